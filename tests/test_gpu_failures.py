"""Failure paths of the decode kernels, made without faulting or hanging the GPU.

* Bounded waits: the test hook ``mentat_decode_set_wait_probe`` makes every
  tensor-core unit CTA wait on a barrier that nothing arrives on, for a few
  microseconds.  The wait gives up before the CTA has issued a copy or an MMA;
  the call must report ``MENTAT_DEV_DECODE_TIMEOUT`` (a ``RuntimeError`` at the
  next check), zero its output, and leave the library usable: the next call,
  with the hook off, must be correct.
* Corrupt block tables: an entry outside ``[0, max_blocks)`` is never read by
  the decode or gather kernels; it is recorded as ``MENTAT_DEV_BAD_BLOCK``
  (``AssertionError``, like the reference's checks at ``paged_kv_cache.py:59,63``).
* Plan overflow: a workspace sized for too few partials gives
  ``MENTAT_DEV_PLAN_OVERFLOW`` and a zeroed output, with no read past the
  workspace.
"""

import math

import numpy as np
import pytest
import torch

from oracle.attention import paged_decode
from tests.golden.cases import ATTN_CASES, attn_inputs
from tests.gpu_util import TORCH_DT, build_tree, round_np

pytestmark = pytest.mark.gpu


def _tol(dtype):
    return dict(atol=1e-5, rtol=0) if dtype == "f32" else dict(atol=2e-3, rtol=1e-2)


def _case(name):
    from mentat_b200 import PagedKVCacheManager
    c = ATTN_CASES[name]
    inp = attn_inputs(c)
    m = PagedKVCacheManager(1, c["hkv"], c["d"], max_blocks=c["pool"], block_size=c["bs"], device="cuda",
                            dtype=TORCH_DT[c["dtype"]], free_order=inp["order"])
    leaves = build_tree(m, c, inp)
    q = torch.from_numpy(inp["q"]).cuda().to(TORCH_DT[c["dtype"]])
    m.check()
    return c, inp, m, leaves, q


def _decode(m, leaves, q):
    from mentat_b200.attention_backend import attn_decode
    k, v, cu, mx = m.build_packed_kv(leaves, 0)
    return attn_decode(q, k, v, None, cu, mx, len(leaves))


def _oracle(c, inp, m, leaves):
    tabs = [m.page_table(s, 0) for s in leaves]
    lens = [m.get_kv_length(s) for s in leaves]
    return paged_decode(round_np(inp["q"], c["dtype"]), m.k_pools[0].float().cpu().numpy(),
                        m.v_pools[0].float().cpu().numpy(), tabs, lens, c["bs"])


@pytest.mark.parametrize("name", ["bf16_g4_wide", "bf16_nested"])
def test_bounded_wait_gives_up_and_zeroes_output(name):
    from mentat_b200 import _lib
    lib = _lib.load()
    c, inp, m, leaves, q = _case(name)
    ref = _oracle(c, inp, m, leaves)
    try:
        assert lib.mentat_decode_set_wait_probe(20000) == 0  # ~10 us at 1.9 GHz
        out = _decode(m, leaves, q)
        torch.cuda.synchronize()
    finally:
        assert lib.mentat_decode_set_wait_probe(0) == 0
    with pytest.raises(RuntimeError, match="bounded wait gave up"):
        m.check()
    assert torch.count_nonzero(out).item() == 0
    m.clear_error()
    for _ in range(2):  # the library and the cache stay usable
        got = _decode(m, leaves, q).float().cpu().numpy()
        m.check()
        np.testing.assert_allclose(got, ref, **_tol(c["dtype"]))


@pytest.mark.parametrize("name", ["bf16_g4_wide", "c1"])
def test_bad_block_id_is_recorded_not_read(name):
    c, inp, m, leaves, q = _case(name)
    ref = _oracle(c, inp, m, leaves)
    slot = m._sequences[leaves[-1]].slot
    nb = len(m.page_table(leaves[-1], 0))
    for j, bad in [(0, c["pool"] + 5), (nb - 1, -3), (nb // 2, 1 << 30)]:
        good = int(m._tables[0, slot, j].item())
        m._tables[0, slot, j] = bad
        _decode(m, leaves, q)
        torch.cuda.synchronize()
        with pytest.raises(AssertionError, match="outside the pool"):
            m.check()
        m.clear_error()
        pk = m.build_packed_kv(leaves, 0)[0]
        pk.materialize()  # the gather kernel checks its entries too
        torch.cuda.synchronize()
        with pytest.raises(AssertionError, match=f"entry {bad} outside"):
            m.check()
        m.clear_error()
        m._tables[0, slot, j] = good
    got = _decode(m, leaves, q).float().cpu().numpy()
    m.check()
    np.testing.assert_allclose(got, ref, **_tol(c["dtype"]))


def test_plan_overflow_zeroes_output():
    from mentat_b200 import _lib
    lib = _lib.load()
    c, inp, m, leaves, q = _case("bf16_nested")
    slots = torch.tensor([m._sequences[s].slot for s in leaves], dtype=torch.int32, device="cuda")
    n, hq, d = q.shape
    parts = 1  # every sequence needs more than one partial (shared and own segments)
    wsb = int(lib.mentat_decode_workspace_bytes(n, hq, d, parts))
    ws = torch.full((wsb,), 0x7F, dtype=torch.uint8, device="cuda")
    out = torch.full_like(q, 3.0)
    st = lib.mentat_paged_decode(m._descp, 0, slots.data_ptr(), n, q.data_ptr(), q.stride(0), hq, out.data_ptr(),
                                 out.stride(0), 1.0 / math.sqrt(d), ws.data_ptr(), wsb, parts,
                                 torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="plan workspace overflow"):
        m.check()
    assert torch.count_nonzero(out).item() == 0
