"""The decode entry point for callers that cannot allocate device memory at call time.

Some hosts cannot give the library a workspace when they decode.  A program that
binds the C ABI directly has no caching allocator, and a cudaMalloc on every
call would synchronise the whole device.  A serving runtime may reserve all
device memory up front and forbid new allocations while it serves.
``mentat_paged_decode_noalloc`` serves them: it uses a fixed scratch array inside
the library instead of a workspace.  This test calls it through the C ABI twice
in a row, on different queries, and checks each result against the ordinary
``mentat_paged_decode``.  It also checks that a request larger than the scratch
is refused without touching the output.

The file name sorts last, so a run that stops at the first failure has run every
other test first.
"""

import ctypes as C
import math

import numpy as np
import pytest
import torch

from tests.golden.cases import ATTN_CASES, attn_inputs
from tests.gpu_util import TORCH_DT, build_tree

pytestmark = pytest.mark.gpu

TOL = dict(atol=2e-3, rtol=1e-2)  # the bf16 tolerance of the attention tests


def _decode_with_workspace(lib, m, slots, q, parts):
    """The existing entry point, with a caller-owned workspace."""
    n, hq, d = q.shape
    out = torch.empty_like(q)
    wsb = int(lib.mentat_decode_workspace_bytes(n, hq, d, parts))
    ws = torch.empty(wsb, dtype=torch.uint8, device=q.device)
    st = lib.mentat_paged_decode(m._descp, 0, slots.data_ptr(), n, q.data_ptr(), q.stride(0), hq, out.data_ptr(),
                                 out.stride(0), 1.0 / math.sqrt(d), ws.data_ptr(), wsb, parts,
                                 torch.cuda.current_stream().cuda_stream)
    assert st == 0, st
    return out


def _decode_no_alloc(lib, m, slots, q, parts, out):
    n, hq, d = q.shape
    return lib.mentat_paged_decode_noalloc(m._descp, 0, slots.data_ptr(), n, q.data_ptr(), q.stride(0), hq,
                                           out.data_ptr(), out.stride(0), 1.0 / math.sqrt(d), parts,
                                           torch.cuda.current_stream().cuda_stream)


def test_no_alloc_decode_matches_workspace_decode_twice():
    from mentat_b200 import PagedKVCacheManager, _lib
    lib = _lib.load()
    c = ATTN_CASES["bf16_nested"]
    inp = attn_inputs(c)
    m = PagedKVCacheManager(1, c["hkv"], c["d"], max_blocks=c["pool"], block_size=c["bs"], device="cuda",
                            dtype=TORCH_DT[c["dtype"]], free_order=inp["order"], strict=True)
    leaves = build_tree(m, c, inp)
    k, _, _, _ = m.build_packed_kv(leaves, 0)
    n = len(leaves)
    parts = int(lib.mentat_decode_max_parts(n, max(k.lens), c["bs"]))
    need = int(lib.mentat_decode_workspace_bytes(n, c["hq"], c["d"], parts))
    assert need <= _lib.NOALLOC_SCRATCH_BYTES
    g = torch.Generator(device="cuda").manual_seed(7)
    for call in range(2):  # two calls in a row share the scratch array
        q = torch.randn((n, c["hq"], c["d"]), generator=g, device="cuda").to(torch.bfloat16)
        ref = _decode_with_workspace(lib, m, k.slots, q, parts)
        out = torch.full_like(q, float("nan"))
        st = _decode_no_alloc(lib, m, k.slots, q, parts, out)
        assert st == 0, lib.mentat_status_string(st)
        torch.cuda.synchronize()
        m.check()
        np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy(), **TOL,
                                   err_msg=f"call {call}")


def test_no_alloc_rejects_requests_beyond_the_scratch():
    from mentat_b200 import PagedKVCacheManager, _lib
    lib = _lib.load()
    m = PagedKVCacheManager(1, 8, 128, max_blocks=64, block_size=16, device="cuda", dtype=torch.bfloat16)
    s = m.allocate_sequence()
    kv = torch.randn((20, 8, 128), device="cuda").to(torch.bfloat16)
    m.append_tokens(s, 0, kv, kv)
    k, _, _, _ = m.build_packed_kv([s], 0)
    q = torch.randn((1, 32, 128), device="cuda").to(torch.bfloat16)
    out = torch.zeros_like(q)
    too_many_parts = 1 + _lib.NOALLOC_SCRATCH_BYTES // (32 * 130 * 4)
    assert lib.mentat_decode_workspace_bytes(1, 32, 128, too_many_parts) > _lib.NOALLOC_SCRATCH_BYTES
    st = _decode_no_alloc(lib, m, k.slots, q, too_many_parts, out)
    assert st == _lib.ERR_SCRATCH_LIMIT
    assert b"scratch" in lib.mentat_status_string(st)
    torch.cuda.synchronize()
    assert torch.all(out == 0)
