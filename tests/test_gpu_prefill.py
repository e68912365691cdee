"""Causal prefill attention on the paged cache against the reference's
``attn_prefill`` (golden fixtures, ``attention_backend.py:175-189`` with its
SDPA backend), the fp64 oracle (``oracle.attention.prefill``) and, at sizes the
oracle is slow for, torch's fp32 SDPA on the GPU.  Tolerances are the north
star's: fp32 1e-5 max-abs; bf16 / fp16 2e-3 max-abs or 1e-2 relative against
exact arithmetic.  The reference's own bf16 / fp16 outputs round their softmax
probabilities to the input dtype and sit up to 8e-3 / 1.1e-3 from exact, which
bounds the comparison with the fixtures."""

import os

import numpy as np
import pytest
import torch

from oracle.attention import gather_seq, prefill
from tests.golden.cases import PREFILL_CASES, prefill_inputs
from tests.gpu_util import HERE, TORCH_DT, round_np

pytestmark = pytest.mark.gpu

GOLDEN_TOL = {"f32": 1e-5, "bf16": 1e-2, "f16": 2e-3}


def _tol(dtype):
    return dict(atol=1e-5, rtol=0) if dtype == "f32" else dict(atol=2e-3, rtol=1e-2)


def _close(got, want, dtype):
    """max-abs within atol, or relative within rtol, element by element."""
    t = _tol(dtype)
    err = np.abs(got - want)
    ok = (err <= t["atol"]) | (err <= t["rtol"] * np.abs(want))
    assert ok.all(), f"max abs {err.max():.3g} at {np.unravel_index(err.argmax(), err.shape)}"


@pytest.mark.parametrize("name", sorted(PREFILL_CASES))
def test_attn_prefill_matches_reference_golden(name):
    """The drop-in attn_prefill (dense K/V read in place as 16-token blocks)."""
    from mentat_b200.attention_backend import attn_prefill
    dt = PREFILL_CASES[name][0]
    g = np.load(os.path.join(HERE, "golden", "prefill.npz"))
    q, k, v = prefill_inputs(name)
    tq, tk, tv = (torch.from_numpy(a).cuda().to(TORCH_DT[dt]) for a in (q, k, v))
    o = attn_prefill(tq, tk, tv)
    torch.cuda.synchronize()
    assert o.shape == tq.shape and o.dtype == tq.dtype
    got = o.float().cpu().numpy()
    np.testing.assert_allclose(got, g[f"{name}__out"], atol=GOLDEN_TOL[dt], rtol=0)
    want = np.stack([prefill(q[b], k[b], v[b]) for b in range(q.shape[0])])
    _close(got, want, dt)


def _manager(dtype, hkv, d, blocks, bs=16):
    from mentat_b200 import PagedKVCacheManager
    return PagedKVCacheManager(1, hkv, d, max_blocks=blocks, block_size=bs, device="cuda", dtype=dtype,
                               strict=True)


def _sdpa_fp32(q, k, v, pos0):
    """torch fp32 causal attention of q (n, Hq, D) at positions pos0.. over k/v (L, Hkv, D)."""
    n, hq, d = q.shape
    L, hkv, _ = k.shape
    g = hq // hkv
    mask = torch.arange(L, device=q.device)[None, :] <= (pos0 + torch.arange(n, device=q.device))[:, None]
    out = torch.empty((n, hq, d), device=q.device)
    for h0 in range(0, hq, 8):  # eight query heads at a time bound the score matrix
        qq = q[:, h0:h0 + 8].float().permute(1, 0, 2)
        kv = [h // g for h in range(h0, min(hq, h0 + 8))]
        kk = k[:, kv].float().permute(1, 0, 2)
        vv = v[:, kv].float().permute(1, 0, 2)
        s = torch.matmul(qq, kk.transpose(1, 2)) / d ** 0.5
        s = s.masked_fill(~mask, float("-inf"))
        out[:, h0:h0 + 8] = torch.matmul(torch.softmax(s, dim=-1), vv).permute(1, 0, 2)
    return out


@pytest.mark.parametrize("dtype,hq,hkv,d,chunks,bs", [
    ("bf16", 32, 4, 128, (700, 1400), 16),  # crosses the tensor-core kernel's 2,048-token chunk
    ("f16", 16, 16, 64, (5, 1, 300), 16),
    ("bf16", 8, 1, 128, (2049,), 16),
    ("f32", 8, 2, 128, (100, 157, 1), 16),   # FFMA kernel
    ("bf16", 32, 32, 128, (4096,), 16),      # every query group in one unit: rows written by the unit kernel
    ("f16", 64, 8, 64, (3000,), 16),         # no query with two partials: no merge
    ("bf16", 32, 2, 128, (1000, 33), 16),    # G = 16: 16 queries per tensor-core unit
    ("bf16", 8, 2, 128, (300, 90), 32),      # 32-token blocks: the FFMA kernel on bf16
])
def test_paged_prefill_in_chunks(dtype, hq, hkv, d, chunks, bs):
    """A prompt appended and attended chunk by chunk (pos0 > 0 for every chunk
    after the first) gives the rows of one causal attention over the prompt."""
    torch.manual_seed(0)
    L = sum(chunks)
    tdt = TORCH_DT[dtype]
    m = _manager(tdt, hkv, d, blocks=(L + bs - 1) // bs + 4, bs=bs)
    sid = m.allocate_sequence()
    q = torch.randn(L, hq, d, device="cuda").to(tdt)
    k = torch.randn(L, hkv, d, device="cuda").to(tdt)
    v = torch.randn(L, hkv, d, device="cuda").to(tdt)
    outs = []
    a = 0
    for n in chunks:
        m.append_tokens(sid, 0, k[a:a + n], v[a:a + n])
        outs.append(m.prefill_attention(sid, 0, q[a:a + n]))
        a += n
    m.check()
    got = torch.cat(outs).float()
    want = _sdpa_fp32(q, k, v, 0)
    err = (got - want).abs()
    t = _tol(dtype)
    ok = (err <= t["atol"]) | (err <= t["rtol"] * want.abs())
    assert bool(ok.all()), f"max abs {err.max().item():.3g}"


def test_prefill_of_a_forked_branch():
    """The suffix of a branch forked off a shared prefix (blocks shared with the
    parent and the siblings, the last shared block copied on write) attends to
    the prefix through the branch's own table."""
    from oracle.attention import prefill as ora
    torch.manual_seed(1)
    hq, hkv, d, dt = 16, 4, 128, "bf16"
    tdt = TORCH_DT[dt]
    m = _manager(tdt, hkv, d, blocks=256)
    root = m.allocate_sequence()
    P, S = 203, 77
    kp, vp = (torch.randn(P, hkv, d, device="cuda").to(tdt) for _ in range(2))
    m.append_tokens(root, 0, kp, vp)
    kids = [m.fork_sequence(root) for _ in range(3)]
    m.free_sequence(root)
    for i, c in enumerate(kids):
        ks, vs = (torch.randn(S + i, hkv, d, device="cuda").to(tdt) for _ in range(2))
        qs = torch.randn(S + i, hq, d, device="cuda").to(tdt)
        m.append_tokens(c, 0, ks, vs)
        o = m.prefill_attention(c, 0, qs).float().cpu().numpy()
        m.check()
        tab, n = m.page_table(c, 0), m.get_kv_length(c)
        assert n == P + S + i
        kk = gather_seq(m.k_pools[0].float().cpu().numpy(), tab, n, 16)
        vv = gather_seq(m.v_pools[0].float().cpu().numpy(), tab, n, 16)
        want = ora(round_np(qs.float().cpu().numpy(), dt), kk, vv, pos0=P)
        _close(o, want, dt)


def test_prefill_argument_errors():
    from mentat_b200.attention_backend import attn_prefill
    m = _manager(torch.bfloat16, 2, 128, blocks=8)
    sid = m.allocate_sequence()
    k = torch.randn(4, 2, 128, device="cuda").to(torch.bfloat16)
    m.append_tokens(sid, 0, k, k)
    with pytest.raises(ValueError):
        m.prefill_attention(sid, 0, torch.randn(5, 4, 128, device="cuda").to(torch.bfloat16))
    with pytest.raises(TypeError):
        m.prefill_attention(sid, 0, torch.randn(4, 4, 128, device="cuda"))
    q = torch.randn(1, 8, 4, 128, device="cuda").to(torch.bfloat16)
    kv = torch.randn(1, 8, 2, 128, device="cuda").to(torch.bfloat16)
    with pytest.raises(NotImplementedError):
        attn_prefill(q, kv, kv, window_size=4)
    assert attn_prefill(q, kv, kv, window_size=8).shape == q.shape  # a window >= S is no window
    assert m.prefill_attention(sid, 0, q[0, :0]).shape == (0, 4, 128)


def test_prefill_refuses_a_short_workspace():
    """A max_parts below the plan's need returns MENTAT_ERR_ARG before any launch."""
    import ctypes as C
    from mentat_b200 import _lib
    lib = _lib.load()
    m = _manager(torch.float32, 2, 128, blocks=400)
    sid = m.allocate_sequence()
    k = torch.randn(5000, 2, 128, device="cuda")
    m.append_tokens(sid, 0, k, k)
    q = torch.randn(1, 4, 128, device="cuda")
    need = int(lib.mentat_prefill_max_parts(m._descp, 1, 4999, 4))
    assert need > 1
    ws = torch.empty(int(lib.mentat_decode_workspace_bytes(1, 4, 128, need)), dtype=torch.uint8, device="cuda")
    out = torch.empty_like(q)
    slot = m._slots_dev([sid])
    stream = torch.cuda.current_stream().cuda_stream
    args = (m._descp, 0, slot.data_ptr(), 1, 4999, q.data_ptr(), 4 * 128, 4, out.data_ptr(), 4 * 128,
            C.c_float(128 ** -0.5), ws.data_ptr(), ws.numel())
    assert lib.mentat_paged_prefill(*args, need - 1, stream) == -1
    assert lib.mentat_paged_prefill(*args, need, stream) == 0
    torch.cuda.synchronize()
    m.check()
    want = _sdpa_fp32(q, k, k, 4999)
    assert float((out - want).abs().max()) < 1e-5
