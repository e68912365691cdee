"""Tree-aware paged decode attention against the reference's outputs (golden
fixtures) and the fp64 oracle.  Tolerances are the north star's: fp32 1e-5
max-abs; bf16 / fp16 2e-3 max-abs or 1e-2 relative."""

import os

import numpy as np
import pytest
import torch

from oracle.attention import decode_one, gather_seq, paged_decode
from tests.golden.cases import ATTN_CASES, attn_inputs
from tests.gpu_util import HERE, TORCH_DT, build_tree, round_np

pytestmark = pytest.mark.gpu


def _tol(dtype):
    return dict(atol=1e-5, rtol=0) if dtype == "f32" else dict(atol=2e-3, rtol=1e-2)


def _mgr(c, inp, **kw):
    from mentat_b200 import PagedKVCacheManager
    return PagedKVCacheManager(1, c["hkv"], c["d"], max_blocks=c["pool"], block_size=c["bs"], device="cuda",
                               dtype=TORCH_DT[c["dtype"]], free_order=inp["order"], strict=True, **kw)


@pytest.mark.parametrize("name", sorted(ATTN_CASES))
def test_decode_matches_reference_golden(name):
    from mentat_b200.attention_backend import attn_decode
    c = ATTN_CASES[name]
    g = np.load(os.path.join(HERE, "golden", "attention.npz"))
    inp = attn_inputs(c)
    m = _mgr(c, inp)
    leaves = build_tree(m, c, inp)
    gt = g[f"{name}__tables"]
    for i, sid in enumerate(leaves):  # the reference's block tables (injected FIFO policy)
        t = m.page_table(sid, 0)
        assert t == list(gt[i][: len(t)])
    assert m.allocator.refcounts == g[f"{name}__refcounts"].tolist()
    q = torch.from_numpy(inp["q"]).cuda().to(TORCH_DT[c["dtype"]])
    k, v, cu, mx = m.build_packed_kv(leaves, 0)
    assert cu.tolist() == g[f"{name}__cu"].tolist() and mx == int(g[f"{name}__maxlen"])
    o = attn_decode(q, k, v, cu_seqlens_q=torch.arange(len(leaves) + 1, dtype=torch.int32, device="cuda"),
                    cu_seqlens_k=cu, max_seqlen_k=mx, N=len(leaves))
    m.check()
    got = o.float().cpu().numpy()
    np.testing.assert_allclose(got, g[f"{name}__out"], **_tol(c["dtype"]))
    tabs = [m.page_table(s, 0) for s in leaves]
    lens = [m.get_kv_length(s) for s in leaves]
    oo = paged_decode(round_np(inp["q"], c["dtype"]), m.k_pools[0].float().cpu().numpy(),
                      m.v_pools[0].float().cpu().numpy(), tabs, lens, c["bs"])
    np.testing.assert_allclose(got, oo, **_tol(c["dtype"]))


def c4_like(n_branch, prefix, lo, hi, seed, hq=32, hkv=8, d=128, dtype=torch.bfloat16):
    """Benchmark config-4 shaped tree built through the cache API."""
    from mentat_b200 import PagedKVCacheManager
    g = torch.Generator(device="cuda").manual_seed(seed)
    suf = np.random.default_rng(seed).integers(lo, hi + 1, n_branch)
    blocks = (prefix + 15) // 16 + int(sum((s + 15) // 16 + 1 for s in suf)) + 8
    m = PagedKVCacheManager(1, hkv, d, max_blocks=blocks, block_size=16, device="cuda", dtype=dtype,
                            max_seqs=n_branch + 2)
    kv = lambda n: torch.randn((n, hkv, d), generator=g, device="cuda").to(dtype)  # noqa: E731
    root = m.allocate_sequence()
    m.append_tokens(root, 0, kv(prefix), kv(prefix))
    kids = [m.fork_sequence(root) for _ in range(n_branch)]
    m.free_sequence(root)
    for kid, n in zip(kids, suf):
        m.append_tokens(kid, 0, kv(int(n)), kv(int(n)))
    q = torch.randn((n_branch, hq, d), generator=g, device="cuda").to(dtype)
    m.check()
    return m, kids, q


def _oracle_one(m, sid, qi):
    n = m.get_kv_length(sid)
    tab = torch.tensor(m.page_table(sid, 0), device="cuda", dtype=torch.long)
    t = torch.arange(n, device="cuda")
    ks = m.k_pools[0][tab[t // 16], t % 16].double().cpu().numpy()
    vs = m.v_pools[0][tab[t // 16], t % 16].double().cpu().numpy()
    return decode_one(qi.double().cpu().numpy(), ks, vs)


def test_c4_shape_every_branch_against_oracle():
    from mentat_b200.attention_backend import attn_decode
    m, kids, q = c4_like(16, 4096, 100, 700, seed=3)
    k, v, cu, mx = m.build_packed_kv(kids, 0)
    o = attn_decode(q, k, v, None, cu, mx, len(kids)).float().cpu().numpy()
    for i, sid in enumerate(kids):
        np.testing.assert_allclose(o[i], _oracle_one(m, sid, q[i]), atol=2e-3, rtol=1e-2)


def test_c4_full_size_sharing_invariance():
    """Full config-4 size: each branch's tree-aware result equals decoding that
    branch alone (no shared segments); sampled branches match the fp64 oracle."""
    from mentat_b200.attention_backend import attn_decode
    m, kids, q = c4_like(64, 32768, 1024, 4096, seed=11)
    k, v, cu, mx = m.build_packed_kv(kids, 0)
    o = attn_decode(q, k, v, None, cu, mx, len(kids))
    m.check()
    for i in (0, 17, 63):
        k1, v1, cu1, mx1 = m.build_packed_kv([kids[i]], 0)
        o1 = attn_decode(q[i:i + 1], k1, v1, None, cu1, mx1, 1)
        torch.testing.assert_close(o[i:i + 1].float(), o1.float(), atol=2e-3, rtol=1e-2)
    for i in (5, 40):
        np.testing.assert_allclose(o[i].float().cpu().numpy(), _oracle_one(m, kids[i], q[i]), atol=2e-3, rtol=1e-2)


def test_empty_and_single_token_sequences():
    from mentat_b200 import PagedKVCacheManager
    from mentat_b200.attention_backend import attn_decode
    m = PagedKVCacheManager(1, 2, 64, max_blocks=16, block_size=16, device="cuda", dtype=torch.float32)
    a = m.allocate_sequence()
    b = m.allocate_sequence()
    kv = torch.randn(1, 2, 64, device="cuda")
    m.append_tokens(b, 0, kv, kv)
    q = torch.randn(2, 4, 64, device="cuda")
    k, v, cu, mx = m.build_packed_kv([a, b], 0)
    o = attn_decode(q, k, v, None, cu, mx, 2)
    assert torch.all(o[0] == 0)  # SDPA with zero keys returns zeros
    torch.testing.assert_close(o[1], kv[0].repeat_interleave(2, dim=0), atol=1e-6, rtol=0)


def test_materialize_matches_oracle_packing():
    c = ATTN_CASES["bf16_nested"]
    inp = attn_inputs(c)
    m = _mgr(c, inp)
    leaves = build_tree(m, c, inp)
    k, v, cu, mx = m.build_packed_kv(leaves, 0)
    pk = k.materialize()
    assert pk.shape == k.shape and pk.dtype == k.dtype


def test_one_launch_of_1000_branches():
    """A 1,000-branch tree decodes in one launch (the per-launch limit is 1,024
    sequences), so the shared prefix is read once for all of them; sampled
    branches match the fp64 oracle and decoding a branch alone gives its row."""
    from mentat_b200 import _lib
    from mentat_b200.attention_backend import attn_decode
    m, kids, q = c4_like(1000, 512, 1, 40, seed=21)
    k, v, cu, mx = m.build_packed_kv(kids, 0)
    n0 = _lib.load().mentat_kernel_launch_count()
    o = attn_decode(q, k, v, None, cu, mx, len(kids))
    assert _lib.load().mentat_kernel_launch_count() - n0 <= 5  # lcp, plan, two unit kernels, merge
    m.check()
    for i in (0, 511, 999):
        np.testing.assert_allclose(o[i].float().cpu().numpy(), _oracle_one(m, kids[i], q[i]), atol=2e-3, rtol=1e-2)
        k1, v1, cu1, mx1 = m.build_packed_kv([kids[i]], 0)
        torch.testing.assert_close(o[i:i + 1].float(), attn_decode(q[i:i + 1], k1, v1, None, cu1, mx1, 1).float(),
                                   atol=2e-3, rtol=1e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_plan_reuse_across_layers(dtype):
    """Layers share the tree's sharing structure, so layer 1 may decode with the
    plan layer 0 left in the workspace: the result is bit-identical to planning
    layer 1 itself.  A workspace planned for another batch size is refused on the
    device (zero output, plan error)."""
    from mentat_b200 import PagedKVCacheManager, ops
    g = torch.Generator(device="cuda").manual_seed(5)
    L, hkv, hq, d = 2, 8, 32, 128
    m = PagedKVCacheManager(L, hkv, d, max_blocks=2048, block_size=16, device="cuda", dtype=dtype, max_seqs=64)
    kv = lambda n: torch.randn((n, hkv, d), generator=g, device="cuda").to(dtype)  # noqa: E731
    root = m.allocate_sequence()
    for layer in range(L):
        m.append_tokens(root, layer, kv(700), kv(700))
    kids = [m.fork_sequence(root) for _ in range(24)]
    m.free_sequence(root)
    for i, kid in enumerate(kids):
        for layer in range(L):
            m.append_tokens(kid, layer, kv(5 + 7 * i), kv(5 + 7 * i))
    slots = m._slots_dev(kids)
    q = torch.randn((len(kids), hq, d), generator=g, device="cuda").to(dtype)
    mx = max(m.get_kv_length(s) for s in kids)
    own1 = ops.paged_decode(q, slots, mx, m._op_id, 1, 0.088)
    ops.paged_decode(q, slots, mx, m._op_id, 0, 0.088)
    reused = ops.paged_decode(q, slots, mx, m._op_id, 1, 0.088, reuse_plan=True)
    m.check()
    assert torch.equal(own1, reused)
    few = ops.paged_decode(q[:10], slots[:10], mx, m._op_id, 1, 0.088, reuse_plan=True)  # planned for 24
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="plan workspace overflow"):
        m.check()
    assert torch.count_nonzero(few).item() == 0
