"""Device allocator, tables, fork / free / append / CoW / trim against the
reference's own op streams (golden fixtures), bit-exact."""

import numpy as np
import pytest
import torch

from oracle.allocator import OraclePagedKV
from tests.golden.cases import ATTN_CASES, attn_inputs, build_tree_ops
from tests.gpu_util import TORCH_DT, build_tree, load_streams, round_np

pytestmark = pytest.mark.gpu


def apply_op(m, op):
    kind = op[0]
    if kind == "alloc":
        return m.allocate_sequence()
    if kind == "fork":
        return m.fork_sequence(op[1])
    if kind == "free":
        return m.free_sequence(op[1])
    if kind == "append":
        _, sid, layer, n = op
        z = torch.zeros((n, 1, 2), device="cuda")
        return m.append_tokens(sid, layer, z, z)
    if kind == "append_batched":
        _, sids, layer = op
        z = torch.zeros((len(sids), 1, 2), device="cuda")
        return m.append_tokens_batched(seq_ids=sids, layer_idx=layer, k=z, v=z)
    if kind == "trim":
        return m.trim_to_window(op[1], op[2])
    raise ValueError(kind)


def snap(m):
    seqs = {str(k): v for k, v in m.sequence_snapshot().items()}
    return {"seqs": seqs, "refcounts": m.allocator.refcounts, "free": m.allocator.free_list(),
            "peak": m.allocator.peak_used, "stats": m.get_stats()}


@pytest.mark.parametrize("idx", range(20))
def test_alloc_stream_bit_exact(idx):
    from mentat_b200 import PagedKVCacheManager
    st = load_streams()[idx]
    p = st["params"]
    m = PagedKVCacheManager(p["L"], 1, 2, max_blocks=p["max_blocks"], block_size=p["bs"], device="cuda",
                            dtype=torch.float32, free_order=st["order"], max_seqs=64, strict=True)
    cps = {c["op"]: c["snap"] for c in st["checkpoints"]}
    err = st["error"]
    for i, op in enumerate(st["ops"]):
        if err and i == err["op"]:
            exc = {"RuntimeError": RuntimeError, "KeyError": KeyError}[err["type"]]
            with pytest.raises(exc) as ei:
                apply_op(m, op)
            assert str(ei.value) == err["msg"]
            return
        apply_op(m, op)
        if i in cps:
            got, exp = snap(m), cps[i]
            assert got["seqs"] == exp["seqs"], f"tables differ after op {i}: {op}"
            assert got["refcounts"] == exp["refcounts"], f"refcounts differ after op {i}"
            assert got["free"] == exp["free"], f"free list differs after op {i}"
            assert got["peak"] == exp["peak"]
            assert got["stats"] == exp["stats"]
    assert err is None


@pytest.mark.parametrize("name", ["c1", "bf16_nested", "f16_g2", "bf16_b8_g8_p17"])
def test_append_cow_data_bit_exact(name):
    """Pool contents after fork / CoW / append equal the oracle's, gathered per leaf."""
    from mentat_b200 import PagedKVCacheManager
    c = ATTN_CASES[name]
    inp = attn_inputs(c)
    m = PagedKVCacheManager(1, c["hkv"], c["d"], max_blocks=c["pool"], block_size=c["bs"], device="cuda",
                            dtype=TORCH_DT[c["dtype"]], free_order=inp["order"], strict=True)
    leaves = build_tree(m, c, inp)
    o = OraclePagedKV(1, c["hkv"], c["d"], c["pool"], c["bs"], order=inp["order"])
    for op in build_tree_ops(c):
        if op[0] == "append":
            o.append_tokens(op[1], 0, round_np(inp[op[2]], c["dtype"]), round_np(inp[op[3]], c["dtype"]))
        elif op[0] == "alloc":
            o.allocate_sequence()
        elif op[0] == "fork":
            o.fork_sequence(op[1])
        elif op[0] == "free":
            o.free_sequence(op[1])
    pk, pv, cu, mx = m.packed_kv_tensors(leaves, 0)
    ok, ov, ocu, omx = o.build_packed_kv(leaves, 0)
    assert cu.tolist() == ocu.tolist() and mx == omx
    np.testing.assert_array_equal(pk.float().cpu().numpy(), ok)
    np.testing.assert_array_equal(pv.float().cpu().numpy(), ov)


def test_decode_steps_append_batched_matches_oracle():
    """Generator-style steps: forks, parent frees and batched appends over layers."""
    from mentat_b200 import PagedKVCacheManager
    rng = np.random.default_rng(5)
    L, hkv, d, bs, pool = 3, 2, 64, 4, 256
    order = rng.permutation(pool).tolist()
    m = PagedKVCacheManager(L, hkv, d, max_blocks=pool, block_size=bs, device="cuda", dtype=torch.bfloat16,
                            free_order=order, strict=True)
    o = OraclePagedKV(L, hkv, d, pool, bs, order=order, elem_bytes=2)
    s = m.allocate_sequence()
    o.allocate_sequence()
    for layer in range(L):  # 6 + 1 tokens at the first fork: a shared partial tail, so CoW happens
        kv = round_np(rng.standard_normal((6, hkv, d), dtype=np.float32), "bf16")
        t = torch.from_numpy(kv).cuda().bfloat16()
        m.append_tokens(s, layer, t, t)
        o.append_tokens(s, layer, kv, kv)
    live = [s]
    for step in range(12):
        if step % 4 == 1:
            p = live.pop(0)
            kids = [m.fork_sequence(p) for _ in range(3)]
            assert kids == [o.fork_sequence(p) for _ in range(3)]
            m.free_sequence(p)
            o.free_sequence(p)
            live += kids
        for layer in range(L):
            kv = round_np(rng.standard_normal((len(live), hkv, d), dtype=np.float32), "bf16")
            t = torch.from_numpy(kv).cuda().bfloat16()
            m.append_tokens_batched(live, layer, t, t)
            o.append_tokens_batched(live, layer, kv, kv)
    for layer in range(L):
        pk, pv, _, _ = m.packed_kv_tensors(live, layer)
        ok, ov, _, _ = o.build_packed_kv(live, layer)
        np.testing.assert_array_equal(pk.float().cpu().numpy(), ok)
        np.testing.assert_array_equal(pv.float().cpu().numpy(), ov)
        for sid in live:
            assert m.page_table(sid, layer) == o._sequences[sid].page_table[layer]
    assert m.allocator.refcounts == o.allocator.refcounts
    assert m.get_stats() == o.get_stats()
    assert m.kernel_counters()["cow_copies"] > 0


def test_duplicate_slot_in_batch_is_sequential():
    from mentat_b200 import PagedKVCacheManager
    m = PagedKVCacheManager(1, 1, 64, max_blocks=32, block_size=4, device="cuda", dtype=torch.float32, strict=True)
    o = OraclePagedKV(1, 1, 64, 32, 4)
    a = m.allocate_sequence()
    o.allocate_sequence()
    base = np.arange(3 * 64, dtype=np.float32).reshape(3, 1, 64)
    m.append_tokens(a, 0, torch.from_numpy(base).cuda(), torch.from_numpy(base).cuda())
    o.append_tokens(a, 0, base, base)
    b = m.fork_sequence(a)
    o.fork_sequence(a)
    kv = np.random.default_rng(0).standard_normal((4, 1, 64)).astype(np.float32)
    t = torch.from_numpy(kv).cuda()
    m.append_tokens_batched([a, b, a, b], 0, t, t)
    o.append_tokens_batched([a, b, a, b], 0, kv, kv)
    for sid in (a, b):
        assert m.page_table(sid, 0) == o._sequences[sid].page_table[0]
    pk, _, _, _ = m.packed_kv_tensors([a, b], 0)
    ok, _, _, _ = o.build_packed_kv([a, b], 0)
    np.testing.assert_array_equal(pk.cpu().numpy(), ok)


def test_out_of_blocks_raises_reference_message():
    """Found on the device (two sequences together exhaust the pool) and raised
    with the reference's message at the next check."""
    from mentat_b200 import PagedKVCacheManager
    m = PagedKVCacheManager(1, 1, 64, max_blocks=3, block_size=4, device="cuda", dtype=torch.float32)
    a, b = m.allocate_sequence(), m.allocate_sequence()
    z = torch.zeros(8, 1, 64, device="cuda")
    m.append_tokens(a, 0, z, z)  # 2 blocks
    m.append_tokens(b, 0, z, z)  # 2 more blocks of a 3-block pool
    with pytest.raises(RuntimeError, match=r"out of blocks \(pool size=3\)"):
        m.check()
    # a single sequence larger than the pool is refused on the host, same message
    m2 = PagedKVCacheManager(1, 1, 64, max_blocks=2, block_size=4, device="cuda", dtype=torch.float32)
    s = m2.allocate_sequence()
    with pytest.raises(RuntimeError, match=r"out of blocks \(pool size=2\)"):
        m2.append_tokens(s, 0, torch.zeros(12, 1, 64, device="cuda"), torch.zeros(12, 1, 64, device="cuda"))


def test_padding_entries_are_skipped():
    """Slot -1 entries of a batched append (padding of a captured graph's batch)
    allocate nothing and write nothing: the cache ends as after the same append
    without them."""
    from mentat_b200 import PagedKVCacheManager

    def build():
        m = PagedKVCacheManager(1, 2, 64, max_blocks=32, block_size=4, device="cuda", dtype=torch.float32,
                                strict=True)
        a = m.allocate_sequence()
        base = torch.arange(3 * 2 * 64, dtype=torch.float32, device="cuda").view(3, 2, 64)
        m.append_tokens(a, 0, base, base)
        b = m.fork_sequence(a)  # shared partial tail: the append below copies it for one of them
        return m, a, b

    kv = torch.from_numpy(np.random.default_rng(1).standard_normal((4, 2, 64)).astype(np.float32)).cuda()
    m1, a, b = build()
    m1.append_tokens_batched([a, b], 0, kv[[0, 2]], kv[[1, 3]])
    m2, a2, b2 = build()
    s = m2._sequences
    slots = torch.tensor([s[a2].slot, -1, s[b2].slot, -1], dtype=torch.int32, device="cuda")
    torch.ops.mentat_b200.append_batched(m2._k_all, m2._v_all, slots, kv[[0, 3, 2, 1]], kv[[1, 0, 3, 2]],
                                         m2._op_id, 0)
    m2.mirror_decode_step([a2, b2])
    assert m2.sequence_snapshot() == m1.sequence_snapshot()
    assert m2.allocator.refcounts == m1.allocator.refcounts
    assert m2.allocator.free_list() == m1.allocator.free_list()
    k1, v1, _, _ = m1.packed_kv_tensors([a, b], 0)
    k2, v2, _, _ = m2.packed_kv_tensors([a2, b2], 0)
    assert torch.equal(k1, k2) and torch.equal(v1, v2)
