"""Seeded case definitions shared by ``make_golden.py`` and the tests.

Everything here is deterministic from numpy ``default_rng`` seeds, so the GPU
box regenerates the same inputs that the reference saw when the fixtures were
made.
"""

from __future__ import annotations

import numpy as np

from oracle.gate import bf16_round

# ---------------------------------------------------------------------------
# Allocator op streams
# ---------------------------------------------------------------------------

ALLOC_STREAM_PARAMS = (
    [dict(seed=s, L=1 + s % 3, max_blocks=64, bs=4, n_ops=60) for s in range(8)]
    + [dict(seed=100 + s, L=2, max_blocks=256, bs=16, n_ops=80) for s in range(6)]
    + [dict(seed=200 + s, L=1, max_blocks=12, bs=4, n_ops=60) for s in range(6)]  # exhausts
)


def random_op_stream(seed, L, max_blocks, bs, n_ops):
    """A random sequence of cache API calls with reference-style seq ids."""
    rng = np.random.default_rng(seed)
    live: list[int] = []
    next_id = 0
    ops = []
    for _ in range(n_ops):
        r = rng.random()
        if not live or r < 0.08:
            ops.append(["alloc"])
            live.append(next_id)
            next_id += 1
        elif r < 0.25:
            p = int(rng.choice(live))
            ops.append(["fork", p])
            live.append(next_id)
            next_id += 1
        elif r < 0.35 and len(live) > 1:
            s = int(rng.choice(live))
            ops.append(["free", s])
            live.remove(s)
        elif r < 0.55:
            s = int(rng.choice(live))
            ops.append(["append", s, int(rng.integers(L)), int(rng.integers(1, 3 * bs))])
        elif r < 0.93:
            k = int(rng.integers(1, len(live) + 1))
            sids = [int(x) for x in rng.choice(live, size=k, replace=False)]
            ops.append(["append_batched", sids, int(rng.integers(L))])
        else:
            s = int(rng.choice(live))
            ops.append(["trim", s, int(rng.integers(0, 4 * bs))])
    if seed % 5 == 4:
        ops.append(["free", next_id + 7])  # unknown seq id -> KeyError
    return ops


# ---------------------------------------------------------------------------
# Attention trees
# ---------------------------------------------------------------------------

def _c(dtype, hq, hkv, d, prefix, levels, seed, pool=1024, bs=16, B=None):
    return dict(dtype=dtype, hq=hq, hkv=hkv, d=d, prefix=prefix, levels=levels,
                seed=seed, pool=pool, bs=bs)


ATTN_CASES = {
    # benchmark config 1: fp32, 8 branches x (512 shared + 64 own), pool 1024.
    "c1": _c("f32", 16, 8, 128, 512, [(8, (64, 64))], seed=1),
    "f32_ragged": _c("f32", 16, 8, 128, 37, [(3, (0, 40))], seed=2),
    "bf16_b1_g1": _c("bf16", 8, 8, 128, 0, [(1, (1, 1))], seed=3),
    "bf16_b2_g2_p15": _c("bf16", 16, 8, 128, 15, [(2, (1, 17))], seed=4),
    "bf16_b8_g4_p16": _c("bf16", 32, 8, 128, 16, [(8, (15, 17))], seed=5),
    "bf16_b8_g8_p17": _c("bf16", 64, 8, 128, 17, [(8, (0, 16))], seed=6),
    "bf16_nested": _c("bf16", 32, 8, 128, 100, [(2, (5, 40)), (3, (1, 33)), (2, (0, 20))], seed=7),
    "bf16_g4_wide": _c("bf16", 32, 8, 128, 300, [(16, (1, 64))], seed=8, pool=2048),
    "bf16_d64": _c("bf16", 8, 4, 64, 70, [(4, (3, 30))], seed=9),
    "f16_g2": _c("f16", 16, 8, 128, 50, [(4, (2, 20))], seed=10),
    "bf16_64branch": _c("bf16", 32, 8, 128, 256, [(64, (16, 48))], seed=11, pool=4096),
}


def build_tree_ops(c):
    """Ops that build the case's tree through the cache API.

    Root gets ``prefix`` tokens; then each level forks every leaf ``fanout``
    times, frees the parent and appends a per-child suffix with a length drawn
    from ``[lo, hi]``.  Leaves come out in DFS order.
    """
    rng = np.random.default_rng(c["seed"] + 77)
    ops = [["alloc"]]
    next_id = 1
    leaves = [0]
    if c["prefix"]:
        ops.append(["append", 0, "k_0", "v_0"])
    for fan, (lo, hi) in c["levels"]:
        new = []
        for p in leaves:
            kids = []
            for _ in range(fan):
                ops.append(["fork", p])
                kids.append(next_id)
                next_id += 1
            ops.append(["free", p])
            for k in kids:
                n = int(rng.integers(lo, hi + 1))
                if n:
                    ops.append(["append", k, f"k_{k}", f"v_{k}", n])
            new.extend(kids)
        leaves = new
    ops.append(["leaves", leaves])
    return ops


# causal prefill (attn_prefill, attention_backend.py:175-189): (dtype, batch,
# prompt length, Hq, Hkv, D, seed); lengths off and on the 16-token block
PREFILL_CASES = {
    "f32_g4_s37": ("f32", 1, 37, 8, 2, 128, 11),
    "f32_g1_d64_s16": ("f32", 2, 16, 4, 4, 64, 12),
    "bf16_g8_s300": ("bf16", 1, 300, 8, 1, 128, 13),
    "bf16_g4_d64_b2_s65": ("bf16", 2, 65, 8, 2, 64, 14),
    "f16_g2_s1": ("f16", 3, 1, 4, 2, 128, 15),
    "f16_g8_s129": ("f16", 1, 129, 16, 2, 128, 16),
}


# semantic pruning (generator.py:400-497): leaves, similarity dtype, cluster spread
# (smaller: more pairs above the threshold), threshold, min_steps_before_prune
PRUNE_CASES = {
    f"p{k}": dict(seed=100 + k, m=m, dtype=dt, spread=sp, thr=thr, min_age=age)
    for k, (m, dt, sp, thr, age) in enumerate([
        (2, "f32", 0.1, 0.85, 0), (5, "f32", 0.3, 0.85, 3), (12, "bf16", 0.3, 0.85, 3),
        (20, "f32", 0.5, 0.85, 5), (33, "bf16", 0.2, 0.85, 2), (40, "f32", 0.4, 0.9, 4),
        (9, "f32", 1.0, 0.0, 0), (17, "bf16", 0.6, -0.25, 1), (6, "f32", 0.05, 0.85, 9),
        (37, "bf16", 0.35, 0.8, 3), (24, "f32", 0.25, 0.95, 0), (3, "bf16", 2.0, 0.85, 0),
    ])
}


def prefill_inputs(name):
    """q (B, S, Hq, D), k and v (B, S, Hkv, D), float32, rounded to the case's dtype."""
    dt, B, S, hq, hkv, d, seed = PREFILL_CASES[name]
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, S, hq, d), dtype=np.float32)
    k = rng.standard_normal((B, S, hkv, d), dtype=np.float32)
    v = rng.standard_normal((B, S, hkv, d), dtype=np.float32)
    rnd = {"f32": lambda a: a, "bf16": bf16_round, "f16": lambda a: a.astype(np.float16).astype(np.float32)}[dt]
    return tuple(rnd(a) for a in (q, k, v))


def attn_inputs(c):
    """q, per-append K/V arrays (float32) and the pool permutation."""
    rng = np.random.default_rng(c["seed"])
    out = {"order": rng.permutation(c["pool"]).tolist()}
    ops = build_tree_ops(c)
    hkv, d = c["hkv"], c["d"]
    if c["prefix"]:
        out["k_0"] = rng.standard_normal((c["prefix"], hkv, d), dtype=np.float32)
        out["v_0"] = rng.standard_normal((c["prefix"], hkv, d), dtype=np.float32)
    for op in ops:
        if op[0] == "append" and op[1] != 0:
            n = op[4]
            out[op[2]] = rng.standard_normal((n, hkv, d), dtype=np.float32)
            out[op[3]] = rng.standard_normal((n, hkv, d), dtype=np.float32)
    nleaves = len(ops[-1][1])
    out["q"] = rng.standard_normal((nleaves, c["hq"], d), dtype=np.float32)
    return out


# ---------------------------------------------------------------------------
# Gate
# ---------------------------------------------------------------------------

def _g(V, seed, scale, offset=0.0, T=0.7, penalty=1.2, K=3, hist=12, ema_old=None,
       alpha=0.3, mult=1.25, M=10, num_active=1, step=1, window=10, initial=0.3):
    return dict(V=V, seed=seed, scale=scale, offset=offset, T=T, penalty=penalty, K=K,
                hist=hist, ema_old=ema_old, alpha=alpha, mult=mult, M=M,
                num_active=num_active, step=step, window=window, initial=initial)


GATE_CASES = (
    [_g(151936, s, sc, ema_old=eo, num_active=na, step=st)
     for s, sc, eo, na, st in [(0, 2.5, None, 1, 0), (1, 0.5, 11.0, 4, 3), (2, 4.0, 3.0, 7, 12),
                               (3, 0.05, 11.9, 2, 5)]]
    + [_g(128256, s, sc, T=1.0, K=2, M=16, ema_old=eo, num_active=na, step=st)
       for s, sc, eo, na, st in [(10, 1.5, 4.0, 3, 20), (11, 0.02, None, 1, 0)]]
    + [_g(V, 20 + i, sc, offset=off, hist=h, K=k, ema_old=eo, num_active=na, step=st, penalty=pen)
       for i, (V, sc, off, h, k, eo, na, st, pen) in enumerate([
           (1000, 0.01, 0.0, 50, 3, 6.0, 2, 2, 1.2),
           (4096, 3.0, -2.0, 0, 3, None, 1, 0, 1.2),
           (4096, 0.3, 1.0, 300, 5, 8.0, 5, 9, 1.2),
           (32000, 1.0, 0.0, 40, 3, 9.0, 3, 4, 1.0),
           (50257, 6.0, 3.0, 100, 4, 2.0, 6, 15, 1.3),
           (257, 0.001, 0.0, 10, 3, 5.0, 1, 1, 1.2),
           (7, 1.0, 0.0, 3, 3, None, 1, 0, 1.2),
       ])]
)


def gate_inputs(c):
    rng = np.random.default_rng(c["seed"])
    x = bf16_round(rng.standard_normal(c["V"], dtype=np.float32) * np.float32(c["scale"])
                   + np.float32(c["offset"]))
    hist = [int(h) for h in rng.integers(0, c["V"], c["hist"])]
    return x, hist


# ---------------------------------------------------------------------------
# entropy-gated rollouts (core/generator.py) on tiny seeded models, fp32 so that
# the decode path's 1e-5 agreement keeps every branch / extend decision exact
# ---------------------------------------------------------------------------
ROLLOUT_CASES = {
    "qwen3_fp32": dict(family="qwen3", seed=11, layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64,
                       intermediate=512, vocab=512, prompts=3, prompt_len=24, max_new_tokens=28,
                       max_active_branches=6, branching_factor=3, eos=2),
    "llama_fp32": dict(family="llama", seed=12, layers=2, hidden=256, heads=4, kv_heads=1, head_dim=64,
                       intermediate=512, vocab=384, prompts=2, prompt_len=17, max_new_tokens=24,
                       max_active_branches=8, branching_factor=2, eos=3),
}


def rollout_model(c, device="cpu"):
    """The case's randomly initialised model (same weights on any device)."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM, Qwen3Config, Qwen3ForCausalLM
    kw = dict(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["intermediate"],
              num_hidden_layers=c["layers"], num_attention_heads=c["heads"], num_key_value_heads=c["kv_heads"],
              head_dim=c["head_dim"], max_position_embeddings=4096, eos_token_id=c["eos"])
    torch.manual_seed(c["seed"])
    model = (Qwen3ForCausalLM(Qwen3Config(**kw)) if c["family"] == "qwen3" else
             LlamaForCausalLM(LlamaConfig(**kw)))
    return model.to(device=device, dtype=torch.float32).eval()


def sharpen(model, factor: float = 40.0):
    """The model with its lm_head (untied from the embedding) scaled by ``factor``.

    A tiny random-init model has nearly uniform next-token distributions; in
    bf16 its top log-probs are then mostly exact ties, whose order torch.topk
    leaves implementation-defined, so bf16 trees would part on tie order alone.
    Sharper logits keep the bf16 comparisons about the arithmetic."""
    import torch
    model.lm_head.weight = torch.nn.Parameter(model.lm_head.weight.detach().clone() * factor)
    return model


def rollout_prompts(c):
    rng = np.random.default_rng(c["seed"] + 1000)
    # ids >= 4 keep the prompt clear of the EOS id
    return [rng.integers(4, c["vocab"], c["prompt_len"]).tolist() for _ in range(c["prompts"])]


# ---------------------------------------------------------------------------
# Gate sweep: GATE_SWEEP_BATCHES x GATE_SWEEP_BATCH leaves from seeds, to measure
# the kernel's residual mismatch against the reference's own gate arithmetic.
# A batch shares what one gate launch shares (vocabulary, temperature, active
# count, step); leaves differ in scale, offset, shape, history and EMA.  Every
# eighth leaf is tie-heavy (logits on a coarse grid, so many exactly equal
# log-probs) and every eighth + 1 is peaked (a few logits far above the rest).
# ---------------------------------------------------------------------------
GATE_SWEEP_BATCH = 256
GATE_SWEEP_BATCHES = 40


def gate_sweep_batch(b):
    rng = np.random.default_rng(900_000 + b)
    V = (151936, 128256)[b % 2]
    T = (0.7, 0.7, 1.0, 0.5)[b % 4]
    leaves = []
    for j in range(GATE_SWEEP_BATCH):
        kind = "ties" if j % 8 == 0 else ("peaked" if j % 8 == 1 else "normal")
        leaves.append(dict(kind=kind, seed=int(rng.integers(1 << 31)),
                           scale=float(np.exp(rng.uniform(np.log(0.02), np.log(8.0)))),
                           offset=float(rng.uniform(-3, 3)), hist=int(rng.integers(0, 300)),
                           ema_old=None if rng.random() < 0.2 else float(rng.uniform(1.0, 12.0))))
    return dict(V=V, T=T, penalty=1.2, K=3, M=10, alpha=0.3, mult=1.25, window=10, initial=0.3,
                num_active=int(rng.integers(1, 11)), step=int(rng.integers(0, 20)), leaves=leaves)


def gate_sweep_leaf(batch, leaf):
    """(bf16-valued float32 logits, generated-token history) of one sweep leaf."""
    V = batch["V"]
    rng = np.random.default_rng(leaf["seed"])
    x = rng.standard_normal(V, dtype=np.float32)
    if leaf["kind"] == "ties":
        q = float((2, 4, 8)[leaf["seed"] % 3])
        x = np.round(x * q) / np.float32(q)
    x = x * np.float32(leaf["scale"]) + np.float32(leaf["offset"])
    if leaf["kind"] == "peaked":
        spikes = rng.integers(0, V, 1 + leaf["seed"] % 4)
        x[spikes] += rng.uniform(8.0, 30.0, spikes.size).astype(np.float32)
    hist = rng.integers(0, V, leaf["hist"]).tolist()
    return bf16_round(x.astype(np.float32)), hist
