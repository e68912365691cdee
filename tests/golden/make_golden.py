"""Generate the golden fixtures under ``tests/golden/`` from the reference itself.

Run in the build container, where the reference source tree is importable::

    MENTAT_REF=<path to the reference checkout> python tests/golden/make_golden.py

The GPU box does not have the reference; the tests there read only the files
this script writes.  Inputs are regenerated from numpy ``default_rng`` seeds
(PCG64 is stable across numpy versions), so the fixtures hold seeds, op lists
and expected outputs, not input tensors.

Reference set-up: ``adapters.attention_backend.BACKEND = "sdpa"`` (flash-attn is
installed here but there is no GPU), the allocator's free list is replaced by
``oracle.allocator.FifoFreeList`` (the reference's ``set.pop()`` order is a
CPython detail), and ``torch.set_num_threads(1)`` for the gate (the CPU bf16
``sum`` rounds per-thread partials, which makes the entropy thread-count
dependent).
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
REF = os.environ.get("MENTAT_REF")
if not REF:
    sys.exit("set MENTAT_REF to the reference checkout (the directory holding core/ and adapters/)")
sys.path.insert(0, REF)

import adapters.attention_backend as ab  # noqa: E402

ab.BACKEND = "sdpa"
from core.paged_kv_cache import PagedKVCacheManager  # noqa: E402
from core import generator_utils as gu  # noqa: E402
from core.generator import MentatGenerator  # noqa: E402

from oracle.allocator import FifoFreeList  # noqa: E402
from tests.golden.cases import (  # noqa: E402
    ALLOC_STREAM_PARAMS, ATTN_CASES, GATE_CASES, attn_inputs, build_tree_ops,
    gate_inputs, random_op_stream,
)


def ref_manager(L, hkv, d, max_blocks, bs, dtype, order):
    m = PagedKVCacheManager(L, hkv, d, max_blocks=max_blocks, block_size=bs,
                            device="cpu", dtype=dtype)
    m.allocator._free = FifoFreeList(order)
    return m


def snapshot(m) -> dict:
    return {
        "seqs": {str(sid): {"tables": [list(map(int, t)) for t in s.page_table],
                            "num_tokens": list(s.num_tokens),
                            "tail": list(s.tokens_in_last_block)}
                 for sid, s in sorted(m._sequences.items())},
        "refcounts": list(m.allocator.refcounts),
        "free": m.allocator._free.as_list(),
        "peak": m.allocator.peak_used,
        "stats": m.get_stats(),
    }


def apply_op(m, op, rng_vals):
    kind = op[0]
    if kind == "alloc":
        return m.allocate_sequence()
    if kind == "fork":
        return m.fork_sequence(op[1])
    if kind == "free":
        return m.free_sequence(op[1])
    if kind == "append":
        _, sid, layer, n = op
        k = torch.from_numpy(rng_vals(n, m))
        return m.append_tokens(sid, layer, k, k.clone())
    if kind == "append_batched":
        _, sids, layer = op
        k = torch.from_numpy(rng_vals(len(sids), m))
        return m.append_tokens_batched(seq_ids=sids, layer_idx=layer, k=k, v=k.clone())
    if kind == "trim":
        return m.trim_to_window(op[1], op[2])
    raise ValueError(kind)


def make_alloc_streams():
    streams = []
    for p in ALLOC_STREAM_PARAMS:
        ops = random_op_stream(**p)
        order = np.random.default_rng(p["seed"] + 1000).permutation(p["max_blocks"]).tolist()
        m = ref_manager(p["L"], 1, 2, p["max_blocks"], p["bs"], torch.float32, order)
        vals = lambda n, mm: np.zeros((n, 1, 2), np.float32)  # noqa: E731
        checkpoints, error = [], None
        for i, op in enumerate(ops):
            try:
                apply_op(m, op, vals)
            except Exception as e:  # record and stop, the state after an error is not compared
                error = {"op": i, "type": type(e).__name__, "msg": str(e)}
                break
            if i % 7 == 6 or i == len(ops) - 1:
                checkpoints.append({"op": i, "snap": snapshot(m)})
        streams.append({"params": p, "order": order, "ops": ops,
                        "checkpoints": checkpoints, "error": error})
    (HERE / "alloc_streams.json").write_text(json.dumps(streams))
    print("alloc streams", len(streams))


def make_attention():
    out = {}
    for name, c in ATTN_CASES.items():
        dt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[c["dtype"]]
        inp = attn_inputs(c)
        order = inp["order"]
        m = ref_manager(1, c["hkv"], c["d"], c["pool"], c["bs"], dt, order)
        leaves = []
        for op in build_tree_ops(c):
            if op[0] == "append":
                sid, arr_k, arr_v = op[1], inp[op[2]], inp[op[3]]
                m.append_tokens(sid, 0, torch.from_numpy(arr_k).to(dt),
                                torch.from_numpy(arr_v).to(dt))
            elif op[0] == "alloc":
                m.allocate_sequence()
            elif op[0] == "fork":
                m.fork_sequence(op[1])
            elif op[0] == "free":
                m.free_sequence(op[1])
            elif op[0] == "leaves":
                leaves = op[1]
        q = torch.from_numpy(inp["q"]).to(dt)
        pk, pv, cu, mx = m.build_packed_kv(leaves, 0)
        o = ab.attn_decode(q, pk, pv, torch.arange(len(leaves) + 1, dtype=torch.int32),
                           cu, mx, len(leaves))
        tables = [m._sequences[s].page_table[0] for s in leaves]
        out[f"{name}__out"] = o.float().numpy()
        out[f"{name}__tables"] = np.array([t + [-1] * (max(map(len, tables)) - len(t)) for t in tables], np.int32) if tables and max(map(len, tables)) else np.zeros((len(leaves), 0), np.int32)
        out[f"{name}__lens"] = np.array([m.get_kv_length(s) for s in leaves], np.int32)
        out[f"{name}__cu"] = cu.numpy()
        out[f"{name}__maxlen"] = np.array(mx)
        out[f"{name}__refcounts"] = np.array(m.allocator.refcounts, np.int32)
    np.savez_compressed(HERE / "attention.npz", **out)
    print("attention cases", len(ATTN_CASES))


def make_prefill():
    """The reference's attn_prefill (SDPA backend, CPU) on the prefill cases, in
    the case's dtype; outputs stored as float32."""
    from tests.golden.cases import PREFILL_CASES, prefill_inputs
    out = {}
    for name, c in PREFILL_CASES.items():
        dt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[c[0]]
        q, k, v = (torch.from_numpy(a).to(dt) for a in prefill_inputs(name))
        o = ab.attn_prefill(q, k, v)
        out[f"{name}__out"] = o.float().numpy()
    np.savez_compressed(HERE / "prefill.npz", **out)
    print("prefill cases", len(PREFILL_CASES))


def make_prune():
    """The reference's MentatGenerator._prune_similar on small fake trees: random
    semantic vectors in clusters (so that pairs cross the threshold), parents
    shared by sibling groups or None, log-prob ties, leaves too young to compare,
    and thresholds 0.85 / 0.0 / -0.25.  Stored per case: the similarity matrix the
    reference computes (same torch ops, same process) over the warmed-up leaves,
    their parent keys and log-probs, the threshold rounded to the matrix dtype,
    and the node ids the reference pruned, in its order."""
    from tests.golden.cases import PRUNE_CASES
    out = {}
    for name, c in PRUNE_CASES.items():
        rng = np.random.default_rng(c["seed"])
        dt = {"f32": torch.float32, "bf16": torch.bfloat16}[c["dtype"]]
        m, d = c["m"], 64
        centers = rng.standard_normal((max(1, m // 3), d))
        vecs = centers[rng.integers(0, len(centers), m)] + c["spread"] * rng.standard_normal((m, d))
        pkeys = rng.integers(-1, max(1, m // 4), m)
        pobj = {int(p): SimpleNamespace(pid=int(p)) for p in set(pkeys.tolist()) if p >= 0}
        parents = [pobj[int(p)] if p >= 0 else None for p in pkeys]
        logp = np.round(rng.standard_normal(m) * 3, 1)  # rounded: ties happen
        ages = rng.integers(0, 8, m)
        step = 20
        leaves = [SimpleNamespace(node_id=100 + i, parent=parents[i], creation_step=step - int(ages[i]),
                                  semantic_vector=torch.from_numpy(vecs[i]).to(dt), cumulative_log_prob=float(logp[i]),
                                  is_active=True) for i in range(m)]
        pruned = []

        class Tree:
            def get_active_leaves(self):
                return [lf for lf in leaves if lf.is_active]

            def prune_branch(self, lf):
                lf.is_active = False
                pruned.append(lf.node_id)

        gen = SimpleNamespace(min_steps_before_prune=c["min_age"], semantic_similarity_threshold=c["thr"],
                              diversity_pruning_events=[])
        warm = [lf for lf in leaves if step - lf.creation_step >= c["min_age"]]
        sv = torch.stack([lf.semantic_vector for lf in warm]) if warm else torch.zeros((0, d), dtype=dt)
        sim = torch.mm(F.normalize(sv, p=2, dim=1), F.normalize(sv, p=2, dim=1).t()) if len(warm) else sv[:, :0]
        MentatGenerator._prune_similar(gen, Tree(), step)
        out[name] = {
            "sim": sim.float().numpy().tolist(),
            "parent": [lf.parent.pid if lf.parent is not None else None for lf in warm],
            "logp": [lf.cumulative_log_prob for lf in warm],
            "node_id": [lf.node_id for lf in warm],
            "thr": float(torch.tensor(c["thr"], dtype=dt).item()),
            "dtype": c["dtype"],
            "pruned": pruned,
        }
    with open(HERE / "prune.json", "w") as f:
        json.dump(out, f)
    print("prune cases", len(PRUNE_CASES))


def make_gate():
    torch.set_num_threads(1)
    gen_self = SimpleNamespace(soft_explore_window=None, soft_explore_initial=None)
    res = []
    for c in GATE_CASES:
        x32, hist = gate_inputs(c)
        x = torch.from_numpy(x32).to(torch.bfloat16)
        assert np.array_equal(x.float().numpy(), x32), "inputs must be bf16 values"
        H = gu.compute_entropy(x, c["T"])
        pen = gu.apply_repetition_penalty(x, hist, penalty=c["penalty"])
        lp = F.log_softmax(pen, dim=-1)
        am = int(torch.argmax(lp).item())
        tv, ti = torch.topk(lp, c["K"])
        gen_self.soft_explore_window = c["window"]
        gen_self.soft_explore_initial = c["initial"]
        ema_old = c["ema_old"]
        ema = H if ema_old is None else (c["alpha"] * H) + ((1.0 - c["alpha"]) * ema_old)
        dyn = gu.adaptive_threshold(c["mult"], c["M"], c["num_active"])
        warm = MentatGenerator._soft_explore_factor(gen_self, c["step"])
        tau = ema * dyn * warm
        branch = (H > tau) and ((c["M"] - c["num_active"]) >= c["K"])
        res.append({
            "case": c, "entropy": H, "ema": ema, "tau": tau, "branch": bool(branch),
            "argmax": am, "argmax_lp": float(lp[am].item()),
            "topk_ids": ti.tolist(), "topk_lps": tv.float().tolist(),
            "pen_entropy": gu.compute_entropy(pen),
            "lp_sha": int(np.frombuffer(lp.view(torch.int16).numpy().tobytes(), np.uint8).astype(np.uint64).sum()),
        })
    (HERE / "gate.json").write_text(json.dumps(res))
    print("gate cases", len(res))


def make_gate_sweep():
    """The reference's gate outputs for every leaf of the sweep (tests/golden/cases.py),
    computed with its own functions on CPU (one thread, as for make_gate)."""
    from tests.golden.cases import GATE_SWEEP_BATCHES, GATE_SWEEP_BATCH, gate_sweep_batch, gate_sweep_leaf
    torch.set_num_threads(1)
    n = GATE_SWEEP_BATCHES * GATE_SWEEP_BATCH
    out = {k: np.zeros(n, np.float64) for k in ("entropy", "pen_entropy", "ema", "tau")}
    out.update(branch=np.zeros(n, np.bool_), argmax=np.zeros(n, np.int32), argmax_lp=np.zeros(n, np.float32),
               topk_ids=np.zeros((n, 3), np.int32), topk_lps=np.zeros((n, 3), np.float32),
               topk_ties=np.zeros((n, 3), np.int32))
    gen_self = SimpleNamespace(soft_explore_window=None, soft_explore_initial=None)
    i = 0
    for b in range(GATE_SWEEP_BATCHES):
        c = gate_sweep_batch(b)
        gen_self.soft_explore_window, gen_self.soft_explore_initial = c["window"], c["initial"]
        dyn = gu.adaptive_threshold(c["mult"], c["M"], c["num_active"])
        warm = MentatGenerator._soft_explore_factor(gen_self, c["step"])
        for leaf in c["leaves"]:
            x32, hist = gate_sweep_leaf(c, leaf)
            x = torch.from_numpy(x32).to(torch.bfloat16)
            H = gu.compute_entropy(x, c["T"])
            pen = gu.apply_repetition_penalty(x, hist, penalty=c["penalty"])
            lp = F.log_softmax(pen, dim=-1)
            am = int(torch.argmax(lp).item())
            tv, ti = torch.topk(lp, c["K"])
            eo = leaf["ema_old"]
            ema = H if eo is None else (c["alpha"] * H) + ((1.0 - c["alpha"]) * eo)
            tau = ema * dyn * warm
            out["entropy"][i], out["ema"][i], out["tau"][i] = H, ema, tau
            out["branch"][i] = (H > tau) and ((c["M"] - c["num_active"]) >= c["K"])
            out["argmax"][i], out["argmax_lp"][i] = am, float(lp[am].item())
            out["topk_ids"][i], out["topk_lps"][i] = ti.numpy(), tv.float().numpy()
            # how many log-probs of the whole vocabulary equal each top-K value: the
            # order of equal values is implementation-defined in torch.topk
            out["topk_ties"][i] = [int((lp == v).sum()) for v in tv]
            out["pen_entropy"][i] = gu.compute_entropy(pen)
            i += 1
        print("gate sweep batch", b, flush=True)
    np.savez_compressed(HERE / "gate_sweep.npz", **out)


class _StubTokenizer:
    """The generator's tokenizer interface over space-separated token ids."""

    def __init__(self, eos):
        self.eos_token_id = eos

    def __call__(self, prompt, return_tensors="pt"):
        return {"input_ids": torch.tensor([[int(t) for t in prompt.split()]], dtype=torch.long)}

    def decode(self, ids, skip_special_tokens=True):
        return " ".join(str(int(t)) for t in ids)


def make_rollout():
    from tests.golden.cases import ROLLOUT_CASES, rollout_model, rollout_prompts
    torch.set_num_threads(1)
    out = {}
    for name, c in ROLLOUT_CASES.items():
        model = rollout_model(c)
        runs = []
        for prompt in rollout_prompts(c):
            gen = MentatGenerator(model, _StubTokenizer(c["eos"]), max_active_branches=c["max_active_branches"],
                                  branching_factor=c["branching_factor"], max_new_tokens=c["max_new_tokens"],
                                  block_size=16, max_blocks=2048)
            res = gen.generate(" ".join(map(str, prompt)))
            d = gen.get_diagnostics()
            runs.append({"results": [{"token_ids": r["token_ids"], "log_prob": r["log_prob"]} for r in res],
                         "branch_points": [[s, n] for s, _, n in d["branch_points"]],
                         "active_branch_trace": d["active_branch_trace"],
                         "decode_tokens_total": d["decode_tokens_total"],
                         "diversity_pruning_events": d["diversity_pruning_events"]})
        out[name] = runs
    with open(HERE / "rollout.json", "w") as f:
        json.dump(out, f)


if __name__ == "__main__":
    parts = sys.argv[1:] or ["alloc", "attention", "prefill", "prune", "gate", "rollout", "gate_sweep"]
    for part in parts:
        globals()[f"make_{part}" if part != "alloc" else "make_alloc_streams"]()
