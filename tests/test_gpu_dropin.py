"""The reference's unmodified generator and adapters on this package (the drop-in).

``tests/dropin_child.py`` runs the reference's ``MentatGenerator`` (the copy
pip-installed under ``baseline/_ref``) in a process of its own.  With this
package's module aliases installed first, the reference's Qwen3 and Llama
adapters (``qwen3_adapter.py:223-269``, ``llama_adapter.py:174-213``) pass the
``PagedKV`` handles of this package's ``build_packed_kv`` straight into its
``attn_decode``, and the generator drives this package's cache (fork, free,
batched append with copy-on-write).

* fp32: the trees must be the ones the reference produced on CPU with its own
  cache and SDPA (``tests/golden/rollout.json``), exactly.
* bf16: three runs of the same seeded tiny models are compared step by step:
  the reference as it ships (its cache; flash-attn, or its SDPA path when
  flash-attn has no kernels for the GPU), the reference on this package's
  backend, and this package's own ``TreeRollout`` (fused gate, device-planned
  steps).  bf16 rounding differs between attention implementations, so the
  trees are allowed to part; the test reports where and how often the
  per-leaf decisions agree, and requires this package's rollout to make the
  same decisions as the reference's generator on the same backend.

Skipped when the reference is not installed under ``baseline/_ref``.
"""

import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from tests.golden.cases import ROLLOUT_CASES, rollout_model, rollout_prompts, sharpen

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(os.path.dirname(HERE), "baseline", "_ref")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "core")),
                                 reason="the reference is not installed under baseline/_ref")]

GOLDEN = json.load(open(os.path.join(HERE, "golden", "rollout.json")))


def _child(mode, specs, tmp_path):
    out = tmp_path / f"{mode}.json"
    r = subprocess.run([sys.executable, os.path.join(HERE, "dropin_child.py"), mode, str(out), *specs],
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-4000:]
    with open(out) as f:
        return json.load(f)


def test_reference_generator_on_this_backend_fp32(tmp_path):
    got = _child("mentat", sorted(ROLLOUT_CASES), tmp_path)
    assert got["backend"] == "mentat_b200"
    for name in sorted(ROLLOUT_CASES):
        for i, run in enumerate(got["cases"][name]):
            want = GOLDEN[name][i]
            assert [r["token_ids"] for r in run["results"]] == [r["token_ids"] for r in want["results"]], \
                f"{name} prompt {i}"
            np.testing.assert_allclose([r["log_prob"] for r in run["results"]],
                                       [r["log_prob"] for r in want["results"]], rtol=1e-4, atol=1e-4)
            assert run["decode_tokens_total"] == want["decode_tokens_total"]


def _compare(a_steps, b_steps):
    """First step whose active leaves differ (None: never), and the fraction of
    leaves present in both runs at a step whose successors at the next step
    (the leaf extended by one token, its K children, or nothing after EOS or
    pruning) are the same in both runs."""
    first = None
    agree = total = 0
    for s in range(min(len(a_steps), len(b_steps))):
        A, B = [tuple(x) for x in a_steps[s]], [tuple(x) for x in b_steps[s]]
        if first is None and A != B:
            first = s + 1  # decode steps count from 1
        if s + 1 >= min(len(a_steps), len(b_steps)):
            break
        nA, nB = [tuple(x) for x in a_steps[s + 1]], [tuple(x) for x in b_steps[s + 1]]
        for leaf in set(A) & set(B):
            succ = lambda nxt: sorted(x for x in nxt if len(x) == len(leaf) + 1 and x[:len(leaf)] == leaf)  # noqa
            total += 1
            agree += succ(nA) == succ(nB)
    if first is None and len(a_steps) != len(b_steps):
        first = min(len(a_steps), len(b_steps)) + 1
    return first, (agree / total if total else 1.0), total


def _our_rollout_steps(name, log_softmax):
    from mentat_b200.rollout import TreeRollout
    c = ROLLOUT_CASES[name]
    model = sharpen(rollout_model(c, device="cuda").to(torch.bfloat16))
    runs = []
    for p in rollout_prompts(c):
        r = TreeRollout(model, eos_token_id=c["eos"], max_active_branches=c["max_active_branches"],
                        branching_factor=c["branching_factor"], max_new_tokens=c["max_new_tokens"], block_size=16,
                        max_blocks=4096, log_softmax=log_softmax)
        r.trace = []
        r.generate(p)
        runs.append([t[0] for t in r.trace])
    return runs


def test_bf16_trees_step_by_step(tmp_path):
    specs = [f"{name}:bf16" for name in sorted(ROLLOUT_CASES)]
    ref = _child("reference", specs, tmp_path)
    drop = _child("mentat", specs, tmp_path)
    report = {"reference_backend": ref["backend"], "cases": {}}
    for spec in specs:
        ours = {mode: _our_rollout_steps(spec.split(":")[0], mode) for mode in ("cpu", "cuda")}
        rows = []
        for i, (r, d) in enumerate(zip(ref["cases"][spec], drop["cases"][spec])):
            f1, a1, n1 = _compare(r["steps"], d["steps"])
            row = {"prompt": i, "steps": len(r["steps"]),
                   "reference_vs_dropin": {"first_divergence_step": f1, "leaf_agreement": a1, "leaves": n1}}
            for mode, runs in ours.items():
                f2, a2, n2 = _compare(d["steps"], runs[i])
                row[f"dropin_vs_rollout_{mode}"] = {"first_divergence_step": f2, "leaf_agreement": a2, "leaves": n2}
            rows.append(row)
        report["cases"][spec] = rows
    path = os.environ.get("MENTAT_BF16_TREES_OUT")
    if path:
        with open(path, "w") as f:
            json.dump(report, f, indent=1)
    for spec, rows in report["cases"].items():
        for row in rows:
            assert row["reference_vs_dropin"]["leaf_agreement"] >= 0.8, (spec, row)
            # the same model arithmetic and attention kernel as the reference's generator on this
            # backend, and the gate in torch's CUDA rounding: the same decisions
            assert row["dropin_vs_rollout_cuda"]["leaf_agreement"] >= 0.95, (spec, row)


def test_gate_vs_reference_on_cuda():
    """The fused gate against the reference's own gate functions run on CUDA
    (compute_entropy, apply_repetition_penalty, log_softmax + argmax / topk, from
    baseline/_ref) on the same bf16 logits: the first 2,048 leaves of the gate
    sweep.  With log_softmax="cuda" the kernel rounds like torch's CUDA kernels;
    the remaining differences come from the softmax sum's summation order.  The
    reference's CUDA results are also compared with its CPU ones (the sweep
    fixture) to show how far the reference agrees with itself across devices."""
    import torch.nn.functional as F
    from mentat_b200.gate import GateConfig, gate_step
    from tests.golden.cases import gate_sweep_batch, gate_sweep_leaf
    sys.path.insert(0, REF)
    try:
        import core.generator_utils as rgu
    finally:
        sys.path.remove(REF)
    g = np.load(os.path.join(HERE, "golden", "gate_sweep.npz"))
    fields = ("entropy", "branch", "argmax", "topk_set")
    miss = {pair: dict.fromkeys(fields, 0) for pair in ("kernel_cuda_vs_ref_cuda", "ref_cuda_vs_ref_cpu")}
    n = 0
    for b in range(8):
        c = gate_sweep_batch(b)
        xs, hists = zip(*(gate_sweep_leaf(c, leaf) for leaf in c["leaves"]))
        logits = torch.from_numpy(np.stack(xs)).cuda().to(torch.bfloat16)
        cfg = GateConfig(temperature=c["T"], repetition_penalty=c["penalty"], entropy_ema_alpha=c["alpha"],
                         relative_entropy_multiplier=c["mult"], soft_explore_initial=c["initial"],
                         branching_factor=c["K"], max_active_branches=c["M"], soft_explore_window=c["window"],
                         log_softmax="cuda")
        out = gate_step(logits, list(hists), [leaf["ema_old"] for leaf in c["leaves"]], cfg,
                        num_active=c["num_active"], step=c["step"])
        dyn = rgu.adaptive_threshold(c["mult"], c["M"], c["num_active"])
        warm = 1.0 if c["step"] >= c["window"] else c["initial"] + (1.0 - c["initial"]) * c["step"] / c["window"]
        for j, leaf in enumerate(c["leaves"]):
            x = logits[j]
            H = rgu.compute_entropy(x, c["T"])
            pen = rgu.apply_repetition_penalty(x, hists[j], penalty=c["penalty"])
            lp = F.log_softmax(pen, dim=-1)
            am = int(torch.argmax(lp).item())
            top = set(torch.topk(lp, c["K"]).indices.tolist())
            eo = leaf["ema_old"]
            ema = H if eo is None else (c["alpha"] * H) + ((1.0 - c["alpha"]) * eo)
            br = (H > ema * dyn * warm) and (c["M"] - c["num_active"] >= c["K"])
            o = out[j]
            i = n + j
            k = miss["kernel_cuda_vs_ref_cuda"]
            k["entropy"] += int(o["entropy"] != H)
            k["branch"] += int(bool(o["branch"]) != br)
            k["argmax"] += int(int(o["argmax"]) != am)
            k["topk_set"] += int(set(int(t) for t in o["topk_ids"][:c["K"]]) != top)
            r = miss["ref_cuda_vs_ref_cpu"]
            r["entropy"] += int(H != g["entropy"][i])
            r["branch"] += int(br != bool(g["branch"][i]))
            r["argmax"] += int(am != int(g["argmax"][i]))
            r["topk_set"] += int(top != set(g["topk_ids"][i].tolist()))
        n += len(c["leaves"])
    rates = {pair: {f: v / n for f, v in m.items()} for pair, m in miss.items()}
    path = os.environ.get("MENTAT_GATE_CUDA_OUT")
    if path:
        with open(path, "w") as f:
            json.dump({"leaves": n, "mismatches": miss, "rates": rates}, f, indent=1)
    k = rates["kernel_cuda_vs_ref_cuda"]
    assert k["branch"] <= 0.01 and k["argmax"] <= 0.01, rates
