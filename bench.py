"""Benchmark of the tree-aware paged decode attention (benchmark config 4).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mentat|reference]

Workload (benchmark config 4): bf16, 32 q / 8 kv heads, head_dim 128, KV
block 16; one 32768-token shared prefix and 64 branches with suffixes drawn
from U[1024, 4096] (seeded).  A step is one ``attn_decode`` over the 64
branches (plan + units + merge kernels).  The unique KV of a step (~0.8 GB) is
larger than the 126 MB L2, so no flush is needed between steps.

metric: decode-attn unique-KV HBM GB/s = distinct physical blocks' valid
tokens x Hkv x D x 2 (K, V) x 2 B per step / step time; the whole-job
aggregate over ranks (each rank decodes its own tree: weak scaling, no
collective on the data path).

``--impl reference`` times the reference's CPU path (oracle/cpu_path.py: the
reference's build_packed_kv + _sdpa_decode restated with the same torch CPU
ops) on the host cores, on a bounded sample of the same tree.
"""

from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HQ, HKV, D, BS = 32, 8, 128, 16
PREFIX, NBR, SUF_LO, SUF_HI = 32768, 64, 1024, 4096
ELEM = 2
METRIC = "decode-attn unique-KV HBM GB/s"


def _env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def combine_ranks(ms, e2e_ms, kv_bytes, e2e_bytes, device, world):
    """Whole-job GB/s of the device-timed loop and of the end-to-end loop.

    Every rank decodes its own tree, so the job moves the sum of the ranks'
    bytes in the time of the slowest rank (max over ranks of its device time).
    Returns (value, e2e value, slowest device time in ms, [(ms, bytes)] per rank)."""
    import torch.distributed as dist
    mine = torch.tensor([ms, e2e_ms, float(kv_bytes), float(e2e_bytes)], dtype=torch.float64, device=device)
    rows = [mine.clone() for _ in range(world)]
    if world > 1:
        dist.all_gather(rows, mine)
    rows = [r.tolist() for r in rows]
    ms_max, e2e_max = max(r[0] for r in rows), max(r[1] for r in rows)
    kv_all, e2e_all = sum(r[2] for r in rows), sum(r[3] for r in rows)
    return (kv_all / (ms_max / 1e3) / 1e9, e2e_all / (e2e_max / 1e3) / 1e9, ms_max,
            [(r[0], r[2]) for r in rows])


def suffixes(seed):
    return np.random.default_rng(seed).integers(SUF_LO, SUF_HI + 1, NBR)


def unique_bytes(prefix, suffix_tokens):
    return int((prefix + int(np.sum(suffix_tokens))) * HKV * D * 2 * ELEM)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic():
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


class Clocks:
    """nvidia-smi sampler running while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100", "-i", str(self.gpu_id)], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.p.kill()
            out, _ = self.p.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def build_shape(prefix, suf, seed, device, extra_blocks):
    """A shared prefix forked into len(suf) branches with the given own lengths."""
    from mentat_b200 import PagedKVCacheManager
    nbr = len(suf)
    blocks = prefix // BS + int(sum((s + BS - 1) // BS for s in suf)) + extra_blocks + 16
    m = PagedKVCacheManager(1, HKV, D, max_blocks=blocks, block_size=BS, device=device, dtype=torch.bfloat16,
                            max_seqs=nbr + 2)
    g = torch.Generator(device=device).manual_seed(seed)
    kv = lambda n: torch.randn((n, HKV, D), generator=g, device=device).to(torch.bfloat16)  # noqa: E731
    root = m.allocate_sequence()
    for a in range(0, prefix, 8192):
        n = min(8192, prefix - a)
        m.append_tokens(root, 0, kv(n), kv(n))
    kids = [m.fork_sequence(root) for _ in range(nbr)]
    m.free_sequence(root)
    for kid, n in zip(kids, suf):
        m.append_tokens(kid, 0, kv(int(n)), kv(int(n)))
    q = torch.randn((nbr, HQ, D), generator=g, device=device).to(torch.bfloat16)
    m.check()
    return m, kids, q


def build_tree(seed, device, extra_blocks, value_seed=None):
    """Config 4's tree: suffix lengths drawn from `seed`, K/V and q values from
    `value_seed` (default `seed`)."""
    suf = suffixes(seed)
    m, kids, q = build_shape(PREFIX, suf, seed if value_seed is None else value_seed, device, extra_blocks)
    return m, kids, q, suf


TREE_CONFIGS = {
    # benchmark config 2: Qwen3-0.6B architecture, random init, bf16; 4 prompts of 256
    # uniform-random ids, 256 new tokens, at most 8 leaves per tree, KV block 16; one
    # B200 (under torchrun every rank rolls out its own 4 prompts: weak scaling)
    2: dict(family="qwen3", vocab=151936, hidden=1024, intermediate=3072, layers=28, heads=16, kv_heads=8,
            head_dim=128, rope_theta=1000000.0, prompts=4, prompt_len=256, max_new_tokens=256, max_active=8,
            eos=151645, shard=False, graphs=True),
    # benchmark config 3: Llama-3.1-8B architecture, random init, bf16; 64 prompts of
    # 2048 ids, trees of up to 16 leaves, 512 new tokens; the 64 trees are sharded
    # across the ranks (strong scaling)
    3: dict(family="llama", vocab=128256, hidden=4096, intermediate=14336, layers=32, heads=32, kv_heads=8,
            head_dim=128, rope_theta=500000.0, prompts=64, prompt_len=2048, max_new_tokens=512, max_active=16,
            eos=128001, shard=True, graphs=True, bucket=64),
    # benchmark config 5: Qwen3-32B architecture, random init, bf16; 32 prompts of 4096
    # ids, trees of up to 32 leaves, 1024 new tokens; tensor parallel by KV head over
    # the ranks (one KV head per GPU at 8), NCCL all-reduce after o_proj and down_proj
    5: dict(family="qwen3", vocab=151936, hidden=5120, intermediate=25600, layers=64, heads=64, kv_heads=8,
            head_dim=128, rope_theta=1000000.0, prompts=32, prompt_len=4096, max_new_tokens=1024, max_active=32,
            eos=151645, shard=False, graphs=True, bucket=64, tp=True, tie=False, min_world=4),
}


def tree_model(c, device, seed):
    """A random-init model of a tree configuration's architecture, in bf16."""
    torch.manual_seed(seed)
    if c["family"] == "qwen3":
        from transformers import Qwen3Config as Cfg, Qwen3ForCausalLM as Model
        cfg = Cfg(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["intermediate"],
                  num_hidden_layers=c["layers"], num_attention_heads=c["heads"], num_key_value_heads=c["kv_heads"],
                  head_dim=c["head_dim"], max_position_embeddings=40960, rms_norm_eps=1e-6,
                  rope_theta=c["rope_theta"], tie_word_embeddings=c.get("tie", True), eos_token_id=c["eos"])
    else:
        from transformers import LlamaConfig as Cfg, LlamaForCausalLM as Model
        cfg = Cfg(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["intermediate"],
                  num_hidden_layers=c["layers"], num_attention_heads=c["heads"], num_key_value_heads=c["kv_heads"],
                  head_dim=c["head_dim"], max_position_embeddings=131072, rms_norm_eps=1e-5,
                  rope_theta=c["rope_theta"], tie_word_embeddings=False, eos_token_id=c["eos"],
                  rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                "high_freq_factor": 4.0, "original_max_position_embeddings": 8192})
    dt = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)  # initialise the weights in bf16 directly
    try:
        with torch.device(device):
            model = Model(cfg).eval()
    finally:
        torch.set_default_dtype(dt)
    return model


def _model_flops_per_token(model) -> float:
    """2 x the parameters every decoded token multiplies (embedding table excluded)."""
    n = sum(p.numel() for name, p in model.named_parameters() if "embed_tokens" not in name)
    return 2.0 * n


def tree_measure(cfg_id, seed, rank, world, device):
    """Tree tokens/s of the entropy-gated rollout on a benchmark model configuration
    (``generator.py:508-511``): decode tokens (one per active leaf per step) over
    decode wall time, summed over the trees; the slowest rank's time.  The branch
    threshold is the 90th percentile of the gate entropies of a seeded 32-step
    warm-up rollout (random-init weights make the adaptive threshold meaningless).
    A full warm-up rollout captures the decode graphs before the timed one.  With
    world > 1 the process group must be up.  Returns a dict (rank 0's view)."""
    import torch.distributed as dist
    from mentat_b200 import _lib
    from mentat_b200.rollout import TreeRollout
    c = TREE_CONFIGS[cfg_id]
    tp = bool(c.get("tp"))
    if world < c.get("min_world", 1):
        return {"unavailable": f"needs >= {c['min_world']} GPUs (KV cache of the tree)"}
    model = tree_model(c, device, seed)
    if tp and world > 1:
        from mentat_b200.tp import shard_model
        full, model = model, shard_model(model, rank, world)
        del full
        torch.cuda.empty_cache()
    if tp:  # every rank rolls out the same trees over its KV heads
        rng = np.random.default_rng(seed * 1000)
        prompts = [rng.integers(0, c["vocab"], c["prompt_len"]).tolist() for _ in range(c["prompts"])]
    elif c["shard"]:
        rng = np.random.default_rng(seed * 1000)
        allp = [rng.integers(0, c["vocab"], c["prompt_len"]).tolist() for _ in range(c["prompts"])]
        prompts = allp[rank::world]
    else:
        rng = np.random.default_rng(seed * 1000 + rank)
        prompts = [rng.integers(0, c["vocab"], c["prompt_len"]).tolist() for _ in range(c["prompts"])]
    M, K = c["max_active"], 3
    n_trees = len(prompts)
    # every live leaf of every tree at once, plus the children of one step's branches
    max_seqs = n_trees * (M + K) + 16 + c.get("bucket", 0)  # + the padding of the last graph bucket
    # a tree's prompt blocks are shared; each live leaf owns at most its generated blocks + a CoW'd tail
    blocks = n_trees * (-(-c["prompt_len"] // 16) + (M + K) * (-(-c["max_new_tokens"] // 16) + 2)) + 64
    r = TreeRollout(model, eos_token_id=c["eos"], max_active_branches=M, branching_factor=K,
                    max_new_tokens=c["max_new_tokens"], max_blocks=blocks, max_seqs=max_seqs,
                    cuda_graphs=c["graphs"], static_decode=not c["graphs"], graph_bucket=c.get("bucket"),
                    max_prompt_len=c["prompt_len"],
                    max_blocks_per_seq=-(-(c["prompt_len"] + c["max_new_tokens"]) // 16) + 2,
                    tp_group=dist.group.WORLD if tp and world > 1 else None)
    lib = _lib.load()
    t_setup = time.perf_counter()
    thr = r.calibrate_threshold(prompts, steps=32, q=90.0)
    if c["graphs"]:
        r.generate_many(prompts)  # warm-up: captures the decode graphs (one per bucket of leaf counts)
    else:
        full = r.max_new_tokens
        r.max_new_tokens = 16     # warm-up of the eager path
        r.generate_many(prompts)
        r.max_new_tokens = full
    warm_s = time.perf_counter() - t_setup
    r.decode_tokens, r.decode_time_s, r.steps, r.step_leaves = 0, 0.0, 0, []
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = lib.mentat_kernel_launch_count() + r.lm.graph_kernel_launches
    clocks = Clocks("GPU-" + str(torch.cuda.get_device_properties(device).uuid))
    clocks.start()
    results = r.generate_many(prompts)
    clk = clocks.stop()
    launches = lib.mentat_kernel_launch_count() + r.lm.graph_kernel_launches - launches0
    # lower bound of this rank's decode time: per step, the weights plus every tree's
    # prompt KV cross HBM once, and the GEMMs do 2 x params flops per decoded token
    peak_bw, _ = peaks()
    peak_fl = _peak_flops()
    kv_tok = 2 * c["kv_heads"] // (world if tp else 1) * c["head_dim"] * 2 * c["layers"]
    w_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
    fl_tok = _model_flops_per_token(model)
    bound_s = sum(max((w_bytes + n_trees * c["prompt_len"] * kv_tok) / (peak_bw * 1e9), n * fl_tok / (peak_fl * 1e12))
                  for n in r.step_leaves)
    stat = torch.tensor([r.decode_time_s, float(r.decode_tokens), bound_s, float(r.steps)], dtype=torch.float64,
                        device=device)
    per_rank = [stat.clone() for _ in range(world)]
    if world > 1:
        dist.all_gather(per_rank, stat)
    per_rank = [x.tolist() for x in per_rank]
    secs = max(x[0] for x in per_rank)
    tokens = per_rank[0][1] if tp else sum(x[1] for x in per_rank)
    leaves = [len(x) for x in results]
    arch = {2: "Qwen3-0.6B", 3: "Llama-3.1-8B", 5: "Qwen3-32B"}[cfg_id]
    out = {
        "metric": f"tree tokens/s (config {cfg_id})", "value": round(tokens / secs, 2), "unit": "tokens/s",
        "n_gpus": world, "steps": r.steps, "ms_per_step": secs / max(r.steps, 1) * 1e3,
        "scaling": "strong" if c["shard"] or tp else "weak",
        "workload": f"BASELINE config {cfg_id}: {arch} architecture, {c['prompts']} prompts x {c['prompt_len']} ids"
                    f"{' split across the ranks' if c['shard'] else (' on every rank' if tp else ' per rank')}, "
                    f"{c['max_new_tokens']} new tokens, <= {M} leaves per tree",
        "decode_tokens": int(tokens), "trees_rank0": n_trees, "entropy_threshold_rank0": round(thr, 4),
        "leaves_per_tree_final_rank0": [min(leaves), float(np.mean(leaves)), max(leaves)],
        "per_rank_s": [round(x[0], 3) for x in per_rank], "per_rank_tokens": [int(x[1]) for x in per_rank],
        "roofline": {"bound_s_rank0": round(per_rank[0][2], 3), "frac_rank0": round(per_rank[0][2] / per_rank[0][0], 4),
                     "frac_slowest": round(max(x[2] for x in per_rank) / secs, 4),
                     "what": "per step max(weights + the trees' prompt KV over measured HBM GB/s, "
                             "2 x params x leaves over measured sustained bf16 TFLOP/s); a lower bound of the "
                             "decode time (generated-token KV and attention flops not counted)"},
        "parallelism": (f"tensor parallel by KV head x{world} (NCCL all-reduce after o_proj and down_proj)"
                        if tp and world > 1 else f"independent trees x{world}"),
        "gpu_launches": int(launches),  # host launches plus the library kernels inside each graph replayed
        "clocks": clk, "setup_and_warmup_s": round(warm_s, 1),
        "note": (("decode steps run as CUDA graphs" + (f" (leaf counts padded to multiples of {c['bucket']})"
                                                       if c.get("bucket") else "")) if c["graphs"] else
                 "eager decode steps planned on the device (no per-layer host work)")
                + "; all trees of a rank advance in lockstep, one forward pass per step; branch threshold = "
                  "90th percentile of a 32-step warm-up's gate entropies",
    }
    # graphs that hold NCCL calls (tensor parallel) go before the process group does
    r.lm._graphs = None
    del r, model
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return out


def _peak_flops(burst=False):
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if burst:
            return float(d["bf16_tflops"])
        return float(d.get("bf16_tflops_sustained") or d["bf16_tflops"])
    return 1590.0 if burst else 1400.0


def run_tree(args):
    """``--tree-config N``: tree tokens/s of one benchmark model configuration as
    its own JSON line (config 2: every rank rolls out its own prompts, weak
    scaling; config 3: the prompts are split across the ranks, strong scaling;
    config 5: tensor parallel by KV head)."""
    import torch.distributed as dist
    rank, world, local = _env_rank()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=600))
    out = tree_measure(args.tree_config, args.seed, rank, world, device)
    if rank == 0:
        line = {"metric": out.pop("metric", f"tree tokens/s (config {args.tree_config})")}
        if "unavailable" not in out:
            line.update({"value": out.pop("value"), "unit": out.pop("unit"), "n_gpus": world,
                         "steps": out.pop("steps"), "warmup": 1, "ms_per_step": out.pop("ms_per_step"),
                         "higher_is_better": True, "scaling": out.pop("scaling"), "vs_baseline": None,
                         "dtype": "bf16", "data": "synthetic (random-init weights, seeded uniform-random prompt ids)",
                         "config": {"workload": out.pop("workload"), "parallelism": out.pop("parallelism")},
                         "gpu_launches": out.pop("gpu_launches"), "clocks": out.pop("clocks")})
        line.update(out)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_profile_kernels(args):
    """The gate, append, fork / free and FFMA decode kernels on benchmark-sized
    inputs, for a profiler capture: the gate over 32 leaves x 151936 bf16 logits
    (config 2's vocabulary) with 200-token histories; one-token batched appends to
    the 64 branches of the config-4 tree (the first append after the forks copies
    every branch's partial tail block); fork + free of one of its branches; and
    config 1's fp32 decode.  Prints time per call and algorithmic GB/s."""
    from mentat_b200.gate import GATE_OUT_DTYPE, Gate, GateConfig
    device = torch.device("cuda", 0)
    steps = max(args.steps, 1)
    n, V = 32, 151936
    g = torch.Generator(device=device).manual_seed(args.seed)
    logits = (torch.randn((n, V), generator=g, device=device) * 2.0).to(torch.bfloat16)
    rng = np.random.default_rng(args.seed)
    hist = [rng.integers(0, V, 200).tolist() for _ in range(n)]
    gate = Gate(device, GateConfig(max_active_branches=64))
    for _ in range(args.warmup):
        gate.launch(logits, hist, [5.0] * n, num_active=n, step=3)
        gate.result()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        gate.launch(logits, hist, [5.0] * n, num_active=n, step=3)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    # the kernel alone: the same operator call, `steps` times in one CUDA graph
    c = gate.cfg
    nb = n * GATE_OUT_DTYPE.itemsize
    op_args = (logits, gate._ptr_dev[: n + 1], gate._hist_dev, gate._ema_dev[:n],
               [c.temperature, c.repetition_penalty, c.entropy_ema_alpha, c.relative_entropy_multiplier,
                c.soft_explore_initial],
               [c.branching_factor, c.max_active_branches, n, 3, c.soft_explore_window], gate._out_dev[:nb])
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(steps):
            torch.ops.mentat_b200.gate_step(*op_args)
    graph.replay()
    torch.cuda.synchronize()
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    kms = e0.elapsed_time(e1) / steps
    del graph
    print(f"gate: {n} x {V} bf16 logits, {ms * 1e3:.1f} us/call through Gate.launch, {kms * 1e3:.1f} us/kernel "
          f"({n * V * 2 / kms / 1e6:.1f} GB/s of logits)", flush=True)
    m, kids, q, suf = build_tree(args.seed, device, extra_blocks=NBR * (args.warmup + steps + 2))
    kv = torch.randn((args.warmup + steps, 2, NBR, HKV, D), generator=g, device=device).to(torch.bfloat16)
    for i in range(args.warmup):
        m.append_tokens_batched(kids, 0, kv[i, 0], kv[i, 1])
    torch.cuda.synchronize()
    e0.record()
    for i in range(steps):
        m.append_tokens_batched(kids, 0, kv[args.warmup + i, 0], kv[args.warmup + i, 1])
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    nb = NBR * HKV * D * 2 * ELEM
    print(f"append: {NBR} sequences x 1 token, {ms * 1e3:.1f} us/call, {nb / ms / 1e6:.2f} GB/s of K/V rows",
          flush=True)
    # fork + free of one branch of the config-4 tree (k_fork refs its 2,000+ blocks,
    # k_free releases them)
    e0.record()
    for _ in range(steps):
        m.free_sequence(m.fork_sequence(kids[0]))
    e1.record()
    torch.cuda.synchronize()
    print(f"fork+free: one branch of {m.get_kv_length(kids[0])} tokens, "
          f"{e0.elapsed_time(e1) / steps * 1e3:.1f} us per pair", flush=True)
    m.check()
    del m
    # benchmark config 1 in fp32 (the FFMA unit kernel): Hq 16, Hkv 8, D 128, block 16,
    # 8 branches sharing a 512-token prefix, 64 tokens of their own each
    from mentat_b200 import PagedKVCacheManager
    from mentat_b200.attention_backend import attn_decode
    m1 = PagedKVCacheManager(1, 8, 128, max_blocks=1024, block_size=16, device=device, dtype=torch.float32,
                             max_seqs=16)
    kv = lambda n: torch.randn((n, 8, 128), generator=g, device=device)  # noqa: E731
    root = m1.allocate_sequence()
    m1.append_tokens(root, 0, kv(512), kv(512))
    br = [m1.fork_sequence(root) for _ in range(8)]
    m1.free_sequence(root)
    for b in br:
        m1.append_tokens(b, 0, kv(64), kv(64))
    q1 = torch.randn((8, 16, 128), generator=g, device=device)
    k1, v1, cu1, mx1 = m1.build_packed_kv(br, 0)
    for _ in range(args.warmup):
        attn_decode(q1, k1, v1, None, cu1, mx1, 8)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        attn_decode(q1, k1, v1, None, cu1, mx1, 8)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    ub = 1024 * 8 * 128 * 2 * 4  # 512 + 8 x 64 distinct tokens
    print(f"config 1 (fp32): {ms * 1e3:.1f} us/call, {ub / ms / 1e6:.1f} GB/s unique KV", flush=True)
    # PagedKV.materialize (k_gather): the reference's packed K of config 1 (4,608 rows of 4 KB)
    for _ in range(args.warmup):
        k1.materialize()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        k1.materialize()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    gb = 4 * 4608 * 8 * 128 * 4  # K and V rows, each read once and written once
    print(f"gather (materialize): {ms * 1e3:.1f} us/call, {gb / ms / 1e6:.1f} GB/s moved", flush=True)
    m1.check()


def run_profile_prefill(args):
    """Causal prefill attention of one prompt per length in --profile-prefill:
    bf16, Hq 32, Hkv 8, D 128 (the benchmark trees' head geometry).  Times the
    paged prefill over the cache (PagedKVCacheManager.prefill_attention), the
    dense drop-in (attn_prefill), and, for comparison, torch's SDPA (flash
    backend) and flash_attn_func on the same tensors.  FLOPs count the causal
    half: 4 x Hq x D x S (S + 1) / 2."""
    import torch.nn.functional as F
    from mentat_b200 import PagedKVCacheManager
    from mentat_b200.attention_backend import attn_prefill
    try:
        from flash_attn import flash_attn_func
    except Exception:  # noqa: BLE001 - optional comparison
        flash_attn_func = None
    device = torch.device("cuda", 0)
    steps = max(args.steps, 1)
    g = torch.Generator(device=device).manual_seed(args.seed)
    hq, hkv, d = 32, 8, 128
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    for S in (int(x) for x in args.profile_prefill.split(",")):
        q = torch.randn((1, S, hq, d), generator=g, device=device).to(torch.bfloat16)
        k = torch.randn((1, S, hkv, d), generator=g, device=device).to(torch.bfloat16)
        v = torch.randn((1, S, hkv, d), generator=g, device=device).to(torch.bfloat16)
        m = PagedKVCacheManager(1, hkv, d, max_blocks=(S + 15) // 16 + 2, block_size=16, device=device,
                                dtype=torch.bfloat16, max_seqs=2)
        sid = m.allocate_sequence()
        m.append_tokens(sid, 0, k[0], v[0])
        flops = 4.0 * hq * d * S * (S + 1) / 2
        row = {"S": S}
        row["paged"] = timed(lambda: m.prefill_attention(sid, 0, q[0]))
        row["dense"] = timed(lambda: attn_prefill(q, k, v))
        qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        row["sdpa"] = timed(lambda: F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, enable_gqa=True))
        if flash_attn_func is not None:
            try:
                row["flash_attn"] = timed(lambda: flash_attn_func(q, k, v, causal=True))
            except Exception as e:  # noqa: BLE001 - no kernels for this GPU
                print(f"flash_attn_func unavailable: {str(e).splitlines()[0][:120]}", flush=True)
        m.check()
        print("prefill S=%d: " % S + ", ".join(
            f"{key} {ms * 1e3:.1f} us ({flops / ms / 1e9:.0f} TFLOP/s)" for key, ms in row.items() if key != "S"),
            flush=True)
        del m


def prefill_measure(device, seed, steps=10, warmup=3):
    """Causal prefill attention of one prompt of benchmark configs 3 and 5 (2,048
    tokens, Llama-3.1-8B heads: Hq 32, Hkv 8; 4,096 tokens, Qwen3-32B heads: Hq 64,
    Hkv 8; D 128, bf16) through PagedKVCacheManager.prefill_attention, on resident
    data, CUDA events around `steps` calls; FLOPs count the causal half.  Reported
    beside the decode headline, not part of it: the rollout's prompt pass."""
    from mentat_b200 import PagedKVCacheManager
    g = torch.Generator(device=device).manual_seed(seed)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    peak_burst = _peak_flops(burst=True)
    out = []
    for cfg, S, hq, hkv in ((3, 2048, 32, 8), (5, 4096, 64, 8)):
        d = 128
        q = torch.randn((S, hq, d), generator=g, device=device).to(torch.bfloat16)
        k = torch.randn((S, hkv, d), generator=g, device=device).to(torch.bfloat16)
        m = PagedKVCacheManager(1, hkv, d, max_blocks=(S + 15) // 16 + 2, block_size=16, device=device,
                                dtype=torch.bfloat16, max_seqs=2)
        sid = m.allocate_sequence()
        m.append_tokens(sid, 0, k, k)
        for _ in range(warmup):
            m.prefill_attention(sid, 0, q)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            m.prefill_attention(sid, 0, q)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        m.check()
        tf = 4.0 * hq * d * S * (S + 1) / 2 / (ms / 1e3) / 1e12
        out.append({"config": cfg, "prompt_tokens": S, "heads": [hq, hkv, d], "us": round(ms * 1e3, 1),
                    "TFLOPs": round(tf, 1), "frac_of_bf16_burst": round(tf / peak_burst, 4)})
        del m, q, k
    torch.cuda.empty_cache()
    return out


def run_profile_case(args):
    """A smaller tree for a profiler capture: warm-up calls, then --steps decode
    calls of attn_decode; prints the mean time per call (no JSON line)."""
    from mentat_b200.attention_backend import attn_decode
    prefix, nbr, suffix = (int(x) for x in args.profile_case.split(","))
    device = torch.device("cuda", 0)
    m, kids, q = build_shape(prefix, [suffix] * nbr, args.seed, device, 0)
    k, v, cu, mx = m.build_packed_kv(kids, 0)
    for _ in range(args.warmup):
        attn_decode(q, k, v, None, cu, mx, nbr)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        attn_decode(q, k, v, None, cu, mx, nbr)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ub = unique_bytes(prefix, [suffix] * nbr)
    print(f"profile case prefix {prefix} x {nbr} branches + {suffix}: {ms:.4f} ms/call, {ub / ms / 1e6:.1f} GB/s "
          f"unique KV", flush=True)
    m.check()


def _cpu_inputs(m, kids, q, nbranch):
    sel = kids[:nbranch]
    tables = [m.page_table(s, 0) for s in sel]
    lens = [m.get_kv_length(s) for s in sel]
    return q[:nbranch].cpu(), m.k_pools[0].cpu(), m.v_pools[0].cpu(), tables, lens


def cpu_sample(m, kids, q, nbranch, budget_s, max_calls=50):
    """Time the reference CPU path on the prefix + the first nbranch branches."""
    from oracle.cpu_path import decode_step
    torch.set_num_threads(os.cpu_count() or 1)
    qc, kp, vp, tables, lens = _cpu_inputs(m, kids, q, nbranch)
    ub = unique_bytes(PREFIX, np.array(lens) - PREFIX)
    decode_step(qc, kp, vp, tables, lens, BS)  # warm
    times = []
    t_end = time.perf_counter() + budget_s
    while not times or (time.perf_counter() < t_end and len(times) < max_calls):
        t = time.perf_counter()
        decode_step(qc, kp, vp, tables, lens, BS)
        times.append(time.perf_counter() - t)
    per = statistics.median(times)
    return {"value": round(ub / per / 1e9, 4), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"shared 32768-token prefix + {nbranch} of 64 branches ({sum(lens)} tokens gathered, {ub} "
                      f"unique KV bytes), median of {len(times)} calls of oracle.cpu_path.decode_step (the "
                      "reference's build_packed_kv + _sdpa_decode, bf16, torch CPU)",
            "seconds_per_call": per}


def host_tree(seed):
    """The config-4 tree built on the host alone (numpy and torch CPU tensors; no
    GPU and no part of this package): the block tables the device allocator
    gives ``build_tree`` (a FIFO pool in id order: the 2,048 prefix blocks, then
    each branch's own blocks in branch order), K/V pools of seeded N(0,1) bf16
    rows, and q.  Returns (q, k_pool, v_pool, tables, lens, suffixes)."""
    suf = suffixes(seed)
    nb_pre = PREFIX // BS
    own = [(int(n) + BS - 1) // BS for n in suf]
    total = nb_pre + sum(own)
    g = torch.Generator().manual_seed(seed)
    k_pool = torch.randn((total, BS, HKV, D), generator=g).to(torch.bfloat16)
    v_pool = torch.randn((total, BS, HKV, D), generator=g).to(torch.bfloat16)
    q = torch.randn((NBR, HQ, D), generator=g).to(torch.bfloat16)
    tables, nxt = [], nb_pre
    for n in own:
        tables.append(list(range(nb_pre)) + list(range(nxt, nxt + n)))
        nxt += n
    lens = [PREFIX + int(n) for n in suf]
    return q, k_pool, v_pool, tables, lens, suf


def config4_config(world, ub):
    return {"workload": "BASELINE config 4: bf16 Hq32/Hkv8/D128, block 16, 32768-token shared prefix "
                        "+ 64 branches x U[1024,4096]-token suffixes",
            "unique_kv_bytes_per_step_per_rank": ub, "global_batch": NBR * world,
            "parallelism": f"independent trees x{world}",
            "l2": "inputs larger than L2 (unique KV > 126 MB), no flush"}


def run_reference(args):
    """The reference's CPU decode path (``oracle/cpu_path.py``: build_packed_kv +
    _sdpa_decode with the same torch CPU ops) on the whole config-4 tree, all 64
    branches per step, on every host thread.  The tree is built on the host, so
    this arm loads nothing of this package.  If the requested steps would take
    more than about four minutes, fewer are timed (the line says how many)."""
    from oracle.cpu_path import decode_step
    rank, world, local = _env_rank()
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    q, kp, vp, tables, lens, suf = host_tree(args.seed)
    ub = unique_bytes(PREFIX, suf)
    t = time.perf_counter()
    decode_step(q, kp, vp, tables, lens, BS)  # warm-up (one full step)
    per = time.perf_counter() - t
    warm = max(0, min(args.warmup, int(60.0 / per)) - 1)
    for _ in range(warm):
        decode_step(q, kp, vp, tables, lens, BS)
    steps = max(1, min(args.steps, int(240.0 / per)))
    t = time.perf_counter()
    for _ in range(steps):
        decode_step(q, kp, vp, tables, lens, BS)
    dt = (time.perf_counter() - t) / steps
    val = round(ub / dt / 1e9, 4)
    sample = (f"the whole config-4 tree per step: 32768-token prefix + all 64 branches ({sum(lens)} tokens gathered, "
              f"{ub} unique KV bytes); the reference's CPU path (build_packed_kv + _sdpa_decode) restated in "
              f"oracle/cpu_path.py; {steps} timed steps after {warm + 1} warm-up")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": val, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": warm + 1, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v, BASELINE config 4 tree)",
        "config": config4_config(1, ub),
        "cpu_baseline": {"value": val, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "steps_requested": args.steps, "warmup_requested": args.warmup,
    }), flush=True)


def run_mentat(args):
    import torch.distributed as dist
    from mentat_b200 import _lib
    from mentat_b200.attention_backend import attn_decode
    rank, world, local = _env_rank()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=600))
    lib = _lib.load()
    # weak scaling: every rank decodes a tree of the same shape (suffix lengths from the
    # base seed) with its own values, so the ranks' work is equal and the max over ranks
    # measures contention, not a larger tree
    m, kids, q, suf = build_tree(args.seed, device, extra_blocks=NBR * ((args.steps + args.warmup) // BS + 2),
                                 value_seed=args.seed + rank)
    ub = unique_bytes(PREFIX, suf)
    # host inputs and outputs of the end-to-end loop, made before anything is timed
    # (each step's [q | new K | new V] in one pinned row, so one copy takes them up)
    g = torch.Generator().manual_seed(args.seed + 1000 + rank)
    n_e2e = args.steps + args.warmup
    nq, nkv = NBR * HQ * D, NBR * HKV * D
    in_host = torch.empty((n_e2e, nq + 2 * nkv), dtype=torch.bfloat16).pin_memory()
    in_host[:, :nq] = q.cpu().reshape(1, -1)
    in_host[:, nq:] = torch.randn((n_e2e, 2 * nkv), generator=g).to(torch.bfloat16)
    out_host = torch.empty((n_e2e, NBR, HQ, D), dtype=torch.bfloat16).pin_memory()
    k, v, cu, mx = m.build_packed_kv(kids, 0)
    for _ in range(args.warmup):
        attn_decode(q, k, v, None, cu, mx, NBR)
    torch.cuda.synchronize()
    try:
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    except Exception:
        gpu_id = str(local)
    clocks = Clocks(gpu_id)
    clocks.start()
    time.sleep(0.3)

    # device-resident timing: one attn_decode per step
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = lib.mentat_kernel_launch_count()
    e0.record()
    for _ in range(args.steps):
        attn_decode(q, k, v, None, cu, mx, NBR)
    e1.record()
    launches = lib.mentat_kernel_launch_count() - launches0
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    m.check()

    # per-kernel durations for the roofline: a second pass with CUDA events
    # recorded between the kernels of every call (which keeps them from
    # overlapping, so this pass is not the headline number)
    prof_steps = min(args.steps, 50)
    _lib.check(lib.mentat_profile_enable(prof_steps), "mentat_profile_enable")
    for _ in range(prof_steps):
        attn_decode(q, k, v, None, cu, mx, NBR)
    stage = (ctypes.c_double * 5)()
    cnt = ctypes.c_int32()
    _lib.check(lib.mentat_profile_collect(stage, ctypes.byref(cnt)), "mentat_profile_collect")
    lib.mentat_profile_enable(0)
    m.check()

    # the same decode with the plan a previous call left in the workspace, as every
    # layer after the first of a decode step runs it (the layers share the tree's
    # shape; mentat_paged_decode_reuse_plan): reported beside the headline, which
    # plans every call
    from mentat_b200 import ops
    scale = ops.default_scale(D)
    ops.paged_decode(q, k.slots, max(k.lens), m._op_id, 0, scale)
    for _ in range(args.warmup):
        ops.paged_decode(q, k.slots, max(k.lens), m._op_id, 0, scale, reuse_plan=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.steps):
        ops.paged_decode(q, k.slots, max(k.lens), m._op_id, 0, scale, reuse_plan=True)
    e1.record()
    torch.cuda.synchronize()
    reuse_ms = e0.elapsed_time(e1) / args.steps
    m.check()

    # end to end through the public API: pinned host inputs in, result out, every
    # step.  The copies run on a second stream: step i+1's inputs go up (into the
    # other of two device slots) while step i decodes, and step i's output comes
    # back while step i+1 runs; events order every hand-over.
    main = torch.cuda.current_stream(device)
    side = torch.cuda.Stream(device)
    x_dev = [torch.empty(nq + 2 * nkv, dtype=torch.bfloat16, device=device) for _ in range(2)]
    # outputs go back from two fixed device slots (a tensor the caching allocator hands
    # out on one stream and frees while another still reads it stalls the host at times)
    o_dev = [torch.empty((NBR, HQ, D), dtype=torch.bfloat16, device=device) for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]    # input slot filled
    ev_free = [torch.cuda.Event() for _ in range(2)]  # input slot read by its step's kernels
    ev_out = [torch.cuda.Event() for _ in range(2)]   # output slot written
    ev_back = [torch.cuda.Event() for _ in range(2)]  # output slot copied to the host

    def upload(i):
        s = i % 2
        if i >= 2:
            side.wait_event(ev_free[s])
        with torch.cuda.stream(side):
            x_dev[s].copy_(in_host[i], non_blocking=True)
            ev_in[s].record(side)

    def e2e_step(i, last):
        s = i % 2
        main.wait_event(ev_in[s])
        qd = x_dev[s][:nq].view(NBR, HQ, D)
        kvd = x_dev[s][nq:].view(2, NBR, HKV, D)
        m.append_tokens_batched(kids, 0, kvd[0], kvd[1])
        kk, vv, cuk, mxk = m.build_packed_kv(kids, 0)
        o = attn_decode(qd, kk, vv, None, cuk, mxk, NBR)
        ev_free[s].record(main)
        if i + 2 <= last:
            upload(i + 2)
        if i >= 2:
            main.wait_event(ev_back[s])
        o_dev[s].copy_(o, non_blocking=True)
        ev_out[s].record(main)
        side.wait_event(ev_out[s])
        with torch.cuda.stream(side):
            out_host[i].copy_(o_dev[s], non_blocking=True)
            ev_back[s].record(side)

    upload(0)
    upload(1)
    for i in range(args.warmup):
        e2e_step(i, args.warmup - 1)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    base = sum(m.get_kv_length(s) for s in kids) - NBR * PREFIX
    e2e_bytes = sum(unique_bytes(PREFIX, [base + NBR * (i + 1)]) for i in range(args.steps))
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(main)
    side.wait_stream(main)
    upload(args.warmup)
    if args.steps > 1:
        upload(args.warmup + 1)
    for i in range(args.steps):
        e2e_step(args.warmup + i, n_e2e - 1)
    main.wait_stream(side)
    a1.record(main)
    torch.cuda.synchronize()
    clk = clocks.stop()
    e2e_ms = a0.elapsed_time(a1)
    m.check()

    value, e2e_val, ms_max, rank_rows = combine_ranks(ms, e2e_ms, ub * args.steps, e2e_bytes, device, world)
    n_prof = max(cnt.value, 1)
    st_ms = {"plan": stage[0] / n_prof, "units_ffma": stage[1] / n_prof, "units_tc": stage[2] / n_prof,
             "units_tcn": stage[3] / n_prof, "merge": stage[4] / n_prof}
    # bytes each unit kernel streams: the shared prefix (64 branches x 4 query heads = 256 rows) goes
    # to the wide tensor-core units, the branch suffixes (4 rows) to the narrow ones (or to the
    # FFMA units when MENTAT_TC_MIN_ROWS routes them there)
    shared_b = unique_bytes(PREFIX, [0])
    suffix_kernel = "units_tcn" if st_ms["units_tcn"] >= st_ms["units_ffma"] else "units_ffma"
    per = {"units_tc": shared_b, suffix_kernel: ub - shared_b}
    # the roofline's kernel is the one that streams most of the bytes (HBM bound); the wide
    # kernel, compute bound on the shared prefix and running beside it on the SMs the plan
    # gives it, is reported in per_kernel with its tensor rate
    dom = max(per, key=lambda k: per[k])
    dom_bytes = per[dom]
    units_ms = st_ms[dom]

    if rank == 0:
        peak, peak_kind = peaks()
        achieved = dom_bytes / (units_ms / 1e3) / 1e9 if units_ms > 0 else None
        kernels = {{"units_tc": "k_units_tc", "units_tcn": "k_units_tcn", "units_ffma": "k_units"}[k]:
                   {"bytes": b, "ms": st_ms[k]} for k, b in per.items()}
        for kv in kernels.values():
            kv["GBps"] = round(kv["bytes"] / (kv["ms"] / 1e3) / 1e9, 1) if kv["ms"] > 0 else None
        # Q K^T and P V for the prefix's 256 rows: 2 x 2 x 256 x D flop per token and kv head
        wide_flop = 4 * 256 * 128 * PREFIX * 8
        if "k_units_tc" in kernels and kernels["k_units_tc"]["ms"] > 0:
            kernels["k_units_tc"]["TFLOPs"] = round(wide_flop / (kernels["k_units_tc"]["ms"] / 1e3) / 1e12, 1)
        cpu = None
        if world == 1 and not args.no_cpu:
            cpu = cpu_sample(m, kids, q, 2, 12.0)
            cpu.pop("seconds_per_call", None)
    h2d_bytes, d2h_bytes = int(in_host[0].numel() * 2), int(out_host[0].numel() * 2)
    del m, k, v, cu, q, in_host
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    # causal prefill of the prompts of configs 3 and 5, on rank 0
    prefill = None
    if rank == 0 and args.tree:
        try:
            prefill = prefill_measure(device, args.seed)
        except Exception as e:  # noqa: BLE001 - the headline line is printed either way
            prefill = {"error": f"{type(e).__name__}: {e}"[:300]}
    # tree tokens/s of benchmark config 3 on the same ranks (the prompts split across them)
    tree = None
    if args.tree:
        try:
            tree = tree_measure(3, args.seed, rank, world, device)
        except Exception as e:  # noqa: BLE001 - the headline line is printed either way
            tree = {"metric": "tree tokens/s (config 3)", "error": f"{type(e).__name__}: {e}"[:300]}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) q/k/v, BASELINE config 4 tree per rank)",
            "config": config4_config(world, ub),
            "roofline": {"bound": "hbm",
                         "kernel": {"units_tc": "k_units_tc", "units_tcn": "k_units_tcn", "units_ffma": "k_units"}[dom],
                         "achieved": round(achieved, 2) if achieved else None, "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4) if achieved else None, "peak_kind": peak_kind,
                         "traffic": ncu_traffic().get(f"{dom}_c4_bytes_per_launch"),
                         "stage_ms_per_launch": st_ms, "per_kernel": kernels,
                         "whole_call": {"bytes": ub, "ms": ms_max / args.steps,
                                        "GBps": round(ub / (ms_max / args.steps / 1e3) / 1e9, 1)},
                         "whole_call_plan_reused": {"ms": round(reuse_ms, 5),
                                                    "GBps": round(ub / (reuse_ms / 1e3) / 1e9, 1)},
                         # each rank's own whole-call rate: imbalance shows as spread, contention
                         # as every rank below the single-GPU figure
                         "per_rank": [{"rank": r, "ms_per_step": round(t / args.steps, 5),
                                       "GBps": round(b / (t / 1e3) / 1e9, 1),
                                       "frac_whole_call": round(b / (t / 1e3) / 1e9 / peak, 4)}
                                      for r, (t, b) in enumerate(rank_rows)]},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d_bytes,
                    "d2h_bytes_per_step": d2h_bytes,
                    "path": "pinned H2D of [q | new K | new V] in one copy -> append_tokens_batched -> "
                            "build_packed_kv -> attn_decode -> D2H output; the copies on a second stream, "
                            "overlapping the neighbouring steps' kernels"},
            "gpu_launches": int(launches),  # counted by the library over the device-timed loop
            "clocks": clk,
            "tree": tree,
            "prefill": prefill,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mentat", choices=["mentat", "reference"])
    ap.add_argument("--seed", type=int, default=4)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-tree", dest="tree", action="store_false",
                    help="skip the config-3 tree tokens/s measurement of the default run")
    ap.add_argument("--profile-case", default=None, metavar="PREFIX,BRANCHES,SUFFIX",
                    help="time a smaller tree for a profiler capture instead of the benchmark")
    ap.add_argument("--profile-prefill", default=None, metavar="LEN[,LEN...]",
                    help="time causal prefill attention of prompts of these lengths (no JSON line)")
    ap.add_argument("--profile-kernels", action="store_true",
                    help="time the gate and append kernels for a profiler capture instead of the benchmark")
    ap.add_argument("--tree-config", type=int, default=None, choices=sorted(TREE_CONFIGS),
                    help="tree tokens/s of the entropy-gated rollout on a benchmark model config")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.profile_prefill:
        run_profile_prefill(args)
        return
    if args.profile_case:
        run_profile_case(args)
    elif args.profile_kernels:
        run_profile_kernels(args)
    elif args.tree_config is not None:
        run_tree(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_mentat(args)


if __name__ == "__main__":
    main()
