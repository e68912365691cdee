"""Tensor parallelism by KV head on two GPUs (NCCL): the decode path under TP.

Each of two ranks builds the same tiny fp32 Qwen3 model, keeps its KV-head shard
(``tp.shard_model``) and runs ``PagedLM`` over its own cache (two of the four KV
heads), prefill plus three decode steps with the library's append and decode
kernels, all-reducing the attention and MLP outputs, eagerly and again with the
decode steps captured as CUDA graphs (all-reduces inside, batch padded).  Both
ranks must end each step with identical logits, equal to the unsplit model's on
one GPU.
Skipped with fewer than two GPUs.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(model, device, group, graphs=False):
    from mentat_b200 import PagedKVCacheManager
    from mentat_b200.rollout import PagedLM
    cfg = model.config
    cache = PagedKVCacheManager(cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim, 256, 16, device,
                                torch.float32, max_seqs=8)
    lm = PagedLM(model, cache, group)
    if graphs:  # the decode steps as CUDA graphs holding the all-reduces, batch padded to 4
        lm.enable_graphs(64, 4, bucket=4)
    sid = cache.allocate_sequence()
    out = [lm.prefill(torch.tensor([3, 14, 15, 92, 65, 35, 89, 79, 32, 38, 46, 26, 43, 38, 32, 79, 50, 28],
                                   device=device), sid).float().cpu().numpy()]
    for t in (7, 1, 8):
        logits, _ = lm.decode(torch.tensor([t], device=device), [sid])
        out.append(logits[0].float().cpu().numpy())
    cache.check()
    lm._graphs = None  # release graphs holding NCCL calls before the process group goes
    return np.stack(out)


def _rank_main(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from mentat_b200.tp import shard_model
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device)
    try:
        torch.manual_seed(11)
        cfg = Qwen3Config(vocab_size=101, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                          num_attention_heads=8, num_key_value_heads=4, head_dim=64, max_position_embeddings=512,
                          rms_norm_eps=1e-6, tie_word_embeddings=True)
        with torch.device(device):
            full = Qwen3ForCausalLM(cfg).float().eval()
        want = _run(full, device, None)
        shard = shard_model(full, rank, world)
        got = _run(shard, device, dist.group.WORLD)
        got_g = _run(shard, device, dist.group.WORLD, graphs=True)
        torch.cuda.synchronize()
        q.put((rank, want, got, got_g))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_kv_head_split_matches_the_whole_model():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, want, got, got_g = q.get(timeout=240)
        res[r] = (want, got, got_g)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    np.testing.assert_array_equal(res[0][1], res[1][1])  # identical logits on both ranks
    np.testing.assert_array_equal(res[0][2], res[1][2])
    for r in range(2):
        np.testing.assert_allclose(res[r][1], res[r][0], atol=1e-4, rtol=1e-4)
        np.testing.assert_allclose(res[r][2], res[r][1], atol=1e-5, rtol=1e-5)  # graphs = eager
