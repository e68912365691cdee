"""Tensor parallelism by KV head (``mentat_b200.tp``), on CPU.

A full tiny Qwen3 / Llama model is split into per-rank shards; a forward pass
that runs every rank's layers and sums the attention and MLP partial outputs
(the all-reduce ``PagedLM`` does) must give the full model's logits.  The same
forward on two gloo ranks, with ``torch.distributed.all_reduce``, must give the
same logits on both ranks.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _model(family, hq=8, hkv=4, inter=96):
    from transformers import LlamaConfig, LlamaForCausalLM, Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(7)
    kw = dict(vocab_size=97, hidden_size=64, intermediate_size=inter, num_hidden_layers=2,
              num_attention_heads=hq, num_key_value_heads=hkv, head_dim=16, max_position_embeddings=256,
              rms_norm_eps=1e-6)
    if family == "qwen3":
        m = Qwen3ForCausalLM(Qwen3Config(**kw, tie_word_embeddings=True))
    else:
        m = LlamaForCausalLM(LlamaConfig(**kw, tie_word_embeddings=False, rope_theta=500000.0))
    return m.float().eval()


def _rope(t, cos, sin):
    h = t.shape[-1] // 2
    return t * cos + torch.cat((-t[..., h:], t[..., :h]), dim=-1) * sin


def _attn_partial(m, li, h, pos):
    blk = m.model.layers[li]
    attn = blk.self_attn
    cfg = m.config
    L, hd = h.shape[1], cfg.head_dim
    x = blk.input_layernorm(h)
    q = attn.q_proj(x).view(1, L, cfg.num_attention_heads, hd)
    k = attn.k_proj(x).view(1, L, cfg.num_key_value_heads, hd)
    v = attn.v_proj(x).view(1, L, cfg.num_key_value_heads, hd)
    if hasattr(attn, "q_norm"):
        q, k = attn.q_norm(q), attn.k_norm(k)
    cos, sin = m.model.rotary_emb(x, pos)
    q, k = _rope(q, cos.unsqueeze(2), sin.unsqueeze(2)), _rope(k, cos.unsqueeze(2), sin.unsqueeze(2))
    g = cfg.num_attention_heads // cfg.num_key_value_heads
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2).repeat_interleave(g, 1),
                                       v.transpose(1, 2).repeat_interleave(g, 1), is_causal=True)
    return attn.o_proj(o.transpose(1, 2).reshape(1, L, -1))


@torch.no_grad()
def _tp_forward(shards, ids, reduce):
    """Every rank's layers in one process (``shards``: this process's ranks);
    ``reduce`` sums the partial outputs over all ranks."""
    m0 = shards[0]
    L = ids.shape[1]
    pos = torch.arange(L).view(1, L)
    h = m0.model.embed_tokens(ids)
    for li in range(m0.config.num_hidden_layers):
        h = h + reduce([_attn_partial(m, li, h, pos) for m in shards])
        h = h + reduce([m.model.layers[li].mlp(m.model.layers[li].post_attention_layernorm(h)) for m in shards])
    return m0.lm_head(m0.model.norm(h))


@pytest.mark.parametrize("family,world", [("qwen3", 2), ("qwen3", 4), ("llama", 2)])
def test_shards_sum_to_full_model(family, world):
    from mentat_b200.tp import shard_model
    full = _model(family)
    ids = torch.tensor([[3, 14, 15, 92, 65, 35, 89, 79, 32, 38]])
    with torch.no_grad():
        want = full(ids).logits
    shards = [shard_model(full, r, world) for r in range(world)]
    c = shards[0].config
    assert c.num_key_value_heads == 4 // world and c.num_attention_heads == 8 // world
    assert shards[0].model.layers[0].self_attn.k_proj.weight.shape == (16 * 4 // world, 64)
    got = _tp_forward(shards, ids, lambda parts: sum(parts))
    np.testing.assert_allclose(got.numpy(), want.numpy(), atol=2e-5, rtol=1e-4)


def test_bad_split_is_refused():
    from mentat_b200.tp import shard_model
    with pytest.raises(ValueError, match="must divide"):
        shard_model(_model("qwen3"), 0, 3)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from mentat_b200.tp import shard_model
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = _model("qwen3")
        shard = shard_model(full, rank, world)
        del full

        def reduce(parts):
            (x,) = parts
            dist.all_reduce(x)
            return x
        ids = torch.tensor([[5, 8, 13, 21, 34, 55]])
        out.put((rank, _tp_forward([shard], ids, reduce).numpy()))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.timeout(180)
def test_two_gloo_ranks_all_reduce_to_the_full_logits():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(out.get(timeout=150) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    with torch.no_grad():
        want = _model("qwen3")(torch.tensor([[5, 8, 13, 21, 34, 55]])).logits.numpy()
    np.testing.assert_array_equal(res[0], res[1])  # every rank ends with the same logits
    np.testing.assert_allclose(res[0], want, atol=2e-5, rtol=1e-4)
