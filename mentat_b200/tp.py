"""Tensor parallelism by KV head for the rollout's model driver.

The largest benchmark model (Qwen3-32B architecture, 8 KV heads) runs split
one KV head per GPU: each rank holds its KV heads' query, key and value
projections (row slices), the matching columns of ``o_proj``, and a slice of
the MLP's intermediate dimension (rows of ``gate_proj`` / ``up_proj``, columns
of ``down_proj``).  The attention output and the MLP output are then partial
sums over the ranks; ``PagedLM`` all-reduces them (NCCL) before the residual
add, the model's two existing reductions per layer.  Norms, the embedding and
the lm_head are replicated, so every rank ends the step with the same hidden
state and the same full-vocabulary logits, and the gate and the tree logic run
identically on every rank (each rank's cache holds only its KV heads).

This follows the reference's adapters (``adapters/qwen3_adapter.py``,
``adapters/llama_adapter.py``): the layer arithmetic is Hugging Face's, only
split; q head ``h`` still reads KV head ``h // G``.
"""

from __future__ import annotations

import copy
import re

import torch

_ROWS = re.compile(r"\.(q_proj|k_proj|v_proj|gate_proj|up_proj)\.(weight|bias)$")
_COLS = re.compile(r"\.(o_proj|down_proj)\.weight$")
_COL_BIAS = re.compile(r"\.(o_proj|down_proj)\.bias$")


def tp_config(cfg, world: int):
    """The per-rank config: heads, KV heads and the MLP width divided by ``world``."""
    hkv, hq, inter = cfg.num_key_value_heads, cfg.num_attention_heads, cfg.intermediate_size
    if hkv % world or hq % world or inter % world:
        raise ValueError(f"tensor parallel size {world} must divide kv heads {hkv}, heads {hq} and "
                         f"intermediate size {inter}")
    c = copy.deepcopy(cfg)
    if getattr(c, "head_dim", None) is None:
        c.head_dim = cfg.hidden_size // hq
    c.num_attention_heads = hq // world
    c.num_key_value_heads = hkv // world
    c.intermediate_size = inter // world
    return c


def shard_state(state: dict, cfg, rank: int, world: int) -> dict:
    """Rank ``rank``'s slices of a full model's state dict (``cfg`` is the full config)."""
    hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    rows = {"q_proj": cfg.num_attention_heads * hd, "k_proj": cfg.num_key_value_heads * hd,
            "v_proj": cfg.num_key_value_heads * hd, "gate_proj": cfg.intermediate_size,
            "up_proj": cfg.intermediate_size}
    out = {}
    for k, t in state.items():
        m = _ROWS.search(k)
        if m:
            n = rows[m.group(1)] // world
            out[k] = t[rank * n:(rank + 1) * n].clone()
            continue
        if _COLS.search(k):
            n = t.shape[1] // world
            out[k] = t[:, rank * n:(rank + 1) * n].clone()
            continue
        if _COL_BIAS.search(k):  # added once, after the reduction's partial sums
            out[k] = t.clone() if rank == 0 else torch.zeros_like(t)
            continue
        out[k] = t.clone()
    return out


def shard_model(model, rank: int, world: int):
    """A per-rank copy of a Hugging Face Qwen3 / Llama causal LM split by KV head;
    the full model is left unchanged (free it after every rank has its shard)."""
    cfg_r = tp_config(model.config, world)
    with torch.device("meta"):
        m = type(model)(cfg_r)
    state = shard_state(model.state_dict(), model.config, rank, world)
    m.load_state_dict(state, assign=True, strict=True)
    if getattr(cfg_r, "tie_word_embeddings", False):
        m.tie_weights()
    # buffers (the rotary inverse frequencies) are not in the state dict: rebuild them
    dev = next(iter(state.values())).device
    m.model.rotary_emb = type(model.model.rotary_emb)(config=cfg_r, device=dev)
    return m.eval()
