"""Drop-in for ``adapters/attention_backend.py`` of SkyeGunasekaran/MENTAT.

Exports the names the reference's adapters import (``BACKEND``,
``attn_prefill``, ``attn_decode``; ``model_adapter.py:34``,
``llama_adapter.py:4``, ``qwen3_adapter.py:5``).  ``attn_decode`` runs the
tree-aware paged decode kernel of libmentat_b200 on the :class:`PagedKV`
handles returned by ``mentat_b200.PagedKVCacheManager.build_packed_kv``; there
is no flash-attn, SDPA or CPU path for decode.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from . import ops
from .paged_kv_cache import PagedKV

BACKEND = "mentat_b200"
MAX_SEQS_PER_LAUNCH = ops.MAX_SEQS_PER_LAUNCH


def attn_decode(q: torch.Tensor, k, v, cu_seqlens_q: torch.Tensor = None, cu_seqlens_k: torch.Tensor = None,
                max_seqlen_k: int = 0, N: int = None, window_size: Optional[int] = None,
                softmax_scale: Optional[float] = None) -> torch.Tensor:
    """Single-query GQA decode for N sequences (``attention_backend.py:192-228``).

    q: (N, num_heads, head_dim); k, v: the PagedKV handles of one
    ``build_packed_kv`` call.  Returns (N, num_heads, head_dim) in q's dtype,
    softmax scale 1/sqrt(head_dim) as in the reference (SDPA / flash default).
    """
    if not isinstance(k, PagedKV) or not isinstance(v, PagedKV):
        raise TypeError("mentat_b200.attn_decode reads KV blocks in place: pass the handles returned by "
                        "mentat_b200.PagedKVCacheManager.build_packed_kv")
    if window_size is not None:
        raise NotImplementedError("sliding-window decode is not used by the reference adapters")
    mgr = k.cache
    n = q.shape[0] if N is None else N
    if n != len(k.lens):
        raise ValueError(f"q has {n} sequences, the KV handle has {len(k.lens)}")
    hq, d = q.shape[1], q.shape[2]
    if d != mgr.head_dim or hq % mgr.num_key_value_heads:
        raise ValueError("q shape does not match the cache geometry")
    if q.dtype != mgr.dtype:
        raise TypeError(f"q dtype {q.dtype} differs from the cache dtype {mgr.dtype}")
    if q.stride(2) != 1 or q.stride(1) != d:
        q = q.contiguous()
    if n == 0:
        return torch.empty((0, hq, d), device=q.device, dtype=q.dtype)
    scale = 1.0 / math.sqrt(d) if softmax_scale is None else float(softmax_scale)
    out = ops.paged_decode(q[:n], k.slots, max(k.lens), mgr._op_id, k.layer, scale)
    if mgr.strict:
        mgr.check()
    return out


def attn_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window_size: Optional[int] = None) -> torch.Tensor:
    """Causal prefill attention, (batch, seq, heads, head_dim) layout
    (``attention_backend.py:175-189``).  Prefill is outside the decode hot
    path; this calls torch's fused SDPA with GQA."""
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    s = q.shape[1]
    if window_size is not None and window_size < s:
        row = torch.arange(s, device=q.device)
        mask = (row[None, :] <= row[:, None]) & (row[None, :] >= (row - window_size + 1)[:, None])
        o = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask, enable_gqa=True)
    else:
        o = F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, enable_gqa=True)
    return o.transpose(1, 2)
