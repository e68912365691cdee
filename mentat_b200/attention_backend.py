"""Drop-in for ``adapters/attention_backend.py`` of SkyeGunasekaran/MENTAT.

Exports the names the reference's adapters import (``BACKEND``,
``attn_prefill``, ``attn_decode``; ``model_adapter.py:34``,
``llama_adapter.py:4``, ``qwen3_adapter.py:5``).  ``attn_decode`` runs the
tree-aware paged decode kernel of libmentat_b200 on the :class:`PagedKV`
handles returned by ``mentat_b200.PagedKVCacheManager.build_packed_kv``;
``attn_prefill`` runs its causal prefill kernel over the dense K and V.  There
is no flash-attn, SDPA or CPU path for either.
"""

from __future__ import annotations

import ctypes as C
import math
from typing import Optional

import torch

from . import _lib, ops
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


_DENSE_INDEX: dict = {}


class _DensePool:
    """A one-layer cache descriptor over the dense (B, S, Hkv, D) K and V of a
    prefill: sequence b is slot b, its blocks are the 16-row slices of k[b]
    (zero-padded to a multiple of 16 rows when S is not one), so the paged
    prefill kernel reads the tensors in place."""

    BLOCK = 16

    def __init__(self, k: torch.Tensor, v: torch.Tensor):
        B, S, hkv, d = k.shape
        nb = (S + self.BLOCK - 1) // self.BLOCK
        sp = nb * self.BLOCK
        dev = k.device

        def pool(t):
            if sp == S and t.is_contiguous():
                return t
            p = torch.zeros((B, sp, hkv, d), device=dev, dtype=t.dtype)
            p[:, :S] = t
            return p
        self.k, self.v = pool(k), pool(v)
        # the index arrays depend only on (B, S) and the device: made once and reused
        # by every layer's call (the reference calls attn_prefill once per layer)
        key = (B, S, dev)
        idx = _DENSE_INDEX.get(key)
        if idx is None:
            i32 = dict(device=dev, dtype=torch.int32)
            idx = (torch.arange(B * nb, **i32), torch.full((B,), nb, **i32), torch.full((B,), S, **i32),
                   torch.full((B,), S - (nb - 1) * self.BLOCK, **i32),
                   torch.zeros(_lib.CTRL_WORDS, device=dev, dtype=torch.int64), torch.arange(B, **i32))
            if len(_DENSE_INDEX) >= 16:
                _DENSE_INDEX.clear()
            _DENSE_INDEX[key] = idx
        self.tables, self.nblocks, self.ntok, self.tail, self.ctrl, self.slots = idx
        desc = _lib.KVCache()
        desc.num_layers, desc.num_blocks, desc.block_size = 1, B * nb, self.BLOCK
        desc.num_kv_heads, desc.head_dim, desc.dtype = hkv, d, ops._DT[k.dtype]
        desc.max_seqs, desc.max_blocks_per_seq = B, nb
        desc.k_pool, desc.v_pool = self.k.data_ptr(), self.v.data_ptr()
        desc.ctrl, desc.tables = self.ctrl.data_ptr(), self.tables.data_ptr()
        desc.nblocks, desc.ntok, desc.tail = self.nblocks.data_ptr(), self.ntok.data_ptr(), self.tail.data_ptr()
        self.desc = desc
        self.descp = C.byref(desc)


def attn_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window_size: Optional[int] = None) -> torch.Tensor:
    """Causal prefill attention, (batch, seq, heads, head_dim) layout
    (``attention_backend.py:175-189``), on libmentat_b200's paged prefill
    kernel (tensor cores for bf16 / fp16) over the dense K and V, softmax scale
    1/sqrt(head_dim) as in the reference.  Sliding windows are not built: the
    reference's generator never passes one (``generator.py`` calls the adapters'
    prefill without ``window_size``)."""
    B, S, hq, d = q.shape
    if window_size is not None and window_size < S:
        raise NotImplementedError("sliding-window prefill is not used by the reference's generator")
    if k.shape[0] != B or k.shape[1] != S or k.shape[3] != d or v.shape != k.shape or hq % k.shape[2]:
        raise ValueError(f"q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)}: not a GQA prefill")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k and v must share one dtype")
    if q.stride(3) != 1 or q.stride(2) != d:
        q = q.contiguous()
    out = torch.empty((B, S, hq, d), device=q.device, dtype=q.dtype)
    if B == 0 or S == 0:
        return out
    pool = _DensePool(k, v)
    scale = 1.0 / math.sqrt(d)
    for b in range(B):
        ops.paged_prefill(pool.descp, 0, pool.slots[b:b + 1], 0, q[b], scale, out=out[b])
    return out
