"""Oracle paged GQA decode and causal prefill attention (test infrastructure only).

Restates the reference's CPU decode path: ``build_packed_kv``
(``core/paged_kv_cache.py:289-368``) gathers every sequence's tokens through its
page table -- token ``t`` of a sequence lives at block ``table[t // bs]``, slot
``t % bs`` -- and ``_sdpa_decode`` (``adapters/attention_backend.py:99-168``)
runs single-query attention per sequence with the GQA expansion of ``:152-155``
(query head ``j`` reads kv head ``j // (Hq // Hkv)``), softmax scale
``1/sqrt(D)`` (the SDPA default) and no mask.  An empty sequence yields zeros
(what ``F.scaled_dot_product_attention`` returns for zero keys).

Arithmetic is float64; callers round to the output dtype.
"""

from __future__ import annotations

import numpy as np


def gather_seq(pool: np.ndarray, table, n_tokens: int, block_size: int) -> np.ndarray:
    """Tokens ``[0, n_tokens)`` of one sequence, ``(n, Hkv, D)`` (``:316-328``)."""
    if n_tokens == 0:
        return pool[:0, 0]
    t = np.arange(n_tokens)
    blocks = np.asarray(table, np.int64)[t // block_size]
    return pool[blocks, t % block_size]


def decode_one(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float | None = None):
    """One sequence: q ``(Hq, D)``, k/v ``(n, Hkv, D)`` -> ``(Hq, D)`` float64."""
    hq, d = q.shape
    n, hkv, _ = k.shape
    if n == 0:
        return np.zeros((hq, d), np.float64)
    g = hq // hkv
    scale = 1.0 / np.sqrt(d) if scale is None else scale
    q64 = q.astype(np.float64).reshape(hkv, g, d)
    k64 = k.astype(np.float64)
    v64 = v.astype(np.float64)
    s = np.einsum("hgd,nhd->hgn", q64, k64) * scale
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    o = np.einsum("hgn,nhd->hgd", p, v64)
    return o.reshape(hq, d)


def paged_decode(q, k_pool, v_pool, tables, lens, block_size, scale=None):
    """All sequences of a batch; q ``(N, Hq, D)`` -> ``(N, Hq, D)`` float64."""
    out = np.zeros(q.shape, np.float64)
    for i, (tab, n) in enumerate(zip(tables, lens)):
        k = gather_seq(k_pool, tab, n, block_size)
        v = gather_seq(v_pool, tab, n, block_size)
        out[i] = decode_one(q[i], k, v, scale)
    return out


def packed_decode(q, packed_k, packed_v, cu_seqlens_k, scale=None):
    """Same computation on a packed (varlen) batch, ``_sdpa_decode`` style."""
    out = np.zeros(q.shape, np.float64)
    cu = np.asarray(cu_seqlens_k)
    for i in range(q.shape[0]):
        a, b = int(cu[i]), int(cu[i + 1])
        out[i] = decode_one(q[i], packed_k[a:b], packed_v[a:b], scale)
    return out


def prefill(q: np.ndarray, k: np.ndarray, v: np.ndarray, pos0: int = 0, scale: float | None = None):
    """Causal prefill attention, the reference's ``_sdpa_prefill``
    (``adapters/attention_backend.py:43-96``): GQA by expanding kv head ``h`` to
    query heads ``h*G .. h*G+G-1`` (``:70-79``), scale ``1/sqrt(D)``, causal mask
    (``is_causal=True``, ``:94``).  Generalised to a chunk: q ``(n, Hq, D)`` are
    the queries of positions ``pos0 .. pos0+n-1`` and k/v ``(pos0+n, Hkv, D)``
    the whole sequence; query ``i`` sees keys ``0 .. pos0+i`` (``pos0 = 0`` is
    the reference's whole-prompt call).  Returns ``(n, Hq, D)`` float64."""
    n, hq, d = q.shape
    L, hkv, _ = k.shape
    assert L == pos0 + n, (L, pos0, n)
    g = hq // hkv
    scale = 1.0 / np.sqrt(d) if scale is None else scale
    q64 = q.astype(np.float64).reshape(n, hkv, g, d)
    k64 = k.astype(np.float64)
    v64 = v.astype(np.float64)
    s = np.einsum("nhgd,lhd->hgnl", q64, k64) * scale
    mask = np.arange(L)[None, :] <= (pos0 + np.arange(n))[:, None]
    s = np.where(mask, s, -np.inf)
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    o = np.einsum("hgnl,lhd->nhgd", p, v64)
    return o.reshape(n, hq, d)


def unique_kv_bytes(tables, lens, block_size, num_kv_heads, head_dim, elem_bytes):
    """Algorithmic bytes of one layer call: distinct physical blocks x their
    valid tokens x Hkv x D x 2 (K and V) x element size."""
    valid = {}
    for tab, n in zip(tables, lens):
        nb = -(-n // block_size)
        for j in range(nb):
            c = min(block_size, n - j * block_size)
            b = int(tab[j])
            valid[b] = max(valid.get(b, 0), c)
    return sum(valid.values()) * num_kv_heads * head_dim * 2 * elem_bytes
