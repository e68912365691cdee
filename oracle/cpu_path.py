"""The reference's CPU decode path restated with the same torch CPU operations
(test and baseline infrastructure only: the ``cpu_baseline`` and
``--impl reference`` legs of ``bench.py`` time it).

* ``packed_gather`` follows ``PagedKVCacheManager.build_packed_kv``
  (``core/paged_kv_cache.py:289-368``): Python lists of (block, slot) per
  token, index tensors, one advanced-index gather for K and one for V, and the
  int32 ``cu_seqlens_k``.
* ``sdpa_decode`` follows ``_sdpa_decode`` (``adapters/attention_backend.py:
  99-168``): one ``F.scaled_dot_product_attention`` per sequence on the GQA-
  expanded K/V slices.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def packed_gather(k_pool, v_pool, tables, lens, block_size):
    blk, slt = [], []
    for tab, n in zip(tables, lens):
        rem = n
        for b in tab:
            c = min(block_size, rem)
            blk.extend([b] * c)
            slt.extend(range(c))
            rem -= c
            if rem == 0:
                break
    b = torch.tensor(blk, dtype=torch.long)
    s = torch.tensor(slt, dtype=torch.long)
    cu = torch.tensor([0] + list(lens), dtype=torch.int32).cumsum(dim=0, dtype=torch.int32)
    return k_pool[b, s], v_pool[b, s], cu, max(lens)


def sdpa_decode(q, packed_k, packed_v, cu_seqlens_k):
    n, hq, d = q.shape
    g = hq // packed_k.shape[1]
    cu = cu_seqlens_k.tolist()
    outs = []
    for i in range(n):
        a, b = cu[i], cu[i + 1]
        L = b - a
        ki, vi = packed_k[a:b], packed_v[a:b]
        if g > 1:
            ki = ki.unsqueeze(2).expand(-1, -1, g, -1).reshape(L, hq, d)
            vi = vi.unsqueeze(2).expand(-1, -1, g, -1).reshape(L, hq, d)
        qi = q[i].unsqueeze(0).unsqueeze(2)
        ki = ki.permute(1, 0, 2).unsqueeze(0)
        vi = vi.permute(1, 0, 2).unsqueeze(0)
        outs.append(F.scaled_dot_product_attention(qi, ki, vi, is_causal=False).squeeze(0).squeeze(1))
    return torch.stack(outs, dim=0)


def decode_step(q, k_pool, v_pool, tables, lens, block_size):
    pk, pv, cu, _ = packed_gather(k_pool, v_pool, tables, lens, block_size)
    return sdpa_decode(q, pk, pv, cu)
