"""Oracle restatement of the reference paged KV cache (test infrastructure only).

Follows ``core/paged_kv_cache.py`` of SkyeGunasekaran/MENTAT line by line in
behaviour, with one deliberate difference: the free list is an injected object.
The reference keeps free block ids in a CPython ``set`` and takes them with
``set.pop()`` (``paged_kv_cache.py:29,51``), whose order is an implementation
detail of CPython's hash table.  Block tables are therefore only comparable
under an injected deterministic policy.  The reference touches ``_free`` only
through ``pop()``, ``add()`` and ``len()`` (``paged_kv_cache.py:34,38,46,51,66,
72``), so :class:`FifoFreeList` can be dropped into the reference
(``mgr.allocator._free = FifoFreeList(order)``) and into this oracle alike; the
CUDA allocator implements the same FIFO policy.
"""

from __future__ import annotations

from collections import deque

import numpy as np

OUT_OF_BLOCKS_MSG = (
    "PagedKVCache: out of blocks (pool size={n}).  "
    "Increase max_blocks or prune more aggressively."
)


class FifoFreeList:
    """Deterministic free list: ``pop`` takes the oldest id, ``add`` appends.

    ``order`` is the initial content (e.g. ``range(n)`` or a seeded
    permutation of it).
    """

    def __init__(self, order):
        self._q = deque(int(b) for b in order)

    def pop(self) -> int:
        if not self._q:
            raise KeyError("pop from an empty free list")
        return self._q.popleft()

    def add(self, b: int) -> None:
        self._q.append(int(b))

    def __len__(self) -> int:
        return len(self._q)

    def __bool__(self) -> bool:
        return bool(self._q)

    def as_list(self) -> list[int]:
        return list(self._q)


class OracleBlockAllocator:
    """``paged_kv_cache.py:21-72``."""

    def __init__(self, num_blocks: int, order=None):
        self.num_blocks = num_blocks
        self.refcounts = [0] * num_blocks
        self._free = FifoFreeList(range(num_blocks) if order is None else order)
        self._peak_used = 0

    @property
    def num_free(self) -> int:          # :33
        return len(self._free)

    @property
    def num_used(self) -> int:          # :37
        return self.num_blocks - len(self._free)

    @property
    def peak_used(self) -> int:         # :41
        return self._peak_used

    def alloc(self) -> int:             # :45-56
        if not self._free:
            raise RuntimeError(OUT_OF_BLOCKS_MSG.format(n=self.num_blocks))
        b = self._free.pop()
        self.refcounts[b] = 1
        used = self.num_blocks - len(self._free)
        if used > self._peak_used:
            self._peak_used = used
        return b

    def ref(self, b: int) -> None:      # :58-60
        assert self.refcounts[b] > 0, f"ref() on free block {b}"
        self.refcounts[b] += 1

    def release(self, b: int) -> None:  # :62-66
        assert self.refcounts[b] > 0, f"release() on free block {b}"
        self.refcounts[b] -= 1
        if self.refcounts[b] == 0:
            self._free.add(b)

    def is_shared(self, b: int) -> bool:  # :68-69
        return self.refcounts[b] > 1


class OracleSeq:
    """``SequenceState`` (``paged_kv_cache.py:80-96``)."""

    def __init__(self, seq_id, L, num_tokens=None, tail=None, tables=None):
        self.seq_id = seq_id
        self.num_tokens = list(num_tokens) if num_tokens else [0] * L
        self.tokens_in_last_block = list(tail) if tail else [0] * L
        self.page_table = [list(t) for t in tables] if tables else [[] for _ in range(L)]


class OraclePagedKV:
    """``PagedKVCacheManager`` (``paged_kv_cache.py:102-455``) on numpy pools.

    ``with_data=False`` keeps only the tables (fast op-stream checks).
    """

    def __init__(self, num_layers, num_kv_heads, head_dim, max_blocks=4096,
                 block_size=16, dtype=np.float32, order=None, with_data=True, elem_bytes=None):
        self.num_layers = num_layers
        self.num_key_value_heads = num_kv_heads
        self.head_dim = head_dim
        self.max_blocks = max_blocks
        self.block_size = block_size
        self.dtype = np.dtype(dtype)
        # bytes per element for get_stats (numpy has no bf16: data may be held wider)
        self.elem_bytes = elem_bytes or self.dtype.itemsize
        self.allocator = OracleBlockAllocator(max_blocks, order)
        self.with_data = with_data
        shape = (max_blocks, block_size, num_kv_heads, head_dim)
        if with_data:
            self.k_pools = [np.zeros(shape, self.dtype) for _ in range(num_layers)]
            self.v_pools = [np.zeros(shape, self.dtype) for _ in range(num_layers)]
        self._sequences: dict[int, OracleSeq] = {}
        self._next_seq_id = 0

    # -- sequences ---------------------------------------------------------
    def allocate_sequence(self) -> int:                    # :143-150
        sid = self._next_seq_id
        self._next_seq_id += 1
        self._sequences[sid] = OracleSeq(sid, self.num_layers)
        return sid

    def fork_sequence(self, parent_id: int) -> int:       # :152-170
        parent = self._sequences[parent_id]
        cid = self._next_seq_id
        self._next_seq_id += 1
        tables = []
        for blocks in parent.page_table:
            tables.append(list(blocks))
            for b in blocks:
                self.allocator.ref(b)
        self._sequences[cid] = OracleSeq(cid, self.num_layers, parent.num_tokens,
                                         parent.tokens_in_last_block, tables)
        return cid

    def free_sequence(self, seq_id: int) -> None:         # :172-176
        seq = self._sequences.pop(seq_id)
        for blocks in seq.page_table:
            for b in blocks:
                self.allocator.release(b)

    # -- append ------------------------------------------------------------
    def _cow_tail(self, layer, table):
        """CoW of a shared tail block (:199-209 and :259-265)."""
        tail = table[-1]
        if self.allocator.is_shared(tail):
            nb = self.allocator.alloc()
            if self.with_data:
                self.k_pools[layer][nb] = self.k_pools[layer][tail]
                self.v_pools[layer][nb] = self.v_pools[layer][tail]
            self.allocator.release(tail)
            table[-1] = nb
            tail = nb
        return tail

    def append_tokens(self, seq_id, layer, k, v) -> None:  # :178-225
        seq = self._sequences[seq_id]
        table = seq.page_table[layer]
        n = k.shape[0]
        written = 0
        while written < n:
            if not table or seq.tokens_in_last_block[layer] == self.block_size:
                table.append(self.allocator.alloc())
                seq.tokens_in_last_block[layer] = 0
            tail = self._cow_tail(layer, table)
            s0 = seq.tokens_in_last_block[layer]
            w = min(self.block_size - s0, n - written)
            if self.with_data:
                self.k_pools[layer][tail, s0:s0 + w] = k[written:written + w]
                self.v_pools[layer][tail, s0:s0 + w] = v[written:written + w]
            written += w
            seq.tokens_in_last_block[layer] += w
        seq.num_tokens[layer] += n

    def append_tokens_batched(self, seq_ids, layer, k, v) -> None:  # :227-284
        if len(seq_ids) == 0:
            return
        dst = []
        for sid in seq_ids:
            seq = self._sequences[sid]
            table = seq.page_table[layer]
            if not table or seq.tokens_in_last_block[layer] == self.block_size:
                table.append(self.allocator.alloc())
                seq.tokens_in_last_block[layer] = 0
            tail = self._cow_tail(layer, table)
            dst.append((tail, seq.tokens_in_last_block[layer]))
            seq.tokens_in_last_block[layer] += 1
            seq.num_tokens[layer] += 1
        if self.with_data:
            for i, (b, s) in enumerate(dst):
                self.k_pools[layer][b, s] = k[i]
                self.v_pools[layer][b, s] = v[i]

    def get_kv_length(self, seq_id) -> int:               # :285-287
        return self._sequences[seq_id].num_tokens[0]

    # -- gather --------------------------------------------------------------
    def gather_indices(self, seq_ids, layer):
        """Flat (block, slot) lists of ``build_packed_kv`` (:316-328)."""
        lens, blk, slt = [], [], []
        for sid in seq_ids:
            seq = self._sequences[sid]
            n = seq.num_tokens[layer]
            lens.append(n)
            rem = n
            for b in seq.page_table[layer]:
                c = min(self.block_size, rem)
                blk.extend([b] * c)
                slt.extend(range(c))
                rem -= c
                if rem == 0:
                    break
        return lens, blk, slt

    def build_packed_kv(self, seq_ids, layer):            # :289-368
        lens, blk, slt = self.gather_indices(seq_ids, layer)
        cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        mx = max(lens) if lens else 0
        if cu[-1] == 0:
            e = np.zeros((0, self.num_key_value_heads, self.head_dim), self.dtype)
            return e, e, np.zeros(len(seq_ids) + 1, np.int32), 0
        b = np.asarray(blk, np.int64)
        s = np.asarray(slt, np.int64)
        return self.k_pools[layer][b, s], self.v_pools[layer][b, s], cu, mx

    # -- sliding window --------------------------------------------------------
    def trim_to_window(self, seq_id, window) -> None:    # :370-417
        seq = self._sequences[seq_id]
        if seq.num_tokens[0] <= window:
            return
        bs = self.block_size
        for layer in range(self.num_layers):
            rem = seq.num_tokens[layer] - window
            table = seq.page_table[layer]
            while rem > 0 and table:
                b = table[0]
                c = min(bs, rem)
                if c >= bs:
                    table.pop(0)
                    self.allocator.release(b)
                    rem -= bs
                else:
                    keep = bs - c
                    if self.allocator.is_shared(b):
                        nb = self.allocator.alloc()
                        if self.with_data:
                            self.k_pools[layer][nb, :keep] = self.k_pools[layer][b, c:c + keep]
                            self.v_pools[layer][nb, :keep] = self.v_pools[layer][b, c:c + keep]
                        self.allocator.release(b)
                        table[0] = nb
                    elif self.with_data:
                        self.k_pools[layer][b, :keep] = self.k_pools[layer][b, c:c + keep].copy()
                        self.v_pools[layer][b, :keep] = self.v_pools[layer][b, c:c + keep].copy()
                    rem = 0
            seq.num_tokens[layer] = window
            if window == 0:
                seq.tokens_in_last_block[layer] = 0
            else:
                t = window % bs
                seq.tokens_in_last_block[layer] = t if t else bs

    # -- stats -------------------------------------------------------------------
    def get_stats(self) -> dict:                          # :419-439
        a = self.allocator
        total = sum(s.num_tokens[0] for s in self._sequences.values())
        bpb = (2 * self.num_layers * self.block_size * self.num_key_value_heads
               * self.head_dim * self.elem_bytes)
        return {
            "num_sequences": len(self._sequences),
            "total_cached_tokens": total,
            "blocks_used": a.num_used,
            "blocks_free": a.num_free,
            "blocks_total": self.max_blocks,
            "blocks_peak": a.peak_used,
            "utilization": a.num_used / self.max_blocks,
            "peak_utilization": a.peak_used / self.max_blocks,
            "pool_memory_bytes": bpb * self.max_blocks,
            "peak_kv_cache_bytes": bpb * a.peak_used,
        }

    def snapshot(self) -> dict:
        """Tables, counters and refcounts in a comparable form."""
        return {
            "seqs": {sid: {"tables": [list(t) for t in s.page_table],
                           "num_tokens": list(s.num_tokens),
                           "tail": list(s.tokens_in_last_block)}
                     for sid, s in sorted(self._sequences.items())},
            "refcounts": list(self.allocator.refcounts),
            "free": self.allocator._free.as_list(),
            "peak": self.allocator.peak_used,
        }
