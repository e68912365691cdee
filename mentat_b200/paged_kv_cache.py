"""Drop-in ``PagedKVCacheManager`` backed by the device-resident allocator.

Mirrors ``core/paged_kv_cache.py`` of SkyeGunasekaran/MENTAT: same constructor,
method names, argument meaning, return values and exceptions.  The block
allocator (refcounts, free FIFO), the per-layer page tables and the counters
live in device memory and are changed only by kernels of libmentat_b200, so
fork, free, append and copy-on-write never wait for the host.  The host keeps
the seq-id -> slot map and a mirror of the counters that do not depend on
block ids (num_tokens, tokens_in_last_block, table lengths).

Differences from the reference, all deliberate:

* The free list is a FIFO of block ids (``free_order`` sets its initial
  order, default ``0..max_blocks-1``).  The reference pops from a CPython
  ``set``, whose order is an interpreter detail (``paged_kv_cache.py:29,51``).
* Errors found on the device (out of blocks, ``paged_kv_cache.py:46-50``) are
  raised at the next synchronisation point: ``check()``, ``get_stats()``,
  ``allocator`` reads, or after every call when ``strict=True``.  Host-side
  errors (``KeyError`` for an unknown ``seq_id``) are raised immediately.
* ``build_packed_kv`` returns lazy :class:`PagedKV` handles instead of
  gathered tensors; ``mentat_b200.attention_backend.attn_decode`` reads the
  blocks in place.  ``PagedKV.materialize()`` produces the reference tensors.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib, ops

_DTYPES = {torch.float32: _lib.MENTAT_F32, torch.bfloat16: _lib.MENTAT_BF16, torch.float16: _lib.MENTAT_F16}

OUT_OF_BLOCKS_MSG = ("PagedKVCache: out of blocks (pool size={n}).  "
                     "Increase max_blocks or prune more aggressively.")


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


@dataclass
class SequenceState:
    """Host mirror of ``SequenceState`` (``paged_kv_cache.py:80-96``) plus its
    device slot; the page table itself lives on the device."""
    seq_id: int
    num_layers: int
    slot: int
    num_tokens: list = field(default_factory=list)
    tokens_in_last_block: list = field(default_factory=list)
    num_blocks: list = field(default_factory=list)

    def __post_init__(self):
        if not self.num_tokens:
            self.num_tokens = [0] * self.num_layers
        if not self.tokens_in_last_block:
            self.tokens_in_last_block = [0] * self.num_layers
        if not self.num_blocks:
            self.num_blocks = [0] * self.num_layers


class DeviceBlockAllocator:
    """Read-only view of the device allocator with ``BlockAllocator``'s
    attribute names (``paged_kv_cache.py:21-72``).  Every read synchronises."""

    def __init__(self, mgr: "PagedKVCacheManager"):
        self._m = mgr
        self.num_blocks = mgr.max_blocks

    def _ctrl(self):
        self._m.check()
        return self._m._ctrl_host()

    @property
    def num_free(self) -> int:
        c = self._ctrl()
        return int(c[_lib.CTRL_TAIL] - c[_lib.CTRL_HEAD])

    @property
    def num_used(self) -> int:
        return self.num_blocks - self.num_free

    @property
    def peak_used(self) -> int:
        return int(self._ctrl()[_lib.CTRL_PEAK])

    @property
    def refcounts(self) -> list:
        self._m.check()
        return self._m._refcounts.tolist()

    def free_list(self) -> list:
        """Free block ids in pop order."""
        c = self._ctrl()
        ring = self._m._free_ring.tolist()
        n, head = self.num_blocks, int(c[_lib.CTRL_HEAD])
        return [ring[(head + k) % n] for k in range(int(c[_lib.CTRL_TAIL]) - head)]

    def is_shared(self, b: int) -> bool:
        return self.refcounts[b] > 1

    def can_alloc(self, n: int = 1) -> bool:
        return self.num_free >= n


class PagedKV:
    """Lazy stand-in for one packed K or V tensor of ``build_packed_kv``.

    Carries what the decode kernel needs (cache, layer, device slots, lengths)
    and looks like the ``(total_tokens, Hkv, D)`` tensor it replaces."""

    def __init__(self, mgr, layer, seq_ids, slots_dev, lens, which):
        self.cache = mgr
        self.layer = layer
        self.seq_ids = seq_ids
        self.slots = slots_dev
        self.lens = lens
        self.which = which  # "k" or "v"
        self.total = sum(lens)
        self.shape = torch.Size((self.total, mgr.num_key_value_heads, mgr.head_dim))
        self.dtype = mgr.dtype
        self.device = mgr.device

    def size(self, dim=None):
        return self.shape if dim is None else self.shape[dim]

    def dim(self):
        return 3

    def materialize(self) -> torch.Tensor:
        k, v = self.cache._gather(self.layer, self.slots, self.lens)
        return k if self.which == "k" else v


class _PinnedRing:
    """Small host-to-device int32 uploads through reused page-locked buffers.

    Each step's sequence lengths change, so a fresh pinned tensor per upload
    would keep the pinned-memory allocator busy; a buffer here is rewritten
    only after the copy that last read it has completed (its event).
    """

    def __init__(self, device, depth: int = 16, cap: int = 1024):
        self.device = device
        self.bufs = [torch.empty(cap, dtype=torch.int32, pin_memory=True) for _ in range(depth)]
        self.views = [b.numpy() for b in self.bufs]
        self.events = [None] * depth
        self.i = 0

    def upload(self, values) -> torch.Tensor:
        """``values``: int32 numpy array or CPU tensor; returns a device copy."""
        if isinstance(values, torch.Tensor):
            values = values.numpy()
        n = values.size
        k = self.i
        self.i = (k + 1) % len(self.bufs)
        if self.events[k] is not None:
            self.events[k].synchronize()
        if self.bufs[k].numel() < n:
            self.bufs[k] = torch.empty(max(n, 2 * self.bufs[k].numel()), dtype=torch.int32, pin_memory=True)
            self.views[k] = self.bufs[k].numpy()
        self.views[k][:n] = values.reshape(-1)
        buf = self.bufs[k][:n]
        dev = torch.empty(n, dtype=torch.int32, device=self.device)
        dev.copy_(buf, non_blocking=True)
        ev = self.events[k] if self.events[k] is not None else torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.events[k] = ev
        return dev


class PagedKVCacheManager:
    """``PagedKVCacheManager`` (``core/paged_kv_cache.py:102-455``) on the device."""

    def __init__(self, num_layers: int, num_key_value_heads: int, head_dim: int,
                 max_blocks: int = 4096, block_size: int = 16,
                 device: str | torch.device = "cuda", dtype: torch.dtype = torch.bfloat16,
                 *, max_seqs: int = 256, max_blocks_per_seq: int | None = None,
                 free_order=None, strict: bool = False):
        self.num_layers = num_layers
        self.num_key_value_heads = num_key_value_heads
        self.head_dim = head_dim
        self.max_blocks = max_blocks
        self.block_size = block_size
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("mentat_b200 runs on CUDA devices only")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        if dtype not in _DTYPES:
            raise TypeError(f"unsupported cache dtype {dtype}")
        self.dtype = dtype
        self.strict = strict
        self.max_seqs = max_seqs
        self.max_blocks_per_seq = min(max_blocks, max_blocks_per_seq or max_blocks)
        # table row stride: a multiple of 4 entries keeps every row 16-byte aligned for vector loads
        self._table_stride = (self.max_blocks_per_seq + 3) // 4 * 4
        self._lib = _lib.load()

        dev, L, mbps = self.device, num_layers, self._table_stride
        shape = (L, max_blocks, block_size, num_key_value_heads, head_dim)
        self._k_all = torch.zeros(shape, device=dev, dtype=dtype)
        self._v_all = torch.zeros(shape, device=dev, dtype=dtype)
        self.k_pools = [self._k_all[i] for i in range(L)]
        self.v_pools = [self._v_all[i] for i in range(L)]
        i32 = dict(device=dev, dtype=torch.int32)
        self._refcounts = torch.zeros(max_blocks, **i32)
        self._free_ring = torch.zeros(max_blocks, **i32)
        self._ctrl = torch.zeros(_lib.CTRL_WORDS, device=dev, dtype=torch.int64)
        self._tables = torch.full((L, max_seqs, mbps), -1, **i32)
        self._nblocks = torch.zeros((L, max_seqs), **i32)
        self._ntok = torch.zeros((L, max_seqs), **i32)
        self._tail = torch.zeros((L, max_seqs), **i32)
        self._scratch = torch.zeros(int(self._lib.mentat_kv_scratch_ints(max_seqs)), **i32)
        self._ctrl_pinned = torch.zeros(_lib.CTRL_WORDS, dtype=torch.int64, pin_memory=True)

        d = _lib.KVCache()
        d.num_layers, d.num_blocks, d.block_size = L, max_blocks, block_size
        d.num_kv_heads, d.head_dim, d.dtype = num_key_value_heads, head_dim, _DTYPES[dtype]
        d.max_seqs, d.max_blocks_per_seq = max_seqs, mbps
        d.k_pool, d.v_pool = self._k_all.data_ptr(), self._v_all.data_ptr()
        d.refcounts, d.free_ring = self._refcounts.data_ptr(), self._free_ring.data_ptr()
        d.ctrl, d.tables = self._ctrl.data_ptr(), self._tables.data_ptr()
        d.nblocks, d.ntok = self._nblocks.data_ptr(), self._ntok.data_ptr()
        d.tail, d.scratch = self._tail.data_ptr(), self._scratch.data_ptr()
        self._desc = d
        self._descp = C.byref(d)

        order = None
        if free_order is not None:
            ids = [int(b) for b in free_order]
            if sorted(ids) != list(range(max_blocks)):
                raise ValueError("free_order must list every block id 0..max_blocks-1 once")
            order = torch.tensor(ids, dtype=torch.int32).to(dev)
        with torch.cuda.device(dev):
            _lib.check(self._lib.mentat_kv_init(self._descp, order.data_ptr() if order is not None else None,
                                                _stream(dev)), "mentat_kv_init")
        self.allocator = DeviceBlockAllocator(self)
        self._sequences: dict[int, SequenceState] = {}
        self._free_slots = list(range(max_seqs - 1, -1, -1))
        self._next_seq_id = 0
        self._cache: dict = {}
        self._ws = None
        self._uploads = _PinnedRing(self.device)
        self._op_id = ops.register_cache(self)
        self._ws_bytes = 0

    # ------------------------------------------------------------------ util
    def _s(self) -> int:
        return _stream(self.device)

    def _ctrl_host(self):
        self._ctrl_pinned.copy_(self._ctrl, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return self._ctrl_pinned.tolist()

    def check(self) -> None:
        """Raise the first error the device recorded (reference exception types)."""
        c = self._ctrl_host()
        err, arg = int(c[_lib.CTRL_ERROR]), int(c[_lib.CTRL_ERRARG])
        if err == 0:
            return
        if err == _lib.DEV_OUT_OF_BLOCKS:
            raise RuntimeError(OUT_OF_BLOCKS_MSG.format(n=self.max_blocks))
        if err == _lib.DEV_REF_FREE:
            raise AssertionError(f"ref() on free block {arg}")
        if err == _lib.DEV_RELEASE_FREE:
            raise AssertionError(f"release() on free block {arg}")
        if err == _lib.DEV_TABLE_OVERFLOW:
            raise RuntimeError(f"PagedKVCache: sequence table overflow (slot {arg}, "
                               f"max_blocks_per_seq={self.max_blocks_per_seq})")
        if err == _lib.DEV_PLAN_OVERFLOW:
            raise RuntimeError("mentat_b200: decode plan workspace overflow")
        if err == _lib.DEV_BAD_BLOCK:
            raise AssertionError(f"block table entry {arg} outside the pool (max_blocks={self.max_blocks})")
        if err == _lib.DEV_DECODE_TIMEOUT:
            raise RuntimeError(f"mentat_b200: a decode kernel's bounded wait gave up (stage {arg}); "
                               "that call's output is invalid")
        raise RuntimeError(f"mentat_b200 device error {err} ({arg})")

    def clear_error(self) -> None:
        """Forget the recorded device error (after the caller has handled it)."""
        self._ctrl[_lib.CTRL_ERROR:_lib.CTRL_ERRARG + 1].zero_()

    def _after(self):
        if self.strict:
            self.check()

    def _remember(self, key, make):
        t = self._cache.get(key)
        if t is None:
            if len(self._cache) > 64:
                self._cache.clear()
            t = self._cache[key] = make()
        return t

    def _slots_dev(self, seq_ids) -> torch.Tensor:
        def make():
            seqs = self._sequences
            return self._uploads.upload(np.fromiter((seqs[s].slot for s in seq_ids), np.int32, len(seq_ids)))
        return self._remember(("slots",) + tuple(seq_ids), make)

    def _cu_seqlens(self, lens) -> torch.Tensor:
        def make():
            a = np.zeros(len(lens) + 1, np.int32)
            np.cumsum(lens, out=a[1:])
            return self._uploads.upload(a)
        return self._remember(("cu",) + tuple(lens), make)

    # ------------------------------------------------------------- sequences
    def _new_slot(self) -> int:
        if not self._free_slots:
            raise RuntimeError(f"PagedKVCache: out of sequence slots (max_seqs={self.max_seqs})")
        return self._free_slots.pop()

    def allocate_sequence(self) -> int:                     # :143-150
        slot = self._new_slot()
        sid = self._next_seq_id
        self._next_seq_id += 1
        self._sequences[sid] = SequenceState(sid, self.num_layers, slot)
        _lib.check(self._lib.mentat_kv_seq_reset(self._descp, slot, self._s()), "allocate_sequence")
        return sid

    def fork_sequence(self, parent_id: int) -> int:         # :152-170
        parent = self._sequences[parent_id]
        slot = self._new_slot()
        cid = self._next_seq_id
        self._next_seq_id += 1
        self._sequences[cid] = SequenceState(cid, self.num_layers, slot, list(parent.num_tokens),
                                             list(parent.tokens_in_last_block), list(parent.num_blocks))
        _lib.check(self._lib.mentat_kv_fork(self._descp, parent.slot, slot, max(parent.num_blocks), self._s()),
                   "fork_sequence")
        self._after()
        return cid

    def free_sequence(self, seq_id: int) -> None:           # :172-176
        seq = self._sequences.pop(seq_id)
        _lib.check(self._lib.mentat_kv_free(self._descp, seq.slot, max(seq.num_blocks), self._s()),
                   "free_sequence")
        self._free_slots.append(seq.slot)
        self._cache.clear()
        self._after()

    # ----------------------------------------------------------------- append
    def _rows(self, t: torch.Tensor, n: int):
        if t.dtype != self.dtype:
            t = t.to(self.dtype)
        if t.device != self.device:
            t = t.to(self.device)
        t = t.reshape(n, self.num_key_value_heads, self.head_dim)
        if t.stride(2) != 1 or t.stride(1) != self.head_dim:
            t = t.contiguous()
        return t, t.stride(0)

    def _mirror_append(self, seq: SequenceState, layer: int, n: int) -> None:
        bs = self.block_size
        nb, tf = seq.num_blocks[layer], seq.tokens_in_last_block[layer]
        w = 0
        while w < n:
            if nb == 0 or tf == bs:
                nb += 1
                tf = 0
            c = min(bs - tf, n - w)
            tf += c
            w += c
        if nb > self.max_blocks_per_seq:
            if self.max_blocks_per_seq >= self.max_blocks:
                # one sequence cannot hold more distinct blocks than the pool has
                raise RuntimeError(OUT_OF_BLOCKS_MSG.format(n=self.max_blocks))
            raise RuntimeError(f"PagedKVCache: sequence {seq.seq_id} needs {nb} blocks per layer, "
                               f"max_blocks_per_seq={self.max_blocks_per_seq}")
        seq.num_blocks[layer], seq.tokens_in_last_block[layer] = nb, tf
        seq.num_tokens[layer] += n

    def mirror_decode_step(self, seq_ids) -> None:
        """Host bookkeeping of one token appended to every layer of each sequence,
        for callers that append on the device without going through this class
        (a replayed CUDA graph of the decode step)."""
        L, bs, cap = self.num_layers, self.block_size, self.max_blocks_per_seq
        for s in seq_ids:
            seq = self._sequences[s]
            nt, nb, tf = seq.num_tokens, seq.num_blocks, seq.tokens_in_last_block
            n0, b0, t0 = nt[0], nb[0], tf[0]
            if nt.count(n0) == L and nb.count(b0) == L and tf.count(t0) == L:
                # every layer alike (the decode case): one token, inline
                if b0 == 0 or t0 == bs:
                    b0, t0 = b0 + 1, 1
                    if b0 > cap:
                        self._mirror_append(seq, 0, 1)  # raises the reference's error
                else:
                    t0 += 1
                nt[:] = [n0 + 1] * L
                nb[:] = [b0] * L
                tf[:] = [t0] * L
            else:
                for layer in range(L):
                    self._mirror_append(seq, layer, 1)

    def append_tokens(self, seq_id: int, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> None:
        seq = self._sequences[seq_id]                       # :178-225
        n = k.shape[0]
        if n == 0:
            return
        k, ks = self._rows(k, n)
        v, vs = self._rows(v, n)
        self._mirror_append(seq, layer_idx, n)
        _lib.check(self._lib.mentat_kv_append(self._descp, layer_idx, seq.slot, n, k.data_ptr(), ks,
                                              v.data_ptr(), vs, self._s()), "append_tokens")
        self._after()

    def append_tokens_batched(self, seq_ids, layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> None:
        N = len(seq_ids)                                    # :227-284
        if N == 0:
            return
        seqs = [self._sequences[s] for s in seq_ids]  # an unknown id raises before any change
        k, ks = self._rows(k, N)
        v, vs = self._rows(v, N)
        # host mirror of one token per sequence, inline (this runs for every layer of
        # every decode step); the general walk only where a new block would overflow
        bs, cap, L = self.block_size, self.max_blocks_per_seq, layer_idx
        for s in seqs:
            nb, tf = s.num_blocks[L], s.tokens_in_last_block[L]
            if nb == 0 or tf == bs:
                if nb + 1 > cap:
                    self._mirror_append(s, L, 1)  # raises the reference's error
                s.num_blocks[L], s.tokens_in_last_block[L] = nb + 1, 1
            else:
                s.tokens_in_last_block[L] = tf + 1
            s.num_tokens[L] += 1
        slots = self._slots_dev(seq_ids)
        ops.append_batched(self._k_all, self._v_all, slots, k, v, self._op_id, layer_idx)
        self._after()

    def get_kv_length(self, seq_id: int) -> int:            # :285-287
        return self._sequences[seq_id].num_tokens[0]

    # ------------------------------------------------------------------ gather
    def build_packed_kv(self, seq_ids, layer_idx: int):     # :289-368
        """Lazy handles ``(k, v, cu_seqlens_k, max_seqlen_k)``; nothing is gathered."""
        lens = [self._sequences[s].num_tokens[layer_idx] for s in seq_ids]
        slots = self._slots_dev(seq_ids)
        cu = self._cu_seqlens(lens)
        mx = max(lens) if lens else 0
        k = PagedKV(self, layer_idx, list(seq_ids), slots, lens, "k")
        v = PagedKV(self, layer_idx, list(seq_ids), slots, lens, "v")
        return k, v, cu, mx

    def _gather(self, layer, slots, lens):
        total = sum(lens)
        shape = (total, self.num_key_value_heads, self.head_dim)
        ok = torch.empty(shape, device=self.device, dtype=self.dtype)
        ov = torch.empty(shape, device=self.device, dtype=self.dtype)
        if total:
            cu = self._cu_seqlens(lens)
            _lib.check(self._lib.mentat_kv_gather(self._descp, layer, slots.data_ptr(), len(lens), cu.data_ptr(),
                                                  total, ok.data_ptr(), ov.data_ptr(), self._s()), "gather")
        return ok, ov

    def packed_kv_tensors(self, seq_ids, layer_idx: int):
        """The reference's materialised return value (for non-kernel consumers)."""
        k, v, cu, mx = self.build_packed_kv(seq_ids, layer_idx)
        pk, pv = self._gather(layer_idx, k.slots, k.lens)
        return pk, pv, cu, mx

    # --------------------------------------------------------- decode workspace
    def decode_workspace(self, n: int, hq: int, max_len: int):
        """The decode workspace for n sequences of up to max_len tokens: (tensor,
        bytes, partials per sequence).  The partial count is a capacity, so the
        last answer is reused while it covers the request (lengths grow by one per
        step), and a new one is sized with headroom."""
        m = self._ws_memo
        if m is not None and n <= m[0] and hq == m[1] and max_len <= m[2]:
            return self._ws, self._ws_bytes, m[3]
        if m is not None and hq == m[1]:
            n, max_len = max(n, m[0]), max(max_len, m[2])
        max_len += 256
        parts = int(self._lib.mentat_decode_max_parts(n, max_len, self.block_size))
        need = int(self._lib.mentat_decode_workspace_bytes(n, hq, self.head_dim, parts))
        if self._ws is None or self._ws_bytes < need:
            if self._ws is not None and self._ws_pinned:
                # captured CUDA graphs hold the old address: it must stay allocated
                self._ws_retired.append(self._ws)
            self._ws_bytes = max(need, int(self._ws_bytes * 1.5))
            self._ws = torch.empty(self._ws_bytes, device=self.device, dtype=torch.uint8)
        self._ws_memo = (n, hq, max_len, parts)
        return self._ws, self._ws_bytes, parts

    _ws_memo = None
    _ws_pinned = False

    def pin_workspace(self) -> None:
        """From now on a workspace that is outgrown stays allocated (for the
        lifetime of the cache), because CUDA graphs captured over it keep
        writing to its address on every replay."""
        if not self._ws_pinned:
            self._ws_pinned = True
            self._ws_retired = []

    # ---------------------------------------------------------------- prefill
    def prefill_attention(self, seq_id: int, layer_idx: int, q: torch.Tensor, scale: float = None) -> torch.Tensor:
        """Causal attention of the last n tokens of ``seq_id`` in layer ``layer_idx``,
        whose K/V ``append_tokens`` has already cached: ``q`` (n, Hq, D) are their
        queries, query i at position num_tokens - n + i.  Returns (n, Hq, D).  The
        paged form of the reference's prefill attention (``attn_prefill``,
        ``attention_backend.py:175-189``, over the K/V before they were cached);
        with n < num_tokens it is a chunk of a longer prompt."""
        seq = self._sequences[seq_id]
        n, hq, d = q.shape
        if d != self.head_dim or hq % self.num_key_value_heads:
            raise ValueError("q shape does not match the cache geometry")
        if q.dtype != self.dtype:
            raise TypeError(f"q dtype {q.dtype} differs from the cache dtype {self.dtype}")
        pos0 = seq.num_tokens[layer_idx] - n
        if pos0 < 0:
            raise ValueError(f"{n} queries but only {seq.num_tokens[layer_idx]} cached tokens")
        if q.stride(2) != 1 or q.stride(1) != d:
            q = q.contiguous()
        out = ops.paged_prefill(self._descp, layer_idx, self._slots_dev([seq_id]), pos0, q,
                                ops.default_scale(d) if scale is None else scale)
        self._after()
        return out

    # ----------------------------------------------------------- sliding window
    def trim_to_window(self, seq_id: int, window_size: int) -> None:   # :370-417
        seq = self._sequences[seq_id]
        if seq.num_tokens[0] <= window_size:
            return
        bs = self.block_size
        for layer in range(self.num_layers):
            rem = seq.num_tokens[layer] - window_size
            nb = seq.num_blocks[layer]
            while rem > 0 and nb > 0:
                if min(bs, rem) >= bs:
                    nb -= 1
                    rem -= bs
                else:
                    rem = 0
            seq.num_blocks[layer] = nb
            seq.num_tokens[layer] = window_size
            t = window_size % bs
            seq.tokens_in_last_block[layer] = 0 if window_size == 0 else (t if t else bs)
        _lib.check(self._lib.mentat_kv_trim(self._descp, seq.slot, window_size, self._s()), "trim_to_window")
        self._cache.clear()
        self._after()

    # ------------------------------------------------------------------ stats
    def get_stats(self) -> dict:                            # :419-439
        self.check()
        c = self._ctrl_pinned.tolist()
        free = int(c[_lib.CTRL_TAIL] - c[_lib.CTRL_HEAD])
        used, peak = self.max_blocks - free, int(c[_lib.CTRL_PEAK])
        total = sum(s.num_tokens[0] for s in self._sequences.values())
        bpb = 2 * self.num_layers * self.block_size * self.num_key_value_heads * self.head_dim * self.dtype_size
        return {
            "num_sequences": len(self._sequences),
            "total_cached_tokens": total,
            "blocks_used": used,
            "blocks_free": free,
            "blocks_total": self.max_blocks,
            "blocks_peak": peak,
            "utilization": used / self.max_blocks,
            "peak_utilization": peak / self.max_blocks,
            "pool_memory_bytes": bpb * self.max_blocks,
            "peak_kv_cache_bytes": bpb * peak,
        }

    def kernel_counters(self) -> dict:
        """Allocations and copy-on-write copies done on the device so far."""
        c = self._ctrl_host()
        return {"allocs": int(c[_lib.CTRL_ALLOCS]), "cow_copies": int(c[_lib.CTRL_COWS])}

    @property
    def dtype_size(self) -> int:
        return torch.tensor([], dtype=self.dtype).element_size()

    # ------------------------------------------------------------ inspection
    def page_table(self, seq_id: int, layer: int) -> list:
        seq = self._sequences[seq_id]
        self.check()
        return self._tables[layer, seq.slot, : seq.num_blocks[layer]].tolist()

    def sequence_snapshot(self) -> dict:
        """Tables and counters of every live sequence, read from the device."""
        self.check()
        tabs = self._tables.cpu()
        nb, nt, tl = self._nblocks.cpu(), self._ntok.cpu(), self._tail.cpu()
        out = {}
        for sid, s in sorted(self._sequences.items()):
            out[sid] = {
                "tables": [tabs[l, s.slot, : int(nb[l, s.slot])].tolist() for l in range(self.num_layers)],
                "num_tokens": [int(nt[l, s.slot]) for l in range(self.num_layers)],
                "tail": [int(tl[l, s.slot]) for l in range(self.num_layers)],
            }
        return out

    def __repr__(self) -> str:
        stats = self.get_stats()
        return (f"PagedKVCacheManager(layers={self.num_layers}, heads={self.num_key_value_heads}, "
                f"head_dim={self.head_dim}, block_size={self.block_size}, "
                f"blocks={stats['blocks_used']}/{self.max_blocks}, "
                f"seqs={stats['num_sequences']}, tokens={stats['total_cached_tokens']})")
