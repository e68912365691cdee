"""torch custom operators over the C ABI (``torch.library``).

The three hot-path calls of the public Python API
(``PagedKVCacheManager.append_tokens_batched``, ``attention_backend.attn_decode``,
``gate.Gate``) are registered as torch operators with schemas and fake (meta)
implementations, so torch.compile can trace a caller that uses them.  The
public API calls them through ``paged_decode``, ``append_batched`` and
``gate_step`` below, which go through the operators while torch.compile traces
and call the implementation directly otherwise (eagerly and under CUDA-graph
capture), which saves the dispatcher's host time.  Each call launches on the
current torch stream and returns without synchronising.

A cache is passed as the integer id it registered under (``register_cache``),
because operator arguments are tensors and scalars.
"""

from __future__ import annotations

import ctypes as C
import itertools
import math
import weakref

import torch

from . import _lib

_caches: "weakref.WeakValueDictionary[int, object]" = weakref.WeakValueDictionary()
_ids = itertools.count(1)

MAX_SEQS_PER_LAUNCH = 1024  # mentat_paged_decode's per-launch sequence limit


def register_cache(mgr) -> int:
    """Registers a ``PagedKVCacheManager``; returns the id the operators take."""
    i = next(_ids)
    _caches[i] = mgr
    return i


def _cache(i: int):
    mgr = _caches.get(i)
    if mgr is None:
        raise RuntimeError(f"mentat_b200: no live cache with id {i}")
    return mgr


def _paged_decode(q: torch.Tensor, slots: torch.Tensor, max_len: int, cache: int, layer: int,
                  scale: float, reuse_plan: bool = False) -> torch.Tensor:
    """Tree-aware decode attention of ``q`` (N, Hq, D) over the cached sequences in
    ``slots`` (N,) int32 of layer ``layer``; ``max_len`` is the longest of their
    lengths (it sizes the workspace).  Wraps ``mentat_paged_decode``; with
    ``reuse_plan``, ``mentat_paged_decode_reuse_plan`` (the previous call on this
    cache planned the same sequences for another layer of the same step; batches
    above the per-launch limit always plan)."""
    mgr = _cache(cache)
    lib = _lib.load()
    n, hq, d = q.shape
    out = torch.empty((n, hq, d), device=q.device, dtype=q.dtype)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    fn = lib.mentat_paged_decode_reuse_plan if reuse_plan and n <= MAX_SEQS_PER_LAUNCH else lib.mentat_paged_decode
    for a in range(0, n, MAX_SEQS_PER_LAUNCH):
        b = min(n, a + MAX_SEQS_PER_LAUNCH)
        ws, wsb, parts = mgr.decode_workspace(b - a, hq, max_len)
        _lib.check(fn(
            mgr._descp, layer, slots.data_ptr() + 4 * a, b - a,
            q.data_ptr() + a * q.stride(0) * q.element_size(), q.stride(0), hq,
            out.data_ptr() + a * out.stride(0) * out.element_size(), out.stride(0), scale,
            ws.data_ptr(), wsb, parts, stream), "mentat_paged_decode")
    return out


paged_decode_op = torch.library.custom_op("mentat_b200::paged_decode", mutates_args=(),
                                          device_types="cuda")(_paged_decode)


@paged_decode_op.register_fake
def _paged_decode_fake(q, slots, max_len, cache, layer, scale, reuse_plan=False):
    return torch.empty_like(q)


def _append_batched(k_pool: torch.Tensor, v_pool: torch.Tensor, slots: torch.Tensor, k: torch.Tensor,
                    v: torch.Tensor, cache: int, layer: int) -> None:
    """Appends one token per sequence (rows of ``k``, ``v``: (N, Hkv, D)) to the
    sequences in ``slots`` of layer ``layer``, allocating and copying-on-write on
    the device.  ``k_pool`` / ``v_pool`` are the cache's pools, named so that
    torch knows what the operator writes.  Wraps ``mentat_kv_append_batched``."""
    mgr = _cache(cache)
    lib = _lib.load()
    n = k.shape[0]
    ks, vs = k.stride(0), v.stride(0)
    stream = torch.cuda.current_stream(k.device).cuda_stream
    for a in range(0, n, 1024):
        b = min(n, a + 1024)
        _lib.check(lib.mentat_kv_append_batched(
            mgr._descp, layer, slots.data_ptr() + 4 * a, b - a,
            k.data_ptr() + a * ks * k.element_size(), ks,
            v.data_ptr() + a * vs * v.element_size(), vs, stream), "append_tokens_batched")


append_batched_op = torch.library.custom_op("mentat_b200::append_batched", mutates_args=("k_pool", "v_pool"),
                                            device_types="cuda")(_append_batched)


@append_batched_op.register_fake
def _append_batched_fake(k_pool, v_pool, slots, k, v, cache, layer):
    return None


# The public API calls these wrappers.  Eagerly (and under CUDA-graph capture) they
# call the implementation directly: the dispatcher round trip of a custom
# operator costs about 15 us of host time per call, which a decode step pays
# for every layer.  While torch.compile traces they go through the operators.
def paged_decode(q, slots, max_len, cache, layer, scale, reuse_plan=False):
    if torch.compiler.is_compiling():
        return torch.ops.mentat_b200.paged_decode(q, slots, max_len, cache, layer, scale, reuse_plan)
    return _paged_decode(q, slots, max_len, cache, layer, scale, reuse_plan)


def append_batched(k_pool, v_pool, slots, k, v, cache, layer):
    if torch.compiler.is_compiling():
        return torch.ops.mentat_b200.append_batched(k_pool, v_pool, slots, k, v, cache, layer)
    return _append_batched(k_pool, v_pool, slots, k, v, cache, layer)


def _gate_step(logits: torch.Tensor, hist_ptr: torch.Tensor, hist_ids: torch.Tensor, ema_old: torch.Tensor,
               params: list[float], ints: list[int], out: torch.Tensor) -> None:
    """The fused entropy gate over ``logits`` (N, V) into ``out`` (N records of
    ``mentat_gate_out`` as bytes).  ``params`` = (temperature, penalty, alpha,
    multiplier, soft-explore initial), ``ints`` = (K, max_active, num_active,
    step, soft-explore window[, flags]).  Wraps ``mentat_gate_step``."""
    lib = _lib.load()
    n, V = logits.shape
    p = _lib.GateParams(*params, *ints[:5], ints[5] if len(ints) > 5 else 0)
    stream = torch.cuda.current_stream(logits.device).cuda_stream
    _lib.check(lib.mentat_gate_step(
        logits.data_ptr(), _DT[logits.dtype], n, V, logits.stride(0), hist_ptr.data_ptr(), hist_ids.data_ptr(),
        ema_old.data_ptr(), C.byref(p), out.data_ptr(), stream), "mentat_gate_step")


gate_step_op = torch.library.custom_op("mentat_b200::gate_step", mutates_args=("out",),
                                       device_types="cuda")(_gate_step)


@gate_step_op.register_fake
def _gate_step_fake(logits, hist_ptr, hist_ids, ema_old, params, ints, out):
    return None


def gate_step(logits, hist_ptr, hist_ids, ema_old, params, ints, out):
    if torch.compiler.is_compiling():
        return torch.ops.mentat_b200.gate_step(logits, hist_ptr, hist_ids, ema_old, params, ints, out)
    return _gate_step(logits, hist_ptr, hist_ids, ema_old, params, ints, out)


_DT = {torch.bfloat16: _lib.MENTAT_BF16, torch.float16: _lib.MENTAT_F16, torch.float32: _lib.MENTAT_F32}


def default_scale(d: int) -> float:
    return 1.0 / math.sqrt(d)


def paged_prefill(descp, layer: int, slot: torch.Tensor, pos0: int, q: torch.Tensor, scale: float,
                  out: torch.Tensor = None) -> torch.Tensor:
    """Causal prefill attention of ``q`` (n, Hq, D), query i at position pos0 + i
    of the sequence in ``slot`` (device int32[1]) of the cache described by
    ``descp`` (a ``ctypes.byref`` of ``_lib.KVCache``); its K/V must already be
    cached.  Wraps ``mentat_paged_prefill``, PREFILL_QUERIES_PER_LAUNCH queries
    per call (the workspace grows with queries x partials); the workspace comes
    from torch's caching allocator on the current stream."""
    lib = _lib.load()
    n, hq, d = q.shape
    if out is None:
        out = torch.empty((n, hq, d), device=q.device, dtype=q.dtype)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    for a in range(0, n, PREFILL_QUERIES_PER_LAUNCH):
        m = min(n - a, PREFILL_QUERIES_PER_LAUNCH)
        parts = int(lib.mentat_prefill_max_parts(descp, m, pos0 + a, hq))
        wsb = int(lib.mentat_decode_workspace_bytes(m, hq, d, parts))
        ws = torch.empty(wsb, device=q.device, dtype=torch.uint8)
        _lib.check(lib.mentat_paged_prefill(
            descp, layer, slot.data_ptr(), m, pos0 + a, q.data_ptr() + a * q.stride(0) * q.element_size(),
            q.stride(0), hq, out.data_ptr() + a * out.stride(0) * out.element_size(), out.stride(0), scale,
            ws.data_ptr(), wsb, parts, stream), "mentat_paged_prefill")
    return out


PREFILL_QUERIES_PER_LAUNCH = 8192


def prune_similar(sim: torch.Tensor, group_off: torch.Tensor, parent_key: torch.Tensor, logp: torch.Tensor,
                  threshold: float, max_group: int) -> torch.Tensor:
    """Pair resolution of semantic pruning (``generator.py:446-484``) on the device:
    ``sim`` (m, m) holds the cosine similarities of the leaves of several trees laid
    out tree after tree (``group_off`` int32, the trees' first rows and m);
    ``parent_key`` (int64) is equal for siblings; ``logp`` (float64) the leaves'
    cumulative log-probs.  Returns one uint8 per leaf, 1 for the pruned ones.
    Wraps ``mentat_prune_similar``; the threshold is rounded to ``sim``'s dtype,
    as torch's ``(sim * mask) > threshold`` compares in that dtype."""
    lib = _lib.load()
    m = sim.shape[0]
    out = torch.empty(m, dtype=torch.uint8, device=sim.device)
    if sim.stride(1) != 1:
        sim = sim.contiguous()
    thr = float(torch.tensor(threshold, dtype=sim.dtype).item())
    stream = torch.cuda.current_stream(sim.device).cuda_stream
    _lib.check(lib.mentat_prune_similar(sim.data_ptr(), _DT[sim.dtype], sim.stride(0), group_off.data_ptr(),
                                        group_off.numel() - 1, max_group, parent_key.data_ptr(), logp.data_ptr(),
                                        thr, out.data_ptr(), stream), "mentat_prune_similar")
    return out
