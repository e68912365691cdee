"""ctypes binding of libmentat_b200.so (the C ABI declared in include/mentat_b200.h).

There is no fallback: if the library is missing or cannot be loaded the kernels
fail with an error that says how to build it.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("MENTAT_B200_LIB", _PKG / "libmentat_b200.so"))

MENTAT_OK = 0
MENTAT_F32, MENTAT_BF16, MENTAT_F16 = 0, 1, 2
CTRL_HEAD, CTRL_TAIL, CTRL_PEAK, CTRL_ERROR, CTRL_ERRARG, CTRL_ALLOCS, CTRL_COWS = range(7)
CTRL_WORDS = 16
DEV_OUT_OF_BLOCKS, DEV_REF_FREE, DEV_RELEASE_FREE, DEV_PLAN_OVERFLOW, DEV_TABLE_OVERFLOW = 1, 2, 3, 4, 5
DEV_DECODE_TIMEOUT, DEV_BAD_BLOCK = 6, 7
GATE_MAXK = 8
GATE_SKIP_PEN_ENTROPY, GATE_FLOAT_LOGSUM = 1, 2
NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024
ERR_SCRATCH_LIMIT = -4


class KVCache(C.Structure):
    _fields_ = [
        ("num_layers", C.c_int32), ("num_blocks", C.c_int32), ("block_size", C.c_int32),
        ("num_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("dtype", C.c_int32),
        ("max_seqs", C.c_int32), ("max_blocks_per_seq", C.c_int32),
        ("k_pool", C.c_void_p), ("v_pool", C.c_void_p),
        ("refcounts", C.c_void_p), ("free_ring", C.c_void_p), ("ctrl", C.c_void_p),
        ("tables", C.c_void_p), ("nblocks", C.c_void_p), ("ntok", C.c_void_p),
        ("tail", C.c_void_p), ("scratch", C.c_void_p),
    ]


class GateParams(C.Structure):
    _fields_ = [
        ("temperature", C.c_double), ("penalty", C.c_double), ("alpha", C.c_double),
        ("mult", C.c_double), ("initial", C.c_double), ("K", C.c_int32), ("M", C.c_int32),
        ("num_active", C.c_int32), ("step", C.c_int32), ("window", C.c_int32), ("flags", C.c_int32),
    ]


class GateOut(C.Structure):
    _fields_ = [
        ("entropy", C.c_double), ("entropy_acc", C.c_double), ("pen_entropy", C.c_double),
        ("ema", C.c_double), ("tau", C.c_double), ("branch", C.c_int32), ("argmax", C.c_int32),
        ("argmax_lp", C.c_float), ("topk_ids", C.c_int32 * GATE_MAXK),
        ("topk_lps", C.c_float * GATE_MAXK), ("pad", C.c_int32 * 3),
    ]


_P, _I32, _I64, _F = C.c_void_p, C.c_int32, C.c_int64, C.c_float
_KV = C.POINTER(KVCache)
# (name, restype, argtypes) for every entry point of include/mentat_b200.h
SIGNATURES = [
    ("mentat_abi_version", C.c_int, []),
    ("mentat_status_string", C.c_char_p, [C.c_int]),
    ("mentat_kv_scratch_ints", _I64, [_I32]),
    ("mentat_kv_init", C.c_int, [_KV, _P, _P]),
    ("mentat_kv_seq_reset", C.c_int, [_KV, _I32, _P]),
    ("mentat_kv_fork", C.c_int, [_KV, _I32, _I32, _I32, _P]),
    ("mentat_kv_free", C.c_int, [_KV, _I32, _I32, _P]),
    ("mentat_kv_append_batched", C.c_int, [_KV, _I32, _P, _I32, _P, _I64, _P, _I64, _P]),
    ("mentat_kv_append", C.c_int, [_KV, _I32, _I32, _I32, _P, _I64, _P, _I64, _P]),
    ("mentat_kv_trim", C.c_int, [_KV, _I32, _I32, _P]),
    ("mentat_kv_gather", C.c_int, [_KV, _I32, _P, _I32, _P, _I64, _P, _P, _P]),
    ("mentat_decode_workspace_bytes", _I64, [_I32, _I32, _I32, _I32]),
    ("mentat_decode_max_parts", _I32, [_I32, _I32, _I32]),
    ("mentat_paged_decode", C.c_int, [_KV, _I32, _P, _I32, _P, _I64, _I32, _P, _I64, _F, _P, _I64, _I32, _P]),
    ("mentat_paged_decode_reuse_plan", C.c_int,
     [_KV, _I32, _P, _I32, _P, _I64, _I32, _P, _I64, _F, _P, _I64, _I32, _P]),
    ("mentat_paged_decode_noalloc", C.c_int, [_KV, _I32, _P, _I32, _P, _I64, _I32, _P, _I64, _F, _I32, _P]),
    ("mentat_decode_set_wait_probe", C.c_int, [_I64]),
    ("mentat_prefill_max_parts", _I32, [_KV, _I32, _I32, _I32]),
    ("mentat_paged_prefill", C.c_int,
     [_KV, _I32, _P, _I32, _I32, _P, _I64, _I32, _P, _I64, _F, _P, _I64, _I32, _P]),
    ("mentat_profile_enable", C.c_int, [_I32]),
    ("mentat_profile_collect", C.c_int, [C.POINTER(C.c_double), C.POINTER(_I32)]),
    ("mentat_kernel_launch_count", C.c_int64, []),
    ("mentat_gate_step", C.c_int, [_P, _I32, _I32, _I32, _I64, _P, _P, _P, C.POINTER(GateParams), _P, _P]),
    ("mentat_prune_similar", C.c_int, [_P, _I32, _I64, _P, _I32, _I32, _P, _P, _F, _P, _P]),
]

_lib = None


def load() -> C.CDLL:
    """Load the library once; raise if it is missing (no CPU fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"libmentat_b200.so not found at {LIB_PATH}; build it with "
                           "`python -m mentat_b200.build` (nvcc, sm_100a)")
    lib = C.CDLL(str(LIB_PATH))
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.mentat_abi_version() != 1:
        raise RuntimeError("libmentat_b200.so ABI mismatch")
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != MENTAT_OK:
        msg = load().mentat_status_string(status).decode()
        raise RuntimeError(f"{what} failed: {msg} ({status})")
