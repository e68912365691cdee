"""The C-ABI library loads and exports every entry point include/mentat_b200.h declares."""

import ctypes
import os
import re

from mentat_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, "include", "mentat_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mentat_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared()
    assert "mentat_paged_decode" in names and "mentat_gate_step" in names
    assert len(names) >= 14


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    bound = {s[0] for s in _lib.SIGNATURES}
    assert set(declared()) <= bound


def test_abi_version_and_host_side_sizing():
    lib = _lib.load()
    assert lib.mentat_abi_version() == 1
    assert lib.mentat_status_string(1) == b"out of blocks"
    assert ctypes.sizeof(_lib.GateOut) % 8 == 0
    assert lib.mentat_decode_workspace_bytes(8, 16, 128, 10) > 8 * 10 * 16 * 128 * 4
    assert lib.mentat_decode_max_parts(8, 576, 16) >= 3
    # argument errors are reported without touching a device
    assert lib.mentat_kv_init(None, None, None) == -1
    assert lib.mentat_paged_decode(None, 0, None, 0, None, 0, 1, None, 0, 1.0, None, 0, 1, None) == -1


def test_prefill_partial_counts():
    """mentat_prefill_max_parts follows the prefill plan's chunk policy on the host:
    a range of at most 2,048 tokens, or one within 1.5 times the average work per SM,
    is one unit (one partial per query); a long range seen by few queries is cut into
    chunks of about the average work per SM (148 SMs assumed without a device)."""
    lib = _lib.load()
    d = _lib.KVCache()
    d.num_layers, d.num_blocks, d.block_size, d.num_kv_heads, d.head_dim = 1, 1024, 16, 8, 128
    d.dtype, d.max_seqs, d.max_blocks_per_seq = _lib.MENTAT_BF16, 4, 1024
    p = ctypes.byref(d)
    assert lib.mentat_prefill_max_parts(p, 1024, 0, 32) == 1
    assert lib.mentat_prefill_max_parts(p, 2048, 0, 32) == 1
    assert lib.mentat_prefill_max_parts(p, 8192, 0, 32) == 1   # 128 query groups fill the GPU
    # one query after 8,191 cached tokens: 8 units' work spread as 512-token chunks
    assert lib.mentat_prefill_max_parts(p, 1, 8191, 32) == 16
    d.dtype = _lib.MENTAT_F32                                   # the FFMA kernel's groups
    assert lib.mentat_prefill_max_parts(p, 1, 8191, 32) == 16
    assert lib.mentat_prefill_max_parts(p, 0, 10, 32) == 0      # invalid: no queries
    assert lib.mentat_prefill_max_parts(p, 4, 0, 30) == 0       # Hq not a multiple of Hkv
    assert lib.mentat_paged_prefill(None, 0, None, 1, 0, None, 0, 32, None, 0, 1.0, None, 0, 1, None) == -1
