"""C ABI checks that need no GPU: the library loads and exports every entry
point declared in include/*.h; argument validation rejects bad calls before
any device work."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for h in sorted(os.listdir(inc)):
        if not h.endswith(".h"):
            continue
        text = open(os.path.join(inc, h)).read()
        for m in re.finditer(r"(?:KVX_API|ADAPTIVE_ENGINE_EXPORT)\s+[\w\s\*]+?\b(\w+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("kvx_append", "kvx_decode", "kvx_append_decode", "kvx_decode_workspace_init",
              "kvx_compress_int8", "kvx_decompress_int8",
              "kvx_f32_to_f16_trunc", "kvx_f16_trunc_to_f32", "kvx_lru_select",
              "kvx_migrate_frames", "kvx_decode_workspace_bytes", "kvx_tier_create", "kvx_tier_step",
              "kvx_tier_wait_resident", "kvx_tier_mark_read", "kvx_tier_sync", "adaptive_engine_get_api"):
        assert n in names


def test_library_exports_every_declared_symbol():
    import kvx
    missing = [n for n in declared_symbols() if not hasattr(kvx.lib, n)]
    assert not missing, missing


def test_version_and_status_strings():
    import kvx
    assert b"sm_100a" in kvx.lib.kvx_version()
    assert kvx.lib.kvx_status_string(-1) == b"invalid argument"
    assert kvx.lib.kvx_status_string(-2) == b"object pinned"


def test_workspace_size_formula():
    import kvx
    # partials: batch * hq * ceil(max_pages/4) rows of (128 + 2) floats, then
    # one int32 arrival counter per (sequence, q-head), rounded up to 16 bytes
    want = 32 * 24 * 136 * 130 * 4 + 32 * 24 * 4
    assert kvx.decode_workspace_bytes(32, 24, 544) == (want + 15) // 16 * 16
    assert kvx.decode_workspace_bytes(1, 3, 4) % 16 == 0
    assert kvx.decode_workspace_bytes(0, 24, 544) == 0


def test_null_arguments_rejected_without_device_work():
    import kvx
    kv = kvx.KvPaged(0, 0, 1, 1, 8, 128, 16)
    assert kvx.lib.kvx_append(C.byref(kv), None, 1, None, 1, None, None, None, None) == -1
    assert kvx.lib.kvx_decode(C.byref(kv), None, 1, None, 1, 24, None, None, 1, 0.0, None, 0,
                              None, None) == -1
    assert kvx.lib.kvx_compress_int8(None, 1, None, None, 1, 2048, None) == -1
    assert kvx.lib.kvx_migrate_frames(None, 1, None, 1, None, None, 1, 64, 0, 0, None, None) == -1
