"""The C-ABI library loads and exports every entry point include/inferd_b200.h declares.

No compute call is made here (no GPU needed): only version / status queries, workspace
sizing and argument validation, which return before touching the device.
"""

from __future__ import annotations

import re
from pathlib import Path

import pytest

from inferd_b200 import _lib

HEADER_DIR = Path(__file__).resolve().parent.parent / "include"


def declared_symbols() -> list[str]:
    names = []
    for h in sorted(HEADER_DIR.glob("*.h")):
        names += re.findall(r"^INFERD_API\s+[\w\s\*]+?\b(inferd_\w+)\s*\(", h.read_text(), re.M)
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ["inferd_reshape_and_cache", "inferd_gather_paged_kv", "inferd_paged_attention",
              "inferd_dense_attention", "inferd_paged_attention_workspace_bytes"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_binding_covers_every_declared_symbol():
    missing = set(declared_symbols()) - set(_lib.exported_symbols())
    assert not missing, f"ctypes binding lacks {sorted(missing)}"


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.inferd_version() >= 100
    assert lib.inferd_status_string(0) == b"ok"
    assert b"pool" in lib.inferd_status_string(_lib.ERR_DEVICE_INDEX)


def test_workspace_sizes():
    lib = _lib.load()
    ws = lib.inferd_paged_attention_workspace_bytes(64, 1, 32, 8, 128, 0)
    assert ws >= lib.inferd_paged_attention_counter_bytes(64, 8) > 0
    assert ws % 256 == 0
    assert lib.inferd_paged_attention_workspace_bytes(0, 1, 32, 8, 128, 0) == 0


def test_argument_validation_without_device():
    lib = _lib.load()
    # invalid sizes are rejected before any device work
    st = lib.inferd_reshape_and_cache(None, None, 0, 0, 0, 0, None, None, None, 1, 0, 128, 16,
                                      4, 2, None, None)
    assert st == _lib.ERR_INVALID_ARGUMENT
    st = lib.inferd_paged_attention(None, None, None, None, None, 4, 0, None, 1, 1, 30, 8, 128,
                                    16, 4, 10, 1.0, 2, None, 0, None, None)
    assert st == _lib.ERR_INVALID_ARGUMENT  # 30 query heads over 8 kv heads
    st = lib.inferd_paged_attention(None, None, None, None, None, 3, 0, None, 1, 1, 32, 8, 128,
                                    16, 4, 10, 1.0, 2, None, 0, None, None)
    assert st == _lib.ERR_INVALID_ARGUMENT  # block-table element size
    st = lib.inferd_gather_paged_kv(None, None, None, None, None, 4, -1, 1, 8, 16, 4, 0, None, None)
    assert st == _lib.ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(IndexError):
        _lib.check(_lib.ERR_DEVICE_INDEX, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_WORKSPACE, "x")


def test_reserved_sms_bounds_without_device():
    # the reserve is host state: negative counts and counts of every SM are refused, a
    # valid one reads back and 0 restores full grids
    lib = _lib.load()
    assert lib.inferd_paged_attention_reserved_sms() == 0
    assert lib.inferd_paged_attention_reserve_sms(-1) == _lib.ERR_INVALID_ARGUMENT
    assert lib.inferd_paged_attention_reserve_sms(1 << 20) == _lib.ERR_INVALID_ARGUMENT
    assert lib.inferd_paged_attention_reserve_sms(8) == _lib.OK
    assert lib.inferd_paged_attention_reserved_sms() == 8
    assert lib.inferd_paged_attention_reserve_sms(0) == _lib.OK
    assert lib.inferd_paged_attention_reserved_sms() == 0
