"""The C-ABI library loads, exports every symbol include/exl3b.h declares, and declines bad calls
before launching anything (no GPU needed: declined calls return before any CUDA work)."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT
from exl3rocm import _lib

HEADER = os.path.join(ROOT, "include", "exl3b.h")


def declared_symbols() -> list[str]:
    text = open(HEADER).read()
    return sorted(set(re.findall(r"EXL3B_API\s+[\w\s\*]+?\b(exl3b_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("exl3b_version", "exl3b_dequant", "exl3b_decode_states", "exl3b_had128", "exl3b_linear",
                 "exl3b_linear_grouped", "exl3b_linear_workspace_bytes"):
        assert must in names


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name
    assert set(declared_symbols()) <= set(_lib.SIGNATURES), "ctypes table misses a declared symbol"


def test_version_and_status_strings():
    L = _lib.lib()
    assert L.exl3b_version() >= 0x000100
    assert b"declined" in L.exl3b_status_string(_lib.EXL3B_DECLINED)
    assert b"workspace" in L.exl3b_status_string(_lib.EXL3B_WORKSPACE)


def test_workspace_size_grows_with_rows_and_columns():
    L = _lib.lib()
    a = L.exl3b_linear_workspace_bytes(1, 5120, 1, 5120)
    b = L.exl3b_linear_workspace_bytes(16, 5120, 1, 5120)
    c = L.exl3b_linear_workspace_bytes(1, 5120, 2, 34816)
    assert 0 < a < b and a < c
    assert L.exl3b_linear_workspace_bytes(0, 5120, 1, 5120) == 0


FAKE = ctypes.c_void_p(0x10000)  # never dereferenced: every call below is declined on the host


@pytest.mark.parametrize("m,k,n,K,cb,expect", [
    (17, 256, 128, 4, 2, _lib.EXL3B_DECLINED),   # more rows than the GEMV takes
    (1, 200, 128, 4, 2, _lib.EXL3B_DECLINED),    # k not a multiple of 128
    (1, 256, 100, 4, 2, _lib.EXL3B_DECLINED),    # n not a multiple of 128
    (1, 256, 128, 9, 2, _lib.EXL3B_DECLINED),    # K out of range
    (1, 256, 128, 4, 3, _lib.EXL3B_DECLINED),    # codebook out of range
])
def test_linear_declines_before_launch(m, k, n, K, cb, expect):
    L = _lib.lib()
    st = L.exl3b_linear(FAKE, m, k, FAKE, n, K, cb, FAKE, FAKE, FAKE, n, FAKE, 1 << 30, None)
    assert st == expect


@pytest.mark.parametrize("m,k,n,K,cb", [
    (17, 256, 128, 4, 2), (0, 256, 128, 4, 2), (1, 200, 128, 4, 2), (1, 256, 100, 4, 2),
    (1, 256, 128, 9, 2), (1, 256, 128, 0, 2), (1, 256, 128, 4, 3), (1, 256, 128 * 8193, 4, 2),
])
def test_supported_query_agrees_with_declines(m, k, n, K, cb):
    L = _lib.lib()
    assert L.exl3b_linear_supported(m, k, n, K, cb) == 0
    assert L.exl3b_linear(FAKE, m, k, FAKE, n, K, cb, FAKE, FAKE, FAKE, n, FAKE, 1 << 30, None) == \
        _lib.EXL3B_DECLINED


def test_supported_query_takes_decode_shapes():
    from exl3rocm import ops
    L = _lib.lib()
    for m in (1, 4, 16):
        for K in range(1, 9):
            for cb in (0, 1, 2, 2 | ops.X_BF16, 2 | ops.Y_ADD):
                assert L.exl3b_linear_supported(m, 5120, 34816, K, cb) == 1
    assert ops.linear_supported(1, 5120, 5120, 4, False, True)
    assert not ops.linear_supported(32, 5120, 5120, 4, False, True)


def test_linear_rejects_small_workspace_and_nulls():
    L = _lib.lib()
    assert L.exl3b_linear(FAKE, 1, 256, FAKE, 128, 4, 2, FAKE, FAKE, FAKE, 128, FAKE, 16, None) == \
        _lib.EXL3B_WORKSPACE
    assert L.exl3b_linear(None, 1, 256, FAKE, 128, 4, 2, FAKE, FAKE, FAKE, 128, FAKE, 1 << 30, None) == \
        _lib.EXL3B_BAD_ARG


def test_dequant_and_had_validate_arguments():
    L = _lib.lib()
    assert L.exl3b_dequant(FAKE, 128, 128, 0, 2, 0, 128, FAKE, 128, None) == _lib.EXL3B_DECLINED
    assert L.exl3b_dequant(FAKE, 128, 128, 4, 2, 8, 128, FAKE, 128, None) == _lib.EXL3B_BAD_ARG
    assert L.exl3b_had128(FAKE, 128, FAKE, 128, 4, 100, None, None, 1.0, None) == _lib.EXL3B_BAD_ARG
    assert L.exl3b_had128(FAKE, 128, FAKE, 128, 0, 128, None, None, 1.0, None) == _lib.EXL3B_OK


def test_missing_library_fails_loudly(monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", "/nonexistent/libexl3b.so")
    with pytest.raises(ImportError, match="no fallback"):
        _lib.lib()
