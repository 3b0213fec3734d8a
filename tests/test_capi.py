"""The C-ABI library builds, loads and exports every symbol include/fused_muon.h
declares; argument validation that happens before any device work."""

import os
import re

import pytest

from muon_fused import _lib
from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "fused_muon.h")


def declared_symbols():
    """Entry points of the shipped library: declarations outside the
    development-only `#ifdef FM_TRACE` block."""
    text = re.sub(r"#ifdef FM_TRACE.*?#endif", "", open(HEADER).read(), flags=re.S)
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(fm_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "fm_fused_newton_schulz" in syms and "fm_newton_schulz_step" in syms
    assert "fm_workspace_size" in syms


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for s in declared_symbols():
        assert hasattr(lib, s), s
    # and the ctypes table covers the header exactly
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_version_and_no_error():
    lib = _lib.load()
    assert lib.fm_version() == 100


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (896, 1152), (1152, 896), (40, 72), (1, 1)])
def test_workspace_size(rows, cols):
    b = _lib.workspace_bytes(rows, cols)
    assert b == _lib.workspace_bytes(cols, rows)
    m, n = min(rows, cols), max(rows, cols)
    r8 = lambda x: (x + 7) // 8 * 8
    # two X buffers, A and B (bf16) + fp32 diagonal
    assert b >= 2 * m * r8(n) * 2 + 2 * m * r8(m) * 2 + 4 * m
    assert b % 256 == 0


def test_workspace_size_rejects_bad_shapes():
    with pytest.raises(_lib.FusedMuonError, match="non-empty"):
        _lib.workspace_bytes(0, 10)


def test_entry_points_validate_before_device_work():
    lib = _lib.load()
    rc = lib.fm_fused_newton_schulz(None, 0, 4, 4, 4, None, 5, None, 0, None)
    assert rc == _lib.FM_E_INVALID
    assert b"null" in lib.fm_last_error()
    rc = lib.fm_fused_newton_schulz(1, 9, 4, 4, 4, 1, 5, 256, 1 << 20, None)
    assert rc == _lib.FM_E_INVALID and b"dtype" in lib.fm_last_error()
    rc = lib.fm_fused_newton_schulz(1, 0, 4, 4, 4, 1, -1, 256, 1 << 20, None)
    assert rc == _lib.FM_E_INVALID and b"steps" in lib.fm_last_error()
    rc = lib.fm_newton_schulz_step(1, 4, 8, 4, 1, 256, 1 << 20, None)
    assert rc == _lib.FM_E_INVALID and b"ldx" in lib.fm_last_error()
