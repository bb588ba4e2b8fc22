"""The C ABI library loads on a machine without a GPU and exports every entry
point ``include/*.h`` declares, with the signatures the ctypes layer binds."""

from __future__ import annotations

import re
from pathlib import Path

import pytest

from conftest import ROOT

HEADER_DECL = re.compile(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b(mgs_\w+)\s*\(", re.M)


def declared_symbols() -> set[str]:
    names: set[str] = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(HEADER_DECL.findall(text))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "mgs_linear_scan_fwd" in names and "mgs_version" in names


def test_library_exports_every_declared_symbol():
    from mingru_b200 import _lib

    lib = _lib.load()
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, f"declared in include/*.h but not exported: {missing}"


def test_ctypes_bindings_cover_the_header():
    from mingru_b200 import _lib

    assert declared_symbols() == set(_lib.SIGNATURES), (
        declared_symbols() ^ set(_lib.SIGNATURES)
    )


def test_size_queries_without_gpu():
    from mingru_b200 import _lib

    lib = _lib.load()
    assert lib.mgs_version() >= 100
    ws = lib.mgs_linear_scan_workspace_size(16, 4096, 1024, 0)
    cs = lib.mgs_linear_scan_carry_size(16, 4096, 1024, 0)
    assert ws > 0 and 0 < cs < 16 * 4096 * 1024 * 4 // 8
    assert lib.mgs_linear_scan_workspace_size(2, 5, 3, 99) == 0  # bad dtype
    assert lib.mgs_status_string(6) == b"look-back wait exceeded its bound"


def test_status_mapping():
    from mingru_b200 import _lib

    _lib.check(0, "op")
    with pytest.raises(ValueError, match="MGS_BAD_SHAPE"):
        _lib.check(1, "op")
    with pytest.raises(RuntimeError, match="MGS_LOOKBACK_TIMEOUT"):
        _lib.check(6, "op")


def test_cpu_tensors_raise_no_fallback():
    import torch

    import mingru_b200 as mb

    a = torch.rand(2, 5, 3)
    with pytest.raises(ValueError, match="CUDA"):
        mb.linear_scan(a, a)
    with pytest.raises(ValueError, match="matching"):
        mb.linear_scan(a, a[:, :4])
