"""The C-ABI library loads and exports every entry point ``include/*.h`` declares.

CPU-only: loads ``libmak_kvcache.so`` with ctypes and inspects symbols; no
kernel is launched.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> list[str]:
    names: list[str] = []
    for header in sorted((ROOT / "include").glob("*.h")):
        text = header.read_text()
        names += re.findall(r"^MAK_API\s+[\w\s\*]+?\b(mak_\w+)\s*\(", text, flags=re.M)
    return names


@pytest.fixture(scope="module")
def lib():
    from musa_aiter import _build

    result = _build.build()
    assert result.ok, result.message
    return ctypes.CDLL(str(_build.LIB_PATH))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert len(names) >= 12
    assert len(set(names)) == len(names)


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    from musa_aiter import _native

    assert set(declared_symbols()) == set(_native.exported_symbols())


def test_abi_version_and_host_only_queries(lib):
    lib.mak_abi_version.restype = ctypes.c_int
    assert lib.mak_abi_version() == 1
    lib.mak_scatter_workspace_bytes.restype = ctypes.c_size_t
    lib.mak_scatter_workspace_bytes.argtypes = [ctypes.c_int64]
    small = lib.mak_scatter_workspace_bytes(10)
    big = lib.mak_scatter_workspace_bytes(1 << 20)
    assert 0 < small < big
    assert big >= (1 << 20) * 8
