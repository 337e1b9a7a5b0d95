"""The C-ABI library loads and exports every entry point include/*.h declares
(no kernel launches: these run without a GPU)."""
import ctypes
import re
from pathlib import Path

import pytest

from mlxz_b200 import _native

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"^MZ_API\s+int\s+(mz_\w+)\s*\(", h.read_text(), re.M))
    return names


@pytest.fixture(scope="module")
def lib():
    if not _native.library_path().exists():
        from mlxz_b200 import build

        build.build()
    return _native.lib()


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"mz_kv_append", "mz_kv_gather", "mz_paged_decode", "mz_block_copy"} <= names


def test_every_declared_symbol_is_exported_and_bound(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _native.exported_symbols(), f"{name} has no ctypes signature"


def test_abi_version(lib):
    assert lib.mz_abi_version() == 6


def test_argument_errors_do_not_launch(lib):
    # Bad dtype / sizes are rejected on the host before any CUDA call.
    rc = lib.mz_kv_append(None, None, None, None, 0, 0, None, 1, 8, 64, 16, 4, 99, None, None)
    assert rc == _native.MZ_ERR_INVALID_ARG
    code, msg = _native.last_error()
    assert code == rc and "dtype" in msg
    rc = lib.mz_paged_decode(None, 1, 0, 0, 0, None, 0, 0, 0, 1, None, None, None, 1, None, 1,
                             32, 8, 96, 16, 4, 1.0, 1, 0, None, 0, None, None)
    assert rc == _native.MZ_ERR_UNSUPPORTED
    rc = lib.mz_block_copy(None, 0, 1, 100, None, None, 1, 4, None, None)
    assert rc in (_native.MZ_ERR_INVALID_ARG, _native.MZ_ERR_ALIGNMENT)
    with pytest.raises(ValueError):
        _native.check(rc)


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setenv("MLXZ_B200_LIB", str(tmp_path / "absent.so"))
    monkeypatch.setattr(_native, "_lib", None)
    with pytest.raises(_native.NativeLibraryError):
        _native.lib()
