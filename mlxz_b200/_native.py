"""ctypes binding of libmlxz_b200.so (the C ABI declared in include/mlxz_b200.h).

There is no fallback: if the library cannot be loaded, every call raises
``NativeLibraryError``.  Status codes from the C ABI become Python exceptions
(``ValueError`` for bad arguments, ``NativeError`` otherwise); device error
words become ``DeviceError``.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libmlxz_b200.so"

MZ_OK = 0
MZ_ERR_INVALID_ARG = -1
MZ_ERR_UNSUPPORTED = -2
MZ_ERR_ALIGNMENT = -3
MZ_ERR_CUDA = -4
MZ_ERR_WORKSPACE = -5
MZ_ERR_TOO_LARGE = -6

MZ_DTYPE_F16 = 0
MZ_DTYPE_BF16 = 1
MZ_DTYPE_F32 = 2

MZ_DEVERR_BLOCK_ID = 1
MZ_DEVERR_SLOT = 2
MZ_DEVERR_CONTEXT = 4
MZ_DEVERR_TIMEOUT = 8
MZ_DEVERR_ROWS = 16

_DEVERR_NAMES = {
    MZ_DEVERR_BLOCK_ID: "block id out of range",
    MZ_DEVERR_SLOT: "slot out of range",
    MZ_DEVERR_CONTEXT: "context length out of range",
    MZ_DEVERR_TIMEOUT: "bounded wait timed out",
    MZ_DEVERR_ROWS: "query rows out of range",
}


class NativeLibraryError(RuntimeError):
    """libmlxz_b200.so is missing or cannot be loaded (build it with mlxz_b200.build)."""


class NativeError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, message: str) -> None:
        self.code = code
        super().__init__(f"[{code}] {message}")


class UnsupportedError(NativeError, ValueError):
    """Valid arguments outside what the kernels implement."""


class DeviceError(RuntimeError):
    """A kernel reported an out-of-range access or a timeout in its error word."""

    def __init__(self, bits: int) -> None:
        self.bits = bits
        names = [n for b, n in _DEVERR_NAMES.items() if bits & b]
        super().__init__("device error: " + ", ".join(names or [hex(bits)]))


_i32, _i64, _f32, _vp, _sz = (ctypes.c_int32, ctypes.c_int64, ctypes.c_float,
                              ctypes.c_void_p, ctypes.c_size_t)

MZ_MAX_RANKS = 8
MZ_IPC_HANDLE_BYTES = 64
MZ_LAUNCH_OVERLAP_PREVIOUS = 1
MZ_DECODE_BATCH_INVARIANT = 2
MZ_LAUNCH_WAIT_PREVIOUS = 4


class PeerOutputs(ctypes.Structure):
    """mz_peer_outputs: one rank's output destinations in a head-sharded group."""

    _fields_ = [("n_ranks", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("out", ctypes.c_void_p * MZ_MAX_RANKS),
                ("signal", ctypes.c_void_p * MZ_MAX_RANKS),
                ("arrivals", ctypes.c_void_p), ("epoch", ctypes.c_uint32)]


# name -> argtypes (every function returns int32 status)
_SIGNATURES: dict[str, list] = {
    "mz_abi_version": [],
    "mz_last_error": [ctypes.c_char_p, _sz],
    "mz_kv_append": [_vp, _vp, _vp, _vp, _i64, _i64, _vp, _i64, _i32, _i32, _i32, _i64, _i32,
                     _vp, _vp],
    "mz_kv_append_paged": [_vp, _vp, _vp, _vp, _i64, _i64, _vp, _i32, _vp, _i32, _i32, _i32,
                           _i32, _i64, _i32, _vp, _vp],
    "mz_kv_gather": [_vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _i32, _i64, _i32, _i32, _i32,
                     _i64, _i32, _vp, _vp],
    "mz_paged_decode_workspace_size": [_i32, _i32, _i32, _i32, _i32, _i32,
                                       ctypes.POINTER(_sz)],
    "mz_paged_decode_workspace_size_ex": [_i32, _i32, _i32, _i32, _i32, _i32, _i32,
                                          ctypes.c_uint32, _i32, ctypes.POINTER(_sz)],
    "mz_paged_decode": [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _vp, _vp,
                        _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _i64, _f32, _i32, _i32,
                        _vp, _sz, _vp, _vp],
    "mz_paged_append_decode": [_vp, _i32, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _i64,
                               _i64, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _i64, _f32,
                               _i32, _i32, _vp, _sz, _vp, _vp],
    "mz_paged_append_decode_ex": [_vp, _i32, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _vp,
                                  _i64, _i64, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32,
                                  _i64, _f32, _i32, _i32, ctypes.c_uint32, _vp, _sz, _vp, _vp],
    "mz_paged_append_decode_allgather": [ctypes.POINTER(PeerOutputs), _i32, _i64, _i64, _vp,
                                         _i64, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _i32,
                                         _vp, _i32, _i32, _i32, _i32, _i32, _i64, _f32, _i32,
                                         _i32, ctypes.c_uint32, _vp, _sz, _vp, _vp],
    "mz_peer_wait": [_vp, _i32, _i32, ctypes.c_uint32, ctypes.c_uint64, _vp, _vp],
    "mz_kv_dequant_blocks": [_vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32,
                             _i32, _i32, _i64, _i32, _vp, _vp],
    "mz_paged_prefill": [_vp, _i32, _i64, _i64, _vp, _i64, _i64, _i32, _vp, _vp, _i32, _vp, _vp, _vp,
                         _i32, _vp, _i32, _i32, _i32, _i32, _i32, _i64, _f32, _i32, _vp, _vp],
    "mz_ipc_export": [_vp, _vp, ctypes.POINTER(ctypes.c_uint64)],
    "mz_ipc_open": [_vp, ctypes.c_uint64, ctypes.POINTER(_vp), ctypes.POINTER(_vp)],
    "mz_ipc_close": [_vp],
    "mz_paged_decode_noalloc": [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _vp,
                                _vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _i64, _f32,
                                _i32, _i32, _vp, _vp],
    "mz_block_copy": [_vp, _i64, _i32, _i64, _vp, _vp, _i32, _i64, _vp, _vp],
    "mz_kv_quant_append": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _i64, _i32,
                           _i32, _i32, _i64, _i32, _i32, _i32, _vp, _vp],
    "mz_kv_quant_append_paged": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _i32,
                                 _vp, _i32, _i32, _i32, _i32, _i64, _i32, _i32, _i32, _vp, _vp],
    "mz_paged_decode_q_workspace_size": [_i32, _i32, _i32, _i32, _i32, _i32, _i32,
                                         ctypes.POINTER(_sz)],
    "mz_paged_decode_q": [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _vp, _vp,
                          _vp, _vp, _vp, _vp, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _i64,
                          _i32, _i32, _f32, _i32, _i32, _vp, _sz, _vp, _vp],
    "mz_block_pack": [_vp, _vp, _i64, _i32, _i64, _vp, _i32, _i64, _vp, _vp],
    "mz_block_unpack": [_vp, _i64, _i32, _i64, _vp, _vp, _i32, _i64, _vp, _vp],
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    return Path(os.environ.get("MLXZ_B200_LIB", _LIB_PATH))


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once); raises NativeLibraryError if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not path.exists():
                raise NativeLibraryError(
                    f"{path} not found: build it with `python -m mlxz_b200.build`")
            try:
                handle = ctypes.CDLL(str(path))
            except OSError as e:  # pragma: no cover - depends on the host
                raise NativeLibraryError(f"cannot load {path}: {e}") from e
            for name, argtypes in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = argtypes
                fn.restype = ctypes.c_int32
            _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def last_error() -> tuple[int, str]:
    buf = ctypes.create_string_buffer(512)
    code = lib().mz_last_error(buf, len(buf))
    return code, buf.value.decode(errors="replace")


def check(status: int) -> None:
    """Raise the exception that matches a C-ABI status code."""
    if status == MZ_OK:
        return
    _, msg = last_error()
    if status in (MZ_ERR_INVALID_ARG, MZ_ERR_ALIGNMENT, MZ_ERR_WORKSPACE, MZ_ERR_TOO_LARGE):
        raise ValueError(f"[{status}] {msg}")
    if status == MZ_ERR_UNSUPPORTED:
        raise UnsupportedError(status, msg)
    raise NativeError(status, msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
