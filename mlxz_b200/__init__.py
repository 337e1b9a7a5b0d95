"""mlxz_b200 -- B200-native (sm_100a) implementation of mlxz's KV-cache hot path.

Host policy (block allocation, prefix hashing and lookup) is Python, mirroring
the reference's API; every byte of KV data moves through the hand-written
CUDA kernels of libmlxz_b200.so (C ABI in include/mlxz_b200.h).  There is no
CPU fallback: without the library, kernel calls raise NativeLibraryError.
"""
from ._native import DeviceError, NativeError, NativeLibraryError, UnsupportedError

__version__ = "0.1.0"

__all__ = ["DeviceError", "NativeError", "NativeLibraryError", "UnsupportedError", "__version__"]
