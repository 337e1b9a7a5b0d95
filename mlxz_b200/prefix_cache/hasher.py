"""Content-addressed prefix hashing at block boundaries (host side).

Same digests as the reference's RollingPrefixHasher
(src/mlxz/prefix_cache/hasher.py:30-53): SHA-256 of each block_size chunk of
the token ids packed as little-endian int32; the last chunk may be partial.
"""
from __future__ import annotations

import hashlib
import struct


class RollingPrefixHasher:
    """Emits one SHA-256 digest per ``block_size`` chunk of a token stream."""

    def __init__(self, block_size: int = 8) -> None:
        if block_size < 1:
            raise ValueError(f"block_size must be >= 1, got {block_size}")
        self._block_size = block_size

    @property
    def block_size(self) -> int:
        return self._block_size

    def hash_chunks(self, tokens: list[int]) -> tuple[bytes, ...]:
        """Digests of tokens[i*bs:(i+1)*bs] for every chunk; () for no tokens."""
        bs = self._block_size
        out = []
        for start in range(0, len(tokens), bs):
            chunk = tokens[start:start + bs]
            out.append(hashlib.sha256(struct.pack(f"<{len(chunk)}i", *chunk)).digest())
        return tuple(out)
