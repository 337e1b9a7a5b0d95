"""Shared data types of the KV-cache path (the subset the reference's prefix
cache uses, src/mlxz/types.py:104-113)."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(slots=True)
class PrefixCacheStats:
    """Point-in-time prefix cache counters."""

    hits: int = 0
    misses: int = 0
    hit_bytes: int = 0
    evictions: int = 0
    memory_used_bytes: int = 0
    disk_used_bytes: int = 0
    host_used_bytes: int = 0
    host_evicted_blocks: int = 0
    host_reloaded_blocks: int = 0
