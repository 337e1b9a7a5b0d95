"""Prefix cache: content-hashed KV reuse for repeated prompts.

``PrefixCacheMemory`` keeps the reference's policy over tensor-state caches;
``PagedPrefixCache`` is the paged form (refcounted block sharing,
copy-on-write, eviction to a pinned host tier).
"""
from .base import CachedPrefix, PrefixMatch, compute_size_bytes
from .disk import PrefixCacheCorruption, PrefixCacheDisk
from .hasher import RollingPrefixHasher
from .host_tier import PinnedHostTier
from .memory import PrefixCacheMemory
from .paged import PagedPrefixCache, PagedPrefixState

__all__ = [
    "CachedPrefix",
    "PagedPrefixCache",
    "PagedPrefixState",
    "PrefixCacheCorruption",
    "PrefixCacheDisk",
    "PinnedHostTier",
    "PrefixCacheMemory",
    "PrefixMatch",
    "RollingPrefixHasher",
    "compute_size_bytes",
]
