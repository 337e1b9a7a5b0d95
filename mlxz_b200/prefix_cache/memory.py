"""In-memory prefix cache with LRU eviction over tensor-state caches.

Same policy as the reference's PrefixCacheMemory
(src/mlxz/prefix_cache/memory.py:38-211):
  * lookup: longest hash-tuple prefix first, optionally filtered by cache
    type; a hit refreshes the entry's LRU position (:56-83);
  * store: deep-copies the caches, then walks the chunk-boundary prefix
    lengths range(bs, n, bs) + [n] from the longest down, trimming the copy
    and snapshotting each length not cached yet (:85-179);
  * eviction: least recently used entries go until the new one fits; an entry
    larger than the whole budget is skipped (:155-162, :181-192).
LRU order uses a monotonically increasing access counter.  The golden traces
in tests/golden pin this policy against the reference's own code.

This class serves contiguous tensor caches (any device).  The paged KV store
uses PagedPrefixCache instead, which shares pool blocks by refcount rather
than copying them.
"""
from __future__ import annotations

import copy
import itertools
from typing import Any

import torch

from ..engine.cache_utils import cache_type_name, trim_prompt_cache
from ..types import PrefixCacheStats
from .base import CachedPrefix, compute_size_bytes

_clock = itertools.count(1)


def _copy_states(kv_states: list[Any]) -> list[Any]:
    """Independent copies of per-layer states (tensors cloned, tuples kept)."""
    def cp(x: Any) -> Any:
        if isinstance(x, torch.Tensor):
            return x.clone()
        if isinstance(x, tuple):
            return tuple(cp(y) for y in x)
        return x

    return [cp(s) if isinstance(s, tuple) else s for s in kv_states]


def _state_len(state: Any) -> int:
    keys = state[0] if isinstance(state, tuple) and state else None
    if isinstance(keys, tuple):
        keys = keys[0]
    if isinstance(keys, torch.Tensor):
        return int(keys.shape[2]) if keys.dim() >= 3 else int(keys.shape[0])
    return 0


class PrefixCacheMemory:
    """Prefix cache with LRU eviction and greedy longest-prefix matching.

    Not thread-safe: one engine thread owns it (as in the reference).
    """

    def __init__(self, memory_budget_bytes: int) -> None:
        self._budget = memory_budget_bytes
        self._entries: dict[tuple[bytes, ...], CachedPrefix] = {}
        self._used_bytes = 0
        self._stats = PrefixCacheStats()

    def lookup_sync(self, token_hashes: tuple[bytes, ...], cache_type: str | None = None
                    ) -> tuple[int, list[Any] | None, str | None]:
        """(n_tokens, kv_states, cache_type) of the longest cached prefix, or
        (0, None, None).  The states are references, not copies."""
        for length in range(len(token_hashes), 0, -1):
            entry = self._entries.get(token_hashes[:length])
            if entry is None:
                continue
            if cache_type is not None and entry.cache_type != cache_type:
                continue
            entry.last_access = next(_clock)
            self._stats.hits += 1
            self._stats.hit_bytes += entry.size_bytes
            return entry.n_tokens, entry.kv_states, entry.cache_type
        self._stats.misses += 1
        return 0, None, None

    def store_sync(self, token_hashes: tuple[bytes, ...], kv_cache_layers: list[Any],
                   n_tokens: int | None = None, block_size: int = 8) -> None:
        """Cache the full prompt state and every chunk-boundary prefix of it."""
        if token_hashes in self._entries:
            return
        ctype = cache_type_name(kv_cache_layers)
        work = copy.deepcopy(kv_cache_layers)
        if n_tokens is None:
            n_tokens = _state_len(work[0].state) if work else 0
        if n_tokens <= 0:
            return
        lengths = list(range(block_size, n_tokens, block_size))
        if not lengths or lengths[-1] != n_tokens:
            lengths.append(n_tokens)
        current = n_tokens
        for plen in reversed(lengths):
            if current > plen:
                trim_prompt_cache(work, current - plen)
                current = plen
            key = token_hashes[: -(-plen // block_size)]
            if not key or key in self._entries:
                continue
            states = _copy_states([layer.state for layer in work])
            size = compute_size_bytes(states)
            self._evict_until_room(size)
            if size > self._budget:
                continue  # larger than the whole budget: not cached
            stamp = next(_clock)
            self._entries[key] = CachedPrefix(token_hashes=key, kv_states=states, n_tokens=plen,
                                              size_bytes=size, cache_type=ctype,
                                              last_access=stamp)
            self._used_bytes += size
            self._stats.memory_used_bytes = self._used_bytes

    def _evict_until_room(self, needed_bytes: int) -> None:
        while self._used_bytes + needed_bytes > self._budget and self._entries:
            oldest = min(self._entries, key=lambda k: self._entries[k].last_access)
            evicted = self._entries.pop(oldest)
            self._used_bytes -= evicted.size_bytes
            self._stats.evictions += 1

    async def lookup(self, token_hashes: list[bytes]) -> tuple[int, Any | None, str | None]:
        return self.lookup_sync(tuple(token_hashes))

    async def store(self, token_hashes: list[bytes], kv: Any) -> None:
        self.store_sync(tuple(token_hashes), kv)

    def stats(self) -> PrefixCacheStats:
        return PrefixCacheStats(hits=self._stats.hits, misses=self._stats.misses,
                                hit_bytes=self._stats.hit_bytes, evictions=self._stats.evictions,
                                memory_used_bytes=self._used_bytes, disk_used_bytes=0)
