"""Prefix cache over a paged KV store: blocks shared by refcount, not copied.

The reference's PrefixCacheMemory deep-copies every layer's KV at every
chunk-boundary prefix (src/mlxz/prefix_cache/memory.py:19-35, :85-179) and
restores by assigning the copies into the request's cache
(src/mlxz/engine/continuous.py:258-259), which mlx_lm copies again on the
next write.  Here, with every layer's K/V in one PagedKVStore:

  * store:   an entry is the list of the sequence's first ceil(n/bs) blocks;
             the cache takes one BlockManager reference per block it holds
             (shared by all entries that use the block) -- no data moves;
  * lookup:  same longest-prefix / cache-type / LRU policy as the reference;
  * restore: the new sequence's table is the entry's block list with one more
             reference each (zero copy); its first write into a shared block
             goes through BlockManager.copy_on_write + mz_block_copy
             (PagedKVStore.make_writable);
  * budget:  the same byte accounting as the reference (an entry of n tokens
             counts n * bytes_per_token), LRU entries dropped until a new one
             fits;
  * host tier: ``evict_to_host`` moves the least recently used entries' blocks
             that only the cache still holds to pinned host memory
             (PinnedHostTier: pack kernel + side-stream D2H) and frees them on
             the device; ``restore`` of such an entry reloads them first;
  * disk tier: ``spill_to_disk`` / ``load_from_disk`` write an entry to and
             read it from a PrefixCacheDisk in the reference's safetensors
             format (src/mlxz/prefix_cache/disk.py).
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass
from typing import Any

import torch

from ..types import PrefixCacheStats
from .base import CachedPrefix
from .host_tier import PinnedHostTier

_clock = itertools.count(1)
CACHE_TYPE = "PagedKVCache"


@dataclass(frozen=True, slots=True)
class PagedPrefixState:
    """A cached prefix: cache-internal logical block ids and its token count."""

    blocks: tuple[int, ...]
    n_tokens: int


class PagedPrefixCache:
    """Refcounted, zero-copy prefix cache for a PagedKVStore."""

    def __init__(self, store: Any, memory_budget_bytes: int,
                 host_tier: PinnedHostTier | None = None) -> None:
        self.store = store
        self._budget = memory_budget_bytes
        self.host_tier = host_tier
        self._entries: dict[tuple[bytes, ...], CachedPrefix] = {}
        self._used = 0
        self._stats = PrefixCacheStats()
        self._loc: dict[int, tuple[str, int]] = {}   # logical block -> ("dev"|"host", id)
        self._users: dict[int, int] = {}             # logical block -> entries using it
        self._by_dev: dict[int, int] = {}            # device block -> logical block
        self._next_lb = 0
        if hasattr(type(store), "bytes_per_token"):
            self.bytes_per_token = store.bytes_per_token
        else:
            elem = store.pools.element_size()
            self.bytes_per_token = store.n_layers * 2 * store.n_kv_heads * store.head_dim * elem

    # -- logical blocks ------------------------------------------------------

    def _hold(self, dev_block: int) -> int:
        lb = self._by_dev.get(dev_block)
        if lb is None:
            lb = self._next_lb
            self._next_lb += 1
            self._loc[lb] = ("dev", dev_block)
            self._by_dev[dev_block] = lb
            self._users[lb] = 0
            self.store.bm.incref([dev_block])  # the cache's own reference
        self._users[lb] += 1
        return lb

    def _release(self, lb: int) -> None:
        self._users[lb] -= 1
        if self._users[lb] > 0:
            return
        del self._users[lb]
        kind, ident = self._loc.pop(lb)
        if kind == "dev":
            del self._by_dev[ident]
            self.store.bm.free([ident])
        else:
            self.host_tier.release([ident])

    # -- reference API -------------------------------------------------------

    def lookup_sync(self, token_hashes: tuple[bytes, ...], cache_type: str | None = None
                    ) -> tuple[int, PagedPrefixState | None, str | None]:
        for length in range(len(token_hashes), 0, -1):
            entry = self._entries.get(token_hashes[:length])
            if entry is None or (cache_type is not None and entry.cache_type != cache_type):
                continue
            entry.last_access = next(_clock)
            self._stats.hits += 1
            self._stats.hit_bytes += entry.size_bytes
            return entry.n_tokens, entry.kv_states, entry.cache_type
        self._stats.misses += 1
        return 0, None, None

    def store_sync(self, token_hashes: tuple[bytes, ...], seq_id: str,
                   n_tokens: int | None = None, block_size: int = 8) -> None:
        """Cache the first n_tokens of `seq_id` and every chunk-boundary prefix."""
        if token_hashes in self._entries:
            return
        table = self.store.tables[seq_id]
        if n_tokens is None:
            n_tokens = self.store.offsets[seq_id]
        if n_tokens <= 0:
            return
        kv_bs = self.store.block_size
        lengths = list(range(block_size, n_tokens, block_size))
        if not lengths or lengths[-1] != n_tokens:
            lengths.append(n_tokens)
        for plen in reversed(lengths):
            key = token_hashes[: -(-plen // block_size)]
            if not key or key in self._entries:
                continue
            size = plen * self.bytes_per_token
            self._evict_until_room(size)
            if size > self._budget:
                continue
            lbs = tuple(self._hold(table[j]) for j in range(-(-plen // kv_bs)))
            self._entries[key] = CachedPrefix(token_hashes=key,
                                              kv_states=PagedPrefixState(lbs, plen),
                                              n_tokens=plen, size_bytes=size,
                                              cache_type=CACHE_TYPE, last_access=next(_clock))
            self._used += size

    def _drop(self, key: tuple[bytes, ...]) -> None:
        entry = self._entries.pop(key)
        self._used -= entry.size_bytes
        self._stats.evictions += 1
        for lb in entry.kv_states.blocks:
            self._release(lb)

    def _evict_until_room(self, needed: int) -> None:
        while self._used + needed > self._budget and self._entries:
            self._drop(min(self._entries, key=lambda k: self._entries[k].last_access))

    def stats(self) -> PrefixCacheStats:
        s = self._stats
        return PrefixCacheStats(hits=s.hits, misses=s.misses, hit_bytes=s.hit_bytes,
                                evictions=s.evictions, memory_used_bytes=self._used,
                                host_used_bytes=self.host_tier.used_bytes() if self.host_tier else 0,
                                host_evicted_blocks=s.host_evicted_blocks,
                                host_reloaded_blocks=s.host_reloaded_blocks)

    # -- restore / host tier ---------------------------------------------------

    def restore(self, seq_id: str, state: PagedPrefixState) -> list[int]:
        """Install a cached prefix as the block table of a new sequence (zero
        copy: one more reference per block; host-resident blocks are reloaded
        first).  Returns the table."""
        self.reload(state)
        table = [self._loc[lb][1] for lb in state.blocks]
        self.store.bm.incref(table)
        self.store.tables[seq_id] = list(table)
        self.store.offsets[seq_id] = state.n_tokens
        return table

    def reload(self, state: PagedPrefixState) -> int:
        """Bring an entry's host-resident blocks back to the device; returns
        the number reloaded."""
        host_lbs = [lb for lb in state.blocks if self._loc[lb][0] == "host"]
        if not host_lbs:
            return 0
        new = self.store.bm.allocate(len(host_lbs))
        slots = [self._loc[lb][1] for lb in host_lbs]
        self.host_tier.reload(self.store.pool_stacks(), slots, new)
        self.host_tier.release(slots)
        for lb, b in zip(host_lbs, new):
            self._loc[lb] = ("dev", b)
            self._by_dev[b] = lb
        self._stats.host_reloaded_blocks += len(host_lbs)
        return len(host_lbs)

    def evict_to_host(self, max_blocks: int) -> int:
        """Move up to `max_blocks` device blocks that only the cache references
        to the host tier, least recently used entries first; returns the count."""
        if self.host_tier is None:
            raise RuntimeError("no host tier configured")
        chosen: list[int] = []
        seen: set[int] = set()
        bm = self.store.bm
        for key in sorted(self._entries, key=lambda k: self._entries[k].last_access):
            for lb in self._entries[key].kv_states.blocks:
                if len(chosen) >= max_blocks:
                    break
                kind, b = self._loc[lb]
                if kind != "dev" or lb in seen or bm.get_refcount(b) != 1:
                    continue
                seen.add(lb)
                chosen.append(lb)
            if len(chosen) >= max_blocks:
                break
        if not chosen:
            return 0
        dev = [self._loc[lb][1] for lb in chosen]
        slots = self.host_tier.evict(self.store.pool_stacks(), dev)
        for lb, b, s in zip(chosen, dev, slots):
            self._loc[lb] = ("host", s)
            del self._by_dev[b]
        bm.free(dev)
        self._stats.host_evicted_blocks += len(chosen)
        return len(chosen)

    def device_blocks(self) -> list[int]:
        """Device blocks the cache currently holds a reference to."""
        return sorted(self._by_dev)

    def entry_location(self, state: PagedPrefixState) -> list[str]:
        return [self._loc[lb][0] for lb in state.blocks]

    # -- disk tier -------------------------------------------------------------

    def _layer_states(self, blocks: list[int], n_tokens: int) -> list[Any]:
        """Per-layer states [1, H, n, W] of the given device blocks: (K, V) for
        a plain store, ((codes, scales, biases) of K, same of V) for a
        quantised one."""
        stacks = self.store.pool_stacks()
        idx = torch.tensor(blocks, dtype=torch.long, device=stacks[0].device)

        def rows(stack, p):
            t = stack[p].index_select(0, idx)             # [nb, H, bs, W]
            nb, H, bs, W = t.shape
            return t.permute(1, 0, 2, 3).reshape(1, H, nb * bs, W)[:, :, :n_tokens]

        states = []
        for l in range(self.store.n_layers):
            if len(stacks) == 1:
                states.append((rows(stacks[0], 2 * l), rows(stacks[0], 2 * l + 1)))
            else:
                states.append((tuple(rows(s, 2 * l) for s in stacks),
                               tuple(rows(s, 2 * l + 1) for s in stacks)))
        return states

    def spill_to_disk(self, token_hashes: tuple[bytes, ...], disk) -> bool:
        """Write the entry stored under ``token_hashes`` to a PrefixCacheDisk in
        its format (host-resident blocks are reloaded first).  False when there
        is no such entry."""
        entry = self._entries.get(token_hashes)
        if entry is None:
            return False
        state = entry.kv_states
        self.reload(state)
        blocks = [self._loc[lb][1] for lb in state.blocks]
        ctype = "QuantizedKVCache" if len(self.store.pool_stacks()) > 1 else "KVCache"
        disk.store_states(token_hashes, self._layer_states(blocks, state.n_tokens),
                          state.n_tokens, ctype)
        return True

    def load_from_disk(self, token_hashes: tuple[bytes, ...], disk, block_size: int = 8
                       ) -> int:
        """Longest prefix of ``token_hashes`` on disk, written into fresh device
        blocks (raw, no requantisation) and cached as an entry; returns its
        token count (0 on a miss or a format this store does not hold)."""
        quantized = len(self.store.pool_stacks()) > 1
        n, states, _ = disk.lookup_sync(token_hashes,
                                        "QuantizedKVCache" if quantized else "KVCache")
        if not n or states is None or len(states) != self.store.n_layers:
            return 0
        bs = self.store.block_size
        nb = -(-n // bs)
        new = self.store.bm.allocate(nb)
        stacks = self.store.pool_stacks()
        idx = torch.tensor(new, dtype=torch.long, device=stacks[0].device)

        def put(stack, p, t):
            H, W = t.shape[1], t.shape[3]
            buf = torch.zeros((H, nb * bs, W), dtype=stack.dtype, device=stack.device)
            buf[:, :n] = t[0].to(stack.device, stack.dtype)
            stack[p].index_copy_(0, idx, buf.view(H, nb, bs, W).permute(1, 0, 2, 3))

        for l, st in enumerate(states):
            if quantized:
                # a quantised layer reads back as its tensors in name order:
                # K's (codes, scales, biases) then V's
                if len(st) != 2 * len(stacks):
                    self.store.bm.free(new)
                    return 0
                k, v = st[:len(stacks)], st[len(stacks):]
                for s, kt, vt in zip(stacks, k, v):
                    put(s, 2 * l, kt)
                    put(s, 2 * l + 1, vt)
            else:
                put(stacks[0], 2 * l, st[0])
                put(stacks[0], 2 * l + 1, st[1])
        key = token_hashes[: -(-n // block_size)]
        size = n * self.bytes_per_token
        if size > self._budget:
            self.store.bm.free(new)
            return 0
        if key not in self._entries:
            self._evict_until_room(size)
            lbs = tuple(self._hold(b) for b in new)
            self._entries[key] = CachedPrefix(token_hashes=key,
                                              kv_states=PagedPrefixState(lbs, n),
                                              n_tokens=n, size_bytes=size,
                                              cache_type=CACHE_TYPE, last_access=next(_clock))
            self._used += size
        self.store.bm.free(new)  # the entry holds its own reference
        return n
