"""Disk tier of the prefix cache: safetensors entries with SHA-256 integrity.

Same behaviour and file format as PrefixCacheDisk
(src/mlxz/prefix_cache/disk.py:21-219), over torch tensors:

* one entry per prefix key: ``<root>/<model_hash>/<sha256(b"".join(hashes))[:32]>
  .safetensors`` holding tensor ``l{layer}_t{i}`` for element i of a layer's
  cache state (K, V) and ``l{layer}_t{i}_q{j}`` for element j of a quantised
  state's tuple (codes, scales, biases);
* a ``.meta.json`` sidecar: ``n_tokens``, ``n_layers``, ``cache_type``,
  ``checksum`` (SHA-256 over the raw bytes of every tensor, in sorted name
  order), ``format_version`` "1", ``tensor_keys``;
* longest-prefix lookup filtered by cache type; a hit touches both files
  (mtime is the LRU clock); a checksum mismatch or unreadable entry is removed
  and reported as a miss;
* eviction of the oldest entries (by mtime) until a new one fits the budget;
* I/O errors degrade to misses / skipped stores, never raise.

``PagedPrefixCache.spill_to_disk`` / ``load_from_disk`` move a paged entry to
and from this format (the KV of its blocks gathered per layer).
"""
from __future__ import annotations

import hashlib
import json
import logging
from pathlib import Path
from typing import Any

import torch

from ..engine.cache_utils import cache_type_name
from ..types import PrefixCacheStats

logger = logging.getLogger(__name__)


class PrefixCacheCorruption(Exception):
    """On-disk prefix cache data failed its checksum (mlxz.exceptions)."""


def _tensor_bytes(t: torch.Tensor) -> bytes:
    """Raw little-endian bytes of a tensor (any dtype, bf16 included)."""
    t = t.detach().contiguous().cpu()
    return t.view(torch.uint8).numpy().tobytes() if t.numel() else b""


def state_checksum(tensors: dict[str, torch.Tensor]) -> str:
    """SHA-256 over every tensor's bytes in sorted name order (disk.py:147-150)."""
    h = hashlib.sha256()
    for name in sorted(tensors):
        h.update(_tensor_bytes(tensors[name]))
    return h.hexdigest()


def flatten_states(kv_states: list[Any]) -> dict[str, torch.Tensor]:
    """Per-layer cache states -> the entry's named tensors (disk.py:129-140)."""
    tensors: dict[str, torch.Tensor] = {}
    for li, state in enumerate(kv_states):
        if not isinstance(state, tuple):
            continue
        for ti, arr in enumerate(state):
            if isinstance(arr, torch.Tensor):
                tensors[f"l{li}_t{ti}"] = arr
            elif isinstance(arr, tuple):
                for qi, qarr in enumerate(arr):
                    if isinstance(qarr, torch.Tensor):
                        tensors[f"l{li}_t{ti}_q{qi}"] = qarr
    return tensors


def unflatten_states(tensors: dict[str, torch.Tensor], n_layers: int) -> list[Any]:
    """Named tensors -> per-layer states: (K, V) for a plain cache, else the
    layer's tensors in name order (disk.py:175-186)."""
    states: list[Any] = []
    for li in range(n_layers):
        k, v = f"l{li}_t0", f"l{li}_t1"
        if k in tensors and v in tensors:
            states.append((tensors[k], tensors[v]))
        else:
            prefix = f"l{li}_"
            states.append(tuple(tensors[n] for n in sorted(tensors) if n.startswith(prefix)))
    return states


class PrefixCacheDisk:
    """Disk-backed prefix cache with integrity validation and model isolation."""

    def __init__(self, disk_path: Path, disk_budget_bytes: int, model_hash: str) -> None:
        self._root = Path(disk_path) / model_hash
        self._budget = disk_budget_bytes
        self._stats = PrefixCacheStats()
        try:
            self._root.mkdir(parents=True, exist_ok=True)
        except OSError as e:
            logger.warning("prefix cache disk init failed: %s", e)

    def _entry_path(self, token_hashes: tuple[bytes, ...]) -> Path:
        key_hash = hashlib.sha256(b"".join(token_hashes)).hexdigest()[:32]
        return self._root / f"{key_hash}.safetensors"

    def _meta_path(self, entry_path: Path) -> Path:
        return entry_path.with_suffix(".meta.json")

    # -- sync interface -------------------------------------------------------

    def lookup_sync(self, token_hashes: tuple[bytes, ...], cache_type: str | None = None
                    ) -> tuple[int, list[Any] | None, str | None]:
        """Longest stored prefix of ``token_hashes``: (n_tokens, per-layer
        states on the CPU, cache type), or (0, None, None)."""
        for length in range(len(token_hashes), 0, -1):
            entry = self._entry_path(token_hashes[:length])
            meta_path = self._meta_path(entry)
            if not (entry.exists() and meta_path.exists()):
                continue
            try:
                meta = json.loads(meta_path.read_text())
                ctype = str(meta.get("cache_type", "KVCache"))
                if cache_type is not None and ctype != cache_type:
                    continue
                states, n_tokens = self._load_entry(entry, meta_path)
                entry.touch()
                meta_path.touch()
                self._stats.hits += 1
                self._stats.hit_bytes += entry.stat().st_size
                return n_tokens, states, ctype
            except Exception as e:  # corrupt or unreadable: drop it, report a miss
                logger.warning("prefix cache disk load failed for %s: %s", entry, e)
                for f in (entry, meta_path):
                    try:
                        f.unlink(missing_ok=True)
                    except OSError:
                        pass
        self._stats.misses += 1
        return 0, None, None

    def store_sync(self, token_hashes: tuple[bytes, ...], kv_cache_layers: list[Any],
                   n_tokens: int | None = None) -> None:
        """Write the layers' states (``.state`` of each cache layer) as one entry."""
        entry = self._entry_path(token_hashes)
        if entry.exists():
            return
        try:
            kv_states = [layer.state for layer in kv_cache_layers]
            ctype = cache_type_name(kv_cache_layers)
            if n_tokens is None:
                first = kv_states[0] if kv_states else None
                n_tokens = 0
                if isinstance(first, tuple) and isinstance(first[0], torch.Tensor) \
                        and first[0].dim() >= 3:
                    n_tokens = int(first[0].shape[2])
            self.store_states(token_hashes, kv_states, n_tokens, ctype)
        except Exception as e:
            logger.warning("prefix cache disk store failed: %s", e)

    def store_states(self, token_hashes: tuple[bytes, ...], kv_states: list[Any], n_tokens: int,
                     cache_type: str) -> None:
        """Write per-layer states (tuples of tensors) as one entry."""
        from safetensors.torch import save_file

        entry = self._entry_path(token_hashes)
        if entry.exists():
            return
        try:
            # own copies: safetensors refuses tensors that share storage
            tensors = {k: v.detach().to("cpu", copy=True).contiguous()
                       for k, v in flatten_states(kv_states).items()}
            checksum = state_checksum(tensors)
            needed = sum(t.numel() * t.element_size() for t in tensors.values())
            self._evict_until_room(needed)
            save_file(tensors, str(entry))
            meta = {"n_tokens": int(n_tokens), "n_layers": len(kv_states),
                    "cache_type": cache_type, "checksum": checksum, "format_version": "1",
                    "tensor_keys": sorted(tensors)}
            self._meta_path(entry).write_text(json.dumps(meta))
            self._stats.disk_used_bytes += needed
        except Exception as e:  # I/O errors of any layer (safetensors has its own type)
            logger.warning("prefix cache disk store failed: %s", e)
            try:
                entry.unlink(missing_ok=True)
            except OSError:
                pass

    def _load_entry(self, entry: Path, meta_path: Path) -> tuple[list[Any], int]:
        from safetensors.torch import load_file

        meta = json.loads(meta_path.read_text())
        tensors = load_file(str(entry))
        if state_checksum(tensors) != meta.get("checksum", ""):
            raise PrefixCacheCorruption(f"checksum mismatch for {entry}")
        return unflatten_states(tensors, int(meta["n_layers"])), int(meta["n_tokens"])

    def _evict_until_room(self, needed: int) -> None:
        try:
            entries = sorted(self._root.glob("*.safetensors"), key=lambda p: p.stat().st_mtime)
            usage = sum(p.stat().st_size for p in entries)
            for e in entries:
                if usage + needed <= self._budget:
                    break
                size = e.stat().st_size
                e.unlink(missing_ok=True)
                self._meta_path(e).unlink(missing_ok=True)
                usage -= size
                self._stats.evictions += 1
        except OSError:
            pass

    # -- async interface ------------------------------------------------------

    async def lookup(self, token_hashes: list[bytes]) -> tuple[int, Any | None, str | None]:
        return self.lookup_sync(tuple(token_hashes))

    async def store(self, token_hashes: list[bytes], kv: Any) -> None:
        self.store_sync(tuple(token_hashes), kv)

    def stats(self) -> PrefixCacheStats:
        return PrefixCacheStats(hits=self._stats.hits, misses=self._stats.misses,
                                hit_bytes=self._stats.hit_bytes,
                                evictions=self._stats.evictions, memory_used_bytes=0,
                                disk_used_bytes=self._stats.disk_used_bytes)
