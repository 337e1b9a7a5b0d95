"""Prefix-cache entry types and size accounting (the reference's
src/mlxz/prefix_cache/base.py:10-57, over torch tensors)."""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any

import torch


@dataclass(slots=True)
class CachedPrefix:
    """One cached prefix.  ``kv_states`` holds per-layer states: ``(keys,
    values)`` tensors, ``((k_data, k_scales, k_biases), (v_data, ...))`` for a
    quantised cache, or a PagedPrefixState for the paged prefix cache."""

    token_hashes: tuple[bytes, ...]
    kv_states: list[Any]
    n_tokens: int
    size_bytes: int
    created_at: float = field(default_factory=time.monotonic)
    last_access: float = field(default_factory=time.monotonic)
    cache_type: str = "KVCache"


@dataclass(frozen=True, slots=True)
class PrefixMatch:
    """Result of a successful lookup (kv_states is a reference, not a copy)."""

    n_matched_tokens: int
    kv_states: list[Any]
    cache_tier: str  # "memory" or "host"


def compute_size_bytes(kv_states: Any) -> int:
    """Sum of the byte sizes of every tensor in a nested list/tuple structure."""
    total = 0

    def walk(obj: Any) -> None:
        nonlocal total
        if isinstance(obj, torch.Tensor):
            total += obj.numel() * obj.element_size()
        elif isinstance(obj, (list, tuple)):
            for item in obj:
                walk(item)

    walk(kv_states)
    return total
