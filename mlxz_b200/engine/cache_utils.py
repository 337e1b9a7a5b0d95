"""Cache-construction and cache-list helpers of the KV path.

Mirrors src/mlxz/engine/cache_utils.py:21-51 (quantise threshold, cache type
name) and the ``trim_prompt_cache`` helper the prefix cache calls
(src/mlxz/prefix_cache/memory.py:138-143), for torch-tensor caches.
"""
from __future__ import annotations

from typing import Any

from ..config import KVConfig


class QuantizedKVCache:
    """Marker base class of quantised KV caches: ``cache_type_name`` reports
    any subclass as "QuantizedKVCache" (as the reference does for mlx_lm's)."""


def should_quantize_cache(kv_config: KVConfig, total_requested_tokens: int) -> bool:
    """True when a request of this many tokens should start on quantised KV
    (cache_utils.py:21-26)."""
    return total_requested_tokens >= kv_config.quantized_kv_start


def cache_type_name(cache_layers: list[Any]) -> str:
    """Type name of the first layer ("" for none), with every quantised cache
    reported as "QuantizedKVCache" (cache_utils.py:44-51)."""
    if not cache_layers:
        return ""
    first = cache_layers[0]
    if isinstance(first, QuantizedKVCache):
        return "QuantizedKVCache"
    return type(first).__name__


def trim_prompt_cache(cache_layers: list[Any], num_tokens: int) -> int:
    """Drop the last ``num_tokens`` tokens of every layer when all layers are
    trimmable; returns the number trimmed (0 when nothing was done)."""
    if num_tokens == 0 or not all(c.is_trimmable() for c in cache_layers):
        return 0
    trimmed = [c.trim(num_tokens) for c in cache_layers]
    return trimmed[0] if trimmed else 0
