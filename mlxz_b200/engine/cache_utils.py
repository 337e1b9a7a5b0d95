"""Cache-construction and cache-list helpers of the KV path.

Mirrors src/mlxz/engine/cache_utils.py:1-115 (quantise threshold, prompt-cache
construction with optional quantisation, the restoring quantised cache, cache
type name, token count of a state) and the ``trim_prompt_cache`` helper the
prefix cache calls (src/mlxz/prefix_cache/memory.py:138-143), over the CUDA
caches of ``kv_cache``.
"""
from __future__ import annotations

from typing import Any

from ..config import KVConfig
from .kv_cache import KVCache, QuantizedKVCache, make_prompt_cache

__all__ = ["KVCache", "QuantizedKVCache", "RestoringQuantizedKVCache", "build_prompt_cache",
           "cache_type_name", "make_prompt_cache", "should_quantize_cache", "trim_prompt_cache"]


class RestoringQuantizedKVCache(QuantizedKVCache):
    """Quantised cache whose ``state`` setter also sets ``offset`` from the
    restored state (cache_utils.py:12-19), so a restored prefix is appended to
    at the right position."""

    @property
    def state(self) -> tuple[Any, Any]:
        return QuantizedKVCache.state.fget(self)

    @state.setter
    def state(self, v: tuple[Any, Any]) -> None:
        self.keys, self.values = v
        self.offset = _state_token_count(v)


def should_quantize_cache(kv_config: KVConfig, total_requested_tokens: int) -> bool:
    """True when a request of this many tokens should start on quantised KV
    (cache_utils.py:21-26)."""
    return total_requested_tokens >= kv_config.quantized_kv_start


def build_prompt_cache(model: Any, *, quantized: bool = False, group_size: int = 64,
                       bits: int = 8, max_kv_size: int | None = None) -> list[Any]:
    """One cache per layer of ``model``; quantised (RestoringQuantizedKVCache)
    when ``quantized`` (cache_utils.py:29-41)."""
    cache = make_prompt_cache(model, max_kv_size=max_kv_size)
    if not quantized:
        return cache
    return [_quantize_layer(layer, group_size=group_size, bits=bits) for layer in cache]


def cache_type_name(cache_layers: list[Any]) -> str:
    """Type name of the first layer ("" for none), with every quantised cache
    reported as "QuantizedKVCache" (cache_utils.py:44-51)."""
    if not cache_layers:
        return ""
    first = cache_layers[0]
    if isinstance(first, QuantizedKVCache):
        return "QuantizedKVCache"
    return type(first).__name__


def _quantize_layer(layer_cache: Any, *, group_size: int, bits: int) -> Any:
    """A layer's cache as a RestoringQuantizedKVCache with its state kept
    (cache_utils.py:54-90): restoring caches are returned as they are, other
    quantised caches are re-wrapped, standard caches are quantised."""
    if isinstance(layer_cache, RestoringQuantizedKVCache):
        return layer_cache
    if isinstance(layer_cache, QuantizedKVCache):
        q = RestoringQuantizedKVCache(group_size=group_size, bits=bits)
        q.keys, q.values = layer_cache.keys, layer_cache.values
        q.offset = getattr(layer_cache, "offset", 0)
        return q
    if isinstance(layer_cache, KVCache):
        quantized = layer_cache.to_quantized(group_size=group_size, bits=bits)
        wrapped = RestoringQuantizedKVCache(group_size=quantized.group_size, bits=quantized.bits)
        wrapped.keys, wrapped.values = quantized.keys, quantized.values
        wrapped.offset = quantized.offset
        return wrapped
    return layer_cache


def _state_token_count(state: tuple[Any, Any]) -> int:
    """Tokens in a cache state: axis 2 of the first array, or of the first
    array of the first tuple for a quantised state (cache_utils.py:93-115)."""
    if not state:
        return 0
    first = state[0]
    if isinstance(first, tuple):
        if not first:
            return 0
        first = first[0]
    shape = getattr(first, "shape", None)
    if shape is None:
        return 0
    if len(shape) >= 3:
        return int(shape[2])
    if len(shape) >= 1:
        return int(shape[0])
    return 0


def trim_prompt_cache(cache_layers: list[Any], num_tokens: int) -> int:
    """Drop the last ``num_tokens`` tokens of every layer when all layers are
    trimmable; returns the number trimmed (0 when nothing was done)."""
    if num_tokens == 0 or not all(c.is_trimmable() for c in cache_layers):
        return 0
    trimmed = [c.trim(num_tokens) for c in cache_layers]
    return trimmed[0] if trimmed else 0
