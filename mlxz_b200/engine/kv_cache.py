"""Per-request contiguous KV caches with the cache protocol the engines use.

The reference's engines drive per-layer caches from mlx_lm (0.22.1):
``KVCache`` and ``QuantizedKVCache``, built by ``make_prompt_cache`` and
``build_prompt_cache`` (src/mlxz/engine/cache_utils.py:7, :29-41) and used
through ``update_and_fetch``, ``state`` (get/set), ``offset``, ``trim`` and
``to_quantized`` (src/mlxz/engine/cache_utils.py:61-90,
src/mlxz/prefix_cache/memory.py:109-143).  These classes give that protocol
over CUDA tensors, with the writes done by this package's kernels:

* ``KVCache``: keys/values ``[B, H, capacity, D]``, grown in steps of 256
  tokens; new rows are written with mz_kv_append (bit-exact), the cache seen as
  a pool of B blocks of ``capacity`` tokens.
* ``QuantizedKVCache``: keys/values are (codes int32 ``[B, H, cap, D*bits/32]``,
  scales fp16 ``[B, H, cap, D/64]``, biases fp16 ``[B, H, cap, D/64]``); new
  rows are quantised on append with mz_kv_quant_append (affine groups of 64,
  4 or 8 bits, LSB-first packing).  The state tuples have the same meaning as
  mlx_lm's (MLX uses uint32 words; torch holds the same bits as int32).
"""
from __future__ import annotations

from typing import Any

import torch

from .. import ops

_STEP = 256


def _grow(t: torch.Tensor | None, batch_head: tuple[int, int], cap: int, last: int,
          dtype: torch.dtype, device, keep: int) -> torch.Tensor:
    """A ``[B, H, cap, last]`` tensor holding the first ``keep`` rows of ``t``."""
    out = torch.zeros((*batch_head, cap, last), dtype=dtype, device=device)
    if t is not None and keep > 0:
        out[:, :, :keep].copy_(t[:, :, :keep])
    return out


def _slots(b: int, cap: int, start: int, n: int, device) -> torch.Tensor:
    base = b * cap + start
    return torch.arange(base, base + n, dtype=torch.int64, device=device)


class KVCache:
    """Growing contiguous K/V cache of one layer (mlx_lm's KVCache protocol)."""

    step = _STEP

    def __init__(self) -> None:
        self.keys: torch.Tensor | None = None
        self.values: torch.Tensor | None = None
        self.offset = 0

    def _reserve(self, keys: torch.Tensor, n: int) -> None:
        B, H, _, D = keys.shape
        need = self.offset + n
        if self.keys is not None and self.keys.shape[2] >= need and \
                self.keys.shape[:2] == (B, H) and self.keys.dtype == keys.dtype:
            return
        cap = -(-need // self.step) * self.step
        self.keys = _grow(self.keys, (B, H), cap, D, keys.dtype, keys.device, self.offset)
        self.values = _grow(self.values, (B, H), cap, D, keys.dtype, keys.device, self.offset)

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor
                         ) -> tuple[torch.Tensor, torch.Tensor]:
        """Append ``keys/values [B, H, n, D]``; return the first ``offset`` tokens."""
        if keys.dim() != 4 or keys.shape != values.shape:
            raise ValueError("keys/values must be [B, H, n, D] of the same shape")
        B, _, n, _ = keys.shape
        self._reserve(keys, n)
        cap = self.keys.shape[2]
        for b in range(B):
            ops.kv_append(self.keys, self.values, keys[b], values[b],
                          _slots(b, cap, self.offset, n, keys.device))
        self.offset += n
        return self.keys[:, :, :self.offset], self.values[:, :, :self.offset]

    @property
    def state(self) -> tuple[Any, Any]:
        if self.keys is None:
            return (None, None)
        if self.offset == self.keys.shape[2]:
            return self.keys, self.values
        return self.keys[:, :, :self.offset], self.values[:, :, :self.offset]

    @state.setter
    def state(self, v: tuple[Any, Any]) -> None:
        self.keys, self.values = v
        self.offset = self.keys.shape[2] if self.keys is not None else 0

    def is_trimmable(self) -> bool:
        return True

    def trim(self, n: int) -> int:
        n = min(self.offset, n)
        self.offset -= n
        return n

    def to_quantized(self, group_size: int = 64, bits: int = 8) -> "QuantizedKVCache":
        """This cache's tokens quantised into a new QuantizedKVCache."""
        q = QuantizedKVCache(group_size=group_size, bits=bits)
        if self.keys is not None and self.offset > 0:
            q.update_and_fetch(self.keys[:, :, :self.offset], self.values[:, :, :self.offset])
        return q


class QuantizedKVCache:
    """Growing contiguous 4/8-bit group-64 quantised K/V cache of one layer
    (mlx_lm's QuantizedKVCache protocol)."""

    step = _STEP

    def __init__(self, group_size: int = 64, bits: int = 8) -> None:
        if group_size != 64:
            raise ValueError(f"group_size {group_size}: the kernels implement groups of 64")
        if bits not in (4, 8):
            raise ValueError(f"bits {bits}: the kernels implement 4 and 8")
        self.group_size = group_size
        self.bits = bits
        self.keys: tuple | None = None
        self.values: tuple | None = None
        self.offset = 0

    def _reserve(self, keys: torch.Tensor, n: int) -> None:
        B, H, _, D = keys.shape
        need = self.offset + n
        if self.keys is not None and self.keys[0].shape[2] >= need and \
                self.keys[0].shape[:2] == (B, H):
            return
        if D % 64:
            raise ValueError(f"head_dim {D} is not a multiple of 64")
        cap = -(-need // self.step) * self.step
        words, groups = D * self.bits // 32, D // 64

        def grown(old):
            return (_grow(old[0] if old else None, (B, H), cap, words, torch.int32, keys.device,
                          self.offset),
                    _grow(old[1] if old else None, (B, H), cap, groups, torch.float16,
                          keys.device, self.offset),
                    _grow(old[2] if old else None, (B, H), cap, groups, torch.float16,
                          keys.device, self.offset))

        self.keys = grown(self.keys)
        self.values = grown(self.values)

    def pools(self) -> tuple[torch.Tensor, ...]:
        """The state as the 6-tuple of quantised pools (B blocks of capacity tokens)."""
        return (*self.keys, *self.values)

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor) -> tuple[tuple, tuple]:
        """Quantise and append ``keys/values [B, H, n, D]``; return the
        quantised state of the first ``offset`` tokens."""
        if keys.dim() != 4 or keys.shape != values.shape:
            raise ValueError("keys/values must be [B, H, n, D] of the same shape")
        B, _, n, _ = keys.shape
        self._reserve(keys, n)
        cap = self.keys[0].shape[2]
        for b in range(B):
            ops.kv_quant_append(self.pools(), keys[b], values[b],
                                _slots(b, cap, self.offset, n, keys.device))
        self.offset += n
        return self.state

    @property
    def state(self) -> tuple[Any, Any]:
        if self.keys is None:
            return (None, None)
        first = self.keys[0] if isinstance(self.keys, tuple) else self.keys
        if self.offset == first.shape[2]:
            return self.keys, self.values
        cut = self.offset

        def head(x):
            return tuple(t[:, :, :cut] for t in x) if isinstance(x, tuple) else x[:, :, :cut]

        return head(self.keys), head(self.values)

    @state.setter
    def state(self, v: tuple[Any, Any]) -> None:
        # as mlx_lm: the offset is kept (RestoringQuantizedKVCache re-derives it)
        self.keys, self.values = v

    def is_trimmable(self) -> bool:
        return True

    def trim(self, n: int) -> int:
        n = min(self.offset, n)
        self.offset -= n
        return n


def make_prompt_cache(model: Any, max_kv_size: int | None = None) -> list[Any]:
    """One empty KVCache per layer of ``model`` (its own ``make_cache`` if it
    has one).  A bounded (rotating) cache is not part of this path."""
    if max_kv_size is not None:
        raise NotImplementedError("max_kv_size (a rotating KV cache) is not supported")
    if hasattr(model, "make_cache"):
        return model.make_cache()
    return [KVCache() for _ in model.layers]
