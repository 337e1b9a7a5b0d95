"""KV-path configuration knobs (the KV / paged / prefix-cache sections of the
reference's RuntimeConfig, src/mlxz/config.py:28-62, with the same defaults
and bounds)."""
from __future__ import annotations

from typing import Literal

from pydantic import BaseModel, Field


class KVConfig(BaseModel):
    """Quantised KV-cache parameters (config.py:28-36)."""

    bits: Literal[4, 8, 16] = 8
    group_size: int = Field(default=64, ge=1, le=256)
    quantized_kv_start: int = Field(default=512, ge=0)
    streaming_sink_size: int = Field(default=4, ge=1)


class PagedConfig(BaseModel):
    """Paged-attention block layout (config.py:39-44)."""

    block_size: int = Field(default=16, ge=1, le=256)
    enabled: bool = False


class PrefixCacheConfig(BaseModel):
    """Prefix cache budgets (config.py:47-62); the disk tier of the reference
    is replaced here by a pinned host-memory tier."""

    memory_budget_gb: float = Field(default=8.0, gt=0)
    host_budget_gb: float = Field(default=32.0, gt=0)
    block_size: int = Field(default=8, ge=1, le=256)
