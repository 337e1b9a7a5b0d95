"""Engine-side KV plumbing: paged stores (bf16/fp16 and 4/8-bit quantised) and
the ragged continuous-batching decode step."""
from .decode_step import (PagedDecodeStep, PagedKVStore, QuantizedPagedDecodeStep,
                          QuantizedPagedKVStore)

__all__ = ["PagedDecodeStep", "PagedKVStore", "QuantizedPagedDecodeStep", "QuantizedPagedKVStore"]
