"""Engine-side KV plumbing: paged stores (bf16/fp16 and 4/8-bit quantised) and
the ragged continuous-batching decode step and chunked prefill."""
from .decode_step import (PagedDecodeStep, PagedKVStore, QuantizedPagedDecodeStep,
                          QuantizedPagedKVStore)
from .prefill import ChunkedPrefillScheduler, PagedPrefillStep, PrefillChunk

__all__ = ["ChunkedPrefillScheduler", "PagedDecodeStep", "PagedKVStore", "PagedPrefillStep",
           "PrefillChunk", "QuantizedPagedDecodeStep", "QuantizedPagedKVStore"]
