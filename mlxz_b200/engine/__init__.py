"""Engine-side KV plumbing: the multi-layer paged store and the ragged decode step."""
from .decode_step import PagedDecodeStep, PagedKVStore

__all__ = ["PagedDecodeStep", "PagedKVStore"]
