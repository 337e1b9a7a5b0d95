"""Paged attention: block-managed KV cache on B200 HBM with fused decode attention."""
from .attention import paged_attention_forward, paged_decode
from .block_manager import BlockManager, DoubleFreeError, OutOfBlocksError, PhysicalBlock
from .paged_kv import PagedKVCache

__all__ = [
    "BlockManager",
    "DoubleFreeError",
    "OutOfBlocksError",
    "PagedKVCache",
    "PhysicalBlock",
    "paged_attention_forward",
    "paged_decode",
]
