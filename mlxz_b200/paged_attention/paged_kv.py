"""Block-table KV cache over B200 HBM pools.

Same interface as the reference's PagedKVCache
(src/mlxz/paged_attention/paged_kv.py:12-154) with torch tensors in place of
mx arrays.  Block tables and offsets stay on the host (as in the reference);
the data moves through the CUDA kernels: ``append_kv`` computes the slots on
the host, allocating blocks exactly as the reference's loop does
(paged_kv.py:72-83), and scatters the rows with one ``mz_kv_append`` launch;
``get_kv`` is one ``mz_kv_gather`` launch.
"""
from __future__ import annotations

import torch

from .. import ops
from .block_manager import BlockManager, OutOfBlocksError


def _device(device) -> torch.device:
    if device is None:
        return torch.device("cuda", torch.cuda.current_device())
    d = torch.device(device)
    if d.type != "cuda":
        raise ValueError("PagedKVCache pools live in GPU memory: pass a CUDA device")
    return d if d.index is not None else torch.device("cuda", torch.cuda.current_device())


class PagedKVCache:
    """KV cache backed by a block table.

    Pools: ``(total_blocks, n_kv_heads, block_size, head_dim)`` per K and V,
    zero-filled, on one CUDA device.
    """

    def __init__(self, block_manager: BlockManager, n_kv_heads: int, head_dim: int,
                 dtype: torch.dtype = torch.float16, device=None) -> None:
        self._bm = block_manager
        self._n_kv_heads = n_kv_heads
        self._head_dim = head_dim
        self._dtype = dtype
        self._block_size = block_manager.block_size
        self._device = _device(device)
        shape = (block_manager.total_blocks, n_kv_heads, self._block_size, head_dim)
        self._key_pool = torch.zeros(shape, dtype=dtype, device=self._device)
        self._value_pool = torch.zeros(shape, dtype=dtype, device=self._device)
        self._block_tables: dict[str, list[int]] = {}
        self._offsets: dict[str, int] = {}

    # -- reference API -----------------------------------------------------

    def allocate_sequence(self, seq_id: str, initial_blocks: int = 1) -> None:
        """Allocate initial blocks for a new sequence."""
        blocks = self._bm.allocate(initial_blocks)
        self._block_tables[seq_id] = blocks
        self._offsets[seq_id] = 0

    def free_sequence(self, seq_id: str) -> None:
        """Free all blocks of a sequence (no-op for an unknown id)."""
        if seq_id in self._block_tables:
            self._bm.free(self._block_tables.pop(seq_id))
            self._offsets.pop(seq_id, None)

    def append_kv(self, seq_id: str, keys: torch.Tensor, values: torch.Tensor) -> None:
        """Append ``(1, n_kv_heads, n_new, head_dim)`` keys/values, growing the
        block table on demand.  If the pool runs out mid-way, the rows before
        the failing token are written, the table keeps the blocks it got, the
        offset is unchanged and OutOfBlocksError propagates (as in the
        reference, whose offset update follows its loop)."""
        n_new = keys.shape[2]
        offset = self._offsets[seq_id]
        blocks = self._block_tables[seq_id]
        bs = self._block_size
        slots: list[int] = []
        err: OutOfBlocksError | None = None
        for i in range(n_new):
            pos = offset + i
            bi = pos // bs
            try:
                while bi >= len(blocks):
                    blocks.extend(self._bm.allocate(1))
            except OutOfBlocksError as e:
                err = e
                break
            slots.append(blocks[bi] * bs + pos % bs)
        if slots:
            k = keys.to(self._device, non_blocking=True)
            v = values.to(self._device, non_blocking=True)
            if len(slots) < n_new:
                k, v = k[:, :, : len(slots)], v[:, :, : len(slots)]
            slot_t = torch.tensor(slots, dtype=torch.int64).to(self._device, non_blocking=True)
            ops.kv_append(self._key_pool, self._value_pool, k, v, slot_t)
        if err is not None:
            raise err
        self._offsets[seq_id] = offset + n_new

    def get_kv(self, seq_id: str) -> tuple[torch.Tensor, torch.Tensor]:
        """Contiguous ``(1, n_kv_heads, offset, head_dim)`` keys and values."""
        offset = self._offsets[seq_id]
        if offset == 0:
            shape = (1, self._n_kv_heads, 0, self._head_dim)
            return (torch.zeros(shape, dtype=self._dtype, device=self._device),
                    torch.zeros(shape, dtype=self._dtype, device=self._device))
        table = self.block_table_tensor([seq_id])
        ctx = torch.tensor([offset], dtype=torch.int32).to(self._device, non_blocking=True)
        return ops.kv_gather(self._key_pool, self._value_pool, table, ctx, [offset])

    def get_block_table(self, seq_id: str) -> list[int]:
        """The block table of a sequence (a copy)."""
        return list(self._block_tables.get(seq_id, []))

    def get_offset(self, seq_id: str) -> int:
        """Number of tokens stored for a sequence."""
        return self._offsets.get(seq_id, 0)

    @property
    def stats(self) -> dict:
        return {
            "total_blocks": self._bm.total_blocks,
            "free_blocks": self._bm.free_blocks,
            "active_sequences": len(self._block_tables),
        }

    # -- batched / kernel-facing helpers -------------------------------------

    @property
    def block_manager(self) -> BlockManager:
        return self._bm

    @property
    def k_pool(self) -> torch.Tensor:
        return self._key_pool

    @property
    def v_pool(self) -> torch.Tensor:
        return self._value_pool

    @property
    def block_size(self) -> int:
        return self._block_size

    @property
    def n_kv_heads(self) -> int:
        return self._n_kv_heads

    @property
    def head_dim(self) -> int:
        return self._head_dim

    @property
    def dtype(self) -> torch.dtype:
        return self._dtype

    @property
    def device(self) -> torch.device:
        return self._device

    def block_table_tensor(self, seq_ids: list[str], min_blocks: int = 1) -> torch.Tensor:
        """int32 ``[len(seq_ids), max_blocks]`` device copy of the tables
        (unused entries are -1)."""
        tabs = [self._block_tables[s] for s in seq_ids]
        width = max([min_blocks] + [len(t) for t in tabs])
        host = torch.full((len(tabs), width), -1, dtype=torch.int32)
        for i, t in enumerate(tabs):
            if t:
                host[i, : len(t)] = torch.tensor(t, dtype=torch.int32)
        return host.to(self._device, non_blocking=True)

    def ctx_tensor(self, seq_ids: list[str]) -> torch.Tensor:
        return torch.tensor([self._offsets[s] for s in seq_ids],
                            dtype=torch.int32).to(self._device, non_blocking=True)

    def ensure_capacity(self, seq_id: str, n_tokens: int) -> None:
        """Grow the table so that `n_tokens` more tokens fit (block growth of
        append_kv done ahead of a batched append)."""
        blocks = self._block_tables[seq_id]
        need = -(-(self._offsets[seq_id] + n_tokens) // self._block_size)
        while len(blocks) < need:
            blocks.extend(self._bm.allocate(1))

    def append_kv_batch(self, seq_ids: list[str], keys: torch.Tensor,
                        values: torch.Tensor) -> None:
        """One decode-step token per sequence: keys/values ``[B, H, 1, D]`` (or
        ``[B, H, D]``), one ``mz_kv_append_paged`` launch."""
        for s in seq_ids:
            self.ensure_capacity(s, 1)
        tables = self.block_table_tensor(seq_ids)
        pos = self.ctx_tensor(seq_ids)
        ops.kv_append_paged(self._key_pool, self._value_pool, keys.to(self._device),
                            values.to(self._device), tables, pos)
        for s in seq_ids:
            self._offsets[s] += 1
