"""Pinned host-memory tier for evicted KV blocks.

Eviction: ``mz_block_pack`` gathers the blocks (every layer's K and V) into a
device staging buffer on the compute stream, then a side stream copies the
staging buffer to pinned host slots with cudaMemcpyAsync.  Reload: the side
stream copies host slots into staging, then ``mz_block_unpack`` scatters them
into freshly allocated device blocks on the compute stream.  Two staging
buffers alternate, so the pack of chunk i+1 overlaps the copy of chunk i;
events order every hand-over between the streams.  Host slots are
[n_pools * block_bytes] rows of one pinned buffer; runs of consecutive slots
move with one copy.

The reference's second tier is a disk cache (src/mlxz/prefix_cache/disk.py);
on this path the slower tier is pinned host RAM reached over the host link.
"""
from __future__ import annotations

import torch

from .. import ops


def _runs(slots: list[int]) -> list[tuple[int, int, int]]:
    """(first index in `slots`, first slot, length) of runs of consecutive slots."""
    out = []
    i = 0
    while i < len(slots):
        j = i
        while j + 1 < len(slots) and slots[j + 1] == slots[j] + 1:
            j += 1
        out.append((i, slots[i], j - i + 1))
        i = j + 1
    return out


class PinnedHostTier:
    """A pool of pinned host slots, each holding one block of every pool."""

    def __init__(self, capacity_blocks: int, n_pools: int, block_bytes: int, device,
                 staging_bytes: int = 256 << 20) -> None:
        self.device = torch.device(device)
        self.n_pools, self.block_bytes = n_pools, block_bytes
        self.slot_bytes = n_pools * block_bytes
        self.capacity = capacity_blocks
        self.host = torch.empty((capacity_blocks, self.slot_bytes), dtype=torch.uint8,
                                pin_memory=True)
        self._free = list(range(capacity_blocks - 1, -1, -1))  # pops lowest slot first
        self.copy_stream = torch.cuda.Stream(self.device)
        self.chunk = max(1, staging_bytes // self.slot_bytes)
        self._staging = [torch.empty((self.chunk, self.slot_bytes), dtype=torch.uint8,
                                     device=self.device) for _ in range(2)]
        self._staging_free = [None, None]  # event after which staging[i] may be reused
        self._last_d2h = None               # event: all evictions so far copied to host

    @property
    def free_slots(self) -> int:
        return len(self._free)

    def used_bytes(self) -> int:
        return (self.capacity - len(self._free)) * self.slot_bytes

    def _take(self, n: int) -> list[int]:
        if n > len(self._free):
            raise MemoryError(f"host tier full: need {n} slots, {len(self._free)} free")
        return [self._free.pop() for _ in range(n)]

    def release(self, slots: list[int]) -> None:
        self._free.extend(sorted(slots, reverse=True))

    def evict(self, pools: torch.Tensor, block_ids: list[int]) -> list[int]:
        """Copy blocks ``block_ids`` of the pool stack to newly taken host slots.

        Returns the slots.  The device blocks may be reused by later work on
        the current stream as soon as this returns (the pack is ordered
        before it); the host copy completes asynchronously (see ``sync``)."""
        slots = self._take(len(block_ids))
        compute = torch.cuda.current_stream(self.device)
        for c, lo in enumerate(range(0, len(block_ids), self.chunk)):
            ids = block_ids[lo:lo + self.chunk]
            k = c % 2
            st = self._staging[k]
            if self._staging_free[k] is not None:
                compute.wait_event(self._staging_free[k])
            ids_t = torch.tensor(ids, dtype=torch.int32).to(self.device, non_blocking=True)
            ops.block_pack(pools, ids_t, st.view(self.chunk, self.n_pools, self.block_bytes))
            packed = torch.cuda.Event()
            packed.record(compute)
            with torch.cuda.stream(self.copy_stream):
                self.copy_stream.wait_event(packed)
                for i0, s0, n in _runs(slots[lo:lo + len(ids)]):
                    self.host[s0:s0 + n].copy_(st[i0:i0 + n], non_blocking=True)
                done = torch.cuda.Event()
                done.record(self.copy_stream)
            self._staging_free[k] = done
            self._last_d2h = done
        return slots

    def reload(self, pools: torch.Tensor, slots: list[int], block_ids: list[int]) -> None:
        """Copy host slots back into device blocks ``block_ids`` (enqueued; the
        unpack runs on the current stream, so later work there sees the data)."""
        if len(slots) != len(block_ids):
            raise ValueError("slots and block_ids differ in length")
        compute = torch.cuda.current_stream(self.device)
        for c, lo in enumerate(range(0, len(slots), self.chunk)):
            sl = slots[lo:lo + self.chunk]
            k = c % 2
            st = self._staging[k]
            with torch.cuda.stream(self.copy_stream):
                if self._last_d2h is not None:
                    self.copy_stream.wait_event(self._last_d2h)
                if self._staging_free[k] is not None:
                    self.copy_stream.wait_event(self._staging_free[k])
                for i0, s0, n in _runs(sl):
                    st[i0:i0 + n].copy_(self.host[s0:s0 + n], non_blocking=True)
                loaded = torch.cuda.Event()
                loaded.record(self.copy_stream)
            compute.wait_event(loaded)
            ids_t = torch.tensor(block_ids[lo:lo + len(sl)], dtype=torch.int32).to(
                self.device, non_blocking=True)
            ops.block_unpack(pools, ids_t, st.view(self.chunk, self.n_pools, self.block_bytes))
            done = torch.cuda.Event()
            done.record(compute)
            self._staging_free[k] = done

    def sync(self) -> None:
        """Wait until every copy issued so far has finished."""
        self.copy_stream.synchronize()
        torch.cuda.current_stream(self.device).synchronize()
