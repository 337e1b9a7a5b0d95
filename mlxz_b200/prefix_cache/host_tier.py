"""Pinned host-memory tier for evicted KV blocks.

A block lives in one or more "stacks" of pools (``[P, n_blocks, ...]``
tensors: K/V of every layer; for quantised stores also their scales and
biases).  Eviction: ``mz_block_pack`` gathers the blocks of each stack into a
device staging buffer on the compute stream, then a side stream copies the
staging buffers to pinned host slots with cudaMemcpyAsync.  Reload: the side
stream copies host slots into staging, then ``mz_block_unpack`` scatters them
into freshly allocated device blocks on the compute stream.  Two staging sets
alternate, so the pack of chunk i+1 overlaps the copy of chunk i; events order
every hand-over between the streams.  Runs of consecutive host slots move
with one copy per stack.

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


def _geometry(stack: torch.Tensor) -> tuple[int, int]:
    """(pools, bytes of one block in one pool) of a ``[P, n_blocks, ...]`` stack."""
    return stack.shape[0], stack[0, 0].numel() * stack.element_size()


class PinnedHostTier:
    """A pool of pinned host slots, each holding one block of every pool of
    every stack.  ``layout``: list of (n_pools, block_bytes) per stack, or one
    (n_pools, block_bytes) pair."""

    def __init__(self, capacity_blocks: int, n_pools_or_layout, block_bytes: int | None = None,
                 device=None, staging_bytes: int = 256 << 20) -> None:
        if block_bytes is not None:
            layout = [(int(n_pools_or_layout), int(block_bytes))]
        else:
            layout = [(int(p), int(b)) for p, b in n_pools_or_layout]
        self.device = torch.device(device)
        self.layout = layout
        self.row_bytes = [p * b for p, b in layout]
        self.slot_bytes = sum(self.row_bytes)
        self.capacity = capacity_blocks
        self.host = [torch.empty((capacity_blocks, rb), dtype=torch.uint8, pin_memory=True)
                     for rb in self.row_bytes]
        self._free = list(range(capacity_blocks - 1, -1, -1))  # pops lowest slot first
        self.copy_stream = torch.cuda.Stream(self.device)
        self.chunk = max(1, staging_bytes // self.slot_bytes)
        self._staging = [[torch.empty((self.chunk, rb), dtype=torch.uint8, device=self.device)
                          for rb in self.row_bytes] for _ in range(2)]
        self._staging_free = [None, None]  # event after which staging set i may be reused
        self._last_d2h = None               # event: all evictions so far copied to host

    @classmethod
    def for_stacks(cls, capacity_blocks: int, stacks: list[torch.Tensor], **kw) -> "PinnedHostTier":
        return cls(capacity_blocks, [_geometry(s) for s in stacks], device=stacks[0].device, **kw)

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

    def _check(self, stacks) -> list[torch.Tensor]:
        stacks = [stacks] if isinstance(stacks, torch.Tensor) else list(stacks)
        if [_geometry(s) for s in stacks] != self.layout:
            raise ValueError("pool stacks do not match the tier's layout")
        return stacks

    def evict(self, stacks, block_ids: list[int]) -> list[int]:
        """Copy blocks ``block_ids`` of the pool stacks to newly taken host slots.

        Returns the slots.  The device blocks may be reused by later work on
        the current stream as soon as this returns (the pack is ordered
        before it); the host copy completes asynchronously (see ``sync``)."""
        stacks = self._check(stacks)
        slots = self._take(len(block_ids))
        compute = torch.cuda.current_stream(self.device)
        for c, lo in enumerate(range(0, len(block_ids), self.chunk)):
            ids = block_ids[lo:lo + self.chunk]
            k = c % 2
            if self._staging_free[k] is not None:
                compute.wait_event(self._staging_free[k])
            ids_t = torch.tensor(ids, dtype=torch.int32).to(self.device, non_blocking=True)
            for stack, st, (P, bb) in zip(stacks, self._staging[k], self.layout):
                ops.block_pack(stack, ids_t, st.view(self.chunk, P, bb))
            packed = torch.cuda.Event()
            packed.record(compute)
            with torch.cuda.stream(self.copy_stream):
                self.copy_stream.wait_event(packed)
                for host, st in zip(self.host, self._staging[k]):
                    for i0, s0, n in _runs(slots[lo:lo + len(ids)]):
                        host[s0:s0 + n].copy_(st[i0:i0 + n], non_blocking=True)
                done = torch.cuda.Event()
                done.record(self.copy_stream)
            self._staging_free[k] = done
            self._last_d2h = done
        return slots

    def reload(self, stacks, slots: list[int], block_ids: list[int]) -> None:
        """Copy host slots back into device blocks ``block_ids`` (enqueued; the
        unpack runs on the current stream, so later work there sees the data)."""
        stacks = self._check(stacks)
        if len(slots) != len(block_ids):
            raise ValueError("slots and block_ids differ in length")
        compute = torch.cuda.current_stream(self.device)
        for c, lo in enumerate(range(0, len(slots), self.chunk)):
            sl = slots[lo:lo + self.chunk]
            k = c % 2
            with torch.cuda.stream(self.copy_stream):
                if self._last_d2h is not None:
                    self.copy_stream.wait_event(self._last_d2h)
                if self._staging_free[k] is not None:
                    self.copy_stream.wait_event(self._staging_free[k])
                for host, st in zip(self.host, self._staging[k]):
                    for i0, s0, n in _runs(sl):
                        st[i0:i0 + n].copy_(host[s0:s0 + n], non_blocking=True)
                loaded = torch.cuda.Event()
                loaded.record(self.copy_stream)
            compute.wait_event(loaded)
            ids_t = torch.tensor(block_ids[lo:lo + len(sl)], dtype=torch.int32).to(
                self.device, non_blocking=True)
            for stack, st, (P, bb) in zip(stacks, self._staging[k], self.layout):
                ops.block_unpack(stack, ids_t, st.view(self.chunk, P, bb))
            done = torch.cuda.Event()
            done.record(compute)
            self._staging_free[k] = done

    def sync(self) -> None:
        """Wait until every copy issued so far has finished."""
        self.copy_stream.synchronize()
        torch.cuda.current_stream(self.device).synchronize()
