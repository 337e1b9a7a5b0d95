"""Fixed-size block pool with reference counting (host policy).

Same contract as the reference's BlockManager
(src/mlxz/paged_attention/block_manager.py:29-147): a LIFO free list popped
from the end, refcount 1 on allocation, ``free`` returning a block to the
list when its count reaches zero, ``incref`` for shared prefix blocks and
``copy_on_write`` that hands back the same id for an unshared block or a
fresh one (the caller copies the data, with ``mz_block_copy``).  Errors and
their partial effects (a ``free``/``incref`` list stops at the first bad
block) match the reference; the golden traces in tests/golden pin them.
"""
from __future__ import annotations

from dataclasses import dataclass


class OutOfBlocksError(Exception):
    """Raised when block allocation cannot be satisfied."""

    def __init__(self, requested: int, available: int) -> None:
        self.requested = requested
        self.available = available
        super().__init__(f"Cannot allocate {requested} blocks; only {available} free")


class DoubleFreeError(Exception):
    """Raised when freeing a block whose refcount is already 0."""

    def __init__(self, block_idx: int) -> None:
        self.block_idx = block_idx
        super().__init__(f"Double free on block {block_idx} (refcount already 0)")


@dataclass(slots=True)
class PhysicalBlock:
    """A single physical block in the pool (index and reference count)."""

    idx: int
    refcount: int = 0


class BlockManager:
    """Block pool with reference counting, copy-on-write and a LIFO free list.

    Invariants: free_blocks + #(refcount > 0) == total_blocks; no refcount is
    negative; freeing a block at refcount 0 raises DoubleFreeError.
    """

    def __init__(self, total_blocks: int, block_size: int) -> None:
        if total_blocks < 1:
            raise ValueError(f"total_blocks must be >= 1, got {total_blocks}")
        if block_size < 1:
            raise ValueError(f"block_size must be >= 1, got {block_size}")
        self._total_blocks = total_blocks
        self._block_size = block_size
        self._refcount: list[int] = [0] * total_blocks
        self._free_list: list[int] = list(range(total_blocks))  # stack, top at the end

    @property
    def total_blocks(self) -> int:
        return self._total_blocks

    @property
    def block_size(self) -> int:
        return self._block_size

    @property
    def free_blocks(self) -> int:
        return len(self._free_list)

    def allocate(self, n_blocks: int) -> list[int]:
        """Pop n blocks off the free list (refcount 1 each)."""
        if n_blocks < 0:
            raise ValueError(f"Cannot allocate negative blocks: {n_blocks}")
        if n_blocks == 0:
            return []
        free = self._free_list
        if n_blocks > len(free):
            raise OutOfBlocksError(n_blocks, len(free))
        out = free[len(free) - n_blocks:][::-1]  # same order as n successive pops
        del free[len(free) - n_blocks:]
        rc = self._refcount
        for idx in out:
            rc[idx] = 1
        return out

    def free(self, block_indices: list[int]) -> None:
        """Decrement each block; a block reaching 0 goes back on the free list."""
        rc = self._refcount
        for idx in block_indices:
            if rc[idx] <= 0:
                raise DoubleFreeError(idx)
            rc[idx] -= 1
            if rc[idx] == 0:
                self._free_list.append(idx)

    def incref(self, block_indices: list[int]) -> None:
        """Share blocks (prefix cache); a freed block raises ValueError."""
        rc = self._refcount
        for idx in block_indices:
            if rc[idx] <= 0:
                raise ValueError(f"Cannot incref freed block {idx}")
            rc[idx] += 1

    def copy_on_write(self, block_idx: int) -> int:
        """Id of a block the caller may write: the same block if unshared,
        otherwise a new block (refcount 1) with the original decremented."""
        rc = self._refcount
        if rc[block_idx] <= 0:
            raise ValueError(f"Cannot COW freed block {block_idx}")
        if rc[block_idx] == 1:
            return block_idx
        new_idx = self.allocate(1)[0]
        rc[block_idx] -= 1
        return new_idx

    def get_refcount(self, block_idx: int) -> int:
        return self._refcount[block_idx]

    def _debug_state(self) -> dict:
        """For testing: internal state summary."""
        return {
            "total": self._total_blocks,
            "free": len(self._free_list),
            "allocated": [(i, r) for i, r in enumerate(self._refcount) if r > 0],
        }

    def blocks(self) -> list[PhysicalBlock]:
        """Snapshot of every block's refcount."""
        return [PhysicalBlock(i, r) for i, r in enumerate(self._refcount)]
