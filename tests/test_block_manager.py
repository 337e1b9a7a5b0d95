"""BlockManager: replay of the reference's own behaviour (golden traces) plus
the example and state-machine properties of the reference's tests
(tests/unit/test_block_manager.py in the reference)."""
import json

import pytest
from hypothesis import settings
from hypothesis import strategies as st
from hypothesis.stateful import RuleBasedStateMachine, invariant, rule

from mlxz_b200.paged_attention.block_manager import (
    BlockManager,
    DoubleFreeError,
    OutOfBlocksError,
)
from tests.conftest import GOLDEN

TRACES = json.loads((GOLDEN / "block_manager_traces.json").read_text())


@pytest.mark.parametrize("ti", range(len(TRACES)))
def test_replay_reference_trace(ti):
    tr = TRACES[ti]
    bm = BlockManager(tr["total_blocks"], tr["block_size"])
    for rec in tr["ops"]:
        fn = getattr(bm, "copy_on_write" if rec["op"] == "cow" else rec["op"])
        if "raises" in rec:
            want = rec["raises"]
            exc = {"OutOfBlocksError": OutOfBlocksError, "DoubleFreeError": DoubleFreeError,
                   "ValueError": ValueError}[want["type"]]
            with pytest.raises(exc) as ei:
                fn(*rec["args"])
            if want["type"] == "OutOfBlocksError":
                assert (ei.value.requested, ei.value.available) == (want["requested"],
                                                                    want["available"])
            elif want["type"] == "DoubleFreeError":
                assert ei.value.block_idx == want["block_idx"]
            else:
                assert str(ei.value) == want["msg"]
        else:
            assert fn(*rec["args"]) == rec["result"]
        s = rec["state"]
        assert bm._free_list == s["free_list"]
        assert [bm.get_refcount(i) for i in range(bm.total_blocks)] == s["refcounts"]
        assert [list(x) for x in bm._debug_state()["allocated"]] == s["allocated"]


def test_examples():
    bm = BlockManager(total_blocks=10, block_size=16)
    assert (bm.total_blocks, bm.free_blocks, bm.block_size) == (10, 10, 16)
    blocks = bm.allocate(3)
    assert blocks == [9, 8, 7] and bm.free_blocks == 7
    bm.free(blocks)
    assert bm.free_blocks == 10
    assert bm.allocate(0) == []
    with pytest.raises(OutOfBlocksError) as e:
        bm.allocate(11)
    assert (e.value.requested, e.value.available) == (11, 10)
    with pytest.raises(ValueError):
        bm.allocate(-1)
    with pytest.raises(ValueError):
        BlockManager(0, 16)
    with pytest.raises(ValueError):
        BlockManager(4, 0)
    b = bm.allocate(1)
    bm.incref(b)
    assert bm.get_refcount(b[0]) == 2
    new = bm.copy_on_write(b[0])
    assert new != b[0] and bm.get_refcount(b[0]) == 1 and bm.get_refcount(new) == 1
    assert bm.copy_on_write(b[0]) == b[0]
    bm.free(b)
    with pytest.raises(DoubleFreeError):
        bm.free(b)
    with pytest.raises(ValueError, match="Cannot incref freed block"):
        bm.incref(b)
    with pytest.raises(ValueError, match="Cannot COW freed block"):
        bm.copy_on_write(b[0])


class BlockManagerMachine(RuleBasedStateMachine):
    """allocate / free / fork (incref) / copy-on-write with leak and refcount
    invariants checked after every step."""

    def __init__(self):
        super().__init__()
        self.bm = BlockManager(total_blocks=32, block_size=16)
        self.owned: dict[int, list[int]] = {}
        self.n = 0

    @rule(k=st.integers(min_value=1, max_value=8))
    def allocate(self, k):
        if self.bm.free_blocks >= k:
            self.n += 1
            self.owned[self.n] = self.bm.allocate(k)

    @rule(data=st.data())
    def free_seq(self, data):
        if self.owned:
            sid = data.draw(st.sampled_from(sorted(self.owned)))
            self.bm.free(self.owned.pop(sid))

    @rule(data=st.data())
    def fork(self, data):
        if self.owned:
            sid = data.draw(st.sampled_from(sorted(self.owned)))
            self.bm.incref(self.owned[sid])
            self.n += 1
            self.owned[self.n] = list(self.owned[sid])

    @rule(data=st.data())
    def cow(self, data):
        if not self.owned:
            return
        sid = data.draw(st.sampled_from(sorted(self.owned)))
        blocks = self.owned[sid]
        i = data.draw(st.integers(min_value=0, max_value=len(blocks) - 1))
        if self.bm.get_refcount(blocks[i]) > 1 and self.bm.free_blocks == 0:
            return
        blocks[i] = self.bm.copy_on_write(blocks[i])

    @invariant()
    def no_leaks(self):
        used = sum(1 for i in range(32) if self.bm.get_refcount(i) > 0)
        assert self.bm.free_blocks + used == 32

    @invariant()
    def refcounts_match_owners(self):
        want = [0] * 32
        for blocks in self.owned.values():
            for b in blocks:
                want[b] += 1
        assert [self.bm.get_refcount(i) for i in range(32)] == want


TestBlockManagerMachine = BlockManagerMachine.TestCase
TestBlockManagerMachine.settings = settings(max_examples=150, stateful_step_count=30,
                                            deadline=None)


def test_step_copy_groups_cover_the_layers_in_order():
    from mlxz_b200.engine.decode_step import _copy_groups

    for L in range(1, 130):
        g = _copy_groups(L)
        assert g[0][0] == 0 and g[-1][1] == L
        assert all(a < b for a, b in g) and all(g[i][1] == g[i + 1][0] for i in range(len(g) - 1))
        if L >= 2:
            assert g[0] == (0, 1) and g[-1] == (L - 1, L)
