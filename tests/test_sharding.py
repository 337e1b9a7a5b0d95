"""KV-head sharding host logic on CPU: HeadShard ranges and the world-size-2
gloo all-gather of head-sharded attention outputs (oracle attention per rank,
compared with the oracle over all heads)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from mlxz_b200.engine.sharding import HeadAllGather, HeadShard


def test_head_shard_ranges():
    s = [HeadShard(r, 4, 8, 64) for r in range(4)]
    assert [x.kv_range for x in s] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert [x.q_range for x in s] == [(0, 16), (16, 32), (32, 48), (48, 64)]
    # every query head of a rank reads a KV head of the same rank (h // G)
    G = 64 // 8
    for x in s:
        lo, hi = x.q_range
        assert {h // G for h in range(lo, hi)} == set(range(*x.kv_range))
    t = torch.arange(2 * 8 * 3).view(2, 8, 3)
    assert torch.equal(s[1].kv_slice(t, 1), t[:, 2:4])


@pytest.mark.parametrize("args", [(0, 3, 8, 32), (2, 2, 8, 32), (0, 2, 8, 12), (0, 0, 8, 32)])
def test_head_shard_rejects(args):
    with pytest.raises(ValueError):
        HeadShard(*args)


def test_world_one_is_identity():
    g = HeadAllGather(HeadShard(0, 1, 8, 32), 4, 16, torch.float32, "cpu")
    x = torch.randn(4, 32, 16)
    assert g.gather(x) is x
    assert g.full(x) is x


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(seed=5, B=3, Hq=8, Hkv=4, D=16, bs=4, n_blocks=40):
    from oracle.rng import normal, permutation

    ctx = np.array([7, 1, 22])
    kp = normal(seed, (n_blocks, Hkv, bs, D), "bf16")
    vp = normal(seed + 1, (n_blocks, Hkv, bs, D), "bf16")
    q = normal(seed + 2, (B, Hq, D), "bf16")
    perm = permutation(seed + 3, n_blocks)
    tables = np.full((B, 8), -1, dtype=np.int64)
    used = 0
    for b in range(B):
        n = -(-int(ctx[b]) // bs)
        tables[b, :n] = perm[used:used + n]
        used += n
    return q, kp, vp, tables, ctx


def _rank(rank: int, world: int, port: int, results) -> None:
    import torch.distributed as dist

    from oracle.paged import paged_decode

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, kp, vp, tables, ctx = _case()
        B, Hq, D = q.shape
        sh = HeadShard(rank, world, kp.shape[1], Hq)
        lo, hi = sh.kv_range
        qlo, qhi = sh.q_range
        local = paged_decode(q[:, qlo:qhi], kp[:, lo:hi], vp[:, lo:hi], tables, ctx, "bf16")
        gat = HeadAllGather(sh, B, D, torch.float64, "cpu")
        full = gat.full(torch.from_numpy(np.ascontiguousarray(local)))
        out = torch.empty(B, Hq, D, dtype=torch.float64)
        gat.full(torch.from_numpy(np.ascontiguousarray(local)), out=out)
        ref = paged_decode(q, kp, vp, tables, ctx, "bf16")
        results[rank] = (float(np.abs(full.numpy() - ref).max()),
                         float(np.abs(out.numpy() - ref).max()))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_head_sharded_gather():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        mp.start_processes(_rank, args=(2, _free_port(), results), nprocs=2, join=True,
                           start_method="spawn")
        got = dict(results)
    assert sorted(got) == [0, 1]
    for r, (e_full, e_out) in got.items():
        assert e_full <= 1e-12 and e_out <= 1e-12, (r, e_full, e_out)


class _FakeStep:
    """Just what PeerAllGather.launch reads from a PagedDecodeStep."""

    class store:  # noqa: N801
        @staticmethod
        def k_pool(l):
            return None

        v_pool = k_pool

    tables = lengths = workspace = None
    scale = 1.0


def _peer_world1(monkeypatch, n_slots):
    """A world-size-1 PeerAllGather on the CPU with the kernel launches
    recorded instead of run (the slot and ordering rules are host logic)."""
    from mlxz_b200 import ops
    from mlxz_b200.engine.sharding import PeerAllGather

    calls = []
    monkeypatch.setattr(ops, "paged_append_decode_allgather",
                        lambda pe, *a, **k: calls.append((pe.epoch, k["wait_previous"])))
    monkeypatch.setattr(ops, "peer_wait", lambda *a, **k: calls.append("wait"))
    pg = PeerAllGather(HeadShard(0, 1, 8, 32), 2, 16, torch.bfloat16, "cpu", n_slots=n_slots)
    return pg, calls


def test_peer_gather_slot_rules(monkeypatch):
    st = _FakeStep()
    pg, calls = _peer_world1(monkeypatch, 3)
    # launch + wait per layer: only the previous launch's slot is off limits
    pg.layer(st, 0, None, None, None, slot=0)
    with pytest.raises(ValueError):
        pg.layer(st, 1, None, None, None, slot=0)
    pg.layer(st, 1, None, None, None, slot=1)
    pg.layer(st, 2, None, None, None, slot=0)
    # chained launches: the launch after a wait_previous launch may not reuse
    # the slot that launch completed
    pg.launch(st, 0, None, None, None, slot=1)
    pg.launch(st, 1, None, None, None, slot=2, wait_previous=True)
    with pytest.raises(ValueError):
        pg.launch(st, 2, None, None, None, slot=1, wait_previous=True)
    pg.launch(st, 2, None, None, None, slot=0, wait_previous=True)
    # a plain launch while the last one was neither waited for nor chained
    with pytest.raises(RuntimeError):
        pg.launch(st, 3, None, None, None, slot=1)
    pg.wait()
    pg.launch(st, 3, None, None, None, slot=1)
    with pytest.raises(ValueError):
        pg.launch(st, 4, None, None, None, slot=3, wait_previous=True)
    epochs = [c[0] for c in calls if c != "wait"]
    assert epochs == list(range(1, len(epochs) + 1))
    assert [c[1] for c in calls if c != "wait"] == [False] * 3 + [False, True, True, False]


def test_peer_gather_needs_two_slots():
    from mlxz_b200.engine.sharding import PeerAllGather

    with pytest.raises(ValueError):
        PeerAllGather(HeadShard(0, 1, 8, 32), 2, 16, torch.bfloat16, "cpu", n_slots=1)
