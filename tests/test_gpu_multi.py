"""Head-sharded decode on 2 GPUs (one process each, NCCL process group):
the all-gather fused into the decode launch over peer memory (PeerAllGather),
waited for after every layer and chained (each launch waiting for the layer
before it), against the NCCL all-gather of the ordinary launch's output
(HeadAllGather), bit for bit, over several layers and steps.  Skipped with
fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

L, B, HKV, G, D, BS = 3, 6, 8, 4, 128, 16
CTX = [1, 17, 300, 2049, 64, 777]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, results) -> None:
    import datetime

    import torch.distributed as dist

    from mlxz_b200 import ops
    from mlxz_b200.engine import PagedDecodeStep, PagedKVStore
    from mlxz_b200.engine.sharding import HeadAllGather, HeadShard, PeerAllGather

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        sh = HeadShard(rank, world, HKV, HKV * G)
        need = [(c + 1 + BS - 1) // BS for c in CTX]
        n_blocks = sum(need) + 4
        g = torch.Generator().manual_seed(1234)
        perm = torch.randperm(n_blocks, generator=g).tolist()
        pools = torch.randn((L, 2, n_blocks, HKV, BS, D), generator=g).to(torch.bfloat16)
        q = torch.randn((2, L, B, HKV * G, D), generator=g).to(torch.bfloat16)
        kn = torch.randn((2, L, B, HKV, D), generator=g).to(torch.bfloat16)
        vn = torch.randn((2, L, B, HKV, D), generator=g).to(torch.bfloat16)

        def make_step():
            store = PagedKVStore(L, n_blocks, sh.kv_local, D, BS, torch.bfloat16, dev, init="empty")
            store.pools.copy_(sh.kv_slice(pools, 3).to(dev))
            used = 0
            for b in range(B):
                store.add_sequence(f"s{b}", CTX[b], blocks=perm[used:used + need[b]])
                used += need[b]
            return PagedDecodeStep(store, [f"s{b}" for b in range(B)], sh.q_local)

        qd = sh.q_slice(q, 3).contiguous().to(dev)
        kd = sh.kv_slice(kn, 3).contiguous().to(dev)
        vd = sh.kv_slice(vn, 3).contiguous().to(dev)

        # NCCL path: ordinary launch, then all-gather + layout copy
        step_a = make_step()
        nccl = HeadAllGather(sh, B, D, torch.bfloat16, dev)
        want = torch.empty((2, L, B, HKV * G, D), dtype=torch.bfloat16, device=dev)
        local = torch.empty((B, sh.q_local, D), dtype=torch.bfloat16, device=dev)
        for t in range(2):
            for l in range(L):
                step_a.layer(l, qd[t, l], kd[t, l], vd[t, l], local)
                nccl.full(local, out=want[t, l])
            step_a.advance()

        # fused path: stores into every rank's buffer + signal + bounded wait
        step_b = make_step()
        peer = PeerAllGather(sh, B, D, torch.bfloat16, dev, n_slots=L)
        got = torch.empty_like(want)
        for t in range(2):
            for l in range(L):
                got[t, l].copy_(peer.layer(step_b, l, qd[t, l], kd[t, l], vd[t, l], slot=l))
            step_b.advance()
        # chained: each layer's launch waits in its prologue for the peers'
        # rows of the layer before it; one wait launch after the last layer
        step_c = make_step()
        chain = PeerAllGather(sh, B, D, torch.bfloat16, dev, n_slots=2 * L)
        got_c = torch.empty_like(want)
        for t in range(2):
            base = L * (t % 2)
            for l in range(L):
                chain.launch(step_c, l, qd[t, l], kd[t, l], vd[t, l], slot=base + l,
                             wait_previous=l > 0)
            chain.wait()
            for l in range(L):
                got_c[t, l].copy_(chain.full[base + l])
            step_c.advance()
        torch.cuda.synchronize()
        ops.check_device_errors(rank)
        same_pools = (torch.equal(step_a.store.pools, step_b.store.pools)
                      and torch.equal(step_a.store.pools, step_c.store.pools))
        peer.close()
        chain.close()
        results[rank] = (bool(torch.equal(got, want) and torch.equal(got_c, want)), same_pools,
                         float((got.float() - want.float()).abs().max()), peer.epoch)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_fused_gather_matches_nccl():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        mp.start_processes(_rank, args=(2, _free_port(), results), nprocs=2, join=True,
                           start_method="spawn")
        got = dict(results)
    assert sorted(got) == [0, 1]
    for r, (equal, same_pools, err, epoch) in got.items():
        assert equal and same_pools, (r, err)
        assert epoch == 2 * L
