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


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_one_process_drives_two_gpus_fused_gather():
    """One process, two GPUs: each GPU runs its half of the KV heads with the
    all-gather fused into the launch, its rows stored into the other GPU's
    buffer through peer access; both gathered buffers equal the two halves'
    ordinary launches side by side, bytewise.  Kernel shared-memory opt-ins
    are per device, so the launch on the second GPU also checks that they are
    set there."""
    from cuda.bindings import runtime as cudart

    from mlxz_b200 import _native as nat
    from mlxz_b200 import ops

    if not (torch.cuda.can_device_access_peer(0, 1) and torch.cuda.can_device_access_peer(1, 0)):
        pytest.skip("GPUs 0 and 1 have no peer access")
    for a, b in ((0, 1), (1, 0)):
        torch.cuda.set_device(a)
        cudart.cudaSetDevice(a)
        err = cudart.cudaDeviceEnablePeerAccess(b, 0)[0]
        assert err in (cudart.cudaError_t.cudaSuccess,
                       cudart.cudaError_t.cudaErrorPeerAccessAlreadyEnabled), err
    N, hkv, hq = 2, HKV // 2, HKV * G // 2
    need = [(c + 1 + BS - 1) // BS for c in CTX]
    n_blocks = sum(need) + 4
    g = torch.Generator().manual_seed(4321)
    perm = torch.randperm(n_blocks, generator=g).to(torch.int32)
    tables = torch.full((B, max(need)), -1, dtype=torch.int32)
    used = 0
    for b in range(B):
        tables[b, :need[b]] = perm[used:used + need[b]]
        used += need[b]
    lens = torch.tensor([c + 1 for c in CTX], dtype=torch.int32)
    ranks = []
    for r in range(N):
        dev = torch.device("cuda", r)
        mk = lambda *shape: torch.randn(shape, generator=g).to(torch.bfloat16).to(dev)  # noqa: E731
        ranks.append(dict(k=mk(n_blocks, hkv, BS, D), v=mk(n_blocks, hkv, BS, D), q=mk(B, hq, D),
                          kn=mk(B, hkv, D), vn=mk(B, hkv, D), tables=tables.to(dev),
                          lens=lens.to(dev),
                          full=torch.zeros((B, N * hq, D), dtype=torch.bfloat16, device=dev),
                          sig=torch.zeros(N, dtype=torch.int32, device=dev),
                          arrivals=torch.zeros(1, dtype=torch.int32, device=dev),
                          ws=ops.decode_workspace(B, hkv, G, D, r, shared=False)))
    local = []
    for r in range(N):
        rk = ranks[r]
        with torch.cuda.device(r):
            local.append(ops.paged_append_decode(rk["q"], rk["k"], rk["v"], rk["kn"], rk["vn"],
                                                 rk["tables"], rk["lens"]).cpu())
    for epoch in (1, 2):
        for r in range(N):
            rk = ranks[r]
            pe = nat.PeerOutputs()
            pe.n_ranks, pe.rank, pe.epoch = N, r, epoch
            for s in range(N):
                pe.out[s] = ranks[s]["full"].data_ptr() + r * hq * D * 2
                pe.signal[s] = ranks[s]["sig"].data_ptr()
            pe.arrivals = rk["arrivals"].data_ptr()
            with torch.cuda.device(r):
                ops.paged_append_decode_allgather(pe, rk["q"], rk["k"], rk["v"], rk["kn"],
                                                  rk["vn"], rk["tables"], rk["lens"], N * hq * D,
                                                  D, torch.bfloat16, workspace=rk["ws"])
        for r in range(N):
            torch.cuda.synchronize(r)
        for r in range(N):
            with torch.cuda.device(r):
                ops.peer_wait(ranks[r]["sig"], N, r, epoch)
            torch.cuda.synchronize(r)
            ops.check_device_errors(r)
    want = torch.cat(local, dim=1).view(torch.int16)
    for r in range(N):
        assert torch.equal(ranks[r]["full"].cpu().view(torch.int16), want)
