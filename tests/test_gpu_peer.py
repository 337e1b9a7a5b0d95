"""All-gather of head-sharded decode outputs fused into the decode launch
(mz_paged_append_decode_allgather + mz_peer_wait), on one GPU.

N ranks are emulated in one process: each "rank" has its own KV-head shard,
gathered buffer, signal words and arrival counter, all in this GPU's memory,
and every launch is queued on one stream before the waits, so each signal a
wait reads is already set when it runs (no kernel waits on another).  The
gathered buffers must equal, bit for bit, the concatenation of the ordinary
fused append+decode launches of each shard (same kernel, same schedule), and
the oracle within the attention tolerance.  The bounded wait's timeout is
exercised with a signal word nothing sets.
"""
import numpy as np
import pytest
import torch

from mlxz_b200 import _native as nat
from mlxz_b200 import ops
from oracle import paged as opaged
from oracle import rng
from tests.gpu_util import attn_err, random_paged_case, to_dev

pytestmark = pytest.mark.gpu
ATOL_REL = 2e-3


def _peers(N, rank, bufs, sigs, arrivals, block_bytes, epoch):
    pe = nat.PeerOutputs()
    pe.n_ranks, pe.rank = N, rank
    for s in range(N):
        pe.out[s] = bufs[s].data_ptr() + rank * block_bytes
        pe.signal[s] = sigs[s].data_ptr()
    pe.arrivals = arrivals.data_ptr()
    pe.epoch = epoch
    return pe


@pytest.mark.parametrize("N,nw", [(2, 0), (4, 0), (8, 0), (2, 40)])
def test_emulated_ranks_gather_bit_exact(cuda, N, nw):
    B, Hkv, G, D, bs = 10, 8, 4, 128, 16
    Hq = Hkv * G
    lengths = [1, 16, 17, 300, 2049, 5, 64, 1000, 33, 4096]
    case = random_paged_case(91, B, Hkv, D, bs, lengths, "bf16", G=G)
    kp, vp = to_dev(case["kp"], "bf16", cuda), to_dev(case["vp"], "bf16", cuda)
    nk_bits = rng.normal(92, (B, Hkv, D), "bf16", stream=1)
    nv_bits = rng.normal(92, (B, Hkv, D), "bf16", stream=2)
    nk, nv = to_dev(nk_bits, "bf16", cuda), to_dev(nv_bits, "bf16", cuda)
    q = to_dev(case["q"][:, 0], "bf16", cuda)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    lens = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    hk, hq = Hkv // N, Hq // N

    shards, refs = [], []
    for r in range(N):
        sl = slice(r * hk, (r + 1) * hk)
        kr, vr = kp[:, sl].contiguous(), vp[:, sl].contiguous()
        qr = q[:, r * hq:(r + 1) * hq].contiguous()
        nkr, nvr = nk[:, sl].contiguous(), nv[:, sl].contiguous()
        refs.append(ops.paged_append_decode(qr, kr.clone(), vr.clone(), nkr, nvr, tables, lens,
                                            num_warps=nw))
        shards.append((kr, vr, qr, nkr, nvr))
    full_ref = torch.cat(refs, dim=1)

    bufs = [torch.empty((B, Hq, D), dtype=torch.bfloat16, device=cuda) for _ in range(N)]
    sigs = [torch.zeros(N, dtype=torch.int32, device=cuda) for _ in range(N)]
    arr = [torch.zeros(1, dtype=torch.int32, device=cuda) for _ in range(N)]
    for epoch in (1, 2):  # two launches in a row: counters reset, epochs advance
        for b in bufs:
            b.fill_(float("nan"))
        for r, (kr, vr, qr, nkr, nvr) in enumerate(shards):
            pe = _peers(N, r, bufs, sigs, arr[r], hq * D * 2, epoch)
            ops.paged_append_decode_allgather(pe, qr, kr, vr, nkr, nvr, tables, lens, Hq * D, D,
                                              torch.bfloat16, num_warps=nw)
        for r in range(N):
            ops.peer_wait(sigs[r], N, r, epoch, timeout_s=2.0)
        torch.cuda.synchronize()
        ops.check_device_errors(0)
        for r in range(N):
            want = [0 if s == r else epoch for s in range(N)]
            assert sigs[r].tolist() == want
            assert arr[r].item() == 0
            assert torch.equal(bufs[r], full_ref), r

    # the new tokens landed in every shard's pools, and the result is the oracle's
    okp, ovp = case["kp"].copy(), case["vp"].copy()
    for b in range(B):
        pos = lengths[b] - 1
        blk = case["tables"][b][pos // bs]
        okp[blk, :, pos % bs] = nk_bits[b]
        ovp[blk, :, pos % bs] = nv_bits[b]
    for r, (kr, vr, *_rest) in enumerate(shards):
        assert np.array_equal(kr.cpu().view(torch.int16).numpy().view(np.uint16),
                              okp[:, r * hk:(r + 1) * hk])
    ref = opaged.paged_decode(case["q"][:, 0], okp, ovp, case["tables"], np.array(lengths), "bf16")
    assert attn_err(bufs[0], ref) <= ATOL_REL


@pytest.mark.parametrize("N", [2, 8])
def test_emulated_ranks_chained_waits(cuda, N):
    """Layers chained with MZ_LAUNCH_WAIT_PREVIOUS: each launch waits inside
    its prologue for the peers' rows of the launch before it, and only the
    last layer is followed by mz_peer_wait.  Launches go on one stream in
    (layer, rank) order without overlap, so every word a launch waits for was
    published by a kernel that completed before it began."""
    B, Hkv, G, D, bs, L = 6, 8, 4, 128, 16, 3
    Hq = Hkv * G
    lengths = [1, 17, 300, 2049, 64, 777]
    case = random_paged_case(93, B, Hkv, D, bs, lengths, "bf16", G=G)
    kp, vp = to_dev(case["kp"], "bf16", cuda), to_dev(case["vp"], "bf16", cuda)
    nk = to_dev(rng.normal(94, (B, Hkv, D), "bf16", stream=1), "bf16", cuda)
    nv = to_dev(rng.normal(94, (B, Hkv, D), "bf16", stream=2), "bf16", cuda)
    qs = [to_dev(rng.normal(95, (B, Hq, D), "bf16", stream=l), "bf16", cuda) for l in range(L)]
    tables = torch.from_numpy(case["tables"]).to(cuda)
    lens = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    hk, hq = Hkv // N, Hq // N
    shards = []
    for r in range(N):
        sl = slice(r * hk, (r + 1) * hk)
        shards.append((kp[:, sl].contiguous(), vp[:, sl].contiguous(), nk[:, sl].contiguous(),
                       nv[:, sl].contiguous()))
    want = []
    for l in range(L):
        parts = [ops.paged_append_decode(qs[l][:, r * hq:(r + 1) * hq].contiguous(),
                                         kr.clone(), vr.clone(), nkr, nvr, tables, lens)
                 for r, (kr, vr, nkr, nvr) in enumerate(shards)]
        want.append(torch.cat(parts, dim=1))
    bufs = [torch.full((L, B, Hq, D), float("nan"), dtype=torch.bfloat16, device=cuda)
            for _ in range(N)]
    sigs = [torch.zeros(N, dtype=torch.int32, device=cuda) for _ in range(N)]
    arr = [torch.zeros(1, dtype=torch.int32, device=cuda) for _ in range(N)]
    for l in range(L):
        epoch = l + 1
        for r, (kr, vr, nkr, nvr) in enumerate(shards):
            pe = nat.PeerOutputs()
            pe.n_ranks, pe.rank = N, r
            for s in range(N):
                pe.out[s] = bufs[s][l].data_ptr() + r * hq * D * 2
                pe.signal[s] = sigs[s].data_ptr()
            pe.arrivals = arr[r].data_ptr()
            pe.epoch = epoch
            ops.paged_append_decode_allgather(pe, qs[l][:, r * hq:(r + 1) * hq].contiguous(), kr,
                                              vr, nkr, nvr, tables, lens, Hq * D, D,
                                              torch.bfloat16, wait_previous=l > 0)
    for r in range(N):
        ops.peer_wait(sigs[r], N, r, L, timeout_s=2.0)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    for r in range(N):
        assert sigs[r].tolist() == [0 if s == r else L for s in range(N)]
        for l in range(L):
            assert torch.equal(bufs[r][l], want[l]), (r, l)


def test_chained_wait_times_out_and_context_survives(cuda):
    """A launch whose folded wait never sees its peer's word gives up after
    the bound, reports MZ_DEVERR_TIMEOUT and still completes its own work."""
    B, Hkv, G, D, bs = 2, 2, 2, 64, 16
    case = random_paged_case(7, B, Hkv, D, bs, [5, 40], "bf16", G=G)
    kp, vp = to_dev(case["kp"], "bf16", cuda), to_dev(case["vp"], "bf16", cuda)
    q = to_dev(case["q"][:, 0], "bf16", cuda)
    nk = torch.zeros(B, Hkv, D, dtype=torch.bfloat16, device=cuda)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    lens = torch.tensor([5, 40], dtype=torch.int32, device=cuda)
    buf = torch.zeros(B, Hkv * G, D, dtype=torch.bfloat16, device=cuda)
    sig = torch.zeros(2, dtype=torch.int32, device=cuda)
    arr = torch.zeros(1, dtype=torch.int32, device=cuda)
    pe = nat.PeerOutputs()
    pe.n_ranks, pe.rank, pe.epoch = 2, 0, 5  # waits for word 1 to reach 4: never set
    pe.out[0] = buf.data_ptr()
    pe.out[1] = buf.data_ptr()  # the "peer" is this buffer too: nothing else is touched
    pe.signal[0] = sig.data_ptr()
    pe.signal[1] = sig.data_ptr()
    pe.arrivals = arr.data_ptr()
    want = ops.paged_append_decode(q, kp.clone(), vp.clone(), nk, nk, tables, lens)
    ops.paged_append_decode_allgather(pe, q, kp, vp, nk, nk, tables, lens, Hkv * G * D, D,
                                      torch.bfloat16, wait_previous=True)
    torch.cuda.synchronize()
    with pytest.raises(nat.DeviceError) as e:
        ops.check_device_errors(0)
    assert e.value.bits & nat.MZ_DEVERR_TIMEOUT
    assert torch.equal(buf, want)
    assert sig.tolist() == [5, 0]  # its own launch still signalled the "peer"
    assert arr.item() == 0


def test_peer_wait_times_out_and_context_survives(cuda):
    sig = torch.zeros(2, dtype=torch.int32, device=cuda)
    ops.peer_wait(sig, 2, 0, 7, timeout_s=0.002)  # word 1 is never set
    torch.cuda.synchronize()
    with pytest.raises(nat.DeviceError) as e:
        ops.check_device_errors(0)
    assert e.value.bits & nat.MZ_DEVERR_TIMEOUT
    x = torch.ones(8, device=cuda)
    assert x.sum().item() == 8.0  # the context is still usable
    sig[1] = 7
    ops.peer_wait(sig, 2, 0, 7, timeout_s=0.002)
    torch.cuda.synchronize()
    ops.check_device_errors(0)


def test_peer_wait_epoch_comparison_wraps(cuda):
    sig = torch.zeros(2, dtype=torch.int32, device=cuda)
    sig[1] = 3  # published after the epochs wrapped: ahead of 2^32 - 1
    ops.peer_wait(sig, 2, 0, 0xFFFFFFFF, timeout_s=0.002)
    torch.cuda.synchronize()
    ops.check_device_errors(0)
    sig[1] = -1  # 2^32 - 1 is behind epoch 2 of the next lap
    ops.peer_wait(sig, 2, 0, 2, timeout_s=0.002)
    torch.cuda.synchronize()
    with pytest.raises(nat.DeviceError):
        ops.check_device_errors(0)


def test_allgather_argument_checks(cuda):
    B, Hkv, G, D, bs = 2, 2, 2, 64, 16
    case = random_paged_case(5, B, Hkv, D, bs, [5, 40], "bf16", G=G)
    kp, vp = to_dev(case["kp"], "bf16", cuda), to_dev(case["vp"], "bf16", cuda)
    q = to_dev(case["q"][:, 0], "bf16", cuda)
    nk = torch.zeros(B, Hkv, D, dtype=torch.bfloat16, device=cuda)
    tables = torch.from_numpy(case["tables"]).to(cuda)
    lens = torch.tensor([5, 40], dtype=torch.int32, device=cuda)
    buf = torch.zeros(B, Hkv * G, D, dtype=torch.bfloat16, device=cuda)
    sig = torch.zeros(2, dtype=torch.int32, device=cuda)
    arr = torch.zeros(1, dtype=torch.int32, device=cuda)
    for N, rank, epoch in [(2, 0, 0), (2, 2, 1), (9, 0, 1), (0, 0, 1)]:
        pe = nat.PeerOutputs()
        pe.n_ranks, pe.rank, pe.epoch = N, rank, epoch
        for s in range(min(N, 8)):
            pe.out[s] = buf.data_ptr()
            pe.signal[s] = sig.data_ptr()
        pe.arrivals = arr.data_ptr()
        with pytest.raises(ValueError):
            ops.paged_append_decode_allgather(pe, q, kp, vp, nk, nk, tables, lens,
                                              Hkv * G * D, D, torch.bfloat16)
    with pytest.raises(ValueError):
        ops.peer_wait(sig, 2, 0, 0)
    with pytest.raises(ValueError):
        ops.peer_wait(sig, 2, 3, 1)
    torch.cuda.synchronize()
    ops.check_device_errors(0)


def test_ipc_export_offsets(cuda):
    t = torch.zeros(1 << 20, dtype=torch.uint8, device=cuda)
    h0, off0 = ops.ipc_export(t)
    h1, off1 = ops.ipc_export(t[4096:])
    assert len(h0) == nat.MZ_IPC_HANDLE_BYTES and h0 == h1
    assert off1 == off0 + 4096
