#!/usr/bin/env python
"""Paged-decode benchmark on the Llama-3.1-8B KV shape, batch 64 per GPU.

One step = for each of 32 layers, one launch of mz_paged_append_decode: append
one new token per sequence into the paged pool, then fused GQA decode
attention over ctx + 1 tokens.  Sequences: 64 with ctx ~ U[512, 8192]
(seeded), block size 16, pools sized to the blocks needed + 10 %, random
block tables, Q/K/V ~ N(0, 1) bf16.  Each step rewrites the same new-token
slots, so every timed step does identical work.

N > 1 GPUs (torchrun): weak scaling by KV-head sharding -- the global batch
is 64 * N sequences, rank r holds KV heads [r*8/N, (r+1)*8/N) of every
sequence (the same bytes per GPU as N = 1), and each layer's head-sharded
output is all-gathered with NCCL.

Printed value: KV bytes read per step (sum_b (ctx_b + 1) * 4096 B * 32
layers, all ranks) / step time.  `--impl reference` times the reference's
CPU algorithm (oracle port) instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
METRIC = ("paged-decode KV-read GB/s (% of HBM peak) and decode tok/s, 8B shape, batch 64")
L, HQ, HKV, D, BS, B_PER_GPU = 32, 32, 8, 128, 16, 64
CTX_LO, CTX_HI = 512, 8192
FALLBACK_HBM_GBS = 6650.0
C5_METRIC = ("head-sharded paged-decode KV-read GB/s (all GPUs) and decode tok/s, "
             "70B shape, batch 256")
C5_L, C5_HQ, C5_B = 80, 64, 256
C5_MEDIAN, C5_SIGMA, C5_LO, C5_HI = 4096, 1.0, 256, 32768


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mlxz_b200", choices=["mlxz_b200", "reference"])
    ap.add_argument("--layers", type=int, default=None,
                    help="layers (decode: default 32); sharded70b: resident layers cap")
    ap.add_argument("--resident-gb", type=float, default=120.0,
                    help="sharded70b: HBM budget for the resident layers' pools")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="approximate CPU time budget of the cpu_baseline sample")
    ap.add_argument("--num-warps", type=int, default=0)
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--separate-append", action="store_true",
                    help="append with mz_kv_append_paged, then mz_paged_decode (two launches)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-sub-records", action="store_true",
                    help="decode: skip the sub-records measured after the headline (sharded70b "
                         "at every N; prefix, quant8 and quant4 at N = 1)")
    ap.add_argument("--batch-invariant", action="store_true",
                    help="decode: MZ_DECODE_BATCH_INVARIANT (whole pairs, batch-independent bytes)")
    ap.add_argument("--config", default="decode",
                    choices=["decode", "prefix", "quant", "sharded70b", "prefill", "kernels",
                             "peer_pair"],
                    help="decode: the paged decode step (headline); prefix: prefix-cache "
                         "restore / copy-on-write / host-tier eviction and reload; quant: "
                         "4/8-bit quantised KV decode step; sharded70b: 70B-shape decode "
                         "step head-sharded over the ranks (strong scaling); prefill: one "
                         "chunked-prefill iteration (append + causal attention per layer); "
                         "kernels: each data-movement kernel timed alone; peer_pair: one "
                         "process driving two GPUs, the 70B-shape fused decode + all-gather "
                         "launch of rank 0 of 2 timed on GPU 0 (its output rows stored into "
                         "GPU 1's buffer over NVLink), for profiling the launch alone")
    ap.add_argument("--bits", type=int, default=8, choices=[4, 8])
    ap.add_argument("--prefill-offset", type=int, default=3584,
                    help="prefill: cached tokens before each 512-token chunk (0 = fresh "
                         "prompts); the headline prefill workload uses 3584")
    ap.add_argument("--kv-bits", type=int, default=16, choices=[4, 8, 16],
                    help="prefill: the K/V store (16 = bf16; 8 / 4 = quantised, "
                         "dequantised per layer into a staging pool)")
    ap.add_argument("--gather", default="p2p", choices=["p2p", "nccl"],
                    help="N > 1: p2p = output rows stored into every rank's buffer by the "
                         "decode launch itself (peer memory over NVLink) + bounded signal "
                         "wait; nccl = ordinary launch, then NCCL all-gather + layout copy")
    return ap.parse_args()


def workload_ctx(seed: int, n: int):
    import numpy as np

    return np.random.default_rng(seed).integers(CTX_LO, CTX_HI + 1, size=n).astype(np.int64)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(name: str):
    """traffic_bytes_per_launch from a committed ncu summary, or None."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


# ---------------------------------------------------------------------------
# clocks sampling (nvidia-smi in the background during the timed region)
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_uuid: str | None, enabled: bool = True):
        self.proc = None
        self.path = None
        if not enabled:
            return
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                   "-lms", "200"]
            if device_uuid:
                cmd += ["-i", device_uuid]
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v == "Active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": reasons}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's algorithm (oracle port) on the host cores
# ---------------------------------------------------------------------------

def cpu_case(seed: int, threads: int, n_seqs: int = 16):
    """One layer of `n_seqs` sequences drawn from the workload's ctx
    distribution, for oracle.cpu_path.decode_layer (torch-CPU restatement of
    the reference's get_kv + GQA attention).  Returns (run, kv_bytes): run()
    times one layer and returns its seconds."""
    import torch

    from oracle import cpu_path

    torch.set_num_threads(threads)
    ctx = workload_ctx(seed + 17, n_seqs)
    need = (ctx + 1 + BS - 1) // BS
    n_blocks = int(need.sum())
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(n_blocks, generator=g)
    tables, used = [], 0
    for n in need:
        tables.append(perm[used:used + int(n)])
        used += int(n)
    kp = torch.randn((n_blocks, HKV, BS, D), generator=g).to(torch.bfloat16)
    vp = torch.randn((n_blocks, HKV, BS, D), generator=g).to(torch.bfloat16)
    q = torch.randn((n_seqs, HQ, D), generator=g).to(torch.bfloat16).float()
    nk = torch.randn((n_seqs, HKV, D), generator=g).to(torch.bfloat16)
    nv = torch.randn((n_seqs, HKV, D), generator=g).to(torch.bfloat16)
    kv_bytes = float((ctx + 1).sum()) * HKV * D * 2 * 2
    ctx_l = [int(c) for c in ctx]

    def run() -> float:
        t0 = time.perf_counter()
        cpu_path.decode_layer(q, kp, vp, tables, ctx_l, nk, nv, D ** -0.5)
        return time.perf_counter() - t0

    return run, kv_bytes


def cpu_sample(seed: int, budget_s: float, threads: int, n_seqs: int = 16):
    """Median time of one layer (cpu_case) over repeats until ~budget_s."""
    run, kv_bytes = cpu_case(seed, threads, n_seqs)
    run()
    times = []
    t_end = time.perf_counter() + budget_s
    while True:
        times.append(run())
        if time.perf_counter() > t_end or len(times) >= 100:
            break
    t = statistics.median(times)
    return {"gbs": kv_bytes / t / 1e9, "tok_s": n_seqs / (t * 32), "reps": len(times),
            "layer_s": t, "n_seqs": n_seqs, "kv_bytes": kv_bytes}


PF_B, PF_CHUNK, PF_CTX = 8, 512, 4096
PF_METRIC = ("chunked-prefill attention TFLOP/s and prefill tok/s, 8B shape, "
             "8 x 512-token chunks at offset 3584")


def set_prefill_offset(offset: int) -> None:
    """Chunks at `offset` cached tokens (the workload constants and metric)."""
    global PF_CTX, PF_METRIC
    if offset < 0 or offset % BS:
        raise SystemExit("--prefill-offset must be a non-negative multiple of 16")
    PF_CTX = offset + PF_CHUNK
    PF_METRIC = ("chunked-prefill attention TFLOP/s and prefill tok/s, 8B shape, "
                 f"8 x 512-token chunks at offset {offset}")


def prefill_flops_layer(n_seqs: int = PF_B) -> float:
    """Causal attention FLOPs of one layer: QK^T and PV, 2 per multiply-add,
    over every (query, visible key) pair."""
    start = PF_CTX - PF_CHUNK
    pairs = PF_CHUNK * start + PF_CHUNK * (PF_CHUNK + 1) // 2
    return 4.0 * D * HQ * pairs * n_seqs


def cpu_prefill_sample(seed: int, threads: int):
    """Times oracle.cpu_path.prefill_layer (torch-CPU restatement of a prompt
    chunk's append + causal GQA attention) on one sequence of one layer."""
    import torch

    from oracle import cpu_path

    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    nb = PF_CTX // BS
    kp = torch.randn((nb, HKV, BS, D), generator=g).to(torch.bfloat16)
    vp = torch.randn((nb, HKV, BS, D), generator=g).to(torch.bfloat16)
    tables = [torch.randperm(nb, generator=g)]
    q = torch.randn((PF_CHUNK, HQ, D), generator=g).to(torch.bfloat16).float()
    nk = torch.randn((PF_CHUNK, HKV, D), generator=g).to(torch.bfloat16)
    nv = torch.randn((PF_CHUNK, HKV, D), generator=g).to(torch.bfloat16)
    args = (q, kp, vp, tables, [PF_CTX], [PF_CHUNK], nk, nv, D ** -0.5)
    cpu_path.prefill_layer(*args)
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        cpu_path.prefill_layer(*args)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"tflops": prefill_flops_layer(1) / t / 1e12, "layer_seq_s": t}


def run_reference_prefill(args, world: int) -> None:
    threads = os.cpu_count() or 1
    vals = [cpu_prefill_sample(args.seed + i, threads)
            for i in range(max(1, min(args.steps, 5)))]
    v = statistics.median(x["tflops"] for x in vals)
    ms = statistics.median(x["layer_seq_s"] for x in vals) * 1000.0 * PF_B * args.layers
    sample = (f"1 of {PF_B} sequences x 1 of {args.layers} layers (a 512-token chunk at "
              f"offset {PF_CTX - PF_CHUNK}), torch-CPU port of append + causal GQA attention, {threads} "
              f"threads; ms_per_step extrapolated to {PF_B} sequences x {args.layers} layers")
    line = {
        "impl": "reference", "metric": PF_METRIC, "value": round(v, 5), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V/Q, random block tables)",
        "config": {"workload": "8B-shape chunked-prefill iteration (CPU sample)",
                   "layers": args.layers, "global_batch": PF_B, "seq_len": PF_CTX,
                   "parallelism": "host threads"},
        "prefill_tok_s": round(PF_B * PF_CHUNK / (ms / 1e3), 3),
        "cpu_baseline": {"value": round(v, 5), "unit": "TFLOP/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(v, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_prefill(args, local_rank: int) -> None:
    """Chunked-prefill iteration, Llama-3.1-8B shape: 32 layers, 32 q heads, 8
    KV heads, head_dim 128, block 16; 8 sequences each prefilling a 512-token
    chunk on top of 3584 cached tokens (--prefill-offset; 0 = fresh prompts).  One step = per layer, through
    PagedPrefillStep.layer: mz_kv_append of the chunk's K/V, then
    mz_paged_prefill (causal GQA attention over cache + chunk).  Every step
    rewrites the same slots, so timed steps do identical work."""
    import numpy as np
    import torch

    from mlxz_b200 import ops
    from mlxz_b200.engine import PagedKVStore, PagedPrefillStep, QuantizedPagedKVStore

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    nl = args.layers
    kv_bits = args.kv_bits
    nb_seq = PF_CTX // BS
    n_blocks = int(math.ceil(PF_B * nb_seq * 1.1))
    perm = np.random.default_rng(args.seed + 1).permutation(n_blocks)
    torch.manual_seed(args.seed)
    if kv_bits == 16:
        store = PagedKVStore(nl, n_blocks, HKV, D, BS, torch.bfloat16, dev, init="empty")
        for l in range(nl):
            store.pools[l].normal_()
    else:
        store = QuantizedPagedKVStore(nl, n_blocks, HKV, D, BS, bits=kv_bits, device=dev,
                                      init="empty")
        allsl = torch.arange(n_blocks * BS, dtype=torch.int64, device=dev)
        for l in range(nl):
            for lo in range(0, n_blocks * BS, 8192):
                sl = allsl[lo:lo + 8192]
                kk = torch.randn(HKV, sl.numel(), D, device=dev).to(torch.bfloat16)
                vv = torch.randn(HKV, sl.numel(), D, device=dev).to(torch.bfloat16)
                ops.kv_quant_append(store.qpools(l), kk, vv, sl)
    ids = []
    for b in range(PF_B):
        store.add_sequence(f"s{b}", PF_CTX - PF_CHUNK,
                           blocks=[int(x) for x in perm[b * nb_seq:(b + 1) * nb_seq]])
        ids.append(f"s{b}")
    step = PagedPrefillStep(store, [(s, PF_CHUNK) for s in ids], HQ)
    T = PF_B * PF_CHUNK
    q = torch.randn(nl, T, HQ, D, device=dev).to(torch.bfloat16)
    kn = torch.randn(nl, T, HKV, D, device=dev).to(torch.bfloat16)
    vn = torch.randn(nl, T, HKV, D, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    flops_layer = prefill_flops_layer()
    warm = max(3, args.warmup)

    def one_step():
        for l in range(nl):
            step.layer(l, q[l], kn[l], vn[l], out=out[l])

    for _ in range(warm):
        one_step()
    torch.cuda.synchronize()
    ops.check_device_errors(local_rank)
    steps = args.steps
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(uuid, enabled=not args.no_clocks)
    t0.record()
    for _ in range(steps):
        one_step()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ops.check_device_errors(local_rank)
    ms = t0.elapsed_time(t1) / steps

    # the attention kernel alone: events around each launch (one extra pass);
    # over a quantised store, the per-layer dequantisation into the staging
    # pool is timed on its own too
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(nl)]
    for l in range(nl):
        if kv_bits == 16:
            kp, vp = store.k_pool(l), store.v_pool(l)
        else:
            kp, vp = step._stage
            evs[l][2].record()
            ops.kv_dequant_blocks(store.qpools(l), step._ids, kp, vp)
            evs[l][3].record()
        evs[l][0].record()
        ops.paged_prefill(q[l], kp, vp, step.tables, step.q_start, step.q_len, step.ctx_lens,
                          step.max_q_len, step.scale, out=out[l])
        evs[l][1].record()
    torch.cuda.synchronize()
    pf_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    dq_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in evs) if kv_bits != 16 else None

    # end to end: per layer the chunk's q/k/v from pinned host memory and the
    # attention output back, copies pipelined against the layers' launches
    e2e = None
    h2d = d2h = 0
    if not args.no_e2e:
        hq = q.cpu().pin_memory()
        hk = kn.cpu().pin_memory()
        hv = vn.cpu().pin_memory()
        ho = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        cs = torch.cuda.Stream(dev)
        stq = [torch.empty_like(q[0]) for _ in range(2)]
        stk = [torch.empty_like(kn[0]) for _ in range(2)]
        stv = [torch.empty_like(vn[0]) for _ in range(2)]
        sto = [torch.empty_like(out[0]) for _ in range(2)]
        main = torch.cuda.current_stream(dev)

        def e2e_step():
            done = [None, None]
            for l in range(nl):
                i = l & 1
                with torch.cuda.stream(cs):
                    if done[i] is not None:
                        cs.wait_event(done[i])
                    stq[i].copy_(hq[l], non_blocking=True)
                    stk[i].copy_(hk[l], non_blocking=True)
                    stv[i].copy_(hv[l], non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(cs)
                main.wait_event(ready)
                step.layer(l, stq[i], stk[i], stv[i], out=sto[i])
                fin = torch.cuda.Event()
                fin.record(main)
                with torch.cuda.stream(cs):
                    cs.wait_event(fin)
                    ho[l].copy_(sto[i], non_blocking=True)
                    done[i] = torch.cuda.Event()
                    done[i].record(cs)
            main.wait_stream(cs)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2e_steps = max(2, min(steps, 5))
        a.record()
        for _ in range(e2e_steps):
            e2e_step()
        z.record()
        torch.cuda.synchronize()
        ops.check_device_errors(local_rank)
        e_ms = a.elapsed_time(z) / e2e_steps
        h2d = nl * (q[0].numel() + 2 * kn[0].numel()) * 2
        d2h = nl * out[0].numel() * 2
        e2e = {"value": round(flops_layer * nl / (e_ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e_ms, 3)}

    cpu = None
    if not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        r = cpu_prefill_sample(args.seed, threads)
        cpu = {"value": round(r["tflops"], 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"1 of 8 sequences x 1 of 32 layers (512-token chunk at offset {PF_CTX - PF_CHUNK}), "
                         f"torch-CPU port of append + causal GQA attention, {threads} threads"}
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    if peaks_path.exists():
        pk = json.loads(peaks_path.read_text())
        peak, peak_kind = float(pk["bf16_tflops_sustained"]), "measured (sustained bf16 GEMM)"
    else:
        peak, peak_kind = 1400.0, "fallback (sustained)"
    achieved = flops_layer / (pf_ms / 1e3) / 1e12
    line = {
        "metric": PF_METRIC, "value": round(flops_layer * nl / (ms / 1e3) / 1e12, 2),
        "unit": "TFLOP/s", "n_gpus": 1, "steps": steps, "warmup": warm,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 K/V/Q, random block tables)",
        "config": {"workload": ("chunked-prefill iteration: 32 layers, 32 q heads, 8 kv heads, "
                                f"head_dim 128, block 16; 8 seqs x 512-token chunk at offset "
                                f"{PF_CTX - PF_CHUNK} (ctx {PF_CTX}); per layer kv_append + paged_prefill"
                                + ("" if kv_bits == 16 else
                                   f"; {kv_bits}-bit store: kv_quant_append, kv_dequant_blocks "
                                   "of the step's blocks into a bf16 staging pool, paged_prefill "
                                   "on it")),
                   "kv_bits": kv_bits,
                   "layers": nl, "global_batch": PF_B, "seq_len": PF_CTX, "chunk": PF_CHUNK,
                   "pool_blocks": n_blocks,
                   "l2": "per layer 134 MB of K/V read > 126 MB L2; layers use distinct pools"},
        "prefill_tok_s": round(T / (ms / 1e3), 1),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "traffic": profile_traffic("paged_prefill_8b.md"),
                     "kernel": ("paged_prefill_tc_kernel<128,bf16>"
                                if os.environ.get("MLXZ_B200_PREFILL_PERSIST", "") == "0"
                                else "paged_prefill_ps_kernel<128,bf16>"), "peak_kind": peak_kind,
                     "prefill_ms_mean": round(pf_ms, 4), "alg_flops_per_launch": flops_layer,
                     "dequant_ms_mean": None if dq_ms is None else round(dq_ms, 4)},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": steps * nl * (2 if kv_bits == 16 else 3),
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Decode workloads (shared by both arms)
# ---------------------------------------------------------------------------

def c5_ctx(seed: int, n: int):
    """70B sharded workload: lognormal context lengths, median 4096, sigma 1,
    clipped to [256, 32768] (seeded)."""
    import numpy as np

    z = np.random.default_rng(seed).standard_normal(n)
    c = np.exp(np.log(C5_MEDIAN) + C5_SIGMA * z)
    return np.clip(np.rint(c), C5_LO, C5_HI).astype(np.int64)


class Workload:
    """Shapes of a decode workload at world size `world` (host side only).

    decode (c5 False): 8B shape, 64 sequences per GPU (weak scaling), `layers`
    model layers, all resident.  sharded70b (c5 True): 70B shape, 256
    sequences in total split by KV head across the ranks (strong scaling);
    the layers whose pools fit in `resident_gb` per GPU are resident and
    timed (`layers` caps them), and the 80-layer step time is the per-layer
    time x 80."""

    def __init__(self, c5: bool, world: int, layers: int | None, resident_gb: float, seed: int,
                 p2p: bool):
        self.c5, self.world, self.p2p = c5, world, p2p
        self.hq_all = C5_HQ if c5 else HQ
        self.hkv = HKV // world
        self.hq = self.hq_all // world
        if c5:
            self.B = C5_B
            self.ctx = c5_ctx(seed, self.B)
            self.model_layers = C5_L
        else:
            self.B = B_PER_GPU * world
            self.ctx = workload_ctx(seed, self.B)
            self.model_layers = layers or L
        self.need = (self.ctx + 1 + BS - 1) // BS
        self.n_blocks = int(math.ceil(self.need.sum() * 1.1))
        layer_pool_bytes = self.n_blocks * self.hkv * BS * D * 2 * 2
        self.nl = self.model_layers
        if c5:
            fit = int(resident_gb * 1e9 // layer_pool_bytes)
            self.nl = max(1, min(layers or C5_L, C5_L, fit))
        # KV bytes one step reads: all heads, all ranks, every model layer
        self.kv_step_total = float((self.ctx + 1).sum()) * HKV * D * 2 * 2 * self.model_layers
        self.kv_layer_rank = float((self.ctx + 1).sum()) * self.hkv * D * 2 * 2
        self.decode_alg_bytes = (self.kv_layer_rank + 2.0 * self.B * self.hq * D * 2
                                 + float(self.need.sum()) * 4)

    @property
    def metric(self) -> str:
        return C5_METRIC if self.c5 else METRIC

    def config(self) -> dict:
        world, nl = self.world, self.nl
        if world == 1:
            par = "1 GPU"
        elif self.p2p:
            par = (f"kv-head sharding x{world}; all-gather fused into the decode launch "
                   f"(peer-memory stores over NVLink; each layer's launch waits for the peers' "
                   f"rows of the layer before it)")
        else:
            par = f"kv-head sharding x{world} + NCCL all-gather per layer"
        if self.c5:
            workload = (f"head-sharded paged decode step, Llama-3.1-70B KV shape: 80 layers "
                        f"({nl} resident and timed, step = per-layer time x 80), 64 q heads, "
                        f"8 kv heads ({self.hkv} per GPU), head_dim 128, block 16; {self.B} "
                        f"seqs, ctx lognormal(median {C5_MEDIAN}, sigma {C5_SIGMA}) clipped to "
                        f"[{C5_LO},{C5_HI}]; append 1 token + attention + all-gather per layer")
            seq_len = f"lognormal median {C5_MEDIAN} sigma {C5_SIGMA} in [{C5_LO},{C5_HI}]"
        else:
            workload = (f"paged decode step, Llama-3.1-8B KV shape: {nl} layers, 32 q heads, "
                        f"8 kv heads, head_dim 128, block 16; {B_PER_GPU} seqs per GPU, "
                        f"ctx U[{CTX_LO},{CTX_HI}]; append 1 token + attention per layer")
            seq_len = f"U[{CTX_LO},{CTX_HI}]"
        return {
            "workload": workload, "layers": self.model_layers, "layers_resident": nl,
            "global_batch": self.B, "seq_len": seq_len,
            "mean_ctx": round(float(self.ctx.mean()), 1), "parallelism": par,
            "l2": (f"KV read per layer {self.kv_layer_rank / 1e9:.2f} GB per GPU >> 126 MB L2"),
            "pool_blocks": self.n_blocks,
        }


def run_reference(args, rank: int, world: int) -> None:
    """The reference's CPU algorithm (oracle port) on this box's host cores,
    on the GPU arm's workload and config.  Each step is measured whole: every
    layer of the step over every sequence of rank 0's KV-head shard (the whole
    workload at N = 1; 1/N of it at N > 1, where the other ranks do nothing).
    One layer's pools are built and every layer pass reads them again (1.2 GB
    per pass from DRAM, far above the host caches), with its own q and new
    tokens."""
    if rank != 0:
        return
    if args.config == "prefill":
        run_reference_prefill(args, world)
        return
    import torch

    from oracle import cpu_path

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = Workload(False, world, args.layers, args.resident_gb, args.seed, args.gather == "p2p")
    hkv, hq, B, nl = w.hkv, w.hq, w.B, w.nl
    g = torch.Generator().manual_seed(args.seed)
    perm = torch.randperm(w.n_blocks, generator=g)
    tables, used = [], 0
    for n in w.need:
        tables.append(perm[used:used + int(n)])
        used += int(n)
    kp = torch.randn((w.n_blocks, hkv, BS, D), generator=g).to(torch.bfloat16)
    vp = torch.randn((w.n_blocks, hkv, BS, D), generator=g).to(torch.bfloat16)
    q = torch.randn((nl, B, hq, D), generator=g).to(torch.bfloat16).float()
    nk = torch.randn((nl, B, hkv, D), generator=g).to(torch.bfloat16)
    nv = torch.randn((nl, B, hkv, D), generator=g).to(torch.bfloat16)
    ctx_l = [int(c) for c in w.ctx]
    scale = D ** -0.5

    def step() -> float:
        t0 = time.perf_counter()
        for l in range(nl):
            cpu_path.decode_layer(q[l], kp, vp, tables, ctx_l, nk[l], nv[l], scale)
        return time.perf_counter() - t0

    times = [step() for _ in range(args.warmup + args.steps)][args.warmup:]
    ms = statistics.median(times) * 1e3
    step_bytes = w.kv_layer_rank * nl
    v = step_bytes / (ms / 1e3) / 1e9
    share = ("the whole workload" if world == 1 else
             f"rank 0's KV-head shard ({hkv} of 8 kv heads of all {B} sequences, 1/{world} "
             f"of the job; the other ranks idle)")
    sample = (f"every step measured whole: {nl} layers x {B} sequences, {share}; "
              f"torch-CPU port of get_kv + GQA attention, {threads} threads; one layer's pools "
              f"re-read by every layer pass ({w.kv_layer_rank / 1e9:.2f} GB per pass)")
    line = {
        "impl": "reference", "metric": w.metric, "value": round(v, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 K/V/Q, random block tables)",
        "config": w.config(),
        "decode_tok_s": round(B / (ms / 1e3), 3),
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU benchmark
# ---------------------------------------------------------------------------

def torch_fp32_attention(store, l: int, table: list[int], length: int, q, scale: float):
    """Plain-torch fp32 decode attention of one sequence over its first
    `length` pool tokens (the parity check inside the bench)."""
    import torch

    kp, vp = store.k_pool(l), store.v_pool(l)
    hkv, bs, Dh = kp.shape[1], kp.shape[2], kp.shape[3]
    idx = torch.tensor(table[: -(-length // bs)], dtype=torch.int64, device=kp.device)
    K = kp.index_select(0, idx).permute(1, 0, 2, 3).reshape(hkv, -1, Dh)[:, :length].float()
    V = vp.index_select(0, idx).permute(1, 0, 2, 3).reshape(hkv, -1, Dh)[:, :length].float()
    hq = q.shape[0]
    s = torch.bmm(q.float().view(hkv, hq // hkv, Dh), K.transpose(1, 2)) * scale
    return torch.bmm(torch.softmax(s, dim=-1), V).reshape(hq, Dh)


def attn_rel_err(out, ref, unit_roundoff: float) -> float:
    """max(|out - ref| - u |ref|, 0) / max |ref|: the error beyond the output
    type's own rounding, relative to the largest reference value."""
    d = ((out.float() - ref).abs() - unit_roundoff * ref.abs()).clamp_min(0)
    return float(d.max() / ref.abs().max())


def measure_decode(args, w: "Workload", rank: int, world: int, local_rank: int, steps: int,
                   warmup: int, e2e: bool, parity: bool) -> dict:
    """Build the workload's pools on this rank, time `steps` decode steps and
    return the rank-max timings (and the parity checks when asked)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from mlxz_b200 import ops
    from mlxz_b200.engine import PagedDecodeStep, PagedKVStore
    from mlxz_b200.engine.decode_step import _copy_groups
    from mlxz_b200.engine.sharding import HeadAllGather, HeadShard, PeerAllGather

    dev = torch.device("cuda", local_rank)
    shard = HeadShard(rank, world, HKV, w.hq_all)
    hkv, hq, B, nl, D_ = w.hkv, w.hq, w.B, w.nl, D
    perm = np.random.default_rng(args.seed + 1).permutation(w.n_blocks)
    torch.manual_seed(args.seed * 1000 + rank)
    store = PagedKVStore(nl, w.n_blocks, hkv, D_, BS, torch.bfloat16, dev, init="empty")
    for l in range(nl):
        store.pools[l].normal_()
    used, ids = 0, []
    for b in range(B):
        sid = f"s{b}"
        store.add_sequence(sid, int(w.ctx[b]),
                           blocks=[int(x) for x in perm[used:used + w.need[b]]])
        used += int(w.need[b])
        ids.append(sid)
    step = PagedDecodeStep(store, ids, hq, batch_invariant=args.batch_invariant)
    q = torch.randn(nl, B, hq, D_, device=dev).to(torch.bfloat16)
    kn = torch.randn(nl, B, hkv, D_, device=dev).to(torch.bfloat16)
    vn = torch.randn(nl, B, hkv, D_, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    p2p = world > 1 and w.p2p
    gat = HeadAllGather(shard, B, D_, torch.bfloat16, dev)
    # two sets of slots, alternated per step in the end-to-end loop (whose
    # outputs are read back while the next step runs)
    peer = PeerAllGather(shard, B, D_, torch.bfloat16, dev, n_slots=2 * nl) if p2p else None
    full = None
    if world > 1 and not p2p:
        full = torch.empty((nl, B, w.hq_all, D_), dtype=torch.bfloat16, device=dev)

    # p2p slots: two sets of nl, alternated per step (all step loops share the
    # round counter), so no slot is reused while its readers may still run
    rounds = [0]

    def one_step(ev=None):
        # p2p: layer l's launch waits (in its prologue) for the peers' rows of
        # layer l - 1; the last layer is followed by a wait launch
        base = nl * (rounds[0] % 2)
        rounds[0] += 1
        for l in range(nl):
            st = step.store
            if args.separate_append:
                ops.kv_append_paged(st.k_pool(l), st.v_pool(l), kn[l], vn[l], step.tables,
                                    step.positions)
            if ev is not None:
                ev[l][0].record()
            if args.separate_append:
                ops.paged_decode(q[l], st.k_pool(l), st.v_pool(l), step.tables, step.lengths,
                                 scale=step.scale, out=out[l], workspace=step.workspace,
                                 num_warps=args.num_warps)
            elif p2p:
                peer.launch(step, l, q[l], kn[l], vn[l], slot=base + l,
                            num_warps=args.num_warps, wait_previous=l > 0)
            else:
                step.layer(l, q[l], kn[l], vn[l], out[l], num_warps=args.num_warps)
            if ev is not None:
                ev[l][1].record()
            if world > 1 and not p2p:
                gat.full(out[l], out=full[l])
        if p2p:
            peer.wait()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(warmup):
        one_step()
    torch.cuda.synchronize()
    ops.check_device_errors(local_rank)

    res = {}
    if parity:
        # (1) at N > 1: the fused gather's output of layer 0, bytewise, against
        # the ordinary launch + NCCL all-gather on the same inputs (every step
        # rewrites the same new tokens, so the pools are the same for both);
        # (2) one sequence per rank against a plain-torch fp32 recomputation
        res_p = {}
        if world > 1:
            if p2p:
                slot0 = nl * (rounds[0] % 2)
                rounds[0] += 1
                peer.launch(step, 0, q[0], kn[0], vn[0], slot=slot0, num_warps=args.num_warps)
                peer.wait()
                full0 = peer.full[slot0]
            else:
                full0 = full[0]
            want = torch.empty((B, w.hq_all, D_), dtype=torch.bfloat16, device=dev)
            local = torch.empty((B, hq, D_), dtype=torch.bfloat16, device=dev)
            step.layer(0, q[0], kn[0], vn[0], local, num_warps=args.num_warps)
            gat.full(local, out=want)
            torch.cuda.synchronize()
            same = torch.equal(full0, want)
            t = torch.tensor([0 if same else 1], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            res_p["fused_vs_nccl_bytewise"] = bool(t.item() == 0) if p2p else None
            got_rows = full0
        else:
            got_rows = out[0]
        ops.check_device_errors(local_rank)
        b = (rank * 37) % B
        table = store.tables[ids[b]]
        ref = torch_fp32_attention(store, 0, table, int(w.ctx[b]) + 1, q[0, b], step.scale)
        got = got_rows[b, rank * hq:(rank + 1) * hq]
        err = attn_rel_err(got, ref, 2.0 ** -8)
        t = torch.tensor([err], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res_p["torch_fp32_max_rel_err"] = float(t.item())
        res_p["tolerance"] = 2e-3
        res_p["sequences_checked"] = f"one per rank (seq (37 r) mod {B}), layer 0"
        res_p["ok"] = (res_p["torch_fp32_max_rel_err"] <= 2e-3
                       and res_p.get("fused_vs_nccl_bytewise", True) is not False)
        res["parity"] = res_p

    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    # The timed region carries events only around the whole run: an event
    # between two launches would stop a layer's launch from starting while the
    # previous layer's drains (MZ_LAUNCH_OVERLAP_PREVIOUS).  The decode kernel's
    # average launch duration is the timed region over its launches (the step
    # is nothing else at N = 1; at N > 1 it includes each layer's gather).
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(uuid, enabled=not args.no_clocks)
    t0.record()
    for _ in range(steps):
        one_step()
    t1.record()
    torch.cuda.synchronize()
    barrier()
    res["clocks"] = clocks.stop()
    ms = t0.elapsed_time(t1) / steps
    dec_mean = ms / nl
    # each decode launch timed on its own (events between launches), two steps
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(nl)]
           for _ in range(2)]
    for k in range(2):
        one_step(evs[k])
    torch.cuda.synchronize()
    iso = [evs[k][l][0].elapsed_time(evs[k][l][1]) for k in range(2) for l in range(nl)]
    dec_iso = sum(iso) / len(iso)
    barrier()
    ops.check_device_errors(local_rank)

    e2e_ms, h2d, d2h = float('nan'), 0, 0
    if e2e:
        # End to end through the public step API: this rank's inputs from
        # pinned host memory; back to the host, this rank's heads of the
        # gathered [B, Hq, D] output (the ranks' parts together are the whole
        # output once).  Bytes are whole-job totals.
        qh = q.cpu().pin_memory()
        kh = kn.cpu().pin_memory()
        vh = vn.cpu().pin_memory()
        qlo, qhi = shard.q_range
        oh = torch.empty((nl, B, hq, D_), dtype=torch.bfloat16).pin_memory()
        h2d = (qh.numel() * 2 + kh.numel() * 2 + vh.numel() * 2) * world
        d2h = oh.numel() * 2 * world
        groups = _copy_groups(nl)
        first = {a for a, _ in groups}
        last = {b - 1 for _, b in groups}

        def gather_layer(l, ql, kl, vl, ol):
            if p2p:
                # chained inside a copy group; the group's last layer is waited
                # for, so the group's outputs are complete when it is copied back
                slot = l + nl * (rounds[0] % 2)
                peer.launch(step, l, ql, kl, vl, slot=slot, num_warps=args.num_warps,
                            wait_previous=l not in first)
                if l in last:
                    peer.wait()
                g = peer.full[slot]
            else:
                step.layer(l, ql, kl, vl, ol)
                g = gat.full(ol, out=full[l])
            return g[:, qlo:qhi]

        def e2e_step():
            step.step_host(qh, kh, vh, oh, layer_fn=None if world == 1 else gather_layer)
            rounds[0] += 1

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        barrier()
        ops.check_device_errors(local_rank)
        e2e_ms = e0.elapsed_time(e1) / steps

    if world > 1:
        t = torch.tensor([ms, e2e_ms, dec_mean, dec_iso], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, dec_mean, dec_iso = (float(x) for x in t.tolist())
    if peer is not None:
        peer.close()
    per_layer_ms = ms / nl
    res.update(ms=ms, e2e_ms=e2e_ms, dec_mean=dec_mean, dec_iso=dec_iso, h2d=h2d, d2h=d2h,
               step_ms=per_layer_ms * w.model_layers,
               e2e_step_ms=e2e_ms / nl * w.model_layers,
               launches=steps * nl * (2 if args.separate_append else 1) + (steps if p2p else 0))
    return res


def run_gpu(args, rank: int, world: int, local_rank: int) -> None:
    """The paged decode step on this rank's KV-head shard.

    decode (default): 8B shape, 64 sequences per GPU (weak scaling), followed
    by a `sharded70b` sub-record measured in the same run (unless
    --no-sub-records).  sharded70b: the 70B-shape line alone."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    c5 = args.config == "sharded70b"
    p2p = args.gather == "p2p"
    w = Workload(c5, world, args.layers, args.resident_gb, args.seed, p2p)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    warm = max(3, args.warmup)
    r = measure_decode(args, w, rank, world, local_rank, args.steps, warm,
                       e2e=not args.no_e2e, parity=True)
    torch.cuda.empty_cache()
    sub = None
    if not c5 and not args.no_sub_records:
        w5 = Workload(True, world, None, args.resident_gb, args.seed, p2p)
        r5 = measure_decode(args, w5, rank, world, local_rank, args.steps, warm, e2e=False,
                            parity=True)
        sub = {
            "metric": w5.metric, "value": round(w5.kv_step_total / (r5["step_ms"] / 1e3) / 1e9, 2),
            "unit": "GB/s", "scaling": "strong", "ms_per_step": round(r5["step_ms"], 4),
            "ms_per_layer": round(r5["ms"] / w5.nl, 5), "layers": w5.model_layers,
            "layers_resident": w5.nl, "steps": args.steps, "warmup": warm,
            "decode_tok_s": round(w5.B / (r5["step_ms"] / 1e3), 1),
            "config": w5.config(), "parity": r5.get("parity"),
            "roofline": {"bound": "hbm", "unit": "GB/s",
                         "achieved": round(w5.decode_alg_bytes / (r5["dec_mean"] / 1e3) / 1e9, 1),
                         "decode_ms_mean": round(r5["dec_mean"], 4),
                         "alg_bytes_per_launch": w5.decode_alg_bytes},
            "gpu_launches": r5["launches"], "clocks": r5["clocks"],
        }
    extra = {}
    if world == 1 and not c5 and not args.no_sub_records:
        # the single-GPU workloads of the other configs, measured in the same
        # run: prefix-cache restore / copy-on-write / host-tier eviction (C3)
        # and the quantised decode step at 8 and 4 bits (C4)
        extra["prefix"] = run_prefix(args, local_rank)
        torch.cuda.empty_cache()
        extra["quant8"] = run_quant(args, local_rank, bits=8)
        extra["quant4"] = run_quant(args, local_rank, bits=4)
    if rank == 0:
        peak, peak_kind = peaks()
        cpu = None
        if world == 1 and not args.no_cpu_baseline and not c5:
            threads = os.cpu_count() or 1
            s = cpu_sample(args.seed, args.cpu_seconds, threads)
            cpu = {"value": round(s["gbs"], 3), "unit": "GB/s", "cores": threads, "kind": "port",
                   "sample": (f"1 layer x {s['n_seqs']} sequences of the same ctx distribution, "
                              f"{s['reps']} reps (median), torch-CPU port of get_kv + GQA attention")}
        value = w.kv_step_total / (r["step_ms"] / 1e3) / 1e9
        achieved = w.decode_alg_bytes / (r["dec_mean"] / 1e3) / 1e9
        if sub is not None:
            sub["roofline"].update(peak=peak, peak_kind=peak_kind,
                                   frac=round(sub["roofline"]["achieved"] / peak, 4))
        result = {
            "metric": w.metric, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": warm, "ms_per_step": round(r["step_ms"], 4),
            "higher_is_better": True, "scaling": "strong" if c5 else "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16 K/V/Q, random block tables)",
            "config": w.config(),
            "decode_tok_s": round(w.B / (r["step_ms"] / 1e3), 1),
            "hbm_frac": round(value / world / peak, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": profile_traffic("paged_decode_c2.md") if not c5 else None,
                         "kernel": "paged_decode_kernel<128,bf16> (fused append + decode"
                                   + (" + peer all-gather)" if world > 1 and p2p else ")"),
                         "peak_kind": peak_kind,
                         "decode_ms_mean": round(r["dec_mean"], 4),
                         "decode_ms_timing": ("timed region / launches" if world == 1 else
                                              "timed region / launches (includes the gather)"),
                         "decode_ms_isolated": round(r["dec_iso"], 4),
                         "alg_bytes_per_launch": w.decode_alg_bytes},
            "cpu_baseline": cpu,
            "e2e": None if args.no_e2e else {
                "value": round(w.kv_step_total / (r["e2e_step_ms"] / 1e3) / 1e9, 2),
                "unit": "GB/s", "ms_per_step": round(r["e2e_step_ms"], 4),
                "h2d_bytes_per_step": int(r["h2d"]), "d2h_bytes_per_step": int(r["d2h"])},
            "gpu_launches": r["launches"],
            "clocks": r["clocks"],
            "parity": r.get("parity"),
        }
        if sub is not None:
            result["sharded70b"] = sub
        result.update(extra)
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_prefix(args, local_rank: int) -> dict:
    """Prefix-cache workload, 8B KV shape (32 layers, 8 KV heads, head_dim 128,
    bf16, block 16): a 2048-token shared prefix cached once; 32 requests
    restore it (zero-copy) and write a U[64, 512]-token suffix; each request's
    full prompt is cached; then the least recently used 25 % of the pool's
    blocks go to the pinned host tier and are reloaded.  Copy-on-write is
    timed as the reference's full-hit path triggers it (re-running the last
    prompt token writes into the shared last prefix block), and as a bulk
    block copy of 25 % of the pool."""
    import numpy as np
    import torch

    from mlxz_b200 import ops
    from mlxz_b200.engine import PagedKVStore
    from mlxz_b200.prefix_cache import PagedPrefixCache, PinnedHostTier, RollingPrefixHasher

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    nl, prefix, n_req = args.layers, 2048, 32
    g = np.random.default_rng(args.seed)
    suffix = g.integers(64, 513, size=n_req)
    need = prefix // BS + int(sum((int(x) + BS - 1) // BS for x in suffix))
    n_blocks = int(math.ceil(need * 1.1))
    store = PagedKVStore(nl, n_blocks, HKV, D, BS, torch.bfloat16, dev, init="zeros")
    bb_all = 2 * nl * store.block_bytes  # one block across every layer's K and V
    tier = PinnedHostTier(n_blocks, 2 * nl, store.block_bytes, dev)
    cache = PagedPrefixCache(store, memory_budget_bytes=1 << 40, host_tier=tier)
    hasher = RollingPrefixHasher(BS)
    torch.manual_seed(args.seed)

    def kv(n):
        return (torch.randn(nl, HKV, n, D, device=dev).to(torch.bfloat16),
                torch.randn(nl, HKV, n, D, device=dev).to(torch.bfloat16))

    prompt0 = list(range(prefix))
    store.add_sequence("p", 0)
    store.append_tokens("p", *kv(prefix))
    cache.store_sync(hasher.hash_chunks(prompt0), "p", block_size=BS)
    store.free_sequence("p")
    torch.cuda.synchronize()

    # restore + suffix write per request
    restore_s, write_s, cow_blocks = [], [], 0
    suffix_kv = [kv(int(n)) for n in suffix]
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    for r in range(n_req):
        prompt = prompt0 + [100000 + 1000 * r + i for i in range(int(suffix[r]))]
        hashes = hasher.hash_chunks(prompt)
        t0 = time.perf_counter()
        n, state, _ = cache.lookup_sync(hashes)
        cache.restore(f"r{r}", state)
        restore_s.append(time.perf_counter() - t0)
        store.append_tokens(f"r{r}", *suffix_kv[r])
        cache.store_sync(hashes, f"r{r}", block_size=BS)
    ev[1].record()
    torch.cuda.synchronize()
    write_ms = ev[0].elapsed_time(ev[1])
    suffix_bytes = float(suffix.sum()) * 2 * nl * HKV * D * 2

    # copy-on-write as the full-hit path triggers it: each of the 32 requests
    # re-runs the last prefix token, writing into the shared block 127
    pairs = []
    for r in range(n_req):
        store.add_sequence(f"h{r}", 0)
        n, state, _ = cache.lookup_sync(hasher.hash_chunks(prompt0))
        cache.restore(f"h{r}", state)
        store.offsets[f"h{r}"] = prefix - 1
        pairs.append(store.make_writable(f"h{r}", prefix - 1))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    store.copy_blocks(pairs)
    e1.record()
    torch.cuda.synchronize()
    cow_ms = e0.elapsed_time(e1)
    cow_blocks = len(pairs)
    for r in range(n_req):
        store.free_sequence(f"h{r}")

    # bulk block copy of 25 % of the pool (HBM roofline of mz_block_copy)
    nb_bulk = max(1, n_blocks // 4)
    free_now = store.bm.free_blocks
    nb_bulk = min(nb_bulk, free_now // 2)
    srcs = store.bm.allocate(nb_bulk)
    dsts = store.bm.allocate(nb_bulk)
    src_t = torch.tensor(srcs, dtype=torch.int32, device=dev)
    dst_t = torch.tensor(dsts, dtype=torch.int32, device=dev)
    for _ in range(3):
        ops.block_copy(store.pool_stack(), src_t, dst_t)
    reps = 20
    e0.record()
    for _ in range(reps):
        ops.block_copy(store.pool_stack(), src_t, dst_t)
    e1.record()
    torch.cuda.synchronize()
    bulk_ms = e0.elapsed_time(e1) / reps
    store.bm.free(srcs + dsts)
    peak, peak_kind = peaks()
    bulk_gbs = 2.0 * nb_bulk * bb_all / (bulk_ms / 1e3) / 1e9

    # host link peaks (pinned, 1 GiB each way)
    big_h = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
    big_d = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    big_d.copy_(big_h, non_blocking=True)
    torch.cuda.synchronize()
    e0.record()
    big_d.copy_(big_h, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    h2d_peak = (1 << 30) / (e0.elapsed_time(e1) / 1e3) / 1e9
    e0.record()
    big_h.copy_(big_d, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    d2h_peak = (1 << 30) / (e0.elapsed_time(e1) / 1e3) / 1e9
    del big_h, big_d

    # LRU eviction of 25 % of the pool to the host tier, then reload
    for r in range(n_req):
        store.free_sequence(f"r{r}")
    n_evict = n_blocks // 4
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    moved = cache.evict_to_host(n_evict)
    tier.sync()
    evict_s = time.perf_counter() - t0
    lookups = [hasher.hash_chunks(prompt0 + [100000 + 1000 * r + i for i in range(int(suffix[r]))])
               for r in range(n_req)]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    reloaded = 0
    for r in range(n_req):
        n, state, _ = cache.lookup_sync(lookups[r])
        reloaded += cache.reload(state)
    tier.sync()
    reload_s = time.perf_counter() - t0
    ops.check_device_errors(local_rank)
    line = {
        "metric": "prefix-cache restore + copy-on-write + host-tier evict/reload, 8B KV shape",
        "value": round(moved * bb_all / evict_s / 1e9, 3), "unit": "GB/s (evict to pinned host)",
        "higher_is_better": True, "n_gpus": 1, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 K/V)",
        "config": {"workload": (f"prefix cache: {prefix}-token shared prefix, {n_req} requests, "
                                f"suffix U[64,512]; {nl} layers, 8 kv heads, head_dim 128, "
                                f"block 16"), "layers": nl, "pool_blocks": n_blocks,
                   "block_bytes_all_layers": bb_all},
        "restore_us_per_request": round(1e6 * statistics.median(restore_s), 1),
        "restore_blocks_per_request": prefix // BS,
        "suffix_write_gbs": round(suffix_bytes / (write_ms / 1e3) / 1e9, 2),
        "cow_full_hit": {"blocks": cow_blocks, "ms": round(cow_ms, 4),
                         "gbs": round(2.0 * cow_blocks * bb_all / (cow_ms / 1e3) / 1e9, 1)},
        "block_copy_bulk": {"blocks": nb_bulk, "ms": round(bulk_ms, 4), "gbs": round(bulk_gbs, 1),
                            "roofline_frac": round(bulk_gbs / peak, 4), "peak": peak,
                            "peak_kind": peak_kind},
        "evict": {"blocks": moved, "bytes": moved * bb_all, "s": round(evict_s, 5),
                  "gbs": round(moved * bb_all / evict_s / 1e9, 2),
                  "frac_of_d2h_peak": round(moved * bb_all / evict_s / 1e9 / d2h_peak, 3)},
        "reload": {"blocks": reloaded, "bytes": reloaded * bb_all, "s": round(reload_s, 5),
                   "gbs": round(reloaded * bb_all / reload_s / 1e9, 2),
                   "frac_of_h2d_peak": round(reloaded * bb_all / reload_s / 1e9 / h2d_peak, 3)},
        "host_link": {"h2d_gbs": round(h2d_peak, 2), "d2h_gbs": round(d2h_peak, 2)},
        "stats": cache.stats().__repr__(),
    }
    return line


def run_quant(args, local_rank: int, bits: int | None = None) -> dict:
    """Quantised KV decode step, Llama-3.1-8B shape: 32 layers, 32 q heads, 8 KV
    heads, head_dim 128, batch 32, ctx ~ U[4096, 16384], affine group-64
    codes at `--bits`, fp16 scales and biases.  Pools are filled by quantising
    seeded N(0,1) bf16 K/V with mz_kv_quant_append.  One step = per layer, the
    quantise-on-append of one new token per sequence then attention with the
    dequantisation fused in."""
    import numpy as np
    import torch

    from mlxz_b200 import ops
    from mlxz_b200.engine import QuantizedPagedDecodeStep, QuantizedPagedKVStore

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    nl, B = args.layers, 32
    bits = args.bits if bits is None else bits
    ctx = np.random.default_rng(args.seed).integers(4096, 16385, size=B).astype(np.int64)
    need = (ctx + 1 + BS - 1) // BS
    n_blocks = int(math.ceil(need.sum() * 1.1))
    perm = np.random.default_rng(args.seed + 1).permutation(n_blocks)
    store = QuantizedPagedKVStore(nl, n_blocks, HKV, D, BS, bits=bits, device=dev, init="empty")
    ids, used = [], 0
    for b in range(B):
        store.add_sequence(f"s{b}", int(ctx[b]), blocks=[int(x) for x in perm[used:used + need[b]]])
        used += int(need[b])
        ids.append(f"s{b}")
    # fill every block slot with quantised N(0,1) data, 8192 slots at a time
    torch.manual_seed(args.seed)
    all_slots = torch.arange(n_blocks * BS, dtype=torch.int64, device=dev)
    for l in range(nl):
        for lo in range(0, n_blocks * BS, 8192):
            sl = all_slots[lo:lo + 8192]
            k = torch.randn(1, HKV, sl.numel(), D, device=dev).to(torch.bfloat16)
            v = torch.randn(1, HKV, sl.numel(), D, device=dev).to(torch.bfloat16)
            ops.kv_quant_append(store.qpools(l), k, v, sl)
    step = QuantizedPagedDecodeStep(store, ids, HQ)
    q = torch.randn(nl, B, HQ, D, device=dev).to(torch.bfloat16)
    kn = torch.randn(nl, B, HKV, D, device=dev).to(torch.bfloat16)
    vn = torch.randn(nl, B, HKV, D, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    per_tok_layer = 2 * HKV * (D * bits // 8 + 2 * 2 * (D // 64))  # codes + scales + biases
    kv_layer = float((ctx + 1).sum()) * per_tok_layer
    alg = kv_layer + 2.0 * B * HQ * D * 2 + float(need.sum()) * 4
    torch.cuda.synchronize()

    def one_step(ev=None):
        for l in range(nl):
            pools = store.qpools(l)
            ops.kv_quant_append_paged(pools, kn[l], vn[l], step.tables, step.positions)
            if ev is not None:
                ev[l][0].record()
            ops.paged_decode_q(q[l], pools, step.tables, step.lengths, scale=step.scale,
                               out=out[l], workspace=step.workspace, num_warps=args.num_warps)
            if ev is not None:
                ev[l][1].record()

    for _ in range(max(3, args.warmup)):
        one_step()
    torch.cuda.synchronize()
    ops.check_device_errors(local_rank)
    steps = args.steps
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(nl)]
           for _ in range(steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid, enabled=not args.no_clocks)
    t0.record()
    for k in range(steps):
        one_step(evs[k])
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ops.check_device_errors(local_rank)
    ms = t0.elapsed_time(t1) / steps
    dec = [evs[k][l][0].elapsed_time(evs[k][l][1]) for k in range(steps) for l in range(nl)]
    dec_ms = sum(dec) / len(dec)
    peak, peak_kind = peaks()
    value = kv_layer * nl / (ms / 1e3) / 1e9
    # the form mz_paged_decode_q dispatches to for this shape (head_dim 128,
    # 4 query rows per KV head): the mma.sync kernel, unless
    # MLXZ_B200_QDECODE_TC=1 selects the tcgen05 form
    use_tc = os.environ.get("MLXZ_B200_QDECODE_TC", "") == "1"
    qkernel = f"paged_decode_qtc_kernel<{bits},4>" if use_tc else f"paged_decode_q_kernel<128,{bits},1>"
    qprof = f"paged_decode_qtc{bits}_c4.md" if use_tc else f"paged_decode_q{bits}_c4.md"
    line = {
        "metric": f"quantised ({bits}-bit) paged-decode KV-read GB/s and decode tok/s, 8B shape, batch 32",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": 1, "steps": steps,
        "warmup": max(3, args.warmup), "ms_per_step": round(ms, 4), "higher_is_better": True,
        "dtype": f"u{bits} codes + fp16 scale/bias, bf16 q",
        "data": "synthetic (seeded N(0,1) bf16 K/V quantised on the GPU, random block tables)",
        "config": {"workload": (f"quantised decode step: {nl} layers, 32 q heads, 8 kv heads, "
                                f"head_dim 128, block 16, group 64, {bits}-bit; 32 seqs, "
                                f"ctx U[4096,16384]"), "layers": nl, "global_batch": B,
                   "mean_ctx": round(float(ctx.mean()), 1), "pool_blocks": n_blocks,
                   "kv_bytes_per_token_layer": per_tok_layer,
                   "bf16_equivalent_step_bytes": float((ctx + 1).sum()) * 2 * HKV * D * 2 * nl},
        "decode_tok_s": round(B / (ms / 1e3), 1),
        "roofline": {"bound": "hbm", "achieved": round(alg / (dec_ms / 1e3) / 1e9, 1),
                     "peak": peak, "unit": "GB/s",
                     "frac": round(alg / (dec_ms / 1e3) / 1e9 / peak, 4),
                     "traffic": profile_traffic(qprof), "kernel": qkernel, "peak_kind": peak_kind,
                     "decode_ms_mean": round(dec_ms, 4), "alg_bytes_per_launch": alg},
        "gpu_launches": steps * nl * 2,
        "clocks": clk,
    }
    del store, step, q, kn, vn, out
    torch.cuda.empty_cache()
    return line


def run_kernels(args, local_rank: int) -> dict:
    """Each data-movement kernel of the path timed alone (CUDA events around
    `--steps` launches after `--warmup`), 8B KV shape (8 KV heads, head_dim
    128, bf16, block 16), against its algorithmic bytes:
      append_slots   mz_kv_append: 8192 prompt tokens to random slots
      append_paged   mz_kv_append_paged: one token for each of 64 sequences
      gather         mz_kv_gather: 16 sequences x 8192 tokens to contiguous KV
      block_copy     mz_block_copy: 2048 blocks x 2 --layers pools (K and V)
      block_pack     mz_block_pack: 2048 blocks into a staging buffer
      block_unpack   mz_block_unpack: the staging buffer back into the pools
      quant_append8/4  mz_kv_quant_append: 8192 tokens, 8 / 4 bits
      dequant8/4     mz_kv_dequant_blocks: 4096 blocks to bf16
    Inputs are far above L2 (126 MB) except the two appends, whose sizes are
    what the decode and prefill steps write."""
    import numpy as np
    import torch

    from mlxz_b200 import ops

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    torch.manual_seed(args.seed)
    H, Dh, bs = HKV, D, BS
    reps, warm = max(1, args.steps), max(1, args.warmup)
    peak, peak_kind = peaks()
    res = {}

    def timed(name, fn, alg_bytes):
        for _ in range(warm):
            fn()
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        z.record()
        torch.cuda.synchronize()
        ops.check_device_errors(local_rank)
        ms = a.elapsed_time(z) / reps
        gbs = alg_bytes / (ms / 1e3) / 1e9
        res[name] = {"ms": round(ms, 5), "alg_bytes": int(alg_bytes), "gbs": round(gbs, 1),
                     "frac": round(gbs / peak, 4)}

    row = H * Dh * 2  # bytes of one token's K (or V) in one layer
    # appends
    n_blocks = 4096
    kp = torch.randn(n_blocks, H, bs, Dh, device=dev).to(torch.bfloat16)
    vp = torch.randn_like(kp)
    n = 8192
    k = torch.randn(1, H, n, Dh, device=dev).to(torch.bfloat16)
    v = torch.randn_like(k)
    slots = torch.randperm(n_blocks * bs, device=dev)[:n].to(torch.int64)
    timed("append_slots", lambda: ops.kv_append(kp, vp, k, v, slots), 2 * 2 * n * row)
    B = 64
    perm = torch.randperm(n_blocks, device=dev).to(torch.int32)
    tables = perm[: B * 32].view(B, 32).contiguous()
    pos = torch.randint(0, 32 * bs, (B,), device=dev, dtype=torch.int32)
    kb = torch.randn(B, H, Dh, device=dev).to(torch.bfloat16)
    vb = torch.randn_like(kb)
    timed("append_paged", lambda: ops.kv_append_paged(kp, vp, kb, vb, tables, pos), 2 * 2 * B * row)
    # gather: 16 sequences x 8192 tokens
    nb_seq, G16 = 512, 16
    gk = torch.randn(G16 * nb_seq + 8, H, bs, Dh, device=dev).to(torch.bfloat16)
    gv = torch.randn_like(gk)
    gt = torch.randperm(G16 * nb_seq, device=dev).to(torch.int32).view(G16, nb_seq).contiguous()
    gl = [nb_seq * bs] * G16
    gld = torch.tensor(gl, dtype=torch.int32, device=dev)
    timed("gather", lambda: ops.kv_gather(gk, gv, gt, gld, gl), 2 * 2 * sum(gl) * row)
    del kp, vp, k, v, gk, gv
    torch.cuda.empty_cache()
    # block moves over the pools of `--layers` layers (K and V of each)
    P, NB = 2 * args.layers, 4608
    pools = torch.empty((P, NB, H, bs, Dh), dtype=torch.bfloat16, device=dev)
    pools.view(torch.int16).random_(-30000, 30000)
    nmove = 2048
    ids = torch.randperm(NB, device=dev).to(torch.int32)
    src, dst = ids[:nmove].contiguous(), ids[nmove:2 * nmove].contiguous()
    bb = H * bs * Dh * 2
    timed("block_copy", lambda: ops.block_copy(pools, src, dst), 2 * nmove * P * bb)
    staging = torch.empty((nmove, P, bb), dtype=torch.uint8, device=dev)
    timed("block_pack", lambda: ops.block_pack(pools, src, staging), 2 * nmove * P * bb)
    timed("block_unpack", lambda: ops.block_unpack(pools, dst, staging), 2 * nmove * P * bb)
    del pools, staging
    torch.cuda.empty_cache()
    # quantised appends and dequantisation
    for bits in (8, 4):
        NQ = 8192
        w = Dh * bits // 32
        qp = (torch.zeros(NQ, H, bs, w, dtype=torch.int32, device=dev),
              torch.zeros(NQ, H, bs, 2, dtype=torch.float16, device=dev),
              torch.zeros(NQ, H, bs, 2, dtype=torch.float16, device=dev),
              torch.zeros(NQ, H, bs, w, dtype=torch.int32, device=dev),
              torch.zeros(NQ, H, bs, 2, dtype=torch.float16, device=dev),
              torch.zeros(NQ, H, bs, 2, dtype=torch.float16, device=dev))
        k = torch.randn(1, H, n, Dh, device=dev).to(torch.bfloat16)
        v = torch.randn_like(k)
        sl = torch.randperm(NQ * bs, device=dev)[:n].to(torch.int64)
        qrow = H * (Dh * bits // 8 + 2 * 2 * 2)  # codes + scales + biases of one token's K
        timed(f"quant_append{bits}", lambda: ops.kv_quant_append(qp, k, v, sl),
              2 * n * row + 2 * n * qrow)
        ndq = 4096
        dids = torch.randperm(NQ, device=dev)[:ndq].to(torch.int32)
        ko = torch.empty(ndq, H, bs, Dh, dtype=torch.bfloat16, device=dev)
        vo = torch.empty_like(ko)
        timed(f"dequant{bits}", lambda: ops.kv_dequant_blocks(qp, dids, ko, vo),
              2 * ndq * bs * qrow + 2 * ndq * bs * row)
        del qp, k, v, ko, vo
        torch.cuda.empty_cache()
    return {"metric": "per-kernel achieved GB/s of the path's data-movement kernels, 8B KV shape",
            "unit": "GB/s", "steps": reps, "warmup": warm, "peak": peak, "peak_kind": peak_kind,
            "data": "synthetic (seeded N(0,1) bf16)", "kernels": res}



def run_peer_pair(args) -> dict:
    """The fused decode + all-gather launch (mz_paged_append_decode_allgather)
    of a 2-rank KV-head split of the 70B-shape workload (256 sequences,
    lognormal ctx; rank r holds KV heads [4r, 4r + 4) and q heads
    [32r, 32r + 32)), both ranks driven from one process: rank r on GPU r, its
    gathered buffer [B, 64, 128] on GPU r, the peer's buffer reached through
    peer access.  One model layer is resident per GPU.  Each step launches
    rank 0 on GPU 0 and rank 1 on GPU 1 (neither waits on the other inside a
    kernel), synchronises both devices, then runs each rank's bounded signal
    wait, which finds the peer's signal already set.  CUDA events on GPU 0
    time rank 0's launches.  Afterwards both gathered buffers must equal,
    bytewise, the two ranks' ordinary fused append + decode outputs side by
    side.  The printed line carries the launch time, its KV read rate and the
    bytes its rows put on NVLink (rows x head_dim x 2 B per pair, to one
    peer), which an ncu capture of GPU 0 (`--devices 0`) can set against the
    NVLink counters."""
    import ctypes

    import numpy as np
    import torch

    from mlxz_b200 import _native as nat
    from mlxz_b200 import ops

    if torch.cuda.device_count() < 2:
        return {"config": "peer_pair", "unavailable": "needs two visible GPUs"}
    if not (torch.cuda.can_device_access_peer(0, 1) and torch.cuda.can_device_access_peer(1, 0)):
        return {"config": "peer_pair", "unavailable": "GPUs 0 and 1 have no peer access"}
    from cuda.bindings import runtime as cudart

    for a, b in ((0, 1), (1, 0)):
        torch.cuda.set_device(a)
        torch.cuda.synchronize(a)
        cudart.cudaSetDevice(a)
        err = cudart.cudaDeviceEnablePeerAccess(b, 0)[0]
        if err not in (cudart.cudaError_t.cudaSuccess,
                       cudart.cudaError_t.cudaErrorPeerAccessAlreadyEnabled):
            return {"config": "peer_pair", "unavailable": f"cudaDeviceEnablePeerAccess: {err}"}
    w = Workload(True, 2, 1, 1e9, args.seed, True)
    N, B, hkv, hq, hq_all = 2, w.B, w.hkv, w.hq, w.hq_all
    gen = torch.Generator().manual_seed(args.seed)
    perm = torch.randperm(w.n_blocks, generator=gen).to(torch.int32)
    width = int(w.need.max())
    tables = torch.full((B, width), -1, dtype=torch.int32)
    pos = 0
    for b in range(B):
        n = int(w.need[b])
        tables[b, :n] = perm[pos:pos + n]
        pos += n
    lens = torch.from_numpy((w.ctx + 1).astype(np.int32))
    elem = 2
    block_bytes = hq * D * elem
    ranks = []
    for r in range(N):
        dev = torch.device("cuda", r)
        torch.cuda.set_device(r)
        g = torch.Generator(device=dev).manual_seed(args.seed * 7 + r)
        pool_shape = (w.n_blocks, hkv, BS, D)
        rk = {
            "dev": dev,
            "k": torch.randn(pool_shape, generator=g, device=dev, dtype=torch.bfloat16),
            "v": torch.randn(pool_shape, generator=g, device=dev, dtype=torch.bfloat16),
            "q": torch.randn((B, hq, D), generator=g, device=dev, dtype=torch.bfloat16),
            "kn": torch.randn((B, hkv, D), generator=g, device=dev, dtype=torch.bfloat16),
            "vn": torch.randn((B, hkv, D), generator=g, device=dev, dtype=torch.bfloat16),
            "tables": tables.to(dev), "lens": lens.to(dev),
            "full": torch.zeros((B, hq_all, D), device=dev, dtype=torch.bfloat16),
            "sig": torch.zeros(N, device=dev, dtype=torch.int32),
            "arrivals": torch.zeros(1, device=dev, dtype=torch.int32),
        }
        rk["ws"] = ops.decode_workspace(B, hkv, hq // hkv, D, r, 0, shared=False)
        ranks.append(rk)
    peers = []
    for r in range(N):
        pe = nat.PeerOutputs()
        pe.n_ranks, pe.rank = N, r
        for s2 in range(N):
            pe.out[s2] = ranks[s2]["full"].data_ptr() + r * block_bytes
            pe.signal[s2] = ranks[s2]["sig"].data_ptr()
        pe.arrivals = ranks[r]["arrivals"].data_ptr()
        peers.append(pe)
    epoch = 0

    def step(timed=None):
        nonlocal epoch
        epoch += 1
        for r in range(N):
            rk = ranks[r]
            peers[r].epoch = epoch
            with torch.cuda.device(r):
                if r == 0 and timed is not None:
                    timed[0].record()
                ops.paged_append_decode_allgather(
                    peers[r], rk["q"], rk["k"], rk["v"], rk["kn"], rk["vn"], rk["tables"],
                    rk["lens"], hq_all * D, D, torch.bfloat16, workspace=rk["ws"])
                if r == 0 and timed is not None:
                    timed[1].record()
        for r in range(N):
            torch.cuda.synchronize(r)
        for r in range(N):
            with torch.cuda.device(r):
                ops.peer_wait(ranks[r]["sig"], N, r, epoch)
        for r in range(N):
            torch.cuda.synchronize(r)
            ops.check_device_errors(r)

    for _ in range(max(1, args.warmup)):
        step()
    ms = []
    for _ in range(max(1, args.steps)):
        with torch.cuda.device(0):
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        step(ev)
        ms.append(ev[0].elapsed_time(ev[1]))
    # parity: each rank's ordinary fused launch, side by side, bytewise
    ok = True
    local = []
    for r in range(N):
        rk = ranks[r]
        with torch.cuda.device(r):
            local.append(ops.paged_append_decode(rk["q"], rk["k"], rk["v"], rk["kn"], rk["vn"],
                                                 rk["tables"], rk["lens"]).to("cuda:0"))
        torch.cuda.synchronize(r)
    want = torch.cat(local, dim=1)
    for r in range(N):
        got = ranks[r]["full"].to("cuda:0")
        ok = ok and bool(torch.equal(got.view(torch.int16), want.view(torch.int16)))
    dec_ms = statistics.median(ms)
    nvlink_bytes = B * hq * D * elem * (N - 1)
    peak, peak_kind = peaks()
    return {
        "config": "peer_pair",
        "workload": (f"rank 0 of a 2-GPU KV-head split of the 70B KV shape: {B} seqs, ctx "
                     f"lognormal(median {C5_MEDIAN}, sigma {C5_SIGMA}) in [{C5_LO},{C5_HI}], "
                     f"{hkv} kv heads and {hq} q heads per GPU, head_dim {D}, block {BS}, bf16; "
                     "one process driving GPUs 0 and 1"),
        "kernel": "paged_decode_gather_kernel<128,bf16> (mz_paged_append_decode_allgather)",
        "steps": len(ms), "launch_ms_median": round(dec_ms, 4),
        "kv_read_gbs": round(w.decode_alg_bytes / (dec_ms / 1e3) / 1e9, 1),
        "hbm_frac": round(w.decode_alg_bytes / (dec_ms / 1e3) / 1e9 / peak, 4),
        "peak": peak, "peak_kind": peak_kind,
        "alg_bytes_per_launch": w.decode_alg_bytes,
        "nvlink_store_bytes_per_launch": nvlink_bytes,
        "parity": {"gathered_equal_to_per_shard_launches": ok},
    }


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world == 1 and args.gpus != 1 and rank == 0:
        print(f"note: --gpus {args.gpus} without torchrun runs 1 rank", file=sys.stderr)
    sys.path.insert(0, str(ROOT))
    if args.layers is None and args.config != "sharded70b":
        args.layers = L
    if args.config == "prefill":
        set_prefill_offset(args.prefill_offset)
    if args.impl == "reference":
        run_reference(args, rank, world)
    elif args.config == "prefix":
        if rank == 0:
            print(json.dumps(run_prefix(args, local_rank)), flush=True)
    elif args.config == "quant":
        if rank == 0:
            print(json.dumps(run_quant(args, local_rank)), flush=True)
    elif args.config == "prefill":
        if rank == 0:
            run_prefill(args, local_rank)
    elif args.config == "kernels":
        if rank == 0:
            print(json.dumps(run_kernels(args, local_rank)), flush=True)
    elif args.config == "peer_pair":
        if world > 1:
            raise SystemExit("--config peer_pair drives both GPUs from one process: run it "
                             "without torchrun")
        print(json.dumps(run_peer_pair(args)), flush=True)
    else:
        run_gpu(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
