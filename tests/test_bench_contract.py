"""CPU: bench.py's reference arm prints the one JSON line the benchmark
contract asks for (decode and prefill workloads; each CPU sample takes a few
seconds)."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _line(*args):
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    _check(d)
    return d


def _check(d):
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    assert "workload" in d["config"]


def test_reference_arm_prefill_line():
    d = _line("--config", "prefill", "--steps", "1", "--warmup", "1")
    assert d["unit"] == "TFLOP/s"


def test_reference_arm_decode_line():
    d = _line("--steps", "3", "--warmup", "1", "--layers", "2")
    assert d["unit"] == "GB/s" and d["steps"] == 3 and d["warmup"] == 1
    # every step is measured whole, on the GPU arm's own config
    assert d["config"]["layers"] == 2 and d["config"]["global_batch"] == 64
    assert d["config"]["parallelism"] == "1 GPU"
    assert "measured whole" in d["cpu_baseline"]["sample"]


def test_reference_arm_config_matches_gpu_arm():
    """The reference arm's config is the GPU arm's (Workload.config), so the
    two lines describe the same workload."""
    sys.path.insert(0, str(ROOT))
    import bench

    for world in (1, 2, 8):
        w = bench.Workload(False, world, 32, 120.0, 0, True)
        assert w.B == 64 * world and w.hkv == 8 // world and w.nl == 32
        assert w.kv_layer_rank * world == w.kv_step_total / 32
    w5 = bench.Workload(True, 8, None, 120.0, 0, True)
    assert w5.B == 256 and w5.hkv == 1 and w5.hq == 8 and w5.nl == 80
    w1 = bench.Workload(True, 1, None, 120.0, 0, True)
    assert 1 <= w1.nl < 80  # 80 layers of the 70B shape do not fit one GPU


def test_peer_pair_reports_unavailable_without_two_gpus():
    """--config peer_pair drives two GPUs from one process; where there are
    fewer, it prints one JSON line saying so and exits 0."""
    import torch

    if torch.cuda.device_count() >= 2:
        return
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--config", "peer_pair",
                        "--steps", "1", "--warmup", "1"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["config"] == "peer_pair" and "unavailable" in d
