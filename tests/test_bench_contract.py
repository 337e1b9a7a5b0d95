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
    d = _line("--steps", "3", "--warmup", "1")
    assert d["unit"] == "GB/s" and d["steps"] == 3 and d["warmup"] == 1
