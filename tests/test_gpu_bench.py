"""bench.py's default line on a GPU: one JSON line with every key the benchmark contract asks for
(roofline of the dominant kernel, CPU baseline, end-to-end figure, clocks, launch count), for a
short run of the default workload."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def test_default_bench_line_carries_the_contract_keys():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--steps", "3", "--warmup", "3",
                          "--cpu-sample-s", "1"], capture_output=True, text=True, cwd=ROOT, timeout=900)
    assert out.returncode == 0, out.stderr[-3000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    a = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "roofline", "cpu_baseline", "e2e", "gpu_launches", "clocks"):
        assert k in a, k
    assert a["n_gpus"] == 1 and a["steps"] == 3 and a["warmup"] == 3 and a["value"] > 0
    assert "workload" in a["config"]
    rf = a["roofline"]
    assert rf["achieved"] > 0 and rf["peak"] > 0 and abs(rf["frac"] - rf["achieved"] / rf["peak"]) < 1e-9
    assert a["cpu_baseline"]["value"] > 0 and a["cpu_baseline"]["cores"] >= 1 and a["cpu_baseline"]["kind"] == "port"
    e = a["e2e"]
    assert e["value"] > 0 and e["h2d_bytes_per_step"] > 0 and e["d2h_bytes_per_step"] > 0
    assert a["gpu_launches"] == 2 * a["steps"]  # one LRU step and one swap-in per timed step
    assert "sm_mhz" in a["clocks"] and "reasons" in a["clocks"]


def _bench_line(*args):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True, cwd=ROOT,
                         timeout=900)
    assert out.returncode == 0, out.stderr[-3000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    return json.loads(lines[0])


def test_multilayer_layer_pipelining_keeps_results():
    """The multi-layer workload with each layer's swap-in on a second stream, overlapping the next
    layer's LRU step: the same LRU statistics as the serial run of the same trace, and every resident
    row of every (layer, request) pool equal to its host record afterwards."""
    common = ["--workload", "multilayer", "--steps", "2", "--warmup", "3", "--prefill", "2", "--no-cpu-baseline",
              "--verify"]
    serial = _bench_line(*common)
    piped = _bench_line(*common, "--overlap-layers")
    assert serial["overlap_layers"] is False and piped["overlap_layers"] is True
    assert piped["job_stats"] == serial["job_stats"]
    assert piped["job_stats"]["installs"] > 0 and piped["job_stats"]["shortages"] == 0
    assert piped["verified_rows"] == serial["verified_rows"] > 0
    assert piped["gpu_launches"] == serial["gpu_launches"] == 2 * 2 * 4
