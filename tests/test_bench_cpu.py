"""The reference arm of bench.py runs on host cores only, so its JSON line is checked here: the
keys the benchmark contract asks for, the same metric / unit / config as the B200 arm, and an
e2e object that moves no bytes across the host link."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3", "--cpu-sample-s", "0.3"], capture_output=True, text=True, env=env,
                         cwd=ROOT, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    a = json.loads(lines[0])
    sys.path.insert(0, str(ROOT))
    import bench

    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config"):
        assert k in a, k
    assert a["impl"] == "reference" and a["metric"] == bench.METRIC and a["unit"] == bench.UNIT
    assert a["value"] > 0 and a["higher_is_better"] is True and a["n_gpus"] == 1
    assert a["config"]["workload"] == bench.RESOLVER_WORKLOADS["resolver"].describe()
    cb = a["cpu_baseline"]
    assert cb["value"] == a["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert a["e2e"] == {"value": a["value"], "unit": a["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_clock_sampler_reads_nvml_and_maps_event_reasons(monkeypatch):
    """The clock sampler on a fake NVML: a sample at start and polls while running, the median SM
    clock, the maximum, and the throttle reasons seen in any sample (power cap here)."""
    import time
    import types

    sys.path.insert(0, str(ROOT))
    import bench

    clocks = iter([1965, 1965, 1800] + [1965] * 1000)
    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=1, nvmlClocksEventReasonSwPowerCap=0x4, nvmlClocksEventReasonHwSlowdown=0x8,
        nvmlInit=lambda: None, nvmlDeviceGetHandleByIndex=lambda i: ("gpu", i),
        nvmlDeviceGetClockInfo=lambda h, c: next(clocks), nvmlDeviceGetMaxClockInfo=lambda h, c: 1965,
        nvmlDeviceGetCurrentClocksEventReasons=lambda h: 0x4)
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    c = bench.ClockSampler(3)
    c.start()
    time.sleep(0.1)
    out = c.stop()
    assert out["samples"] >= 2 and out["sm_max_mhz"] == 1965 and out["sm_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"] and out["source"].startswith("NVML")
    # a sampler whose NVML is missing falls back to nvidia-smi, or reports that it has none
    monkeypatch.setitem(sys.modules, "pynvml", None)
    c = bench.ClockSampler(0)
    c.start()
    out = c.stop()
    assert "sm_mhz" in out and "reasons" in out
