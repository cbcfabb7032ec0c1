"""bench.py's output contract, checked on the CPU.

The reference arm (`--impl reference`) runs the CPU restatement of the
reference's forward on the host cores, so its JSON line can be produced
here: one line, BASELINE.json's metric, the keys the driver reads, and the
reference arm's own e2e / cpu_baseline objects.  The clock sampler's
summary logic is checked against synthetic NVML readings.
"""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _baseline_metric():
    return json.loads((ROOT / "BASELINE.json").read_text())["metric"]


def test_reference_arm_json_line():
    env = dict(os.environ, OMP_NUM_THREADS="2")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == _baseline_metric()
    assert d["unit"] == "embeddings/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["n_gpus"] == 1
    assert d["config"]["workload"] == "bge-base-b256xL128"
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_bench_workloads_name_the_baseline_config():
    sys.path.insert(0, str(ROOT))
    try:
        import bench
    finally:
        sys.path.pop(0)
    assert "bge-base-b256xL128" in bench.WORKLOADS
    wl = bench.WORKLOADS["bge-base-b256xL128"]
    assert wl["preset"] == "bge-base" and wl["nseq"] == 256 and wl.get("lo", 128) == 128


class _FakeNvml:
    """The few NVML names NvmlClockSampler.summary reads."""
    NVML_CLOCK_SM = 1
    nvmlClocksEventReasonHwSlowdown = 0x8
    nvmlClocksEventReasonHwThermalSlowdown = 0x40
    nvmlClocksEventReasonSwThermalSlowdown = 0x20
    nvmlClocksEventReasonSwPowerCap = 0x4
    nvmlClocksEventReasonGpuIdle = 0x1
    nvmlClocksEventReasonApplicationsClocksSetting = 0x2
    nvmlClocksEventReasonSyncBoost = 0x10
    nvmlClocksEventReasonHwPowerBrakeSlowdown = 0x80
    nvmlClocksEventReasonDisplayClockSetting = 0x100
    nvmlClocksEventReasonUserDefinedClocks = 0x200

    class NVMLError(Exception):
        pass

    @staticmethod
    def nvmlDeviceGetMaxClockInfo(h, kind):
        return 1965


def test_clock_summary_names_throttle_reasons():
    sys.path.insert(0, str(ROOT))
    try:
        import bench
    finally:
        sys.path.pop(0)
    s = bench.NvmlClockSampler.__new__(bench.NvmlClockSampler)
    s.nv, s.h = _FakeNvml, None
    s.rows = [{"sm": 1965.0, "power": 700.0, "reasons": 0x4}, {"sm": 1800.0, "power": 990.0, "reasons": 0x4 | 0x200},
              {"sm": 1890.0, "power": 950.0, "reasons": 0}]
    out = s.summary()
    assert out["sm_mhz"] == 1890.0 and out["sm_max_mhz"] == 1965.0 and out["samples"] == 3
    assert out["reasons"] == ["sw_power_cap"]
    assert out["other_reasons"] == ["user_defined_clocks"]
    assert out["sm_mhz_range"] == [1800.0, 1965.0]
    s.rows = []
    assert s.summary()["reasons"] == ["no samples"]
