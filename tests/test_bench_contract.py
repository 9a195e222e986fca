# SPDX-License-Identifier: Apache-2.0
"""bench.py's reference arm (CPU only) prints one JSON line with the keys
the benchmark contract names."""
from __future__ import annotations

import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _run(*args) -> dict:
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                         capture_output=True, text=True, timeout=600, cwd=ROOT, check=True)
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_json_line():
    line = _run("--impl", "reference", "--config", "c2_mxfp8_b64_ctx512-4096", "--steps", "1",
                "--warmup", "3", "--cpu-seconds", "0.5")
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["config"]["workload"] == "c2_mxfp8_b64_ctx512-4096"
    assert line["value"] > 0 and line["unit"] == "GB/s"
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["warmup"] >= 3


def test_reference_arm_table_build():
    """The block-table build's reference arm runs the reference's own path
    (OpenSSL SHA256 keys + cache_index.c lookups) when oracle/_ref has it."""
    import pytest
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    line = _run("--impl", "reference", "--config", "t5_tables_b16_2048_prefix1024", "--steps",
                "2", "--warmup", "3")
    if oracle.ref_index_lib() is None:
        assert "unavailable" in line
        pytest.skip("reference index library not built")
    assert line["impl"] == "reference" and line["unit"] == "blocks/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "reference"
    assert line["e2e"]["h2d_bytes_per_step"] == 0


def test_reference_arm_unavailable_lines():
    """Paths the reference only stubs print the contract's unavailable line."""
    for cfg in ("w3_kv_arrival_4096x36k", "l3_lm_head_llama3-8b_b256_greedy"):
        line = _run("--impl", "reference", "--config", cfg)
        assert line["impl"] == "reference" and line["unavailable"]


def test_clock_sampler_reads_nvml_during_the_region(monkeypatch):
    """The bench's clock record comes from NVML samples taken every 10 ms on
    a thread (checked here against a fake NVML: the median SM clock, the
    maximum, and the clock-event reason bits mapped to their names)."""
    import time
    import types
    sys.path.insert(0, ROOT)
    import bench

    calls = {"n": 0}
    fake = types.ModuleType("pynvml")
    fake.NVML_CLOCK_SM = 1
    fake.nvmlInit = lambda: None
    fake.nvmlDeviceGetHandleByIndex = lambda i: ("gpu", i)
    fake.nvmlDeviceGetMaxClockInfo = lambda h, kind: 1965

    def clock(h, kind):
        calls["n"] += 1
        return 1965 if calls["n"] % 2 else 1755

    fake.nvmlDeviceGetClockInfo = clock
    fake.nvmlDeviceGetCurrentClocksEventReasons = lambda h: 0x4 | 0x20   # power cap, sw thermal
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    c = bench.Clocks(3)
    c.start()
    time.sleep(0.08)
    r = c.stop()
    assert r["samples"] >= 3, r
    assert r["sm_max_mhz"] == 1965.0
    assert 1755.0 <= r["sm_mhz"] <= 1965.0
    assert r["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]
    assert r["source"].startswith("nvml")
