"""The `bench.py --impl reference` line on the CPU: the fields the round's
driver reads (one JSON line on stdout, the same metric / unit / direction as
the GPU arm, a cpu_baseline that describes the run, an e2e block with no
copies), and that ranks other than 0 exit cleanly without work."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(args, env_extra=None, timeout=600):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=timeout)


def test_reference_arm_prints_one_contract_line():
    import bench

    p = _run(["--impl", "reference", "--steps", "1", "--warmup", "0", "--batch", "8"])
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, p.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC
    assert line["unit"] == "embeddings/s" and line["higher_is_better"] is True
    assert line["n_gpus"] == 1 and line["steps"] == 1 and line["warmup"] == 0
    assert line["value"] > 0 and line["ms_per_step"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "workload" in line["config"]


def test_reference_arm_other_ranks_exit_without_work():
    p = _run(["--impl", "reference", "--steps", "1", "--warmup", "0", "--batch", "8"],
             {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, timeout=120)
    assert p.returncode == 0, p.stderr[-2000:]
    assert p.stdout.strip() == ""


FAKE_SMI = r'''#!/usr/bin/env python3
import sys, time
# the bench's query: index, clocks.sm, clocks.max.sm, power.draw, reasons.active,
# hw_slowdown, hw_thermal_slowdown, sw_thermal_slowdown, sw_power_cap
time.sleep(0.3)  # nvidia-smi's start-up before its first sample
cap = "Active" if "cap" in sys.argv[0] else "Not Active"
for i in range(1000):
    sm = 1965 if i % 2 == 0 else 1900
    print(f"0, {sm}, 1965, 900.5, 0x0, Not Active, Not Active, Not Active, {cap}", flush=True)
    time.sleep(0.05)
'''


def _fake_smi(tmp_path, name):
    d = tmp_path / name
    d.mkdir()
    exe = d / "nvidia-smi"
    exe.write_text(FAKE_SMI.replace('"cap" in sys.argv[0]', repr(name == "cap")))
    exe.chmod(0o755)
    return d


def test_clock_sampler_is_live_when_the_timed_region_starts(tmp_path, monkeypatch):
    """The sampler returns from __enter__ only once the first sample is in,
    so a 0.2 s region gets several samples; the summary reads the clocks and
    the throttle reasons from nvidia-smi's CSV fields (a fake here)."""
    import time

    import bench

    for name, reasons in (("clean", []), ("cap", ["sw_power_cap"])):
        monkeypatch.setenv("PATH", f"{_fake_smi(tmp_path, name)}{os.pathsep}{os.environ['PATH']}")
        with bench.ClockSampler(0) as clk:
            time.sleep(0.2)
        s = clk.summary()
        assert s["samples"] >= 3, s
        assert s["sm_max_mhz"] == 1965.0 and 1900.0 <= s["sm_mhz"] <= 1965.0
        assert s["reasons"] == reasons


def test_clock_sampler_without_nvidia_smi(tmp_path, monkeypatch):
    import bench

    monkeypatch.setenv("PATH", str(tmp_path))
    with bench.ClockSampler(0) as clk:
        pass
    assert clk.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
