"""bench.py's clock record against a fake nvidia-smi (CPU): the sampler waits
for the first sample before the timed region, keeps the samples that bracket
the region however short it is, and reports the throttle reasons it saw."""
import os
import stat
import time

import pytest

FAKE = """#!/usr/bin/env python3
import sys, time
interval = 0.05
for a, b in zip(sys.argv, sys.argv[1:]):
    if a == "-lms":
        interval = int(b) / 1000.0
time.sleep({startup})  # slow start, as with several ranks starting nvidia-smi at once
i = 0
while True:
    cap = "Active" if i == {cap_at} else "Not Active"
    print(f"{{1900 + i % 3}}, 1965, 300.5, 0x0, Not Active, Not Active, Not Active, {{cap}}", flush=True)
    i += 1
    time.sleep(interval)
"""


@pytest.fixture
def fake_smi(tmp_path, monkeypatch):
    def make(startup: float, cap_at: int = -1):
        path = tmp_path / "nvidia-smi"
        path.write_text(FAKE.format(startup=startup, cap_at=cap_at))
        path.chmod(path.stat().st_mode | stat.S_IEXEC)
        monkeypatch.setenv("PATH", str(tmp_path) + os.pathsep + os.environ.get("PATH", ""))

    return make


def test_short_region_is_bracketed_after_a_slow_start(fake_smi):
    import bench

    fake_smi(startup=0.6)
    cs = bench.ClockSampler(0)
    cs.start()
    cs.mark()
    time.sleep(0.02)  # a timed region much shorter than the sampling interval
    rec = cs.stop()
    assert rec["samples"] >= 2, rec
    assert rec["sm_max_mhz"] == 1965.0
    assert 1900.0 <= rec["sm_mhz"] <= 1902.0
    assert rec["reasons"] == []


def test_reasons_inside_the_region_are_reported(fake_smi):
    import bench

    fake_smi(startup=0.0, cap_at=3)
    cs = bench.ClockSampler(0)
    cs.start()
    cs.mark()
    time.sleep(0.4)
    rec = cs.stop()
    assert rec["samples"] >= 5, rec
    assert rec["reasons"] == ["sw_power_cap"]


def test_missing_nvidia_smi_reports_unsampled(monkeypatch, tmp_path):
    import bench

    monkeypatch.setenv("PATH", str(tmp_path))
    cs = bench.ClockSampler(0)
    cs.start()
    rec = cs.stop()
    assert rec["samples"] == 0 and rec["reasons"] == ["unsampled"]
