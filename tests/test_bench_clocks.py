"""bench.py's clock sampler: only samples that arrive inside the timed region
are reported, slowdown reasons are collected, and a missing nvidia-smi gives
an empty record instead of an error.  A shell loop stands in for nvidia-smi."""
import os
import sys
import time

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

import bench  # noqa: E402


def _loop(line: str) -> list:
    return ["bash", "-c", f"while true; do echo '{line}'; sleep 0.02; done"]


def test_samples_inside_region_only():
    s = bench.ClockSampler(0, cmd=_loop("1965, 1965, Not Active, Not Active, Not Active, Active"))
    s.start()
    s.wait_first()
    time.sleep(0.1)  # samples before the region are dropped
    s.mark_start()
    time.sleep(0.25)
    s.mark_end()
    time.sleep(0.1)  # and after it
    rec = s.stop()
    assert 3 <= rec["samples"] <= 20, rec
    assert rec["sm_mhz"] == 1965.0 and rec["sm_max_mhz"] == 1965.0
    assert rec["reasons"] == ["sw_power_cap"]


def test_missing_sampler_gives_empty_record():
    s = bench.ClockSampler(0, cmd=["/nonexistent/nvidia-smi"])
    s.start()
    s.wait_first(0.2)
    s.mark_start()
    s.mark_end()
    rec = s.stop()
    assert rec["samples"] == 0 and rec["sm_mhz"] is None and rec["reasons"] == []
