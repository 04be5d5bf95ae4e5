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


def test_nvml_sampler_with_a_fake_nvml(monkeypatch):
    """The NVML sampler reads (never sets) the SM clock and the clock-event
    reason bits, finds the GPU by PCI bus id and keeps only in-region samples."""
    import types
    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=1, nvmlInit=lambda: None,
        nvmlDeviceGetHandleByPciBusId=lambda bus: ("h", bus),
        nvmlDeviceGetMaxClockInfo=lambda h, c: 1965,
        nvmlDeviceGetClockInfo=lambda h, c: 1900,
        nvmlDeviceGetCurrentClocksEventReasons=lambda h: 0x4 | 0x1)
    monkeypatch.setitem(sys.modules, "pynvml", fake)

    class Props:
        pci_bus_id, pci_device_id, pci_domain_id = 0x1b, 0, 0

    import torch
    monkeypatch.setattr(torch.cuda, "get_device_properties", lambda i: Props())
    s = bench.NvmlClockSampler(0, interval_ms=2)
    assert s.h == ("h", "00000000:1b:00.0")
    s.start()
    s.wait_first()
    time.sleep(0.02)
    s.mark_start()
    time.sleep(0.05)
    s.mark_end()
    rec = s.stop()
    assert rec["samples"] >= 5 and rec["sm_mhz"] == 1900.0 and rec["sm_max_mhz"] == 1965.0
    assert rec["reasons"] == ["sw_power_cap"] and rec["source"] == "nvml"


def test_profile_figures_are_read_from_summaries(tmp_path, monkeypatch):
    p = tmp_path / "k.md"
    p.write_text("# kernel\n- dram_bytes_per_launch: 224301824\n- other: 1\n")
    monkeypatch.setattr(bench, "PROFILES", str(tmp_path))
    assert bench.profile_figure("k.md", "dram_bytes_per_launch") == 224301824
    assert bench.profile_figure("k.md", "missing") is None
    assert bench.profile_figure("absent.md", "x") is None
