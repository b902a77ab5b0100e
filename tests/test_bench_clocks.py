"""bench.py's clock sampler against a fake NVML: samples land only inside the marked timed
window, the reason bits decode to names, and a window with no samples reports None.  (The
sampler only reads; it never sets clocks or any other GPU state.)"""

import sys
import time
import types

import bench


class _Props:
    pci_domain_id, pci_bus_id, pci_device_id = 0, 0x3B, 0


def _fake_nvml(bits):
    nv = types.SimpleNamespace()
    nv.NVML_CLOCK_SM = 1
    nv.bus = None
    nv.nvmlInit = lambda: None

    def by_bus(b):
        nv.bus = b
        return "h"

    nv.nvmlDeviceGetHandleByPciBusId = by_bus
    nv.nvmlDeviceGetMaxClockInfo = lambda h, c: 1965
    nv.nvmlDeviceGetClockInfo = lambda h, c: 1850
    nv.nvmlDeviceGetCurrentClocksEventReasons = lambda h: bits
    return nv


def _sampler(monkeypatch, bits):
    nv = _fake_nvml(bits)
    monkeypatch.setitem(sys.modules, "pynvml", nv)
    monkeypatch.setattr(bench.torch.cuda, "get_device_properties", lambda d: _Props())
    return bench.ClockSampler("cuda:0"), nv


def test_samples_inside_window_and_reason_names(monkeypatch):
    cs, nv = _sampler(monkeypatch, 0x4 | 0x1)   # sw_power_cap + gpu idle (not reported)
    assert nv.bus == "00000000:3b:00.0"
    cs.start()
    time.sleep(0.05)
    cs.mark_begin()
    time.sleep(0.12)
    cs.mark_end()
    time.sleep(0.05)
    r = cs.stop()
    assert r["sm_mhz"] == 1850 and r["sm_max_mhz"] == 1965
    assert r["reasons"] == ["sw_power_cap"]
    assert r["reason_bits"] == "0x5"           # every bit seen, named or not (gpu idle included)
    assert r["sm_mhz_range"] == [1850, 1850]
    assert 3 <= r["samples"] <= 20   # 10 ms period over a 120 ms window, none outside it
    assert r["source"].startswith("nvml")


def test_thermal_reasons_are_reported(monkeypatch):
    cs, _ = _sampler(monkeypatch, 0x8 | 0x40)
    cs.start()
    cs.mark_begin()
    time.sleep(0.05)
    cs.mark_end()
    assert cs.stop()["reasons"] == ["hw_slowdown", "hw_thermal_slowdown"]


def test_empty_window_reports_none(monkeypatch):
    cs, _ = _sampler(monkeypatch, 0)
    cs.start()
    time.sleep(0.03)
    cs.mark_begin()
    cs.mark_end()            # an empty window: no sample can fall inside
    assert cs.stop() is None
