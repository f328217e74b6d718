"""Host-side pieces of bench.py that need no GPU: the clock sampler's NVML polling and its
summary, against a fake NVML module (read-only queries only; nothing is set)."""
import sys
import time
import types

import bench


def _fake_nvml(clocks, reasons, max_mhz=1965):
    it = {"n": 0}
    nv = types.SimpleNamespace()
    nv.NVML_CLOCK_SM = 1
    nv.nvmlClocksEventReasonHwSlowdown = 0x8
    nv.nvmlClocksEventReasonHwThermalSlowdown = 0x40
    nv.nvmlClocksEventReasonSwThermalSlowdown = 0x20
    nv.nvmlClocksEventReasonSwPowerCap = 0x4
    nv.calls = []
    nv.nvmlInit = lambda: nv.calls.append("init")
    nv.nvmlShutdown = lambda: nv.calls.append("shutdown")
    nv.nvmlDeviceGetHandleByIndex = lambda i: ("dev", i)
    nv.nvmlDeviceGetMaxClockInfo = lambda h, c: max_mhz

    def clock(h, c):
        i = it["n"]
        it["n"] += 1
        return clocks[min(i, len(clocks) - 1)]
    nv.nvmlDeviceGetClockInfo = clock
    nv.nvmlDeviceGetCurrentClocksEventReasons = lambda h: reasons[min(it["n"] - 1, len(reasons) - 1)]
    return nv


def test_nvml_samples_and_reasons(monkeypatch):
    nv = _fake_nvml([1965, 1965, 1800, 1965], [0, 0x4, 0x4, 0])
    monkeypatch.setitem(sys.modules, "pynvml", nv)
    monkeypatch.setattr(bench.subprocess, "Popen", lambda *a, **k: (_ for _ in ()).throw(OSError("no smi")))
    with bench.ClockSampler(3) as c:
        time.sleep(0.15)
    s = c.summary()
    assert s["source"] == "nvml" and s["samples"] >= 4
    assert s["sm_max_mhz"] == 1965 and s["sm_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]
    assert nv.calls[0] == "init" and nv.calls[-1] == "shutdown"


def test_nvml_failure_falls_back_to_nvidia_smi(monkeypatch):
    nv = _fake_nvml([1965], [0])

    def broken():
        raise RuntimeError("NVML Shared Library Not Found")
    nv.nvmlInit = broken
    monkeypatch.setitem(sys.modules, "pynvml", nv)

    class FakeProc:
        def terminate(self):
            pass

        def communicate(self, timeout=None):
            row = "0, 1950, 1965, 700.0, 0x4, Not Active, Not Active, Not Active, Active"
            return row + "\n" + row.replace("1950", "1960") + "\n", ""
    monkeypatch.setattr(bench.subprocess, "Popen", lambda *a, **k: FakeProc())
    with bench.ClockSampler(0) as c:
        time.sleep(0.02)
    s = c.summary()
    assert s["source"] == "nvidia-smi" and s["samples"] == 2
    assert s["sm_mhz"] == 1955 and s["sm_max_mhz"] == 1965 and s["reasons"] == ["sw_power_cap"]


def test_unsampled_when_nothing_answers(monkeypatch):
    nv = _fake_nvml([1965], [0])
    nv.nvmlDeviceGetHandleByIndex = lambda i: (_ for _ in ()).throw(RuntimeError("bad index"))
    monkeypatch.setitem(sys.modules, "pynvml", nv)
    monkeypatch.setattr(bench.subprocess, "Popen", lambda *a, **k: (_ for _ in ()).throw(OSError("no smi")))
    with bench.ClockSampler(0) as c:
        pass
    assert c.summary()["reasons"] == ["unsampled"]
    assert nv.calls == ["init", "shutdown"]


def test_nvml_device_found_by_uuid(monkeypatch):
    """The CUDA device's UUID picks the NVML handle; the index is only the fallback."""
    nv = _fake_nvml([1700], [0])
    nv.nvmlDeviceGetCount = lambda: 4
    nv.nvmlDeviceGetUUID = lambda h: f"GPU-0000000{h[1]}-aaaa".encode()
    seen = []

    def clock(h, c):
        seen.append(h)
        return 1700
    nv.nvmlDeviceGetClockInfo = clock
    monkeypatch.setitem(sys.modules, "pynvml", nv)
    monkeypatch.setattr(bench.subprocess, "Popen", lambda *a, **k: (_ for _ in ()).throw(OSError("no smi")))
    with bench.ClockSampler(0, uuid="00000002-aaaa") as c:
        time.sleep(0.03)
    assert c.summary()["samples"] >= 1 and set(seen) == {("dev", 2)}
    seen.clear()
    with bench.ClockSampler(1, uuid="not-present") as c:
        time.sleep(0.03)
    assert set(seen) == {("dev", 1)}
