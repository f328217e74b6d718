"""Host-side pieces of bench.py that need no GPU: the clock sampler's NVML polling and its
summary, against a fake NVML module (read-only queries only; nothing is set), and the reference
arm's JSON line (the CPU restatement on the tiny config), alone and under torchrun."""
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


def _json_lines(out):
    import json
    return [json.loads(line) for line in out.splitlines() if line.startswith("{")]


def _check_reference_line(line, n_gpus):
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["n_gpus"] == n_gpus and line["steps"] == 2 and line["warmup"] == 3
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] in ("port", "reference") and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["model"] == "tiny"


def test_reference_arm_line_one_process():
    """`bench.py --impl reference` times the CPU restatement and prints one contract line."""
    import os
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "tiny", "--steps", "2",
                        "--warmup", "3"], cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    _check_reference_line(lines[0], 1)


def test_reference_arm_under_torchrun_prints_once():
    """Launched as the driver launches it for N > 1: rank 0 alone runs and prints, the other rank
    exits 0 without work."""
    import os
    import socket
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
                        "--config", "tiny", "--gpus", "2", "--steps", "2", "--warmup", "3"],
                       cwd=root, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    _check_reference_line(lines[0], 2)
