"""The C-ABI library loads and exports every symbol include/llmdot_cuda.h
declares; on a machine without a GPU its entry points fail with a status, never
crash and never compute on the CPU."""
import ctypes as C
import subprocess

import numpy as np
import pytest

from dotllm_b200 import native


def test_library_exists_and_loads():
    L = native.lib()
    assert L.llmdot_cuda_version().decode().startswith("llmdot-cuda")


def test_exports_every_header_function():
    declared = native.header_functions()
    assert len(declared) >= 35
    out = subprocess.run(["nm", "-D", "--defined-only", native.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [f for f in declared if f not in exported]
    assert not missing, f"not exported: {missing}"
    # nothing else leaks: internal symbols are hidden
    extra = [s for s in exported if s.startswith("llmdot") and s not in declared]
    assert not extra, f"undeclared exports: {extra}"


def test_bindings_cover_header():
    assert set(native.header_functions()) <= set(native._SIGS)


def test_device_count_without_gpu_is_zero_or_more():
    n = native.device_count()
    assert n >= 0


def test_no_cpu_fallback_without_device():
    if native.device_count() > 0:
        pytest.skip("a GPU is present; this checks the device-less error path")
    h = C.c_void_p()
    rc = native.lib().llmdot_cuda_create(0, C.byref(h))
    assert rc == -3 and not h.value
    assert "no CUDA device" in native.lib().llmdot_cuda_last_error().decode()
    with pytest.raises(native.CudaBackendError):
        from dotllm_b200.backend import CudaBackend
        CudaBackend(0)


def test_seeded_draw_matches_oracle():
    """llmdot_cuda_sampling_seeded_draw (host only) is the oracle's new Random(seed).NextSingle()."""
    from oracle import oracle as O
    # int.MinValue has its own case in the seeding (its absolute value does not fit an int)
    seeds = [0, 1, 7, 42, 99, 12345, -5, 2147483647, -2147483648]
    seeds += [int(x) for x in np.random.default_rng(3).integers(-2**31, 2**31, size=500)]
    for seed in seeds:
        d = native.lib().llmdot_cuda_sampling_seeded_draw(seed)
        assert d == O.net_random_single(seed) and 0.0 <= d < 1.0, seed


def test_header_is_plain_c99(tmp_path):
    """The boundary is a C ABI: the header compiles as strict C99 and the sampling struct has
    the layout the ctypes binding uses."""
    import os
    hdr = native.HEADER
    out = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-fsyntax-only", "-x", "c", hdr],
                         capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    src = tmp_path / "size.c"
    src.write_text(f'#include "{os.path.abspath(hdr)}"\n#include <stdio.h>\n'
                   'int main(void) { printf("%zu %zu", sizeof(llmdot_sampling), sizeof(llmdot_config)); return 0; }\n')
    exe = tmp_path / "size"
    subprocess.run(["gcc", "-std=c99", str(src), "-o", str(exe)], check=True)
    s_sampling, s_config = map(int, subprocess.run([str(exe)], capture_output=True, text=True).stdout.split())
    assert s_sampling == C.sizeof(native.LlmdotSampling)
    assert s_config == C.sizeof(native.LlmdotConfig)


def test_sampling_defaults_are_the_references():
    """SamplingOptions.cs:7-14: TopK 40, TopP 0.95, Temperature 0.8, RepeatPenalty 1.1, window 64, Seed -1."""
    o = native.LlmdotSampling()
    assert (o.top_k, o.repeat_window, o.seed) == (40, 64, -1)
    assert (o.top_p, o.temperature, o.repeat_penalty) == (pytest.approx(0.95), pytest.approx(0.8), pytest.approx(1.1))


def test_backend_rejects_short_host_arrays_before_the_call():
    """Entry points that take one length for several host spans would read a shorter array past
    its end; the binding refuses it first (no device is needed to see that)."""
    from dotllm_b200.backend import CudaBackend
    b = CudaBackend.__new__(CudaBackend)  # no device handle: every case must fail before the call
    b._h = None
    x = np.ones(16, np.float32)
    with pytest.raises(ValueError):
        b.rms_norm(x, np.ones(8, np.float32), 1e-5)
    with pytest.raises(ValueError):
        b.layer_norm(x, np.ones(16, np.float32), np.ones(4, np.float32), 1e-5)
    with pytest.raises(ValueError):
        b.add(x, np.ones(15, np.float32))
    with pytest.raises(ValueError):
        b.mul(x, np.ones(3, np.float32))
    with pytest.raises(ValueError):
        b.add_in_place(x.copy(), np.ones(15, np.float32))
    with pytest.raises(ValueError):
        b.conv1d(np.ones(8, np.float32), np.ones(12, np.float32), 3, 4)
    with pytest.raises(TypeError):
        b.add_in_place(np.ones(16, np.float64), x)
    with pytest.raises(TypeError):
        b.scale_in_place(np.ones(16, np.float64), 2.0)
    with pytest.raises(TypeError):
        b.silu_in_place(x[::2])


def test_engine_rejects_token_and_draw_counts_the_library_would_overrun():
    """decode / decode_steps read one token per session and generate_sampled one
    draw per token: other counts are refused before the call (no device needed)."""
    from types import SimpleNamespace

    from dotllm_b200 import engine
    fake = [SimpleNamespace(_h=None), SimpleNamespace(_h=None)]
    for call in (lambda: engine.decode_batch(fake, [1]),
                 lambda: engine.decode_steps(fake, [1, 2, 3], 4)):
        with pytest.raises(ValueError):
            call()
    s = engine.CudaSession.__new__(engine.CudaSession)
    s._h = None
    with pytest.raises(ValueError):
        s.generate_sampled([1, 2], 8, native.LlmdotSampling(), draws=np.full(7, 0.5, np.float32))


def test_csharp_bindings_name_declared_entry_points():
    """Every entry point the C# [LibraryImport] bindings bind (the list in
    tests/golden/csharp_bindings.json) is a function the header declares: a binding must not name
    a symbol that does not exist."""
    import json
    import os
    here = os.path.dirname(os.path.abspath(__file__))
    entry_points = set(json.load(open(os.path.join(here, "golden", "csharp_bindings.json")))["entry_points"])
    assert entry_points and entry_points <= set(native.header_functions())


def test_sampler_mirror_draws_like_the_reference():
    """backend.Sampler passes no draw for a seed >= 0 (the backend then uses the seeded draw) and a
    fresh uniform draw in [0, 1) otherwise."""
    from dotllm_b200.backend import Sampler
    calls = []

    class FakeBackend:
        def sample(self, logits, options, recent, r):
            calls.append(r)
            return 7
    s = Sampler(FakeBackend())
    assert s.sample([0.0, 1.0], native.LlmdotSampling(seed=42), [1]) == 7
    s.sample([0.0, 1.0], native.LlmdotSampling(seed=-1), [])
    s.sample([0.0, 1.0], native.LlmdotSampling(seed=-1), [])
    assert calls[0] is None
    assert all(0.0 <= r < 1.0 for r in calls[1:]) and calls[1] != calls[2]
