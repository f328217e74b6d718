"""Per-operation adapter (IComputeBackend) on the GPU vs the CPU oracle.

Bit-exact wherever the reference uses only IEEE +,-,*,/ (dequantisation, the
ExpApprox/TanhApprox vector lanes, RoPE with host cos/sin, argmax, element-wise
ops).  Reductions with a different summation order and the MathF tail lanes
(expf/tanhf: CUDA vs glibc differ by <= 2 ulp) use the tolerances written
beside each check.
"""
import base64
import json
import os

import numpy as np
import pytest

from dotllm_b200 import gguf, quant

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
KAT = json.load(open(os.path.join(HERE, "golden", "kquant_kat.json")))["cases"]


def bits_equal(a, b):
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all(nan | (a.view(np.uint32) == b.view(np.uint32))))


@pytest.mark.parametrize("case", KAT, ids=[c["name"] for c in KAT])
def test_dequant_golden_bit_exact(backend, case):
    data = np.frombuffer(base64.b64decode(case["data"]), dtype=np.uint8).copy()
    exp = np.frombuffer(base64.b64decode(case["expected_f32"]), dtype="<f4")
    out = backend.dequantize_to_float(data, case["type"], case["rows"], case["row_elems"])
    assert bits_equal(out, exp)


@pytest.mark.parametrize("t", [gguf.GGML_Q4_K, gguf.GGML_Q5_K, gguf.GGML_Q6_K, gguf.GGML_Q8_0, gguf.GGML_Q4_0,
                               gguf.GGML_Q2_K, gguf.GGML_Q3_K, gguf.GGML_F16, gguf.GGML_BF16, gguf.GGML_F32])
def test_dequant_random_bit_exact(backend, oracle, t):
    """Random bytes (incl. NaN/Inf/subnormal f16 scales) over many rows."""
    rng = np.random.default_rng(100 + t)
    be, bb = gguf.BLOCK[t]
    rows, elems = 37, 1024
    nbytes = rows * (elems // be) * bb + (2 if t == gguf.GGML_Q3_K else 0)
    data = rng.integers(0, 256, nbytes, dtype=np.uint8)
    ref = oracle.dequantize(data, t, rows, elems)
    out = backend.dequantize_to_float(data, t, rows, elems)
    assert bits_equal(out, ref)


def test_dequant_q3k_needs_slack(backend):
    from dotllm_b200.native import CudaBackendError
    with pytest.raises(CudaBackendError, match="Q3_K"):
        backend.dequantize_to_float(np.zeros(110, dtype=np.uint8), gguf.GGML_Q3_K, 1, 256)


def test_dequant_empty_and_short(backend):
    from dotllm_b200.native import CudaBackendError
    assert backend.dequantize_to_float(np.zeros(0, dtype=np.uint8), gguf.GGML_Q4_K, 0, 256).size == 0
    with pytest.raises(CudaBackendError):
        backend.dequantize_to_float(np.zeros(100, dtype=np.uint8), gguf.GGML_Q4_K, 1, 256)
    with pytest.raises(CudaBackendError):
        backend.dequantize_to_float(np.zeros(100, dtype=np.uint8), 16, 1, 256)  # IQ2_XXS: unsupported


@pytest.mark.parametrize("n", [8, 64, 1000, 4097])
def test_elementwise_exact(backend, oracle, n):
    rng = np.random.default_rng(n)
    a = rng.standard_normal(n).astype(np.float32) * 3
    b = rng.standard_normal(n).astype(np.float32)
    assert bits_equal(backend.add(a, b), oracle.add(a, b))
    assert bits_equal(backend.mul(a, b), oracle.mul(a, b))
    assert bits_equal(backend.scale(a, 0.37), oracle.scale(a, 0.37))
    c = a.copy()
    backend.add_in_place(c, b)
    assert bits_equal(c, oracle.add(a, b))
    nv = n - n % 8  # reference vector lanes: bit-exact; MathF tail: <= 4 ulp
    for name in ("silu", "gelu"):
        g, r = getattr(backend, name)(a), getattr(oracle, name)(a)
        assert bits_equal(g[:nv], r[:nv]), name
        assert np.allclose(g[nv:], r[nv:], rtol=1e-6, atol=1e-7), name
    g, r = backend.softcap(a * 20, 30.0), oracle.softcap(a * 20, 30.0)
    assert bits_equal(g[:nv], r[:nv])
    assert np.allclose(g[nv:], r[nv:], rtol=1e-6, atol=1e-6)


def test_gelu_scalar(backend, oracle):
    for x in (-3.0, -1.0, 0.0, 0.5, 1.0, 2.5):
        assert abs(backend.gelu_scalar(x) - oracle.gelu_scalar(x)) <= 1e-6 * max(1.0, abs(x))


@pytest.mark.parametrize("n,cap", [(1, None), (7, None), (64, None), (1001, None), (4096, 50.0), (13, 5.0)])
def test_softmax(backend, oracle, n, cap):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32) * 4
    g, r = backend.softmax(x, cap), oracle.softmax(x, cap)
    # the sum is reduced in a different order: agreement to a few ulp of each probability
    assert np.allclose(g, r, rtol=2e-6, atol=1e-9)


def test_softmax_empty(backend):
    assert backend.softmax(np.zeros(0, dtype=np.float32)).size == 0


@pytest.mark.parametrize("n", [2, 512, 2048, 2304, 4099])
def test_rmsnorm(backend, oracle, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    w = (1 + 0.01 * rng.standard_normal(n)).astype(np.float32)
    # different sum-of-squares order: the scale factor may differ by 1-2 ulp
    assert np.allclose(backend.rms_norm(x, w, 1e-5), oracle.rmsnorm(x, w, 1e-5), rtol=3e-7, atol=0)


def test_layernorm(backend, oracle):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(777).astype(np.float32) + 3
    w = rng.standard_normal(777).astype(np.float32)
    b = rng.standard_normal(777).astype(np.float32)
    assert np.allclose(backend.layer_norm(x, w, b, 1e-5), oracle.layernorm(x, w, b, 1e-5), rtol=1e-5, atol=1e-5)
    assert np.allclose(backend.layer_norm(x, w, None, 1e-5), oracle.layernorm(x, w, None, 1e-5), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("hd,pos,base", [(64, 0, 10000.0), (64, 17, 500000.0), (96, 1000, 10000.0), (128, 4095, 500000.0)])
def test_rope_exact(backend, oracle, hd, pos, base):
    rng = np.random.default_rng(hd + pos)
    q = rng.standard_normal(4 * hd).astype(np.float32)
    k = rng.standard_normal(2 * hd).astype(np.float32)
    gq, gk = backend.apply_rope(q[:hd], k[:hd], hd, pos, base, hd)
    rq, rk = oracle.rope(q[:hd], k[:hd], hd, pos, base, hd)
    assert bits_equal(gq, rq) and bits_equal(gk, rk)
    freq = (1.0 / np.power(np.float32(base), (2.0 * np.arange(hd // 2, dtype=np.float32) / hd))).astype(np.float32)
    gq, _ = backend.apply_rope_table(q[:hd], None, hd, pos, freq)
    rq, _ = oracle.rope_table(q[:hd], None, pos, freq)
    assert bits_equal(gq, rq)


@pytest.mark.parametrize("n", [1, 5, 32000, 128256])
def test_argmax(backend, oracle, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    assert backend.arg_max(x) == oracle.argmax(x)
    if n > 10:
        x[3] = x[n - 2] = x.max() + 1  # tie: lowest index wins
        assert backend.arg_max(x) == 3 == oracle.argmax(x)


def _special_rows(rng, n):
    """Rows of n floats with NaN, signed zeros and infinities placed where VectorMath.ArgMax's strict
    `>` scan from element 0 decides differently from a plain order on the float values."""
    from test_oracle_kats import ARGMAX_SPECIAL
    rows = [np.array(r, dtype=np.float32) for r, _ in ARGMAX_SPECIAL]
    nan, inf = np.float32("nan"), np.float32("inf")
    base = -np.abs(rng.standard_normal(n).astype(np.float32)) - 1.0
    x = base.copy(); x[0] = nan; x[n // 2] = inf; rows.append(x)            # NaN first: index 0
    x = base.copy(); x[n // 3] = nan; x[n - 1] = nan; rows.append(x)        # NaN never wins
    x = base.copy(); x[5] = -0.0; x[n - 7] = 0.0; rows.append(x)             # -0 then +0: the first
    x = base.copy(); x[9] = 0.0; x[11] = -0.0; x[3] = nan; rows.append(x)
    x = np.full(n, -inf, dtype=np.float32); x[n - 3] = nan; rows.append(x)  # all -Inf: index 0
    x = np.full(n, nan, dtype=np.float32); rows.append(x)                    # all NaN: index 0
    x = base.copy(); x[n - 1] = inf; x[n - 2] = inf; x[n - 4] = nan; rows.append(x)
    return rows


@pytest.mark.parametrize("n", [64, 32000, 128256])
def test_argmax_special_values(backend, oracle, n):
    """Index-exact against the reference's ArgMax on NaN, +-0 and +-Inf rows (argmax_kernel)."""
    for x in _special_rows(np.random.default_rng(n), n):
        assert backend.arg_max(x) == oracle.argmax(x), x[:16]


@pytest.mark.parametrize("n", [64, 32000])
def test_sampler_greedy_special_values(backend, oracle, n):
    """Sampler.Sample with Temperature <= 0 is ArgMax (Sampler.cs:26-27): same special rows."""
    from dotllm_b200.native import LlmdotSampling
    opt = LlmdotSampling(temperature=0.0, seed=1)
    for x in _special_rows(np.random.default_rng(n + 1), n):
        assert backend.sample(x, opt, r=0.5) == oracle.argmax(x), x[:16]


def test_conv1d(backend):
    rng = np.random.default_rng(9)
    x = rng.standard_normal(64 * 3).astype(np.float32)
    w = rng.standard_normal(64 * 3).astype(np.float32)
    out = backend.conv1d(x, w, 3, 64)
    assert np.allclose(out, (x.reshape(64, 3) * w.reshape(64, 3)).sum(1), rtol=1e-6, atol=1e-6)
    out1 = backend.conv1d(x[:64], w[:64], 1, 64)
    assert bits_equal(out1, x[:64] * w[:64])


MM_TYPES = [gguf.GGML_Q4_K, gguf.GGML_Q5_K, gguf.GGML_Q6_K, gguf.GGML_Q8_0, gguf.GGML_Q4_0]


@pytest.mark.parametrize("t", MM_TYPES)
@pytest.mark.parametrize("a_rows", [1, 3])
def test_matmul_vs_oracle(backend, oracle, t, a_rows):
    rng = np.random.default_rng(t * 10 + a_rows)
    cols, rows = 2048, 300
    w = quant.quantize(rng.standard_normal((rows, cols), dtype=np.float32) * 0.02, t)
    a = rng.standard_normal(a_rows * cols).astype(np.float32)
    g = backend.mat_mul(a, w, t, cols, rows, weight_key=f"w{t}_{a_rows}")
    r = oracle.matmul(a, w, t, cols, rows)
    # fp32 sums of 2048 products in a different order: bound by eps * sum|a*w|
    deq = oracle.dequantize(w, t, rows, cols).reshape(rows, cols)
    bound = 2e-6 * (np.abs(a.reshape(a_rows, cols)) @ np.abs(deq).T).ravel() + 1e-7
    assert np.all(np.abs(g - r) <= bound)
    # cached weight: a second call with the same key ignores b's bytes
    g2 = backend.mat_mul(a, np.zeros_like(w), t, cols, rows, weight_key=f"w{t}_{a_rows}")
    assert np.array_equal(g, g2)


def test_matmul_f32(backend, oracle):
    rng = np.random.default_rng(2)
    a = rng.standard_normal(2 * 37).astype(np.float32)
    b = rng.standard_normal(37 * 11).astype(np.float32)
    assert np.allclose(backend.mat_mul_f32(a, b, 37, 11), oracle.matmul_f32(a, b, 37, 11), rtol=1e-5, atol=1e-5)
