"""Pin the CPU oracle against the reference's own unit-test expectations.

Each test restates one assertion from tests/Llmdot.Core.Tests (file:line given)
against the oracle, which is the checker for every GPU parity test.
"""
import math

import numpy as np
import pytest

from dotllm_b200 import gguf


def test_dequant_q4_0_all_minus8(oracle):  # Tensors/DequantizeTests.cs:25-42
    src = np.zeros(36, dtype=np.uint8)
    src[0:2] = [0x00, 0x3C]
    src[18:20] = [0x00, 0x3C]
    out = oracle.dequantize(src, gguf.GGML_Q4_0, 1, 64)
    assert np.all(out == -8.0)


def test_dequant_q8_0_zeros(oracle):  # DequantizeTests.cs:44-61
    src = np.zeros(68, dtype=np.uint8)
    src[0:2] = [0x00, 0x3C]
    src[34:36] = [0x00, 0x3C]
    assert np.all(oracle.dequantize(src, gguf.GGML_Q8_0, 1, 64) == 0.0)


def test_f16_known_values(oracle):  # DequantizeTests.cs:63-70
    assert oracle.half_to_float(0x3C00) == 1.0
    assert oracle.half_to_float(0xBC00) == -1.0
    assert oracle.half_to_float(0x3800) == 0.5
    assert oracle.half_to_float(0x0000) == 0.0


def test_f16_subnormal_and_specials(oracle):  # HalfHelper.cs:7-40
    assert oracle.half_to_float(0x0001) == 2.0 ** -24
    assert oracle.half_to_float(0x03FF) == 1023 * 2.0 ** -24
    assert oracle.half_to_float(0x7C00) == math.inf
    assert oracle.half_to_float(0xFC00) == -math.inf
    assert math.isnan(oracle.half_to_float(0x7E00))
    assert math.copysign(1.0, oracle.half_to_float(0x8000)) == -1.0


def test_bf16_known_values(oracle):  # DequantizeTests.cs:72-89
    out = oracle.dequantize(np.array([0x80, 0x3F, 0x00, 0x40, 0x80, 0xBF], dtype=np.uint8), gguf.GGML_BF16, 1, 3)
    assert list(out) == [1.0, 2.0, -1.0]


def test_f32_identity(oracle):  # DequantizeTests.cs:12-23
    v = np.array([1.0, -2.5, 3.14, 0.0], dtype=np.float32)
    assert np.array_equal(oracle.dequantize(v.view(np.uint8), gguf.GGML_F32, 1, 4), v)


def test_matmul_f32_identity(oracle):  # Tensors/TensorOpsTests.cs:8-19
    r = oracle.matmul_f32([1, 2, 3], [1, 0, 0, 0, 1, 0, 0, 0, 1], 3, 3)
    assert list(r) == [1, 2, 3]


def test_matmul_f32_2x3(oracle):  # TensorOpsTests.cs:21-33
    r = oracle.matmul_f32([1, 2, 3, 4, 5, 6], [7, 8, 9, 10, 11, 12], 3, 2)
    assert np.allclose(r, [50, 68, 122, 167], atol=1e-3)


def test_rope_modifies(oracle):  # TensorOpsTests.cs:35-46
    q, k = oracle.rope(np.ones(128), np.ones(128), 128, 1, 10000.0, 128)
    assert q[64] != 1.0 and k[64] != 1.0


def test_rope_position_zero(oracle):  # TensorOpsTests.cs:48-61
    q, k = oracle.rope([1, 0, 1, 0], [1, 0, 1, 0], 4, 0, 10000.0, 4)
    assert abs(q[0] - 1) < 1e-3 and abs(q[1]) < 1e-3 and abs(k[0] - 1) < 1e-3


def test_rope_same_span(oracle):  # TensorOpsTests.cs:63-81
    a, _ = oracle.rope(np.ones(128), None, 128, 1, 10000.0, 128)
    q, _ = oracle.rope(np.ones(128), np.ones(128), 128, 1, 10000.0, 128)
    assert np.allclose(a, q, atol=1e-4)


def test_rmsnorm_3_4(oracle):  # Tensors/VectorMathTests.cs:9-20
    out = oracle.rmsnorm([3, 4], [1, 1], 1e-5)
    mag = math.sqrt((9 + 16) / 2 + 1e-5)
    assert abs(out[0] - 3 / mag) < 1e-3 and abs(out[1] - 4 / mag) < 1e-3


def test_layernorm_zero_mean(oracle):  # VectorMathTests.cs:22-35
    out = oracle.layernorm([1, 2, 3], [1, 1, 1], [0, 0, 0], 1e-5)
    assert abs(out.mean()) < 0.01


def test_softmax_sums_to_one(oracle):  # VectorMathTests.cs:37-46
    assert abs(oracle.softmax([1, 2, 3, 4]).sum() - 1) < 1e-3


def test_softmax_softcap_sums_to_one(oracle):  # VectorMathTests.cs:48-56
    assert abs(oracle.softmax([10, 20, 30, 40], softcap=5.0).sum() - 1) < 1e-3


def test_silu_zero_and_large(oracle):  # VectorMathTests.cs:58-78
    assert abs(oracle.silu([0.0])[0]) < 1e-3
    assert abs(oracle.silu([100.0])[0] - 100) < 0.1


def test_argmax(oracle):  # VectorMathTests.cs:80-86
    assert oracle.argmax([1, 5, 3, 2]) == 1


def test_argmax_ties_lowest_index(oracle):  # VectorMath.cs:412-425 (strict >)
    assert oracle.argmax([1, 7, 7, 2]) == 1


# VectorMath.ArgMax (VectorMath.cs:412-425) starts from element 0 and moves only on `>`: a NaN never
# becomes the maximum, a NaN at element 0 is never replaced, and -0 / +0 compare equal.
ARGMAX_SPECIAL = [
    ([1.0, float("nan"), 3.0, 2.0], 2),
    ([float("nan"), 1.0, 5.0, float("inf")], 0),
    ([1.0, float("nan"), float("nan")], 0),
    ([-0.0, 0.0, -1.0], 0),
    ([-1.0, 0.0, -0.0], 1),
    ([-1.0, -0.0, 0.0], 1),
    ([float("-inf"), float("-inf"), -3.0], 2),
    ([float("-inf"), float("nan"), float("-inf")], 0),
    ([2.0, float("inf"), float("nan"), float("inf")], 1),
]


@pytest.mark.parametrize("row,want", ARGMAX_SPECIAL)
def test_argmax_special_values(oracle, row, want):
    assert oracle.argmax(np.array(row, dtype=np.float32)) == want


def test_add_scale_mul(oracle):  # VectorMathTests.cs:88-108, VectorMathExtendedTests.cs:50-80
    assert list(oracle.add([1, 2, 3], [4, 5, 6])) == [5, 7, 9]
    assert list(oracle.scale([1, 2, 3], 2.0)) == [2, 4, 6]
    assert list(oracle.mul([1, 2, 3, 4], [5, 6, 7, 8])) == [5, 12, 21, 32]


def test_silu_vector_matches_tail(oracle):  # VectorMathExtendedTests.cs:10-20
    x = np.array([-3, -1, 0, 0.5, 1, 2, 5, 10], dtype=np.float32)
    a = oracle.silu(x)
    b = np.array([oracle.silu(np.array([v], dtype=np.float32))[0] for v in x])  # tail lanes (MathF.Exp)
    # the 8-wide vector lanes use the reference's ExpApprox; its error is what the
    # reference's own test tolerates only loosely, so compare at that scale
    assert np.allclose(a, b, atol=0.1)


def test_gelu_vector_vs_scalar(oracle):  # VectorMathExtendedTests.cs:22-32 (tol 0.05)
    x = np.array([-1, 0, 0.5, 1, -1, 0, 0.5, 1], dtype=np.float32)
    v = oracle.gelu(x)
    for i, xi in enumerate(x):
        assert abs(v[i] - oracle.gelu_scalar(float(xi))) < 0.05


def test_gelu_scalar_signs(oracle):  # VectorMathExtendedTests.cs:34-48
    assert abs(oracle.gelu_scalar(0.0)) < 1e-4
    assert 0 < oracle.gelu_scalar(1.0) < 1
    assert -1 < oracle.gelu_scalar(-1.0) < 0


def test_softcap_vs_tanh(oracle):  # VectorMathExtendedTests.cs:84-96 (tol 0.05)
    vals = np.array([-2, 0, 1, 2, -2, 0, 1, 2], dtype=np.float32)
    out = oracle.softcap(vals, 3.0)
    assert np.allclose(out, 3 * np.tanh(vals / 3), atol=0.05)


@pytest.mark.parametrize("t,n,expected", [(gguf.GGML_F32, 1024, 4096), (gguf.GGML_F16, 1024, 2048),
                                          (gguf.GGML_Q8_0, 256, 272), (gguf.GGML_Q4_0, 256, 144)])
def test_tensor_size(oracle, t, n, expected):  # Tensors/TensorSizeTests.cs:9-19
    assert oracle.byte_count(t, n) == expected
    assert gguf.byte_count(t, n) == expected


def test_tensor_size_unsupported():  # TensorSizeTests.cs:21-25
    with pytest.raises(NotImplementedError):
        gguf.byte_count(999, 1024)


def test_exp_approx_known_points(oracle):
    """ExpApprox (VectorMath.cs:137-166): exact at 0, clamps, and its known
    negative-argument error (y^4/10 Pade-like polynomial with truncating k)."""
    assert oracle.exp_approx(0.0) == 1.0
    assert oracle.exp_approx(-100.0) == 0.0
    assert oracle.exp_approx(100.0) == math.inf
    assert abs(oracle.exp_approx(-1.0) - (1 - 1 + 0.5 - 1 / 6 + 0.1)) < 1e-6


def test_tanh_approx_known_points(oracle):  # VectorMath.cs:196-209
    assert oracle.tanh_approx(5.0) == 1.0 and oracle.tanh_approx(-5.0) == -1.0
    assert abs(oracle.tanh_approx(1.0) - 28 / 36) < 1e-7
    assert oracle.tanh_approx(0.0) == 0.0
