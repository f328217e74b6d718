"""The decode step's quantised matvec (tensor-core path for Q4_K / Q6_K, generic
kernel otherwise) against the oracle's restatement of TensorOps.MatMul, on every
weight matrix of the small synthetic models.

Bound: the device and the reference both sum in fp32 but in different orders,
and the device feeds the tensor cores an exact fp16 hi/lo split of x; the
difference is bounded by 4e-6 * sum_i |x_i * w_i| per output (a few fp32 ulps of
the absolute sum).
"""
import numpy as np
import pytest

from dotllm_b200 import gguf, synth
from dotllm_b200.engine import CudaModel

pytestmark = pytest.mark.gpu

_cache = {}


def loaded(name):
    if name not in _cache:
        path = synth.build_model(synth.get(name))
        _cache[name] = (CudaModel.load(path), gguf.GgufFile(path))
    return _cache[name]


def bound(x, deq):
    return 4e-6 * (np.abs(x) @ np.abs(deq).T) + 1e-6


@pytest.mark.parametrize("name", ["micro", "micro-gemma", "micro-phi3", "tiny"])
@pytest.mark.parametrize("nv", [1, 2, 3, 4])
def test_matvec_every_weight(oracle, name, nv):
    m, f = loaded(name)
    rng = np.random.default_rng(nv)
    for tname, info in f.tensors.items():
        if len(info.dims) != 2 or info.ggml_type not in (gguf.GGML_Q4_K, gguf.GGML_Q6_K, gguf.GGML_Q5_K,
                                                          gguf.GGML_Q8_0):
            continue
        cols, rows = info.dims
        raw = np.array(f.tensor_bytes(tname))
        x = rng.standard_normal((nv, cols)).astype(np.float32)
        x[0, :7] *= 1e-4  # a few tiny entries (exercise the fp16 hi/lo split)
        y = m.matvec(tname, x, rows, mode=0)
        deq = oracle.dequantize(raw, info.ggml_type, rows, cols).reshape(rows, cols)
        for v in range(nv):
            ref = oracle.matmul(x[v], raw, info.ggml_type, cols, rows)
            err = np.abs(y[v] - ref)
            assert np.all(err <= bound(x[v:v + 1], deq)[0]), f"{tname} v={v}: max err {err.max()}"


@pytest.mark.parametrize("name", ["micro", "micro-phi3", "tiny"])
@pytest.mark.parametrize("nv", [5, 8, 13, 32])
def test_matmul_batched_every_weight(oracle, name, nv):
    """5..32 input rows: the batched tensor-core kernel (gemm_tc.cu) on every Q4_K / Q6_K matrix."""
    m, f = loaded(name)
    rng = np.random.default_rng(100 + nv)
    for tname, info in f.tensors.items():
        if len(info.dims) != 2 or info.ggml_type not in (gguf.GGML_Q4_K, gguf.GGML_Q6_K):
            continue
        cols, rows = info.dims
        raw = np.array(f.tensor_bytes(tname))
        x = rng.standard_normal((nv, cols)).astype(np.float32)
        x[nv - 1] *= 1e-3  # rows of very different scale in one batch
        y = m.matvec(tname, x, rows, mode=0)
        deq = oracle.dequantize(raw, info.ggml_type, rows, cols).reshape(rows, cols)
        for v in range(nv):
            ref = oracle.matmul(x[v], raw, info.ggml_type, cols, rows)
            err = np.abs(y[v] - ref)
            assert np.all(err <= bound(x[v:v + 1], deq)[0]), f"{tname} v={v}: max err {err.max()}"


def test_matmul_batched_fused_rmsnorm(oracle):
    name = "tiny"
    m, f = loaded(name)
    cfg = synth.get(name)
    rng = np.random.default_rng(6)
    wn = (1 + 0.01 * rng.standard_normal(cfg.hidden)).astype(np.float32)
    for tname in ("blk.0.attn_v.weight", "blk.1.ffn_up.weight", "output.weight"):
        info = f.tensors[tname]
        cols, rows = info.dims
        raw = np.array(f.tensor_bytes(tname))
        h = (rng.standard_normal((7, cols)) * 3).astype(np.float32)
        y = m.matvec(tname, h, rows, mode=2, norm_w=wn)
        deq = oracle.dequantize(raw, info.ggml_type, rows, cols).reshape(rows, cols)
        for v in range(7):
            xn = oracle.rmsnorm(h[v], wn, cfg.eps)
            ref = oracle.matmul(xn, raw, info.ggml_type, cols, rows)
            assert np.all(np.abs(y[v] - ref) <= bound(xn[None], deq)[0] + 1e-6)


@pytest.mark.parametrize("name", ["micro", "tiny"])
def test_matvec_fused_rmsnorm(oracle, name):
    m, f = loaded(name)
    cfg = synth.get(name)
    rng = np.random.default_rng(5)
    wn = (1 + 0.01 * rng.standard_normal(cfg.hidden)).astype(np.float32)
    for tname in ("blk.0.attn_q.weight", "blk.1.ffn_gate.weight", "token_embd.weight"):
        info = f.tensors[tname]
        cols, rows = info.dims
        raw = np.array(f.tensor_bytes(tname))
        h = (rng.standard_normal((2, cols)) * 3).astype(np.float32)
        y = m.matvec(tname, h, rows, mode=2, norm_w=wn)
        deq = oracle.dequantize(raw, info.ggml_type, rows, cols).reshape(rows, cols)
        for v in range(2):
            xn = oracle.rmsnorm(h[v], wn, cfg.eps)
            ref = oracle.matmul(xn, raw, info.ggml_type, cols, rows)
            assert np.all(np.abs(y[v] - ref) <= bound(xn[None], deq)[0] + 1e-6)


def test_matvec_fast_matches_generic(oracle):
    m, f = loaded("tiny")
    rng = np.random.default_rng(9)
    for tname in ("blk.2.ffn_down.weight", "output.weight", "blk.3.attn_v.weight"):
        info = f.tensors[tname]
        cols, rows = info.dims
        x = rng.standard_normal((1, cols)).astype(np.float32)
        a = m.matvec(tname, x, rows, mode=0)
        b = m.matvec(tname, x, rows, mode=1)
        raw = np.array(f.tensor_bytes(tname))
        deq = oracle.dequantize(raw, info.ggml_type, rows, cols).reshape(rows, cols)
        assert np.all(np.abs(a - b) <= 2 * bound(x, deq))


def test_matvec_extreme_inputs(oracle):
    """Large and tiny magnitudes, exact zeros: the power-of-two pre-scaling keeps fp16 in range."""
    m, f = loaded("micro")
    tname = "blk.0.ffn_gate.weight"
    info = f.tensors[tname]
    cols, rows = info.dims
    raw = np.array(f.tensor_bytes(tname))
    deq = oracle.dequantize(raw, info.ggml_type, rows, cols).reshape(rows, cols)
    for scale in (1e-30, 1e-6, 1e4, 1e20):
        x = (np.random.default_rng(1).standard_normal((1, cols)) * scale).astype(np.float32)
        y = m.matvec(tname, x, rows)
        ref = oracle.matmul(x[0], raw, info.ggml_type, cols, rows)
        assert np.all(np.abs(y[0] - ref) <= bound(x, deq)[0])
    y = m.matvec(tname, np.zeros((1, cols), dtype=np.float32), rows)
    assert np.all(y == 0)
