"""CudaBackend: the per-operation adapter, one method per IComputeBackend member
(src/Llmdot.Core/Inference/Backends/IComputeBackend.cs:7-28), over the C ABI.

Arguments and results are host numpy arrays (the interface passes host spans);
each call copies to the device, runs the kernel and copies back.  Weights are
cached on the device under their ``weight_key`` like the reference's Metal
backend does.  Method names follow the C# interface in snake_case.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from .native import F32P, I32P, U8P, VP, check, lib


def _f(a: np.ndarray):
    return a.ctypes.data_as(F32P)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _need(name: str, a: np.ndarray, n: int) -> None:
    """The C entry points take one length for all their spans and read that many elements of
    each; a shorter host array would be read past its end (the C# spans throw instead)."""
    if a.size < n:
        raise ValueError(f"{name}: {a.size} elements, {n} needed")


def _inplace(name: str, a) -> None:
    if not (isinstance(a, np.ndarray) and a.dtype == np.float32 and a.flags.c_contiguous and a.flags.writeable):
        raise TypeError(f"{name}: needs a writeable C-contiguous float32 array")


class CudaBackend:
    def __init__(self, device: int = 0):
        self._h = VP()
        check(lib().llmdot_cuda_create(device, C.byref(self._h)))

    def dispose(self) -> None:
        if self._h:
            lib().llmdot_cuda_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass

    # MatMul(a, b, result, bType, aCols, bCols, weightKey)
    def mat_mul(self, a, b, b_type: int, a_cols: int, b_cols: int, weight_key: Optional[str] = None,
                result_len: Optional[int] = None) -> np.ndarray:
        a = _f32(a)
        b = np.ascontiguousarray(b, dtype=np.uint8)
        n = result_len if result_len is not None else (a.size // a_cols) * b_cols
        res = np.empty(n, dtype=np.float32)
        check(lib().llmdot_cuda_matmul(self._h, _f(a), a.size, b.ctypes.data_as(U8P), b.nbytes, b_type, a_cols, b_cols,
                                       weight_key.encode() if weight_key else None, _f(res), res.size))
        return res

    def mat_mul_f32(self, a, b, a_cols: int, b_cols: int, weight_key: Optional[str] = None) -> np.ndarray:
        a, b = _f32(a), _f32(b)
        res = np.empty((a.size // a_cols) * b_cols, dtype=np.float32)
        check(lib().llmdot_cuda_matmul_f32(self._h, _f(a), a.size, _f(b), b.size, a_cols, b_cols,
                                           weight_key.encode() if weight_key else None, _f(res), res.size))
        return res

    def rms_norm(self, x, w, eps: float) -> np.ndarray:
        x, w = _f32(x), _f32(w)
        _need("rms_norm weight", w, x.size)
        out = np.empty_like(x)
        check(lib().llmdot_cuda_rmsnorm(self._h, _f(x), _f(w), _f(out), x.size, eps))
        return out

    def layer_norm(self, x, w, bias, eps: float) -> np.ndarray:
        x, w = _f32(x), _f32(w)
        _need("layer_norm weight", w, x.size)
        out = np.empty_like(x)
        b = _f32(bias) if bias is not None and len(bias) else None
        if b is not None:
            _need("layer_norm bias", b, x.size)
        check(lib().llmdot_cuda_layernorm(self._h, _f(x), _f(w), _f(b) if b is not None else None, _f(out), x.size, eps))
        return out

    def apply_rope(self, q, k, head_dim: int, position: int, freq_base: float, rotary_dim: int):
        """ApplyRoPE(query, key, headDim, position, freqBase, rotaryDim); k=None means same span."""
        q = np.array(q, dtype=np.float32, copy=True)
        kk = q if k is None else np.array(k, dtype=np.float32, copy=True)
        check(lib().llmdot_cuda_rope(self._h, _f(q), q.size, _f(kk), kk.size, head_dim, position, freq_base, rotary_dim))
        return q, (None if k is None else kk)

    def apply_rope_table(self, q, k, head_dim: int, position: int, freq_table):
        q = np.array(q, dtype=np.float32, copy=True)
        kk = q if k is None else np.array(k, dtype=np.float32, copy=True)
        ft = _f32(freq_table)
        check(lib().llmdot_cuda_rope_table(self._h, _f(q), q.size, _f(kk), kk.size, head_dim, position, _f(ft), ft.size))
        return q, (None if k is None else kk)

    def softmax(self, x, softcap: Optional[float] = None) -> np.ndarray:
        x = np.array(x, dtype=np.float32, copy=True)
        check(lib().llmdot_cuda_softmax(self._h, _f(x), x.size, 0 if softcap is None else 1, float(softcap or 0.0)))
        return x

    def silu(self, x) -> np.ndarray:
        x = _f32(x)
        out = np.empty_like(x)
        check(lib().llmdot_cuda_silu(self._h, _f(x), _f(out), x.size))
        return out

    def silu_in_place(self, x: np.ndarray) -> None:
        _inplace("silu_in_place", x)
        check(lib().llmdot_cuda_silu_inplace(self._h, _f(x), x.size))

    def gelu(self, x) -> np.ndarray:
        x = _f32(x)
        out = np.empty_like(x)
        check(lib().llmdot_cuda_gelu(self._h, _f(x), _f(out), x.size))
        return out

    def gelu_scalar(self, x: float) -> float:
        r = C.c_float()
        check(lib().llmdot_cuda_gelu_scalar(self._h, x, C.byref(r)))
        return r.value

    def add(self, a, b) -> np.ndarray:
        a, b = _f32(a), _f32(b)
        _need("add b", b, a.size)
        out = np.empty_like(a)
        check(lib().llmdot_cuda_add(self._h, _f(a), _f(b), _f(out), a.size))
        return out

    def add_in_place(self, a: np.ndarray, b) -> None:
        _inplace("add_in_place", a)
        b = _f32(b)
        _need("add_in_place b", b, a.size)
        check(lib().llmdot_cuda_add_inplace(self._h, _f(a), _f(b), a.size))

    def scale(self, x, s: float) -> np.ndarray:
        x = _f32(x)
        out = np.empty_like(x)
        check(lib().llmdot_cuda_scale(self._h, _f(x), s, _f(out), x.size))
        return out

    def scale_in_place(self, x: np.ndarray, s: float) -> None:
        _inplace("scale_in_place", x)
        check(lib().llmdot_cuda_scale_inplace(self._h, _f(x), x.size, s))

    def mul(self, a, b) -> np.ndarray:
        a, b = _f32(a), _f32(b)
        _need("mul b", b, a.size)
        out = np.empty_like(a)
        check(lib().llmdot_cuda_mul(self._h, _f(a), _f(b), _f(out), a.size))
        return out

    def softcap(self, x, cap: float) -> np.ndarray:
        x = np.array(x, dtype=np.float32, copy=True)
        check(lib().llmdot_cuda_softcap(self._h, _f(x), x.size, cap))
        return x

    def conv1d(self, x, w, kernel_size: int, input_dim: int) -> np.ndarray:
        x, w = _f32(x), _f32(w)
        span = input_dim if kernel_size == 1 else kernel_size * input_dim
        _need("conv1d input", x, span)
        _need("conv1d weights", w, span)
        out = np.empty(input_dim, dtype=np.float32)
        check(lib().llmdot_cuda_conv1d(self._h, _f(x), _f(w), _f(out), kernel_size, input_dim))
        return out

    def dequantize_to_float(self, src, ggml_type: int, num_rows: int, row_elements: int) -> np.ndarray:
        src = np.ascontiguousarray(src, dtype=np.uint8)
        dst = np.empty(num_rows * row_elements, dtype=np.float32)
        check(lib().llmdot_cuda_dequantize(self._h, src.ctypes.data_as(U8P), src.nbytes, ggml_type, num_rows,
                                           row_elements, _f(dst)))
        return dst

    def arg_max(self, x) -> int:
        x = _f32(x)
        r = C.c_int()
        check(lib().llmdot_cuda_argmax(self._h, _f(x), x.size, C.byref(r)))
        return r.value

    def sample(self, logits, options, recent=(), r=None) -> int:
        """Sampler.Sample (Sampler.cs:24-62) on the device.  options: native.LlmdotSampling;
        r: the uniform draw (the seeded draw of options.seed when omitted and seed >= 0)."""
        from .native import LlmdotSampling
        x = _f32(logits)
        rec = np.ascontiguousarray(recent, dtype=np.int32)
        if r is None:
            if options.seed < 0:
                raise ValueError("an unseeded sample needs its draw r")
            r = lib().llmdot_cuda_sampling_seeded_draw(options.seed)
        out = C.c_int32()
        o = LlmdotSampling(options.top_k, options.top_p, options.temperature, options.repeat_penalty,
                           options.repeat_window, options.seed)
        check(lib().llmdot_cuda_sample(self._h, _f(x), x.size, C.byref(o), rec.ctypes.data_as(I32P), rec.size,
                                       float(r), C.byref(out)))
        return out.value


class Sampler:
    """Sampler (src/Llmdot.Core/Sampling/Sampler.cs:11-165) over a CudaBackend: ``sample(logits,
    options, recent_tokens)`` with the reference's draw -- ``new Random(seed).NextSingle()`` when
    seed >= 0 (the same draw for every call, as the reference re-seeds per call), a fresh uniform
    draw otherwise.  Option sets the device refuses (the top-p-only branch) raise CudaBackendError."""

    def __init__(self, backend: "CudaBackend"):
        import random
        self._backend = backend
        self._rng = random.Random()

    def sample(self, logits, options, recent_tokens=()) -> int:
        r = None if options.seed >= 0 else self._rng.random()
        return self._backend.sample(logits, options, recent_tokens, r)
