"""ctypes wrapper of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference arm of bench.py -- never by the product package.
The C source restates llmdot's managed CPU path; see llmdot_oracle.c.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

F32P = C.POINTER(C.c_float)
U8P = C.POINTER(C.c_uint8)
I32P = C.POINTER(C.c_int32)


class OrcConfig(C.Structure):
    """Same field order as llmdot_config in include/llmdot_cuda.h."""
    _fields_ = [
        ("template_id", C.c_int32), ("hidden", C.c_int32), ("layers", C.c_int32), ("context", C.c_int32),
        ("vocab", C.c_int32), ("ffn", C.c_int32), ("heads", C.c_int32), ("heads_kv", C.c_int32),
        ("head_dim", C.c_int32), ("qkv_fused", C.c_int32), ("norm_is_rms", C.c_int32), ("eps", C.c_float),
        ("has_post_norm", C.c_int32), ("rope_base", C.c_float), ("rope_dim", C.c_int32),
        ("rope_scaling", C.c_int32), ("rope_factor", C.c_float), ("ffn_type", C.c_int32),
        ("parallel_residual", C.c_int32), ("tied", C.c_int32), ("emb_scale", C.c_float),
        ("sliding_window", C.c_int32), ("has_attn_cap", C.c_int32), ("attn_cap", C.c_float),
        ("has_final_cap", C.c_int32), ("final_cap", C.c_float), ("expert_count", C.c_int32),
        ("bos", C.c_int32), ("eos", C.c_int32),
    ]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


def build() -> str:
    src = os.path.join(_HERE, "llmdot_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(_LIB_PATH)
        L.orc_half_to_float.restype = C.c_float
        L.orc_half_to_float.argtypes = [C.c_uint32]
        L.orc_byte_count.restype = C.c_uint64
        L.orc_byte_count.argtypes = [C.c_uint32, C.c_uint64]
        L.orc_dequantize.argtypes = [U8P, F32P, C.c_uint32, C.c_int, C.c_int]
        L.orc_matmul.argtypes = [F32P, U8P, F32P, C.c_int, C.c_uint32, C.c_int, C.c_int]
        L.orc_matmul_f32.argtypes = [F32P, F32P, F32P, C.c_int, C.c_int, C.c_int]
        L.orc_exp_approx.restype = C.c_float
        L.orc_exp_approx.argtypes = [C.c_float]
        L.orc_tanh_approx.restype = C.c_float
        L.orc_tanh_approx.argtypes = [C.c_float]
        L.orc_gelu_scalar.restype = C.c_float
        L.orc_gelu_scalar.argtypes = [C.c_float]
        for n in ("orc_silu", "orc_gelu"):
            getattr(L, n).argtypes = [F32P, F32P, C.c_int]
        L.orc_softmax.argtypes = [F32P, C.c_int, C.c_int, C.c_float]
        L.orc_softcap.argtypes = [F32P, C.c_int, C.c_float]
        L.orc_rmsnorm.argtypes = [F32P, F32P, F32P, C.c_int, C.c_float]
        L.orc_layernorm.argtypes = [F32P, F32P, F32P, F32P, C.c_int, C.c_float]
        L.orc_argmax.argtypes = [F32P, C.c_int]
        L.orc_add.argtypes = [F32P, F32P, F32P, C.c_int]
        L.orc_mul.argtypes = [F32P, F32P, F32P, C.c_int]
        L.orc_scale.argtypes = [F32P, C.c_float, F32P, C.c_int]
        L.orc_rope_table.argtypes = [F32P, F32P, C.c_int, C.c_int, F32P, C.c_int]
        L.orc_rope.argtypes = [F32P, F32P, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int]
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_set_kv_fp16.argtypes = [C.c_int]
        L.orc_set_hsum_order.argtypes = [C.c_int]
        L.orc_last_error.restype = C.c_char_p
        L.orc_model_load.restype = C.c_void_p
        L.orc_model_load.argtypes = [C.c_char_p]
        L.orc_model_free.argtypes = [C.c_void_p]
        L.orc_model_config.argtypes = [C.c_void_p, C.POINTER(OrcConfig)]
        L.orc_model_rope_freq.restype = F32P
        L.orc_model_rope_freq.argtypes = [C.c_void_p, C.POINTER(C.c_int)]
        L.orc_session_new.restype = C.c_void_p
        L.orc_session_new.argtypes = [C.c_void_p]
        L.orc_session_free.argtypes = [C.c_void_p]
        L.orc_process_token.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.orc_session_logits.restype = F32P
        L.orc_session_logits.argtypes = [C.c_void_p]
        L.orc_session_hidden.restype = F32P
        L.orc_session_hidden.argtypes = [C.c_void_p]
        L.orc_generate.argtypes = [C.c_void_p, I32P, C.c_int, C.c_int, I32P, F32P]
        L.orc_sample.argtypes = [F32P, C.c_int, C.c_int, C.c_float, C.c_float, C.c_float, C.c_int, I32P, C.c_int,
                                 C.c_float]
        L.orc_net_random_single.restype = C.c_float
        L.orc_net_random_single.argtypes = [C.c_int]
        L.orc_generate_sampled.argtypes = [C.c_void_p, I32P, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float,
                                           C.c_float, C.c_int, F32P, I32P]
        L.orc_session_reset.argtypes = [C.c_void_p]
        L.orc_conv_state_new.restype = C.c_void_p
        L.orc_conv_state_new.argtypes = [C.c_int, C.c_int, C.c_int]
        L.orc_conv_state_free.argtypes = [C.c_void_p]
        L.orc_conv_state_store.argtypes = [C.c_void_p, C.c_int, F32P]
        L.orc_conv_state_build.restype = F32P
        L.orc_conv_state_build.argtypes = [C.c_void_p, C.c_int, F32P, C.c_int]
        L.orc_conv_state_reset.argtypes = [C.c_void_p]
        L.orc_conv1d.argtypes = [F32P, F32P, F32P, C.c_int, C.c_int]
        L.orc_moe_route.argtypes = [F32P, U8P, C.c_uint32, C.c_int, C.c_int, C.c_int, F32P, I32P, F32P]
        L.orc_nucleus.argtypes = [F32P, C.c_int, C.c_float, C.c_int, I32P, F32P]
        _lib = L
    return _lib


def _f(a):
    return a.ctypes.data_as(F32P)


def _u8(a):
    return a.ctypes.data_as(U8P)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def set_kv_fp16(on: bool) -> None:
    """Diagnostic: round cached K/V to fp16 (what a device fp16 KV cache stores)."""
    lib().orc_set_kv_fp16(1 if on else 0)


def set_hsum_order(order: int) -> None:
    """Diagnostic: 0 sums the 8 vector lanes as the pairwise tree the oracle assumes for the
    reference's Vector.Dot, 1 left to right (the order the reference's source does not fix)."""
    lib().orc_set_hsum_order(int(order))


def max_threads() -> int:
    return int(lib().orc_get_max_threads())


def half_to_float(h: int) -> float:
    return lib().orc_half_to_float(h)


def byte_count(t: int, n: int) -> int:
    return int(lib().orc_byte_count(t, n))


def dequantize(src: np.ndarray, ggml_type: int, rows: int, row_elems: int) -> np.ndarray:
    src = np.ascontiguousarray(src, dtype=np.uint8)
    dst = np.empty(rows * row_elems, dtype=np.float32)
    if lib().orc_dequantize(_u8(src), _f(dst), ggml_type, rows, row_elems) != 0:
        raise NotImplementedError(f"type {ggml_type}")
    return dst


def matmul(a: np.ndarray, b: np.ndarray, ggml_type: int, a_cols: int, b_cols: int) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.uint8)
    res = np.empty((a.size // a_cols) * b_cols, dtype=np.float32)
    if lib().orc_matmul(_f(a), _u8(b), _f(res), res.size, ggml_type, a_cols, b_cols) != 0:
        raise NotImplementedError(f"type {ggml_type}")
    return res


def matmul_f32(a, b, a_cols, b_cols):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    res = np.empty((a.size // a_cols) * b_cols, dtype=np.float32)
    lib().orc_matmul_f32(_f(a), _f(b), _f(res), res.size, a_cols, b_cols)
    return res


def exp_approx(x: float) -> float:
    return lib().orc_exp_approx(x)


def tanh_approx(x: float) -> float:
    return lib().orc_tanh_approx(x)


def _unary(name, x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    getattr(lib(), name)(_f(x), _f(out), x.size)
    return out


def silu(x):
    return _unary("orc_silu", x)


def gelu(x):
    return _unary("orc_gelu", x)


def gelu_scalar(x: float) -> float:
    return lib().orc_gelu_scalar(x)


def softmax(x, softcap=None):
    x = np.array(x, dtype=np.float32, copy=True)
    lib().orc_softmax(_f(x), x.size, 1 if softcap is not None else 0, float(softcap or 0.0))
    return x


def softcap(x, cap):
    x = np.array(x, dtype=np.float32, copy=True)
    lib().orc_softcap(_f(x), x.size, float(cap))
    return x


def rmsnorm(x, w, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib().orc_rmsnorm(_f(x), _f(w), _f(out), x.size, eps)
    return out


def layernorm(x, w, b, eps):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    bp = _f(np.ascontiguousarray(b, dtype=np.float32)) if b is not None else None
    lib().orc_layernorm(_f(x), _f(w), bp, _f(out), x.size, eps)
    return out


def argmax(x) -> int:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return int(lib().orc_argmax(_f(x), x.size))


def add(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    out = np.empty_like(a)
    lib().orc_add(_f(a), _f(b), _f(out), a.size)
    return out


def mul(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    out = np.empty_like(a)
    lib().orc_mul(_f(a), _f(b), _f(out), a.size)
    return out


def scale(a, s):
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty_like(a)
    lib().orc_scale(_f(a), float(s), _f(out), a.size)
    return out


def rope_table(q, k, position, freq):
    """ApplyRoPE with a frequency table; q and k are rotated copies (k may be None = same span)."""
    q = np.array(q, dtype=np.float32, copy=True)
    freq = np.ascontiguousarray(freq, dtype=np.float32)
    if k is None:
        lib().orc_rope_table(_f(q), _f(q), 1, position, _f(freq), freq.size)
        return q, None
    k = np.array(k, dtype=np.float32, copy=True)
    lib().orc_rope_table(_f(q), _f(k), 0, position, _f(freq), freq.size)
    return q, k


def rope(q, k, head_dim, position, freq_base, rotary_dim):
    q = np.array(q, dtype=np.float32, copy=True)
    if k is None:
        lib().orc_rope(_f(q), _f(q), 1, head_dim, position, freq_base, rotary_dim)
        return q, None
    k = np.array(k, dtype=np.float32, copy=True)
    lib().orc_rope(_f(q), _f(k), 0, head_dim, position, freq_base, rotary_dim)
    return q, k


class Model:
    """LoadedModel + TransformerConfig restatement over a GGUF file."""

    def __init__(self, path: str):
        self._h = lib().orc_model_load(path.encode())
        if not self._h:
            raise ValueError(lib().orc_last_error().decode())
        c = OrcConfig()
        lib().orc_model_config(self._h, C.byref(c))
        self.config = c.as_dict()
        n = C.c_int()
        p = lib().orc_model_rope_freq(self._h, C.byref(n))
        self.rope_freq = np.ctypeslib.as_array(p, shape=(n.value,)).copy()

    def close(self):
        if self._h:
            lib().orc_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class SamplingOptions:
    """SamplingOptions (src/Llmdot.Core/Sampling/SamplingOptions.cs:7-14), same defaults."""

    def __init__(self, top_k=40, top_p=0.95, temperature=0.8, repeat_penalty=1.1, repeat_window=64, seed=-1):
        self.top_k, self.top_p, self.temperature = int(top_k), float(top_p), float(temperature)
        self.repeat_penalty, self.repeat_window, self.seed = float(repeat_penalty), int(repeat_window), int(seed)


class ConvState:
    """ConvStateCache (src/Llmdot.Core/Inference/ConvStateCache.cs:3-65)."""

    def __init__(self, layers: int, hidden: int, kernel: int):
        self.hidden, self.kernel = hidden, kernel
        self._h = lib().orc_conv_state_new(layers, hidden, kernel)
        if not self._h:
            raise ValueError("bad conv state shape")

    def store(self, layer: int, x) -> None:
        lib().orc_conv_state_store(self._h, layer, _f(np.ascontiguousarray(x, dtype=np.float32)))

    def build_input(self, layer: int, current, position: int) -> np.ndarray:
        cur = np.ascontiguousarray(current, dtype=np.float32)
        p = lib().orc_conv_state_build(self._h, layer, _f(cur), position)
        return np.ctypeslib.as_array(p, shape=(self.kernel * self.hidden,)).copy()

    def reset(self) -> None:
        lib().orc_conv_state_reset(self._h)

    def close(self):
        if self._h:
            lib().orc_conv_state_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def conv1d(x, w, kernel_size: int, dim: int) -> np.ndarray:
    """TensorOps.Conv1D (TensorOps.cs:745-778)."""
    x, w = np.ascontiguousarray(x, dtype=np.float32), np.ascontiguousarray(w, dtype=np.float32)
    out = np.zeros(dim, dtype=np.float32)
    lib().orc_conv1d(_f(x), _f(w), _f(out), kernel_size, dim)
    return out


def moe_route(hidden_state, gate: np.ndarray, gate_type: int, experts: int, top_k: int):
    """MoeRouter.Route (MoeRouter.cs:12-59): (gate logits, selected experts, routing weights)."""
    h = np.ascontiguousarray(hidden_state, dtype=np.float32)
    g = np.ascontiguousarray(gate).view(np.uint8)
    logits = np.zeros(experts, dtype=np.float32)
    sel = np.zeros(max(top_k, 1), dtype=np.int32)
    w = np.zeros(max(top_k, 1), dtype=np.float32)
    if lib().orc_moe_route(_f(h), _u8(g), gate_type, h.size, experts, top_k, _f(logits), sel.ctypes.data_as(I32P),
                           _f(w)) != 0:
        raise ValueError("unsupported gate type")
    return logits, sel[:top_k], w[:top_k]


def nucleus(p, top_p: float, fast: bool):
    """FindNucleus (Sampler.cs:129-151) on a copy of p, literally (quadratic selection sort) or
    by the sort-and-replay form: (count, idx[:count], the buffer after its aliased writes)."""
    p = np.ascontiguousarray(p, dtype=np.float32)
    idx = np.zeros(max(p.size, 1), dtype=np.int32)
    buf = np.zeros(max(p.size, 1), dtype=np.float32)
    n = lib().orc_nucleus(_f(p), p.size, top_p, 1 if fast else 0, idx.ctypes.data_as(I32P), _f(buf))
    return n, idx[:n], buf[:p.size]


def net_random_single(seed: int) -> float:
    """new System.Random(seed).NextSingle() (restated, see the C source)."""
    return float(lib().orc_net_random_single(int(seed)))


def sample(logits, opts: SamplingOptions, recent=(), r: float = None) -> int:
    """Sampler.Sample (Sampler.cs:24-62).  r defaults to the seeded draw (opts.seed >= 0)."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    rec = np.ascontiguousarray(recent, dtype=np.int32)
    if r is None:
        if opts.seed < 0:
            raise ValueError("an unseeded draw needs r")
        r = net_random_single(opts.seed)
    return int(lib().orc_sample(_f(x), x.size, opts.top_k, opts.top_p, opts.temperature, opts.repeat_penalty,
                                opts.repeat_window, rec.ctypes.data_as(I32P), rec.size, float(r)))


class Session:
    """One InferenceEngine's KvCache + buffers over a Model."""

    def __init__(self, model: Model):
        self.model = model
        self._h = lib().orc_session_new(model._h)
        if not self._h:
            raise MemoryError(lib().orc_last_error().decode())

    def reset(self) -> None:
        """Generate's KvCache / ConvStateCache reset (InferenceEngine.cs:79-80)."""
        lib().orc_session_reset(self._h)

    def process_token(self, token: int, position: int) -> np.ndarray:
        if lib().orc_process_token(self._h, int(token), int(position)) != 0:
            raise RuntimeError(lib().orc_last_error().decode())
        V = self.model.config["vocab"]
        return np.ctypeslib.as_array(lib().orc_session_logits(self._h), shape=(V,)).copy()

    def generate_sampled(self, prompt, max_tokens: int, opts: SamplingOptions, r=None):
        """Generate with Sampler.Sample; r[i] is the draw for token i (the seeded draw when omitted)."""
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        if r is None:
            r = np.full(max(max_tokens, 1), net_random_single(opts.seed), dtype=np.float32)
        r = np.ascontiguousarray(r, dtype=np.float32)
        out = np.zeros(max(max_tokens, 1), dtype=np.int32)
        n = lib().orc_generate_sampled(self._h, prompt.ctypes.data_as(I32P), prompt.size, max_tokens, opts.top_k,
                                       opts.top_p, opts.temperature, opts.repeat_penalty, opts.repeat_window, _f(r),
                                       out.ctypes.data_as(I32P))
        if n < 0:
            raise RuntimeError(lib().orc_last_error().decode())
        return out[:n]

    def generate(self, prompt, max_tokens: int, want_logits: bool = False):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max_tokens, dtype=np.int32)
        V = self.model.config["vocab"]
        logits = np.zeros((max_tokens, V), dtype=np.float32) if want_logits else None
        n = lib().orc_generate(self._h, prompt.ctypes.data_as(I32P), prompt.size, max_tokens,
                               out.ctypes.data_as(I32P), _f(logits) if logits is not None else None)
        if n < 0:
            raise RuntimeError(lib().orc_last_error().decode())
        return (out[:n], logits[:n] if logits is not None else None)

    def close(self):
        if self._h:
            lib().orc_session_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
