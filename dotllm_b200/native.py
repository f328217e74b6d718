"""ctypes binding of libllmdot_cuda.so (the C ABI in include/llmdot_cuda.h).

The library is built in-tree (``make -C dotllm_b200/csrc``); importing this
module never falls back to a CPU implementation: a missing library or a
failing call raises ``CudaBackendError`` with the native status and message.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from typing import Dict, List

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libllmdot_cuda.so")
HEADER = os.path.join(os.path.dirname(_HERE), "include", "llmdot_cuda.h")

STATUS = {0: "OK", -1: "INVALID", -2: "UNSUPPORTED", -3: "CUDA", -4: "NOMEM", -5: "FORMAT", -6: "NCCL", -7: "TIMEOUT"}
KV_F16, KV_F32 = 0, 1


class CudaBackendError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"llmdot_cuda status {status} ({STATUS.get(status, '?')}): {message}")
        self.status = status
        self.message = message


class LlmdotConfig(C.Structure):
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

    def as_dict(self) -> Dict[str, float]:
        return {k: getattr(self, k) for k, _ in self._fields_}


class TensorDesc(C.Structure):
    _fields_ = [("name", C.c_char_p), ("type", C.c_uint32), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 4),
                ("data", C.c_void_p), ("n_bytes", C.c_uint64)]


class LlmdotSampling(C.Structure):
    """llmdot_sampling = SamplingOptions (SamplingOptions.cs:7-14), the reference's defaults."""
    _fields_ = [("top_k", C.c_int32), ("top_p", C.c_float), ("temperature", C.c_float),
                ("repeat_penalty", C.c_float), ("repeat_window", C.c_int32), ("seed", C.c_int32)]

    def __init__(self, top_k=40, top_p=0.95, temperature=0.8, repeat_penalty=1.1, repeat_window=64, seed=-1):
        super().__init__(top_k, top_p, temperature, repeat_penalty, repeat_window, seed)


F32P = C.POINTER(C.c_float)
U8P = C.POINTER(C.c_uint8)
I32P = C.POINTER(C.c_int32)
VP = C.c_void_p

# name -> (restype, argtypes)
_SIGS = {
    "llmdot_cuda_last_error": (C.c_char_p, []),
    "llmdot_cuda_version": (C.c_char_p, []),
    "llmdot_cuda_device_count": (C.c_int, [C.POINTER(C.c_int)]),
    "llmdot_cuda_create": (C.c_int, [C.c_int, C.POINTER(VP)]),
    "llmdot_cuda_destroy": (C.c_int, [VP]),
    "llmdot_cuda_matmul": (C.c_int, [VP, F32P, C.c_int, U8P, C.c_size_t, C.c_uint32, C.c_int, C.c_int, C.c_char_p, F32P, C.c_int]),
    "llmdot_cuda_matmul_f32": (C.c_int, [VP, F32P, C.c_int, F32P, C.c_size_t, C.c_int, C.c_int, C.c_char_p, F32P, C.c_int]),
    "llmdot_cuda_rmsnorm": (C.c_int, [VP, F32P, F32P, F32P, C.c_int, C.c_float]),
    "llmdot_cuda_layernorm": (C.c_int, [VP, F32P, F32P, F32P, F32P, C.c_int, C.c_float]),
    "llmdot_cuda_rope": (C.c_int, [VP, F32P, C.c_int, F32P, C.c_int, C.c_int, C.c_int, C.c_float, C.c_int]),
    "llmdot_cuda_rope_table": (C.c_int, [VP, F32P, C.c_int, F32P, C.c_int, C.c_int, C.c_int, F32P, C.c_int]),
    "llmdot_cuda_softmax": (C.c_int, [VP, F32P, C.c_int, C.c_int, C.c_float]),
    "llmdot_cuda_silu": (C.c_int, [VP, F32P, F32P, C.c_int]),
    "llmdot_cuda_silu_inplace": (C.c_int, [VP, F32P, C.c_int]),
    "llmdot_cuda_gelu": (C.c_int, [VP, F32P, F32P, C.c_int]),
    "llmdot_cuda_gelu_scalar": (C.c_int, [VP, C.c_float, F32P]),
    "llmdot_cuda_add_inplace": (C.c_int, [VP, F32P, F32P, C.c_int]),
    "llmdot_cuda_add": (C.c_int, [VP, F32P, F32P, F32P, C.c_int]),
    "llmdot_cuda_scale": (C.c_int, [VP, F32P, C.c_float, F32P, C.c_int]),
    "llmdot_cuda_scale_inplace": (C.c_int, [VP, F32P, C.c_int, C.c_float]),
    "llmdot_cuda_mul": (C.c_int, [VP, F32P, F32P, F32P, C.c_int]),
    "llmdot_cuda_softcap": (C.c_int, [VP, F32P, C.c_int, C.c_float]),
    "llmdot_cuda_conv1d": (C.c_int, [VP, F32P, F32P, F32P, C.c_int, C.c_int]),
    "llmdot_cuda_dequantize": (C.c_int, [VP, U8P, C.c_size_t, C.c_uint32, C.c_int, C.c_int, F32P]),
    "llmdot_cuda_argmax": (C.c_int, [VP, F32P, C.c_int, C.POINTER(C.c_int)]),
    "llmdot_cuda_model_load": (C.c_int, [C.c_int, C.POINTER(LlmdotConfig), C.POINTER(TensorDesc), C.c_int, C.POINTER(VP)]),
    "llmdot_cuda_model_load_gguf": (C.c_int, [C.c_int, C.c_char_p, C.POINTER(VP)]),
    "llmdot_cuda_model_config": (C.c_int, [VP, C.POINTER(LlmdotConfig)]),
    "llmdot_cuda_gguf_config": (C.c_int, [C.c_char_p, C.POINTER(LlmdotConfig)]),
    "llmdot_cuda_model_weight_bytes": (C.c_int, [VP, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "llmdot_cuda_model_free": (C.c_int, [VP]),
    "llmdot_cuda_session_create": (C.c_int, [VP, C.c_int, C.c_int, C.POINTER(VP)]),
    "llmdot_cuda_session_reset": (C.c_int, [VP]),
    "llmdot_cuda_session_position": (C.c_int, [VP, C.POINTER(C.c_int)]),
    "llmdot_cuda_session_free": (C.c_int, [VP]),
    "llmdot_cuda_prefill": (C.c_int, [VP, I32P, C.c_int, F32P, I32P]),
    "llmdot_cuda_decode": (C.c_int, [C.POINTER(VP), C.c_int, I32P, I32P, F32P]),
    "llmdot_cuda_generate": (C.c_int, [VP, I32P, C.c_int, C.c_int, I32P, C.POINTER(C.c_int)]),
    "llmdot_cuda_sampling_seeded_draw": (C.c_float, [C.c_int32]),
    "llmdot_cuda_sample": (C.c_int, [VP, F32P, C.c_int, C.POINTER(LlmdotSampling), I32P, C.c_int, C.c_float,
                                     C.POINTER(C.c_int32)]),
    "llmdot_cuda_generate_sampled": (C.c_int, [VP, I32P, C.c_int, C.c_int, C.POINTER(LlmdotSampling), F32P, I32P,
                                               C.POINTER(C.c_int)]),
    "llmdot_cuda_decode_steps": (C.c_int, [C.POINTER(VP), C.c_int, I32P, C.c_int, I32P, F32P, C.POINTER(C.c_int)]),
    "llmdot_cuda_model_load_gguf_tp": (C.c_int, [C.c_int, C.c_char_p, C.c_int, C.c_int, C.POINTER(VP)]),
    "llmdot_cuda_tp_unique_id": (C.c_int, [C.POINTER(C.c_uint8)]),
    "llmdot_cuda_tp_init": (C.c_int, [VP, C.POINTER(C.c_uint8)]),
    "llmdot_cuda_tp_exchange_handle": (C.c_int, [VP, C.POINTER(C.c_uint8)]),
    "llmdot_cuda_tp_exchange_open": (C.c_int, [VP, C.POINTER(C.c_uint8)]),
    "llmdot_cuda_tp_exchange_use": (C.c_int, [VP, C.c_int]),
    "llmdot_cuda_tp_shard": (C.c_int, [C.POINTER(LlmdotConfig), C.c_int, C.c_int, I32P]),
    "llmdot_cuda_profile_step": (C.c_int, [C.POINTER(VP), C.c_int, I32P, I32P, C.c_int, F32P, C.POINTER(C.c_int)]),
    "llmdot_cuda_profile_matvec": (C.c_int, [VP, C.c_char_p, C.c_int, C.c_int, F32P, C.POINTER(C.c_uint64)]),
    "llmdot_cuda_argmax_noalloc": (C.c_int, [VP, C.c_int, C.c_int, C.c_int, VP, VP]),
    "llmdot_cuda_model_matvec": (C.c_int, [VP, C.c_char_p, F32P, C.c_int, C.c_int, F32P, F32P]),
}

_lib = None


def header_functions() -> List[str]:
    """Every function the public header declares (used by the export test)."""
    src = open(HEADER).read()
    return sorted(set(re.findall(r"LLMDOT_API\s+[\w\s\*]+?\b(llmdot_cuda_\w+)\s*\(", src)))


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise CudaBackendError(-2, f"{LIB_PATH} is missing: build it with `make -C dotllm_b200/csrc`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != 0:
        raise CudaBackendError(rc, lib().llmdot_cuda_last_error().decode(errors="replace"))


def device_count() -> int:
    n = C.c_int(0)
    check(lib().llmdot_cuda_device_count(C.byref(n)))
    return n.value
