"""Device-resident decode/prefill over the C ABI (Tier B).

Mirrors the reference's engine surface: ``LoadedModel.Load`` ->
``CudaModel.load``; ``new InferenceEngine(model, backend)`` + ``Generate`` ->
``CudaSession.generate`` (greedy, src/Llmdot.Core/Inference/InferenceEngine.cs:74-132);
the per-token ``ProcessToken`` -> ``prefill`` / ``decode``.  Everything runs
in the native library on the GPU; there is no CPU path here.
"""
from __future__ import annotations

import ctypes as C
import weakref
from typing import List, Optional, Sequence, Tuple

import numpy as np

from .native import (KV_F16, KV_F32, LlmdotConfig, TensorDesc, VP, F32P, I32P, check, lib)


class CudaModel:
    def __init__(self, handle: int, device: int):
        self._sessions = weakref.WeakSet()
        self._h = C.c_void_p(handle)
        self.device = device
        cfg = LlmdotConfig()
        check(lib().llmdot_cuda_model_config(self._h, C.byref(cfg)))
        self.config = cfg.as_dict()

    @classmethod
    def load(cls, path: str, device: int = 0) -> "CudaModel":
        """LoadedModel.Load + upload: native GGUF parse, tensors streamed to the device."""
        h = VP()
        check(lib().llmdot_cuda_model_load_gguf(device, path.encode(), C.byref(h)))
        return cls(h.value, device)

    @classmethod
    def load_tp(cls, path: str, tp_size: int, tp_rank: int, device: int = 0) -> "CudaModel":
        """This rank's tensor-parallel shard of the model (attach the group with tp_init)."""
        h = VP()
        check(lib().llmdot_cuda_model_load_gguf_tp(device, path.encode(), tp_size, tp_rank, C.byref(h)))
        return cls(h.value, device)

    def tp_init(self, unique_id: bytes) -> None:
        """Join the NCCL group whose id rank 0 obtained from tp_unique_id()."""
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        check(lib().llmdot_cuda_tp_init(self._h, buf))

    def tp_exchange_handle(self) -> bytes:
        """This rank's 128-byte exchange-buffer handle (CUDA IPC handle + GPU UUID) for the
        peer-memory all-reduce."""
        buf = (C.c_uint8 * 128)()
        check(lib().llmdot_cuda_tp_exchange_handle(self._h, buf))
        return bytes(buf)

    def tp_exchange_open(self, handles) -> None:
        """Open every rank's handle (rank order); the step's residual sums then run over peer
        memory instead of NCCL."""
        blob = b"".join(handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        check(lib().llmdot_cuda_tp_exchange_open(self._h, buf))

    def tp_exchange_use(self, on: bool) -> None:
        """Residual sums on the opened peer-memory all-reduce (True) or on NCCL (False)."""
        check(lib().llmdot_cuda_tp_exchange_use(self._h, 1 if on else 0))

    @classmethod
    def from_tensors(cls, cfg: dict, tensors: Sequence[Tuple[str, int, Sequence[int], np.ndarray]],
                     device: int = 0) -> "CudaModel":
        """Upload tensors the host already holds (the .NET LoadedModel path)."""
        c = LlmdotConfig(**{k: v for k, v in cfg.items() if k in dict(LlmdotConfig._fields_)})
        keep = []
        descs = (TensorDesc * len(tensors))()
        for i, (name, gtype, dims, data) in enumerate(tensors):
            data = np.ascontiguousarray(data)
            nb = name.encode()
            keep += [data, nb]
            descs[i].name = nb
            descs[i].type = gtype
            descs[i].n_dims = len(dims)
            for j, d in enumerate(dims):
                descs[i].dims[j] = d
            descs[i].data = data.ctypes.data
            descs[i].n_bytes = data.nbytes
        h = VP()
        check(lib().llmdot_cuda_model_load(device, C.byref(c), descs, len(tensors), C.byref(h)))
        return cls(h.value, device)

    def profile_matvec(self, tensor: str, batch: int = 1, iters: int = 20) -> Tuple[float, int]:
        """(average ms per launch, bytes per launch) of the matvec over one weight tensor."""
        ms, nb = C.c_float(), C.c_uint64()
        check(lib().llmdot_cuda_profile_matvec(self._h, tensor.encode(), batch, iters, C.byref(ms), C.byref(nb)))
        return ms.value, nb.value

    def matvec(self, tensor: str, x, rows: int, mode: int = 0, norm_w=None) -> np.ndarray:
        """y [batch, rows] = W.x for one uploaded weight (mode 0: the decode step's kernel,
        1: the generic kernel, 2: the step's kernel with the fused RMSNorm of x by norm_w)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim == 1:
            x = x[None, :]
        nw = np.ascontiguousarray(norm_w, dtype=np.float32) if norm_w is not None else None
        y = np.empty((x.shape[0], rows), dtype=np.float32)
        check(lib().llmdot_cuda_model_matvec(self._h, tensor.encode(), x.ctypes.data_as(F32P), x.shape[0], mode,
                                             nw.ctypes.data_as(F32P) if nw is not None else None,
                                             y.ctypes.data_as(F32P)))
        return y

    def weight_bytes(self) -> Tuple[int, int]:
        a, b = C.c_uint64(), C.c_uint64()
        check(lib().llmdot_cuda_model_weight_bytes(self._h, C.byref(a), C.byref(b)))
        return a.value, b.value

    def session(self, max_ctx: int = 0, kv: str = "f16") -> "CudaSession":
        s = CudaSession(self, max_ctx, KV_F16 if kv == "f16" else KV_F32)
        self._sessions.add(s)
        return s

    def close(self) -> None:
        """Free the model; sessions still open are closed first."""
        if self._h:
            for s in list(self._sessions):
                s.close()
            lib().llmdot_cuda_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaSession:
    def __init__(self, model: CudaModel, max_ctx: int = 0, kv_type: int = KV_F16):
        self.model = model
        self._h = VP()
        check(lib().llmdot_cuda_session_create(model._h, max_ctx, kv_type, C.byref(self._h)))

    @property
    def position(self) -> int:
        p = C.c_int()
        check(lib().llmdot_cuda_session_position(self._h, C.byref(p)))
        return p.value

    def reset(self) -> None:
        check(lib().llmdot_cuda_session_reset(self._h))

    def prefill(self, tokens, want_logits: bool = False):
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        V = self.model.config["vocab"]
        logits = np.empty(V, dtype=np.float32) if want_logits else None
        nxt = C.c_int32()
        check(lib().llmdot_cuda_prefill(self._h, toks.ctypes.data_as(I32P), toks.size,
                                        logits.ctypes.data_as(F32P) if logits is not None else None, C.byref(nxt)))
        return nxt.value, logits

    def decode(self, token: int, want_logits: bool = False):
        nxt, lg = decode_batch([self], [token], want_logits)
        return int(nxt[0]), (lg[0] if lg is not None else None)

    def generate(self, prompt, max_tokens: int) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(max_tokens, 1), dtype=np.int32)
        n = C.c_int()
        check(lib().llmdot_cuda_generate(self._h, p.ctypes.data_as(I32P), p.size, max_tokens,
                                         out.ctypes.data_as(I32P), C.byref(n)))
        return out[:n.value]

    def generate_sampled(self, prompt, max_tokens: int, options, draws=None) -> np.ndarray:
        """Generate with Sampler.Sample on the device (llmdot_cuda_generate_sampled).  options:
        native.LlmdotSampling; draws: per-token uniform draws (default: seeded / fresh)."""
        from .native import LlmdotSampling
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(max_tokens, 1), dtype=np.int32)
        n = C.c_int()
        o = LlmdotSampling(options.top_k, options.top_p, options.temperature, options.repeat_penalty,
                           options.repeat_window, options.seed)
        d = None if draws is None else np.ascontiguousarray(draws, dtype=np.float32)
        if d is not None and d.size < max_tokens:  # the library reads one draw per token
            raise ValueError(f"generate_sampled: {d.size} draws for {max_tokens} tokens")
        check(lib().llmdot_cuda_generate_sampled(self._h, p.ctypes.data_as(I32P), p.size, max_tokens, C.byref(o),
                                                 d.ctypes.data_as(F32P) if d is not None else None,
                                                 out.ctypes.data_as(I32P), C.byref(n)))
        return out[:n.value]

    def close(self) -> None:
        if self._h:
            lib().llmdot_cuda_session_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _batch_tokens(name: str, tokens, batch: int) -> np.ndarray:
    """One input token per session: the library reads exactly `batch` of them."""
    toks = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
    if toks.size != batch:
        raise ValueError(f"{name}: {toks.size} tokens for {batch} sessions")
    return toks


def decode_steps(sessions: List[CudaSession], tokens, n_steps: int):
    """Device-resident greedy decode of n_steps tokens for sessions in lockstep.
    Returns (ids [n_steps, batch], device ms, kernel launches per step)."""
    B = len(sessions)
    arr = (VP * B)(*[s._h for s in sessions])
    toks = _batch_tokens("decode_steps", tokens, B)
    out = np.zeros((max(n_steps, 1), B), dtype=np.int32)
    ms = C.c_float()
    kps = C.c_int()
    check(lib().llmdot_cuda_decode_steps(arr, B, toks.ctypes.data_as(I32P), n_steps, out.ctypes.data_as(I32P),
                                         C.byref(ms), C.byref(kps)))
    return out[:n_steps], ms.value, kps.value


FAMILIES = ("matvec", "attention", "other", "collective")


def profile_step(sessions: List[CudaSession], tokens):
    """One greedy step launched operation by operation with CUDA events around each operation:
    returns (next ids, {family: (ms, operations)}); see llmdot_cuda_profile_step."""
    B = len(sessions)
    arr = (VP * B)(*[s._h for s in sessions])
    toks = _batch_tokens("profile_step", tokens, B)
    nxt = np.zeros(B, dtype=np.int32)
    nf = len(FAMILIES)
    ms = np.zeros(nf, dtype=np.float32)
    cnt = (C.c_int * nf)()
    check(lib().llmdot_cuda_profile_step(arr, B, toks.ctypes.data_as(I32P), nxt.ctypes.data_as(I32P), nf,
                                         ms.ctypes.data_as(F32P), cnt))
    return nxt, {f: (float(ms[i]), int(cnt[i])) for i, f in enumerate(FAMILIES)}


def decode_batch(sessions: List[CudaSession], tokens, want_logits: bool = False):
    """One greedy step for several sessions of one model (batched decode)."""
    B = len(sessions)
    arr = (VP * B)(*[s._h for s in sessions])
    toks = _batch_tokens("decode", tokens, B)
    nxt = np.zeros(B, dtype=np.int32)
    V = sessions[0].model.config["vocab"]
    logits = np.empty((B, V), dtype=np.float32) if want_logits else None
    check(lib().llmdot_cuda_decode(arr, B, toks.ctypes.data_as(I32P), nxt.ctypes.data_as(I32P),
                                   logits.ctypes.data_as(F32P) if logits is not None else None))
    return nxt, logits


def gguf_config(path: str) -> dict:
    """GgufReader.Read + ArchitectureResolver.Resolve of a GGUF file, natively and without a
    device (llmdot_cuda_gguf_config)."""
    c = LlmdotConfig()
    check(lib().llmdot_cuda_gguf_config(path.encode(), C.byref(c)))
    return c.as_dict()


def tp_open_peer(model, all_gather) -> Optional[str]:
    """Collective switch of a tensor-parallel group's residual sums to the peer-memory all-reduce.

    Every rank calls it with its model and `all_gather(obj) -> [obj of rank 0, .., rank tp-1]`
    (e.g. torch.distributed.all_gather_object).  Each rank exports its handle, the handles are
    gathered, each rank opens them, and the ranks then agree: the peer form is used only if every
    rank opened it; otherwise the ranks that did open turn it off again, so that all ranks keep
    NCCL.  Returns None on success, else the first failing rank's reason.
    """
    why = None
    try:
        h = model.tp_exchange_handle()
    except Exception as e:  # CudaBackendError: unsupported TP size, no device memory, ...
        h, why = None, str(e)[:300]
    handles = all_gather(h)
    opened = False
    if why is None:
        if all(x is not None for x in handles):
            try:
                model.tp_exchange_open(list(handles))
                opened = True
            except Exception as e:
                why = str(e)[:300]
        else:
            why = "a peer could not export its exchange buffer"
    whys = all_gather(why)
    first = next((w for w in whys if w), None)
    if first is not None and opened:
        model.tp_exchange_use(False)
    return first


def tp_unique_id() -> bytes:
    """An NCCL unique id (128 bytes) for llmdot_cuda_tp_init."""
    buf = (C.c_uint8 * 128)()
    check(lib().llmdot_cuda_tp_unique_id(buf))
    return bytes(buf)


def tp_shard(config: dict, tp_size: int, tp_rank: int) -> dict:
    """Rows / columns of the full matrices that rank tp_rank holds (host only)."""
    c = LlmdotConfig(**{k: v for k, v in config.items() if k in dict(LlmdotConfig._fields_)})
    out = (C.c_int32 * 8)()
    check(lib().llmdot_cuda_tp_shard(C.byref(c), tp_size, tp_rank, out))
    keys = ["q_lo", "q_n", "kv_lo", "kv_n", "ffn_lo", "ffn_n", "vocab_lo", "vocab_n"]
    return dict(zip(keys, list(out)))
