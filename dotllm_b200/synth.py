"""Seeded synthetic GGUF models for the benchmark configurations.

No checkpoints or datasets exist on these machines, so every model is random:
weight matrices N(0, 0.02) quantised to the stated K-quant types with the
reference-layout encoders in ``quant.py``; norm weights 1 + N(0, 0.01) stored
as F32; prompts uniform token ids.  The metadata carries exactly the keys
llmdot's ArchitectureResolver reads (src/Llmdot.Core/Loading/ArchitectureResolver.cs:14-112),
plus ``tokenizer.ggml.tokens`` of length V (which sets the vocabulary) and an
EOS id of -1 so the reference's Generate never stops early
(src/Llmdot.Core/Inference/InferenceEngine.cs:114).

Each tensor is generated from its own seed (config seed, tensor index), so a
file is identical whatever order or process builds it.
"""
from __future__ import annotations

import hashlib
import os
from dataclasses import dataclass, field, replace
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import gguf
from .gguf import (F32, I32, STR, U32, ARR, GGML_F32, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K, GGML_Q8_0,
                   Metadata, TensorInfo, write_gguf)
from .quant import quantize

GEN_VERSION = 3  # bump when the generator's output changes


@dataclass(frozen=True)
class SynthConfig:
    name: str
    arch: str
    layers: int
    hidden: int
    heads: int
    heads_kv: int
    head_dim: int
    ffn: int
    vocab: int
    context: int
    rope_base: float = 10000.0
    eps: float = 1e-5
    tied: bool = False
    default_type: int = GGML_Q4_K
    # tensor-name role -> ggml type ("token_embd", "output", "attn_q", "attn_k", "attn_v",
    # "attn_qkv", "attn_output", "ffn_gate", "ffn_up", "ffn_down")
    overrides: Tuple[Tuple[str, int], ...] = ()
    qkv_fused: bool = False
    post_norm: bool = False
    attn_softcap: Optional[float] = None
    final_softcap: Optional[float] = None
    sliding_window: int = 0
    # Lfm2Like: layers whose operator is the short conv (the others are attention), its kernel
    conv_layers: Tuple[int, ...] = ()
    conv_kernel: int = 3
    qk_norm: bool = False
    # LayerNorm (attention.layer_norm_epsilon, attn_norm.bias) instead of RMSNorm; FFN with a gate
    layer_norm: bool = False
    gated_ffn: bool = True
    # MoE FFN: expert count, experts used per token, each expert's FFN width
    experts: int = 0
    experts_used: int = 0
    expert_ffn: int = 0
    seed: int = 1
    # workload
    prompt_len: int = 64
    decode_len: int = 128
    batch: int = 1

    def type_of(self, role: str) -> int:
        return dict(self.overrides).get(role, self.default_type)

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.heads_kv * self.head_dim


Q6 = GGML_Q6_K
# F32 tensors and the std of their random values (norm vectors are 1 + N(0, 0.01))
F32_ROLES = {"norm": None, "conv": 0.5, "router": 0.1, "bias": 0.01}

# BASELINE.json configs[0..4]
CONFIGS: Dict[str, SynthConfig] = {
    "tiny": SynthConfig(
        name="tiny", arch="llama", layers=6, hidden=512, heads=8, heads_kv=4, head_dim=64, ffn=1536,
        vocab=32000, context=2048, rope_base=10000.0, tied=False,
        overrides=(("token_embd", Q6), ("output", Q6)), seed=1001, prompt_len=64, decode_len=128),
    "llama1b": SynthConfig(
        name="llama1b", arch="llama", layers=16, hidden=2048, heads=32, heads_kv=8, head_dim=64, ffn=8192,
        vocab=128256, context=4096, rope_base=500000.0, tied=True,
        overrides=(("attn_v", Q6), ("ffn_down", Q6)), seed=2001, prompt_len=512, decode_len=256),
    "phi3mini": SynthConfig(
        name="phi3mini", arch="phi3", layers=32, hidden=3072, heads=32, heads_kv=32, head_dim=96, ffn=8192,
        vocab=32064, context=4096, rope_base=10000.0, tied=False, qkv_fused=True,
        overrides=(("output", Q6),), seed=3001, prompt_len=1024, decode_len=256, batch=32),
    "gemma2b": SynthConfig(
        name="gemma2b", arch="gemma2", layers=26, hidden=2304, heads=8, heads_kv=4, head_dim=256, ffn=9216,
        vocab=256000, context=8192, rope_base=10000.0, eps=1e-6, tied=True, post_norm=True,
        attn_softcap=50.0, final_softcap=30.0, sliding_window=4096,
        overrides=(("token_embd", Q6), ("attn_v", Q6), ("ffn_down", Q6)), seed=4001,
        prompt_len=6144, decode_len=256, batch=4),
    "llama8b": SynthConfig(
        name="llama8b", arch="llama", layers=32, hidden=4096, heads=32, heads_kv=8, head_dim=128, ffn=14336,
        vocab=128256, context=8192, rope_base=500000.0, tied=False,
        overrides=(("attn_v", Q6), ("ffn_down", Q6), ("output", Q6)), seed=5001,
        prompt_len=2048, decode_len=256, batch=1),
}

# Small shapes for fast tests; they exercise the same features as the big configs.
TEST_CONFIGS: Dict[str, SynthConfig] = {
    "micro": SynthConfig(
        name="micro", arch="llama", layers=2, hidden=256, heads=4, heads_kv=2, head_dim=64, ffn=512,
        vocab=1000, context=256, tied=True, overrides=(("attn_v", Q6), ("ffn_down", Q6)), seed=11,
        prompt_len=8, decode_len=16),
    "micro-gemma": SynthConfig(
        name="micro-gemma", arch="gemma2", layers=2, hidden=256, heads=4, heads_kv=2, head_dim=128, ffn=768,
        vocab=1000, context=256, eps=1e-6, tied=True, post_norm=True, attn_softcap=50.0, final_softcap=30.0,
        sliding_window=24, overrides=(("token_embd", Q6), ("attn_v", Q6), ("ffn_down", Q6)), seed=12,
        prompt_len=20, decode_len=16),
    "micro-phi3": SynthConfig(
        name="micro-phi3", arch="phi3", layers=2, hidden=512, heads=8, heads_kv=8, head_dim=96, ffn=512,
        vocab=1000, context=256, qkv_fused=True, overrides=(("output", Q6),), seed=13,
        prompt_len=8, decode_len=16),
    "micro-q5q8": SynthConfig(
        name="micro-q5q8", arch="qwen2", layers=2, hidden=256, heads=4, heads_kv=1, head_dim=64, ffn=512,
        vocab=1000, context=256, default_type=GGML_Q5_K,
        overrides=(("attn_v", GGML_Q8_0), ("ffn_down", GGML_Q8_0), ("output", Q6)), seed=14,
        prompt_len=8, decode_len=16),
    # the templates the device does not run yet (checked by the oracle only): LFM2's short-conv
    # layers with QK-normed attention layers, a Llama-like MoE, and LFM2 with MoE
    "micro-lfm2": SynthConfig(
        name="micro-lfm2", arch="lfm2", layers=4, hidden=256, heads=4, heads_kv=2, head_dim=64, ffn=512,
        vocab=1000, context=256, tied=True, conv_layers=(0, 2), qk_norm=True, seed=15,
        prompt_len=8, decode_len=16),
    "micro-neox": SynthConfig(
        name="micro-neox", arch="phi2", layers=2, hidden=256, heads=4, heads_kv=4, head_dim=64, ffn=512,
        vocab=1000, context=256, layer_norm=True, gated_ffn=False, seed=18, prompt_len=8, decode_len=16),
    "micro-moe": SynthConfig(
        name="micro-moe", arch="llama", layers=2, hidden=256, heads=4, heads_kv=2, head_dim=64, ffn=512,
        vocab=1000, context=256, experts=4, experts_used=2, expert_ffn=256, seed=16, prompt_len=8, decode_len=16),
    "micro-lfm2moe": SynthConfig(
        name="micro-lfm2moe", arch="lfm2_moe", layers=3, hidden=256, heads=4, heads_kv=2, head_dim=64, ffn=512,
        vocab=1000, context=256, tied=True, conv_layers=(0,), qk_norm=True, experts=4, experts_used=2,
        expert_ffn=256, seed=17, prompt_len=8, decode_len=16),
}

# Full-width, few-layer copies of the BASELINE models: every matrix, head and vocabulary shape
# of the real config (head_dim 96 / 128 / 256, fused QKV, 256000-row tied head) at a size the
# CPU oracle checks in seconds.  Prompts of 40 tokens cross one 32-token prefill chunk; the
# Gemma copy narrows its sliding window so that the window is active within the test.
for _n, _kw in (("llama1b", {}), ("phi3mini", {}), ("gemma2b", {"sliding_window": 32}), ("llama8b", {"layers": 1})):
    _c = replace(CONFIGS[_n], name=f"{_n}-shape", prompt_len=40, decode_len=16, batch=1, **{"layers": 2, **_kw})
    TEST_CONFIGS[_c.name] = _c
del _n, _kw, _c

ALL_CONFIGS = {**CONFIGS, **TEST_CONFIGS}


def tensor_plan(cfg: SynthConfig) -> List[Tuple[TensorInfo, str]]:
    """(TensorInfo, role) for every tensor, in file order.  Role "norm" = F32 norm vector."""
    d, q, kv, f, V = cfg.hidden, cfg.q_dim, cfg.kv_dim, cfg.ffn, cfg.vocab
    out: List[Tuple[TensorInfo, str]] = []

    def add(name: str, dims: List[int], role: str):
        t = GGML_F32 if role in F32_ROLES else cfg.type_of(role)
        out.append((TensorInfo(name, dims, t), role))

    add("token_embd.weight", [d, V], "token_embd")
    for l in range(cfg.layers):
        p = f"blk.{l}."
        add(p + "attn_norm.weight", [d], "norm")
        if cfg.layer_norm:
            add(p + "attn_norm.bias", [d], "bias")
        if l in cfg.conv_layers:
            # TensorNameResolver.cs:79-89: in_proj -> (B, C, x), the depthwise kernel [K][d], out_proj
            add(p + "shortconv.in_proj.weight", [d, 3 * d], "conv_in")
            add(p + "shortconv.conv.weight", [cfg.conv_kernel, d], "conv")
            add(p + "shortconv.out_proj.weight", [d, d], "conv_out")
        else:
            if cfg.qkv_fused:
                add(p + "attn_qkv.weight", [d, q + 2 * kv], "attn_qkv")
            else:
                add(p + "attn_q.weight", [d, q], "attn_q")
                add(p + "attn_k.weight", [d, kv], "attn_k")
                add(p + "attn_v.weight", [d, kv], "attn_v")
            if cfg.qk_norm:
                add(p + "attn_q_norm.weight", [cfg.head_dim], "norm")
                add(p + "attn_k_norm.weight", [cfg.head_dim], "norm")
            add(p + "attn_output.weight", [q, d], "attn_output")
        if cfg.post_norm:
            add(p + "post_attention_norm.weight", [d], "norm")
        add(p + "ffn_norm.weight", [d], "norm")
        if cfg.experts:
            # MoeFfnForward (InferenceEngine.cs:489-542): the router and per-expert SwiGLU
            # tensors; the dense ffn_up / ffn_down exist only because ResolveLayer requires them
            add(p + "ffn_gate_inp.weight", [d, cfg.experts], "router")
            for e in range(cfg.experts):
                add(p + f"ffn_gate.{e}.weight", [d, cfg.expert_ffn], "ffn_gate")
                add(p + f"ffn_up.{e}.weight", [d, cfg.expert_ffn], "ffn_up")
                add(p + f"ffn_down.{e}.weight", [cfg.expert_ffn, d], "ffn_down")
            add(p + "ffn_up.weight", [d, f], "ffn_up")
            add(p + "ffn_down.weight", [f, d], "ffn_down")
        else:
            if cfg.gated_ffn:
                add(p + "ffn_gate.weight", [d, f], "ffn_gate")
            add(p + "ffn_up.weight", [d, f], "ffn_up")
            add(p + "ffn_down.weight", [f, d], "ffn_down")
        if cfg.post_norm:
            add(p + "post_ffw_norm.weight", [d], "norm")
    add("output_norm.weight", [d], "norm")
    if not cfg.tied:
        add("output.weight", [d, V], "output")
    return out


def metadata_for(cfg: SynthConfig) -> Metadata:
    a = cfg.arch
    md = Metadata()
    md.add("general.architecture", STR, a)
    md.add("general.name", STR, f"synthetic-{cfg.name}")
    md.add(f"{a}.embedding_length", U32, cfg.hidden)
    md.add(f"{a}.block_count", U32, cfg.layers)
    md.add(f"{a}.context_length", U32, cfg.context)
    md.add(f"{a}.feed_forward_length", U32, cfg.ffn)
    md.add(f"{a}.attention.head_count", U32, cfg.heads)
    if cfg.conv_layers:  # per-layer kv heads, 0 for the conv layers (HeadCountKvPerLayer)
        md.add(f"{a}.attention.head_count_kv", ARR,
               [0 if l in cfg.conv_layers else cfg.heads_kv for l in range(cfg.layers)], U32)
        md.add(f"{a}.shortconv.l_cache", U32, cfg.conv_kernel)
    else:
        md.add(f"{a}.attention.head_count_kv", U32, cfg.heads_kv)
    if cfg.experts:
        md.add(f"{a}.expert_count", U32, cfg.experts)
        md.add(f"{a}.expert_used_count", U32, cfg.experts_used)
    md.add(f"{a}.attention.key_length", U32, cfg.head_dim)
    md.add(f"{a}.attention.value_length", U32, cfg.head_dim)
    md.add(f"{a}.attention.layer_norm_epsilon" if cfg.layer_norm else f"{a}.attention.layer_norm_rms_epsilon",
           F32, cfg.eps)
    md.add(f"{a}.rope.freq_base", F32, cfg.rope_base)
    md.add(f"{a}.rope.dimension_count", U32, cfg.head_dim)
    if cfg.sliding_window:
        md.add(f"{a}.attention.sliding_window", U32, cfg.sliding_window)
    if cfg.attn_softcap is not None:
        md.add(f"{a}.attn_logit_softcapping", F32, cfg.attn_softcap)
    if cfg.final_softcap is not None:
        md.add(f"{a}.final_logit_softcapping", F32, cfg.final_softcap)
    md.add("tokenizer.ggml.model", STR, "synthetic")
    md.add("tokenizer.ggml.tokens", ARR, [f"<t{i}>" for i in range(cfg.vocab)], STR)
    md.add("tokenizer.ggml.bos_token_id", U32, 1)
    md.add("tokenizer.ggml.eos_token_id", I32, -1)
    return md


def _tensor_seed(cfg: SynthConfig, idx: int) -> int:
    return (cfg.seed * 1_000_003 + idx * 7919) & 0x7FFFFFFF


def tensor_bytes(cfg: SynthConfig, info: TensorInfo, role: str, idx: int) -> bytes:
    rng = np.random.default_rng(_tensor_seed(cfg, idx))
    if role == "norm":
        w = 1.0 + 0.01 * rng.standard_normal(info.dims[0], dtype=np.float32)
        return w.astype("<f4").tobytes()
    if role in F32_ROLES:  # the conv kernel and the MoE router stay F32, as in released GGUFs
        n = int(np.prod(info.dims))
        return (rng.standard_normal(n, dtype=np.float32) * np.float32(F32_ROLES[role])).astype("<f4").tobytes()
    cols, rows = info.dims[0], info.dims[1]
    chunk = max(1, (1 << 24) // cols)
    starts = range(0, rows, chunk)
    if len(starts) == 1:
        x = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
        return quantize(x, info.ggml_type).tobytes()
    # the random stream is drawn in order; quantisation of the drawn chunks (row-independent,
    # numpy releases the GIL) runs on threads, so the bytes do not depend on the thread count
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        futs, parts = [], []
        for r0 in starts:
            n = min(chunk, rows - r0)
            x = rng.standard_normal((n, cols), dtype=np.float32) * np.float32(0.02)
            futs.append(ex.submit(lambda a: quantize(a, info.ggml_type).tobytes(), x))
            if len(futs) - len(parts) > 16:  # bound the drawn chunks held in memory
                parts.append(futs[len(parts)].result())
        parts += [f.result() for f in futs[len(parts):]]
        return b"".join(parts)


def cache_dir() -> str:
    d = os.environ.get("LLMDOT_SYNTH_DIR") or os.path.join(os.path.expanduser("~"), ".cache", "llmdot_synth")
    os.makedirs(d, exist_ok=True)
    return d


def model_path(cfg: SynthConfig) -> str:
    key = hashlib.sha1(repr((cfg, GEN_VERSION)).encode()).hexdigest()[:12]
    return os.path.join(cache_dir(), f"{cfg.name}-{key}.gguf")


def _tensor_job(args):
    cfg, info, role, idx = args
    return tensor_bytes(cfg, info, role, idx)


def build_model(cfg: SynthConfig, path: Optional[str] = None, workers: Optional[int] = None) -> str:
    """Write (or reuse) the synthetic GGUF for ``cfg`` and return its path.

    Large models are generated by a pool of worker processes.  The pool runs inside a
    fresh interpreter (``python -m dotllm_b200.synth``), so callers may be scripts without
    a ``__main__`` guard and may already have initialised CUDA; the file is identical to a
    single-process build because every tensor has its own seed."""
    path = path or model_path(cfg)
    if os.path.exists(path):
        return path
    total = sum(t.n_bytes for t, _ in tensor_plan(cfg))
    if workers is None and total > (64 << 20) and cfg.name in ALL_CONFIGS and ALL_CONFIGS[cfg.name] == cfg:
        import subprocess
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        subprocess.run([sys.executable, "-m", "dotllm_b200.synth", cfg.name, path], check=True, cwd=root,
                       timeout=1800)
        return path
    return _build_local(cfg, path, workers)


def _build_local(cfg: SynthConfig, path: str, workers: Optional[int]) -> str:
    plan = tensor_plan(cfg)
    infos = [t for t, _ in plan]
    roles = {t.name: (r, i) for i, (t, r) in enumerate(plan)}
    tmp = path + f".tmp{os.getpid()}"
    total = sum(t.n_bytes for t in infos)
    if workers is None:
        workers = min(os.cpu_count() or 1, 24) if total > (64 << 20) else 1
    if workers <= 1:
        def produce(info: TensorInfo) -> bytes:
            role, idx = roles[info.name]
            return tensor_bytes(cfg, info, role, idx)

        write_gguf(tmp, metadata_for(cfg), infos, produce)
    else:
        import multiprocessing as mp
        ctx = mp.get_context("spawn")
        jobs = [(cfg, t, r, i) for i, (t, r) in enumerate(plan)]
        with ctx.Pool(workers) as pool:
            it = pool.imap(_tensor_job, jobs, chunksize=1)
            write_gguf(tmp, metadata_for(cfg), infos, lambda info: next(it))
    os.replace(tmp, path)
    return path


def prompt_tokens(cfg: SynthConfig, n: Optional[int] = None, session: int = 0) -> np.ndarray:
    """Uniform token ids in [0, V) seeded by (config seed, session)."""
    n = cfg.prompt_len if n is None else n
    rng = np.random.default_rng(cfg.seed * 1000 + 1 + session)
    return rng.integers(0, cfg.vocab, size=n, dtype=np.int64).astype(np.int32)


def weight_bytes(cfg: SynthConfig) -> Dict[str, int]:
    """Quantised bytes read per decode step (embedding excluded: one row per session)."""
    layer = 0
    head = 0
    for info, role in tensor_plan(cfg):
        if role == "token_embd":
            if cfg.tied:
                head += info.n_bytes
            continue
        if role == "output":
            head += info.n_bytes
            continue
        layer += info.n_bytes
    return {"layers": layer, "logits": head}


def get(name: str) -> SynthConfig:
    return ALL_CONFIGS[name]


def with_overrides(cfg: SynthConfig, **kw) -> SynthConfig:
    return replace(cfg, **kw)


if __name__ == "__main__":
    import sys

    # python -m dotllm_b200.synth NAME [PATH]: generate one synthetic model (worker pool)
    _cfg = get(sys.argv[1])
    _path = sys.argv[2] if len(sys.argv) > 2 else model_path(_cfg)
    if not os.path.exists(_path):
        _build_local(_cfg, _path, min(os.cpu_count() or 1, 24))
    print(_path)
