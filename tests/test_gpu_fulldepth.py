"""The BASELINE models at full depth against the CPU oracle (the north star's parity bar).

The benchmarked configuration itself: the Llama-3.2-1B-shape model with all 16 layers, its
512-token prompt and 64 greedy decode steps.  Greedy ids must be identical to the reference
algorithm's with an fp32 KV cache; logits before every generated token (the device fed the
oracle's tokens) must be within max-abs 2e-2 plus relative 1e-2 of the reference's with the fp16
KV cache the benchmark runs, and with the fp32 cache.  The other BASELINE models (Phi-3-mini,
Gemma-2-2B, Llama-3-8B) run at full depth with a 64-token prompt and 8 greedy steps under the same
bars; the oracle's cost on the host cores bounds their length.

When a greedy step differs, the message reports the oracle's top-2 logit margin at that step, so
a flip at a near-tie is told apart from a real divergence.
"""
import numpy as np
import pytest

from dotllm_b200 import synth
from dotllm_b200.engine import CudaModel

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
ATOL, RTOL = 2e-2, 1e-2


def _oracle(oracle, cfg, prompt, steps):
    m = oracle.Model(synth.build_model(cfg))
    s = oracle.Session(m)
    try:
        return s.generate(prompt, steps, want_logits=True)
    finally:
        s.close()
        m.close()


def _teacher_forced(m, prompt, toks, kv, ctx):
    s = m.session(max_ctx=ctx, kv=kv)
    try:
        _, lg0 = s.prefill(prompt, want_logits=True)
        out = [lg0]
        for t in toks[:-1]:
            out.append(s.decode(int(t), want_logits=True)[1])
    finally:
        s.close()
    return np.stack(out)


def _check(name, n_prompt, steps, gpu, oracle):
    cfg = synth.get(name)
    prompt = synth.prompt_tokens(cfg, n_prompt)
    toks, ref = _oracle(oracle, cfg, prompt, steps)
    ctx = ((n_prompt + steps + 64 + 63) // 64) * 64
    m = CudaModel.load(synth.build_model(cfg))
    try:
        s = m.session(max_ctx=ctx, kv="f32")
        got = list(s.generate(prompt, steps))
        s.close()
        want = list(toks)
        if got != want:
            i = next(j for j in range(min(len(got), len(want))) if got[j] != want[j])
            top2 = np.sort(ref[i])[-2:]
            pytest.fail(f"{name}: greedy id {i} is {got[i]}, the reference's {want[i]} "
                        f"(reference top-2 margin {top2[1] - top2[0]:.3e})")
        for kv in ("f32", "f16"):
            lg = _teacher_forced(m, prompt, toks, kv, ctx)
            err = np.abs(lg - ref)
            assert np.all(err <= ATOL + RTOL * np.abs(ref)), f"{name} {kv} KV: max abs err {err.max():.3e}"
            if kv == "f32":
                assert err.max() < 1e-3, f"{name} fp32 KV: max abs err {err.max():.3e}"
    finally:
        m.close()


def test_llama1b_full_depth_512_prompt_64_greedy(gpu, oracle):
    """BASELINE configs[1], the benchmarked model: 16 layers, 512-token prompt, 64 greedy steps."""
    _check("llama1b", 512, 64, gpu, oracle)


@pytest.mark.parametrize("name", ["phi3mini", "gemma2b", "llama8b"])
def test_baseline_models_full_depth(gpu, oracle, name):
    """Phi-3-mini (32 layers, hd96, fused QKV), Gemma-2-2B (26 layers, hd256, softcaps, post-norms,
    GeGLU, 256000-row head), Llama-3-8B (32 layers, hd128, FFN 14336): 64-token prompt, 8 steps."""
    _check(name, 64, 8, gpu, oracle)
