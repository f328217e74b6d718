"""The BASELINE models at full depth against the CPU oracle (the north star's parity bar).

The benchmarked configuration itself: the Llama-3.2-1B-shape model with all 16 layers, its
512-token prompt and 64 greedy decode steps, device and oracle both with an fp32 KV cache (the
reference's cache; the fp16 cache the benchmark runs is checked against the oracle run with the
same fp16 rounding in the micro, tiny and full-width shape tests).  The
other BASELINE models (Phi-3-mini, Gemma-2-2B, Llama-3-8B) run at full depth with a 32-token prompt
and 6 greedy steps under the same bars; the oracle's cost on the host cores bounds their length.

Greedy identity over 64 steps is a property of one compilation of the reference, not of its
algorithm: the reference's softmax uses ExpApprox, which jumps by up to ~18 % where its integer
part switches, so fp32 rounding-level changes upstream move some attention weights by a visible
step.  The reference's source leaves one order open (the horizontal add of Vector.Dot, decided by
the JIT and the vector unit); running the oracle with only that order changed (its diagnostic
switch, set_hsum_order(1)) moves the 16-layer Llama-3.2-1B-shape logits by up to 1.4e-2 at every
step and flips its own greedy ids from step 45 on.  The device's fp32 sums run in yet other orders
(tensor-core tiles, split K), so its distance from the oracle is of that same kind and size.  Each
test therefore measures the reference's own sensitivity on its model and prompt (the oracle
teacher-forced again with the other horizontal-add order) and the bars are:
  * logits before every generated token within max-abs 2e-2 + relative 1e-2 of the reference's
    (teacher-forced), or, where an element is outside that, the step's largest device error within
    SENS_FACTOR times the reference's own change at that step;
  * the device's argmax equals the reference's at every step whose reference top-2 margin exceeds
    twice the reference's largest own change over the run;
  * free-running greedy ids identical to the reference's up to the end, or up to a first difference
    at a step whose reference top-2 margin is below that largest own change (a step the reference
    algorithm does not itself decide).
"""
import numpy as np
import pytest

from dotllm_b200 import synth
from dotllm_b200.engine import CudaModel

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
ATOL, RTOL = 2e-2, 1e-2
# the device's summation orders differ from the oracle's in more places than the one order the
# sensitivity run changes, so its error may exceed that run's change by this factor
SENS_FACTOR = 4.0


def _oracle(oracle, cfg, prompt, steps):
    m = oracle.Model(synth.build_model(cfg))
    s = oracle.Session(m)
    try:
        return s.generate(prompt, steps, want_logits=True)
    finally:
        s.close()
        m.close()


def _oracle_other_order(oracle, cfg, prompt, toks):
    """The reference algorithm teacher-forced on the same tokens with the other horizontal-add
    order of its 8-lane reductions: logits before every generated token."""
    oracle.set_hsum_order(1)
    m = oracle.Model(synth.build_model(cfg))
    s = oracle.Session(m)
    try:
        lg = None
        for i, t in enumerate(prompt):
            lg = s.process_token(int(t), i)
        out = [lg]
        for j, t in enumerate(toks[:-1]):
            out.append(s.process_token(int(t), len(prompt) + j))
        return np.stack(out)
    finally:
        oracle.set_hsum_order(0)
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
    sens = np.abs(_oracle_other_order(oracle, cfg, prompt, toks) - ref).max(axis=1)  # per step
    eps = float(sens.max())
    ctx = ((n_prompt + steps + 64 + 63) // 64) * 64
    m = CudaModel.load(synth.build_model(cfg))
    try:
        srt = np.sort(ref, axis=1)
        margin = srt[:, -1] - srt[:, -2]
        s = m.session(max_ctx=ctx, kv="f32")
        got = list(s.generate(prompt, steps))
        s.close()
        want = list(toks)
        if got != want:
            i = next(j for j in range(min(len(got), len(want))) if got[j] != want[j])
            assert margin[i] < eps, (f"{name}: greedy id {i} is {got[i]}, the reference's {want[i]} at a "
                                     f"reference top-2 margin of {margin[i]:.3e} (reference's own change {eps:.3e})")
        for kv in ("f32",):
            lg = _teacher_forced(m, prompt, toks, kv, ctx)
            err = np.abs(lg - ref)
            inside = np.all(err <= ATOL + RTOL * np.abs(ref), axis=1)
            step_err = err.max(axis=1)
            bad = [i for i in range(steps) if not inside[i] and step_err[i] > SENS_FACTOR * sens[i]]
            assert not bad, (f"{name} {kv} KV: steps {bad} outside the bar: device error "
                             f"{[round(float(step_err[i]), 5) for i in bad]}, reference's own change "
                             f"{[round(float(sens[i]), 5) for i in bad]}")
            decided = margin > 2 * eps
            top = lg.argmax(axis=1)
            wrong = [i for i in range(steps) if decided[i] and top[i] != toks[i]]
            assert not wrong, f"{name} {kv} KV: argmax differs at decided steps {wrong}"
    finally:
        m.close()


def test_llama1b_full_depth_512_prompt_64_greedy(gpu, oracle):
    """BASELINE configs[1], the benchmarked model: 16 layers, 512-token prompt, 64 greedy steps."""
    _check("llama1b", 512, 64, gpu, oracle)


@pytest.mark.parametrize("name", ["phi3mini", "gemma2b", "llama8b"])
def test_baseline_models_full_depth(gpu, oracle, name):
    """Phi-3-mini (32 layers, hd96, fused QKV), Gemma-2-2B (26 layers, hd256, softcaps, post-norms,
    GeGLU, 256000-row head), Llama-3-8B (32 layers, hd128, FFN 14336): 32-token prompt, 6 steps."""
    _check(name, 32, 6, gpu, oracle)
