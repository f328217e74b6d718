"""Sampler.Sample on the device (llmdot_cuda_sample, llmdot_cuda_generate_sampled) against the
oracle's restatement (Sampler.cs:24-165), on the same logits, history and uniform draws.

Logits are continuous random values, so no two tie; the sampled index must be identical.  The
softmax's 8-wide ExpApprox lanes are bit-exact on the device; only its MathF.Exp tail (the last
k mod 8 entries) may differ by an ulp, so a draw within an ulp of a cumulative-probability
boundary could in principle pick the neighbour.  The seeds and draws are fixed, and none of them
lands that close.  The full-row path (top_k <= 0 or >= n) is also checked on rows with many exactly
tied probabilities, where the nucleus replays the reference's selection sort, and the top-k path on
rows with tied winners, where the device replays FindTopK's replacement scan.
"""
import numpy as np
import pytest

from dotllm_b200 import synth
from dotllm_b200.native import CudaBackendError, LlmdotSampling
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _opts(**kw):
    return LlmdotSampling(**kw)


def _oracle_opts(o):
    return O.SamplingOptions(o.top_k, o.top_p, o.temperature, o.repeat_penalty, o.repeat_window, o.seed)


CASES = [
    dict(top_k=40, top_p=0.95, temperature=0.8, repeat_penalty=1.1, repeat_window=64),  # the defaults
    dict(top_k=1, top_p=1.0, temperature=1.0, repeat_penalty=1.0, repeat_window=0),
    dict(top_k=5, top_p=1.0, temperature=0.5, repeat_penalty=2.0, repeat_window=8),
    dict(top_k=200, top_p=1.0, temperature=1.5, repeat_penalty=1.3, repeat_window=64),
    dict(top_k=1024, top_p=1.0, temperature=2.0, repeat_penalty=1.0, repeat_window=64),
    dict(top_k=3, top_p=1.0, temperature=0.0, repeat_penalty=1.5, repeat_window=64),  # greedy
    # the whole row (Sampler.cs:42-61): top-p nucleus, plain softmax, top_k at or above the vocabulary
    dict(top_k=0, top_p=0.95, temperature=0.8, repeat_penalty=1.1, repeat_window=64),
    dict(top_k=0, top_p=1.0, temperature=1.0, repeat_penalty=1.0, repeat_window=0),
    dict(top_k=-1, top_p=0.5, temperature=0.7, repeat_penalty=1.3, repeat_window=16),
    dict(top_k=1 << 20, top_p=0.9, temperature=1.2, repeat_penalty=1.1, repeat_window=64),
    dict(top_k=0, top_p=0.05, temperature=2.0, repeat_penalty=1.0, repeat_window=0),
]


@pytest.mark.parametrize("vocab", [1000, 32064, 128256])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_sample_matches_oracle(backend, vocab, case):
    rng = np.random.default_rng(1000 * case + vocab)
    o = _opts(**CASES[case])
    if 1024 < o.top_k < vocab:
        pytest.skip("top_k above the device's top-k limit")
    for trial in range(4):
        logits = (rng.standard_normal(vocab) * 3.0).astype(np.float32)
        # a history with repeats and negative logits among the penalised tokens
        recent = rng.integers(0, vocab, size=30).astype(np.int32)
        recent[5] = recent[9] = recent[20]
        logits[recent[:4]] = -np.abs(logits[recent[:4]])
        r = float(rng.uniform(0.02, 0.98))
        want = O.sample(logits, _oracle_opts(o), recent, r)
        got = backend.sample(logits, o, recent, r)
        assert got == want, (vocab, CASES[case], trial, got, want)


def test_sample_seeded_draw_and_errors(backend):
    logits = np.random.default_rng(5).standard_normal(5000).astype(np.float32)
    o = _opts(seed=42)
    want = O.sample(logits, _oracle_opts(o), [])
    assert backend.sample(logits, o, []) == want
    with pytest.raises(CudaBackendError):  # top_k between the device's 1024 and the vocabulary
        backend.sample(logits, _opts(top_k=2000, temperature=1.0), [], 0.5)


@pytest.mark.parametrize("vocab", [7, 8, 1000, 32000])
def test_sample_full_row_ties(backend, vocab):
    """Whole-row softmax and nucleus on rows whose logits take a few values only, so equal
    probabilities fill the nucleus and the selection sort's replay decides the order; also rows
    shorter than the 8-wide lanes, NaN-free infinities, and nuclei that cover the whole row."""
    rng = np.random.default_rng(vocab)
    for trial in range(6):
        logits = rng.integers(-3, 4, size=vocab).astype(np.float32) * 0.5
        if trial == 1:
            logits[rng.integers(0, vocab, size=max(1, vocab // 10))] = -np.inf
        recent = rng.integers(0, vocab, size=12).astype(np.int32)
        for top_p, r in [(0.9, 0.37), (0.5, 0.81), (0.999999, 0.55), (1.0, 0.93), (0.2, 0.05)]:
            o = _opts(top_k=0, top_p=top_p, temperature=0.9, repeat_penalty=1.2, repeat_window=8)
            want = O.sample(logits, _oracle_opts(o), recent, r)
            got = backend.sample(logits, o, recent, r)
            assert got == want, (vocab, trial, top_p, r, got, want)


@pytest.mark.parametrize("vocab", [1000, 32064, 128256])
@pytest.mark.parametrize("top_k", [2, 5, 40, 200, 1024])
def test_sample_top_k_ties(backend, vocab, top_k):
    """Top-k on rows whose values repeat (a few levels, signed zeros among them): the winners tie,
    within the top k and across the k-th place, and the device replays FindTopK's replacement scan
    (Sampler.cs:83-127), so both which equal values win and their order are the reference's."""
    rng = np.random.default_rng(7 * vocab + top_k)
    for trial, (levels, temp) in enumerate([(3, 0.7), (8, 1.0), (60, 1.3)]):
        logits = (rng.integers(-levels, levels + 1, size=vocab) * 0.25).astype(np.float32)
        logits[rng.integers(0, vocab, size=20)] = -0.0
        recent = rng.integers(0, vocab, size=24).astype(np.int32)
        o = _opts(top_k=top_k, top_p=1.0, temperature=temp, repeat_penalty=1.1, repeat_window=32)
        for r in (0.03, 0.5, 0.97):
            want = O.sample(logits, _oracle_opts(o), recent, r)
            got = backend.sample(logits, o, recent, r)
            assert got == want, (vocab, top_k, trial, r, got, want)


@pytest.mark.parametrize("name", ["micro", "micro-gemma", "tiny"])
def test_generate_sampled_matches_oracle(gpu, name):
    from dotllm_b200.engine import CudaModel
    cfg = synth.get(name)
    path = synth.build_model(cfg)
    prompt = synth.prompt_tokens(cfg)
    steps = 24
    rng = np.random.default_rng(77)
    draws = rng.uniform(0.02, 0.98, size=steps).astype(np.float32)
    o = _opts(top_k=40, top_p=0.95, temperature=0.8, repeat_penalty=1.1, repeat_window=16)
    om = O.Model(path)
    os_ = O.Session(om)
    try:
        want = list(os_.generate_sampled(prompt, steps, _oracle_opts(o), draws))
    finally:
        os_.close()
        om.close()
    m = CudaModel.load(path)
    try:
        s = m.session(kv="f32")
        got = list(s.generate_sampled(prompt, steps, o, draws))
        assert got == want
        # a second call resets the session and draws the same tokens
        assert list(s.generate_sampled(prompt, steps, o, draws)) == want
        # the seeded draw when no draws are given
        seeded = _opts(top_k=40, top_p=0.95, temperature=0.8, repeat_penalty=1.1, repeat_window=16, seed=7)
        os_ = O.Session(om := O.Model(path))
        try:
            want7 = list(os_.generate_sampled(prompt, 8, _oracle_opts(seeded)))
        finally:
            os_.close()
            om.close()
        assert list(s.generate_sampled(prompt, 8, seeded)) == want7
        # the whole-row path: softmax over the vocabulary, then the top-p nucleus.  A nucleus of
        # thousands of nearly equal probabilities (the random-weight "tiny" model) orders them by
        # differences far below the logits' fp32 tolerance, so there the draw is checked on the
        # device's own logits; the micro models' nuclei are small enough for the whole sequence.
        top_p = _opts(top_k=0, top_p=0.9, temperature=0.9, repeat_penalty=1.1, repeat_window=16)
        got_p = list(s.generate_sampled(prompt, steps, top_p, draws))
        if name == "tiny":
            s2 = m.session(kv="f32")
            _, lg = s2.prefill(prompt, want_logits=True)
            s2.close()
            assert got_p[0] == O.sample(lg, _oracle_opts(top_p), prompt, float(draws[0]))
        else:
            os_ = O.Session(om := O.Model(path))
            try:
                want_p = list(os_.generate_sampled(prompt, steps, _oracle_opts(top_p), draws))
            finally:
                os_.close()
                om.close()
            assert got_p == want_p
        s.close()
    finally:
        m.close()
