"""The oracle's restatement of Sampler.Sample (src/Llmdot.Core/Sampling/Sampler.cs:24-165),
pinned by the assertions of the reference's own tests
(tests/Llmdot.Core.Tests/Sampling/SamplerTests.cs, line of each test cited).  CPU only.

The seeded draw restates new System.Random(seed).NextSingle() (the .NET-5-compatible seeded
generator); the reference tests only assert properties of it (determinism, range), and so do
these.  Its first doubles for seeds 0 and 42 are the widely quoted 0.72624326996796 and
0.668106465911542, which the float draws below round from.
"""
import numpy as np
import pytest

from oracle import oracle as O


def opts(**kw):
    return O.SamplingOptions(**kw)


def peak(size, idx, value=10.0):  # MakeLogits :11-17
    x = np.full(size, 0.01, dtype=np.float32)
    x[idx] = value
    return x


def test_seeded_draw_is_the_first_net_random_double():
    assert O.net_random_single(0) == pytest.approx(0.72624326996796, abs=1e-7)
    assert O.net_random_single(42) == pytest.approx(0.668106465911542, abs=1e-7)
    assert O.net_random_single(-42) == O.net_random_single(42)  # Math.Abs(seed)
    assert 0.0 <= O.net_random_single(12345) < 1.0


def test_temperature_zero_is_argmax():  # :20, :34, :539
    assert O.sample(peak(100, 42), opts(temperature=0), [], 0.5) == 42
    assert O.sample(peak(100, 7), opts(temperature=0, top_k=5, top_p=0.5, repeat_penalty=2.0), [7], 0.5) == 7
    assert O.sample(peak(100, 3), opts(temperature=-1.0), [], 0.5) == 3


def test_top_k_limits_and_seed_determines():  # :73, :99
    x = np.full(100, 0.001, dtype=np.float32)
    x[:3] = [100, 90, 80]
    o = opts(temperature=1, top_k=3, top_p=1, repeat_penalty=1, repeat_window=0, seed=99)
    a, b = O.sample(x, o), O.sample(x, o)
    assert a == b and 0 <= a <= 2


def test_top_p():  # :127, :153
    x = np.full(100, 0.001, dtype=np.float32)
    x[:3] = [10, 5, 3]
    assert O.sample(x, opts(temperature=1, top_k=0, top_p=0.5, repeat_penalty=1, repeat_window=0, seed=42)) <= 2
    y = np.full(100, 0.01, dtype=np.float32)
    y[0] = 100
    assert O.sample(y, opts(temperature=1, top_k=0, top_p=0.01, repeat_penalty=1, repeat_window=0, seed=42)) == 0


def test_repeat_penalty():  # :177, :201, :240, :263, :286
    x = np.zeros(100, dtype=np.float32)
    x[50], x[51] = 100, 50
    o = opts(temperature=0.5, top_k=100, top_p=1, repeat_penalty=100, repeat_window=64, seed=42)
    assert O.sample(x, o, [50]) != 50
    y = np.full(100, -1.0, dtype=np.float32)
    y[50], y[30] = -0.5, 10
    no = opts(temperature=1, top_k=0, top_p=1, repeat_penalty=1, repeat_window=64, seed=42)
    pen = opts(temperature=1, top_k=0, top_p=1, repeat_penalty=100, repeat_window=64, seed=42)
    assert O.sample(y, no, []) == 30
    assert O.sample(y, pen, [30]) != 30
    z = peak(100, 42)
    assert O.sample(z, opts(temperature=0.5, top_k=0, top_p=1, repeat_penalty=100, repeat_window=0, seed=42), [42]) == 42
    assert O.sample(z, opts(temperature=0.5, top_k=0, top_p=1, repeat_penalty=1, repeat_window=64, seed=42), [42]) == 42
    assert O.sample(z, opts(temperature=0.5, top_k=0, top_p=1, repeat_penalty=100, repeat_window=64, seed=42), []) == 42


def test_seed_determinism_and_spread():  # :309, :333
    x = (np.arange(100) * 0.1).astype(np.float32)
    o = opts(temperature=0.8, top_k=40, top_p=0.95, repeat_penalty=1, repeat_window=64, seed=12345)
    assert O.sample(x, o) == O.sample(x, o)
    y = (np.arange(100) * 0.5).astype(np.float32)
    seen = {O.sample(y, opts(temperature=1, top_k=10, top_p=0.95, repeat_penalty=1, repeat_window=64, seed=s))
            for s in range(20)}
    assert len(seen) > 1


def test_defaults_and_top_k_one():  # :360, :376, :391
    x = (np.arange(32000) * 0.001).astype(np.float32)
    x[100] = 5
    assert 0 <= O.sample(x, opts(seed=42)) < 32000
    y = (np.arange(100) * 0.1).astype(np.float32)
    assert 0 <= O.sample(y, opts(seed=7)) < 100
    assert O.sample(peak(100, 42), opts(temperature=1, top_k=1, top_p=1, repeat_penalty=1, repeat_window=0, seed=42)) == 42


def test_pick_is_the_first_cumulative_probability_reaching_r():
    """SampleFromProbabilities :153-165 on a hand-computed top-2: softmax([1, 0]) = [e/(e+1), 1/(e+1)]."""
    x = np.full(10, -50.0, dtype=np.float32)
    x[3], x[7] = 1.0, 0.0
    o = opts(temperature=1, top_k=2, top_p=1, repeat_penalty=1, repeat_window=0)
    p0 = np.e / (np.e + 1)
    assert O.sample(x, o, [], r=p0 - 1e-3) == 3
    assert O.sample(x, o, [], r=p0 + 1e-3) == 7
    assert O.sample(x, o, [], r=1.0) == 7


def test_sampled_generation_matches_golden():
    """The oracle's Generate with Sampler.Sample against tests/golden/sampled_tokens.json (made by
    tests/golden/make_golden.py): a regression pin for the restatement."""
    import json
    import os

    from dotllm_b200 import synth
    gold = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "sampled_tokens.json")))
    so = gold["options"]
    O.set_threads(max(1, O.max_threads()))
    for name in ("micro", "micro-gemma", "tiny"):
        g = gold[name]
        cfg = synth.get(name)
        m = O.Model(synth.build_model(cfg))
        s = O.Session(m)
        try:
            prompt = synth.prompt_tokens(cfg)
            seeded = s.generate_sampled(prompt, g["steps"], O.SamplingOptions(seed=g["seed"], **so))
            drawn = s.generate_sampled(prompt, g["steps"], O.SamplingOptions(**so), np.asarray(g["draws"], np.float32))
        finally:
            s.close()
            m.close()
        assert list(seeded) == g["seeded_tokens"], name
        assert list(drawn) == g["drawn_tokens"], name
