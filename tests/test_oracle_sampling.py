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


def _nucleus_literal(p, top_p, r, aliased=True):
    """Sample :46-58 with FindNucleus :129-151 and SampleFromProbabilities :153-165, restated
    line by line in numpy float32.  With aliased=True `values` is the softmax row itself (the
    reference passes samplingBuf for both); aliased=False is what a separate buffer would give."""
    f32 = np.float32
    buf = np.array(p, dtype=np.float32)
    vals = buf if aliased else np.zeros_like(buf)
    n = buf.size
    idx = list(range(n))
    for i in range(n - 1):
        mx = i
        for j in range(i + 1, n):
            if buf[idx[j]] > buf[idx[mx]]:
                mx = j
        if mx != i:
            idx[i], idx[mx] = idx[mx], idx[i]
    cum, count = f32(0), 0
    for i in range(n):
        vals[i] = buf[idx[i]]
        cum = f32(cum + vals[i])
        count += 1
        if cum >= f32(top_p):
            break

    def pick(q):
        c = f32(0)
        for i in range(q.size):
            c = f32(c + q[i])
            if f32(r) <= c:
                return i
        return q.size - 1

    if count < n:
        s = f32(0)
        for i in range(count):
            s = f32(s + vals[i])
        inv = f32(1) / s
        return idx[pick((vals[:count] * inv).astype(np.float32))]
    return pick(buf)


def test_top_p_only_reads_the_overwritten_row():
    """TopK <= 0 (or >= the vocabulary) with TopP < 1: FindNucleus writes its values into the
    softmax row it is still reading (Sample :48-50 passes samplingBuf as both), so a token whose
    id is below its rank reads an already-overwritten slot.  Hand-worked on probabilities about
    [0.3, 0.4, 0.2, 0.05, 0.05], TopP 0.85: the order is ids [1, 0, 2, 3, 4]; the aliased values
    are [0.4, 0.4, 0.2] (id 0 reads slot 0, which already holds id 1's 0.4), a separate buffer
    would give [0.4, 0.3, 0.2].  And on [0.1, 0.55, 0.35] with TopP 0.95 the nucleus is the
    whole row, so the fall-through pick reads the overwritten row [0.55, 0.35, 0.55] and returns
    a position."""
    cases = [(np.log(np.array([0.3, 0.4, 0.2, 0.05, 0.05])), 0.85),
             (np.log(np.array([0.1, 0.55, 0.35])), 0.95)]
    for logits, top_p in cases:
        logits = logits.astype(np.float32)
        p = O.softmax(logits.copy())
        differs = False
        for top_k in (0, -3, logits.size):
            o = opts(temperature=1, top_k=top_k, top_p=top_p, repeat_penalty=1, repeat_window=0)
            for r in np.linspace(0.01, 0.99, 99):
                want = _nucleus_literal(p, top_p, r)
                assert O.sample(logits, o, [], r=float(r)) == want, (top_k, top_p, r)
                differs |= want != _nucleus_literal(p, top_p, r, aliased=False)
        assert differs, "the case does not separate the aliased reading from a separate buffer"


def test_top_p_only_random_rows_with_ties():
    """The same restatement on random rows whose logits are coarse (many exact ties, so the
    selection sort's unstable tie order matters), with temperature and repeat penalty applied
    first (Sample :33-34)."""
    rng = np.random.default_rng(11)
    for trial in range(60):
        n = int(rng.integers(3, 40))
        logits = (np.round(rng.standard_normal(n) * 4) / 2).astype(np.float32)
        top_p = float(rng.uniform(0.2, 0.999))
        temp = float(rng.uniform(0.5, 1.5))
        recent = rng.integers(0, n, size=5).astype(np.int32)
        o = opts(temperature=temp, top_k=0, top_p=top_p, repeat_penalty=1.3, repeat_window=4)
        x = logits.copy()
        for t in recent[-4:]:  # ApplyRepeatPenalty :64-81
            x[t] = x[t] / np.float32(1.3) if x[t] > 0 else x[t] * np.float32(1.3)
        x = (x * (np.float32(1) / np.float32(temp))).astype(np.float32)
        p = O.softmax(x)
        for r in rng.uniform(0, 1, size=8):
            assert O.sample(logits, o, recent, r=float(r)) == _nucleus_literal(p, top_p, r), trial


def test_fast_nucleus_equals_the_selection_sort():
    """The sort-and-replay nucleus (the form a device port follows) against the literal quadratic
    selection sort with its aliased writes, on rows full of exact ties (values from a few levels,
    zeros included) and on continuous rows, for nuclei that stop early and that take the whole row."""
    rng = np.random.default_rng(21)
    for trial in range(300):
        n = int(rng.integers(1, 1200))
        if trial % 3 == 0:
            p = rng.standard_normal(n).astype(np.float32) ** 2
        else:
            levels = rng.uniform(0, 1, size=int(rng.integers(1, 6))).astype(np.float32)
            levels[0] = 0.0
            p = rng.choice(levels, size=n).astype(np.float32)
        s = float(p.astype(np.float64).sum())
        top_p = float(rng.uniform(0.0, 1.3)) * max(s, 1e-6)
        a = O.nucleus(p, top_p, fast=False)
        b = O.nucleus(p, top_p, fast=True)
        assert a[0] == b[0], trial
        assert np.array_equal(a[1], b[1]), trial
        assert np.array_equal(a[2], b[2]), trial
