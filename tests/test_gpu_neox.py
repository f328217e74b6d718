"""The GPT-NeoX-like execution template on the device (ProcessGptNeoXLikeLayer,
src/Llmdot.Core/Inference/InferenceEngine.cs:198-207) against the oracle, on the phi2-shaped
synthetic model (LayerNorm, non-gated GELU FFN).

The reference's layer adds only the FFN result to the hidden state (the attention result lands in a
buffer the hidden state never reads), so the device computes h += FFN(LayerNorm(h)) per layer and
skips the attention; the oracle restates the full reference layer, attention included.  Bars: the
committed greedy tokens of the oracle (tests/golden/template_tokens.json) identical, logits within
the north star's 2e-2 + 1e-2 relative at every step (and within 1e-3 here, a shallow model).
"""
import json
import os

import numpy as np
import pytest

from dotllm_b200 import synth
from dotllm_b200.engine import CudaModel

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "golden", "template_tokens.json")))
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def neox():
    m = CudaModel.load(synth.build_model(synth.get("micro-neox")))
    yield m
    m.close()


def test_neox_greedy_matches_golden(gpu, neox):
    g = GOLD["micro-neox"]
    cfg = synth.get("micro-neox")
    for kv in ("f32", "f16"):
        s = neox.session(kv=kv)
        assert list(s.generate(synth.prompt_tokens(cfg), g["steps"])) == g["tokens"], kv
        s.close()


def test_neox_logits_vs_oracle(gpu, oracle, neox):
    cfg = synth.get("micro-neox")
    prompt = synth.prompt_tokens(cfg)
    om = oracle.Model(synth.build_model(cfg))
    os_ = oracle.Session(om)
    toks, ref = os_.generate(prompt, 12, want_logits=True)
    s = neox.session(kv="f32")
    _, lg0 = s.prefill(prompt, want_logits=True)
    got = [lg0]
    for t in toks[:-1]:
        got.append(s.decode(int(t), want_logits=True)[1])
    err = np.abs(np.stack(got) - ref)
    assert np.all(err <= ATOL + RTOL * np.abs(ref)), err.max()
    assert err.max() < 1e-3, err.max()


def test_neox_batched_matches_single(gpu, neox):
    """Several sessions per step (the batched matmul and per-row LayerNorm) equal one-session steps."""
    from dotllm_b200.engine import decode_batch
    cfg = synth.get("micro-neox")
    prompts = [synth.prompt_tokens(cfg, n, session=i) for i, n in enumerate([3, 8, 17, 5, 9, 4])]
    singles = [neox.session(kv="f32").generate(p, 6) for p in prompts]
    ss = [neox.session(kv="f32") for _ in prompts]
    cur = [s.prefill(p)[0] for s, p in zip(ss, prompts)]
    outs = [[c] for c in cur]
    for _ in range(5):
        cur = [int(c) for c in decode_batch(ss, cur)[0]]
        for o, c in zip(outs, cur):
            o.append(c)
    assert outs == [list(x) for x in singles]
