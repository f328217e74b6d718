"""The device-resident decode loop (llmdot_cuda_decode_steps) and the per-element matvec path.

decode_steps replays the captured decode-step graph n times with the greedy id of each step fed
back on the device; its tokens must equal step-by-step Generate.  A model loaded with
LLMDOT_REFERENCE_MATVEC=1 runs every matvec through the generic per-element kernel and the prompt
token by token, and must still reproduce the oracle's greedy ids.
"""
import json
import os

import pytest

from dotllm_b200 import synth
from dotllm_b200.engine import CudaModel, decode_batch, decode_steps

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
GREEDY = json.load(open(os.path.join(HERE, "golden", "greedy_tokens.json")))

_models = {}


def load_with(name, env):
    key = (name, tuple(sorted(env.items())))
    if key not in _models:
        saved = {k: os.environ.get(k) for k in env}
        os.environ.update(env)
        try:
            _models[key] = CudaModel.load(synth.build_model(synth.get(name)))
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
    return _models[key]


def test_device_loop_matches_generate(gpu):
    """decode_steps: n greedy steps fed back on the device == step-by-step generate."""
    name = "tiny"
    cfg = synth.get(name)
    m = load_with(name, {})
    prompt = synth.prompt_tokens(cfg)
    ref = m.session(kv="f16").generate(prompt, 40)
    s = m.session(kv="f16")
    first, _ = s.prefill(prompt)
    toks, ms, kps = decode_steps([s], [first], 39)
    assert [first] + [int(t) for t in toks[:, 0]] == list(ref)
    assert kps > 0 and ms > 0
    assert s.position == len(prompt) + 39


def test_device_loop_batched_matches_single(gpu):
    name = "micro"
    cfg = synth.get(name)
    m = load_with(name, {})
    prompts = [synth.prompt_tokens(cfg, n, session=i) for i, n in enumerate([3, 8, 17])]
    singles = [m.session(kv="f32").generate(p, 15) for p in prompts]
    sessions = [m.session(kv="f32") for _ in prompts]
    cur = [s.prefill(p)[0] for s, p in zip(sessions, prompts)]
    outs = [[c] for c in cur]
    for _ in range(9):
        cur = [int(c) for c in decode_batch(sessions, cur)[0]]
        for o, c in zip(outs, cur):
            o.append(c)
    more, _, _ = decode_steps(sessions, cur, 5)
    assert more.shape == (5, 3)
    for i, o in enumerate(outs):
        o.extend(int(t) for t in more[:, i])
    assert outs == [list(x) for x in singles]


@pytest.mark.parametrize("name", ["micro", "micro-gemma"])
def test_reference_matvec_path(gpu, name):
    """Per-element matvec everywhere, prompt token by token: the oracle's greedy ids."""
    g = GREEDY[name]
    m = load_with(name, {"LLMDOT_REFERENCE_MATVEC": "1"})
    s = m.session(kv="f32")
    assert list(s.generate(synth.prompt_tokens(synth.get(name)), g["steps"])) == g["tokens"]
