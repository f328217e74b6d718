"""Device-resident decode/prefill (Tier B) vs the CPU oracle on seeded synthetic GGUFs.

Parity bar (the north star's): final logits within max-abs 2e-2 and relative
1e-2 of the reference's managed path at every step, and greedy token ids
identical.  Greedy identity is asserted with an fp32 KV cache.  With the fp16
KV cache the device stores K/V rounded to binary16, which changes logits by
~1e-3 and flips greedy choices wherever the reference's own top-2 margin is
smaller than that (the tiny config has a 1.3e-5 margin at step 21); there the
device is checked against the oracle run with the same fp16 rounding of its
cache, and the logits against the fp32 reference within the tolerance.
"""
import json
import os

import numpy as np
import pytest

from dotllm_b200 import synth
from dotllm_b200.engine import CudaModel, decode_batch
from dotllm_b200.native import CudaBackendError

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
GREEDY = json.load(open(os.path.join(HERE, "golden", "greedy_tokens.json")))
ATOL, RTOL = 2e-2, 1e-2

_models = {}


def model(name):
    if name not in _models:
        _models[name] = CudaModel.load(synth.build_model(synth.get(name)))
    return _models[name]


def oracle_run(oracle, name, steps, prompt=None, kv_fp16=False):
    cfg = synth.get(name)
    m = oracle.Model(synth.build_model(cfg))
    s = oracle.Session(m)
    oracle.set_kv_fp16(kv_fp16)
    try:
        toks, lg = s.generate(synth.prompt_tokens(cfg) if prompt is None else prompt, steps, want_logits=True)
    finally:
        oracle.set_kv_fp16(False)
    return toks, lg


def gpu_teacher_forced(name, prompt, tokens, kv):
    """Prefill the prompt, then feed the oracle's tokens; logits before each sampled token."""
    s = model(name).session(kv=kv)
    nxt, lg0 = s.prefill(prompt, want_logits=True)
    out = [lg0]
    for t in tokens[:-1]:
        _, lg = s.decode(int(t), want_logits=True)
        out.append(lg)
    s.close()
    return np.stack(out)


@pytest.mark.parametrize("name", ["micro", "micro-gemma", "micro-phi3", "micro-q5q8"])
def test_micro_greedy_fp32_kv(gpu, name):
    g = GREEDY[name]
    cfg = synth.get(name)
    s = model(name).session(kv="f32")
    toks = s.generate(synth.prompt_tokens(cfg), g["steps"])
    assert list(toks) == g["tokens"]


@pytest.mark.parametrize("name", ["micro", "micro-gemma", "micro-phi3", "micro-q5q8"])
@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_micro_logits(gpu, oracle, name, kv):
    cfg = synth.get(name)
    prompt = synth.prompt_tokens(cfg)
    toks, ref = oracle_run(oracle, name, 12, prompt, kv_fp16=(kv == "f16"))
    got = gpu_teacher_forced(name, prompt, toks, kv)
    err = np.abs(got - ref)
    assert np.all(err <= ATOL + RTOL * np.abs(ref)), f"max abs err {err.max()}"
    if kv == "f32":
        assert err.max() < 1e-3, err.max()


def test_tiny_greedy_64_fp32_kv(gpu):
    """BASELINE config 0 (tiny LLaMA-like, 64-token prompt): 64 greedy steps identical."""
    g = GREEDY["tiny"]
    cfg = synth.get("tiny")
    s = model("tiny").session(kv="f32")
    toks = s.generate(synth.prompt_tokens(cfg), 64)
    assert list(toks) == g["tokens"][:64]


def test_tiny_logits_fp16_kv(gpu, oracle):
    cfg = synth.get("tiny")
    prompt = synth.prompt_tokens(cfg)
    toks32, ref32 = oracle_run(oracle, "tiny", 64, prompt)
    got = gpu_teacher_forced("tiny", prompt, toks32, "f16")
    err = np.abs(got - ref32)
    assert np.all(err <= ATOL + RTOL * np.abs(ref32)), f"max abs err {err.max()}"
    # greedy with fp16 KV agrees with the reference algorithm run on an fp16-rounded cache
    toks16, _ = oracle_run(oracle, "tiny", 64, prompt, kv_fp16=True)
    s = model("tiny").session(kv="f16")
    assert list(s.generate(prompt, 64)) == list(toks16)


def test_batched_decode_matches_single(gpu):
    name = "micro"
    cfg = synth.get(name)
    m = model(name)
    prompts = [synth.prompt_tokens(cfg, n, session=i) for i, n in enumerate([3, 8, 17])]
    singles = [m.session(kv="f32").generate(p, 10) for p in prompts]
    sessions = [m.session(kv="f32") for _ in prompts]
    cur = [s.prefill(p)[0] for s, p in zip(sessions, prompts)]
    outs = [[c] for c in cur]
    for _ in range(9):
        nxt, _ = decode_batch(sessions, cur)
        cur = list(nxt)
        for o, c in zip(outs, cur):
            o.append(int(c))
    for a, b in zip(outs, singles):
        assert a == list(b)


def test_generate_empty_prompt_uses_bos(gpu, oracle):
    name = "micro"
    toks, _ = oracle_run(oracle, name, 5, prompt=np.zeros(0, dtype=np.int32))
    s = model(name).session(kv="f32")
    assert list(s.generate(np.zeros(0, dtype=np.int32), 5)) == list(toks)


def test_session_errors(gpu):
    m = model("micro")
    s = m.session(max_ctx=16, kv="f32")
    with pytest.raises(CudaBackendError):
        s.prefill(np.arange(17, dtype=np.int32))  # beyond the session's context
    with pytest.raises(CudaBackendError):
        s.prefill(np.array([m.config["vocab"]], dtype=np.int32))  # token outside the vocabulary
    s.prefill(np.arange(16, dtype=np.int32))
    assert s.position == 16
    with pytest.raises(CudaBackendError):
        s.decode(1)  # context full
    s.reset()
    assert s.position == 0


def test_model_load_rejects_garbage(gpu, tmp_path):
    p = tmp_path / "x.gguf"
    p.write_bytes(b"GGUF" + b"\xff" * 100)
    with pytest.raises(CudaBackendError):
        CudaModel.load(str(p))


@pytest.mark.parametrize("B", [6, 20])
def test_large_batch_decode_matches_single(gpu, B):
    """5..32 sessions per step run the batched matmul; logits agree with one-session steps."""
    name = "tiny"
    cfg = synth.get(name)
    m = model(name)
    prompts = [synth.prompt_tokens(cfg, 4 + 3 * i, session=i) for i in range(B)]
    sessions = [m.session(kv="f32") for _ in prompts]
    cur = [s.prefill(p)[0] for s, p in zip(sessions, prompts)]
    singles = [m.session(kv="f32") for _ in prompts]
    for s, p in zip(singles, prompts):
        s.prefill(p)
    for _ in range(3):
        nxt, lg = decode_batch(sessions, cur, want_logits=True)
        for i, s in enumerate(singles):
            n1, l1 = s.decode(int(cur[i]), want_logits=True)
            assert np.abs(lg[i] - l1).max() < 1e-3
            top2 = np.sort(l1)[-2:]
            if top2[1] - top2[0] > 1e-3:
                assert int(nxt[i]) == int(n1)
        cur = [int(t) for t in nxt]


def test_session_outlives_model(gpu):
    """Freeing a model detaches its open sessions: calls on them fail cleanly, free still works."""
    from dotllm_b200 import native
    cfg = synth.get("micro")
    m = CudaModel.load(synth.build_model(cfg))
    s = m.session(kv="f32")
    s.prefill(synth.prompt_tokens(cfg))
    h = native.VP(s._h.value)
    s._h = None  # keep the native session open past the model
    m.close()
    nxt = native.C.c_int32()
    toks = np.zeros(1, dtype=np.int32)
    rc = native.lib().llmdot_cuda_prefill(h, toks.ctypes.data_as(native.I32P), 1, None, native.C.byref(nxt))
    assert rc == -1  # LLMDOT_E_INVALID
    assert native.lib().llmdot_cuda_session_free(h) == 0
