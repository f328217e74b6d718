"""Host-side data formats: reference-layout quantisers, the GGUF writer/reader,
config resolution, and the oracle's greedy output pinned by committed fixtures."""
import json
import os

import numpy as np
import pytest

from dotllm_b200 import gguf, quant, synth

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("t,tol", [(gguf.GGML_Q4_K, 0.12), (gguf.GGML_Q5_K, 0.06), (gguf.GGML_Q6_K, 0.03),
                                   (gguf.GGML_Q8_0, 0.01), (gguf.GGML_Q4_0, 0.15)])
def test_quantiser_roundtrip(oracle, t, tol):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((6, 1024), dtype=np.float32) * 0.02
    b = quant.quantize(x, t)
    assert b.shape == (6, gguf.byte_count(t, 1024))
    y = oracle.dequantize(b, t, 6, 1024).reshape(6, 1024)
    assert np.linalg.norm(y - x) / np.linalg.norm(x) < tol


def test_quantiser_uses_min_offsets(oracle):
    """Q4_K blocks must exercise the dmin*m term of the reference formula."""
    rng = np.random.default_rng(3)
    b = quant.quantize(rng.standard_normal((4, 2048), dtype=np.float32) * 0.02, gguf.GGML_Q4_K).reshape(-1, 144)
    scales = b[:, 4:16].astype(np.uint32)
    w = scales[:, 0::3] | (scales[:, 1::3] << 8) | (scales[:, 2::3] << 16)
    m_even = (w >> 6) & 63
    assert (m_even > 0).mean() > 0.2


def test_quantiser_rejects_ragged_rows():
    with pytest.raises(ValueError):
        quant.quantize(np.zeros((2, 300), dtype=np.float32), gguf.GGML_Q4_K)


def test_gguf_roundtrip(tmp_path):
    md = gguf.Metadata().add("general.architecture", gguf.STR, "llama").add("x.y", gguf.F32, 1.5)
    md.add("arr", gguf.ARR, [1, 2, 3], gguf.I32)
    rng = np.random.default_rng(1)
    w = quant.quantize(rng.standard_normal((3, 256), dtype=np.float32), gguf.GGML_Q6_K)
    n = np.arange(5, dtype=np.float32)
    infos = [gguf.TensorInfo("a.weight", [256, 3], gguf.GGML_Q6_K), gguf.TensorInfo("n.weight", [5], gguf.GGML_F32)]
    data = {"a.weight": w.tobytes(), "n.weight": n.tobytes()}
    p = str(tmp_path / "t.gguf")
    gguf.write_gguf(p, md, infos, lambda t: data[t.name])
    f = gguf.GgufFile(p)
    assert f.metadata["general.architecture"] == "llama"
    assert f.metadata["x.y"] == pytest.approx(1.5)
    assert f.metadata["arr"] == [1, 2, 3]
    assert f.tensors["a.weight"].dims == [256, 3]
    assert bytes(f.tensor_bytes("a.weight")) == w.tobytes()
    assert np.array_equal(np.frombuffer(bytes(f.tensor_bytes("n.weight")), dtype=np.float32), n)
    assert f.tensors["a.weight"].data_offset % 32 == 0 and f.tensors["n.weight"].data_offset % 32 == 0


def test_gguf_rejects_bad_magic(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGML" + b"\0" * 64)
    with pytest.raises(ValueError):
        gguf.GgufFile(str(p))


@pytest.mark.parametrize("name", ["micro", "micro-gemma", "micro-phi3", "micro-q5q8"])
def test_config_resolution(oracle, name):
    """ArchitectureResolver restatement: the oracle resolves what the generator wrote."""
    cfg = synth.get(name)
    m = oracle.Model(synth.build_model(cfg))
    c = m.config
    assert (c["hidden"], c["layers"], c["heads"], c["heads_kv"], c["head_dim"], c["ffn"], c["vocab"]) == (
        cfg.hidden, cfg.layers, cfg.heads, cfg.heads_kv, cfg.head_dim, cfg.ffn, cfg.vocab)
    assert c["tied"] == int(cfg.tied)
    assert c["qkv_fused"] == int(cfg.qkv_fused)
    assert c["template_id"] == (2 if cfg.arch.startswith("gemma") else 0)
    assert c["ffn_type"] == (2 if cfg.arch.startswith("gemma") else 1)
    assert c["eos"] == -1
    if cfg.arch.startswith("gemma"):
        assert c["emb_scale"] == pytest.approx(np.sqrt(np.float32(cfg.hidden)))
        assert c["has_attn_cap"] and c["has_final_cap"] and c["has_post_norm"]
        assert c["sliding_window"] == cfg.sliding_window
    m.close()


def test_oracle_rejects_unknown_arch(oracle, tmp_path):
    md = gguf.Metadata().add("general.architecture", gguf.STR, "mamba")
    p = str(tmp_path / "m.gguf")
    gguf.write_gguf(p, md, [], lambda t: b"")
    with pytest.raises(ValueError, match="Unsupported GGUF architecture"):
        oracle.Model(p)


GREEDY = json.load(open(os.path.join(HERE, "golden", "greedy_tokens.json")))


@pytest.mark.parametrize("name", ["micro", "micro-gemma", "micro-phi3", "micro-q5q8", "tiny"])
def test_oracle_greedy_regression(oracle, name):
    """The oracle reproduces its committed greedy tokens (catches drift in the checker)."""
    g = GREEDY[name]
    cfg = synth.get(name)
    m = oracle.Model(synth.build_model(cfg))
    s = oracle.Session(m)
    toks, lg = s.generate(synth.prompt_tokens(cfg), g["steps"], want_logits=True)
    assert list(toks) == g["tokens"]
    assert np.allclose(lg.astype(np.float64).sum(axis=1), g["logit_sum"], rtol=1e-5, atol=1e-3)
    s.close()
    m.close()


def test_oracle_threads_do_not_change_results(oracle):
    cfg = synth.get("micro")
    m = oracle.Model(synth.build_model(cfg))
    s = oracle.Session(m)
    prompt = synth.prompt_tokens(cfg)
    oracle.set_threads(1)
    a = s.generate(prompt, 6, want_logits=True)[1]
    oracle.set_threads(max(1, oracle.max_threads()))
    b = s.generate(prompt, 6, want_logits=True)[1]
    assert np.array_equal(a, b)


def test_weight_bytes_llama1b():
    """Bytes streamed per decode step for the Llama-3.2-1B shape (roofline numerator)."""
    wb = synth.weight_bytes(synth.get("llama1b"))
    assert wb["layers"] == 620888064 + 16 * 2 * 2048 * 4 + 2048 * 4  # + per-layer and final norm vectors
    assert wb["logits"] == 147750912
