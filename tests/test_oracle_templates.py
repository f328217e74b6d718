"""The oracle's layer templates against a second restatement.  CPU only.

LFM2 short-conv layers and the MoE FFN (InferenceEngine.cs:222-301, 489-542; ConvStateCache.cs;
MoeRouter.cs; TensorOps.Conv1D), which the device does not run yet, are pinned by the assertions
of the reference's own tests (tests/Llmdot.Core.Tests/Inference/ConvLayerTests.cs,
ConvStateCacheTests.cs, MoeRouterTests.cs, line of each test cited).  Every template the
synthetic models use -- LlamaLike (Llama, Qwen2 with Q5_K/Q8_0, Phi-3 with fused QKV), GemmaLike
(embedding scale, attention softcap, sliding window, post-norms, GeGLU) and Lfm2Like with dense or
MoE FFNs -- is also restated a second time in numpy below, from the reference's source, with the
oracle's pinned primitives (dequantisation, softmax with ExpApprox, SiLU / GELU lanes) as its only
shared parts; it must reproduce the oracle's logits.  The GPT-NeoX-like layer is pinned by a
property of the reference's residual (its logits do not depend on the attention weights).
"""
import math

import numpy as np
import pytest

from dotllm_b200 import gguf, synth
from oracle import oracle as O

F32 = gguf.GGML_F32


# ---- ConvLayerTests.cs ------------------------------------------------------------------

def test_conv_state_kernel1_store_is_a_no_op():  # :9-16
    cs = O.ConvState(1, 4, 1)
    cs.store(0, [1, 2, 3, 4])
    assert list(cs.build_input(0, [5, 6, 7, 8], 3)) == [5, 6, 7, 8]


def test_conv_state_kernel4_window():  # :18-47
    cs = O.ConvState(1, 2, 4)
    for d in ([1, 2], [3, 4], [5, 6]):
        cs.store(0, d)
    x = cs.build_input(0, [7, 8], 3)
    assert x.size == 8
    assert list(x) == [1, 3, 5, 7, 2, 4, 6, 8]


def test_conv_state_early_positions_zero_padded():  # :49-65
    cs = O.ConvState(1, 2, 3)
    x = cs.build_input(0, [1, 2], 0)
    assert list(x[:3]) == [0, 0, 1]


def test_conv1d_kernels():  # :67-115
    assert list(O.conv1d([3.0, 5.0], [1.0, 1.0], 1, 2)) == pytest.approx([3.0, 5.0], abs=1e-4)
    third = np.float32(1.0) / np.float32(3)
    assert O.conv1d([1.0, 2.0, 3.0], [third] * 3, 3, 1)[0] == pytest.approx(2.0, abs=1e-2)
    assert list(O.conv1d([1, 2, 3, 4], [1.0, 0.5, 0.5, 1.0], 2, 2)) == pytest.approx([2.0, 5.5], abs=1e-4)


def test_conv1d_lanes_and_tail():
    """Kernels of 8 and more take the 8-lane body, the rest the in-order tail (TensorOps.cs:762-777)."""
    rng = np.random.default_rng(3)
    K, dim = 11, 5
    x = rng.standard_normal(K * dim).astype(np.float32)
    w = rng.standard_normal(K * dim).astype(np.float32)
    want = np.zeros(dim, np.float32)
    for c in range(dim):
        p = x[c * K:(c + 1) * K] * w[c * K:(c + 1) * K]
        lanes = p[:8]
        s = np.float32(((lanes[0] + lanes[1]) + (lanes[2] + lanes[3])) + ((lanes[4] + lanes[5]) + (lanes[6] + lanes[7])))
        for k in range(8, K):
            s = np.float32(s + p[k])
        want[c] = s
    assert np.array_equal(O.conv1d(x, w, K, dim), want)


# ---- ConvStateCacheTests.cs ---------------------------------------------------------------

def test_store_and_build_returns_stored_data():  # :9-27
    cs = O.ConvState(1, 2, 3)
    cs.store(0, [1, 2])
    cs.store(0, [3, 4])
    assert list(cs.build_input(0, [5, 6], 2)) == [1, 3, 5, 2, 4, 6]


def test_rolling_buffer_overwrites_oldest():  # :29-47
    cs = O.ConvState(1, 1, 3)
    for v in (1, 2, 3):
        cs.store(0, [v])
    assert list(cs.build_input(0, [4], 3)) == [2, 3, 4]


def test_reset_clears_state():  # :49-64
    cs = O.ConvState(1, 1, 3)
    cs.store(0, [42])
    cs.reset()
    assert list(cs.build_input(0, [99], 0)) == [0, 0, 99]


def test_multi_layer_isolation():  # :66-86
    cs = O.ConvState(2, 1, 3)
    cs.store(0, [10])
    cs.store(0, [20])
    assert list(cs.build_input(0, [50], 2)) == [10, 20, 50]
    assert list(cs.build_input(1, [50], 2)) == [0, 0, 50]


# ---- MoeRouterTests.cs ------------------------------------------------------------------

def test_route_selects_top_k():  # :10-47
    g = np.zeros((4, 4), np.float32)
    for i in range(4):
        g[i, i] = 1.0
    logits, sel, w = O.moe_route([0.1, 0.9, 0.5, 0.2], g, F32, 4, 2)
    assert list(sel) == [1, 2]
    assert 0.99 <= w.sum() <= 1.01 and w[0] > w[1]
    assert list(logits) == pytest.approx([0.1, 0.9, 0.5, 0.2])


def test_route_single_expert_full_weight():  # :49-76
    g = np.zeros((3, 2), np.float32)
    g[0, 0], g[1, 1], g[2, 0] = 1.0, 10.0, 0.5
    _, sel, w = O.moe_route([1.0, 1.0], g, F32, 3, 1)
    assert list(sel) == [1] and w[0] == 1.0


def test_route_equal_logits_selects_first_k():  # :78-112
    g = np.ones((4, 2), np.float32)
    _, sel, w = O.moe_route([1.0, 1.0], g, F32, 4, 2)
    assert list(sel) == [0, 1]
    assert 0.49 <= w[0] <= 0.51 and 0.49 <= w[1] <= 0.51


def test_route_more_used_than_experts_leaves_minus_one():
    """The scan starts from float.MinValue with a strict >, so once every expert is taken the
    slot stays -1 with weight MinValue, which the softmax turns into 0 (MoeRouter.cs:27-58)."""
    g = np.eye(2, dtype=np.float32)
    _, sel, w = O.moe_route([1.0, 2.0], g, F32, 2, 3)
    assert list(sel) == [1, 0, -1]
    assert w[2] == 0.0 and w.sum() == pytest.approx(1.0)


# ---- an independent restatement of the layer wiring -----------------------------------------

class _Weights:
    def __init__(self, path):
        self.f = gguf.GgufFile(path)
        self.cache = {}

    def has(self, name):
        return name in self.f.tensors

    def __call__(self, name):
        """Dequantised [rows, cols] float32 (rows = dims[1])."""
        if name not in self.cache:
            t = self.f.tensors[name]
            cols = t.dims[0]
            rows = int(np.prod(t.dims[1:])) if len(t.dims) > 1 else 1
            raw = np.frombuffer(bytes(self.f.tensor_bytes(name)), np.uint8)
            self.cache[name] = O.dequantize(raw, t.ggml_type, rows, cols).reshape(rows, cols)
        return self.cache[name]


def _rms(x, w, eps):
    ss = np.float32(np.mean(x.astype(np.float64) ** 2)) + np.float32(eps)
    return (w * x * (np.float32(1) / np.float32(math.sqrt(ss)))).astype(np.float32)


def _rope(v, pos, freq):
    half = freq.size
    ang = (np.float32(pos) * freq).astype(np.float32)
    c, s = np.cos(ang.astype(np.float64)), np.sin(ang.astype(np.float64))
    a, b = v[:half].astype(np.float64), v[half:2 * half].astype(np.float64)
    out = v.copy()
    out[:half], out[half:2 * half] = a * c - b * s, a * s + b * c
    return out


class _Model:
    """Generate's ProcessToken restated from the reference's source in numpy (float64 products,
    float32 state), for the LlamaLike / Lfm2Like templates with dense or MoE FFNs."""

    def __init__(self, cfg, path):
        self.cfg, self.W = cfg, _Weights(path)
        self.freq = (1.0 / np.power(np.float32(cfg.rope_base),
                                    np.arange(0, cfg.head_dim, 2, dtype=np.float32) / np.float32(cfg.head_dim))
                     ).astype(np.float32)
        self.k = {l: [] for l in range(cfg.layers)}
        self.v = {l: [] for l in range(cfg.layers)}
        self.conv = {l: [] for l in range(cfg.layers)}  # conv inputs by position

    def mv(self, name, x):
        return (self.W(name).astype(np.float64) @ x.astype(np.float64)).astype(np.float32)

    def attention(self, l, x, pos):
        c, p = self.cfg, f"blk.{l}."
        hd, H, Hk = c.head_dim, c.heads, c.heads_kv
        if c.qkv_fused:  # one projection, split q | k | v (InferenceEngine.cs:321-331)
            f = self.mv(p + "attn_qkv.weight", x)
            q, k, v = f[:H * hd], f[H * hd:(H + Hk) * hd], f[(H + Hk) * hd:]
        else:
            q, k, v = self.mv(p + "attn_q.weight", x), self.mv(p + "attn_k.weight", x), self.mv(p + "attn_v.weight", x)
        qn = self.W(p + "attn_q_norm.weight")[0] if self.W.has(p + "attn_q_norm.weight") else None
        kn = self.W(p + "attn_k_norm.weight")[0] if self.W.has(p + "attn_k_norm.weight") else None
        q, k = q.reshape(H, hd), k.reshape(Hk, hd)
        if qn is not None:
            q = np.stack([_rms(h, qn, c.eps) for h in q])
        q = np.stack([_rope(h, pos, self.freq) for h in q])
        if kn is not None:
            k = np.stack([_rms(h, kn, c.eps) for h in k])
        k = np.stack([_rope(h, pos, self.freq) for h in k])
        self.k[l].append(k)
        self.v[l].append(v.reshape(Hk, hd))
        K, V = np.stack(self.k[l]), np.stack(self.v[l])  # [t, Hk, hd]
        if c.sliding_window:  # every layer, window start max(0, p + 1 - SW) (:381-383)
            K, V = K[max(0, pos + 1 - c.sliding_window):], V[max(0, pos + 1 - c.sliding_window):]
        out = np.zeros((H, hd), np.float32)
        g = H // Hk
        for h in range(H):
            sc = (K[:, h // g].astype(np.float64) @ q[h].astype(np.float64)).astype(np.float32)
            sc = (sc * (np.float32(1) / np.float32(math.sqrt(hd)))).astype(np.float32)
            pr = O.softmax(sc, softcap=c.attn_softcap)
            out[h] = (pr.astype(np.float64) @ V[:, h // g].astype(np.float64)).astype(np.float32)
        return self.mv(p + "attn_output.weight", out.reshape(-1))

    def conv_op(self, l, x, pos):
        c, p, hid = self.cfg, f"blk.{l}.", self.cfg.hidden
        ip = self.mv(p + "shortconv.in_proj.weight", x)
        b, cc, xx = ip[:hid], ip[hid:2 * hid], ip[2 * hid:]
        bx = (b * xx).astype(np.float32)
        K = c.conv_kernel
        hist = self.conv[l]
        win = np.zeros((hid, K), np.float32)
        for kk in range(K - 1):
            t = pos - (K - 1) + kk
            if t >= 0:
                win[:, kk] = hist[t]
        win[:, K - 1] = bx
        hist.append(bx)
        w = self.W(p + "shortconv.conv.weight")  # [hid, K]
        y = (win.astype(np.float64) * w.astype(np.float64)).sum(axis=1).astype(np.float32)
        y = (y * cc).astype(np.float32)
        return self.mv(p + "shortconv.out_proj.weight", y)

    def ffn(self, l, x):
        c, p = self.cfg, f"blk.{l}."
        if not c.experts:
            gate = self.mv(p + "ffn_gate.weight", x)
            gt = O.gelu(gate) if c.arch.startswith("gemma") else O.silu(gate)  # GeGLU / SwiGLU
            return self.mv(p + "ffn_down.weight", (gt * self.mv(p + "ffn_up.weight", x)).astype(np.float32))
        logits = self.mv(p + "ffn_gate_inp.weight", x)
        sel = []
        for _ in range(c.experts_used):  # first maximum among the experts not yet taken
            best = max((e for e in range(c.experts) if e not in sel), key=lambda e: (logits[e], -e))
            sel.append(best)
        vals = [float(logits[e]) for e in sel]
        ex = [math.exp(v - max(vals)) for v in vals]
        wts = [v / sum(ex) for v in ex]
        acc = np.zeros(c.hidden, np.float64)
        for e, wt in zip(sel, wts):
            gt = O.silu(self.mv(p + f"ffn_gate.{e}.weight", x))
            h = (gt * self.mv(p + f"ffn_up.{e}.weight", x)).astype(np.float32)
            acc += wt * self.mv(p + f"ffn_down.{e}.weight", h).astype(np.float64)
        return acc.astype(np.float32)

    def token(self, tok, pos):
        c, W = self.cfg, self.W
        h = W("token_embd.weight")[tok].astype(np.float32).copy()
        if c.arch.startswith("gemma"):  # EmbeddingScale = MathF.Sqrt(hidden) (ArchitectureResolver.cs:164-166)
            h = (h * np.float32(math.sqrt(np.float32(c.hidden)))).astype(np.float32)
        for l in range(c.layers):
            p = f"blk.{l}."
            x = _rms(h, W(p + "attn_norm.weight")[0], c.eps)
            op = self.conv_op(l, x, pos) if l in c.conv_layers else self.attention(l, x, pos)
            h = (h + op).astype(np.float32)
            if c.post_norm:  # GemmaLike post-norms of h after each residual add (:209-220)
                h = _rms(h, W(p + "post_attention_norm.weight")[0], c.eps)
            x = _rms(h, W(p + "ffn_norm.weight")[0], c.eps)
            h = (h + self.ffn(l, x)).astype(np.float32)
            if c.post_norm:
                h = _rms(h, W(p + "post_ffw_norm.weight")[0], c.eps)
        h = _rms(h, W("output_norm.weight")[0], c.eps)
        head = "output.weight" if W.has("output.weight") else "token_embd.weight"
        return self.mv(head, h)


@pytest.mark.parametrize("name", ["micro-lfm2", "micro-moe", "micro-lfm2moe",
                                  "micro", "micro-gemma", "micro-phi3", "micro-q5q8"])
def test_oracle_templates_match_independent_restatement(name):
    cfg = synth.get(name)
    path = synth.build_model(cfg)
    ref = _Model(cfg, path)
    m = O.Model(path)
    s = O.Session(m)
    s.reset()
    try:
        # past the micro-gemma sliding window (24) so the window start moves
        toks = list(synth.prompt_tokens(cfg, 28 if cfg.sliding_window else 6))
        for pos, t in enumerate(toks):
            want = ref.token(int(t), pos)
            got = s.process_token(int(t), pos)
            # products and sums in another order (float64 here): agreement to fp32 rounding
            assert np.allclose(got, want, rtol=0, atol=2e-4), (name, pos, float(np.abs(got - want).max()))
    finally:
        s.close()
        m.close()


def test_template_resolution():
    """LayerTypes from the attention tensors present (ResolveLayerTypes, ArchitectureResolver.cs:
    226-238) and the per-layer kv heads (0 on conv layers) resolve as the generator wrote them."""
    from dotllm_b200.engine import gguf_config
    for name in ("micro-lfm2", "micro-moe", "micro-lfm2moe"):
        cfg = synth.get(name)
        c = gguf_config(synth.build_model(cfg))
        assert c["template_id"] == (3 if cfg.conv_layers else 0)
        assert c["expert_count"] == cfg.experts and c["heads_kv"] == cfg.heads_kv


def test_golden_template_tokens():
    """Regression pins for the oracle's greedy tokens on the three template models."""
    import json
    import os
    gold = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "template_tokens.json")))
    for name, g in gold.items():
        cfg = synth.get(name)
        m = O.Model(synth.build_model(cfg))
        s = O.Session(m)
        toks, lg = s.generate(synth.prompt_tokens(cfg), g["steps"], want_logits=True)
        s.close()
        m.close()
        assert list(toks) == g["tokens"], name
        assert np.allclose(lg.astype(np.float64).sum(axis=1), g["logit_sum"], rtol=1e-5, atol=1e-3), name


def _with_new_attention(src: str, dst: str, seed: int) -> None:
    """A copy of the GGUF whose attn_q/k/v/output tensors hold other random weights."""
    from dotllm_b200 import quant
    f = gguf.GgufFile(src)
    raw = bytearray(open(src, "rb").read())
    rng = np.random.default_rng(seed)
    for name, t in f.tensors.items():
        if any(k in name for k in ("attn_q.", "attn_k.", "attn_v.", "attn_output.")):
            x = rng.standard_normal((t.dims[1], t.dims[0]), dtype=np.float32) * np.float32(0.05)
            b = quant.quantize(x, t.ggml_type).tobytes()
            assert len(b) == t.n_bytes
            raw[t.data_offset:t.data_offset + t.n_bytes] = b
    open(dst, "wb").write(bytes(raw))


@pytest.mark.parametrize("name,dropped", [("micro-neox", True), ("micro", False)])
def test_neox_layer_adds_only_the_ffn_output(tmp_path, name, dropped):
    """ProcessGptNeoXLikeLayer (InferenceEngine.cs:198-207) adds the FFN result into the attention
    buffer and then only the FFN result into the hidden state (the two-argument Add writes its
    first argument, VectorMath.cs:27-42), so a NeoX model's logits do not depend on its attention
    weights at all; a LlamaLike model's do (the control case)."""
    cfg = synth.get(name)
    a = synth.build_model(cfg)
    b = str(tmp_path / "other_attention.gguf")
    _with_new_attention(a, b, 99)
    prompt = synth.prompt_tokens(cfg)[:6]
    outs = []
    for p in (a, b):
        m = O.Model(p)
        s = O.Session(m)
        outs.append(np.stack([s.process_token(int(t), i) for i, t in enumerate(prompt)]))
        s.close()
        m.close()
    assert np.array_equal(outs[0], outs[1]) == dropped


def test_neox_config_resolves_layer_norm_standard_ffn_parallel_residual():
    c = O.Model(synth.build_model(synth.get("micro-neox"))).config
    assert (c["template_id"], c["norm_is_rms"], c["ffn_type"], c["parallel_residual"]) == (1, 0, 0, 1)
