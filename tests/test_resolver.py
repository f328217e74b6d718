"""ArchitectureResolver.Resolve (src/Llmdot.Core/Loading/ArchitectureResolver.cs:14-112) in the
library's native GGUF parser (llmdot_cuda_gguf_config, host only) and in the oracle, on the
files of the reference's tests/Llmdot.Core.Tests/Loading/ArchitectureResolverTests.cs,
SmolLm2ResolverTests.cs and GgufReaderTests.cs (line of each test cited), and against each other.
CPU only.

The files are written byte for byte as that test's WriteGguf helper (:179-245) writes them:
GGUF v3, no tensors, UInt32 / Float32 / String values, and Bool written as a 4-byte UInt32
(the reader takes its first byte; the other three fall into the empty data section).
"""
import struct

import numpy as np
import pytest

from dotllm_b200.engine import gguf_config
from dotllm_b200.native import CudaBackendError
from oracle import oracle as O

U32, F32, BOOL, STR = 4, 6, 7, 8  # GgufValueType


def _s(v: str) -> bytes:
    b = v.encode()
    return struct.pack("<Q", len(b)) + b


def write_meta_gguf(path, entries, tensor_names=()):
    """Metadata, then (SmolLm2ResolverTests.cs:188-215) one tensor info per name -- 1 dim of 1,
    F32, offset 0 -- padding to 32 bytes and a 0f per tensor."""
    out = b"GGUF" + struct.pack("<IQQ", 3, len(tensor_names), len(entries))
    for key, t, v in entries:
        if t == "raw":  # type tag and payload already encoded
            out += _s(key) + v
            continue
        out += _s(key) + struct.pack("<I", t)
        if t == U32:
            out += struct.pack("<I", v)
        elif t == F32:
            out += struct.pack("<f", v)
        elif t == STR:
            out += _s(v)
        elif t == BOOL:
            out += struct.pack("<I", 1 if v else 0)
    for name in tensor_names:
        out += _s(name) + struct.pack("<IQIQ", 1, 1, 0, 0)
    if tensor_names:
        out += b"\0" * ((32 - len(out) % 32) % 32) + struct.pack("<f", 0.0) * len(tensor_names)
    with open(path, "wb") as f:
        f.write(out)
    return str(path)


def _arch(name, hidden, layers, ctx, ffn, heads, heads_kv, eps):
    return [("general.architecture", STR, name), (f"{name}.embedding_length", U32, hidden),
            (f"{name}.block_count", U32, layers), (f"{name}.context_length", U32, ctx),
            (f"{name}.feed_forward_length", U32, ffn), (f"{name}.attention.head_count", U32, heads),
            (f"{name}.attention.head_count_kv", U32, heads_kv),
            (f"{name}.attention.layer_norm_rms_epsilon", F32, eps)]


LLAMA = _arch("llama", 4096, 32, 4096, 11008, 32, 32, 1e-5)                             # :34-58
PHI2 = _arch("phi2", 2560, 32, 2048, 10240, 32, 32, 1e-5) + [("phi2.use_parallel_residual", BOOL, True)]  # :61-82
GEMMA = _arch("gemma", 2048, 18, 8192, 16384, 8, 1, 1e-6)                               # :85-106
GQA = _arch("llama", 4096, 32, 8192, 14336, 32, 8, 1e-5)                                # :109-128
LFM2 = _arch("lfm2", 2048, 16, 32768, 6656, 16, 8, 1e-5) + [("lfm2.conv_L_cache", U32, 3)]  # :131-155


def attention_type(c):  # DetermineAttentionType :123-128
    return "MHA" if c["heads"] == c["heads_kv"] else ("MQA" if c["heads_kv"] == 1 else "GQA")


def both(path):
    """The library's resolution, and the oracle's (which must agree field for field)."""
    c = gguf_config(path)
    m = O.Model(path)
    try:
        o = m.config
    finally:
        m.close()
    for k, v in o.items():
        assert c[k] == pytest.approx(v, rel=0, abs=0), k
    return c


def test_missing_architecture(tmp_path):  # :11-19
    p = write_meta_gguf(tmp_path / "a.gguf", [])
    with pytest.raises(CudaBackendError, match="missing 'general.architecture'"):
        gguf_config(p)
    with pytest.raises(ValueError, match="missing 'general.architecture'"):
        O.Model(p)


def test_unsupported_architecture(tmp_path):  # :21-31
    p = write_meta_gguf(tmp_path / "a.gguf", [("general.architecture", STR, "fancy_new_model")])
    with pytest.raises(CudaBackendError, match="Unsupported GGUF architecture"):
        gguf_config(p)
    with pytest.raises(ValueError, match="Unsupported GGUF architecture"):
        O.Model(p)


def test_llama_is_llama_like(tmp_path):  # :34-58
    c = both(write_meta_gguf(tmp_path / "a.gguf", LLAMA))
    assert c["template_id"] == 0 and c["hidden"] == 4096 and c["layers"] == 32
    assert attention_type(c) == "MHA"
    assert c["norm_is_rms"] == 1 and c["eps"] == np.float32(1e-5)
    # the defaults the test file leaves to the resolver
    assert (c["vocab"], c["bos"], c["eos"], c["head_dim"], c["rope_dim"]) == (0, 1, 2, 128, 128)
    assert c["rope_base"] == 10000.0 and c["emb_scale"] == 1.0 and c["tied"] == 1
    assert c["parallel_residual"] == 0 and c["ffn_type"] == 0 and c["qkv_fused"] == 0


def test_phi2_is_neox_like_with_parallel_residual(tmp_path):  # :61-82
    c = both(write_meta_gguf(tmp_path / "a.gguf", PHI2))
    assert c["template_id"] == 1 and c["parallel_residual"] == 1


def test_gemma_is_gemma_like_mqa_with_embedding_scale(tmp_path):  # :85-106
    c = both(write_meta_gguf(tmp_path / "a.gguf", GEMMA))
    assert c["template_id"] == 2 and attention_type(c) == "MQA"
    assert c["emb_scale"] == np.sqrt(np.float32(2048), dtype=np.float32)


def test_gqa_detected(tmp_path):  # :109-128
    c = both(write_meta_gguf(tmp_path / "a.gguf", GQA))
    assert attention_type(c) == "GQA" and c["heads_kv"] == 8


def test_lfm2_is_lfm2_like(tmp_path):  # :131-155 (the oracle stops at LFM2: outside its path)
    c = gguf_config(write_meta_gguf(tmp_path / "a.gguf", LFM2))
    assert c["template_id"] == 3 and c["layers"] == 16 and attention_type(c) == "GQA"


def test_non_lfm2_has_no_conv_template(tmp_path):  # :158-178
    c = both(write_meta_gguf(tmp_path / "a.gguf", LLAMA))
    assert c["template_id"] != 3


def test_no_norm_epsilon_is_refused(tmp_path):  # ResolveNormType :131-141
    p = write_meta_gguf(tmp_path / "a.gguf", LLAMA[:-1])
    with pytest.raises(CudaBackendError, match="No norm epsilon"):
        gguf_config(p)
    with pytest.raises(ValueError, match="No norm epsilon"):
        O.Model(p)


def test_layer_norm_epsilon_and_rope_scaling(tmp_path):
    """ResolveNormType's LayerNorm branch and ResolveRopeScaling (:169-183), case-insensitive."""
    e = LLAMA[:-1] + [("llama.attention.layer_norm_epsilon", F32, 1e-6),
                      ("llama.rope.scaling.type", STR, "Linear"), ("llama.rope.scaling.factor", F32, 4.0),
                      ("llama.rope.freq_base", F32, 500000.0), ("llama.attention.sliding_window", U32, 4096),
                      ("llama.final_logit_softcapping", F32, 30.0), ("tokenizer.ggml.eos_token_id", U32, 7)]
    c = both(write_meta_gguf(tmp_path / "a.gguf", e))
    assert c["norm_is_rms"] == 0 and c["eps"] == np.float32(1e-6)
    assert c["rope_scaling"] == 1 and c["rope_factor"] == 4.0 and c["rope_base"] == 500000.0
    assert c["sliding_window"] == 4096 and c["has_final_cap"] == 1 and c["final_cap"] == 30.0
    assert c["has_attn_cap"] == 0 and c["eos"] == 7


def test_synthetic_models_resolve_alike(tmp_path):
    """Full generated models (tensors included: fused QKV, gate, post-norms, tied heads)."""
    from dotllm_b200 import synth
    for name in ("micro", "micro-gemma", "micro-phi3", "micro-q5q8"):
        both(synth.build_model(synth.get(name)))


def test_gguf_reader_cases(tmp_path):
    """tests/Llmdot.Core.Tests/Loading/GgufReaderTests.cs through the resolving entry points:
    bad magic is refused by the reader (:8-18); the minimal v3 header (:20-31) parses and then
    stops at the resolver's missing-architecture check; the one-string metadata file (:33-55)
    parses its value, which the resolver names in its missing-epsilon message."""
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"\0\0\0\0")
    with pytest.raises(CudaBackendError, match="Invalid GGUF magic"):
        gguf_config(str(bad))
    with pytest.raises(ValueError, match="Invalid GGUF magic"):
        O.Model(str(bad))
    p = write_meta_gguf(tmp_path / "min.gguf", [])
    with pytest.raises(CudaBackendError, match="missing 'general.architecture'"):
        gguf_config(p)
    p = write_meta_gguf(tmp_path / "phi2.gguf", [("general.architecture", STR, "phi2")])
    with pytest.raises(CudaBackendError, match="architecture 'phi2'"):
        gguf_config(p)
    with pytest.raises(ValueError, match="architecture 'phi2'"):
        O.Model(p)
    old = tmp_path / "v1.gguf"  # GgufReader.cs: versions below 2 are refused
    old.write_bytes(b"GGUF" + struct.pack("<IQQ", 1, 0, 0))
    with pytest.raises(CudaBackendError, match="Unsupported GGUF version"):
        gguf_config(str(old))


# ---- tests/Llmdot.Core.Tests/Loading/SmolLm2ResolverTests.cs --------------------------------

def _smol(hidden, layers, ffn, heads, heads_kv, key_length=True, rope=False):
    e = [("general.architecture", STR, "llama"), ("llama.embedding_length", U32, hidden),
         ("llama.block_count", U32, layers), ("llama.context_length", U32, 2048),
         ("llama.feed_forward_length", U32, ffn), ("llama.attention.head_count", U32, heads),
         ("llama.attention.head_count_kv", U32, heads_kv)]
    if key_length:
        e.append(("llama.attention.key_length", U32, 64))
    e.append(("llama.attention.layer_norm_rms_epsilon", F32, 1e-5))
    if rope:
        e.append(("llama.rope.freq_base", F32, 10000.0))
    return e


@pytest.mark.parametrize("entries,want", [
    (_smol(576, 30, 1536, 9, 3, rope=True),                                            # :11-44
     dict(template_id=0, hidden=576, layers=30, context=2048, ffn=1536, heads=9, heads_kv=3, head_dim=64,
          ffn_type=1, norm_is_rms=1, rope_base=10000.0, tied=1)),
    (_smol(960, 32, 2560, 15, 5), dict(hidden=960, layers=32, ffn=2560, heads=15, heads_kv=5)),     # :46-71
    (_smol(2048, 24, 8192, 32, 32), dict(hidden=2048, layers=24, ffn=8192, heads=32, heads_kv=32)),  # :73-98
])
def test_smollm2_configs(tmp_path, entries, want):
    c = both(write_meta_gguf(tmp_path / "a.gguf", entries, ["blk.0.ffn_gate.weight"]))
    for k, v in want.items():
        assert c[k] == v, k
    assert attention_type(c) == ("MHA" if c["heads"] == c["heads_kv"] else "GQA")


def test_smollm2_tied_and_separate_output(tmp_path):  # :100-140
    e = _smol(576, 30, 1536, 9, 3, key_length=False)
    assert both(write_meta_gguf(tmp_path / "t.gguf", e, ["token_embd.weight"]))["tied"] == 1
    assert both(write_meta_gguf(tmp_path / "s.gguf", e, ["token_embd.weight", "output.weight"]))["tied"] == 0


def test_smollm2_swiglu_from_gate_tensor(tmp_path):  # :142-161
    e = _smol(576, 30, 1536, 9, 3, key_length=False)
    assert both(write_meta_gguf(tmp_path / "a.gguf", e, ["blk.0.ffn_gate.weight"]))["ffn_type"] == 1
    assert both(write_meta_gguf(tmp_path / "b.gguf", e, ["blk.0.ffn_up.weight"]))["ffn_type"] == 0


def test_smollm2_rope_parameters(tmp_path):  # :163-186
    e = _smol(576, 30, 1536, 9, 3, rope=True) + [("llama.rope.dimension_count", U32, 64)]
    c = both(write_meta_gguf(tmp_path / "a.gguf", e))
    assert c["rope_base"] == 10000.0 and c["rope_dim"] == 64


ARR = 9


def _nested(depth_payloads):
    """ARR of ARR of U32, and ARR of ARR of STR (GgufReader.ReadGgufArray recurses)."""
    inner_u32 = struct.pack("<IQ", U32, 2) + struct.pack("<II", 7, 8)
    inner_str = struct.pack("<IQ", STR, 1) + _s("x")
    return [("x.nested_u32", "raw", struct.pack("<IIQ", ARR, ARR, 2) + inner_u32 + inner_u32),
            ("x.nested_str", "raw", struct.pack("<IIQ", ARR, ARR, 1) + inner_str)]


def test_nested_metadata_arrays_are_read_past(tmp_path):
    """A file whose metadata holds arrays of arrays resolves like one without them: both parsers
    read past the nested values, as GgufReader does (GgufReader.cs:84-96)."""
    plain = both(write_meta_gguf(tmp_path / "a.gguf", LLAMA))
    nested = both(write_meta_gguf(tmp_path / "b.gguf", _nested(2) + LLAMA))
    assert plain == nested


def test_duplicate_metadata_key_last_wins(tmp_path):
    """GgufReader stores `values[key] = ...`, so a repeated key keeps its last value."""
    e = LLAMA + [("llama.block_count", U32, 7)]
    assert both(write_meta_gguf(tmp_path / "a.gguf", e))["layers"] == 7


def test_unsupported_tensor_type_refused_even_when_empty(tmp_path):
    """TensorSize.ByteCount throws for a type it does not know (TensorSize.cs:7-24), before any
    element count matters: a zero-element IQ2_XXS tensor still fails the load."""
    out = bytearray(open(write_meta_gguf(tmp_path / "a.gguf", LLAMA), "rb").read())
    struct.pack_into("<Q", out, 8, 1)  # one tensor
    out += _s("blk.0.odd.weight") + struct.pack("<IIQ", 0, 16, 0)  # 0 dims, type 16, offset 0
    p = tmp_path / "b.gguf"
    p.write_bytes(bytes(out))
    with pytest.raises(CudaBackendError, match="Unsupported GGML type"):
        gguf_config(str(p))
    with pytest.raises(ValueError, match="Unsupported GGML type"):
        O.Model(str(p))


def test_duplicate_tensor_name_last_loaded_wins(tmp_path):
    """LoadedModel.LoadTensors stores `tensors[info.Name] = ...` (case-insensitive keys), so a
    repeated tensor name resolves to the last one: the oracle's logits with an output_norm repeated
    (different values, other case) equal those of the model whose only output_norm has the new values."""
    import numpy as np

    from dotllm_b200 import gguf, synth
    cfg = synth.get("micro")
    plan = synth.tensor_plan(cfg)
    data = {t.name: synth.tensor_bytes(cfg, t, r, i) for i, (t, r) in enumerate(plan)}
    md = synth.metadata_for(cfg)
    new_norm = (1.0 + 0.2 * np.random.default_rng(5).standard_normal(cfg.hidden)).astype("<f4").tobytes()
    single = str(tmp_path / "single.gguf")
    gguf.write_gguf(single, md, [t for t, _ in plan],
                    lambda t: new_norm if t.name == "output_norm.weight" else data[t.name])
    dup_infos = [t for t, _ in plan] + [gguf.TensorInfo("OUTPUT_NORM.weight", [cfg.hidden], gguf.GGML_F32)]
    dup = str(tmp_path / "dup.gguf")
    gguf.write_gguf(dup, synth.metadata_for(cfg), dup_infos,
                    lambda t: new_norm if t.name == "OUTPUT_NORM.weight" else data[t.name])
    outs = []
    for p in (single, dup):
        m = O.Model(p)
        s = O.Session(m)
        outs.append(s.process_token(3, 0))
        s.close()
        m.close()
    assert np.array_equal(outs[0], outs[1])


def test_parsers_agree_on_mutated_files(tmp_path):
    """Seeded byte flips, truncations and insertions of valid files (metadata-only and a real model's head): the library's GGUF parser
    (which runs inside the caller's process) and the oracle's must neither crash nor disagree --
    both refuse the file, or both resolve it to the same configuration."""
    import random
    rng = random.Random(1)
    from dotllm_b200 import synth
    bases = [open(write_meta_gguf(tmp_path / f"b{i}.gguf", e, names), "rb").read() for i, (e, names) in enumerate(
        [(LLAMA, ["token_embd.weight", "blk.0.ffn_gate.weight"]), (GEMMA, []), (PHI2, ["output.weight"]),
         (LFM2, ["blk.1.attn_q.weight", "blk.0.shortconv.conv.weight"])])]
    # and the head of a real synthetic model: its tensor infos and the start of its data
    bases.append(open(synth.build_model(synth.get("micro-lfm2")), "rb").read()[:200000])
    p = str(tmp_path / "f.gguf")
    resolved = 0
    for it in range(2500):
        b = bytearray(rng.choice(bases))
        for _ in range(rng.randint(1, 4)):
            op = rng.random()
            if op < 0.5:
                i = rng.randrange(len(b))
                b[i] = rng.randrange(256)
            elif op < 0.75:
                b = b[:rng.randrange(len(b))]
            else:
                i = rng.randrange(len(b))
                b[i:i] = bytes(rng.randrange(256) for _ in range(rng.randint(1, 8)))
            if not b:
                b = bytearray(b"G")
        with open(p, "wb") as f:
            f.write(bytes(b))
        try:
            c = gguf_config(p)
        except CudaBackendError:
            c = None
        try:
            m = O.Model(p)
            o = m.config
            m.close()
        except ValueError:
            o = None
        assert (c is None) == (o is None), it
        if c is not None:
            resolved += 1
            for k, v in o.items():
                assert c[k] == v or (c[k] != c[k] and v != v), (it, k)
    assert resolved > 50  # the mutations leave enough files valid to compare configurations
