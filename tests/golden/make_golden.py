"""Generate the committed golden fixtures in tests/golden/.

  kquant_kat.json   dequantisation known-answer vectors for every type the
                    reference decodes.  Expected values come from a second,
                    independent restatement of the reference decoders written
                    here in numpy (float32 arithmetic, same operation order as
                    src/Llmdot.Core/Tensors/Dequantize/DequantizeK.cs and
                    DequantizeBlock.cs), plus hand-worked blocks whose expected
                    values are derived in the comments below.
  greedy_tokens.json  greedy token ids and logit checksums produced by the CPU
                    oracle for the small synthetic models (regression pins for
                    the oracle itself).
  sampled_tokens.json  token ids of the oracle's Generate with Sampler.Sample on
                    the same models: seeded (one draw, new Random(42).NextSingle())
                    and with per-token draws listed in the file.
  template_tokens.json  greedy token ids and logit checksums of the oracle on the
                    LFM2 short-conv, MoE and GPT-NeoX-like synthetic models.

Run:  python tests/golden/make_golden.py              (every fixture)
      python tests/golden/make_golden.py sampled      (sampled_tokens.json only)
      python tests/golden/make_golden.py templates    (template_tokens.json only)
"""
from __future__ import annotations

import base64
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

F = np.float32

# ---------------------------------------------------------------------- independent decoders


def h2f(b0: int, b1: int) -> np.float32:
    return np.frombuffer(bytes([b0, b1]), dtype="<f2")[0].astype(F)


def ex6(blk: bytes, base: int, bit: int) -> int:
    bi, sh = bit // 8, bit % 8
    if sh <= 2:
        return (blk[base + bi] >> sh) & 0x3F
    return ((blk[base + bi] >> sh) | (blk[base + bi + 1] << (8 - sh))) & 0x3F


def dec_block(t: int, data: bytes, off: int) -> np.ndarray:
    """Decode the block at data[off:]; Q3_K reads up to byte off+111, one past its 110-byte
    block, exactly as DequantizeK.cs:65 does (the caller supplies that slack)."""
    bb = BLOCK[t][1]
    blk = data[off:off + (112 if t == 11 else bb)]
    out = []
    if t == 12:  # Q4_K: d*sc*(q-8) - dmin*m
        d, dmin = h2f(blk[0], blk[1]), h2f(blk[2], blk[3])
        for i in range(256):
            g = i // 32
            sc, m = ex6(blk, 4, g * 12), ex6(blk, 4, g * 12 + 6)
            q = (blk[16 + i // 2] >> ((i % 2) * 4)) & 0xF
            out.append(F(F(d * F(sc)) * F(q - 8)) - F(dmin * F(m)))
    elif t == 13:  # Q5_K
        d, dmin = h2f(blk[0], blk[1]), h2f(blk[2], blk[3])
        for i in range(256):
            g = i // 32
            sc, m = ex6(blk, 4, g * 12), ex6(blk, 4, g * 12 + 6)
            ql = (blk[48 + i // 2] >> ((i % 2) * 4)) & 0xF
            qh = (blk[16 + i // 8] >> (i % 8)) & 1
            out.append(F(F(d * F(sc)) * F(ql + (qh << 4) - 16)) - F(dmin * F(m)))
    elif t == 14:  # Q6_K
        d = h2f(blk[208], blk[209])
        vals = [None] * 256
        for n in (0, 128):
            ql, qh, sc = n // 2, 128 + n // 4, 192 + n // 16
            for l in range(32):
                s = l // 16
                q1 = ((blk[ql + l] & 0xF) | ((blk[qh + l] & 3) << 4)) - 32
                q2 = ((blk[ql + l + 32] & 0xF) | (((blk[qh + l] >> 2) & 3) << 4)) - 32
                q3 = ((blk[ql + l] >> 4) | (((blk[qh + l] >> 4) & 3) << 4)) - 32
                q4 = ((blk[ql + l + 32] >> 4) | (((blk[qh + l] >> 6) & 3) << 4)) - 32
                scs = [np.int8(np.uint8(blk[sc + s + k])) for k in (0, 2, 4, 6)]
                for off, q, scv in zip((0, 32, 64, 96), (q1, q2, q3, q4), scs):
                    vals[n + l + off] = F(F(d * F(scv)) * F(q))
        out = vals
    elif t == 10:  # Q2_K: d*sc*(q-0.5) - dmin*m
        d, dmin = h2f(blk[0], blk[1]), h2f(blk[2], blk[3])
        for i in range(256):
            idx = (i // 64) * 4 + (i % 64) // 16
            sc, m = blk[4 + idx * 2] & 0xF, blk[4 + idx * 2 + 1] & 0xF
            q = (blk[20 + i // 4] >> ((i % 4) * 2)) & 3
            out.append(F(F(d * F(sc)) * F(F(q) - F(0.5))) - F(dmin * F(m)))
    elif t == 11:  # Q3_K: d*sc*(q - 4m)
        d = h2f(blk[0], blk[1])
        for i in range(256):
            sc = ex6(blk, 4, (i // 16) * 6)
            q = (blk[48 + i // 4] >> ((i % 4) * 2)) & 3
            m = (blk[16 + i // 8] >> (i % 8)) & 1
            out.append(F(F(d * F(sc)) * F(q - (m << 2))))
    elif t == 8:  # Q8_0
        d = h2f(blk[0], blk[1])
        out = [F(F(np.int8(np.uint8(blk[2 + i]))) * d) for i in range(32)]
    elif t == 2:  # Q4_0
        d = h2f(blk[0], blk[1])
        out = [F(F((blk[2 + (i % 16)] >> (4 * (i // 16)) & 0xF) - 8) * d) for i in range(32)]
    elif t == 3:  # Q4_1
        d, m = h2f(blk[0], blk[1]), h2f(blk[2], blk[3])
        out = [F(F(d * F((blk[4 + (i % 16)] >> (4 * (i // 16))) & 0xF)) + m) for i in range(32)]
    elif t == 6:  # Q5_0
        d = h2f(blk[0], blk[1])
        qh = int.from_bytes(blk[2:6], "little")
        for i in range(32):
            j = i % 16
            if i < 16:
                x = ((blk[6 + j] & 0xF) | (((qh >> j) << 4) & 0x10)) - 16
            else:
                x = (((blk[6 + j] >> 4) & 0xF) | ((qh >> (j + 12)) & 0x10)) - 16
            out.append(F(F(x) * d))
    elif t == 7:  # Q5_1
        d, m = h2f(blk[0], blk[1]), h2f(blk[2], blk[3])
        qh = int.from_bytes(blk[4:8], "little")
        for i in range(32):
            j = i % 16
            if i < 16:
                x = (blk[8 + j] & 0xF) | (((qh >> j) << 4) & 0x10)
            else:
                x = ((blk[8 + j] >> 4) & 0xF) | ((qh >> (j + 12)) & 0x10)
            out.append(F(F(d * F(x)) + m))
    elif t == 1:  # F16
        out = [h2f(blk[0], blk[1])]
    elif t == 25:  # BF16
        out = [np.frombuffer(bytes([0, 0, blk[0], blk[1]]), dtype="<f4")[0]]
    elif t == 0:
        out = [np.frombuffer(blk[:4], dtype="<f4")[0]]
    return np.array(out, dtype=F)


BLOCK = {0: (1, 4), 1: (1, 2), 25: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34),
         10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210)}


def decode(t: int, data: bytes, rows: int, row_elems: int) -> np.ndarray:
    be, bb = BLOCK[t]
    res = []
    for r in range(rows):
        for b in range(row_elems // be):
            off = (r * (row_elems // be) + b) * bb
            res.append(dec_block(t, data, off))
    return np.concatenate(res)


# ---------------------------------------------------------------------- hand-worked blocks

def hand_q4k() -> bytes:
    """d = 1.0 (0x3C00), dmin = 0.5 (0x3800); sub-block g has sc = g+1, m = 2g; nibble i = i % 16.
    Element i (g = i//32, q = i%16): x = (g+1)*(q-8) - g.  E.g. x[0] = -8, x[33] = 2*(1-8) - 1 = -15,
    x[255] = 8*(15-8) - 7 = 49."""
    b = bytearray(144)
    b[0:2] = bytes([0x00, 0x3C])
    b[2:4] = bytes([0x00, 0x38])
    for j in range(4):
        sc0, m0, sc1, m1 = 2 * j + 1, 4 * j, 2 * j + 2, 4 * j + 2
        w = sc0 | (m0 << 6) | (sc1 << 12) | (m1 << 18)
        b[4 + 3 * j:7 + 3 * j] = w.to_bytes(3, "little")
    for i in range(0, 256, 2):
        b[16 + i // 2] = (i % 16) | (((i + 1) % 16) << 4)
    return bytes(b)


def hand_q4k_expected() -> np.ndarray:
    return np.array([(i // 32 + 1) * (i % 16 - 8) - (i // 32) for i in range(256)], dtype=F)


def hand_q6k() -> bytes:
    """d = 0.5 (0x3800), sc[s] = s - 8 (int8), every 6-bit q = 33 (value 1).  Element e uses sc[e//16]:
    x[e] = 0.5 * (e//16 - 8) * 1, e.g. x[0] = -4, x[255] = 3.5."""
    b = bytearray(210)
    q = 33  # low nibble 1, high bits 2
    for n in range(2):
        for l in range(64):
            b[n * 64 + l] = (q & 0xF) | ((q & 0xF) << 4)
        for l in range(32):
            h = (q >> 4) & 3
            b[128 + n * 32 + l] = h | (h << 2) | (h << 4) | (h << 6)
    for s in range(16):
        b[192 + s] = (s - 8) & 0xFF
    b[208:210] = bytes([0x00, 0x38])
    return bytes(b)


def hand_q6k_expected() -> np.ndarray:
    return np.array([0.5 * (e // 16 - 8) for e in range(256)], dtype=F)


def hand_q5k() -> bytes:
    """d = 2.0 (0x4000), dmin = 1.0; sc = 1, m = 1 for every sub-block; q5 = i % 32 (high bit set
    for i%32 >= 16).  x[i] = 2*(i%32 - 16) - 1, e.g. x[0] = -33, x[31] = 29."""
    b = bytearray(176)
    b[0:2] = bytes([0x00, 0x40])
    b[2:4] = bytes([0x00, 0x3C])
    for j in range(4):
        w = 1 | (1 << 6) | (1 << 12) | (1 << 18)
        b[4 + 3 * j:7 + 3 * j] = w.to_bytes(3, "little")
    for i in range(256):
        q = i % 32
        if q >> 4:
            b[16 + i // 8] |= 1 << (i % 8)
        b[48 + i // 2] |= (q & 0xF) << ((i % 2) * 4)
    return bytes(b)


def hand_q5k_expected() -> np.ndarray:
    return np.array([2 * (i % 32 - 16) - 1 for i in range(256)], dtype=F)


def b64(x: bytes) -> str:
    return base64.b64encode(x).decode()


def make_kquant() -> dict:
    rng = np.random.default_rng(20261201)
    cases = []
    # the reference's own unit-test blocks (tests/Llmdot.Core.Tests/Tensors/DequantizeTests.cs:25-61)
    q40 = bytearray(36)
    q40[0:2] = bytes([0x00, 0x3C])
    q40[18:20] = bytes([0x00, 0x3C])
    cases.append(dict(name="ref_q4_0_all_minus8", type=2, rows=1, row_elems=64, data=bytes(q40),
                      expected=np.full(64, -8.0, dtype=F)))
    q80 = bytearray(68)
    q80[0:2] = bytes([0x00, 0x3C])
    q80[34:36] = bytes([0x00, 0x3C])
    cases.append(dict(name="ref_q8_0_zeros", type=8, rows=1, row_elems=64, data=bytes(q80),
                      expected=np.zeros(64, dtype=F)))
    cases.append(dict(name="ref_f16_values", type=1, rows=1, row_elems=4,
                      data=bytes([0x00, 0x3C, 0x00, 0xBC, 0x00, 0x38, 0x00, 0x00]),
                      expected=np.array([1.0, -1.0, 0.5, 0.0], dtype=F)))
    cases.append(dict(name="ref_bf16_values", type=25, rows=1, row_elems=3,
                      data=bytes([0x80, 0x3F, 0x00, 0x40, 0x80, 0xBF]), expected=np.array([1.0, 2.0, -1.0], dtype=F)))
    # hand-worked K-quant blocks
    cases.append(dict(name="hand_q4_k", type=12, rows=1, row_elems=256, data=hand_q4k(), expected=hand_q4k_expected()))
    cases.append(dict(name="hand_q5_k", type=13, rows=1, row_elems=256, data=hand_q5k(), expected=hand_q5k_expected()))
    cases.append(dict(name="hand_q6_k", type=14, rows=1, row_elems=256, data=hand_q6k(), expected=hand_q6k_expected()))
    # random blocks for every type; f16 scales drawn from a wide range incl. subnormals
    for t, rows, elems in [(12, 3, 512), (13, 2, 512), (14, 3, 512), (10, 2, 512), (11, 2, 512), (8, 2, 128),
                           (2, 2, 128), (3, 2, 64), (6, 2, 64), (7, 2, 64), (1, 1, 64), (25, 1, 64)]:
        be, bb = BLOCK[t]
        n = rows * (elems // be) * bb + (2 if t == 11 else 0)  # Q3_K: 2 bytes of slack, see dec_block
        data = bytearray(rng.integers(0, 256, size=n, dtype=np.uint8).tobytes())
        # keep scale fields finite: replace f16 fields with values from [-2^3, 2^3] incl. subnormals
        scales = {12: (0, 2), 13: (0, 2), 10: (0, 2), 11: (0,), 14: (208,), 8: (0,), 2: (0,), 3: (0, 2), 6: (0,),
                  7: (0, 2)}.get(t, ())
        for bi in range(rows * (elems // be)):
            for off in scales:
                exp = rng.integers(-20, 4)
                v = np.float16(rng.uniform(0.5, 1.0) * (2.0 ** exp) * rng.choice([-1, 1]))
                data[bi * bb + off:bi * bb + off + 2] = v.tobytes()
        if t in (1,):
            vals = (rng.standard_normal(elems) * 4).astype(np.float16)
            vals[:3] = [np.float16(6e-8), np.float16(-0.0), np.float16(65504)]
            data = bytearray(vals.tobytes())
        data = bytes(data)
        cases.append(dict(name=f"rand_type{t}", type=t, rows=rows, row_elems=elems, data=data,
                          expected=decode(t, data, rows, elems)))
    out = []
    for c in cases:
        out.append(dict(name=c["name"], type=c["type"], rows=c["rows"], row_elems=c["row_elems"],
                        data=b64(c["data"]), expected_f32=b64(np.asarray(c["expected"], dtype="<f4").tobytes())))
    return {"generator": "tests/golden/make_golden.py", "cases": out}


def make_greedy() -> dict:
    from dotllm_b200 import synth
    from oracle import oracle as O
    O.set_threads(max(1, O.max_threads()))
    res = {}
    for name, steps in [("micro", 16), ("micro-gemma", 16), ("micro-phi3", 16), ("micro-q5q8", 16), ("tiny", 64)]:
        cfg = synth.get(name)
        m = O.Model(synth.build_model(cfg))
        s = O.Session(m)
        prompt = synth.prompt_tokens(cfg)
        toks, lg = s.generate(prompt, steps, want_logits=True)
        srt = np.sort(lg, axis=1)
        res[name] = dict(prompt_len=int(prompt.size), steps=steps, tokens=[int(t) for t in toks],
                         logit_sum=[float(x) for x in lg.astype(np.float64).sum(axis=1)],
                         top2_margin=[float(x) for x in (srt[:, -1] - srt[:, -2])])
        s.close()
        m.close()
    return res


def make_templates() -> dict:
    from dotllm_b200 import synth
    from oracle import oracle as O
    O.set_threads(max(1, O.max_threads()))
    res = {}
    for name in ("micro-lfm2", "micro-moe", "micro-lfm2moe", "micro-neox"):
        cfg = synth.get(name)
        m = O.Model(synth.build_model(cfg))
        s = O.Session(m)
        toks, lg = s.generate(synth.prompt_tokens(cfg), 16, want_logits=True)
        res[name] = dict(steps=16, tokens=[int(t) for t in toks],
                         logit_sum=[float(x) for x in lg.astype(np.float64).sum(axis=1)])
        s.close()
        m.close()
    return res


SAMPLED_OPTIONS = dict(top_k=40, top_p=0.95, temperature=0.8, repeat_penalty=1.1, repeat_window=16)


def make_sampled() -> dict:
    from dotllm_b200 import synth
    from oracle import oracle as O
    O.set_threads(max(1, O.max_threads()))
    res = {"options": SAMPLED_OPTIONS}
    for name, steps in [("micro", 16), ("micro-gemma", 16), ("tiny", 32)]:
        cfg = synth.get(name)
        m = O.Model(synth.build_model(cfg))
        s = O.Session(m)
        prompt = synth.prompt_tokens(cfg)
        seeded = s.generate_sampled(prompt, steps, O.SamplingOptions(seed=42, **SAMPLED_OPTIONS))
        draws = np.random.default_rng(2024).uniform(0.0, 1.0, size=steps).astype(np.float32)
        drawn = s.generate_sampled(prompt, steps, O.SamplingOptions(**SAMPLED_OPTIONS), draws)
        res[name] = dict(steps=steps, seed=42, seeded_tokens=[int(t) for t in seeded],
                         draws=[float(x) for x in draws], drawn_tokens=[int(t) for t in drawn])
        s.close()
        m.close()
    return res


if __name__ == "__main__":
    only = sys.argv[1] if len(sys.argv) > 1 else None
    if only is None:
        with open(os.path.join(HERE, "kquant_kat.json"), "w") as f:
            json.dump(make_kquant(), f, indent=1)
        with open(os.path.join(HERE, "greedy_tokens.json"), "w") as f:
            json.dump(make_greedy(), f, indent=1)
    if only in (None, "sampled"):
        with open(os.path.join(HERE, "sampled_tokens.json"), "w") as f:
            json.dump(make_sampled(), f, indent=1)
    if only in (None, "templates"):
        with open(os.path.join(HERE, "template_tokens.json"), "w") as f:
            json.dump(make_templates(), f, indent=1)
    print("wrote", os.listdir(HERE))
