"""Quantisers that encode for llmdot's own K-quant decode formulas.

llmdot ships decoders only (src/Llmdot.Core/Tensors/Dequantize/DequantizeK.cs,
DequantizeBlock.cs); its Q4_K/Q5_K layouts are not ggml's (linear 6-bit scale
packing, sequential nibbles), so a ggml quantiser would produce bytes that the
reference decodes differently.  These encoders target exactly the reference's
decoders:

* Q4_K (144 B / 256): f16 d @0, f16 dmin @2, 8 x (6-bit sc, 6-bit m) packed at
  bit g*12 / g*12+6 of bytes 4..15, nibble i at byte 16+i/2 (even i = low);
  x = d*sc*(q-8) - dmin*m                         (DequantizeK.cs:76-106)
* Q5_K (176 B / 256): scales as Q4_K, high bit i at byte 16+i/8 bit i%8, low
  nibble at byte 48+i/2; x = d*sc*(q5-16) - dmin*m (DequantizeK.cs:108-140)
* Q6_K (210 B / 256): ggml layout, ql[128] qh[64] int8 sc[16] f16 d
  (DequantizeK.cs:142-187); element e uses sc[e/16]
* Q8_0 (34 B / 32): f16 d, int8 q[32]              (DequantizeBlock.cs:35-59)
* Q4_0 (18 B / 32): f16 d, byte j = q[j] | q[j+16]<<4 (DequantizeBlock.cs:7-33)

All functions take float32 arrays whose last dimension is a multiple of the
block size and return uint8 arrays of shape [rows, row_bytes].  They are
vectorised over blocks; the encode choices (min/max fit, rounding) only need to
be reasonable, because parity is checked on the bytes they produce.
"""
from __future__ import annotations

import numpy as np

from .gguf import (BLOCK, GGML_BF16, GGML_F16, GGML_F32, GGML_Q4_0, GGML_Q4_K, GGML_Q5_K,
                   GGML_Q6_K, GGML_Q8_0)


def _f16(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float16)


def _pack_scales_k(sc: np.ndarray, m: np.ndarray) -> np.ndarray:
    """Pack 8 (sc, m) 6-bit pairs per block into 12 bytes: pair (2j, 2j+1) ->
    24-bit word sc0 | m0<<6 | sc1<<12 | m1<<18 at bytes 3j..3j+2.  Matches
    Extract6Bit(base, g*12) / (base, g*12+6) (DequantizeK.cs:189-199)."""
    sc = sc.astype(np.uint32)
    m = m.astype(np.uint32)
    w = sc[:, 0::2] | (m[:, 0::2] << 6) | (sc[:, 1::2] << 12) | (m[:, 1::2] << 18)  # [nb, 4]
    out = np.empty((sc.shape[0], 12), dtype=np.uint8)
    out[:, 0::3] = (w & 0xFF).astype(np.uint8)
    out[:, 1::3] = ((w >> 8) & 0xFF).astype(np.uint8)
    out[:, 2::3] = ((w >> 16) & 0xFF).astype(np.uint8)
    return out


def _fit_min_offset(sub: np.ndarray, qmax: int, zero: int):
    """Per sub-block (step, offset >= 0) so that step*(q-zero) - offset spans [min, max]."""
    mn = sub.min(axis=-1)
    mx = sub.max(axis=-1)
    step = (mx - mn) / qmax
    off = -mn - zero * step
    neg = off < 0
    alt = np.maximum(mx / max(qmax - zero, 1), -mn / zero)
    step = np.where(neg, alt, step)
    off = np.where(neg, 0.0, off)
    return step.astype(np.float32), off.astype(np.float32)


def _k_scales(step: np.ndarray, off: np.ndarray):
    d = step.max(axis=-1) / 63.0
    dmin = off.max(axis=-1) / 63.0
    d16 = _f16(d)
    dm16 = _f16(dmin)
    d32 = d16.astype(np.float32)
    dm32 = dm16.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d32[:, None] > 0, np.rint(step / d32[:, None]), 0)
        m = np.where(dm32[:, None] > 0, np.rint(off / dm32[:, None]), 0)
    sc = np.clip(sc, 0, 63).astype(np.int32)
    m = np.clip(m, 0, 63).astype(np.int32)
    return d16, dm16, d32, dm32, sc, m


def quantize_q4_k(x: np.ndarray) -> np.ndarray:
    rows = x.shape[0]
    blocks = x.reshape(-1, 256).astype(np.float32)
    nb = blocks.shape[0]
    sub = blocks.reshape(nb, 8, 32)
    step, off = _fit_min_offset(sub, 15, 8)
    d16, dm16, d32, dm32, sc, m = _k_scales(step, off)
    eff_step = (d32[:, None] * sc)[:, :, None]
    eff_off = (dm32[:, None] * m)[:, :, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(eff_step > 0, np.rint((sub + eff_off) / eff_step) + 8, 8)
    q = np.clip(q, 0, 15).astype(np.uint8).reshape(nb, 256)
    out = np.empty((nb, 144), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dm16.view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = _pack_scales_k(sc, m)
    out[:, 16:144] = q[:, 0::2] | (q[:, 1::2] << 4)
    return out.reshape(rows, -1)


def quantize_q5_k(x: np.ndarray) -> np.ndarray:
    rows = x.shape[0]
    blocks = x.reshape(-1, 256).astype(np.float32)
    nb = blocks.shape[0]
    sub = blocks.reshape(nb, 8, 32)
    step, off = _fit_min_offset(sub, 31, 16)
    d16, dm16, d32, dm32, sc, m = _k_scales(step, off)
    eff_step = (d32[:, None] * sc)[:, :, None]
    eff_off = (dm32[:, None] * m)[:, :, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(eff_step > 0, np.rint((sub + eff_off) / eff_step) + 16, 16)
    q = np.clip(q, 0, 31).astype(np.uint8).reshape(nb, 256)
    out = np.empty((nb, 176), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = dm16.view(np.uint8).reshape(nb, 2)
    out[:, 4:16] = _pack_scales_k(sc, m)
    out[:, 16:48] = np.packbits((q >> 4).astype(np.uint8), axis=1, bitorder="little")
    lo = q & 0xF
    out[:, 48:176] = lo[:, 0::2] | (lo[:, 1::2] << 4)
    return out.reshape(rows, -1)


def quantize_q6_k(x: np.ndarray) -> np.ndarray:
    rows = x.shape[0]
    blocks = x.reshape(-1, 256).astype(np.float32)
    nb = blocks.shape[0]
    sub = blocks.reshape(nb, 16, 16)
    sreal = np.abs(sub).max(axis=-1) / 31.0
    d = sreal.max(axis=-1) / 127.0
    d16 = _f16(d)
    d32 = d16.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d32[:, None] > 0, np.rint(sreal / d32[:, None]), 0)
    sc = np.clip(sc, -128, 127).astype(np.int32)
    eff = (d32[:, None] * sc)[:, :, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(eff != 0, np.rint(sub / eff), 0)
    q = (np.clip(q, -32, 31).astype(np.int32) + 32).astype(np.uint8).reshape(nb, 2, 4, 32)
    # q[:, h, t, l] is element h*128 + t*32 + l
    lo = q & 0xF
    hi = q >> 4
    ql = np.empty((nb, 2, 64), dtype=np.uint8)
    ql[:, :, 0:32] = lo[:, :, 0, :] | (lo[:, :, 2, :] << 4)
    ql[:, :, 32:64] = lo[:, :, 1, :] | (lo[:, :, 3, :] << 4)
    qh = hi[:, :, 0, :] | (hi[:, :, 1, :] << 2) | (hi[:, :, 2, :] << 4) | (hi[:, :, 3, :] << 6)
    out = np.empty((nb, 210), dtype=np.uint8)
    out[:, 0:128] = ql.reshape(nb, 128)
    out[:, 128:192] = qh.reshape(nb, 64)
    out[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    out[:, 208:210] = d16.view(np.uint8).reshape(nb, 2)
    return out.reshape(rows, -1)


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    rows = x.shape[0]
    blocks = x.reshape(-1, 32).astype(np.float32)
    nb = blocks.shape[0]
    d = np.abs(blocks).max(axis=-1) / 127.0
    d16 = _f16(d)
    d32 = d16.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(d32[:, None] > 0, np.rint(blocks / d32[:, None]), 0)
    q = np.clip(q, -127, 127).astype(np.int8)
    out = np.empty((nb, 34), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:34] = q.view(np.uint8)
    return out.reshape(rows, -1)


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    rows = x.shape[0]
    blocks = x.reshape(-1, 32).astype(np.float32)
    nb = blocks.shape[0]
    d = np.abs(blocks).max(axis=-1) / 8.0
    d16 = _f16(d)
    d32 = d16.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(d32[:, None] > 0, np.rint(blocks / d32[:, None]) + 8, 8)
    q = np.clip(q, 0, 15).astype(np.uint8)
    out = np.empty((nb, 18), dtype=np.uint8)
    out[:, 0:2] = d16.view(np.uint8).reshape(nb, 2)
    out[:, 2:18] = q[:, 0:16] | (q[:, 16:32] << 4)
    return out.reshape(rows, -1)


QUANTIZERS = {
    GGML_Q4_K: quantize_q4_k,
    GGML_Q5_K: quantize_q5_k,
    GGML_Q6_K: quantize_q6_k,
    GGML_Q8_0: quantize_q8_0,
    GGML_Q4_0: quantize_q4_0,
    GGML_F32: lambda x: np.ascontiguousarray(x, dtype="<f4").view(np.uint8).reshape(x.shape[0], -1),
    GGML_F16: lambda x: np.ascontiguousarray(x, dtype="<f2").view(np.uint8).reshape(x.shape[0], -1),
    GGML_BF16: lambda x: (np.ascontiguousarray(x, dtype="<f4").view("<u4") >> 16).astype("<u2").view(np.uint8).reshape(x.shape[0], -1),
}


def quantize(x: np.ndarray, ggml_type: int) -> np.ndarray:
    """Quantise a 2-D float array [rows, cols] row-major into [rows, row_bytes]."""
    x = np.asarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    be = BLOCK[ggml_type][0]
    if x.shape[1] % be:
        raise ValueError(f"row length {x.shape[1]} is not a multiple of the {be}-element block")
    return QUANTIZERS[ggml_type](x)
