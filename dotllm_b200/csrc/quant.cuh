// quant.cuh -- bit-exact element decoders for every GGUF type the reference reads.
//
// deq1(type, blk, i) returns element i of the block at `blk` (for F32/F16/BF16 the
// "block" is a single element and i must be 0).  Each formula restates the
// reference decoder with the same operation order, using explicitly rounded
// float ops so that nvcc cannot contract them into FMAs:
//   Q2_K DequantizeK.cs:8-41     Q3_K DequantizeK.cs:43-74   Q4_K DequantizeK.cs:76-106
//   Q5_K DequantizeK.cs:108-140  Q6_K DequantizeK.cs:142-187 Q4_0/Q8_0/F16/BF16/F32
//   DequantizeBlock.cs:7-104     Q4_1/Q5_0/Q5_1 TensorOps.cs:580-652
#pragma once
#include "common.cuh"

namespace llmdot {

__device__ __forceinline__ uint32_t ld_u32_unaligned(const uint8_t *p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

__device__ __forceinline__ float deq1(uint32_t type, const uint8_t *o, int i)
{
    switch (type) {
    case T_F32:
        return __uint_as_float(ld_u32_unaligned(o));
    case T_F16:
        return ld_half(o);
    case T_BF16:
        return __uint_as_float(((uint32_t)o[1] << 24) | ((uint32_t)o[0] << 16));
    case T_Q4_0: {
        float s = ld_half(o);
        int q = i < 16 ? (o[2 + i] & 0x0F) : ((o[2 + i - 16] >> 4) & 0x0F);
        return __fmul_rn((float)(q - 8), s);
    }
    case T_Q8_0:
        return __fmul_rn((float)(int8_t)o[2 + i], ld_half(o));
    case T_Q4_1: {
        float d = ld_half(o), m = ld_half(o + 2);
        int q = i < 16 ? (o[4 + i] & 0x0F) : ((o[4 + i - 16] >> 4) & 0x0F);
        return __fadd_rn(__fmul_rn(d, (float)q), m);
    }
    case T_Q5_0: {
        float d = ld_half(o);
        uint32_t qh = ld_u32_unaligned(o + 2);
        int j = i & 15, x;
        if (i < 16) x = ((o[6 + j] & 0x0F) | (int)(((qh >> j) << 4) & 0x10)) - 16;
        else x = (((o[6 + j] >> 4) & 0x0F) | (int)((qh >> (j + 12)) & 0x10)) - 16;
        return __fmul_rn((float)x, d);
    }
    case T_Q5_1: {
        float d = ld_half(o), m = ld_half(o + 2);
        uint32_t qh = ld_u32_unaligned(o + 4);
        int j = i & 15, x;
        if (i < 16) x = (o[8 + j] & 0x0F) | (int)(((qh >> j) << 4) & 0x10);
        else x = ((o[8 + j] >> 4) & 0x0F) | (int)((qh >> (j + 12)) & 0x10);
        return __fadd_rn(__fmul_rn(d, (float)x), m);
    }
    case T_Q2_K: {
        float d = ld_half(o), dmin = ld_half(o + 2);
        int g = i / 64, sub = (i % 64) / 16, scIdx = g * 4 + sub;
        int sc = o[4 + scIdx * 2] & 0x0F, mi = o[4 + scIdx * 2 + 1] & 0x0F;
        int q = (o[20 + i / 4] >> ((i % 4) * 2)) & 0x3;
        return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), __fsub_rn((float)q, 0.5f)), __fmul_rn(dmin, (float)mi));
    }
    case T_Q3_K: {
        float d = ld_half(o);
        int sc = extract6(o + 4, (i / 16) * 6);
        int q = (o[48 + i / 4] >> ((i % 4) * 2)) & 0x3;
        int m = (o[16 + i / 8] >> (i % 8)) & 0x1;
        return __fmul_rn(__fmul_rn(d, (float)sc), (float)(q - (m << 2)));
    }
    case T_Q4_K: {
        float d = ld_half(o), dmin = ld_half(o + 2);
        int g = i / 32;
        int sc = extract6(o + 4, g * 12), mi = extract6(o + 4, g * 12 + 6);
        int q = (o[16 + i / 2] >> ((i % 2) * 4)) & 0xF;
        return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)(q - 8)), __fmul_rn(dmin, (float)mi));
    }
    case T_Q5_K: {
        float d = ld_half(o), dmin = ld_half(o + 2);
        int g = i / 32;
        int sc = extract6(o + 4, g * 12), mi = extract6(o + 4, g * 12 + 6);
        int ql = (o[48 + i / 2] >> ((i % 2) * 4)) & 0xF;
        int qh = (o[16 + i / 8] >> (i % 8)) & 0x1;
        return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)(ql + (qh << 4) - 16)), __fmul_rn(dmin, (float)mi));
    }
    case T_Q6_K: {
        float d = ld_half(o + 208);
        int n = i / 128, r = i % 128, t = r / 32, l = r % 32;
        const uint8_t *ql = o + n * 64, *qh = o + 128 + n * 32, *scb = o + 192 + n * 8;
        int lo = (t & 1) ? ql[l + 32] : ql[l];
        lo = (t & 2) ? (lo >> 4) : (lo & 0xF);
        int hi = (qh[l] >> (2 * t)) & 3;
        int q = (lo | (hi << 4)) - 32;
        float sc = (float)(int8_t)scb[l / 16 + 2 * t];
        return __fmul_rn(__fmul_rn(d, sc), (float)q);
    }
    default:
        return 0.0f;
    }
}

}  // namespace llmdot
