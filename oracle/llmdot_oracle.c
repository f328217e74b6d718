/*
 * llmdot_oracle.c -- TEST INFRASTRUCTURE ONLY. Never linked into, imported by or
 * called from the product library; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference arm of bench.py load it, and only as the checker or
 * as the timed CPU baseline.
 *
 * A plain-C restatement of llmdot's managed CPU decode path (cognisoc/dotllm,
 * C#): GGUF loading, config resolution, K-quant dequantisation, the fused
 * dequant-matvecs, VectorMath (incl. its exp/tanh approximations and 8-lane
 * partial sums), RoPE, inline GQA attention, the Llama/Gemma/NeoX layer
 * templates and the greedy Generate loop.  Every function names the reference
 * file:line it follows (paths relative to the reference project root).
 *
 * Numerics contract (why the build flags matter):
 *   - compile with -O2 -ffp-contract=off -fno-fast-math: .NET RyuJIT does not
 *     contract a*b+c into FMA and does not reassociate, so neither may we;
 *   - System.Numerics.Vector<float> is 8 lanes wide on AVX2 hosts: every
 *     "vector lane" loop below keeps 8 independent partial sums and the scalar
 *     tail runs after the vector loop, exactly like the C#;
 *   - Vector.Dot(acc, One) is restated as the pairwise tree
 *     ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)) (x86 dpps per 128-bit half, then the
 *     two halves added) -- the reference cannot run here, so this horizontal
 *     order is an assumption; it only moves the last ulp of a reduction;
 *   - MathF.Exp/Cos/Sin/Pow/Tanh/Sqrt call the C runtime, so expf/cosf/sinf/
 *     powf/tanhf/sqrtf from glibc are the faithful counterparts;
 *   - Vector.ConvertToInt32 truncates toward zero (cvttps2dq): a C (int) cast.
 *
 * OpenMP is used only across independent output rows / heads; the per-row
 * accumulation order never changes, so results are identical for any thread
 * count.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <strings.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define VEC 8 /* Vector<float>.Count on AVX2 */

#define EXPORT __attribute__((visibility("default")))

/* GgmlType values, src/Llmdot.Core/Loading/GgmlType.cs:3-27 */
enum {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8,
    T_Q8_1 = 9, T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_BF16 = 25
};

static float bits_f(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t f_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* .NET float.NaN bit pattern (0xFFC00000) */
static float net_nan(void) { return bits_f(0xFFC00000u); }

/* ------------------------------------------------------------------------ */
/* HalfHelper.HalfToFloat -- src/Llmdot.Core/Tensors/Numeric/HalfHelper.cs:7-40 */
EXPORT float orc_half_to_float(uint32_t half)
{
    uint32_t sign = (half >> 15) & 1u, exponent = (half >> 10) & 0x1Fu, mant = half & 0x3FFu;
    if (exponent == 0) {
        if (mant == 0) return sign ? -0.0f : 0.0f;
        uint32_t norm = mant;
        int shift = 0;
        while ((norm & 0x400u) == 0) { norm <<= 1; shift++; }
        uint32_t newExp = (uint32_t)(127 - 14 - shift);
        uint32_t b = (sign << 31) | (newExp << 23) | ((norm & 0x3FFu) << 13);
        return bits_f(b);
    }
    if (exponent == 31)
        return mant == 0 ? (sign ? -INFINITY : INFINITY) : net_nan();
    uint32_t b = (sign << 31) | ((exponent - 15 + 127) << 23) | (mant << 13);
    return bits_f(b);
}
static float rd_half(const uint8_t *p) { return orc_half_to_float((uint32_t)p[0] | ((uint32_t)p[1] << 8)); }

/* DequantizeK.Extract6Bit -- src/Llmdot.Core/Tensors/Dequantize/DequantizeK.cs:189-199 */
static int extract6(const uint8_t *base, int bitOffset)
{
    int byteIdx = bitOffset / 8, bitShift = bitOffset % 8;
    if (bitShift <= 2) return (base[byteIdx] >> bitShift) & 0x3F;
    return ((base[byteIdx] >> bitShift) | (base[byteIdx + 1] << (8 - bitShift))) & 0x3F;
}

/* TensorSize.ByteCount -- src/Llmdot.Core/Tensors/TensorSize.cs:7-24 (returns 0 if unsupported) */
EXPORT uint64_t orc_byte_count(uint32_t type, uint64_t n)
{
    switch (type) {
    case T_F32: return n * 4;
    case T_F16: case T_BF16: return n * 2;
    case T_Q4_0: return n / 32 * 18;
    case T_Q4_1: return n / 32 * 20;
    case T_Q5_0: return n / 32 * 22;
    case T_Q5_1: return n / 32 * 24;
    case T_Q8_0: return n / 32 * 34;
    case T_Q8_1: return n / 32 * 40;
    case T_Q2_K: return n / 256 * 84;
    case T_Q3_K: return n / 256 * 110;
    case T_Q4_K: return n / 256 * 144;
    case T_Q5_K: return n / 256 * 176;
    case T_Q6_K: return n / 256 * 210;
    default: return 0;
    }
}

/* ------------------------------------------------------------------------ */
/* Dequantisation: DequantizeK.cs:8-187, DequantizeBlock.cs:7-104, TensorOps.cs:580-652 */

static void deq_q2k(const uint8_t *src, float *dst, int numRows, int rowElements)
{   /* DequantizeK.cs:8-41 */
    int bpr = rowElements / 256;
    for (int r = 0; r < numRows; r++)
        for (int b = 0; b < bpr; b++) {
            const uint8_t *o = src + ((size_t)r * bpr + b) * 84;
            float d = rd_half(o), dmin = rd_half(o + 2);
            for (int i = 0; i < 256; i++) {
                int g = i / 64, local = i % 64, sub = local / 16, scIdx = g * 4 + sub;
                int sc = o[4 + scIdx * 2] & 0x0F, mi = o[4 + scIdx * 2 + 1] & 0x0F;
                int q = (o[20 + i / 4] >> ((i % 4) * 2)) & 0x3;
                dst[(size_t)r * rowElements + b * 256 + i] = d * (float)sc * ((float)q - 0.5f) - dmin * (float)mi;
            }
        }
}

static void deq_q3k(const uint8_t *src, float *dst, int numRows, int rowElements)
{   /* DequantizeK.cs:43-74 */
    int bpr = rowElements / 256;
    for (int r = 0; r < numRows; r++)
        for (int b = 0; b < bpr; b++) {
            const uint8_t *o = src + ((size_t)r * bpr + b) * 110;
            float d = rd_half(o);
            for (int i = 0; i < 256; i++) {
                int g = i / 16;
                int sc = extract6(o + 4, g * 6);
                int q = (o[48 + i / 4] >> ((i % 4) * 2)) & 0x3;
                int m = (o[16 + i / 8] >> (i % 8)) & 0x1;
                int value = q - (m << 2);
                dst[(size_t)r * rowElements + b * 256 + i] = d * (float)sc * (float)value;
            }
        }
}

static void deq_q4k(const uint8_t *src, float *dst, int numRows, int rowElements)
{   /* DequantizeK.cs:76-106 */
    int bpr = rowElements / 256;
    for (int r = 0; r < numRows; r++)
        for (int b = 0; b < bpr; b++) {
            const uint8_t *o = src + ((size_t)r * bpr + b) * 144;
            float d = rd_half(o), dmin = rd_half(o + 2);
            for (int i = 0; i < 256; i++) {
                int g = i / 32;
                int sc = extract6(o + 4, g * 12), mi = extract6(o + 4, g * 12 + 6);
                int q = (o[16 + i / 2] >> ((i % 2) * 4)) & 0xF;
                dst[(size_t)r * rowElements + b * 256 + i] = d * (float)sc * (float)(q - 8) - dmin * (float)mi;
            }
        }
}

static void deq_q5k(const uint8_t *src, float *dst, int numRows, int rowElements)
{   /* DequantizeK.cs:108-140 */
    int bpr = rowElements / 256;
    for (int r = 0; r < numRows; r++)
        for (int b = 0; b < bpr; b++) {
            const uint8_t *o = src + ((size_t)r * bpr + b) * 176;
            float d = rd_half(o), dmin = rd_half(o + 2);
            for (int i = 0; i < 256; i++) {
                int g = i / 32;
                int sc = extract6(o + 4, g * 12), mi = extract6(o + 4, g * 12 + 6);
                int qLow = (o[48 + i / 2] >> ((i % 2) * 4)) & 0xF;
                int qHigh = (o[16 + i / 8] >> (i % 8)) & 0x1;
                int q5 = qLow + (qHigh << 4);
                dst[(size_t)r * rowElements + b * 256 + i] = d * (float)sc * (float)(q5 - 16) - dmin * (float)mi;
            }
        }
}

static void deq_q6k(const uint8_t *src, float *dst, int numRows, int rowElements)
{   /* DequantizeK.cs:142-187 */
    int bpr = rowElements / 256;
    for (int r = 0; r < numRows; r++)
        for (int b = 0; b < bpr; b++) {
            const uint8_t *o = src + ((size_t)r * bpr + b) * 210;
            float d = rd_half(o + 208);
            for (int n = 0; n < 256; n += 128) {
                const uint8_t *ql = o + n / 2, *qh = o + 128 + n / 4, *scb = o + 192 + n / 16;
                for (int l = 0; l < 32; l++) {
                    int is = l / 16;
                    int q1 = ((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                    int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    float sc0 = (float)(int8_t)scb[is + 0], sc2 = (float)(int8_t)scb[is + 2];
                    float sc4 = (float)(int8_t)scb[is + 4], sc6 = (float)(int8_t)scb[is + 6];
                    float *dd = dst + (size_t)r * rowElements + b * 256 + n;
                    dd[l] = d * sc0 * (float)q1;
                    dd[l + 32] = d * sc2 * (float)q2;
                    dd[l + 64] = d * sc4 * (float)q3;
                    dd[l + 96] = d * sc6 * (float)q4;
                }
            }
        }
}

static void deq_q4_0(const uint8_t *src, float *dst, int numRows, int rowElements)
{   /* DequantizeBlock.cs:7-33 */
    int bpr = rowElements / 32;
    for (int r = 0; r < numRows; r++)
        for (int b = 0; b < bpr; b++) {
            const uint8_t *o = src + ((size_t)r * bpr + b) * 18;
            float scale = rd_half(o);
            for (int j = 0; j < 16; j++) {
                int qs = o[2 + j];
                dst[(size_t)r * rowElements + b * 32 + j] = (float)((qs & 0x0F) - 8) * scale;
                dst[(size_t)r * rowElements + b * 32 + j + 16] = (float)(((qs >> 4) & 0x0F) - 8) * scale;
            }
        }
}

static void deq_q8_0(const uint8_t *src, float *dst, int numRows, int rowElements)
{   /* DequantizeBlock.cs:35-59 */
    int bpr = rowElements / 32;
    for (int r = 0; r < numRows; r++)
        for (int b = 0; b < bpr; b++) {
            const uint8_t *o = src + ((size_t)r * bpr + b) * 34;
            float scale = rd_half(o);
            for (int i = 0; i < 32; i++)
                dst[(size_t)r * rowElements + b * 32 + i] = (float)(int8_t)o[2 + i] * scale;
        }
}

static void deq_q4_1(const uint8_t *src, float *dst, int numRows, int rowElements)
{   /* TensorOps.cs:584-603 */
    int bpr = rowElements / 32;
    for (int r = 0; r < numRows; r++)
        for (int b = 0; b < bpr; b++) {
            const uint8_t *o = src + ((size_t)r * bpr + b) * 20;
            float d = rd_half(o), m = rd_half(o + 2);
            for (int j = 0; j < 16; j++) {
                int qs = o[4 + j];
                dst[(size_t)r * rowElements + b * 32 + j] = d * (float)(qs & 0x0F) + m;
                dst[(size_t)r * rowElements + b * 32 + j + 16] = d * (float)((qs >> 4) & 0x0F) + m;
            }
        }
}

static uint32_t rd_u32(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); }

static void deq_q5_0(const uint8_t *src, float *dst, int numRows, int rowElements)
{   /* TensorOps.cs:604-625 */
    int bpr = rowElements / 32;
    for (int r = 0; r < numRows; r++)
        for (int b = 0; b < bpr; b++) {
            const uint8_t *o = src + ((size_t)r * bpr + b) * 22;
            float d = rd_half(o);
            uint32_t qh = rd_u32(o + 2);
            for (int j = 0; j < 16; j++) {
                int qs = o[6 + j];
                int x0 = ((qs & 0x0F) | (int)(((qh >> (j + 0)) << 4) & 0x10)) - 16;
                int x1 = (((qs >> 4) & 0x0F) | (int)((qh >> (j + 12)) & 0x10)) - 16;
                dst[(size_t)r * rowElements + b * 32 + j] = (float)x0 * d;
                dst[(size_t)r * rowElements + b * 32 + j + 16] = (float)x1 * d;
            }
        }
}

static void deq_q5_1(const uint8_t *src, float *dst, int numRows, int rowElements)
{   /* TensorOps.cs:626-648 */
    int bpr = rowElements / 32;
    for (int r = 0; r < numRows; r++)
        for (int b = 0; b < bpr; b++) {
            const uint8_t *o = src + ((size_t)r * bpr + b) * 24;
            float d = rd_half(o), m = rd_half(o + 2);
            uint32_t qh = rd_u32(o + 4);
            for (int j = 0; j < 16; j++) {
                int qs = o[8 + j];
                int x0 = (qs & 0x0F) | (int)(((qh >> (j + 0)) << 4) & 0x10);
                int x1 = ((qs >> 4) & 0x0F) | (int)((qh >> (j + 12)) & 0x10);
                dst[(size_t)r * rowElements + b * 32 + j] = d * (float)x0 + m;
                dst[(size_t)r * rowElements + b * 32 + j + 16] = d * (float)x1 + m;
            }
        }
}

/* TensorOps.DequantizeToFloat -- TensorOps.cs:18-56; returns 0 ok, -1 unsupported */
EXPORT int orc_dequantize(const uint8_t *src, float *dst, uint32_t type, int numRows, int rowElements)
{
    size_t count = (size_t)numRows * rowElements;
    switch (type) {
    case T_F32: memcpy(dst, src, count * 4); return 0;                        /* DequantizeBlock.cs:97-104 */
    case T_F16: for (size_t i = 0; i < count; i++) dst[i] = rd_half(src + 2 * i); return 0;
    case T_BF16:                                                             /* DequantizeBlock.cs:70-95 */
        for (size_t i = 0; i < count; i++) dst[i] = bits_f(((uint32_t)src[2 * i + 1] << 24) | ((uint32_t)src[2 * i] << 16));
        return 0;
    case T_Q4_0: deq_q4_0(src, dst, numRows, rowElements); return 0;
    case T_Q8_0: deq_q8_0(src, dst, numRows, rowElements); return 0;
    case T_Q2_K: deq_q2k(src, dst, numRows, rowElements); return 0;
    case T_Q3_K: deq_q3k(src, dst, numRows, rowElements); return 0;
    case T_Q4_K: deq_q4k(src, dst, numRows, rowElements); return 0;
    case T_Q5_K: deq_q5k(src, dst, numRows, rowElements); return 0;
    case T_Q6_K: deq_q6k(src, dst, numRows, rowElements); return 0;
    case T_Q4_1: deq_q4_1(src, dst, numRows, rowElements); return 0;
    case T_Q5_0: deq_q5_0(src, dst, numRows, rowElements); return 0;
    case T_Q5_1: deq_q5_1(src, dst, numRows, rowElements); return 0;
    default: return -1;
    }
}

/* ------------------------------------------------------------------------ */
/* 8-lane helpers */

/* Vector.Dot(acc, Vector<float>.One): see header for the assumed tree order.  The order is the
 * one thing the reference's source leaves to the JIT and the host's vector unit; a diagnostic
 * switch (orc_set_hsum_order(1)) sums the lanes left to right instead, to measure how far the
 * reference algorithm's own result moves when only that order changes. */
static int g_hsum_order = 0;
EXPORT void orc_set_hsum_order(int order) { g_hsum_order = order; }
static float hsum8(const float *v)
{
    if (g_hsum_order == 1) return ((((((v[0] + v[1]) + v[2]) + v[3]) + v[4]) + v[5]) + v[6]) + v[7];
    return ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
}

/* TensorOps.DotProduct -- TensorOps.cs:510-531 */
static float dot_product(const float *a, const float *b, int n)
{
    float acc[VEC] = {0};
    int i = 0;
    for (; i <= n - VEC; i += VEC)
        for (int l = 0; l < VEC; l++) acc[l] = acc[l] + a[i + l] * b[i + l];
    float dot = hsum8(acc);
    for (; i < n; i++) dot += a[i] * b[i];
    return dot;
}

/* ------------------------------------------------------------------------ */
/* Fused single-row matvecs, TensorOps.cs:116-431 */

static int g_threads = 1;
/* Diagnostic knob (tests only): round the cached K/V to IEEE binary16, as a device
 * fp16 KV cache stores them.  Off by default; the reference keeps fp32. */
static int g_kv_fp16 = 0;
EXPORT void orc_set_kv_fp16(int on) { g_kv_fp16 = on; }
static void kv_store(float *dst, const float *src, int n)
{
    for (int i = 0; i < n; i++) dst[i] = g_kv_fp16 ? (float)(_Float16)src[i] : src[i];
}
EXPORT void orc_set_threads(int n) { g_threads = n > 0 ? n : 1; }
EXPORT int orc_get_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_num_procs();
#else
    return 1;
#endif
}

static void mm_q4_0(const float *a, const uint8_t *b, float *res, int aCols, int bCols)
{   /* TensorOps.cs:118-173 */
    int nb = aCols / 32;
#pragma omp parallel num_threads(g_threads)
    {
        float *fused = (float *)malloc(sizeof(float) * (size_t)aCols);
#pragma omp for schedule(static)
        for (int c = 0; c < bCols; c++) {
            const uint8_t *row = b + (size_t)c * nb * 18;
            for (int blk = 0; blk < nb; blk++) {
                const uint8_t *o = row + blk * 18;
                float d = rd_half(o);
                int base = blk * 32;
                for (int i = 0; i < 16; i++) {
                    int qs = o[2 + i];
                    fused[base + i] = a[base + i] * (((float)(qs & 0x0F) - 8.0f) * d);
                    fused[base + i + 16] = a[base + i + 16] * (((float)((qs >> 4) & 0x0F) - 8.0f) * d);
                }
            }
            float acc[VEC] = {0};
            int k = 0;
            for (; k <= aCols - VEC; k += VEC)
                for (int l = 0; l < VEC; l++) acc[l] = acc[l] + fused[k + l];
            float dot = hsum8(acc);
            for (; k < aCols; k++) dot += fused[k];
            res[c] = dot;
        }
        free(fused);
    }
}

static void mm_q8_0(const float *a, const uint8_t *b, float *res, int aCols, int bCols)
{   /* TensorOps.cs:179-224 */
    int nb = aCols / 32;
#pragma omp parallel num_threads(g_threads)
    {
        float *fused = (float *)malloc(sizeof(float) * (size_t)aCols);
#pragma omp for schedule(static)
        for (int c = 0; c < bCols; c++) {
            const uint8_t *row = b + (size_t)c * nb * 34;
            int fi = 0;
            for (int blk = 0; blk < nb; blk++) {
                const uint8_t *o = row + blk * 34;
                float d = rd_half(o);
                for (int i = 0; i < 32; i++) { fused[fi] = a[fi] * ((float)(int8_t)o[2 + i] * d); fi++; }
            }
            float acc[VEC] = {0};
            int k = 0;
            for (; k <= aCols - VEC; k += VEC)
                for (int l = 0; l < VEC; l++) acc[l] = acc[l] + fused[k + l];
            float r = hsum8(acc);
            for (; k < aCols; k++) r += fused[k];
            res[c] = r;
        }
        free(fused);
    }
}

static void mm_q6k(const float *a, const uint8_t *b, float *res, int aCols, int bCols)
{   /* TensorOps.cs:230-287: dequantise the row, then DotProduct */
    int nb = aCols / 256;
#pragma omp parallel num_threads(g_threads)
    {
        float *deq = (float *)malloc(sizeof(float) * (size_t)aCols);
#pragma omp for schedule(static)
        for (int c = 0; c < bCols; c++) {
            deq_q6k(b + (size_t)c * nb * 210, deq, 1, aCols);
            res[c] = dot_product(a, deq, aCols);
        }
        free(deq);
    }
}

static void mm_q2k(const float *a, const uint8_t *b, float *res, int aCols, int bCols)
{   /* TensorOps.cs:293-329 */
    int nb = aCols / 256;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int c = 0; c < bCols; c++) {
        float dot = 0.0f;
        for (int blk = 0; blk < nb; blk++) {
            const uint8_t *o = b + ((size_t)c * nb + blk) * 84;
            float d = rd_half(o), dmin = rd_half(o + 2);
            int base = blk * 256;
            for (int i = 0; i < 256; i++) {
                int g = i / 64, local = i % 64, sub = local / 16, scIdx = g * 4 + sub;
                int sc = o[4 + scIdx * 2] & 0x0F, mi = o[4 + scIdx * 2 + 1] & 0x0F;
                int q = (o[20 + i / 4] >> ((i % 4) * 2)) & 0x3;
                dot += a[base + i] * (d * (float)sc * ((float)q - 0.5f) - dmin * (float)mi);
            }
        }
        res[c] = dot;
    }
}

static void mm_q3k(const float *a, const uint8_t *b, float *res, int aCols, int bCols)
{   /* TensorOps.cs:331-362 (note the association a*d*sc*value) */
    int nb = aCols / 256;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int c = 0; c < bCols; c++) {
        float dot = 0.0f;
        for (int blk = 0; blk < nb; blk++) {
            const uint8_t *o = b + ((size_t)c * nb + blk) * 110;
            float d = rd_half(o);
            int base = blk * 256;
            for (int i = 0; i < 256; i++) {
                int g = i / 16;
                int sc = extract6(o + 4, g * 6);
                int q = (o[48 + i / 4] >> ((i % 4) * 2)) & 0x3;
                int m = (o[16 + i / 8] >> (i % 8)) & 0x1;
                int value = q - (m << 2);
                dot += a[base + i] * d * (float)sc * (float)value;
            }
        }
        res[c] = dot;
    }
}

static void mm_q4k(const float *a, const uint8_t *b, float *res, int aCols, int bCols)
{   /* TensorOps.cs:364-395 */
    int nb = aCols / 256;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int c = 0; c < bCols; c++) {
        float dot = 0.0f;
        for (int blk = 0; blk < nb; blk++) {
            const uint8_t *o = b + ((size_t)c * nb + blk) * 144;
            float d = rd_half(o), dmin = rd_half(o + 2);
            int base = blk * 256;
            for (int i = 0; i < 256; i++) {
                int g = i / 32;
                int sc = extract6(o + 4, g * 12), mi = extract6(o + 4, g * 12 + 6);
                int q = (o[16 + i / 2] >> ((i % 2) * 4)) & 0xF;
                dot += a[base + i] * (d * (float)sc * (float)(q - 8) - dmin * (float)mi);
            }
        }
        res[c] = dot;
    }
}

static void mm_q5k(const float *a, const uint8_t *b, float *res, int aCols, int bCols)
{   /* TensorOps.cs:397-431 */
    int nb = aCols / 256;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int c = 0; c < bCols; c++) {
        float dot = 0.0f;
        for (int blk = 0; blk < nb; blk++) {
            const uint8_t *o = b + ((size_t)c * nb + blk) * 176;
            float d = rd_half(o), dmin = rd_half(o + 2);
            int base = blk * 256;
            for (int i = 0; i < 256; i++) {
                int g = i / 32;
                int sc = extract6(o + 4, g * 12), mi = extract6(o + 4, g * 12 + 6);
                int qLow = (o[48 + i / 2] >> ((i % 2) * 4)) & 0xF;
                int qHigh = (o[16 + i / 8] >> (i % 8)) & 0x1;
                int q5 = qLow + (qHigh << 4);
                dot += a[base + i] * (d * (float)sc * (float)(q5 - 16) - dmin * (float)mi);
            }
        }
        res[c] = dot;
    }
}

/* TensorOps.MatMulF32 -- TensorOps.cs:437-504 (single-row and multi-row paths share the math) */
EXPORT void orc_matmul_f32(const float *a, const float *b, float *res, int resLen, int aCols, int bCols)
{
    int aRows = resLen / bCols;
    for (int r = 0; r < aRows; r++) {
        const float *ar = a + (size_t)r * aCols;
#pragma omp parallel for num_threads(g_threads) schedule(static)
        for (int c = 0; c < bCols; c++)
            res[(size_t)r * bCols + c] = dot_product(ar, b + (size_t)c * aCols, aCols);
    }
}

/* TensorOps.MatMul -- TensorOps.cs:60-112.  resLen = result.Length; returns -1 on unsupported type */
EXPORT int orc_matmul(const float *a, const uint8_t *b, float *res, int resLen, uint32_t bType, int aCols, int bCols)
{
    int aRows = resLen / bCols;
    if (aRows == 1) {
        switch (bType) {
        case T_Q4_0: mm_q4_0(a, b, res, aCols, bCols); return 0;
        case T_Q8_0: mm_q8_0(a, b, res, aCols, bCols); return 0;
        case T_Q6_K: mm_q6k(a, b, res, aCols, bCols); return 0;
        case T_Q4_K: mm_q4k(a, b, res, aCols, bCols); return 0;
        case T_Q2_K: mm_q2k(a, b, res, aCols, bCols); return 0;
        case T_Q3_K: mm_q3k(a, b, res, aCols, bCols); return 0;
        case T_Q5_K: mm_q5k(a, b, res, aCols, bCols); return 0;
        default: break;
        }
    }
    uint64_t rowBytes = orc_byte_count(bType, (uint64_t)aCols);
    if (rowBytes == 0) return -1;
    int err = 0;
    for (int r = 0; r < aRows; r++) {
#pragma omp parallel num_threads(g_threads)
        {
            float *tmp = (float *)malloc(sizeof(float) * (size_t)aCols);
#pragma omp for schedule(static)
            for (int c = 0; c < bCols; c++) {
                if (orc_dequantize(b + (size_t)c * rowBytes, tmp, bType, 1, aCols) != 0) { err = -1; continue; }
                res[(size_t)r * bCols + c] = dot_product(a + (size_t)r * aCols, tmp, aCols);
            }
            free(tmp);
        }
    }
    return err;
}

/* ------------------------------------------------------------------------ */
/* VectorMath -- src/Llmdot.Core/Tensors/Numeric/VectorMath.cs */

/* ExpApproxVector, VectorMath.cs:137-166 (one lane) */
EXPORT float orc_exp_approx(float x)
{
    float clamped = x > -87.3f ? x : -87.3f;
    clamped = clamped < 88.4f ? clamped : 88.4f;
    int k = (int)(clamped * 1.4426950408889634f + 0.5f);
    float kf = (float)k;
    float y = clamped - kf * 0.693145751953125f - kf * 1.42860677e-6f;
    float c = y * y * 0.5f;
    float pade = 1.0f + y + c + c * y * 0.3333333f + c * y * y * 0.2f;
    float scale = bits_f((uint32_t)(k + 127) << 23);
    float result = pade * scale;
    if (x < -87.3f) result = 0.0f;
    if (x > 88.4f) result = INFINITY;
    return result;
}

/* TanhApproxVector, VectorMath.cs:196-209 (one lane) */
EXPORT float orc_tanh_approx(float x)
{
    float x2 = x * x;
    float approx = x * (27.0f + x2) / (27.0f + 9.0f * x2);
    if (fabsf(x) > 4.0f) return x > 0.0f ? 1.0f : -1.0f;
    return approx;
}

/* VectorMath.Add(Span a, b) :27-42; Add(a,b,result) :10-25 (same per-element op) */
EXPORT void orc_add(const float *a, const float *b, float *res, int n) { for (int i = 0; i < n; i++) res[i] = a[i] + b[i]; }
/* Scale :44-76 */
EXPORT void orc_scale(const float *in, float s, float *res, int n) { for (int i = 0; i < n; i++) res[i] = in[i] * s; }
/* Mul :78-93 */
EXPORT void orc_mul(const float *a, const float *b, float *res, int n) { for (int i = 0; i < n; i++) res[i] = a[i] * b[i]; }

/* Silu / SiluInPlace :99-135 -- vector lanes use ExpApprox, tail uses MathF.Exp */
EXPORT void orc_silu(const float *in, float *res, int n)
{
    int i = 0;
    for (; i <= n - VEC; i += VEC)
        for (int l = 0; l < VEC; l++) { float x = in[i + l]; res[i + l] = x / (1.0f + orc_exp_approx(-x)); }
    for (; i < n; i++) { float x = in[i]; res[i] = x / (1.0f + expf(-x)); }
}

/* Gelu(float) :168-170 */
EXPORT float orc_gelu_scalar(float x) { return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x))); }

/* Gelu(span) :172-194 -- vector lanes use TanhApprox with a different association */
EXPORT void orc_gelu(const float *in, float *res, int n)
{
    int i = 0;
    for (; i <= n - VEC; i += VEC)
        for (int l = 0; l < VEC; l++) {
            float x = in[i + l];
            float t = orc_tanh_approx(x * 0.7978845608028654f * (1.0f + 0.044715f * x * x * x));
            res[i + l] = 0.5f * x * (1.0f + t);
        }
    for (; i < n; i++) res[i] = orc_gelu_scalar(in[i]);
}

/* FindMax :260-284 */
static float find_max(const float *x, int n)
{
    if (n >= VEC) {
        float lm[VEC];
        for (int l = 0; l < VEC; l++) lm[l] = x[l];
        int mi = VEC;
        for (; mi <= n - VEC; mi += VEC)
            for (int l = 0; l < VEC; l++) lm[l] = x[mi + l] > lm[l] ? x[mi + l] : lm[l];
        float m = -INFINITY;
        for (int k = 0; k < VEC; k++) if (lm[k] > m) m = lm[k];
        for (; mi < n; mi++) if (x[mi] > m) m = x[mi];
        return m;
    }
    float m = x[0];
    for (int i = 1; i < n; i++) if (x[i] > m) m = x[i];
    return m;
}

/* Softmax(span, softcap) :215-258 */
EXPORT void orc_softmax(float *x, int n, int hasCap, float cap)
{
    if (n == 0) return;
    if (hasCap) {
        float invCap = 1.0f / cap;
        int si = 0;
        for (; si <= n - VEC; si += VEC)
            for (int l = 0; l < VEC; l++) x[si + l] = cap * orc_tanh_approx(x[si + l] * invCap);
        for (; si < n; si++) x[si] = cap * tanhf(x[si] / cap);
    }
    float max = find_max(x, n);
    float acc[VEC] = {0};
    int j = 0;
    for (; j <= n - VEC; j += VEC)
        for (int l = 0; l < VEC; l++) { float e = orc_exp_approx(x[j + l] - max); x[j + l] = e; acc[l] = acc[l] + e; }
    float sum = hsum8(acc);
    for (; j < n; j++) { x[j] = expf(x[j] - max); sum += x[j]; }
    float invSum = 1.0f / sum;
    for (int i = 0; i < n; i++) x[i] = x[i] * invSum;
}

/* Softcap :286-302 */
EXPORT void orc_softcap(float *x, int n, float cap)
{
    float invCap = 1.0f / cap;
    int i = 0;
    for (; i <= n - VEC; i += VEC)
        for (int l = 0; l < VEC; l++) x[i + l] = cap * orc_tanh_approx(x[i + l] * invCap);
    for (; i < n; i++) x[i] = cap * tanhf(x[i] / cap);
}

/* RmsNorm :308-340 */
EXPORT void orc_rmsnorm(const float *in, const float *w, float *out, int n, float eps)
{
    float acc[VEC] = {0};
    int i = 0;
    for (; i <= n - VEC; i += VEC)
        for (int l = 0; l < VEC; l++) acc[l] = acc[l] + in[i + l] * in[i + l];
    float ss = hsum8(acc);
    for (; i < n; i++) ss += in[i] * in[i];
    ss /= (float)n;
    ss += eps;
    float inv = 1.0f / sqrtf(ss);
    i = 0;
    for (; i <= n - VEC; i += VEC)
        for (int l = 0; l < VEC; l++) out[i + l] = w[i + l] * in[i + l] * inv;
    for (; i < n; i++) out[i] = w[i] * (in[i] * inv);
}

/* LayerNorm :342-406 (bias may be NULL) */
EXPORT void orc_layernorm(const float *in, const float *w, const float *bias, float *out, int n, float eps)
{
    float acc[VEC] = {0};
    int i = 0;
    for (; i <= n - VEC; i += VEC)
        for (int l = 0; l < VEC; l++) acc[l] = acc[l] + in[i + l];
    float mean = hsum8(acc);
    for (; i < n; i++) mean += in[i];
    mean /= (float)n;
    float vacc[VEC] = {0};
    i = 0;
    for (; i <= n - VEC; i += VEC)
        for (int l = 0; l < VEC; l++) { float d = in[i + l] - mean; vacc[l] = vacc[l] + d * d; }
    float var = hsum8(vacc);
    for (; i < n; i++) { float d = in[i] - mean; var += d * d; }
    var /= (float)n;
    float invStd = 1.0f / sqrtf(var + eps);
    i = 0;
    for (; i <= n - VEC; i += VEC)
        for (int l = 0; l < VEC; l++) {
            float v = w[i + l] * (in[i + l] - mean) * invStd;
            out[i + l] = bias ? v + bias[i + l] : v;
        }
    for (; i < n; i++) {
        float v = w[i] * (in[i] - mean) * invStd;
        out[i] = bias ? v + bias[i] : v;
    }
}

/* ArgMax :412-425 (strict '>': ties go to the lowest index) */
EXPORT int orc_argmax(const float *x, int n)
{
    int mi = 0;
    float mv = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mv) { mv = x[i]; mi = i; }
    return mi;
}

/* ------------------------------------------------------------------------ */
/* RoPE -- TensorOps.cs:656-743 (half-split pairs (i, i+half)) */

static void rope_core(float *q, float *k, int same, const float *cs, const float *sn, int half)
{
    for (int i = 0; i < half; i++) {
        float c = cs[i], s = sn[i];
        float q0 = q[i], q1 = q[i + half];
        q[i] = q0 * c - q1 * s;
        q[i + half] = q0 * s + q1 * c;
        if (same) continue;
        float k0 = k[i], k1 = k[i + half];
        k[i] = k0 * c - k1 * s;
        k[i + half] = k0 * s + k1 * c;
    }
}

/* ApplyRoPE(query, key, headDim, position, freqTable) :679-696 */
EXPORT void orc_rope_table(float *q, float *k, int same, int position, const float *freq, int half)
{
    float cs[512], sn[512];
    for (int i = 0; i < half; i++) {
        float angle = (float)position * freq[i];
        cs[i] = cosf(angle);
        sn[i] = sinf(angle);
    }
    rope_core(q, k, same, cs, sn, half);
}

/* ApplyRoPE(query, key, headDim, position, freqBase, rotaryDim) :658-677 */
EXPORT void orc_rope(float *q, float *k, int same, int headDim, int position, float freqBase, int rotaryDim)
{
    int rd = rotaryDim > 0 ? rotaryDim : headDim;
    int half = rd / 2;
    float cs[512], sn[512];
    for (int i = 0; i < half; i++) {
        float freq = 1.0f / powf(freqBase, 2.0f * (float)i / (float)rd);
        float angle = (float)position * freq;
        cs[i] = cosf(angle);
        sn[i] = sinf(angle);
    }
    rope_core(q, k, same, cs, sn, half);
}

/* ------------------------------------------------------------------------ */
/* GGUF reader -- src/Llmdot.Core/Loading/GgufReader.cs:8-126 */

enum { V_U8 = 0, V_I8, V_U16, V_I16, V_U32, V_I32, V_F32, V_BOOL, V_STR, V_ARR, V_U64, V_I64, V_F64 };

typedef struct {
    char *key;
    uint32_t type;
    double num;          /* scalar numeric value (ints, floats, bool) */
    char *str;           /* string value */
    uint32_t arr_type;   /* array element type */
    uint64_t arr_n;      /* array length */
    double *arr_num;     /* numeric array values (NULL for string arrays) */
} okv;

typedef struct {
    char *name;
    uint64_t name_len;  /* bytes read: a name may hold a NUL that C string functions stop at */
    uint32_t type, ndims;
    uint64_t dims[4];
    uint64_t nelem, offset;
    const uint8_t *data;
    uint64_t nbytes;
} otensor;

typedef struct { const uint8_t *p, *end; int err; } rd_t;

static uint64_t rd_n(rd_t *r, int n)
{
    if (r->p + n > r->end) { r->err = 1; return 0; }
    uint64_t v = 0;
    for (int i = 0; i < n; i++) v |= (uint64_t)r->p[i] << (8 * i);
    r->p += n;
    return v;
}
static char *rd_str_len(rd_t *r, uint64_t *out_len)
{
    uint64_t len = rd_n(r, 8);
    if (out_len) *out_len = len;
    if (r->err || len > (uint64_t)(r->end - r->p)) { r->err = 1; return NULL; }
    char *s = (char *)malloc(len + 1);
    memcpy(s, r->p, len);
    s[len] = 0;
    r->p += len;
    return s;
}
static char *rd_str(rd_t *r) { return rd_str_len(r, NULL); }
static double rd_scalar(rd_t *r, uint32_t t);
/* a nested array's contents: GgufReader.ReadGgufArray reads them recursively (GgufReader.cs:84-96);
 * nothing on the path uses them.  Depth-limited. */
static void rd_skip_array(rd_t *r, int depth)
{
    if (depth > 64) { r->err = 1; return; }
    uint32_t t = (uint32_t)rd_n(r, 4);
    uint64_t cnt = rd_n(r, 8);
    for (uint64_t j = 0; j < cnt && !r->err; j++) {
        if (t == V_STR) { uint64_t len = rd_n(r, 8); if (len > (uint64_t)(r->end - r->p)) r->err = 1; else r->p += len; }
        else if (t == V_ARR) rd_skip_array(r, depth + 1);
        else rd_scalar(r, t);
    }
}
static double rd_scalar(rd_t *r, uint32_t t)
{
    switch (t) {
    case V_U8: return (double)(uint8_t)rd_n(r, 1);
    case V_I8: return (double)(int8_t)rd_n(r, 1);
    case V_U16: return (double)(uint16_t)rd_n(r, 2);
    case V_I16: return (double)(int16_t)rd_n(r, 2);
    case V_U32: return (double)(uint32_t)rd_n(r, 4);
    case V_I32: return (double)(int32_t)rd_n(r, 4);
    case V_F32: { uint32_t b = (uint32_t)rd_n(r, 4); return (double)bits_f(b); }
    case V_BOOL: return rd_n(r, 1) != 0 ? 1.0 : 0.0;
    case V_U64: return (double)rd_n(r, 8);
    case V_I64: return (double)(int64_t)rd_n(r, 8);
    case V_F64: { uint64_t b = rd_n(r, 8); double d; memcpy(&d, &b, 8); return d; }
    default: r->err = 1; return 0;
    }
}

/* ------------------------------------------------------------------------ */
/* Model: TransformerConfig (doc/architecture.md:171-225) resolved by
 * ArchitectureResolver.Resolve (src/Llmdot.Core/Loading/ArchitectureResolver.cs:14-112). */

enum { TPL_LLAMA = 0, TPL_NEOX = 1, TPL_GEMMA = 2, TPL_LFM2 = 3 };
enum { FFN_STANDARD = 0, FFN_SWIGLU = 1, FFN_GEGLU = 2 };
enum { ROPE_NONE = 0, ROPE_LINEAR = 1, ROPE_YARN = 2, ROPE_LONGROPE = 3 };

/* Mirror of the C-ABI llmdot_config struct (include/llmdot_cuda.h); field order is shared. */
typedef struct {
    int32_t template_id, hidden, layers, context, vocab, ffn, heads, heads_kv, head_dim;
    int32_t qkv_fused, norm_is_rms;
    float eps;
    int32_t has_post_norm;
    float rope_base;
    int32_t rope_dim, rope_scaling;
    float rope_factor;
    int32_t ffn_type, parallel_residual, tied;
    float emb_scale;
    int32_t sliding_window, has_attn_cap;
    float attn_cap;
    int32_t has_final_cap;
    float final_cap;
    int32_t expert_count, bos, eos;
} orc_config;

typedef struct {
    uint8_t *file;
    size_t file_size;
    okv *kv;
    int nkv;
    otensor *t;
    int nt;
    orc_config cfg;
    int32_t *hkv_per_layer;
    int n_hkv_per_layer;
    float *rope_freq;
    int rope_half;
    char arch[64];
    int conv_kernel;      /* ConvKernelSize (0 unless HasConvLayers) */
    int bad_rope;         /* a negative rotary dimension, refused when a session is created */
    int expert_used;      /* ExpertUsedCount */
    uint8_t *layer_attn;  /* LayerTypes: 1 Attention, 0 Conv */
} omodel;

/* the last entry of a key wins, as GgufReader's `values[key] = ...` (GgufReader.cs:44-53) */
static okv *find_kv(omodel *m, const char *key)
{
    for (int i = m->nkv - 1; i >= 0; i--) if (m->kv[i].key && strcmp(m->kv[i].key, key) == 0) return &m->kv[i];
    return NULL;
}
static okv *find_arch_kv(omodel *m, const char *key)
{
    char buf[256];
    snprintf(buf, sizeof buf, "%s.%s", m->arch, key);
    return find_kv(m, buf);
}
static int kv_is_num(const okv *v) { return v && v->type != V_STR && v->type != V_ARR; }
/* Convert.ToInt32 rounds floats to nearest-even */
static int to_i32(double d) { return (int)nearbyint(d); }
static int get_int(omodel *m, const char *key, int def)
{
    okv *v = find_arch_kv(m, key);
    return kv_is_num(v) ? to_i32(v->num) : def;
}
static float get_float(omodel *m, const char *key, float def, int *present)
{
    okv *v = find_arch_kv(m, key);
    if (present) *present = kv_is_num(v);
    return kv_is_num(v) ? (float)v->num : def;
}

/* case-insensitive tensor lookup (TensorNameResolver uses OrdinalIgnoreCase) */
/* LoadedModel.LoadTensors (LoadedModel.cs:77-107): tensors with data, keyed OrdinalIgnoreCase, a
 * later one replacing an earlier one of the same name -- the last loaded match wins */
static otensor *find_t(omodel *m, const char *name)
{
    for (int i = m->nt - 1; i >= 0; i--) if (m->t[i].data && strcasecmp(m->t[i].name, name) == 0) return &m->t[i];
    return NULL;
}
static otensor *find_tf(omodel *m, const char *fmt, int layer)
{
    char buf[128];
    snprintf(buf, sizeof buf, fmt, layer);
    return find_t(m, buf);
}
/* a tensor of that name exists in TensorInfos, data or not (case-insensitive) */
static int has_name(omodel *m, const char *fmt, int layer)
{
    char buf[128];
    snprintf(buf, sizeof buf, fmt, layer);
    for (int i = 0; i < m->nt; i++) if (strcasecmp(m->t[i].name, buf) == 0) return 1;
    return 0;
}
/* TensorInfos.Any(t => t.Name.Contains(sub)): over the whole name, NUL bytes included */
static int any_name_contains(omodel *m, const char *sub)
{
    for (int i = 0; i < m->nt; i++)
        if (m->t[i].name && memmem(m->t[i].name, (size_t)m->t[i].name_len, sub, strlen(sub))) return 1;
    return 0;
}

static char g_err[512];
EXPORT const char *orc_last_error(void) { return g_err; }

EXPORT void orc_model_free(omodel *m)
{
    if (!m) return;
    for (int i = 0; i < m->nkv; i++) { free(m->kv[i].key); free(m->kv[i].str); free(m->kv[i].arr_num); }
    for (int i = 0; i < m->nt; i++) free(m->t[i].name);
    free(m->kv); free(m->t); free(m->file); free(m->hkv_per_layer); free(m->rope_freq); free(m->layer_attn);
    free(m);
}

EXPORT omodel *orc_model_load(const char *path)
{
    FILE *f = fopen(path, "rb");
    if (!f) { snprintf(g_err, sizeof g_err, "cannot open %s", path); return NULL; }
    fseek(f, 0, SEEK_END);
    long sz = ftell(f);
    fseek(f, 0, SEEK_SET);
    omodel *m = (omodel *)calloc(1, sizeof(omodel));
    m->file = (uint8_t *)malloc((size_t)sz);
    m->file_size = (size_t)sz;
    if (fread(m->file, 1, (size_t)sz, f) != (size_t)sz) { fclose(f); snprintf(g_err, sizeof g_err, "short read"); orc_model_free(m); return NULL; }
    fclose(f);

    rd_t r = {m->file, m->file + sz, 0};
    if (sz < 4 || memcmp(m->file, "GGUF", 4) != 0) { snprintf(g_err, sizeof g_err, "Invalid GGUF magic. Expected 'GGUF'."); orc_model_free(m); return NULL; }
    r.p += 4;
    uint32_t version = (uint32_t)rd_n(&r, 4);
    if (version < 2) { snprintf(g_err, sizeof g_err, "Unsupported GGUF version: %u", version); orc_model_free(m); return NULL; }
    uint64_t nt = rd_n(&r, 8), nkv = rd_n(&r, 8);
    /* a count the file cannot hold (a key-value pair takes at least 12 bytes, a tensor info 24)
     * is a truncated header, not an allocation to attempt */
    const uint64_t left = (uint64_t)(r.end - r.p);
    if (r.err || nkv > left / 12 || nt > left / 24) { snprintf(g_err, sizeof g_err, "truncated GGUF header"); orc_model_free(m); return NULL; }
    m->kv = (okv *)calloc(nkv ? nkv : 1, sizeof(okv));
    for (uint64_t i = 0; i < nkv && !r.err; i++) {
        okv *v = &m->kv[m->nkv++];
        v->key = rd_str(&r);
        v->type = (uint32_t)rd_n(&r, 4);
        if (v->type == V_STR) v->str = rd_str(&r);
        else if (v->type == V_ARR) {
            v->arr_type = (uint32_t)rd_n(&r, 4);
            v->arr_n = rd_n(&r, 8);
            if (v->arr_type == V_STR) {
                for (uint64_t j = 0; j < v->arr_n && !r.err; j++) { uint64_t len = rd_n(&r, 8); if (len > (uint64_t)(r.end - r.p)) r.err = 1; else r.p += len; }
            } else if (v->arr_type == V_ARR) {
                for (uint64_t j = 0; j < v->arr_n && !r.err; j++) rd_skip_array(&r, 1);
            } else {
                if (v->arr_n > (uint64_t)(r.end - r.p)) { r.err = 1; break; }  /* >= 1 byte per element */
                v->arr_num = (double *)malloc(sizeof(double) * (v->arr_n ? v->arr_n : 1));
                if (!v->arr_num) { r.err = 1; break; }
                for (uint64_t j = 0; j < v->arr_n && !r.err; j++) v->arr_num[j] = rd_scalar(&r, v->arr_type);
            }
        } else v->num = rd_scalar(&r, v->type);
    }
    m->t = (otensor *)calloc(nt ? nt : 1, sizeof(otensor));
    for (uint64_t i = 0; i < nt && !r.err; i++) {
        otensor *t = &m->t[m->nt++];
        t->name = rd_str_len(&r, &t->name_len);
        t->ndims = (uint32_t)rd_n(&r, 4);
        if (t->ndims > 4) { r.err = 1; break; }
        uint32_t ne = 1; /* the reference multiplies the uint dims in 32-bit arithmetic */
        for (uint32_t d = 0; d < t->ndims; d++) { t->dims[d] = (uint32_t)rd_n(&r, 8); ne *= (uint32_t)t->dims[d]; }
        t->nelem = t->ndims ? ne : 0;
        t->type = (uint32_t)rd_n(&r, 4);
        t->offset = rd_n(&r, 8);
    }
    if (r.err) { snprintf(g_err, sizeof g_err, "truncated GGUF header"); orc_model_free(m); return NULL; }
    okv *al = find_kv(m, "general.alignment");
    uint64_t alignment = kv_is_num(al) ? (uint64_t)al->num : 32;
    uint64_t dataOff = (uint64_t)(r.p - m->file);
    dataOff += (alignment - dataOff % alignment) % alignment;
    /* LoadedModel.LoadTensors (src/Llmdot.Core/Inference/LoadedModel.cs:77-107): skip truncated tensors */
    for (int i = 0; i < m->nt; i++) {
        otensor *t = &m->t[i];
        t->nbytes = orc_byte_count(t->type, t->nelem);
        /* TensorSize.ByteCount throws for a type it does not know, whatever the element count */
        if (orc_byte_count(t->type, 256) == 0) { snprintf(g_err, sizeof g_err, "Unsupported GGML type: %u", t->type); orc_model_free(m); return NULL; }
        /* overflow-safe form of dataOff + offset + nbytes > file size */
        if (t->nbytes == 0 || dataOff > (uint64_t)sz || t->offset > (uint64_t)sz - dataOff ||
            t->nbytes > (uint64_t)sz - dataOff - t->offset) { t->data = NULL; continue; }
        t->data = m->file + dataOff + t->offset;
    }

    /* ArchitectureResolver.Resolve */
    okv *a = find_kv(m, "general.architecture");
    if (!a || a->type != V_STR || !a->str[0]) { snprintf(g_err, sizeof g_err, "GGUF model missing 'general.architecture' metadata key."); orc_model_free(m); return NULL; }
    snprintf(m->arch, sizeof m->arch, "%s", a->str);
    const char *sup[] = {"llama", "phi3", "qwen2", "phi2", "gptneox", "gemma", "gemma2", "stablelm", "lfm2", "lfm2_moe"};
    int ok = 0;
    for (int i = 0; i < 10; i++) if (strcasecmp(m->arch, sup[i]) == 0) ok = 1;
    if (!ok) { snprintf(g_err, sizeof g_err, "Unsupported GGUF architecture: '%s'", m->arch); orc_model_free(m); return NULL; }
    orc_config *c = &m->cfg;
    if (!strcasecmp(m->arch, "phi2") || !strcasecmp(m->arch, "gptneox")) c->template_id = TPL_NEOX;
    else if (!strcasecmp(m->arch, "gemma") || !strcasecmp(m->arch, "gemma2")) c->template_id = TPL_GEMMA;
    else if (!strcasecmp(m->arch, "lfm2") || !strcasecmp(m->arch, "lfm2_moe")) c->template_id = TPL_LFM2;
    else c->template_id = TPL_LLAMA;
    c->hidden = get_int(m, "embedding_length", 0);
    c->layers = get_int(m, "block_count", 0);
    c->context = get_int(m, "context_length", 0);
    c->ffn = get_int(m, "feed_forward_length", 0);
    c->heads = get_int(m, "attention.head_count", 0);
    okv *hkv = find_arch_kv(m, "attention.head_count_kv");
    if (hkv && hkv->type == V_ARR && hkv->arr_num && hkv->arr_n > 0) {
        m->n_hkv_per_layer = (int)hkv->arr_n;
        m->hkv_per_layer = (int32_t *)malloc(sizeof(int32_t) * hkv->arr_n);
        int mx = 0;
        for (uint64_t j = 0; j < hkv->arr_n; j++) { m->hkv_per_layer[j] = to_i32(hkv->arr_num[j]); if (m->hkv_per_layer[j] > mx) mx = m->hkv_per_layer[j]; }
        c->heads_kv = mx;
    } else c->heads_kv = get_int(m, "attention.head_count_kv", c->heads);
    c->head_dim = get_int(m, "attention.key_length", c->hidden / (c->heads > 1 ? c->heads : 1));
    okv *toks = find_kv(m, "tokenizer.ggml.tokens");
    c->vocab = (toks && toks->type == V_ARR) ? (int)toks->arr_n : 0;
    int present = 0;
    c->eps = get_float(m, "attention.layer_norm_rms_epsilon", 0, &present);
    if (present) c->norm_is_rms = 1;
    else {
        c->eps = get_float(m, "attention.layer_norm_epsilon", 0, &present);
        if (!present) { snprintf(g_err, sizeof g_err, "No norm epsilon found for architecture '%s'.", m->arch); orc_model_free(m); return NULL; }
        c->norm_is_rms = 0;
    }
    c->rope_base = get_float(m, "rope.freq_base", 10000.0f, NULL);
    c->rope_dim = get_int(m, "rope.dimension_count", c->head_dim);
    {   /* ResolveRopeScaling :169-183 */
        okv *st = find_arch_kv(m, "rope.scaling.type");
        c->rope_scaling = ROPE_NONE;
        if (st && st->type == V_STR) {
            if (!strcasecmp(st->str, "linear")) c->rope_scaling = ROPE_LINEAR;
            else if (!strcasecmp(st->str, "yarn")) c->rope_scaling = ROPE_YARN;
            else if (!strcasecmp(st->str, "longrope")) c->rope_scaling = ROPE_LONGROPE;
        }
        c->rope_factor = get_float(m, "rope.scaling.factor", 1.0f, NULL);
    }
    c->qkv_fused = any_name_contains(m, "attn_qkv");
    c->ffn_type = any_name_contains(m, "ffn_gate") ? (c->template_id == TPL_GEMMA ? FFN_GEGLU : FFN_SWIGLU) : FFN_STANDARD;
    okv *pr = find_arch_kv(m, "use_parallel_residual");
    c->parallel_residual = kv_is_num(pr) ? (pr->num != 0) : (c->template_id == TPL_NEOX);
    c->tied = 1;  /* !TensorInfos.Any(t => t.Name == "output.weight"), exact and case-sensitive */
    for (int i = 0; i < m->nt; i++) if (strcmp(m->t[i].name, "output.weight") == 0) c->tied = 0;
    {
        int es_present = 0;
        float es = get_float(m, "embedding_scale", 0, &es_present);
        c->emb_scale = es_present ? es : (c->template_id == TPL_GEMMA ? sqrtf((float)c->hidden) : 1.0f);
    }
    c->has_post_norm = any_name_contains(m, "post_attention_norm") || any_name_contains(m, "post_ffw_norm");
    c->sliding_window = get_int(m, "attention.sliding_window", 0);
    c->attn_cap = get_float(m, "attn_logit_softcapping", 0, &present);
    c->has_attn_cap = present;
    c->final_cap = get_float(m, "final_logit_softcapping", 0, &present);
    c->has_final_cap = present;
    c->expert_count = get_int(m, "expert_count", 0);
    m->expert_used = get_int(m, "expert_used_count", 0);
    /* HasConvLayers / ConvKernelSize / LayerTypes (:66-70); ResolveLayerTypes :226-238: a layer
     * is Attention when blk.N.attn_q, attn_k or attn_qkv is among the tensor infos */
    m->layer_attn = (uint8_t *)malloc(c->layers > 0 ? (size_t)c->layers : 1);
    if (!m->layer_attn) { snprintf(g_err, sizeof g_err, "out of memory (%d layers)", c->layers); orc_model_free(m); return NULL; }
    m->conv_kernel = 0;
    for (int l = 0; l < c->layers; l++) m->layer_attn[l] = 1;
    if (c->template_id == TPL_LFM2) {
        m->conv_kernel = get_int(m, "shortconv.l_cache", 3);
        for (int l = 0; l < c->layers; l++)
            m->layer_attn[l] = (uint8_t)(has_name(m, "blk.%d.attn_q.weight", l) || has_name(m, "blk.%d.attn_k.weight", l) ||
                                         has_name(m, "blk.%d.attn_qkv.weight", l));
    }
    {
        okv *b = find_kv(m, "tokenizer.ggml.bos_token_id");
        okv *e = find_kv(m, "tokenizer.ggml.eos_token_id");
        c->bos = kv_is_num(b) ? to_i32(b->num) : 1;
        c->eos = kv_is_num(e) ? to_i32(e->num) : 2;
    }
    /* PrecomputeRopeFrequencies -- InferenceEngine.cs:57-72 */
    int rd = c->rope_dim > 0 ? c->rope_dim : c->head_dim;
    /* the reference builds this table in the InferenceEngine constructor, not at load: a rope
     * dimension it cannot size fails the session (orc_session_new), as `new float[halfDim]` would */
    m->rope_half = rd / 2 > 0 ? rd / 2 : 0;
    m->bad_rope = rd / 2 < 0 ? rd : 0;
    m->rope_freq = (float *)malloc(sizeof(float) * (m->rope_half ? (size_t)m->rope_half : 1));
    if (!m->rope_freq) { snprintf(g_err, sizeof g_err, "out of memory (rope dimension %d)", rd); orc_model_free(m); return NULL; }
    for (int i = 0; i < m->rope_half; i++) {
        float freq = 1.0f / powf(c->rope_base, 2.0f * (float)i / (float)rd);
        if (c->rope_scaling == ROPE_LINEAR && c->rope_factor > 1.0f) freq /= c->rope_factor;
        m->rope_freq[i] = freq;
    }
    if (c->template_id == TPL_LFM2 && m->conv_kernel < 1) {
        snprintf(g_err, sizeof g_err, "conv kernel size %d", m->conv_kernel);
        orc_model_free(m);
        return NULL;
    }
    return m;
}

EXPORT void orc_model_config(omodel *m, orc_config *out) { *out = m->cfg; }
EXPORT const float *orc_model_rope_freq(omodel *m, int *half) { *half = m->rope_half; return m->rope_freq; }

/* ------------------------------------------------------------------------ */
/* ConvStateCache (src/Llmdot.Core/Inference/ConvStateCache.cs:3-65): per layer a ring of the
 * last kernel-1 conv inputs; BuildInput lays the window out channel-major, [c * K + k], zeros
 * before position 0; Store writes at the layer's head, which counts stores, not positions. */
typedef struct {
    int layers, hidden, hist, k;
    float *buf;      /* [layers][hist][hidden] */
    float *scratch;  /* [k * hidden] */
    int *head;       /* [layers] */
} oconv;

EXPORT void orc_conv_state_free(oconv *cs)
{
    if (!cs) return;
    free(cs->buf); free(cs->scratch); free(cs->head);
    free(cs);
}

EXPORT oconv *orc_conv_state_new(int layers, int hidden, int kernel)
{
    if (layers < 0 || hidden <= 0 || kernel < 1) return NULL;
    oconv *cs = (oconv *)calloc(1, sizeof(oconv));
    cs->layers = layers; cs->hidden = hidden; cs->hist = kernel - 1; cs->k = kernel;
    size_t nb = (size_t)layers * cs->hist * hidden;
    cs->buf = (float *)calloc(nb ? nb : 1, sizeof(float));
    cs->scratch = (float *)calloc((size_t)kernel * hidden, sizeof(float));
    cs->head = (int *)calloc(layers ? (size_t)layers : 1, sizeof(int));
    return cs;
}

EXPORT void orc_conv_state_store(oconv *cs, int layer, const float *x)   /* Store :24-31 */
{
    if (cs->hist == 0) return;
    int pos = cs->head[layer];
    memcpy(cs->buf + ((size_t)layer * cs->hist + pos) * cs->hidden, x, sizeof(float) * cs->hidden);
    cs->head[layer] = (pos + 1) % cs->hist;
}

EXPORT const float *orc_conv_state_build(oconv *cs, int layer, const float *cur, int position)  /* BuildInput :33-56 */
{
    const int K = cs->k, H = cs->hist;
    float *r = cs->scratch;
    for (int c = 0; c < cs->hidden; c++) {
        for (int k = 0; k < H; k++) {
            int req = position - H + k;
            r[(size_t)c * K + k] = req < 0 ? 0.0f : cs->buf[((size_t)layer * H + req % H) * cs->hidden + c];
        }
        r[(size_t)c * K + H] = cur[c];
    }
    return r;
}

EXPORT void orc_conv_state_reset(oconv *cs)   /* Reset :58-62 */
{
    memset(cs->buf, 0, sizeof(float) * (size_t)cs->layers * cs->hist * cs->hidden);
    memset(cs->head, 0, sizeof(int) * (size_t)(cs->layers ? cs->layers : 1));
}

/* TensorOps.Conv1D (TensorOps.cs:745-778): kernel 1 is an elementwise product; otherwise per
 * channel 8-lane products summed in lanes, the lanes added (Vector.Dot with One), then the tail
 * k's added in order -- for kernels below 8 only the tail runs, after a +0 from the empty lanes */
EXPORT void orc_conv1d(const float *in, const float *w, float *out, int K, int dim)
{
    if (K == 1) {
        for (int i = 0; i < dim; i++) out[i] = in[i] * w[i];
        return;
    }
    for (int c = 0; c < dim; c++) {
        const float *x = in + (size_t)c * K, *wk = w + (size_t)c * K;
        float acc[VEC] = {0};
        int k = 0;
        for (; k <= K - VEC; k += VEC)
            for (int l = 0; l < VEC; l++) acc[l] = acc[l] + x[k + l] * wk[k + l];
        float sum = hsum8(acc);
        for (; k < K; k++) sum += x[k] * wk[k];
        out[c] = sum;
    }
}

/* MoeRouter.Route (src/Llmdot.Core/Inference/MoeRouter.cs:12-59): gate logits by the backend's
 * MatMul (the generic dequantise-and-dot path for F32 gates), top-k by repeated first-maximum
 * scans over the experts not yet taken (strict >, starting from float.MinValue, so an
 * exhausted scan leaves index -1), then MathF.Exp softmax over the k selected values. */
EXPORT int orc_moe_route(const float *hidden_state, const uint8_t *gate, uint32_t gate_type, int hidden, int experts,
                         int top_k, float *logits, int *selected, float *weights)
{
    if (orc_matmul(hidden_state, gate, logits, experts, gate_type, hidden, experts) != 0) return -1;
    for (int i = 0; i < top_k; i++) {
        int best = -1;
        float bv = -FLT_MAX;
        for (int j = 0; j < experts; j++) {
            int skip = 0;
            for (int k = 0; k < i; k++) if (selected[k] == j) { skip = 1; break; }
            if (skip) continue;
            if (logits[j] > bv) { bv = logits[j]; best = j; }
        }
        selected[i] = best;
        weights[i] = bv;
    }
    float mx = -FLT_MAX;
    for (int i = 0; i < top_k; i++) if (weights[i] > mx) mx = weights[i];
    float sum = 0.0f;
    for (int i = 0; i < top_k; i++) {
        weights[i] = expf(weights[i] - mx);
        sum += weights[i];
    }
    for (int i = 0; i < top_k; i++) weights[i] /= sum;
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Session: KvCache (src/Llmdot.Core/Inference/KvCache.cs:3-43) and InferenceBuffers
 * (InferenceBuffers.cs:29-62), fp32 throughout like the reference. */

typedef struct {
    omodel *m;
    float *kc, *vc;          /* [layers][ctx][kvDim] */
    int pos;
    float *h, *logits, *norm, *norm2, *normtmp, *q, *k, *v, *attnout, *attnres, *ffn, *ffnres, *score;
    float *scratch;
    oconv *conv;                         /* ConvStateCache when HasConvLayers */
    float *convb, *convq, *convw;        /* ConvBuf, the conv output, the dequantised conv weights */
    float *moe_logits, *moe_w, *moe_acc, *moe_res;
    int *moe_sel;
} osess;

EXPORT void orc_session_free(osess *s)
{
    if (!s) return;
    free(s->kc); free(s->vc); free(s->h); free(s->logits); free(s->norm); free(s->norm2); free(s->normtmp);
    free(s->q); free(s->k); free(s->v); free(s->attnout); free(s->attnres); free(s->ffn); free(s->ffnres);
    free(s->score); free(s->scratch);
    orc_conv_state_free(s->conv);
    free(s->convb); free(s->convq); free(s->convw);
    free(s->moe_logits); free(s->moe_w); free(s->moe_acc); free(s->moe_res); free(s->moe_sel);
    free(s);
}

EXPORT osess *orc_session_new(omodel *m)
{
    orc_config *c = &m->cfg;
    if (m->bad_rope) { snprintf(g_err, sizeof g_err, "bad rope dimension %d", m->bad_rope); return NULL; }
    osess *s = (osess *)calloc(1, sizeof(osess));
    s->m = m;
    size_t kvDim = (size_t)c->heads_kv * c->head_dim, qDim = (size_t)c->heads * c->head_dim;
    size_t kvsz = (size_t)c->layers * c->context * kvDim;
    s->kc = (float *)calloc(kvsz ? kvsz : 1, sizeof(float));
    s->vc = (float *)calloc(kvsz ? kvsz : 1, sizeof(float));
    size_t hid = (size_t)c->hidden;
    s->h = (float *)calloc(hid, 4); s->logits = (float *)calloc((size_t)c->vocab, 4);
    s->norm = (float *)calloc(hid, 4); s->norm2 = (float *)calloc(hid, 4); s->normtmp = (float *)calloc(hid, 4);
    s->q = (float *)calloc(qDim, 4); s->k = (float *)calloc(kvDim, 4); s->v = (float *)calloc(kvDim, 4);
    s->attnout = (float *)calloc(hid, 4);
    s->attnres = (float *)calloc(qDim > hid ? qDim : hid, 4);
    size_t inter = 2 * (size_t)c->ffn > 3 * hid ? 2 * (size_t)c->ffn : 3 * hid;
    s->ffn = (float *)calloc(inter, 4); s->ffnres = (float *)calloc(hid, 4);
    s->score = (float *)calloc(hid > (size_t)c->context ? hid : (size_t)c->context, 4);
    s->scratch = (float *)calloc(qDim + 2 * kvDim + hid, 4);
    if (c->template_id == TPL_LFM2) {   /* InferenceEngine.cs:52 */
        s->conv = orc_conv_state_new(c->layers, c->hidden, m->conv_kernel);
        s->convb = (float *)calloc(hid, 4);
        s->convq = (float *)calloc(hid, 4);
        s->convw = (float *)calloc((size_t)m->conv_kernel * hid, 4);
    }
    if (c->expert_count > 0) {          /* InferenceBuffers.cs:56-60 */
        int tk = m->expert_used > 0 ? m->expert_used : 1;
        s->moe_logits = (float *)calloc((size_t)c->expert_count, 4);
        s->moe_w = (float *)calloc((size_t)tk, 4);
        s->moe_sel = (int *)calloc((size_t)tk, sizeof(int));
        s->moe_acc = (float *)calloc(hid, 4);
        s->moe_res = (float *)calloc(hid, 4);
    }
    if (!s->kc || !s->vc) { orc_session_free(s); snprintf(g_err, sizeof g_err, "out of memory"); return NULL; }
    return s;
}

/* Generate's _kvCache.Reset() / _convCache?.Reset() (InferenceEngine.cs:79-80) */
EXPORT void orc_session_reset(osess *s)
{
    s->pos = 0;
    if (s->conv) orc_conv_state_reset(s->conv);
}

static float *norm_weights(omodel *m, otensor *t, float *buf)
{   /* LoadedModel.GetDequantizedWeights :63-75 (norm vectors are F32 or dequantised) */
    int rows = t->ndims > 1 ? (int)t->dims[1] : 1;
    orc_dequantize(t->data, buf, t->type, rows, (int)(t->nelem / (uint64_t)rows));
    (void)m;
    return buf;
}

/* InferenceEngine.MatMulFromTensor :604-617 */
static int matmul_tensor(const float *input, otensor *w, float *out, int cols)
{
    int inDim = (int)w->dims[0];
    if (w->type == T_F32) { orc_matmul_f32(input, (const float *)w->data, out, cols, inDim, cols); return 0; }
    return orc_matmul(input, w->data, out, cols, w->type, inDim, cols);
}

/* ApplyNorm :544-562 */
static void apply_norm(osess *s, const float *in, float *out, int layer, int isAttn)
{
    omodel *m = s->m;
    orc_config *c = &m->cfg;
    otensor *w = isAttn ? find_tf(m, "blk.%d.attn_norm.weight", layer) : find_tf(m, "blk.%d.ffn_norm.weight", layer);
    if (!w) w = find_tf(m, "blk.%d.attn_norm.weight", layer);
    float *wb = s->scratch;
    norm_weights(m, w, wb);
    if (c->norm_is_rms) orc_rmsnorm(in, wb, out, c->hidden, c->eps);
    else {
        otensor *bt = isAttn ? find_tf(m, "blk.%d.attn_norm.bias", layer) : NULL;
        float *bb = NULL;
        if (bt) { bb = s->scratch + c->hidden; norm_weights(m, bt, bb); }
        orc_layernorm(in, wb, bb, out, c->hidden, c->eps);
    }
}

/* ApplyPostNorm :564-573 */
static void apply_post_norm(osess *s, int layer, int isAttn)
{
    omodel *m = s->m;
    orc_config *c = &m->cfg;
    otensor *w = isAttn ? find_tf(m, "blk.%d.post_attention_norm.weight", layer) : find_tf(m, "blk.%d.post_ffw_norm.weight", layer);
    if (!w) return;
    norm_weights(m, w, s->scratch);
    memcpy(s->normtmp, s->h, sizeof(float) * c->hidden);
    orc_rmsnorm(s->normtmp, s->scratch, s->h, c->hidden, c->eps);
}

/* AttentionForward :304-450 */
static int attention_forward(osess *s, int layer, int position, const float *input)
{
    omodel *m = s->m;
    orc_config *c = &m->cfg;
    int hd = c->head_dim, H = c->heads, hidden = c->hidden;
    int hkvl = (m->n_hkv_per_layer > layer) ? (m->hkv_per_layer[layer] > 1 ? m->hkv_per_layer[layer] : 1) : c->heads_kv;
    int qDim = H * hd, kvDimL = hkvl * hd, gKv = c->heads_kv * hd;
    float *q = s->q, *k = s->k, *v = s->v;
    int rc = 0;
    if (c->qkv_fused) {
        otensor *ft = find_tf(m, "blk.%d.attn_qkv.weight", layer);
        if (!ft) { snprintf(g_err, sizeof g_err, "missing attn_qkv"); return -1; }
        int fc = qDim + 2 * kvDimL;
        float *fb = fc <= 2 * c->ffn ? s->ffn : (float *)malloc(sizeof(float) * fc);
        rc |= matmul_tensor(input, ft, fb, fc);
        memcpy(q, fb, sizeof(float) * qDim);
        memcpy(k, fb + qDim, sizeof(float) * kvDimL);
        memcpy(v, fb + qDim + kvDimL, sizeof(float) * kvDimL);
        if (fb != s->ffn) free(fb);
    } else {
        otensor *qt = find_tf(m, "blk.%d.attn_q.weight", layer), *kt = find_tf(m, "blk.%d.attn_k.weight", layer), *vt = find_tf(m, "blk.%d.attn_v.weight", layer);
        if (!qt || !kt || !vt) { snprintf(g_err, sizeof g_err, "missing q/k/v"); return -1; }
        rc |= matmul_tensor(input, qt, q, (int)(qt->nelem / (uint64_t)hidden));
        rc |= matmul_tensor(input, kt, k, (int)(kt->nelem / (uint64_t)hidden));
        rc |= matmul_tensor(input, vt, v, (int)(vt->nelem / (uint64_t)hidden));
    }
    otensor *qn = find_tf(m, "blk.%d.attn_q_norm.weight", layer);
    if (qn) {
        float *w = s->scratch;
        norm_weights(m, qn, w);
        for (int h = 0; h < H; h++) orc_rmsnorm(q + h * hd, w, q + h * hd, hd, c->eps);
    }
    for (int h = 0; h < H; h++) orc_rope_table(q + h * hd, q + h * hd, 1, position, m->rope_freq, m->rope_half);
    otensor *kn = find_tf(m, "blk.%d.attn_k_norm.weight", layer);
    if (kn) {
        float *w = s->scratch;
        norm_weights(m, kn, w);
        for (int h = 0; h < hkvl; h++) orc_rmsnorm(k + h * hd, w, k + h * hd, hd, c->eps);
    }
    size_t lbase = (size_t)layer * c->context * gKv;
    for (int h = 0; h < hkvl; h++) {
        orc_rope_table(k + h * hd, k + h * hd, 1, position, m->rope_freq, m->rope_half);
        kv_store(s->kc + lbase + (size_t)position * gKv + h * hd, k + h * hd, hd);
        kv_store(s->vc + lbase + (size_t)position * gKv + h * hd, v + h * hd, hd);
    }
    int seqLen = position + 1;
    int attnStart = c->sliding_window > 0 ? (seqLen - c->sliding_window > 0 ? seqLen - c->sliding_window : 0) : 0;
    int attnLen = seqLen - attnStart;
    float *result = s->attnres;
    const float *keys = s->kc + lbase, *values = s->vc + lbase;
    int group = H / hkvl;
    float invSqrt = 1.0f / sqrtf((float)hd);
#pragma omp parallel num_threads(g_threads)
    {
        float *score = (float *)malloc(sizeof(float) * (size_t)(attnLen > 0 ? attnLen : 1));
#pragma omp for schedule(static)
        for (int h = 0; h < H; h++) {
            int kvH = h / group;
            const float *qs = q + h * hd;
            for (int sIdx = attnStart; sIdx < seqLen; sIdx++) {
                const float *kr = keys + (size_t)sIdx * gKv + kvH * hd;
                float acc[VEC] = {0};
                int d = 0;
                for (; d <= hd - VEC; d += VEC)
                    for (int l = 0; l < VEC; l++) acc[l] = acc[l] + qs[d + l] * kr[d + l];
                float dot = hsum8(acc);
                for (; d < hd; d++) dot += qs[d] * kr[d];
                score[sIdx - attnStart] = dot * invSqrt;
            }
            orc_softmax(score, attnLen, c->has_attn_cap, c->attn_cap);
            float *rs = result + h * hd;
            for (int d = 0; d < hd; d++) rs[d] = 0.0f;
            for (int t = 0; t < attnLen; t++) {
                float p = score[t];
                const float *vr = values + (size_t)(attnStart + t) * gKv + kvH * hd;
                int d = 0;
                for (; d <= hd - VEC; d += VEC)
                    for (int l = 0; l < VEC; l++) rs[d + l] = rs[d + l] + vr[d + l] * p;
                for (d = hd - hd % VEC; d < hd; d++) rs[d] += p * vr[d];
            }
        }
        free(score);
    }
    otensor *ot = find_tf(m, "blk.%d.attn_output.weight", layer);
    if (!ot) { snprintf(g_err, sizeof g_err, "missing attn_output"); return -1; }
    int outCols = (int)(ot->nelem / (uint64_t)(H * hd));
    rc |= matmul_tensor(result, ot, s->attnout, outCols);
    memcpy(s->attnres, s->attnout, sizeof(float) * hidden);
    return rc;
}

/* FfnForward :452-487 */
static int ffn_forward(osess *s, int layer, const float *input)
{
    omodel *m = s->m;
    orc_config *c = &m->cfg;
    int hidden = c->hidden, rc = 0;
    otensor *up = find_tf(m, "blk.%d.ffn_up.weight", layer), *down = find_tf(m, "blk.%d.ffn_down.weight", layer);
    if (!up || !down) { snprintf(g_err, sizeof g_err, "missing ffn tensors"); return -1; }
    if (c->ffn_type == FFN_SWIGLU || c->ffn_type == FFN_GEGLU) {
        otensor *gate = find_tf(m, "blk.%d.ffn_gate.weight", layer);
        int gc = (int)(gate->nelem / (uint64_t)hidden), uc = (int)(up->nelem / (uint64_t)hidden);
        rc |= matmul_tensor(input, gate, s->ffn, gc);
        if (c->ffn_type == FFN_SWIGLU) orc_silu(s->ffn, s->ffn, gc);
        else orc_gelu(s->ffn, s->ffn, gc);
        rc |= matmul_tensor(input, up, s->ffn + gc, uc);
        orc_mul(s->ffn, s->ffn + gc, s->ffn, gc);
        rc |= matmul_tensor(s->ffn, down, s->ffnres, hidden);
    } else {
        int uc = (int)(up->nelem / (uint64_t)hidden);
        rc |= matmul_tensor(input, up, s->ffn, uc);
        orc_gelu(s->ffn, s->ffn, uc);
        rc |= matmul_tensor(s->ffn, down, s->ffnres, hidden);
    }
    return rc;
}

/* ProcessConvLayer :222-277, the operator half: in_proj -> (B, C, x) chunks; B*x through the
 * short causal conv over the ConvStateCache window; times C; out_proj; residual add.  A conv
 * layer without in_proj or conv weights only stores its normed input. */
static int conv_forward(osess *s, int layer, int position)
{
    omodel *m = s->m;
    orc_config *c = &m->cfg;
    const int hidden = c->hidden, K = m->conv_kernel;
    otensor *inp = find_tf(m, "blk.%d.shortconv.in_proj.weight", layer);
    otensor *cw = find_tf(m, "blk.%d.conv1d.weight", layer);
    if (!cw) cw = find_tf(m, "blk.%d.shortconv.conv.weight", layer);
    if (!inp || !cw || !s->conv) {
        if (s->conv) orc_conv_state_store(s->conv, layer, s->norm);
        return 0;
    }
    /* GetDequantizedConvWeights :279-301 */
    if (cw->type == T_F32) memcpy(s->convw, cw->data, sizeof(float) * (size_t)K * hidden);
    else orc_dequantize(cw->data, s->convw, cw->type, cw->ndims > 1 ? (int)cw->dims[1] : 1, (int)cw->dims[0]);
    int inCols = (int)(inp->nelem / (uint64_t)hidden);
    size_t ffnLen = 2 * (size_t)c->ffn > 3 * (size_t)hidden ? 2 * (size_t)c->ffn : 3 * (size_t)hidden;
    float *ib = (size_t)inCols <= ffnLen ? s->ffn : (float *)malloc(sizeof(float) * (size_t)inCols);
    int rc = matmul_tensor(s->norm, inp, ib, inCols);
    const float *bch = ib, *cch = ib + hidden, *xch = ib + 2 * hidden;
    orc_mul(bch, xch, s->convb, hidden);
    const float *win = orc_conv_state_build(s->conv, layer, s->convb, position);
    orc_conv1d(win, s->convw, s->convq, K, hidden);
    orc_conv_state_store(s->conv, layer, s->convb);
    orc_mul(s->convq, cch, s->convq, hidden);
    otensor *op = find_tf(m, "blk.%d.shortconv.out_proj.weight", layer);
    if (op) rc |= matmul_tensor(s->convq, op, s->attnres, (int)(op->nelem / (uint64_t)hidden));
    else memcpy(s->attnres, s->convq, sizeof(float) * hidden);
    orc_add(s->h, s->attnres, s->h, hidden);
    if (ib != s->ffn) free(ib);
    return rc;
}

/* MoeFfnForward :489-542: route, then per selected expert a SwiGLU FFN through its own
 * blk.N.ffn_{gate,up,down}.E tensors, scaled by the routing weight and added in selection
 * order; experts whose tensors are missing are skipped.  ResolveLayer (TensorNameResolver.cs:
 * 109-165) requires the dense ffn_up / ffn_down names to exist even though they are unused. */
static int moe_forward(osess *s, int layer, const float *input)
{
    omodel *m = s->m;
    orc_config *c = &m->cfg;
    const int hidden = c->hidden, E = c->expert_count, topK = m->expert_used;
    if (!has_name(m, "blk.%d.ffn_up.weight", layer) || !has_name(m, "blk.%d.ffn_down.weight", layer)) {
        snprintf(g_err, sizeof g_err, "Tensor 'blk.%d.ffn_up/ffn_down.weight' not found in model.", layer);
        return -1;
    }
    otensor *gate = find_tf(m, "blk.%d.ffn_gate_inp.weight", layer);
    if (!gate) { snprintf(g_err, sizeof g_err, "missing blk.%d.ffn_gate_inp.weight", layer); return -1; }
    if (orc_moe_route(input, gate->data, gate->type, hidden, E, topK, s->moe_logits, s->moe_sel, s->moe_w) != 0) return -1;
    memset(s->moe_acc, 0, sizeof(float) * hidden);
    int rc = 0;
    size_t ffnLen = 2 * (size_t)c->ffn > 3 * (size_t)hidden ? 2 * (size_t)c->ffn : 3 * (size_t)hidden;
    for (int i = 0; i < topK; i++) {
        int e = s->moe_sel[i];
        char nb[128];
        otensor *g, *u, *d;
        snprintf(nb, sizeof nb, "blk.%d.ffn_gate.%d.weight", layer, e); g = find_t(m, nb);
        snprintf(nb, sizeof nb, "blk.%d.ffn_up.%d.weight", layer, e); u = find_t(m, nb);
        snprintf(nb, sizeof nb, "blk.%d.ffn_down.%d.weight", layer, e); d = find_t(m, nb);
        if (!g || !u || !d) continue;
        int gc = (int)(g->nelem / (uint64_t)hidden), uc = (int)(u->nelem / (uint64_t)hidden);
        float *fb = (size_t)gc + uc <= ffnLen ? s->ffn : (float *)malloc(sizeof(float) * ((size_t)gc + uc));
        rc |= matmul_tensor(input, g, fb, gc);
        orc_silu(fb, fb, gc);
        rc |= matmul_tensor(input, u, fb + gc, uc);
        orc_mul(fb, fb + gc, fb, gc);
        rc |= matmul_tensor(fb, d, s->moe_res, hidden);
        orc_scale(s->moe_res, s->moe_w[i], s->moe_res, hidden);
        orc_add(s->moe_acc, s->moe_res, s->moe_acc, hidden);
        if (fb != s->ffn) free(fb);
    }
    memcpy(s->ffnres, s->moe_acc, sizeof(float) * hidden);
    return rc;
}

/* ProcessToken :134-146 with ProcessLayer :158-220 and ComputeLogits :583-602.
 * Writes the raw logits (before any final softcap) to s->logits. */
EXPORT int orc_process_token(osess *s, int token, int position)
{
    omodel *m = s->m;
    orc_config *c = &m->cfg;
    int hidden = c->hidden, rc = 0;
    if (position < 0 || position >= c->context) { snprintf(g_err, sizeof g_err, "position %d outside context %d", position, c->context); return -1; }
    otensor *emb = find_t(m, "token_embd.weight");
    if (!emb || token < 0 || (uint64_t)token >= emb->dims[1]) { snprintf(g_err, sizeof g_err, "bad token %d", token); return -1; }
    uint64_t rowBytes = orc_byte_count(emb->type, (uint64_t)hidden);
    orc_dequantize(emb->data + (size_t)token * rowBytes, s->h, emb->type, 1, hidden);
    if (c->emb_scale != 1.0f) orc_scale(s->h, c->emb_scale, s->h, hidden);
    for (int l = 0; l < c->layers; l++) {
        if (c->template_id == TPL_NEOX) {                        /* :198-207 */
            apply_norm(s, s->h, s->norm, l, 1);
            rc |= attention_forward(s, l, position, s->norm);
            apply_norm(s, s->h, s->norm2, l, 0);
            rc |= ffn_forward(s, l, s->norm2);
            /* Add(AttnResultBuf, FfnResultBuf) then Add(hs, FfnResultBuf): the two-argument Add
             * writes its first argument (VectorMath.cs:27-42), so the sum lands in the attention
             * buffer and only the FFN output reaches the hidden state */
            orc_add(s->attnres, s->ffnres, s->attnres, hidden);
            orc_add(s->h, s->ffnres, s->h, hidden);
        } else if (c->template_id == TPL_LFM2 && !m->layer_attn[l]) {   /* ProcessConvLayer :222-277 */
            apply_norm(s, s->h, s->norm, l, 1);
            rc |= conv_forward(s, l, position);
            apply_norm(s, s->h, s->norm2, l, 0);
            rc |= c->expert_count > 0 ? moe_forward(s, l, s->norm2) : ffn_forward(s, l, s->norm2);
            orc_add(s->h, s->ffnres, s->h, hidden);
        } else {                                                  /* :184-196, :209-220 */
            apply_norm(s, s->h, s->norm, l, 1);
            rc |= attention_forward(s, l, position, s->norm);
            orc_add(s->h, s->attnres, s->h, hidden);
            if (c->template_id == TPL_GEMMA && c->has_post_norm) apply_post_norm(s, l, 1);
            apply_norm(s, s->h, s->norm, l, 0);
            /* LlamaLike (and Lfm2Like attention layers) route through the experts when present */
            if (c->template_id != TPL_GEMMA && c->expert_count > 0) rc |= moe_forward(s, l, s->norm);
            else rc |= ffn_forward(s, l, s->norm);
            orc_add(s->h, s->ffnres, s->h, hidden);
            if (c->template_id == TPL_GEMMA && c->has_post_norm) apply_post_norm(s, l, 0);
        }
        if (rc) return rc;
    }
    /* ApplyFinalNorm :575-581 */
    otensor *fn = find_t(m, "output_norm.weight");
    if (!fn) fn = find_t(m, "token_embd_norm.weight");
    norm_weights(m, fn, s->scratch);
    memcpy(s->normtmp, s->h, sizeof(float) * hidden);
    orc_rmsnorm(s->normtmp, s->scratch, s->h, hidden, c->eps);
    otensor *out = find_t(m, "output.weight");
    if (!out) out = emb;
    if (out->type == T_F32) orc_matmul_f32(s->h, (const float *)out->data, s->logits, c->vocab, hidden, c->vocab);
    else rc |= orc_matmul(s->h, out->data, s->logits, c->vocab, out->type, hidden, c->vocab);
    return rc;
}

EXPORT const float *orc_session_logits(osess *s) { return s->logits; }
EXPORT const float *orc_session_hidden(osess *s) { return s->h; }

/* InferenceEngine.Generate :74-132, greedy (Sampler.Sample with Temperature<=0 -> ArgMax,
 * src/Llmdot.Core/Sampling/Sampler.cs:24-27).  Stops at EOS like the reference.
 * out_logits (nullable) receives, per generated token, the raw logits it was sampled from
 * (before the final softcap).  Returns the number of tokens written, or -1 on error. */
EXPORT int orc_generate(osess *s, const int *prompt, int nPrompt, int maxTokens, int *outTokens, float *outLogits)
{
    omodel *m = s->m;
    orc_config *c = &m->cfg;
    orc_session_reset(s);
    int have = 0;
    for (int i = 0; i < nPrompt; i++) {
        if (orc_process_token(s, prompt[i], i)) return -1;
        s->pos++;
        have = 1;
    }
    if (!have) {
        int init = c->bos > 0 ? c->bos : 0;
        if (orc_process_token(s, init, 0)) return -1;
        s->pos++;
    }
    int generated = 0;
    float *lg = (float *)malloc(sizeof(float) * c->vocab);
    while (generated < maxTokens) {
        if (outLogits) memcpy(outLogits + (size_t)generated * c->vocab, s->logits, sizeof(float) * c->vocab);
        memcpy(lg, s->logits, sizeof(float) * c->vocab);
        if (c->has_final_cap) orc_softcap(lg, c->vocab, c->final_cap);
        int next = orc_argmax(lg, c->vocab);
        outTokens[generated] = next;
        if (next == c->eos) { generated++; break; }
        if (generated + 1 == maxTokens) { generated++; break; } /* the reference's last forward is unused */
        if (orc_process_token(s, next, s->pos)) { free(lg); return -1; }
        s->pos++;
        generated++;
    }
    free(lg);
    return generated;
}


/* ---------------------------------------------------------------- sampling
 * Sampler.Sample (src/Llmdot.Core/Sampling/Sampler.cs:24-62) with SamplingOptions
 * (SamplingOptions.cs:7-14).  The uniform draw r is the caller's: Sampler takes
 * Random(seed).NextSingle() for seed >= 0 (orc_net_random_single) and Random.Shared otherwise. */

/* ApplyRepeatPenalty :64-81: the last `window` tokens of the history, in order, each applied once */
static void repeat_penalty(float *x, int n, float penalty, int window, const int *recent, int nRecent)
{
    if (penalty == 1.0f || nRecent == 0 || window <= 0) return;
    int start = nRecent - window > 0 ? nRecent - window : 0;
    for (int i = start; i < nRecent; i++) {
        int t = recent[i];
        if (t >= 0 && t < n) {
            if (x[t] > 0) x[t] = x[t] / penalty;
            else x[t] = x[t] * penalty;
        }
    }
}

/* FindTopK :83-127: the first k entries seed the set; a later entry replaces the first minimum
 * of the set when it is strictly larger; then an insertion sort, descending */
static void find_top_k(const float *x, int n, int k, int *idx, float *val)
{
    for (int i = 0; i < k; i++) { idx[i] = i; val[i] = x[i]; }
    for (int i = k; i < n; i++) {
        int mi = 0;
        for (int j = 1; j < k; j++) if (val[j] < val[mi]) mi = j;
        if (x[i] > val[mi]) { idx[mi] = i; val[mi] = x[i]; }
    }
    for (int i = 1; i < k; i++) {
        int ki = idx[i];
        float kv = val[i];
        int j = i - 1;
        while (j >= 0 && val[j] < kv) { idx[j + 1] = idx[j]; val[j + 1] = val[j]; j--; }
        idx[j + 1] = ki;
        val[j + 1] = kv;
    }
}

/* FindNucleus :129-151: selection sort by probability, descending, then the prefix whose
 * running sum first reaches top_p.  Sample (:48-50) passes its samplingBuf both as the
 * probabilities and as `values`, so the caller passes val == p: each `val[i] = p[idx[i]]` may
 * read a slot an earlier iteration already overwrote (when idx[i] < i), as the reference's
 * aliased spans do.  No restrict: the aliasing is the behaviour being restated. */
static int find_nucleus(const float *p, int n, float topP, int *idx, float *val)
{
    for (int i = 0; i < n; i++) idx[i] = i;
    for (int i = 0; i < n - 1; i++) {
        int mx = i;
        for (int j = i + 1; j < n; j++) if (p[idx[j]] > p[idx[mx]]) mx = j;
        if (mx != i) { int t = idx[i]; idx[i] = idx[mx]; idx[mx] = t; }
    }
    float cum = 0.0f;
    int count = 0;
    for (int i = 0; i < n; i++) {
        val[i] = p[idx[i]];
        cum += val[i];
        count++;
        if (cum >= topP) break;
    }
    return count;
}

/* FindNucleus's result without its quadratic sort, for rows of any size (same idx prefix, same
 * aliased writes into p, same count).  The selection sort takes, at each pass, the first
 * maximum in the CURRENT order and swaps it with the pass position; values are distinct across
 * tie groups, so groups come out in descending value, and inside a group the members leave in the
 * order of their positions at the moment the group becomes the maximum: the only element a pass
 * displaces is the occupant of the pass position, the smallest remaining position, and an
 * occupant that belongs to the current group is itself that group's first member.  So: sort by
 * value, and per group order the members by their current positions while replaying the swaps. */
typedef struct { float v; int i; } vkey;
static int vkey_desc(const void *a, const void *b)
{
    const vkey *x = (const vkey *)a, *y = (const vkey *)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return x->i - y->i;
}
static int *g_pos_for_cmp;
static int pos_asc(const void *a, const void *b)
{
    return g_pos_for_cmp[*(const int *)a] - g_pos_for_cmp[*(const int *)b];
}
static int find_nucleus_fast(float *p, int n, float topP, int *idx)
{
    vkey *ord = (vkey *)malloc(sizeof(vkey) * (size_t)n);
    int *pos = (int *)malloc(sizeof(int) * (size_t)n), *at = (int *)malloc(sizeof(int) * (size_t)n);
    int *grp = (int *)malloc(sizeof(int) * (size_t)n);
    for (int e = 0; e < n; e++) { ord[e].v = p[e]; ord[e].i = e; pos[e] = e; at[e] = e; }
    qsort(ord, (size_t)n, sizeof(vkey), vkey_desc);
    float cum = 0.0f;
    int i = 0, count = n;
    for (int g = 0; g < n && count == n;) {
        int ge = g + 1;
        while (ge < n && !(ord[ge].v < ord[g].v)) ge++;
        int m = ge - g;
        for (int k = 0; k < m; k++) grp[k] = ord[g + k].i;
        g_pos_for_cmp = pos;
        qsort(grp, (size_t)m, sizeof(int), pos_asc);
        for (int k = 0; k < m; k++) {
            int sel = grp[k], o = at[i];
            if (o != sel) { at[pos[sel]] = o; pos[o] = pos[sel]; at[i] = sel; pos[sel] = i; }
            idx[i] = sel;
            float v = p[sel];  /* slot sel already holds a written value when sel < i */
            p[i] = v;
            cum += v;
            i++;
            if (cum >= topP) { count = i; break; }
        }
        g = ge;
    }
    free(ord); free(pos); free(at); free(grp);
    return count;
}

/* Both forms on a copy of p (test hook): count; idx[0..count) and the written buffer out */
EXPORT int orc_nucleus(const float *p, int n, float topP, int fast, int *idx, float *buf)
{
    memcpy(buf, p, sizeof(float) * (size_t)n);
    return fast ? find_nucleus_fast(buf, n, topP, idx) : find_nucleus(buf, n, topP, idx, buf);
}

/* SampleFromProbabilities :153-165 */
static int pick(const float *p, int n, float r)
{
    float cum = 0.0f;
    for (int i = 0; i < n; i++) {
        cum += p[i];
        if (r <= cum) return i;
    }
    return n - 1;
}

EXPORT int orc_sample(const float *logits, int n, int topK, float topP, float temperature, float penalty, int window,
                      const int *recent, int nRecent, float r)
{
    if (temperature <= 0.0f) return orc_argmax(logits, n);
    float *x = (float *)malloc(sizeof(float) * n * 2);
    int *idx = (int *)malloc(sizeof(int) * n);
    memcpy(x, logits, sizeof(float) * n);
    repeat_penalty(x, n, penalty, window, recent, nRecent);
    float s = 1.0f / temperature;
    for (int i = 0; i < n; i++) x[i] = x[i] * s; /* VectorMath.Scale: x * s in every lane */
    int out;
    if (topK > 0 && topK < n) {
        float *val = x + n;
        find_top_k(x, n, topK, idx, val);
        orc_softmax(val, topK, 0, 0.0f);
        out = idx[pick(val, topK, r)];
    } else {
        orc_softmax(x, n, 0, 0.0f);
        out = -1;
        if (topP < 1.0f) {
            /* values alias the softmax row (Sample :48-50); when the nucleus is the whole row the
             * fall-through pick below reads the overwritten row and returns a position.  The
             * sort-and-replay form gives the selection sort's result (tests hold the two equal) */
            float *val = x;
            int ns = find_nucleus_fast(x, n, topP, idx);
            if (ns < n) {
                float sum = 0.0f;
                for (int i = 0; i < ns; i++) sum += val[i];
                float inv = 1.0f / sum;
                for (int i = 0; i < ns; i++) val[i] = val[i] * inv;
                out = idx[pick(val, ns, r)];
            }
        }
        if (out < 0) out = pick(x, n, r);
    }
    free(x);
    free(idx);
    return out;
}

/* new System.Random(seed).NextSingle(): the seeded generator is Knuth's subtractive generator
 * (the .NET 5-compatible seeded implementation), NextSingle = (float)(sample / int.MaxValue).
 * Restated from the published algorithm; not checked against .NET here (no runtime). */
EXPORT float orc_net_random_single(int seed)
{
    const int MBIG = 2147483647, MSEED = 161803398;
    int sa[56];
    memset(sa, 0, sizeof(sa));
    int sub = seed == (-2147483647 - 1) ? 2147483647 : (seed < 0 ? -seed : seed);
    int mj = MSEED - sub;
    sa[55] = mj;
    int mk = 1;
    for (int i = 1; i < 55; i++) {
        int ii = (21 * i) % 55;
        sa[ii] = mk;
        mk = mj - mk;
        if (mk < 0) mk += MBIG;
        mj = sa[ii];
    }
    for (int k = 1; k < 5; k++)
        for (int i = 1; i < 56; i++) {
            sa[i] -= sa[1 + (i + 30) % 55];
            if (sa[i] < 0) sa[i] += MBIG;
        }
    int inext = 1, inextp = 22; /* 0 and 21, advanced once */
    int ret = sa[inext] - sa[inextp];
    if (ret == MBIG) ret--;
    if (ret < 0) ret += MBIG;
    return (float)(ret * (1.0 / MBIG));
}

/* Generate (InferenceEngine.cs:74-131) with Sampler.Sample: the history starts as the prompt
 * and keeps the last window + 1 tokens; r[i] is the draw for generated token i */
EXPORT int orc_generate_sampled(osess *s, const int *prompt, int nPrompt, int maxTokens, int topK, float topP,
                                float temperature, float penalty, int window, const float *r, int *outTokens)
{
    omodel *m = s->m;
    orc_config *c = &m->cfg;
    orc_session_reset(s);
    int have = 0;
    for (int i = 0; i < nPrompt; i++) {
        if (orc_process_token(s, prompt[i], i)) return -1;
        s->pos++;
        have = 1;
    }
    if (!have) {
        int init = c->bos > 0 ? c->bos : 0;
        if (orc_process_token(s, init, 0)) return -1;
        s->pos++;
    }
    int cap = nPrompt + maxTokens + 1;
    int *recent = (int *)malloc(sizeof(int) * (cap > 1 ? cap : 1));
    int nRecent = 0;
    for (int i = 0; i < nPrompt; i++) recent[nRecent++] = prompt[i];
    float *lg = (float *)malloc(sizeof(float) * c->vocab);
    int generated = 0;
    while (generated < maxTokens) {
        memcpy(lg, s->logits, sizeof(float) * c->vocab);
        if (c->has_final_cap) orc_softcap(lg, c->vocab, c->final_cap);
        int next = orc_sample(lg, c->vocab, topK, topP, temperature, penalty, window, recent, nRecent, r[generated]);
        recent[nRecent++] = next;
        if (nRecent > window + 1) {
            int drop = nRecent - window - 1;
            memmove(recent, recent + drop, sizeof(int) * (nRecent - drop));
            nRecent -= drop;
        }
        outTokens[generated] = next;
        if (next == c->eos) { generated++; break; }
        if (generated + 1 == maxTokens) { generated++; break; }
        if (orc_process_token(s, next, s->pos)) { free(lg); free(recent); return -1; }
        s->pos++;
        generated++;
    }
    free(lg);
    free(recent);
    return generated;
}
