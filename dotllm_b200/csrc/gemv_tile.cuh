// gemv_tile.cuh -- per-warp tensor-core math on one 16-row x 256-weight quantised tile.
//
// Shared by the standalone matvec kernel (gemv.cu) and the persistent decode-step kernel
// (step.cu).  A tile is one super-block of 16 consecutive rows, re-laid out at load time so
// that lane L = 4g + t of a warp finds its bytes as one 16-byte slot per 512-byte plane:
//   Q4_K (2304 bytes): planes 0..3 = nibbles of sub-blocks 2t, 2t+1 of rows g and g+8,
//                      headers (d, dmin, 12 scale bytes) of both rows at 2048 + g*32;
//   Q6_K (3360 bytes): planes 0..5 = low nibbles / high bits of rows g and g+8,
//                      int8 scales at 3072 + g*32, fp16 d at 3328 + g*4.
// The activation enters as fp16 hi/lo pairs (B operand columns 2v, 2v+1) of an exactly
// power-of-two-scaled x, so every product is exact and the sums are fp32.  Lanes whose B column
// is past the last vector (g >= 2*NV) load the last vector's fragment again: their C columns are
// never read, and an unconditional shared load costs no predication.
#pragma once
#include "common.cuh"

namespace llmdot {

enum { QT_Q4K = 0, QT_Q6K = 1 };

constexpr int Q4K_TILE = 16 * 144;  // 2304
constexpr int Q6K_TILE = 16 * 210;  // 3360

// ------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c)
{  // (a & b) | c
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c)
{
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b)
{
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ void mma_f16(float &d0, float &d1, float &d2, float &d3, uint32_t a0, uint32_t a1,
                                        uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi)
{
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}
__device__ __forceinline__ float half_bits(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)v)); }

// x fragments in shared memory: 16-byte units u(sb, t, w, v, part) holding the B operands of
// MMAs 2w and 2w+1 for lane-column (v, part); XOR-swizzled so a quarter-warp hits 8 distinct
// bank groups.
template <int NV> __device__ __forceinline__ int xunit(int sb, int t, int w, int v, int part)
{
    return (sb * 4 + t) * (16 * NV) + ((w * 2 * NV + v * 2 + part) ^ (2 * t));
}

// Per-lane view of one weight tile (Q4_K uses 6 of the registers, Q6_K 9), read from the slot.
struct TileRegs {
    uint4 r[9];
};

__device__ __forceinline__ void read_tile(TileRegs &T, const uint8_t *slot, int qt, int lane)
{
    const int g = lane >> 2;
    if (qt == QT_Q4K) {
#pragma unroll
        for (int p = 0; p < 4; p++) T.r[p] = *(const uint4 *)(slot + p * 512 + lane * 16);
        T.r[4] = *(const uint4 *)(slot + 2048 + g * 32);
        T.r[5] = *(const uint4 *)(slot + 2048 + g * 32 + 16);
    } else {
#pragma unroll
        for (int p = 0; p < 6; p++) T.r[p] = *(const uint4 *)(slot + p * 512 + lane * 16);
        T.r[6] = *(const uint4 *)(slot + 3072 + g * 32);
        T.r[7] = *(const uint4 *)(slot + 3072 + g * 32 + 16);
        T.r[8].x = *(const uint32_t *)(slot + 3328 + g * 4);
    }
}

template <int NV>
__device__ __forceinline__ void q4k_tile(const TileRegs &T, const uint4 *__restrict__ xs, const float *__restrict__ S,
                                         int nsb, int sb, int t, int bv, int bpart, float &acc0, float &acc1,
                                         float *corr0, float *corr1)
{
    float d_r[2], dm_r[2];
    uint32_t sc2[2][2], nsc2[2][2], sc16[2][2], nsc16[2][2];
    float coef[2][2];
    const uint32_t sh = (24u * (uint32_t)t) & 31u;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint4 hd = T.r[4 + h];
        d_r[h] = half_bits(hd.x & 0xFFFF);
        dm_r[h] = half_bits(hd.x >> 16);
        // the 24-bit (sc, m) pair of sub-blocks 2t, 2t+1 starts at byte 4 + 3t of the block
        const uint32_t lo = t < 2 ? hd.y : (t == 2 ? hd.z : hd.w), hi = t < 2 ? hd.z : hd.w;
        const uint32_t pr = __funnelshift_r(lo, hi, sh);
        const uint32_t scA = pr & 63u, mA = (pr >> 6) & 63u, scB = (pr >> 12) & 63u, mB = (pr >> 18) & 63u;
        const uint32_t sA = hsub2(0x64006400u | (scA * 0x10001u), 0x64006400u);
        const uint32_t sB = hsub2(0x64006400u | (scB * 0x10001u), 0x64006400u);
        sc2[h][0] = sA;
        sc2[h][1] = sB;
        nsc2[h][0] = hfma2(sA, 0xE400E400u, 0u);  // * -1024
        nsc2[h][1] = hfma2(sB, 0xE400E400u, 0u);
        // high nibbles taken in place (16q): (1024 + 16q) * (sc/16) - 64 sc = q sc, one rounding
        sc16[h][0] = hfma2(sA, 0x2C002C00u, 0u);    // * 1/16
        sc16[h][1] = hfma2(sB, 0x2C002C00u, 0u);
        nsc16[h][0] = hfma2(sA, 0xD400D400u, 0u);   // * -64
        nsc16[h][1] = hfma2(sB, 0xD400D400u, 0u);
        coef[h][0] = fmaf(8.0f * d_r[h], (float)scA, dm_r[h] * (float)mA);
        coef[h][1] = fmaf(8.0f * d_r[h], (float)scB, dm_r[h] * (float)mB);
    }
    // independent accumulator chains (MMA i goes to chain i % QC): the tensor-core latency of one
    // chain of 16 dependent MMAs would otherwise bound the tile
    constexpr int QC = 2;
    float c[QC][4];
#pragma unroll
    for (int q = 0; q < QC; q++) c[q][0] = c[q][1] = c[q][2] = c[q][3] = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const int j = w >> 2;  // sub-block 2t + j
        const uint32_t W0 = (&T.r[j].x)[w & 3], W1 = (&T.r[2 + j].x)[w & 3];
        const uint4 b = xs[xunit<NV>(sb, t, w, bv, bpart)];
        float *ca = c[(2 * w) % QC], *cb = c[(2 * w + 1) % QC];
        uint32_t a0 = hfma2(and_or(W0, 0x000F000Fu, 0x64006400u), sc2[0][j], nsc2[0][j]);
        uint32_t a1 = hfma2(and_or(W1, 0x000F000Fu, 0x64006400u), sc2[1][j], nsc2[1][j]);
        uint32_t a2 = hfma2(and_or(W0, 0x00F000F0u, 0x64006400u), sc16[0][j], nsc16[0][j]);
        uint32_t a3 = hfma2(and_or(W1, 0x00F000F0u, 0x64006400u), sc16[1][j], nsc16[1][j]);
        mma_f16(ca[0], ca[1], ca[2], ca[3], a0, a1, a2, a3, b.x, b.y);
        const uint32_t V0 = W0 >> 8, V1 = W1 >> 8;
        a0 = hfma2(and_or(V0, 0x000F000Fu, 0x64006400u), sc2[0][j], nsc2[0][j]);
        a1 = hfma2(and_or(V1, 0x000F000Fu, 0x64006400u), sc2[1][j], nsc2[1][j]);
        a2 = hfma2(and_or(V0, 0x00F000F0u, 0x64006400u), sc16[0][j], nsc16[0][j]);
        a3 = hfma2(and_or(V1, 0x00F000F0u, 0x64006400u), sc16[1][j], nsc16[1][j]);
        mma_f16(cb[0], cb[1], cb[2], cb[3], a0, a1, a2, a3, b.z, b.w);
    }
    float c0 = c[0][0], c1 = c[0][1], c2 = c[0][2], c3 = c[0][3];
#pragma unroll
    for (int q = 1; q < QC; q++) {
        c0 += c[q][0];
        c1 += c[q][1];
        c2 += c[q][2];
        c3 += c[q][3];
    }
    acc0 = fmaf(d_r[0], c0 + c1, acc0);
    acc1 = fmaf(d_r[1], c2 + c3, acc1);
#pragma unroll
    for (int v = 0; v < NV; v++) {
        const float *Sv = S + v * nsb * 8 + sb * 8 + 2 * t;
        corr0[v] = fmaf(coef[0][0], Sv[0], fmaf(coef[0][1], Sv[1], corr0[v]));
        corr1[v] = fmaf(coef[1][0], Sv[0], fmaf(coef[1][1], Sv[1], corr1[v]));
    }
}

// ---------------------------------------------------------------- Q4_K, int8 tensor-core form
// For one or two input vectors.  x enters as four signed 8-bit digits of X = x * 2^k (k per
// super-block, |X| <= 2^30), one MMA column per (vector, digit); the nibbles are the unsigned
// A operand of mma.m16n8k32 (one 32-weight sub-block per MMA, so its 6-bit scale multiplies
// the int32 result exactly).  Every product and sum of a super-block is exact integer
// arithmetic; the float result differs from the fp32 dot only by x's rounding at 2^-30 of the
// block's largest |x|.
// Tile (2304 bytes), lane L = 4g + t: plane p (0..3) at p*512 + L*16 holds the words
// {A row g, A row g+8, B row g, B row g+8} of sub-blocks j = 2p (low nibbles) and j' = 2p+1
// (high nibbles): byte b of A holds weight 4t+b, byte b of B weight 16+4t+b.  The low nibbles
// (W & 0x0F0F0F0F) are j's operand as they are, the high ones (W & 0xF0F0F0F0) are j''s times
// 16 (exact; divided out once per tile).  Headers at 2048 + g*32 (row g, then row g+8), 16
// bytes each: d, dmin (fp16), bytes 4..11: sc_j | (m_j & 3) << 6, bytes 12..15: m_j >> 2 in
// nibble j.
__device__ __forceinline__ void mma_u8s8_zero(int &d0, int &d1, int &d2, int &d3, uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1)
{
    const int z = 0;
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(z));
}

// x digit fragments: unit (sb, j, t, col) of 8 bytes, col = 4v + digit; lane (g, t) reads
// col g mod (4 NV).
template <int NV> __device__ __forceinline__ int x8unit(int sb, int j, int t, int col)
{
    return ((sb * 8 + j) * 4 + t) * (4 * NV) + col;
}

// One tile: accf[0..1] += rows g (columns 2t, 2t+1), accf[2..3] the same for row g+8, in units of
// d * 2^-k (the digit weights are applied when a unit ends); corr*[v] += the offset term of this
// lane's sub-blocks 2t, 2t+1 (coef = 8 d sc + dmin m, times the sub-block sums S of x).
template <int NV>
__device__ __forceinline__ void q4k_tile_i8(const TileRegs &T, const uint2 *__restrict__ xs8, const float *__restrict__ S,
                                            const float *__restrict__ xinv, int nsb, int sb, int g, int t,
                                            float (&accf)[4], float *corr0, float *corr1)
{
    const uint4 h0 = T.r[4], h1 = T.r[5];
    const uint32_t s0a = h0.y & 0x3F3F3F3Fu, s0b = h0.z & 0x3F3F3F3Fu;
    const uint32_t s1a = h1.y & 0x3F3F3F3Fu, s1b = h1.z & 0x3F3F3F3Fu;
    const uint2 *xp = xs8 + x8unit<NV>(sb, 0, t, g % (4 * NV));
    int ai0 = 0, ai1 = 0, ai2 = 0, ai3 = 0;  // low-nibble sub-blocks
    int ah0 = 0, ah1 = 0, ah2 = 0, ah3 = 0;  // high-nibble sub-blocks, times 16
#pragma unroll
    for (int p = 0; p < 4; p++) {
        const uint4 W = T.r[p];  // A row g, A row g+8, B row g, B row g+8
#pragma unroll
        for (int hi = 0; hi < 2; hi++) {
            const int j = 2 * p + hi;
            const uint32_t mk = hi ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
            const uint2 b = xp[j * 4 * (4 * NV)];
            int c0, c1, c2, c3;
            mma_u8s8_zero(c0, c1, c2, c3, W.x & mk, W.y & mk, W.z & mk, W.w & mk, b.x, b.y);
            const int sg = (int)__byte_perm(j < 4 ? s0a : s0b, 0u, 0x4440u | (j & 3));
            const int sg8 = (int)__byte_perm(j < 4 ? s1a : s1b, 0u, 0x4440u | (j & 3));
            if (hi) {
                ah0 += sg * c0;
                ah1 += sg * c1;
                ah2 += sg8 * c2;
                ah3 += sg8 * c3;
            } else {
                ai0 += sg * c0;
                ai1 += sg * c1;
                ai2 += sg8 * c2;
                ai3 += sg8 * c3;
            }
        }
    }
    ai0 += ah0 >> 4;  // exact: every high-nibble product is a multiple of 16
    ai1 += ah1 >> 4;
    ai2 += ah2 >> 4;
    ai3 += ah3 >> 4;
    const float d0 = half_bits(h0.x & 0xFFFF), d1 = half_bits(h1.x & 0xFFFF);
    const int v = min(t >> 1, NV - 1);
    const float xi = xinv[v * nsb + sb];
    const float f0 = d0 * xi, f1 = d1 * xi;
    accf[0] = fmaf(f0, (float)ai0, accf[0]);
    accf[1] = fmaf(f0, (float)ai1, accf[1]);
    accf[2] = fmaf(f1, (float)ai2, accf[2]);
    accf[3] = fmaf(f1, (float)ai3, accf[3]);
    // offset term of sub-blocks 2t, 2t+1
    const float dm0 = half_bits(h0.x >> 16), dm1 = half_bits(h1.x >> 16);
    const uint32_t r0 = t < 2 ? h0.y : h0.z, r1 = t < 2 ? h1.y : h1.z;  // bytes of sub-blocks 4*(t>=2) ..
#pragma unroll
    for (int jj = 0; jj < 2; jj++) {
        const int j = 2 * t + jj;
        const uint32_t bsel = (uint32_t)(j & 3);
        const uint32_t by0 = __byte_perm(r0, 0u, 0x4440u | bsel), by1 = __byte_perm(r1, 0u, 0x4440u | bsel);
        const float m0 = (float)((by0 >> 6) | (((h0.w >> (4 * j)) & 15u) << 2));
        const float m1 = (float)((by1 >> 6) | (((h1.w >> (4 * j)) & 15u) << 2));
        const float cf0 = fmaf(8.0f * d0, (float)(by0 & 63u), dm0 * m0);
        const float cf1 = fmaf(8.0f * d1, (float)(by1 & 63u), dm1 * m1);
#pragma unroll
        for (int vv = 0; vv < NV; vv++) {
            const float sj = S[(vv * nsb + sb) * 8 + j];
            corr0[vv] = fmaf(cf0, sj, corr0[vv]);
            corr1[vv] = fmaf(cf1, sj, corr1[vv]);
        }
    }
}

template <int NV>
__device__ __forceinline__ void q6k_tile(const TileRegs &T, const uint4 *__restrict__ xs, int sb, int t, int bv,
                                         int bpart, float &acc0, float &acc1)
{
    const float d0 = half_bits(T.r[8].x & 0xFFFF);
    const float d1 = half_bits(T.r[8].x >> 16);
#pragma unroll
    for (int s = 0; s < 16; s++) {
        const int w = s >> 1, u = s >> 2, k0 = (s & 1) ? 2 : 0;
        float c0 = 0.0f, c1 = 0.0f, c2 = 0.0f, c3 = 0.0f;
        uint32_t av[4];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t Lw = (&T.r[3 * h + (w >> 2)].x)[w & 3];
            const uint32_t Hu = (&T.r[3 * h + 2].x)[u];
#pragma unroll
            for (int kk = 0; kk < 2; kk++) {
                const int k = k0 + kk;
                uint32_t hb;
                if ((w & 1) == 0) hb = Hu >> (2 * k);
                else hb = k == 0 ? (Hu << 4) : k == 1 ? (Hu << 2) : k == 2 ? (Hu >> 8) : (Hu >> 10);
                uint32_t q = and_or(hb, 0x00300030u, and_or(Lw >> (4 * k), 0x000F000Fu, 0x64006400u));
                av[kk * 2 + h] = hsub2(q, 0x64206420u);  // - (1024 + 32)
            }
        }
        const uint4 bb = xs[xunit<NV>(sb, t, w, bv, bpart)];
        const uint2 b = (s & 1) ? make_uint2(bb.z, bb.w) : make_uint2(bb.x, bb.y);
        mma_f16(c0, c1, c2, c3, av[0], av[1], av[2], av[3], b.x, b.y);
        const float s0 = d0 * (float)(int8_t)((&T.r[6].x)[s >> 2] >> (8 * (s & 3)));
        const float s1 = d1 * (float)(int8_t)((&T.r[7].x)[s >> 2] >> (8 * (s & 3)));
        acc0 = fmaf(s0, c0 + c1, acc0);
        acc1 = fmaf(s1, c2 + c3, acc1);
    }
}

}  // namespace llmdot
