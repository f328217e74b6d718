// gemm.cu -- quantised matmul for 5..32 input rows: batched decode steps and prompt chunks.
//
// Same contract as the matvec (TensorOps.MatMulFusedQ4_K / Q6_K, src/Llmdot.Core/Tensors/TensorOps.cs:230-395,
// with aRows > 1 from TensorOps.cs:62): y[v][row] = sum_k x[v][k] * W[row][k], fp32 result.
//
// The weights keep the 16-row x 256-weight tile layout of gemv.cu and are still streamed once
// (TMA bulk copies into a 3-slot ring per warp); what changes with many input rows is that
// every dequantised weight fragment now feeds NB tensor-core MMAs (NB = ceil(rows / 4) column
// groups of 8 = 4 input rows x {hi, lo} halves of the fp16 split of x):
//
// * x is turned into B fragments ONCE per input by gemm_prepare (one CTA per input row: RMSNorm
//   statistics, exact power-of-two scale, fp16 hi/lo, in the tile's K order), into global
//   memory laid out per super-block.  Each CTA copies one super-block of fragments at a time
//   into shared memory with a bulk copy (double-buffered), shared by its 8 warps.
// * A CTA owns 8 row tiles (one per warp) and a K range; small matrices split K over CTAs
//   and a second kernel sums the K parts in a fixed order.
// * Q4_K offset term  sum_j (8 d sc_j + dmin m_j) S_j(x)  (S_j = sub-block sums of x) is itself
//   a tiny product: each lane already holds the coefficients of sub-blocks 2t, 2t+1 of rows
//   g, g+8, which is exactly an m16n8k16 A fragment (k = 2t, 2t+1); with the sub-block sums as
//   B fragments (hi/lo split, scaled by powers of two) two MMAs per column group reduce it
//   across the lanes in the tensor core.
#include <vector>

#include "engine.cuh"
#include "gemm.cuh"
#include "gemv.cuh"
#include "gemv_tile.cuh"

namespace llmdot {

namespace {

constexpr int GW = 8;        // warps per CTA, one 16-row tile each
constexpr int GRING = 3;     // weight tiles in flight per warp
constexpr int GSLOT = Q6K_TILE;
constexpr int NB_MAX = 8;    // column groups (4 input rows each)
constexpr float S_FAC = 1.0f / 64.0f;  // sub-block sums (< 2^20) scaled into fp16 range
constexpr float C_FAC = 16.0f;         // correction coefficients scaled up (lo half stays normal)
constexpr unsigned long long GEMM_WAIT_NS = 2000000000ull;

__host__ __device__ inline int gcols(int nb) { return 8 * nb; }
// B-fragment units of one super-block: [t][8 w][C columns] uint4, rows of 8C+2 units so that a
// quarter-warp (t = 0..3, g = 0..1) hits 8 distinct 16-byte bank groups
__host__ __device__ inline int xsb_units(int nb) { return 4 * (8 * gcols(nb) + 2); }
__host__ __device__ inline size_t xsb_bytes(int nb) { return (size_t)xsb_units(nb) * 16; }
// correction B operands of one super-block: [t][C + 8] uint32 (padding: distinct banks)
__host__ __device__ inline int ssb_words(int nb) { return 4 * (gcols(nb) + 8); }
__host__ __device__ inline size_t ssb_bytes(int nb) { return (size_t)ssb_words(nb) * 4; }

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t gtimer()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t *b, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity)
{
    if (mbar_test(b, parity)) return true;
    const uint64_t t0 = gtimer();
    while (!mbar_test(b, parity))
        if (gtimer() - t0 > GEMM_WAIT_NS) return false;
    return true;
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *b)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(b))
                 : "memory");
}

// ------------------------------------------------------------------ input fragments
// One CTA per (padded) input row.  Rows v >= nv get zero fragments.
__global__ void __launch_bounds__(256) gemm_prep_kernel(const float *__restrict__ x, int ldx, int nv, int nsb,
                                                        const float *__restrict__ norm_w, float eps, int lay, int nb,
                                                        uint4 *__restrict__ xf, uint32_t *__restrict__ sf,
                                                        float *__restrict__ isc)
{
    extern __shared__ float P[];  // [nsb][4][8] partial sums of 8 weights (Q4_K layout)
    __shared__ float red[2][8];
    __shared__ float stat[2];
    const int v = blockIdx.x, tid = threadIdx.x, C = gcols(nb), cols = nsb * 256;
    const bool live = v < nv;
    const float *xv = x + (size_t)v * ldx;
    if (live) {
        float ss = 0.0f, mx = 0.0f;
        for (int i = tid; i < cols; i += 256) {
            const float h = xv[i];
            ss = fmaf(h, h, ss);
            mx = fmaxf(mx, fabsf(norm_w ? __fmul_rn(norm_w[i], h) : h));
        }
        ss = warp_sum(ss);
        mx = warp_max(mx);
        if ((tid & 31) == 0) {
            red[0][tid >> 5] = ss;
            red[1][tid >> 5] = mx;
        }
        __syncthreads();
        if (tid == 0) {
            float s = 0.0f, m = 0.0f;
            for (int w = 0; w < 8; w++) {
                s += red[0][w];
                m = fmaxf(m, red[1][w]);
            }
            float iv = 1.0f;
            if (norm_w) {  // VectorMath.RmsNorm: 1 / sqrt(ss/n + eps); x = (w*h)*inv
                iv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)cols), eps)));
                m = __fmul_rn(m, iv);
            }
            float sc = 1.0f;  // exact power of two putting max|x|*sc in [2^14, 2^15)
            if (m > 0.0f && m < INFINITY) {
                int e;
                frexpf(m, &e);
                sc = ldexpf(1.0f, 15 - e);
            }
            stat[0] = iv;
            stat[1] = sc;
            isc[v] = 1.0f / sc;
        }
        __syncthreads();
    } else if (tid == 0) {
        isc[v] = 0.0f;
    }
    const float f = live ? (norm_w ? stat[0] * stat[1] : stat[1]) : 0.0f;
    for (int it = tid; it < nsb * 32; it += 256) {
        const int w = it & 7, tt = (it >> 3) & 3, sb = it >> 5;
        // Q4_K: 8 consecutive weights 64t+8w.. in slot order {0,4,1,5,2,6,3,7};
        // Q6_K: 4 at 32w+4t.. and 4 at 32w+16+4t.. in order
        const int e0 = lay == 0 ? sb * 256 + 64 * tt + 8 * w : sb * 256 + 32 * w + 4 * tt;
        const int e1 = lay == 0 ? e0 + 4 : e0 + 16;
        float c[8];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            c[k] = 0.0f;
            c[4 + k] = 0.0f;
            if (live) {
                if (norm_w) {  // ((w*h)*inv)*sc == (w*h)*(inv*sc): sc is a power of two
                    c[k] = __fmul_rn(__fmul_rn(norm_w[e0 + k], xv[e0 + k]), f);
                    c[4 + k] = __fmul_rn(__fmul_rn(norm_w[e1 + k], xv[e1 + k]), f);
                } else {
                    c[k] = xv[e0 + k] * f;
                    c[4 + k] = xv[e1 + k] * f;
                }
            }
        }
        if (lay == 0) {
            float psum = 0.0f;
#pragma unroll
            for (int k = 0; k < 8; k++) psum += c[k];
            P[(sb * 4 + tt) * 8 + w] = psum;
        }
        float o[8];
#pragma unroll
        for (int k = 0; k < 8; k++) o[k] = lay == 0 ? c[(k >> 1) + 4 * (k & 1)] : c[k];
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            __half2 hh = __floats2half2_rn(o[2 * k], o[2 * k + 1]);
            float2 hf = __half22float2(hh);
            hi[k] = *reinterpret_cast<uint32_t *>(&hh);
            lo[k] = pack_half2(o[2 * k] - hf.x, o[2 * k + 1] - hf.y);
        }
        uint4 *u = xf + (size_t)sb * xsb_units(nb) + tt * (8 * C + 2) + w * C;
        u[2 * v] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        u[2 * v + 1] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    if (lay == 0) {
        __syncthreads();
        // B operand of the offset product: column (v, hi|lo) holds (S_2t, S_2t+1) for lane t
        for (int it = tid; it < nsb * 4; it += 256) {
            const int sb = it >> 2, t = it & 3;
            const float *pp = P + (sb * 4 + t) * 8;
            const float s0 = (((pp[0] + pp[1]) + pp[2]) + pp[3]) * S_FAC;
            const float s1 = (((pp[4] + pp[5]) + pp[6]) + pp[7]) * S_FAC;
            const __half2 h = __floats2half2_rn(s0, s1);
            const float2 hf = __half22float2(h);
            uint32_t *q = sf + (size_t)sb * ssb_words(nb) + t * (C + 8);
            q[2 * v] = *reinterpret_cast<const uint32_t *>(&h);
            q[2 * v + 1] = pack_half2(s0 - hf.x, s1 - hf.y);
        }
    }
}

// ------------------------------------------------------------------ tile math, NB column groups
template <int NB>
__device__ __forceinline__ void q4k_tile_nb(const TileRegs &T, const uint4 *__restrict__ xs,
                                            const uint32_t *__restrict__ ss, int t, int g, float (&acc)[NB][2],
                                            float (&cc)[NB][4])
{
    constexpr int C = 8 * NB;
    float d_r[2];
    uint32_t sc2[2][2], nsc2[2][2], sc16[2][2], nsc16[2][2], ahi[2], alo[2];
    const uint32_t sh = (24u * (uint32_t)t) & 31u;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint4 hd = T.r[4 + h];
        d_r[h] = half_bits(hd.x & 0xFFFF);
        const float dm = half_bits(hd.x >> 16);
        const uint32_t lo = t < 2 ? hd.y : (t == 2 ? hd.z : hd.w), hi = t < 2 ? hd.z : hd.w;
        const uint32_t pr = __funnelshift_r(lo, hi, sh);
        const uint32_t scA = pr & 63u, mA = (pr >> 6) & 63u, scB = (pr >> 12) & 63u, mB = (pr >> 18) & 63u;
        const uint32_t sA = hsub2(0x64006400u | (scA * 0x10001u), 0x64006400u);
        const uint32_t sB = hsub2(0x64006400u | (scB * 0x10001u), 0x64006400u);
        sc2[h][0] = sA;
        sc2[h][1] = sB;
        nsc2[h][0] = hfma2(sA, 0xE400E400u, 0u);
        nsc2[h][1] = hfma2(sB, 0xE400E400u, 0u);
        sc16[h][0] = hfma2(sA, 0x2C002C00u, 0u);
        sc16[h][1] = hfma2(sB, 0x2C002C00u, 0u);
        nsc16[h][0] = hfma2(sA, 0xD400D400u, 0u);
        nsc16[h][1] = hfma2(sB, 0xD400D400u, 0u);
        // offset coefficients of sub-blocks 2t, 2t+1 as an A fragment (k = 2t, 2t+1), hi/lo
        const float c0 = fmaf(8.0f * d_r[h], (float)scA, dm * (float)mA) * C_FAC;
        const float c1 = fmaf(8.0f * d_r[h], (float)scB, dm * (float)mB) * C_FAC;
        const __half2 ch = __floats2half2_rn(c0, c1);
        const float2 cf = __half22float2(ch);
        ahi[h] = *reinterpret_cast<const uint32_t *>(&ch);
        alo[h] = pack_half2(c0 - cf.x, c1 - cf.y);
    }
    float c[NB][4];
#pragma unroll
    for (int j = 0; j < NB; j++) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const int jj = w >> 2;  // sub-block 2t + jj
        const uint32_t W0 = (&T.r[jj].x)[w & 3], W1 = (&T.r[2 + jj].x)[w & 3];
        const uint32_t a0 = hfma2(and_or(W0, 0x000F000Fu, 0x64006400u), sc2[0][jj], nsc2[0][jj]);
        const uint32_t a1 = hfma2(and_or(W1, 0x000F000Fu, 0x64006400u), sc2[1][jj], nsc2[1][jj]);
        const uint32_t a2 = hfma2(and_or(W0, 0x00F000F0u, 0x64006400u), sc16[0][jj], nsc16[0][jj]);
        const uint32_t a3 = hfma2(and_or(W1, 0x00F000F0u, 0x64006400u), sc16[1][jj], nsc16[1][jj]);
        const uint32_t V0 = W0 >> 8, V1 = W1 >> 8;
        const uint32_t a4 = hfma2(and_or(V0, 0x000F000Fu, 0x64006400u), sc2[0][jj], nsc2[0][jj]);
        const uint32_t a5 = hfma2(and_or(V1, 0x000F000Fu, 0x64006400u), sc2[1][jj], nsc2[1][jj]);
        const uint32_t a6 = hfma2(and_or(V0, 0x00F000F0u, 0x64006400u), sc16[0][jj], nsc16[0][jj]);
        const uint32_t a7 = hfma2(and_or(V1, 0x00F000F0u, 0x64006400u), sc16[1][jj], nsc16[1][jj]);
#pragma unroll
        for (int j = 0; j < NB; j++) {
            const uint4 b = xs[t * (8 * C + 2) + w * C + 8 * j + g];
            mma_f16(c[j][0], c[j][1], c[j][2], c[j][3], a0, a1, a2, a3, b.x, b.y);
            mma_f16(c[j][0], c[j][1], c[j][2], c[j][3], a4, a5, a6, a7, b.z, b.w);
        }
    }
#pragma unroll
    for (int j = 0; j < NB; j++) {
        acc[j][0] = fmaf(d_r[0], c[j][0] + c[j][1], acc[j][0]);
        acc[j][1] = fmaf(d_r[1], c[j][2] + c[j][3], acc[j][1]);
        const uint32_t sb = ss[t * (C + 8) + 8 * j + g];
        mma_f16(cc[j][0], cc[j][1], cc[j][2], cc[j][3], ahi[0], ahi[1], 0u, 0u, sb, 0u);
        mma_f16(cc[j][0], cc[j][1], cc[j][2], cc[j][3], alo[0], alo[1], 0u, 0u, sb, 0u);
    }
}

template <int NB>
__device__ __forceinline__ void q6k_tile_nb(const TileRegs &T, const uint4 *__restrict__ xs, int t, int g,
                                            float (&acc)[NB][2])
{
    constexpr int C = 8 * NB;
    const float d0 = half_bits(T.r[8].x & 0xFFFF);
    const float d1 = half_bits(T.r[8].x >> 16);
#pragma unroll
    for (int s = 0; s < 16; s++) {
        const int w = s >> 1, u = s >> 2, k0 = (s & 1) ? 2 : 0;
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
                const uint32_t q = and_or(hb, 0x00300030u, and_or(Lw >> (4 * k), 0x000F000Fu, 0x64006400u));
                av[kk * 2 + h] = hsub2(q, 0x64206420u);  // - (1024 + 32)
            }
        }
        const float s0 = d0 * (float)(int8_t)((&T.r[6].x)[s >> 2] >> (8 * (s & 3)));
        const float s1 = d1 * (float)(int8_t)((&T.r[7].x)[s >> 2] >> (8 * (s & 3)));
#pragma unroll
        for (int j = 0; j < NB; j++) {
            const uint4 bb = xs[t * (8 * C + 2) + w * C + 8 * j + g];
            const uint32_t b0 = (s & 1) ? bb.z : bb.x, b1 = (s & 1) ? bb.w : bb.y;
            float c0 = 0.0f, c1 = 0.0f, c2 = 0.0f, c3 = 0.0f;
            mma_f16(c0, c1, c2, c3, av[0], av[1], av[2], av[3], b0, b1);
            acc[j][0] = fmaf(s0, c0 + c1, acc[j][0]);
            acc[j][1] = fmaf(s1, c2 + c3, acc[j][1]);
        }
    }
}

// ------------------------------------------------------------------ the batched kernel
struct GemmArgs {
    const uint8_t *w;  // tiled weights
    int qt, rows, nrt, nsb, ksplit, nv, nvpad;
    const uint4 *xf;
    const uint32_t *sf;
    const float *isc;
    float *y;
    int ldy, mode;
    float *part;  // [ksplit][nvpad][rows] when ksplit > 1
    int *err;
};

__host__ __device__ inline size_t gemm_smem(int nb)
{
    return 256 + 2 * (xsb_bytes(nb) + ssb_bytes(nb)) + (size_t)GW * GRING * GSLOT;
}

template <int NB>
__global__ void __launch_bounds__(GW * 32, 1) gemm_q_kernel(const __grid_constant__ GemmArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int rtb = blockIdx.x / a.ksplit, kp = blockIdx.x % a.ksplit;
    const int rt = rtb * GW + warp;
    const bool active = rt < a.nrt;
    const int sb0 = kp * a.nsb / a.ksplit, sb1 = (kp + 1) * a.nsb / a.ksplit, n = sb1 - sb0;
    const bool q4 = a.qt == QT_Q4K;
    uint64_t *mb = (uint64_t *)smem;  // [GW][GRING] weight slots, then 2 fragment buffers
    uint64_t *xbar = mb + GW * GRING;
    const size_t XB = xsb_bytes(NB) + ssb_bytes(NB);
    uint8_t *xb = smem + 256;
    uint8_t *ring = xb + 2 * XB + (size_t)warp * GRING * GSLOT;
    uint64_t *mb_w = mb + warp * GRING;
    if (tid < GW * GRING + 2) mbar_init(mb + tid, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    const uint32_t xbytes = (uint32_t)(xsb_bytes(NB) + (q4 ? ssb_bytes(NB) : 0));
    auto issue_x = [&](int i) {  // fragments of the CTA's i-th super-block into buffer i & 1
        if (i >= n) return;
        const int buf = i & 1;
        mbar_expect_tx(xbar + buf, xbytes);
        bulk_load(xb + buf * XB, a.xf + (size_t)(sb0 + i) * xsb_units(NB), (uint32_t)xsb_bytes(NB), xbar + buf);
        if (q4)
            bulk_load(xb + buf * XB + xsb_bytes(NB), a.sf + (size_t)(sb0 + i) * ssb_words(NB), (uint32_t)ssb_bytes(NB),
                      xbar + buf);
    };
    if (tid == 0) {
        issue_x(0);
        issue_x(1);
    }
    const uint32_t tb = q4 ? Q4K_TILE : Q6K_TILE;
    const uint8_t *wsrc = a.w + ((size_t)rt * a.nsb + sb0) * tb;
    if (active && lane == 0)
        for (int r = 0; r < GRING && r < n; r++) {
            mbar_expect_tx(mb_w + r, tb);
            bulk_load(ring + (size_t)r * GSLOT, wsrc + (size_t)r * tb, tb, mb_w + r);
        }
    float acc[NB][2], cc[NB][4];
#pragma unroll
    for (int j = 0; j < NB; j++) {
        acc[j][0] = acc[j][1] = 0.0f;
        cc[j][0] = cc[j][1] = cc[j][2] = cc[j][3] = 0.0f;
    }
    bool ok = true;
    int w_issued = active ? min(GRING, n) : 0, w_done = 0, x_issued = min(2, n), x_done = 0;
    for (int i = 0; i < n; i++) {
        const int buf = i & 1;
        const bool xok = __all_sync(0xffffffffu, mbar_wait(xbar + buf, (uint32_t)(i >> 1) & 1u));
        if (xok) x_done = i + 1;
        else ok = false;
        if (active && xok) {
            const int slot = i % GRING;
            if (!__all_sync(0xffffffffu, mbar_wait(mb_w + slot, (uint32_t)(i / GRING) & 1u))) {
                ok = false;
            } else {
                w_done = i + 1;
                TileRegs T;
                read_tile(T, ring + (size_t)slot * GSLOT, a.qt, lane);
                __syncwarp();  // the tile is in registers: refill its slot before the math
                if (i + GRING < n) {
                    if (lane == 0) {
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        mbar_expect_tx(mb_w + slot, tb);
                        bulk_load(ring + (size_t)slot * GSLOT, wsrc + (size_t)(i + GRING) * tb, tb, mb_w + slot);
                    }
                    w_issued = i + 1 + GRING;
                }
                const uint4 *xs = (const uint4 *)(xb + buf * XB);
                if (q4) q4k_tile_nb<NB>(T, xs, (const uint32_t *)(xb + buf * XB + xsb_bytes(NB)), t, g, acc, cc);
                else q6k_tile_nb<NB>(T, xs, t, g, acc);
            }
        }
        if (!__syncthreads_and(ok)) {  // every warp is done with fragment buffer `buf`, or one gave up
            if (tid == 0) atomicExch(a.err, 4);
            // bounded drain of the copies still in flight into this CTA's shared memory
            for (int k = w_done; k < w_issued; k++) mbar_wait(mb_w + k % GRING, (uint32_t)(k / GRING) & 1u);
            if (tid == 0)
                for (int k = x_done; k < x_issued; k++) mbar_wait(xbar + (k & 1), (uint32_t)(k >> 1) & 1u);
            return;
        }
        if (tid == 0 && i + 2 < n) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_x(i + 2);
            x_issued = i + 3;
        }
    }
    if (!active) return;
#pragma unroll
    for (int j = 0; j < NB; j++) {
        const int v = 4 * j + t;
        if (v >= a.nv) continue;
        float o0 = acc[j][0], o1 = acc[j][1];
        if (q4) {  // minus the offset product (scaled by C_FAC * S_FAC)
            o0 -= (cc[j][0] + cc[j][1]) * (1.0f / (C_FAC * S_FAC));
            o1 -= (cc[j][2] + cc[j][3]) * (1.0f / (C_FAC * S_FAC));
        }
        const float s = a.isc[v];
        o0 *= s;
        o1 *= s;
        const int r0 = rt * 16 + g, r1 = r0 + 8;
        if (a.ksplit == 1) {
            float *yv = a.y + (size_t)v * a.ldy;
            if (r0 < a.rows) yv[r0] = a.mode == GEMV_ADD ? __fadd_rn(yv[r0], o0) : o0;
            if (r1 < a.rows) yv[r1] = a.mode == GEMV_ADD ? __fadd_rn(yv[r1], o1) : o1;
        } else {
            float *pv = a.part + ((size_t)kp * a.nvpad + v) * a.rows;
            if (r0 < a.rows) pv[r0] = o0;
            if (r1 < a.rows) pv[r1] = o1;
        }
    }
}

// K parts summed in a fixed order, then the epilogue.
__global__ void gemm_reduce_kernel(const float *__restrict__ part, int ksplit, int nvpad, int nv, int rows, float *y,
                                   int ldy, int mode)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nv * rows) return;
    const int v = i / rows, r = i % rows;
    float s = 0.0f;
    for (int k = 0; k < ksplit; k++) s += part[((size_t)k * nvpad + v) * rows + r];
    float *yp = y + (size_t)v * ldy + r;
    *yp = mode == GEMV_ADD ? __fadd_rn(*yp, s) : s;
}

int nb_for(int nv) { return nv <= 8 ? 2 : (nv <= 16 ? 4 : 8); }

}  // namespace

int gemm_scratch_alloc(GemmScratch &s, int cols_max, int rows_max, std::vector<void *> &allocs)
{
    const int nsb = (cols_max + 255) / 256;
    const size_t xbytes = (size_t)nsb * xsb_bytes(NB_MAX), sbytes = (size_t)nsb * ssb_bytes(NB_MAX);
    auto get = [&](void **p, size_t bytes) -> int {
        if (cudaMalloc(p, bytes) != cudaSuccess) {
            cudaGetLastError();
            return fail(LLMDOT_E_NOMEM, "batched matmul scratch allocation failed");
        }
        allocs.push_back(*p);
        return LLMDOT_OK;
    };
    LLMDOT_TRY(get(&s.xf[0], xbytes));
    LLMDOT_TRY(get(&s.xf[1], xbytes));
    LLMDOT_TRY(get(&s.sf, 2 * sbytes));
    LLMDOT_TRY(get((void **)&s.isc[0], sizeof(float) * 2 * 4 * NB_MAX));
    s.isc[1] = s.isc[0] + 4 * NB_MAX;
    s.part_floats = (size_t)16 * 4 * NB_MAX * rows_max;
    LLMDOT_TRY(get((void **)&s.part, sizeof(float) * s.part_floats));
    s.cols_max = cols_max;
    s.rows_max = rows_max;
    return LLMDOT_OK;
}

bool gemm_supported(const DevMat &W, int nv)
{
    return W.tiled && (W.type == T_Q4_K || W.type == T_Q6_K) && W.cols % 256 == 0 && nv >= 1 && nv <= GEMM_MAX_ROWS;
}

int gemm_prepare(const float *x, int ldx, int nv, int cols, const float *norm_w, float eps, uint32_t qtype, int slot,
                 GemmScratch &s, GemmInput *out, cudaStream_t st)
{
    if (nv < 1 || nv > GEMM_MAX_ROWS || cols % 256 || cols > s.cols_max || slot < 0 || slot > 1)
        return fail(LLMDOT_E_INVALID, "batched matmul: bad input shape");
    const int nb = nb_for(nv), nsb = cols / 256, lay = qtype == T_Q4_K ? 0 : 1;
    uint32_t *sf = (uint32_t *)s.sf + (size_t)slot * nsb * ssb_words(NB_MAX);
    gemm_prep_kernel<<<4 * nb, 256, sizeof(float) * nsb * 32, st>>>(x, ldx, nv, nsb, norm_w, eps, lay, nb,
                                                                    (uint4 *)s.xf[slot], sf, s.isc[slot]);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    out->xf = s.xf[slot];
    out->sf = sf;
    out->isc = s.isc[slot];
    out->nv = nv;
    out->nsb = nsb;
    out->layout = lay;
    return LLMDOT_OK;
}

template <int NB> static int launch_nb(const GemmArgs &a, int grid, cudaStream_t st)
{
    static std::atomic<unsigned long long> attr_done{0};
    LLMDOT_CUDA_TRY(smem_attr_once(attr_done, gemm_q_kernel<NB>, (int)gemm_smem(NB)));
    gemm_q_kernel<NB><<<grid, GW * 32, gemm_smem(NB), st>>>(a);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

int launch_gemm(const DevMat &W, const GemmInput &in, float *y, int ldy, int mode, GemmScratch &s, int *err,
                cudaStream_t st)
{
    if (!gemm_supported(W, in.nv) || W.cols != in.nsb * 256 || (mode != GEMV_STORE && mode != GEMV_ADD))
        return fail(LLMDOT_E_UNSUPPORTED, "batched matmul: unsupported matrix");
    if ((W.type == T_Q4_K) != (in.layout == 0)) return fail(LLMDOT_E_INVALID, "batched matmul: fragment layout mismatch");
    const int nb = nb_for(in.nv);
    GemmArgs a{};
    a.w = W.tiled;
    a.qt = W.type == T_Q4_K ? QT_Q4K : QT_Q6K;
    a.rows = W.rows;
    a.nrt = (W.rows + 15) / 16;
    a.nsb = in.nsb;
    a.nv = in.nv;
    a.nvpad = 4 * nb;
    a.xf = (const uint4 *)in.xf;
    a.sf = (const uint32_t *)in.sf;
    a.isc = in.isc;
    a.y = y;
    a.ldy = ldy;
    a.mode = mode;
    a.err = err;
    const int blocks = (a.nrt + GW - 1) / GW;
    // split K until the grid covers the SMs (one CTA per SM fits the shared memory)
    int ks = 1;
    while (blocks * ks < 148 && ks * 2 <= a.nsb && ks * 2 <= 16 &&
           (size_t)(ks * 2) * a.nvpad * a.rows <= s.part_floats)
        ks *= 2;
    a.ksplit = ks;
    a.part = s.part;
    const int grid = blocks * ks;
    if (nb == 2) LLMDOT_TRY(launch_nb<2>(a, grid, st));
    else if (nb == 4) LLMDOT_TRY(launch_nb<4>(a, grid, st));
    else LLMDOT_TRY(launch_nb<8>(a, grid, st));
    if (ks > 1) {
        const int n = in.nv * a.rows;
        gemm_reduce_kernel<<<(n + 255) / 256, 256, 0, st>>>(s.part, ks, a.nvpad, in.nv, a.rows, y, ldy, mode);
        LLMDOT_CUDA_TRY(cudaGetLastError());
    }
    return LLMDOT_OK;
}

}  // namespace llmdot
