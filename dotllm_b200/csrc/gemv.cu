// gemv.cu -- tensor-core quantised matvec for decode (1..4 input rows).
//
// Replaces TensorOps.MatMulFusedQ4_K / MatMulFusedQ6_K (src/Llmdot.Core/Tensors/TensorOps.cs:230-395)
// on the device.  The matvec is HBM-bound, so the design goal is to stream every weight byte
// exactly once with fully coalesced 128-bit loads and to spend as few issue slots per weight
// as possible turning it into tensor-core operands:
//
// * Layout.  At model load every Q4_K / Q6_K matrix is re-laid out (same byte count) into
//   tiles of 16 rows x one 256-weight super-block.  Inside a tile, the bytes lane L of a warp
//   needs are one 16-byte slot of each 512-byte "plane", so each plane is one fully coalesced
//   warp load; the per-row headers (d, dmin, scales) sit behind the planes.
// * Math.  mma.sync m16n8k16 (fp16 in, fp32 accumulate).  The weights enter as exact small
//   integers in fp16, built from nibbles with one LOP3 (magic 0x6400 = 1024.0) and one packed
//   HFMA2/HSUB2.  The activation x is split into x_hi + x_lo (two fp16 columns of the MMA) after
//   an exact power-of-two scaling, so each product is exact and the sum is fp32: the result
//   agrees with the reference's fp32 dot to fp32 rounding, not to fp16 precision.
//     Q4_K: A = q*sc (<= 945, exact), one MMA chain per super-block, then
//           y += d*C - sum_j (8*d*sc_j + dmin*m_j) * S_j   with S_j the sub-block sums of x;
//     Q6_K: A = q-32 (exact), one MMA per 16-weight sub-block, y += (d*sc_s) * C_s.
// * One launch covers up to three matrices that read the same input (Q, K, V), each with its
//   own type, and an optional RMSNorm of the input in the prologue (ApplyNorm,
//   InferenceEngine.cs:544-562).  Epilogues: store, residual add (Add, :189/:195), or
//   silu/gelu(gate)*up for the FFN (FfnForward :466-474, both matrices in one launch).
// * Programmatic dependent launch: each warp fetches its first weight tile before waiting for
//   the previous kernel, so weight streaming overlaps the predecessor's tail.
#include <string.h>

#include "gemv.cuh"
#include "gemv_tile.cuh"
#include "ops.cuh"

namespace llmdot {

enum { GM_STORE = GEMV_STORE, GM_ADD = GEMV_ADD, GM_SILU_MUL = GEMV_SILU_MUL, GM_GELU_MUL = GEMV_GELU_MUL };

// ------------------------------------------------------------------ repack kernels
// Q4_K tile (16 rows x 1 super-block), lane L = 4g + t owns rows g, g+8 and sub-blocks 2t, 2t+1:
//   plane p (0..3) at p*512 + L*16: nibble bytes of sub-block 2t + (p&1) of row (p < 2 ? g : g+8)
//   header at 2048 + g*32: bytes 0..15 of row g's block, then of row g+8's block
__global__ void repack_q4k_kernel(const uint8_t *__restrict__ raw, uint8_t *__restrict__ tiled, int rows, int nsb,
                                  uint64_t rbytes, int ntiles)
{
    int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= ntiles * 32) return;
    int tile = idx >> 5, L = idx & 31, g = L >> 2, t = L & 3;
    int rt = tile / nsb, sb = tile % nsb;
    uint8_t *dst = tiled + (uint64_t)tile * Q4K_TILE;
    for (int p = 0; p < 4; p++) {
        int row = rt * 16 + (p < 2 ? g : g + 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (row < rows) v = *(const uint4 *)(raw + (uint64_t)row * rbytes + (uint64_t)sb * 144 + 16 + 16 * (2 * t + (p & 1)));
        *(uint4 *)(dst + p * 512 + L * 16) = v;
    }
    if (t == 0)
        for (int h = 0; h < 2; h++) {
            int row = rt * 16 + g + 8 * h;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (row < rows) v = *(const uint4 *)(raw + (uint64_t)row * rbytes + (uint64_t)sb * 144);
            *(uint4 *)(dst + 2048 + g * 32 + h * 16) = v;
        }
}

// Q4_K tile in the int8 tensor-core lane order (gemv_tile.cuh, q4k_tile_i8): same bytes, nibbles
// re-paired per lane and the 6-bit (sc, m) pairs re-packed so that sc_j is a byte.
__global__ void repack_q4k_i8_kernel(const uint8_t *__restrict__ raw, uint8_t *__restrict__ tiled, int rows, int nsb,
                                     uint64_t rbytes, int ntiles)
{
    int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= ntiles * 32) return;
    int tile = idx >> 5, L = idx & 31, g = L >> 2, t = L & 3;
    int rt = tile / nsb, sb = tile % nsb;
    uint8_t *dst = tiled + (uint64_t)tile * Q4K_TILE;
    for (int p = 0; p < 4; p++) {
        uint32_t w[4];
        for (int q = 0; q < 4; q++) {  // A row g, A row g+8, B row g, B row g+8
            const int row = rt * 16 + g + 8 * (q & 1), half = (q >> 1) * 16;
            uint32_t word = 0;
            if (row < rows) {
                const uint8_t *qs = raw + (uint64_t)row * rbytes + (uint64_t)sb * 144 + 16;
                for (int b = 0; b < 4; b++) {
                    // element e of the super-block is nibble (e & 1) of byte e / 2
                    const int e0 = 32 * (2 * p) + half + 4 * t + b, e1 = e0 + 32;  // sub-blocks 2p and 2p+1
                    const uint32_t lo = (qs[e0 >> 1] >> ((e0 & 1) * 4)) & 15u, hi = (qs[e1 >> 1] >> ((e1 & 1) * 4)) & 15u;
                    word |= (lo | (hi << 4)) << (8 * b);
                }
            }
            w[q] = word;
        }
        *(uint4 *)(dst + p * 512 + L * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    if (t == 0)
        for (int h = 0; h < 2; h++) {
            const int row = rt * 16 + g + 8 * h;
            uint8_t hd[16] = {0};
            if (row < rows) {
                const uint8_t *blk = raw + (uint64_t)row * rbytes + (uint64_t)sb * 144;
                for (int i = 0; i < 4; i++) hd[i] = blk[i];  // d, dmin
                uint32_t mhi = 0;
                for (int j = 0; j < 8; j++) {
                    auto f6 = [&](int bit) {  // 6 bits of the little-endian bit stream at blk + 4
                        const int bi = bit >> 3, sh = bit & 7;
                        const uint32_t v = blk[4 + bi] | (bi + 1 < 12 ? (uint32_t)blk[5 + bi] << 8 : 0u);
                        return (v >> sh) & 63u;
                    };
                    const uint32_t sc = f6(12 * j), m = f6(12 * j + 6);
                    hd[4 + j] = (uint8_t)(sc | ((m & 3u) << 6));
                    mhi |= (m >> 2) << (4 * j);
                }
                memcpy(hd + 12, &mhi, 4);
            }
            uint4 v;
            memcpy(&v, hd, 16);
            *(uint4 *)(dst + 2048 + g * 32 + h * 16) = v;
        }
}

// Q6_K element (sub-block s, lane t, i) = super-block element 16s + 4t + i.  Per lane and row:
//   L_w (w = 0..7): nibbles of sub-blocks 2w (bits 0-3 i0, 16-19 i1, 4-7 i2, 20-23 i3) and
//                   2w+1 (bits 8-11 i0, 24-27 i1, 12-15 i2, 28-31 i3);
//   H_u (u = 0..3): 2-bit highs of L_{2u} pair k at bits 4+2k / 20+2k, of L_{2u+1} pair k at
//                   {0,2,12,14}[k] / {16,18,28,30}[k]  (pair k = (s odd ? 2 : 0) + (i >= 2)).
//   planes 0,1 = L_0..3, L_4..7 of row g; plane 2 = H_0..3 of row g; planes 3..5 the same for row g+8;
//   sc at 3072 + g*32 (16 int8 of row g, then row g+8); d at 3328 + g*4 (row g, row g+8).
__device__ __forceinline__ int q6_value(const uint8_t *blk, int e)
{
    int n = e >> 7, rr = e & 127, tt = rr >> 5, l = rr & 31;
    int lo = (tt & 1) ? blk[n * 64 + l + 32] : blk[n * 64 + l];
    lo = (tt & 2) ? (lo >> 4) : (lo & 0xF);
    int hi = (blk[128 + n * 32 + l] >> (2 * tt)) & 3;
    return lo | (hi << 4);
}

__global__ void repack_q6k_kernel(const uint8_t *__restrict__ raw, uint8_t *__restrict__ tiled, int rows, int nsb,
                                  uint64_t rbytes, int ntiles)
{
    int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= ntiles * 32) return;
    int tile = idx >> 5, L = idx & 31, g = L >> 2, t = L & 3;
    int rt = tile / nsb, sb = tile % nsb;
    uint8_t *dst = tiled + (uint64_t)tile * Q6K_TILE;
    for (int h = 0; h < 2; h++) {
        int row = rt * 16 + g + 8 * h;
        uint32_t Lw[8] = {0, 0, 0, 0, 0, 0, 0, 0}, Hu[4] = {0, 0, 0, 0};
        if (row < rows) {
            const uint8_t *blk = raw + (uint64_t)row * rbytes + (uint64_t)sb * 210;
            for (int s = 0; s < 16; s++)
                for (int i = 0; i < 4; i++) {
                    int q = q6_value(blk, 16 * s + 4 * t + i);
                    int w = s >> 1, odd = s & 1, k = (odd ? 2 : 0) + (i >> 1), high = i & 1;
                    int lobit = 4 * k + (high ? 16 : 0);
                    Lw[w] |= (uint32_t)(q & 0xF) << lobit;
                    int hb;
                    if ((w & 1) == 0) hb = 4 + 2 * k + (high ? 16 : 0);
                    else {
                        const int pl[4] = {0, 2, 12, 14};
                        hb = pl[k] + (high ? 16 : 0);
                    }
                    Hu[w >> 1] |= (uint32_t)((q >> 4) & 3) << hb;
                }
        }
        *(uint4 *)(dst + (3 * h) * 512 + L * 16) = make_uint4(Lw[0], Lw[1], Lw[2], Lw[3]);
        *(uint4 *)(dst + (3 * h + 1) * 512 + L * 16) = make_uint4(Lw[4], Lw[5], Lw[6], Lw[7]);
        *(uint4 *)(dst + (3 * h + 2) * 512 + L * 16) = make_uint4(Hu[0], Hu[1], Hu[2], Hu[3]);
        if (t == 0) {
            uint8_t *scd = dst + 3072 + g * 32 + h * 16;
            uint8_t *dd = dst + 3328 + g * 4 + h * 2;
            if (row < rows) {
                const uint8_t *blk = raw + (uint64_t)row * rbytes + (uint64_t)sb * 210;
                for (int s = 0; s < 16; s++) scd[s] = blk[192 + s];
                dd[0] = blk[208];
                dd[1] = blk[209];
            } else {
                for (int s = 0; s < 16; s++) scd[s] = 0;
                dd[0] = dd[1] = 0;
            }
        }
    }
}

int prepare_tiled(llmdot_model *m, DevMat &W)
{
    if (W.type != T_Q4_K && W.type != T_Q6_K) return LLMDOT_OK;
    if (W.cols % 256 != 0) return LLMDOT_OK;
    const int nsb = W.cols / 256, nrt = (W.rows + 15) / 16, ntiles = nsb * nrt;
    const size_t tb = W.type == T_Q4_K ? Q4K_TILE : Q6K_TILE;
    cudaError_t e = cudaMalloc(&W.tiled, tb * (size_t)ntiles);
    if (e != cudaSuccess) {
        cudaGetLastError();
        W.tiled = nullptr;
        return fail(LLMDOT_E_NOMEM, "tiled weight allocation failed");
    }
    m->allocs.push_back(W.tiled);
    int threads = ntiles * 32;
    if (W.type == T_Q4_K)
        repack_q4k_kernel<<<(threads + 255) / 256, 256, 0, m->stream>>>(W.raw, W.tiled, W.rows, nsb, W.rbytes, ntiles);
    else
        repack_q6k_kernel<<<(threads + 255) / 256, 256, 0, m->stream>>>(W.raw, W.tiled, W.rows, nsb, W.rbytes, ntiles);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    if (W.type == T_Q4_K && W.rows >= GEMV_I8_MIN_ROWS) {  // the copy the 1..2-vector matvec streams
        e = cudaMalloc(&W.tiled8, tb * (size_t)ntiles);
        if (e != cudaSuccess) {
            cudaGetLastError();
            W.tiled8 = nullptr;
            return fail(LLMDOT_E_NOMEM, "tiled weight allocation failed");
        }
        m->allocs.push_back(W.tiled8);
        repack_q4k_i8_kernel<<<(threads + 255) / 256, 256, 0, m->stream>>>(W.raw, W.tiled8, W.rows, nsb, W.rbytes,
                                                                            ntiles);
        LLMDOT_CUDA_TRY(cudaGetLastError());
    }
    return LLMDOT_OK;
}

// ------------------------------------------------------------------ the matvec kernel
struct GemvSeg {
    const uint8_t *w;   // tiled weights
    const uint8_t *w1;  // second ("up") matrix of the *_MUL epilogues (segment 0 only)
    float *y;           // [nv][ldy]
    int rows, nrt, qt, ldy;
};

struct GemvArgs {
    GemvSeg seg[3];
    int nseg, rt_total, nsb;
    const float *x;  // [nv][ldx]
    int ldx;
    const float *norm_w;  // fused RMSNorm weight (nullable)
    float eps;
    int need_q4, need_q6;  // x layouts the segments use
    int lks;               // log2 of the K split: each row tile is 2^lks units of consecutive super-blocks
    int i8;                // Q4_K segments are int8-order tiles (1..2 vectors)
    GemvPrefetch pf;       // weights of the next operation, pulled into L2 while this one runs
};

// Tiles in flight per warp: each warp streams its tiles through a private ring of RING (2 or 3)
// shared-memory slots.  Lane 0 fetches a whole tile with one TMA bulk copy (cp.async.bulk, tiles
// are contiguous) completing on the slot's mbarrier; the refill of a slot is issued as soon as
// the warp has consumed it, so RING tiles are always on their way.  Every wait is bounded.
constexpr unsigned long long GEMV_WAIT_NS = 2000000000ull;
__device__ int g_gemv_timeout;  // set when a bounded wait gave up (read by gemv_timeout_check)

__device__ __forceinline__ uint32_t gsm_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t g_timer()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void gmbar_init(uint64_t *b)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(gsm_u32(b)) : "memory");
}
__device__ __forceinline__ bool gmbar_test(uint64_t *b, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(gsm_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait for the fill with the given parity; the answer is uniform across the warp
__device__ __forceinline__ bool gmbar_wait(uint64_t *b, uint32_t parity)
{
    bool ok = gmbar_test(b, parity);
    if (!ok) {
        const uint64_t t0 = g_timer();
        while (!(ok = gmbar_test(b, parity)))
            if (g_timer() - t0 > GEMV_WAIT_NS) break;
    }
    return __all_sync(0xffffffffu, ok);
}
// lane 0: one bulk copy of a tile into a ring slot
__device__ __forceinline__ void issue_bulk(uint8_t *slot, const uint8_t *src, uint32_t bytes, uint64_t *b)
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(gsm_u32(b)), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     gsm_u32(slot)),
                 "l"(src), "r"(bytes), "r"(gsm_u32(b))
                 : "memory");
}

__device__ __forceinline__ int find_seg(const GemvArgs &a, int gt, int &rt)
{
    int s = 0;
    rt = gt;
    while (s + 1 < a.nseg && rt >= a.seg[s].nrt) {
        rt -= a.seg[s].nrt;
        s++;
    }
    return s;
}

#ifndef LLMDOT_GEMV_WARPS
#define LLMDOT_GEMV_WARPS 16
#endif
constexpr int GEMV_WARPS = LLMDOT_GEMV_WARPS;  // warps per CTA (one CTA per SM)

// This CTA's share of the next operation's weights into L2 (bulk prefetch, no data returned):
// consecutive matvec launches are latency-bound, so while one runs the next one's tiles move
// from HBM to L2 and its streaming starts from L2.
__device__ __forceinline__ void l2_prefetch_share(const GemvPrefetch &pf)
{
#pragma unroll
    for (int r = 0; r < GEMV_PREFETCH_MAX; r++) {
        const unsigned long long n = pf.n[r];
        if (!pf.p[r] || n == 0) continue;
        const unsigned long long share = (n / gridDim.x + 15) & ~15ull, lo = (unsigned long long)blockIdx.x * share;
        if (lo >= n) continue;
        unsigned long long len = n - lo < share ? n - lo : share;
        const uint8_t *src = (const uint8_t *)pf.p[r] + lo;
        while (len > 0) {
            const uint32_t piece = len > (1u << 20) ? (1u << 20) : (uint32_t)len;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(piece) : "memory");
            src += piece;
            len -= piece;
        }
    }
}

// Shared memory of one CTA (byte offsets; all 16-byte aligned).
struct GemvSmem {
    int xs4, xs6, S, P, xi, red, stat, wred, ring, total, slot;  // byte offsets (slot: bytes per ring slot)
};
__host__ __device__ inline GemvSmem gemv_layout(int nv, int nsb, int nmat, bool q4, bool q6, int max_rt_cta,
                                                int ks, int ring)
{
    GemvSmem L;
    const int xsz = nsb * 64 * nv * 16;
    int o = GEMV_WARPS * 3 * 8;  // slot mbarriers [GEMV_WARPS][3]
    L.xs4 = o;
    o += q4 ? xsz : 0;
    L.xs6 = o;
    o += q6 ? xsz : 0;
    L.S = o;
    o += q4 ? nv * nsb * 8 * 4 : 0;
    L.P = o;
    o += q4 ? nv * nsb * 32 * 4 : 0;
    L.xi = o;  // int8 form (nv <= 2): per (vector, super-block) max |x| bits, then 2^k, and 2^-k
    o += q4 && nv <= 2 ? (2 * nv * nsb * 4 + 15) / 16 * 16 : 0;
    L.red = o;  // unit partials [max_rt_cta][ks][nmat][16][nv]
    o += (max_rt_cta * ks * nmat * 16 * nv * 4 + 15) / 16 * 16;
    L.stat = o;
    o += 16 * ((2 * nv * 4 + 15) / 16);
    L.wred = o;
    o += (GEMV_WARPS * 2 * nv * 4 + 15) / 16 * 16;
    L.slot = q6 ? Q6K_TILE : Q4K_TILE;
    L.ring = o;
    o += GEMV_WARPS * ring * L.slot;
    L.total = o;
    return L;
}

// Where a unit's tiles are: unit u of a CTA is K part (u mod ks) of its row tile (u / ks);
// its tiles run over matrix 0 then matrix 1 (the *_MUL epilogues), super-blocks [sb_lo, sb_hi).
struct UnitPos {
    const uint8_t *p0, *p1;  // first tile of the unit in matrix 0 / 1
    int tb, qt, rtl, kp, sb_lo, n;  // tile bytes, type, local row tile, K part, first super-block, tiles per matrix
};
template <int NMAT>
__device__ __forceinline__ void unit_pos(const GemvArgs &a, int rt_lo, int u, UnitPos &P)
{
    const int ks1 = (1 << a.lks) - 1;
    P.rtl = u >> a.lks;
    P.kp = u & ks1;
    P.sb_lo = (P.kp * a.nsb) >> a.lks;
    P.n = (((P.kp + 1) * a.nsb) >> a.lks) - P.sb_lo;
    int rt;
    const GemvSeg &sg = a.seg[find_seg(a, rt_lo + P.rtl, rt)];
    P.qt = sg.qt;
    P.tb = sg.qt == QT_Q4K ? Q4K_TILE : Q6K_TILE;
    const size_t off = ((size_t)rt * a.nsb + P.sb_lo) * P.tb;
    P.p0 = sg.w + off;
    P.p1 = NMAT == 2 ? sg.w1 + off : nullptr;
}

// TM: 0 every segment Q4_K, 1 every segment Q6_K, 2 mixed (the type is read per unit).
// I8 (1..2 vectors): Q4_K segments run the int8 tensor-core form on the int8-order tile copy.
template <int NV, int MODE, int RING, int TM, bool I8>
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_mma_kernel(GemvArgs a, int max_rt_cta)
{
    constexpr int NMAT = (MODE >= GM_SILU_MUL) ? 2 : 1;
    constexpr int NT = GEMV_WARPS * 32;
    static_assert(!I8 || NV <= 2, "int8 form: at most two vectors (4 digit columns each)");
    extern __shared__ __align__(16) uint8_t smem[];
    const int nsb = a.nsb, cols = nsb * 256, ks = 1 << a.lks;
    const GemvSmem L = gemv_layout(NV, nsb, NMAT, a.need_q4, a.need_q6, max_rt_cta, ks, RING);
    uint4 *xs4 = (uint4 *)(smem + L.xs4), *xs6 = (uint4 *)(smem + L.xs6);
    float *S = (float *)(smem + L.S), *P = (float *)(smem + L.P), *red = (float *)(smem + L.red);
    float *stat = (float *)(smem + L.stat), *wred = (float *)(smem + L.wred);
    float *xsc = (float *)(smem + L.xi), *xinv = xsc + NV * nsb;  // [NV][nsb] each (int8 form)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    uint8_t *ring = smem + L.ring + (size_t)warp * RING * L.slot;
    uint64_t *mb = (uint64_t *)smem + warp * 3;  // this warp's slot mbarriers
    // this CTA owns row tiles [rt_lo, rt_hi) of the concatenated segments, i.e. units
    // [0, nrt * ks); warp w takes units w, w + 16, ...
    const int rt_lo = (int)((long long)blockIdx.x * a.rt_total / gridDim.x);
    const int rt_hi = (int)((long long)(blockIdx.x + 1) * a.rt_total / gridDim.x);
    const int nrt = rt_hi - rt_lo, nunit = nrt * ks;
    // issue cursor: unit iu, tile ij of it; i_n tiles issued so far
    // tiles go through the ring in order, so the slot of a warp's k-th tile is k mod RING: both
    // loops below walk the slots with compile-time indices (ring slot bytes = L.slot)
    constexpr int SLOTB = TM == QT_Q4K ? Q4K_TILE : Q6K_TILE;
    int iu = warp, ij = 0, i_n = 0;
    UnitPos IP;
    if (iu < nunit) unit_pos<NMAT>(a, rt_lo, iu, IP);
    auto issue = [&](int slot) {  // the warp's next tile into ring slot `slot`
        if (iu >= nunit) return;
        if (lane == 0) {
            const int mat = (NMAT == 2 && ij >= IP.n) ? 1 : 0;
            issue_bulk(ring + slot * SLOTB, (mat ? IP.p1 : IP.p0) + (size_t)(ij - mat * IP.n) * IP.tb, IP.tb,
                       mb + slot);
        }
        i_n++;
        if (++ij == NMAT * IP.n) {
            ij = 0;
            iu += GEMV_WARPS;
            if (iu < nunit) unit_pos<NMAT>(a, rt_lo, iu, IP);
        }
    };
    if (tid < GEMV_WARPS * 3) gmbar_init((uint64_t *)smem + tid);
    if (I8 && a.need_q4)
        for (int i = tid; i < NV * nsb; i += NT) xsc[i] = 0.0f;  // per super-block max |x| (as uint bits)
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    // weights are constant: start streaming before waiting for the previous kernel
#pragma unroll
    for (int f = 0; f < RING; f++) issue(f);
    if (tid == 0) l2_prefetch_share(a.pf);
    pdl_launch();
    pdl_wait();

    // ---- prologue.  Short form (no int8 layout, 1/2/4 vectors, at most two fragment items per
    // thread): each thread loads the x (and norm weight) elements of its fragment items once, the
    // statistics need one barrier (every thread then derives the scales itself), and the offset
    // term's sub-block sums come from the four partials' lanes by shuffles, in the same order as
    // the general form below.
    const int nlay = (a.need_q4 ? 1 : 0) + (a.need_q6 ? 1 : 0), per_lay = nsb * 32 * NV;
    const bool short_pro = !I8 && (NV == 1 || NV == 2 || NV == 4) && nlay * per_lay <= 2 * NT;
    if (short_pro) {
        constexpr int IPT = 2;
        const int ss_lay = a.need_q4 ? 0 : 1;  // the layout whose items cover x once
        float c[IPT][8], nw[IPT][8];
        int lay_of[IPT], it_of[IPT];
#pragma unroll
        for (int k = 0; k < IPT; k++) {
            const int gi = tid + k * NT;
            lay_of[k] = -1;
            it_of[k] = 0;
            if (gi < nlay * per_lay) {
                const int lay = nlay == 2 ? (gi >= per_lay ? 1 : 0) : ss_lay, it = gi >= per_lay ? gi - per_lay : gi;
                lay_of[k] = lay;
                it_of[k] = it;
                const int v = it % NV, r = it / NV, w = r & 7, tt = (r >> 3) & 3, sb = r >> 5;
                const int e0 = lay == 0 ? sb * 256 + 64 * tt + 8 * w : sb * 256 + 32 * w + 4 * tt;
                const int e1 = lay == 0 ? e0 + 4 : e0 + 16;
                const float *h = a.x + (size_t)v * a.ldx;
                const float4 p0 = *(const float4 *)(h + e0), p1 = *(const float4 *)(h + e1);
                c[k][0] = p0.x, c[k][1] = p0.y, c[k][2] = p0.z, c[k][3] = p0.w;
                c[k][4] = p1.x, c[k][5] = p1.y, c[k][6] = p1.z, c[k][7] = p1.w;
                if (a.norm_w) {
                    const float4 n0 = *(const float4 *)(a.norm_w + e0), n1 = *(const float4 *)(a.norm_w + e1);
                    nw[k][0] = n0.x, nw[k][1] = n0.y, nw[k][2] = n0.z, nw[k][3] = n0.w;
                    nw[k][4] = n1.x, nw[k][5] = n1.y, nw[k][6] = n1.z, nw[k][7] = n1.w;
                }
            }
        }
        float ss[NV], mx[NV];
#pragma unroll
        for (int v = 0; v < NV; v++) ss[v] = mx[v] = 0.0f;
#pragma unroll
        for (int k = 0; k < IPT; k++) {
            if (lay_of[k] != ss_lay) continue;
            const int v = it_of[k] % NV;
#pragma unroll
            for (int vv = 0; vv < NV; vv++) {
                if (vv != v) continue;
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    ss[vv] = fmaf(c[k][q], c[k][q], ss[vv]);
                    mx[vv] = fmaxf(mx[vv], fabsf(a.norm_w ? __fmul_rn(nw[k][q], c[k][q]) : c[k][q]));
                }
            }
        }
#pragma unroll
        for (int v = 0; v < NV; v++) {
            ss[v] = warp_sum(ss[v]);
            mx[v] = warp_max(mx[v]);
        }
        if (lane == 0)
#pragma unroll
            for (int v = 0; v < NV; v++) {
                wred[warp * 2 * NV + v] = ss[v];
                wred[warp * 2 * NV + NV + v] = mx[v];
            }
        __syncthreads();
        float f_of[NV], sc_of[NV];
#pragma unroll
        for (int v = 0; v < NV; v++) {
            float s2 = 0.0f, m = 0.0f;
            for (int w = 0; w < GEMV_WARPS; w++) {
                s2 += wred[w * 2 * NV + v];
                m = fmaxf(m, wred[w * 2 * NV + NV + v]);
            }
            float inv = 1.0f;
            if (a.norm_w) {  // VectorMath.RmsNorm: 1 / sqrt(ss/n + eps); x = (w*h)*inv
                inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s2, (float)cols), a.eps)));
                m = __fmul_rn(m, inv);
            }
            float sc = 1.0f;  // exact power of two putting max|x|*sc in [2^14, 2^15)
            if (m > 0.0f && m < INFINITY) {
                int e;
                frexpf(m, &e);
                sc = ldexpf(1.0f, 15 - e);
            }
            sc_of[v] = sc;
            f_of[v] = a.norm_w ? inv * sc : sc;  // ((w*h)*inv)*sc == (w*h)*(inv*sc): sc is a power of two
            if (tid == 0) {
                stat[v] = inv;
                stat[NV + v] = sc;
            }
        }
#pragma unroll
        for (int k = 0; k < IPT; k++) {
            if (lay_of[k] < 0) continue;  // warp-uniform: a layout's items fill whole warps
            const int lay = lay_of[k], it = it_of[k];
            const int v = it % NV, r = it / NV, w = r & 7, tt = (r >> 3) & 3, sb = r >> 5;
            float f = 1.0f, scv = 1.0f;
#pragma unroll
            for (int vv = 0; vv < NV; vv++)
                if (vv == v) {
                    f = f_of[vv];
                    scv = sc_of[vv];
                }
            float cc[8];
#pragma unroll
            for (int q = 0; q < 8; q++) cc[q] = a.norm_w ? __fmul_rn(__fmul_rn(nw[k][q], c[k][q]), f) : c[k][q] * scv;
            if (lay == 0) {
                float psum = 0.0f;
#pragma unroll
                for (int q = 0; q < 8; q++) psum += cc[q];
                // S_j: the partials of w = 4 (j & 1) .. + 3 sit NV lanes apart in this warp
                const float p1 = __shfl_down_sync(0xffffffffu, psum, NV), p2 = __shfl_down_sync(0xffffffffu, psum, 2 * NV),
                            p3 = __shfl_down_sync(0xffffffffu, psum, 3 * NV);
                if ((w & 3) == 0) S[(v * nsb + sb) * 8 + 2 * tt + (w >> 2)] = ((psum + p1) + p2) + p3;
            }
            float o[8];
#pragma unroll
            for (int q = 0; q < 8; q++) o[q] = lay == 0 ? cc[(q >> 1) + 4 * (q & 1)] : cc[q];
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                __half2 hh = __floats2half2_rn(o[2 * q], o[2 * q + 1]);
                float2 hf = __half22float2(hh);
                hi[q] = *reinterpret_cast<uint32_t *>(&hh);
                lo[q] = pack_half2(o[2 * q] - hf.x, o[2 * q + 1] - hf.y);
            }
            uint4 *xs = lay == 0 ? xs4 : xs6;
            xs[xunit<NV>(sb, tt, w, v, 0)] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            xs[xunit<NV>(sb, tt, w, v, 1)] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
    } else {
        // ---- prologue pass A: sum of squares (norm) and max |x| per vector, all threads
        {
            float ss[NV], mx[NV];
    #pragma unroll
            for (int v = 0; v < NV; v++) ss[v] = mx[v] = 0.0f;
            for (int i = tid; i < cols; i += NT) {
                const float wn = a.norm_w ? a.norm_w[i] : 1.0f;
    #pragma unroll
                for (int v = 0; v < NV; v++) {
                    const float h = a.x[(size_t)v * a.ldx + i];
                    ss[v] = fmaf(h, h, ss[v]);
                    const float ax = fabsf(a.norm_w ? __fmul_rn(wn, h) : h);
                    mx[v] = fmaxf(mx[v], ax);
                    if (I8 && a.need_q4) {  // the warp's 32 consecutive elements share a super-block
                        const float wm = warp_max(ax);
                        if (lane == 0) atomicMax((unsigned *)xsc + v * nsb + (i >> 8), __float_as_uint(wm));
                    }
                }
            }
    #pragma unroll
            for (int v = 0; v < NV; v++) {
                ss[v] = warp_sum(ss[v]);
                mx[v] = warp_max(mx[v]);
            }
            if (lane == 0)
    #pragma unroll
                for (int v = 0; v < NV; v++) {
                    wred[warp * 2 * NV + v] = ss[v];
                    wred[warp * 2 * NV + NV + v] = mx[v];
                }
            __syncthreads();
            if (tid < NV) {
                float s = 0.0f, m = 0.0f;
                for (int w = 0; w < GEMV_WARPS; w++) {
                    s += wred[w * 2 * NV + tid];
                    m = fmaxf(m, wred[w * 2 * NV + NV + tid]);
                }
                float inv = 1.0f;
                if (a.norm_w) {  // VectorMath.RmsNorm: 1 / sqrt(ss/n + eps); x = (w*h)*inv
                    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)cols), a.eps)));
                    m = __fmul_rn(m, inv);  // rounding is monotone: max of the products
                }
                float sc = 1.0f;  // exact power of two putting max|x|*sc in [2^14, 2^15)
                if (m > 0.0f && m < INFINITY) {
                    int e;
                    frexpf(m, &e);
                    sc = ldexpf(1.0f, 15 - e);
                }
                stat[tid] = inv;
                stat[NV + tid] = sc;
            }
            __syncthreads();
            if (I8 && a.need_q4)  // X = x * 2^k with the super-block's max |x| * 2^k in [2^29, 2^30)
                for (int i = tid; i < NV * nsb; i += NT) {
                    float m = __uint_as_float(((const unsigned *)xsc)[i]);
                    if (a.norm_w) m = __fmul_rn(m, stat[i / nsb]);
                    int e = 0;
                    if (m > 0.0f && m < INFINITY) frexpf(m, &e);
                    e = max(e, -90);
                    xsc[i] = ldexpf(1.0f, 30 - e);
                    xinv[i] = ldexpf(1.0f, e - 30);
                }
        }
        // ---- pass B: fp16 hi/lo fragments of the scaled x for the layouts in use
        if (I8 && a.need_q4) {
            __syncthreads();
            // int8 form: item (v, sb, j, t) = elements 32j + 4t + b and 32j + 16 + 4t + b (b = 0..3) of
            // super-block sb, as four signed digits of X (one 8-byte unit per digit); P gets the sum
            // of the 8 normed values for the sub-block sums S
            uint2 *xs8 = (uint2 *)xs4;
            for (int it = tid; it < NV * nsb * 32; it += NT) {
                const int tt = it & 3, j = (it >> 2) & 7, sb = (it >> 5) % nsb, v = it / (nsb * 32);
                const int e0 = sb * 256 + 32 * j + 4 * tt;
                const float *h = a.x + (size_t)v * a.ldx;
                const float4 p0 = *(const float4 *)(h + e0), p1 = *(const float4 *)(h + e0 + 16);
                float c[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
                if (a.norm_w) {
                    const float inv = stat[v];
                    const float4 n0 = *(const float4 *)(a.norm_w + e0), n1 = *(const float4 *)(a.norm_w + e0 + 16);
                    const float nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
    #pragma unroll
                    for (int k = 0; k < 8; k++) c[k] = __fmul_rn(__fmul_rn(nw[k], c[k]), inv);
                }
                float psum = 0.0f;
    #pragma unroll
                for (int k = 0; k < 8; k++) psum += c[k];
                P[((v * nsb + sb) * 4 + (j >> 1)) * 8 + 4 * (j & 1) + tt] = psum;
                const float scale = xsc[v * nsb + sb];
                uint32_t dg[4][2] = {{0, 0}, {0, 0}, {0, 0}, {0, 0}};
    #pragma unroll
                for (int k = 0; k < 8; k++) {
                    int X = __float2int_rn(c[k] * scale);
    #pragma unroll
                    for (int dd = 0; dd < 4; dd++) {  // balanced base-256 digits
                        const int dgt = dd < 3 ? (int)(int8_t)(X & 0xFF) : X;
                        X = (X - dgt) >> 8;
                        dg[dd][k >> 2] |= ((uint32_t)dgt & 0xFFu) << (8 * (k & 3));
                    }
                }
    #pragma unroll
                for (int dd = 0; dd < 4; dd++) xs8[x8unit<NV>(sb, j, tt, 4 * v + dd)] = make_uint2(dg[dd][0], dg[dd][1]);
            }
        }
        for (int lay = 0; lay < 2; lay++) {
            if ((lay == 0 && (I8 || !a.need_q4)) || (lay == 1 && !a.need_q6)) continue;
            uint4 *xs = lay == 0 ? xs4 : xs6;
            for (int it = tid; it < nsb * 32 * NV; it += NT) {
                const int v = it % NV, r = it / NV, w = r & 7, tt = (r >> 3) & 3, sb = r >> 5;
                // Q4_K: 8 consecutive weights 64t+8w.. in slot order {0,4,1,5,2,6,3,7};
                // Q6_K: 4 at 32w+4t.. and 4 at 32w+16+4t.. in order
                const int e0 = lay == 0 ? sb * 256 + 64 * tt + 8 * w : sb * 256 + 32 * w + 4 * tt;
                const int e1 = lay == 0 ? e0 + 4 : e0 + 16;
                const float *h = a.x + (size_t)v * a.ldx;
                float4 p0 = *(const float4 *)(h + e0), p1 = *(const float4 *)(h + e1);
                float c[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
                const float sc = stat[NV + v];
                if (a.norm_w) {
                    // ((w*h)*inv)*sc == (w*h)*(inv*sc): sc is a power of two
                    const float f = stat[v] * sc;
                    const float4 n0 = *(const float4 *)(a.norm_w + e0), n1 = *(const float4 *)(a.norm_w + e1);
                    const float nw[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
    #pragma unroll
                    for (int k = 0; k < 8; k++) c[k] = __fmul_rn(__fmul_rn(nw[k], c[k]), f);
                } else {
    #pragma unroll
                    for (int k = 0; k < 8; k++) c[k] *= sc;
                }
                if (lay == 0) {
                    float psum = 0.0f;
    #pragma unroll
                    for (int k = 0; k < 8; k++) psum += c[k];
                    P[((v * nsb + sb) * 4 + tt) * 8 + w] = psum;
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
                xs[xunit<NV>(sb, tt, w, v, 0)] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                xs[xunit<NV>(sb, tt, w, v, 1)] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
        }
        if (a.need_q4) {
            __syncthreads();
            // pass C: sub-block sums S_j = sum of its four 8-weight partials, fixed order
            for (int it = tid; it < NV * nsb * 8; it += NT) {
                const int v = it / (nsb * 8), jj = it % (nsb * 8), sb = jj >> 3, j = jj & 7;
                const float *pp = P + ((v * nsb + sb) * 4 + (j >> 1)) * 8 + 4 * (j & 1);
                S[it] = ((pp[0] + pp[1]) + pp[2]) + pp[3];
            }
        }
    }
    __syncthreads();

    // ---- streaming loop: no CTA-wide barrier inside, warps run independently.  A warp sums a
    // whole (unit, matrix) in registers and stores it once; nothing else is written per tile.
    const int bv = min(g >> 1, NV - 1), bpart = g & 1;  // this lane's B column (vector, part)
    int cu = warp, cj = 0, c_n = 0, s_fail = 0;
    uint32_t cpar = 0;
    UnitPos CP;
    if (cu < nunit) unit_pos<NMAT>(a, rt_lo, cu, CP);
    float acc0 = 0.0f, acc1 = 0.0f;  // rows g, g+8 for vector t (MMA columns 2t, 2t+1)
    float accf[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // int8 form: rows g, g+8 x this lane's two digit columns
    float corr0[NV], corr1[NV];
#pragma unroll
    for (int v = 0; v < NV; v++) corr0[v] = corr1[v] = 0.0f;
    bool ok = true;
    while (ok && cu < nunit) {
#pragma unroll
      for (int slot = 0; slot < RING; slot++) {  // one lap of the ring per iteration
        if (cu >= nunit) break;
        if (!gmbar_wait(mb + slot, cpar)) {
            ok = false;
            s_fail = slot;
            if (lane == 0) atomicExch(&g_gemv_timeout, 1);
            break;
        }
        const int qt = TM == 2 ? CP.qt : TM;
        TileRegs T;
        read_tile(T, ring + slot * SLOTB, qt, lane);
        __syncwarp();  // the tile is in registers: refill its slot before the math
        c_n++;
        issue(slot);
        const int mat = (NMAT == 2 && cj >= CP.n) ? 1 : 0;
        const int sb = CP.sb_lo + cj - mat * CP.n;
        if (TM != 1 && qt == QT_Q4K) {
            if (I8) q4k_tile_i8<NV>(T, (const uint2 *)xs4, S, xinv, nsb, sb, g, t, accf, corr0, corr1);
            else q4k_tile<NV>(T, xs4, S, nsb, sb, t, bv, bpart, acc0, acc1, corr0, corr1);
        }
        if (TM != 0 && qt == QT_Q6K) q6k_tile<NV>(T, xs6, sb, t, bv, bpart, acc0, acc1);
        ++cj;
        if (I8 && TM != 1 && qt == QT_Q4K && (cj == CP.n || cj == NMAT * CP.n)) {
            // int8 form: weight this lane's digit columns (2t, 2t+1 -> digits 2(t&1), 2(t&1)+1 of
            // vector t/2), add the partner lane's two digits, subtract the offset term
            const float w0 = (t & 1) ? 65536.0f : 1.0f, w1 = (t & 1) ? 16777216.0f : 256.0f;
            float r0 = fmaf(accf[1], w1, accf[0] * w0), r1 = fmaf(accf[3], w1, accf[2] * w0);
            r0 += __shfl_xor_sync(0xffffffffu, r0, 1);
            r1 += __shfl_xor_sync(0xffffffffu, r1, 1);
            float k0 = 0.0f, k1 = 0.0f;
#pragma unroll
            for (int v = 0; v < NV; v++) {
                float c0v = corr0[v], c1v = corr1[v];
                c0v += __shfl_xor_sync(0xffffffffu, c0v, 1);
                c0v += __shfl_xor_sync(0xffffffffu, c0v, 2);
                c1v += __shfl_xor_sync(0xffffffffu, c1v, 1);
                c1v += __shfl_xor_sync(0xffffffffu, c1v, 2);
                if (v == (t >> 1)) {
                    k0 = c0v;
                    k1 = c1v;
                }
                corr0[v] = corr1[v] = 0.0f;
            }
            if ((t & 1) == 0 && (t >> 1) < NV) {
                float *rp = red + ((size_t)((CP.rtl * ks + CP.kp) * NMAT + mat) * 16) * NV;
                rp[g * NV + (t >> 1)] = r0 - k0;
                rp[(g + 8) * NV + (t >> 1)] = r1 - k1;
            }
            accf[0] = accf[1] = accf[2] = accf[3] = 0.0f;
            if (cj == NMAT * CP.n) {
                cj = 0;
                cu += GEMV_WARPS;
                if (cu < nunit) unit_pos<NMAT>(a, rt_lo, cu, CP);
            }
        } else if (cj == CP.n || cj == NMAT * CP.n) {  // end of this (unit, matrix): one store of its partial
            if (TM != 1 && qt == QT_Q4K) {
                // offset term: each lane of a row group covered 2 sub-blocks; sum over the group
                float k0 = 0.0f, k1 = 0.0f;
#pragma unroll
                for (int v = 0; v < NV; v++) {
                    float c0v = corr0[v], c1v = corr1[v];
                    c0v += __shfl_xor_sync(0xffffffffu, c0v, 1);
                    c0v += __shfl_xor_sync(0xffffffffu, c0v, 2);
                    c1v += __shfl_xor_sync(0xffffffffu, c1v, 1);
                    c1v += __shfl_xor_sync(0xffffffffu, c1v, 2);
                    if (v == t) {
                        k0 = c0v;
                        k1 = c1v;
                    }
                    corr0[v] = corr1[v] = 0.0f;
                }
                acc0 -= k0;
                acc1 -= k1;
            }
            if (t < NV) {
                float *rp = red + ((size_t)((CP.rtl * ks + CP.kp) * NMAT + mat) * 16) * NV;
                rp[g * NV + t] = acc0;
                rp[(g + 8) * NV + t] = acc1;
            }
            acc0 = acc1 = 0.0f;
            if (cj == NMAT * CP.n) {
                cj = 0;
                cu += GEMV_WARPS;
                if (cu < nunit) unit_pos<NMAT>(a, rt_lo, cu, CP);
            }
        }
      }
        if (ok) cpar ^= 1u;  // the next lap waits for the slots' next phases
    }
    if (!ok) {  // bounded drain of this warp's copies still in flight, then leave the output untouched
        int ds = s_fail;
        for (int k = c_n; k < i_n; k++) {
            gmbar_wait(mb + ds, cpar);
            if (++ds == RING) {
                ds = 0;
                cpar ^= 1u;
            }
        }
    }
    if (!__syncthreads_and(ok)) return;

    // ---- epilogue: every (row tile, row, vector) of the CTA, K parts summed in a fixed order
    for (int it = tid; it < nrt * 16 * NV; it += NT) {
        const int rtl = it / (16 * NV), rr = (it / NV) % 16, v = it % NV;
        int rt;
        const GemvSeg &sg = a.seg[find_seg(a, rt_lo + rtl, rt)];
        const int row = rt * 16 + rr;
        if (row >= sg.rows) continue;
        float o[NMAT];
#pragma unroll
        for (int mtx = 0; mtx < NMAT; mtx++) {
            float s = 0.0f;
            for (int kp = 0; kp < ks; kp++) s += red[(((rtl * ks + kp) * NMAT + mtx) * 16 + rr) * NV + v];
            o[mtx] = (I8 && sg.qt == QT_Q4K) ? s : s * (1.0f / stat[NV + v]);  // int8 form is in x's units
        }
        float *yp = sg.y + (size_t)v * sg.ldy + row;
        if (MODE == GM_STORE) *yp = o[0];
        else if (MODE == GM_ADD) *yp = __fadd_rn(*yp, o[0]);
        else {
            const bool vl = row < sg.rows - sg.rows % 8;
            const float act = MODE == GM_SILU_MUL ? silu_ref(o[0], vl) : gelu_ref(o[0], vl);
            *yp = __fmul_rn(act, o[NMAT - 1]);
        }
    }
}

constexpr int GEMV_SMEM_MAX = 220 * 1024;

// Shared memory needed for `nv` rows through matrices with nsb super-blocks (worst case over the
// row-tile blocking, K split 2^lks); 0 when it does not fit even with a 2-deep ring.
static size_t gemv_need(int nv, int nsb, int nmat, bool q4, bool q6, int max_rt, int lks, int *ring)
{
    for (int r = 3; r >= 2; r--) {
        const GemvSmem L = gemv_layout(nv, nsb, nmat, q4, q6, max_rt, 1 << lks, r);
        if (L.total <= GEMV_SMEM_MAX) {
            if (ring) *ring = r;
            return (size_t)L.total;
        }
    }
    return 0;
}

int gemv_timeout_check()
{
    int v = 0;
    LLMDOT_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_gemv_timeout, sizeof(int)));
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_gemv_timeout, &zero, sizeof(int));
        return fail(LLMDOT_E_TIMEOUT, "matvec: a weight tile wait timed out");
    }
    return LLMDOT_OK;
}

bool gemv_fast_supported(const DevMat &W, int nv)
{
    if (!W.tiled || nv < 1 || nv > 4) return false;
    const bool q4 = W.type == T_Q4_K;
    return gemv_need(nv, W.cols / 256, 2, q4, !q4, 4, 0, nullptr) != 0;
}

template <int NV, int MODE, int RING, int TM, bool I8>
static int launch_r(const GemvArgs &a, int grid, int max_rt, size_t sm, bool pdl, cudaStream_t st)
{
    auto kern = gemv_mma_kernel<NV, MODE, RING, TM, I8>;
    static std::atomic<unsigned long long> attr_done{0};  // per instantiation, per device
    LLMDOT_CUDA_TRY(smem_attr_once(attr_done, kern, GEMV_SMEM_MAX));
    LLMDOT_CUDA_TRY(launch_kernel(pdl, kern, dim3(grid), dim3(GEMV_WARPS * 32), sm, st, a, max_rt));
    return LLMDOT_OK;
}

template <int NV, int MODE, int RING, bool I8>
static int launch_tm(const GemvArgs &a, int grid, int max_rt, size_t sm, bool pdl, cudaStream_t st)
{
    if (a.need_q4 && a.need_q6) return launch_r<NV, MODE, RING, 2, I8>(a, grid, max_rt, sm, pdl, st);
    if (a.need_q6) return launch_r<NV, MODE, RING, QT_Q6K, false>(a, grid, max_rt, sm, pdl, st);
    return launch_r<NV, MODE, RING, QT_Q4K, I8>(a, grid, max_rt, sm, pdl, st);
}
template <int NV, int MODE, int RING>
static int launch_i8(const GemvArgs &a, int grid, int max_rt, size_t sm, bool pdl, cudaStream_t st)
{
    if constexpr (NV <= 2)
        if (a.i8) return launch_tm<NV, MODE, RING, true>(a, grid, max_rt, sm, pdl, st);
    return launch_tm<NV, MODE, RING, false>(a, grid, max_rt, sm, pdl, st);
}

template <int NV, int MODE> static int launch_t(GemvArgs a, bool pdl, cudaStream_t st)
{
    constexpr int NMAT = (MODE >= GM_SILU_MUL) ? 2 : 1;
    // one CTA per SM (148 on B200), each with a contiguous block of row tiles; more CTAs only
    // when the per-unit partial sums would not fit in shared memory
    int grid = a.rt_total < 148 ? a.rt_total : 148;
    int max_rt = (a.rt_total + grid - 1) / grid, ring = 0;
    // K split: enough units per CTA (about 6 per warp) that warps finish together, but at least
    // one super-block per unit
    const int min_rt = a.rt_total / grid;
    int lks = 0;
    while ((2 << lks) <= a.nsb && (min_rt << lks) < 6 * GEMV_WARPS) lks++;
    size_t sm = gemv_need(NV, a.nsb, NMAT, a.need_q4, a.need_q6, max_rt, lks, &ring);
    while (sm == 0 && lks > 0) sm = gemv_need(NV, a.nsb, NMAT, a.need_q4, a.need_q6, max_rt, --lks, &ring);
    while (sm == 0 && grid < a.rt_total) {
        grid += 148;
        if (grid > a.rt_total) grid = a.rt_total;
        max_rt = (a.rt_total + grid - 1) / grid;
        sm = gemv_need(NV, a.nsb, NMAT, a.need_q4, a.need_q6, max_rt, lks, &ring);
    }
    if (sm == 0) return fail(LLMDOT_E_UNSUPPORTED, "fast matvec: shared memory");
    a.lks = lks;
    if (ring == 3) return launch_i8<NV, MODE, 3>(a, grid, max_rt, sm, pdl, st);
    return launch_i8<NV, MODE, 2>(a, grid, max_rt, sm, pdl, st);
}

template <int MODE> static int launch_mode(const GemvArgs &a, int nv, bool pdl, cudaStream_t st)
{
    switch (nv) {
    case 1: return launch_t<1, MODE>(a, pdl, st);
    case 2: return launch_t<2, MODE>(a, pdl, st);
    case 3: return launch_t<3, MODE>(a, pdl, st);
    default: return launch_t<4, MODE>(a, pdl, st);
    }
}

int launch_gemv_multi(const GemvTarget *tg, int ntarget, const float *norm_w, float eps, const float *x, int ldx,
                      int nv, int mode, bool pdl, cudaStream_t st, const GemvPrefetch *pf)
{
    if (ntarget < 1 || ntarget > 3 || (mode >= GEMV_SILU_MUL && ntarget != 1))
        return fail(LLMDOT_E_INVALID, "fast matvec: bad target list");
    GemvArgs a = {};
    if (pf) {
        for (int r = 0; r < GEMV_PREFETCH_MAX; r++)  // bulk prefetches want 16-byte aligned, 16-byte multiples
            if (((uintptr_t)pf->p[r] & 15) || (pf->n[r] & 15)) return fail(LLMDOT_E_INVALID, "fast matvec: prefetch range");
        a.pf = *pf;
    }
    a.nseg = ntarget;
    a.nsb = tg[0].W->cols / 256;
    a.x = x;
    a.ldx = ldx;
    a.norm_w = norm_w;
    a.eps = eps;
    for (int i = 0; i < ntarget; i++) {
        const DevMat &W = *tg[i].W;
        if (!gemv_fast_supported(W, nv) || W.cols != tg[0].W->cols)
            return fail(LLMDOT_E_UNSUPPORTED, "fast matvec: unsupported matrix");
        if (tg[i].W1 && (tg[i].W1->type != W.type || tg[i].W1->rows != W.rows || tg[i].W1->cols != W.cols ||
                         !tg[i].W1->tiled))
            return fail(LLMDOT_E_UNSUPPORTED, "fast matvec: gate/up matrices differ");
        GemvSeg &s = a.seg[i];
        s.w = W.tiled;
        s.w1 = tg[i].W1 ? tg[i].W1->tiled : nullptr;
        s.y = tg[i].y;
        s.ldy = tg[i].ldy;
        s.rows = W.rows;
        s.nrt = (W.rows + 15) / 16;
        s.qt = W.type == T_Q4_K ? QT_Q4K : QT_Q6K;
        a.rt_total += s.nrt;
        a.need_q4 |= s.qt == QT_Q4K;
        a.need_q6 |= s.qt == QT_Q6K;
    }
    // the int8 form when every Q4_K segment has its int8-order copy (the large logits matrices)
    bool i8 = nv <= 2 && a.need_q4;
    for (int i = 0; i < ntarget; i++)
        if (tg[i].W->type == T_Q4_K) i8 = i8 && tg[i].W->tiled8 && (!tg[i].W1 || tg[i].W1->tiled8);
    if (i8) {
        a.i8 = 1;
        for (int i = 0; i < ntarget; i++)
            if (tg[i].W->type == T_Q4_K) {
                a.seg[i].w = tg[i].W->tiled8;
                if (tg[i].W1) a.seg[i].w1 = tg[i].W1->tiled8;
            }
    }
    switch (mode) {
    case GM_STORE: return launch_mode<GM_STORE>(a, nv, pdl, st);
    case GM_ADD: return launch_mode<GM_ADD>(a, nv, pdl, st);
    case GM_SILU_MUL: return launch_mode<GM_SILU_MUL>(a, nv, pdl, st);
    default: return launch_mode<GM_GELU_MUL>(a, nv, pdl, st);
    }
}

int launch_gemv_fast_ex(const DevMat &W0, const DevMat *W1, const float *norm_w, float eps, const float *x, int ldx,
                        int nv, float *y, int ldy, int mode, cudaStream_t st, bool pdl, const GemvPrefetch *pf)
{
    GemvTarget tg = {&W0, W1, y, ldy};
    return launch_gemv_multi(&tg, 1, norm_w, eps, x, ldx, nv, mode, pdl, st, pf);
}

int launch_gemv_fast(const DevMat &W, const float *x, int ldx, int nv, float *y, int ldy, bool accumulate,
                     cudaStream_t st)
{
    return launch_gemv_fast_ex(W, nullptr, nullptr, 0.0f, x, ldx, nv, y, ldy, accumulate ? GM_ADD : GM_STORE, st,
                               false);
}

}  // namespace llmdot
