// step.cu -- the whole greedy decode step as ONE persistent cooperative kernel.
//
// Reference: InferenceEngine.ProcessToken (src/Llmdot.Core/Inference/InferenceEngine.cs:134-146)
// over LlamaLike / GemmaLike templates, i.e. per layer ApplyNorm (:544-562), Q/K/V (:321-353),
// RoPE + KV append + attention (:362-442), attn_output + residual (:444-449), FfnForward
// (:452-487) + residual, then ApplyFinalNorm (:575-581), ComputeLogits (:583-602), final softcap
// and greedy argmax (:105-108, Sampler.cs:26-27).
//
// Batch-1 decode streams ~0.77 GB of quantised weights per token, i.e. ~120 us at HBM speed,
// while a launch per operation costs several microseconds of fixed latency each (about 100
// launches per step).  Here one CTA per SM runs all of it:
//
// * The step is a static list of phases (per layer: QKV matvec, attention scores, attention
//   P.V, attn_output matvec, gate/up matvec, down matvec; then the logits head), separated by
//   grid barriers (an arrival counter in global memory, spins bounded by %globaltimer).
// * Matvec phases split the output rows in 16-row tiles over the CTAs (a CTA owns a contiguous
//   run of row tiles) and each row tile in `ks` K-parts; a "unit" (row tile, K-part) belongs to
//   one warp, which accumulates its partial in registers.  Units are reduced in shared memory
//   in a fixed order, so results do not depend on timing.
// * Weights never depend on activations, so each warp streams the tiles of ITS units with
//   cp.async.bulk (TMA bulk copies) into a private ring of shared-memory slots completed by
//   mbarriers, and keeps the ring full across phase boundaries: while the CTA waits at a grid
//   barrier, computes the attention or builds the next input, the next phases' weights are
//   already on their way.
// * The input of every matvec phase (with its RMSNorm, and Gemma's post-norms of the residual
//   stream deferred into the next phase) is rebuilt by every CTA from L2 in a prologue, as the
//   fp16 hi/lo fragments the tensor-core tile math consumes (gemv_tile.cuh).
// * Attention: the units are (session, kv head, page of 64 positions).  The reference's softmax
//   evaluates ExpApprox against the window max, so the scores phase (RoPE, append, q.k, softcap,
//   page max) and the P.V phase (exp against the window max, page partials, last page combines)
//   are separate phases.
// * The argmax is folded into the head's epilogue (64-bit keys, atomicMax); the next step reads
//   its token from the keys, so `n_steps` greedy steps run inside one launch.
#include <algorithm>
#include <cstdlib>
#include <vector>

#include "engine.cuh"
#include "gemv_tile.cuh"
#include "quant.cuh"
#include "step.cuh"

namespace llmdot {

namespace {

constexpr int SW = 16;            // warps per CTA (every warp streams and computes)
constexpr int ST = SW * 32;       // threads per CTA
constexpr int SLOT = Q6K_TILE;    // ring slot bytes: the largest tile
constexpr int UMAX = 128;         // (row tile, K-part) units per CTA and phase
constexpr int NV_MAX = 3;         // batch rows the kernel is built for
constexpr unsigned long long WAIT_NS = 2000000000ull;  // every spin gives up after 2 s

enum { PK_MATVEC = 0, PK_SCORES = 1, PK_PV = 2, PK_EMBED = 3 };
enum { SM_STORE = 0, SM_ADD = 1, SM_SILU = 2, SM_GELU = 3, SM_HEAD = 4 };
enum { PF_LAST_ONLY = 1 };
enum { ERR_TOKEN = 1, ERR_BARRIER = 2, ERR_TILE = 3 };

struct StepSeg {
    const uint8_t *w, *w1;  // tiled weights (w1: the "up" matrix of gate/up)
    float *y;               // [nv][ldy]
    int rows, nrt, qt, ldy;
};

struct StepPhase {
    int kind, mode, flags, layer;
    int nseg, nsb, nmat, rt_total, ks, tpu, need_q4, need_q6;
    StepSeg seg[3];
    const float *x;           // matvec input [nv][ldx]
    int ldx;
    const float *norm_w;      // fused RMSNorm of the input (nullable)
    const float *pend_w;      // deferred post-norm of the residual, applied to the input first
    const float *add_pend_w;  // SM_ADD: deferred post-norm applied to the residual before the add
    const float *q, *k, *v;   // attention inputs (raw projections)
    int ldq, ldkv;
    float *out;               // attention output [nv][ldo]
    int ldo;
};

struct StepArgs {
    const StepPhase *ph;
    int nph, n_steps, nv;
    const uint8_t *emb;
    uint32_t emb_type;
    int emb_apply;
    uint64_t emb_rbytes;
    int vocab;
    float emb_scale, eps;
    AttnShape sh;
    const float *cos_t, *sin_t;
    float *h;
    int ldh;
    float *scores, *part_m, *part_s, *part_o;
    int *counters;
    unsigned long long *keys;  // [2][nv] argmax keys of even / odd steps
    int32_t *next, *pos, *hist, *hist_step;
    const int32_t *forced;
    const KvView *views;
    int *err;
    unsigned *bar;  // [0] barrier arrivals, [1] CTAs that finished
    int has_final_cap;
    float final_cap;
    unsigned long long *trace;  // optional: [phase][cta][16] %globaltimer stamps of step 0
    int ring;                   // tile slots per warp (2 or 3)
    int evict_first;            // tag the weight stream L2 evict-first
    int kv_f16;                 // KV cache element: fp16 (1) or fp32 (0)
};

// ------------------------------------------------------------------ PTX helpers
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
        : "r"(smem_u32(b)), "r"(parity), "r"(1000000u)  // suspend up to 1 ms instead of spinning
        : "memory");
    return ok != 0;
}
// contiguous global -> shared copy by the TMA unit, completing `bytes` on the mbarrier
// The weight stream is read once per step and would evict everything else from L2 (KV pages,
// activations, norm weights, phase descriptors): it is tagged evict-first.
__device__ __forceinline__ uint64_t evict_first_policy()
{
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *b)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(b))
                 : "memory");
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *b, uint64_t pol)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(b)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Waits (bounded) for the fill with the given parity; the answer is uniform across the warp.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *b, uint32_t parity)
{
    bool ok = mbar_test(b, parity);
    if (!ok) {
        const uint64_t t0 = gtimer();
        while (!(ok = mbar_test(b, parity)))
            if (gtimer() - t0 > WAIT_NS) break;
    }
    return __all_sync(0xffffffffu, ok);
}
__host__ __device__ inline size_t align16(size_t n) { return (n + 15) / 16 * 16; }

// ------------------------------------------------------------------ static schedule
__device__ __forceinline__ bool phase_runs(const StepArgs &a, const StepPhase &ph, int s)
{
    return !((ph.flags & PF_LAST_ONLY) && a.forced && s != a.n_steps - 1);
}
// contiguous block of row tiles owned by this CTA
__device__ __forceinline__ void cta_rows(const StepPhase &ph, int &lo, int &hi)
{
    lo = (int)(blockIdx.x * (unsigned)ph.rt_total / gridDim.x);
    hi = (int)((blockIdx.x + 1) * (unsigned)ph.rt_total / gridDim.x);
}
__device__ __forceinline__ int seg_of(const StepPhase &ph, int rt, int &rts)
{
    int s = 0;
    rts = rt;
    while (s + 1 < ph.nseg && rts >= ph.seg[s].nrt) {
        rts -= ph.seg[s].nrt;
        s++;
    }
    return s;
}

// Position of a warp in its own tile stream: step s, phase pi, unit u (= warp mod SW), tile j
// of the unit, with the current phase's and unit's constants cached so that advancing by one
// tile is a pointer increment.
struct Cur {
    int s, pi, u, j, U, ks, tpu, lo;
    uint32_t tb;          // bytes of one tile of the current unit
    const uint8_t *src;   // next tile to fetch
};
__device__ __forceinline__ void cur_unit(const StepPhase &ph, Cur &c)
{
    const int rt = c.lo + c.u / c.ks, f0 = (c.u % c.ks) * c.tpu;
    const int mat = f0 / ph.nsb, sb0 = f0 - mat * ph.nsb;
    int rts;
    const StepSeg &sg = ph.seg[seg_of(ph, rt, rts)];
    c.tb = sg.qt == QT_Q4K ? Q4K_TILE : Q6K_TILE;
    c.src = (mat ? sg.w1 : sg.w) + ((size_t)rts * ph.nsb + sb0) * c.tb;  // a unit's tiles are contiguous
    c.j = 0;
}
// Per-phase constants the tile cursor scans, cached in shared memory at kernel start.
struct PhHdr {
    int kind, flags, rt_total, ks;
};
constexpr int PH_MAX = 256;  // phases a plan may hold (6 per layer + 2)

// First unit of this warp at or after phase (s, pi).
__device__ void cur_seek(const StepArgs &a, const PhHdr *hdr, Cur &c, int warp)
{
    while (c.s < a.n_steps) {
        const PhHdr hh = hdr[c.pi];
        if (hh.kind == PK_MATVEC && !((hh.flags & PF_LAST_ONLY) && a.forced && c.s != a.n_steps - 1)) {
            const int lo = (int)(blockIdx.x * (unsigned)hh.rt_total / gridDim.x);
            const int hi = (int)((blockIdx.x + 1) * (unsigned)hh.rt_total / gridDim.x);
            const int U = (hi - lo) * hh.ks;
            if (warp < U) {
                const StepPhase &ph = a.ph[c.pi];
                c.u = warp;
                c.U = U;
                c.ks = hh.ks;
                c.tpu = ph.tpu;
                c.lo = lo;
                cur_unit(ph, c);
                return;
            }
        }
        if (++c.pi == a.nph) {
            c.pi = 0;
            c.s++;
        }
    }
}
// Ring position of one side (issue or consume) of a warp's tile stream.
struct RingPos {
    int n, slot;       // tiles so far, slot of the next one
    uint32_t parity;   // fill parity the next tile completes
    __device__ __forceinline__ void step(int ring)
    {
        n++;
        if (++slot == ring) {
            slot = 0;
            parity ^= 1u;
        }
    }
};

// Lane 0 starts the bulk copy of the warp's next tile into its next ring slot.
__device__ __forceinline__ void issue_next(const StepArgs &a, const PhHdr *hdr, Cur &c, int warp, int lane, uint8_t *ring_w,
                                           uint64_t *mb_w, RingPos &ip)
{
    if (c.s >= a.n_steps) return;
    const int slot = ip.slot;
    if (lane == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the slot's last reads come first
        mbar_expect_tx(mb_w + slot, c.tb);
        if (a.evict_first) bulk_load(ring_w + (size_t)slot * SLOT, c.src, c.tb, mb_w + slot, evict_first_policy());
        else bulk_load(ring_w + (size_t)slot * SLOT, c.src, c.tb, mb_w + slot);
    }
    ip.step(a.ring);
    c.src += c.tb;
    if (++c.j == c.tpu) {
        c.u += SW;
        if (c.u < c.U) {
            cur_unit(a.ph[c.pi], c);
        } else {
            if (++c.pi == a.nph) {
                c.pi = 0;
                c.s++;
            }
            cur_seek(a, hdr, c, warp);
        }
    }
}

// ------------------------------------------------------------------ grid barrier
__device__ __forceinline__ bool grid_barrier(const StepArgs &a, unsigned &nbar, volatile int *abort_flag)
{
    __syncthreads();
    if (threadIdx.x == 0) {
        nbar++;
        const unsigned target = nbar * gridDim.x;
        __threadfence();
        atomicAdd(a.bar, 1u);
        if (ld_acquire(a.bar) < target) {
            const uint64_t t0 = gtimer();
            while (ld_acquire(a.bar) < target)
                if (gtimer() - t0 > WAIT_NS) {
                    atomicExch(a.err, ERR_BARRIER);
                    *abort_flag = 1;
                    break;
                }
        }
        __threadfence();
    }
    __syncthreads();
    return *abort_flag == 0;
}

// ------------------------------------------------------------------ matvec phase
// Shared-memory layout of one matvec phase's input inside the scratch region X.
template <int NV> struct XLayout {
    uint4 *xs4, *xs6;
    float *S, *P;
    __device__ XLayout(uint8_t *X, const StepPhase &ph)
    {
        const size_t xsz = (size_t)ph.nsb * 1024 * NV;
        xs4 = (uint4 *)X;
        xs6 = (uint4 *)(X + (ph.need_q4 ? xsz : 0));
        S = (float *)(X + (ph.need_q4 ? xsz : 0) + (ph.need_q6 ? xsz : 0));
        P = S + NV * ph.nsb * 8;
    }
};

// Builds the phase input: optional deferred post-norm of the residual (pinv kept for the next
// SM_ADD epilogue), the phase's own RMSNorm, an exact power-of-two scale, then the fp16 hi/lo
// B fragments for the tile layouts the phase uses and, for Q4_K, the sub-block sums of x.
// Every thread owns "items" of 8 elements (the group one fragment unit holds) and keeps the
// first PRO_KEEP of them in registers between the statistics and the fragment pass, so the
// input crosses L2 once per layout.
constexpr int PRO_KEEP = 2;

template <int NV>
__device__ void mv_prologue(const StepArgs &a, const StepPhase &ph, const int *tok, float *stat, float *wred,
                            const XLayout<NV> &L, unsigned long long *tr)
{
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nsb = ph.nsb, cols = nsb * 256, nitem = nsb * 32 * NV;
    float *inv = stat, *scl = stat + NV, *pinv = stat + 2 * NV;
    const int lay0 = ph.need_q4 ? 0 : 1;  // the layout whose items carry the statistics
    // item it of layout lay: vector v, elements e0..e0+3 and e1..e1+3
    // Q4_K: 8 consecutive weights 64t+8w.. in slot order {0,4,1,5,2,6,3,7};
    // Q6_K: 4 at 32w+4t.. and 4 at 32w+16+4t.. in order
    auto item = [&](int lay, int it, int &v, int &e0, int &e1) {
        v = it % NV;
        const int r = it / NV, w = r & 7, tt = (r >> 3) & 3, sb = r >> 5;
        e0 = lay == 0 ? sb * 256 + 64 * tt + 8 * w : sb * 256 + 32 * w + 4 * tt;
        e1 = lay == 0 ? e0 + 4 : e0 + 16;
    };
    // the activation the last phase wrote (other CTAs: read through L2)
    auto load8 = [&](int v, int e0, int e1, float *c) {
        const float4 p0 = __ldcg((const float4 *)(ph.x + (size_t)v * ph.ldx + e0));
        const float4 p1 = __ldcg((const float4 *)(ph.x + (size_t)v * ph.ldx + e1));
        c[0] = p0.x, c[1] = p0.y, c[2] = p0.z, c[3] = p0.w, c[4] = p1.x, c[5] = p1.y, c[6] = p1.z, c[7] = p1.w;
    };
    // cols is a multiple of 8, so every element is a "vector lane" of the reference's RmsNorm:
    // (w * x) * inv
    auto pend = [&](int v, int e0, int e1, float *c) {
        if (!ph.pend_w) return;
        const float4 w0 = __ldg((const float4 *)(ph.pend_w + e0)), w1 = __ldg((const float4 *)(ph.pend_w + e1));
        const float wn[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int k = 0; k < 8; k++) c[k] = __fmul_rn(__fmul_rn(wn[k], c[k]), pinv[v]);
    };
    auto block_stats = [&](float *ss, float *mx) {
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
    };
    float keep[PRO_KEEP][8];
    // visits this thread's items; the first PRO_KEEP (fully unrolled) may keep their values in
    // registers between passes
    auto each_item = [&](auto &&fn) {
#pragma unroll
        for (int q = 0; q < PRO_KEEP; q++) {
            const int it = tid + q * ST;
            if (it < nitem) fn(it, keep[q], true);
        }
        for (int it = tid + PRO_KEEP * ST; it < nitem; it += ST) {
            float tmp[8];
            fn(it, tmp, false);
        }
    };
    if (ph.pend_w) {  // VectorMath.RmsNorm of the residual (Gemma post-norm): statistics first
        float ss[NV], mx[NV];
#pragma unroll
        for (int v = 0; v < NV; v++) ss[v] = mx[v] = 0.0f;
        each_item([&](int it, float(&c)[8], bool) {
            int v, e0, e1;
            item(lay0, it, v, e0, e1);
            load8(v, e0, e1, c);
#pragma unroll
            for (int vv = 0; vv < NV; vv++)
                if (vv == v)
#pragma unroll
                    for (int k = 0; k < 8; k++) ss[vv] = fmaf(c[k], c[k], ss[vv]);
        });
        block_stats(ss, mx);
        if (tid < NV) {
            float t = 0.0f;
            for (int w = 0; w < SW; w++) t += wred[w * 2 * NV + tid];
            pinv[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)cols), a.eps)));
        }
        __syncthreads();
    }
    {
        float ss[NV], mx[NV];
#pragma unroll
        for (int v = 0; v < NV; v++) ss[v] = mx[v] = 0.0f;
        each_item([&](int it, float(&c)[8], bool kept) {
            int v, e0, e1;
            item(lay0, it, v, e0, e1);
            if (!(ph.pend_w && kept)) load8(v, e0, e1, c);  // kept values already hold the raw input
            pend(v, e0, e1, c);
            float wn[8] = {1, 1, 1, 1, 1, 1, 1, 1};
            if (ph.norm_w) {
                const float4 w0 = __ldg((const float4 *)(ph.norm_w + e0)), w1 = __ldg((const float4 *)(ph.norm_w + e1));
                wn[0] = w0.x, wn[1] = w0.y, wn[2] = w0.z, wn[3] = w0.w, wn[4] = w1.x, wn[5] = w1.y, wn[6] = w1.z,
                wn[7] = w1.w;
            }
#pragma unroll
            for (int vv = 0; vv < NV; vv++)
                if (vv == v)
#pragma unroll
                    for (int k = 0; k < 8; k++) {
                        ss[vv] = fmaf(c[k], c[k], ss[vv]);
                        mx[vv] = fmaxf(mx[vv], fabsf(ph.norm_w ? __fmul_rn(wn[k], c[k]) : c[k]));
                    }
        });
        if (tr) tr[8] = gtimer();  // thread 0's input loads and statistics done
        block_stats(ss, mx);
        if (tr) tr[9] = gtimer();  // whole CTA's statistics done
        if (tid < NV) {
            float t = 0.0f, m = 0.0f;
            for (int w = 0; w < SW; w++) {
                t += wred[w * 2 * NV + tid];
                m = fmaxf(m, wred[w * 2 * NV + NV + tid]);
            }
            float iv = 1.0f;
            if (ph.norm_w) {  // 1 / sqrt(ss/n + eps); x = (w*h)*inv
                iv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)cols), a.eps)));
                m = __fmul_rn(m, iv);  // rounding is monotone: max of the products
            }
            float sc = 1.0f;  // exact power of two putting max|x|*sc in [2^14, 2^15)
            if (m > 0.0f && m < INFINITY) {
                int e;
                frexpf(m, &e);
                sc = ldexpf(1.0f, 15 - e);
            }
            inv[tid] = iv;
            scl[tid] = sc;
        }
        __syncthreads();
    }
    for (int lay = 0; lay < 2; lay++) {
        if ((lay == 0 && !ph.need_q4) || (lay == 1 && !ph.need_q6)) continue;
        uint4 *xs = lay == 0 ? L.xs4 : L.xs6;
        each_item([&](int it, float(&kq)[8], bool kept) {
            int v, e0, e1;
            item(lay, it, v, e0, e1);
            const int r = it / NV, w = r & 7, tt = (r >> 3) & 3, sb = r >> 5;
            float c[8];
            if (lay == lay0 && kept) {
#pragma unroll
                for (int k = 0; k < 8; k++) c[k] = kq[k];
            } else {
                load8(v, e0, e1, c);
                pend(v, e0, e1, c);
            }
            const float sc = scl[v];
            if (ph.norm_w) {
                const float f = inv[v] * sc;  // ((w*h)*inv)*sc == (w*h)*(inv*sc): sc is a power of two
                const float4 w0 = __ldg((const float4 *)(ph.norm_w + e0)), w1 = __ldg((const float4 *)(ph.norm_w + e1));
                const float wn[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int k = 0; k < 8; k++) c[k] = __fmul_rn(__fmul_rn(wn[k], c[k]), f);
            } else {
#pragma unroll
                for (int k = 0; k < 8; k++) c[k] *= sc;
            }
            if (lay == 0) {
                float psum = 0.0f;
#pragma unroll
                for (int k = 0; k < 8; k++) psum += c[k];
                L.P[((v * nsb + sb) * 4 + tt) * 8 + w] = psum;
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
        });
    }
    if (tr) tr[10] = gtimer();  // thread 0's fragments written
    if (ph.need_q4) {
        __syncthreads();
        // sub-block sums S_j = sum of its four 8-weight partials, fixed order
        for (int it = tid; it < NV * nsb * 8; it += ST) {
            const int v = it / (nsb * 8), jj = it % (nsb * 8), sb = jj >> 3, j = jj & 7;
            const float *pp = L.P + ((v * nsb + sb) * 4 + (j >> 1)) * 8 + 4 * (j & 1);
            L.S[it] = ((pp[0] + pp[1]) + pp[2]) + pp[3];
        }
    }
    __syncthreads();
}

// The warp's units of this phase: wait for each tile in its ring, refill the slot with the
// warp's next tile (possibly of a later phase), accumulate, store the unit partial.
template <int NV>
__device__ bool mv_tiles(const StepArgs &a, const StepPhase &ph, int lo, int hi, const XLayout<NV> &L, float *red,
                         uint8_t *ring_w, uint64_t *mb_w, const PhHdr *hdr, Cur &cur, RingPos &ip, RingPos &cp,
                         unsigned long long *tr)
{
    unsigned long long t_wait = 0, t_comp = 0, n_tiles = 0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int bv = min(g >> 1, NV - 1), bpart = g & 1;  // this lane's B column (vector, part)
    const int ks = ph.ks, tpu = ph.tpu, nsb = ph.nsb;  // registers: the loop stores would force reloads
    const int U = (hi - lo) * ks;
    for (int u = warp; u < U; u += SW) {
        const int rt = lo + u / ks, kp = u % ks;
        int rts;
        const int qt = ph.seg[seg_of(ph, rt, rts)].qt;
        const int sb0 = (kp * tpu) % nsb;
        float acc0 = 0.0f, acc1 = 0.0f;  // rows g, g+8 for vector t (MMA columns 2t, 2t+1)
        float corr0[NV], corr1[NV];
#pragma unroll
        for (int v = 0; v < NV; v++) corr0[v] = corr1[v] = 0.0f;
        for (int j = 0; j < tpu; j++) {
            const int sb = sb0 + j;
            const int slot = cp.slot;
            const unsigned long long w0 = tr ? gtimer() : 0;
            if (!mbar_wait_warp(mb_w + slot, cp.parity)) return false;
            const unsigned long long w1 = tr ? gtimer() : 0;
            TileRegs T;
            read_tile(T, ring_w + (size_t)slot * SLOT, qt, lane);
            __syncwarp();  // the tile is in registers: refill its slot before the math
            cp.step(a.ring);
            issue_next(a, hdr, cur, warp, lane, ring_w, mb_w, ip);
            if (qt == QT_Q4K) q4k_tile<NV>(T, L.xs4, L.S, nsb, sb, t, bv, bpart, acc0, acc1, corr0, corr1);
            else q6k_tile<NV>(T, L.xs6, sb, t, bv, bpart, acc0, acc1);
            if (tr) {
                t_wait += w1 - w0;
                t_comp += gtimer() - w1;
                n_tiles++;
            }
        }
        if (qt == QT_Q4K) {
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
            }
            acc0 -= k0;
            acc1 -= k1;
        }
        if (t < NV) {
            red[(u * 16 + g) * NV + t] = acc0;
            red[(u * 16 + g + 8) * NV + t] = acc1;
        }
    }
    if (tr && lane == 0) {  // warp 0 of the CTA: time waiting for tiles vs computing them
        tr[4] = t_wait;
        tr[5] = t_comp;
        tr[6] = n_tiles;
    }
    return true;
}

// Sums each row tile's K-parts in a fixed order and applies the phase's epilogue.
template <int NV>
__device__ void mv_epilogue(const StepArgs &a, const StepPhase &ph, int s, int lo, int hi, const float *red,
                            const float *stat)
{
    const int tid = threadIdx.x, lane = tid & 31;
    const int n = (hi - lo) * 16;
    const float *scl = stat + NV, *pinv = stat + 2 * NV;
    const bool head = ph.mode == SM_HEAD;
    const float inv_cap = (head && a.has_final_cap) ? __fdiv_rn(1.0f, a.final_cap) : 0.0f;
    unsigned long long best[NV];
#pragma unroll
    for (int v = 0; v < NV; v++) best[v] = 0ull;
    for (int it = tid; it < n * NV; it += ST) {
        const int v = it / n, r2 = it % n, rtl = r2 >> 4, rr = r2 & 15;
        int rts;
        const StepSeg &sg = ph.seg[seg_of(ph, lo + rtl, rts)];
        const int row = rts * 16 + rr;
        if (row >= sg.rows) continue;
        float o0 = 0.0f, o1 = 0.0f;
        for (int kp = 0; kp < ph.ks; kp++) {
            const float pv = red[(((rtl * ph.ks + kp) << 4) + rr) * NV + v];
            if ((kp * ph.tpu) / ph.nsb == 0) o0 += pv;
            else o1 += pv;
        }
        const float isc = 1.0f / scl[v];
        o0 *= isc;
        o1 *= isc;
        float *yp = sg.y + (size_t)v * sg.ldy + row;
        if (ph.mode == SM_STORE) {
            *yp = o0;
        } else if (ph.mode == SM_ADD) {  // Add (InferenceEngine.cs:189/:195) onto the residual
            float hv = __ldcg(yp);
            if (ph.add_pend_w) hv = __fmul_rn(__fmul_rn(__ldg(ph.add_pend_w + row), hv), pinv[v]);
            *yp = __fadd_rn(hv, o0);
        } else if (head) {
            *yp = o0;
            const float f = a.has_final_cap ? softcap_ref(o0, a.final_cap, inv_cap, row < sg.rows - sg.rows % 8) : o0;
            const unsigned long long k = ((unsigned long long)float_key(f) << 32) | (0xFFFFFFFFu - (uint32_t)row);
#pragma unroll
            for (int vv = 0; vv < NV; vv++)
                if (vv == v && k > best[vv]) best[vv] = k;
        } else {
            const bool vl = row < sg.rows - sg.rows % 8;
            const float act = ph.mode == SM_SILU ? silu_ref(o0, vl) : gelu_ref(o0, vl);
            *yp = __fmul_rn(act, o1);
        }
    }
    if (head) {
#pragma unroll
        for (int v = 0; v < NV; v++) {
            unsigned long long b = best[v];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, b, o);
                b = other > b ? other : b;
            }
            if (lane == 0 && b) atomicMax(a.keys + (s & 1) * NV + v, b);
        }
    }
}

// ------------------------------------------------------------------ attention phases
template <typename T> struct KvT;
template <> struct KvT<float> {
    static __device__ __forceinline__ float ld(const float *p) { return *p; }
    static __device__ __forceinline__ float st(float v) { return v; }
};
template <> struct KvT<__half> {
    static __device__ __forceinline__ float ld(const __half *p) { return __half2float(*p); }
    static __device__ __forceinline__ __half st(float v) { return __float2half_rn(v); }
};

__device__ __forceinline__ void att_window(int p, int sw, int &start, int &seq_len)
{
    seq_len = p + 1;
    start = sw > 0 ? max(0, seq_len - sw) : 0;
}

// Positions [j0, j1) of one page into shared-memory rows of `stride` elements, read through L2
// (pages are appended by other CTAs during the launch).
template <typename T>
__device__ __forceinline__ void stage_cg(T *dst, const T *src, int hd, int stride, int j0, int j1)
{
    constexpr int E = 16 / sizeof(T);
    const int per_row = hd / E;
    for (int i = threadIdx.x; i < (j1 - j0) * per_row; i += ST) {
        const int j = j0 + i / per_row, c = (i % per_row) * E;
        const uint4 v = __ldcg((const uint4 *)(src + (size_t)j * hd + c));
        const T *pv = (const T *)&v;
#pragma unroll
        for (int e = 0; e < E; e++) dst[j * stride + c + e] = pv[e];
    }
}

// Units (session b, kv head, page) of the attention window of every session at step s.
struct AttUnits {
    int c0[NV_MAX], nc[NV_MAX], total;
    __device__ AttUnits(const StepArgs &a, const int *pos0, int s)
    {
        total = 0;
        for (int b = 0; b < a.nv; b++) {
            int start, seq_len;
            att_window(pos0[b] + s, a.sh.sliding_window, start, seq_len);
            c0[b] = start / KV_PAGE;
            nc[b] = (seq_len - 1) / KV_PAGE - c0[b] + 1;
            total += a.sh.heads_kv * nc[b];
        }
    }
    __device__ void unit(int u, int hkv, int &b, int &kvh, int &chunk) const
    {
        b = 0;
        while (u >= hkv * nc[b]) {
            u -= hkv * nc[b];
            b++;
        }
        kvh = u / nc[b];
        chunk = c0[b] + u % nc[b];
    }
};

// RoPE of q (and of the new k, appended with v by the page that holds the position),
// s = (q . k) / sqrt(hd) with softcap, page max (InferenceEngine.cs:362-414).
template <typename T>
__device__ void att_scores(const StepArgs &a, const StepPhase &ph, int s, const int *pos0, uint8_t *X)
{
    const AttnShape &sh = a.sh;
    const int hd = sh.head_dim, half = sh.rope_half, G = sh.heads / sh.heads_kv, nchunk = sh.max_ctx / KV_PAGE;
    const int stride = hd + (sizeof(T) == 2 ? 2 : 1);  // odd word stride: no bank conflicts across positions
    T *ks = (T *)X;
    float *qs = (float *)(X + align16((size_t)KV_PAGE * stride * sizeof(T)));  // [G][hd]
    uint32_t *mk = (uint32_t *)(qs + G * hd);                                   // [G]
    const AttUnits au(a, pos0, s);
    const float inv_cap = sh.has_cap ? __fdiv_rn(1.0f, sh.cap) : 0.0f;
    for (int u = blockIdx.x; u < au.total; u += gridDim.x) {
        int b, kvh, chunk;
        au.unit(u, sh.heads_kv, b, kvh, chunk);
        const int p = pos0[b] + s;
        int start, seq_len;
        att_window(p, sh.sliding_window, start, seq_len);
        const int s0 = chunk * KV_PAGE;
        const KvView vw = a.views[b];
        const int page = vw.pages[chunk];
        const size_t head_off = ((size_t)page * sh.heads_kv + kvh) * KV_PAGE * hd;
        T *kg = (T *)vw.k + (size_t)ph.layer * vw.layer_stride + head_off;
        T *vg = (T *)vw.v + (size_t)ph.layer * vw.layer_stride + head_off;
        const int jlo = max(start - s0, 0), jhi = min(seq_len - s0, KV_PAGE);
        const bool has_new = p >= s0 && p < s0 + KV_PAGE;
        stage_cg<T>(ks, kg, hd, stride, jlo, has_new ? p - s0 : jhi);
        const float *cs = a.cos_t + (size_t)p * half, *sn = a.sin_t + (size_t)p * half;
        for (int i = threadIdx.x; i < G * hd; i += ST) {  // TensorOps.ApplyRoPE, half-split pairs
            const int hg = i / hd, d = i % hd;
            const float *x = ph.q + (size_t)b * ph.ldq + (size_t)(kvh * G + hg) * hd;
            float r;
            if (d < half) r = __fsub_rn(__fmul_rn(__ldcg(x + d), cs[d]), __fmul_rn(__ldcg(x + d + half), sn[d]));
            else if (d < 2 * half)
                r = __fadd_rn(__fmul_rn(__ldcg(x + d - half), sn[d - half]), __fmul_rn(__ldcg(x + d), cs[d - half]));
            else r = __ldcg(x + d);
            qs[i] = r;
        }
        for (int i = threadIdx.x; i < G; i += ST) mk[i] = 0u;
        if (has_new) {  // RoPE of the new key, then K/V cache append (InferenceEngine.cs:375-382)
            const float *kx = ph.k + (size_t)b * ph.ldkv + (size_t)kvh * hd;
            const float *vx = ph.v + (size_t)b * ph.ldkv + (size_t)kvh * hd;
            const int slot = p - s0;
            for (int d = threadIdx.x; d < hd; d += ST) {
                float r;
                if (d < half) r = __fsub_rn(__fmul_rn(__ldcg(kx + d), cs[d]), __fmul_rn(__ldcg(kx + d + half), sn[d]));
                else if (d < 2 * half)
                    r = __fadd_rn(__fmul_rn(__ldcg(kx + d - half), sn[d - half]), __fmul_rn(__ldcg(kx + d), cs[d - half]));
                else r = __ldcg(kx + d);
                const T kt = KvT<T>::st(r);
                kg[(size_t)slot * hd + d] = kt;
                ks[slot * stride + d] = kt;
                vg[(size_t)slot * hd + d] = KvT<T>::st(__ldcg(vx + d));
            }
        }
        __syncthreads();
        const int len = seq_len - start, nvec = len - len % 8;
        for (int idx = threadIdx.x; idx < G * KV_PAGE; idx += ST) {
            const int hg = idx / KV_PAGE, j = idx % KV_PAGE, sp = s0 + j;
            if (j < jlo || j >= jhi) continue;
            const T *kr = ks + j * stride;
            const float *qh = qs + hg * hd;
            float dot = 0.0f;
            for (int d = 0; d < hd; d++) dot = fmaf(qh[d], KvT<T>::ld(kr + d), dot);
            float sc = __fmul_rn(dot, sh.inv_sqrt_hd);
            if (sh.has_cap) sc = softcap_ref(sc, sh.cap, inv_cap, (sp - start) < nvec);
            a.scores[((size_t)b * sh.heads + kvh * G + hg) * sh.max_ctx + sp] = sc;
            atomicMax(mk + hg, float_key(sc));
        }
        __syncthreads();
        for (int hg = threadIdx.x; hg < G; hg += ST)
            a.part_m[((size_t)b * sh.heads + kvh * G + hg) * nchunk + chunk] = key_float(mk[hg]);
        __syncthreads();  // the staging buffers are reused by the next unit
    }
}

// p = exp(s - M) against the window max M, page sums and sum p*V; the last page of each
// (session, kv head) combines the pages and scales by 1/sum (VectorMath.Softmax, :415-442).
template <typename T>
__device__ void att_pv(const StepArgs &a, const StepPhase &ph, int s, const int *pos0, uint8_t *X, int *last_flag)
{
    const AttnShape &sh = a.sh;
    const int hd = sh.head_dim, G = sh.heads / sh.heads_kv, nchunk = sh.max_ctx / KV_PAGE;
    T *vs = (T *)X;                                                                 // [KV_PAGE][hd]
    float *ps = (float *)(X + align16((size_t)KV_PAGE * hd * sizeof(T)));          // [G][KV_PAGE]
    float *mx = ps + G * KV_PAGE;                                                   // [G]
    const AttUnits au(a, pos0, s);
    for (int u = blockIdx.x; u < au.total; u += gridDim.x) {
        int b, kvh, chunk;
        au.unit(u, sh.heads_kv, b, kvh, chunk);
        const int p = pos0[b] + s;
        int start, seq_len;
        att_window(p, sh.sliding_window, start, seq_len);
        const int s0 = chunk * KV_PAGE;
        const KvView vw = a.views[b];
        const int page = vw.pages[chunk];
        const T *vg =
            (const T *)vw.v + (size_t)ph.layer * vw.layer_stride + ((size_t)page * sh.heads_kv + kvh) * KV_PAGE * hd;
        const int jlo = max(start - s0, 0), jhi = min(seq_len - s0, KV_PAGE);
        stage_cg<T>(vs, vg, hd, hd, jlo, jhi);
        const int len = seq_len - start, nvec = len - len % 8;
        const int c0 = start / KV_PAGE, c1 = (seq_len - 1) / KV_PAGE;
        for (int hg = threadIdx.x; hg < G; hg += ST) {
            const float *pm = a.part_m + ((size_t)b * sh.heads + kvh * G + hg) * nchunk;
            float m = -INFINITY;
            for (int c = c0; c <= c1; c++) m = fmaxf(m, __ldcg(pm + c));
            mx[hg] = m;
        }
        __syncthreads();
        for (int idx = threadIdx.x; idx < G * KV_PAGE; idx += ST) {
            const int hg = idx / KV_PAGE, j = idx % KV_PAGE, sp = s0 + j;
            float pr = 0.0f;
            if (j >= jlo && j < jhi) {
                const float d =
                    __fsub_rn(__ldcg(a.scores + ((size_t)b * sh.heads + kvh * G + hg) * sh.max_ctx + sp), mx[hg]);
                pr = (sp - start) < nvec ? exp_approx(d) : expf(d);
            }
            ps[idx] = pr;
        }
        __syncthreads();
        const size_t hbase = ((size_t)b * sh.heads + kvh * G) * nchunk;
        for (int hg = threadIdx.x >> 5; hg < G; hg += ST >> 5) {
            float tsum = 0.0f;
            for (int j = threadIdx.x & 31; j < KV_PAGE; j += 32) tsum += ps[hg * KV_PAGE + j];
            tsum = warp_sum(tsum);
            if ((threadIdx.x & 31) == 0) a.part_s[hbase + (size_t)hg * nchunk + chunk] = tsum;
        }
        for (int idx = threadIdx.x; idx < G * hd; idx += ST) {
            const int hg = idx / hd, d = idx % hd;
            const float *pp = ps + hg * KV_PAGE;
            float acc = 0.0f;
            for (int j = jlo; j < jhi; j++) acc = fmaf(pp[j], KvT<T>::ld(vs + j * hd + d), acc);
            a.part_o[((hbase + (size_t)hg * nchunk) + chunk) * hd + d] = acc;
        }
        __threadfence();
        __syncthreads();
        int *cnt = a.counters + (size_t)b * sh.heads_kv + kvh;
        if (threadIdx.x == 0) *last_flag = atomicAdd(cnt, 1) == (c1 - c0);
        __syncthreads();
        if (*last_flag) {
            __threadfence();
            for (int idx = threadIdx.x; idx < G * hd; idx += ST) {
                const int hg = idx / hd, d = idx % hd;
                const size_t hb = hbase + (size_t)hg * nchunk;
                float sum = 0.0f, o = 0.0f;
                for (int c = c0; c <= c1; c++) {
                    sum += __ldcg(a.part_s + hb + c);
                    o += __ldcg(a.part_o + (hb + c) * hd + d);
                }
                ph.out[(size_t)b * ph.ldo + (size_t)(kvh * G + hg) * hd + d] = __fmul_rn(o, __fdiv_rn(1.0f, sum));
            }
            if (threadIdx.x == 0) *cnt = 0;  // ready for the next layer / step
        }
        __syncthreads();
    }
}

// GetEmbedding + EmbeddingScale (InferenceEngine.cs:138-140): every CTA dequantises its share
// of the residual stream h for each row.
__device__ void embed_phase(const StepArgs &a, const int *tok, int cols)
{
    const uint32_t be = (uint32_t)block_elems(a.emb_type), bb = (uint32_t)block_bytes(a.emb_type);
    const int lo = (int)(blockIdx.x * (unsigned)cols / gridDim.x), hi = (int)((blockIdx.x + 1) * (unsigned)cols / gridDim.x);
    for (int it = threadIdx.x; it < (hi - lo) * a.nv; it += ST) {
        const int v = it / (hi - lo), i = lo + it % (hi - lo);
        const float val = deq1(a.emb_type, a.emb + (size_t)tok[v] * a.emb_rbytes + (size_t)(i / be) * bb, (int)(i % be));
        a.h[(size_t)v * a.ldh + i] = a.emb_apply ? __fmul_rn(val, a.emb_scale) : val;
    }
}

__device__ __forceinline__ int key_token(unsigned long long k) { return (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)); }

// Fixed part of the dynamic shared memory ahead of the phase scratch region.
__host__ __device__ inline size_t step_fixed_smem(int nv, int ring)
{
    return (size_t)SW * 3 * 8 + (size_t)SW * ring * SLOT + (size_t)UMAX * 16 * nv * 4 + 64 + (size_t)SW * 8 * 4 + 64 +
           (size_t)PH_MAX * sizeof(PhHdr);
}

// ------------------------------------------------------------------ the kernel
template <int NV>
__global__ void __launch_bounds__(ST, 1) decode_step_kernel(const __grid_constant__ StepArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, ring = a.ring;
    uint64_t *mb = (uint64_t *)smem;                      // [SW][3] tile-slot mbarriers
    uint8_t *ring_all = smem + SW * 3 * 8;                // [SW][ring][SLOT]
    uint8_t *ring_w = ring_all + (size_t)warp * ring * SLOT;
    uint64_t *mb_w = mb + warp * 3;
    float *red = (float *)(ring_all + (size_t)SW * ring * SLOT);  // [UMAX][16][NV] unit partials
    float *stat = red + UMAX * 16 * NV;          // inv[NV] scale[NV] pending-inv[NV]
    float *wred = stat + 16;                     // [SW][2*NV] block reductions
    int *ist = (int *)(wred + SW * 8);           // tok[4] pos0[4] abort last hist0
    PhHdr *hdr = (PhHdr *)(ist + 16);            // [PH_MAX] phase headers
    uint8_t *X = (uint8_t *)(hdr + PH_MAX);      // phase scratch
    int *tok = ist, *pos0 = ist + 4;
    volatile int *abort_flag = ist + 8;
    int *last_flag = ist + 9;

    if (tid < SW * 3) mbar_init(mb + tid, 1);
    for (int i = tid; i < a.nph; i += ST) {
        const StepPhase &ph = a.ph[i];
        hdr[i] = PhHdr{ph.kind, ph.flags, ph.rt_total, ph.ks};
    }
    if (tid < NV) pos0[tid] = a.pos[tid];
    if (tid == 0) {
        *abort_flag = 0;
        ist[10] = a.hist_step ? *a.hist_step : 0;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();

    // every warp starts streaming its first tiles right away
    Cur cur = {};
    cur_seek(a, hdr, cur, warp);
    RingPos ip = {0, 0, 0u}, cp = {0, 0, 0u};
    for (int r = 0; r < ring; r++) issue_next(a, hdr, cur, warp, lane, ring_w, mb_w, ip);

    unsigned nbar = 0;
    bool ok = true;
    for (int s = 0; s < a.n_steps && ok; s++) {
        if (tid < NV) {  // this step's token: given, fed by the host, or the previous argmax
            int tk;
            if (a.forced) tk = a.forced[s * NV + tid];
            else if (s == 0) tk = a.next[tid];
            else tk = key_token(__ldcg(a.keys + ((s - 1) & 1) * NV + tid));
            if (tk < 0 || tk >= a.vocab) {
                if (blockIdx.x == 0) atomicExch(a.err, ERR_TOKEN);
                tk = 0;
            }
            tok[tid] = tk;
            if (blockIdx.x == 0) {
                if (!a.forced && s > 0) a.hist[((ist[10] + s - 1) % HIST_STEPS) * NV + tid] = tk;
                a.keys[(s & 1) * NV + tid] = 0ull;  // last read as step s-1's input, two barriers ago
            }
        }
        __syncthreads();
        for (int pi = 0; pi < a.nph && ok; pi++) {
            const StepPhase &ph = a.ph[pi];
            if (!phase_runs(a, ph, s)) continue;
            unsigned long long *tr =
                (a.trace && s == 0 && tid == 0) ? a.trace + ((size_t)pi * gridDim.x + blockIdx.x) * 16 : nullptr;
            if (tr) tr[0] = gtimer();
            if (ph.kind == PK_MATVEC) {
                const XLayout<NV> L(X, ph);
                mv_prologue<NV>(a, ph, tok, stat, wred, L, tr);
                if (tr) tr[1] = gtimer();
                int lo, hi;
                cta_rows(ph, lo, hi);
                if (!mv_tiles<NV>(a, ph, lo, hi, L, red, ring_w, mb_w, hdr, cur, ip, cp,
                                  (a.trace && s == 0 && warp == 0)
                                      ? a.trace + ((size_t)pi * gridDim.x + blockIdx.x) * 16
                                      : nullptr)) {
                    if (lane == 0) {
                        atomicExch(a.err, ERR_TILE);
                        *abort_flag = 1;
                    }
                }
                __syncthreads();
                if (tr) tr[2] = gtimer();
                if (*abort_flag) {
                    ok = false;
                    break;
                }
                mv_epilogue<NV>(a, ph, s, lo, hi, red, stat);
            } else if (ph.kind == PK_EMBED) {
                embed_phase(a, tok, a.ldh);
            } else if (ph.kind == PK_SCORES) {
                if (a.kv_f16) att_scores<__half>(a, ph, s, pos0, X);
                else att_scores<float>(a, ph, s, pos0, X);
            } else {
                if (a.kv_f16) att_pv<__half>(a, ph, s, pos0, X, last_flag);
                else att_pv<float>(a, ph, s, pos0, X, last_flag);
            }
            if (tr) tr[3] = gtimer();
            ok = grid_barrier(a, nbar, abort_flag);
        }
    }
    if (ok) {
        if (blockIdx.x == 0 && tid < NV) {
            const int tk = key_token(__ldcg(a.keys + ((a.n_steps - 1) & 1) * NV + tid));
            a.next[tid] = tk;
            if (!a.forced) a.hist[((ist[10] + a.n_steps - 1) % HIST_STEPS) * NV + tid] = tk;
            a.pos[tid] = pos0[tid] + a.n_steps;
        }
        if (blockIdx.x == 0 && tid == 0 && !a.forced && a.hist_step) *a.hist_step = ist[10] + a.n_steps;
        __syncthreads();
        if (tid == 0) {  // the last CTA out re-arms the barrier counters for the next launch
            __threadfence();
            if (atomicAdd(a.bar + 1, 1u) == gridDim.x - 1) {
                atomicExch(a.bar, 0u);
                atomicExch(a.bar + 1, 0u);
            }
        }
    } else {
        // error path: give the warp's copies still in flight (bounded) time to land before exit
        while (cp.n < ip.n) {
            mbar_wait_warp(mb_w + cp.slot, cp.parity);
            cp.step(ring);
        }
    }
}

}  // namespace

// ------------------------------------------------------------------ host side
struct StepPlan {
    int batch = 0, gen = -1, nph = 0, ring = 0, grid = 0, status = LLMDOT_OK;
    size_t smem = 0;
    StepPhase *d_ph = nullptr;
    unsigned *bar = nullptr;
    unsigned long long *keys = nullptr;
};
struct StepCache {
    std::vector<StepPlan> plans;
};

static void free_plan(StepPlan &p)
{
    if (p.d_ph) cudaFree(p.d_ph);
    if (p.bar) cudaFree(p.bar);
    if (p.keys) cudaFree(p.keys);
    p.d_ph = nullptr;
    p.bar = nullptr;
    p.keys = nullptr;
}

void step_cache_free(llmdot_model *m)
{
    if (!m || !m->step_cache) return;
    for (auto &p : m->step_cache->plans) free_plan(p);
    delete m->step_cache;
    m->step_cache = nullptr;
}

static void *pick_kernel(int nv)
{
    switch (nv) {
    case 1: return (void *)decode_step_kernel<1>;
    case 2: return (void *)decode_step_kernel<2>;
    case 3: return (void *)decode_step_kernel<3>;
    default: return nullptr;
    }
}

static bool tiled_ok(const DevMat &W) { return W.valid() && W.tiled && W.cols % 256 == 0; }

// Builds the phase list for `batch` rows (the workspace must already hold `batch` rows).
static int build_plan(llmdot_model *m, int batch, StepPlan &P)
{
    const llmdot_config &c = m->cfg;
    const Workspace &w = m->ws;
    const int H = c.hidden, qDim = c.heads * c.head_dim, kvDim = c.heads_kv * c.head_dim;
    const bool gemma = c.template_id == 2;
    int dev_sms = 0, optin = 0;
    LLMDOT_CUDA_TRY(cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, m->device));
    LLMDOT_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device));
    int coop = 0;
    LLMDOT_CUDA_TRY(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->device));
    if (!coop) return fail(LLMDOT_E_UNSUPPORTED, "step kernel: no cooperative launch");
    if (batch < 1 || batch > NV_MAX) return fail(LLMDOT_E_UNSUPPORTED, "step kernel: batch outside 1..3");
    const int grid = dev_sms;

    std::vector<StepPhase> ph;
    auto seg = [&](const DevMat &W, const DevMat *W1, float *y, int ldy) {
        StepSeg s{};
        s.w = W.tiled;
        s.w1 = W1 ? W1->tiled : nullptr;
        s.y = y;
        s.rows = W.rows;
        s.nrt = (W.rows + 15) / 16;
        s.qt = W.type == T_Q4_K ? QT_Q4K : QT_Q6K;
        s.ldy = ldy;
        return s;
    };
    auto matvec = [&](int mode, std::vector<StepSeg> segs, int cols, int nmat, const float *x, int ldx,
                      const float *norm_w, const float *pend_w, const float *add_pend_w, int flags) -> int {
        StepPhase p{};
        p.kind = PK_MATVEC;
        p.mode = mode;
        p.flags = flags;
        p.nseg = (int)segs.size();
        p.nsb = cols / 256;
        p.nmat = nmat;
        for (int i = 0; i < p.nseg; i++) {
            p.seg[i] = segs[i];
            p.rt_total += segs[i].nrt;
            p.need_q4 |= segs[i].qt == QT_Q4K;
            p.need_q6 |= segs[i].qt == QT_Q6K;
        }
        // K-parts per row tile: enough units for the CTA's 16 warps, a unit within one matrix
        const int nrt_max = (p.rt_total + grid - 1) / grid;
        p.ks = nmat;
        p.tpu = p.nsb;
        while (p.tpu % 2 == 0 && nrt_max * p.ks < SW) {
            p.ks *= 2;
            p.tpu /= 2;
        }
        if (nrt_max * p.ks > UMAX) return fail(LLMDOT_E_UNSUPPORTED, "step kernel: too many row tiles per SM");
        p.x = x;
        p.ldx = ldx;
        p.norm_w = norm_w;
        p.pend_w = pend_w;
        p.add_pend_w = add_pend_w;
        ph.push_back(p);
        return LLMDOT_OK;
    };
    const DevMat &head = m->out.valid() ? m->out : m->emb;
    if (!tiled_ok(head)) return fail(LLMDOT_E_UNSUPPORTED, "step kernel: head matrix without tile layout");
    {
        StepPhase p{};
        p.kind = PK_EMBED;
        ph.push_back(p);
    }
    for (int l = 0; l < c.layers; l++) {
        const LayerW &L = m->layers[l];
        const float *prev_post = (gemma && l > 0) ? m->layers[l - 1].post_ffw : nullptr;
        const float *q, *k, *v;
        int ldq, ldkv;
        std::vector<StepSeg> qkv;
        if (L.qkv.valid()) {
            if (!tiled_ok(L.qkv)) return fail(LLMDOT_E_UNSUPPORTED, "step kernel: qkv without tile layout");
            const int ld = qDim + 2 * kvDim;
            qkv.push_back(seg(L.qkv, nullptr, w.qkv, ld));
            q = w.qkv;
            k = w.qkv + qDim;
            v = w.qkv + qDim + kvDim;
            ldq = ldkv = ld;
        } else {
            if (!tiled_ok(L.q) || !tiled_ok(L.k) || !tiled_ok(L.v))
                return fail(LLMDOT_E_UNSUPPORTED, "step kernel: q/k/v without tile layout");
            qkv.push_back(seg(L.q, nullptr, w.q, qDim));
            qkv.push_back(seg(L.k, nullptr, w.k, kvDim));
            qkv.push_back(seg(L.v, nullptr, w.v, kvDim));
            q = w.q;
            k = w.k;
            v = w.v;
            ldq = qDim;
            ldkv = kvDim;
        }
        LLMDOT_TRY(matvec(SM_STORE, qkv, H, 1, w.h, H, L.attn_norm, prev_post, nullptr, 0));
        for (int kind : {PK_SCORES, PK_PV}) {
            StepPhase p{};
            p.kind = kind;
            p.layer = l;
            p.q = q;
            p.k = k;
            p.v = v;
            p.ldq = ldq;
            p.ldkv = ldkv;
            p.out = w.attn;
            p.ldo = qDim;
            ph.push_back(p);
        }
        if (!tiled_ok(L.o) || !tiled_ok(L.gate) || !tiled_ok(L.up) || !tiled_ok(L.down) || L.gate.type != L.up.type)
            return fail(LLMDOT_E_UNSUPPORTED, "step kernel: o/ffn matrices without tile layout");
        LLMDOT_TRY(matvec(SM_ADD, {seg(L.o, nullptr, w.h, H)}, qDim, 1, w.attn, qDim, nullptr, nullptr, prev_post, 0));
        const float *post_attn = (gemma && L.post_attn) ? L.post_attn : nullptr;
        LLMDOT_TRY(matvec(c.ffn_type == 2 ? SM_GELU : SM_SILU, {seg(L.gate, &L.up, w.gate, c.ffn)}, H, 2, w.h, H,
                          L.ffn_norm ? L.ffn_norm : L.attn_norm, post_attn, nullptr, 0));
        LLMDOT_TRY(matvec(SM_ADD, {seg(L.down, nullptr, w.h, H)}, c.ffn, 1, w.gate, c.ffn, nullptr, nullptr, post_attn,
                          0));
    }
    const float *last_post = (gemma && c.layers > 0) ? m->layers[c.layers - 1].post_ffw : nullptr;
    LLMDOT_TRY(matvec(SM_HEAD, {seg(head, nullptr, w.logits, c.vocab)}, H, 1, w.h, H, m->out_norm, last_post, nullptr,
                      PF_LAST_ONLY));

    // scratch region: the largest phase input or attention staging
    const int G = c.heads / c.heads_kv, hd = c.head_dim;
    size_t xreg = 0;
    for (const StepPhase &p : ph) {
        if (p.kind != PK_MATVEC) continue;
        const size_t xsz = (size_t)p.nsb * 1024 * batch;
        xreg = std::max(xreg, (p.need_q4 ? xsz : 0) + (p.need_q6 ? xsz : 0) + (size_t)batch * p.nsb * 8 * 4 +
                                  (p.need_q4 ? (size_t)batch * p.nsb * 32 * 4 : 0));
    }
    for (size_t esz : {(size_t)2, (size_t)4}) {
        const size_t stride = hd + (esz == 2 ? 2 : 1);
        xreg = std::max(xreg, align16(KV_PAGE * stride * esz) + (size_t)G * hd * 4 + (size_t)G * 4);
        xreg = std::max(xreg, align16(KV_PAGE * hd * esz) + (size_t)G * KV_PAGE * 4 + (size_t)G * 4);
    }
    xreg = align16(xreg);
    int ring = 0;
    for (int r = 3; r >= 2 && !ring; r--)
        if (step_fixed_smem(batch, r) + xreg <= (size_t)optin) ring = r;
    if (!ring) return fail(LLMDOT_E_UNSUPPORTED, "step kernel: shared memory plan does not fit");
    if ((int)ph.size() > PH_MAX) return fail(LLMDOT_E_UNSUPPORTED, "step kernel: too many layers");
    P.batch = batch;
    P.gen = w.gen;
    P.nph = (int)ph.size();
    P.ring = ring;
    P.grid = grid;
    P.smem = step_fixed_smem(batch, ring) + xreg;
    {
        void *k = pick_kernel(batch);
        // the attribute is per kernel, shared by every model's plan: allow the device maximum
        LLMDOT_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
        int nb = 0;
        LLMDOT_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k, ST, P.smem));
        if (nb < 1) return fail(LLMDOT_E_UNSUPPORTED, "step kernel: does not fit one SM");
    }
    LLMDOT_CUDA_TRY(cudaMalloc(&P.d_ph, sizeof(StepPhase) * ph.size()));
    LLMDOT_CUDA_TRY(cudaMalloc(&P.bar, sizeof(unsigned) * 2));
    LLMDOT_CUDA_TRY(cudaMalloc(&P.keys, sizeof(unsigned long long) * 2 * batch));
    LLMDOT_CUDA_TRY(cudaMemcpy(P.d_ph, ph.data(), sizeof(StepPhase) * ph.size(), cudaMemcpyHostToDevice));
    LLMDOT_CUDA_TRY(cudaMemset(P.bar, 0, sizeof(unsigned) * 2));
    LLMDOT_CUDA_TRY(cudaMemset(P.keys, 0, sizeof(unsigned long long) * 2 * batch));
    return LLMDOT_OK;
}

static StepPlan *get_plan(llmdot_model *m, int batch)
{
    if (!m->step_cache) m->step_cache = new StepCache();
    auto &plans = m->step_cache->plans;
    for (size_t i = 0; i < plans.size();)
        if (plans[i].gen != m->ws.gen) {  // built on buffers that were reallocated since
            free_plan(plans[i]);
            plans.erase(plans.begin() + i);
        } else {
            i++;
        }
    for (auto &p : plans)
        if (p.batch == batch) return &p;
    StepPlan P;
    P.status = build_plan(m, batch, P);
    if (P.status != LLMDOT_OK) free_plan(P);
    P.batch = batch;
    P.gen = m->ws.gen;
    plans.push_back(P);
    return &plans.back();
}

bool step_kernel_supported(llmdot_model *m, int batch)
{
    if (!m->use_step_kernel || !m->use_fast_gemv || m->tp > 1 || batch < 1 || batch > NV_MAX) return false;
    if (ensure_workspace(m, batch) != LLMDOT_OK) return false;
    return get_plan(m, batch)->status == LLMDOT_OK;
}

int launch_step_kernel(llmdot_model *m, int batch, int kv_type, int n_steps, const int32_t *forced, cudaStream_t st,
                       unsigned long long *trace)
{
    if (n_steps <= 0) return LLMDOT_OK;
    LLMDOT_TRY(ensure_workspace(m, batch));
    StepPlan *P = get_plan(m, batch);
    if (P->status != LLMDOT_OK) return fail(P->status, "step kernel unavailable for this model / batch");
    const llmdot_config &c = m->cfg;
    Workspace &w = m->ws;
    StepArgs a{};
    a.ph = P->d_ph;
    a.nph = P->nph;
    a.n_steps = n_steps;
    a.nv = batch;
    a.emb = m->emb.raw;
    a.emb_type = m->emb.type;
    a.emb_rbytes = m->emb.rbytes;
    a.vocab = c.vocab;
    a.emb_scale = c.emb_scale;
    a.emb_apply = c.emb_scale != 1.0f;
    a.eps = c.eps;
    AttnShape &sh = a.sh;
    sh.heads = c.heads;
    sh.heads_kv = c.heads_kv;
    sh.head_dim = c.head_dim;
    sh.max_ctx = m->max_ctx;
    sh.sliding_window = c.sliding_window;
    sh.has_cap = c.has_attn_cap;
    sh.cap = c.attn_cap;
    sh.inv_sqrt_hd = 1.0f / sqrtf((float)c.head_dim);
    sh.rope_half = m->rope_half;
    a.cos_t = m->cos_t;
    a.sin_t = m->sin_t;
    a.h = w.h;
    a.ldh = c.hidden;
    a.scores = w.scores;
    a.part_m = w.part_m;
    a.part_s = w.part_s;
    a.part_o = w.part_o;
    a.counters = w.counters;
    a.keys = P->keys;
    a.next = w.next;
    a.pos = w.pos;
    a.hist = w.hist;
    a.hist_step = w.hist_step;
    a.forced = forced;
    a.views = w.views;
    a.err = w.err;
    a.bar = P->bar;
    a.has_final_cap = c.has_final_cap;
    a.final_cap = c.final_cap;
    a.trace = trace;
    a.ring = P->ring;
    a.evict_first = getenv("LLMDOT_STEP_NO_EVICT_FIRST") == nullptr;
    a.kv_f16 = kv_type == LLMDOT_KV_F16;
    void *k = pick_kernel(batch);
    if (!k) return fail(LLMDOT_E_UNSUPPORTED, "step kernel: no instance for this batch");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(P->grid);
    cfg.blockDim = dim3(ST);
    cfg.dynamicSmemBytes = P->smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident: the grid barriers rely on it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {&a};
    LLMDOT_CUDA_TRY(cudaLaunchKernelExC(&cfg, k, args));
    return LLMDOT_OK;
}

int step_kernel_shape(llmdot_model *m, int batch, int *n_phases, int *n_cta, int *kinds, int max_kinds)
{
    LLMDOT_TRY(ensure_workspace(m, batch));
    StepPlan *P = get_plan(m, batch);
    if (P->status != LLMDOT_OK) return fail(P->status, "step kernel unavailable for this model / batch");
    *n_phases = P->nph;
    *n_cta = P->grid;
    if (kinds) {
        std::vector<StepPhase> ph(P->nph);
        LLMDOT_CUDA_TRY(cudaMemcpy(ph.data(), P->d_ph, sizeof(StepPhase) * P->nph, cudaMemcpyDeviceToHost));
        for (int i = 0; i < P->nph && i < max_kinds; i++) kinds[i] = ph[i].kind == PK_MATVEC ? 10 + ph[i].mode : ph[i].kind;
    }
    return LLMDOT_OK;
}

int step_kernel_reset(llmdot_model *m, cudaStream_t st)
{
    if (!m->step_cache) return LLMDOT_OK;
    for (auto &p : m->step_cache->plans) {
        if (p.bar) LLMDOT_CUDA_TRY(cudaMemsetAsync(p.bar, 0, sizeof(unsigned) * 2, st));
        if (p.keys) LLMDOT_CUDA_TRY(cudaMemsetAsync(p.keys, 0, sizeof(unsigned long long) * 2 * p.batch, st));
    }
    const llmdot_config &c = m->cfg;
    if (m->ws.counters)
        LLMDOT_CUDA_TRY(cudaMemsetAsync(m->ws.counters, 0, sizeof(int) * m->ws.batch * c.heads_kv, st));
    return LLMDOT_OK;
}

}  // namespace llmdot
