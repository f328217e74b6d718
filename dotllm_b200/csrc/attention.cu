// attention.cu -- GQA decode attention over the paged KV cache, with RoPE and the KV append.
//
// Reference: InferenceEngine.AttentionForward (src/Llmdot.Core/Inference/InferenceEngine.cs:304-450)
// with VectorMath.Softmax (src/Llmdot.Core/Tensors/Numeric/VectorMath.cs:215-258).
// The reference's softmax evaluates ExpApprox(s - max) against the GLOBAL max of the
// window (an approximation whose error is up to ~18 % for some arguments, so an
// online/rescaled softmax would not reproduce it).  The device therefore runs two kernels
// over pages of KV_PAGE positions, one CTA per (page, kv head, session):
//   1. scores: RoPE of q (and of the new k, which the CTA owning the current position appends
//      to the cache together with v), s = (q . k) * 1/sqrt(hd), softcap, per-page max;
//   2. p = exp(s - M) with M the window max, per-page sum and sum p*V; the last CTA of each
//      (session, kv head) to finish combines the pages and scales by 1/sum.
// "Vector lane" vs "tail" (ExpApprox/TanhApprox vs MathF.Exp/Tanh) is decided by the
// position's index inside the window, exactly as the reference's 8-wide loops do.
// Both kernels stage their KV page in shared memory before waiting on the previous kernel
// (programmatic dependent launch): pages of earlier positions are constant during a step.
#include "attention.cuh"

#include <stdlib.h>

#include <algorithm>
#include <cooperative_groups.h>

namespace llmdot {

namespace cg = cooperative_groups;

template <typename T> struct KvT;
template <> struct KvT<float> {
    static __device__ __forceinline__ float ld(const float *p) { return *p; }
    static __device__ __forceinline__ float st(float v) { return v; }
};
template <> struct KvT<__half> {
    static __device__ __forceinline__ float ld(const __half *p) { return __half2float(*p); }
    static __device__ __forceinline__ __half st(float v) { return __float2half_rn(v); }
};

__device__ __forceinline__ void window(int p, int sw, int &start, int &seq_len)
{
    seq_len = p + 1;
    start = sw > 0 ? max(0, seq_len - sw) : 0;
}

// Copy positions [j0, j1) of one page (KV_PAGE x hd elements, contiguous) into shared memory
// rows of `stride` elements, 16 bytes at a time.
template <typename T>
__device__ __forceinline__ void stage_page(T *dst, const T *src, int hd, int stride, int j0, int j1)
{
    constexpr int E = 16 / sizeof(T);  // elements per 16 bytes
    const int per_row = hd / E;
    for (int i = threadIdx.x; i < (j1 - j0) * per_row; i += blockDim.x) {
        const int j = j0 + i / per_row, c = (i % per_row) * E;
        const uint4 v = *(const uint4 *)(src + (size_t)j * hd + c);
        const T *pv = (const T *)&v;
#pragma unroll
        for (int e = 0; e < E; e++) dst[j * stride + c + e] = pv[e];
    }
}

// ---------------------------------------------------------------- kernel 1: RoPE, append, scores
template <typename T>
__global__ void __launch_bounds__(256) attn_scores_kernel(const float *__restrict__ q, int ldq, const float *__restrict__ k,
                                                          const float *__restrict__ v, int ldkv,
                                                          const int32_t *__restrict__ pos,
                                                          const float *__restrict__ cos_t, const float *__restrict__ sin_t,
                                                          const KvView *__restrict__ views, int layer, AttnShape sh,
                                                          float *__restrict__ scores, float *__restrict__ part_m,
                                                          int appended)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    const int chunk = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int hd = sh.head_dim, half = sh.rope_half, G = sh.heads / sh.heads_kv, nchunk = sh.max_ctx / KV_PAGE;
    const int p = pos[b];  // positions change only between steps
    int start, seq_len;
    window(p, sh.sliding_window, start, seq_len);
    const int s0 = chunk * KV_PAGE;
    if (s0 >= seq_len || s0 + KV_PAGE <= start) {
        pdl_launch();
        return;
    }
    const int stride = hd + (sizeof(T) == 2 ? 2 : 1);  // odd word stride: no bank conflicts across positions
    T *ks = (T *)smem_raw;                                            // [KV_PAGE][stride]
    float *qs = (float *)(smem_raw + (size_t)KV_PAGE * stride * sizeof(T));  // [G][hd]
    uint32_t *mk = (uint32_t *)(qs + G * hd);                         // [G]
    const KvView vw = views[b];
    const int page = vw.pages[chunk];
    const size_t head_off = ((size_t)page * sh.heads_kv + kvh) * KV_PAGE * hd;
    T *kg = (T *)vw.k + (size_t)layer * vw.layer_stride + head_off;
    T *vg = (T *)vw.v + (size_t)layer * vw.layer_stride + head_off;
    const int jlo = max(start - s0, 0), jhi = min(seq_len - s0, KV_PAGE);
    const bool has_new = !appended && p >= s0 && p < s0 + KV_PAGE;
    // earlier positions of the page are constant: stage them before the dependency wait (with
    // `appended`, the previous kernel wrote positions of this step: stage after the wait)
    if (!appended) stage_page<T>(ks, kg, hd, stride, jlo, has_new ? p - s0 : jhi);
    pdl_launch();
    pdl_wait();
    if (appended) stage_page<T>(ks, kg, hd, stride, jlo, jhi);
    const float *cs = cos_t + (size_t)p * half, *sn = sin_t + (size_t)p * half;
    // RoPE of the G query heads (TensorOps.ApplyRoPE, half-split pairs)
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
        const int hg = i / hd, d = i % hd;
        const float *x = q + (size_t)b * ldq + (size_t)(kvh * G + hg) * hd;
        float r;
        if (d < half) r = __fsub_rn(__fmul_rn(x[d], cs[d]), __fmul_rn(x[d + half], sn[d]));
        else if (d < 2 * half) r = __fadd_rn(__fmul_rn(x[d - half], sn[d - half]), __fmul_rn(x[d], cs[d - half]));
        else r = x[d];
        qs[i] = r;
    }
    for (int i = threadIdx.x; i < G; i += blockDim.x) mk[i] = 0u;
    if (has_new) {
        // RoPE of the new key, then K/V cache append (InferenceEngine.cs:375-382)
        const float *kx = k + (size_t)b * ldkv + (size_t)kvh * hd;
        const float *vx = v + (size_t)b * ldkv + (size_t)kvh * hd;
        const int slot = p - s0;
        for (int d = threadIdx.x; d < hd; d += blockDim.x) {
            float r;
            if (d < half) r = __fsub_rn(__fmul_rn(kx[d], cs[d]), __fmul_rn(kx[d + half], sn[d]));
            else if (d < 2 * half) r = __fadd_rn(__fmul_rn(kx[d - half], sn[d - half]), __fmul_rn(kx[d], cs[d - half]));
            else r = kx[d];
            const T kt = KvT<T>::st(r);
            kg[(size_t)slot * hd + d] = kt;
            ks[slot * stride + d] = kt;
            vg[(size_t)slot * hd + d] = KvT<T>::st(vx[d]);
        }
    }
    __syncthreads();
    const int len = seq_len - start, nvec = len - len % 8;
    const float inv_cap = sh.has_cap ? __fdiv_rn(1.0f, sh.cap) : 0.0f;
    for (int idx = threadIdx.x; idx < G * KV_PAGE; idx += blockDim.x) {
        const int hg = idx / KV_PAGE, j = idx % KV_PAGE, s = s0 + j;
        if (j < jlo || j >= jhi) continue;
        const T *kr = ks + j * stride;
        const float *qh = qs + hg * hd;
        float dot = 0.0f;
        for (int d = 0; d < hd; d++) dot = fmaf(qh[d], KvT<T>::ld(kr + d), dot);
        float sc = __fmul_rn(dot, sh.inv_sqrt_hd);
        if (sh.has_cap) sc = softcap_ref(sc, sh.cap, inv_cap, (s - start) < nvec);
        scores[((size_t)b * sh.heads + kvh * G + hg) * sh.max_ctx + s] = sc;
        atomicMax(mk + hg, float_key(sc));
    }
    __syncthreads();
    for (int hg = threadIdx.x; hg < G; hg += blockDim.x)
        part_m[((size_t)b * sh.heads + kvh * G + hg) * nchunk + chunk] = key_float(mk[hg]);
}

// ---------------------------------------------------------------- kernel 2: exp, PV, combine
template <typename T>
__global__ void __launch_bounds__(256) attn_pv_kernel(const int32_t *__restrict__ pos, const KvView *__restrict__ views,
                                                      int layer, AttnShape sh, const float *__restrict__ scores,
                                                      const float *__restrict__ part_m, float *__restrict__ part_s,
                                                      float *__restrict__ part_o, int *__restrict__ counters,
                                                      float *__restrict__ out, int ldo, int appended)
{
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ int last;
    const int chunk = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int hd = sh.head_dim, G = sh.heads / sh.heads_kv, nchunk = sh.max_ctx / KV_PAGE;
    const int p = pos[b];
    int start, seq_len;
    window(p, sh.sliding_window, start, seq_len);
    const int s0 = chunk * KV_PAGE;
    if (s0 >= seq_len || s0 + KV_PAGE <= start) {
        pdl_launch();
        return;
    }
    T *vs = (T *)smem_raw;                                                  // [KV_PAGE][hd]
    float *ps = (float *)(smem_raw + (size_t)KV_PAGE * hd * sizeof(T));     // [G][KV_PAGE]
    float *mx = ps + G * KV_PAGE;                                           // [G]
    const KvView vw = views[b];
    const int page = vw.pages[chunk];
    const T *vg = (const T *)vw.v + (size_t)layer * vw.layer_stride + ((size_t)page * sh.heads_kv + kvh) * KV_PAGE * hd;
    const int jlo = max(start - s0, 0), jhi = min(seq_len - s0, KV_PAGE);
    const bool has_new = p >= s0 && p < s0 + KV_PAGE;
    if (!appended) stage_page<T>(vs, vg, hd, hd, jlo, has_new ? p - s0 : jhi);
    pdl_launch();
    pdl_wait();
    if (appended) stage_page<T>(vs, vg, hd, hd, jlo, jhi);
    else if (has_new) stage_page<T>(vs, vg, hd, hd, p - s0, p - s0 + 1);  // appended by kernel 1
    const int len = seq_len - start, nvec = len - len % 8;
    const int c0 = start / KV_PAGE, c1 = (seq_len - 1) / KV_PAGE;
    for (int hg = threadIdx.x; hg < G; hg += blockDim.x) {
        const float *pm = part_m + ((size_t)b * sh.heads + kvh * G + hg) * nchunk;
        float m = -INFINITY;
        for (int c = c0; c <= c1; c++) m = fmaxf(m, pm[c]);
        mx[hg] = m;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * KV_PAGE; idx += blockDim.x) {
        const int hg = idx / KV_PAGE, j = idx % KV_PAGE, s = s0 + j;
        float pr = 0.0f;
        if (j >= jlo && j < jhi) {
            const float d = __fsub_rn(scores[((size_t)b * sh.heads + kvh * G + hg) * sh.max_ctx + s], mx[hg]);
            pr = (s - start) < nvec ? exp_approx(d) : expf(d);
        }
        ps[idx] = pr;
    }
    __syncthreads();
    const size_t hbase = ((size_t)b * sh.heads + kvh * G) * nchunk;
    for (int hg = threadIdx.x >> 5; hg < G; hg += blockDim.x >> 5) {
        float t = 0.0f;
        for (int j = threadIdx.x & 31; j < KV_PAGE; j += 32) t += ps[hg * KV_PAGE + j];
        t = warp_sum(t);
        if ((threadIdx.x & 31) == 0) part_s[hbase + (size_t)hg * nchunk + chunk] = t;
    }
    for (int idx = threadIdx.x; idx < G * hd; idx += blockDim.x) {
        const int hg = idx / hd, d = idx % hd;
        const float *pp = ps + hg * KV_PAGE;
        float acc = 0.0f;
        for (int j = jlo; j < jhi; j++) acc = fmaf(pp[j], KvT<T>::ld(vs + j * hd + d), acc);
        part_o[((hbase + (size_t)hg * nchunk) + chunk) * hd + d] = acc;
    }
    // the last page of this (session, kv head) to finish combines all pages
    __threadfence();
    __syncthreads();
    int *cnt = counters + (size_t)b * sh.heads_kv + kvh;
    if (threadIdx.x == 0) last = atomicAdd(cnt, 1) == (c1 - c0);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int idx = threadIdx.x; idx < G * hd; idx += blockDim.x) {
        const int hg = idx / hd, d = idx % hd;
        const size_t hb = hbase + (size_t)hg * nchunk;
        float sum = 0.0f, o = 0.0f;
        for (int c = c0; c <= c1; c++) {
            sum += __ldcg(part_s + hb + c);
            o += __ldcg(part_o + (hb + c) * hd + d);
        }
        out[(size_t)b * ldo + (size_t)(kvh * G + hg) * hd + d] = __fmul_rn(o, __fdiv_rn(1.0f, sum));
    }
    if (threadIdx.x == 0) *cnt = 0;  // ready for the next layer / step
}

// RoPE of the new keys and the K/V append of every row, ahead of the attention kernels: used
// when several rows of one step belong to the same session (a prompt chunk), so that row i
// sees the keys of rows < i (InferenceEngine.cs:375-382).
template <typename T>
__global__ void append_kv_kernel(const float *__restrict__ k, const float *__restrict__ v, int ldkv,
                                 const int32_t *__restrict__ pos, const float *__restrict__ cos_t,
                                 const float *__restrict__ sin_t, const KvView *__restrict__ views, int layer,
                                 AttnShape sh)
{
    pdl_launch();
    pdl_wait();
    const int kvh = blockIdx.x, b = blockIdx.y, hd = sh.head_dim, half = sh.rope_half;
    const int p = pos[b];
    const KvView vw = views[b];
    const int page = vw.pages[p / KV_PAGE], slot = p % KV_PAGE;
    const size_t off = (size_t)layer * vw.layer_stride + (((size_t)page * sh.heads_kv + kvh) * KV_PAGE + slot) * hd;
    const float *kx = k + (size_t)b * ldkv + (size_t)kvh * hd, *vx = v + (size_t)b * ldkv + (size_t)kvh * hd;
    const float *cs = cos_t + (size_t)p * half, *sn = sin_t + (size_t)p * half;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float r;
        if (d < half) r = __fsub_rn(__fmul_rn(kx[d], cs[d]), __fmul_rn(kx[d + half], sn[d]));
        else if (d < 2 * half) r = __fadd_rn(__fmul_rn(kx[d - half], sn[d - half]), __fmul_rn(kx[d], cs[d - half]));
        else r = kx[d];
        ((T *)vw.k)[off + d] = KvT<T>::st(r);
        ((T *)vw.v)[off + d] = KvT<T>::st(vx[d]);
    }
}

// ---------------------------------------------------------------- one-kernel cluster attention
// One thread-block cluster of C CTAs per (kv head, session); rank r of the cluster takes an even
// share of the window's pages.  Each CTA streams its K pages, then its V pages, through two
// shared-memory slots with cp.async (rows padded by 16 bytes: 16-byte reads of 8 consecutive
// rows hit distinct bank groups), keeping the scores of all its positions in shared memory.
// The window max (the reference's softmax subtracts the GLOBAL max before ExpApprox) and the
// final sums cross the cluster through distributed shared memory: every rank pushes its per-head
// maxima into every rank's shared memory and its partial P.V slices to the rank that finishes
// them, each exchange closed by one cluster barrier (release / acquire); the output is reduced
// over the ranks in rank order, so the result does not depend on scheduling.  No global scratch,
// no atomics, one launch per layer.
constexpr int AC_THREADS = 256;
constexpr int AC_SBUF = 32 * 1024;  // bytes of scores per CTA (G heads x pages x 64 positions)

struct AcLayout {
    int rstride, mbar, ring, sbuf, qs, kn, pv, lo, stat, xmax, xsum, xpart, total;  // rstride: bytes per staged row
};
// slice of the G * hd outputs that rank q of a C-CTA cluster finishes
__host__ __device__ inline int ac_slice(int G, int hd, int C) { return (G * hd + C - 1) / C; }
__host__ __device__ inline AcLayout ac_layout(int hd, int esz, int G, int maxp, int slots, int C)
{
    AcLayout L;
    int o = 0;
    L.rstride = hd * esz + 16;
    L.mbar = o;  // one mbarrier per slot
    o += (slots * 8 + 15) / 16 * 16;
    L.ring = o;
    o += slots * KV_PAGE * L.rstride;
    L.sbuf = o;  // [G][maxp * KV_PAGE] scores, then probabilities
    o += G * maxp * KV_PAGE * 4;
    L.qs = o;  // [G][hd] roped queries
    o += G * hd * 4;
    L.kn = o;  // new k row, new v row (cache type), 16-byte rounded each
    o += 2 * ((hd * esz + 15) / 16 * 16);
    L.pv = o;  // per-group partial P.V: at most AC_THREADS x 8 floats
    o += AC_THREADS * 8 * 4;
    L.lo = o;  // [G][hd] this CTA's P.V
    o += G * hd * 4;
    L.stat = o;  // lmax[G], M[G], lsum[G]
    o += (3 * G * 4 + 15) / 16 * 16;
    L.xmax = o;  // [C][G] every rank's per-head maxima (pushed by the ranks)
    o += (C * G * 4 + 15) / 16 * 16;
    L.xsum = o;  // [C][G] every rank's per-head sums
    o += (C * G * 4 + 15) / 16 * 16;
    L.xpart = o;  // [C][slice] every rank's P.V partials of this rank's output slice
    o += (C * ac_slice(G, hd, C) * 4 + 15) / 16 * 16;
    L.total = o;
    return L;
}

// Bounded waits of the attention kernel: a wait that gives up sets this flag (read by
// attention_timeout_check) and the kernel finishes without valid output.
constexpr unsigned long long ATTN_WAIT_NS = 2000000000ull;
__device__ int g_attn_timeout;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool ac_mbar_wait(uint64_t *b, uint32_t parity)
{
    uint32_t ok = 0;
    uint64_t t0 = 0;
    for (int it = 0;; it++) {
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(smem_u32(b)), "r"(parity)
            : "memory");
        if (ok) return true;
        uint64_t now;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
        if (it == 0) t0 = now;
        else if (now - t0 > ATTN_WAIT_NS) return false;
    }
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}

// 16 bytes of cache elements as floats
__device__ __forceinline__ void chunk_f32(const uint4 &u, const float *, float (&o)[4]) 
{
    o[0] = __uint_as_float(u.x);
    o[1] = __uint_as_float(u.y);
    o[2] = __uint_as_float(u.z);
    o[3] = __uint_as_float(u.w);
}
__device__ __forceinline__ void chunk_f32(const uint4 &u, const __half *, float (&o)[8])
{
    const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
    for (int e = 0; e < 4; e++) {
        const float2 f = __half22float2(h[e]);
        o[2 * e] = f.x;
        o[2 * e + 1] = f.y;
    }
}

template <typename T>
__global__ void __launch_bounds__(AC_THREADS) attn_cluster_kernel(const float *__restrict__ q, int ldq,
                                                                  const float *__restrict__ k, const float *__restrict__ v,
                                                                  int ldkv, const int32_t *__restrict__ pos,
                                                                  const float *__restrict__ cos_t,
                                                                  const float *__restrict__ sin_t,
                                                                  const KvView *__restrict__ views, int layer, AttnShape sh,
                                                                  float *__restrict__ out, int ldo, int appended, int maxp,
                                                                  int slots)
{
    constexpr int E = 16 / sizeof(T);  // cache elements per 16-byte chunk
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(16) uint8_t smem[];
    const int C = (int)cluster.num_blocks(), rank = (int)cluster.block_rank();
    const int kvh = blockIdx.y, b = blockIdx.z, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hd = sh.head_dim, half = sh.rope_half, G = sh.heads / sh.heads_kv, cpr = hd / E;
    const AcLayout L = ac_layout(hd, (int)sizeof(T), G, maxp, slots, C);
    uint8_t *ring = smem + L.ring;
    uint64_t *mbar = (uint64_t *)(smem + L.mbar);
    if (tid < slots)
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(mbar + tid)), "r"(AC_THREADS) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    // cluster barrier 0: every rank has started (its shared memory may receive pushes); waited
    // on just before the first push
    __syncwarp();
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    float *sbuf = (float *)(smem + L.sbuf), *qs = (float *)(smem + L.qs), *pv = (float *)(smem + L.pv);
    float *lmax = (float *)(smem + L.stat), *lsum = lmax + 2 * G;
    T *kn = (T *)(smem + L.kn), *vn = (T *)(smem + L.kn + (hd * sizeof(T) + 15) / 16 * 16);
    const int sstride = maxp * KV_PAGE;  // scores per head in sbuf

    // positions and page tables are constant during a step: read before the dependency wait
    const int p = pos[b];
    int start, seq_len;
    window(p, sh.sliding_window, start, seq_len);
    const int c0 = start / KV_PAGE, np = (seq_len - 1) / KV_PAGE - c0 + 1;
    const int pg_lo = c0 + (int)((long long)rank * np / C), n = c0 + (int)((long long)(rank + 1) * np / C) - pg_lo;
    const KvView vw = views[b];
    const size_t lbase = (size_t)layer * vw.layer_stride;
    // stream f = 0..2n-1: K pages 0..n-1 then V pages 0..n-1, page f in slot f % slots; every
    // thread's copies of a page arrive on the slot's mbarrier (cp.async.mbarrier.arrive.noinc).
    // Thread tid copies 16-byte chunk tid % cpr of rows tid / cpr, + rpp, ... (no division per copy)
    const int rpp = AC_THREADS / cpr, crow = tid / cpr, cchunk = tid % cpr;
    auto issue = [&](int f) {
        const int i = f < n ? f : f - n;
        const int s0 = (pg_lo + i) * KV_PAGE, jlo = max(start - s0, 0), jhi = min(seq_len - s0, KV_PAGE);
        const T *src = (const T *)(f < n ? vw.k : vw.v) + lbase +
                       ((size_t)vw.pages[pg_lo + i] * sh.heads_kv + kvh) * KV_PAGE * hd;
        const int slot = f % slots;
        uint8_t *dst = ring + (size_t)slot * KV_PAGE * L.rstride;
        if (crow < rpp)
            for (int j = jlo + crow; j < jhi; j += rpp)
                cp_async16(dst + j * L.rstride + cchunk * 16, src + (size_t)j * hd + cchunk * E);
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(mbar + slot)) : "memory");
    };
    bool ok = true;
    auto consume = [&](int f) -> uint8_t * {  // wait until page f is in its slot
        const int slot = f % slots;
        if (ok && !ac_mbar_wait(mbar + slot, (uint32_t)(f / slots) & 1u)) {
            ok = false;
            atomicExch(&g_attn_timeout, 1);
        }
        __syncthreads();
        return ring + (size_t)slot * KV_PAGE * L.rstride;
    };
    const int first = min(slots, 2 * n);  // pages in flight from the start
    // earlier positions are constant: fetch before the wait (with `appended`, the previous
    // kernel wrote rows of this step, so fetch after it)
    if (!appended)
        for (int f = 0; f < first; f++) issue(f);
    pdl_launch();
    pdl_wait();
    if (appended)
        for (int f = 0; f < first; f++) issue(f);

    const float *cs = cos_t + (size_t)p * half, *sn = sin_t + (size_t)p * half;
    for (int i = tid; i < G * hd; i += AC_THREADS) {  // RoPE of the G query heads (half-split pairs)
        const int hg = i / hd, d = i % hd;
        const float *x = q + (size_t)b * ldq + (size_t)(kvh * G + hg) * hd;
        float r;
        if (d < half) r = __fsub_rn(__fmul_rn(x[d], cs[d]), __fmul_rn(x[d + half], sn[d]));
        else if (d < 2 * half) r = __fadd_rn(__fmul_rn(x[d - half], sn[d - half]), __fmul_rn(x[d], cs[d - half]));
        else r = x[d];
        qs[i] = r;
    }
    // the CTA whose pages hold the current position ropes the new key and appends k and v
    const bool has_new = !appended && n > 0 && p >= pg_lo * KV_PAGE && p < (pg_lo + n) * KV_PAGE;
    if (has_new) {
        const float *kx = k + (size_t)b * ldkv + (size_t)kvh * hd, *vx = v + (size_t)b * ldkv + (size_t)kvh * hd;
        const size_t row = lbase + (((size_t)vw.pages[p / KV_PAGE] * sh.heads_kv + kvh) * KV_PAGE + p % KV_PAGE) * hd;
        for (int d = tid; d < hd; d += AC_THREADS) {
            float r;
            if (d < half) r = __fsub_rn(__fmul_rn(kx[d], cs[d]), __fmul_rn(kx[d + half], sn[d]));
            else if (d < 2 * half) r = __fadd_rn(__fmul_rn(kx[d - half], sn[d - half]), __fmul_rn(kx[d], cs[d - half]));
            else r = kx[d];
            kn[d] = KvT<T>::st(r);
            vn[d] = KvT<T>::st(vx[d]);
            ((T *)vw.k)[row + d] = kn[d];
            ((T *)vw.v)[row + d] = vn[d];
        }
    }
    __syncthreads();

    const int len = seq_len - start, nvec = len - len % 8;
    const float inv_cap = sh.has_cap ? __fdiv_rn(1.0f, sh.cap) : 0.0f;
    // threads per dot product: 256 threads over G x 64 dots
    const int LTPD = G >= 4 ? 0 : (G == 2 ? 1 : 2), TPD = 1 << LTPD;
    // ---- pass 1: scores of this CTA's positions
    for (int f = 0; f < n; f++) {
        uint8_t *slot = consume(f);
        const int s0 = (pg_lo + f) * KV_PAGE, jlo = max(start - s0, 0), jhi = min(seq_len - s0, KV_PAGE);
        if (has_new && p >= s0 && p < s0 + KV_PAGE) {
            for (int d = tid; d < hd; d += AC_THREADS) ((T *)(slot + (p - s0) * L.rstride))[d] = kn[d];
            __syncthreads();
        }
        for (int base = 0; base < G * KV_PAGE * TPD; base += AC_THREADS) {
            const int idx = base + tid, dot = idx >> LTPD, part = idx & (TPD - 1), hg = dot / KV_PAGE, j = dot % KV_PAGE;
            const bool valid = idx < G * KV_PAGE * TPD && j >= jlo && j < jhi;
            float acc = 0.0f;
            if (valid) {
                const uint8_t *kr = slot + j * L.rstride;
                const float *qh = qs + hg * hd;
                for (int ch = part; ch < cpr; ch += TPD) {
                    float kf[E];
                    chunk_f32(*(const uint4 *)(kr + ch * 16), (const T *)nullptr, kf);
#pragma unroll
                    for (int e = 0; e < E; e++) acc = fmaf(qh[ch * E + e], kf[e], acc);
                }
            }
            if (TPD > 1) acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            if (TPD > 2) acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            if (valid && part == 0) {
                float sc = __fmul_rn(acc, sh.inv_sqrt_hd);
                if (sh.has_cap) sc = softcap_ref(sc, sh.cap, inv_cap, (s0 + j - start) < nvec);
                sbuf[hg * sstride + f * KV_PAGE + j] = sc;
            }
        }
        __syncthreads();  // the slot is free again
        if (f + slots < 2 * n) issue(f + slots);
    }
    // this CTA's max per head: warp hg reduces head hg's positions, and lane r pushes it into
    // rank r's exchange slots; after the barrier every rank holds all ranks' maxima
    const int plo = max(start - pg_lo * KV_PAGE, 0), phi = min(seq_len - pg_lo * KV_PAGE, n * KV_PAGE);  // CTA's positions
    float *xmax = (float *)(smem + L.xmax), *xsum = (float *)(smem + L.xsum), *xpart = (float *)(smem + L.xpart);
    __syncwarp();
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // barrier 0
    for (int hg = warp; hg < G; hg += AC_THREADS / 32) {
        float m = -INFINITY;
        for (int j = plo + lane; j < phi; j += 32) m = fmaxf(m, sbuf[hg * sstride + j]);
        m = warp_max(m);
        if (lane < C) *cluster.map_shared_rank(xmax + rank * G + hg, lane) = m;
    }
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");  // barrier 1
    // p = exp(s - M) in place (ExpApprox in the reference's 8-wide lanes, MathF.Exp in the tail);
    // warp hg takes head hg: the window max over the ranks, the exponentials, this CTA's sum
    for (int hg = warp; hg < G; hg += AC_THREADS / 32) {
        float M = -INFINITY;
        for (int r = 0; r < C; r++) M = fmaxf(M, xmax[r * G + hg]);
        float sum = 0.0f;
        for (int j = plo + lane; j < phi; j += 32) {
            float *sp = sbuf + hg * sstride + j;
            const float d = __fsub_rn(*sp, M);
            const float pr = (pg_lo * KV_PAGE + j - start) < nvec ? exp_approx(d) : expf(d);
            *sp = pr;
            sum += pr;
        }
        sum = warp_sum(sum);
        if (lane == 0) lsum[hg] = sum;
    }
    __syncthreads();
    // ---- pass 2: P.V.  A set of G*hd/E threads covers every (head, 16-byte chunk) once; the NG
    // sets take the positions of each page round robin and are summed in set order at the end.
    const int SET = G * cpr, NG = AC_THREADS / SET, gi = tid / SET, w = tid % SET, hg = w / cpr, ch = w % cpr;
    float acc[E];
#pragma unroll
    for (int e = 0; e < E; e++) acc[e] = 0.0f;
    for (int f = n; f < 2 * n; f++) {
        uint8_t *slot = consume(f);
        const int i = f - n, s0 = (pg_lo + i) * KV_PAGE, jlo = max(start - s0, 0), jhi = min(seq_len - s0, KV_PAGE);
        if (has_new && p >= s0 && p < s0 + KV_PAGE) {
            for (int d = tid; d < hd; d += AC_THREADS) ((T *)(slot + (p - s0) * L.rstride))[d] = vn[d];
            __syncthreads();
        }
        if (gi < NG)
            for (int j = jlo + gi; j < jhi; j += NG) {
                const float pj = sbuf[hg * sstride + i * KV_PAGE + j];
                float vf[E];
                chunk_f32(*(const uint4 *)(slot + j * L.rstride + ch * 16), (const T *)nullptr, vf);
#pragma unroll
                for (int e = 0; e < E; e++) acc[e] = fmaf(pj, vf[e], acc[e]);
            }
        __syncthreads();
        if (f + slots < 2 * n) issue(f + slots);
    }
    if (!ok) asm volatile("cp.async.wait_all;" ::: "memory");  // after a timeout: no copy may still land
    if (gi < NG)
#pragma unroll
        for (int e = 0; e < E; e++) pv[gi * G * hd + hg * hd + ch * E + e] = acc[e];
    __syncthreads();
    // this CTA's P.V partials go to the rank finishing their slice, its sums to every rank
    const int SL = ac_slice(G, hd, C);
    for (int o = tid; o < G * hd; o += AC_THREADS) {
        float sacc = 0.0f;
        for (int g2 = 0; g2 < NG; g2++) sacc += pv[g2 * G * hd + o];
        const int q = o / SL;
        *cluster.map_shared_rank(xpart + rank * SL + (o - q * SL), q) = sacc;
    }
    for (int i = tid; i < C * G; i += AC_THREADS) {
        const int r = i / G, hg = i % G;
        *cluster.map_shared_rank(xsum + rank * G + hg, r) = lsum[hg];
    }
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");  // barrier 2: no access to a peer after it
    // this rank's slice of the (head, dim) outputs, the ranks summed in rank order
    for (int ol = tid; ol < SL; ol += AC_THREADS) {
        const int o = rank * SL + ol;
        if (o >= G * hd) break;
        const int h = o / hd;
        float tot = 0.0f, ssum = 0.0f;
        for (int r = 0; r < C; r++) {
            tot += xpart[r * SL + ol];
            ssum += xsum[r * G + h];
        }
        out[(size_t)b * ldo + (size_t)kvh * G * hd + o] = __fmul_rn(tot, __fdiv_rn(1.0f, ssum));
    }
}

// Cluster size and pages per CTA for a shape, or false when the cluster kernel does not apply
// (a window longer than 8 CTAs' score buffers, or a P.V set wider than the block).
static bool cluster_plan(const AttnShape &sh, int batch, size_t esz, int *C_out, int *maxp_out, int *slots_out,
                         size_t *smem_out)
{
    const int G = sh.heads / sh.heads_kv;
    if (G < 1 || sh.heads % sh.heads_kv || sh.head_dim % 8) return false;
    if (G * sh.head_dim / (int)(16 / esz) > AC_THREADS) return false;
    int npg = sh.max_ctx / KV_PAGE;
    if (sh.sliding_window > 0) npg = std::min(npg, (sh.sliding_window + KV_PAGE - 1) / KV_PAGE + 1);
    // the score buffer holds AC_SBUF bytes: that many pages per CTA
    const int maxp_lim = std::max(1, AC_SBUF / (G * KV_PAGE * 4));
    static const int c_cap = [] {  // LLMDOT_ATTN_CLUSTER: upper bound on the cluster size (tuning)
        const char *e = getenv("LLMDOT_ATTN_CLUSTER");
        return e ? std::min(8, std::max(1, atoi(e))) : 8;
    }();
    int C = 1;
    while (C < 8 && (npg + C - 1) / C > maxp_lim) C++;
    while (C < c_cap && (long long)batch * sh.heads_kv * C < 2 * 148) C++;  // enough CTAs for every SM
    const int maxp = (npg + C - 1) / C;
    if (maxp > maxp_lim) return false;
    // page slots: as many pages in flight as the CTAs sharing an SM leave room for (at most
    // every page of the CTA, at least two)
    const long long ctas = (long long)batch * sh.heads_kv * C;
    const int per_sm = (int)std::min<long long>(4, std::max<long long>(1, (ctas + 147) / 148));
    const int budget = std::min(200 * 1024, 220 * 1024 / per_sm - 2048);
    // Large pages (24 KB and up: head_dim 256 in fp16) stream best two at a time with the CTAs
    // small enough to pair up on an SM; small pages are latency-bound, and their CTAs run best
    // one per SM with every page in flight (measured on Gemma-2-2B and Llama-3.2-1B shapes).
    const bool big_pages = (size_t)KV_PAGE * (sh.head_dim * esz + 16) >= 24 * 1024;
    int slots = big_pages ? 2 : 2 * maxp;
    static const int slots_cap = [] {  // LLMDOT_ATTN_SLOTS: upper bound on the page slots (tuning)
        const char *e = getenv("LLMDOT_ATTN_SLOTS");
        return e ? std::max(2, atoi(e)) : 1 << 20;
    }();
    slots = std::min(slots, slots_cap);
    while (slots > 2 && ac_layout(sh.head_dim, (int)esz, G, maxp, slots, C).total > budget) slots--;
    const AcLayout L = ac_layout(sh.head_dim, (int)esz, G, maxp, slots, C);
    if (L.total > 200 * 1024) return false;
    static const int min_smem = [] {  // LLMDOT_ATTN_MIN_SMEM: shared-memory floor per CTA in KB (tuning)
        const char *e = getenv("LLMDOT_ATTN_MIN_SMEM");
        return e ? std::min(200, std::max(0, atoi(e))) * 1024 : 0;
    }();
    *C_out = C;
    *maxp_out = maxp;
    *slots_out = slots;
    *smem_out = (size_t)std::max(L.total, min_smem);
    return true;
}

int attention_timeout_check()
{
    int v = 0;
    LLMDOT_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_attn_timeout, sizeof(int)));
    if (v) {
        const int zero = 0;
        cudaMemcpyToSymbol(g_attn_timeout, &zero, sizeof(int));
        return fail(LLMDOT_E_TIMEOUT, "attention: a KV page wait timed out");
    }
    return LLMDOT_OK;
}

template <typename T>
static int launch_cluster_t(const float *q, int ldq, const float *k, const float *v, int ldkv, const int32_t *pos,
                            const float *cos_t, const float *sin_t, const KvView *views, int layer, const AttnShape &sh,
                            int batch, float *out, int ldo, int appended, int C, int maxp, int slots, size_t smem,
                            bool pdl, cudaStream_t st)
{
    static std::atomic<unsigned long long> attr_done{0};
    LLMDOT_CUDA_TRY(smem_attr_once(attr_done, attn_cluster_kernel<T>, 200 * 1024));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C, sh.heads_kv, batch);
    cfg.blockDim = dim3(AC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    LLMDOT_CUDA_TRY(cudaLaunchKernelEx(&cfg, attn_cluster_kernel<T>, q, ldq, k, v, ldkv, pos, cos_t, sin_t, views, layer,
                                       sh, out, ldo, appended, maxp, slots));
    return LLMDOT_OK;
}

static size_t scores_smem(const AttnShape &sh, size_t esz)
{
    const int G = sh.heads / sh.heads_kv;
    return (size_t)KV_PAGE * (sh.head_dim + (esz == 2 ? 2 : 1)) * esz + 16 + sizeof(float) * (G * sh.head_dim + G) + 16;
}
static size_t pv_smem(const AttnShape &sh, size_t esz)
{
    const int G = sh.heads / sh.heads_kv;
    return (size_t)KV_PAGE * sh.head_dim * esz + sizeof(float) * (G * KV_PAGE + G) + 16;
}

template <typename T>
static int launch_attn_t(const float *q, int ldq, const float *k, const float *v, int ldkv, const int32_t *pos,
                         const float *cos_t, const float *sin_t, const KvView *views, int layer, const AttnShape &sh,
                         int batch, float *scores, float *part_m, float *part_s, float *part_o, int *counters,
                         float *out, int ldo, bool append_first, bool pdl, cudaStream_t st)
{
    const int nchunk = sh.max_ctx / KV_PAGE;
    dim3 grid(nchunk, sh.heads_kv, batch);
    if (append_first)
        LLMDOT_CUDA_TRY(launch_kernel(pdl, append_kv_kernel<T>, dim3(sh.heads_kv, batch), dim3(128), 0, st, k, v, ldkv,
                                      pos, cos_t, sin_t, views, layer, sh));
    const int appended = append_first ? 1 : 0;
    static std::atomic<unsigned long long> attr_s{0}, attr_p{0};
    LLMDOT_CUDA_TRY(smem_attr_once(attr_s, attn_scores_kernel<T>, 200 * 1024));
    LLMDOT_CUDA_TRY(smem_attr_once(attr_p, attn_pv_kernel<T>, 200 * 1024));
    LLMDOT_CUDA_TRY(launch_kernel(pdl, attn_scores_kernel<T>, grid, dim3(256), scores_smem(sh, sizeof(T)), st, q, ldq, k,
                                  v, ldkv, pos, cos_t, sin_t, views, layer, sh, scores, part_m, appended));
    LLMDOT_CUDA_TRY(launch_kernel(pdl, attn_pv_kernel<T>, grid, dim3(256), pv_smem(sh, sizeof(T)), st, pos, views, layer,
                                  sh, (const float *)scores, (const float *)part_m, part_s, part_o, counters, out, ldo,
                                  appended));
    return LLMDOT_OK;
}

int launch_attention_step(const float *q, int ldq, const float *k, const float *v, int ldkv, const int32_t *pos,
                          const float *cos_t, const float *sin_t, const KvView *views, int layer, int kv_type,
                          const AttnShape &sh, int batch, float *scores, float *part_m, float *part_s, float *part_o,
                          int *counters, float *out, int ldo, bool append_first, bool pdl, cudaStream_t st)
{
    const size_t esz = kv_type == LLMDOT_KV_F16 ? 2 : 4;
    int C = 0, maxp = 0, slots = 0;
    size_t csm = 0;
    if (cluster_plan(sh, batch, esz, &C, &maxp, &slots, &csm)) {
        if (append_first)
            LLMDOT_CUDA_TRY(kv_type == LLMDOT_KV_F16
                                ? launch_kernel(pdl, append_kv_kernel<__half>, dim3(sh.heads_kv, batch), dim3(128), 0, st,
                                                k, v, ldkv, pos, cos_t, sin_t, views, layer, sh)
                                : launch_kernel(pdl, append_kv_kernel<float>, dim3(sh.heads_kv, batch), dim3(128), 0, st,
                                                k, v, ldkv, pos, cos_t, sin_t, views, layer, sh));
        const int appended = append_first ? 1 : 0;
        if (kv_type == LLMDOT_KV_F16)
            return launch_cluster_t<__half>(q, ldq, k, v, ldkv, pos, cos_t, sin_t, views, layer, sh, batch, out, ldo,
                                            appended, C, maxp, slots, csm, pdl, st);
        return launch_cluster_t<float>(q, ldq, k, v, ldkv, pos, cos_t, sin_t, views, layer, sh, batch, out, ldo,
                                       appended, C, maxp, slots, csm, pdl, st);
    }
    // long windows: the two-kernel path with global scratch
    if (scores_smem(sh, 4) > 200 * 1024 || pv_smem(sh, 4) > 200 * 1024)
        return fail(LLMDOT_E_UNSUPPORTED, "attention: head too large for the page staging");
    if (kv_type == LLMDOT_KV_F16)
        return launch_attn_t<__half>(q, ldq, k, v, ldkv, pos, cos_t, sin_t, views, layer, sh, batch, scores, part_m,
                                     part_s, part_o, counters, out, ldo, append_first, pdl, st);
    return launch_attn_t<float>(q, ldq, k, v, ldkv, pos, cos_t, sin_t, views, layer, sh, batch, scores, part_m, part_s,
                                part_o, counters, out, ldo, append_first, pdl, st);
}

}  // namespace llmdot
