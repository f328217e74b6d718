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

namespace llmdot {

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
    static bool attr_set = false;
    if (!attr_set) {
        LLMDOT_CUDA_TRY(cudaFuncSetAttribute(attn_scores_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        LLMDOT_CUDA_TRY(cudaFuncSetAttribute(attn_pv_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        attr_set = true;
    }
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
    if (scores_smem(sh, 4) > 200 * 1024 || pv_smem(sh, 4) > 200 * 1024)
        return fail(LLMDOT_E_UNSUPPORTED, "attention: head too large for the page staging");
    if (kv_type == LLMDOT_KV_F16)
        return launch_attn_t<__half>(q, ldq, k, v, ldkv, pos, cos_t, sin_t, views, layer, sh, batch, scores, part_m,
                                     part_s, part_o, counters, out, ldo, append_first, pdl, st);
    return launch_attn_t<float>(q, ldq, k, v, ldkv, pos, cos_t, sin_t, views, layer, sh, batch, scores, part_m, part_s,
                                part_o, counters, out, ldo, append_first, pdl, st);
}

}  // namespace llmdot
