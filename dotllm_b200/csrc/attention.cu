// attention.cu -- RoPE + KV append and GQA decode attention over the paged cache.
//
// Reference: InferenceEngine.AttentionForward (src/Llmdot.Core/Inference/InferenceEngine.cs:304-450)
// with VectorMath.Softmax (src/Llmdot.Core/Tensors/Numeric/VectorMath.cs:215-258).
// The reference's softmax evaluates ExpApprox(s - max) against the GLOBAL max of the
// window (an approximation whose error is up to ~18 % for some arguments, so an
// online/rescaled softmax would not reproduce it).  The device therefore works in
// three passes over pages of KV_PAGE positions:
//   1. scores: s = (q . k) * 1/sqrt(hd), softcap, per-page max;
//   2. p = exp(s - M) with M the window max, per-page sum and sum p*V;
//   3. combine the pages and scale by 1/sum.
// "Vector lane" vs "tail" (ExpApprox/TanhApprox vs MathF.Exp/Tanh) is decided by the
// position's index inside the window, exactly as the reference's 8-wide loops do.
#include "attention.cuh"

namespace llmdot {

template <typename T> __device__ __forceinline__ float ldf(const T *p);
template <> __device__ __forceinline__ float ldf<float>(const float *p) { return *p; }
template <> __device__ __forceinline__ float ldf<__half>(const __half *p) { return __half2float(*p); }
template <typename T> __device__ __forceinline__ T stf(float v);
template <> __device__ __forceinline__ float stf<float>(float v) { return v; }
template <> __device__ __forceinline__ __half stf<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ void window(int p, int sw, int &start, int &seq_len)
{
    seq_len = p + 1;
    start = sw > 0 ? max(0, seq_len - sw) : 0;
}

// ---------------------------------------------------------------- RoPE + append
template <typename T>
__global__ void rope_append_kernel(float *__restrict__ q, int ldq, const float *__restrict__ k,
                                   const float *__restrict__ v, int ldkv, const int32_t *__restrict__ pos,
                                   const float *__restrict__ cos_t, const float *__restrict__ sin_t,
                                   const KvView *__restrict__ views, int layer, AttnShape sh)
{
    const int b = blockIdx.y, h = blockIdx.x, hd = sh.head_dim, half = sh.rope_half;
    const int p = pos[b];
    const float *cs = cos_t + (uint64_t)p * half, *sn = sin_t + (uint64_t)p * half;
    if (h < sh.heads) {
        float *x = q + (uint64_t)b * ldq + (uint64_t)h * hd;
        for (int i = threadIdx.x; i < half; i += blockDim.x) {
            float c = cs[i], s = sn[i], x0 = x[i], x1 = x[i + half];
            x[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
            x[i + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        }
        return;
    }
    const int kh = h - sh.heads;
    const KvView vw = views[b];
    const int page = vw.pages[p / KV_PAGE], slot = p % KV_PAGE;
    const uint64_t off = (uint64_t)layer * vw.layer_stride +
                         (((uint64_t)page * sh.heads_kv + kh) * KV_PAGE + slot) * hd;
    T *kd = (T *)vw.k + off;
    T *vd = (T *)vw.v + off;
    const float *ks = k + (uint64_t)b * ldkv + (uint64_t)kh * hd;
    const float *vs = v + (uint64_t)b * ldkv + (uint64_t)kh * hd;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float r;
        if (i < half) r = __fsub_rn(__fmul_rn(ks[i], cs[i]), __fmul_rn(ks[i + half], sn[i]));
        else if (i < 2 * half) r = __fadd_rn(__fmul_rn(ks[i - half], sn[i - half]), __fmul_rn(ks[i], cs[i - half]));
        else r = ks[i];
        kd[i] = stf<T>(r);
        vd[i] = stf<T>(vs[i]);
    }
}

int launch_rope_append(float *q, int ldq, const float *k, const float *v, int ldkv, const int32_t *pos,
                       const float *cos_t, const float *sin_t, const KvView *views, int layer, int kv_type,
                       const AttnShape &sh, int batch, cudaStream_t st)
{
    dim3 grid(sh.heads + sh.heads_kv, batch);
    if (kv_type == LLMDOT_KV_F16)
        rope_append_kernel<__half><<<grid, 128, 0, st>>>(q, ldq, k, v, ldkv, pos, cos_t, sin_t, views, layer, sh);
    else
        rope_append_kernel<float><<<grid, 128, 0, st>>>(q, ldq, k, v, ldkv, pos, cos_t, sin_t, views, layer, sh);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

// ---------------------------------------------------------------- pass 1: scores
template <typename T>
__global__ void __launch_bounds__(256) attn_scores_kernel(const float *__restrict__ q, int ldq,
                                                          const int32_t *__restrict__ pos,
                                                          const KvView *__restrict__ views, int layer, AttnShape sh,
                                                          float *__restrict__ scores, float *__restrict__ part_m)
{
    extern __shared__ float smem[];
    const int chunk = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int hd = sh.head_dim, G = sh.heads / sh.heads_kv, nchunk = sh.max_ctx / KV_PAGE;
    int start, seq_len;
    window(pos[b], sh.sliding_window, start, seq_len);
    const int s0 = chunk * KV_PAGE;
    if (s0 >= seq_len || s0 + KV_PAGE <= start) return;
    const int len = seq_len - start, nvec = len - len % 8;
    float *qs = smem;                                // [G][hd]
    uint32_t *mk = (uint32_t *)(smem + G * hd);      // [G]
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x)
        qs[i] = q[(uint64_t)b * ldq + (uint64_t)(kvh * G) * hd + i];
    for (int i = threadIdx.x; i < G; i += blockDim.x) mk[i] = 0u;
    __syncthreads();
    const KvView vw = views[b];
    const int page = vw.pages[chunk];
    const T *kb = (const T *)vw.k + (uint64_t)layer * vw.layer_stride +
                  ((uint64_t)page * sh.heads_kv + kvh) * KV_PAGE * hd;
    const float inv_cap = sh.has_cap ? __fdiv_rn(1.0f, sh.cap) : 0.0f;
    for (int idx = threadIdx.x; idx < G * KV_PAGE; idx += blockDim.x) {
        const int hg = idx / KV_PAGE, j = idx % KV_PAGE, s = s0 + j;
        if (s < start || s >= seq_len) continue;
        const T *kr = kb + (uint64_t)j * hd;
        const float *qh = qs + hg * hd;
        float dot = 0.0f;
        for (int d = 0; d < hd; d++) dot = fmaf(qh[d], ldf<T>(kr + d), dot);
        float sc = __fmul_rn(dot, sh.inv_sqrt_hd);
        if (sh.has_cap) sc = softcap_ref(sc, sh.cap, inv_cap, (s - start) < nvec);
        const int h = kvh * G + hg;
        scores[((uint64_t)b * sh.heads + h) * sh.max_ctx + s] = sc;
        atomicMax(mk + hg, float_key(sc));
    }
    __syncthreads();
    for (int hg = threadIdx.x; hg < G; hg += blockDim.x)
        part_m[((uint64_t)b * sh.heads + kvh * G + hg) * nchunk + chunk] = key_float(mk[hg]);
}

// ---------------------------------------------------------------- pass 2: exp + PV
template <typename T>
__global__ void __launch_bounds__(256) attn_pv_kernel(const int32_t *__restrict__ pos, const KvView *__restrict__ views,
                                                      int layer, AttnShape sh, const float *__restrict__ scores,
                                                      const float *__restrict__ part_m, float *__restrict__ part_s,
                                                      float *__restrict__ part_o)
{
    extern __shared__ float smem[];
    const int chunk = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int hd = sh.head_dim, G = sh.heads / sh.heads_kv, nchunk = sh.max_ctx / KV_PAGE;
    int start, seq_len;
    window(pos[b], sh.sliding_window, start, seq_len);
    const int s0 = chunk * KV_PAGE;
    if (s0 >= seq_len || s0 + KV_PAGE <= start) return;
    const int len = seq_len - start, nvec = len - len % 8;
    const int c0 = start / KV_PAGE, c1 = (seq_len - 1) / KV_PAGE;
    float *ps = smem;                  // [G][KV_PAGE]
    float *mx = smem + G * KV_PAGE;    // [G]
    float *sm = mx + G;                // [G]
    for (int hg = threadIdx.x; hg < G; hg += blockDim.x) {
        const float *pm = part_m + ((uint64_t)b * sh.heads + kvh * G + hg) * nchunk;
        float m = -INFINITY;
        for (int c = c0; c <= c1; c++) m = fmaxf(m, pm[c]);
        mx[hg] = m;
        sm[hg] = 0.0f;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * KV_PAGE; idx += blockDim.x) {
        const int hg = idx / KV_PAGE, j = idx % KV_PAGE, s = s0 + j;
        float p = 0.0f;
        if (s >= start && s < seq_len) {
            const int h = kvh * G + hg;
            float d = __fsub_rn(scores[((uint64_t)b * sh.heads + h) * sh.max_ctx + s], mx[hg]);
            p = (s - start) < nvec ? exp_approx(d) : expf(d);
        }
        ps[idx] = p;
    }
    __syncthreads();
    for (int hg = threadIdx.x >> 5; hg < G; hg += blockDim.x >> 5) {
        float t = 0.0f;
        for (int j = threadIdx.x & 31; j < KV_PAGE; j += 32) t += ps[hg * KV_PAGE + j];
        t = warp_sum(t);
        if ((threadIdx.x & 31) == 0) part_s[((uint64_t)b * sh.heads + kvh * G + hg) * nchunk + chunk] = t;
    }
    const KvView vw = views[b];
    const int page = vw.pages[chunk];
    const T *vb = (const T *)vw.v + (uint64_t)layer * vw.layer_stride +
                  ((uint64_t)page * sh.heads_kv + kvh) * KV_PAGE * hd;
    const int jlo = max(start - s0, 0), jhi = min(seq_len - s0, KV_PAGE);
    for (int idx = threadIdx.x; idx < G * hd; idx += blockDim.x) {
        const int hg = idx / hd, d = idx % hd;
        const float *p = ps + hg * KV_PAGE;
        float acc = 0.0f;
        for (int j = jlo; j < jhi; j++) acc = fmaf(p[j], ldf<T>(vb + (uint64_t)j * hd + d), acc);
        part_o[(((uint64_t)b * sh.heads + kvh * G + hg) * nchunk + chunk) * hd + d] = acc;
    }
}

// ---------------------------------------------------------------- pass 3: combine
__global__ void attn_combine_kernel(const int32_t *__restrict__ pos, AttnShape sh, const float *__restrict__ part_s,
                                    const float *__restrict__ part_o, float *__restrict__ out, int ldo)
{
    const int h = blockIdx.x, b = blockIdx.y, hd = sh.head_dim, nchunk = sh.max_ctx / KV_PAGE;
    int start, seq_len;
    window(pos[b], sh.sliding_window, start, seq_len);
    const int c0 = start / KV_PAGE, c1 = (seq_len - 1) / KV_PAGE;
    const uint64_t base = ((uint64_t)b * sh.heads + h) * nchunk;
    float sum = 0.0f;
    for (int c = c0; c <= c1; c++) sum += part_s[base + c];
    const float inv = __fdiv_rn(1.0f, sum);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.0f;
        for (int c = c0; c <= c1; c++) o += part_o[(base + c) * hd + d];
        out[(uint64_t)b * ldo + (uint64_t)h * hd + d] = __fmul_rn(o, inv);
    }
}

int launch_attention_decode(const float *q, int ldq, const int32_t *pos, const KvView *views, int layer, int kv_type,
                            const AttnShape &sh, int batch, float *scores, float *part_m, float *part_s, float *part_o,
                            float *out, int ldo, cudaStream_t st)
{
    const int G = sh.heads / sh.heads_kv, nchunk = sh.max_ctx / KV_PAGE;
    dim3 grid(nchunk, sh.heads_kv, batch);
    size_t sm1 = sizeof(float) * (G * sh.head_dim + G);
    size_t sm2 = sizeof(float) * (G * KV_PAGE + 2 * G);
    if (kv_type == LLMDOT_KV_F16) {
        attn_scores_kernel<__half><<<grid, 256, sm1, st>>>(q, ldq, pos, views, layer, sh, scores, part_m);
        attn_pv_kernel<__half><<<grid, 256, sm2, st>>>(pos, views, layer, sh, scores, part_m, part_s, part_o);
    } else {
        attn_scores_kernel<float><<<grid, 256, sm1, st>>>(q, ldq, pos, views, layer, sh, scores, part_m);
        attn_pv_kernel<float><<<grid, 256, sm2, st>>>(pos, views, layer, sh, scores, part_m, part_s, part_o);
    }
    LLMDOT_CUDA_TRY(cudaGetLastError());
    attn_combine_kernel<<<dim3(sh.heads, batch), sh.head_dim < 256 ? sh.head_dim : 256, 0, st>>>(pos, sh, part_s, part_o,
                                                                                              out, ldo);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

}  // namespace llmdot
