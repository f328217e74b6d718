// ops.cu -- element-wise / reduction kernels and the generic (reference) quantised
// matvec.  These serve the per-operation adapter (Tier A) directly and the decode
// step wherever no fused kernel replaces them.
#include <cuda_runtime.h>

#include "ops.cuh"
#include "quant.cuh"

namespace llmdot {

// ------------------------------------------------------------------ dequantise
// TensorOps.DequantizeToFloat (TensorOps.cs:18-56): bit-exact with the reference.
__global__ void dequant_kernel(const uint8_t *__restrict__ src, float *__restrict__ dst, uint32_t type,
                               int rows, int row_elems, uint64_t rbytes)
{
    const uint64_t total = (uint64_t)rows * row_elems;
    const uint32_t be = (uint32_t)block_elems(type), bb = (uint32_t)block_bytes(type);
    for (uint64_t idx = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; idx < total;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        uint64_t r = idx / row_elems;
        uint32_t e = (uint32_t)(idx - r * row_elems);
        const uint8_t *blk = src + r * rbytes + (uint64_t)(e / be) * bb;
        dst[idx] = deq1(type, blk, e % be);
    }
}

int launch_dequant(const uint8_t *src, float *dst, uint32_t type, int rows, int row_elems, cudaStream_t st)
{
    if (block_elems(type) == 0) return fail(LLMDOT_E_UNSUPPORTED, "dequantize: unsupported type " + std::to_string(type));
    uint64_t total = (uint64_t)rows * row_elems;
    if (total == 0) return LLMDOT_OK;
    int blocks = (int)((total + 255) / 256);
    if (blocks > 148 * 32) blocks = 148 * 32;
    dequant_kernel<<<blocks, 256, 0, st>>>(src, dst, type, rows, row_elems, row_bytes(type, row_elems));
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

// ------------------------------------------------------------------ generic matvec
// y[v][c] (+)= sum_i x[v][i] * deq(W row c, i) for NV input rows.  One warp per
// output row; lanes take 8 consecutive elements at a time so weight reads are
// coalesced.  Every weight value is decoded bit-exactly; accumulation is fp32.
template <int NV>
__global__ void __launch_bounds__(256) gemv_ref_kernel(const uint8_t *__restrict__ W, uint32_t type, int rows, int cols,
                                                       uint64_t rbytes, const float *__restrict__ x, int ldx,
                                                       float *__restrict__ y, int ldy, int accumulate, int nv)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + warp;
    if (row >= rows) return;
    const uint32_t be = (uint32_t)block_elems(type), bb = (uint32_t)block_bytes(type);
    const uint8_t *wr = W + (uint64_t)row * rbytes;
    float acc[NV];
#pragma unroll
    for (int v = 0; v < NV; v++) acc[v] = 0.0f;
    for (int e0 = lane * 8; e0 < cols; e0 += 256) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int e = e0 + j;
            if (e >= cols) break;
            float w = deq1(type, wr + (uint64_t)(e / be) * bb, e % be);
#pragma unroll
            for (int v = 0; v < NV; v++)
                if (v < nv) acc[v] = fmaf(x[(uint64_t)v * ldx + e], w, acc[v]);
        }
    }
#pragma unroll
    for (int v = 0; v < NV; v++) {
        float s = warp_sum(acc[v]);
        if (lane == 0 && v < nv) {
            float *o = y + (uint64_t)v * ldy + row;
            *o = accumulate ? *o + s : s;
        }
    }
}

int launch_gemv_ref(const uint8_t *W, uint32_t type, int rows, int cols, const float *x, int ldx, int nv, float *y,
                    int ldy, bool accumulate, cudaStream_t st)
{
    if (block_elems(type) == 0) return fail(LLMDOT_E_UNSUPPORTED, "matmul: unsupported type " + std::to_string(type));
    if (cols % (int)block_elems(type) != 0) return fail(LLMDOT_E_INVALID, "matmul: aCols not a multiple of the block size");
    uint64_t rb = row_bytes(type, (uint64_t)cols);
    dim3 grid((rows + 7) / 8);
    for (int v0 = 0; v0 < nv; v0 += 8) {
        int n = nv - v0 < 8 ? nv - v0 : 8;
        const float *xv = x + (uint64_t)v0 * ldx;
        float *yv = y + (uint64_t)v0 * ldy;
        if (n == 1)
            gemv_ref_kernel<1><<<grid, 256, 0, st>>>(W, type, rows, cols, rb, xv, ldx, yv, ldy, accumulate, n);
        else if (n <= 4)
            gemv_ref_kernel<4><<<grid, 256, 0, st>>>(W, type, rows, cols, rb, xv, ldx, yv, ldy, accumulate, n);
        else
            gemv_ref_kernel<8><<<grid, 256, 0, st>>>(W, type, rows, cols, rb, xv, ldx, yv, ldy, accumulate, n);
        LLMDOT_CUDA_TRY(cudaGetLastError());
    }
    return LLMDOT_OK;
}

// ------------------------------------------------------------------ norms
// VectorMath.RmsNorm (VectorMath.cs:308-340), nv independent rows of n.  The sum of
// squares is reduced in a fixed tree (not the reference's 8-lane order); the
// scaling keeps the reference's association: (w*x)*inv for the first n - n%8
// elements, w*(x*inv) for the tail.
__global__ void rmsnorm_kernel(const float *__restrict__ in, int ldin, const float *__restrict__ w, float *__restrict__ out,
                               int ldout, int n, float eps)
{
    const float *x = in + (uint64_t)blockIdx.x * ldin;
    float *o = out + (uint64_t)blockIdx.x * ldout;
    __shared__ float red[32];
    pdl_launch();  // no-ops unless launched with programmatic dependent launch
    pdl_wait();
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    float mean = __fadd_rn(__fdiv_rn(red[0], (float)n), eps);
    float inv = __fdiv_rn(1.0f, __fsqrt_rn(mean));
    const int nvec = n - n % 8;
    __syncthreads();  // in-place (in == out) safety: everybody has read red[0]
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float xi = x[i];
        o[i] = i < nvec ? __fmul_rn(__fmul_rn(w[i], xi), inv) : __fmul_rn(w[i], __fmul_rn(xi, inv));
    }
}

int launch_rmsnorm(const float *in, int ldin, const float *w, float *out, int ldout, int n, int nv, float eps,
                   cudaStream_t st, bool pdl)
{
    LLMDOT_CUDA_TRY(launch_kernel(pdl, rmsnorm_kernel, dim3(nv), dim3(256), 0, st, in, ldin, w, out, ldout, n, eps));
    return LLMDOT_OK;
}

// VectorMath.LayerNorm (VectorMath.cs:342-406); bias may be null.
__global__ void layernorm_kernel(const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ b,
                                 float *__restrict__ o, int n, float eps)
{
    __shared__ float red[32];
    __shared__ float stat[2];
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        v = warp_sum(v);
        if (threadIdx.x == 0) stat[0] = __fdiv_rn(v, (float)n);
    }
    __syncthreads();
    float mean = stat[0];
    float q = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float d = __fsub_rn(x[i], mean);
        q = fmaf(d, d, q);
    }
    q = warp_sum(q);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = q;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        v = warp_sum(v);
        if (threadIdx.x == 0) stat[1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(v, (float)n), eps)));
    }
    __syncthreads();
    float inv = stat[1];
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = __fmul_rn(__fmul_rn(w[i], __fsub_rn(x[i], mean)), inv);
        o[i] = b ? __fadd_rn(v, b[i]) : v;
    }
}

int launch_layernorm(const float *x, const float *w, const float *b, float *o, int n, float eps, cudaStream_t st)
{
    layernorm_kernel<<<1, 1024, 0, st>>>(x, w, b, o, n, eps);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

// ------------------------------------------------------------------ element-wise
// `row` is the length of the reference's span: lane i of a row is a "vector lane" when
// (i % row) < row - row % 8.
__global__ void eltwise_kernel(int op, const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ o,
                               int n, float s, int row)
{
    const int nvec = row - row % 8;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        float r;
        const bool vl = (i % row) < nvec;
        switch (op) {
        case OP_ADD: r = __fadd_rn(a[i], b[i]); break;
        case OP_MUL: r = __fmul_rn(a[i], b[i]); break;
        case OP_SCALE: r = __fmul_rn(a[i], s); break;
        case OP_SILU: r = silu_ref(a[i], vl); break;
        case OP_GELU: r = gelu_ref(a[i], vl); break;
        case OP_SOFTCAP: r = softcap_ref(a[i], s, __fdiv_rn(1.0f, s), vl); break;
        case OP_SILU_MUL: r = __fmul_rn(silu_ref(a[i], vl), b[i]); break;
        case OP_GELU_MUL: r = __fmul_rn(gelu_ref(a[i], vl), b[i]); break;
        default: r = 0.0f;
        }
        o[i] = r;
    }
}

int launch_eltwise(int op, const float *a, const float *b, float *o, int n, float s, cudaStream_t st, int row)
{
    if (n <= 0) return LLMDOT_OK;
    if (row <= 0) row = n;
    int blocks = (n + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    eltwise_kernel<<<blocks, 256, 0, st>>>(op, a, b, o, n, s, row);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

// FfnForward's SiluInPlace/Gelu of the gate followed by Mul(gate, up) (InferenceEngine.cs:466-474)
int launch_act_mul(bool gelu, const float *gate, const float *up, float *out, int ffn, int batch, cudaStream_t st)
{
    return launch_eltwise(gelu ? OP_GELU_MUL : OP_SILU_MUL, gate, up, out, ffn * batch, 0.0f, st, ffn);
}

__global__ void gelu_scalar_kernel(float x, float *o)
{
    *o = gelu_ref(x, false);
}

int launch_gelu_scalar(float x, float *o, cudaStream_t st)
{
    gelu_scalar_kernel<<<1, 1, 0, st>>>(x, o);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

// ------------------------------------------------------------------ RoPE
// TensorOps.ApplyRoPE with precomputed cos/sin (TensorOps.cs:679-743): half-split
// pairs (i, i+half) of every head; cos/sin come from the host (MathF.Cos/Sin of the
// fp32 angle position*freq[i]).
__global__ void rope_kernel(float *__restrict__ x, int nheads, int head_dim, const float *__restrict__ cs,
                            const float *__restrict__ sn, int half)
{
    int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= nheads * half) return;
    int h = idx / half, i = idx % half;
    float *p = x + (uint64_t)h * head_dim;
    float c = cs[i], s = sn[i];
    float x0 = p[i], x1 = p[i + half];
    p[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    p[i + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

int launch_rope(float *x, int nheads, int head_dim, const float *cs, const float *sn, int half, cudaStream_t st)
{
    int n = nheads * half;
    if (n <= 0) return LLMDOT_OK;
    rope_kernel<<<(n + 127) / 128, 128, 0, st>>>(x, nheads, head_dim, cs, sn, half);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

// ------------------------------------------------------------------ softmax (Tier A)
// VectorMath.Softmax (VectorMath.cs:215-258) on one vector: softcap (vector/tail
// lanes), max, exp (ExpApprox lanes / MathF.Exp tail) of x - max, scale by 1/sum.
__global__ void softmax_kernel(float *__restrict__ x, int n, int has_cap, float cap)
{
    __shared__ float red[32];
    __shared__ float bc;
    const int nvec = n - n % 8;
    float inv_cap = has_cap ? __fdiv_rn(1.0f, cap) : 0.0f;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = x[i];
        if (has_cap) { v = softcap_ref(v, cap, inv_cap, i < nvec); x[i] = v; }
        m = fmaxf(m, v);
    }
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
        v = warp_max(v);
        if (threadIdx.x == 0) bc = v;
    }
    __syncthreads();
    m = bc;
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float d = __fsub_rn(x[i], m);
        float e = i < nvec ? exp_approx(d) : expf(d);
        x[i] = e;
        s = __fadd_rn(s, e);
    }
    s = warp_sum(s);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
        v = warp_sum(v);
        if (threadIdx.x == 0) bc = __fdiv_rn(1.0f, v);
    }
    __syncthreads();
    float inv = bc;
    for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] = __fmul_rn(x[i], inv);
}

int launch_softmax(float *x, int n, bool has_cap, float cap, cudaStream_t st)
{
    if (n <= 0) return LLMDOT_OK;
    softmax_kernel<<<1, 1024, 0, st>>>(x, n, has_cap ? 1 : 0, cap);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

// ------------------------------------------------------------------ argmax
// VectorMath.ArgMax (VectorMath.cs:412-425): first index of the maximum.  Packed
// 64-bit keys (argmax_key: value key << 32 | ~index) reduced with atomicMax, so the largest
// value wins and, among equal values, the lowest index; NaN and -0 are keyed so that the result
// is the reference's strict-`>` scan from element 0.  Optional in-kernel final
// softcap of the logits first (Generate applies it before sampling,
// InferenceEngine.cs:105-106); the capped logits are written back to `capped` if given.
// Under tensor parallelism x holds vocabulary entries [off, off + n) of `ntot`: keys carry the
// global index, and the vector-lane / tail choice of the softcap uses the global position.
__global__ void argmax_kernel(const float *__restrict__ x, int ldx, int n, unsigned long long *__restrict__ keys,
                              int has_cap, float cap, float *__restrict__ capped, int off, int ntot)
{
    const int v = blockIdx.y;
    const float *xv = x + (uint64_t)v * ldx;
    const int nvec = ntot - ntot % 8 - off;
    float inv_cap = has_cap ? __fdiv_rn(1.0f, cap) : 0.0f;
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        float f = xv[i];
        if (has_cap) {
            f = softcap_ref(f, cap, inv_cap, i < nvec);
            if (capped) capped[(uint64_t)v * ldx + i] = f;
        }
        const unsigned long long k = argmax_key(f, (uint32_t)(i + off));
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) atomicMax(keys + v, best);
}

__global__ void argmax_finish_kernel(const unsigned long long *__restrict__ keys, int nv, int32_t *__restrict__ out)
{
    int v = blockIdx.x * blockDim.x + threadIdx.x;
    if (v < nv) out[v] = (int32_t)(0xFFFFFFFFu - (uint32_t)(keys[v] & 0xFFFFFFFFull));
}

int launch_argmax_keys(const float *x, int ldx, int n, int nv, unsigned long long *keys, bool has_cap, float cap,
                       float *capped, int off, int ntot, cudaStream_t st)
{
    LLMDOT_CUDA_TRY(cudaMemsetAsync(keys, 0, sizeof(unsigned long long) * nv, st));
    int blocks = (n + 1023) / 1024;
    if (blocks > 148) blocks = 148;
    argmax_kernel<<<dim3(blocks, nv), 256, 0, st>>>(x, ldx, n, keys, has_cap ? 1 : 0, cap, capped, off, ntot);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

int launch_argmax_finish(const unsigned long long *keys, int nv, int32_t *out, cudaStream_t st)
{
    argmax_finish_kernel<<<(nv + 63) / 64, 64, 0, st>>>(keys, nv, out);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

int launch_argmax(const float *x, int ldx, int n, int nv, unsigned long long *keys, int32_t *out, bool has_cap,
                  float cap, float *capped, cudaStream_t st)
{
    LLMDOT_TRY(launch_argmax_keys(x, ldx, n, nv, keys, has_cap, cap, capped, 0, n, st));
    return launch_argmax_finish(keys, nv, out, st);
}

// ------------------------------------------------------------------ conv1d
// TensorOps.Conv1D (TensorOps.cs:745-779); the per-channel dot keeps 8 lanes + tail.
__global__ void conv1d_kernel(const float *__restrict__ in, const float *__restrict__ w, float *__restrict__ o, int ks,
                              int dim)
{
    int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= dim) return;
    if (ks == 1) { o[c] = __fmul_rn(in[c], w[c]); return; }
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int k = 0;
    const float *ip = in + (uint64_t)c * ks, *wp = w + (uint64_t)c * ks;
    for (; k <= ks - 8; k += 8)
        for (int l = 0; l < 8; l++) acc[l] = __fadd_rn(acc[l], __fmul_rn(ip[k + l], wp[k + l]));
    float s = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3])),
                        __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7])));
    for (; k < ks; k++) s = __fadd_rn(s, __fmul_rn(ip[k], wp[k]));
    o[c] = s;
}

int launch_conv1d(const float *in, const float *w, float *o, int ks, int dim, cudaStream_t st)
{
    if (dim <= 0) return LLMDOT_OK;
    conv1d_kernel<<<(dim + 127) / 128, 128, 0, st>>>(in, w, o, ks, dim);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

// ------------------------------------------------------------------ embedding
// GetEmbedding (InferenceEngine.cs:148-156) + EmbeddingScale (:138-139) for nv tokens.
__global__ void embed_kernel(const uint8_t *__restrict__ emb, uint32_t type, int hidden, uint64_t rbytes, int vocab,
                             const int32_t *__restrict__ tokens, float scale, int apply_scale, float *__restrict__ h,
                             int ldh, int *__restrict__ err)
{
    const int v = blockIdx.y;
    int tok = tokens[v];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(err, 1);
        tok = 0;
    }
    const uint32_t be = (uint32_t)block_elems(type), bb = (uint32_t)block_bytes(type);
    const uint8_t *row = emb + (uint64_t)tok * rbytes;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x) {
        float val = deq1(type, row + (uint64_t)(i / be) * bb, i % be);
        h[(uint64_t)v * ldh + i] = apply_scale ? __fmul_rn(val, scale) : val;
    }
}

int launch_embed(const uint8_t *emb, uint32_t type, int hidden, int vocab, const int32_t *tokens, int nv, float scale,
                 float *h, int ldh, int *err, cudaStream_t st)
{
    embed_kernel<<<dim3((hidden + 255) / 256, nv), 256, 0, st>>>(emb, type, hidden, row_bytes(type, hidden), vocab, tokens,
                                                                 scale, scale != 1.0f, h, ldh, err);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

}  // namespace llmdot
