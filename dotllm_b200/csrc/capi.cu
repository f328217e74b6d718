// capi.cu -- the extern "C" entry points declared in include/llmdot_cuda.h.
#include <string.h>

#include <algorithm>
#include <random>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "engine.cuh"
#include "sample.cuh"
#include "gemv.cuh"
#include "gguf_loader.h"
#include "tp.cuh"
#include "ops.cuh"

namespace llmdot {

static thread_local std::string g_err = "";

void set_error(const std::string &msg) { g_err = msg; }
int fail(int code, const std::string &msg)
{
    g_err = msg;
    return code;
}
int cuda_fail(cudaError_t e, const char *what)
{
    g_err = std::string(what) + ": " + cudaGetErrorString(e);
    return LLMDOT_E_CUDA;
}

}  // namespace llmdot

using namespace llmdot;

// ===================================================================== misc
extern "C" const char *llmdot_cuda_last_error(void) { return g_err.c_str(); }
extern "C" const char *llmdot_cuda_version(void) { return "llmdot-cuda 0.1 sm_100a"; }
extern "C" int llmdot_cuda_device_count(int *count)
{
    if (!count) return fail(LLMDOT_E_INVALID, "count is null");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    *count = n;
    return LLMDOT_OK;
}

// ===================================================================== Tier A
struct llmdot_backend {
    int device = 0;
    cudaStream_t st = nullptr;
    struct Cached {
        void *ptr = nullptr;
        size_t bytes = 0;
    };
    std::map<std::string, Cached> weights;
    void *scratch[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};  // 4: the sampler's full-row work
    size_t scratch_bytes[5] = {0, 0, 0, 0, 0};
    unsigned long long *keys = nullptr;
    int32_t *idx = nullptr;
};

static int scratch(llmdot_backend *h, int slot, size_t bytes, void **out)
{
    if (h->scratch_bytes[slot] < bytes) {
        if (h->scratch[slot]) cudaFree(h->scratch[slot]);
        h->scratch[slot] = nullptr;
        h->scratch_bytes[slot] = 0;
        size_t want = (bytes < 4096 ? 4096 : bytes) + 256;  // slack: no kernel reads past an allocation
        cudaError_t e = cudaMalloc(&h->scratch[slot], want);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return fail(LLMDOT_E_NOMEM, "scratch allocation failed");
        }
        h->scratch_bytes[slot] = want;
    }
    *out = h->scratch[slot];
    return LLMDOT_OK;
}

static int enter(llmdot_backend *h)
{
    if (!h) return fail(LLMDOT_E_INVALID, "backend handle is null");
    LLMDOT_CUDA_TRY(cudaSetDevice(h->device));
    return LLMDOT_OK;
}

static int finish(llmdot_backend *h)
{
    LLMDOT_CUDA_TRY(cudaStreamSynchronize(h->st));
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

static int up(llmdot_backend *h, int slot, const void *src, size_t bytes, void **dev)
{
    LLMDOT_TRY(scratch(h, slot, bytes, dev));
    if (bytes) LLMDOT_CUDA_TRY(cudaMemcpyAsync(*dev, src, bytes, cudaMemcpyHostToDevice, h->st));
    return LLMDOT_OK;
}

static int down(llmdot_backend *h, void *dst, const void *dev, size_t bytes)
{
    if (bytes) LLMDOT_CUDA_TRY(cudaMemcpyAsync(dst, dev, bytes, cudaMemcpyDeviceToHost, h->st));
    return finish(h);
}

// Weight upload keyed by the tensor name, like MetalBackend's persistent buffers
// (src/Llmdot.Metal/MetalBackend.cs:85-104).
static int weight(llmdot_backend *h, const char *key, const void *src, size_t bytes, const void **dev)
{
    if (!key) {
        void *p;
        LLMDOT_TRY(up(h, 3, src, bytes, &p));
        *dev = p;
        return LLMDOT_OK;
    }
    auto it = h->weights.find(key);
    if (it != h->weights.end() && it->second.bytes >= bytes) {
        *dev = it->second.ptr;
        return LLMDOT_OK;
    }
    if (!src) return fail(LLMDOT_E_INVALID, "weight data is null");
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes + 256);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(LLMDOT_E_NOMEM, "weight allocation failed");
    }
    LLMDOT_CUDA_TRY(cudaMemsetAsync((uint8_t *)p + bytes, 0, 256, h->st));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(p, src, bytes, cudaMemcpyHostToDevice, h->st));
    if (it != h->weights.end()) cudaFree(it->second.ptr);
    h->weights[key] = {p, bytes};
    *dev = p;
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_create(int device, llmdot_backend **out)
{
    if (!out) return fail(LLMDOT_E_INVALID, "out is null");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(LLMDOT_E_CUDA, "no CUDA device available");
    }
    if (device < 0 || device >= n) return fail(LLMDOT_E_INVALID, "device index out of range");
    LLMDOT_CUDA_TRY(cudaSetDevice(device));
    auto *h = new llmdot_backend();
    h->device = device;
    if (cudaStreamCreateWithFlags(&h->st, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&h->keys, 64 * sizeof(unsigned long long)) != cudaSuccess ||
        cudaMalloc(&h->idx, 64 * sizeof(int32_t)) != cudaSuccess) {
        cudaGetLastError();
        llmdot_cuda_destroy(h);
        return fail(LLMDOT_E_CUDA, "backend initialisation failed");
    }
    *out = h;
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_destroy(llmdot_backend *h)
{
    if (!h) return LLMDOT_OK;
    cudaSetDevice(h->device);
    if (h->st) cudaStreamSynchronize(h->st);
    for (auto &kv : h->weights) cudaFree(kv.second.ptr);
    for (int i = 0; i < 5; i++)
        if (h->scratch[i]) cudaFree(h->scratch[i]);
    if (h->keys) cudaFree(h->keys);
    if (h->idx) cudaFree(h->idx);
    if (h->st) cudaStreamDestroy(h->st);
    delete h;
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_matmul(llmdot_backend *h, const float *a, int aLen, const uint8_t *b, size_t bBytes,
                                  uint32_t bType, int aCols, int bCols, const char *weightKey, float *result,
                                  int resultLen)
{
    LLMDOT_TRY(enter(h));
    if (!a || !result || aCols <= 0 || bCols <= 0) return fail(LLMDOT_E_INVALID, "matmul: bad arguments");
    int aRows = resultLen / bCols;  // TensorOps.cs:62
    if (aRows <= 0 || (int64_t)aRows * aCols > aLen) return fail(LLMDOT_E_INVALID, "matmul: a is shorter than aRows*aCols");
    if (block_elems(bType) == 0) return fail(LLMDOT_E_UNSUPPORTED, "matmul: unsupported type " + std::to_string(bType));
    uint64_t need = row_bytes(bType, (uint64_t)aCols) * (uint64_t)bCols;
    if (bType == T_Q3_K) need += 2;  // the reference's Q3_K decode reads one byte past each block
    if (bBytes < need && !(weightKey && h->weights.count(weightKey)))
        return fail(LLMDOT_E_INVALID, bType == T_Q3_K ? "matmul: Q3_K reads one byte past its last block; b needs 2 bytes of slack"
                                                      : "matmul: b is shorter than bCols rows");
    const void *wd;
    LLMDOT_TRY(weight(h, weightKey, b, need, &wd));
    void *xa, *yd;
    LLMDOT_TRY(up(h, 0, a, sizeof(float) * (size_t)aRows * aCols, &xa));
    LLMDOT_TRY(scratch(h, 1, sizeof(float) * (size_t)aRows * bCols, &yd));
    LLMDOT_TRY(launch_gemv_ref((const uint8_t *)wd, bType, bCols, aCols, (const float *)xa, aCols, aRows, (float *)yd,
                               bCols, false, h->st));
    return down(h, result, yd, sizeof(float) * (size_t)aRows * bCols);
}

extern "C" int llmdot_cuda_matmul_f32(llmdot_backend *h, const float *a, int aLen, const float *b, size_t bLen, int aCols,
                                      int bCols, const char *weightKey, float *result, int resultLen)
{
    LLMDOT_TRY(enter(h));
    if (!a || !result || aCols <= 0 || bCols <= 0) return fail(LLMDOT_E_INVALID, "matmul_f32: bad arguments");
    int aRows = resultLen / bCols;
    if (aRows <= 0 || (int64_t)aRows * aCols > aLen) return fail(LLMDOT_E_INVALID, "matmul_f32: a too short");
    size_t need = sizeof(float) * (size_t)aCols * bCols;
    if (bLen < (size_t)aCols * bCols && !(weightKey && h->weights.count(weightKey)))
        return fail(LLMDOT_E_INVALID, "matmul_f32: b too short");
    const void *wd;
    LLMDOT_TRY(weight(h, weightKey, b, need, &wd));
    void *xa, *yd;
    LLMDOT_TRY(up(h, 0, a, sizeof(float) * (size_t)aRows * aCols, &xa));
    LLMDOT_TRY(scratch(h, 1, sizeof(float) * (size_t)aRows * bCols, &yd));
    LLMDOT_TRY(launch_gemv_ref((const uint8_t *)wd, T_F32, bCols, aCols, (const float *)xa, aCols, aRows, (float *)yd,
                               bCols, false, h->st));
    return down(h, result, yd, sizeof(float) * (size_t)aRows * bCols);
}

extern "C" int llmdot_cuda_rmsnorm(llmdot_backend *h, const float *input, const float *weights, float *output, int n,
                                   float epsilon)
{
    LLMDOT_TRY(enter(h));
    if (!input || !weights || !output || n <= 0) return fail(LLMDOT_E_INVALID, "rmsnorm: bad arguments");
    void *x, *w;
    LLMDOT_TRY(up(h, 0, input, sizeof(float) * n, &x));
    LLMDOT_TRY(up(h, 1, weights, sizeof(float) * n, &w));
    LLMDOT_TRY(launch_rmsnorm((float *)x, n, (float *)w, (float *)x, n, n, 1, epsilon, h->st));
    return down(h, output, x, sizeof(float) * n);
}

extern "C" int llmdot_cuda_layernorm(llmdot_backend *h, const float *input, const float *weights, const float *bias,
                                     float *output, int n, float epsilon)
{
    LLMDOT_TRY(enter(h));
    if (!input || !weights || !output || n <= 0) return fail(LLMDOT_E_INVALID, "layernorm: bad arguments");
    void *x, *w, *b = nullptr, *o;
    LLMDOT_TRY(up(h, 0, input, sizeof(float) * n, &x));
    LLMDOT_TRY(up(h, 1, weights, sizeof(float) * n, &w));
    if (bias) LLMDOT_TRY(up(h, 2, bias, sizeof(float) * n, &b));
    LLMDOT_TRY(scratch(h, 3, sizeof(float) * n, &o));
    LLMDOT_TRY(launch_layernorm((float *)x, (float *)w, (float *)b, (float *)o, n, epsilon, h->st));
    return down(h, output, o, sizeof(float) * n);
}

static int rope_common(llmdot_backend *h, float *query, int qLen, float *key, int kLen, int headDim, const float *cs,
                       const float *sn, int half)
{
    if (!query || !key || half <= 0 || 2 * half > qLen || (key != query && 2 * half > kLen))
        return fail(LLMDOT_E_INVALID, "rope: bad arguments");
    (void)headDim;
    // TensorOps.ApplyRoPECore (TensorOps.cs:699-743) rotates the pairs (i, i+half) of the
    // first 2*half elements of each span and leaves the rest untouched, whatever the span
    // length (InferenceEngine calls it once per head).
    void *tab;
    LLMDOT_TRY(scratch(h, 2, sizeof(float) * 2 * half, &tab));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(tab, cs, sizeof(float) * half, cudaMemcpyHostToDevice, h->st));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync((float *)tab + half, sn, sizeof(float) * half, cudaMemcpyHostToDevice, h->st));
    void *q;
    LLMDOT_TRY(up(h, 0, query, sizeof(float) * qLen, &q));
    LLMDOT_TRY(launch_rope((float *)q, 1, 2 * half, (float *)tab, (float *)tab + half, half, h->st));
    if (key != query) {
        void *k;
        LLMDOT_TRY(up(h, 1, key, sizeof(float) * kLen, &k));
        LLMDOT_TRY(launch_rope((float *)k, 1, 2 * half, (float *)tab, (float *)tab + half, half, h->st));
        LLMDOT_CUDA_TRY(cudaMemcpyAsync(key, k, sizeof(float) * kLen, cudaMemcpyDeviceToHost, h->st));
    }
    return down(h, query, q, sizeof(float) * qLen);
}

extern "C" int llmdot_cuda_rope(llmdot_backend *h, float *query, int qLen, float *key, int kLen, int headDim,
                                int position, float freqBase, int rotaryDim)
{
    LLMDOT_TRY(enter(h));
    // TensorOps.ApplyRoPE(.., freqBase, rotaryDim) (TensorOps.cs:658-677): the cos/sin table
    // is built on the host with the C runtime, as MathF does.
    int rd = rotaryDim > 0 ? rotaryDim : headDim;
    int half = rd / 2;
    std::vector<float> cs(half), sn(half);
    for (int i = 0; i < half; i++) {
        float f = 1.0f / powf(freqBase, 2.0f * (float)i / (float)rd);
        float a = (float)position * f;
        cs[i] = cosf(a);
        sn[i] = sinf(a);
    }
    return rope_common(h, query, qLen, key, kLen, headDim, cs.data(), sn.data(), half);
}

extern "C" int llmdot_cuda_rope_table(llmdot_backend *h, float *query, int qLen, float *key, int kLen, int headDim,
                                      int position, const float *freqTable, int halfDim)
{
    LLMDOT_TRY(enter(h));
    if (!freqTable) return fail(LLMDOT_E_INVALID, "rope_table: freqTable is null");
    std::vector<float> cs(halfDim), sn(halfDim);
    for (int i = 0; i < halfDim; i++) {
        float a = (float)position * freqTable[i];
        cs[i] = cosf(a);
        sn[i] = sinf(a);
    }
    return rope_common(h, query, qLen, key, kLen, headDim, cs.data(), sn.data(), halfDim);
}

extern "C" int llmdot_cuda_softmax(llmdot_backend *h, float *x, int n, int hasSoftcap, float softcap)
{
    LLMDOT_TRY(enter(h));
    if (n == 0) return LLMDOT_OK;  // VectorMath.cs:217
    if (!x || n < 0) return fail(LLMDOT_E_INVALID, "softmax: bad arguments");
    void *d;
    LLMDOT_TRY(up(h, 0, x, sizeof(float) * n, &d));
    LLMDOT_TRY(launch_softmax((float *)d, n, hasSoftcap != 0, softcap, h->st));
    return down(h, x, d, sizeof(float) * n);
}

static int unary(llmdot_backend *h, int op, const float *a, const float *b, float *out, int n, float s)
{
    LLMDOT_TRY(enter(h));
    if (n == 0) return LLMDOT_OK;
    if (!a || !out || n < 0) return fail(LLMDOT_E_INVALID, "element-wise op: bad arguments");
    void *da, *db = nullptr;
    LLMDOT_TRY(up(h, 0, a, sizeof(float) * n, &da));
    if (b) LLMDOT_TRY(up(h, 1, b, sizeof(float) * n, &db));
    LLMDOT_TRY(launch_eltwise(op, (float *)da, (float *)db, (float *)da, n, s, h->st, n));
    return down(h, out, da, sizeof(float) * n);
}

extern "C" int llmdot_cuda_silu(llmdot_backend *h, const float *input, float *result, int n)
{
    return unary(h, OP_SILU, input, nullptr, result, n, 0.0f);
}
extern "C" int llmdot_cuda_silu_inplace(llmdot_backend *h, float *x, int n) { return unary(h, OP_SILU, x, nullptr, x, n, 0.0f); }
extern "C" int llmdot_cuda_gelu(llmdot_backend *h, const float *input, float *result, int n)
{
    return unary(h, OP_GELU, input, nullptr, result, n, 0.0f);
}
extern "C" int llmdot_cuda_gelu_scalar(llmdot_backend *h, float x, float *result)
{
    LLMDOT_TRY(enter(h));
    if (!result) return fail(LLMDOT_E_INVALID, "gelu_scalar: result is null");
    void *d;
    LLMDOT_TRY(scratch(h, 0, sizeof(float), &d));
    LLMDOT_TRY(launch_gelu_scalar(x, (float *)d, h->st));
    return down(h, result, d, sizeof(float));
}
extern "C" int llmdot_cuda_add_inplace(llmdot_backend *h, float *a, const float *b, int n)
{
    if (!b && n) return fail(LLMDOT_E_INVALID, "add: b is null");
    return unary(h, OP_ADD, a, b, a, n, 0.0f);
}
extern "C" int llmdot_cuda_add(llmdot_backend *h, const float *a, const float *b, float *result, int n)
{
    if (!b && n) return fail(LLMDOT_E_INVALID, "add: b is null");
    return unary(h, OP_ADD, a, b, result, n, 0.0f);
}
extern "C" int llmdot_cuda_scale(llmdot_backend *h, const float *input, float scale, float *result, int n)
{
    return unary(h, OP_SCALE, input, nullptr, result, n, scale);
}
extern "C" int llmdot_cuda_scale_inplace(llmdot_backend *h, float *x, int n, float scale)
{
    return unary(h, OP_SCALE, x, nullptr, x, n, scale);
}
extern "C" int llmdot_cuda_mul(llmdot_backend *h, const float *a, const float *b, float *result, int n)
{
    if (!b && n) return fail(LLMDOT_E_INVALID, "mul: b is null");
    return unary(h, OP_MUL, a, b, result, n, 0.0f);
}
extern "C" int llmdot_cuda_softcap(llmdot_backend *h, float *x, int n, float cap)
{
    return unary(h, OP_SOFTCAP, x, nullptr, x, n, cap);
}

extern "C" int llmdot_cuda_conv1d(llmdot_backend *h, const float *input, const float *weights, float *output,
                                  int kernelSize, int inputDim)
{
    LLMDOT_TRY(enter(h));
    if (!input || !weights || !output || kernelSize <= 0 || inputDim <= 0)
        return fail(LLMDOT_E_INVALID, "conv1d: bad arguments");
    size_t n = (size_t)kernelSize * inputDim;
    void *di, *dw, *dout;
    LLMDOT_TRY(up(h, 0, input, sizeof(float) * (kernelSize == 1 ? inputDim : n), &di));
    LLMDOT_TRY(up(h, 1, weights, sizeof(float) * (kernelSize == 1 ? inputDim : n), &dw));
    LLMDOT_TRY(scratch(h, 2, sizeof(float) * inputDim, &dout));
    LLMDOT_TRY(launch_conv1d((float *)di, (float *)dw, (float *)dout, kernelSize, inputDim, h->st));
    return down(h, output, dout, sizeof(float) * inputDim);
}

extern "C" int llmdot_cuda_dequantize(llmdot_backend *h, const uint8_t *src, size_t srcBytes, uint32_t type, int numRows,
                                      int rowElements, float *dst)
{
    LLMDOT_TRY(enter(h));
    if (!src || !dst || numRows < 0 || rowElements < 0) return fail(LLMDOT_E_INVALID, "dequantize: bad arguments");
    if (block_elems(type) == 0) return fail(LLMDOT_E_UNSUPPORTED, "dequantize: unsupported type " + std::to_string(type));
    uint64_t need = row_bytes(type, (uint64_t)rowElements) * (uint64_t)numRows;
    if (srcBytes < need) return fail(LLMDOT_E_INVALID, "dequantize: src shorter than numRows rows");
    // The reference's Q3_K decoder reads byte 111 of each 110-byte block (DequantizeK.cs:65),
    // i.e. one byte of the next block; on the final block it throws IndexOutOfRangeException.
    if (type == T_Q3_K && numRows > 0) {
        if (srcBytes < need + 2)
            return fail(LLMDOT_E_INVALID, "dequantize: Q3_K reads one byte past its last block (as the reference does); "
                                          "src needs 2 bytes after the final block");
        need += 2;
    }
    size_t outBytes = sizeof(float) * (size_t)numRows * rowElements;
    if (outBytes == 0) return LLMDOT_OK;
    void *ds, *dd;
    LLMDOT_TRY(up(h, 0, src, need, &ds));
    LLMDOT_TRY(scratch(h, 1, outBytes, &dd));
    LLMDOT_TRY(launch_dequant((const uint8_t *)ds, (float *)dd, type, numRows, rowElements, h->st));
    return down(h, dst, dd, outBytes);
}

extern "C" int llmdot_cuda_argmax(llmdot_backend *h, const float *x, int n, int *index)
{
    LLMDOT_TRY(enter(h));
    if (!x || !index || n <= 0) return fail(LLMDOT_E_INVALID, "argmax: bad arguments");
    void *d;
    LLMDOT_TRY(up(h, 0, x, sizeof(float) * n, &d));
    LLMDOT_TRY(launch_argmax((float *)d, n, n, 1, h->keys, h->idx, false, 0.0f, nullptr, h->st));
    int32_t r = 0;
    LLMDOT_TRY(down(h, &r, h->idx, sizeof(int32_t)));
    *index = r;
    return LLMDOT_OK;
}

// new System.Random(seed).NextSingle(): Knuth's subtractive generator as the .NET-5-compatible
// seeded Random implements it (55-entry state, MSEED 161803398, modulus int.MaxValue), first
// sample divided by int.MaxValue, then rounded to float.
extern "C" float llmdot_cuda_sampling_seeded_draw(int32_t seed)
{
    const int MBIG = 2147483647, MSEED = 161803398;
    int sa[56] = {0};
    const int sub = seed == INT32_MIN ? MBIG : (seed < 0 ? -seed : seed);
    int mj = MSEED - sub, mk = 1;
    sa[55] = mj;
    for (int i = 1; i < 55; i++) {
        const int ii = (21 * i) % 55;
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
    int v = sa[1] - sa[22];  // the first draw reads entries 1 and 22
    if (v == MBIG) v--;
    if (v < 0) v += MBIG;
    return (float)(v * (1.0 / MBIG));
}

namespace llmdot {
static SampleArgs sample_args(const llmdot_sampling &o, int n)
{
    SampleArgs a = {};
    a.n = n;
    a.ld = n;
    a.temperature = o.temperature;
    a.inv_temp = o.temperature > 0.0f ? 1.0f / o.temperature : 0.0f;  // 1f / options.Temperature
    a.top_k = o.top_k;
    a.top_p = o.top_p;
    a.penalty = o.repeat_penalty;
    a.window = o.repeat_window > 0 ? o.repeat_window : 0;
    return a;
}
}  // namespace llmdot

extern "C" int llmdot_cuda_sample(llmdot_backend *h, const float *logits, int n, const llmdot_sampling *opt,
                                  const int32_t *recent, int n_recent, float r, int32_t *index)
{
    LLMDOT_TRY(enter(h));
    if (!logits || !opt || !index || n <= 0 || n_recent < 0 || (n_recent > 0 && !recent))
        return fail(LLMDOT_E_INVALID, "sample: bad arguments");
    SampleArgs a = sample_args(*opt, n);
    void *dl, *dr, *dp;
    LLMDOT_TRY(up(h, 0, logits, sizeof(float) * n, &dl));
    if (n_recent > 0) LLMDOT_TRY(up(h, 1, recent, sizeof(int32_t) * n_recent, &dr));
    const int32_t hp[4] = {n_recent, 0, 0, 0};  // [recent length, out, pad, r]
    int32_t hpr[4];
    memcpy(hpr, hp, sizeof(hp));
    memcpy(&hpr[3], &r, sizeof(float));
    LLMDOT_TRY(up(h, 2, hpr, sizeof(hpr), &dp));
    a.logits = (const float *)dl;
    a.recent = n_recent > 0 ? (const int32_t *)dr : nullptr;
    a.recent_len = (const int32_t *)dp;
    a.recent_ld = n_recent;
    a.out = (int32_t *)dp + 1;
    a.r = (const float *)((int32_t *)dp + 3);
    if (sample_full_row(a.temperature, a.top_k, n)) LLMDOT_TRY(scratch(h, 4, sample_work_bytes(n), &a.work));
    LLMDOT_TRY(launch_sample(a, 1, h->st));
    int32_t out = 0;
    LLMDOT_TRY(down(h, &out, (int32_t *)dp + 1, sizeof(int32_t)));
    if (out < 0) return fail(LLMDOT_E_UNSUPPORTED, "sample: a tie group of the nucleus above 8192 tokens");
    *index = out;
    return LLMDOT_OK;
}

// ===================================================================== Tier B
namespace llmdot {

// Decode-step graphs: one per (batch, kv type); the step reads tokens / positions /
// views from the workspace, so replays only need those arrays refreshed.
struct StepGraph {
    cudaGraphExec_t exec = nullptr;
    int batch = 0, kv_type = 0, kernels = 0, gen = 0;
};

struct ModelExtra {
    std::vector<StepGraph> graphs;
    int32_t *h_pinned = nullptr;  // pinned staging: tokens | pos | next  (3 * cap)
    KvView *h_views = nullptr;
    int cap = 0;
    // the sampled Generate's buffers, kept across calls: history | length | out | draw (pinned and
    // device copies), and the sampler's whole-row work
    int32_t *h_samp = nullptr, *d_samp = nullptr;
    size_t samp_n = 0;
    void *d_work = nullptr;
    size_t work_bytes = 0;
};

static std::mutex g_extra_mu;
static std::map<const llmdot_model *, ModelExtra> g_extra;

static ModelExtra &extra(const llmdot_model *m)
{
    std::lock_guard<std::mutex> lk(g_extra_mu);
    return g_extra[m];
}

static int ensure_pinned(llmdot_model *m, int batch)
{
    ModelExtra &x = extra(m);
    if (x.cap >= batch) return LLMDOT_OK;
    if (x.h_pinned) cudaFreeHost(x.h_pinned);
    if (x.h_views) cudaFreeHost(x.h_views);
    x.h_pinned = nullptr;
    x.h_views = nullptr;
    int cap = batch < 64 ? 64 : batch;
    if (cudaMallocHost(&x.h_pinned, sizeof(int32_t) * 3 * cap) != cudaSuccess ||
        cudaMallocHost(&x.h_views, sizeof(KvView) * cap) != cudaSuccess) {
        cudaGetLastError();
        return fail(LLMDOT_E_NOMEM, "pinned staging allocation failed");
    }
    x.cap = cap;
    return LLMDOT_OK;
}

// After a captured step: advance every row's position by one and record the step's greedy
// ids into the history ring (one block; batch <= 1024).
__global__ void advance_record_kernel(int32_t *pos, const int32_t *next, int32_t *hist, int32_t *hist_step, int n)
{
    int i = threadIdx.x;
    int step = *hist_step;
    if (i < n) {
        pos[i] += 1;
        hist[(step % HIST_STEPS) * n + i] = next[i];
    }
    __syncthreads();
    if (i == 0) *hist_step = step + 1;
}

static int step_graph(llmdot_model *m, int batch, int kv_type, cudaGraphExec_t *out, int *kernels = nullptr)
{
    ModelExtra &x = extra(m);
    for (size_t i = 0; i < x.graphs.size();)  // graphs captured before the workspace was reallocated
        if (x.graphs[i].gen != m->ws.gen) {
            cudaGraphExecDestroy(x.graphs[i].exec);
            x.graphs.erase(x.graphs.begin() + i);
        } else {
            i++;
        }
    for (auto &g : x.graphs)
        if (g.batch == batch && g.kv_type == kv_type) {
            *out = g.exec;
            if (kernels) *kernels = g.kernels;
            return LLMDOT_OK;
        }
    if (batch > 1024) return fail(LLMDOT_E_INVALID, "batch above 1024");
    Workspace &w = m->ws;
    cudaGraph_t graph;
    LLMDOT_CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int rc = forward_step(m, batch, kv_type, w.next, w.pos, w.views, w.next, m->stream);
    if (rc == LLMDOT_OK) {
        advance_record_kernel<<<1, batch < 32 ? 32 : batch, 0, m->stream>>>(w.pos, w.next, w.hist, w.hist_step, batch);
        if (cudaGetLastError() != cudaSuccess) rc = fail(LLMDOT_E_CUDA, "advance launch failed");
    }
    cudaError_t e = cudaStreamEndCapture(m->stream, &graph);
    if (rc != LLMDOT_OK) return rc;
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    // count the kernel nodes of one step (reported by the benchmark as launches per step)
    size_t nn = 0;
    cudaGraphGetNodes(graph, nullptr, &nn);
    std::vector<cudaGraphNode_t> nodes(nn);
    cudaGraphGetNodes(graph, nodes.data(), &nn);
    int kn = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        cudaGraphNodeGetType(nd, &t);
        kn += t == cudaGraphNodeTypeKernel;
    }
    cudaGraphExec_t exec;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
    x.graphs.push_back({exec, batch, kv_type, kn, m->ws.gen});
    *out = exec;
    if (kernels) *kernels = kn;
    return LLMDOT_OK;
}

static void drop_graphs(llmdot_model *m)
{
    std::lock_guard<std::mutex> lk(g_extra_mu);
    auto it = g_extra.find(m);
    if (it == g_extra.end()) return;
    for (auto &g : it->second.graphs) cudaGraphExecDestroy(g.exec);
    if (it->second.h_pinned) cudaFreeHost(it->second.h_pinned);
    if (it->second.h_views) cudaFreeHost(it->second.h_views);
    if (it->second.h_samp) cudaFreeHost(it->second.h_samp);
    if (it->second.d_samp) cudaFree(it->second.d_samp);
    if (it->second.d_work) cudaFree(it->second.d_work);
    g_extra.erase(it);
}

}  // namespace llmdot

extern "C" int llmdot_cuda_model_load(int device, const llmdot_config *cfg, const llmdot_tensor_desc *tensors,
                                      int n_tensors, llmdot_model **out)
{
    if (!out) return fail(LLMDOT_E_INVALID, "out is null");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(LLMDOT_E_CUDA, "no CUDA device available");
    }
    if (device < 0 || device >= n) return fail(LLMDOT_E_INVALID, "device index out of range");
    return model_upload(device, cfg, tensors, n_tensors, out);
}

extern "C" int llmdot_cuda_model_load_gguf(int device, const char *path, llmdot_model **out)
{
    if (!out || !path) return fail(LLMDOT_E_INVALID, "null argument");
    GgufModelFile f;
    LLMDOT_TRY(gguf_open(path, &f));
    std::vector<llmdot_tensor_desc> descs;
    gguf_descs(f, &descs);
    int rc = llmdot_cuda_model_load(device, &f.cfg, descs.data(), (int)descs.size(), out);
    gguf_close(&f);
    return rc;
}

extern "C" int llmdot_cuda_gguf_config(const char *path, llmdot_config *out)
{
    if (!out || !path) return fail(LLMDOT_E_INVALID, "null argument");
    GgufModelFile f;
    LLMDOT_TRY(gguf_open(path, &f));  // host only: parse and resolve, no device touched
    *out = f.cfg;
    gguf_close(&f);
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_model_load_gguf_tp(int device, const char *path, int tp_size, int tp_rank,
                                              llmdot_model **out)
{
    if (!out || !path) return fail(LLMDOT_E_INVALID, "null argument");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(LLMDOT_E_CUDA, "no CUDA device available");
    }
    if (device < 0 || device >= n) return fail(LLMDOT_E_INVALID, "device index out of range");
    GgufModelFile f;
    LLMDOT_TRY(gguf_open(path, &f));
    std::vector<llmdot_tensor_desc> descs;
    gguf_descs(f, &descs);
    int rc = model_upload(device, &f.cfg, descs.data(), (int)descs.size(), out, tp_size, tp_rank);
    gguf_close(&f);
    return rc;
}

extern "C" int llmdot_cuda_tp_shard(const llmdot_config *cfg, int tp_size, int tp_rank, int32_t *out8)
{
    if (!cfg || !out8) return fail(LLMDOT_E_INVALID, "null argument");
    TpShard sh{};
    LLMDOT_TRY(tp_shard(*cfg, tp_size, tp_rank, &sh));
    const int32_t v[8] = {sh.q_lo, sh.q_n, sh.kv_lo, sh.kv_n, sh.f_lo, sh.f_n, sh.v_lo, sh.v_n};
    memcpy(out8, v, sizeof(v));
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_tp_unique_id(uint8_t *out128)
{
    if (!out128) return fail(LLMDOT_E_INVALID, "null argument");
    return tp_unique_id(out128);
}

extern "C" int llmdot_cuda_tp_init(llmdot_model *m, const uint8_t *id128)
{
    if (!m || !id128) return fail(LLMDOT_E_INVALID, "null argument");
    if (m->tp < 2) return fail(LLMDOT_E_INVALID, "tp_init: the model was loaded without tensor parallelism");
    return tp_comm_init(m, id128);
}

extern "C" int llmdot_cuda_tp_exchange_handle(llmdot_model *m, uint8_t *out128)
{
    if (!m || !out128) return fail(LLMDOT_E_INVALID, "null argument");
    if (!m->nccl) return fail(LLMDOT_E_INVALID, "tp_exchange_handle: call llmdot_cuda_tp_init first");
    return tp_exchange_handle(m, out128);
}

extern "C" int llmdot_cuda_tp_exchange_open(llmdot_model *m, const uint8_t *handles)
{
    if (!m || !handles) return fail(LLMDOT_E_INVALID, "null argument");
    LLMDOT_TRY(tp_exchange_open(m, handles));
    drop_graphs(m);  // steps captured before use NCCL's all-reduce; the next capture uses the exchange
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_tp_exchange_use(llmdot_model *m, int on)
{
    if (!m) return fail(LLMDOT_E_INVALID, "null argument");
    LLMDOT_TRY(tp_exchange_use(m, on != 0));
    drop_graphs(m);  // captured steps hold the other all-reduce form
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_model_config(const llmdot_model *m, llmdot_config *out)
{
    if (!m || !out) return fail(LLMDOT_E_INVALID, "null argument");
    *out = m->full_cfg;
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_model_weight_bytes(const llmdot_model *m, uint64_t *layer_bytes, uint64_t *head_bytes)
{
    if (!m) return fail(LLMDOT_E_INVALID, "model is null");
    if (layer_bytes) *layer_bytes = m->layer_bytes;
    if (head_bytes) *head_bytes = m->head_bytes;
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_model_free(llmdot_model *m)
{
    if (!m) return LLMDOT_OK;
    cudaSetDevice(m->device);
    // sessions still open keep their cache until llmdot_cuda_session_free; every other call on
    // them fails instead of touching the freed model
    for (llmdot_session *s : m->sessions) s->m = nullptr;
    m->sessions.clear();
    drop_graphs(m);
    model_destroy(m);
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_session_create(llmdot_model *m, int max_ctx, int kv_type, llmdot_session **out)
{
    if (!m || !out) return fail(LLMDOT_E_INVALID, "null argument");
    if (kv_type != LLMDOT_KV_F16 && kv_type != LLMDOT_KV_F32) return fail(LLMDOT_E_INVALID, "bad kv_type");
    *out = nullptr;
    LLMDOT_CUDA_TRY(cudaSetDevice(m->device));
    if (max_ctx <= 0 || max_ctx > m->cfg.context) max_ctx = m->cfg.context;
    auto *s = new llmdot_session();
    s->device = m->device;
    s->kv_type = kv_type;
    s->n_pages = (max_ctx + KV_PAGE - 1) / KV_PAGE;
    s->max_ctx = max_ctx;
    const llmdot_config &c = m->cfg;
    size_t esz = kv_type == LLMDOT_KV_F16 ? 2 : 4;
    int64_t layer_stride = (int64_t)s->n_pages * c.heads_kv * KV_PAGE * c.head_dim;
    size_t bytes = (size_t)layer_stride * c.layers * esz;
    if (cudaMalloc(&s->k, bytes) != cudaSuccess || cudaMalloc(&s->v, bytes) != cudaSuccess ||
        cudaMalloc(&s->pages, sizeof(int32_t) * s->n_pages) != cudaSuccess) {
        cudaGetLastError();
        llmdot_cuda_session_free(s);
        return fail(LLMDOT_E_NOMEM, "KV cache allocation failed (" + std::to_string(2 * bytes) + " bytes)");
    }
    std::vector<int32_t> pt(s->n_pages);
    for (int i = 0; i < s->n_pages; i++) pt[i] = i;
    if (cudaMemcpy(s->pages, pt.data(), sizeof(int32_t) * s->n_pages, cudaMemcpyHostToDevice) != cudaSuccess) {
        const int rc = cuda_fail(cudaGetLastError(), "page table upload");
        llmdot_cuda_session_free(s);
        return rc;
    }
    s->view = {s->k, s->v, s->pages, layer_stride};
    s->m = m;
    m->sessions.push_back(s);
    *out = s;
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_session_reset(llmdot_session *s)
{
    if (!s) return fail(LLMDOT_E_INVALID, "session is null");
    s->pos = 0;  // KvCache.Reset (KvCache.cs:40): stale entries are never read past pos
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_session_position(const llmdot_session *s, int *pos)
{
    if (!s || !pos) return fail(LLMDOT_E_INVALID, "null argument");
    *pos = s->pos;
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_session_free(llmdot_session *s)
{
    if (!s) return LLMDOT_OK;
    if (s->m) {
        auto &v = s->m->sessions;
        v.erase(std::remove(v.begin(), v.end(), s), v.end());
        cudaSetDevice(s->m->device);
        cudaStreamSynchronize(s->m->stream);
    } else {
        cudaSetDevice(s->device);
    }
    if (s->k) cudaFree(s->k);
    if (s->v) cudaFree(s->v);
    if (s->pages) cudaFree(s->pages);
    delete s;
    return LLMDOT_OK;
}

// logits[v][r * rows + j] = gathered[r][v][j]
__global__ void logits_unshard_kernel(const float *__restrict__ g, float *__restrict__ full, int tp, int batch, int rows,
                                      int vocab)
{
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)tp * batch * rows) return;
    const int j = (int)(i % rows), v = (int)((i / rows) % batch), r = (int)(i / ((size_t)rows * batch));
    full[(size_t)v * vocab + (size_t)r * rows + j] = g[i];
}

// Copies row `row` (or all `batch` rows when row < 0) of the step's logits to host memory; under
// tensor parallelism the vocabulary shards are gathered from every rank first (even split only).
static int read_logits(llmdot_model *m, int batch, int row, float *host, cudaStream_t st)
{
    const int V = m->cfg.vocab;
    const size_t count = (size_t)V * (row < 0 ? batch : 1);
    if (m->tp > 1) {
        if (V % m->tp) return fail(LLMDOT_E_UNSUPPORTED, "logits read-back under TP needs vocab % tp == 0");
        const size_t per = (size_t)batch * m->head_rows;
        float *g = nullptr;
        LLMDOT_CUDA_TRY(cudaMallocAsync(&g, sizeof(float) * (per * m->tp + (size_t)batch * V), st));
        float *full = g + per * m->tp;
        int rc = tp_allgather(m, m->ws.logits, g, per, st);
        if (rc == LLMDOT_OK) {
            const size_t n = per * m->tp;
            logits_unshard_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, full, m->tp, batch, m->head_rows, V);
            if (cudaGetLastError() != cudaSuccess) rc = fail(LLMDOT_E_CUDA, "logits unshard launch");
        }
        if (rc == LLMDOT_OK && cudaMemcpyAsync(host, full + (row < 0 ? 0 : (size_t)row * V), sizeof(float) * count,
                                               cudaMemcpyDeviceToHost, st) != cudaSuccess)
            rc = cuda_fail(cudaGetLastError(), "logits copy");
        cudaStreamSynchronize(st);
        cudaFreeAsync(g, st);
        return rc;
    }
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(host, m->ws.logits + (row < 0 ? 0 : (size_t)row * V), sizeof(float) * count,
                                    cudaMemcpyDeviceToHost, st));
    return LLMDOT_OK;
}

static int check_err_flag(llmdot_model *m)
{
    LLMDOT_TRY(gemv_timeout_check());
    LLMDOT_TRY(attention_timeout_check());
    int e = 0;
    LLMDOT_CUDA_TRY(cudaMemcpy(&e, m->ws.err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
        cudaMemset(m->ws.err, 0, sizeof(int));
        if (e == 1) return fail(LLMDOT_E_INVALID, "token id outside the vocabulary");
        if (e == 5) return fail(LLMDOT_E_TIMEOUT, "tensor-core matmul: a bounded wait gave up");
        if (e == 6) return fail(LLMDOT_E_TIMEOUT, "tensor parallel: a peer exchange wait gave up");
        return fail(LLMDOT_E_CUDA, "device error flag " + std::to_string(e));
    }
    return LLMDOT_OK;
}

static int prefill_rows(llmdot_session *s, const int32_t *tokens, int n, float *logits, int32_t *next_token,
                        int *last_row_out);

extern "C" int llmdot_cuda_prefill(llmdot_session *s, const int32_t *tokens, int n, float *logits, int32_t *next_token)
{
    return prefill_rows(s, tokens, n, logits, next_token, nullptr);
}

// The prefill; *last_row_out (nullable) receives the workspace row of the last token's logits.
static int prefill_rows(llmdot_session *s, const int32_t *tokens, int n, float *logits, int32_t *next_token,
                        int *last_row_out)
{
    if (!s || (!tokens && n > 0) || n < 0) return fail(LLMDOT_E_INVALID, "prefill: bad arguments");
    llmdot_model *m = s->m;
    if (!m) return fail(LLMDOT_E_INVALID, "prefill: the session's model was freed");
    LLMDOT_CUDA_TRY(cudaSetDevice(m->device));
    if (s->pos + n > s->max_ctx) return fail(LLMDOT_E_INVALID, "prefill: context length exceeded");
    if (n == 0) return LLMDOT_OK;
    const llmdot_config &c = m->cfg;
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= c.vocab) return fail(LLMDOT_E_INVALID, "prefill: token id outside the vocabulary");
    LLMDOT_TRY(ensure_workspace(m, 1));
    Workspace &w = m->ws;
    cudaStream_t st = m->stream;
    // The reference feeds the prompt token by token (InferenceEngine.cs:84-88); here runs of up
    // to 32 consecutive tokens go through each layer together (same arithmetic per token, the
    // K/V of a chunk appended before its attention so every token still sees only its prefix)
    int32_t *dtok = nullptr, *dpos = nullptr;
    LLMDOT_CUDA_TRY(cudaMallocAsync(&dtok, sizeof(int32_t) * 2 * n, st));
    dpos = dtok + n;
    std::vector<int32_t> hp(2 * (size_t)n);
    for (int i = 0; i < n; i++) {
        hp[i] = tokens[i];
        hp[n + i] = s->pos + i;
    }
    cudaMemcpyAsync(dtok, hp.data(), sizeof(int32_t) * 2 * n, cudaMemcpyHostToDevice, st);
    int rc = LLMDOT_OK;
    int last_row = 0;  // row of the workspace that holds the last prompt token's logits
    if (m->use_fast_gemv) {
        // prompt chunks of up to TC_MAX_ROWS consecutive positions, one batched step each
        const int CH = n < TC_MAX_ROWS ? n : TC_MAX_ROWS;
        rc = ensure_workspace(m, CH);
        if (rc == LLMDOT_OK) {
            std::vector<KvView> vs(CH, s->view);
            if (cudaMemcpyAsync(w.views, vs.data(), sizeof(KvView) * CH, cudaMemcpyHostToDevice, st) != cudaSuccess)
                rc = cuda_fail(cudaGetLastError(), "prefill views");
            for (int c0 = 0; c0 < n && rc == LLMDOT_OK; c0 += CH) {
                const int T = n - c0 < CH ? n - c0 : CH;
                const bool last = c0 + T == n;
                rc = forward_step(m, T, s->kv_type, dtok + c0, dpos + c0, w.views, w.next, st,
                                  STEP_CHUNK | (last ? 0 : STEP_NO_HEAD));
                last_row = T - 1;
            }
        }
    } else {
        cudaMemcpyAsync(w.views, &s->view, sizeof(KvView), cudaMemcpyHostToDevice, st);
        for (int i = 0; i < n && rc == LLMDOT_OK; i++)
            rc = forward_step(m, 1, s->kv_type, dtok + i, dpos + i, w.views, w.next, st);
    }
    cudaFreeAsync(dtok, st);
    if (rc != LLMDOT_OK) return rc;
    if (logits) LLMDOT_TRY(read_logits(m, last_row + 1, last_row, logits, st));
    int32_t nt = 0;
    // the device loop of generate feeds next[0]: the last prompt token's argmax goes there
    if (last_row > 0)
        LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.next, w.next + last_row, sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(&nt, w.next, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    LLMDOT_CUDA_TRY(cudaStreamSynchronize(st));
    LLMDOT_TRY(check_err_flag(m));
    s->pos += n;
    if (next_token) *next_token = nt;
    if (last_row_out) *last_row_out = last_row;
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_decode(llmdot_session **sessions, int batch, const int32_t *tokens, int32_t *next_tokens,
                                  float *logits)
{
    if (!sessions || batch <= 0 || !tokens || !next_tokens) return fail(LLMDOT_E_INVALID, "decode: bad arguments");
    llmdot_model *m = sessions[0] ? sessions[0]->m : nullptr;
    if (!m) return fail(LLMDOT_E_INVALID, "decode: null session, or its model was freed");
    const int kv_type = sessions[0]->kv_type;
    for (int i = 0; i < batch; i++) {
        llmdot_session *s = sessions[i];
        if (!s || s->m != m) return fail(LLMDOT_E_INVALID, "decode: sessions must share one model");
        if (s->kv_type != kv_type) return fail(LLMDOT_E_INVALID, "decode: sessions must share one KV type");
        if (s->pos >= s->max_ctx) return fail(LLMDOT_E_INVALID, "decode: context length exceeded");
        if (tokens[i] < 0 || tokens[i] >= m->cfg.vocab) return fail(LLMDOT_E_INVALID, "decode: token id outside the vocabulary");
        for (int j = 0; j < i; j++)
            if (sessions[j] == s) return fail(LLMDOT_E_INVALID, "decode: a session appears twice in the batch");
    }
    LLMDOT_CUDA_TRY(cudaSetDevice(m->device));
    LLMDOT_TRY(ensure_workspace(m, batch));
    LLMDOT_TRY(ensure_pinned(m, batch));
    ModelExtra &x = extra(m);
    Workspace &w = m->ws;
    cudaStream_t st = m->stream;
    for (int i = 0; i < batch; i++) {
        x.h_pinned[i] = tokens[i];
        x.h_pinned[x.cap + i] = sessions[i]->pos;
        x.h_views[i] = sessions[i]->view;
    }
    cudaGraphExec_t g = nullptr;
    LLMDOT_TRY(step_graph(m, batch, kv_type, &g));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.next, x.h_pinned, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, st));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.pos, x.h_pinned + x.cap, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, st));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.views, x.h_views, sizeof(KvView) * batch, cudaMemcpyHostToDevice, st));
    LLMDOT_CUDA_TRY(cudaGraphLaunch(g, st));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(x.h_pinned + 2 * x.cap, w.next, sizeof(int32_t) * batch, cudaMemcpyDeviceToHost, st));
    if (logits) LLMDOT_TRY(read_logits(m, batch, -1, logits, st));
    LLMDOT_CUDA_TRY(cudaStreamSynchronize(st));
    LLMDOT_TRY(check_err_flag(m));
    for (int i = 0; i < batch; i++) {
        next_tokens[i] = x.h_pinned[2 * x.cap + i];
        sessions[i]->pos += 1;
    }
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_generate(llmdot_session *s, const int32_t *prompt, int n_prompt, int max_tokens,
                                    int32_t *out_tokens, int *n_out)
{
    if (!s || !out_tokens || !n_out || max_tokens < 0 || n_prompt < 0 || (n_prompt > 0 && !prompt))
        return fail(LLMDOT_E_INVALID, "generate: bad arguments");
    llmdot_model *m = s->m;
    if (!m) return fail(LLMDOT_E_INVALID, "generate: the session's model was freed");
    *n_out = 0;
    LLMDOT_TRY(llmdot_cuda_session_reset(s));  // InferenceEngine.cs:79
    int32_t next = 0;
    if (n_prompt > 0) {
        LLMDOT_TRY(llmdot_cuda_prefill(s, prompt, n_prompt, nullptr, &next));
    } else {
        int32_t init = m->cfg.bos > 0 ? m->cfg.bos : 0;  // InferenceEngine.cs:90-95
        LLMDOT_TRY(llmdot_cuda_prefill(s, &init, 1, nullptr, &next));
    }
    if (max_tokens == 0) return LLMDOT_OK;
    LLMDOT_CUDA_TRY(cudaSetDevice(m->device));
    LLMDOT_TRY(ensure_pinned(m, 1));
    ModelExtra &x = extra(m);
    Workspace &w = m->ws;
    cudaStream_t st = m->stream;
    cudaGraphExec_t g = nullptr;
    LLMDOT_TRY(step_graph(m, 1, s->kv_type, &g));
    // device state: w.next holds the token to feed, w.pos its position
    x.h_pinned[x.cap] = s->pos;
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.pos, x.h_pinned + x.cap, sizeof(int32_t), cudaMemcpyHostToDevice, st));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.views, &s->view, sizeof(KvView), cudaMemcpyHostToDevice, st));
    int produced = 0;
    while (true) {
        out_tokens[produced++] = next;
        if (next == m->cfg.eos || produced == max_tokens) break;
        if (s->pos >= s->max_ctx) return fail(LLMDOT_E_INVALID, "generate: context length exceeded");
        LLMDOT_CUDA_TRY(cudaGraphLaunch(g, st));
        LLMDOT_CUDA_TRY(cudaMemcpyAsync(x.h_pinned + 2 * x.cap, w.next, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
        LLMDOT_CUDA_TRY(cudaStreamSynchronize(st));
        next = x.h_pinned[2 * x.cap];
        s->pos += 1;
    }
    *n_out = produced;
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_generate_sampled(llmdot_session *s, const int32_t *prompt, int n_prompt, int max_tokens,
                                            const llmdot_sampling *opt, const float *draws, int32_t *out_tokens,
                                            int *n_out)
{
    if (!s || !opt || !out_tokens || !n_out || max_tokens < 0 || n_prompt < 0 || (n_prompt > 0 && !prompt))
        return fail(LLMDOT_E_INVALID, "generate_sampled: bad arguments");
    llmdot_model *m = s->m;
    if (!m) return fail(LLMDOT_E_INVALID, "generate_sampled: the session's model was freed");
    if (m->tp > 1) return fail(LLMDOT_E_UNSUPPORTED, "generate_sampled: not under tensor parallelism");
    const llmdot_config &c = m->cfg;
    SampleArgs a = sample_args(*opt, c.vocab);
    const bool full_row = sample_full_row(a.temperature, a.top_k, c.vocab);
    if (a.temperature > 0.0f && !full_row && a.top_k > SAMPLE_MAX_TOP_K)
        return fail(LLMDOT_E_UNSUPPORTED, "generate_sampled: top_k above 1024 (and below the vocabulary)");
    if (a.window > SAMPLE_MAX_WINDOW) return fail(LLMDOT_E_UNSUPPORTED, "generate_sampled: repeat window above 1024");
    *n_out = 0;
    LLMDOT_TRY(llmdot_cuda_session_reset(s));  // InferenceEngine.cs:79
    int last_row = 0;
    int32_t first = 0;
    if (n_prompt > 0) {
        LLMDOT_TRY(prefill_rows(s, prompt, n_prompt, nullptr, &first, &last_row));
    } else {
        const int32_t init = c.bos > 0 ? c.bos : 0;  // InferenceEngine.cs:90-95
        LLMDOT_TRY(prefill_rows(s, &init, 1, nullptr, &first, &last_row));
    }
    if (max_tokens == 0) return LLMDOT_OK;
    LLMDOT_CUDA_TRY(cudaSetDevice(m->device));
    Workspace &w = m->ws;
    cudaStream_t st = m->stream;
    cudaGraphExec_t g = nullptr;
    LLMDOT_TRY(step_graph(m, 1, s->kv_type, &g));
    // the decode step's position and KV view
    ModelExtra &x = extra(m);
    LLMDOT_TRY(ensure_pinned(m, 1));
    x.h_pinned[x.cap] = s->pos;
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.pos, x.h_pinned + x.cap, sizeof(int32_t), cudaMemcpyHostToDevice, st));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.views, &s->view, sizeof(KvView), cudaMemcpyHostToDevice, st));
    // history: the prompt, then every generated token, the last window + 1 kept (:100, :109-111)
    const int keep = a.window + 1;
    std::vector<int32_t> recent(prompt, prompt + n_prompt);
    // device: [history (keep)] [length] [out] [r]
    // kept by the model across calls (a per-call pinned allocation cost more than a short
    // generation); pinned, so the per-token upload is a plain DMA
    const size_t need = (size_t)keep + 3;
    if (x.samp_n < need) {
        if (x.h_samp) cudaFreeHost(x.h_samp);
        if (x.d_samp) cudaFree(x.d_samp);
        x.h_samp = x.d_samp = nullptr;
        x.samp_n = 0;
        if (cudaMallocHost(&x.h_samp, sizeof(int32_t) * need) != cudaSuccess ||
            cudaMalloc(&x.d_samp, sizeof(int32_t) * need) != cudaSuccess) {
            cudaGetLastError();
            return fail(LLMDOT_E_NOMEM, "generate_sampled: staging allocation failed");
        }
        x.samp_n = need;
    }
    if (full_row && x.work_bytes < sample_work_bytes(c.vocab)) {
        if (x.d_work) cudaFree(x.d_work);
        x.d_work = nullptr;
        x.work_bytes = 0;
        if (cudaMalloc(&x.d_work, sample_work_bytes(c.vocab)) != cudaSuccess) {
            cudaGetLastError();
            return fail(LLMDOT_E_NOMEM, "generate_sampled: sampler work allocation failed");
        }
        x.work_bytes = sample_work_bytes(c.vocab);
    }
    int32_t *dbuf = x.d_samp, *hbuf = x.h_samp;
    if (full_row) a.work = x.d_work;
    std::mt19937 rng(std::random_device{}());
    const float seeded = opt->seed >= 0 ? llmdot_cuda_sampling_seeded_draw(opt->seed) : 0.0f;
    a.has_cap = c.has_final_cap;
    a.cap = c.final_cap;
    a.inv_cap = c.has_final_cap ? 1.0f / c.final_cap : 0.0f;
    a.recent = dbuf;
    a.recent_ld = keep;
    a.recent_len = dbuf + keep;
    a.out = dbuf + keep + 1;
    a.r = (const float *)(dbuf + keep + 2);
    a.next = w.next;  // the next decode step's input token
    int rc = LLMDOT_OK, produced = 0;
    for (int i = 0; i < max_tokens && rc == LLMDOT_OK; i++) {
        // the logits: the last prompt row after the prefill, row 0 after each decode step
        a.logits = w.logits + (size_t)(i == 0 ? last_row : 0) * c.vocab;
        const int len = (int)std::min<size_t>(recent.size(), (size_t)keep);
        std::copy(recent.end() - len, recent.end(), hbuf);
        hbuf[keep] = len;
        float r = draws ? draws[i] : (opt->seed >= 0 ? seeded : (float)(rng() >> 8) * (1.0f / 16777216.0f));
        memcpy(&hbuf[keep + 2], &r, sizeof(float));
        if (cudaMemcpyAsync(dbuf, hbuf, sizeof(int32_t) * (keep + 3), cudaMemcpyHostToDevice, st) != cudaSuccess) {
            rc = cuda_fail(cudaGetLastError(), "generate_sampled upload");
            break;
        }
        rc = launch_sample(a, 1, st);
        if (rc != LLMDOT_OK) break;
        int32_t tok = 0;
        if (cudaMemcpyAsync(x.h_pinned + 2 * x.cap, a.out, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess) {
            rc = cuda_fail(cudaGetLastError(), "generate_sampled step");
            break;
        }
        tok = x.h_pinned[2 * x.cap];
        if (tok < 0) {
            rc = fail(LLMDOT_E_UNSUPPORTED, "generate_sampled: a tie group of the nucleus above 8192 tokens");
            break;
        }
        out_tokens[produced++] = tok;
        recent.push_back(tok);
        if (recent.size() > (size_t)keep) recent.erase(recent.begin(), recent.end() - keep);
        if (tok == c.eos || produced == max_tokens) break;
        if (s->pos >= s->max_ctx) {
            rc = fail(LLMDOT_E_INVALID, "generate_sampled: context length exceeded");
            break;
        }
        if (cudaGraphLaunch(g, st) != cudaSuccess) {
            rc = cuda_fail(cudaGetLastError(), "generate_sampled decode");
            break;
        }
        s->pos += 1;
    }
    cudaStreamSynchronize(st);
    if (rc == LLMDOT_OK) rc = check_err_flag(m);
    *n_out = produced;
    return rc;
}

extern "C" int llmdot_cuda_decode_steps(llmdot_session **sessions, int batch, const int32_t *tokens, int n_steps,
                                        int32_t *out_tokens, float *elapsed_ms, int *kernels_per_step)
{
    if (!sessions || batch <= 0 || !tokens || !out_tokens || n_steps < 0)
        return fail(LLMDOT_E_INVALID, "decode_steps: bad arguments");
    llmdot_model *m = sessions[0] ? sessions[0]->m : nullptr;
    if (!m) return fail(LLMDOT_E_INVALID, "decode_steps: null session, or its model was freed");
    const int kv_type = sessions[0]->kv_type;
    for (int i = 0; i < batch; i++) {
        llmdot_session *s = sessions[i];
        if (!s || s->m != m || s->kv_type != kv_type)
            return fail(LLMDOT_E_INVALID, "decode_steps: sessions must share one model and KV type");
        if (s->pos + n_steps > s->max_ctx) return fail(LLMDOT_E_INVALID, "decode_steps: context length exceeded");
        if (tokens[i] < 0 || tokens[i] >= m->cfg.vocab) return fail(LLMDOT_E_INVALID, "decode_steps: token id outside the vocabulary");
        for (int j = 0; j < i; j++)
            if (sessions[j] == s) return fail(LLMDOT_E_INVALID, "decode_steps: a session appears twice in the batch");
    }
    LLMDOT_CUDA_TRY(cudaSetDevice(m->device));
    LLMDOT_TRY(ensure_workspace(m, batch));
    LLMDOT_TRY(ensure_pinned(m, batch));
    ModelExtra &x = extra(m);
    Workspace &w = m->ws;
    cudaStream_t st = m->stream;
    for (int i = 0; i < batch; i++) {
        x.h_pinned[i] = tokens[i];
        x.h_pinned[x.cap + i] = sessions[i]->pos;
        x.h_views[i] = sessions[i]->view;
    }
    cudaGraphExec_t g = nullptr;
    LLMDOT_TRY(step_graph(m, batch, kv_type, &g, kernels_per_step));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.next, x.h_pinned, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, st));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.pos, x.h_pinned + x.cap, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, st));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.views, x.h_views, sizeof(KvView) * batch, cudaMemcpyHostToDevice, st));
    cudaEvent_t e0, e1;
    LLMDOT_CUDA_TRY(cudaEventCreate(&e0));
    if (cudaEventCreate(&e1) != cudaSuccess) {
        const int erc = cuda_fail(cudaGetLastError(), "cudaEventCreate");
        cudaEventDestroy(e0);
        return erc;
    }
    float total_ms = 0.0f;
    int rc = LLMDOT_OK;
    for (int done = 0; done < n_steps && rc == LLMDOT_OK;) {
        int chunk = n_steps - done < HIST_STEPS ? n_steps - done : HIST_STEPS;
        cudaMemsetAsync(w.hist_step, 0, sizeof(int32_t), st);
        cudaEventRecord(e0, st);
        for (int i = 0; i < chunk; i++)
            if (cudaGraphLaunch(g, st) != cudaSuccess) {
                rc = cuda_fail(cudaGetLastError(), "cudaGraphLaunch");
                break;
            }
        cudaEventRecord(e1, st);
        if (rc == LLMDOT_OK &&
            cudaMemcpyAsync(out_tokens + (size_t)done * batch, w.hist, sizeof(int32_t) * (size_t)chunk * batch,
                            cudaMemcpyDeviceToHost, st) != cudaSuccess)
            rc = cuda_fail(cudaGetLastError(), "history copy");
        if (cudaStreamSynchronize(st) != cudaSuccess) rc = cuda_fail(cudaGetLastError(), "decode_steps");
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, e0, e1);
        total_ms += ms;
        done += chunk;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    LLMDOT_TRY(rc);
    LLMDOT_TRY(check_err_flag(m));
    for (int i = 0; i < batch; i++) sessions[i]->pos += n_steps;
    if (elapsed_ms) *elapsed_ms = total_ms;
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_profile_step(llmdot_session **sessions, int batch, const int32_t *tokens,
                                        int32_t *next_tokens, int n_families, float *family_ms, int *family_launches)
{
    if (!sessions || batch <= 0 || !tokens || n_families < 0 || (n_families > 0 && (!family_ms || !family_launches)))
        return fail(LLMDOT_E_INVALID, "profile_step: bad arguments");
    llmdot_model *m = sessions[0] ? sessions[0]->m : nullptr;
    if (!m) return fail(LLMDOT_E_INVALID, "profile_step: null session, or its model was freed");
    const int kv_type = sessions[0]->kv_type;
    for (int i = 0; i < batch; i++) {
        llmdot_session *s = sessions[i];
        if (!s || s->m != m || s->kv_type != kv_type)
            return fail(LLMDOT_E_INVALID, "profile_step: sessions must share one model and KV type");
        if (s->pos >= s->max_ctx) return fail(LLMDOT_E_INVALID, "profile_step: context length exceeded");
        if (tokens[i] < 0 || tokens[i] >= m->cfg.vocab) return fail(LLMDOT_E_INVALID, "profile_step: token id outside the vocabulary");
        for (int j = 0; j < i; j++)
            if (sessions[j] == s) return fail(LLMDOT_E_INVALID, "profile_step: a session appears twice in the batch");
    }
    LLMDOT_CUDA_TRY(cudaSetDevice(m->device));
    LLMDOT_TRY(ensure_workspace(m, batch));
    LLMDOT_TRY(ensure_pinned(m, batch));
    ModelExtra &x = extra(m);
    Workspace &w = m->ws;
    cudaStream_t st = m->stream;
    for (int i = 0; i < batch; i++) {
        x.h_pinned[i] = tokens[i];
        x.h_pinned[x.cap + i] = sessions[i]->pos;
        x.h_views[i] = sessions[i]->view;
    }
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.next, x.h_pinned, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, st));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.pos, x.h_pinned + x.cap, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, st));
    LLMDOT_CUDA_TRY(cudaMemcpyAsync(w.views, x.h_views, sizeof(KvView) * batch, cudaMemcpyHostToDevice, st));
    StepTimer tm;
    m->timer = &tm;
    int rc = forward_step(m, batch, kv_type, w.next, w.pos, w.views, w.next, st);
    m->timer = nullptr;
    if (rc == LLMDOT_OK &&
        cudaMemcpyAsync(x.h_pinned + 2 * x.cap, w.next, sizeof(int32_t) * batch, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        rc = cuda_fail(cudaGetLastError(), "profile_step copy");
    if (cudaStreamSynchronize(st) != cudaSuccess && rc == LLMDOT_OK) rc = cuda_fail(cudaGetLastError(), "profile_step");
    for (int f = 0; f < n_families; f++) {
        family_ms[f] = 0.0f;
        family_launches[f] = 0;
    }
    for (int i = 0; rc == LLMDOT_OK && i < tm.n; i++) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, tm.ev[2 * i], tm.ev[2 * i + 1]) != cudaSuccess) {
            rc = cuda_fail(cudaGetLastError(), "profile_step elapsed");
            break;
        }
        if (tm.fam[i] < n_families) {
            family_ms[tm.fam[i]] += ms;
            family_launches[tm.fam[i]] += 1;
        }
    }
    tm.destroy();
    LLMDOT_TRY(rc);
    LLMDOT_TRY(check_err_flag(m));
    for (int i = 0; i < batch; i++) {
        if (next_tokens) next_tokens[i] = x.h_pinned[2 * x.cap + i];
        sessions[i]->pos += 1;
    }
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_profile_matvec(llmdot_model *m, const char *tensor, int batch, int iters, float *avg_ms,
                                          uint64_t *bytes)
{
    if (!m || !tensor || batch <= 0 || iters <= 0) return fail(LLMDOT_E_INVALID, "profile_matvec: bad arguments");
    // "blk.*.<name>" walks the same matrix of every layer in turn, so the weights stream from HBM
    // the way they do inside a decode step instead of staying resident in L2
    std::vector<const DevMat *> mats;
    const std::string name(tensor);
    if (name.rfind("blk.*.", 0) == 0) {
        for (int l = 0; l < m->cfg.layers; l++) {
            const std::string nm = "blk." + std::to_string(l) + "." + name.substr(6);
            auto it = m->by_name.find(nm);
            if (it == m->by_name.end() || !it->second->valid()) return fail(LLMDOT_E_INVALID, "no weight " + nm);
            mats.push_back(it->second);
        }
    } else {
        auto it = m->by_name.find(name);
        if (it == m->by_name.end() || !it->second->valid()) return fail(LLMDOT_E_INVALID, "no weight " + name);
        mats.push_back(it->second);
    }
    size_t max_rows = 0, max_cols = 0;
    uint64_t total = 0;
    for (const DevMat *W : mats) {
        max_rows = std::max<size_t>(max_rows, W->rows);
        max_cols = std::max<size_t>(max_cols, W->cols);
        total += W->bytes();
    }
    LLMDOT_CUDA_TRY(cudaSetDevice(m->device));
    // as in the decode step: 5..32 rows run the batched kernel (input fragments + matmul per
    // launch), and so do 2..4 rows whose input does not fit the matvec kernel's shared memory
    bool batched = m->use_fast_gemv && batch >= 2 && batch <= TC_MAX_ROWS;
    bool any_wide = batch >= TC_MIN_ROWS;
    for (const DevMat *W : mats) {
        batched = batched && tc_supported(*W);
        any_wide = any_wide || !gemv_fast_supported(*W, batch);
    }
    batched = batched && any_wide;
    if (batched) LLMDOT_TRY(ensure_workspace(m, batch));
    float *x = nullptr, *y = nullptr;
    LLMDOT_CUDA_TRY(cudaMalloc(&x, sizeof(float) * (size_t)batch * max_cols));
    LLMDOT_CUDA_TRY(cudaMalloc(&y, sizeof(float) * (size_t)batch * max_rows));
    cudaStream_t st = m->stream;
    cudaMemsetAsync(x, 0, sizeof(float) * (size_t)batch * max_cols, st);
    auto pass = [&]() {
        for (const DevMat *W : mats) {
            int rc;
            if (batched) {
                rc = tc_prepare(x, W->cols, batch, W->cols, nullptr, m->cfg.eps, W->type == T_Q4_K, W->type == T_Q6_K,
                                m->ws.tc, st);
                const TcSeg sg = {W, y, W->rows};
                if (rc == LLMDOT_OK) rc = tc_gemm(&sg, 1, batch, GEMV_STORE, m->ws.tc, m->ws.err, st);
            } else {
                rc = gemv(*W, x, W->cols, batch, y, W->rows, false, m->use_fast_gemv, st);
            }
            if (rc != LLMDOT_OK) return rc;
        }
        return (int)LLMDOT_OK;
    };
    // the launches are replayed from a CUDA graph so the figure is device time, not the host's launch rate
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = pass();  // warm-up, sets kernel attributes outside the capture
    if (rc == LLMDOT_OK && cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
        for (int i = 0; i < iters && rc == LLMDOT_OK; i++) rc = pass();
        const cudaError_t ce = cudaStreamEndCapture(st, &graph);
        if (rc == LLMDOT_OK && ce != cudaSuccess) rc = cuda_fail(ce, "profile_matvec capture");
    } else if (rc == LLMDOT_OK) {
        rc = cuda_fail(cudaGetLastError(), "profile_matvec capture");
    }
    if (rc == LLMDOT_OK && cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess)
        rc = cuda_fail(cudaGetLastError(), "profile_matvec instantiate");
    float ms = 0.0f;
    if (rc == LLMDOT_OK) {
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaGraphLaunch(exec, st);  // first replay uploads the graph
        cudaEventRecord(e0, st);
        cudaGraphLaunch(exec, st);
        cudaEventRecord(e1, st);
        const cudaError_t ce = cudaStreamSynchronize(st);
        if (ce != cudaSuccess) rc = cuda_fail(ce, "profile_matvec");
        else cudaEventElapsedTime(&ms, e0, e1);
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    cudaFree(x);
    cudaFree(y);
    LLMDOT_TRY(rc);
    if (avg_ms) *avg_ms = ms / ((float)iters * mats.size());
    if (bytes) *bytes = total / mats.size();
    return LLMDOT_OK;
}

extern "C" int llmdot_cuda_model_matvec(llmdot_model *m, const char *tensor, const float *x, int batch, int mode,
                                        const float *norm_w, float *y)
{
    if (!m || !tensor || !x || !y || batch <= 0 || mode < 0 || mode > 2 || (mode == 2 && !norm_w))
        return fail(LLMDOT_E_INVALID, "model_matvec: bad arguments");
    auto it = m->by_name.find(tensor);
    if (it == m->by_name.end() || !it->second->valid()) return fail(LLMDOT_E_INVALID, std::string("no weight ") + tensor);
    const DevMat &W = *it->second;
    LLMDOT_CUDA_TRY(cudaSetDevice(m->device));
    auto up64 = [](size_t n) { return (n + 63) / 64 * 64; };  // keep every buffer 256-byte aligned
    const size_t nx = (size_t)batch * W.cols, ny = (size_t)batch * W.rows;
    float *dx = nullptr, *dy = nullptr, *dn = nullptr;
    LLMDOT_CUDA_TRY(cudaMalloc(&dx, sizeof(float) * (up64(nx) + up64(ny) + up64(W.cols))));
    dy = dx + up64(nx);
    dn = dy + up64(ny);
    cudaStream_t st = m->stream;
    int rc = LLMDOT_OK;
    if (cudaMemcpyAsync(dx, x, sizeof(float) * nx, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        (norm_w && cudaMemcpyAsync(dn, norm_w, sizeof(float) * W.cols, cudaMemcpyHostToDevice, st) != cudaSuccess))
        rc = cuda_fail(cudaGetLastError(), "model_matvec upload");
    const bool batched = mode != 1 && m->use_fast_gemv && batch >= 2 && batch <= TC_MAX_ROWS && tc_supported(W) &&
                         (batch >= TC_MIN_ROWS || !gemv_fast_supported(W, batch));
    if (rc == LLMDOT_OK && batched) rc = ensure_workspace(m, batch);
    if (rc == LLMDOT_OK) {
        if (batched) {
            rc = tc_prepare(dx, W.cols, batch, W.cols, mode == 2 ? dn : nullptr, m->cfg.eps, W.type == T_Q4_K,
                            W.type == T_Q6_K, m->ws.tc, st);
            const TcSeg sg = {&W, dy, W.rows};
            if (rc == LLMDOT_OK) rc = tc_gemm(&sg, 1, batch, GEMV_STORE, m->ws.tc, m->ws.err, st);
        } else if (mode == 1 || !m->use_fast_gemv || !gemv_fast_supported(W, batch)) {
            if (mode == 2) rc = fail(LLMDOT_E_UNSUPPORTED, "model_matvec: fused norm needs the tensor-core path");
            else rc = launch_gemv_ref(W.raw, W.type, W.rows, W.cols, dx, W.cols, batch, dy, W.rows, false, st);
        } else {
            rc = launch_gemv_fast_ex(W, nullptr, mode == 2 ? dn : nullptr, m->cfg.eps, dx, W.cols, batch, dy, W.rows,
                                     GEMV_STORE, st);
        }
    }
    if (rc == LLMDOT_OK && cudaMemcpyAsync(y, dy, sizeof(float) * ny, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        rc = cuda_fail(cudaGetLastError(), "model_matvec download");
    cudaError_t e = cudaStreamSynchronize(st);
    cudaFree(dx);
    LLMDOT_TRY(rc);
    if (e != cudaSuccess) return cuda_fail(e, "model_matvec");
    return LLMDOT_OK;
}
