// common.cuh -- shared host/device helpers for the llmdot B200 backend.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "../../include/llmdot_cuda.h"

namespace llmdot {

// ---------------------------------------------------------------- host errors
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
int cuda_fail(cudaError_t e, const char *what);

#define LLMDOT_CUDA_TRY(expr)                                       \
    do {                                                            \
        cudaError_t _e = (expr);                                    \
        if (_e != cudaSuccess) return ::llmdot::cuda_fail(_e, #expr); \
    } while (0)

// cudaFuncSetAttribute applies to the current device only: raise a kernel's dynamic shared-memory
// limit once per device it is launched on (done: one bit per device, one variable per kernel).
template <typename K>
inline cudaError_t smem_attr_once(std::atomic<unsigned long long> &done, K kern, int bytes)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
    return e;
}

#define LLMDOT_TRY(expr)              \
    do {                              \
        int _rc = (expr);             \
        if (_rc != LLMDOT_OK) return _rc; \
    } while (0)

// ---------------------------------------------------------------- ggml types
enum : uint32_t {
    T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8,
    T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_BF16 = 25
};

// TensorSize.ByteCount (src/Llmdot.Core/Tensors/TensorSize.cs:7-24); 0 = unsupported
__host__ __device__ inline uint64_t block_elems(uint32_t t)
{
    switch (t) {
    case T_F32: case T_F16: case T_BF16: return 1;
    case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: return 32;
    case T_Q2_K: case T_Q3_K: case T_Q4_K: case T_Q5_K: case T_Q6_K: return 256;
    default: return 0;
    }
}
__host__ __device__ inline uint64_t block_bytes(uint32_t t)
{
    switch (t) {
    case T_F32: return 4;
    case T_F16: case T_BF16: return 2;
    case T_Q4_0: return 18;
    case T_Q4_1: return 20;
    case T_Q5_0: return 22;
    case T_Q5_1: return 24;
    case T_Q8_0: return 34;
    case T_Q2_K: return 84;
    case T_Q3_K: return 110;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    default: return 0;
    }
}
__host__ __device__ inline uint64_t row_bytes(uint32_t t, uint64_t elems)
{
    uint64_t be = block_elems(t);
    return be ? elems / be * block_bytes(t) : 0;
}

// ---------------------------------------------------------------- device numerics
// Every helper below restates a reference formula with explicitly rounded IEEE
// operations (no FMA contraction), so the device result is bit-identical to the
// managed code wherever the reference uses only +, -, *, / and sqrt.

// HalfHelper.HalfToFloat (src/Llmdot.Core/Tensors/Numeric/HalfHelper.cs:7-40): exact
// binary16 -> binary32, NaN returned as the .NET float.NaN pattern 0xFFC00000.
__device__ __forceinline__ float half_to_float_ref(uint32_t h)
{
    uint32_t sign = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0) {
        if (m == 0) return __uint_as_float(sign << 31);
        int shift = __clz(m) - 21;  // leading zeros within the 11-bit field
        uint32_t norm = m << shift;
        return __uint_as_float((sign << 31) | ((uint32_t)(127 - 14 - shift) << 23) | ((norm & 0x3FFu) << 13));
    }
    if (e == 31) return m == 0 ? __uint_as_float((sign << 31) | 0x7F800000u) : __uint_as_float(0xFFC00000u);
    return __uint_as_float((sign << 31) | ((e - 15 + 127) << 23) | (m << 13));
}
__device__ __forceinline__ float ld_half(const uint8_t *p)
{
    return half_to_float_ref((uint32_t)p[0] | ((uint32_t)p[1] << 8));
}

// ExpApproxVector lane (src/Llmdot.Core/Tensors/Numeric/VectorMath.cs:137-166)
__device__ __forceinline__ float exp_approx(float x)
{
    float cl = fminf(fmaxf(x, -87.3f), 88.4f);
    int k = __float2int_rz(__fadd_rn(__fmul_rn(cl, 1.4426950408889634f), 0.5f));
    float kf = __int2float_rn(k);
    float y = __fsub_rn(__fsub_rn(cl, __fmul_rn(kf, 0.693145751953125f)), __fmul_rn(kf, 1.42860677e-6f));
    float c = __fmul_rn(__fmul_rn(y, y), 0.5f);
    float cy = __fmul_rn(c, y);
    float p = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(1.0f, y), c), __fmul_rn(cy, 0.3333333f)),
                        __fmul_rn(__fmul_rn(cy, y), 0.2f));
    float r = __fmul_rn(p, __int_as_float((k + 127) << 23));
    if (x < -87.3f) r = 0.0f;
    if (x > 88.4f) r = __int_as_float(0x7F800000);
    return r;
}

// TanhApproxVector lane (VectorMath.cs:196-209)
__device__ __forceinline__ float tanh_approx(float x)
{
    float x2 = __fmul_rn(x, x);
    float a = __fdiv_rn(__fmul_rn(x, __fadd_rn(27.0f, x2)), __fadd_rn(27.0f, __fmul_rn(9.0f, x2)));
    if (fabsf(x) > 4.0f) return x > 0.0f ? 1.0f : -1.0f;
    return a;
}

// Silu lane (VectorMath.cs:118-135): vector lanes use ExpApprox, the n%8 tail MathF.Exp
__device__ __forceinline__ float silu_ref(float x, bool vec_lane)
{
    float e = vec_lane ? exp_approx(-x) : expf(-x);
    return __fdiv_rn(x, __fadd_rn(1.0f, e));
}

// Gelu lane (VectorMath.cs:168-194)
__device__ __forceinline__ float gelu_ref(float x, bool vec_lane)
{
    if (vec_lane) {
        float inner = __fmul_rn(__fmul_rn(x, 0.7978845608028654f),
                                __fadd_rn(1.0f, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x)));
        return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanh_approx(inner)));
    }
    float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(x, __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

// Softcap lane (VectorMath.cs:286-302, and the softcap prologue of Softmax :222-235)
__device__ __forceinline__ float softcap_ref(float v, float cap, float inv_cap, bool vec_lane)
{
    if (vec_lane) return __fmul_rn(cap, tanh_approx(__fmul_rn(v, inv_cap)));
    return __fmul_rn(cap, tanhf(__fdiv_rn(v, cap)));
}

// DequantizeK.Extract6Bit (DequantizeK.cs:189-199)
__device__ __forceinline__ int extract6(const uint8_t *base, int bit)
{
    int bi = bit >> 3, sh = bit & 7;
    if (sh <= 2) return (base[bi] >> sh) & 0x3F;
    return ((base[bi] >> sh) | (base[bi + 1] << (8 - sh))) & 0x3F;
}

// Order-preserving float <-> uint key for max-reductions (larger float -> larger key).
__device__ __forceinline__ uint32_t float_key(float f)
{
    uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k)
{
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// VectorMath.ArgMax (src/Llmdot.Core/Tensors/Numeric/VectorMath.cs:412-425) as a max-reduction of
// packed keys (value key << 32 | (0xFFFFFFFF - index)), so that among equal value keys the lowest
// index wins.  The reference starts from element 0 and moves only on a strict `>`, hence:
//   * a NaN never replaces the running maximum: NaN gets the lowest value key (0, below -Inf);
//   * a NaN at index 0 is never replaced by anything: there it gets the highest key (0xFFFFFFFF,
//     above +Inf);
//   * -0 and +0 compare equal: -0 is keyed as +0, so the earlier of the two stays.
// gidx is the index in the whole row (the vocabulary index under tensor parallelism).
__device__ __forceinline__ unsigned long long argmax_key(float f, uint32_t gidx)
{
    uint32_t b = __float_as_uint(f), vk;
    if ((b & 0x7FFFFFFFu) > 0x7F800000u) {
        vk = gidx == 0 ? 0xFFFFFFFFu : 0u;
    } else {
        if (b == 0x80000000u) b = 0u;
        vk = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    }
    return ((unsigned long long)vk << 32) | (unsigned long long)(0xFFFFFFFFu - gidx);
}
__device__ __forceinline__ int32_t argmax_key_index(unsigned long long k)
{
    return (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
}

// Programmatic dependent launch.  A kernel launched with the programmatic-serialization
// attribute may start while its predecessor in the stream is still running; it must call
// pdl_wait() before it reads anything the predecessor writes and before it writes any
// global memory.  Before the wait it may only read data no in-flight kernel writes (weights,
// tables, KV entries of earlier steps).  pdl_launch() lets the successor start early.  Both
// are no-ops for kernels launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace llmdot
