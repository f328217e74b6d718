// noalloc.cu -- greedy argmax over device-resident logits that allocates no device memory.
//
// Who needs it: a host that owns all device memory itself -- for example one that reserves
// the weights, the KV pages and its logits buffers from its own pool at start-up and runs the
// token loop under a fixed memory budget.  For such a caller a cudaMalloc inside a library
// call can fail when the pool has taken the memory, and it can also stall the device while
// other streams are busy.  This entry point therefore keeps its only scratch (one 64-bit key
// per row) in a fixed array compiled into the library and takes every other buffer from the
// caller.
//
// The array's name is only a host-side stand-in in host code, so the host looks up its real
// device address once per device with cudaGetSymbolAddress (with that device current) and
// passes the address to the kernels.  That first call also loads the library's device code
// (CUDA loads modules lazily), which may make the driver take device memory: hosts make one
// warm-up call per device before they reserve their pools.  The cached address belongs to the
// device's primary context; a cudaDeviceReset invalidates it.
#include <mutex>

#include "common.cuh"

namespace llmdot {

// One key per row: (orderable float << 32) | (0xFFFFFFFF - index).  Every GPU that loads the
// library holds these 32 KiB until the process exits.
static __device__ __align__(256) unsigned long long g_argmax_keys[LLMDOT_ARGMAX_NOALLOC_MAX_ROWS];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_keys_mu;
void *g_keys_addr[kMaxDevices] = {};  // device address of g_argmax_keys, per device
}  // namespace

__global__ void argmax_noalloc_kernel(const float *__restrict__ x, int ld, int n, unsigned long long *__restrict__ keys)
{
    const int row = blockIdx.y;
    const float *xr = x + (uint64_t)row * ld;
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const unsigned long long k = argmax_key(xr[i], (uint32_t)i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) atomicMax(keys + row, best);
}

__global__ void argmax_noalloc_finish_kernel(const unsigned long long *__restrict__ keys, int rows,
                                             int32_t *__restrict__ out)
{
    int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < rows) out[r] = (int32_t)(0xFFFFFFFFu - (uint32_t)(keys[r] & 0xFFFFFFFFull));
}

}  // namespace llmdot

using namespace llmdot;

extern "C" int llmdot_cuda_argmax_noalloc(const float *d_logits, int n, int rows, int ld, int32_t *d_index,
                                          void *stream)
{
    if (!d_logits || !d_index) return fail(LLMDOT_E_INVALID, "argmax_noalloc: null device pointer");
    if (n <= 0 || rows <= 0 || ld < n) return fail(LLMDOT_E_INVALID, "argmax_noalloc: need n > 0, rows > 0, ld >= n");
    if (rows > LLMDOT_ARGMAX_NOALLOC_MAX_ROWS)
        return fail(LLMDOT_E_INVALID, "argmax_noalloc: rows=" + std::to_string(rows) + " exceeds the fixed scratch of " +
                                          std::to_string(LLMDOT_ARGMAX_NOALLOC_MAX_ROWS) + " rows");
    int dev = 0;
    LLMDOT_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(LLMDOT_E_INVALID, "argmax_noalloc: device index above 63");
    void *keys = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_keys_mu);
        if (!g_keys_addr[dev]) {
            // one-time set-up for this device (the caller's current device)
            cudaError_t e = cudaGetSymbolAddress(&g_keys_addr[dev], g_argmax_keys);
            if (e != cudaSuccess) {
                g_keys_addr[dev] = nullptr;
                return cuda_fail(e, "argmax_noalloc: cudaGetSymbolAddress");
            }
        }
        keys = g_keys_addr[dev];
    }
    cudaStream_t st = (cudaStream_t)stream;
    // the array keeps the previous call's keys: clear this call's rows first
    LLMDOT_CUDA_TRY(cudaMemsetAsync(keys, 0, sizeof(unsigned long long) * (size_t)rows, st));
    int blocks = (n + 1023) / 1024;
    if (blocks > 148) blocks = 148;
    argmax_noalloc_kernel<<<dim3(blocks, rows), 256, 0, st>>>(d_logits, ld, n, (unsigned long long *)keys);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    argmax_noalloc_finish_kernel<<<(rows + 255) / 256, 256, 0, st>>>((const unsigned long long *)keys, rows, d_index);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}
