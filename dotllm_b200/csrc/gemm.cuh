// gemm.cuh -- quantised matmul for 5..32 input rows (batched decode steps, prompt chunks).
#pragma once
#include <vector>

#include "common.cuh"

struct llmdot_model;

namespace llmdot {

struct DevMat;

constexpr int GEMM_MIN_ROWS = 5;   // below this the matvec kernel (gemv.cu), where its input fits
constexpr int GEMM_MAX_ROWS = 32;

// Activation fragments of one input, built once and shared by every matrix that reads it.
struct GemmInput {
    const void *xf = nullptr;   // fp16 hi/lo B operands, per super-block
    const void *sf = nullptr;   // Q4_K offset-correction B operands (Q4_K layout only)
    const float *isc = nullptr; // per row: 1 / (power-of-two scale)
    int nv = 0, nsb = 0, layout = 0;
};

// Device scratch of the batched path, sized for `cols_max` inputs and `rows_max` outputs.
struct GemmScratch {
    void *xf[2] = {nullptr, nullptr};
    void *sf = nullptr;
    float *isc[2] = {nullptr, nullptr};
    float *part = nullptr;
    int cols_max = 0, rows_max = 0;
    size_t part_floats = 0;
};

int gemm_scratch_alloc(GemmScratch &s, int cols_max, int rows_max, std::vector<void *> &allocs);

// True when W has the tile layout the batched kernel reads (Q4_K / Q6_K, cols % 256 == 0).
bool gemm_supported(const DevMat &W, int nv);

// Builds the fragments of x ([nv][ldx], optional fused RMSNorm with norm_w) for the tile layout
// of `qtype` (Q4_K or Q6_K) into scratch slot `slot` (0 or 1).
int gemm_prepare(const float *x, int ldx, int nv, int cols, const float *norm_w, float eps, uint32_t qtype, int slot,
                 GemmScratch &s, GemmInput *out, cudaStream_t st);

// y[v][row] (=, +=) W . x_v for the nv rows of `in`; mode GEMV_STORE or GEMV_ADD.
int launch_gemm(const DevMat &W, const GemmInput &in, float *y, int ldy, int mode, GemmScratch &s, int *err,
                cudaStream_t st);

}  // namespace llmdot
