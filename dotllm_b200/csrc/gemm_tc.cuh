// gemm_tc.cuh -- quantised matmul for 2..32 input rows on the tcgen05 tensor cores (TMEM
// accumulators), for batched decode steps and prompt chunks.
#pragma once
#include <vector>

#include "common.cuh"

namespace llmdot {

struct DevMat;
struct GemvPrefetch;

constexpr int TC_MIN_ROWS = 5;   // below this the matvec kernel (gemv.cu), where its input fits
constexpr int TC_MAX_ROWS = 32;  // input rows per launch (MMA N = 2 x 32: the hi and lo fp16 halves)

// Device scratch of the tensor-core matmul: the prepared B operands of one input (both weight
// layouts), per-row scales, K-split partial outputs and their arrival counters.
struct TcScratch {
    uint8_t *b4 = nullptr;  // Q4_K operand layout, 34 KB per super-block (two K halves + offset-term sums)
    uint8_t *b6 = nullptr;  // Q6_K operand layout, 32 KB per super-block
    float *isc = nullptr;   // [TC_MAX_ROWS] 1 / (power-of-two scale of the row)
    float *part = nullptr;  // [grid][2][TC_MAX_ROWS][128] partial row tiles
    int *cnt = nullptr;     // [tiles_max] arrivals per 128-row tile (left at zero)
    size_t b4s = 0, b6s = 0;  // bytes of one replica of each layout
    int reps = 1;             // replicas of the prepared operands (CTA c reads replica c % reps)
    int cols_max = 0, grid_max = 0, tiles_max = 0;
    bool ready() const { return b4 != nullptr; }
};

// One output of a launch: y[v][row] (=, +=) W[row] . x_v.  Segments of one launch share the input.
struct TcSeg {
    const DevMat *W;
    float *y;
    int ldy;
};

int tc_scratch_alloc(TcScratch &s, int cols_max, int tiles_max, std::vector<void *> &allocs);

// True when W has the 16-row tile layout the kernel reads (Q4_K / Q6_K, cols % 256 == 0).
bool tc_supported(const DevMat &W);

// Builds the B operands of x ([nv][ldx], optional fused RMSNorm with norm_w) for the layouts
// the following launches read (q4: Q4_K matrices, q6: Q6_K matrices).
int tc_prepare(const float *x, int ldx, int nv, int cols, const float *norm_w, float eps, bool q4, bool q6,
               TcScratch &s, cudaStream_t st);

// y = W . x for the prepared input, for 1..3 segments of the same input width; mode GEMV_STORE or
// GEMV_ADD (residual add).  err: device flag set to 5 when a bounded wait gave up.  pf (nullable):
// weights of the next operation, prefetched into L2 while this one runs.
int tc_gemm(const TcSeg *seg, int nseg, int nv, int mode, TcScratch &s, int *err, cudaStream_t st,
            const GemvPrefetch *pf = nullptr);

}  // namespace llmdot
