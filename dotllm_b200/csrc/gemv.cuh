// gemv.cuh -- tensor-core quantised matvec over 16-row tiled weights (see gemv.cu).
#pragma once
#include "engine.cuh"

namespace llmdot {
// Epilogues of the fast matvec
enum { GEMV_STORE = 0, GEMV_ADD = 1, GEMV_SILU_MUL = 2, GEMV_GELU_MUL = 3 };

// One output of a multi-matrix launch: y[v][row] (ldy) = epilogue(W . x[v]); W1 is the "up"
// matrix of the GEMV_*_MUL epilogues.
struct GemvTarget {
    const DevMat *W;
    const DevMat *W1;
    float *y;
    int ldy;
};

// Up to GEMV_PREFETCH_MAX byte ranges (16-byte aligned, multiples of 16 bytes) that a matvec
// launch pulls into L2 for the operation after it.
constexpr int GEMV_PREFETCH_MAX = 3;
struct GemvPrefetch {
    const void *p[GEMV_PREFETCH_MAX];
    unsigned long long n[GEMV_PREFETCH_MAX];
};

// Q4_K matrices with at least this many rows (the logits heads) also get the int8-order tile
// copy that the 1..2-vector matvec streams with int8 MMAs; on smaller matrices the per-CTA input
// conversion it needs costs more than its tile math saves.
constexpr int GEMV_I8_MIN_ROWS = 16384;

// Allocate and fill W.tiled (the tensor-core layout) for Q4_K / Q6_K matrices.
int prepare_tiled(llmdot_model *m, DevMat &W);
// LLMDOT_E_TIMEOUT (and the flag cleared) when a bounded wait of the matvec kernel gave up.
int gemv_timeout_check();
bool gemv_fast_supported(const DevMat &W, int nv);
int launch_gemv_fast(const DevMat &W, const float *x, int ldx, int nv, float *y, int ldy, bool accumulate,
                     cudaStream_t st);
// y = epilogue(W0 . rmsnorm(x)); norm_w == null means no fused norm.
int launch_gemv_fast_ex(const DevMat &W0, const DevMat *W1, const float *norm_w, float eps, const float *x, int ldx,
                        int nv, float *y, int ldy, int mode, cudaStream_t st, bool pdl = false,
                        const GemvPrefetch *pf = nullptr);
// Up to three matrices with the same input (e.g. Q, K, V) in one launch.
int launch_gemv_multi(const GemvTarget *tg, int ntarget, const float *norm_w, float eps, const float *x, int ldx,
                      int nv, int mode, bool pdl, cudaStream_t st, const GemvPrefetch *pf = nullptr);
}  // namespace llmdot
