// gemv.cuh -- tensor-core quantised matvec over 16-row tiled weights.
#pragma once
#include "engine.cuh"

namespace llmdot {
// Allocate and fill W.tiled (the tensor-core layout) when the type has a fast kernel.
int prepare_tiled(llmdot_model *m, DevMat &W);
bool gemv_fast_supported(const DevMat &W, int nv);
int launch_gemv_fast(const DevMat &W, const float *x, int ldx, int nv, float *y, int ldy, bool accumulate,
                     cudaStream_t st);
}  // namespace llmdot
