// gemv.cu -- tensor-core quantised matvec (placeholder until the tiled kernel lands).
#include "gemv.cuh"

namespace llmdot {
int prepare_tiled(llmdot_model *, DevMat &) { return LLMDOT_OK; }
bool gemv_fast_supported(const DevMat &, int) { return false; }
int launch_gemv_fast(const DevMat &, const float *, int, int, float *, int, bool, cudaStream_t)
{
    return fail(LLMDOT_E_UNSUPPORTED, "fast matvec not built");
}
}  // namespace llmdot
