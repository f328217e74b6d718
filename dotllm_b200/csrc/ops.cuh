// ops.cuh -- launchers of the element-wise, reduction and generic matvec kernels.
#pragma once
#include "common.cuh"

namespace llmdot {

enum { OP_ADD = 0, OP_MUL, OP_SCALE, OP_SILU, OP_GELU, OP_SOFTCAP, OP_SILU_MUL, OP_GELU_MUL };

int launch_dequant(const uint8_t *src, float *dst, uint32_t type, int rows, int row_elems, cudaStream_t st);
int launch_gemv_ref(const uint8_t *W, uint32_t type, int rows, int cols, const float *x, int ldx, int nv, float *y,
                    int ldy, bool accumulate, cudaStream_t st);
int launch_rmsnorm(const float *in, int ldin, const float *w, float *out, int ldout, int n, int nv, float eps,
                   cudaStream_t st, bool pdl = false);
int launch_layernorm(const float *x, const float *w, const float *b, float *o, int n, float eps, cudaStream_t st);
int launch_eltwise(int op, const float *a, const float *b, float *o, int n, float s, cudaStream_t st, int row = 0);
int launch_act_mul(bool gelu, const float *gate, const float *up, float *out, int ffn, int batch, cudaStream_t st);
int launch_gelu_scalar(float x, float *o, cudaStream_t st);
int launch_rope(float *x, int nheads, int head_dim, const float *cs, const float *sn, int half, cudaStream_t st);
int launch_softmax(float *x, int n, bool has_cap, float cap, cudaStream_t st);
int launch_argmax(const float *x, int ldx, int n, int nv, unsigned long long *keys, int32_t *out, bool has_cap,
                  float cap, float *capped, cudaStream_t st);
// The two halves of launch_argmax, for a vocabulary shard [off, off + n) of ntot entries (keys
// reduced across ranks in between).
int launch_argmax_keys(const float *x, int ldx, int n, int nv, unsigned long long *keys, bool has_cap, float cap,
                       float *capped, int off, int ntot, cudaStream_t st);
int launch_argmax_finish(const unsigned long long *keys, int nv, int32_t *out, cudaStream_t st);
int launch_conv1d(const float *in, const float *w, float *o, int ks, int dim, cudaStream_t st);
int launch_embed(const uint8_t *emb, uint32_t type, int hidden, int vocab, const int32_t *tokens, int nv, float scale,
                 float *h, int ldh, int *err, cudaStream_t st);

}  // namespace llmdot
