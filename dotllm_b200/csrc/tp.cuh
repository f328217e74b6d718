// tp.cuh -- tensor parallelism: shard geometry and the NCCL collectives of the decode step.
#pragma once
#include "common.cuh"

struct llmdot_model;
struct llmdot_config;

namespace llmdot {

// What rank `rank` of `tp` holds (Megatron-style split):
//   q rows [q_lo, q_lo+q_n)            (its heads / tp query heads)
//   k, v rows [kv_lo, kv_lo+kv_n)      (its heads_kv / tp kv heads)
//   attn_output columns [q_lo, q_lo+q_n)
//   gate, up rows / down columns [f_lo, f_lo+f_n)
//   logits rows [v_lo, v_lo+v_n)       (vocabulary shard; the embedding stays whole)
struct TpShard {
    int q_lo, q_n, kv_lo, kv_n, f_lo, f_n, v_lo, v_n;
};

// Fills `s`; fails when the model does not split evenly into `tp` ranks (heads, kv heads and FFN
// rows divisible by tp, and the column splits on whole 256-weight super-blocks).
int tp_shard(const llmdot_config &c, int tp, int rank, TpShard *s);

// NCCL is loaded at run time (libnccl.so.2) the first time tensor parallelism is used, so the
// library has no link-time NCCL dependency and shares the process's NCCL when torch loaded one.
int tp_unique_id(void *out128);
int tp_comm_init(llmdot_model *m, const void *id128);
void tp_comm_destroy(llmdot_model *m);
// In-place sum of `n` floats across the ranks, on stream st.
int tp_allreduce_sum(llmdot_model *m, float *buf, size_t n, cudaStream_t st);
// In-place max of `n` packed (value key, index) argmax keys across the ranks.
int tp_allreduce_max_u64(llmdot_model *m, unsigned long long *buf, size_t n, cudaStream_t st);
// All-gather of `n` floats per rank: recv holds rank r's block at r*n.
int tp_allgather(llmdot_model *m, const float *send, float *recv, size_t n, cudaStream_t st);

// Peer-memory one-shot all-reduce: each rank's exchange buffer (a sequence counter and two receive
// slots) is exported with CUDA IPC; once every rank opened every handle, tp_allreduce_sum runs as
// one kernel that pushes this rank's partial into every peer's slot and sums the ranks' values in
// rank order (the same order on every rank, so every rank ends with identical values);
// tp_allreduce_max_u64 runs over the same buffers.
constexpr int TPX_HANDLE_BYTES = 128;  // cudaIpcMemHandle_t (64) + device UUID (16), zero padded
constexpr int TPX_MAX_RANKS = 8;
int tp_exchange_handle(llmdot_model *m, void *out128);
int tp_exchange_open(llmdot_model *m, const void *handles);  // tp x TPX_HANDLE_BYTES, rank order
int tp_exchange_use(llmdot_model *m, bool on);  // whether the step's sums use it (after open)
void tp_exchange_close(llmdot_model *m);

}  // namespace llmdot
