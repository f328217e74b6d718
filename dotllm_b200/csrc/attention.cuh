// attention.cuh -- paged KV cache views and the decode-attention launcher.
#pragma once
#include "common.cuh"

namespace llmdot {

// Positions per KV page.  A page of one KV head holds KV_PAGE consecutive positions,
// head_dim contiguous elements each, so one page is one contiguous run per head.
constexpr int KV_PAGE = 64;

// Device-side view of one session's cache (one entry per batch row).
struct KvView {
    void *k;              // base of the session's K pool, element type = kv_type
    void *v;              // base of the V pool
    const int32_t *pages; // logical page -> physical page
    int64_t layer_stride; // elements per layer = n_pages * heads_kv * KV_PAGE * head_dim
};

struct AttnShape {
    int heads, heads_kv, head_dim, max_ctx, sliding_window, has_cap;
    float cap, inv_sqrt_hd;
    int rope_half;
};

// One layer of decode attention for `batch` sessions: RoPE of q and of the new k, append of
// k and v at pos[b], softmax(q K^T / sqrt(hd), softcap) V over the window, written to
// out[b][h*hd + d].  q/k/v are the raw projections.  Scratch: scores [batch][heads][max_ctx],
// part_m/part_s [batch][heads][max_ctx/KV_PAGE], part_o [..][head_dim], counters
// [batch][heads_kv] (zero on entry, left zero).  append_first: append every row's k/v in a
// separate kernel before the attention, for rows of one session in one step (prompt chunks).
// LLMDOT_E_TIMEOUT (and the flag cleared) when a bounded wait of the attention kernel gave up.
int attention_timeout_check();

int launch_attention_step(const float *q, int ldq, const float *k, const float *v, int ldkv, const int32_t *pos,
                          const float *cos_t, const float *sin_t, const KvView *views, int layer, int kv_type,
                          const AttnShape &sh, int batch, float *scores, float *part_m, float *part_s, float *part_o,
                          int *counters, float *out, int ldo, bool append_first, bool pdl, cudaStream_t st);

}  // namespace llmdot
