// sample.cuh -- Sampler.Sample on the device (see sample.cu).
#pragma once
#include "common.cuh"

namespace llmdot {

constexpr int SAMPLE_MAX_TOP_K = 1024;   // top-k candidates sorted in shared memory
constexpr int SAMPLE_MAX_WINDOW = 1024;  // repeat-penalty history tokens

struct SampleArgs {
    const float *logits;  // [rows][ld], raw (before the final softcap)
    int ld, n;            // row stride, vocabulary
    int has_cap;          // Gemma's final-logit softcap, applied first
    float cap, inv_cap;
    float temperature, inv_temp;  // inv_temp = 1 / temperature as the reference computes it (float)
    int top_k;
    float penalty;
    int window;
    const int32_t *recent;      // [rows][recent_ld] history (device), oldest first; may be null
    const int32_t *recent_len;  // [rows] entries of each history (device)
    int recent_ld;
    const float *r;  // [rows] uniform draws (device)
    int32_t *out;    // [rows] sampled ids (device); -2 when the full-row path met a tie group above its limit
    int32_t *next;   // optional second copy of the ids (the next step's input tokens)
    float top_p;     // the nucleus mass (full-row path, top_p < 1)
    void *work;      // device scratch of the full-row path: sample_work_bytes(n) bytes
};

// Scratch of the full-row path (top_k <= 0 or top_k >= n), carved from SampleArgs::work.
struct SampleWork {
    float *p, *val;         // [n] probabilities in token order; nucleus values in sorted order
    uint32_t *kin, *kout;   // [n] sort keys (probabilities), before and after the sort
    int32_t *iin, *iout;    // [n] token ids with the keys
    int32_t *pos, *at;      // [n] selection-sort replay: position of each token, token at each position
    void *cub;              // radix-sort scratch
    size_t cub_bytes;
};

// Sampler.cs:42-61 runs the whole row (softmax, then top-p) when top_k <= 0 or top_k >= n.
inline bool sample_full_row(float temperature, int top_k, int n) { return temperature > 0.0f && (top_k <= 0 || top_k >= n); }

int launch_sample(const SampleArgs &a, int rows, cudaStream_t st);
size_t sample_smem(int n, int window, int top_k);
size_t sample_work_bytes(int n);  // device bytes of SampleArgs::work for a vocabulary of n

}  // namespace llmdot
