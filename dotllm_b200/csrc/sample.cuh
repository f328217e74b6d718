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
    int32_t *out;    // [rows] sampled ids (device)
    int32_t *next;   // optional second copy of the ids (the next step's input tokens)
};

int launch_sample(const SampleArgs &a, int rows, cudaStream_t st);
size_t sample_smem(int n, int window, int top_k);

}  // namespace llmdot
