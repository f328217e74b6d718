// step.cuh -- the greedy decode step (and prompt prefill) as one persistent kernel launch.
#pragma once
#include "common.cuh"

struct llmdot_model;

namespace llmdot {

struct StepCache;
void step_cache_free(llmdot_model *m);

// True when every matrix of the model has the tensor-core tile layout, the batch is 1..3 and
// the whole step fits the persistent kernel's shared-memory plan on this device.
bool step_kernel_supported(llmdot_model *m, int batch);

// Runs n_steps steps of ProcessToken for the workspace's `batch` rows in ONE cooperative
// launch on stream st.  Device state in the workspace: next[b] is the token fed to the first
// step, pos[b] its position, views[b] the session's KV pages.  Without `forced`, every step
// feeds the greedy argmax of the previous one (records it in hist, advances hist_step); with
// `forced` ([n_steps][batch] device token ids) the steps consume those tokens (prompt
// prefill) and only the last step computes logits.  On return next[b] holds the argmax of
// the last step, pos[b] has advanced by n_steps and ws.logits holds the last step's logits.
// trace (optional): [phase][cta][4] %globaltimer stamps of the first step (phase start, input
// built, tiles done, phase end).
int launch_step_kernel(llmdot_model *m, int batch, int kv_type, int n_steps, const int32_t *forced, cudaStream_t st,
                       unsigned long long *trace = nullptr);

// Phase count, CTA count and per-phase kind (1 scores, 2 P.V, 10 + epilogue mode for matvecs).
int step_kernel_shape(llmdot_model *m, int batch, int *n_phases, int *n_cta, int *kinds, int max_kinds);

// Clears the grid-barrier, attention and argmax state after a launch that reported an error.
int step_kernel_reset(llmdot_model *m, cudaStream_t st);

}  // namespace llmdot
