// engine.cuh -- device-resident model, sessions and the decode step.
#pragma once
#include <map>
#include <string>
#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "gemm_tc.cuh"

namespace llmdot {

// One weight matrix on the device: `rows` output features of `cols` inputs, stored
// exactly as GGUF holds it (row-major, quantised blocks), plus an optional copy
// re-laid out in 16-row tiles for the tensor-core matvec (see gemv.cu).
struct DevMat {
    uint32_t type = 0;
    int rows = 0, cols = 0;
    uint64_t rbytes = 0;
    uint8_t *raw = nullptr;
    uint8_t *tiled = nullptr;
    uint8_t *tiled8 = nullptr;  // Q4_K only: the same tiles in the int8 tensor-core lane order
    bool valid() const { return raw != nullptr; }
    uint64_t bytes() const { return rbytes * (uint64_t)rows; }
};

struct LayerW {
    DevMat q, k, v, qkv, o, gate, up, down;
    float *attn_norm = nullptr, *ffn_norm = nullptr, *post_attn = nullptr, *post_ffw = nullptr;
};

// Step scratch, sized for `batch` rows.
struct Workspace {
    int batch = 0;
    int gen = 0;  // bumped whenever the buffers are reallocated (captured graphs and plans go stale)
    float *h = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *qkv = nullptr, *attn = nullptr;
    float *gate = nullptr, *up = nullptr, *logits = nullptr;
    float *scores = nullptr, *part_m = nullptr, *part_s = nullptr, *part_o = nullptr;
    unsigned long long *keys = nullptr;
    int32_t *tokens = nullptr, *pos = nullptr, *next = nullptr;
    KvView *views = nullptr;
    int *err = nullptr;
    int *counters = nullptr;   // [batch][heads_kv] attention page-combine arrival counters
    int32_t *hist = nullptr;   // [HIST_STEPS][batch] greedy ids recorded by captured steps
    int32_t *hist_step = nullptr;
    TcScratch tc;  // tensor-core matmul (2..32 rows): prepared operands and K-split partials
    std::vector<void *> allocs;
};
constexpr int HIST_STEPS = 4096;

// Per-launch device timing of one forward step (the measurement hook llmdot_cuda_profile_step):
// while a StepTimer is attached to the model, forward_step brackets each launch (or the launches
// of one operation) with CUDA events on its stream and files the span under a kernel family.
enum { FAM_MATVEC = 0, FAM_ATTENTION = 1, FAM_OTHER = 2, FAM_COLLECTIVE = 3, FAM_COUNT = 4 };
struct StepTimer {
    std::vector<cudaEvent_t> ev;  // pairs (start, end), reused across steps
    std::vector<int> fam;         // family of each recorded span
    int n = 0;                    // spans recorded in the current step
    int begin(cudaStream_t st, int family);
    int end(cudaStream_t st);
    void destroy();
};

}  // namespace llmdot

struct llmdot_session;
struct llmdot_model {
    int device = 0;
    std::vector<llmdot_session *> sessions;  // live sessions, detached when the model is freed
    llmdot_config cfg{};
    cudaStream_t stream = nullptr;
    std::vector<llmdot::LayerW> layers;
    llmdot::DevMat emb, out;
    float *out_norm = nullptr;
    float *cos_t = nullptr, *sin_t = nullptr;
    int rope_half = 0;
    int max_ctx = 0;  // context rounded up to whole KV pages
    uint64_t layer_bytes = 0, head_bytes = 0;
    std::vector<void *> allocs;
    std::map<std::string, llmdot::DevMat *> by_name;
    llmdot::Workspace ws;
    bool use_fast_gemv = true;
    bool use_pdl = true;
    // tensor parallelism: cfg above holds THIS rank's local heads / kv heads / FFN rows; full_cfg
    // the model's; the logits head (m->out) holds vocabulary rows [head_lo, head_lo + head_rows)
    int tp = 1, tp_rank = 0, head_lo = 0, head_rows = 0;
    llmdot_config full_cfg{};
    void *nccl = nullptr;  // ncclComm_t once llmdot_cuda_tp_init ran
    // peer-memory all-reduce (tp.cu): this rank's exchange buffer, every rank's mapped into this
    // process (own included), floats per slot row, and whether the step uses it
    uint8_t *tpx = nullptr;
    uint8_t *tpx_peer[8] = {};
    size_t tpx_cap = 0;
    bool tpx_open = false, tpx_use = false;
    llmdot::StepTimer *timer = nullptr;  // attached only while llmdot_cuda_profile_step runs
};

struct llmdot_session {
    llmdot_model *m = nullptr;  // null once the model was freed (the session then only accepts free)
    int device = 0;
    int max_ctx = 0, kv_type = 0, n_pages = 0, pos = 0;
    void *k = nullptr, *v = nullptr;
    int32_t *pages = nullptr;
    llmdot::KvView view{};
};

namespace llmdot {
int model_upload(int device, const llmdot_config *cfg, const llmdot_tensor_desc *t, int n, llmdot_model **out,
                 int tp = 1, int tp_rank = 0);
void model_destroy(llmdot_model *m);
int ensure_workspace(llmdot_model *m, int batch);
// One forward step (ProcessToken) for `batch` rows: token ids, positions and KV views are
// device arrays of `batch` entries.  Raw logits land in ws.logits, greedy ids in next.
// tokens may alias next (the step reads its tokens before it writes the argmax).
// flags: STEP_CHUNK = the rows are consecutive positions of one session (a prompt chunk): K/V
// of every row are appended before attention; STEP_NO_HEAD = skip final norm, logits, argmax.
enum { STEP_CHUNK = 1, STEP_NO_HEAD = 2 };
int forward_step(llmdot_model *m, int batch, int kv_type, const int32_t *tokens, const int32_t *pos,
                 const KvView *views, int32_t *next, cudaStream_t st, int flags = 0);
int gemv(const DevMat &W, const float *x, int ldx, int nv, float *y, int ldy, bool accumulate, bool fast,
         cudaStream_t st);
}  // namespace llmdot
