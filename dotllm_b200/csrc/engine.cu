// engine.cu -- model upload, sessions, and the decode step (the device-resident
// counterpart of InferenceEngine.ProcessToken, src/Llmdot.Core/Inference/InferenceEngine.cs:134-602).
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <strings.h>

#include <algorithm>

#include "engine.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"
#include "gemv_tile.cuh"
#include "ops.cuh"
#include "tp.cuh"

namespace llmdot {

static int dmalloc(std::vector<void *> &allocs, void **p, size_t bytes)
{
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(LLMDOT_E_NOMEM, std::string("cudaMalloc(") + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    }
    allocs.push_back(*p);
    return LLMDOT_OK;
}

template <typename T> static int dalloc(std::vector<void *> &a, T **p, size_t n)
{
    return dmalloc(a, (void **)p, n * sizeof(T));
}

// LoadedModel.LoadTensors keys tensors OrdinalIgnoreCase and a later tensor of the same name
// replaces an earlier one (LoadedModel.cs:77-107): the last match wins
static const llmdot_tensor_desc *find_desc(const llmdot_tensor_desc *t, int n, const std::string &name)
{
    for (int i = n - 1; i >= 0; i--)
        if (t[i].name && strcasecmp(t[i].name, name.c_str()) == 0) return &t[i];
    return nullptr;
}

// A run of `n` consecutive rows of a weight starting at row `lo`.
struct RowRange {
    int lo, n;
};

// Uploads the rows `ranges` (concatenated, in order) and the columns [col_lo, col_lo + col_n) of a
// weight (col_n <= 0: all columns).  Without tensor parallelism that is the whole matrix.
static int upload_mat(llmdot_model *m, const llmdot_tensor_desc *d, DevMat &out, int expect_cols, int expect_rows,
                      std::vector<RowRange> ranges = {}, int col_lo = 0, int col_n = 0)
{
    if (!d) return LLMDOT_OK;
    m->by_name[d->name] = &out;
    if (d->n_dims < 2) return fail(LLMDOT_E_FORMAT, std::string(d->name) + ": expected a 2-D weight");
    out.type = d->type;
    const int full_cols = (int)d->dims[0], full_rows = (int)d->dims[1];
    if (block_elems(out.type) == 0 || out.type == T_F16 || out.type == T_BF16)
        return fail(LLMDOT_E_UNSUPPORTED, std::string(d->name) + ": weight type " + std::to_string(out.type) +
                                              " is not supported by the device matvec");
    if ((expect_cols > 0 && full_cols != expect_cols) || (expect_rows > 0 && full_rows != expect_rows))
        return fail(LLMDOT_E_FORMAT, std::string(d->name) + ": unexpected shape " + std::to_string(full_cols) + "x" +
                                         std::to_string(full_rows));
    const int be = (int)block_elems(out.type);
    if (full_cols % be != 0) return fail(LLMDOT_E_FORMAT, std::string(d->name) + ": columns not a multiple of the block size");
    if (ranges.empty()) ranges.push_back({0, full_rows});
    if (col_n <= 0) {
        col_lo = 0;
        col_n = full_cols;
    }
    if (col_lo % be || col_n % be || col_lo + col_n > full_cols)
        return fail(LLMDOT_E_UNSUPPORTED, std::string(d->name) + ": column shard not on block boundaries");
    out.cols = col_n;
    out.rows = 0;
    for (const RowRange &r : ranges) {
        if (r.lo < 0 || r.n < 0 || r.lo + r.n > full_rows) return fail(LLMDOT_E_INVALID, "row shard out of range");
        out.rows += r.n;
    }
    const uint64_t full_rb = row_bytes(out.type, (uint64_t)full_cols), col_off = row_bytes(out.type, (uint64_t)col_lo);
    out.rbytes = row_bytes(out.type, (uint64_t)out.cols);
    const uint64_t nb = out.rbytes * (uint64_t)out.rows;
    if (!d->data || d->n_bytes < full_rb * (uint64_t)full_rows)
        return fail(LLMDOT_E_FORMAT, std::string(d->name) + ": data too short");
    // 256 zeroed bytes of slack: the Q3_K decoder reads one byte past each block
    LLMDOT_TRY(dmalloc(m->allocs, (void **)&out.raw, nb + 256));
    LLMDOT_CUDA_TRY(cudaMemsetAsync(out.raw + nb, 0, 256, m->stream));
    uint64_t dst_row = 0;
    for (const RowRange &r : ranges) {
        if (r.n == 0) continue;
        const uint8_t *src = (const uint8_t *)d->data + (uint64_t)r.lo * full_rb + col_off;
        if (out.rbytes == full_rb)
            LLMDOT_CUDA_TRY(cudaMemcpyAsync(out.raw + dst_row * out.rbytes, src, out.rbytes * r.n,
                                            cudaMemcpyHostToDevice, m->stream));
        else
            LLMDOT_CUDA_TRY(cudaMemcpy2DAsync(out.raw + dst_row * out.rbytes, out.rbytes, src, full_rb, out.rbytes, r.n,
                                              cudaMemcpyHostToDevice, m->stream));
        dst_row += r.n;
    }
    LLMDOT_TRY(prepare_tiled(m, out));
    return LLMDOT_OK;
}

// LoadedModel.GetDequantizedWeights (LoadedModel.cs:63-75) for norm vectors.
static int upload_vec(llmdot_model *m, const llmdot_tensor_desc *d, float **out, int n)
{
    if (!d) return LLMDOT_OK;
    uint64_t elems = 1;
    for (uint32_t i = 0; i < d->n_dims; i++) elems *= d->dims[i];
    if ((int)elems != n) return fail(LLMDOT_E_FORMAT, std::string(d->name) + ": unexpected length");
    uint64_t nb = row_bytes(d->type, elems);
    if (nb == 0) return fail(LLMDOT_E_UNSUPPORTED, std::string(d->name) + ": unsupported type");
    if (!d->data || d->n_bytes < nb) return fail(LLMDOT_E_FORMAT, std::string(d->name) + ": data too short");
    LLMDOT_TRY(dalloc(m->allocs, out, (size_t)n));
    if (d->type == T_F32) {
        LLMDOT_CUDA_TRY(cudaMemcpyAsync(*out, d->data, nb, cudaMemcpyHostToDevice, m->stream));
        return LLMDOT_OK;
    }
    uint8_t *tmp = nullptr;
    LLMDOT_CUDA_TRY(cudaMalloc(&tmp, nb));
    cudaMemcpyAsync(tmp, d->data, nb, cudaMemcpyHostToDevice, m->stream);
    int rc = launch_dequant(tmp, *out, d->type, 1, n, m->stream);
    cudaStreamSynchronize(m->stream);
    cudaFree(tmp);
    return rc;
}

int model_upload(int device, const llmdot_config *cfg, const llmdot_tensor_desc *t, int n, llmdot_model **out, int tp,
                 int tp_rank)
{
    *out = nullptr;
    if (!cfg || !t || n <= 0) return fail(LLMDOT_E_INVALID, "model_load: null config or tensors");
    const llmdot_config &c = *cfg;
    const bool neox = c.template_id == 1;
    if (c.template_id != 0 && c.template_id != 1 && c.template_id != 2)
        return fail(LLMDOT_E_UNSUPPORTED,
                    "model_load: only the LlamaLike, GptNeoXLike and GemmaLike execution templates run on the device");
    if (c.expert_count > 0) return fail(LLMDOT_E_UNSUPPORTED, "model_load: MoE models are not supported on the device");
    if (!c.norm_is_rms && !neox)
        return fail(LLMDOT_E_UNSUPPORTED, "model_load: LayerNorm is supported on the device for the GptNeoXLike template only");
    if (neox && tp > 1) return fail(LLMDOT_E_UNSUPPORTED, "model_load: the GptNeoXLike template runs on one GPU");
    if (c.hidden <= 0 || c.layers <= 0 || c.heads <= 0 || c.heads_kv <= 0 || c.head_dim <= 0 || c.vocab <= 0 ||
        c.context <= 0 || c.heads % c.heads_kv != 0)
        return fail(LLMDOT_E_FORMAT, "model_load: invalid dimensions in config");
    if (c.ffn_type == 0 && !neox)
        return fail(LLMDOT_E_UNSUPPORTED, "model_load: the non-gated FFN is supported on the device for the GptNeoXLike template only");
    int rd = c.rope_dim > 0 ? c.rope_dim : c.head_dim;
    if (rd > c.head_dim || rd % 2) return fail(LLMDOT_E_FORMAT, "model_load: bad rope dimension");
    if (c.head_dim % 8 != 0) return fail(LLMDOT_E_UNSUPPORTED, "model_load: head_dim must be a multiple of 8");

    TpShard sh{};
    LLMDOT_TRY(tp_shard(c, tp, tp_rank, &sh));
    LLMDOT_CUDA_TRY(cudaSetDevice(device));
    llmdot_model *m = new llmdot_model();
    m->device = device;
    m->full_cfg = c;
    m->cfg = c;
    m->tp = tp;
    m->tp_rank = tp_rank;
    m->head_lo = sh.v_lo;
    m->head_rows = sh.v_n;
    if (tp > 1) {  // this rank's local shapes drive every kernel; the vocabulary stays global
        m->cfg.heads /= tp;
        m->cfg.heads_kv /= tp;
        m->cfg.ffn /= tp;
    }
    // LLMDOT_REFERENCE_MATVEC=1 selects the generic (per-element) matvec everywhere; the tests
    // use it to check the tensor-core path against the straightforward one.
    m->use_fast_gemv = getenv("LLMDOT_REFERENCE_MATVEC") == nullptr;
    // programmatic dependent launch between the step's kernels (LLMDOT_NO_PDL=1 turns it off)
    m->use_pdl = getenv("LLMDOT_NO_PDL") == nullptr;
    int rc = LLMDOT_OK;
    auto bail = [&](int code) { model_destroy(m); return code; };
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(LLMDOT_E_CUDA, "stream create failed"));

    const int qDim = c.heads * c.head_dim, kvDim = c.heads_kv * c.head_dim, H = c.hidden;
    const bool tps = tp > 1;
    auto D = [&](const std::string &s) { return find_desc(t, n, s); };
    const llmdot_tensor_desc *emb = D("token_embd.weight");
    if (!emb) return bail(fail(LLMDOT_E_FORMAT, "token_embd.weight missing"));
    if ((rc = upload_mat(m, emb, m->emb, H, c.vocab))) return bail(rc);
    // ComputeLogits (InferenceEngine.cs:583-602) looks the head up with TryGetTensor, whose keys
    // compare OrdinalIgnoreCase like every other lookup here
    const llmdot_tensor_desc *outw = D("output.weight");
    if (tps) {
        // the logits head holds this rank's vocabulary rows (tied models: a shard of the embedding,
        // which itself stays whole for the lookup)
        if ((rc = upload_mat(m, outw ? outw : emb, m->out, H, c.vocab, {{sh.v_lo, sh.v_n}}))) return bail(rc);
        m->by_name["output.weight"] = &m->out;
        m->by_name[emb->name] = &m->emb;
    } else if (outw && (rc = upload_mat(m, outw, m->out, H, c.vocab))) {
        return bail(rc);
    }
    const llmdot_tensor_desc *on = D("output_norm.weight");
    if (!on) on = D("token_embd_norm.weight");
    if (!on) return bail(fail(LLMDOT_E_FORMAT, "output_norm.weight missing"));
    if ((rc = upload_vec(m, on, &m->out_norm, H))) return bail(rc);

    m->layers.resize(c.layers);
    for (int l = 0; l < c.layers; l++) {
        LayerW &L = m->layers[l];
        std::string p = "blk." + std::to_string(l) + ".";
        if (D(p + "attn_q_norm.weight") || D(p + "attn_k_norm.weight"))
            return bail(fail(LLMDOT_E_UNSUPPORTED, "q/k norm tensors are not supported on the device"));
        if (!D(p + "attn_norm.weight")) return bail(fail(LLMDOT_E_FORMAT, p + "attn_norm.weight missing"));
        if ((rc = upload_vec(m, D(p + "attn_norm.weight"), &L.attn_norm, H))) return bail(rc);
        if ((rc = upload_vec(m, D(p + "ffn_norm.weight"), &L.ffn_norm, H))) return bail(rc);
        if (c.template_id == 2 && c.has_post_norm) {
            if ((rc = upload_vec(m, D(p + "post_attention_norm.weight"), &L.post_attn, H))) return bail(rc);
            if ((rc = upload_vec(m, D(p + "post_ffw_norm.weight"), &L.post_ffw, H))) return bail(rc);
        }
        // shards (tp > 1): q/k/v and gate/up by output rows, attn_output and ffn_down by input columns
        const std::vector<RowRange> all;
        const std::vector<RowRange> qr = tps ? std::vector<RowRange>{{sh.q_lo, sh.q_n}} : all;
        const std::vector<RowRange> kvr = tps ? std::vector<RowRange>{{sh.kv_lo, sh.kv_n}} : all;
        const std::vector<RowRange> fr = tps ? std::vector<RowRange>{{sh.f_lo, sh.f_n}} : all;
        if (neox) {
            // ProcessGptNeoXLikeLayer (InferenceEngine.cs:198-207) adds only the FFN result to the hidden
            // state: the attention result goes into a buffer the hidden state never reads.  So the
            // layer's output depends on the FFN weights alone; attention tensors are not uploaded.
            const bool gated = c.ffn_type != 0;
            if (!D(p + "ffn_up.weight") || !D(p + "ffn_down.weight") || (gated && !D(p + "ffn_gate.weight")))
                return bail(fail(LLMDOT_E_FORMAT, p + "FFN tensors missing"));
            if (gated && (rc = upload_mat(m, D(p + "ffn_gate.weight"), L.gate, H, c.ffn))) return bail(rc);
            if ((rc = upload_mat(m, D(p + "ffn_up.weight"), L.up, H, c.ffn))) return bail(rc);
            if ((rc = upload_mat(m, D(p + "ffn_down.weight"), L.down, c.ffn, H))) return bail(rc);
            for (const DevMat *w : {&L.gate, &L.up, &L.down})
                if (w->valid()) m->layer_bytes += w->bytes();
            m->layer_bytes += (uint64_t)H * 4;
            continue;
        }
        if (c.qkv_fused) {
            if (!D(p + "attn_qkv.weight")) return bail(fail(LLMDOT_E_FORMAT, p + "attn_qkv.weight missing"));
            const std::vector<RowRange> qkvr =
                tps ? std::vector<RowRange>{{sh.q_lo, sh.q_n}, {qDim + sh.kv_lo, sh.kv_n}, {qDim + kvDim + sh.kv_lo, sh.kv_n}}
                    : all;
            if ((rc = upload_mat(m, D(p + "attn_qkv.weight"), L.qkv, H, qDim + 2 * kvDim, qkvr))) return bail(rc);
        } else {
            if (!D(p + "attn_q.weight") || !D(p + "attn_k.weight") || !D(p + "attn_v.weight"))
                return bail(fail(LLMDOT_E_FORMAT, p + "attn_q/k/v missing"));
            if ((rc = upload_mat(m, D(p + "attn_q.weight"), L.q, H, qDim, qr))) return bail(rc);
            if ((rc = upload_mat(m, D(p + "attn_k.weight"), L.k, H, kvDim, kvr))) return bail(rc);
            if ((rc = upload_mat(m, D(p + "attn_v.weight"), L.v, H, kvDim, kvr))) return bail(rc);
        }
        if (!D(p + "attn_output.weight") || !D(p + "ffn_gate.weight") || !D(p + "ffn_up.weight") ||
            !D(p + "ffn_down.weight"))
            return bail(fail(LLMDOT_E_FORMAT, p + "attention output / FFN tensors missing"));
        if ((rc = upload_mat(m, D(p + "attn_output.weight"), L.o, qDim, H, all, tps ? sh.q_lo : 0, tps ? sh.q_n : 0)))
            return bail(rc);
        if ((rc = upload_mat(m, D(p + "ffn_gate.weight"), L.gate, H, c.ffn, fr))) return bail(rc);
        if ((rc = upload_mat(m, D(p + "ffn_up.weight"), L.up, H, c.ffn, fr))) return bail(rc);
        if ((rc = upload_mat(m, D(p + "ffn_down.weight"), L.down, c.ffn, H, all, tps ? sh.f_lo : 0, tps ? sh.f_n : 0)))
            return bail(rc);
        for (const DevMat *w : {&L.q, &L.k, &L.v, &L.qkv, &L.o, &L.gate, &L.up, &L.down})
            if (w->valid()) m->layer_bytes += w->bytes();
        m->layer_bytes += (uint64_t)H * 4 * (L.post_attn ? 4 : 2);
    }
    m->head_bytes = (m->out.valid() ? m->out.bytes() : m->emb.bytes()) + (uint64_t)H * 4;

    // RoPE tables: PrecomputeRopeFrequencies (InferenceEngine.cs:57-72), then
    // MathF.Cos/Sin of position*freq (TensorOps.cs:688-693), evaluated on the host
    // with the same C runtime functions the reference calls.
    m->rope_half = rd / 2;
    m->max_ctx = (c.context + KV_PAGE - 1) / KV_PAGE * KV_PAGE;
    {
        std::vector<float> freq(m->rope_half), cs((size_t)m->max_ctx * m->rope_half), sn(cs.size());
        for (int i = 0; i < m->rope_half; i++) {
            float f = 1.0f / powf(c.rope_base, 2.0f * (float)i / (float)rd);
            if (c.rope_scaling == 1 && c.rope_factor > 1.0f) f /= c.rope_factor;
            freq[i] = f;
        }
        for (int p = 0; p < m->max_ctx; p++)
            for (int i = 0; i < m->rope_half; i++) {
                float a = (float)p * freq[i];
                cs[(size_t)p * m->rope_half + i] = cosf(a);
                sn[(size_t)p * m->rope_half + i] = sinf(a);
            }
        if ((rc = dalloc(m->allocs, &m->cos_t, cs.size())) || (rc = dalloc(m->allocs, &m->sin_t, sn.size())))
            return bail(rc);
        cudaMemcpy(m->cos_t, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(m->sin_t, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    }
    if (cudaStreamSynchronize(m->stream) != cudaSuccess) return bail(cuda_fail(cudaGetLastError(), "model upload"));
    if ((rc = ensure_workspace(m, 1))) return bail(rc);
    *out = m;
    return LLMDOT_OK;
}

void model_destroy(llmdot_model *m)
{
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    tp_exchange_close(m);
    tp_comm_destroy(m);
    for (void *p : m->ws.allocs) cudaFree(p);
    for (void *p : m->allocs) cudaFree(p);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

int ensure_workspace(llmdot_model *m, int batch)
{
    Workspace &w = m->ws;
    if (w.batch >= batch) return LLMDOT_OK;
    cudaStreamSynchronize(m->stream);
    for (void *p : w.allocs) cudaFree(p);
    const int gen = w.gen + 1;
    w = Workspace();
    w.gen = gen;
    const llmdot_config &c = m->cfg;
    const size_t B = (size_t)batch, qDim = (size_t)c.heads * c.head_dim, kvDim = (size_t)c.heads_kv * c.head_dim;
    const size_t nchunk = (size_t)m->max_ctx / KV_PAGE;
    auto &a = w.allocs;
    LLMDOT_TRY(dalloc(a, &w.h, B * c.hidden));
    LLMDOT_TRY(dalloc(a, &w.xn, B * c.hidden));
    LLMDOT_TRY(dalloc(a, &w.q, B * qDim));
    LLMDOT_TRY(dalloc(a, &w.k, B * kvDim));
    LLMDOT_TRY(dalloc(a, &w.v, B * kvDim));
    LLMDOT_TRY(dalloc(a, &w.qkv, B * (qDim + 2 * kvDim)));
    LLMDOT_TRY(dalloc(a, &w.attn, B * qDim));
    LLMDOT_TRY(dalloc(a, &w.gate, B * c.ffn));
    LLMDOT_TRY(dalloc(a, &w.up, B * c.ffn));
    LLMDOT_TRY(dalloc(a, &w.logits, B * c.vocab));
    LLMDOT_TRY(dalloc(a, &w.scores, B * c.heads * (size_t)m->max_ctx));
    LLMDOT_TRY(dalloc(a, &w.part_m, B * c.heads * nchunk));
    LLMDOT_TRY(dalloc(a, &w.part_s, B * c.heads * nchunk));
    LLMDOT_TRY(dalloc(a, &w.part_o, B * c.heads * nchunk * c.head_dim));
    LLMDOT_TRY(dalloc(a, &w.keys, B));
    LLMDOT_TRY(dalloc(a, &w.tokens, B));
    LLMDOT_TRY(dalloc(a, &w.pos, B));
    LLMDOT_TRY(dalloc(a, &w.next, B));
    LLMDOT_TRY(dalloc(a, &w.views, B));
    LLMDOT_TRY(dalloc(a, &w.err, 1));
    LLMDOT_TRY(dalloc(a, &w.hist, (size_t)HIST_STEPS * B));
    LLMDOT_TRY(dalloc(a, &w.hist_step, 1));
    LLMDOT_TRY(dalloc(a, &w.counters, B * c.heads_kv));
    LLMDOT_CUDA_TRY(cudaMemset(w.counters, 0, sizeof(int) * B * c.heads_kv));
    LLMDOT_CUDA_TRY(cudaMemset(w.err, 0, sizeof(int)));
    LLMDOT_CUDA_TRY(cudaMemset(w.hist_step, 0, sizeof(int32_t)));
    if (batch >= 2) {  // the batched kernel also takes 2..4 rows whose input does not fit the matvec's smem
        const int cols_max = std::max(std::max(c.hidden, (int)qDim), c.ffn);
        // 128-row tiles of the largest launch: Q+K+V, gate+up, the logits head
        const int rows_max = std::max(std::max(c.hidden, (int)(qDim + 2 * kvDim)), std::max(2 * c.ffn, c.vocab));
        LLMDOT_TRY(tc_scratch_alloc(w.tc, cols_max, (rows_max + 127) / 128 + 8, a));
    }
    w.batch = batch;
    return LLMDOT_OK;
}

int gemv(const DevMat &W, const float *x, int ldx, int nv, float *y, int ldy, bool accumulate, bool fast, cudaStream_t st)
{
    if (fast && W.tiled && gemv_fast_supported(W, nv)) return launch_gemv_fast(W, x, ldx, nv, y, ldy, accumulate, st);
    return launch_gemv_ref(W.raw, W.type, W.rows, W.cols, x, ldx, nv, y, ldy, accumulate, st);
}

int StepTimer::begin(cudaStream_t st, int family)
{
    if ((size_t)(2 * n + 2) > ev.size()) {
        cudaEvent_t a, b;
        LLMDOT_CUDA_TRY(cudaEventCreate(&a));
        if (cudaEventCreate(&b) != cudaSuccess) {
            cudaEventDestroy(a);
            return cuda_fail(cudaGetLastError(), "cudaEventCreate");
        }
        ev.push_back(a);
        ev.push_back(b);
    }
    if ((size_t)n >= fam.size()) fam.resize(n + 1);
    fam[n] = family;
    LLMDOT_CUDA_TRY(cudaEventRecord(ev[2 * n], st));
    return LLMDOT_OK;
}

int StepTimer::end(cudaStream_t st)
{
    LLMDOT_CUDA_TRY(cudaEventRecord(ev[2 * n + 1], st));
    n++;
    return LLMDOT_OK;
}

void StepTimer::destroy()
{
    for (cudaEvent_t e : ev) cudaEventDestroy(e);
    ev.clear();
    fam.clear();
    n = 0;
}

// ProcessToken (InferenceEngine.cs:134-146) for `batch` independent sessions at once.
int forward_step(llmdot_model *m, int batch, int kv_type, const int32_t *tokens, const int32_t *pos,
                 const KvView *views, int32_t *next, cudaStream_t st, int flags)
{
    const llmdot_config &c = m->cfg;
    Workspace &w = m->ws;
    const int H = c.hidden, qDim = c.heads * c.head_dim, kvDim = c.heads_kv * c.head_dim;
    const bool gemma = c.template_id == 2;
    const bool fast = m->use_fast_gemv;
    const bool pdl = m->use_pdl;
    AttnShape sh;
    sh.heads = c.heads;
    sh.heads_kv = c.heads_kv;
    sh.head_dim = c.head_dim;
    sh.max_ctx = m->max_ctx;
    sh.sliding_window = c.sliding_window;
    sh.has_cap = c.has_attn_cap;
    sh.cap = c.attn_cap;
    sh.inv_sqrt_hd = 1.0f / sqrtf((float)c.head_dim);
    sh.rope_half = m->rope_half;

    // y = epilogue(W . [rmsnorm](x)); the tensor-core kernel fuses the norm and the epilogue,
    // the generic kernel runs them as separate launches.
    const bool batched = fast && batch <= TC_MAX_ROWS && w.tc.ready();
    // the weights of the next matvec, handed to the current one for an L2 prefetch
    auto tiled_bytes = [](const DevMat *W) -> unsigned long long {
        if (!W || !W->tiled) return 0;
        return (unsigned long long)((W->rows + 15) / 16) * (W->cols / 256) * (W->type == T_Q4_K ? Q4K_TILE : Q6K_TILE);
    };
    auto prefetch = [&](const DevMat *a, const DevMat *b = nullptr, const DevMat *d = nullptr,
                        unsigned long long cap = ~0ull) {
        GemvPrefetch pf = {};
        const DevMat *ms[GEMV_PREFETCH_MAX] = {a, b, d};
        for (int i = 0; i < GEMV_PREFETCH_MAX; i++) {
            const bool i8 = ms[i] && batch <= 2 && ms[i]->tiled8;  // the copy it will read
            pf.p[i] = ms[i] && ms[i]->tiled ? (i8 ? ms[i]->tiled8 : ms[i]->tiled) : nullptr;
            pf.n[i] = pf.p[i] ? std::min(tiled_bytes(ms[i]), cap) : 0;
        }
        return pf;
    };
    auto mv = [&](const DevMat &W, const DevMat *W1, const float *x, int ldx, const float *norm_w, float *y, int ldy,
                  int mode, const GemvPrefetch *pf = nullptr) -> int {
        if (fast && gemv_fast_supported(W, batch) && (!W1 || gemv_fast_supported(*W1, batch)))
            return launch_gemv_fast_ex(W, W1, norm_w, c.eps, x, ldx, batch, y, ldy, mode, st, pdl, pf);
        if (batched && tc_supported(W) && (!W1 || (tc_supported(*W1) && W1->cols == W.cols))) {
            // tensor-core matmul: the input's B operands are built once for the layouts in use
            const bool q4 = W.type == T_Q4_K || (W1 && W1->type == T_Q4_K);
            const bool q6 = W.type == T_Q6_K || (W1 && W1->type == T_Q6_K);
            LLMDOT_TRY(tc_prepare(x, ldx, batch, W.cols, norm_w, c.eps, q4, q6, w.tc, st));
            if (mode == GEMV_SILU_MUL || mode == GEMV_GELU_MUL) {
                const TcSeg sg[2] = {{&W, w.gate, c.ffn}, {W1, w.up, c.ffn}};
                LLMDOT_TRY(tc_gemm(sg, 2, batch, GEMV_STORE, w.tc, w.err, st, pf));
                return launch_act_mul(mode == GEMV_GELU_MUL, w.gate, w.up, y, c.ffn, batch, st);
            }
            const TcSeg sg = {&W, y, ldy};
            return tc_gemm(&sg, 1, batch, mode == GEMV_ADD ? GEMV_ADD : GEMV_STORE, w.tc, w.err, st, pf);
        }
        const float *xin = x;
        int ld = ldx;
        if (norm_w) {
            LLMDOT_TRY(launch_rmsnorm(x, ldx, norm_w, w.xn, H, H, batch, c.eps, st));
            xin = w.xn;
            ld = H;
        }
        if (mode == GEMV_SILU_MUL || mode == GEMV_GELU_MUL) {
            LLMDOT_TRY(launch_gemv_ref(W.raw, W.type, W.rows, W.cols, xin, ld, batch, w.gate, c.ffn, false, st));
            LLMDOT_TRY(launch_gemv_ref(W1->raw, W1->type, W1->rows, W1->cols, xin, ld, batch, w.up, c.ffn, false, st));
            return launch_act_mul(mode == GEMV_GELU_MUL, w.gate, w.up, y, c.ffn, batch, st);
        }
        return launch_gemv_ref(W.raw, W.type, W.rows, W.cols, xin, ld, batch, y, ldy, mode == GEMV_ADD, st);
    };

    // measurement hook: brackets the launches of one operation with events (no-op unless attached)
    StepTimer *tm = m->timer;
    auto tb = [&](int fam) { return tm ? tm->begin(st, fam) : (int)LLMDOT_OK; };
    auto te = [&]() { return tm ? tm->end(st) : (int)LLMDOT_OK; };

    // GetEmbedding + EmbeddingScale
    LLMDOT_TRY(tb(FAM_OTHER));
    LLMDOT_TRY(launch_embed(m->emb.raw, m->emb.type, H, c.vocab, tokens, batch, c.emb_scale, w.h, H, w.err, st));
    LLMDOT_TRY(te());
    for (int l = 0; l < c.layers; l++) {
        const LayerW &L = m->layers[l];
        if (c.template_id == 1) {
            // ProcessGptNeoXLikeLayer (InferenceEngine.cs:198-207): h += FFN(ApplyNorm(h, ffn)).  Its
            // attention result only reaches a buffer the hidden state never reads (the two-argument
            // Add writes its first argument), and no later step reads that layer's K/V either, so
            // neither is computed.  ApplyNorm (:544-562): RMSNorm, or LayerNorm without a bias for
            // the FFN norm; FfnForward (:452-487): gated as in LlamaLike, else up -> Gelu -> down.
            const float *nw = L.ffn_norm ? L.ffn_norm : L.attn_norm;
            const float *xin = w.h, *fused = nullptr;
            LLMDOT_TRY(tb(FAM_OTHER));
            if (c.norm_is_rms) {
                fused = nw;
            } else {
                for (int v = 0; v < batch; v++)
                    LLMDOT_TRY(launch_layernorm(w.h + (size_t)v * H, nw, nullptr, w.xn + (size_t)v * H, H, c.eps, st));
                xin = w.xn;
            }
            LLMDOT_TRY(te());
            LLMDOT_TRY(tb(FAM_MATVEC));
            if (c.ffn_type != 0) {
                LLMDOT_TRY(mv(L.gate, &L.up, xin, H, fused, w.gate, c.ffn, c.ffn_type == 2 ? GEMV_GELU_MUL : GEMV_SILU_MUL));
            } else {
                LLMDOT_TRY(mv(L.up, nullptr, xin, H, fused, w.gate, c.ffn, GEMV_STORE));
                LLMDOT_TRY(launch_eltwise(OP_GELU, w.gate, nullptr, w.gate, c.ffn * batch, 0.0f, st, c.ffn));
            }
            LLMDOT_TRY(mv(L.down, nullptr, w.gate, c.ffn, nullptr, w.h, H, GEMV_ADD));
            LLMDOT_TRY(te());
            continue;
        }
        // L2 prefetches: each matvec pulls in the weights of the one after it (the attention
        // sits between Q/K/V and the output projection)
        const GemvPrefetch pf_o = prefetch(&L.o), pf_ffn = prefetch(&L.gate, &L.up), pf_down = prefetch(&L.down);
        GemvPrefetch pf_next;
        if (l + 1 < c.layers) {
            const LayerW &N = m->layers[l + 1];
            pf_next = N.qkv.valid() ? prefetch(&N.qkv) : prefetch(&N.q, &N.k, &N.v);
        } else {
            const DevMat &head = m->out.valid() ? m->out : m->emb;
            pf_next = prefetch(&head, nullptr, nullptr, 64ull << 20);  // as much of the head as L2 keeps
        }
        // ApplyNorm(attn_norm) :544-562 fused into the Q/K/V projections :321-353
        float *q, *k, *v;
        int ldq, ldkv;
        LLMDOT_TRY(tb(FAM_MATVEC));
        if (L.qkv.valid()) {
            LLMDOT_TRY(mv(L.qkv, nullptr, w.h, H, L.attn_norm, w.qkv, qDim + 2 * kvDim, GEMV_STORE, &pf_o));
            q = w.qkv;
            k = w.qkv + qDim;
            v = w.qkv + qDim + kvDim;
            ldq = ldkv = qDim + 2 * kvDim;
        } else {
            int qkv_rc = LLMDOT_E_UNSUPPORTED;
            if (fast && gemv_fast_supported(L.q, batch) && gemv_fast_supported(L.k, batch) &&
                gemv_fast_supported(L.v, batch)) {
                // Q, K and V share the normed input: one launch
                const GemvTarget tg[3] = {{&L.q, nullptr, w.q, qDim}, {&L.k, nullptr, w.k, kvDim},
                                          {&L.v, nullptr, w.v, kvDim}};
                qkv_rc = launch_gemv_multi(tg, 3, L.attn_norm, c.eps, w.h, H, batch, GEMV_STORE, pdl, st, &pf_o);
                if (qkv_rc != LLMDOT_OK && qkv_rc != LLMDOT_E_UNSUPPORTED) return qkv_rc;
            }
            if (qkv_rc != LLMDOT_OK && batched && tc_supported(L.q) && tc_supported(L.k) && tc_supported(L.v)) {
                // batched: Q, K and V in one tensor-core launch over the normed input
                const DevMat *mats[3] = {&L.q, &L.k, &L.v};
                bool q4 = false, q6 = false;
                for (const DevMat *M : mats) {
                    q4 = q4 || M->type == T_Q4_K;
                    q6 = q6 || M->type == T_Q6_K;
                }
                LLMDOT_TRY(tc_prepare(w.h, H, batch, H, L.attn_norm, c.eps, q4, q6, w.tc, st));
                const TcSeg sg[3] = {{&L.q, w.q, qDim}, {&L.k, w.k, kvDim}, {&L.v, w.v, kvDim}};
                LLMDOT_TRY(tc_gemm(sg, 3, batch, GEMV_STORE, w.tc, w.err, st, &pf_o));
                qkv_rc = LLMDOT_OK;
            }
            if (qkv_rc != LLMDOT_OK) {
                // mixed Q4_K/Q6_K segments whose shared-memory layout does not fit one launch
                LLMDOT_TRY(mv(L.q, nullptr, w.h, H, L.attn_norm, w.q, qDim, GEMV_STORE));
                LLMDOT_TRY(mv(L.k, nullptr, w.h, H, L.attn_norm, w.k, kvDim, GEMV_STORE));
                LLMDOT_TRY(mv(L.v, nullptr, w.h, H, L.attn_norm, w.v, kvDim, GEMV_STORE));
            }
            q = w.q;
            k = w.k;
            v = w.v;
            ldq = qDim;
            ldkv = kvDim;
        }
        LLMDOT_TRY(te());
        // RoPE of q and k, K/V cache append :362-382, attention :384-442
        LLMDOT_TRY(tb(FAM_ATTENTION));
        LLMDOT_TRY(launch_attention_step(q, ldq, k, v, ldkv, pos, m->cos_t, m->sin_t, views, l, kv_type, sh, batch,
                                         w.scores, w.part_m, w.part_s, w.part_o, w.counters, w.attn, qDim,
                                         (flags & STEP_CHUNK) != 0, pdl, st));
        LLMDOT_TRY(te());
        // attn_output matvec + residual add :444-449, :189
        // tensor parallel: rank 0 adds its partial onto the residual, the others store theirs, and
        // the all-reduce leaves h + the sum of the partials on every rank
        const int res_mode = (m->tp > 1 && m->tp_rank != 0) ? GEMV_STORE : GEMV_ADD;
        LLMDOT_TRY(tb(FAM_MATVEC));
        LLMDOT_TRY(mv(L.o, nullptr, w.attn, qDim, nullptr, w.h, H, res_mode, &pf_ffn));
        LLMDOT_TRY(te());
        if (m->tp > 1) {
            LLMDOT_TRY(tb(FAM_COLLECTIVE));
            LLMDOT_TRY(tp_allreduce_sum(m, w.h, (size_t)batch * H, st));
            LLMDOT_TRY(te());
        }
        if (gemma && L.post_attn) {
            LLMDOT_TRY(tb(FAM_OTHER));
            LLMDOT_TRY(launch_rmsnorm(w.h, H, L.post_attn, w.h, H, H, batch, c.eps, st, pdl));
            LLMDOT_TRY(te());
        }
        // FfnForward :452-487: ApplyNorm(ffn_norm ?? attn_norm), gate and up, act(gate)*up in one launch
        LLMDOT_TRY(tb(FAM_MATVEC));
        LLMDOT_TRY(mv(L.gate, &L.up, w.h, H, L.ffn_norm ? L.ffn_norm : L.attn_norm, w.gate, c.ffn,
                      c.ffn_type == 2 ? GEMV_GELU_MUL : GEMV_SILU_MUL, &pf_down));
        LLMDOT_TRY(te());
        // down projection + residual add
        LLMDOT_TRY(tb(FAM_MATVEC));
        LLMDOT_TRY(mv(L.down, nullptr, w.gate, c.ffn, nullptr, w.h, H, res_mode, &pf_next));
        LLMDOT_TRY(te());
        if (m->tp > 1) {
            LLMDOT_TRY(tb(FAM_COLLECTIVE));
            LLMDOT_TRY(tp_allreduce_sum(m, w.h, (size_t)batch * H, st));
            LLMDOT_TRY(te());
        }
        if (gemma && L.post_ffw) {
            LLMDOT_TRY(tb(FAM_OTHER));
            LLMDOT_TRY(launch_rmsnorm(w.h, H, L.post_ffw, w.h, H, H, batch, c.eps, st, pdl));
            LLMDOT_TRY(te());
        }
    }
    if (flags & STEP_NO_HEAD) return LLMDOT_OK;  // prompt chunk before the last: no logits needed
    // ApplyFinalNorm :575-581 fused into ComputeLogits :583-602
    const DevMat &head = m->out.valid() ? m->out : m->emb;
    // logits rows [head_lo, head_lo + head_rows): the whole vocabulary without tensor parallelism
    LLMDOT_TRY(tb(FAM_MATVEC));
    LLMDOT_TRY(mv(head, nullptr, w.h, H, m->out_norm, w.logits, m->head_rows, GEMV_STORE));
    LLMDOT_TRY(te());
    // final softcap + greedy argmax (InferenceEngine.cs:105-108, Sampler.cs:26-27); across ranks the
    // packed (value, index) keys reduce with max
    LLMDOT_TRY(tb(FAM_OTHER));
    LLMDOT_TRY(launch_argmax_keys(w.logits, m->head_rows, m->head_rows, batch, w.keys, c.has_final_cap != 0,
                                  c.final_cap, nullptr, m->head_lo, c.vocab, st));
    LLMDOT_TRY(te());
    if (m->tp > 1) {
        LLMDOT_TRY(tb(FAM_COLLECTIVE));
        LLMDOT_TRY(tp_allreduce_max_u64(m, w.keys, batch, st));
        LLMDOT_TRY(te());
    }
    LLMDOT_TRY(tb(FAM_OTHER));
    LLMDOT_TRY(launch_argmax_finish(w.keys, batch, next, st));
    return te();
}

}  // namespace llmdot
