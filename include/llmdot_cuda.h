/*
 * llmdot_cuda.h -- C ABI of the B200 (sm_100a) backend for llmdot.
 *
 * Plain C types only (no CUDA or torch types): the .NET package binds these
 * with [LibraryImport] (blittable pointers, ints, nint handles, UTF-8 keys);
 * tests and the benchmark bind them with Python ctypes.
 *
 * Every function returns 0 on success or a negative LLMDOT_E* status; the
 * message of the last failure on the calling thread is available from
 * llmdot_cuda_last_error().  There is no CPU fallback: a missing device, an
 * unsupported tensor type or a CUDA error is reported, never emulated.
 *
 * Two tiers:
 *   Tier A mirrors llmdot's per-operation backend adapter IComputeBackend
 *     (src/Llmdot.Core/Inference/Backends/IComputeBackend.cs:7-28) one call per
 *     interface method, over HOST buffers (the interface passes host spans).
 *     Weight matrices are uploaded once and cached on the device under their
 *     weightKey (the tensor name), as MetalBackend does
 *     (src/Llmdot.Metal/MetalBackend.cs:85-104).
 *   Tier B is the device-resident decode/prefill path: model upload, sessions
 *     with a paged KV cache, prefill, batched greedy decode and a greedy
 *     Generate loop that mirrors InferenceEngine.Generate
 *     (src/Llmdot.Core/Inference/InferenceEngine.cs:74-132).
 */
#ifndef LLMDOT_CUDA_H
#define LLMDOT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define LLMDOT_API __declspec(dllexport)
#else
#define LLMDOT_API __attribute__((visibility("default")))
#endif

/* ---- status codes ---------------------------------------------------------------- */
#define LLMDOT_OK 0
#define LLMDOT_E_INVALID (-1)     /* bad argument (null pointer, size mismatch, range) */
#define LLMDOT_E_UNSUPPORTED (-2) /* tensor type / model feature not implemented on the device */
#define LLMDOT_E_CUDA (-3)        /* CUDA runtime / driver error */
#define LLMDOT_E_NOMEM (-4)       /* device or host allocation failed */
#define LLMDOT_E_FORMAT (-5)      /* malformed GGUF / model description */
#define LLMDOT_E_NCCL (-6)        /* collective communication error */
#define LLMDOT_E_TIMEOUT (-7)     /* a bounded device-side wait gave up */

/* GgmlType values (src/Llmdot.Core/Loading/GgmlType.cs:3-27) */
#define LLMDOT_F32 0u
#define LLMDOT_F16 1u
#define LLMDOT_Q4_0 2u
#define LLMDOT_Q4_1 3u
#define LLMDOT_Q5_0 6u
#define LLMDOT_Q5_1 7u
#define LLMDOT_Q8_0 8u
#define LLMDOT_Q2_K 10u
#define LLMDOT_Q3_K 11u
#define LLMDOT_Q4_K 12u
#define LLMDOT_Q5_K 13u
#define LLMDOT_Q6_K 14u
#define LLMDOT_BF16 25u

/* Thread-local message of the last failure (never NULL). */
LLMDOT_API const char *llmdot_cuda_last_error(void);
/* Library version string, e.g. "llmdot-cuda 0.1 sm_100a". */
LLMDOT_API const char *llmdot_cuda_version(void);
/* Number of CUDA devices visible to the process (0 on a machine without GPUs). */
LLMDOT_API int llmdot_cuda_device_count(int *count);

/* ====================================================================================
 * Tier A -- per-operation adapter, one entry point per IComputeBackend method.
 * All float/byte pointers are HOST memory owned by the caller and valid only for
 * the duration of the call (the interface's span semantics).  Calls on one handle
 * are serialised on its CUDA stream and synchronous.
 * ==================================================================================== */
typedef struct llmdot_backend llmdot_backend;

/* new CudaBackend(device) -- replaces the CpuBackend ctor (CpuBackend.cs:8). */
LLMDOT_API int llmdot_cuda_create(int device, llmdot_backend **out);
/* IDisposable.Dispose (IComputeBackend.cs:7) -- frees cached weights and scratch. */
LLMDOT_API int llmdot_cuda_destroy(llmdot_backend *h);

/* MatMul(a, b, result, bType, aCols, bCols, weightKey) (IComputeBackend.cs:9).
 * aRows = resultLen / bCols (TensorOps.cs:62).  b holds bCols rows of aCols quantised
 * elements (bBytes bytes).  weightKey != NULL caches b on the device under that key;
 * later calls with the same key reuse the device copy and ignore b's contents. */
LLMDOT_API int llmdot_cuda_matmul(llmdot_backend *h, const float *a, int aLen, const uint8_t *b,
                                  size_t bBytes, uint32_t bType, int aCols, int bCols,
                                  const char *weightKey, float *result, int resultLen);
/* MatMulF32(a, b, result, aCols, bCols, weightKey) (IComputeBackend.cs:10). */
LLMDOT_API int llmdot_cuda_matmul_f32(llmdot_backend *h, const float *a, int aLen, const float *b,
                                      size_t bLen, int aCols, int bCols, const char *weightKey,
                                      float *result, int resultLen);
/* RmsNorm(input, weights, output, epsilon) (IComputeBackend.cs:11). */
LLMDOT_API int llmdot_cuda_rmsnorm(llmdot_backend *h, const float *input, const float *weights,
                                   float *output, int n, float epsilon);
/* LayerNorm(input, weights, bias, output, epsilon) (IComputeBackend.cs:12); bias may be NULL. */
LLMDOT_API int llmdot_cuda_layernorm(llmdot_backend *h, const float *input, const float *weights,
                                     const float *bias, float *output, int n, float epsilon);
/* ApplyRoPE(query, key, headDim, position, freqBase, rotaryDim) (IComputeBackend.cs:13).
 * query and key are rotated in place; key == query means "same span" (applied once). */
LLMDOT_API int llmdot_cuda_rope(llmdot_backend *h, float *query, int qLen, float *key, int kLen,
                                int headDim, int position, float freqBase, int rotaryDim);
/* ApplyRoPE(query, key, headDim, position, freqTable) (IComputeBackend.cs:14). */
LLMDOT_API int llmdot_cuda_rope_table(llmdot_backend *h, float *query, int qLen, float *key,
                                      int kLen, int headDim, int position, const float *freqTable,
                                      int halfDim);
/* Softmax(input, softcap) (IComputeBackend.cs:15); hasSoftcap=0 means null. */
LLMDOT_API int llmdot_cuda_softmax(llmdot_backend *h, float *x, int n, int hasSoftcap, float softcap);
/* Silu(input, result) / SiluInPlace(input) (IComputeBackend.cs:16-17). */
LLMDOT_API int llmdot_cuda_silu(llmdot_backend *h, const float *input, float *result, int n);
LLMDOT_API int llmdot_cuda_silu_inplace(llmdot_backend *h, float *x, int n);
/* Gelu(input, result) (IComputeBackend.cs:18). */
LLMDOT_API int llmdot_cuda_gelu(llmdot_backend *h, const float *input, float *result, int n);
/* GeluScalar(x) (IComputeBackend.cs:19), evaluated on the device. */
LLMDOT_API int llmdot_cuda_gelu_scalar(llmdot_backend *h, float x, float *result);
/* Add(a, b) in place / Add(a, b, result) (IComputeBackend.cs:20-21). */
LLMDOT_API int llmdot_cuda_add_inplace(llmdot_backend *h, float *a, const float *b, int n);
LLMDOT_API int llmdot_cuda_add(llmdot_backend *h, const float *a, const float *b, float *result, int n);
/* Scale(input, scale, result) / Scale(input, scale) in place (IComputeBackend.cs:22-23). */
LLMDOT_API int llmdot_cuda_scale(llmdot_backend *h, const float *input, float scale, float *result, int n);
LLMDOT_API int llmdot_cuda_scale_inplace(llmdot_backend *h, float *x, int n, float scale);
/* Mul(a, b, result) (IComputeBackend.cs:24). */
LLMDOT_API int llmdot_cuda_mul(llmdot_backend *h, const float *a, const float *b, float *result, int n);
/* Softcap(input, cap) in place (IComputeBackend.cs:25). */
LLMDOT_API int llmdot_cuda_softcap(llmdot_backend *h, float *x, int n, float cap);
/* Conv1D(input, weights, output, kernelSize, inputDim) (IComputeBackend.cs:26). */
LLMDOT_API int llmdot_cuda_conv1d(llmdot_backend *h, const float *input, const float *weights,
                                  float *output, int kernelSize, int inputDim);
/* DequantizeToFloat(src, dst, type, numRows, rowElements) (IComputeBackend.cs:27).
 * Bit-exact with the reference's fp32 dequantisation for every supported type. */
LLMDOT_API int llmdot_cuda_dequantize(llmdot_backend *h, const uint8_t *src, size_t srcBytes,
                                      uint32_t type, int numRows, int rowElements, float *dst);
/* ArgMax(input) (IComputeBackend.cs:28): first index of the maximum. */
LLMDOT_API int llmdot_cuda_argmax(llmdot_backend *h, const float *x, int n, int *index);

/* ====================================================================================
 * Tier B -- device-resident decode / prefill.
 * ==================================================================================== */

/* Resolved hyper-parameters: TransformerConfig (doc/architecture.md:171-225) as
 * produced by ArchitectureResolver.Resolve (src/Llmdot.Core/Loading/ArchitectureResolver.cs:14-112). */
typedef struct llmdot_config {
    int32_t template_id;  /* ExecutionTemplate: 0 LlamaLike, 1 GptNeoXLike, 2 GemmaLike, 3 Lfm2Like */
    int32_t hidden;       /* HiddenSize */
    int32_t layers;       /* LayerCount */
    int32_t context;      /* ContextLength */
    int32_t vocab;        /* VocabSize */
    int32_t ffn;          /* FfnDim */
    int32_t heads;        /* HeadCount */
    int32_t heads_kv;     /* HeadCountKv */
    int32_t head_dim;     /* HeadDim */
    int32_t qkv_fused;    /* QkvLayout == Fused */
    int32_t norm_is_rms;  /* NormType == RmsNorm */
    float eps;            /* NormEpsilon */
    int32_t has_post_norm;
    float rope_base;      /* RopeFreqBase */
    int32_t rope_dim;     /* RopeDimensionCount */
    int32_t rope_scaling; /* RopeScalingType: 0 None, 1 Linear, 2 YaRN, 3 LongRoPE */
    float rope_factor;
    int32_t ffn_type;     /* FfnType: 0 Standard, 1 SwiGLU, 2 GeGLU */
    int32_t parallel_residual;
    int32_t tied;         /* TiedEmbeddings */
    float emb_scale;      /* EmbeddingScale */
    int32_t sliding_window;
    int32_t has_attn_cap;
    float attn_cap;       /* AttnLogitSoftcap */
    int32_t has_final_cap;
    float final_cap;      /* FinalLogitSoftcap */
    int32_t expert_count;
    int32_t bos;          /* BosTokenId */
    int32_t eos;          /* EosTokenId */
} llmdot_config;

/* One GGUF tensor as LoadedModel holds it (src/Llmdot.Core/Inference/LoadedModel.cs:77-107;
 * Tensor.cs: dims[0] = columns / in-features, dims[1] = rows). */
typedef struct llmdot_tensor_desc {
    const char *name;
    uint32_t type;      /* GgmlType */
    uint32_t n_dims;
    uint64_t dims[4];
    const void *data;   /* host bytes, TensorSize.ByteCount(type, elements) long */
    uint64_t n_bytes;
} llmdot_tensor_desc;

typedef struct llmdot_model llmdot_model;
typedef struct llmdot_session llmdot_session;

/* KV element types for sessions */
#define LLMDOT_KV_F16 0
#define LLMDOT_KV_F32 1

/* Upload a model that the host has already parsed (LoadedModel + TransformerConfig).
 * Weights are copied to the device once and re-laid out for the kernels. */
LLMDOT_API int llmdot_cuda_model_load(int device, const llmdot_config *cfg,
                                      const llmdot_tensor_desc *tensors, int n_tensors,
                                      llmdot_model **out);
/* Parse a GGUF file natively (GgufReader + ArchitectureResolver restated in C++),
 * stream its tensors to the device and upload the model. */
LLMDOT_API int llmdot_cuda_model_load_gguf(int device, const char *path, llmdot_model **out);
/* The same parse and ArchitectureResolver.Resolve (ArchitectureResolver.cs:14-112) without
 * loading anything: host only, no device needed.  Fails with LLMDOT_E_FORMAT and the
 * reference's message for a missing or unsupported general.architecture or a missing norm
 * epsilon. */
LLMDOT_API int llmdot_cuda_gguf_config(const char *path, llmdot_config *out);
LLMDOT_API int llmdot_cuda_model_config(const llmdot_model *m, llmdot_config *out);
/* Quantised weight bytes the decode step streams per token (layers + logits head). */
LLMDOT_API int llmdot_cuda_model_weight_bytes(const llmdot_model *m, uint64_t *layer_bytes,
                                              uint64_t *head_bytes);
/* Sessions of the model that are still open stay valid for llmdot_cuda_session_free only;
 * every other call on them returns LLMDOT_E_INVALID. */
LLMDOT_API int llmdot_cuda_model_free(llmdot_model *m);

/* A session = one InferenceEngine's KvCache (src/Llmdot.Core/Inference/KvCache.cs), held on
 * the device as pages of LLMDOT_KV_PAGE positions.  max_ctx <= 0 means the model's context. */
LLMDOT_API int llmdot_cuda_session_create(llmdot_model *m, int max_ctx, int kv_type,
                                          llmdot_session **out);
LLMDOT_API int llmdot_cuda_session_reset(llmdot_session *s);       /* KvCache.Reset */
LLMDOT_API int llmdot_cuda_session_position(const llmdot_session *s, int *pos);
LLMDOT_API int llmdot_cuda_session_free(llmdot_session *s);

/* Feed n prompt tokens (positions pos..pos+n-1), i.e. the prefill loop of Generate
 * (InferenceEngine.cs:84-88).  logits (host, nullable) receives the raw logits of the last
 * token; next_token (nullable) its greedy argmax after the final softcap. */
LLMDOT_API int llmdot_cuda_prefill(llmdot_session *s, const int32_t *tokens, int n, float *logits,
                                   int32_t *next_token);

/* One greedy decode step for `batch` sessions of the same model: token[i] is appended to
 * sessions[i] at its current position.  next_tokens (host) receives the argmax of each
 * session's new logits (after the final softcap, Sampler.cs:26-27); logits (host, nullable)
 * receives the raw logits [batch][vocab]. */
LLMDOT_API int llmdot_cuda_decode(llmdot_session **sessions, int batch, const int32_t *tokens,
                                  int32_t *next_tokens, float *logits);

/* Greedy InferenceEngine.Generate (InferenceEngine.cs:74-132) on the device: reset the
 * session, prefill the prompt, then decode up to max_tokens tokens, stopping after EOS.
 * The loop runs without host round trips (CUDA graph).  out_tokens receives the generated
 * ids, n_out their count. */
LLMDOT_API int llmdot_cuda_generate(llmdot_session *s, const int32_t *prompt, int n_prompt,
                                    int max_tokens, int32_t *out_tokens, int *n_out);

/* SamplingOptions (src/Llmdot.Core/Sampling/SamplingOptions.cs:7-14); the reference's defaults are
 * top_k 40, top_p 0.95, temperature 0.8, repeat_penalty 1.1, repeat_window 64, seed -1. */
typedef struct llmdot_sampling {
    int32_t top_k;
    float top_p;
    float temperature;
    float repeat_penalty;
    int32_t repeat_window;
    int32_t seed; /* >= 0: every draw is new System.Random(seed).NextSingle(); < 0: fresh draws */
} llmdot_sampling;

/* new System.Random(seed).NextSingle(): the draw Sampler.SampleFromProbabilities uses for
 * seed >= 0 (Sampler.cs:155-157).  Host only. */
LLMDOT_API float llmdot_cuda_sampling_seeded_draw(int32_t seed);

/* Sampler.Sample (Sampler.cs:24-62) for one row of host logits (vocabulary n), on the device:
 * repeat penalty over the last repeat_window entries of recent (oldest first), scaling by
 * 1/temperature, then
 *   0 < top_k < n: top-k, softmax over the k, and the first index whose running probability
 *                  reaches r (the uniform draw in [0, 1)); top_k <= 1024 on the device;
 *   otherwise:     softmax over the whole row, then with top_p < 1 the nucleus (FindNucleus,
 *                  including the reference's aliased value buffer: a nucleus that is the whole
 *                  row returns a position of the sorted order, as the reference does), else the
 *                  pick over the whole row.
 * temperature <= 0 is the argmax.  repeat_window <= 1024.  Exactly tied logits at the k-th place
 * are taken lowest index first.  LLMDOT_E_UNSUPPORTED: top_k in (1024, n), or a tie group of
 * more than 8192 equal probabilities inside the nucleus. */
LLMDOT_API int llmdot_cuda_sample(llmdot_backend *h, const float *logits, int n, const llmdot_sampling *opt,
                                  const int32_t *recent, int n_recent, float r, int32_t *index);

/* InferenceEngine.Generate (InferenceEngine.cs:74-131) with Sampler.Sample: reset, prefill, then
 * per token the final softcap, the sample over the device logits (history = the prompt, then every
 * generated token, the last repeat_window + 1 kept) and the decode step, stopping after EOS or
 * max_tokens.  draws (nullable, max_tokens entries) are the uniform draws of the tokens; null means
 * the seeded draw for seed >= 0 and a fresh draw per token (host generator) for seed < 0.
 * Same device limits as llmdot_cuda_sample; not under tensor parallelism. */
LLMDOT_API int llmdot_cuda_generate_sampled(llmdot_session *s, const int32_t *prompt, int n_prompt,
                                            int max_tokens, const llmdot_sampling *opt, const float *draws,
                                            int32_t *out_tokens, int *n_out);

/* Device-resident greedy decode of n_steps tokens for `batch` sessions in lockstep (the decode
 * loop of Generate without the per-token EOS / stop-sequence check): tokens[b] is fed first, and
 * out_tokens[step * batch + b] receives every step's argmax.  Steps run as back-to-back CUDA-graph
 * replays with no host round trip.  elapsed_ms (nullable) receives the device time of the n_steps
 * replays (CUDA events on the model's stream); kernels_per_step (nullable) the number of kernel
 * launches one step performs. */
LLMDOT_API int llmdot_cuda_decode_steps(llmdot_session **sessions, int batch, const int32_t *tokens,
                                        int n_steps, int32_t *out_tokens, float *elapsed_ms,
                                        int *kernels_per_step);

/* Diagnostic (no counterpart in the reference): y = W . x for one uploaded weight tensor and
 * `batch` host input rows x [batch][cols] -> y [batch][rows] (host), through the same device
 * matvec the decode step uses for that tensor (mode 0), the generic per-element kernel (mode 1),
 * or with the step's fused RMSNorm of x by norm_w (mode 2, norm_w host [cols]). */
LLMDOT_API int llmdot_cuda_model_matvec(llmdot_model *m, const char *tensor, const float *x, int batch,
                                        int mode, const float *norm_w, float *y);

/* ---- tensor parallelism (Megatron-style, one process per GPU) ---------------------------
 * One process per GPU (in place of a single-process `tp_init(model, tpSize, devices)`): every
 * rank loads ITS shard of the model, rank 0 creates an NCCL unique id that the host distributes
 * (e.g. with torch.distributed), and every rank attaches it.  Shards: attn_q/k/v and
 * ffn_gate/up by output rows (whole heads), attn_output and ffn_down by input columns, the
 * logits head by vocabulary rows; the embedding and norms stay whole.  Each decode step then
 * does one in-place all-reduce of the residual after attn_output and one after ffn_down, and a
 * max all-reduce of the packed argmax keys (NCCL's, or the peer exchange's once it is open).  All ranks must make the same prefill /
 * decode / generate calls in the same order (they contain collectives); logits read back under
 * TP are gathered from every rank (needs vocab % tp_size == 0).  llmdot_cuda_model_config
 * returns the full model's configuration. */
LLMDOT_API int llmdot_cuda_model_load_gguf_tp(int device, const char *path, int tp_size, int tp_rank,
                                              llmdot_model **out);
/* 128 bytes of ncclUniqueId (NCCL is loaded at run time from libnccl.so.2). */
LLMDOT_API int llmdot_cuda_tp_unique_id(uint8_t *out128);
/* Attaches the NCCL communicator (ncclCommInitRank on the model's device). */
LLMDOT_API int llmdot_cuda_tp_init(llmdot_model *m, const uint8_t *id128);
/* Peer-memory all-reduce for the step's two residual sums (one kernel over NVLink instead of
 * NCCL's all-reduce), after llmdot_cuda_tp_init: every rank exports a 128-byte handle (the CUDA IPC
 * handle of its exchange buffer and its GPU's UUID) into out128, the host hands all ranks' handles
 * to every rank in rank order (tp x 128 bytes), and every rank opens them; two ranks on one GPU
 * are refused (LLMDOT_E_UNSUPPORTED).  Each sum then adds the ranks' partials in rank order on
 * every rank (identical results everywhere), and the greedy argmax's max-reduce of the ranks' keys
 * runs over the same buffers; sums larger than 64 rows of the hidden state stay on NCCL, as do the
 * logits all-gathers.  Every wait is bounded (10 s, then LLMDOT_E_TIMEOUT).
 * Needs 2 to 8 ranks whose GPUs can map each other's memory.  Once open, llmdot_cuda_model_free
 * is collective too: it waits (at most 5 s) for every rank to reach its own free before releasing
 * the buffer, and leaves the buffer allocated if a rank never does.  Replaces no reference
 * interface: the reference has no multi-GPU path; this is the NVLink form of the NCCL sum above. */
LLMDOT_API int llmdot_cuda_tp_exchange_handle(llmdot_model *m, uint8_t *out128);
LLMDOT_API int llmdot_cuda_tp_exchange_open(llmdot_model *m, const uint8_t *handles);
/* Whether the step's residual sums use the opened peer-memory all-reduce (on = 1, the state after
 * open) or NCCL's (on = 0).  Every rank must make the same choice before its next step: a rank
 * whose open succeeded turns it off when another rank's open failed. */
LLMDOT_API int llmdot_cuda_tp_exchange_use(llmdot_model *m, int on);
/* Shard geometry of rank tp_rank (host only, no device needed): out8 = {q_lo, q_n, kv_lo, kv_n,
 * ffn_lo, ffn_n, vocab_lo, vocab_n} in rows / columns of the full matrices. */
LLMDOT_API int llmdot_cuda_tp_shard(const llmdot_config *cfg, int tp_size, int tp_rank, int32_t *out8);

/* Profiling hook (no counterpart in the reference): average device time of one matvec launch
 * over the named weight tensor for `batch` input rows; `iters` launches are captured into a CUDA
 * graph and one replay is timed with CUDA events on the model's stream.  A name of the form
 * "blk.*.<suffix>" walks that matrix of every layer in turn (weights stream from HBM as in a
 * decode step).  bytes receives the quantised bytes one launch streams (layer average). */
LLMDOT_API int llmdot_cuda_profile_matvec(llmdot_model *m, const char *tensor, int batch, int iters,
                                          float *avg_ms, uint64_t *bytes);

/* Measurement hook (no counterpart in the reference): ONE greedy decode step for `batch` sessions
 * fed `tokens`, launched operation by operation (not from the captured step graph) with CUDA events
 * around each operation's launches on the model's stream.  family_ms[f] and family_launches[f]
 * receive the summed device time (ms) and the number of timed operations of kernel family f, for
 * f < n_families: 0 quantised matvec / matmul (with its fused norm, activation and residual
 * epilogues), 1 attention (RoPE, KV append, attention), 2 other element-wise kernels (embedding,
 * Gemma post-norms, argmax), 3 collectives (tensor parallelism).  next_tokens (nullable) receives
 * the greedy ids; the sessions advance by one token, as with llmdot_cuda_decode.  Under tensor
 * parallelism every rank makes the same call. */
LLMDOT_API int llmdot_cuda_profile_step(llmdot_session **sessions, int batch, const int32_t *tokens,
                                        int32_t *next_tokens, int n_families, float *family_ms, int *family_launches);

/* Greedy argmax over logits that are already in device memory, without allocating any device
 * memory.  No counterpart in the reference: it exists for hosts that own all device memory
 * themselves (e.g. pools reserved at start-up for weights, KV pages and logits) and cannot let
 * a library call cudaMalloc during the token loop, where it could fail or stall the device.
 *   d_logits  device pointer, `rows` vectors of `n` floats, row r starting at d_logits + r*ld
 *   d_index   device pointer, receives `rows` int32 results: first index of each row's maximum
 *   stream    a cudaStream_t passed as a plain pointer (NULL = the legacy default stream)
 * The only scratch is one fixed array inside the library: LLMDOT_ARGMAX_NOALLOC_MAX_ROWS 64-bit
 * keys (32 KiB), which every GPU that loads the library holds until the process exits; more rows
 * are rejected with LLMDOT_E_INVALID.  The call is asynchronous on `stream`.  All calls on a
 * device share that array and it keeps the last call's contents (each call clears the rows it
 * uses): calls that overlap on the GPU race and return wrong indices.  The first call on each
 * device looks the array's address up (cudaGetSymbolAddress) with that device current and is
 * the first launch of its two kernels; with CUDA's lazy module loading both load the library's
 * device code, for which the driver itself may take device memory.  So make one warm-up call on
 * each device before the host reserves its memory pools, and before any stream capture; later
 * calls allocate nothing.  The address is kept per device for the life of the process: after a
 * cudaDeviceReset (or anything else that destroys the device's primary context) the cached
 * address is stale, so do not reset a device that this entry point has been used on. */
#define LLMDOT_ARGMAX_NOALLOC_MAX_ROWS 4096
LLMDOT_API int llmdot_cuda_argmax_noalloc(const float *d_logits, int n, int rows, int ld, int32_t *d_index,
                                          void *stream);

#ifdef __cplusplus
}
#endif
#endif /* LLMDOT_CUDA_H */
