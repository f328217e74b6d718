// tp.cu -- tensor-parallel shard geometry and NCCL collectives (NCCL loaded at run time).
#include <dlfcn.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "engine.cuh"
#include "tp.cuh"

namespace llmdot {

int tp_shard(const llmdot_config &c, int tp, int rank, TpShard *s)
{
    if (tp < 1 || rank < 0 || rank >= tp) return fail(LLMDOT_E_INVALID, "tensor parallel: bad size or rank");
    if (c.heads % tp || c.heads_kv % tp || c.ffn % tp)
        return fail(LLMDOT_E_UNSUPPORTED, "tensor parallel: heads, kv heads and FFN rows must divide by the TP size");
    const int qn = c.heads / tp * c.head_dim, kvn = c.heads_kv / tp * c.head_dim, fn = c.ffn / tp;
    if (tp > 1 && (qn % 256 || fn % 256))
        return fail(LLMDOT_E_UNSUPPORTED, "tensor parallel: attn_output / ffn_down column shards must be whole super-blocks");
    s->q_lo = rank * qn;
    s->q_n = qn;
    s->kv_lo = rank * kvn;
    s->kv_n = kvn;
    s->f_lo = rank * fn;
    s->f_n = fn;
    s->v_lo = (int)((long long)rank * c.vocab / tp);
    s->v_n = (int)((long long)(rank + 1) * c.vocab / tp) - s->v_lo;
    return LLMDOT_OK;
}

// ------------------------------------------------------------------ NCCL, resolved at run time
namespace {

struct NcclId {
    char internal[128];  // ncclUniqueId
};
typedef void *NcclComm;
enum { NCCL_UINT64 = 5, NCCL_FLOAT = 7, NCCL_SUM = 0, NCCL_MAX = 2 };  // ncclDataType_t / ncclRedOp_t values

struct Nccl {
    bool tried = false, ok = false;
    std::string why;
    int (*getUniqueId)(NcclId *) = nullptr;
    int (*commInitRank)(NcclComm *, int, NcclId, int) = nullptr;
    int (*commDestroy)(NcclComm) = nullptr;
    int (*allReduce)(const void *, void *, size_t, int, int, NcclComm, cudaStream_t) = nullptr;
    int (*allGather)(const void *, void *, size_t, int, NcclComm, cudaStream_t) = nullptr;
    const char *(*getErrorString)(int) = nullptr;
};

Nccl &nccl()
{
    static Nccl n;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (n.tried) return n;
    n.tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        n.why = std::string("libnccl.so.2 not loadable: ") + dlerror();
        return n;
    }
    n.getUniqueId = (int (*)(NcclId *))dlsym(h, "ncclGetUniqueId");
    n.commInitRank = (int (*)(NcclComm *, int, NcclId, int))dlsym(h, "ncclCommInitRank");
    n.commDestroy = (int (*)(NcclComm))dlsym(h, "ncclCommDestroy");
    n.allReduce = (int (*)(const void *, void *, size_t, int, int, NcclComm, cudaStream_t))dlsym(h, "ncclAllReduce");
    n.allGather = (int (*)(const void *, void *, size_t, int, NcclComm, cudaStream_t))dlsym(h, "ncclAllGather");
    n.getErrorString = (const char *(*)(int))dlsym(h, "ncclGetErrorString");
    n.ok = n.getUniqueId && n.commInitRank && n.commDestroy && n.allReduce && n.allGather && n.getErrorString;
    if (!n.ok) n.why = "libnccl.so.2 lacks an expected symbol";
    return n;
}

int nccl_fail(int r, const char *what)
{
    Nccl &n = nccl();
    return fail(LLMDOT_E_NCCL, std::string(what) + ": " + (n.getErrorString ? n.getErrorString(r) : "error"));
}

}  // namespace

int tp_unique_id(void *out128)
{
    Nccl &n = nccl();
    if (!n.ok) return fail(LLMDOT_E_NCCL, n.why);
    NcclId id;
    const int r = n.getUniqueId(&id);
    if (r) return nccl_fail(r, "ncclGetUniqueId");
    memcpy(out128, &id, sizeof(id));
    return LLMDOT_OK;
}

int tp_comm_init(llmdot_model *m, const void *id128)
{
    Nccl &n = nccl();
    if (!n.ok) return fail(LLMDOT_E_NCCL, n.why);
    if (m->nccl) return fail(LLMDOT_E_INVALID, "tensor parallel: communicator already initialised");
    NcclId id;
    memcpy(&id, id128, sizeof(id));
    LLMDOT_CUDA_TRY(cudaSetDevice(m->device));
    NcclComm comm = nullptr;
    const int r = n.commInitRank(&comm, m->tp, id, m->tp_rank);
    if (r) return nccl_fail(r, "ncclCommInitRank");
    m->nccl = comm;
    return LLMDOT_OK;
}

void tp_comm_destroy(llmdot_model *m)
{
    if (!m->nccl) return;
    Nccl &n = nccl();
    if (n.ok) n.commDestroy((NcclComm)m->nccl);
    m->nccl = nullptr;
}

// ------------------------------------------------------------------ peer-memory all-reduce
// Exchange buffer of one rank (device memory, exported with CUDA IPC):
//   u32 [0]  sequence number of the last finished all-reduce (advanced by its last CTA)
//   u32 [1]  CTAs of the running all-reduce that finished
//   u32 [2]  set once a wait of this rank gave up (later waits give up at once)
//   u32 [3]  set by the close barrier when it gave up
//   u32 [16 + q]  set by rank q when it reached its close barrier
//   byte TPX_DATA: u64 slots [2 parities][tp source ranks][cap elements]
// One all-reduce, generation g = sequence + 1: every rank stores each element of its partial as a
// word (g << 32 | float bits) into every peer's slot [g & 1][own rank][element], then polls its own
// slots for the other ranks' words tagged g.  A 64-bit store is single-copy atomic, so the tag and
// the value arrive together and no flag or fence is needed.  Two parities make reuse safe: a rank
// starts generation g + 2 only after finishing g + 1, which needed every peer's g + 1 words, which
// each peer stores only after its generation g kernel (and all its reads of parity g & 1) ended.
namespace {

constexpr size_t TPX_DATA = 4096;
constexpr int TPX_THREADS = 256;
constexpr int TPX_MAX_CTAS = 148;  // at most one CTA per SM: every CTA resident, none waits on a queued one
constexpr unsigned long long TPX_WAIT_NS = 10ull * 1000 * 1000 * 1000;
constexpr unsigned long long TPX_CLOSE_NS = 5ull * 1000 * 1000 * 1000;
constexpr int TPX_ERR_TIMEOUT = 6;  // device error flag value the host maps to LLMDOT_E_TIMEOUT

struct TpxArgs {
    uint8_t *peer[TPX_MAX_RANKS];  // every rank's exchange buffer as mapped here (own included)
    uint8_t *own;
    float *buf;
    long long n, cap;
    int tp, rank;
    int *err;
};

__device__ __forceinline__ unsigned long long tpx_now()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void tpx_store2(uint8_t *p, unsigned long long a, unsigned long long b)
{
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ void tpx_load2(const uint8_t *p, unsigned long long &a, unsigned long long &b)
{
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Polls the four words at p until all carry tag gen; false (and the error flag) once the wait ran
// past its deadline or an earlier wait of this rank already gave up.
__device__ bool tpx_wait4(const uint8_t *p, unsigned gen, float4 &v, volatile unsigned *hdr, int *err)
{
    unsigned long long w0, w1, w2, w3, t0 = 0;
    for (unsigned it = 0;; it++) {
        tpx_load2(p, w0, w1);
        tpx_load2(p + 16, w2, w3);
        if ((unsigned)(w0 >> 32) == gen && (unsigned)(w1 >> 32) == gen && (unsigned)(w2 >> 32) == gen &&
            (unsigned)(w3 >> 32) == gen)
            break;
        if ((it & 255) == 0) {
            const unsigned long long t = tpx_now();
            if (it == 0) t0 = t;
            if (hdr[2] || t - t0 > TPX_WAIT_NS) {
                hdr[2] = 1;
                atomicCAS(err, 0, TPX_ERR_TIMEOUT);
                v = make_float4(0.f, 0.f, 0.f, 0.f);
                return false;
            }
        }
    }
    v = make_float4(__uint_as_float((unsigned)w0), __uint_as_float((unsigned)w1), __uint_as_float((unsigned)w2),
                    __uint_as_float((unsigned)w3));
    return true;
}

// Polls the two words at p until both carry tag gen; their low halves, or false as above.
__device__ bool tpx_wait2(const uint8_t *p, unsigned gen, unsigned &lo0, unsigned &lo1, volatile unsigned *hdr,
                          int *err)
{
    unsigned long long w0, w1, t0 = 0;
    for (unsigned it = 0;; it++) {
        tpx_load2(p, w0, w1);
        if ((unsigned)(w0 >> 32) == gen && (unsigned)(w1 >> 32) == gen) break;
        if ((it & 255) == 0) {
            const unsigned long long t = tpx_now();
            if (it == 0) t0 = t;
            if (hdr[2] || t - t0 > TPX_WAIT_NS) {
                hdr[2] = 1;
                atomicCAS(err, 0, TPX_ERR_TIMEOUT);
                lo0 = lo1 = 0;
                return false;
            }
        }
    }
    lo0 = (unsigned)w0;
    lo1 = (unsigned)w1;
    return true;
}

// The last CTA of an exchange to finish publishes its generation (every CTA read the old one
// before arriving).
__device__ __forceinline__ void tpx_finish(uint8_t *own, volatile unsigned *hdr, unsigned gen)
{
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd((unsigned *)(own + 4), 1u) == gridDim.x - 1) {
            hdr[1] = 0;
            hdr[0] = gen;
            __threadfence();
        }
    }
}

__device__ __forceinline__ unsigned long long tpx_word(unsigned gen, float x)
{
    return ((unsigned long long)gen << 32) | __float_as_uint(x);
}

__global__ void __launch_bounds__(TPX_THREADS) tpx_allreduce_kernel(TpxArgs a)
{
    volatile unsigned *hdr = (volatile unsigned *)a.own;
    const unsigned gen = hdr[0] + 1;
    const long long par = gen & 1;
    const long long stride = (long long)gridDim.x * TPX_THREADS * 4;
    const long long e0 = ((long long)blockIdx.x * TPX_THREADS + threadIdx.x) * 4;
    const size_t src_off = TPX_DATA + (size_t)((par * a.tp + a.rank) * a.cap) * 8;
    // push: this rank's partial into every peer's slot row [par][rank]
    for (long long e = e0; e < a.n; e += stride) {
        const float4 v = *(const float4 *)(a.buf + e);
        const unsigned long long w0 = tpx_word(gen, v.x), w1 = tpx_word(gen, v.y), w2 = tpx_word(gen, v.z),
                                 w3 = tpx_word(gen, v.w);
        for (int q = 0; q < a.tp; q++) {
            if (q == a.rank) continue;
            uint8_t *d = a.peer[q] + src_off + (size_t)e * 8;
            tpx_store2(d, w0, w1);
            tpx_store2(d + 16, w2, w3);
        }
    }
    // gather: every rank's partial, summed in rank order (the same order on every rank)
    for (long long e = e0; e < a.n; e += stride) {
        const float4 mine = *(const float4 *)(a.buf + e);
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < a.tp; q++) {
            float4 v = mine;
            if (q != a.rank)
                tpx_wait4(a.own + TPX_DATA + (size_t)((par * a.tp + q) * a.cap + e) * 8, gen, v, hdr, a.err);
            if (q == 0) {
                s = v;
            } else {
                s.x += v.x;
                s.y += v.y;
                s.z += v.z;
                s.w += v.w;
            }
        }
        *(float4 *)(a.buf + e) = s;
    }
    tpx_finish(a.own, hdr, gen);
}

// Max of n packed argmax keys (value key << 32 | ~index) across the ranks: one exchange of the
// same protocol, each key sent as two tagged words (high half, low half) in slot elements 2j, 2j+1.
__global__ void __launch_bounds__(TPX_THREADS) tpx_allmax_u64_kernel(TpxArgs a, unsigned long long *keys, int n)
{
    volatile unsigned *hdr = (volatile unsigned *)a.own;
    const unsigned gen = hdr[0] + 1;
    const long long par = gen & 1;
    const int j = blockIdx.x * TPX_THREADS + threadIdx.x;
    if (j < n) {
        const unsigned long long k = keys[j];
        const unsigned long long w0 = ((unsigned long long)gen << 32) | (unsigned)(k >> 32),
                                 w1 = ((unsigned long long)gen << 32) | (unsigned)k;
        const size_t src_off = TPX_DATA + (size_t)((par * a.tp + a.rank) * a.cap + 2 * (long long)j) * 8;
        for (int q = 0; q < a.tp; q++)
            if (q != a.rank) tpx_store2(a.peer[q] + src_off, w0, w1);
        unsigned long long best = k;
        for (int q = 0; q < a.tp; q++) {
            if (q == a.rank) continue;
            unsigned hi, lo;
            tpx_wait2(a.own + TPX_DATA + (size_t)((par * a.tp + q) * a.cap + 2 * (long long)j) * 8, gen, hi, lo, hdr,
                      a.err);
            const unsigned long long kq = ((unsigned long long)hi << 32) | lo;
            best = kq > best ? kq : best;
        }
        keys[j] = best;
    }
    tpx_finish(a.own, hdr, gen);
}

// Close barrier: every rank marks its arrival in every peer's header and waits (bounded) for the
// others' marks, so that no rank frees its buffer while a peer may still store into it.
__global__ void tpx_close_kernel(TpxArgs a)
{
    volatile unsigned *hdr = (volatile unsigned *)a.own;
    const int q = threadIdx.x;
    if (q < a.tp && q != a.rank) {
        volatile unsigned *peer_hdr = (volatile unsigned *)a.peer[q];
        peer_hdr[16 + a.rank] = 1;
        __threadfence_system();
        const unsigned long long t0 = tpx_now();
        while (hdr[16 + q] == 0) {
            if (tpx_now() - t0 > TPX_CLOSE_NS) {
                hdr[3] = 1;
                break;
            }
        }
    }
}

TpxArgs tpx_args(llmdot_model *m, float *buf, long long n)
{
    TpxArgs a{};
    for (int q = 0; q < m->tp && q < TPX_MAX_RANKS; q++) a.peer[q] = m->tpx_peer[q];
    a.own = m->tpx;
    a.buf = buf;
    a.n = n;
    a.cap = (long long)m->tpx_cap;
    a.tp = m->tp;
    a.rank = m->tp_rank;
    a.err = m->ws.err;
    return a;
}

}  // namespace

int tp_exchange_handle(llmdot_model *m, void *out128)
{
    if (m->tp < 2 || m->tp > TPX_MAX_RANKS)
        return fail(LLMDOT_E_UNSUPPORTED, "peer all-reduce: needs 2 to 8 tensor-parallel ranks");
    if (m->tpx_open) return fail(LLMDOT_E_INVALID, "peer all-reduce: already open");
    LLMDOT_CUDA_TRY(cudaSetDevice(m->device));
    if (!m->tpx) {
        // the step's residual sums of up to 64 rows of the hidden state
        const size_t cap = (size_t)64 * ((m->cfg.hidden + 3) / 4 * 4);
        const size_t bytes = TPX_DATA + 2 * (size_t)m->tp * cap * 8;
        LLMDOT_CUDA_TRY(cudaMalloc((void **)&m->tpx, bytes));
        LLMDOT_CUDA_TRY(cudaMemset(m->tpx, 0, bytes));
        LLMDOT_CUDA_TRY(cudaDeviceSynchronize());
        m->tpx_cap = cap;
    }
    cudaIpcMemHandle_t h;
    LLMDOT_CUDA_TRY(cudaIpcGetMemHandle(&h, m->tpx));
    cudaDeviceProp prop;
    LLMDOT_CUDA_TRY(cudaGetDeviceProperties(&prop, m->device));
    static_assert(sizeof(h) + sizeof(prop.uuid) <= TPX_HANDLE_BYTES, "handle layout");
    memset(out128, 0, TPX_HANDLE_BYTES);
    memcpy(out128, &h, sizeof(h));
    memcpy((uint8_t *)out128 + 64, &prop.uuid, sizeof(prop.uuid));
    return LLMDOT_OK;
}

int tp_exchange_open(llmdot_model *m, const void *handles)
{
    if (!m->tpx) return fail(LLMDOT_E_INVALID, "peer all-reduce: call tp_exchange_handle first");
    if (m->tpx_open) return fail(LLMDOT_E_INVALID, "peer all-reduce: already open");
    const uint8_t *hb = (const uint8_t *)handles;
    LLMDOT_CUDA_TRY(cudaSetDevice(m->device));
    cudaDeviceProp prop;
    LLMDOT_CUDA_TRY(cudaGetDeviceProperties(&prop, m->device));
    if (memcmp(hb + (size_t)m->tp_rank * TPX_HANDLE_BYTES + 64, &prop.uuid, sizeof(prop.uuid)))
        return fail(LLMDOT_E_INVALID, "peer all-reduce: this rank's handle is not at its rank's position");
    // ranks that wait on one another must not share a GPU (nothing makes their kernels co-resident)
    for (int p = 0; p < m->tp; p++)
        for (int q = p + 1; q < m->tp; q++)
            if (!memcmp(hb + (size_t)p * TPX_HANDLE_BYTES + 64, hb + (size_t)q * TPX_HANDLE_BYTES + 64, 16))
                return fail(LLMDOT_E_UNSUPPORTED, "peer all-reduce: two ranks share one GPU");
    uint8_t *peer[TPX_MAX_RANKS] = {};
    for (int q = 0; q < m->tp; q++) {
        if (q == m->tp_rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + (size_t)q * TPX_HANDLE_BYTES, sizeof(h));
        void *p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int r = 0; r < q; r++)
                if (peer[r]) cudaIpcCloseMemHandle(peer[r]);
            return fail(LLMDOT_E_CUDA, std::string("peer all-reduce: cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
        }
        peer[q] = (uint8_t *)p;
    }
    peer[m->tp_rank] = m->tpx;
    for (int q = 0; q < TPX_MAX_RANKS; q++) m->tpx_peer[q] = peer[q];
    m->tpx_open = m->tpx_use = true;
    return LLMDOT_OK;
}

int tp_exchange_use(llmdot_model *m, bool on)
{
    if (on && !m->tpx_open) return fail(LLMDOT_E_INVALID, "peer all-reduce: not open");
    m->tpx_use = on;
    return LLMDOT_OK;
}

void tp_exchange_close(llmdot_model *m)
{
    if (!m->tpx) return;
    cudaSetDevice(m->device);
    bool safe = false;  // whether no peer can store into this rank's buffer any more
    if (m->tpx_open) {
        TpxArgs a = tpx_args(m, nullptr, 0);
        tpx_close_kernel<<<1, 32, 0, m->stream>>>(a);
        unsigned gave_up = 1;
        if (cudaGetLastError() == cudaSuccess && cudaStreamSynchronize(m->stream) == cudaSuccess &&
            cudaMemcpy(&gave_up, m->tpx + 12, sizeof(gave_up), cudaMemcpyDeviceToHost) == cudaSuccess)
            safe = gave_up == 0;
        for (int q = 0; q < m->tp && q < TPX_MAX_RANKS; q++)
            if (q != m->tp_rank && m->tpx_peer[q]) cudaIpcCloseMemHandle(m->tpx_peer[q]);
    }
    // A buffer whose handle went out but whose close barrier did not complete stays allocated: a
    // peer that opened it may still store into it.
    if (safe) cudaFree(m->tpx);
    m->tpx = nullptr;
    for (int q = 0; q < TPX_MAX_RANKS; q++) m->tpx_peer[q] = nullptr;
    m->tpx_cap = 0;
    m->tpx_open = m->tpx_use = false;
}

int tp_allreduce_sum(llmdot_model *m, float *buf, size_t n, cudaStream_t st)
{
    if (!m->nccl) return fail(LLMDOT_E_INVALID, "tensor parallel: call llmdot_cuda_tp_init first");
    if (m->tpx_use && n <= m->tpx_cap && n % 4 == 0 && ((uintptr_t)buf & 15) == 0) {
        const long long G = std::min<long long>(TPX_MAX_CTAS, ((long long)n + TPX_THREADS * 4 - 1) / (TPX_THREADS * 4));
        if (n == 0) return LLMDOT_OK;
        tpx_allreduce_kernel<<<(unsigned)G, TPX_THREADS, 0, st>>>(tpx_args(m, buf, (long long)n));
        LLMDOT_CUDA_TRY(cudaGetLastError());
        return LLMDOT_OK;
    }
    const int r = nccl().allReduce(buf, buf, n, NCCL_FLOAT, NCCL_SUM, (NcclComm)m->nccl, st);
    return r ? nccl_fail(r, "ncclAllReduce") : LLMDOT_OK;
}

int tp_allreduce_max_u64(llmdot_model *m, unsigned long long *buf, size_t n, cudaStream_t st)
{
    if (!m->nccl) return fail(LLMDOT_E_INVALID, "tensor parallel: call llmdot_cuda_tp_init first");
    // one key per thread, at most one CTA per SM (every CTA resident, as for the sums)
    if (m->tpx_use && 2 * n <= m->tpx_cap && n <= (size_t)TPX_MAX_CTAS * TPX_THREADS) {
        if (n == 0) return LLMDOT_OK;
        const unsigned G = (unsigned)((n + TPX_THREADS - 1) / TPX_THREADS);
        tpx_allmax_u64_kernel<<<G, TPX_THREADS, 0, st>>>(tpx_args(m, nullptr, 0), buf, (int)n);
        LLMDOT_CUDA_TRY(cudaGetLastError());
        return LLMDOT_OK;
    }
    const int r = nccl().allReduce(buf, buf, n, NCCL_UINT64, NCCL_MAX, (NcclComm)m->nccl, st);
    return r ? nccl_fail(r, "ncclAllReduce") : LLMDOT_OK;
}

int tp_allgather(llmdot_model *m, const float *send, float *recv, size_t n, cudaStream_t st)
{
    if (!m->nccl) return fail(LLMDOT_E_INVALID, "tensor parallel: call llmdot_cuda_tp_init first");
    const int r = nccl().allGather(send, recv, n, NCCL_FLOAT, (NcclComm)m->nccl, st);
    return r ? nccl_fail(r, "ncclAllGather") : LLMDOT_OK;
}

}  // namespace llmdot
