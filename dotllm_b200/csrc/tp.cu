// tp.cu -- tensor-parallel shard geometry and NCCL collectives (NCCL loaded at run time).
#include <dlfcn.h>
#include <string.h>

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

int tp_allreduce_sum(llmdot_model *m, float *buf, size_t n, cudaStream_t st)
{
    if (!m->nccl) return fail(LLMDOT_E_INVALID, "tensor parallel: call llmdot_cuda_tp_init first");
    const int r = nccl().allReduce(buf, buf, n, NCCL_FLOAT, NCCL_SUM, (NcclComm)m->nccl, st);
    return r ? nccl_fail(r, "ncclAllReduce") : LLMDOT_OK;
}

int tp_allreduce_max_u64(llmdot_model *m, unsigned long long *buf, size_t n, cudaStream_t st)
{
    if (!m->nccl) return fail(LLMDOT_E_INVALID, "tensor parallel: call llmdot_cuda_tp_init first");
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
