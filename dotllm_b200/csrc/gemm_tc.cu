// gemm_tc.cu -- quantised matmul for 2..32 input rows on the 5th-generation tensor cores:
// batched decode steps (several sessions) and prompt chunks (consecutive tokens of one session).
//
// Same contract as the matvec (TensorOps.MatMulFusedQ4_K / Q6_K, src/Llmdot.Core/Tensors/TensorOps.cs:230-395,
// several input rows as in TensorOps.MatMul's aRows > 1 branch, TensorOps.cs:92-111):
// y[v][row] = sum_k x[v][k] * W[row][k], fp32 result.
//
// Arithmetic (exact products, fp32 sums, as in the matvec):
// * x is scaled per input row by a power of two and split into fp16 hi + lo: MMA column v holds
//   x_hi, column 32 + v holds x_lo (N = 64).
// * Q4_K: the A operand is q * sc (integers <= 945, exact in fp16), one accumulator per super-block,
//   read back from TMEM and scaled by the row's d on the CUDA cores; the offset term
//   sum_j (8 d sc_j + dmin m_j) * S_j (S_j = sub-block sums of x) is one more MMA per super-block
//   (coefficients and sums as fp16 hi/lo pairs) into a second accumulator that spans the whole K.
// * Q6_K: the A operand sc * (q - 32) (|.| <= 4096) is split into an fp16 hi (rounded) and its exact
//   residual lo (0 or +-1), two MMAs per K step; d applied per super-block as for Q4_K.
//
// Kernel structure (one CTA of 16 warps per SM, persistent over a contiguous range of work units;
// a unit is one 128-row tile x one 256-weight super-block):
//   warp 0        producer: one cp.async.bulk of the prepared B operand per super-block into a
//                 3-slot ring;
//   warp 1        TMEM allocator and MMA issuer (one thread): tcgen05.mma.cta_group::1.kind::f16,
//                 M = 128, N = 64, K = 16, A from TMEM, B from shared memory (no-swizzle K-major core
//                 matrices), commits to mbarriers;
//   warps 4-7     epilogue: tcgen05.ld of the accumulators (one TMEM lane = one weight row per
//                 thread), d scaling, output or K-split partial;
//   warps 8-15    dequantisation: raw tile bytes (shared memory, streamed by these warps with
//                 bulk copies) -> fp16 A operand written straight into TMEM (tcgen05.st, one thread
//                 per weight row), which the MMA reads from there.
// The A operand lives in TMEM in three quarter super-block (K = 64) stages; three raw super-blocks and
// three B super-blocks are in flight; accumulators are double-buffered in TMEM.  A
// 128-row tile whose super-blocks are split between CTAs is finished by the last CTA to arrive,
// which adds the partials in CTA order (deterministic).  Every wait is bounded (%globaltimer).
#include "engine.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"
#include "gemv_tile.cuh"

namespace llmdot {

namespace {

constexpr int TC_THREADS = 512;
constexpr int TM = 128, TN = 64, QK = 64;           // tile rows, MMA N, K per pipeline stage (quarter super-block)
constexpr uint32_t B_BYTES = TN * QK * 2;           // 8192: B operand of a quarter super-block
constexpr int NSTAGE = 3;                           // A operand stages in TMEM (quarter super-blocks)
constexpr int NB = 3;                               // B operand slots (whole super-blocks) in shared memory
constexpr int NRAW = 3;                             // raw super-block slots (units in flight)
constexpr uint32_t RAW_SLOT = 8 * Q6K_TILE;         // eight 16-row tiles of one super-block
constexpr uint32_t AM_BYTES = TM * 16 * 2;          // Q4_K offset-term A operand (K = 16)
constexpr uint32_t BM_BYTES = TN * 16 * 2;
constexpr uint32_t B4_SB = 4 * B_BYTES + BM_BYTES;  // prepared B per super-block, Q4_K layout
constexpr uint32_t B6_SB = 4 * B_BYTES;             // Q6_K layout
constexpr uint32_t OFF_B = 0;
constexpr uint32_t OFF_RAW = OFF_B + NB * B4_SB;
constexpr uint32_t OFF_AM = OFF_RAW + NRAW * RAW_SLOT;
constexpr uint32_t OFF_DSM = OFF_AM + 2 * AM_BYTES;
constexpr uint32_t OFF_BAR = OFF_DSM + 2 * TM * 4;
constexpr int NBAR = 72;
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
constexpr uint32_t SMEM_BYTES = OFF_MISC + 64;
static_assert(SMEM_BYTES <= 227 * 1024, "tensor-core matmul: shared memory");
// TMEM columns: accumulators 0..63 and 64..127 (one per super-block in flight), the Q4_K offset
// term 128..191, then NSTAGE A stages of 64 columns (32 for fp16 A of K = 64, 32 for the Q6_K lo part)
constexpr int TMEM_COLS = 512;
constexpr uint32_t A_COL = 192;
constexpr float S_FAC = 1.0f / 64.0f;  // sub-block sums (< 2^20) scaled into fp16 range
constexpr float C_FAC = 256.0f;        // offset coefficients scaled up (their lo half stays normal)
constexpr unsigned long long TC_WAIT_NS = 2000000000ull;
constexpr int TC_DEFAULT_REPLICAS = 1;

enum {
    B_B_FULL = 0, B_B_EMPTY = B_B_FULL + NB, B_RAW_FULL = B_B_EMPTY + NB, B_RAW_EMPTY = B_RAW_FULL + 8 * NRAW,
    B_A_FULL = B_RAW_EMPTY + 8 * NRAW, B_ST_EMPTY = B_A_FULL + NSTAGE, B_ACC_FULL = B_ST_EMPTY + NSTAGE,
    B_ACC_EMPTY = B_ACC_FULL + 2, B_ACCM_EMPTY = B_ACC_EMPTY + 2, B_DRAIN = B_ACCM_EMPTY + 1, B_COUNT = B_DRAIN + 1
};
static_assert(B_COUNT <= NBAR, "tensor-core matmul: barrier slots");

struct TcArgs {
    const uint8_t *w[3];
    float *y[3];
    int ldy[3], rows[3], qt[3], nrt16[3], cum[4];  // cum: first 128-row tile of each segment
    int nseg, nsb, U, nv, mode;
    const uint8_t *b4, *b6;
    size_t b4s, b6s;  // bytes between the replicas of the prepared operands
    int reps;         // replicas: CTA c reads replica c % reps (spreads the hot lines over L2)
    const float *isc;
    float *part;
    int *cnt;
    int *err;
    GemvPrefetch pf;  // weights of the next operation, pulled into L2 while this one runs
};

__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t gtime()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void bar_init(uint64_t *b, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t *b)
{
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t *b, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void cp16(void *dst, const void *src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(su32(dst)), "l"(src) : "memory");
}
// arrives on b once every cp.async this thread issued so far has landed (no pending-count change)
__device__ __forceinline__ void cp_arrive(uint64_t *b)
{
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(su32(b)) : "memory");
}
// shared-memory matrix descriptor: no swizzle, K-major core matrices of 8 rows x 16 bytes; lbo =
// byte distance of K-adjacent core matrices, sbo = of 8-row groups; bit 46 = descriptor version 1
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo)
{
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// kind::f16 instruction descriptor: fp32 accumulator, fp16 A and B, both K-major, N = 64, M = 128
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(TN >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t acc)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(da), "l"(db), "r"(IDESC), "r"(acc)
        : "memory");
}
// A operand from TMEM: row m in lane m, K element k in column k/2 (low half for even k)
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t db, uint32_t acc)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(db), "r"(IDESC), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *b)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 64 consecutive fp32 TMEM columns of this thread's lane
__device__ __forceinline__ void tmem_ld64(uint32_t ta, float (&f)[64])
{
    uint32_t v[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,"
        "%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]), "=r"(v[32]),
          "=r"(v[33]), "=r"(v[34]), "=r"(v[35]), "=r"(v[36]), "=r"(v[37]), "=r"(v[38]), "=r"(v[39]), "=r"(v[40]),
          "=r"(v[41]), "=r"(v[42]), "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]), "=r"(v[48]),
          "=r"(v[49]), "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]), "=r"(v[55]), "=r"(v[56]),
          "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63])
        : "r"(ta));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 64; i++) f[i] = __uint_as_float(v[i]);
}

// 16 consecutive 32-bit TMEM columns of this thread's lane
__device__ __forceinline__ void tmem_st16(uint32_t ta, const uint32_t (&v)[16])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(ta),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

__device__ __forceinline__ uint32_t half2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

// The CTA whose unit range holds unit u (ranges [c U / G, (c + 1) U / G)).
__device__ __forceinline__ int cta_of(long long u, int U, int G) { return (int)(((u + 1) * G + U - 1) / U) - 1; }

struct Unit {
    int seg, rt, gt, sb, qt;
    bool first, last;
};

__device__ __forceinline__ void l2_prefetch(const void *src, uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__global__ void __launch_bounds__(TC_THREADS, 1) tc_gemm_kernel(const __grid_constant__ TcArgs a)
{
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, c = blockIdx.x;
    const int u0 = (int)((long long)c * a.U / G), u1 = (int)((long long)(c + 1) * a.U / G), n = u1 - u0;
    uint64_t *bars = (uint64_t *)(smem + OFF_BAR);
    uint32_t *tmem_slot = (uint32_t *)(smem + OFF_MISC);
    volatile int *abort_f = (volatile int *)(smem + OFF_MISC + 4);
    volatile int *last_f = (volatile int *)(smem + OFF_MISC + 8);
    float *dsm = (float *)(smem + OFF_DSM);
    const int nsb = a.nsb;

    auto unit = [&](int i) {
        Unit U;
        const int u = u0 + i;
        U.gt = u / nsb;
        U.sb = u % nsb;
        int s = 0;
        while (s + 1 < a.nseg && U.gt >= a.cum[s + 1]) s++;
        U.seg = s;
        U.rt = U.gt - a.cum[s];
        U.qt = a.qt[s];
        U.first = i == 0 || U.sb == 0;
        U.last = i == n - 1 || U.sb == nsb - 1;
        return U;
    };
    // bounded wait; gives up on another role's abort as well
    auto wait = [&](int bi, uint32_t parity) -> bool {
        uint64_t *b = bars + bi;
        if (bar_try(b, parity)) return true;
        const uint64_t t0 = gtime();
        while (!bar_try(b, parity)) {
            if (*abort_f || gtime() - t0 > TC_WAIT_NS) {
                if (!*abort_f) {
                    *abort_f = 1;
                    atomicExch(a.err, 5);
                }
                return false;
            }
        }
        return true;
    };

    if (tid == 0) {
        for (int i = 0; i < B_COUNT; i++) {
            uint32_t cnt = 1;
            if (i >= B_B_FULL && i < B_B_FULL + NB) cnt = 64;            // the B loader threads
            if (i >= B_RAW_FULL && i < B_RAW_FULL + 8 * NRAW) cnt = 32;  // the copying warp's lanes
            if (i >= B_RAW_EMPTY && i < B_RAW_EMPTY + 8 * NRAW) cnt = 2;  // the two warps reading a tile
            if (i >= B_A_FULL && i < B_A_FULL + NSTAGE) cnt = 8;         // the dequantisation warps
            if (i == B_ACC_EMPTY || i == B_ACC_EMPTY + 1 || i == B_ACCM_EMPTY) cnt = 4;
            bar_init(bars + i, cnt);
        }
        *abort_f = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- producer: B operands
        if (lane == 0 && n > 0) {
            // this CTA's share of the next operation's weights into L2
#pragma unroll
            for (int r = 0; r < GEMV_PREFETCH_MAX; r++) {
                const unsigned long long nb = a.pf.n[r];
                if (!a.pf.p[r] || nb == 0) continue;
                const unsigned long long share = (nb / G + 15) & ~15ull, lo = (unsigned long long)c * share;
                if (lo >= nb) continue;
                unsigned long long len = nb - lo < share ? nb - lo : share;
                const uint8_t *src = (const uint8_t *)a.pf.p[r] + lo;
                while (len > 0) {
                    const uint32_t piece = len > (1u << 20) ? (1u << 20) : (uint32_t)len;
                    l2_prefetch(src, piece);
                    src += piece;
                    len -= piece;
                }
            }
        }
    } else if (warp == 2 || warp == 3) {
        // ---------------------------------------------------------------- B loader (64 threads)
        // cp.async 16-byte pieces of the prepared B of each super-block into a 3-slot ring; a unit's
        // slot is signalled once its copies have landed and are made visible to the tensor core
        const int lt = tid - 64;
        auto issue_b = [&](int k) {
            const Unit U = unit(k);
            const bool q4 = U.qt == QT_Q4K;
            const int rr = c % a.reps;
            const uint32_t bytes = q4 ? B4_SB : B6_SB;
            const uint8_t *src = q4 ? a.b4 + rr * a.b4s + (size_t)U.sb * B4_SB : a.b6 + rr * a.b6s + (size_t)U.sb * B6_SB;
            uint8_t *dst = smem + OFF_B + (k % NB) * B4_SB;
            for (uint32_t o = (uint32_t)lt * 16; o < bytes; o += 64 * 16) cp16(dst + o, src + o);
            asm volatile("cp.async.commit_group;" ::: "memory");
        };
        int issued = 0;
        for (; issued < NB && issued < n; issued++) issue_b(issued);
        // unit k is signalled as soon as its copies land; the slot of unit k - 1 is refilled with unit
        // k - 1 + NB once the tensor core is done with it, so signalling never waits on the MMA
        for (int k = 0; k < n; k++) {
            const int pend = issued - k - 1;  // copy groups issued after unit k's
            if (pend >= 2) asm volatile("cp.async.wait_group 2;" ::: "memory");
            else if (pend == 1) asm volatile("cp.async.wait_group 1;" ::: "memory");
            else asm volatile("cp.async.wait_group 0;" ::: "memory");
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy writes -> tensor core
            bar_arrive(bars + B_B_FULL + k % NB);
            if (k >= 1 && issued < n) {
                if (!wait(B_B_EMPTY + (k - 1) % NB, ((k - 1) / NB) & 1)) break;
                issue_b(issued++);
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");  // no copy may land after the CTA exits
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0 && n > 0) {
            int run = 0;
            bool ok = true;
            for (int i = 0; i < n && ok; i++) {
                const Unit U = unit(i);
                const bool q4 = U.qt == QT_Q4K;
                const int b = i & 1, bs = i % NB;
                if (i >= 2 && !(ok = wait(B_ACC_EMPTY + b, ((i - 2) >> 1) & 1))) break;
                if (!(ok = wait(B_B_FULL + bs, (i / NB) & 1))) break;
                const uint32_t Bsm = su32(smem + OFF_B + bs * B4_SB);
                for (int qt = 0; qt < 4 && ok; qt++) {
                    const int Q = 4 * i + qt, st = Q % NSTAGE;
                    if (!(ok = wait(B_A_FULL + st, (Q / NSTAGE) & 1))) break;
                    tc_fence_after();
                    const uint32_t A = tmem + A_COL + st * 64;
#pragma unroll
                    for (int kk = 0; kk < QK / 16; kk++) {
                        const uint64_t db = sdesc(Bsm + qt * B_BYTES + kk * 256, 128, 1024);
                        umma_ts(tmem + b * 64, A + kk * 8, db, (qt | kk) != 0);
                        if (!q4) umma_ts(tmem + b * 64, A + 32 + kk * 8, db, 1u);
                    }
                    if (q4 && qt == 3) {
                        if (U.first && run >= 1 && !(ok = wait(B_ACCM_EMPTY, (run - 1) & 1))) break;
                        tc_fence_after();
                        umma(tmem + 128, sdesc(su32(smem + OFF_AM + b * AM_BYTES), 128, 256),
                             sdesc(Bsm + 4 * B_BYTES, 128, 256), U.first ? 0u : 1u);
                    }
                    umma_commit(bars + B_ST_EMPTY + st);
                }
                if (!ok) break;
                umma_commit(bars + B_B_EMPTY + bs);
                umma_commit(bars + B_ACC_FULL + b);
                if (U.last) run++;
            }
            // every MMA issued so far completes before the TMEM is released
            umma_commit(bars + B_DRAIN);
            const uint64_t t0 = gtime();
            while (!bar_try(bars + B_DRAIN, 0) && gtime() - t0 < TC_WAIT_NS) {}
        }
    } else if (warp >= 4 && warp < 8) {
        // ---------------------------------------------------------------- epilogue
        const int e = warp - 4, row = 32 * e + lane, te = tid - 128;
        float acc[TC_MAX_ROWS];
#pragma unroll
        for (int t = 0; t < TC_MAX_ROWS; t++) acc[t] = 0.0f;
        int run = 0, run_sb0 = 0;
        for (int i = 0; i < n; i++) {
            const Unit U = unit(i);
            const int b = i & 1;
            if (U.first) run_sb0 = U.sb;
            if (!wait(B_ACC_FULL + b, (i >> 1) & 1)) break;
            tc_fence_after();
            float v[64];
            tmem_ld64(tmem + ((uint32_t)(32 * e) << 16) + b * 64, v);
            const float d = dsm[b * TM + row];
#pragma unroll
            for (int t = 0; t < TC_MAX_ROWS; t++) acc[t] = fmaf(d, v[t] + v[t + 32], acc[t]);
            if (U.last && U.qt == QT_Q4K) {
                tmem_ld64(tmem + ((uint32_t)(32 * e) << 16) + 128, v);
#pragma unroll
                for (int t = 0; t < TC_MAX_ROWS; t++) acc[t] -= (v[t] + v[t + 32]) * (1.0f / (C_FAC * S_FAC));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                bar_arrive(bars + B_ACC_EMPTY + b);
                if (U.last) bar_arrive(bars + B_ACCM_EMPTY);
            }
            if (!U.last) continue;
            // ---- a 128-row tile (or this CTA's share of its super-blocks) is complete
            const int s = U.seg, rowg = 128 * U.rt + row;
            const bool whole = run_sb0 == 0 && U.sb == nsb - 1;
            float *y = a.y[s];
            if (whole) {
                if (rowg < a.rows[s])
#pragma unroll
                    for (int t = 0; t < TC_MAX_ROWS; t++) {
                        if (t >= a.nv) break;
                        const float val = acc[t] * __ldg(a.isc + t);
                        float *yp = y + (size_t)t * a.ldy[s] + rowg;
                        *yp = a.mode == GEMV_ADD ? __fadd_rn(*yp, val) : val;
                    }
            } else {
                float *pp = a.part + ((size_t)(c * 2 + (run == 0 ? 0 : 1)) * TC_MAX_ROWS) * TM;
#pragma unroll
                for (int t = 0; t < TC_MAX_ROWS; t++) pp[t * TM + row] = acc[t];
                __threadfence();
                asm volatile("bar.sync 1, 128;" ::: "memory");
                const long long ub = (long long)U.gt * nsb;
                const int c_lo = cta_of(ub, a.U, G), c_hi = cta_of(ub + nsb - 1, a.U, G);
                if (te == 0) {
                    const int old = atomicAdd(a.cnt + U.gt, 1);
                    *last_f = old == c_hi - c_lo;
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
                if (*last_f) {
                    __threadfence();
                    float tot[TC_MAX_ROWS];
#pragma unroll
                    for (int t = 0; t < TC_MAX_ROWS; t++) tot[t] = 0.0f;
                    for (int cc = c_lo; cc <= c_hi; cc++) {
                        const int first_gt = (int)((long long)cc * a.U / G) / nsb;
                        const float *qp = a.part + ((size_t)(cc * 2 + (first_gt == U.gt ? 0 : 1)) * TC_MAX_ROWS) * TM;
#pragma unroll
                        for (int t = 0; t < TC_MAX_ROWS; t++) tot[t] += __ldcg(qp + t * TM + row);
                    }
                    if (rowg < a.rows[s])
#pragma unroll
                        for (int t = 0; t < TC_MAX_ROWS; t++) {
                            if (t >= a.nv) break;
                            const float val = tot[t] * __ldg(a.isc + t);
                            float *yp = y + (size_t)t * a.ldy[s] + rowg;
                            *yp = a.mode == GEMV_ADD ? __fadd_rn(*yp, val) : val;
                        }
                    if (te == 0) a.cnt[U.gt] = 0;
                }
                asm volatile("bar.sync 1, 128;" ::: "memory");
            }
#pragma unroll
            for (int t = 0; t < TC_MAX_ROWS; t++) acc[t] = 0.0f;
            run++;
        }
    } else if (warp >= 8) {
        // ---------------------------------------------------------------- dequantisation
        // warp 8 + 4 kh + lq: TMEM lanes (weight rows) 32 lq .. 32 lq + 31, K half kh of each quarter
        // super-block; one thread per row writes its A columns with tcgen05.st.  Warp 8 + r also
        // streams raw 16-row tile r of every unit into the ring; tile r is read by the two warps of
        // lane quarter r / 2.
        const int dw = warp - 8, lq = dw & 3, kh = dw >> 2, row = 32 * lq + lane;
        const int rt8 = row >> 4, r16 = row & 15, g = r16 & 7, h = r16 >> 3;
        const int my_tile = dw;  // the tile this warp copies
        auto issue_tile = [&](int k) {  // cp.async by all 32 lanes; each lane arrives when its pieces land
            const Unit V = unit(k);
            const uint32_t tb = V.qt == QT_Q4K ? Q4K_TILE : Q6K_TILE;
            if (8 * V.rt + my_tile < a.nrt16[V.seg]) {  // else no such rows: the lanes only arrive
                uint8_t *dst = smem + OFF_RAW + (k % NRAW) * RAW_SLOT + my_tile * tb;
                const uint8_t *src = a.w[V.seg] + ((size_t)(8 * V.rt + my_tile) * nsb + V.sb) * tb;
                for (uint32_t o = (uint32_t)lane * 16; o < tb; o += 32 * 16) cp16(dst + o, src + o);
            }
            cp_arrive(bars + B_RAW_FULL + (k % NRAW) * 8 + my_tile);
        };
        for (int k = 0; k < NRAW && k < n; k++) issue_tile(k);
        bool ok = true;
        for (int i = 0; i < n && ok; i++) {
            const Unit U = unit(i);
            const int b = i & 1, slot = i % NRAW;
            const bool q4 = U.qt == QT_Q4K;
            if (!(ok = wait(B_RAW_FULL + slot * 8 + rt8, (i / NRAW) & 1))) break;
            if (i >= 2 && !(ok = wait(B_ACC_EMPTY + b, ((i - 2) >> 1) & 1))) break;
            const uint8_t *tile = smem + OFF_RAW + slot * RAW_SLOT + rt8 * (q4 ? Q4K_TILE : Q6K_TILE);
            uint4 hd = make_uint4(0, 0, 0, 0);
            if (q4) {
                hd = *(const uint4 *)(tile + 2048 + g * 32 + h * 16);
                if (kh == 0) dsm[b * TM + row] = half_bits(hd.x & 0xFFFF);
            } else if (kh == 0) {
                dsm[b * TM + row] = half_bits(*(const uint16_t *)(tile + 3328 + g * 4 + h * 2));
            }
            for (int qt = 0; qt < 4; qt++) {
                const int Q = 4 * i + qt, st = Q % NSTAGE;
                if (Q >= NSTAGE && !(ok = wait(B_ST_EMPTY + st, (Q / NSTAGE - 1) & 1))) break;
                tc_fence_after();
                const uint32_t ta = tmem + ((uint32_t)(32 * lq) << 16) + A_COL + st * 64 + kh * 16;
                if (q4) {
                    // sub-block j = 2 qt + kh of this row: 32 weights q * sc as 16 columns of fp16 pairs
                    const int j = 2 * qt + kh;
                    const uint4 W = *(const uint4 *)(tile + ((j & 1) + 2 * h) * 512 + (4 * g + (j >> 1)) * 16);
                    const int bit = 12 * j, wi = bit >> 5;
                    const uint32_t lo = wi == 0 ? hd.y : (wi == 1 ? hd.z : hd.w);
                    const uint32_t hi = wi == 0 ? hd.z : hd.w;
                    const uint32_t pr = __funnelshift_r(lo, hi, bit & 31);
                    const uint32_t sc = pr & 63u, mm = (pr >> 6) & 63u;
                    const uint32_t sc2 = hsub2(0x64006400u | (sc * 0x10001u), 0x64006400u);
                    const uint32_t nsc2 = hfma2(sc2, 0xE400E400u, 0u);   // * -1024
                    const uint32_t sc16 = hfma2(sc2, 0x2C002C00u, 0u);   // * 1/16
                    const uint32_t nsc16 = hfma2(sc2, 0xD400D400u, 0u);  // * -64
                    const uint32_t Ws[4] = {W.x, W.y, W.z, W.w};
                    uint32_t o[16];
#pragma unroll
                    for (int i4 = 0; i4 < 4; i4++) {
                        const uint32_t w = Ws[i4], w8 = w >> 8;
                        o[4 * i4 + 0] = hfma2(and_or(w, 0x000F000Fu, 0x64006400u), sc2, nsc2);
                        o[4 * i4 + 1] = hfma2(and_or(w, 0x00F000F0u, 0x64006400u), sc16, nsc16);
                        o[4 * i4 + 2] = hfma2(and_or(w8, 0x000F000Fu, 0x64006400u), sc2, nsc2);
                        o[4 * i4 + 3] = hfma2(and_or(w8, 0x00F000F0u, 0x64006400u), sc16, nsc16);
                    }
                    tmem_st16(ta, o);
                    // offset coefficient of sub-block j as an fp16 hi/lo pair (K = 2j, 2j + 1)
                    const float dd = half_bits(hd.x & 0xFFFF), dm = half_bits(hd.x >> 16);
                    const float cf = fmaf(8.0f * dd, (float)sc, dm * (float)mm) * C_FAC;
                    const __half chh = __float2half_rn(cf);
                    const __half2 pair = __halves2half2(chh, __float2half_rn(cf - __half2float(chh)));
                    *(uint32_t *)(smem + OFF_AM + b * AM_BYTES + (row >> 3) * 256 + (j >> 2) * 128 + (row & 7) * 16 +
                                  (j & 3) * 4) = half2_bits(pair);
                } else {
                    // group w = 2 qt + kh (sub-blocks 2w, 2w + 1) of this row: the four tile lanes
                    // t = 0..3 each hold its 4-element pieces; sc * (q - 32) as fp16 hi + exact lo
                    const int w = 2 * qt + kh;
                    const uint8_t *lwp = tile + (3 * h + (w >> 2)) * 512 + (4 * g) * 16 + (w & 3) * 4;
                    const uint8_t *hup = tile + (3 * h + 2) * 512 + (4 * g) * 16 + (w >> 1) * 4;
                    const uint32_t SCa = *(const uint16_t *)(tile + 3072 + g * 32 + h * 16 + 2 * w);  // int8 sc of 2w, 2w + 1
                    uint32_t ohi[16], olo[16];
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        const uint32_t Lw = *(const uint32_t *)(lwp + t * 16), Hu = *(const uint32_t *)(hup + t * 16);
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            uint32_t hb;
                            if ((w & 1) == 0) hb = Hu >> (2 * k);
                            else hb = k == 0 ? (Hu << 4) : k == 1 ? (Hu << 2) : k == 2 ? (Hu >> 8) : (Hu >> 10);
                            const uint32_t qv = and_or(hb, 0x00300030u, and_or(Lw >> (4 * k), 0x000F000Fu, 0x64006400u));
                            const uint32_t pq = hsub2(qv, 0x64206420u);  // q - 32, exact
                            const int scv = (int)(int8_t)(SCa >> (8 * (k >> 1)));
                            const __half shv = __int2half_rn(scv);  // |sc| <= 128: exact
                            const uint32_t sc2 = half2_bits(__halves2half2(shv, shv));
                            uint32_t hv;
                            asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(hv) : "r"(pq), "r"(sc2));
                            ohi[4 * t + k] = hv;
                            olo[4 * t + k] = hfma2(pq, sc2, hv ^ 0x80008000u);  // exact residual of the product
                        }
                    }
                    tmem_st16(ta, ohi);
                    tmem_st16(ta + 32, olo);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the offset-term operand in smem
                tc_fence_before();
                __syncwarp();
                if (lane == 0) bar_arrive(bars + B_A_FULL + st);
            }
            if (!ok) break;
            // this warp is done with its lane quarter's two tiles of unit i
            __syncwarp();
            if (lane == 0) {
                bar_arrive(bars + B_RAW_EMPTY + slot * 8 + 2 * lq);
                bar_arrive(bars + B_RAW_EMPTY + slot * 8 + 2 * lq + 1);
            }
            if (i + NRAW < n) {
                // refill this warp's tile of the slot once both readers of it are done with unit i
                if (!(ok = wait(B_RAW_EMPTY + slot * 8 + my_tile, (i / NRAW) & 1))) break;
                issue_tile(i + NRAW);
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");  // no copy may land after the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

// ------------------------------------------------------------------ input operands
// CTA (v, c) for input row v and chunk c of the super-blocks: RMSNorm statistics of the whole row
// (optional), an exact power-of-two scale putting max |x| in [2^14, 2^15), then fp16 hi (column v)
// and lo (column 32 + v) of the chunk's elements, in the K order of each weight layout; for Q4_K
// also the sub-block sums as the offset term's B operand.
__global__ void __launch_bounds__(256) tc_prep_kernel(const float *__restrict__ x, int ldx, int nsb,
                                                      const float *__restrict__ norm_w, float eps, int q4, int q6,
                                                      uint8_t *__restrict__ b4, uint8_t *__restrict__ b6,
                                                      float *__restrict__ isc, int reps, size_t b4s, size_t b6s)
{
    __shared__ float red[2][8];
    __shared__ float stat[2];
    const int v = blockIdx.x, tid = threadIdx.x, cols = nsb * 256;
    const int sb_lo = (int)((long long)blockIdx.y * nsb / gridDim.y), sb_n = (int)((long long)(blockIdx.y + 1) * nsb / gridDim.y) - sb_lo;
    const float *xv = x + (size_t)v * ldx;
    float ss = 0.0f, mx = 0.0f;
    for (int i = tid; i < cols; i += 256) {
        const float h = xv[i];
        ss = fmaf(h, h, ss);
        mx = fmaxf(mx, fabsf(norm_w ? __fmul_rn(norm_w[i], h) : h));
    }
    ss = warp_sum(ss);
    mx = warp_max(mx);
    if ((tid & 31) == 0) {
        red[0][tid >> 5] = ss;
        red[1][tid >> 5] = mx;
    }
    __syncthreads();
    if (tid == 0) {
        float s = 0.0f, m = 0.0f;
        for (int w = 0; w < 8; w++) {
            s += red[0][w];
            m = fmaxf(m, red[1][w]);
        }
        float iv = 1.0f;
        if (norm_w) {  // VectorMath.RmsNorm: 1 / sqrt(ss/n + eps); x = (w*h)*inv
            iv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)cols), eps)));
            m = __fmul_rn(m, iv);
        }
        float sc = 1.0f;
        if (m > 0.0f && m < INFINITY) {
            int e;
            frexpf(m, &e);
            sc = ldexpf(1.0f, 15 - e);
        }
        stat[0] = iv;
        stat[1] = sc;
        if (blockIdx.y == 0) isc[v] = 1.0f / sc;
    }
    __syncthreads();
    // ((w*h)*inv)*sc == (w*h)*(inv*sc): sc is a power of two
    const float f = norm_w ? stat[0] * stat[1] : stat[1];
    auto val = [&](int e) { return norm_w ? __fmul_rn(__fmul_rn(norm_w[e], xv[e]), f) : xv[e] * f; };
    const int n_hi = v, n_lo = v + 32;
    const int off_hi = (n_hi >> 3) * 1024 + (n_hi & 7) * 16, off_lo = (n_lo >> 3) * 1024 + (n_lo & 7) * 16;
    // one core row (8 weights, 16 bytes) per item: (super-block, quarter qt, core row kc of the quarter)
    for (int it = tid; it < sb_n * 32; it += 256) {
        const int sb = sb_lo + (it >> 5), kc32 = it & 31, qt = kc32 >> 3, kc = kc32 & 7;
        float c[8];
        if (q4) {  // elements 32 (kc / 4) + 8 (kc % 4) + {0,4,1,5,2,6,3,7} of the quarter
            const int e0 = sb * 256 + qt * 64 + 32 * (kc >> 2) + 8 * (kc & 3);
            float nat[8];
#pragma unroll
            for (int k = 0; k < 8; k++) nat[k] = val(e0 + k);
            const int perm[8] = {0, 4, 1, 5, 2, 6, 3, 7};
#pragma unroll
            for (int k = 0; k < 8; k++) c[k] = nat[perm[k]];
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const __half2 hh = __floats2half2_rn(c[2 * k], c[2 * k + 1]);
                const float2 hf2 = __half22float2(hh);
                hi[k] = half2_bits(hh);
                lo[k] = pack_half2(c[2 * k] - hf2.x, c[2 * k + 1] - hf2.y);
            }
            uint8_t *base = b4 + (size_t)sb * B4_SB + qt * B_BYTES + kc * 128;
            for (int r = 0; r < reps; r++) {
                *(uint4 *)(base + r * b4s + off_hi) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *(uint4 *)(base + r * b4s + off_lo) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
        }
        if (q6) {  // elements 32 w2 + 4 t + {0..3} and 32 w2 + 16 + 4 t + {0..3} of the quarter (kc = 4 w2 + t)
            const int e0 = sb * 256 + qt * 64 + 32 * (kc >> 2) + 4 * (kc & 3);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                c[k] = val(e0 + k);
                c[4 + k] = val(e0 + 16 + k);
            }
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const __half2 hh = __floats2half2_rn(c[2 * k], c[2 * k + 1]);
                const float2 hf2 = __half22float2(hh);
                hi[k] = half2_bits(hh);
                lo[k] = pack_half2(c[2 * k] - hf2.x, c[2 * k + 1] - hf2.y);
            }
            uint8_t *base = b6 + (size_t)sb * B6_SB + qt * B_BYTES + kc * 128;
            for (int r = 0; r < reps; r++) {
                *(uint4 *)(base + r * b6s + off_hi) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *(uint4 *)(base + r * b6s + off_lo) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
        }
    }
    if (q4) {
        // sub-block sums S_j (fixed order: four 8-element partials), hi and lo, at K = 2j and 2j + 1
        for (int it = tid; it < sb_n * 8; it += 256) {
            const int sb = sb_lo + (it >> 3), j = it & 7;
            float p[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                float s = 0.0f;
#pragma unroll
                for (int k = 0; k < 8; k++) s += val(sb * 256 + 32 * j + 8 * q + k);
                p[q] = s;
            }
            const float S = (((p[0] + p[1]) + p[2]) + p[3]) * S_FAC;
            const __half sh = __float2half_rn(S);
            const __half sl = __float2half_rn(S - __half2float(sh));
            uint8_t *base = b4 + (size_t)sb * B4_SB + 4 * B_BYTES + (j >> 2) * 128 + (j & 3) * 4;
            for (int r = 0; r < reps; r++) {
                *(uint32_t *)(base + r * b4s + (n_hi >> 3) * 256 + (n_hi & 7) * 16) = half2_bits(__halves2half2(sh, sh));
                *(uint32_t *)(base + r * b4s + (n_lo >> 3) * 256 + (n_lo & 7) * 16) = half2_bits(__halves2half2(sl, sl));
            }
        }
    }
}

int sm_count()
{
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

}  // namespace

int tc_scratch_alloc(TcScratch &s, int cols_max, int tiles_max, std::vector<void *> &allocs)
{
    const int nsb = (cols_max + 255) / 256;
    const int grid = sm_count();
    auto get = [&](void **p, size_t bytes) -> int {
        if (cudaMalloc(p, bytes) != cudaSuccess) {
            cudaGetLastError();
            return fail(LLMDOT_E_NOMEM, "tensor-core matmul scratch allocation failed");
        }
        allocs.push_back(*p);
        return LLMDOT_OK;
    };
    // replicas of the prepared operands (CTA c reads replica c % reps): every CTA reads all of one
    // input's B from L2; spreading the readers over copies measured no faster, so one by default
    static const int reps_env = [] {
        const char *e = getenv("LLMDOT_TC_REPLICAS");
        return e ? std::max(1, std::min(16, atoi(e))) : TC_DEFAULT_REPLICAS;
    }();
    s.reps = reps_env;
    s.b4s = (size_t)nsb * B4_SB;
    s.b6s = (size_t)nsb * B6_SB;
    LLMDOT_TRY(get((void **)&s.b4, s.b4s * s.reps));
    LLMDOT_TRY(get((void **)&s.b6, s.b6s * s.reps));
    LLMDOT_TRY(get((void **)&s.isc, sizeof(float) * TC_MAX_ROWS));
    LLMDOT_TRY(get((void **)&s.part, sizeof(float) * (size_t)grid * 2 * TC_MAX_ROWS * TM));
    LLMDOT_TRY(get((void **)&s.cnt, sizeof(int) * (size_t)tiles_max));
    LLMDOT_CUDA_TRY(cudaMemset(s.cnt, 0, sizeof(int) * (size_t)tiles_max));
    // stale columns of unused input rows must not hold NaN bit patterns that the MMA would read as
    // values of live columns: every column is independent, so zeroing once is only for tidiness
    LLMDOT_CUDA_TRY(cudaMemset(s.b4, 0, s.b4s * s.reps));
    LLMDOT_CUDA_TRY(cudaMemset(s.b6, 0, s.b6s * s.reps));
    s.cols_max = nsb * 256;
    s.grid_max = grid;
    s.tiles_max = tiles_max;
    return LLMDOT_OK;
}

bool tc_supported(const DevMat &W)
{
    return W.tiled && (W.type == T_Q4_K || W.type == T_Q6_K) && W.cols % 256 == 0;
}

int tc_prepare(const float *x, int ldx, int nv, int cols, const float *norm_w, float eps, bool q4, bool q6,
               TcScratch &s, cudaStream_t st)
{
    if (!s.ready() || nv < 1 || nv > TC_MAX_ROWS || cols % 256 || cols > s.cols_max)
        return fail(LLMDOT_E_INVALID, "tensor-core matmul: bad input shape");
    // about four super-blocks per CTA: the statistics are re-read per chunk, the conversion spreads
    const int chunks = std::max(1, std::min(16, cols / 1024));
    tc_prep_kernel<<<dim3(nv, chunks), 256, 0, st>>>(x, ldx, cols / 256, norm_w, eps, q4 ? 1 : 0, q6 ? 1 : 0, s.b4,
                                                      s.b6, s.isc, s.reps, s.b4s, s.b6s);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

int tc_gemm(const TcSeg *seg, int nseg, int nv, int mode, TcScratch &s, int *err, cudaStream_t st,
            const GemvPrefetch *pf)
{
    if (!s.ready() || nseg < 1 || nseg > 3 || nv < 1 || nv > TC_MAX_ROWS || (mode != GEMV_STORE && mode != GEMV_ADD))
        return fail(LLMDOT_E_INVALID, "tensor-core matmul: bad arguments");
    TcArgs a{};
    a.nseg = nseg;
    a.nsb = seg[0].W->cols / 256;
    a.nv = nv;
    a.mode = mode;
    int tiles = 0;
    for (int i = 0; i < nseg; i++) {
        const DevMat &W = *seg[i].W;
        if (!tc_supported(W) || W.cols != seg[0].W->cols || W.cols > s.cols_max)
            return fail(LLMDOT_E_UNSUPPORTED, "tensor-core matmul: unsupported matrix");
        a.w[i] = W.tiled;
        a.y[i] = seg[i].y;
        a.ldy[i] = seg[i].ldy;
        a.rows[i] = W.rows;
        a.qt[i] = W.type == T_Q4_K ? QT_Q4K : QT_Q6K;
        a.nrt16[i] = (W.rows + 15) / 16;
        a.cum[i] = tiles;
        tiles += (W.rows + TM - 1) / TM;
    }
    a.cum[nseg] = tiles;
    if (tiles > s.tiles_max) return fail(LLMDOT_E_UNSUPPORTED, "tensor-core matmul: more row tiles than scratch");
    a.U = tiles * a.nsb;
    a.b4 = s.b4;
    a.b6 = s.b6;
    a.b4s = s.b4s;
    a.b6s = s.b6s;
    a.reps = s.reps;
    a.isc = s.isc;
    a.part = s.part;
    a.cnt = s.cnt;
    a.err = err;
    if (pf) {
        for (int r = 0; r < GEMV_PREFETCH_MAX; r++)  // bulk prefetches want 16-byte aligned, 16-byte multiples
            if (((uintptr_t)pf->p[r] & 15) || (pf->n[r] & 15)) return fail(LLMDOT_E_INVALID, "tensor-core matmul: prefetch range");
        a.pf = *pf;
    }
    const int grid = a.U < s.grid_max ? a.U : s.grid_max;
    static std::atomic<unsigned long long> attr_done{0};
    LLMDOT_CUDA_TRY(smem_attr_once(attr_done, tc_gemm_kernel, (int)SMEM_BYTES));
    tc_gemm_kernel<<<grid, TC_THREADS, SMEM_BYTES, st>>>(a);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

}  // namespace llmdot
