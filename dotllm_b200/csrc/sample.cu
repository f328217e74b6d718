// sample.cu -- Sampler.Sample on the device (temperature, top-k, repeat penalty).
//
// Reference: src/Llmdot.Core/Sampling/Sampler.cs:24-165 with SamplingOptions.cs:7-14, called by
// InferenceEngine.Generate (InferenceEngine.cs:103-111) after the final-logit softcap.  One CTA per
// row of logits:
//   1. the row's value of token i is softcap(logits[i]) (Gemma; the reference's vector/tail rule),
//      then the repeat penalty of the last `window` history tokens, each applied once in history
//      order (a token that appears twice is divided twice), then times 1/T (VectorMath.Scale);
//   2. top-k by a 4-pass radix select on order-preserving 32-bit keys of the values, the k winners
//      sorted by value (bitonic sort of (key, index) pairs in shared memory);
//   3. VectorMath.Softmax over the k sorted values (ExpApprox in the 8-wide lanes, exp in the tail,
//      the 8 lane sums added as ((0+1)+(2+3))+((4+5)+(6+7))), then the first index whose running
//      sum of probabilities reaches the draw r (SampleFromProbabilities).
// Temperature <= 0 is the greedy argmax of the softcapped row (lowest index on ties).  When two of
// the k winners have equal values, or equal values straddle the k-th place, which of them win and
// their order come from FindTopK's replacement scan (:83-127), so such rows replay it exactly
// (topk_replay: one warp scanning the row in index order); rows without ties skip the replay, as
// their winners and order are then unique.
//
// top_k <= 0 or top_k >= n (Sampler.cs:42-61): VectorMath.Softmax over the whole row (the FindMax
// lane rule, ExpApprox in the 8-wide lanes with the lanes' running sums, exp in the tail), then
//   * top_p >= 1: the first index whose running sum reaches r;
//   * top_p < 1: FindNucleus (:129-151) -- the selection sort by probability, the prefix whose
//     running sum first reaches top_p, renormalised, and the pick inside it.  The reference passes
//     one buffer as both the probabilities and the nucleus values (:48-50), so the value written at
//     sorted position i is the probability of token idx[i] unless that token's slot was already
//     overwritten (idx[i] < i), in which case it is the value written there; when the nucleus is
//     the whole row the pick then runs over the overwritten row and returns a position.  The device
//     sorts (value, index) pairs with a stable radix sort; while no two of the prefix's values tie,
//     that is the selection sort's order, and the aliased values follow the chain
//     i -> idx[i] while idx[i] < i.  A tie inside the prefix replays the selection sort's swaps on
//     one thread (each tie group ordered by its members' current positions).
// The running sums are sequential fp32 adds in the reference's order, on one thread.
#include "sample.cuh"

#include <cub/device/device_radix_sort.cuh>
#include <string>

namespace llmdot {

constexpr int SMP_THREADS = 1024;
constexpr int SMP_UNROLL = 4;  // row values loaded per thread before any is used (loads in flight)

constexpr int SMP_CAND = 4096;     // candidates the sampled threshold may collect
constexpr int SMP_SAMPLES = 2048;  // keys of the strided sample that places the threshold

struct SampleSmem {
    int bitmap, ptok, pval, hist, cand, skey, prob, total;  // byte offsets
};
__host__ __device__ inline SampleSmem sample_layout(int n, int window, int k2)
{
    SampleSmem L;
    int o = 0;
    L.bitmap = o;  // one bit per token: penalised tokens
    o += ((n + 31) / 32 * 4 + 15) / 16 * 16;
    L.ptok = o;  // penalised tokens and their values
    o += (window * 4 + 15) / 16 * 16;
    L.pval = o;
    o += (window * 4 + 15) / 16 * 16;
    L.hist = o;  // radix histogram, then scan state
    o += 260 * 4;
    L.cand = o;  // (key << 32 | ~index) pairs: the candidates, at least k2
    o += (k2 > SMP_CAND ? k2 : SMP_CAND) * 8;
    L.skey = o;  // strided sample of the row's keys
    o += SMP_SAMPLES * 4;
    L.prob = o;  // k probabilities
    o += k2 * 4;
    L.total = o;
    return L;
}

// The row's values as the sampler sees them: softcap (vector-lane rule), repeat penalty, 1/T.
struct RowValues {
    const float *x;
    int nvec, has_cap, np;
    float cap, inv_cap, inv_temp;
    const uint32_t *bitmap;
    const int *ptok;
    const float *pval;
    __device__ __forceinline__ float capped(int i) const
    {
        const float v = x[i];
        return has_cap ? softcap_ref(v, cap, inv_cap, i < nvec) : v;
    }
    // the scaled value of token i (VectorMath.Scale: x * (1/T) in every lane)
    __device__ __forceinline__ float value(int i) const
    {
        float v;
        if (np && ((bitmap[i >> 5] >> (i & 31)) & 1u)) {
            int j = 0;
            while (ptok[j] != i) j++;
            v = pval[j];
        } else {
            v = capped(i);
        }
        return __fmul_rn(v, inv_temp);
    }
};

// Repeat penalty (ApplyRepeatPenalty :64-81), by the whole block: the last `window` history tokens
// in order, each occurrence applied once (a token that appears twice is divided twice).  The
// window's values are loaded in parallel into wval; one thread then applies the penalty.  Fills
// the bitmap and (ptok, pval) of the distinct penalised tokens and returns their number.
__device__ int penalty_setup(const SampleArgs &a, int row, RowValues &rv, uint32_t *bitmap, int *ptok, float *pval,
                             float *wval, int *np_slot)
{
    const int tid = threadIdx.x, n = a.n, window = a.window;
    for (int i = tid; i < (n + 31) / 32; i += blockDim.x) bitmap[i] = 0u;
    const bool pen = a.penalty != 1.0f && window > 0 && a.recent;
    const int plen = pen ? a.recent_len[row] : 0, p0 = max(0, plen - window);
    const int32_t *rec = pen ? a.recent + (size_t)row * a.recent_ld : nullptr;
    for (int i = p0 + tid; i < plen; i += blockDim.x) {
        const int t = rec[i];
        wval[i - p0] = (t >= 0 && t < n) ? rv.capped(t) : 0.0f;
    }
    __syncthreads();
    if (tid == 0) {
        int np = 0;
        for (int i = p0; i < plen; i++) {
            const int t = rec[i];
            if (t < 0 || t >= n) continue;
            int j = 0;
            while (j < np && ptok[j] != t) j++;
            if (j == np) {
                ptok[np] = t;
                pval[np] = wval[i - p0];
                np++;
                bitmap[t >> 5] |= 1u << (t & 31);
            }
            pval[j] = pval[j] > 0.0f ? __fdiv_rn(pval[j], a.penalty) : __fmul_rn(pval[j], a.penalty);
        }
        *np_slot = np;
    }
    __syncthreads();
    const int np = *np_slot;
    rv.bitmap = bitmap;
    rv.ptok = ptok;
    rv.pval = pval;
    rv.np = np;
    return np;
}

__device__ __forceinline__ RowValues row_values(const SampleArgs &a, int row)
{
    RowValues rv;
    rv.x = a.logits + (size_t)row * a.ld;
    rv.nvec = a.n - a.n % 8;
    rv.has_cap = a.has_cap;
    rv.cap = a.cap;
    rv.inv_cap = a.inv_cap;
    rv.inv_temp = a.inv_temp;
    rv.np = 0;
    rv.bitmap = nullptr;
    rv.ptok = nullptr;
    rv.pval = nullptr;
    return rv;
}

// First slot holding the smallest of tv[0..k) (FindTopK's minIdx scan, :93-98: a later slot
// replaces the current one only when strictly smaller, so equal values keep the lowest slot),
// reduced over the calling warp; every lane gets the same (value, slot).
__device__ __forceinline__ void topk_min(const float *tv, int k, int lane, float &minv, int &mins)
{
    float bv = 0.0f;
    int bs = INT_MAX;
    for (int j = lane; j < k; j += 32) {
        const float t = tv[j];
        if (bs == INT_MAX || t < bv) {
            bv = t;
            bs = j;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int os = __shfl_xor_sync(0xffffffffu, bs, o);
        if (os != INT_MAX && (bs == INT_MAX || ov < bv || (ov == bv && os < bs))) {
            bv = ov;
            bs = os;
        }
    }
    minv = bv;
    mins = bs;
}

// FindTopK (Sampler.cs:83-127) replayed exactly, for rows whose winners tie: slots 0..k-1 start
// as tokens 0..k-1; each later token, in index order, replaces the first slot holding the minimum
// when it is strictly larger; the slots are then ordered by value, equal values by slot (the
// insertion sort is stable).  Warp 0 scans the row 32 tokens at a time and handles the tokens
// above the current minimum lane by lane in index order (re-testing them after each replacement);
// the whole block then sorts (value, slot) pairs.  Leaves the k winners in cand as
// (key << 32 | ~token), sorted.  Rows are taken NaN-free (a NaN never enters, as in the reference,
// but one among the first k slots is ordered differently).
__device__ void topk_replay(const RowValues &rv, int n, int k, int k2, unsigned long long *cand, int *tix,
                            float *tv)
{
    const int tid = threadIdx.x;
    if (tid < 32) {
        const int lane = tid;
        for (int j = lane; j < k; j += 32) {
            tix[j] = j;
            tv[j] = rv.value(j);
        }
        __syncwarp();
        float minv;
        int mins;
        topk_min(tv, k, lane, minv, mins);
        for (int base = k; base < n; base += 4 * 32) {
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = base + u * 32 + lane;
                v[u] = i < n ? rv.value(i) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int b = base + u * 32;
                unsigned m = __ballot_sync(0xffffffffu, b + lane < n && v[u] > minv);
                while (m) {
                    const int l = __ffs(m) - 1;
                    const float vl = __shfl_sync(0xffffffffu, v[u], l);
                    if (lane == 0) {
                        tix[mins] = b + l;
                        tv[mins] = vl;
                    }
                    __syncwarp();
                    topk_min(tv, k, lane, minv, mins);
                    m &= ~(1u << l);
                    m &= __ballot_sync(0xffffffffu, b + lane < n && v[u] > minv);
                }
            }
        }
    }
    __syncthreads();
    // (value, slot) pairs: descending value (-0 as +0), then ascending slot
    for (int j = tid; j < k2; j += SMP_THREADS)
        cand[j] = j < k ? ((unsigned long long)float_key(tv[j] == 0.0f ? 0.0f : tv[j]) << 32) | (uint32_t)~j : 0ull;
    __syncthreads();
    for (int size = 2; size <= k2; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < k2 / 2; i += SMP_THREADS) {
                const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const unsigned long long A = cand[lo], B = cand[hi];
                if ((A < B) == desc) {
                    cand[lo] = B;
                    cand[hi] = A;
                }
            }
            __syncthreads();
        }
    for (int j = tid; j < k; j += SMP_THREADS) {
        const int slot = (int)~(uint32_t)cand[j];
        cand[j] = ((unsigned long long)float_key(tv[slot]) << 32) | (uint32_t)~tix[slot];
    }
    __syncthreads();
}

__global__ void __launch_bounds__(SMP_THREADS) sample_kernel(SampleArgs a, int k2)
{
    extern __shared__ __align__(16) uint8_t smem[];
    const int row = blockIdx.x, tid = threadIdx.x, n = a.n;
    const int window = a.window;
    const SampleSmem L = sample_layout(n, window, k2);
    uint32_t *bitmap = (uint32_t *)(smem + L.bitmap);
    int *ptok = (int *)(smem + L.ptok);
    float *pval = (float *)(smem + L.pval);
    int *hist = (int *)(smem + L.hist);
    unsigned long long *cand = (unsigned long long *)(smem + L.cand);
    uint32_t *skey = (uint32_t *)(smem + L.skey);
    float *prob = (float *)(smem + L.prob);
    RowValues rv = row_values(a, row);
    auto capped = [&](int i) { return rv.capped(i); };

    if (a.temperature <= 0.0f) {  // Temperature <= 0: ArgMax (Sampler.cs:26-27)
        unsigned long long best = 0;
        for (int base = 0; base < n; base += SMP_THREADS * SMP_UNROLL) {
            float vals[SMP_UNROLL];
#pragma unroll
            for (int u = 0; u < SMP_UNROLL; u++) {
                const int i = base + u * SMP_THREADS + tid;
                vals[u] = i < n ? capped(i) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < SMP_UNROLL; u++) {
                const int i = base + u * SMP_THREADS + tid;
                if (i >= n) continue;
                const unsigned long long kk = argmax_key(vals[u], (uint32_t)i);
                best = kk > best ? kk : best;
            }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
            best = v > best ? v : best;
        }
        if ((tid & 31) == 0) cand[tid >> 5] = best;
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < SMP_THREADS / 32; w++) best = cand[w] > best ? cand[w] : best;
            const int idx = (int)~(uint32_t)best;
            a.out[row] = idx;
            if (a.next) a.next[row] = idx;
        }
        return;
    }

    // ---- repeat penalty (the window's values are staged in the candidate buffer, not yet in use)
    penalty_setup(a, row, rv, bitmap, ptok, pval, (float *)cand, &hist[256]);
    auto value = [&](int i) { return rv.value(i); };

    const int k = a.top_k;
    int sort_n = k2;  // entries of cand to sort
    bool fast = false;
    int ncand = 0;         // fast path: candidates collected (sorted, so cand[k] is the (k+1)-th largest)
    bool thr_tie = false;  // radix path: more keys equal the k-th than places are left for them
    // ---- fast path: a threshold tau from a strided sample, then one pass collecting every key
    // >= tau.  When at least k keys reach tau, the k largest (ties included) are all among them,
    // so sorting the candidates gives exactly the radix select's answer; otherwise (tau above
    // the k-th key, or more than SMP_CAND candidates) the radix select below runs.
    {
        const int ns = n < SMP_SAMPLES ? n : SMP_SAMPLES;
        for (int j = tid; j < SMP_SAMPLES; j += SMP_THREADS)
            skey[j] = j < ns ? float_key(value((int)((long long)j * n / ns))) : 0u;
        if (tid == 0) {
            hist[0] = 0;
            hist[1] = 0;
        }
        __syncthreads();
        for (int size = 2; size <= SMP_SAMPLES; size <<= 1)  // sort the sample, descending
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = tid; i < SMP_SAMPLES / 2; i += SMP_THREADS) {
                    const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
                    const bool desc = (lo & size) == 0;
                    const uint32_t A = skey[lo], B = skey[hi];
                    if ((A < B) == desc) {
                        skey[lo] = B;
                        skey[hi] = A;
                    }
                }
                __syncthreads();
            }
        // about 2k + a margin of the row's keys are expected at or above the sample's r-th key
        const int rk = (int)(((long long)2 * k * ns + n - 1) / n) + 4;
        const uint32_t tau = skey[rk < ns ? rk : ns - 1];
        for (int base = 0; base < n; base += SMP_THREADS * SMP_UNROLL) {
            uint32_t keys[SMP_UNROLL];
#pragma unroll
            for (int u = 0; u < SMP_UNROLL; u++) {
                const int i = base + u * SMP_THREADS + tid;
                keys[u] = i < n ? float_key(value(i)) : 0u;
            }
#pragma unroll
            for (int u = 0; u < SMP_UNROLL; u++) {
                const int i = base + u * SMP_THREADS + tid;
                if (i < n && keys[u] >= tau) {
                    const int slot = atomicAdd(&hist[0], 1);
                    if (slot < SMP_CAND) cand[slot] = ((unsigned long long)keys[u] << 32) | (uint32_t)~i;
                }
            }
        }
        __syncthreads();
        const int got = hist[0];
        __syncthreads();
        ncand = got;
        if (got >= k && got <= SMP_CAND) {
            int c2 = k2;
            while (c2 < got) c2 <<= 1;
            for (int i = got + tid; i < c2; i += SMP_THREADS) cand[i] = 0ull;
            __syncthreads();
            sort_n = c2;
            fast = true;
        }
    }
    if (!fast) {  // uniform: every thread read the same count
    // ---- radix select of the k-th largest key
    uint32_t prefix = 0, mask = 0;
    int need = k;  // rank wanted inside the current prefix
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += SMP_THREADS) hist[i] = 0;
        __syncthreads();
        // nearly every logit shares the top key byte: lanes with the same bin add once per warp
        for (int base = 0; base < n; base += SMP_THREADS * SMP_UNROLL) {
            uint32_t keys[SMP_UNROLL];
#pragma unroll
            for (int u = 0; u < SMP_UNROLL; u++) {
                const int i = base + u * SMP_THREADS + tid;
                keys[u] = i < n ? float_key(value(i)) : 0u;
            }
#pragma unroll
            for (int u = 0; u < SMP_UNROLL; u++) {
                const int i = base + u * SMP_THREADS + tid;
                const bool act = i < n && (keys[u] & mask) == prefix;
                const unsigned am = __ballot_sync(0xffffffffu, act);
                if (act) {
                    const uint32_t bin = (keys[u] >> shift) & 255u;
                    const unsigned same = __match_any_sync(am, bin);
                    if ((tid & 31) == __ffs(same) - 1) atomicAdd(&hist[bin], __popc(same));
                }
            }
        }
        __syncthreads();
        if (tid == 0) {
            int above = 0, b = 255;
            for (; b > 0; b--) {
                if (above + hist[b] >= need) break;
                above += hist[b];
            }
            hist[257] = b;
            hist[258] = need - above;  // rank inside bin b
            hist[259] = hist[b];       // keys in bin b
        }
        __syncthreads();
        prefix |= (uint32_t)hist[257] << shift;
        mask |= 255u << shift;
        need = hist[258];
        __syncthreads();
    }
    const uint32_t thr = prefix;
    const int eq_total = hist[259], eq_take = need;  // keys equal to thr: all of them / how many to take
    thr_tie = eq_take < eq_total;
    // ---- the k winners: every key above thr, and the eq_take lowest indices with key == thr
    if (tid == 0) hist[0] = 0;
    for (int i = tid; i < k2; i += SMP_THREADS) cand[i] = 0ull;
    __syncthreads();
    for (int base = 0; base < n; base += SMP_THREADS * SMP_UNROLL) {
        uint32_t keys[SMP_UNROLL];
#pragma unroll
        for (int u = 0; u < SMP_UNROLL; u++) {
            const int i = base + u * SMP_THREADS + tid;
            keys[u] = i < n ? float_key(value(i)) : 0u;
        }
#pragma unroll
        for (int u = 0; u < SMP_UNROLL; u++) {
            const int i = base + u * SMP_THREADS + tid;
            if (i < n && (keys[u] > thr || (keys[u] == thr && eq_take == eq_total))) {
                const int slot = atomicAdd(&hist[0], 1);
                cand[slot] = ((unsigned long long)keys[u] << 32) | (uint32_t)~i;
            }
        }
    }
    __syncthreads();
    if (eq_take < eq_total) {  // ties across the k-th place: the lowest indices, in index order
        if (tid == 0) {
            int slot = hist[0];
            for (int i = 0, got = 0; i < n && got < eq_take; i++)
                if (float_key(value(i)) == thr) {
                    cand[slot++] = ((unsigned long long)thr << 32) | (uint32_t)~i;
                    got++;
                }
        }
        __syncthreads();
    }
    }
    // ---- bitonic sort, descending: by value, then by lower index (the first k are the winners)
    for (int size = 2; size <= sort_n; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < sort_n / 2; i += SMP_THREADS) {
                const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const unsigned long long A = cand[lo], B = cand[hi];
                if ((A < B) == desc) {
                    cand[lo] = B;
                    cand[hi] = A;
                }
            }
            __syncthreads();
        }
    // ---- exactly equal values among the winners or across the k-th place: FindTopK's order
    if (tid == 0) {
        const float kth = key_float((uint32_t)(cand[k - 1] >> 32));
        // -0 and +0 compare equal in the reference but have distinct keys: a zero k-th value
        // may hide a tie across the k-th place, so it is treated as one
        hist[0] = thr_tie || kth == 0.0f || (fast && ncand > k && key_float((uint32_t)(cand[k] >> 32)) == kth);
    }
    __syncthreads();
    for (int j = 1 + tid; j < k; j += SMP_THREADS)  // sorted: equal values are neighbours
        if (key_float((uint32_t)(cand[j - 1] >> 32)) == key_float((uint32_t)(cand[j] >> 32))) hist[0] = 1;
    __syncthreads();
    if (hist[0]) topk_replay(rv, n, k, k2, cand, (int *)skey, prob);
    // ---- VectorMath.Softmax over the k values (Sampler.cs:39), then the pick (:153-165)
    if (tid < 32) {
        const int lane = tid;
        const float mx = key_float((uint32_t)(cand[0] >> 32));  // sorted: the first is the largest
        const int kvec = k - k % 8;
        float acc = 0.0f;
        if (lane < 8)
            for (int j = lane; j < kvec; j += 8) {
                const float e = exp_approx(__fsub_rn(key_float((uint32_t)(cand[j] >> 32)), mx));
                prob[j] = e;
                acc = __fadd_rn(acc, e);
            }
        // ((l0 + l1) + (l2 + l3)) + ((l4 + l5) + (l6 + l7))
        const float s1 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
        const float s2 = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, 2));
        const float s4 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, 4));
        if (lane == 0) {
            float sum = s4;
            for (int j = kvec; j < k; j++) {
                const float e = expf(__fsub_rn(key_float((uint32_t)(cand[j] >> 32)), mx));
                prob[j] = e;
                sum = __fadd_rn(sum, e);
            }
            const float inv = __fdiv_rn(1.0f, sum);
            const float r = a.r[row];
            float cum = 0.0f;
            int pick = k - 1;
            for (int j = 0; j < k; j++) {
                cum = __fadd_rn(cum, __fmul_rn(prob[j], inv));
                if (r <= cum) {
                    pick = j;
                    break;
                }
            }
            const int idx = (int)~(uint32_t)cand[pick];
            a.out[row] = idx;
            if (a.next) a.next[row] = idx;
        }
    }
}

// ---------------------------------------------------------------- full-row path (top_k <= 0 or >= n)
constexpr int SF_CHUNK = 8192;    // values staged in shared memory per step of a sequential scan
constexpr int SF_GROUP = 8192;    // largest tie group the selection-sort replay orders in shared memory
constexpr int SF_TIE_GROUP_TOO_LARGE = -2;  // written as the sampled id when SF_GROUP is exceeded

static size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

static size_t cub_sort_bytes(int n)
{
    size_t tb = 0;
    cub::DeviceRadixSort::SortPairsDescending(nullptr, tb, (const uint32_t *)nullptr, (uint32_t *)nullptr,
                                              (const int32_t *)nullptr, (int32_t *)nullptr, n);
    return tb;
}

size_t sample_work_bytes(int n)
{
    return 8 * align256(sizeof(float) * (size_t)n) + align256(cub_sort_bytes(n));
}

static SampleWork work_carve(void *base, int n)
{
    SampleWork w;
    uint8_t *p = (uint8_t *)base;
    const size_t a = align256(sizeof(float) * (size_t)n);
    w.p = (float *)p;
    w.val = (float *)(p + a);
    w.kin = (uint32_t *)(p + 2 * a);
    w.kout = (uint32_t *)(p + 3 * a);
    w.iin = (int32_t *)(p + 4 * a);
    w.iout = (int32_t *)(p + 5 * a);
    w.pos = (int32_t *)(p + 6 * a);
    w.at = (int32_t *)(p + 7 * a);
    w.cub = p + 8 * a;
    w.cub_bytes = cub_sort_bytes(n);
    return w;
}

struct SampleFullSmem {
    int bitmap, ptok, pval, wval, misc, chunk, group, total;  // byte offsets
};
__host__ __device__ inline SampleFullSmem sample_full_layout(int n, int window, bool probs)
{
    SampleFullSmem L;
    int o = 0;
    L.bitmap = o;
    o += probs ? ((n + 31) / 32 * 4 + 15) / 16 * 16 : 0;
    L.ptok = o;
    o += probs ? (window * 4 + 15) / 16 * 16 : 0;
    L.pval = o;
    o += probs ? (window * 4 + 15) / 16 * 16 : 0;
    L.wval = o;
    o += probs ? (window * 4 + 15) / 16 * 16 : 0;
    L.misc = o;  // 32 floats / ints of block reductions and broadcasts
    o += 32 * 4 + 16 * 4;
    L.chunk = o;
    o += SF_CHUNK * 4;
    L.group = o;  // (position << 32 | token) keys of one tie group
    o += probs ? 0 : SF_GROUP * 8;
    L.total = o;
    return L;
}

// The first i in [0, len) at which the running fp32 sum of v[0..i] (each times `scale` first when
// `scaled`) reaches thr, or -1.  One thread adds in index order (the reference's loops); the block
// stages the values in shared memory.  *sum_out (thread 0): the running sum where the scan stopped.
__device__ int seq_reach(const float *v, int len, bool scaled, float scale, float thr, float *chunk, int *flag,
                         float *sum_out)
{
    float cum = 0.0f;
    int hit = -1;
    for (int base = 0; base < len; base += SF_CHUNK) {
        const int m = min(SF_CHUNK, len - base);
        for (int j = threadIdx.x; j < m; j += blockDim.x) chunk[j] = v[base + j];
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int j = 0; j < m; j++) {
                cum = __fadd_rn(cum, scaled ? __fmul_rn(chunk[j], scale) : chunk[j]);
                if (cum >= thr) {  // SampleFromProbabilities: r <= cum; FindNucleus: cum >= top_p
                    hit = base + j;
                    break;
                }
            }
            *flag = hit;
        }
        __syncthreads();
        hit = *flag;
        __syncthreads();
        if (hit >= 0) break;
    }
    if (threadIdx.x == 0 && sum_out) *sum_out = cum;
    return hit;
}

// Softmax of the whole row into w.p (and the sort keys when the nucleus follows); without the
// nucleus, also the pick.
__global__ void __launch_bounds__(SMP_THREADS) sample_probs_kernel(SampleArgs a, SampleWork w, int nucleus)
{
    extern __shared__ __align__(16) uint8_t smem[];
    const int n = a.n, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const SampleFullSmem L = sample_full_layout(n, a.window, true);
    float *misc = (float *)(smem + L.misc), *chunk = (float *)(smem + L.chunk);
    int *imisc = (int *)(misc + 32);
    RowValues rv = row_values(a, 0);
    penalty_setup(a, 0, rv, (uint32_t *)(smem + L.bitmap), (int *)(smem + L.ptok), (float *)(smem + L.pval),
                  (float *)(smem + L.wval), &imisc[0]);
    // ---- values, and FindMax (:260-284): with n >= 8, lane l of the 8-wide loop starts from
    // element l and keeps it if it is NaN (no later element compares greater); NaN never wins; so
    // the max is over the non-NaN elements outside NaN-started lanes.  With n < 8: x[0], then `>`.
    const int nv8 = n - n % 8;
    uint32_t nan_lanes = 0;
    if (n >= 8)
        for (int l = 0; l < 8; l++) nan_lanes |= (uint32_t)(rv.value(l) != rv.value(l)) << l;
    float mx = -INFINITY;
    for (int i = tid; i < n; i += SMP_THREADS) {
        const float v = rv.value(i);
        w.p[i] = v;
        const bool ok = v == v && !(i < nv8 && ((nan_lanes >> (i & 7)) & 1u));
        if (ok) mx = fmaxf(mx, v);
    }
    mx = warp_max(mx);
    if (lane == 0) misc[warp] = mx;
    __syncthreads();
    if (tid == 0) {
        float m = -INFINITY;
        for (int q = 0; q < SMP_THREADS / 32; q++) m = fmaxf(m, misc[q]);
        if (n < 8) {
            m = w.p[0];
            for (int i = 1; i < n; i++)
                if (w.p[i] > m) m = w.p[i];
        }
        misc[0] = m;
    }
    __syncthreads();
    const float M = misc[0];
    // ---- e = ExpApprox(x - max) in the 8-wide lanes, exp in the tail (Softmax :215-258)
    for (int i = tid; i < n; i += SMP_THREADS) {
        const float d = __fsub_rn(w.p[i], M);
        w.p[i] = i < nv8 ? exp_approx(d) : expf(d);
    }
    __syncthreads();
    // ---- the lanes' running sums (lane l adds elements l, l + 8, ... in order), staged in chunks
    float acc = 0.0f;
    for (int base = 0; base < nv8; base += SF_CHUNK) {
        const int m = min(SF_CHUNK, nv8 - base);
        for (int j = tid; j < m; j += SMP_THREADS) chunk[j] = w.p[base + j];
        __syncthreads();
        if (tid < 8)
            for (int j = tid; j < m; j += 8) acc = __fadd_rn(acc, chunk[j]);
        __syncthreads();
    }
    if (warp == 0) {
        // ((l0 + l1) + (l2 + l3)) + ((l4 + l5) + (l6 + l7)), then the tail in order
        if (lane >= 8) acc = 0.0f;
        const float s1 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
        const float s2 = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, 2));
        const float s4 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, 4));
        if (lane == 0) {
            float sum = n >= 8 ? s4 : 0.0f;
            for (int j = nv8; j < n; j++) sum = __fadd_rn(sum, w.p[j]);
            misc[1] = __fdiv_rn(1.0f, sum);
        }
    }
    __syncthreads();
    const float inv = misc[1];
    for (int i = tid; i < n; i += SMP_THREADS) {
        const float pr = __fmul_rn(w.p[i], inv);
        w.p[i] = pr;
        if (nucleus) {
            w.kin[i] = float_key(pr);
            w.iin[i] = i;
        }
    }
    __syncthreads();
    if (nucleus) return;
    // ---- SampleFromProbabilities (:153-165) over the whole row
    const int hit = seq_reach(w.p, n, false, 1.0f, a.r[0], chunk, &imisc[1], nullptr);
    if (tid == 0) {
        const int idx = hit >= 0 ? hit : n - 1;
        a.out[0] = idx;
        if (a.next) a.next[0] = idx;
    }
}

// FindNucleus on the sorted (probability, token) pairs, then the pick.
__global__ void __launch_bounds__(SMP_THREADS) sample_nucleus_kernel(SampleArgs a, SampleWork w)
{
    extern __shared__ __align__(16) uint8_t smem[];
    const int n = a.n, tid = threadIdx.x;
    const SampleFullSmem L = sample_full_layout(n, a.window, false);
    float *misc = (float *)(smem + L.misc), *chunk = (float *)(smem + L.chunk);
    int *imisc = (int *)(misc + 32);
    unsigned long long *grp = (unsigned long long *)(smem + L.group);
    const float top_p = a.top_p;
    // first sorted position i whose value equals the next one's
    if (tid == 0) imisc[0] = n;
    __syncthreads();
    for (int i = tid; i + 1 < n; i += SMP_THREADS)
        if (w.kout[i] == w.kout[i + 1]) atomicMin(&imisc[0], i);
    // values written at each sorted position (the aliased buffer): follow i -> idx[i] while idx[i] < i
    for (int i = tid; i < n; i += SMP_THREADS) {
        int j = i, sel = w.iout[i];
        while (sel < j) {
            j = sel;
            sel = w.iout[j];
        }
        w.val[i] = w.p[sel];
    }
    __syncthreads();
    const int t0 = imisc[0];
    const int hit = seq_reach(w.val, n, false, 1.0f, top_p, chunk, &imisc[1], &misc[0]);
    int count = hit >= 0 ? hit + 1 : n;
    const float *vals = w.val;
    const int32_t *idx = w.iout;
    if (t0 <= count - 1) {
        // ---- a tie inside the prefix: replay the selection sort.  pos / at: current position of
        // each token / token at each position; the aliased writes go to w.p in place.
        int32_t *nidx = (int32_t *)w.kin;  // the sorted order this replay produces
        for (int e = tid; e < n; e += SMP_THREADS) {
            w.pos[e] = e;
            w.at[e] = e;
        }
        __syncthreads();
        // thread 0's state: pass i, group start g, running sum, done (count found), group size
        int i = 0, g = 0;
        float cum = 0.0f;
        if (tid == 0) imisc[2] = 0;  // done
        for (;;) {
            if (tid == 0) {
                int done = 0, m = 0;
                auto take = [&](int sel) {  // one pass of the selection sort selects token sel
                    const int o = w.at[i];
                    if (o != sel) {
                        const int ps = w.pos[sel];
                        w.at[ps] = o;
                        w.pos[o] = ps;
                        w.at[i] = sel;
                        w.pos[sel] = i;
                    }
                    nidx[i] = sel;
                    const float v = w.p[sel];  // slot sel holds a written value when sel < i
                    w.p[i] = v;
                    cum = __fadd_rn(cum, v);
                    i++;
                    if (cum >= top_p) done = 1;
                };
                while (!done && g < n) {
                    int ge = g + 1;
                    while (ge < n && w.kout[ge] == w.kout[g]) ge++;
                    if (ge - g == 1) {
                        take(w.iout[g]);
                        g = ge;
                    } else {
                        m = ge - g;
                        break;
                    }
                }
                imisc[2] = done || g >= n ? 1 : 0;
                imisc[3] = g;
                imisc[4] = m;
                misc[0] = cum;
            }
            __syncthreads();
            if (imisc[2]) break;
            const int gs = imisc[3], m = imisc[4];
            if (m > SF_GROUP) {
                if (tid == 0) a.out[0] = SF_TIE_GROUP_TOO_LARGE;
                return;
            }
            // the group's members ordered by their current positions (bitonic sort, ascending)
            int m2 = 2;
            while (m2 < m) m2 <<= 1;
            for (int k = tid; k < m2; k += SMP_THREADS) {
                const int e = k < m ? w.iout[gs + k] : 0;
                grp[k] = k < m ? ((unsigned long long)(uint32_t)w.pos[e] << 32) | (uint32_t)e : ~0ull;
            }
            __syncthreads();
            for (int size = 2; size <= m2; size <<= 1)
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    for (int q = tid; q < m2 / 2; q += SMP_THREADS) {
                        const int lo = 2 * q - (q & (stride - 1)), hi = lo + stride;
                        const bool asc = (lo & size) == 0;
                        const unsigned long long A = grp[lo], B = grp[hi];
                        if ((A > B) == asc) {
                            grp[lo] = B;
                            grp[hi] = A;
                        }
                    }
                    __syncthreads();
                }
            if (tid == 0) {
                int done = 0;
                for (int k = 0; k < m && !done; k++) {
                    const int sel = (int)(uint32_t)grp[k];
                    const int o = w.at[i];
                    if (o != sel) {
                        const int ps = w.pos[sel];
                        w.at[ps] = o;
                        w.pos[o] = ps;
                        w.at[i] = sel;
                        w.pos[sel] = i;
                    }
                    nidx[i] = sel;
                    const float v = w.p[sel];
                    w.p[i] = v;
                    cum = __fadd_rn(cum, v);
                    i++;
                    if (cum >= top_p) done = 1;
                }
                g = gs + m;
                imisc[2] = done || g >= n ? 1 : 0;
                misc[0] = cum;
            }
            __syncthreads();
            if (imisc[2]) break;
        }
        if (tid == 0) imisc[5] = i;  // passes run: the count (n when the sum never reached top_p)
        __syncthreads();
        count = imisc[5];
        vals = w.p;
        idx = nidx;
    }
    __syncthreads();
    // ---- Sample :51-61: the nucleus renormalised (its sum is the running sum where it stopped),
    // or, when it is the whole row, the pick over the overwritten row (a position)
    const float sum = misc[0];
    __syncthreads();
    int out;
    if (count < n) {
        const float inv = __fdiv_rn(1.0f, sum);
        const int h2 = seq_reach(vals, count, true, inv, a.r[0], chunk, &imisc[1], nullptr);
        out = idx[h2 >= 0 ? h2 : count - 1];
    } else {
        const int h2 = seq_reach(vals, n, false, 1.0f, a.r[0], chunk, &imisc[1], nullptr);
        out = h2 >= 0 ? h2 : n - 1;
    }
    if (tid == 0) {
        a.out[0] = out;
        if (a.next) a.next[0] = out;
    }
}

static int launch_sample_full(const SampleArgs &a, int rows, cudaStream_t st)
{
    if (rows != 1) return fail(LLMDOT_E_UNSUPPORTED, "sample: the full-row path takes one row");
    if (!a.work) return fail(LLMDOT_E_INVALID, "sample: the full-row path needs its work buffer");
    if (a.n > (1 << 30) / 8) return fail(LLMDOT_E_UNSUPPORTED, "sample: vocabulary too large for the full-row path");
    const SampleWork w = work_carve(a.work, a.n);
    const bool nucleus = a.top_p < 1.0f;
    const size_t s1 = sample_full_layout(a.n, a.window, true).total, s2 = sample_full_layout(a.n, a.window, false).total;
    if (s1 > 200 * 1024 || s2 > 200 * 1024)
        return fail(LLMDOT_E_UNSUPPORTED, "sample: vocabulary too large for the token bitmap");
    static std::atomic<unsigned long long> attr1{0}, attr2{0};
    LLMDOT_CUDA_TRY(smem_attr_once(attr1, sample_probs_kernel, 200 * 1024));
    LLMDOT_CUDA_TRY(smem_attr_once(attr2, sample_nucleus_kernel, 200 * 1024));
    sample_probs_kernel<<<1, SMP_THREADS, s1, st>>>(a, w, nucleus ? 1 : 0);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    if (!nucleus) return LLMDOT_OK;
    size_t tb = w.cub_bytes;
    LLMDOT_CUDA_TRY(cub::DeviceRadixSort::SortPairsDescending(w.cub, tb, w.kin, w.kout, w.iin, w.iout, a.n, 0, 32, st));
    sample_nucleus_kernel<<<1, SMP_THREADS, s2, st>>>(a, w);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

// candidates, a power of two: at least one per warp (the greedy path parks warp maxima there)
static int k2_for(int k)
{
    int k2 = SMP_THREADS / 32;
    while (k2 < k) k2 <<= 1;
    return k2;
}

size_t sample_smem(int n, int window, int top_k)
{
    return (size_t)sample_layout(n, window, k2_for(top_k > 0 ? top_k : 1)).total;
}

int launch_sample(const SampleArgs &a, int rows, cudaStream_t st)
{
    if (rows < 1 || a.n < 1 || !a.logits || !a.out || !a.r)
        return fail(LLMDOT_E_INVALID, "sample: bad arguments");
    if (a.window < 0 || a.window > SAMPLE_MAX_WINDOW)
        return fail(LLMDOT_E_UNSUPPORTED, "sample: repeat window above " + std::to_string(SAMPLE_MAX_WINDOW));
    if (sample_full_row(a.temperature, a.top_k, a.n)) return launch_sample_full(a, rows, st);
    if (a.temperature > 0.0f && a.top_k > SAMPLE_MAX_TOP_K)
        return fail(LLMDOT_E_UNSUPPORTED, "sample: top_k above " + std::to_string(SAMPLE_MAX_TOP_K) +
                                              " (and below the vocabulary) is not on the device");
    const int k2 = k2_for(a.top_k > 0 ? a.top_k : 1);
    const size_t sm = sample_smem(a.n, a.window, a.top_k);
    if (sm > 200 * 1024) return fail(LLMDOT_E_UNSUPPORTED, "sample: vocabulary too large for the token bitmap");
    static std::atomic<unsigned long long> attr_done{0};
    LLMDOT_CUDA_TRY(smem_attr_once(attr_done, sample_kernel, 200 * 1024));
    sample_kernel<<<rows, SMP_THREADS, sm, st>>>(a, k2);
    LLMDOT_CUDA_TRY(cudaGetLastError());
    return LLMDOT_OK;
}

}  // namespace llmdot
