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
// Temperature <= 0 is the greedy argmax of the softcapped row (lowest index on ties).  Equal values
// at the k-th place are taken lowest index first and equal winners are ordered by index; the
// reference orders them by its replacement scan instead (FindTopK :83-127), which only matters for
// exactly tied logits.  The top-p-only path (top_k <= 0 or >= n) is not on the device.
#include "sample.cuh"

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
    const float *x = a.logits + (size_t)row * a.ld;
    const int nvec = n - n % 8;
    auto capped = [&](int i) {
        const float v = x[i];
        return a.has_cap ? softcap_ref(v, a.cap, a.inv_cap, i < nvec) : v;
    };

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

    // ---- repeat penalty (ApplyRepeatPenalty :64-81): the last `window` tokens, in order.  The
    // window's values are loaded in parallel (into the candidate buffer, not yet in use);
    // one thread then applies the penalty occurrence by occurrence.
    for (int i = tid; i < (n + 31) / 32; i += SMP_THREADS) bitmap[i] = 0u;
    const bool pen = a.penalty != 1.0f && window > 0 && a.recent;
    const int plen = pen ? a.recent_len[row] : 0, p0 = max(0, plen - window);
    const int32_t *rec = pen ? a.recent + (size_t)row * a.recent_ld : nullptr;
    float *wval = (float *)cand;  // window values, index i - p0 (the candidates come later)
    for (int i = p0 + tid; i < plen; i += SMP_THREADS) {
        const int t = rec[i];
        wval[i - p0] = (t >= 0 && t < n) ? capped(t) : 0.0f;
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
        hist[256] = np;
    }
    __syncthreads();
    const int np = hist[256];
    // the scaled value of token i (VectorMath.Scale: x * (1/T) in every lane)
    auto value = [&](int i) {
        float v;
        if (np && ((bitmap[i >> 5] >> (i & 31)) & 1u)) {
            int j = 0;
            while (ptok[j] != i) j++;
            v = pval[j];
        } else {
            v = capped(i);
        }
        return __fmul_rn(v, a.inv_temp);
    };

    const int k = a.top_k;
    int sort_n = k2;  // entries of cand to sort
    bool fast = false;
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
    if (a.temperature > 0.0f && (a.top_k <= 0 || a.top_k >= a.n || a.top_k > SAMPLE_MAX_TOP_K))
        return fail(LLMDOT_E_UNSUPPORTED, "sample: temperature > 0 needs 0 < top_k < vocabulary and top_k <= " +
                                              std::to_string(SAMPLE_MAX_TOP_K) + " on the device");
    if (a.window < 0 || a.window > SAMPLE_MAX_WINDOW)
        return fail(LLMDOT_E_UNSUPPORTED, "sample: repeat window above " + std::to_string(SAMPLE_MAX_WINDOW));
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
