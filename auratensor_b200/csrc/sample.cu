// Sampler.sample (inference/Sampler.java:37-121) on the device, one CTA of
// 1024 threads per logits row, with the reference's float arithmetic:
//  1. repetition penalty over the history, in place (logits / p when
//     positive, else * p, once per occurrence);
//  2. greedy fast path (temperature 0, or topK 1 with topP >= 1): the first
//     index of the maximum, a NaN winning only at index 0;
//  3. adj = logits * (1 / T); the candidates are the topK largest adj in the
//     order of the reference's stable descending sort (Double.compare: NaN
//     above +inf, -0.0 below 0.0; equal values keep index order). They are
//     found by a radix select of the topK-th key (four 8-bit passes over the
//     row), an index-ordered compaction of the keys above and equal to it,
//     and a bitonic sort of the at most 1024 candidates;
//  4. probs = (float) exp((double)(adj - max)) in parallel, then one thread
//     runs the sequential float sums of the reference (sumExp, the top-p
//     running sum, the renormalization, the CDF scan with r).
// r is the caller's draw for the row (the reference draws it from a fresh
// java.util.Random(seed) on every call, so a fixed seed gives a fixed r); an
// unseeded row instead advances its own java.util.Random state per call.
#include <cstdint>

#include "at_internal.h"
#include "dev_common.cuh"

namespace at {

namespace {

constexpr int SMP_THREADS = 1024;
constexpr int SMP_KMAX = 1024;

// Order-preserving bits with Double.compare's order: NaN above +inf.
__device__ __forceinline__ uint32_t dc_bits(float v) {
    if (v != v) return 0xFFFFFFFFu;
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exclusive prefix sum over the block (values per thread); returns the total.
__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int* excl) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = (lane < SMP_THREADS / 32) ? s_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < SMP_THREADS / 32) s_warp[lane] = w;  // inclusive warp totals
    }
    __syncthreads();
    const int before = (warp > 0 ? s_warp[warp - 1] : 0) + x - v;
    *excl = before;
    const int total = s_warp[SMP_THREADS / 32 - 1];
    __syncthreads();
    return total;
}

__global__ void __launch_bounds__(SMP_THREADS) sample_kernel(float* __restrict__ logits, int V, int stride,
                                                             const SampleRow* __restrict__ rows,
                                                             int* __restrict__ out) {
    __shared__ unsigned long long s_cand[SMP_KMAX];
    __shared__ float s_prob[SMP_KMAX];
    __shared__ unsigned s_hist[256];
    __shared__ int s_warp[32];
    __shared__ unsigned long long s_best[32];
    __shared__ uint32_t s_prefix;
    __shared__ int s_remaining;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = blockIdx.x;
    const SampleRow row = rows[b];
    float* lg = logits + (size_t)b * stride;

    // 1) repetition penalty (Sampler.java:44-53). The reference applies it
    // once per history entry, in order; every application to a token is the
    // same map (v > 0 ? v / p : v * p), so applying it count(t) times to each
    // distinct t in one thread gives the same floats. Counts go through the
    // row's zeroed [V] array, which each token's leader zeroes again.
    const int hist_len = row.hist_len ? *row.hist_len : 0;
    if (row.penalty != 1.0f && row.hist && row.cnt && hist_len > 0) {
        for (int i = tid; i < hist_len; i += SMP_THREADS) {
            const int t = row.hist[i];
            if (t >= 0 && t < V) atomicAdd(&row.cnt[t], 1);
        }
        __syncthreads();
        for (int i = tid; i < hist_len; i += SMP_THREADS) {
            const int t = row.hist[i];
            if (t < 0 || t >= V) continue;
            const int c = atomicExch(&row.cnt[t], 0);
            if (c > 0) {
                float v = lg[t];
                for (int j = 0; j < c; ++j) v = (v > 0) ? __fdiv_rn(v, row.penalty) : __fmul_rn(v, row.penalty);
                lg[t] = v;
            }
        }
    }
    __syncthreads();

    // 2) greedy fast path (Sampler.java:56-67)
    if (row.temperature == 0.0f || (row.top_k == 1 && row.top_p >= 1.0f)) {
        unsigned long long best = 0ull;
        for (int i = tid; i < V; i += SMP_THREADS) {
            const unsigned long long k = ((unsigned long long)ordered_bits(lg[i]) << 32) | (0xFFFFFFFFu - (uint32_t)i);
            best = k > best ? k : best;
        }
        if (tid == 0 && lg[0] != lg[0]) best = ~0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0) s_best[warp] = best;
        __syncthreads();
        if (tid == 0) {
            for (int w = 0; w < SMP_THREADS / 32; ++w) best = s_best[w] > best ? s_best[w] : best;
            out[b] = key_index(best);
        }
        return;
    }

    // 3) candidates: the k largest adj in stable descending order
    const float inv_t = __fdiv_rn(1.0f, row.temperature);
    const int k = min(row.top_k, V);
    if (k < 1 || k > SMP_KMAX) {  // the host refuses these; never index past the candidate buffer
        if (tid == 0) out[b] = -1;
        return;
    }
    if (tid == 0) {
        s_prefix = 0u;
        s_remaining = k;
    }
    uint32_t mask = 0u;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += SMP_THREADS) s_hist[i] = 0u;
        __syncthreads();
        const uint32_t prefix = s_prefix;
        for (int i = tid; i < V; i += SMP_THREADS) {
            const uint32_t key = dc_bits(__fmul_rn(lg[i], inv_t));
            if ((key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & 0xFFu], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            int rem = s_remaining;
            int bin = 255;
            for (; bin > 0; --bin) {
                if ((int)s_hist[bin] >= rem) break;
                rem -= (int)s_hist[bin];
            }
            s_remaining = rem;  // keys still needed from this bin
            s_prefix = prefix | ((uint32_t)bin << shift);
        }
        mask |= 0xFFu << shift;
        __syncthreads();
    }
    const uint32_t thr = s_prefix;     // the k-th largest key
    const int need_eq = s_remaining;   // keys equal to thr to take, lowest indices first
    // index-ordered compaction: each thread owns a contiguous index range
    const int chunk = (V + SMP_THREADS - 1) / SMP_THREADS;
    const int i0 = min(V, tid * chunk), i1 = min(V, i0 + chunk);
    int n_gt = 0, n_eq = 0;
    for (int i = i0; i < i1; ++i) {
        const uint32_t key = dc_bits(__fmul_rn(lg[i], inv_t));
        n_gt += key > thr;
        n_eq += key == thr;
    }
    int gt_before, eq_before;
    const int total_gt = block_exclusive_scan(n_gt, s_warp, &gt_before);
    block_exclusive_scan(n_eq, s_warp, &eq_before);
    for (int i = i0; i < i1; ++i) {
        const uint32_t key = dc_bits(__fmul_rn(lg[i], inv_t));
        const unsigned long long ck = ((unsigned long long)key << 32) | (0xFFFFFFFFu - (uint32_t)i);
        if (key > thr) {
            s_cand[gt_before++] = ck;
        } else if (key == thr) {
            if (eq_before < need_eq) s_cand[total_gt + eq_before] = ck;
            ++eq_before;
        }
    }
    for (int i = k + tid; i < SMP_KMAX; i += SMP_THREADS) s_cand[i] = 0ull;  // padding sorts last
    __syncthreads();
    // bitonic sort, descending
    for (int size = 2; size <= SMP_KMAX; size <<= 1) {
        for (int stride2 = size >> 1; stride2 > 0; stride2 >>= 1) {
            for (int i = tid; i < SMP_KMAX; i += SMP_THREADS) {
                const int j = i ^ stride2;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned long long a = s_cand[i], c = s_cand[j];
                    if (desc ? (a < c) : (a > c)) {
                        s_cand[i] = c;
                        s_cand[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    // 4) probabilities (Sampler.java:79-110)
    const int top_idx = (int)(0xFFFFFFFFu - (uint32_t)(s_cand[0] & 0xFFFFFFFFull));
    const float max_logit = __fmul_rn(lg[top_idx], inv_t);
    for (int i = tid; i < k; i += SMP_THREADS) {
        const int idx = (int)(0xFFFFFFFFu - (uint32_t)(s_cand[i] & 0xFFFFFFFFull));
        const float a = __fmul_rn(lg[idx], inv_t);
        s_prob[i] = (float)exp((double)__fsub_rn(a, max_logit));
    }
    __syncthreads();
    if (tid == 0) {
        float sum_exp = 0.0f;
        for (int i = 0; i < k; ++i) sum_exp = __fadd_rn(sum_exp, s_prob[i]);
        int cutoff = k;
        if (row.top_p < 1.0f) {
            float running = 0.0f;
            for (int i = 0; i < k; ++i) {
                running = __fadd_rn(running, s_prob[i]);
                if (__fdiv_rn(running, sum_exp) >= row.top_p) {
                    cutoff = i + 1;
                    break;
                }
            }
        }
        float new_sum = 0.0f;
        for (int i = 0; i < cutoff; ++i) new_sum = __fadd_rn(new_sum, s_prob[i]);
        float r = row.r;
        if (row.rng) {  // java.util.Random.nextFloat: next(24) / 2^24
            const unsigned long long st = (*row.rng * 0x5DEECE66DULL + 0xBULL) & ((1ULL << 48) - 1);
            *row.rng = st;
            r = (float)(int)(st >> 24) * 0x1.0p-24f;
        }
        float cum = 0.0f;
        int pick = cutoff - 1;
        for (int i = 0; i < cutoff; ++i) {
            cum = __fadd_rn(cum, __fdiv_rn(s_prob[i], new_sum));
            if (r <= cum) {
                pick = i;
                break;
            }
        }
        out[b] = (int)(0xFFFFFFFFu - (uint32_t)(s_cand[pick] & 0xFFFFFFFFull));
    }
}

// Sampled tokens -> the next step's inputs: token, position + 1, the output
// sequence and the penalty history of each row.
__global__ void sample_advance_kernel(const int* __restrict__ picked, int B, int* __restrict__ tokens,
                                      int64_t* __restrict__ pos, int* __restrict__ seq, int seq_stride, int* step,
                                      int* __restrict__ hist, int hist_stride, int* __restrict__ hist_len,
                                      const int* __restrict__ append) {
    const int b = threadIdx.x;
    const int st = step ? *step : 0;
    if (b < B) {
        const int t = picked[b];
        tokens[b] = t;
        pos[b] += 1;
        if (seq) seq[(size_t)b * seq_stride + st] = t;
        if (hist && (!append || append[b]) && hist_len[b] < hist_stride) hist[(size_t)b * hist_stride + hist_len[b]++] = t;
    }
    __syncthreads();
    if (b == 0 && step) *step = st + 1;
}

}  // namespace

void launch_sample(float* logits_dev, int B, int V, int stride, const SampleRow* rows_dev, int* out_dev,
                   cudaStream_t s) {
    sample_kernel<<<B, SMP_THREADS, 0, s>>>(logits_dev, V, stride, rows_dev, out_dev);
    AT_CUDA(cudaGetLastError());
}

void launch_sample_advance(const int* picked, int B, int* tokens, int64_t* pos, int* seq, int seq_stride, int* step,
                           int* hist, int hist_stride, int* hist_len, const int* append, cudaStream_t s) {
    sample_advance_kernel<<<1, 32, 0, s>>>(picked, B, tokens, pos, seq, seq_stride, step, hist, hist_stride, hist_len,
                                           append);
    AT_CUDA(cudaGetLastError());
}

int sample_k_max() { return SMP_KMAX; }

}  // namespace at
