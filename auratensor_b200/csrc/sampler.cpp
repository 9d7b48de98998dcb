// Sampler.sample (inference/Sampler.java:37-121) on the host, with the same
// float arithmetic and the java.util.Random generator it seeds per call.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>
#if defined(__SSE2__)
#include <immintrin.h>
#endif

#include "at_internal.h"

namespace {

// java.util.Random: the 48-bit LCG specified in the Java SE API documentation.
struct JavaRandom {
    uint64_t seed;
    explicit JavaRandom(int64_t s) : seed(((uint64_t)s ^ 0x5DEECE66DULL) & ((1ULL << 48) - 1)) {}
    int32_t next(int bits) {
        seed = (seed * 0x5DEECE66DULL + 0xBULL) & ((1ULL << 48) - 1);
        return (int32_t)(int64_t)(seed >> (48 - bits));
    }
    float next_float() { return (float)next(24) / (float)(1 << 24); }
};

// Order-preserving bits of a float under Double.compare: NaN above +inf,
// -0.0 below 0.0, every NaN equal.
uint32_t double_compare_bits(float v) {
    if (std::isnan(v)) return 0xFFFFFFFFu;
    uint32_t u;
    std::memcpy(&u, &v, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Sampler.java's greedy loop (inference/Sampler.java:56-67): scanning left
// to right, an element replaces the running maximum only if it is greater.
// So a NaN wins only at index 0 (nothing is greater than it, and it is
// greater than nothing), later NaNs are skipped, and equal values (-0.0 and
// 0.0 included) keep the first index. Computed as the maximum over 16
// independent lanes seeded with element 0 (no compare chain carried from one
// element to the next) and then the first index holding that maximum: the
// same index as the scan. With SSE, lane update max(x, m) is MAXPS(x, m),
// which yields m when x is NaN or equal, exactly the scan's rule.
int greedy_index(const float* x, int n) {
    const float x0 = x[0];
    if (std::isnan(x0)) return 0;
    constexpr int W = 16;
    float m[W];
    int i = 0;
#if defined(__SSE2__)
    __m128 a0 = _mm_set1_ps(x0), a1 = a0, a2 = a0, a3 = a0;
    for (; i + W <= n; i += W) {
        a0 = _mm_max_ps(_mm_loadu_ps(x + i), a0);
        a1 = _mm_max_ps(_mm_loadu_ps(x + i + 4), a1);
        a2 = _mm_max_ps(_mm_loadu_ps(x + i + 8), a2);
        a3 = _mm_max_ps(_mm_loadu_ps(x + i + 12), a3);
    }
    _mm_storeu_ps(m, a0);
    _mm_storeu_ps(m + 4, a1);
    _mm_storeu_ps(m + 8, a2);
    _mm_storeu_ps(m + 12, a3);
#else
    for (int j = 0; j < W; ++j) m[j] = x0;
    for (; i + W <= n; i += W)
        for (int j = 0; j < W; ++j) m[j] = x[i + j] > m[j] ? x[i + j] : m[j];
#endif
    for (; i < n; ++i) m[0] = x[i] > m[0] ? x[i] : m[0];
    float top = m[0];
    for (int j = 1; j < W; ++j) top = m[j] > top ? m[j] : top;
    int k = 0;
#if defined(__SSE2__)
    const __m128 t = _mm_set1_ps(top);
    for (; k + W <= n; k += W) {
        const int hit = _mm_movemask_ps(_mm_cmpeq_ps(_mm_loadu_ps(x + k), t)) |
                        (_mm_movemask_ps(_mm_cmpeq_ps(_mm_loadu_ps(x + k + 4), t)) << 4) |
                        (_mm_movemask_ps(_mm_cmpeq_ps(_mm_loadu_ps(x + k + 8), t)) << 8) |
                        (_mm_movemask_ps(_mm_cmpeq_ps(_mm_loadu_ps(x + k + 12), t)) << 12);
        if (hit) return k + __builtin_ctz((unsigned)hit);
    }
#endif
    for (; k < n; ++k)
        if (x[k] == top) return k;
    return 0;  // not reached: top is one of the elements
}

}  // namespace

namespace at {
float sampler_r(int64_t seed) {
    int64_t s = seed;
    if (s == 0) s = (int64_t)std::chrono::steady_clock::now().time_since_epoch().count();
    return JavaRandom(s).next_float();
}
}  // namespace at

extern "C" int at_sample(float* logits, int vocab, const int* history, int n_history, float temperature, int top_k,
                         float top_p, float rep_penalty, int64_t seed, int* out_token) {
    return at::guard([&] {
        AT_REQUIRE(logits && out_token && vocab > 0, AT_ERR_INVALID_ARG, "bad sampler argument");
        // 1) repetition penalty, in place (Sampler.java:44-53)
        if (rep_penalty != 1.0f && history && n_history > 0) {
            for (int i = 0; i < n_history; ++i) {
                const int t = history[i];
                if (t >= 0 && t < vocab) {
                    if (logits[t] > 0) logits[t] = logits[t] / rep_penalty;
                    else logits[t] = logits[t] * rep_penalty;
                }
            }
        }
        // 2) greedy fast path (Sampler.java:56-67)
        if (temperature == 0.0f || (top_k == 1 && top_p >= 1.0f)) {
            *out_token = greedy_index(logits, vocab);
            return;
        }
        // 3) temperature, stable descending sort, top-k, top-p (Sampler.java:71-110)
        const float inv_t = 1.0f / temperature;
        std::vector<float> adj(vocab);
        for (int i = 0; i < vocab; ++i) adj[i] = logits[i] * inv_t;
        // Comparator.comparingDouble(..).reversed() under List.sort (stable):
        // descending in Double.compare's order, equal values in index order.
        // Only the first k places are read, and they are the k largest of the
        // keys (order bits, then the complemented index), sorted.
        const int k = std::min(top_k, vocab);
        AT_REQUIRE(k >= 1, AT_ERR_INVALID_ARG, "topK must be positive");
        std::vector<uint64_t> keys(vocab);
        for (int i = 0; i < vocab; ++i) keys[i] = ((uint64_t)double_compare_bits(adj[i]) << 32) | (0xFFFFFFFFu - (uint32_t)i);
        auto desc = [](uint64_t a, uint64_t b) { return a > b; };
        if (k < vocab) std::nth_element(keys.begin(), keys.begin() + (k - 1), keys.end(), desc);
        std::sort(keys.begin(), keys.begin() + k, desc);
        std::vector<int> idx(k);
        for (int i = 0; i < k; ++i) idx[i] = (int)(0xFFFFFFFFu - (uint32_t)(keys[i] & 0xFFFFFFFFu));
        const float max_logit = adj[idx[0]];
        std::vector<float> probs(k);
        float sum_exp = 0.0f;
        for (int i = 0; i < k; ++i) {
            const float p = (float)std::exp((double)(adj[idx[i]] - max_logit));
            probs[i] = p;
            sum_exp += p;
        }
        int cutoff = k;
        if (top_p < 1.0f) {
            float running = 0.0f;
            const float total = sum_exp;
            for (int i = 0; i < k; ++i) {
                running += probs[i];
                if (running / total >= top_p) { cutoff = i + 1; break; }
            }
        }
        float new_sum = 0.0f;
        for (int i = 0; i < cutoff; ++i) new_sum += probs[i];
        for (int i = 0; i < cutoff; ++i) probs[i] /= new_sum;
        // 4) r from a fresh java.util.Random(seed); seed 0 means an unseeded generator
        int64_t s = seed;
        if (s == 0) s = (int64_t)std::chrono::steady_clock::now().time_since_epoch().count();
        const float r = JavaRandom(s).next_float();
        float cum = 0.0f;
        for (int i = 0; i < cutoff; ++i) {
            cum += probs[i];
            if (r <= cum) { *out_token = idx[i]; return; }
        }
        *out_token = idx[cutoff - 1];
    });
}
