// Device-resident Llama decode (LlamaModel.forwardStep, inference/LlamaModel.java:141-308)
// with Megatron tensor parallelism over NCCL.
//
// Per step and per layer the work is five kernels plus, under tensor
// parallelism, two all-reduces:
//   1. QKV GEMV (orientation T) with the attention RMSNorm in its prologue
//      (x = norm(x + y), F7 residual semantics) and RoPE + KV append in its
//      epilogue;
//   2. split-KV attention over the fp32 KV cache;  3. log-sum-exp combine;
//   4. wo GEMV (T) -> y  [all-reduce y];
//   5. gate/up GEMV (N) with the FFN RMSNorm prologue and SiLU*up epilogue;
//   6. down GEMV (N) -> y  [all-reduce y].
// The embedding row dequant starts the step, the lm_head GEMV with the output
// norm prologue and an argmax end it. The whole sequence is captured once per
// batch size into a CUDA graph and replayed; token ids and positions are read
// from device memory so the graph does not change between steps.
#include <dlfcn.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cooperative_groups.h>
#include <cuda_bf16.h>

#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "at_internal.h"
#include "dev_common.cuh"
#include "nccl_dl.h"

namespace at {

// ---------------------------------------------------------------------------
// NCCL loader
// ---------------------------------------------------------------------------
const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    static std::string err;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            err = std::string("cannot load libnccl.so.2: ") + dlerror();
            return;
        }
#define AT_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name))
        AT_SYM(GetUniqueId, "ncclGetUniqueId");
        AT_SYM(CommInitRank, "ncclCommInitRank");
        AT_SYM(CommDestroy, "ncclCommDestroy");
        AT_SYM(CommAbort, "ncclCommAbort");
        AT_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
        AT_SYM(AllReduce, "ncclAllReduce");
        AT_SYM(AllGather, "ncclAllGather");
        AT_SYM(GetErrorString, "ncclGetErrorString");
#undef AT_SYM
        if (!api.GetUniqueId || !api.CommInitRank || !api.AllReduce || !api.AllGather || !api.CommDestroy)
            err = "libnccl.so.2 lacks required symbols";
    });
    if (!err.empty()) fail(AT_ERR_NCCL, err);
    return api;
}

void nccl_check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess) {
        const char* s = nccl().GetErrorString ? nccl().GetErrorString(r) : "?";
        fail(AT_ERR_NCCL, std::string(what) + ": " + s);
    }
}

namespace {

constexpr int CH = 32;  // KV positions per attention CTA

// ---------------------------------------------------------------------------
// Step kernels
// ---------------------------------------------------------------------------
// writeTokenEmbedding (inference/LlamaModel.java:181-186): one dequantized row
// of token_embd into xa; y <- 0 so the first layer's prologue reads x + 0.
// Also advances the step sequence number the tensor-parallel all-reduces
// match on (every rank runs the same steps, so the numbers agree).
template <int QT>
__global__ void embed_kernel(const uint8_t* __restrict__ tiles, QTileMap map, const int* __restrict__ tokens, int d,
                             float* __restrict__ xa, float* __restrict__ y, unsigned long long* __restrict__ argkeys,
                             unsigned* __restrict__ step) {
    const int b = blockIdx.x;
    if (threadIdx.x == 0 && argkeys) argkeys[b] = 0ull;
    if (b == 0 && threadIdx.x == 0 && step) *step += 1u;
    const int64_t tok = tokens[b];
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        int64_t d_off, q_off;
        map.offsets(tok, i >> 5, &d_off, &q_off);
        const int w = i & 31;
        int q;
        if constexpr (QT == AT_GGML_Q4_0) {
            const uint32_t pack = tiles[q_off + (w >> 1)];
            q = ((w & 1) ? (int)(pack >> 4) : (int)(pack & 0xF)) - 8;
        } else {
            q = (int)(int8_t)tiles[q_off + w];
        }
        const uint32_t h = (uint32_t)tiles[d_off] | ((uint32_t)tiles[d_off + 1] << 8);
        xa[(size_t)b * d + i] = __fmul_rn((float)q, fp16_ftz(h));
        y[(size_t)b * d + i] = 0.f;
    }
}

__device__ __forceinline__ float exp_ref(float v) { return (float)exp((double)v); }

// LlamaModel.attention (inference/LlamaModel.java:255-297) split over KV
// chunks of CH positions: for the G query heads sharing KV head `kvh`, scores
// over positions [p0, p0 + n) = (K q) * scale, chunk max m, l = sum exp(s - m),
// o = sum exp(s - m) V. K and V of the chunk are staged in shared memory with
// all of the CTA's 128-bit loads in flight at once.
// CHK positions per CTA (K and V of the chunk staged in dynamic shared
// memory, attn_smem_bytes).
// MODE 0 (prompt path): the chunk partials go to `part` for attn_combine_kernel.
// MODE 1 (decode step): the last CTA of a (sequence, KV head) to finish its
// chunk (ticket per pair in `cnt`, reset by that CTA) merges the chunk
// partials of the G heads into `att` (the log-sum-exp combine of
// attn_combine_kernel, without a second launch). Needs G * chunks <= CH * HD
// (the merge weights reuse the K staging buffer).
// MODE 2 (decode step, CHK = 64, launched with clusters of CS CTAs along the chunks):
// the CTAs of a cluster keep their partials in shared memory; after a cluster
// barrier every rank merges a slice of the G * HD outputs, reading one float4
// of each rank's partial per thread through distributed shared memory. When
// one cluster covers the sequence the ranks write `att` directly; otherwise
// the cluster partials (one per CS * CHK positions) are merged as in MODE 1
// by rank 0 of the last cluster to arrive. A cluster
// whose first chunk lies past the sequence exits as a whole; idle CTAs of a
// partly used cluster take part in its barriers with an empty partial.
// 16-byte asynchronous copy global -> shared (L2 only).
__device__ __forceinline__ void cp_async16_smem(void* smem, const void* g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(g)
                 : "memory");
}

// Dynamic shared memory of attn_split_kernel: K (rows padded by two float4)
// and V of a chunk of chk positions.
constexpr size_t attn_smem_bytes(int hd, int chk) { return (size_t)chk * (hd / 4 + 2 + hd / 4) * 16; }
constexpr int kAttnClusterChunk = 64;  // positions per CTA of the cluster-merged decode attention

// Four K or V elements of a Q8_0 KV cache row chunk (float4 index i of the
// chunk starting at quant pointer qb, scales sb of the same elements / 32).
__device__ __forceinline__ float4 kv_dq4(const int8_t* __restrict__ qb, const uint16_t* __restrict__ sb, int i) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(qb + 4 * (size_t)i);
    const float d = fp16_ftz_fast(sb[i >> 3]);
    return make_float4(__fmul_rn((float)(int8_t)(w & 0xFFu), d), __fmul_rn((float)(int8_t)((w >> 8) & 0xFFu), d),
                       __fmul_rn((float)(int8_t)((w >> 16) & 0xFFu), d), __fmul_rn((float)(int8_t)(w >> 24), d));
}

// KVQ: kc / vc are the int8 quants of a Q8_0 KV cache (same element index)
// and ksc / vsc its fp16 scales; the chunk's rows are dequantized into the
// same shared-memory rows the fp32 cache is copied into.
template <int HD, int MODE = 0, int CHK = CH, bool KVQ = false>
__global__ void __launch_bounds__(256) attn_split_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                                         const float* __restrict__ vc,
                                                         const int64_t* __restrict__ pos, float* __restrict__ part,
                                                         int Hl, int Hkvl, int ctx, int64_t slot_stride,
                                                         int nchunk_max, float scale,
                                                         unsigned* __restrict__ cnt = nullptr,
                                                         float* __restrict__ att = nullptr,
                                                         const uint16_t* __restrict__ ksc = nullptr,
                                                         const uint16_t* __restrict__ vsc = nullptr) {
    constexpr int G_MAX = 8;
    constexpr int F4 = HD / 4;  // float4 per row
    // K rows padded by two float4: the 8 lanes of a quarter-warp (4 rows x 2
    // interleaved halves) read 8 distinct 16-byte bank groups.
    constexpr int KP = F4 + 2;
    static_assert(CHK % 16 == 0 && CHK <= 64, "a warp's 16 score pairs share one head");
    // K and V of the chunk in dynamic shared memory: CHK x (KP + F4) float4
    extern __shared__ __align__(16) float4 kv_smem[];
    float4 (*ks)[KP] = reinterpret_cast<float4 (*)[KP]>(kv_smem);
    float4 (*vs)[F4] = reinterpret_cast<float4 (*)[F4]>(kv_smem + CHK * KP);
    __shared__ __align__(16) float4 qs[G_MAX][F4];
    __shared__ float sc[G_MAX][CHK];
    __shared__ float s_m[G_MAX], s_l[G_MAX];
    __shared__ __align__(16) float s_o[MODE == 2 ? G_MAX : 1][HD];  // MODE 2: this CTA's partial
    __shared__ float s_cm[G_MAX], s_cl[G_MAX];                       // MODE 2: cluster statistics
    __shared__ int s_last;
    const int kvh = blockIdx.x, chunk = blockIdx.y, b = blockIdx.z;
    const int G = Hl / Hkvl;
    // MODE 2 lets the next kernel launch only once its chunk work is done: the
    // next kernel's CTAs copy their weights before their own wait, and that
    // flood of copies slows this kernel's shared-memory work on the same SM
    if constexpr (MODE != 2) pdl_trigger();
    // The position was advanced by an earlier step; the rows of positions
    // before it were appended by earlier steps, so they are loaded before
    // waiting on the QKV kernel, which appends row P - 1 and writes q.
    const int64_t P = pos[b] + 1;
    const int64_t p0 = (int64_t)chunk * CHK;
    int cs = 1, crank = 0;
    if constexpr (MODE == 2) {
        cs = (int)cooperative_groups::this_cluster().num_blocks();  // cluster dims (1, cs, 1)
        crank = chunk % cs;
        if ((int64_t)(chunk - crank) * CHK >= P) return;  // the whole cluster is past the sequence
    } else {
        if (p0 >= P) return;
    }
    const bool active = p0 < P;  // MODE 2 only can be false here (CTA-uniform)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (active) {
    const int n = (int)((P - p0) < CHK ? (P - p0) : CHK);
    const int n_past = (p0 + n == P) ? n - 1 : n;
    const size_t e0 = (size_t)b * slot_stride + ((size_t)kvh * ctx + p0) * HD;  // first element of the chunk
    const float4* qbase = reinterpret_cast<const float4*>(q + (size_t)b * Hl * HD + (size_t)kvh * G * HD);
    if constexpr (KVQ) {
        // rows before P - 1 are dequantized before the wait
        const int8_t* kq = reinterpret_cast<const int8_t*>(kc) + e0;
        const int8_t* vq = reinterpret_cast<const int8_t*>(vc) + e0;
        const uint16_t* kss = ksc + (e0 >> 5);
        const uint16_t* vss = vsc + (e0 >> 5);
        for (int i = tid; i < n_past * F4; i += 256) {
            ks[i / F4][i % F4] = kv_dq4(kq, kss, i);
            vs[i / F4][i % F4] = kv_dq4(vq, vss, i);
        }
        pdl_wait();
        for (int i = n_past * F4 + tid; i < n * F4; i += 256) {
            ks[i / F4][i % F4] = kv_dq4(kq, kss, i);
            vs[i / F4][i % F4] = kv_dq4(vq, vss, i);
        }
    } else {
        const float4* kbase = reinterpret_cast<const float4*>(kc + e0);
        const float4* vbase = reinterpret_cast<const float4*>(vc + e0);
        // K and V rows go straight to shared memory (cp.async, all in flight, no
        // registers); rows before P - 1 are copied before the wait
        for (int i = tid; i < n_past * F4; i += 256) {
            cp_async16_smem(&ks[i / F4][i % F4], kbase + i);
            cp_async16_smem(&vs[i / F4][i % F4], vbase + i);
        }
        pdl_wait();
        for (int i = n_past * F4 + tid; i < n * F4; i += 256) {
            cp_async16_smem(&ks[i / F4][i % F4], kbase + i);
            cp_async16_smem(&vs[i / F4][i % F4], vbase + i);
        }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int i = tid; i < G * F4; i += 256) qs[i / F4][i % F4] = qbase[i];
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // scores: lanes 2p and 2p + 1 take (position p % CHK, head p / CHK), each
    // half of head_dim (interleaved float4), summed with one shuffle
    for (int pr = tid >> 1; pr < CHK * G; pr += 128) {
        const int i = pr & (CHK - 1), g = pr / CHK, h = tid & 1;
        float acc = 0.f;
        if (i < n) {
#pragma unroll
            for (int j = 0; j < F4 / 2; ++j) {
                const float4 kv = ks[i][2 * j + h], qv = qs[g][2 * j + h];
                acc = fmaf(kv.x, qv.x, acc);
                acc = fmaf(kv.y, qv.y, acc);
                acc = fmaf(kv.z, qv.z, acc);
                acc = fmaf(kv.w, qv.w, acc);
            }
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        if (h == 0 && i < n) sc[g][i] = __fmul_rn(acc, scale);
    }
    __syncthreads();
    if (warp < G) {
        const int g = warp;
        float m = -INFINITY;
        for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[g][i]);
        m = warp_max(m);
        float l = 0.f;
        for (int i = lane; i < n; i += 32) {
            const float e = exp_ref(__fsub_rn(sc[g][i], m));
            sc[g][i] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { s_m[g] = m; s_l[g] = l; }
    }
    __syncthreads();
    // o = sum_i p_i V_i: a thread takes outputs o0 and o0 + 256, each summed
    // as even and odd positions (four independent FMA chains)
    const float* vsf = reinterpret_cast<const float*>(vs);
    for (int o0 = tid; o0 < G * HD; o0 += 512) {
        const int o1 = o0 + 256;
        const bool has1 = o1 < G * HD;
        const int g0 = o0 / HD, d0 = o0 - g0 * HD;
        const int g1 = has1 ? o1 / HD : g0, d1 = has1 ? o1 - g1 * HD : d0;
        float a0 = 0.f, a1 = 0.f, c0 = 0.f, c1 = 0.f;
        int i = 0;
        for (; i + 2 <= n; i += 2) {
            a0 = fmaf(sc[g0][i], vsf[i * HD + d0], a0);
            a1 = fmaf(sc[g1][i], vsf[i * HD + d1], a1);
            c0 = fmaf(sc[g0][i + 1], vsf[(i + 1) * HD + d0], c0);
            c1 = fmaf(sc[g1][i + 1], vsf[(i + 1) * HD + d1], c1);
        }
        if (i < n) {
            a0 = fmaf(sc[g0][i], vsf[i * HD + d0], a0);
            a1 = fmaf(sc[g1][i], vsf[i * HD + d1], a1);
        }
        if constexpr (MODE == 2) {
            s_o[g0][d0] = a0 + c0;
            if (has1) s_o[g1][d1] = a1 + c1;
        } else {
            float* dst0 = part + (((size_t)b * Hl + kvh * G + g0) * nchunk_max + chunk) * (HD + 2);
            dst0[d0] = a0 + c0;
            if (d0 == 0) { dst0[HD] = s_m[g0]; dst0[HD + 1] = s_l[g0]; }
            if (has1) {
                float* dst1 = part + (((size_t)b * Hl + kvh * G + g1) * nchunk_max + chunk) * (HD + 2);
                dst1[d1] = a1 + c1;
                if (d1 == 0) { dst1[HD] = s_m[g1]; dst1[HD + 1] = s_l[g1]; }
            }
        }
    }
    }  // active
    int nparts = (int)((P + CHK - 1) / CHK);  // partials the global merge combines (MODE 1: chunks)
    if constexpr (MODE == 2) {
        namespace cg = cooperative_groups;
        cg::cluster_group cluster = cg::this_cluster();
        if (!active) {
            for (int i = tid; i < G * HD; i += 256) s_o[i / HD][i % HD] = 0.f;
            if (tid < G) { s_m[tid] = -INFINITY; s_l[tid] = 0.f; }
        }
        pdl_trigger();
        cluster.sync();  // every rank's partial is in its shared memory
        // Every rank merges a slice of per = G * HD / cs outputs (a whole
        // number of float4): weights of all heads from the ranks' (m, l), then
        // one float4 of each rank's o per thread through DSMEM.
        float* cw = reinterpret_cast<float*>(ks);  // [G][cs] merge weights
        if (warp < G) {
            const int g = warp;
            const float mk = lane < cs ? cluster.map_shared_rank(&s_m[0], lane)[g] : -INFINITY;
            const float lk = lane < cs ? cluster.map_shared_rank(&s_l[0], lane)[g] : 0.f;
            const float M = warp_max(mk);  // rank 0 is active: finite
            const float w = lane < cs ? exp_ref(__fsub_rn(mk, M)) : 0.f;
            const float L = warp_sum(lk * w);
            if (lane < cs) cw[g * cs + lane] = w;
            if (lane == 0) { s_cm[g] = M; s_cl[g] = L; }
        }
        const int per = (G * HD) / cs, nq = per / 4, o_lo = crank * per;
        float4* pv = reinterpret_cast<float4*>(vs);  // [cs][nq] the ranks' float4 of this slice
        if (tid < cs * nq) {
            const int k = tid / nq, j = tid - k * nq;
            pv[k * nq + j] = *reinterpret_cast<const float4*>(cluster.map_shared_rank(&s_o[0][0], k) + o_lo + 4 * j);
        }
        __syncthreads();
        cluster.sync();  // every rank has read what it needs from its peers
        const int nclu = (nparts + cs - 1) / cs;  // clusters over the sequence
        const int cl_idx = chunk / cs;
        if (tid < nq) {
            const int o = o_lo + 4 * tid, g = o / HD, dd = o - g * HD;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int k = 0; k < cs; ++k) {
                const float4 v = pv[k * nq + tid];
                const float w = cw[g * cs + k];
                acc = make_float4(fmaf(v.x, w, acc.x), fmaf(v.y, w, acc.y), fmaf(v.z, w, acc.z), fmaf(v.w, w, acc.w));
            }
            if (nclu == 1) {
                const float L = s_cl[g];
                *reinterpret_cast<float4*>(att + (size_t)b * Hl * HD + (size_t)kvh * G * HD + o) =
                    make_float4(__fdiv_rn(acc.x, L), __fdiv_rn(acc.y, L), __fdiv_rn(acc.z, L), __fdiv_rn(acc.w, L));
            } else {
                // this cluster's partial number cl_idx, merged below across clusters
                // partial rows are HD + 2 floats: only 4-byte aligned, so scalar stores
                float* dst = part + (((size_t)b * Hl + kvh * G + g) * nchunk_max + cl_idx) * (HD + 2);
                dst[dd] = acc.x;
                dst[dd + 1] = acc.y;
                dst[dd + 2] = acc.z;
                dst[dd + 3] = acc.w;
                if (dd == 0) { dst[HD] = s_cm[g]; dst[HD + 1] = s_cl[g]; }
                __threadfence();
            }
        }
        if (nclu == 1) return;
        cluster.sync();  // every slice of the cluster partial is written and fenced
        if (crank != 0) return;
        nparts = nclu;
    }
    if constexpr (MODE >= 1) {
        const int nch = nparts;
        // Publish this CTA's partial (barrier, then a device-scope fence that
        // is cumulative over the stores ordered before it) and take a ticket.
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            const unsigned t = atomicAdd(&cnt[b * Hkvl + kvh], 1u);
            s_last = (t == (unsigned)(nch - 1));
            if (s_last) {
                cnt[b * Hkvl + kvh] = 0u;
                __threadfence();
            }
        }
        __syncthreads();
        if (!s_last) return;
        float* sw = reinterpret_cast<float*>(ks);  // [G][nch] chunk maxima, then merge weights
        float* sl = reinterpret_cast<float*>(vs);  // [G][nch] chunk sums
        if (warp < G) {
            // both statistics of every chunk in one round of loads
            const int g = warp;
            const float* base = part + ((size_t)b * Hl + kvh * G + g) * nchunk_max * (HD + 2);
            float mx = -INFINITY;
            for (int c = lane; c < nch; c += 32) {
                const float mc = __ldcg(base + (size_t)c * (HD + 2) + HD);
                sl[g * nch + c] = __ldcg(base + (size_t)c * (HD + 2) + HD + 1);
                sw[g * nch + c] = mc;
                mx = fmaxf(mx, mc);
            }
            mx = warp_max(mx);
            float l = 0.f;
            for (int c = lane; c < nch; c += 32) {
                const float w = exp_ref(__fsub_rn(sw[g * nch + c], mx));
                sw[g * nch + c] = w;
                l = fmaf(sl[g * nch + c], w, l);
            }
            l = warp_sum(l);
            if (lane == 0) s_l[g] = l;
        }
        __syncthreads();
        // outputs o0 and o0 + 256 per thread, 16 chunks of both in flight
        for (int o0 = tid; o0 < G * HD; o0 += 512) {
            const int o1 = o0 + 256;
            const bool has1 = o1 < G * HD;
            const int g0 = o0 / HD, d0 = o0 - g0 * HD;
            const int g1 = has1 ? o1 / HD : g0, d1 = has1 ? o1 - g1 * HD : d0;
            const float* base0 = part + ((size_t)b * Hl + kvh * G + g0) * nchunk_max * (HD + 2) + d0;
            const float* base1 = part + ((size_t)b * Hl + kvh * G + g1) * nchunk_max * (HD + 2) + d1;
            const float* w0 = sw + g0 * nch;
            const float* w1 = sw + g1 * nch;
            float acc0 = 0.f, acc1 = 0.f;
            for (int c = 0; c < nch; c += 16) {
                float v0[16], v1[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const bool in = c + k < nch;
                    v0[k] = in ? __ldcg(base0 + (size_t)(c + k) * (HD + 2)) : 0.f;
                    v1[k] = (in && has1) ? __ldcg(base1 + (size_t)(c + k) * (HD + 2)) : 0.f;
                }
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    if (c + k < nch) {
                        acc0 = fmaf(v0[k], w0[c + k], acc0);
                        acc1 = fmaf(v1[k], w1[c + k], acc1);
                    }
                }
            }
            att[(size_t)b * Hl * HD + (size_t)(kvh * G + g0) * HD + d0] = __fdiv_rn(acc0, s_l[g0]);
            if (has1) att[(size_t)b * Hl * HD + (size_t)(kvh * G + g1) * HD + d1] = __fdiv_rn(acc1, s_l[g1]);
        }
    }
}

// Merges the chunk partials of one (sequence, head): out = sum_c o_c e^(m_c-M) / sum_c l_c e^(m_c-M).
// All chunk statistics are loaded at once (one round of loads, not one per chunk).
template <int HD>
__global__ void __launch_bounds__(HD) attn_combine_kernel(const float* __restrict__ part,
                                                          const int64_t* __restrict__ pos, float* __restrict__ att,
                                                          int Hl, int nchunk_max) {
    constexpr int MAXC = 1024;  // chunks per head handled (context <= 32768 positions)
    __shared__ float sw[MAXC];
    __shared__ float sred[HD / 32];
    __shared__ float s_M, s_L;
    const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_trigger();
    const int64_t P = pos[b] + 1;
    const int nch = (int)((P + CH - 1) / CH);
    pdl_wait();
    const float* base = part + ((size_t)b * Hl + h) * nchunk_max * (HD + 2);
    float m = -INFINITY;
    for (int c = tid; c < nch; c += HD) {
        const float mc = base[(size_t)c * (HD + 2) + HD];
        sw[c] = mc;
        m = fmaxf(m, mc);
    }
    m = warp_max(m);
    if (lane == 0) sred[warp] = m;
    __syncthreads();
    if (tid == 0) {
        float t = sred[0];
        for (int w = 1; w < HD / 32; ++w) t = fmaxf(t, sred[w]);
        s_M = t;
    }
    __syncthreads();
    const float M = s_M;
    float l = 0.f;
    for (int c = tid; c < nch; c += HD) {
        const float w = exp_ref(__fsub_rn(sw[c], M));
        sw[c] = w;
        l = fmaf(base[(size_t)c * (HD + 2) + HD + 1], w, l);
    }
    l = warp_sum(l);
    __syncthreads();
    if (lane == 0) sred[warp] = l;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < HD / 32; ++w) t += sred[w];
        s_L = t;
    }
    __syncthreads();
    float o = 0.f;
    int c = 0;
    for (; c + 8 <= nch; c += 8) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = base[(size_t)(c + k) * (HD + 2) + tid];
#pragma unroll
        for (int k = 0; k < 8; ++k) o = fmaf(v[k], sw[c + k], o);
    }
    for (; c < nch; ++c) o = fmaf(base[(size_t)c * (HD + 2) + tid], sw[c], o);
    att[(size_t)b * Hl * HD + (size_t)h * HD + tid] = __fdiv_rn(o, s_L);
}

// ---------------------------------------------------------------------------
// Tensor-parallel exchanges through NVLink peer memory (no NCCL inside a
// step). Every rank owns receive areas, mapped by every other rank (CUDA IPC):
// per exchange site one slot per rank, plus flags. A sender pushes its data
// into slot `rank` of a peer's area with plain peer stores and, after a
// system-scope fence, sets its flag there to the step number (release store);
// a receiver polls only its own memory. All waits are bounded (iterations
// and 1 s of device time); a peer that never arrives sets *err, later waits
// are skipped, and the host fails the call.
//   Sites 0 .. 2L-1: all-reduce of the wo / w2 outputs (B x d floats). The
//     rank's GEMV writes its partial straight into its own slot; the sums are
//     taken in rank order, so every rank gets bit-identical results.
//   Site 2L: the logits shards (B x Vl floats), concatenated on every rank.
//   Site 2L + 1: flags only, the teardown barrier.
// A slot is written once per site and step, and a rank cannot reach the same
// site of the next step before every rank has read it (that needs the
// peers' data of all later sites of this step).
// ---------------------------------------------------------------------------
constexpr int kMaxRanks = 8;
constexpr int kPushCtas = 8;                            // CTAs that may push to one peer (flag slots per sender)
constexpr int kArSpinLimit = 1 << 24;                   // polls of a flag before giving up ...
constexpr unsigned long long kArWaitNs = 1000000000ull;  // ... or 1 s of device time, whichever comes first

struct ArPeers {
    float* base[kMaxRanks];  // rank r's receive areas, mapped into this process
};

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Flag of (site, sender, part) inside an area base (as u32).
__device__ __forceinline__ unsigned* flag_at(float* base, int64_t flag_off, int site, int world, int sender, int part) {
    return reinterpret_cast<unsigned*>(base + flag_off) + ((int64_t)site * world + sender) * kPushCtas + part;
}

// After this CTA's stores to a peer: publish flag (site, rank, part) there.
__device__ __forceinline__ void publish(float* peer_base, int64_t flag_off, int site, int world, int rank, int part,
                                       unsigned seq) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        st_release_sys(flag_at(peer_base, flag_off, site, world, rank, part), seq);
    }
}

// Waits (thread 0, bounded) until every peer's flags (site, r, 0..parts-1) in
// this rank's own area reach seq; returns the CTA-wide verdict.
__device__ __forceinline__ bool arrived(unsigned flag, unsigned seq, bool exact) {
    return exact ? flag == seq : (int)(flag - seq) >= 0;
}

__device__ __forceinline__ bool wait_peers(float* mine, int64_t flag_off, int site, int world, int rank, int parts,
                                           unsigned seq, int* err, int* s_ok, bool exact = false) {
    if (threadIdx.x == 0) {
        int ok = *reinterpret_cast<volatile int*>(err) == 0;
        const unsigned long long t0 = global_ns();
        for (int r = 0; r < world && ok; ++r) {
            if (r == rank) continue;
            for (int part = 0; part < parts && ok; ++part) {
                const unsigned* f = flag_at(mine, flag_off, site, world, r, part);
                int it = 0;
                while (!arrived(ld_acquire_sys(f), seq, exact)) {
                    if (++it > kArSpinLimit || global_ns() - t0 > kArWaitNs) {
                        ok = 0;
                        atomicExch(err, 1);
                        break;
                    }
                    if (it > 64) __nanosleep(64);
                }
            }
        }
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

// All-reduce site: grid = world - 1 CTAs, CTA k pushes to peer rank + 1 + k;
// then every CTA sums its share of the n4 float4s in rank order into out.
__global__ void __launch_bounds__(512) allreduce_push_kernel(ArPeers peers, int world, int rank, int64_t area_off,
                                                             int64_t slot_floats, int64_t flag_off, int site, int n4,
                                                             const unsigned* __restrict__ step,
                                                             float* __restrict__ out, int* __restrict__ err) {
    pdl_trigger();
    pdl_wait();  // this rank's partial (written by the previous kernel) is complete
    __shared__ int s_ok;
    const unsigned seq = *step;
    float* mine = peers.base[rank];
    const float4* own = reinterpret_cast<const float4*>(mine + area_off + rank * slot_floats);
    const int k = blockIdx.x;
    if (k < world - 1) {
        const int peer = (rank + 1 + k) % world;
        float4* dst = reinterpret_cast<float4*>(peers.base[peer] + area_off + rank * slot_floats);
        for (int i = threadIdx.x; i < n4; i += blockDim.x) dst[i] = own[i];
        publish(peers.base[peer], flag_off, site, world, rank, 0, seq);
    }
    if (!wait_peers(mine, flag_off, site, world, rank, 1, seq, err, &s_ok)) return;
    const int per = (n4 + gridDim.x - 1) / gridDim.x;
    const int i0 = k * per, i1 = min(n4, i0 + per);
    const float4* slot0 = reinterpret_cast<const float4*>(mine + area_off);
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        float4 acc = __ldcv(slot0 + i);
        for (int r = 1; r < world; ++r) {
            const float4 v = __ldcv(slot0 + r * (slot_floats / 4) + i);
            acc.x = __fadd_rn(acc.x, v.x); acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z); acc.w = __fadd_rn(acc.w, v.w);
        }
        reinterpret_cast<float4*>(out)[i] = acc;
    }
}

// Logits site: grid = (world - 1) * kPushCtas CTAs; CTA k pushes part
// k % kPushCtas of this rank's B x Vl shard to peer rank + 1 + k / kPushCtas,
// then the CTAs assemble out[b][r * Vl + j] (j < Vl, r * Vl + j < V) from
// the local shard and the received slots.
__global__ void __launch_bounds__(512) gather_push_kernel(ArPeers peers, int world, int rank, int64_t area_off,
                                                          int64_t slot_floats, int64_t flag_off, int site,
                                                          const float* __restrict__ shard, int B, int Vl, int V,
                                                          const unsigned* __restrict__ step, float* __restrict__ out,
                                                          int* __restrict__ err) {
    pdl_trigger();
    pdl_wait();
    __shared__ int s_ok;
    const unsigned seq = *step;
    float* mine = peers.base[rank];
    const int n = B * Vl;
    const int k = blockIdx.x;
    {
        const int peer = (rank + 1 + k / kPushCtas) % world, part = k % kPushCtas;
        const int j0 = (int)((int64_t)part * n / kPushCtas), j1 = (int)((int64_t)(part + 1) * n / kPushCtas);
        float* dst = peers.base[peer] + area_off + rank * slot_floats;
        for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) dst[j] = shard[j];
        publish(peers.base[peer], flag_off, site, world, rank, part, seq);
    }
    if (!wait_peers(mine, flag_off, site, world, rank, kPushCtas, seq, err, &s_ok)) return;
    const int64_t total = (int64_t)B * V;
    for (int64_t t = (int64_t)k * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(t / V), v = (int)(t - (t / V) * V);
        const int r = v / Vl, j = v - r * Vl;
        out[t] = (r == rank) ? shard[(int64_t)b * Vl + j] : __ldcv(mine + area_off + r * slot_floats + (int64_t)b * Vl + j);
    }
}

// Teardown barrier: flags only (site 2L + 1), one CTA per peer. The flag
// value is a fixed sentinel that only the peer's own teardown push writes, so
// passing the barrier means the peer has made its last store into this
// rank's areas, whatever steps either rank ran.
constexpr unsigned kTeardownFlag = 0xC0FFEE01u;

__global__ void peer_barrier_kernel(ArPeers peers, int world, int rank, int64_t flag_off, int site,
                                    int* __restrict__ err) {
    __shared__ int s_ok;
    const int peer = (rank + 1 + blockIdx.x) % world;
    publish(peers.base[peer], flag_off, site, world, rank, 0, kTeardownFlag);
    wait_peers(peers.base[rank], flag_off, site, world, rank, 1, kTeardownFlag, err, &s_ok, true);
}

// Greedy fast path of Sampler.sample (inference/Sampler.java:56-67): the
// first index of the maximum; a NaN never wins unless it is element 0 (then
// the reference returns 0). Every CTA reduces a slice and folds
// (order-preserving bits of the value, ~index) into a 64-bit key with
// atomicMax, so the result does not depend on CTA order. Keys are zeroed by
// the embedding kernel at the start of the step.
__global__ void __launch_bounds__(256) argmax_kernel(const float* __restrict__ logits, int V, int stride,
                                                     unsigned long long* __restrict__ keys) {
    __shared__ unsigned long long sk[8];
    const int b = blockIdx.y;
    const float* row = logits + (size_t)b * stride;
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * 256 + threadIdx.x; i < V; i += gridDim.x * 256) {
        const unsigned long long k = ((unsigned long long)ordered_bits(row[i]) << 32) | (0xFFFFFFFFu - (uint32_t)i);
        best = k > best ? k : best;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0 && row[0] != row[0]) best = ~0ull;  // NaN at index 0 wins
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) sk[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) best = sk[w] > best ? sk[w] : best;
        atomicMax(&keys[b], best);
    }
}

// Writes the argmax index of each of the B keys.
__global__ void argmax_index_kernel(const unsigned long long* __restrict__ keys, int B, int* __restrict__ out) {
    if (threadIdx.x < B) out[threadIdx.x] = key_index(keys[threadIdx.x]);
}

// ---------------------------------------------------------------------------
// Batched prompt kernels (one row per prompt token)
// ---------------------------------------------------------------------------
// Row-wise x_out = rmsNorm(x_in + y_in) * gamma with the reference's rounding
// (the F7 residual stream): one CTA per row; with xbf, x_out also rounded to
// bf16 [T][d] for the next tensor-core GEMM.
// Element i of y summed over `splits` (<= 4) K-split GEMM partials `stride`
// floats apart, in split order (the order of splitk_sum_kernel); the
// partials' loads are predicated, not a loop, so they are all in flight.
constexpr int kMaxPromptSplits = 4;
__device__ __forceinline__ float4 split_sum4(const float* __restrict__ y, int splits, size_t stride, size_t i) {
    float4 acc = *reinterpret_cast<const float4*>(y + i);
    float4 p[kMaxPromptSplits - 1];
#pragma unroll
    for (int z = 1; z < kMaxPromptSplits; ++z)
        if (z < splits) p[z - 1] = *reinterpret_cast<const float4*>(y + (size_t)z * stride + i);
#pragma unroll
    for (int z = 1; z < kMaxPromptSplits; ++z)
        if (z < splits) {
            acc.x += p[z - 1].x;
            acc.y += p[z - 1].y;
            acc.z += p[z - 1].z;
            acc.w += p[z - 1].w;
        }
    return acc;
}

// One prompt row (CTA of 256 threads): t = x + y (y summed over its K-split
// partials), RMSNorm of t into xout (FP32, the reference's rounding) and
// xbf (bf16, the next GEMM's operand). t is staged in shared memory once
// (d <= 8192, a multiple of 4).
constexpr int kRowsMaxDim = 8192;
__global__ void __launch_bounds__(256) rows_addnorm_kernel(const float* __restrict__ xin, const float* __restrict__ yin,
                                                           const float* __restrict__ gamma, float* __restrict__ xout,
                                                           __nv_bfloat16* __restrict__ xbf, int d, float eps,
                                                           int ysplits = 1, size_t ysplit_stride = 0) {
    __shared__ float4 s_t[kRowsMaxDim / 4];
    __shared__ float s_red[8];
    const size_t row = blockIdx.x;
    const int n4 = d >> 2;
    const float4* a = reinterpret_cast<const float4*>(xin + row * d);
    float acc = 0.f;
#pragma unroll 4
    for (int i = threadIdx.x; i < n4; i += 256) {
        const float4 y = split_sum4(yin, ysplits, ysplit_stride, row * d + 4 * (size_t)i);
        const float4 x = a[i];
        const float4 t = make_float4(__fadd_rn(x.x, y.x), __fadd_rn(x.y, y.y), __fadd_rn(x.z, y.z), __fadd_rn(x.w, y.w));
        s_t[i] = t;
        acc = fmaf(t.x, t.x, acc);
        acc = fmaf(t.y, t.y, acc);
        acc = fmaf(t.z, t.z, acc);
        acc = fmaf(t.w, t.w, acc);
    }
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = acc;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += s_red[w];
    const float inv = rms_inv(tot, d, eps);
    const float4* g4 = reinterpret_cast<const float4*>(gamma);
    for (int i = threadIdx.x; i < n4; i += 256) {
        const float4 t = s_t[i], g = g4[i];
        const float4 o = make_float4(norm_apply(t.x, inv, g.x), norm_apply(t.y, inv, g.y), norm_apply(t.z, inv, g.z),
                                     norm_apply(t.w, inv, g.w));
        reinterpret_cast<float4*>(xout + row * d)[i] = o;
        if (xbf) {
            const __nv_bfloat162 lo = __floats2bfloat162_rn(o.x, o.y), hi = __floats2bfloat162_rn(o.z, o.w);
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t*>(&lo);
            u.y = *reinterpret_cast<const uint32_t*>(&hi);
            reinterpret_cast<uint2*>(xbf + row * d)[i] = u;
        }
    }
}

// Causal attention of a prompt chunk (LlamaModel.attention, inference/
// LlamaModel.java:255-297, for T consecutive query positions p0 .. p0+T-1).
// CTA (KV head h, query block) holds R = 32 query rows (QB = 32 / G tokens x
// the G query heads of h) and streams the keys 0 .. (its last position) in
// tiles of 64 through shared memory (K and V of the tile; Q8_0 caches are
// dequantized on the way in): warp w scores rows 4w .. 4w+3 against keys
// lane and lane + 32 (q rows are broadcast reads, K rows padded to spread the
// banks), keeps a running max and sum per row (online softmax; keys past a
// row's own position are masked), writes the tile's probabilities to shared
// memory and adds P V into its rows' outputs (lane: HD / 32 dimensions).
// Every K/V row a query block needs is read once per block instead of once
// per query token. Scores are dot * scale as the reference; the prompt
// path's tolerance is 2e-2 of the logit range.
constexpr int PA_R = 32, PA_KT = 64;
constexpr size_t prompt_attn_smem(int hd) {
    return (size_t)(PA_R * (hd + 4) + PA_KT * (hd + 4) + PA_KT * hd + PA_R * PA_KT) * 4;
}

template <int HD, int G, bool KVQ>
__global__ void __launch_bounds__(256) prompt_attn_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                                          const float* __restrict__ vc,
                                                          const uint16_t* __restrict__ ksc,
                                                          const uint16_t* __restrict__ vsc, float* __restrict__ att,
                                                          int T, int64_t p0, int Hl, int ctx, float scale) {
    constexpr int QB = PA_R / G;   // tokens per CTA
    constexpr int KP = HD + 4;     // padded q / K row (floats)
    constexpr int F4 = HD / 4;
    constexpr int DPL = HD / 32;   // output dimensions per lane
    extern __shared__ __align__(16) float pa_smem[];
    float* qs = pa_smem;                 // [R][KP]
    float* ks = qs + PA_R * KP;          // [KT][KP]
    float* vs = ks + PA_KT * KP;         // [KT][HD]
    float* ps = vs + PA_KT * HD;         // [R][KT]
    const int kvh = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nq = Hl * HD;
    const int t0 = blockIdx.y * QB;
    const int ntok = min(QB, T - t0);
    // q rows: row r = ti * G + g is token t0 + ti, query head kvh * G + g
    for (int i = tid; i < PA_R * F4; i += 256) {
        const int r = i / F4, f = i - r * F4;
        const int ti = r / G, g = r - ti * G;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ti < ntok) v = *reinterpret_cast<const float4*>(q + (size_t)(t0 + ti) * nq + (size_t)(kvh * G + g) * HD + 4 * f);
        *reinterpret_cast<float4*>(qs + r * KP + 4 * f) = v;
    }
    int64_t rpos[4];  // position of this warp's rows (-1: no token)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int ti = (4 * warp + j) / G;
        rpos[j] = ti < ntok ? p0 + t0 + ti : -1;
    }
    const int64_t last = p0 + t0 + ntok - 1;
    const size_t kvbase = (size_t)kvh * ctx * HD;
    float m[4], l[4], o[4][DPL];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        m[j] = -INFINITY;
        l[j] = 0.f;
#pragma unroll
        for (int d = 0; d < DPL; ++d) o[j][d] = 0.f;
    }
    for (int64_t k0 = 0; k0 <= last; k0 += PA_KT) {
        const int nk = (last + 1 - k0) < PA_KT ? (int)(last + 1 - k0) : PA_KT;
        __syncthreads();  // the previous tile's K and V are no longer read
        for (int i = tid; i < PA_KT * F4; i += 256) {
            const int kr = i / F4, f = i - kr * F4;
            float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
            if (kr < nk) {
                const size_t e = kvbase + (size_t)(k0 + kr) * HD;
                if constexpr (KVQ) {
                    kv4 = kv_dq4(reinterpret_cast<const int8_t*>(kc) + e, ksc + (e >> 5), f);
                    vv4 = kv_dq4(reinterpret_cast<const int8_t*>(vc) + e, vsc + (e >> 5), f);
                } else {
                    kv4 = *reinterpret_cast<const float4*>(kc + e + 4 * f);
                    vv4 = *reinterpret_cast<const float4*>(vc + e + 4 * f);
                }
            }
            *reinterpret_cast<float4*>(ks + kr * KP + 4 * f) = kv4;
            *reinterpret_cast<float4*>(vs + kr * HD + 4 * f) = vv4;
        }
        __syncthreads();
        float sc[4][2];
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[j][0] = sc[j][1] = 0.f;
#pragma unroll 4
        for (int f = 0; f < F4; ++f) {
            const float4 ka = *reinterpret_cast<const float4*>(ks + lane * KP + 4 * f);
            const float4 kb = *reinterpret_cast<const float4*>(ks + (lane + 32) * KP + 4 * f);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float4 qv = *reinterpret_cast<const float4*>(qs + (4 * warp + j) * KP + 4 * f);
                sc[j][0] = fmaf(qv.x, ka.x, fmaf(qv.y, ka.y, fmaf(qv.z, ka.z, fmaf(qv.w, ka.w, sc[j][0]))));
                sc[j][1] = fmaf(qv.x, kb.x, fmaf(qv.y, kb.y, fmaf(qv.z, kb.z, fmaf(qv.w, kb.w, sc[j][1]))));
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const bool ia = lane < nk && k0 + lane <= rpos[j];
            const bool ib = lane + 32 < nk && k0 + lane + 32 <= rpos[j];
            const float a = ia ? __fmul_rn(sc[j][0], scale) : -INFINITY;
            const float bq = ib ? __fmul_rn(sc[j][1], scale) : -INFINITY;
            const float mn = fmaxf(m[j], warp_max(fmaxf(a, bq)));
            const float alpha = (mn == -INFINITY) ? 1.f : expf(m[j] - mn);
            const float pa = ia ? expf(a - mn) : 0.f;
            const float pb = ib ? expf(bq - mn) : 0.f;
            l[j] = fmaf(l[j], alpha, warp_sum(pa + pb));
            m[j] = mn;
            ps[(4 * warp + j) * PA_KT + lane] = pa;
            ps[(4 * warp + j) * PA_KT + lane + 32] = pb;
#pragma unroll
            for (int d = 0; d < DPL; ++d) o[j][d] *= alpha;
        }
        __syncwarp();  // this warp's probabilities are visible to its lanes
        for (int kk = 0; kk < nk; ++kk) {
            float vv[DPL];
            if constexpr (DPL == 4) {
                const float4 t = *reinterpret_cast<const float4*>(vs + kk * HD + 4 * lane);
                vv[0] = t.x; vv[1] = t.y; vv[2] = t.z; vv[3] = t.w;
            } else {
                const float2 t = *reinterpret_cast<const float2*>(vs + kk * HD + 2 * lane);
                vv[0] = t.x; vv[1] = t.y;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float pj = ps[(4 * warp + j) * PA_KT + kk];
#pragma unroll
                for (int d = 0; d < DPL; ++d) o[j][d] = fmaf(pj, vv[d], o[j][d]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int r = 4 * warp + j, ti = r / G, g = r - ti * G;
        if (ti < ntok) {
            float* dst = att + (size_t)(t0 + ti) * nq + (size_t)(kvh * G + g) * HD + DPL * lane;
#pragma unroll
            for (int d = 0; d < DPL; ++d) dst[d] = __fdiv_rn(o[j][d], l[j]);
        }
    }
}

template <int HD, bool KVQ, int G>
void launch_prompt_attn_g(int Hkvl, int T, cudaStream_t s, const float* q, const float* kc, const float* vc,
                          const uint16_t* ksc, const uint16_t* vsc, float* att, int64_t p0, int Hl, int ctx,
                          float scale) {
    auto kern = prompt_attn_kernel<HD, G, KVQ>;
    const size_t smem = prompt_attn_smem(HD);
    AT_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    constexpr int QB = PA_R / G;
    kern<<<dim3(Hkvl, (T + QB - 1) / QB), 256, smem, s>>>(q, kc, vc, ksc, vsc, att, T, p0, Hl, ctx, scale);
    AT_CUDA(cudaGetLastError());
}

template <int HD, bool KVQ>
void launch_prompt_attn(int G, int Hkvl, int T, cudaStream_t s, const float* q, const float* kc, const float* vc,
                        const uint16_t* ksc, const uint16_t* vsc, float* att, int64_t p0, int Hl, int ctx,
                        float scale) {
    switch (G) {
#define AT_PA(GG) \
    case GG: launch_prompt_attn_g<HD, KVQ, GG>(Hkvl, T, s, q, kc, vc, ksc, vsc, att, p0, Hl, ctx, scale); break;
        AT_PA(1) AT_PA(2) AT_PA(3) AT_PA(4) AT_PA(5) AT_PA(6) AT_PA(7) AT_PA(8)
#undef AT_PA
        default: fail(AT_ERR_UNSUPPORTED, "query heads per KV head must be 1..8");
    }
}

// Q8_0 KV cache of one layer (all slots; the slot offset is in the element index).
struct KvQ {
    int8_t* kq = nullptr;
    int8_t* vq = nullptr;
    uint16_t* ks = nullptr;
    uint16_t* vs = nullptr;
};

// RoPE of q and k (core/Kernels.java:296-309: a' = fma(a, c, b * -s),
// b' = fma(b, c, a * s)) and the KV-cache append (inference/KVCache.java:79-95)
// of prompt row t at position p0 + t; q goes to q_out [T][nq].
// One prompt token (CTA of 256 threads): the QKV GEMM's row (summed over
// its K-split partials, staged in shared memory; qcols <= 10240) gets RoPE
// on q and k; q goes to q_out, k and v are appended to the KV cache.
constexpr int kRopeMaxCols = 10240;
__global__ void __launch_bounds__(256) rope_append_kernel(const float* __restrict__ qkv, int qcols,
                                                          float* __restrict__ q_out, float* __restrict__ kc,
                                                          float* __restrict__ vc, KvQ kvq,
                                                          const float* __restrict__ rcos,
                                                          const float* __restrict__ rsin, int hd, int nq, int nkv,
                                                          int ctx, int64_t p0, int splits = 1,
                                                          size_t split_stride = 0) {
    __shared__ float4 s_row4[kRopeMaxCols / 4];
    const float* s_row = reinterpret_cast<const float*>(s_row4);
    const int t = blockIdx.x;
    const int64_t pos = p0 + t;
#pragma unroll 4
    for (int i = threadIdx.x; i < qcols / 4; i += 256)
        s_row4[i] = split_sum4(qkv, splits, split_stride, (size_t)t * qcols + 4 * (size_t)i);
    __syncthreads();
#pragma unroll 4
    for (int j = threadIdx.x; j < qcols; j += 256) {
        const float val = s_row[j];
        if (j < nq + nkv) {
            const int dd = (j < nq ? j : j - nq) % hd;
            const float partner = s_row[j ^ 1];
            const float cs = rcos[pos * hd + dd], sn = rsin[pos * hd + dd];
            const float out = ((dd & 1) == 0) ? fmaf(val, cs, __fmul_rn(partner, -sn)) : fmaf(val, cs, __fmul_rn(partner, sn));
            if (j < nq) {
                q_out[(size_t)t * nq + j] = out;
            } else {
                const int jj = j - nq, kvh = jj / hd;
                const size_t e = ((size_t)kvh * ctx + pos) * hd + dd;
                if (kvq.kq) kv_store_q8(kvq.kq, kvq.ks, e, out);  // warp-uniform: 32-aligned column blocks
                else kc[e] = out;
            }
        } else {
            const int jj = j - nq - nkv, kvh = jj / hd, dd = jj - kvh * hd;
            const size_t e = ((size_t)kvh * ctx + pos) * hd + dd;
            if (kvq.kq) kv_store_q8(kvq.vq, kvq.vs, e, val);
            else vc[e] = val;
        }
    }
}

// KVCache.append of one position: block h (one per KV head), thread dd.
__global__ void kv_put_kernel(const float* __restrict__ k, const float* __restrict__ v, float* __restrict__ kc,
                              float* __restrict__ vc, KvQ kvq, int ctx, int hd, int64_t pos) {
    const int h = blockIdx.x, dd = threadIdx.x;
    const size_t e = ((size_t)h * ctx + pos) * hd + dd;
    const float kv = k[h * hd + dd], vv = v[h * hd + dd];
    if (kvq.kq) {  // hd is a multiple of 32: every warp holds one block
        kv_store_q8(kvq.kq, kvq.ks, e, kv);
        kv_store_q8(kvq.vq, kvq.vs, e, vv);
    } else {
        kc[e] = kv;
        vc[e] = vv;
    }
}

// RoPE and the KV-cache append for B batch rows of a plain QKV output
// [B][qcols] (attention weights stored [out][in], computed by the
// orientation-N GEMV): the arithmetic of the fused QKV epilogue
// (core/Kernels.java:296-309, inference/KVCache.java:79-95), slot b at
// position pos[b].
__global__ void __launch_bounds__(256) qkv_rope_rows_kernel(const float* __restrict__ qkv, int qcols,
                                                            float* __restrict__ q_out, float* __restrict__ kc,
                                                            float* __restrict__ vc, KvQ kvq, int64_t slot_stride,
                                                            const float* __restrict__ rcos,
                                                            const float* __restrict__ rsin,
                                                            const int64_t* __restrict__ pos, int hd, int nq, int nkv,
                                                            int ctx) {
    const int b = blockIdx.x;
    const int64_t p = pos[b];
    const float* row = qkv + (size_t)b * qcols;
    for (int j = threadIdx.x; j < qcols; j += 256) {
        const float val = row[j];
        if (j < nq + nkv) {
            const int dd = (j < nq ? j : j - nq) % hd;
            const float partner = row[j ^ 1];
            const float cs = rcos[p * hd + dd], sn = rsin[p * hd + dd];
            const float out = ((dd & 1) == 0) ? fmaf(val, cs, __fmul_rn(partner, -sn)) : fmaf(val, cs, __fmul_rn(partner, sn));
            if (j < nq) {
                q_out[(size_t)b * nq + j] = out;
            } else {
                const int jj = j - nq, kvh = jj / hd;
                const size_t e = (size_t)b * slot_stride + ((size_t)kvh * ctx + p) * hd + dd;
                if (kvq.kq) kv_store_q8(kvq.kq, kvq.ks, e, out);  // warp-uniform: 32-aligned column blocks
                else kc[e] = out;
            }
        } else {
            const int jj = j - nq - nkv, kvh = jj / hd, dd = jj - kvh * hd;
            const size_t e = (size_t)b * slot_stride + ((size_t)kvh * ctx + p) * hd + dd;
            if (kvq.kq) kv_store_q8(kvq.vq, kvq.vs, e, val);
            else vc[e] = val;
        }
    }
}

// h = silu(g) * u rounded to bf16: the w2 GEMM's staged input.
__global__ void silu_mul_bf16_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                     __nv_bfloat16* __restrict__ h, int64_t n) {
    const int64_t n4 = n / 4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const float4 a = reinterpret_cast<const float4*>(g)[i], b = reinterpret_cast<const float4*>(u)[i];
        const __nv_bfloat162 lo = __floats2bfloat162_rn(silu_mul(a.x, b.x), silu_mul(a.y, b.y));
        const __nv_bfloat162 hi = __floats2bfloat162_rn(silu_mul(a.z, b.z), silu_mul(a.w, b.w));
        reinterpret_cast<__nv_bfloat162*>(h)[2 * i] = lo;
        reinterpret_cast<__nv_bfloat162*>(h)[2 * i + 1] = hi;
    }
    for (int64_t i = 4 * n4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        h[i] = __float2bfloat16_rn(silu_mul(g[i], u[i]));
}


inline int grid_for(int64_t n, int tpb = 256) {
    int64_t g = (n + tpb - 1) / tpb;
    if (g > 65535 * 16) g = 65535 * 16;
    return (int)(g < 1 ? 1 : g);
}

// Greedy loop step: the argmax becomes the next token, the position advances.
__global__ void advance_kernel(const int* __restrict__ argmax, int* __restrict__ tokens, int64_t* __restrict__ pos,
                               int* __restrict__ out, int* __restrict__ counter) {
    const int t = argmax[0];
    out[*counter] = t;
    *counter += 1;
    tokens[0] = t;
    pos[0] += 1;
}

struct Layer {
    at_qmat qkv, wo, w1, w3, w2;
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
};

}  // namespace
}  // namespace at

using namespace at;

// Fp16.toFloat with flush-to-zero (core/Fp16.java:19-37), on the host.
static float fp16_ftz_host(uint16_t h) {
    const uint32_t sgn = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, mt = h & 0x3FFu;
    uint32_t bits = (sgn << 31) | ((e + 112u) << 23) | (mt << 13);
    if (e == 0u) bits = sgn << 31;
    if (e == 31u) bits = mt ? 0x7FC00000u : ((sgn << 31) | 0x7F800000u);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

struct at_model {
    at_ctx* ctx = nullptr;
    at_model_config cfg{};
    int d = 0, hd = 0, H = 0, Hkv = 0, F = 0, V = 0, L = 0, ctx_len = 0, B = 1;
    int Hl = 0, Hkvl = 0, Fl = 0, Vl = 0;  // per-rank shares
    int wtype = -1;                        // type of the first quantized matrix seen (Q4_0 / Q8_0)
    int layout = 0;                        // AT_LAYOUT_* bits of the tensors' bytes
    bool attn_n = false;                   // attention weights [out][in]: orientation-N GEMVs
    float* qkvbuf = nullptr;               // attn_n: plain QKV output [max_batch][(Hl + 2 Hkvl) hd]
    std::vector<Layer> layers;
    at_qmat tok, out;
    float* out_norm = nullptr;
    // activations
    float *xa = nullptr, *xb = nullptr, *y = nullptr, *q = nullptr, *att = nullptr, *h = nullptr;
    float *logits = nullptr, *logits_local = nullptr, *att_part = nullptr;
    unsigned* attn_cnt = nullptr;  // [max_batch][Hkvl] tickets of the fused decode attention
    int attn_cs = 0;               // decode attention cluster size (0: merge through global memory)
    float *kcache = nullptr, *vcache = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    bool kv_q8 = false;                   // Q8_0 KV cache: quants + fp16 scales instead of kcache / vcache
    int8_t *kq8 = nullptr, *vq8 = nullptr;
    uint16_t *ksc = nullptr, *vsc = nullptr;
    float* kv_stage = nullptr;            // at_model_kv_append staging: k then v, [Hkvl * hd] each
    float* scratch = nullptr;
    unsigned* counters = nullptr;
    int* d_tokens = nullptr;
    int64_t* d_pos = nullptr;
    unsigned* d_step = nullptr;           // step sequence number (advanced by the embedding kernel)
    // tensor parallelism: one-shot all-reduce through peer memory
    float* ar_base = nullptr;             // this rank's receive areas [sites][world][site_floats] + flags (IPC-exported)
    float* ar_peer[8] = {};               // every rank's ar_base, mapped into this process (own rank: ar_base)
    int64_t ar_site_floats = 0, ar_logit_floats = 0, ar_flag_off = 0;
    int* d_ar_err = nullptr;
    int* h_ar_err = nullptr;              // pinned copy, read after each step
    // batched prompt chunks (allocated on the first forwardPrompt that uses them)
    float *pf_xa = nullptr, *pf_xb = nullptr, *pf_y = nullptr, *pf_qkv = nullptr, *pf_q = nullptr;
    float *pf_att = nullptr, *pf_g = nullptr, *pf_u = nullptr;
    void* pf_xbf = nullptr;               // bf16 activations of the prompt GEMMs
    size_t pf_xbf_bytes = 0;
    float* pf_ws = nullptr;               // split-K partials of the prompt GEMMs
    size_t pf_ws_bytes = 0;
    int* pf_tok = nullptr;
    int64_t* pf_pos = nullptr;
    int* pf_err = nullptr;
    int* h_pf_tok = nullptr;              // pinned
    int64_t* h_pf_pos = nullptr;          // pinned
    int* d_argmax = nullptr;
    unsigned long long* d_argkey = nullptr;  // packed (value, index) max per row
    int* h_tokens = nullptr;      // pinned
    int64_t* h_pos = nullptr;     // pinned
    int nchunk_max = 0;
    int64_t slot_stride = 0;      // floats per KV slot (all layers)
    std::vector<int64_t> kv_size;
    std::map<std::string, bool> seen;
    cudaGraphExec_t graph[9] = {};
    cudaGraphExec_t graph_gen = nullptr;  // step + greedy advance (slot 0)
    cudaGraphExec_t graph_prof = nullptr; // step with an event pair around every launch
    int graph_prof_batch = 0;
    int* d_gen_out = nullptr;             // [ctx] generated tokens
    int* d_gen_count = nullptr;
    // eager profiling: event pairs around each launch
    bool profiling = false;
    bool pdl = true;                      // programmatic dependent launch between step kernels
    std::vector<cudaEvent_t> prof_ev;
    std::vector<int> prof_cls;
    size_t prof_used = 0;
    // persistent decode step (batch 1, one GPU): one launch per token
    bool use_ds = false;
    DsParams ds{};
    DsLayer* d_ds_layers = nullptr;
    float *ds_qkv_part = nullptr, *ds_wo_part = nullptr, *ds_apart = nullptr;
    unsigned *ds_tickets = nullptr, *ds_bar = nullptr;
    int* ds_err = nullptr;
    int* h_ds_err = nullptr;              // pinned copy, read after each launch sequence
    unsigned long long* ds_stamps = nullptr;
    // device sampling (allocated on first use)
    SampleRow* d_rows = nullptr;
    SampleRow* h_rows = nullptr;          // pinned, [max_batch]
    int* d_hist = nullptr;                // [max_batch][hist_cap] penalty histories
    int64_t hist_cap = 0;                 // max(maxContext, 8192) ids per row
    int* d_hist_len = nullptr;            // [max_batch]
    int* d_pen_cnt = nullptr;             // [max_batch][V] occurrence counts, zero between calls
    unsigned long long* d_rng = nullptr;  // [max_batch] generator states of unseeded rows
    int* d_sampled = nullptr;             // [max_batch]
    int* d_seq = nullptr;                 // [max_batch][ctx] sampled sequences
    int* d_step_ctr = nullptr;
    int* d_append = nullptr;              // [max_batch] history-append flags of a scheduler step
    int* h_i32 = nullptr;                 // pinned staging, [max_batch]
    unsigned long long* h_rng = nullptr;  // pinned staging, [max_batch]
    cudaGraphExec_t graph_samp[9] = {};   // step + sample + advance, per batch
    bool finalized = false;
};

namespace {

void alloc_zero(void** p, size_t bytes) {
    AT_CUDA(cudaMalloc(p, bytes ? bytes : 16));
    AT_CUDA(cudaMemset(*p, 0, bytes ? bytes : 16));
}

void make_qmat(at_qmat& m, int type, int orient, int64_t rows, int64_t cols) {
    if (m.tiles || m.f32) return;
    m.type = type;
    m.orient = orient;
    m.rows = rows;
    m.cols = cols;
    qmat_alloc(&m);  // zeroed: blocks never written stay zero (scale 0)
}

bool parse_layer(const std::string& name, int* layer, std::string* leaf) {
    if (name.rfind("blk.", 0) != 0) return false;
    const size_t dot = name.find('.', 4);
    if (dot == std::string::npos) return false;
    *layer = std::stoi(name.substr(4, dot - 4));
    *leaf = name.substr(dot + 1);
    return true;
}

// Model dimensions a tensor-parallel rank's shard cut depends on.
struct ShardDims {
    int64_t d, hd, H, Hkv, F, V, Hl, Hkvl, Fl, Vl;
    int W, r;
    bool attn_n;  // attention weights [out][in] (llama.cpp) instead of [in][out]
};

ShardDims shard_dims(const at_model* m, int W, int r) {
    return ShardDims{m->d, m->hd, m->H, m->Hkv, m->F, m->V, m->Hl, m->Hkvl, m->Fl, m->Vl, W, r, m->attn_n};
}

// The part of a logical weight tensor that rank r of W keeps and where it
// lands in the rank's device matrix (Megatron: wq/wk/wv by heads into the
// fused [q|k|v] matrix, wo by its head rows, w1/w3 by output rows, w2 by
// input columns, lm_head by vocabulary rows; norms and the embedding whole).
// The tensor's shape follows Weights.wrapByName (inference/Weights.java:84-112);
// the upload (at_model_set_tensor) and at_tp_shard_region both use this.
void shard_region(const ShardDims& s, const std::string& name, at_shard_region* o) {
    *o = at_shard_region{};
    o->target = AT_SHARD_NONE;
    o->orient = AT_ORIENT_N;
    int layer = -1;
    std::string leaf;
    const bool is_layer = parse_layer(name, &layer, &leaf);
    const int64_t nq = s.Hl * s.hd, nkv = s.Hkvl * s.hd, qcols = nq + 2 * nkv;
    auto set = [&](int target, int orient, int64_t rows, int64_t cols, int64_t lr, int64_t lc, int64_t sr0,
                   int64_t sc0, int64_t nr, int64_t nc, int64_t dr0, int64_t dc0) {
        *o = at_shard_region{target, orient, rows, cols, lr, lc, sr0, sc0, nr, nc, dr0, dc0};
    };
    if (name == "output_norm.weight" || (is_layer && (leaf == "attn_norm.weight" || leaf == "ffn_norm.weight"))) {
        set(AT_SHARD_NORM, AT_ORIENT_N, 1, s.d, 1, s.d, 0, 0, 1, s.d, 0, 0);
    } else if (name == "token_embd.weight") {
        set(AT_SHARD_TOKEN_EMBD, AT_ORIENT_N, s.V, s.d, s.V, s.d, 0, 0, s.V, s.d, 0, 0);
    } else if (name == "output.weight") {
        const int64_t v0 = (int64_t)s.r * s.Vl;
        const int64_t nv = std::max<int64_t>(0, std::min<int64_t>(s.Vl, s.V - v0));
        set(AT_SHARD_OUTPUT, AT_ORIENT_N, s.V, s.d, s.Vl, s.d, v0, 0, nv, s.d, 0, 0);
    } else if (!is_layer) {
        return;
    } else if (s.attn_n) {  // [out][in]: the rank's heads are rows (wq/wk/wv) or input columns (wo)
        if (leaf == "attn_q.weight")
            set(AT_SHARD_QKV, AT_ORIENT_N, s.H * s.hd, s.d, qcols, s.d, s.r * nq, 0, nq, s.d, 0, 0);
        else if (leaf == "attn_k.weight")
            set(AT_SHARD_QKV, AT_ORIENT_N, s.Hkv * s.hd, s.d, qcols, s.d, s.r * nkv, 0, nkv, s.d, nq, 0);
        else if (leaf == "attn_v.weight")
            set(AT_SHARD_QKV, AT_ORIENT_N, s.Hkv * s.hd, s.d, qcols, s.d, s.r * nkv, 0, nkv, s.d, nq + nkv, 0);
        else if (leaf == "attn_output.weight")
            set(AT_SHARD_WO, AT_ORIENT_N, s.d, s.H * s.hd, s.d, nq, 0, s.r * nq, s.d, nq, 0, 0);
    } else {  // the reference's [in][out] attention: the rank's heads are columns (wq/wk/wv) or rows (wo)
        if (leaf == "attn_q.weight")
            set(AT_SHARD_QKV, AT_ORIENT_T, s.d, s.H * s.hd, s.d, qcols, 0, s.r * nq, s.d, nq, 0, 0);
        else if (leaf == "attn_k.weight")
            set(AT_SHARD_QKV, AT_ORIENT_T, s.d, s.Hkv * s.hd, s.d, qcols, 0, s.r * nkv, s.d, nkv, 0, nq);
        else if (leaf == "attn_v.weight")
            set(AT_SHARD_QKV, AT_ORIENT_T, s.d, s.Hkv * s.hd, s.d, qcols, 0, s.r * nkv, s.d, nkv, 0, nq + nkv);
        else if (leaf == "attn_output.weight")
            set(AT_SHARD_WO, AT_ORIENT_T, s.H * s.hd, s.d, nq, s.d, s.r * nq, 0, nq, s.d, 0, 0);
    }
    if (o->target != AT_SHARD_NONE || !is_layer) return;
    if (leaf == "ffn_gate.weight")
        set(AT_SHARD_W1, AT_ORIENT_N, s.F, s.d, s.Fl, s.d, s.r * s.Fl, 0, s.Fl, s.d, 0, 0);
    else if (leaf == "ffn_up.weight")
        set(AT_SHARD_W3, AT_ORIENT_N, s.F, s.d, s.Fl, s.d, s.r * s.Fl, 0, s.Fl, s.d, 0, 0);
    else if (leaf == "ffn_down.weight")
        set(AT_SHARD_W2, AT_ORIENT_N, s.d, s.F, s.d, s.Fl, 0, s.r * s.Fl, s.d, s.Fl, 0, 0);
}

// Brackets the launches of one kernel class with events when profiling.
struct ProfScope {
    at_model* m;
    int cls;
    size_t idx = 0;
    ProfScope(at_model* mm, int c) : m(mm), cls(c) {
        if (!m->profiling) return;
        if (m->prof_used + 2 > m->prof_ev.size()) {
            for (int k = 0; k < 64; ++k) {
                cudaEvent_t e;
                AT_CUDA(cudaEventCreate(&e));
                m->prof_ev.push_back(e);
            }
        }
        idx = m->prof_used;
        m->prof_used += 2;
        m->prof_cls.push_back(cls);
        AT_CUDA(cudaEventRecordWithFlags(m->prof_ev[idx], m->ctx->stream, cudaEventRecordExternal));
    }
    ~ProfScope() {
        if (m->profiling) cudaEventRecordWithFlags(m->prof_ev[idx + 1], m->ctx->stream, cudaEventRecordExternal);
    }
};

// Launches kern<<<grid, block, 0, s>>>(args...), with programmatic stream
// serialization when pdl is set (the kernel calls pdl_wait before reading
// what the previous kernel writes).
template <class... KArgs, class... Args>
void launch_kc(void (*kern)(KArgs...), dim3 grid, dim3 block, dim3 cluster, size_t smem, cudaStream_t s, bool pdl,
               Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (cluster.x * cluster.y * cluster.z > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = cluster.x;
        attr[na].val.clusterDim.y = cluster.y;
        attr[na].val.clusterDim.z = cluster.z;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    AT_CUDA(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...));
}
template <class... KArgs, class... Args>
void launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, bool pdl, Args... args) {
    launch_kc(kern, grid, block, dim3(1, 1, 1), 0, s, pdl, args...);
}

// One attention launch over the fp32 or the Q8_0 KV cache of a layer.
template <int HD, int MODE, int CHK>
void launch_attn(const KvQ& kvq, const float* kc, const float* vc, dim3 grid, dim3 cluster, size_t smem,
                 cudaStream_t s, bool pdl, const float* q, const int64_t* pos, float* part, int Hl, int Hkvl, int ctx,
                 int64_t slot_stride, int nchunk_max, float scale, unsigned* cnt, float* att) {
    if (kvq.kq)
        launch_kc(attn_split_kernel<HD, MODE, CHK, true>, grid, 256, cluster, smem, s, pdl, q,
                  (const float*)kvq.kq, (const float*)kvq.vq, pos, part, Hl, Hkvl, ctx, slot_stride, nchunk_max,
                  scale, cnt, att, (const uint16_t*)kvq.ks, (const uint16_t*)kvq.vs);
    else
        launch_kc(attn_split_kernel<HD, MODE, CHK, false>, grid, 256, cluster, smem, s, pdl, q, kc, vc, pos, part,
                  Hl, Hkvl, ctx, slot_stride, nchunk_max, scale, cnt, att, (const uint16_t*)nullptr,
                  (const uint16_t*)nullptr);
}

// The Q8_0 KV cache of layer L (null pointers for an fp32 cache).
KvQ kv_layer(const at_model* m, int L);

// Cluster size of the decode attention (clusters of chunk CTAs of one KV head
// merge through distributed shared memory): 16 where the device can place
// such clusters (non-portable size), else 8, else 0 (no clusters: MODE 1).
template <int HD>
int attn_cluster_size(int hkv, int nchunk, int batch) {
    auto kern = attn_split_kernel<HD, 2, kAttnClusterChunk>;
    const size_t smem = attn_smem_bytes(HD, kAttnClusterChunk);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    // the Q8_0-KV variant has the same footprint and launch shape
    auto kern_q = attn_split_kernel<HD, 2, kAttnClusterChunk, true>;
    if (cudaFuncSetAttribute(kern_q, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess ||
        cudaFuncSetAttribute(kern_q, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        cudaGetLastError();
    }
    for (int cs : {16, 8}) {
        if (cs == 16 &&
            cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(hkv, (nchunk + cs - 1) / cs * cs, batch);
        cfg.blockDim = dim3(256);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = cs;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n >= hkv * batch) return cs;
        cudaGetLastError();
    }
    return 0;
}

KvQ kv_layer(const at_model* m, int L) {
    if (!m->kv_q8) return KvQ{};
    const size_t off = (size_t)L * m->Hkvl * m->ctx_len * m->hd;
    return KvQ{m->kq8 + off, m->vq8 + off, m->ksc + off / 32, m->vsc + off / 32};
}

void enqueue_step(at_model* m, int B) {
    at_ctx* c = m->ctx;
    cudaStream_t s = c->stream;
    const int d = m->d, hd = m->hd;
    // Under tensor parallelism the wo and w2 GEMVs write their partial sums
    // into the peer-visible slot of their all-reduce site; the all-reduce
    // kernel leaves the sum in y.
    ArPeers peers{};
    for (int r = 0; r < c->world && r < kMaxRanks; ++r) peers.base[r] = m->ar_peer[r];
    auto area_off = [&](int site) -> int64_t { return (int64_t)site * c->world * m->ar_site_floats; };
    auto proj_out = [&](int site) -> float* {
        return (c->world > 1) ? m->ar_base + area_off(site) + (int64_t)c->rank * m->ar_site_floats : m->y;
    };
    auto allreduce_y = [&](int site) {
        if (c->world <= 1) return;
        ProfScope p(m, AT_PROF_COMM);
        launch_k(allreduce_push_kernel, dim3(c->world - 1), dim3(512), s, m->pdl, peers, c->world, c->rank,
                 area_off(site), m->ar_site_floats, m->ar_flag_off, site, B * d / 4, (const unsigned*)m->d_step,
                 m->y, m->d_ar_err);
    };
    {
        ProfScope p(m, AT_PROF_EMBED);
        if (m->tok.type == AT_GGML_Q6_K)
            launch_q6k_embed(&m->tok, m->d_tokens, B, d, m->xa, m->y, m->d_argkey, m->d_step, s);
        else if (m->tok.type == AT_GGML_Q4_0)
            embed_kernel<AT_GGML_Q4_0><<<B, 256, 0, s>>>(m->tok.tiles, tile_map(&m->tok), m->d_tokens, d, m->xa,
                                                          m->y, m->d_argkey, m->d_step);
        else
            embed_kernel<AT_GGML_Q8_0><<<B, 256, 0, s>>>(m->tok.tiles, tile_map(&m->tok), m->d_tokens, d, m->xa,
                                                          m->y, m->d_argkey, m->d_step);
        AT_CUDA(cudaGetLastError());
    }
    const float scale = (float)(1.0 / std::sqrt((double)hd));
    const size_t layer_kv = (size_t)m->Hkvl * m->ctx_len * hd;
    for (int L = 0; L < m->L; ++L) {
        Layer& ly = m->layers[L];
        float* kc = m->kv_q8 ? nullptr : m->kcache + L * layer_kv;
        float* vc = m->kv_q8 ? nullptr : m->vcache + L * layer_kv;
        const KvQ kvq = kv_layer(m, L);
        {
            ProfScope p(m, AT_PROF_QKV);
            GemvArgs a;
            a.xin = m->xa; a.yin = m->y; a.gamma = ly.attn_norm; a.xout = m->xb; a.eps = m->cfg.rms_norm_eps;
            a.x_stride = d;
            a.y = m->q; a.y_stride = m->Hl * hd;
            a.rope_cos = m->rope_cos; a.rope_sin = m->rope_sin; a.pos = m->d_pos;
            a.kcache = kc; a.vcache = vc;
            a.kq = kvq.kq; a.vq = kvq.vq; a.ksc = kvq.ks; a.vsc = kvq.vs;
            a.kv_slot_stride = m->slot_stride;
            a.head_dim = hd; a.n_q_cols = m->Hl * hd; a.n_kv_cols = m->Hkvl * hd; a.ctx_len = m->ctx_len;
            a.scratch = m->scratch; a.counters = m->counters;
            if (m->attn_n) {
                // [out][in] attention weights: plain QKV rows, then RoPE + KV append
                const int qcols = (m->Hl + 2 * m->Hkvl) * hd;
                a.y = m->qkvbuf; a.y_stride = qcols;
                launch_gemv_n(&ly.qkv, B, Pro::AddNorm, Epi::Plain, a, c->num_sms, s, m->pdl);
                qkv_rope_rows_kernel<<<B, 256, 0, s>>>(m->qkvbuf, qcols, m->q, kc, vc, kvq, m->slot_stride,
                                                       m->rope_cos, m->rope_sin, m->d_pos, hd, m->Hl * hd,
                                                       m->Hkvl * hd, m->ctx_len);
                AT_CUDA(cudaGetLastError());
            } else {
                launch_gemv_t(&ly.qkv, B, Pro::AddNorm, Epi::QkvRope, a, c->num_sms, s, m->pdl);
            }
        }
        {
            ProfScope p(m, AT_PROF_ATTN);
            dim3 g1(m->Hkvl, m->nchunk_max, B);
            const float* qp = m->q;
            const int64_t* dp = m->d_pos;
            // one launch (split + merge by the last CTA) when the merge
            // weights of a KV head's query heads fit the K staging buffer
            const bool fused = (m->Hl / m->Hkvl) * m->nchunk_max <= CH * hd;
            const int cs = m->attn_cs;
            // each cluster rank merges a whole number of float4 outputs
            if (fused && cs > 1 && ((m->Hl / m->Hkvl) * hd) % (4 * cs) == 0) {
                // 64-position chunks merged per cluster through distributed shared memory
                const int nch64 = (m->ctx_len + kAttnClusterChunk - 1) / kAttnClusterChunk;
                dim3 gc(m->Hkvl, (nch64 + cs - 1) / cs * cs, B);
                const size_t sm = attn_smem_bytes(hd, kAttnClusterChunk);
                if (hd == 128)
                    launch_attn<128, 2, kAttnClusterChunk>(kvq, kc, vc, gc, dim3(1, cs, 1), sm, s, m->pdl, qp, dp,
                                                           m->att_part, m->Hl, m->Hkvl, m->ctx_len, m->slot_stride,
                                                           m->nchunk_max, scale, m->attn_cnt, m->att);
                else
                    launch_attn<64, 2, kAttnClusterChunk>(kvq, kc, vc, gc, dim3(1, cs, 1), sm, s, m->pdl, qp, dp,
                                                          m->att_part, m->Hl, m->Hkvl, m->ctx_len, m->slot_stride,
                                                          m->nchunk_max, scale, m->attn_cnt, m->att);
            } else if (fused) {
                if (hd == 128)
                    launch_attn<128, 1, CH>(kvq, kc, vc, g1, dim3(1, 1, 1), attn_smem_bytes(128, CH), s, m->pdl, qp, dp,
                                            m->att_part, m->Hl, m->Hkvl, m->ctx_len, m->slot_stride, m->nchunk_max,
                                            scale, m->attn_cnt, m->att);
                else
                    launch_attn<64, 1, CH>(kvq, kc, vc, g1, dim3(1, 1, 1), attn_smem_bytes(64, CH), s, m->pdl, qp, dp,
                                           m->att_part, m->Hl, m->Hkvl, m->ctx_len, m->slot_stride, m->nchunk_max,
                                           scale, m->attn_cnt, m->att);
            } else {
                if (hd == 128)
                    launch_attn<128, 0, CH>(kvq, kc, vc, g1, dim3(1, 1, 1), attn_smem_bytes(128, CH), s, m->pdl, qp, dp,
                                            m->att_part, m->Hl, m->Hkvl, m->ctx_len, m->slot_stride, m->nchunk_max,
                                            scale, nullptr, nullptr);
                else
                    launch_attn<64, 0, CH>(kvq, kc, vc, g1, dim3(1, 1, 1), attn_smem_bytes(64, CH), s, m->pdl, qp, dp,
                                           m->att_part, m->Hl, m->Hkvl, m->ctx_len, m->slot_stride, m->nchunk_max,
                                           scale, nullptr, nullptr);
                dim3 g2(m->Hl, B);
                const float* pp = m->att_part;
                if (hd == 128)
                    launch_k(attn_combine_kernel<128>, g2, 128, s, m->pdl, pp, dp, m->att, m->Hl, m->nchunk_max);
                else
                    launch_k(attn_combine_kernel<64>, g2, 64, s, m->pdl, pp, dp, m->att, m->Hl, m->nchunk_max);
            }
        }
        {
            ProfScope p(m, AT_PROF_WO);
            GemvArgs o;
            o.x = m->att; o.x_stride = m->Hl * hd; o.y = proj_out(2 * L); o.y_stride = d;
            o.scratch = m->scratch; o.counters = m->counters;
            if (m->attn_n) launch_gemv_n(&ly.wo, B, Pro::Plain, Epi::Plain, o, c->num_sms, s, m->pdl);
            else launch_gemv_t(&ly.wo, B, Pro::Plain, Epi::Plain, o, c->num_sms, s, m->pdl);
        }
        allreduce_y(2 * L);
        {
            ProfScope p(m, AT_PROF_FFN_UP);
            GemvArgs f;
            f.xin = m->xb; f.yin = m->y; f.gamma = ly.ffn_norm; f.xout = m->xa; f.eps = m->cfg.rms_norm_eps;
            f.x_stride = d; f.y = m->h; f.y_stride = m->Fl; f.m2 = &ly.w3;
            f.scratch = m->scratch; f.counters = m->counters;
            launch_gemv_n(&ly.w1, B, Pro::AddNorm, Epi::SiluMul, f, c->num_sms, s, m->pdl);
        }
        {
            ProfScope p(m, AT_PROF_FFN_DOWN);
            GemvArgs dn;
            dn.x = m->h; dn.x_stride = m->Fl; dn.y = proj_out(2 * L + 1); dn.y_stride = d;
            dn.scratch = m->scratch; dn.counters = m->counters;
            launch_gemv_n(&ly.w2, B, Pro::Plain, Epi::Plain, dn, c->num_sms, s, m->pdl);
        }
        allreduce_y(2 * L + 1);
    }
    {
        ProfScope p(m, AT_PROF_LM_HEAD);
        GemvArgs ha;
        ha.xin = m->xa; ha.yin = m->y; ha.gamma = m->out_norm; ha.xout = m->xb;
        ha.eps = m->cfg.rms_norm_eps; ha.x_stride = d;
        ha.y = (c->world > 1) ? m->logits_local : m->logits; ha.y_stride = m->Vl;
        ha.scratch = m->scratch; ha.counters = m->counters;
        launch_gemv_n(&m->out, B, Pro::AddNorm, Epi::Plain, ha, c->num_sms, s, m->pdl);
    }
    if (c->world > 1) {
        ProfScope p(m, AT_PROF_COMM);
        const int site = 2 * m->L;
        launch_k(gather_push_kernel, dim3((c->world - 1) * kPushCtas), dim3(512), s, m->pdl, peers, c->world,
                 c->rank, area_off(site), m->ar_logit_floats, m->ar_flag_off, site, (const float*)m->logits_local, B,
                 m->Vl, m->V, (const unsigned*)m->d_step, m->logits, m->d_ar_err);
    }
    {
        ProfScope p(m, AT_PROF_ARGMAX);
        argmax_kernel<<<dim3(c->num_sms, B), 256, 0, s>>>(m->logits, m->V, m->V, m->d_argkey);
        AT_CUDA(cudaGetLastError());
        argmax_index_kernel<<<1, 32, 0, s>>>(m->d_argkey, B, m->d_argmax);
        AT_CUDA(cudaGetLastError());
    }
}

cudaGraphExec_t capture(at_model* m, void (*body)(at_model*, int), int B) {
    at_ctx* c = m->ctx;
    cudaGraph_t g = nullptr;
    AT_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    try {
        body(m, B);
    } catch (...) {
        cudaStreamEndCapture(c->stream, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    AT_CUDA(cudaStreamEndCapture(c->stream, &g));
    cudaGraphExec_t e = nullptr;
    const cudaError_t err = cudaGraphInstantiate(&e, g, 0);
    cudaGraphDestroy(g);
    AT_CUDA(err);
    return e;
}

void enqueue_generate_step(at_model* m, int) {
    enqueue_step(m, 1);
    advance_kernel<<<1, 1, 0, m->ctx->stream>>>(m->d_argmax, m->d_tokens, m->d_pos, m->d_gen_out, m->d_gen_count);
    AT_CUDA(cudaGetLastError());
}

// Fails the call when a tensor-parallel all-reduce gave up waiting for a peer
// (the peer died or never reached the step); the model is unusable after it.
void check_peer_allreduce(at_model* m) {
    if (m->ctx->world > 1 && m->h_ar_err && *m->h_ar_err)
        fail(AT_ERR_NCCL, "tensor-parallel all-reduce: a peer rank did not arrive within the wait limit");
}

void ds_launch(at_model* m, bool greedy);
void ds_check(at_model* m);

// Checks a step's inputs and enqueues it (copies in, the step); no wait.
void run_step_enqueue_only(at_model* m, const int* tokens, const int64_t* positions, int B) {
    AT_REQUIRE(m && m->finalized, AT_ERR_STATE, "model is not finalized");
    AT_REQUIRE(B >= 1 && B <= m->B, AT_ERR_INVALID_ARG, "batch exceeds the model's max_batch");
    AT_REQUIRE(tokens && positions, AT_ERR_INVALID_ARG, "null tokens/positions");
    for (int b = 0; b < B; ++b) {
        AT_REQUIRE(tokens[b] >= 0 && tokens[b] < m->V, AT_ERR_INVALID_ARG,
                   "token id " + std::to_string(tokens[b]) + " out of range");
        AT_REQUIRE(positions[b] >= 0, AT_ERR_INVALID_ARG, "negative position");
        // KVCache.append (inference/KVCache.java:83-85)
        AT_REQUIRE(positions[b] < m->ctx_len, AT_ERR_STATE,
                   "position " + std::to_string(positions[b]) + " exceeds maxContext " + std::to_string(m->ctx_len));
    }
    at_ctx* c = m->ctx;
    AT_CUDA(cudaSetDevice(c->device));
    // previous step's copies out of the pinned buffers are complete (stream order + sync below)
    for (int b = 0; b < B; ++b) { m->h_tokens[b] = tokens[b]; m->h_pos[b] = positions[b]; }
    AT_CUDA(cudaMemcpyAsync(m->d_tokens, m->h_tokens, sizeof(int) * B, cudaMemcpyHostToDevice, c->stream));
    AT_CUDA(cudaMemcpyAsync(m->d_pos, m->h_pos, sizeof(int64_t) * B, cudaMemcpyHostToDevice, c->stream));
    if (B == 1 && m->use_ds) {
        ds_launch(m, false);
        AT_CUDA(cudaMemcpyAsync(m->h_ds_err, m->ds_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    } else {
        if (!m->graph[B]) m->graph[B] = capture(m, enqueue_step, B);
        AT_CUDA(cudaGraphLaunch(m->graph[B], c->stream));
    }
}

void run_step(at_model* m, const int* tokens, const int64_t* positions, int B, float* logits_host) {
    run_step_enqueue_only(m, tokens, positions, B);
    at_ctx* c = m->ctx;
    if (logits_host)
        AT_CUDA(cudaMemcpyAsync(logits_host, m->logits, sizeof(float) * (size_t)B * m->V, cudaMemcpyDeviceToHost,
                                c->stream));
    if (c->world > 1)
        AT_CUDA(cudaMemcpyAsync(m->h_ar_err, m->d_ar_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    AT_CUDA(cudaStreamSynchronize(c->stream));
    check_peer_allreduce(m);
    ds_check(m);
    for (int b = 0; b < B; ++b) m->kv_size[b] = std::max<int64_t>(m->kv_size[b], positions[b] + 1);
}

void destroy_model(at_model* m) {
    if (!m) return;
    at_ctx* c = m->ctx;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    if (c->world > 1 && m->ar_base) {
        // No peer may still write into this rank's areas when they are freed:
        // the teardown barrier completes only after every peer's last push.
        // A peer that never arrives ends the wait at its bound instead (and
        // the areas are then left allocated, below).
        ArPeers peers{};
        for (int r = 0; r < c->world; ++r) peers.base[r] = m->ar_peer[r];
        peer_barrier_kernel<<<c->world - 1, 32, 0, c->stream>>>(peers, c->world, c->rank, m->ar_flag_off,
                                                                2 * m->L + 1, m->d_ar_err);
        cudaStreamSynchronize(c->stream);
        for (int r = 0; r < c->world; ++r)
            if (r != c->rank && m->ar_peer[r]) cudaIpcCloseMemHandle(m->ar_peer[r]);
        int err = 0;
        if (m->d_ar_err) cudaMemcpy(&err, m->d_ar_err, sizeof(int), cudaMemcpyDeviceToHost);
        // After a failed wait a live peer may still push into the receive
        // areas, so they are left allocated rather than freed under it.
        if (err) m->ar_base = nullptr;
    }
    for (auto& g : m->graph)
        if (g) cudaGraphExecDestroy(g);
    for (auto& g : m->graph_samp)
        if (g) cudaGraphExecDestroy(g);
    if (m->graph_gen) cudaGraphExecDestroy(m->graph_gen);
    if (m->graph_prof) cudaGraphExecDestroy(m->graph_prof);
    for (cudaEvent_t e : m->prof_ev) cudaEventDestroy(e);
    for (auto& ly : m->layers) {
        qmat_free(&ly.qkv); qmat_free(&ly.wo); qmat_free(&ly.w1); qmat_free(&ly.w3); qmat_free(&ly.w2);
        cudaFree(ly.attn_norm); cudaFree(ly.ffn_norm);
    }
    qmat_free(&m->tok);
    qmat_free(&m->out);
    void* bufs[] = {m->out_norm, m->xa, m->xb, m->y, m->q, m->att, m->h, m->logits, m->logits_local,
                    m->att_part, m->attn_cnt, m->kcache, m->vcache, m->rope_cos, m->rope_sin, m->scratch, m->counters,
                    m->d_tokens, m->d_pos, m->d_argmax, m->d_gen_out, m->d_gen_count, m->d_argkey,
                    m->d_step, m->ar_base, m->d_ar_err, m->pf_xa, m->pf_xb, m->pf_y, m->pf_qkv, m->pf_q,
                    m->pf_att, m->pf_g, m->pf_u, m->pf_tok, m->pf_pos, m->pf_err, m->pf_xbf, m->pf_ws,
                    m->d_ds_layers, m->ds_qkv_part, m->ds_wo_part, m->ds_apart, m->ds_tickets, m->ds_bar,
                    m->ds_err, m->ds_stamps, m->qkvbuf, m->d_rows, m->d_hist, m->d_hist_len, m->d_pen_cnt,
                    m->d_rng, m->d_sampled, m->d_seq, m->d_step_ctr, m->d_append, m->kq8, m->vq8, m->ksc, m->vsc, m->kv_stage};
    for (void* p : bufs)
        if (p) cudaFree(p);
    if (m->h_tokens) cudaFreeHost(m->h_tokens);
    if (m->h_pos) cudaFreeHost(m->h_pos);
    if (m->h_ar_err) cudaFreeHost(m->h_ar_err);
    if (m->h_pf_tok) cudaFreeHost(m->h_pf_tok);
    if (m->h_pf_pos) cudaFreeHost(m->h_pf_pos);
    if (m->h_ds_err) cudaFreeHost(m->h_ds_err);
    if (m->h_rows) cudaFreeHost(m->h_rows);
    if (m->h_i32) cudaFreeHost(m->h_i32);
    if (m->h_rng) cudaFreeHost(m->h_rng);
    delete m;
}

// Persistent decode step (opt-in with AT_DECODE_STEP=1 at load): batch 1 on
// one GPU when every matrix (token embedding and lm_head included) shares one
// quantized type the kernel supports. Measured slower than the per-kernel
// step graph on B200 (Llama-3-8B Q4_0: 3.23 against 1.97 ms per token), so
// the graph stays the default.
void setup_decode_step(at_model* m) {
    at_ctx* c = m->ctx;
    const char* env = std::getenv("AT_DECODE_STEP");
    if (!env || env[0] != '1') return;
    if (c->world != 1 || m->layers.empty() || m->layout != 0 || m->kv_q8) return;
    const int qt = m->layers[0].qkv.type;
    for (auto& ly : m->layers)
        for (const at_qmat* q : {&ly.qkv, &ly.wo, &ly.w1, &ly.w3, &ly.w2})
            if (q->type != qt || !q->tiles) return;
    if (m->out.type != qt || !m->out.tiles || m->tok.type != qt || !m->tok.tiles) return;
    DsParams p{};
    p.qtype = qt;
    p.hd = m->hd;
    p.d = m->d;
    p.Hl = m->Hl;
    p.Hkvl = m->Hkvl;
    p.Fl = m->Fl;
    p.Vl = m->Vl;
    p.ctx = m->ctx_len;
    p.L = m->L;
    p.eps = m->cfg.rms_norm_eps;
    p.scale = (float)(1.0 / std::sqrt((double)m->hd));
    if (!decode_step_configure(&p, c->num_sms)) return;
    if (const char* ns = std::getenv("AT_DS_NST")) {  // ring depth override (measurement knob)
        const int v = std::atoi(ns);
        if (v == 2 || v == 4 || v == 8) {
            DsParams q = p;
            q.nst = v;
            if (decode_step_smem(q) <= 232448 - 20 * 1024) p = q;
        }
    }
    const Layer& l0 = m->layers[0];
    if (l0.qkv.tile_bytes != p.tile_t || l0.w1.tile_bytes != p.tile_n || l0.qkv.ngroups != p.qkv.ngroups ||
        l0.wo.ngroups != p.wo.ngroups || l0.w1.nsteps != p.gu.nsteps || l0.w2.nsteps != p.dn.nsteps ||
        m->out.nsteps != p.head.nsteps || m->out.ngroups != p.head.ngroups)
        return;
    std::vector<DsLayer> tab(m->L);
    const size_t layer_kv = (size_t)m->Hkvl * m->ctx_len * m->hd;
    for (int L = 0; L < m->L; ++L) {
        const Layer& ly = m->layers[L];
        tab[L] = DsLayer{ly.qkv.tiles, ly.wo.tiles, ly.w1.tiles, ly.w3.tiles, ly.w2.tiles, ly.attn_norm, ly.ffn_norm,
                         m->kcache + L * layer_kv, m->vcache + L * layer_kv};
    }
    AT_CUDA(cudaMalloc(&m->d_ds_layers, sizeof(DsLayer) * m->L));
    AT_CUDA(cudaMemcpy(m->d_ds_layers, tab.data(), sizeof(DsLayer) * m->L, cudaMemcpyHostToDevice));
    const int G = m->Hl / m->Hkvl;
    alloc_zero((void**)&m->ds_qkv_part, (size_t)p.qkv.ncols * p.qkv.S * 32 * 4);
    alloc_zero((void**)&m->ds_wo_part, (size_t)p.wo.ncols * p.wo.S * 32 * 4);
    alloc_zero((void**)&m->ds_apart, (size_t)m->Hkvl * p.att_max_ctas * G * (m->hd + 2) * 4);
    alloc_zero((void**)&m->ds_tickets, (size_t)(m->Hkvl + 1) * sizeof(unsigned));
    alloc_zero((void**)&m->ds_bar, 2 * sizeof(unsigned));
    alloc_zero((void**)&m->ds_err, sizeof(int));
    AT_CUDA(cudaMallocHost(&m->h_ds_err, sizeof(int)));
    *m->h_ds_err = 0;
    p.layers = m->d_ds_layers;
    p.tok_tiles = m->tok.tiles;
    p.tok_map = tile_map(&m->tok);
    p.out_tiles = m->out.tiles;
    p.out_norm = m->out_norm;
    p.rope_cos = m->rope_cos;
    p.rope_sin = m->rope_sin;
    p.tokens = m->d_tokens;
    p.pos = m->d_pos;
    p.res0 = m->xa;
    p.res1 = m->xb;
    p.ydown = m->y;
    p.qkv_part = m->ds_qkv_part;
    p.wo_part = m->ds_wo_part;
    p.h = m->h;
    p.att = m->att;
    p.apart = m->ds_apart;
    p.logits = m->logits;
    p.tickets = m->ds_tickets;
    p.bar = m->ds_bar;
    p.err = m->ds_err;
    p.argkey = m->d_argkey;
    p.argmax_out = m->d_argmax;
    p.gen_out = m->d_gen_out;
    p.gen_count = m->d_gen_count;
    p.greedy = 0;
    p.stamps = nullptr;
    m->ds = p;
    m->use_ds = true;
}

void ds_launch(at_model* m, bool greedy) {
    DsParams p = m->ds;
    p.greedy = greedy ? 1 : 0;
    p.stamps = m->ds_stamps;
    launch_decode_step(p, m->ctx->num_sms, m->ctx->stream);
}

// After the stream has synchronized: fails the call when a bounded wait of
// the step kernel ran out, after clearing its counters for the next launch.
void ds_check(at_model* m) {
    if (!m->use_ds || !*m->h_ds_err) return;
    const int code = *m->h_ds_err;
    *m->h_ds_err = 0;
    cudaMemset(m->ds_err, 0, sizeof(int));
    cudaMemset(m->ds_bar, 0, 2 * sizeof(unsigned));
    cudaMemset(m->ds_tickets, 0, (size_t)(m->Hkvl + 1) * sizeof(unsigned));
    cudaMemset(m->d_argkey, 0, sizeof(unsigned long long));
    cudaDeviceSynchronize();
    fail(AT_ERR_CUDA, std::string("decode step: a bounded wait ran out (") +
                          (code == 1 ? "weight copy" : "grid barrier") + ")");
}

// --- GGUF ------------------------------------------------------------------
struct GgufView {
    const uint8_t* base = nullptr;
    size_t len = 0;
    size_t pos = 0;
    void need(size_t n) {
        if (pos + n > len) fail(AT_ERR_IO, "truncated GGUF file");
    }
    template <class T>
    T rd() {
        need(sizeof(T));
        T v;
        memcpy(&v, base + pos, sizeof(T));
        pos += sizeof(T);
        return v;
    }
    std::string str() {
        const int64_t n = rd<int64_t>();
        if (n < 0 || n > 0x7fffffff) fail(AT_ERR_IO, "implausible string length");
        need((size_t)n);
        std::string s(reinterpret_cast<const char*>(base + pos), (size_t)n);
        pos += (size_t)n;
        return s;
    }
};

struct MetaVal {
    int type = -1;
    double num = 0;
    bool is_num = false;
    std::string s;
};

// GgufFile.readValue (format/GgufFile.java:259-294); arrays are skipped.
MetaVal read_value(GgufView& v, int vt) {
    MetaVal r;
    r.type = vt;
    switch (vt) {
        case 0: r.num = v.rd<uint8_t>(); r.is_num = true; break;
        case 1: r.num = v.rd<int8_t>(); r.is_num = true; break;
        case 2: r.num = v.rd<uint16_t>(); r.is_num = true; break;
        case 3: r.num = v.rd<int16_t>(); r.is_num = true; break;
        case 4: r.num = v.rd<uint32_t>(); r.is_num = true; break;
        case 5: r.num = v.rd<int32_t>(); r.is_num = true; break;
        case 6: r.num = v.rd<float>(); r.is_num = true; break;
        case 7: r.num = v.rd<uint8_t>() != 0; break;
        case 8: r.s = v.str(); break;
        case 9: {
            const int et = v.rd<int32_t>();
            const int64_t n = v.rd<int64_t>();
            if (n < 0 || n > (1 << 26)) fail(AT_ERR_IO, "implausible array length");
            for (int64_t i = 0; i < n; ++i) read_value(v, et);
            break;
        }
        case 10: r.num = (double)v.rd<uint64_t>(); r.is_num = true; break;
        case 11: r.num = (double)v.rd<int64_t>(); r.is_num = true; break;
        case 12: r.num = v.rd<double>(); r.is_num = true; break;
        default: fail(AT_ERR_IO, "Unknown GGUF metadata value type: " + std::to_string(vt));
    }
    return r;
}

}  // namespace

extern "C" {

int at_tp_unique_id(uint8_t out_id[128]) {
    return guard([&] {
        AT_REQUIRE(out_id, AT_ERR_INVALID_ARG, "null output");
        ncclUniqueId id;
        nccl_check(nccl().GetUniqueId(&id), "ncclGetUniqueId");
        static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
        memcpy(out_id, &id, 128);
    });
}

int at_ctx_create_tp(int device, int rank, int world, const uint8_t id[128], at_ctx** out) {
    at_ctx* c = nullptr;
    const int rc = guard([&] {
        AT_REQUIRE(out && id, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(world >= 1 && rank >= 0 && rank < world, AT_ERR_INVALID_ARG, "bad rank/world");
        const int r0 = at_ctx_create(device, &c);
        if (r0 != AT_OK) fail(r0, "context creation failed");
        c->rank = rank;
        c->world = world;
        if (world > 1) {
            ncclUniqueId uid;
            memcpy(&uid, id, 128);
            ncclComm_t comm;
            AT_CUDA(cudaSetDevice(device));
            nccl_check(nccl().CommInitRank(&comm, world, uid, rank), "ncclCommInitRank");
            c->nccl_comm = comm;
        }
        *out = c;
    });
    if (rc != AT_OK && c) at_ctx_destroy(c);
    return rc;
}

int at_ctx_destroy(at_ctx* ctx) {
    return guard([&] {
        if (!ctx) return;
        cudaSetDevice(ctx->device);
        if (ctx->stream) cudaStreamSynchronize(ctx->stream);
        if (ctx->nccl_comm) nccl().CommDestroy((ncclComm_t)ctx->nccl_comm);
        if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
        delete ctx;
    });
}

int at_model_create(at_ctx* ctx, const at_model_config* cfg, at_model** out) {
    at_model* m = nullptr;
    const int rc = guard([&] {
        AT_REQUIRE(ctx && cfg && out, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(cfg->head_count > 0, AT_ERR_STATE, "headCount == 0");
        AT_REQUIRE(cfg->context_length > 0 && cfg->embedding_length > 0 && cfg->block_count > 0 &&
                       cfg->head_count_kv > 0 && cfg->feed_forward_length > 0 && cfg->vocab_size > 0,
                   AT_ERR_INVALID_ARG, "model dims must be positive");
        AT_CUDA(cudaSetDevice(ctx->device));
        m = new at_model();
        m->ctx = ctx;
        m->cfg = *cfg;
        AT_REQUIRE((cfg->layout & ~AT_LAYOUT_LLAMA_CPP) == 0, AT_ERR_INVALID_ARG, "unknown layout bits");
        m->layout = cfg->layout;
        m->attn_n = (cfg->layout & AT_LAYOUT_ATTN_OUT_IN) != 0;
        AT_REQUIRE(cfg->kv_type == AT_GGML_F32 || cfg->kv_type == AT_GGML_Q8_0, AT_ERR_UNSUPPORTED,
                   "KV cache type must be F32 or Q8_0");
        m->kv_q8 = cfg->kv_type == AT_GGML_Q8_0;
        m->B = cfg->max_batch < 1 ? 1 : cfg->max_batch;
        AT_REQUIRE(m->B <= 8, AT_ERR_INVALID_ARG, "max_batch must be in [1, 8]");
        m->d = (int)cfg->embedding_length;
        m->H = (int)cfg->head_count;
        m->Hkv = (int)cfg->head_count_kv;
        m->hd = m->d / m->H;  // LlamaConfig.headDim (inference/LlamaConfig.java:293-296)
        m->F = (int)cfg->feed_forward_length;
        m->V = (int)cfg->vocab_size;
        m->L = (int)cfg->block_count;
        m->ctx_len = (int)cfg->context_length;
        const int W = ctx->world;
        AT_REQUIRE(m->hd == 64 || m->hd == 128, AT_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
        AT_REQUIRE(cfg->context_length <= 32768, AT_ERR_UNSUPPORTED, "context_length above 32768");
        AT_REQUIRE(m->d % 32 == 0, AT_ERR_INVALID_ARG, "embedding_length must be a multiple of 32");
        AT_REQUIRE(m->H % m->Hkv == 0 && m->H / m->Hkv <= 8, AT_ERR_UNSUPPORTED, "query heads per KV head must be 1..8");
        AT_REQUIRE(m->Hkv % W == 0, AT_ERR_INVALID_ARG, "KV heads must divide evenly across tensor-parallel ranks");
        AT_REQUIRE(m->F % (32 * W) == 0, AT_ERR_INVALID_ARG, "FFN width must split into 32-aligned shards");
        m->Hl = m->H / W;
        m->Hkvl = m->Hkv / W;
        m->Fl = m->F / W;
        m->Vl = (m->V + W - 1) / W;
        m->layers.resize(m->L);
        m->kv_size.assign(m->B, 0);
        *out = m;
    });
    if (rc != AT_OK && m) destroy_model(m);
    return rc;
}

int at_tp_shard_region(const at_model_config* cfg, int world, int rank, const char* tensor_name,
                       at_shard_region* out) {
    return guard([&] {
        AT_REQUIRE(cfg && tensor_name && out, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(world >= 1 && world <= 8 && rank >= 0 && rank < world, AT_ERR_INVALID_ARG,
                   "rank must be in [0, world) and world in [1, 8]");
        AT_REQUIRE(cfg->head_count > 0 && cfg->head_count_kv > 0 && cfg->embedding_length % cfg->head_count == 0,
                   AT_ERR_INVALID_ARG, "embedding_length must be a multiple of head_count");
        const int64_t H = cfg->head_count, Hkv = cfg->head_count_kv, F = cfg->feed_forward_length;
        const int64_t V = cfg->vocab_size, d = cfg->embedding_length;
        AT_REQUIRE(Hkv % world == 0, AT_ERR_INVALID_ARG, "KV heads must divide evenly across tensor-parallel ranks");
        AT_REQUIRE(F % (32 * world) == 0, AT_ERR_INVALID_ARG, "FFN width must split into 32-aligned shards");
        const ShardDims s{d, d / H, H, Hkv, F, V, H / world, Hkv / world, F / world, (V + world - 1) / world,
                          world, rank, (cfg->layout & AT_LAYOUT_ATTN_OUT_IN) != 0};
        shard_region(s, tensor_name, out);
    });
}

int at_model_set_tensor(at_model* m, const char* cname, int type, const void* data, size_t bytes, int on_device) {
    void* staging = nullptr;
    const int rc = guard([&] {
        AT_REQUIRE(m && cname && data, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(!m->finalized, AT_ERR_STATE, "model already finalized");
        at_ctx* c = m->ctx;
        AT_CUDA(cudaSetDevice(c->device));
        const std::string name(cname);
        const int d = m->d;
        int layer = -1;
        std::string leaf;
        const bool is_layer = parse_layer(name, &layer, &leaf);
        if (is_layer) AT_REQUIRE(layer >= 0 && layer < m->L, AT_ERR_INVALID_ARG, "layer index out of range: " + name);
        at_shard_region rg;
        shard_region(shard_dims(m, c->world, c->rank), name, &rg);
        const bool is_norm = rg.target == AT_SHARD_NORM;
        if (rg.target == AT_SHARD_NONE) return;  // tensors the decode path does not read are ignored, as in Weights.load
        const int64_t rows = rg.rows, cols = rg.cols;
        const int64_t numel = rows * cols;
        size_t expect;
        const bool emb_or_out = name == "token_embd.weight" || name == "output.weight";
        if (type == AT_GGML_F32) expect = (size_t)numel * 4;
        else if (type == AT_GGML_F16) expect = (size_t)numel * 2;
        else if (type == AT_GGML_Q4_0 || type == AT_GGML_Q8_0) expect = (size_t)raw_bytes(type, numel);
        else if (type == AT_GGML_Q6_K && emb_or_out && cols % 256 == 0) expect = (size_t)raw_bytes(type, numel);
        else fail(AT_ERR_UNSUPPORTED, "tensor '" + name + "' has unsupported type " + std::to_string(type));
        AT_REQUIRE(bytes == expect, AT_ERR_INVALID_ARG,
                   "tensor '" + name + "' has " + std::to_string(bytes) + " bytes, expected " + std::to_string(expect));
        const void* src = data;
        if (!on_device) {
            AT_CUDA(cudaMalloc(&staging, bytes));
            AT_CUDA(cudaMemcpyAsync(staging, data, bytes, cudaMemcpyHostToDevice, c->stream));
            src = staging;
        }
        const uint8_t* s8 = static_cast<const uint8_t*>(src);
        if (is_norm) {
            float** dst = (name == "output_norm.weight") ? &m->out_norm
                          : (leaf == "attn_norm.weight" ? &m->layers[layer].attn_norm : &m->layers[layer].ffn_norm);
            if (!*dst) alloc_zero((void**)dst, (size_t)d * 4);
            at_qmat tmp;
            tmp.type = AT_GGML_F32; tmp.rows = 1; tmp.cols = d; tmp.f32 = *dst; tmp.owns = false;
            qmat_fill_from_float(&tmp, src, type, d, 0, 0, c->stream);
        } else {
            AT_REQUIRE(type == AT_GGML_Q4_0 || type == AT_GGML_Q8_0 || (type == AT_GGML_Q6_K && emb_or_out),
                       AT_ERR_UNSUPPORTED,
                       "tensor '" + name + "': the device path keeps weight matrices in Q4_0 or Q8_0 "
                       "(Q6_K for token_embd and output)");
            if (m->wtype < 0 && type != AT_GGML_Q6_K) m->wtype = type;
            const int nib_split = m->layout & AT_LAYOUT_Q4_SPLIT_HALVES;
            auto place = [&](at_qmat& q, int orient, int64_t qr, int64_t qc, int64_t sr0, int64_t sc0, int64_t nr,
                             int64_t nc, int64_t dr0, int64_t dc0) {
                make_qmat(q, type, orient, qr, qc);
                AT_REQUIRE(q.type == type, AT_ERR_UNSUPPORTED,
                           "tensor '" + name + "' differs in type from the tensors fused with it");
                qmat_fill_region(&q, s8, cols, sr0, sc0, nr, nc, dr0, dc0, c->stream, nib_split);
            };
            at_qmat* dst = nullptr;
            switch (rg.target) {
                case AT_SHARD_TOKEN_EMBD: dst = &m->tok; break;
                case AT_SHARD_OUTPUT: dst = &m->out; break;
                case AT_SHARD_QKV: dst = &m->layers[layer].qkv; break;
                case AT_SHARD_WO: dst = &m->layers[layer].wo; break;
                case AT_SHARD_W1: dst = &m->layers[layer].w1; break;
                case AT_SHARD_W3: dst = &m->layers[layer].w3; break;
                case AT_SHARD_W2: dst = &m->layers[layer].w2; break;
                default: fail(AT_ERR_INVALID_ARG, "tensor '" + name + "' has no device matrix");
            }
            place(*dst, rg.orient, rg.local_rows, rg.local_cols, rg.src_row0, rg.src_col0, rg.n_rows, rg.n_cols,
                  rg.dst_row0, rg.dst_col0);
        }
        AT_CUDA(cudaStreamSynchronize(c->stream));
        m->seen[name] = true;
    });
    if (staging) cudaFree(staging);
    return rc;
}

// Allocates this rank's receive areas (2 all-reduce sites per layer with one
// max-batch x dim slot per rank, the logits site with one shard slot per
// rank, then the flags of every site plus the teardown site), exports them
// with CUDA IPC, and maps
// every peer's slots: the 64-byte handles travel through one ncclAllGather.
void setup_peer_allreduce(at_model* m) {
    at_ctx* c = m->ctx;
    AT_REQUIRE(c->world <= kMaxRanks, AT_ERR_UNSUPPORTED, "tensor parallelism supports at most 8 ranks");
    // sites 0..2L-1: all-reduce slots; site 2L: logits shards; site 2L+1: teardown flags
    const int sites = 2 * m->L;
    m->ar_site_floats = ((int64_t)m->B * m->d + 63) / 64 * 64;
    m->ar_logit_floats = ((int64_t)m->B * m->Vl + 63) / 64 * 64;
    m->ar_flag_off = ((int64_t)sites * m->ar_site_floats + m->ar_logit_floats) * c->world;
    AT_REQUIRE(m->ar_logit_floats >= m->ar_site_floats, AT_ERR_UNSUPPORTED, "vocabulary shard smaller than dim");
    const int64_t nflags = (int64_t)(sites + 2) * c->world * kPushCtas;
    const size_t bytes = (size_t)(m->ar_flag_off + (nflags + 63) / 64 * 64) * 4;
    alloc_zero((void**)&m->ar_base, bytes);
    cudaIpcMemHandle_t mine;
    AT_CUDA(cudaIpcGetMemHandle(&mine, m->ar_base));
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    uint8_t* d_h = nullptr;
    AT_CUDA(cudaMalloc(&d_h, 64 * (size_t)(c->world + 1)));
    AT_CUDA(cudaMemcpyAsync(d_h + 64 * c->world, &mine, 64, cudaMemcpyHostToDevice, c->stream));
    nccl_check(nccl().AllGather(d_h + 64 * c->world, d_h, 64, ncclUint8, (ncclComm_t)c->nccl_comm, c->stream),
               "ncclAllGather(IPC handles)");
    std::vector<cudaIpcMemHandle_t> all(c->world);
    AT_CUDA(cudaMemcpyAsync(all.data(), d_h, 64 * (size_t)c->world, cudaMemcpyDeviceToHost, c->stream));
    AT_CUDA(cudaStreamSynchronize(c->stream));
    cudaFree(d_h);
    for (int r = 0; r < c->world; ++r) {
        if (r == c->rank) {
            m->ar_peer[r] = m->ar_base;
        } else {
            void* p = nullptr;
            AT_CUDA(cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess));
            m->ar_peer[r] = static_cast<float*>(p);
        }
    }
}

int at_model_finalize(at_model* m) {
    return guard([&] {
        AT_REQUIRE(m, AT_ERR_INVALID_ARG, "null model");
        if (m->finalized) return;
        at_ctx* c = m->ctx;
        AT_CUDA(cudaSetDevice(c->device));
        const int d = m->d, hd = m->hd, B = m->B;
        const int wt = m->wtype < 0 ? AT_GGML_Q8_0 : m->wtype;
        const int64_t qcols = (int64_t)(m->Hl + 2 * m->Hkvl) * hd;
        // Missing tensors become zeros (inference/Weights.java:131-135).
        make_qmat(m->tok, wt, AT_ORIENT_N, m->V, d);
        make_qmat(m->out, wt, AT_ORIENT_N, m->Vl, d);
        if (!m->out_norm) alloc_zero((void**)&m->out_norm, (size_t)d * 4);
        for (auto& ly : m->layers) {
            if (m->attn_n) {
                make_qmat(ly.qkv, wt, AT_ORIENT_N, qcols, d);
                make_qmat(ly.wo, wt, AT_ORIENT_N, d, (int64_t)m->Hl * hd);
            } else {
                make_qmat(ly.qkv, wt, AT_ORIENT_T, d, qcols);
                make_qmat(ly.wo, wt, AT_ORIENT_T, (int64_t)m->Hl * hd, d);
            }
            make_qmat(ly.w1, wt, AT_ORIENT_N, m->Fl, d);
            make_qmat(ly.w3, ly.w1.type, AT_ORIENT_N, m->Fl, d);
            make_qmat(ly.w2, wt, AT_ORIENT_N, d, m->Fl);
            if (!ly.attn_norm) alloc_zero((void**)&ly.attn_norm, (size_t)d * 4);
            if (!ly.ffn_norm) alloc_zero((void**)&ly.ffn_norm, (size_t)d * 4);
            AT_REQUIRE(ly.w1.type == ly.w3.type, AT_ERR_UNSUPPORTED, "ffn_gate and ffn_up must share a type");
        }
        // activations
        alloc_zero((void**)&m->xa, (size_t)B * d * 4);
        alloc_zero((void**)&m->xb, (size_t)B * d * 4);
        alloc_zero((void**)&m->y, (size_t)B * d * 4);
        alloc_zero((void**)&m->q, (size_t)B * m->Hl * hd * 4);
        alloc_zero((void**)&m->att, (size_t)B * m->Hl * hd * 4);
        alloc_zero((void**)&m->h, (size_t)B * m->Fl * 4);
        alloc_zero((void**)&m->logits, (size_t)B * m->V * 4);
        if (c->world > 1) {
            alloc_zero((void**)&m->logits_local, (size_t)B * m->Vl * 4);
        }
        m->nchunk_max = (m->ctx_len + CH - 1) / CH;
        {
            const int nch64 = (m->ctx_len + kAttnClusterChunk - 1) / kAttnClusterChunk;
            m->attn_cs = (hd == 128) ? attn_cluster_size<128>(m->Hkvl, nch64, B)
                                     : attn_cluster_size<64>(m->Hkvl, nch64, B);
        }
        alloc_zero((void**)&m->att_part, (size_t)B * m->Hl * m->nchunk_max * (hd + 2) * 4);
        alloc_zero((void**)&m->attn_cnt, (size_t)B * m->Hkvl * sizeof(unsigned));
        // KV cache (inference/KVCache.java:43-63): [slot][layer][kvHead][ctx][headDim] fp32
        m->slot_stride = (int64_t)m->L * m->Hkvl * m->ctx_len * hd;
        if (m->kv_q8) {
            alloc_zero((void**)&m->kq8, (size_t)B * m->slot_stride);
            alloc_zero((void**)&m->vq8, (size_t)B * m->slot_stride);
            alloc_zero((void**)&m->ksc, (size_t)B * m->slot_stride / 32 * 2);
            alloc_zero((void**)&m->vsc, (size_t)B * m->slot_stride / 32 * 2);
        } else {
            alloc_zero((void**)&m->kcache, (size_t)B * m->slot_stride * 4);
            alloc_zero((void**)&m->vcache, (size_t)B * m->slot_stride * 4);
        }
        // RoPE tables (inference/RopeCache.java:154-177): freq = (float) pow(base, -2i/hd)
        // in double, angle = pos * freq in float, cos/sin in double then float.
        {
            std::vector<float> cs((size_t)m->ctx_len * hd), sn((size_t)m->ctx_len * hd);
            const double base = (double)m->cfg.rope_freq_base;
            for (int64_t p = 0; p < m->ctx_len; ++p)
                for (int i = 0; i < hd / 2; ++i) {
                    const float freq = (float)std::pow(base, -2.0 * i / (double)hd);
                    const float ang = (float)p * freq;
                    const float cv = (float)std::cos((double)ang), sv = (float)std::sin((double)ang);
                    cs[p * hd + 2 * i] = cv; cs[p * hd + 2 * i + 1] = cv;
                    sn[p * hd + 2 * i] = sv; sn[p * hd + 2 * i + 1] = sv;
                }
            AT_CUDA(cudaMalloc(&m->rope_cos, cs.size() * 4));
            AT_CUDA(cudaMalloc(&m->rope_sin, sn.size() * 4));
            AT_CUDA(cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
            AT_CUDA(cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
        }
        // split scratch for the GEMVs at every batch size (launches are serialized on the stream)
        size_t nf = 16, nc = 16;
        for (int b = 1; b <= B; ++b) {
            size_t f1, c1;
            for (const at_qmat* q : {&m->layers[0].qkv, &m->layers[0].wo, &m->layers[0].w1, &m->layers[0].w2, &m->out}) {
                if (q->orient == AT_ORIENT_T) gemv_t_scratch_need(q, b, c->num_sms, &f1, &c1);
                else gemv_n_scratch_need(q, b, c->num_sms, &f1, &c1);
                nf = std::max(nf, f1); nc = std::max(nc, c1);
            }
        }
        if (m->attn_n) alloc_zero((void**)&m->qkvbuf, (size_t)B * qcols * 4);
        alloc_zero((void**)&m->scratch, nf * 4);
        alloc_zero((void**)&m->counters, nc * 4);
        alloc_zero((void**)&m->d_tokens, 8 * sizeof(int));
        alloc_zero((void**)&m->d_pos, 8 * sizeof(int64_t));
        alloc_zero((void**)&m->d_step, sizeof(unsigned));
        alloc_zero((void**)&m->d_ar_err, sizeof(int));
        AT_CUDA(cudaMallocHost(&m->h_ar_err, sizeof(int)));
        *m->h_ar_err = 0;
        if (c->world > 1) setup_peer_allreduce(m);
        alloc_zero((void**)&m->d_argmax, 8 * sizeof(int));
        alloc_zero((void**)&m->d_argkey, 8 * sizeof(unsigned long long));
        alloc_zero((void**)&m->d_gen_out, (size_t)m->ctx_len * sizeof(int));
        alloc_zero((void**)&m->d_gen_count, sizeof(int));
        AT_CUDA(cudaMallocHost(&m->h_tokens, 8 * sizeof(int)));
        AT_CUDA(cudaMallocHost(&m->h_pos, 8 * sizeof(int64_t)));
        setup_decode_step(m);
        AT_CUDA(cudaDeviceSynchronize());
        m->finalized = true;
    });
}

int at_model_load_gguf(at_ctx* ctx, const char* path, int max_batch, at_model** out) {
    return at_model_load_gguf_ex(ctx, path, max_batch, 0, AT_GGML_F32, out);
}

int at_model_load_gguf_ex(at_ctx* ctx, const char* path, int max_batch, int layout, int kv_type, at_model** out) {
    int fd = -1;
    void* map = MAP_FAILED;
    size_t len = 0;
    at_model* m = nullptr;
    const int rc = guard([&] {
        AT_REQUIRE(ctx && path && out, AT_ERR_INVALID_ARG, "null argument");
        fd = open(path, O_RDONLY);
        AT_REQUIRE(fd >= 0, AT_ERR_IO, std::string("cannot open ") + path);
        struct stat st;
        AT_REQUIRE(fstat(fd, &st) == 0, AT_ERR_IO, "fstat failed");
        len = (size_t)st.st_size;
        AT_REQUIRE(len >= 24, AT_ERR_IO, "Not a GGUF file: too short");
        map = mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0);
        AT_REQUIRE(map != MAP_FAILED, AT_ERR_IO, "mmap failed");
        GgufView v{static_cast<const uint8_t*>(map), len, 0};
        const uint32_t magic = v.rd<uint32_t>();
        if (magic != 0x46554747u) {
            char buf[64];
            snprintf(buf, sizeof buf, "Not a GGUF file: magic=0x%x", magic);
            fail(AT_ERR_IO, buf);
        }
        const uint32_t version = v.rd<uint32_t>();
        AT_REQUIRE(version == 3, AT_ERR_IO,
                   "Unsupported GGUF version: " + std::to_string(version) + " (AuraTensor supports v3)");
        const int64_t n_tensors = v.rd<int64_t>();
        const int64_t n_kv = v.rd<int64_t>();
        AT_REQUIRE(n_tensors >= 0 && n_kv >= 0, AT_ERR_IO, "negative counts in GGUF header");
        std::map<std::string, MetaVal> meta;
        for (int64_t i = 0; i < n_kv; ++i) {
            std::string k = v.str();
            const int vt = v.rd<int32_t>();
            meta[k] = read_value(v, vt);
        }
        struct TI { std::string name; int type; int64_t numel; uint64_t off; };
        std::vector<TI> tis;
        for (int64_t i = 0; i < n_tensors; ++i) {
            TI t;
            t.name = v.str();
            const int nd = v.rd<int32_t>();
            AT_REQUIRE(nd >= 1 && nd <= 4, AT_ERR_IO, "Unsupported rank: " + std::to_string(nd) + " (" + t.name + ")");
            t.numel = 1;
            for (int k = 0; k < nd; ++k) t.numel *= v.rd<int64_t>();
            t.type = v.rd<int32_t>();
            t.off = v.rd<uint64_t>();
            tis.push_back(t);
        }
        // LlamaConfig.fromGguf (inference/LlamaConfig.java:30-53)
        auto s_or = [&](const std::string& k, const std::string& dflt) {
            auto it = meta.find(k);
            return (it == meta.end() || it->second.type != 8) ? dflt : it->second.s;
        };
        auto n_or = [&](const std::string& k, double dflt) {
            auto it = meta.find(k);
            if (it == meta.end()) return dflt;
            AT_REQUIRE(it->second.is_num, AT_ERR_STATE, "Metadata '" + k + "' is not a number");
            return it->second.num;
        };
        const std::string arch = s_or("general.architecture", "llama");
        at_model_config cfg{};
        cfg.context_length = (int64_t)n_or(arch + ".context_length", 4096);
        cfg.embedding_length = (int64_t)n_or(arch + ".embedding_length", 4096);
        cfg.block_count = (int64_t)n_or(arch + ".block_count", 32);
        cfg.head_count = (int64_t)n_or(arch + ".attention.head_count", 32);
        cfg.head_count_kv = (int64_t)n_or(arch + ".attention.head_count_kv", (double)cfg.head_count);
        cfg.feed_forward_length = (int64_t)n_or(arch + ".feed_forward_length", 11008);
        const bool llama_big = arch.find("llama") != std::string::npos && cfg.embedding_length >= 4096;
        cfg.rope_freq_base = (float)n_or(arch + ".rope.freq_base", llama_big ? 500000.0 : 10000.0);
        cfg.rms_norm_eps = (float)n_or(arch + ".attention.layer_norm_rms_epsilon", 1e-5);
        cfg.vocab_size = (int64_t)n_or(arch + ".vocab_size", n_or("tokenizer.ggml.vocab_size", 32000));
        cfg.max_batch = max_batch < 1 ? 1 : max_batch;
        cfg.layout = layout;
        cfg.kv_type = kv_type;
        const int64_t align = (int64_t)n_or("general.alignment", 32);
        AT_REQUIRE(align > 0, AT_ERR_IO, "bad general.alignment");
        const uint64_t data_off = ((v.pos + align - 1) / align) * align;
        int rc2 = at_model_create(ctx, &cfg, &m);
        if (rc2 != AT_OK) fail(rc2, "model creation failed");
        for (const TI& t : tis) {
            int64_t bytes;
            if (t.type == AT_GGML_F32) bytes = t.numel * 4;
            else if (t.type == AT_GGML_F16) bytes = t.numel * 2;
            else if (t.type == AT_GGML_Q4_0) bytes = (t.numel + 31) / 32 * 18;
            else if (t.type == AT_GGML_Q8_0) bytes = (t.numel + 31) / 32 * 34;
            else if (t.type == AT_GGML_Q6_K) bytes = (t.numel + 255) / 256 * 210;
            else continue;  // types the decode path cannot use stay zero stand-ins (inference/Weights.java:143-149)
            AT_REQUIRE(data_off + t.off + (uint64_t)bytes <= len, AT_ERR_IO, "tensor '" + t.name + "' past end of file");
            rc2 = at_model_set_tensor(m, t.name.c_str(), t.type, static_cast<const uint8_t*>(map) + data_off + t.off,
                                      (size_t)bytes, 0);
            if (rc2 != AT_OK) {
                char msg[512];
                at_last_error(msg, sizeof msg);
                fail(rc2, msg);
            }
        }
        rc2 = at_model_finalize(m);
        if (rc2 != AT_OK) {
            char msg[512];
            at_last_error(msg, sizeof msg);
            fail(rc2, msg);
        }
        *out = m;
    });
    if (map != MAP_FAILED) munmap(map, len);
    if (fd >= 0) close(fd);
    if (rc != AT_OK && m) destroy_model(m);
    return rc;
}

int at_model_get_config(const at_model* m, at_model_config* out) {
    return guard([&] {
        AT_REQUIRE(m && out, AT_ERR_INVALID_ARG, "null argument");
        *out = m->cfg;
    });
}

int at_model_destroy(at_model* m) {
    return guard([&] { destroy_model(m); });
}

int at_model_forward_step(at_model* m, int token, int64_t position, float* logits_host) {
    return guard([&] { run_step(m, &token, &position, 1, logits_host); });
}

// Prompt chunks of up to PF_T tokens go through every layer together: the
// projections are tensor-core GEMMs (bf16 operands, FP32 sums; the prompt
// path's tolerance is 2e-2 of the logit range), attention is the causal
// prompt kernel over the KV cache of the target slot. Only the KV cache carries
// over to the decode steps, so the last layer's feed-forward and the lm_head
// are not needed; they are skipped. A chunk of 512 tokens is one CTA row of
// the GEMMs (two 256-token tiles per dequantized weight tile).
constexpr int PF_T = 512;

bool prompt_batched_ok(const at_model* m) {
    if (m->ctx->world != 1) return false;
    if (m->hd != 64 && m->hd != 128) return false;
    if (m->d % 64 || (m->Hl * m->hd) % 64 || m->Fl % 64) return false;
    // one row of the norm and of the QKV output fits the row kernels' shared memory
    if (m->d > kRowsMaxDim || (m->Hl + 2 * m->Hkvl) * m->hd > kRopeMaxCols) return false;
    for (const auto& ly : m->layers)
        for (const at_qmat* q : {&ly.qkv, &ly.wo, &ly.w1, &ly.w3, &ly.w2})
            if (q->type != AT_GGML_Q4_0 && q->type != AT_GGML_Q8_0) return false;
    return m->tok.type == AT_GGML_Q4_0 || m->tok.type == AT_GGML_Q8_0 || m->tok.type == AT_GGML_Q6_K;
}

void ensure_prompt_buffers(at_model* m) {
    if (m->pf_xa) return;
    const int64_t d = m->d, qcols = (int64_t)(m->Hl + 2 * m->Hkvl) * m->hd, nq = (int64_t)m->Hl * m->hd;
    alloc_zero((void**)&m->pf_xa, PF_T * d * 4);
    alloc_zero((void**)&m->pf_xb, PF_T * d * 4);
    alloc_zero((void**)&m->pf_y, PF_T * d * 4);
    alloc_zero((void**)&m->pf_qkv, PF_T * qcols * 4);
    alloc_zero((void**)&m->pf_q, PF_T * nq * 4);
    alloc_zero((void**)&m->pf_att, PF_T * nq * 4);
    alloc_zero((void**)&m->pf_g, PF_T * (int64_t)m->Fl * 4);
    alloc_zero((void**)&m->pf_u, PF_T * (int64_t)m->Fl * 4);
    alloc_zero((void**)&m->pf_tok, PF_T * sizeof(int));
    alloc_zero((void**)&m->pf_pos, PF_T * sizeof(int64_t));
    alloc_zero((void**)&m->pf_err, sizeof(int));
    m->pf_xbf_bytes = (size_t)PF_T * std::max<int64_t>(std::max<int64_t>(d, nq), m->Fl) * 2;
    alloc_zero(&m->pf_xbf, m->pf_xbf_bytes);
    {
        size_t ws = 16;
        const Layer& ly = m->layers[0];
        for (const at_qmat* q : {&ly.qkv, &ly.wo, &ly.w1, &ly.w3, &ly.w2}) {
            const int64_t outn = (q->orient == AT_ORIENT_N) ? q->rows : q->cols;
            ws = std::max(ws, (size_t)gemm_tc_splits(q, PF_T, m->ctx->num_sms) * PF_T * outn * 4);
        }
        m->pf_ws_bytes = ws;
        alloc_zero((void**)&m->pf_ws, ws);
    }
    AT_CUDA(cudaMallocHost(&m->h_pf_tok, PF_T * sizeof(int)));
    AT_CUDA(cudaMallocHost(&m->h_pf_pos, PF_T * sizeof(int64_t)));
}

void run_prompt_batched(at_model* m, const int* tokens, int n, int slot) {
    at_ctx* c = m->ctx;
    cudaStream_t s = c->stream;
    AT_CUDA(cudaSetDevice(c->device));
    ensure_prompt_buffers(m);
    const int d = m->d, hd = m->hd;
    const int nq = m->Hl * hd, nkv = m->Hkvl * hd, qcols = nq + 2 * nkv;
    const float eps = m->cfg.rms_norm_eps;
    const float scale = (float)(1.0 / std::sqrt((double)hd));
    const size_t layer_kv = (size_t)m->Hkvl * m->ctx_len * hd;
    __nv_bfloat16* xbf = static_cast<__nv_bfloat16*>(m->pf_xbf);
    for (int p0 = 0; p0 < n; p0 += PF_T) {
        const int T = std::min(PF_T, n - p0);
        AT_CUDA(cudaStreamSynchronize(s));  // the pinned staging buffers are free again
        for (int t = 0; t < T; ++t) {
            m->h_pf_tok[t] = tokens[p0 + t];
            m->h_pf_pos[t] = p0 + t;
        }
        AT_CUDA(cudaMemcpyAsync(m->pf_tok, m->h_pf_tok, sizeof(int) * T, cudaMemcpyHostToDevice, s));
        AT_CUDA(cudaMemcpyAsync(m->pf_pos, m->h_pf_pos, sizeof(int64_t) * T, cudaMemcpyHostToDevice, s));
        if (m->tok.type == AT_GGML_Q6_K)
            launch_q6k_embed(&m->tok, m->pf_tok, T, d, m->pf_xa, m->pf_y, nullptr, nullptr, s);
        else if (m->tok.type == AT_GGML_Q4_0)
            embed_kernel<AT_GGML_Q4_0><<<T, 256, 0, s>>>(m->tok.tiles, tile_map(&m->tok), m->pf_tok, d, m->pf_xa,
                                                          m->pf_y, nullptr, nullptr);
        else
            embed_kernel<AT_GGML_Q8_0><<<T, 256, 0, s>>>(m->tok.tiles, tile_map(&m->tok), m->pf_tok, d, m->pf_xa,
                                                          m->pf_y, nullptr, nullptr);
        AT_CUDA(cudaGetLastError());
        // The residual update y of the attention norm: the embedding's zeros,
        // then the down projection's output or its K-split partials in pf_ws
        // (summed by the consumer in split order)
        const float* ysrc = m->pf_y;
        int ysp = 1;
        for (int L = 0; L < m->L; ++L) {
            Layer& ly = m->layers[L];
            const size_t kv_off = (size_t)slot * m->slot_stride + L * layer_kv;
            float* kc = m->kv_q8 ? nullptr : m->kcache + kv_off;
            float* vc = m->kv_q8 ? nullptr : m->vcache + kv_off;
            KvQ kvq;
            if (m->kv_q8) kvq = KvQ{m->kq8 + kv_off, m->vq8 + kv_off, m->ksc + kv_off / 32, m->vsc + kv_off / 32};
            // attention block: xb = norm(xa + y); q, k, v; RoPE + append; attention; y = wo att
            rows_addnorm_kernel<<<T, 256, 0, s>>>(m->pf_xa, ysrc, ly.attn_norm, m->pf_xb, xbf, d, eps, ysp,
                                                  (size_t)T * d);
            AT_CUDA(cudaGetLastError());
            int sp = 1;
            GemmTcOut defer;
            defer.defer = &sp;
            launch_gemm_tc(&ly.qkv, nullptr, d, m->pf_qkv, qcols, T, m->pf_xbf, m->pf_xbf_bytes, m->pf_ws, m->pf_ws_bytes,
                           c->num_sms, m->pf_err, s, defer);
            AT_REQUIRE(sp <= kMaxPromptSplits, AT_ERR_STATE, "prompt GEMM split count above the consumers' limit");
            rope_append_kernel<<<T, 256, 0, s>>>(sp > 1 ? m->pf_ws : m->pf_qkv, qcols, m->pf_q, kc, vc, kvq, m->rope_cos,
                                                 m->rope_sin, hd, nq, nkv, m->ctx_len, p0, sp, (size_t)T * qcols);
            AT_CUDA(cudaGetLastError());
            bool att_bf = false;  // the attention output already sits in the bf16 staging buffer
            {
                const int G = m->Hl / m->Hkvl;
                const float* kq = m->kv_q8 ? reinterpret_cast<const float*>(kvq.kq) : kc;
                const float* vq = m->kv_q8 ? reinterpret_cast<const float*>(kvq.vq) : vc;
                // tensor-core attention for head_dim 64 / 128 and 1, 2, 4 or 8 query heads per KV head
                // (the last layer's attention output is not needed: write nothing)
                if (launch_prompt_attn_tc(hd, G, m->kv_q8, m->Hkvl, T, s, m->pf_q, kq, vq, kvq.ks, kvq.vs, m->pf_att,
                                          p0, m->Hl, m->ctx_len, scale, m->pf_err, xbf)) {
                    att_bf = true;
                } else if (hd == 128) {
                    if (m->kv_q8)
                        launch_prompt_attn<128, true>(G, m->Hkvl, T, s, m->pf_q, kq, vq, kvq.ks, kvq.vs, m->pf_att, p0,
                                                      m->Hl, m->ctx_len, scale);
                    else
                        launch_prompt_attn<128, false>(G, m->Hkvl, T, s, m->pf_q, kq, vq, nullptr, nullptr, m->pf_att,
                                                       p0, m->Hl, m->ctx_len, scale);
                } else {
                    if (m->kv_q8)
                        launch_prompt_attn<64, true>(G, m->Hkvl, T, s, m->pf_q, kq, vq, kvq.ks, kvq.vs, m->pf_att, p0,
                                                     m->Hl, m->ctx_len, scale);
                    else
                        launch_prompt_attn<64, false>(G, m->Hkvl, T, s, m->pf_q, kq, vq, nullptr, nullptr, m->pf_att,
                                                      p0, m->Hl, m->ctx_len, scale);
                }
            }
            AT_CUDA(cudaGetLastError());
            if (L == m->L - 1) break;  // later layers' inputs only; the KV cache is complete
            launch_gemm_tc(&ly.wo, att_bf ? nullptr : m->pf_att, nq, m->pf_y, d, T, m->pf_xbf, m->pf_xbf_bytes, m->pf_ws,
                           m->pf_ws_bytes, c->num_sms, m->pf_err, s, defer);
            // feed-forward block: xa = norm(xb + y); h = silu(w1 xa) * (w3 xa); y = w2 h
            // the norm, silu * mul and their bf16 copies feed w1 / w3 / w2 through the staging buffer
            rows_addnorm_kernel<<<T, 256, 0, s>>>(m->pf_xb, sp > 1 ? m->pf_ws : m->pf_y, ly.ffn_norm, m->pf_xa, xbf, d,
                                                  eps, sp, (size_t)T * d);
            AT_CUDA(cudaGetLastError());
            launch_gemm_tc(&ly.w1, nullptr, d, m->pf_g, m->Fl, T, m->pf_xbf, m->pf_xbf_bytes, m->pf_ws, m->pf_ws_bytes,
                           c->num_sms, m->pf_err, s);
            launch_gemm_tc(&ly.w3, nullptr, d, m->pf_u, m->Fl, T, m->pf_xbf, m->pf_xbf_bytes, m->pf_ws, m->pf_ws_bytes,
                           c->num_sms, m->pf_err, s);
            silu_mul_bf16_kernel<<<grid_for((int64_t)T * m->Fl / 4), 256, 0, s>>>(m->pf_g, m->pf_u, xbf,
                                                                                (int64_t)T * m->Fl);
            AT_CUDA(cudaGetLastError());
            launch_gemm_tc(&ly.w2, nullptr, m->Fl, m->pf_y, d, T, m->pf_xbf, m->pf_xbf_bytes, m->pf_ws, m->pf_ws_bytes,
                           c->num_sms, m->pf_err, s, defer);
            ysrc = sp > 1 ? m->pf_ws : m->pf_y;
            ysp = sp;
        }
    }
    int err = 0;
    AT_CUDA(cudaMemcpyAsync(&err, m->pf_err, sizeof(int), cudaMemcpyDeviceToHost, s));
    AT_CUDA(cudaStreamSynchronize(s));
    AT_REQUIRE(err == 0, AT_ERR_CUDA, "prompt GEMM or attention: an mbarrier wait ran out");
    m->kv_size[slot] = std::max<int64_t>(m->kv_size[slot], n);
}

void check_prompt(const at_model* m, const int* tokens, int n) {
    AT_REQUIRE(m && (n == 0 || tokens), AT_ERR_INVALID_ARG, "null argument");
    // LlamaModel.forwardPrompt (inference/LlamaModel.java:167-170)
    AT_REQUIRE(n >= 0 && n < m->ctx_len, AT_ERR_INVALID_ARG,
               "Prompt length " + std::to_string(n) + " exceeds contextLength " + std::to_string(m->ctx_len));
    AT_REQUIRE(m->finalized, AT_ERR_STATE, "model is not finalized");
    for (int i = 0; i < n; ++i)
        AT_REQUIRE(tokens[i] >= 0 && tokens[i] < m->V, AT_ERR_INVALID_ARG,
                   "token id " + std::to_string(tokens[i]) + " out of range");
}

int at_model_forward_prompt(at_model* m, const int* tokens, int n) {
    return guard([&] {
        check_prompt(m, tokens, n);
        if (n > 1 && prompt_batched_ok(m)) {
            run_prompt_batched(m, tokens, n, 0);
            return;
        }
        for (int i = 0; i < n; ++i) {
            const int64_t p = i;
            run_step(m, tokens + i, &p, 1, nullptr);
        }
    });
}

int at_model_forward_batch(at_model* m, const int* tokens, const int64_t* positions, int batch, float* logits_host) {
    return guard([&] { run_step(m, tokens, positions, batch, logits_host); });
}

int at_model_generate(at_model* m, int first_token, int64_t start_pos, int n_steps, int* tokens_out_host) {
    return guard([&] {
        AT_REQUIRE(m && m->finalized, AT_ERR_STATE, "model is not finalized");
        AT_REQUIRE(n_steps >= 0, AT_ERR_INVALID_ARG, "negative step count");
        AT_REQUIRE(first_token >= 0 && first_token < m->V, AT_ERR_INVALID_ARG, "token id out of range");
        AT_REQUIRE(start_pos >= 0, AT_ERR_INVALID_ARG, "negative position");
        AT_REQUIRE(start_pos + n_steps <= m->ctx_len, AT_ERR_STATE,
                   "position " + std::to_string(start_pos + n_steps - 1) + " exceeds maxContext " +
                       std::to_string(m->ctx_len));
        if (n_steps == 0) return;
        at_ctx* c = m->ctx;
        AT_CUDA(cudaSetDevice(c->device));
        m->h_tokens[0] = first_token;
        m->h_pos[0] = start_pos;
        AT_CUDA(cudaMemcpyAsync(m->d_tokens, m->h_tokens, sizeof(int), cudaMemcpyHostToDevice, c->stream));
        AT_CUDA(cudaMemcpyAsync(m->d_pos, m->h_pos, sizeof(int64_t), cudaMemcpyHostToDevice, c->stream));
        AT_CUDA(cudaMemsetAsync(m->d_gen_count, 0, sizeof(int), c->stream));
        if (m->use_ds) {
            for (int i = 0; i < n_steps; ++i) ds_launch(m, true);
            AT_CUDA(cudaMemcpyAsync(m->h_ds_err, m->ds_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
        } else {
            if (!m->graph_gen) m->graph_gen = capture(m, enqueue_generate_step, 1);
            for (int i = 0; i < n_steps; ++i) AT_CUDA(cudaGraphLaunch(m->graph_gen, c->stream));
        }
        m->kv_size[0] = std::max<int64_t>(m->kv_size[0], start_pos + n_steps);
        if (c->world > 1)
            AT_CUDA(cudaMemcpyAsync(m->h_ar_err, m->d_ar_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
        if (tokens_out_host) {
            AT_CUDA(cudaMemcpyAsync(tokens_out_host, m->d_gen_out, sizeof(int) * n_steps, cudaMemcpyDeviceToHost,
                                    c->stream));
            AT_CUDA(cudaStreamSynchronize(c->stream));
            check_peer_allreduce(m);
            ds_check(m);
        }
    });
}

int at_model_forward_prompt_slot(at_model* m, int slot, const int* tokens, int n) {
    return guard([&] {
        check_prompt(m, tokens, n);
        AT_REQUIRE(slot >= 0 && slot < m->B, AT_ERR_INVALID_ARG, "slot out of range");
        if (n == 0) return;
        if (prompt_batched_ok(m) && (n > 1 || slot > 0)) {
            run_prompt_batched(m, tokens, n, slot);
            return;
        }
        // A decode step writes the KV of every slot below its batch size, so
        // slots other than 0 need the batched prompt path.
        AT_REQUIRE(slot == 0, AT_ERR_UNSUPPORTED,
                   "a prompt into slot " + std::to_string(slot) + " needs the batched prompt path (one GPU, "
                   "Q4_0/Q8_0 layer matrices, head_dim 64 or 128)");
        for (int i = 0; i < n; ++i) {
            const int64_t p = i;
            run_step(m, tokens + i, &p, 1, nullptr);
        }
    });
}

}  // extern "C"

namespace at {

int64_t history_cap(const at_model* m) { return std::max<int64_t>(m->ctx_len, 8192); }

void ensure_sample_buffers(at_model* m) {
    if (m->d_rows) return;
    const size_t B = m->B;
    alloc_zero((void**)&m->d_rows, B * sizeof(SampleRow));
    m->hist_cap = history_cap(m);
    alloc_zero((void**)&m->d_hist, B * m->hist_cap * sizeof(int));
    alloc_zero((void**)&m->d_hist_len, B * sizeof(int));
    alloc_zero((void**)&m->d_pen_cnt, B * m->V * sizeof(int));
    alloc_zero((void**)&m->d_rng, B * sizeof(unsigned long long));
    alloc_zero((void**)&m->d_sampled, B * sizeof(int));
    alloc_zero((void**)&m->d_seq, B * m->ctx_len * sizeof(int));
    alloc_zero((void**)&m->d_step_ctr, sizeof(int));
    alloc_zero((void**)&m->d_append, B * sizeof(int));
    AT_CUDA(cudaMallocHost(&m->h_rows, B * sizeof(SampleRow)));
    AT_CUDA(cudaMallocHost(&m->h_i32, B * sizeof(int)));
    AT_CUDA(cudaMallocHost(&m->h_rng, B * sizeof(unsigned long long)));
    for (size_t b = 0; b < B; ++b) m->h_rows[b] = SampleRow{0.f, 1, 1.f, 1.f, 0.f, nullptr, nullptr, nullptr, nullptr};
}

bool sampler_greedy(const at_sampler_config& c) {
    return c.temperature == 0.0f || (c.top_k == 1 && c.top_p >= 1.0f);
}

// Sampler.Config checks: the reference fails on a non-positive topK
// outside the greedy path (inference/Sampler.java:77-80); the device
// sampler holds at most sample_k_max() candidates.
void check_sampler_config(const at_model* m, const at_sampler_config& c, int64_t history_cap) {
    if (!sampler_greedy(c)) {
        AT_REQUIRE(c.top_k >= 1, AT_ERR_INVALID_ARG, "topK must be positive");
        AT_REQUIRE(std::min(c.top_k, m->V) <= sample_k_max(), AT_ERR_UNSUPPORTED,
                   "topK above " + std::to_string(sample_k_max()) + " is not supported by the device sampler");
    }
    AT_REQUIRE(c.history_len >= 0 && (c.history_len == 0 || c.history), AT_ERR_INVALID_ARG, "bad history");
    AT_REQUIRE(c.history_len <= history_cap, AT_ERR_INVALID_ARG,
               "history of " + std::to_string(c.history_len) + " tokens exceeds the " + std::to_string(history_cap) +
                   " the device keeps for the row");
}

// Row b's sampler settings and penalty history (host ids, n of them) staged
// for the next sample launch; the caller uploads h_rows.
void set_sample_row(at_model* m, int b, const at_sampler_config& c, const int* history, int n) {
    at_ctx* ctx = m->ctx;
    SampleRow r{};
    r.temperature = c.temperature;
    r.top_k = c.top_k;
    r.top_p = c.top_p;
    r.penalty = c.repetition_penalty;
    r.hist = m->d_hist + (size_t)b * m->hist_cap;
    r.hist_len = m->d_hist_len + b;
    r.cnt = m->d_pen_cnt + (size_t)b * m->V;
    if (c.seed != 0) {
        r.r = sampler_r(c.seed);
    } else {  // an unseeded generator, advanced on the device per call
        const uint64_t t = (uint64_t)std::chrono::steady_clock::now().time_since_epoch().count();
        m->h_rng[b] = ((t + 0x9E3779B97F4A7C15ULL * (uint64_t)(b + 1)) ^ 0x5DEECE66DULL) & ((1ULL << 48) - 1);
        AT_CUDA(cudaMemcpyAsync(m->d_rng + b, m->h_rng + b, sizeof(unsigned long long), cudaMemcpyHostToDevice,
                                ctx->stream));
        r.rng = m->d_rng + b;
    }
    m->h_rows[b] = r;
    m->h_i32[b] = n;
    if (n > 0)
        AT_CUDA(cudaMemcpyAsync(m->d_hist + (size_t)b * m->hist_cap, history, sizeof(int) * n, cudaMemcpyHostToDevice,
                                ctx->stream));
    AT_CUDA(cudaMemcpyAsync(m->d_hist_len + b, m->h_i32 + b, sizeof(int), cudaMemcpyHostToDevice, ctx->stream));
}

void upload_sample_rows(at_model* m, int B) {
    AT_CUDA(cudaMemcpyAsync(m->d_rows, m->h_rows, sizeof(SampleRow) * B, cudaMemcpyHostToDevice, m->ctx->stream));
}

void enqueue_sampled_step(at_model* m, int B) {
    cudaStream_t s = m->ctx->stream;
    enqueue_step(m, B);
    launch_sample(m->logits, B, m->V, m->V, m->d_rows, m->d_sampled, s);
    launch_sample_advance(m->d_sampled, B, m->d_tokens, m->d_pos, m->d_seq, m->ctx_len, m->d_step_ctr, m->d_hist,
                          m->hist_cap, m->d_hist_len, nullptr, s);
}

}  // namespace at

extern "C" {

int at_model_sample(at_model* m, int batch, const at_sampler_config* cfgs, int* tokens_host) {
    return guard([&] {
        AT_REQUIRE(m && cfgs && tokens_host, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(m->finalized, AT_ERR_STATE, "model is not finalized");
        AT_REQUIRE(batch >= 1 && batch <= m->B, AT_ERR_INVALID_ARG, "batch out of range");
        for (int b = 0; b < batch; ++b) check_sampler_config(m, cfgs[b], history_cap(m));
        at_ctx* c = m->ctx;
        AT_CUDA(cudaSetDevice(c->device));
        AT_CUDA(cudaStreamSynchronize(c->stream));  // the pinned staging buffers are free
        ensure_sample_buffers(m);
        for (int b = 0; b < batch; ++b) set_sample_row(m, b, cfgs[b], cfgs[b].history, cfgs[b].history_len);
        upload_sample_rows(m, batch);
        launch_sample(m->logits, batch, m->V, m->V, m->d_rows, m->d_sampled, c->stream);
        AT_CUDA(cudaMemcpyAsync(tokens_host, m->d_sampled, sizeof(int) * batch, cudaMemcpyDeviceToHost, c->stream));
        AT_CUDA(cudaStreamSynchronize(c->stream));
    });
}

int at_model_generate_sampled(at_model* m, int batch, const int* first_tokens, const int64_t* start_pos, int n_steps,
                              const at_sampler_config* cfgs, int* tokens_out_host) {
    return guard([&] {
        AT_REQUIRE(m && first_tokens && start_pos && cfgs, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(m->finalized, AT_ERR_STATE, "model is not finalized");
        AT_REQUIRE(batch >= 1 && batch <= m->B, AT_ERR_INVALID_ARG, "batch out of range");
        AT_REQUIRE(n_steps >= 0, AT_ERR_INVALID_ARG, "negative step count");
        for (int b = 0; b < batch; ++b) {
            AT_REQUIRE(first_tokens[b] >= 0 && first_tokens[b] < m->V, AT_ERR_INVALID_ARG, "token id out of range");
            AT_REQUIRE(start_pos[b] >= 0, AT_ERR_INVALID_ARG, "negative position");
            AT_REQUIRE(start_pos[b] + n_steps <= m->ctx_len, AT_ERR_STATE,
                       "position " + std::to_string(start_pos[b] + n_steps - 1) + " exceeds maxContext " +
                           std::to_string(m->ctx_len));
            check_sampler_config(m, cfgs[b], history_cap(m) - n_steps);
        }
        if (n_steps == 0) return;
        at_ctx* c = m->ctx;
        AT_CUDA(cudaSetDevice(c->device));
        AT_CUDA(cudaStreamSynchronize(c->stream));
        ensure_sample_buffers(m);
        for (int b = 0; b < batch; ++b) {
            set_sample_row(m, b, cfgs[b], cfgs[b].history, cfgs[b].history_len);
            m->h_tokens[b] = first_tokens[b];
            m->h_pos[b] = start_pos[b];
        }
        upload_sample_rows(m, batch);
        AT_CUDA(cudaMemcpyAsync(m->d_tokens, m->h_tokens, sizeof(int) * batch, cudaMemcpyHostToDevice, c->stream));
        AT_CUDA(cudaMemcpyAsync(m->d_pos, m->h_pos, sizeof(int64_t) * batch, cudaMemcpyHostToDevice, c->stream));
        AT_CUDA(cudaMemsetAsync(m->d_step_ctr, 0, sizeof(int), c->stream));
        if (!m->graph_samp[batch]) m->graph_samp[batch] = capture(m, enqueue_sampled_step, batch);
        for (int i = 0; i < n_steps; ++i) AT_CUDA(cudaGraphLaunch(m->graph_samp[batch], c->stream));
        if (c->world > 1)
            AT_CUDA(cudaMemcpyAsync(m->h_ar_err, m->d_ar_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
        if (tokens_out_host)
            AT_CUDA(cudaMemcpy2DAsync(tokens_out_host, sizeof(int) * n_steps, m->d_seq, sizeof(int) * m->ctx_len,
                                      sizeof(int) * n_steps, batch, cudaMemcpyDeviceToHost, c->stream));
        AT_CUDA(cudaStreamSynchronize(c->stream));
        check_peer_allreduce(m);
        for (int b = 0; b < batch; ++b) m->kv_size[b] = std::max<int64_t>(m->kv_size[b], start_pos[b] + n_steps);
    });
}

}  // extern "C"

namespace at {

// Scheduler hooks (sched.cpp).
int model_max_batch(const at_model* m) { return m->B; }
int64_t model_ctx_len(const at_model* m) { return m->ctx_len; }
int model_vocab(const at_model* m) { return m->V; }
bool model_slot_prompt(const at_model* m) { return prompt_batched_ok(m); }

void sched_set_row(at_model* m, int slot, const at_sampler_config* cfg, const int* history, int n) {
    AT_REQUIRE(m->finalized, AT_ERR_STATE, "model is not finalized");
    at_ctx* c = m->ctx;
    AT_CUDA(cudaSetDevice(c->device));
    AT_CUDA(cudaStreamSynchronize(c->stream));
    ensure_sample_buffers(m);
    if (cfg) {
        check_sampler_config(m, *cfg, history_cap(m));
        AT_REQUIRE(n <= history_cap(m), AT_ERR_INVALID_ARG, "history exceeds the device history buffer");
        set_sample_row(m, slot, *cfg, history, n);
    } else {  // an idle row: greedy, no penalty
        m->h_rows[slot] = SampleRow{0.f, 1, 1.f, 1.f, 0.f, nullptr, nullptr, nullptr, nullptr};
    }
    AT_CUDA(cudaMemcpyAsync(m->d_rows + slot, m->h_rows + slot, sizeof(SampleRow), cudaMemcpyHostToDevice,
                            c->stream));
    AT_CUDA(cudaStreamSynchronize(c->stream));
}

// One decode step of rows 0..B-1 (tokens at positions), device sampling of
// every row and the history append of rows with append[b] set; picked
// receives the B sampled ids.
void sched_step(at_model* m, int B, const int* tokens, const int64_t* positions, const int* append, int* picked) {
    AT_REQUIRE(m->d_rows, AT_ERR_STATE, "no sampler rows were set");
    at_ctx* c = m->ctx;
    for (int b = 0; b < B; ++b) m->h_i32[b] = append[b] ? 1 : 0;
    AT_CUDA(cudaMemcpyAsync(m->d_append, m->h_i32, sizeof(int) * B, cudaMemcpyHostToDevice, c->stream));
    run_step_enqueue_only(m, tokens, positions, B);
    launch_sample(m->logits, B, m->V, m->V, m->d_rows, m->d_sampled, c->stream);
    launch_sample_advance(m->d_sampled, B, m->d_tokens, m->d_pos, nullptr, 0, nullptr, m->d_hist, m->hist_cap,
                          m->d_hist_len, m->d_append, c->stream);
    AT_CUDA(cudaMemcpyAsync(picked, m->d_sampled, sizeof(int) * B, cudaMemcpyDeviceToHost, c->stream));
    if (c->world > 1)
        AT_CUDA(cudaMemcpyAsync(m->h_ar_err, m->d_ar_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    AT_CUDA(cudaStreamSynchronize(c->stream));
    check_peer_allreduce(m);
    ds_check(m);
    for (int b = 0; b < B; ++b) m->kv_size[b] = std::max<int64_t>(m->kv_size[b], positions[b] + 1);
}

void sched_prompt(at_model* m, int slot, const int* tokens, int n) {
    check_prompt(m, tokens, n);
    run_prompt_batched(m, tokens, n, slot);
}

void sched_reset_slot(at_model* m, int slot) { m->kv_size[slot] = 0; }

}  // namespace at

extern "C" {

int at_model_profile_batch(at_model* m, int batch, const int* tokens, const int64_t* positions, float* class_ms,
                           int* class_launches) {
    return guard([&] {
        AT_REQUIRE(m && m->finalized && class_ms && class_launches && tokens && positions, AT_ERR_INVALID_ARG,
                   "bad argument");
        AT_REQUIRE(batch >= 1 && batch <= m->B, AT_ERR_INVALID_ARG, "batch out of range");
        for (int b = 0; b < batch; ++b) {
            AT_REQUIRE(tokens[b] >= 0 && tokens[b] < m->V, AT_ERR_INVALID_ARG, "token id out of range");
            AT_REQUIRE(positions[b] >= 0 && positions[b] < m->ctx_len, AT_ERR_STATE, "position exceeds maxContext");
        }
        at_ctx* c = m->ctx;
        AT_CUDA(cudaSetDevice(c->device));
        AT_CUDA(cudaStreamSynchronize(c->stream));  // the pinned staging buffers are free
        for (int b = 0; b < batch; ++b) {
            m->h_tokens[b] = tokens[b];
            m->h_pos[b] = positions[b];
        }
        AT_CUDA(cudaMemcpyAsync(m->d_tokens, m->h_tokens, sizeof(int) * batch, cudaMemcpyHostToDevice, c->stream));
        AT_CUDA(cudaMemcpyAsync(m->d_pos, m->h_pos, sizeof(int64_t) * batch, cudaMemcpyHostToDevice, c->stream));
        // The step is captured into a graph with an event pair around every
        // launch and no programmatic overlap, so each pair times one kernel on
        // the device without host submission gaps (recaptured when the batch
        // changes; the event pairs are shared).
        if (!m->graph_prof || m->graph_prof_batch != batch) {
            if (m->graph_prof) {
                cudaGraphExecDestroy(m->graph_prof);
                m->graph_prof = nullptr;
            }
            m->profiling = true;
            m->pdl = false;
            m->prof_used = 0;
            m->prof_cls.clear();
            try {
                m->graph_prof = capture(m, enqueue_step, batch);
            } catch (...) {
                m->profiling = false;
                m->pdl = true;
                throw;
            }
            m->profiling = false;
            m->pdl = true;
            m->graph_prof_batch = batch;
        }
        AT_CUDA(cudaGraphLaunch(m->graph_prof, c->stream));
        if (c->world > 1)
            AT_CUDA(cudaMemcpyAsync(m->h_ar_err, m->d_ar_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
        AT_CUDA(cudaStreamSynchronize(c->stream));
        check_peer_allreduce(m);
        for (int k = 0; k < AT_PROF_CLASSES; ++k) { class_ms[k] = 0.f; class_launches[k] = 0; }
        for (size_t i = 0; i < m->prof_cls.size(); ++i) {
            float ms = 0.f;
            AT_CUDA(cudaEventElapsedTime(&ms, m->prof_ev[2 * i], m->prof_ev[2 * i + 1]));
            class_ms[m->prof_cls[i]] += ms;
            class_launches[m->prof_cls[i]] += 1;
        }
        for (int b = 0; b < batch; ++b) m->kv_size[b] = std::max<int64_t>(m->kv_size[b], positions[b] + 1);
    });
}

int at_model_profile_step(at_model* m, int token, int64_t position, float* class_ms, int* class_launches) {
    return at_model_profile_batch(m, 1, &token, &position, class_ms, class_launches);
}

int at_model_logits_device(at_model* m, float** logits_dev) {
    return guard([&] {
        AT_REQUIRE(m && logits_dev && m->finalized, AT_ERR_INVALID_ARG, "bad argument");
        *logits_dev = m->logits;
    });
}

int at_model_argmax(at_model* m, int batch, int* tokens_host) {
    return guard([&] {
        AT_REQUIRE(m && tokens_host && m->finalized, AT_ERR_INVALID_ARG, "bad argument");
        AT_REQUIRE(batch >= 1 && batch <= m->B, AT_ERR_INVALID_ARG, "batch out of range");
        AT_CUDA(cudaMemcpyAsync(tokens_host, m->d_argmax, sizeof(int) * batch, cudaMemcpyDeviceToHost, m->ctx->stream));
        AT_CUDA(cudaStreamSynchronize(m->ctx->stream));
    });
}

int at_model_step_kernel(const at_model* m, int* persistent) {
    return guard([&] {
        AT_REQUIRE(m && persistent, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(m->finalized, AT_ERR_STATE, "model is not finalized");
        *persistent = m->use_ds ? 1 : 0;
    });
}

int at_model_step_stamps(at_model* m, int token, int64_t position, unsigned long long* stamps_host, int64_t n,
                         int* n_ctas) {
    return guard([&] {
        AT_REQUIRE(m && stamps_host && n_ctas, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(m->finalized, AT_ERR_STATE, "model is not finalized");
        AT_REQUIRE(m->use_ds, AT_ERR_STATE, "the model does not use the persistent step kernel");
        AT_REQUIRE(token >= 0 && token < m->V, AT_ERR_INVALID_ARG, "token id out of range");
        AT_REQUIRE(position >= 0 && position < m->ctx_len, AT_ERR_STATE, "position exceeds maxContext");
        at_ctx* c = m->ctx;
        const int64_t need = (int64_t)c->num_sms * (5 * m->L + 1) * 4;
        AT_REQUIRE(n >= need, AT_ERR_INVALID_ARG, "stamp buffer needs " + std::to_string(need) + " values");
        AT_CUDA(cudaSetDevice(c->device));
        if (!m->ds_stamps) alloc_zero((void**)&m->ds_stamps, (size_t)need * sizeof(unsigned long long));
        m->h_tokens[0] = token;
        m->h_pos[0] = position;
        AT_CUDA(cudaMemcpyAsync(m->d_tokens, m->h_tokens, sizeof(int), cudaMemcpyHostToDevice, c->stream));
        AT_CUDA(cudaMemcpyAsync(m->d_pos, m->h_pos, sizeof(int64_t), cudaMemcpyHostToDevice, c->stream));
        ds_launch(m, false);
        AT_CUDA(cudaMemcpyAsync(m->h_ds_err, m->ds_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
        AT_CUDA(cudaMemcpyAsync(stamps_host, m->ds_stamps, (size_t)need * sizeof(unsigned long long),
                                cudaMemcpyDeviceToHost, c->stream));
        AT_CUDA(cudaStreamSynchronize(c->stream));
        cudaFree(m->ds_stamps);  // later steps run without stamps
        m->ds_stamps = nullptr;
        ds_check(m);
        m->kv_size[0] = std::max<int64_t>(m->kv_size[0], position + 1);
        *n_ctas = c->num_sms;
    });
}

int at_model_kv_size(const at_model* m, int slot, int64_t* size) {
    return guard([&] {
        AT_REQUIRE(m && size, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(slot >= 0 && slot < m->B, AT_ERR_INVALID_ARG, "slot out of range");
        *size = m->kv_size[slot];
    });
}

int at_model_kv_read(at_model* m, int slot, int layer, int kv_head, int64_t position, float* k_host, float* v_host) {
    return guard([&] {
        AT_REQUIRE(m && m->finalized && k_host && v_host, AT_ERR_INVALID_ARG, "bad argument");
        // KVCache.offsetOf bounds (inference/KVCache.java:70-76); kv_head is rank-local under TP
        AT_REQUIRE(slot >= 0 && slot < m->B, AT_ERR_INVALID_ARG, "slot oob");
        AT_REQUIRE(layer >= 0 && layer < m->L, AT_ERR_INVALID_ARG, "layer oob");
        AT_REQUIRE(kv_head >= 0 && kv_head < m->Hkvl, AT_ERR_INVALID_ARG, "kvHead oob");
        AT_REQUIRE(position >= 0 && position < m->ctx_len, AT_ERR_INVALID_ARG, "position oob");
        const size_t off = (size_t)slot * m->slot_stride +
                           (((size_t)layer * m->Hkvl + kv_head) * m->ctx_len + (size_t)position) * m->hd;
        if (m->kv_q8) {
            // quants and scales to the host, read back as q * d (fp16 scale with flush-to-zero)
            std::vector<int8_t> kq(m->hd), vq(m->hd);
            std::vector<uint16_t> ks(m->hd / 32), vs(m->hd / 32);
            AT_CUDA(cudaMemcpyAsync(kq.data(), m->kq8 + off, m->hd, cudaMemcpyDeviceToHost, m->ctx->stream));
            AT_CUDA(cudaMemcpyAsync(vq.data(), m->vq8 + off, m->hd, cudaMemcpyDeviceToHost, m->ctx->stream));
            AT_CUDA(cudaMemcpyAsync(ks.data(), m->ksc + off / 32, m->hd / 32 * 2, cudaMemcpyDeviceToHost, m->ctx->stream));
            AT_CUDA(cudaMemcpyAsync(vs.data(), m->vsc + off / 32, m->hd / 32 * 2, cudaMemcpyDeviceToHost, m->ctx->stream));
            AT_CUDA(cudaStreamSynchronize(m->ctx->stream));
            for (int i = 0; i < m->hd; ++i) {
                k_host[i] = (float)kq[i] * fp16_ftz_host(ks[i / 32]);
                v_host[i] = (float)vq[i] * fp16_ftz_host(vs[i / 32]);
            }
            return;
        }
        AT_CUDA(cudaMemcpyAsync(k_host, m->kcache + off, m->hd * 4, cudaMemcpyDeviceToHost, m->ctx->stream));
        AT_CUDA(cudaMemcpyAsync(v_host, m->vcache + off, m->hd * 4, cudaMemcpyDeviceToHost, m->ctx->stream));
        AT_CUDA(cudaStreamSynchronize(m->ctx->stream));
    });
}

int at_model_kv_append(at_model* m, int slot, int64_t layer, int64_t position, const float* k_host,
                       const float* v_host) {
    return guard([&] {
        AT_REQUIRE(m && m->finalized && k_host && v_host, AT_ERR_INVALID_ARG, "bad argument");
        AT_REQUIRE(slot >= 0 && slot < m->B, AT_ERR_INVALID_ARG, "slot out of range");
        // KVCache.append (inference/KVCache.java:79-95)
        AT_REQUIRE(layer >= 0 && layer < m->L, AT_ERR_INVALID_ARG,
                   "layer " + std::to_string(layer) + " out of range " + std::to_string(m->L));
        AT_REQUIRE(position >= 0, AT_ERR_INVALID_ARG, "negative position");
        AT_REQUIRE(position < m->ctx_len, AT_ERR_STATE,
                   "position " + std::to_string(position) + " exceeds maxContext " + std::to_string(m->ctx_len));
        at_ctx* c = m->ctx;
        AT_CUDA(cudaSetDevice(c->device));
        const int n = m->Hkvl * m->hd;
        if (!m->kv_stage) alloc_zero((void**)&m->kv_stage, (size_t)2 * n * 4);
        AT_CUDA(cudaMemcpyAsync(m->kv_stage, k_host, (size_t)n * 4, cudaMemcpyHostToDevice, c->stream));
        AT_CUDA(cudaMemcpyAsync(m->kv_stage + n, v_host, (size_t)n * 4, cudaMemcpyHostToDevice, c->stream));
        const size_t base = (size_t)slot * m->slot_stride + (size_t)layer * m->Hkvl * m->ctx_len * m->hd;
        KvQ kvq;
        if (m->kv_q8) kvq = KvQ{m->kq8 + base, m->vq8 + base, m->ksc + base / 32, m->vsc + base / 32};
        kv_put_kernel<<<m->Hkvl, m->hd, 0, c->stream>>>(m->kv_stage, m->kv_stage + n,
                                                         m->kv_q8 ? nullptr : m->kcache + base,
                                                         m->kv_q8 ? nullptr : m->vcache + base, kvq, m->ctx_len,
                                                         m->hd, position);
        AT_CUDA(cudaGetLastError());
        AT_CUDA(cudaStreamSynchronize(c->stream));
        m->kv_size[slot] = std::max<int64_t>(m->kv_size[slot], position + 1);
    });
}

int at_model_kv_offset(const at_model* m, int64_t layer, int64_t kv_head, int64_t position, int64_t dim,
                       int64_t* byte_offset) {
    return guard([&] {
        AT_REQUIRE(m && byte_offset, AT_ERR_INVALID_ARG, "null argument");
        // KVCache.offsetOf (inference/KVCache.java:70-76), with its checks and messages
        AT_REQUIRE(layer >= 0 && layer < m->L, AT_ERR_INVALID_ARG, "layer oob");
        AT_REQUIRE(kv_head >= 0 && kv_head < m->Hkvl, AT_ERR_INVALID_ARG, "kvHead oob");
        AT_REQUIRE(position >= 0 && position < m->ctx_len, AT_ERR_INVALID_ARG, "position oob");
        AT_REQUIRE(dim < m->hd, AT_ERR_INVALID_ARG, "dim oob");
        const int64_t row_bytes = (int64_t)m->ctx_len * m->hd * 4;
        *byte_offset = (layer * m->Hkvl + kv_head) * row_bytes + position * m->hd * 4 + dim * 4;
    });
}

int at_model_kv_reset(at_model* m, int slot) {
    return guard([&] {
        AT_REQUIRE(m && m->finalized, AT_ERR_INVALID_ARG, "bad argument");
        AT_REQUIRE(slot >= 0 && slot < m->B, AT_ERR_INVALID_ARG, "slot out of range");
        const size_t off = (size_t)slot * m->slot_stride;
        if (m->kv_q8) {
            AT_CUDA(cudaMemsetAsync(m->kq8 + off, 0, (size_t)m->slot_stride, m->ctx->stream));
            AT_CUDA(cudaMemsetAsync(m->vq8 + off, 0, (size_t)m->slot_stride, m->ctx->stream));
            AT_CUDA(cudaMemsetAsync(m->ksc + off / 32, 0, (size_t)m->slot_stride / 32 * 2, m->ctx->stream));
            AT_CUDA(cudaMemsetAsync(m->vsc + off / 32, 0, (size_t)m->slot_stride / 32 * 2, m->ctx->stream));
        } else {
            AT_CUDA(cudaMemsetAsync(m->kcache + off, 0, (size_t)m->slot_stride * 4, m->ctx->stream));
            AT_CUDA(cudaMemsetAsync(m->vcache + off, 0, (size_t)m->slot_stride * 4, m->ctx->stream));
        }
        AT_CUDA(cudaStreamSynchronize(m->ctx->stream));
        m->kv_size[slot] = 0;
    });
}

}  // extern "C"
