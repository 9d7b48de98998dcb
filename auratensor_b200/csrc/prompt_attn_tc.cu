// Causal attention of a prompt chunk on the 5th-generation tensor cores
// (tcgen05): LlamaModel.attention (inference/LlamaModel.java:255-297) for the
// T consecutive query positions p0 .. p0+T-1 of one slot, every query head.
//
// CTA (KV head h, query block): 128 query rows = 128 / G tokens x the G query
// heads of h, so every K/V row the block needs is read once for all G heads.
// The keys 0 .. (the block's last position) are walked in tiles of 128:
//   1. the tile's K and V rows (FP32 or Q8_0 cache) are converted to bf16 in
//      one of two shared-memory tile buffers: K K-major (the B operand of
//      Q K^T), V M-major (the B operand of P V, dimensions contiguous: no
//      transpose); all threads load the first tile, then warps 4-7 load
//      tile k + 1 while warps 0-3 run the softmax of tile k;
//   2. one thread issues S = Q K^T (M 128, N 128 keys, K = HD) into TMEM
//      columns 0..127;
//   3. warps 0-3 (TMEM lane quarters; thread = query row) read S, apply the
//      scale (dot * scale, as the reference), the causal mask and the online
//      softmax (running max and sum), write P in bf16 (K-major A operand)
//      and rescale the output accumulator O (TMEM columns 128..) by the
//      tile's correction;
//   4. one thread issues O += P V (N = HD) into those TMEM columns;
//   5. after the last tile, warps 0-3 read O and store o / l.
// Operands are bf16 with FP32 sums (the prompt path's tolerance is 2e-2 of
// the logit range). Every wait on an mbarrier is bounded: a wait that runs
// out records an error code and the CTA frees its TMEM and returns.
#include <cuda_bf16.h>

#include <cstdint>

#include "at_internal.h"
#include "dev_common.cuh"

namespace at {

namespace {

constexpr int PT_ROWS = 128;     // query rows per CTA (MMA M)
constexpr int PT_KT = 128;       // keys per tile (MMA N of Q K^T, K of P V)
constexpr int PT_THREADS = 256;  // 8 warps: all load, warps 0-3 run the softmax
constexpr uint32_t PT_TMEM_COLS = 256;
constexpr int kPtSpinLimit = 1 << 22;

__device__ __forceinline__ uint32_t pt_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool pt_wait(uint32_t bar, uint32_t parity) {
    for (int it = 0; it < kPtSpinLimit; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

// Instruction descriptor of tcgen05.mma kind::f16: D f32, A and B bf16,
// A K-major, B K-major (bit 16 = 0) or M/N-major (bit 16 = 1), N >> 3 at bits
// 17-22, M >> 4 at bits 24-28.
constexpr uint32_t pt_idesc(int m, int n, bool b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn ? (1u << 16) : 0u) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}
static_assert(pt_idesc(128, 128, false) == 0x08200490u, "tcgen05 instruction descriptor");

// Shared-memory descriptors, 128-byte swizzle, version 1 (bit 46), layout
// type 2 (bits 61-63). K-major: stride byte offset 1024 B between 8-row
// groups (leading offset unused, encoded 1). M/N-major: leading byte offset =
// stride between 64-element atoms along M/N, stride byte offset = stride
// between 8-row groups along K.
__device__ __forceinline__ uint64_t pt_desc_k(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ uint64_t pt_desc_mn(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void pt_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void pt_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void pt_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void pt_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive FP32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void pt_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pt_pack(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // a -> low half (lower address)
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Byte offset of the 16-byte chunk c (0..7) of row r in a K-major swizzled
// tile of 64-element rows (one 128-byte atom column).
__device__ __forceinline__ uint32_t pt_sw128(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Eight consecutive elements of a cache row (FP32, or Q8_0 quants + fp16
// scales: the same element index), as four packed bf16 pairs.
template <bool KVQ>
__device__ __forceinline__ uint4 pt_row8(const float* __restrict__ c, const uint16_t* __restrict__ sc, size_t e) {
    float f[8];
    if constexpr (KVQ) {
        const uint2 w = *reinterpret_cast<const uint2*>(reinterpret_cast<const int8_t*>(c) + e);
        const float d = fp16_ftz_fast(sc[e >> 5]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            f[i] = __fmul_rn((float)(int8_t)((w.x >> (8 * i)) & 0xFFu), d);
            f[4 + i] = __fmul_rn((float)(int8_t)((w.y >> (8 * i)) & 0xFFu), d);
        }
    } else {
        const float4 a = *reinterpret_cast<const float4*>(c + e), b = *reinterpret_cast<const float4*>(c + e + 4);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    }
    return make_uint4(pt_pack(f[0], f[1]), pt_pack(f[2], f[3]), pt_pack(f[4], f[5]), pt_pack(f[6], f[7]));
}

// K (K-major, 128-row atom columns) and V (M-major) of the key tile at k0
// (nk valid rows, the rest zero) into one tile buffer, by NT threads (index
// lt), LB chunks' loads in flight per thread.
template <int HD, bool KVQ, int NT>
__device__ __forceinline__ void pt_load_kv(uint8_t* ks, uint8_t* vs, const float* __restrict__ kc,
                                           const float* __restrict__ vc, const uint16_t* __restrict__ ksc,
                                           const uint16_t* __restrict__ vsc, size_t kvbase, int64_t k0, int nk,
                                           int lt) {
    constexpr int NA = HD / 64;
    constexpr uint32_t ATOM_COL = 128 * 128;        // bytes of one atom column of a 128-row K-major tile
    constexpr int CH = 128 * HD / 8 / NT;           // 8-element chunks of K (and of V) per thread
    constexpr int LB = CH < 8 ? CH : 8;             // chunks whose loads are in flight together
    static_assert(CH % LB == 0, "load batches");
#pragma unroll
    for (int b = 0; b < CH; b += LB) {
        uint4 kv[LB], vv[LB];
#pragma unroll
        for (int u = 0; u < LB; ++u) {
            const int i = lt + (b + u) * NT;
            const int kr = i / (HD / 8), c8 = i % (HD / 8);
            kv[u] = vv[u] = make_uint4(0u, 0u, 0u, 0u);
            if (kr < nk) {
                const size_t e = kvbase + (size_t)(k0 + kr) * HD + 8 * c8;
                kv[u] = pt_row8<KVQ>(kc, ksc, e);
                vv[u] = pt_row8<KVQ>(vc, vsc, e);
            }
        }
#pragma unroll
        for (int u = 0; u < LB; ++u) {
            const int i = lt + (b + u) * NT;
            const int kr = i / (HD / 8), c8 = i % (HD / 8);
            *reinterpret_cast<uint4*>(ks + (c8 >> 3) * ATOM_COL + pt_sw128(kr, c8 & 7)) = kv[u];
            *reinterpret_cast<uint4*>(vs + (kr >> 3) * (NA * 1024) + (c8 >> 3) * 1024 + (kr & 7) * 128 +
                                      (((c8 & 7) ^ (kr & 7)) << 4)) = vv[u];
        }
    }
}

// 32 consecutive FP32 columns of this warp's 32 TMEM lanes, written.
__device__ __forceinline__ void pt_st32(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
          "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
          "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
          "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
          "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
          "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
          "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
          "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
          "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
          "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
          "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// The output accumulator O (FP32) lives in TMEM columns 128 .. 128 + HD and
// P V of each tile is added into it by the MMA; before that, the softmax
// warps rescale it by the tile's correction exp(m_old - m_new) (tcgen05.ld /
// st). The S MMA of a tile is issued after the previous tile's P V, so its
// completion also means the previous P V is done.
template <int HD, int G, bool KVQ>
__global__ void __launch_bounds__(PT_THREADS, 1)
    prompt_attn_tc_kernel(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                          const uint16_t* __restrict__ ksc, const uint16_t* __restrict__ vsc, float* __restrict__ att,
                          int T, int64_t p0, int Hl, int ctx, float scale, int* err,
                          __nv_bfloat16* __restrict__ att_bf) {
    constexpr int QB = PT_ROWS / G;  // tokens per CTA
    constexpr int NA = HD / 64;      // 128-byte atom columns of a Q / K row
    constexpr uint32_t QK_BYTES = PT_ROWS * HD * 2, V_BYTES = PT_KT * HD * 2;
    constexpr uint32_t ATOM_COL = PT_ROWS * 128;  // bytes of one atom column of a 128-row K-major tile
    constexpr uint32_t idesc_s = pt_idesc(PT_ROWS, PT_KT, false);
    constexpr uint32_t idesc_o = pt_idesc(PT_ROWS, HD, true);
    static_assert(PT_KT == PT_ROWS, "K tiles share the 128-row atom layout of Q");
    extern __shared__ uint8_t pt_raw[];
    __shared__ __align__(8) uint64_t s_bar[2];  // S complete, P V complete
    __shared__ uint32_t s_tmem;
    __shared__ int s_bad;
    uint8_t* qs = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pt_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ps = qs + QK_BYTES;
    // two K / V tile buffers: tile k uses buffer k & 1
    auto ks = [&](int buf) { return ps + PT_ROWS * PT_KT * 2 + buf * (QK_BYTES + V_BYTES); };
    auto vs = [&](int buf) { return ks(buf) + QK_BYTES; };
    const int kvh = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nq = Hl * HD;
    const int t0 = blockIdx.y * QB;
    const int ntok = min(QB, T - t0);
    const int64_t last = p0 + t0 + ntok - 1;  // the block's last query position
    const int ntiles = (int)(last / PT_KT) + 1;
    const size_t kvbase = (size_t)kvh * ctx * HD;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(pt_smem_u32(&s_tmem)),
                     "r"(PT_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(pt_smem_u32(&s_bar[0])) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(pt_smem_u32(&s_bar[1])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_bad = 0;
    }
    // q rows -> bf16, K-major: row r = ti * G + g is token t0 + ti, query head kvh * G + g
    for (int i = tid; i < PT_ROWS * HD / 8; i += PT_THREADS) {
        const int r = i / (HD / 8), c8 = i % (HD / 8);
        const int ti = r / G, g = r % G;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (ti < ntok) v = pt_row8<false>(q, nullptr, (size_t)(t0 + ti) * nq + (size_t)(kvh * G + g) * HD + 8 * c8);
        *reinterpret_cast<uint4*>(qs + (c8 >> 3) * ATOM_COL + pt_sw128(r, c8 & 7)) = v;
    }
    // the first key tile, by all threads
    pt_load_kv<HD, KVQ, PT_THREADS>(ks(0), vs(0), kc, vc, ksc, vsc, kvbase, 0, (last + 1) < PT_KT ? (int)(last + 1) : PT_KT,
                                    tid);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> the MMAs' async proxy
    pt_fence_before();
    __syncthreads();
    pt_fence_after();
    const uint32_t tmem = s_tmem;

    // this thread's query row (warps 0-3: TMEM lane quarter warp, lane = row)
    const int row = 32 * (warp & 3) + lane;
    const int64_t qpos = (row / G < ntok) ? p0 + t0 + row / G : -1;
    const uint32_t trow = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    float m = -INFINITY, l = 0.f;

    for (int kt = 0; kt < ntiles; ++kt) {
        const int64_t k0 = (int64_t)kt * PT_KT;
        const int buf = kt & 1;
        // 2. S = Q K^T
        if (tid == 0) {
            pt_fence_after();
            const uint32_t qa = pt_smem_u32(qs), ka = pt_smem_u32(ks(buf));
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk)
                pt_mma(tmem, pt_desc_k(qa + (kk >> 2) * ATOM_COL + 32 * (kk & 3)),
                       pt_desc_k(ka + (kk >> 2) * ATOM_COL + 32 * (kk & 3)), idesc_s, kk > 0 ? 1u : 0u);
            pt_commit(pt_smem_u32(&s_bar[0]));
        }
        // 3. scale, causal mask, online softmax; P (bf16, K-major) to shared
        //    memory; O rescaled by the correction
        if (warp < 4) {
            if (!pt_wait(pt_smem_u32(&s_bar[0]), kt & 1)) {
                atomicExch(err, 2);
                s_bad = 1;
            }
            pt_fence_after();
            float mx = -INFINITY;
#pragma unroll 1
            for (int c = 0; c < PT_KT / 32; ++c) {
                float sv[32];
                pt_ld32(trow + 32 * c, sv);
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (k0 + 32 * c + i <= qpos) mx = fmaxf(mx, __fmul_rn(sv[i], scale));
            }
            const float mn = fmaxf(m, mx);
            const float alpha = (mn == -INFINITY) ? 1.f : expf(m - mn);
            float sum = 0.f;
#pragma unroll 1
            for (int c = 0; c < PT_KT / 32; ++c) {
                float sv[32];
                pt_ld32(trow + 32 * c, sv);
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float a = (k0 + 32 * c + i <= qpos) ? expf(__fmul_rn(sv[i], scale) - mn) : 0.f;
                    const float b = (k0 + 32 * c + i + 1 <= qpos) ? expf(__fmul_rn(sv[i + 1], scale) - mn) : 0.f;
                    sum += a + b;
                    pk[i / 2] = pt_pack(a, b);
                }
                // keys 32c .. 32c+31: atom column c / 2, chunks 4 (c & 1) .. + 3
                uint8_t* prow = ps + (c >> 1) * ATOM_COL;
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    *reinterpret_cast<uint4*>(prow + pt_sw128(row, 4 * (c & 1) + j)) =
                        make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            }
            l = fmaf(l, alpha, sum);
            m = mn;
            // warp-uniform (tcgen05.ld / st are warp-collective); the previous
            // P V is complete: it precedes this S
            if (kt > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
                for (int c = 0; c < HD / 32; ++c) {
                    float ov[32];
                    pt_ld32(trow + PT_KT + 32 * c, ov);
#pragma unroll
                    for (int i = 0; i < 32; ++i) ov[i] *= alpha;
                    pt_st32(trow + PT_KT + 32 * c, ov);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        } else if (kt + 1 < ntiles) {
            // 1'. warps 4-7: the next tile into the other buffer, once the
            //     previous tile's P V (the last reader of that buffer) is done
            if (kt > 0 && !pt_wait(pt_smem_u32(&s_bar[1]), (kt - 1) & 1)) {
                atomicExch(err, 2);
                s_bad = 1;
            } else {
                const int64_t k1 = k0 + PT_KT;
                pt_load_kv<HD, KVQ, PT_THREADS - 128>(ks(buf ^ 1), vs(buf ^ 1), kc, vc, ksc, vsc, kvbase, k1,
                                                      (last + 1 - k1) < PT_KT ? (int)(last + 1 - k1) : PT_KT, tid - 128);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            }
        }
        pt_fence_before();
        __syncthreads();
        if (s_bad) break;
        // 4. O (+)= P V
        if (tid == 0) {
            pt_fence_after();
            const uint32_t pa = pt_smem_u32(ps), va = pt_smem_u32(vs(buf));
#pragma unroll
            for (int kk = 0; kk < PT_KT / 16; ++kk)
                pt_mma(tmem + PT_KT, pt_desc_k(pa + (kk >> 2) * ATOM_COL + 32 * (kk & 3)),
                       pt_desc_mn(va + kk * 2 * (NA * 1024), 1024, NA * 1024), idesc_o, (kt > 0 || kk > 0) ? 1u : 0u);
            pt_commit(pt_smem_u32(&s_bar[1]));
        }
    }
    // 5. the last P V; o / l (the TMEM reads by whole warps, stores by the rows that hold a token)
    if (!s_bad && warp < 4) {
        const bool done = __all_sync(0xffffffffu, pt_wait(pt_smem_u32(&s_bar[1]), (ntiles - 1) & 1));
        if (!done) {
            if (lane == 0) atomicExch(err, 2);
        } else {
            pt_fence_after();
            const int ti = row / G, g = row % G;
            const size_t off = (size_t)(t0 + ti) * nq + (size_t)(kvh * G + g) * HD;
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                float ov[32];
                pt_ld32(trow + PT_KT + 32 * c, ov);
                if (qpos >= 0) {
                    if (att_bf) {  // the wo GEMM's bf16 operand (round to nearest even, as its conversion)
#pragma unroll
                        for (int d = 0; d < 32; d += 8) {
                            uint4 u;
                            u.x = pt_pack(__fdiv_rn(ov[d], l), __fdiv_rn(ov[d + 1], l));
                            u.y = pt_pack(__fdiv_rn(ov[d + 2], l), __fdiv_rn(ov[d + 3], l));
                            u.z = pt_pack(__fdiv_rn(ov[d + 4], l), __fdiv_rn(ov[d + 5], l));
                            u.w = pt_pack(__fdiv_rn(ov[d + 6], l), __fdiv_rn(ov[d + 7], l));
                            *reinterpret_cast<uint4*>(att_bf + off + 32 * c + d) = u;
                        }
                    } else {
#pragma unroll
                        for (int d = 0; d < 32; d += 4)
                            *reinterpret_cast<float4*>(att + off + 32 * c + d) =
                                make_float4(__fdiv_rn(ov[d], l), __fdiv_rn(ov[d + 1], l), __fdiv_rn(ov[d + 2], l),
                                            __fdiv_rn(ov[d + 3], l));
                    }
                }
            }
        }
    }
    pt_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PT_TMEM_COLS) : "memory");
}

// q, P and two K / V tile buffers (bf16) + alignment slack
constexpr size_t pt_smem(int hd) {
    return (size_t)(PT_ROWS * hd * 2 + PT_ROWS * PT_KT * 2 + 2 * (PT_KT * hd * 2 + PT_KT * hd * 2)) + 1024;
}
static_assert(pt_smem(128) <= 227 * 1024, "shared memory per CTA");

template <int HD, int G, bool KVQ>
void pt_launch(int Hkvl, int T, cudaStream_t s, const float* q, const float* kc, const float* vc, const uint16_t* ksc,
               const uint16_t* vsc, float* att, int64_t p0, int Hl, int ctx, float scale, int* err,
               __nv_bfloat16* att_bf) {
    auto kern = prompt_attn_tc_kernel<HD, G, KVQ>;
    static bool attr = false;  // per instance
    if (!attr) {
        AT_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pt_smem(HD)));
        attr = true;
    }
    constexpr int QB = PT_ROWS / G;
    kern<<<dim3(Hkvl, (T + QB - 1) / QB), PT_THREADS, pt_smem(HD), s>>>(q, kc, vc, ksc, vsc, att, T, p0, Hl, ctx,
                                                                       scale, err, att_bf);
    AT_CUDA(cudaGetLastError());
}

template <int HD, bool KVQ>
bool pt_dispatch_g(int G, int Hkvl, int T, cudaStream_t s, const float* q, const float* kc, const float* vc,
                   const uint16_t* ksc, const uint16_t* vsc, float* att, int64_t p0, int Hl, int ctx, float scale,
                   int* err, __nv_bfloat16* att_bf) {
    switch (G) {
        case 1: pt_launch<HD, 1, KVQ>(Hkvl, T, s, q, kc, vc, ksc, vsc, att, p0, Hl, ctx, scale, err, att_bf); return true;
        case 2: pt_launch<HD, 2, KVQ>(Hkvl, T, s, q, kc, vc, ksc, vsc, att, p0, Hl, ctx, scale, err, att_bf); return true;
        case 4: pt_launch<HD, 4, KVQ>(Hkvl, T, s, q, kc, vc, ksc, vsc, att, p0, Hl, ctx, scale, err, att_bf); return true;
        case 8: pt_launch<HD, 8, KVQ>(Hkvl, T, s, q, kc, vc, ksc, vsc, att, p0, Hl, ctx, scale, err, att_bf); return true;
        default: return false;
    }
}

}  // namespace

bool launch_prompt_attn_tc(int hd, int G, bool kvq, int Hkvl, int T, cudaStream_t s, const float* q, const float* kc,
                           const float* vc, const uint16_t* ksc, const uint16_t* vsc, float* att, int64_t p0, int Hl,
                           int ctx, float scale, int* err, __nv_bfloat16* att_bf) {
    if (hd == 128)
        return kvq ? pt_dispatch_g<128, true>(G, Hkvl, T, s, q, kc, vc, ksc, vsc, att, p0, Hl, ctx, scale, err, att_bf)
                   : pt_dispatch_g<128, false>(G, Hkvl, T, s, q, kc, vc, ksc, vsc, att, p0, Hl, ctx, scale, err, att_bf);
    if (hd == 64)
        return kvq ? pt_dispatch_g<64, true>(G, Hkvl, T, s, q, kc, vc, ksc, vsc, att, p0, Hl, ctx, scale, err, att_bf)
                   : pt_dispatch_g<64, false>(G, Hkvl, T, s, q, kc, vc, ksc, vsc, att, p0, Hl, ctx, scale, err, att_bf);
    return false;
}

}  // namespace at
