// Fused-dequant Q4_0 / Q8_0 matrix-vector kernels for sm_100a.
//
// Replaces Kernels.sgemv over load-time dequantized FP32 weights
// (core/Kernels.java:350-371 fed by inference/Weights.java:185-203): the raw
// GGUF blocks stay resident in HBM and are dequantized in registers.
//
// Dequant: Q4_0 w = (q - 8) * d with the interleaved nibble order of
// quant/Q4_0.java:39-42 (element 2k = low nibble of byte k, 2k+1 = high
// nibble); Q8_0 w = q * d (quant/Q8_0.java:130-132); d decoded by
// Fp16.toFloat with flush-to-zero. A nibble/byte becomes the exact float
// q - 8 (or q) through one byte permute into the mantissa of 2^23 and one
// packed f32x2 subtraction; products and sums are FP32 (packed f32x2 FMA), so
// each (q - 8) * x term equals the reference's dequantized weight times x and
// only the summation order differs.
//
// Weights use the tiled layout of at_qmat (a lossless re-layout of whole
// blocks): the bytes one warp step consumes are one contiguous tile.
// Orientation N (rows = outputs, blocks along the row): a warp streams the
// tiles (4 rows x 32 blocks) of its row group through a cp.async ring in
// shared memory, one block per lane per step; x is staged once per CTA in
// shared memory (natural order, 36 floats per 32-element block so a
// quarter-warp of 128-bit reads touches 32 distinct banks).
// Orientation T (rows = inputs, blocks along the outputs): a lane owns rows
// of one block column (tiles of 32 rows) and accumulates its 32 (or 8)
// outputs; lanes combine by a butterfly reduce-scatter, warps through shared
// memory, and CTAs that split the rows through an ordered reduction by the
// last CTA to arrive (counter per block column, reset by that CTA).
// All kernels support programmatic dependent launch: weights (never written
// by an earlier kernel) are prefetched before griddepcontrol.wait; every
// activation read comes after it.
#include <cuda_fp16.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>

#include "at_internal.h"
#include "dev_common.cuh"

namespace at {

namespace {

constexpr int THREADS = 256;
constexpr int XPAD = 36;                 // floats per staged 32-element block
constexpr int kMaxXSmemChunk = 96 * 1024;

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <int QT>
struct QTraits;
template <>
struct QTraits<AT_GGML_Q4_0> { static constexpr int QB = 16; static constexpr int NV = 1; };
template <>
struct QTraits<AT_GGML_Q8_0> { static constexpr int QB = 32; static constexpr int NV = 2; };

// Decodes the 32 weights of one block (unscaled: q - 8 for Q4_0, q for Q8_0)
// into 16 float pairs of consecutive elements (2k, 2k+1).
template <int QT>
__device__ __forceinline__ void decode32(const uint4* q, float2* w) {
    if constexpr (QT == AT_GGML_Q4_0) {
        const float2 moff = f2(-8388616.f, -8388616.f);  // -(2^23 + 8)
        const uint32_t ws[4] = {q[0].x, q[0].y, q[0].z, q[0].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = ws[i] & 0x0F0F0F0Fu, hi = (ws[i] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                w[4 * i + k] = __fadd2_rn(f2(magic_byte(lo, k), magic_byte(hi, k)), moff);  // elements 8i+2k, +1
        }
    } else {
        const float2 moff = f2(-8388736.f, -8388736.f);  // -(2^23 + 128)
        const uint32_t ws[8] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t u = ws[i] ^ 0x80808080u;  // int8 q -> unsigned q + 128
            w[2 * i + 0] = __fadd2_rn(f2(magic_byte(u, 0), magic_byte(u, 1)), moff);  // elements 4i, 4i+1
            w[2 * i + 1] = __fadd2_rn(f2(magic_byte(u, 2), magic_byte(u, 3)), moff);  // elements 4i+2, 4i+3
        }
    }
}

// Unscaled dot of one block with x (natural order, xr[t] = x[4t..4t+3]).
// Each nibble (byte) is placed in the low mantissa byte of 2^23 by one byte
// permute, and one packed f32x2 subtraction of 2^23 + 8 (or 2^23 + 128 after
// flipping the sign bit of an int8) leaves the exact integer weight.
template <int QT>
__device__ __forceinline__ float dot32(const uint4* q, const float4* xr) {
    float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
    if constexpr (QT == AT_GGML_Q4_0) {
        const float2 moff = f2(-8388616.f, -8388616.f);  // -(2^23 + 8)
        const uint32_t ws[4] = {q[0].x, q[0].y, q[0].z, q[0].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = ws[i] & 0x0F0F0F0Fu, hi = (ws[i] >> 4) & 0x0F0F0F0Fu;
            // pair k = elements (8i + 2k, 8i + 2k + 1) = (low, high) nibble of byte k
            const float2 p0 = __fadd2_rn(f2(magic_byte(lo, 0), magic_byte(hi, 0)), moff);
            const float2 p1 = __fadd2_rn(f2(magic_byte(lo, 1), magic_byte(hi, 1)), moff);
            const float2 p2 = __fadd2_rn(f2(magic_byte(lo, 2), magic_byte(hi, 2)), moff);
            const float2 p3 = __fadd2_rn(f2(magic_byte(lo, 3), magic_byte(hi, 3)), moff);
            a0 = __ffma2_rn(p0, f2(xr[2 * i].x, xr[2 * i].y), a0);
            a1 = __ffma2_rn(p1, f2(xr[2 * i].z, xr[2 * i].w), a1);
            a0 = __ffma2_rn(p2, f2(xr[2 * i + 1].x, xr[2 * i + 1].y), a0);
            a1 = __ffma2_rn(p3, f2(xr[2 * i + 1].z, xr[2 * i + 1].w), a1);
        }
    } else {
        const float2 moff = f2(-8388736.f, -8388736.f);  // -(2^23 + 128)
        const uint32_t ws[8] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t u = ws[i] ^ 0x80808080u;  // int8 q -> unsigned q + 128
            const float2 v01 = __fadd2_rn(f2(magic_byte(u, 0), magic_byte(u, 1)), moff);
            const float2 v23 = __fadd2_rn(f2(magic_byte(u, 2), magic_byte(u, 3)), moff);
            a0 = __ffma2_rn(v01, f2(xr[i].x, xr[i].y), a0);
            a1 = __ffma2_rn(v23, f2(xr[i].z, xr[i].w), a1);
        }
    }
    return (a0.x + a0.y) + (a1.x + a1.y);
}

// Stages x (or the normed x + y) for blocks [b0, b0 + nbc) of B rows into
// shared memory, natural order, XPAD floats per block.
// float4 global loads, eight in flight per thread before any is stored.
template <int QT, int B, Pro PRO, int NT = THREADS>
__device__ __forceinline__ void stage_x(float* xs, const GemvArgs& a, int b0, int nbc, int chunk_blocks,
                                        const float* s_inv) {
    const int nf4 = nbc * 8;
    const int total = B * nf4;
    for (int base = 0; base < total; base += NT * 8) {
        float4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int idx = base + k * NT + threadIdx.x;
            if (idx < total) {
                const int bb = idx / nf4, r = idx - bb * nf4;
                const size_t off = (size_t)bb * a.x_stride + (size_t)(b0 + (r >> 3)) * 32 + (r & 7) * 4;
                if constexpr (PRO == Pro::Plain) {
                    v[k] = *reinterpret_cast<const float4*>(a.x + off);
                } else {
                    float4 t = *reinterpret_cast<const float4*>(a.xin + off);
                    if (a.yin) {
                        const float4 u = *reinterpret_cast<const float4*>(a.yin + off);
                        t.x = __fadd_rn(t.x, u.x); t.y = __fadd_rn(t.y, u.y);
                        t.z = __fadd_rn(t.z, u.z); t.w = __fadd_rn(t.w, u.w);
                    }
                    v[k] = t;
                }
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int idx = base + k * NT + threadIdx.x;
            if (idx < total) {
                const int bb = idx / nf4, r = idx - bb * nf4;
                const int blk = r >> 3, q4 = r & 7;
                float4 o = v[k];
                if constexpr (PRO == Pro::AddNorm) {
                    const float4 g = *reinterpret_cast<const float4*>(a.gamma + (size_t)(b0 + blk) * 32 + q4 * 4);
                    const float inv = s_inv[bb];
                    o = make_float4(norm_apply(o.x, inv, g.x), norm_apply(o.y, inv, g.y), norm_apply(o.z, inv, g.z),
                                    norm_apply(o.w, inv, g.w));
                }
                *reinterpret_cast<float4*>(xs + ((size_t)bb * chunk_blocks + blk) * XPAD + q4 * 4) = o;
            }
        }
    }
}

// Writes the normed x (x + y scaled, F7 residual stream) for all B rows: CTA 0 only.
template <int B, int NT = THREADS>
__device__ __forceinline__ void write_xout(const GemvArgs& a, int d, const float* s_inv) {
    for (int idx = threadIdx.x; idx < B * d / 4; idx += NT) {
        const int bb = idx / (d / 4), i4 = idx - bb * (d / 4);
        const size_t off = (size_t)bb * a.x_stride + (size_t)i4 * 4;
        float4 t = *reinterpret_cast<const float4*>(a.xin + off);
        if (a.yin) {
            const float4 u = *reinterpret_cast<const float4*>(a.yin + off);
            t.x = __fadd_rn(t.x, u.x); t.y = __fadd_rn(t.y, u.y); t.z = __fadd_rn(t.z, u.z); t.w = __fadd_rn(t.w, u.w);
        }
        const float4 g = *reinterpret_cast<const float4*>(a.gamma + (size_t)i4 * 4);
        const float inv = s_inv[bb];
        *reinterpret_cast<float4*>(a.xout + off) = make_float4(
            norm_apply(t.x, inv, g.x), norm_apply(t.y, inv, g.y), norm_apply(t.z, inv, g.z), norm_apply(t.w, inv, g.w));
    }
}

template <Epi EPI>
__device__ __forceinline__ float n_epilogue(float g, float u) {
    if constexpr (EPI == Epi::SiluMul) {
        // Kernels.siluInPlace then elementwiseMul (core/Kernels.java:86-87,
        // inference/LlamaModel.java:372-380): g / (1 + exp(-g)) * u
        return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    } else {
        return g;
    }
}

// ---------------------------------------------------------------------------
// Orientation N, tile streams through per-warp cp.async rings
// ---------------------------------------------------------------------------
// A warp owns a 4-row group and a contiguous range of its 32-block steps; one
// step is one tile (4 rows x 32 blocks, scales then quant bytes), copied
// 16 bytes per lane into the warp's ring slot with cp.async. Lanes then read
// their own block of each row. Warps that split one group's steps (KS > 1)
// combine through shared memory in a fixed order. A CTA stages x once and
// walks `per` rounds of groups.
constexpr int N4_THREADS = 512;
constexpr int N4_WARPS = N4_THREADS / 32;

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int QT>
struct NTile {
    static constexpr int QB = QTraits<QT>::QB;
    static constexpr int BYTES = 4 * 32 * (2 + QB);  // 2304 (Q4_0) or 4352 (Q8_0)
    static constexpr int CHUNKS = BYTES / 16;
};

struct N4Params {
    const uint8_t* tiles[2];
    int rows, nb, ngroups, nsteps;
    int KS;         // warps splitting the steps of one group
    int gpc;        // groups per CTA round = N4_WARPS / KS
    int per;        // rounds per CTA
    int steps_ks;   // steps per step range = ceil(nsteps / KS)
    int ring_off;
    GemvArgs a;
};

template <int QT, int NM>
__device__ __forceinline__ void n4_issue(uint32_t slot, const N4Params& p, int g, int s, int lane) {
    using TL = NTile<QT>;
    if (g < p.ngroups) {
#pragma unroll
        for (int m = 0; m < NM; ++m) {
            const uint8_t* src = p.tiles[m] + ((size_t)g * p.nsteps + s) * TL::BYTES;
#pragma unroll
            for (int u = 0; u < (TL::CHUNKS + 31) / 32; ++u) {
                const int k = lane + 32 * u;
                if (k < TL::CHUNKS) cp_async16(slot + (uint32_t)(m * TL::BYTES + 16 * k), src + 16 * k);
            }
        }
    }
    cp_commit();
}

template <int QT, int B, Pro PRO, Epi EPI, int NST>
__global__ void __launch_bounds__(N4_THREADS, 1) gemv_n4_kernel(const N4Params p) {
    static_assert((NST & (NST - 1)) == 0, "ring depth is a power of two");
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    using TL = NTile<QT>;
    constexpr int SLOT = NM * TL::BYTES;
    constexpr int NV = QTraits<QT>::NV;
    extern __shared__ __align__(16) float xs[];
    __shared__ float s_red[N4_WARPS * B];
    __shared__ float s_inv[B];
    __shared__ float red[N4_WARPS][NM * 4 * B];

    pdl_trigger();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kpart = warp % p.KS, gslot = warp / p.KS;
    const int s0 = kpart * p.steps_ks;
    const int nsk = max(0, min(p.nsteps, s0 + p.steps_ks) - s0);  // steps of this warp per round
    const int T = p.per * nsk;
    const uint8_t* ring_ptr = reinterpret_cast<const uint8_t*>(xs) + p.ring_off + warp * NST * SLOT;
    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(ring_ptr);
    const int g_base = blockIdx.x * p.per * p.gpc + gslot;  // group of round r: g_base + r * gpc

    // Issue iterator: (round, step) of the next step to copy. Weights are
    // never written by earlier kernels, so the first NST copies start before
    // waiting on those kernels.
    int i_round = 0, i_step = 0, issued = 0;
    auto issue_next = [&](uint32_t slot) {
        if (issued < T) {
            n4_issue<QT, NM>(slot, p, g_base + i_round * p.gpc, s0 + i_step, lane);
            if (++i_step == nsk) { i_step = 0; ++i_round; }
        } else {
            cp_commit();
        }
        ++issued;
    };
#pragma unroll
    for (int k = 0; k < NST; ++k) issue_next(ring + k * SLOT);
    pdl_wait();

    const int d_model = p.nb * 32;
    if constexpr (PRO == Pro::AddNorm) {
        block_rms_inv<B, N4_THREADS>(p.a.xin, p.a.yin, p.a.x_stride, d_model, p.a.eps, s_red, s_inv);
        if (blockIdx.x == 0) write_xout<B, N4_THREADS>(p.a, d_model, s_inv);
    }
    stage_x<QT, B, PRO, N4_THREADS>(xs, p.a, 0, p.nb, p.nb, s_inv);
    __syncthreads();

    float acc[NM * 4][B];
#pragma unroll
    for (int i = 0; i < NM * 4; ++i)
#pragma unroll
        for (int b = 0; b < B; ++b) acc[i][b] = 0.f;

    int t = 0;
    for (int round = 0; round < p.per; ++round) {
        const int g = g_base + round * p.gpc;
        const bool g_ok = g < p.ngroups;
        const float* xrow = xs + ((size_t)s0 * 32 + lane) * XPAD;  // x of this lane's first block
        for (int ks = 0; ks < nsk; ++ks, ++t) {
            cp_wait<NST - 1>();
            __syncwarp();  // every lane's 16-byte pieces of this slot have landed
            const int slot = t & (NST - 1);
            const uint8_t* sp = ring_ptr + slot * SLOT;
            const int j = (s0 + ks) * 32 + lane;  // this lane's block
            if (g_ok && j < p.nb) {
                uint4 q[NM * 4][NV];
                float dsc[NM * 4];
#pragma unroll
                for (int m = 0; m < NM; ++m)
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const uint8_t* tb = sp + m * TL::BYTES;
#pragma unroll
                        for (int v = 0; v < NV; ++v)
                            q[m * 4 + r][v] = *reinterpret_cast<const uint4*>(tb + 256 + (r * 32 + lane) * TL::QB + 16 * v);
                        dsc[m * 4 + r] = fp16_ftz_fast(*reinterpret_cast<const uint16_t*>(tb + (r * 32 + lane) * 2));
                    }
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float4* xv = reinterpret_cast<const float4*>(xrow + (size_t)b * p.nb * XPAD + (size_t)ks * 32 * XPAD);
                    float4 xr[8];
#pragma unroll
                    for (int k = 0; k < 8; ++k) xr[k] = xv[k];
#pragma unroll
                    for (int i = 0; i < NM * 4; ++i) acc[i][b] = fmaf(dsc[i], dot32<QT>(q[i], xr), acc[i][b]);
                }
            }
            __syncwarp();  // every lane is done with this slot before it is refilled
            issue_next(ring + slot * SLOT);
        }
        // round complete: reduce over lanes, then over the KS warps of each group
#pragma unroll
        for (int i = 0; i < NM * 4; ++i)
#pragma unroll
            for (int b = 0; b < B; ++b) acc[i][b] = warp_sum(acc[i][b]);
        if (lane == 0) {
#pragma unroll
            for (int i = 0; i < NM * 4; ++i)
#pragma unroll
                for (int b = 0; b < B; ++b) red[warp][i * B + b] = acc[i][b];
        }
#pragma unroll
        for (int i = 0; i < NM * 4; ++i)
#pragma unroll
            for (int b = 0; b < B; ++b) acc[i][b] = 0.f;
        __syncthreads();
        if (kpart == 0 && lane < 4 * B) {
            const int r = lane / B, b = lane - (lane / B) * B;
            const int row = g * 4 + r;
            if (g_ok && row < p.rows) {
                float v0 = 0.f, v1 = 0.f;
                for (int k = 0; k < p.KS; ++k) {
                    v0 += red[warp + k][(0 * 4 + r) * B + b];
                    if constexpr (NM == 2) v1 += red[warp + k][(1 * 4 + r) * B + b];
                }
                p.a.y[(size_t)b * p.a.y_stride + row] = n_epilogue<EPI>(v0, v1);
            }
        }
        __syncthreads();
    }
    cp_wait<0>();
}

// ---------------------------------------------------------------------------
// Orientation N, K staged in chunks (x larger than the shared-memory budget)
// ---------------------------------------------------------------------------
struct NCParams {
    const uint8_t* tiles[2];
    QTileMap map;
    int rows, nb;
    int chunk_blocks, nchunks;
    int wk;        // warps splitting the blocks of a row (1, 2, 4, 8)
    int n_tiles;   // row tiles of (8 / wk) * R rows
    GemvArgs a;
};

template <int QT, int B, Pro PRO, Epi EPI>
__global__ void __launch_bounds__(THREADS) gemv_nc_kernel(const NCParams p) {
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    constexpr int R = (NM == 2) ? 2 : 4;
    constexpr int NV = QTraits<QT>::NV;
    constexpr int NVAL = NM * R * B;

    extern __shared__ __align__(16) float xs[];
    __shared__ float red[8][NVAL];
    __shared__ float s_red[8 * B];
    __shared__ float s_inv[B];

    pdl_trigger();
    pdl_wait();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wk = p.wk, wrn = 8 / wk;
    const int wr = warp / wk, wki = warp - wr * wk;
    const int d_model = p.nb * 32;

    if constexpr (PRO == Pro::AddNorm) {
        block_rms_inv<B>(p.a.xin, p.a.yin, p.a.x_stride, d_model, p.a.eps, s_red, s_inv);
        if (blockIdx.x == 0) write_xout<B>(p.a, d_model, s_inv);
    }
    for (int tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
        const int row0 = (tile * wrn + wr) * R;
        float acc[NM][R][B];
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int b = 0; b < B; ++b) acc[m][r][b] = 0.f;
        for (int ch = 0; ch < p.nchunks; ++ch) {
            const int b0 = ch * p.chunk_blocks;
            const int nbc = min(p.chunk_blocks, p.nb - b0);
            if (p.nchunks > 1 || tile == (int)blockIdx.x) {
                __syncthreads();
                stage_x<QT, B, PRO>(xs, p.a, b0, nbc, p.chunk_blocks, s_inv);
                __syncthreads();
            }
            for (int j = lane + 32 * wki; j < nbc; j += 32 * wk) {
                uint4 q[NM][R][NV];
                float dsc[NM][R];
#pragma unroll
                for (int m = 0; m < NM; ++m)
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const int row = row0 + r;
                        if (row < p.rows) {
                            int64_t d_off, q_off;
                            p.map.offsets(row, b0 + j, &d_off, &q_off);
#pragma unroll
                            for (int v = 0; v < NV; ++v) q[m][r][v] = ld_stream_u4(p.tiles[m] + q_off + 16 * v);
                            dsc[m][r] = fp16_ftz(ld_stream_u16(reinterpret_cast<const uint16_t*>(p.tiles[m] + d_off)));
                        } else {
#pragma unroll
                            for (int v = 0; v < NV; ++v) q[m][r][v] = make_uint4(0, 0, 0, 0);
                            dsc[m][r] = 0.f;
                        }
                    }
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float4* xv = reinterpret_cast<const float4*>(xs + ((size_t)b * p.chunk_blocks + j) * XPAD);
                    float4 xr[8];
#pragma unroll
                    for (int t = 0; t < 8; ++t) xr[t] = xv[t];
#pragma unroll
                    for (int m = 0; m < NM; ++m)
#pragma unroll
                        for (int r = 0; r < R; ++r) acc[m][r][b] = fmaf(dsc[m][r], dot32<QT>(q[m][r], xr), acc[m][r][b]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int b = 0; b < B; ++b) acc[m][r][b] = warp_sum(acc[m][r][b]);
        __syncthreads();
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < NM; ++m)
#pragma unroll
                for (int r = 0; r < R; ++r)
#pragma unroll
                    for (int b = 0; b < B; ++b) red[warp][(m * R + r) * B + b] = acc[m][r][b];
        }
        __syncthreads();
        if (wki == 0 && lane < R * B) {
            const int r = lane / B, b = lane - (lane / B) * B;
            const int row = row0 + r;
            if (row < p.rows) {
                float v0 = 0.f, v1 = 0.f;
                for (int k = 0; k < wk; ++k) {
                    v0 += red[wr * wk + k][(0 * R + r) * B + b];
                    if constexpr (NM == 2) v1 += red[wr * wk + k][(1 * R + r) * B + b];
                }
                p.a.y[(size_t)b * p.a.y_stride + row] = n_epilogue<EPI>(v0, v1);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Orientation T (tiles of 32 rows x 1 block column)
// ---------------------------------------------------------------------------
struct TParams {
    const uint8_t* tiles;
    int64_t tile_bytes;
    int E;             // input rows
    int ngroups;       // 32-row groups
    int n_bc;          // block columns (outputs / 32)
    int S;             // CTAs splitting the rows of a block column
    int e_per_split;   // rows per CTA (multiple of the CTA row step)
    GemvArgs a;
};

// Columns per lane: 32 (a whole block) for B <= 2, else 8 (a quarter block).
template <int B>
struct TCfg {
    static constexpr int CPL = (B <= 2) ? 32 : 8;
    static constexpr int LPB = 32 / CPL;           // lanes per block
    static constexpr int ROWS_PER_WARP = 32 / LPB; // rows a warp covers per step
    static constexpr int STEP = 8 * ROWS_PER_WARP; // rows a CTA covers per step
    static constexpr int U = 4;                    // steps in flight
};

template <int QT, int CPL>
__device__ __forceinline__ void t_load(uint4* q, float& dsc, const uint8_t* col, int64_t tb, int e, int quarter) {
    constexpr int QB = QTraits<QT>::QB;
    const uint8_t* tile = col + (int64_t)(e >> 5) * tb;
    const int l = e & 31;
    const uint8_t* qp = tile + 64 + l * QB;
    if constexpr (CPL == 32) {
        q[0] = ld_stream_u4(qp);
        if constexpr (QT == AT_GGML_Q8_0) q[1] = ld_stream_u4(qp + 16);
    } else {
        // the 16-byte vector holding this lane's quarter (4 or 8 bytes)
        q[0] = ld_stream_u4(qp + (QT == AT_GGML_Q8_0 ? 16 * (quarter >> 1) : 0));
    }
    dsc = fp16_ftz(ld_stream_u16(reinterpret_cast<const uint16_t*>(tile + l * 2)));
}

// Decodes this lane's CPL weights into CPL/2 pairs of consecutive columns.
template <int QT, int CPL>
__device__ __forceinline__ void t_decode(const uint4* q, int quarter, float2* wv) {
    if constexpr (CPL == 32) {
        decode32<QT>(q, wv);
    } else if constexpr (QT == AT_GGML_Q4_0) {
        const uint32_t a4[4] = {q[0].x, q[0].y, q[0].z, q[0].w};
        const uint32_t w = a4[quarter];  // bytes 4*quarter..: columns 8*quarter + 0..7
        const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
        const float2 moff = f2(-8388616.f, -8388616.f);
#pragma unroll
        for (int k = 0; k < 4; ++k) wv[k] = __fadd2_rn(f2(magic_byte(lo, k), magic_byte(hi, k)), moff);
    } else {
        const uint32_t a4[4] = {q[0].x, q[0].y, q[0].z, q[0].w};
        const int h = quarter & 1;  // which 8 bytes of the loaded 16
        const float2 moff = f2(-8388736.f, -8388736.f);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint32_t u = a4[2 * h + i] ^ 0x80808080u;
            wv[2 * i + 0] = __fadd2_rn(f2(magic_byte(u, 0), magic_byte(u, 1)), moff);
            wv[2 * i + 1] = __fadd2_rn(f2(magic_byte(u, 2), magic_byte(u, 3)), moff);
        }
    }
}

template <int QT, int B, Pro PRO, Epi EPI>
__global__ void __launch_bounds__(THREADS, 2) gemv_t_kernel(const TParams p) {
    using C = TCfg<B>;
    constexpr int CPL = C::CPL, LPB = C::LPB, U = C::U;
    constexpr int NPAIR = CPL / 2;

    extern __shared__ __align__(16) float xs[];  // [B][e_per_split]
    __shared__ float red[8][B][32];
    __shared__ float s_red[8 * B];
    __shared__ float s_inv[B];
    __shared__ int s_last;

    pdl_trigger();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x / p.S, s = blockIdx.x - (blockIdx.x / p.S) * p.S;
    const int e_lo = s * p.e_per_split;
    const int e_hi = min(p.E, e_lo + p.e_per_split);
    const int ne = e_hi - e_lo;
    const int quarter = (LPB == 1) ? 0 : (lane & (LPB - 1));
    const int row_in_warp = lane / LPB;
    const uint8_t* col = p.tiles + (size_t)c * p.ngroups * p.tile_bytes;

    // first U steps of weights before waiting on earlier kernels
    uint4 q[U][2];
    float dsc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int i = u * C::STEP + warp * C::ROWS_PER_WARP + row_in_warp;
        if (i < ne) t_load<QT, CPL>(q[u], dsc[u], col, p.tile_bytes, e_lo + i, quarter);
    }
    pdl_wait();

    if constexpr (PRO == Pro::AddNorm) {
        block_rms_inv<B>(p.a.xin, p.a.yin, p.a.x_stride, p.E, p.a.eps, s_red, s_inv);
        if (blockIdx.x == 0) write_xout<B>(p.a, p.E, s_inv);
    }
    if ((p.a.x_stride & 3) != 0 || (ne & 3) != 0) {
        // rows not 16-byte aligned: scalar staging
        for (int idx = tid; idx < B * ne; idx += THREADS) {
            const int bb = idx / ne, i = idx - bb * ne;
            const size_t off = (size_t)bb * p.a.x_stride + e_lo + i;
            float v;
            if constexpr (PRO == Pro::Plain) {
                v = p.a.x[off];
            } else {
                float t = p.a.xin[off];
                if (p.a.yin) t = __fadd_rn(t, p.a.yin[off]);
                v = norm_apply(t, s_inv[bb], p.a.gamma[e_lo + i]);
            }
            xs[bb * p.e_per_split + i] = v;
        }
    } else {
        // x slice [e_lo, e_hi) of each of the B rows, float4 (e_lo is a multiple of 64)
        const int n4 = ne >> 2;
        for (int base = 0; base < B * n4; base += THREADS * 4) {
            float4 v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int idx = base + k * THREADS + tid;
                if (idx < B * n4) {
                    const int bb = idx / n4, i4 = idx - bb * n4;
                    const size_t off = (size_t)bb * p.a.x_stride + e_lo + 4 * i4;
                    if constexpr (PRO == Pro::Plain) {
                        v[k] = *reinterpret_cast<const float4*>(p.a.x + off);
                    } else {
                        float4 t = *reinterpret_cast<const float4*>(p.a.xin + off);
                        if (p.a.yin) {
                            const float4 u = *reinterpret_cast<const float4*>(p.a.yin + off);
                            t.x = __fadd_rn(t.x, u.x); t.y = __fadd_rn(t.y, u.y);
                            t.z = __fadd_rn(t.z, u.z); t.w = __fadd_rn(t.w, u.w);
                        }
                        v[k] = t;
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int idx = base + k * THREADS + tid;
                if (idx < B * n4) {
                    const int bb = idx / n4, i4 = idx - bb * n4;
                    float4 o = v[k];
                    if constexpr (PRO == Pro::AddNorm) {
                        const float4 g = *reinterpret_cast<const float4*>(p.a.gamma + e_lo + 4 * i4);
                        const float inv = s_inv[bb];
                        o = make_float4(norm_apply(o.x, inv, g.x), norm_apply(o.y, inv, g.y),
                                        norm_apply(o.z, inv, g.z), norm_apply(o.w, inv, g.w));
                    }
                    *reinterpret_cast<float4*>(xs + bb * p.e_per_split + 4 * i4) = o;
                }
            }
        }
    }
    __syncthreads();

    float2 acc[B][NPAIR];
#pragma unroll
    for (int b = 0; b < B; ++b)
#pragma unroll
        for (int k = 0; k < NPAIR; ++k) acc[b][k] = f2(0.f, 0.f);

    for (int base = 0; base < ne; base += C::STEP * U) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = base + u * C::STEP + warp * C::ROWS_PER_WARP + row_in_warp;
            if (i < ne) {
                float2 wv[NPAIR];
                t_decode<QT, CPL>(q[u], quarter, wv);
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float sv = __fmul_rn(dsc[u], xs[b * p.e_per_split + i]);
                    const float2 s2 = f2(sv, sv);
#pragma unroll
                    for (int k = 0; k < NPAIR; ++k) acc[b][k] = __ffma2_rn(wv[k], s2, acc[b][k]);
                }
            }
            const int in = i + C::STEP * U;
            if (in < ne) t_load<QT, CPL>(q[u], dsc[u], col, p.tile_bytes, e_lo + in, quarter);
        }
    }

    // Butterfly reduce-scatter across the lanes sharing a block column.
#pragma unroll
    for (int b = 0; b < B; ++b) {
        float v[CPL];
#pragma unroll
        for (int k = 0; k < NPAIR; ++k) {
            v[2 * k] = acc[b][k].x;
            v[2 * k + 1] = acc[b][k].y;
        }
        int n = CPL;
#pragma unroll
        for (int bit = 16; bit >= LPB; bit >>= 1) {
            const bool upper = (lane & bit) != 0;
            n >>= 1;
#pragma unroll
            for (int t = 0; t < CPL / 2; ++t) {
                if (t < n) {
                    const float send = upper ? v[t] : v[t + n];
                    const float keep = upper ? v[t + n] : v[t];
                    v[t] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
                }
            }
        }
        // v[0] is column: CPL == 32 -> lane; CPL == 8 -> 8 * quarter + (lane >> 2)
        const int colx = (CPL == 32) ? lane : (8 * quarter + (lane >> 2));
        red[warp][b][colx] = v[0];
    }
    __syncthreads();

    // CTA partial for (block column c, rows [e_lo, e_hi)): thread (b = warp, col = lane)
    float val = 0.f;
    const int b_me = warp, cl = lane;
    if (b_me < B) {
#pragma unroll
        for (int w = 0; w < 8; ++w) val += red[w][b_me][cl];
    }
    if (p.S > 1) {
        if (b_me < B) p.a.scratch[(((size_t)c * p.S + s) * B + b_me) * 32 + cl] = val;
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const unsigned prev = atomicAdd(&p.a.counters[c], 1u);
            s_last = (prev == (unsigned)(p.S - 1));
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (b_me < B) {
            val = 0.f;
            for (int k = 0; k < p.S; ++k)
                val += __ldcg(&p.a.scratch[(((size_t)c * p.S + k) * B + b_me) * 32 + cl]);
        }
        if (tid == 0) p.a.counters[c] = 0u;
    }
    if (b_me >= B) return;

    const int j = c * 32 + cl;  // output column
    if constexpr (EPI == Epi::Plain) {
        p.a.y[(size_t)b_me * p.a.y_stride + j] = val;
    } else {
        // QKV epilogue: RoPE on q and k (core/Kernels.java:296-309 vector path:
        // a' = fma(a, c, b * -s), b' = fma(b, c, a * s)), then the KV-cache
        // append of k and v (inference/KVCache.java:79-95).
        const int hd = p.a.head_dim;
        const int nq = p.a.n_q_cols, nkv = p.a.n_kv_cols;
        const int64_t pos = p.a.pos[b_me];
        const float partner = __shfl_xor_sync(0xffffffffu, val, 1);
        float out = val;
        if (j < nq + nkv) {
            const int dd = (j < nq ? j : j - nq) % hd;
            const float cs = p.a.rope_cos[pos * hd + dd];
            const float sn = p.a.rope_sin[pos * hd + dd];
            if ((dd & 1) == 0) out = fmaf(val, cs, __fmul_rn(partner, -sn));
            else out = fmaf(val, cs, __fmul_rn(partner, sn));
        }
        if (j < nq) {
            p.a.y[(size_t)b_me * p.a.y_stride + j] = out;
        } else {
            const bool is_k = j < nq + nkv;
            const int jj = is_k ? j - nq : j - nq - nkv;
            const int kvh = jj / hd, dd = jj - kvh * hd;
            float* cache = is_k ? p.a.kcache : p.a.vcache;
            cache[(size_t)b_me * p.a.kv_slot_stride + ((size_t)kvh * p.a.ctx_len + pos) * hd + dd] = out;
        }
    }
}

// ---------------------------------------------------------------------------
// Host-side launch configuration
// ---------------------------------------------------------------------------
std::mutex g_attr_mu;
std::map<const void*, int> g_smem_set;  // kernel -> dynamic smem attribute already set
std::map<std::pair<const void*, int>, int> g_occ;

void ensure_smem(const void* fn, int smem) {
    std::lock_guard<std::mutex> lk(g_attr_mu);
    auto it = g_smem_set.find(fn);
    if (it != g_smem_set.end() && it->second >= smem) return;
    AT_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    g_smem_set[fn] = smem;
}

int occupancy(const void* fn, int smem) {
    {
        std::lock_guard<std::mutex> lk(g_attr_mu);
        auto it = g_occ.find({fn, smem});
        if (it != g_occ.end()) return it->second;
    }
    int n = 0;
    AT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, THREADS, smem));
    n = n < 1 ? 1 : n;
    std::lock_guard<std::mutex> lk(g_attr_mu);
    g_occ[{fn, smem}] = n;
    return n;
}

template <class P>
void launch(const void* fn, int grid, int smem, cudaStream_t s, bool pdl, const P& params, int threads = THREADS) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    void* args[] = {const_cast<P*>(&params)};
    AT_CUDA(cudaLaunchKernelExC(&cfg, fn, args));
}

// Chooses how many warps split the steps of a 4-row group (KS), and how many
// rounds of groups each CTA (one per SM) walks, minimising the steps per warp.
void n4_config(int ngroups, int nsteps, int num_sms, int* KS, int* gpc, int* per, int* grid, int* steps_ks) {
    int best = -1;
    for (int ks = 1; ks <= N4_WARPS; ks *= 2) {
        if (ks > 1 && ks > nsteps) break;
        const int g = N4_WARPS / ks;
        const int ctas = (ngroups + g - 1) / g;
        const int pr = (ctas + num_sms - 1) / num_sms;
        const int sk = (nsteps + ks - 1) / ks;
        const int cost = pr * sk;
        if (best < 0 || cost < best) {
            best = cost;
            *KS = ks;
            *gpc = g;
            *per = pr;
            *grid = (ngroups + g * pr - 1) / (g * pr);
            *steps_ks = sk;
        }
    }
}

template <int QT, int B, Pro PRO, Epi EPI, int NST>
void run_n4(const at_qmat* m, const GemvArgs& a, int num_sms, cudaStream_t s, bool pdl, int xbytes) {
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    N4Params p{};
    p.tiles[0] = m->tiles;
    p.tiles[1] = (NM == 2) ? a.m2->tiles : m->tiles;
    p.rows = (int)m->rows;
    p.nb = (int)(m->cols / QK);
    p.ngroups = (int)m->ngroups;
    p.nsteps = (int)m->nsteps;
    p.ring_off = xbytes;
    p.a = a;
    int grid = 1;
    n4_config(p.ngroups, p.nsteps, num_sms, &p.KS, &p.gpc, &p.per, &grid, &p.steps_ks);
    const int smem = xbytes + N4_WARPS * NST * NM * NTile<QT>::BYTES;
    const void* fn = reinterpret_cast<const void*>(&gemv_n4_kernel<QT, B, PRO, EPI, NST>);
    ensure_smem(fn, smem);
    launch(fn, grid, smem, s, pdl, p, N4_THREADS);
}

template <int QT, int B, Pro PRO, Epi EPI>
void run_n(const at_qmat* m, const GemvArgs& a, int num_sms, cudaStream_t s, bool pdl) {
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    const int nb = (int)(m->cols / QK);
    const int xbytes = B * nb * XPAD * 4;
    const int slot = NM * NTile<QT>::BYTES;
    constexpr int kBudget = 200 * 1024;
    if constexpr (B <= 2) {
        // deepest ring (4 or 2 steps per warp) that fits next to the staged x
        if (xbytes + N4_WARPS * 4 * slot <= kBudget) { run_n4<QT, B, PRO, EPI, 4>(m, a, num_sms, s, pdl, xbytes); return; }
        if (xbytes + N4_WARPS * 2 * slot <= kBudget) { run_n4<QT, B, PRO, EPI, 2>(m, a, num_sms, s, pdl, xbytes); return; }
    }
    constexpr int R = (NM == 2) ? 2 : 4;
    NCParams p{};
    p.tiles[0] = m->tiles;
    p.tiles[1] = (NM == 2) ? a.m2->tiles : m->tiles;
    p.map = tile_map(m);
    p.rows = (int)m->rows;
    p.nb = nb;
    p.chunk_blocks = std::min(p.nb, std::max(32, kMaxXSmemChunk / (B * XPAD * 4)));
    p.nchunks = (p.nb + p.chunk_blocks - 1) / p.chunk_blocks;
    p.a = a;
    const int smem = B * p.chunk_blocks * XPAD * 4;
    const void* fn = reinterpret_cast<const void*>(&gemv_nc_kernel<QT, B, PRO, EPI>);
    ensure_smem(fn, smem);
    const int occ = occupancy(fn, smem);
    int wk = 1;
    auto tiles = [&](int w) { return (p.rows + (8 / w) * R - 1) / ((8 / w) * R); };
    while (wk < 8 && tiles(wk) < 2 * num_sms && p.chunk_blocks >= 64 * wk) wk *= 2;
    p.wk = wk;
    p.n_tiles = tiles(wk);
    const int grid = std::max(1, std::min(p.n_tiles, num_sms * occ));
    launch(fn, grid, smem, s, pdl, p);
}

void t_config(const at_qmat* m, int batch, int num_sms, int* S, int* eps_rows) {
    const int step = (batch <= 2) ? 256 : 64;
    const int E = (int)m->rows;
    const int n_bc = (int)(m->cols / QK);
    // enough CTAs for every SM, each with at least 4 steps of rows per warp
    int s = std::max(1, (5 * num_sms / 4 + n_bc - 1) / n_bc);
    s = std::min(s, std::max(1, E / (4 * step)));
    int per = (E + s - 1) / s;
    per = ((per + step - 1) / step) * step;
    // the staged x slice must fit the shared-memory budget
    const int cap = std::max(step, (kMaxXSmemChunk / (4 * batch)) / step * step);
    per = std::min(per, cap);
    *eps_rows = per;
    *S = (E + per - 1) / per;
}

template <int QT, int B, Pro PRO, Epi EPI>
void run_t(const at_qmat* m, const GemvArgs& a, int num_sms, cudaStream_t s, bool pdl) {
    TParams p{};
    p.tiles = m->tiles;
    p.tile_bytes = m->tile_bytes;
    p.E = (int)m->rows;
    p.ngroups = (int)m->ngroups;
    p.n_bc = (int)(m->cols / QK);
    t_config(m, B, num_sms, &p.S, &p.e_per_split);
    p.a = a;
    if (p.S > 1) AT_REQUIRE(a.scratch && a.counters, AT_ERR_STATE, "T GEMV needs split scratch");
    const int smem = B * p.e_per_split * 4;
    const void* fn = reinterpret_cast<const void*>(&gemv_t_kernel<QT, B, PRO, EPI>);
    ensure_smem(fn, smem);
    launch(fn, p.n_bc * p.S, smem, s, pdl, p);
}

template <int QT, Pro PRO, Epi EPI, bool IS_T>
void dispatch_b(const at_qmat* m, int batch, const GemvArgs& a, int num_sms, cudaStream_t s, bool pdl) {
#define AT_CASE(BB)                                                           \
    case BB:                                                                  \
        if constexpr (IS_T) run_t<QT, BB, PRO, EPI>(m, a, num_sms, s, pdl);   \
        else run_n<QT, BB, PRO, EPI>(m, a, num_sms, s, pdl);                  \
        break;
    switch (batch) {
        AT_CASE(1) AT_CASE(2) AT_CASE(3) AT_CASE(4) AT_CASE(5) AT_CASE(6) AT_CASE(7) AT_CASE(8)
        default: fail(AT_ERR_INVALID_ARG, "batch must be in [1, 8]");
    }
#undef AT_CASE
}

template <Pro PRO, Epi EPI, bool IS_T>
void dispatch_q(const at_qmat* m, int batch, const GemvArgs& a, int num_sms, cudaStream_t s, bool pdl) {
    if (m->type == AT_GGML_Q4_0) dispatch_b<AT_GGML_Q4_0, PRO, EPI, IS_T>(m, batch, a, num_sms, s, pdl);
    else if (m->type == AT_GGML_Q8_0) dispatch_b<AT_GGML_Q8_0, PRO, EPI, IS_T>(m, batch, a, num_sms, s, pdl);
    else fail(AT_ERR_UNSUPPORTED, "fused GEMV supports Q4_0 and Q8_0");
}

}  // namespace

void gemv_t_scratch_need(const at_qmat* m, int batch, int num_sms, size_t* floats, size_t* counters) {
    int S = 1, per = 0;
    t_config(m, batch, num_sms, &S, &per);
    const size_t n_bc = (size_t)(m->cols / QK);
    *floats = (S > 1) ? n_bc * S * batch * 32 : 0;
    *counters = (S > 1) ? n_bc : 0;
}

void launch_gemv_n(const at_qmat* m, int batch, Pro pro, Epi epi, const GemvArgs& a, int num_sms,
                   cudaStream_t s, bool pdl) {
    AT_REQUIRE(m->cols % QK == 0, AT_ERR_INVALID_ARG, "cols must be a multiple of 32");
    AT_REQUIRE(m->orient == AT_ORIENT_N, AT_ERR_INVALID_ARG, "matrix is not stored for orientation N");
    if (pro == Pro::Plain && epi == Epi::Plain) dispatch_q<Pro::Plain, Epi::Plain, false>(m, batch, a, num_sms, s, pdl);
    else if (pro == Pro::AddNorm && epi == Epi::Plain) dispatch_q<Pro::AddNorm, Epi::Plain, false>(m, batch, a, num_sms, s, pdl);
    else if (pro == Pro::AddNorm && epi == Epi::SiluMul) {
        AT_REQUIRE(a.m2 && a.m2->type == m->type && a.m2->rows == m->rows && a.m2->cols == m->cols,
                   AT_ERR_INVALID_ARG, "gate/up matrices must match");
        dispatch_q<Pro::AddNorm, Epi::SiluMul, false>(m, batch, a, num_sms, s, pdl);
    } else fail(AT_ERR_UNSUPPORTED, "unsupported N prologue/epilogue combination");
}

void launch_gemv_t(const at_qmat* m, int batch, Pro pro, Epi epi, const GemvArgs& a, int num_sms,
                   cudaStream_t s, bool pdl) {
    AT_REQUIRE(m->cols % QK == 0, AT_ERR_INVALID_ARG, "cols must be a multiple of 32");
    AT_REQUIRE(m->orient == AT_ORIENT_T, AT_ERR_INVALID_ARG, "matrix is not stored for orientation T");
    if (pro == Pro::Plain && epi == Epi::Plain) dispatch_q<Pro::Plain, Epi::Plain, true>(m, batch, a, num_sms, s, pdl);
    else if (pro == Pro::AddNorm && epi == Epi::QkvRope) dispatch_q<Pro::AddNorm, Epi::QkvRope, true>(m, batch, a, num_sms, s, pdl);
    else fail(AT_ERR_UNSUPPORTED, "unsupported T prologue/epilogue combination");
}

// ---------------------------------------------------------------------------
// FP32 GEMV (Kernels.sgemv on FP32 operands): one warp per output row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(THREADS) sgemv_f32_kernel(const float* __restrict__ A, const float* __restrict__ x,
                                                              float* __restrict__ y, int M, int K, int batch, int lda) {
    const int warp = (blockIdx.x * THREADS + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= M) return;
    const float* a = A + (size_t)warp * lda;
    for (int b = 0; b < batch; ++b) {
        float acc = 0.f;
        for (int k = lane; k < K; k += 32) acc = fmaf(a[k], x[(size_t)b * K + k], acc);
        acc = warp_sum(acc);
        if (lane == 0) y[(size_t)b * M + warp] = acc;
    }
}

void launch_sgemv_f32(const float* A, const float* x, float* y, int M, int K, int batch, int a_ld,
                      cudaStream_t s) {
    if (M <= 0) return;
    const int grid = (M * 32 + THREADS - 1) / THREADS;
    sgemv_f32_kernel<<<grid, THREADS, 0, s>>>(A, x, y, M, K, batch, a_ld);
    AT_CUDA(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Orientation T with its split scratch in a static device array
// ---------------------------------------------------------------------------
// For callers that cannot allocate device memory: the split-K partials and
// the per-column arrival counters of the orientation-T GEMV live in one
// file-scope array instead of cudaMalloc'd scratch. Every GPU that loads the
// library holds this array (256 KiB) until the process exits.
namespace {
constexpr size_t kStaticSplitFloats = 61440;   // partials (240 KiB)
constexpr size_t kStaticSplitCounters = 4096;  // arrival counters (16 KiB)
constexpr int kMaxDevices = 64;
static __device__ __align__(256) uint32_t g_static_split_scratch[kStaticSplitFloats + kStaticSplitCounters];

std::mutex g_static_mu;
void* g_static_addr[kMaxDevices] = {};

// Device address of g_static_split_scratch on `device`, looked up once per
// device with that device current (the host-side name is not a device address).
void* static_split_scratch(int device) {
    AT_REQUIRE(device >= 0 && device < kMaxDevices, AT_ERR_INVALID_ARG, "device index out of range");
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_addr[device]) {
        int cur = -1;
        AT_CUDA(cudaGetDevice(&cur));
        if (cur != device) AT_CUDA(cudaSetDevice(device));
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_split_scratch);
        if (cur != device) cudaSetDevice(cur);
        AT_CUDA(e);
        g_static_addr[device] = p;
    }
    return g_static_addr[device];
}
}  // namespace
}  // namespace at

extern "C" int at_gemv_t_static_scratch(at_ctx* ctx, const at_qmat* m, const float* x, float* y, int batch) {
    using namespace at;
    return guard([&] {
        AT_REQUIRE(ctx && m && x && y, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(m->orient == AT_ORIENT_T, AT_ERR_INVALID_ARG,
                   "at_gemv_t_static_scratch takes an orientation-T matrix (use at_gemv for orientation N)");
        AT_REQUIRE(m->type == AT_GGML_Q4_0 || m->type == AT_GGML_Q8_0, AT_ERR_UNSUPPORTED,
                   "at_gemv_t_static_scratch supports Q4_0 and Q8_0");
        AT_REQUIRE(batch >= 1 && batch <= 8, AT_ERR_INVALID_ARG, "batch must be in [1, 8]");
        AT_REQUIRE(((uintptr_t)x & 15) == 0, AT_ERR_INVALID_ARG, "x must be 16-byte aligned");
        size_t nf = 0, nc = 0;
        gemv_t_scratch_need(m, batch, ctx->num_sms, &nf, &nc);
        AT_REQUIRE(nf <= kStaticSplitFloats && nc <= kStaticSplitCounters, AT_ERR_INVALID_ARG,
                   "split scratch of " + std::to_string(nf) + " partials and " + std::to_string(nc) +
                       " counters exceeds the static maximum of " + std::to_string(kStaticSplitFloats) + " and " +
                       std::to_string(kStaticSplitCounters));
        uint32_t* base = static_cast<uint32_t*>(static_split_scratch(ctx->device));
        float* partials = reinterpret_cast<float*>(base);
        unsigned* counters = base + kStaticSplitFloats;
        // the array keeps the previous call's contents: the counters must start at zero
        if (nc) AT_CUDA(cudaMemsetAsync(counters, 0, nc * sizeof(unsigned), ctx->stream));
        GemvArgs a;
        a.x = x;
        a.y = y;
        a.x_stride = (int)m->rows;
        a.y_stride = (int)m->cols;
        a.scratch = partials;
        a.counters = counters;
        launch_gemv_t(m, batch, Pro::Plain, Epi::Plain, a, ctx->num_sms, ctx->stream);
    });
}
