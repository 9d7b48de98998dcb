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
// Orientation N (rows = outputs, blocks along the row), batch <= 2: the
// tiles (4 rows x 32 blocks) form one stream split evenly over one CTA per
// SM and its 16 warps; a warp copies its tiles through a cp.async ring in
// shared memory, one block per lane per step, and x is staged once per CTA
// in shared memory (natural order, 36 floats per 32-element block so a
// quarter-warp of 128-bit reads touches 32 distinct banks). The RMSNorm of
// an AddNorm prologue is folded into the result (the GEMV runs on
// (x + y) * gamma and 1/rms multiplies the finished dot products), so the
// prologue is one pass over x. Larger batches stage x in chunks.
// Orientation T (rows = inputs, blocks along the outputs): a lane owns rows
// of one block column (tiles of 32 rows) and accumulates its 32 (or 8)
// outputs; lanes combine by a butterfly reduce-scatter, warps through shared
// memory, and CTAs that split the rows through an ordered reduction by the
// last CTA to arrive (counter per block column, reset by that CTA).
// All kernels support programmatic dependent launch: weights (never written
// by an earlier kernel) are prefetched before griddepcontrol.wait; every
// activation read comes after it.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>

#include "at_internal.h"
#include "dev_common.cuh"
#include "qdecode.cuh"

namespace at {

namespace {

constexpr int THREADS = 256;
constexpr int XPAD = 36;                 // floats per staged 32-element block
constexpr int kMaxXSmemChunk = 96 * 1024;


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

// The same for the slice [c*n4/C, (c+1)*n4/C) of float4s of each row: CTA c of C.
template <int B, int NT>
__device__ __forceinline__ void write_xout_slice(const GemvArgs& a, int d, const float* s_inv, int c, int C) {
    const int n4 = d / 4;
    const int i0 = (int)((int64_t)c * n4 / C), i1 = (int)((int64_t)(c + 1) * n4 / C);
    for (int idx = threadIdx.x; idx < B * (i1 - i0); idx += NT) {
        const int bb = idx / (i1 - i0), i4 = i0 + idx - bb * (i1 - i0);
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
        return silu_mul(g, u);
    } else {
        return g;
    }
}

// ---------------------------------------------------------------------------
// Balanced unit streams (orientation N and T, batch <= 2)
// ---------------------------------------------------------------------------
// The tiles of a matrix form one stream of units in storage order:
//   N: unit (g, s) = tile of rows 4g..4g+3 x blocks 32s..32s+31 (the steps of
//      a row group are consecutive); segment = row group g;
//   T: unit (c, g) = tile of rows 32g..32g+31 of block column c (the tiles
//      of a column are consecutive); segment = block column c.
// CTA c (one per SM) streams units [start[c], start[c+1]) of a host-computed
// map (whole segments when that costs little balance, else an even split)
// and its 16 warps split that range evenly, so every SM streams the same
// bytes within a unit or a segment. A warp copies its units into a per-warp
// ring of NST slots with cp.async (16 bytes per lane-copy; a __syncwarp after
// each wait publishes the slot), accumulates in registers while consecutive
// units belong to one segment, and stores the segment's partial sums to its
// shared-memory slot when the segment changes. After one barrier each
// segment inside the CTA is summed over its warps in warp order. A segment
// shared with neighbouring CTAs goes through global scratch: every CTA
// stores its partial (slot 2c for its first segment, 2c + 1 for its last),
// and the last CTA to arrive (counter per segment, reset by that CTA) sums
// them in CTA order and applies the epilogue. Results do not depend on
// timing.
//
// Activation loads are issued before the bulk of the weight copies: the
// copies of one SM drain at its share of HBM bandwidth, and a load queued
// behind them would wait for all of them.
constexpr int S_THREADS = 512;
constexpr int S_WARPS = S_THREADS / 32;
constexpr int kMaxStreamCtas = 160;

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Unit ranges of the CTAs: CTA c streams units [start[c], start[c + 1]).
struct StreamMap {
    int len;                           // units per segment
    int start[kMaxStreamCtas + 1];
};

template <int QT>
struct NTile {
    static constexpr int QB = QTraits<QT>::QB;
    static constexpr int BYTES = 4 * 32 * (2 + QB);  // 2304 (Q4_0) or 4352 (Q8_0)
    static constexpr int CHUNKS = BYTES / 16;
};

// Copies one unit (CHUNKS x 16 bytes) from src into a ring slot.
template <int CHUNKS>
__device__ __forceinline__ void copy_unit(uint32_t slot, const uint8_t* src, int lane) {
#pragma unroll
    for (int u = 0; u < (CHUNKS + 31) / 32; ++u) {
        const int k = lane + 32 * u;
        if (k < CHUNKS) cp_async16(slot + (uint32_t)(16 * k), src + 16 * k);
    }
}

// Warp w of a CTA with n units streams units [floor(w n / 16), floor((w+1) n / 16))
// of the CTA's range; warp_of(x) is the warp holding unit x of the range.
__device__ __forceinline__ int warp_of(int x, int n) {
    const int w = (16 * x + 15) / n;
    return w < S_WARPS - 1 ? w : S_WARPS - 1;
}

// This CTA's sum of the warp partials of segment `seg` (units [s0, s1) of the
// CTA range, relative), value v, in warp order. Warp w stored its partial of
// its k-th segment at red[(w * slots + k) * vals + v].
__device__ __forceinline__ float sum_warp_partials(const float* red, int slots, int vals, int seg, int s0, int s1,
                                                   int n, int u_lo, int len, int v) {
    const int wa = warp_of(s0, n), wb = warp_of(s1 - 1, n);
    float acc = 0.f;
    for (int w = wa; w <= wb; ++w) {
        const int first_unit = u_lo + ((w * n) >> 4);
        const int k = seg - first_unit / len;
        if (k >= 0 && k < slots) acc += red[((size_t)w * slots + k) * vals + v];
    }
    return acc;
}

// CTAs [first, last] whose ranges overlap segment `seg` (one of them is `cta`).
__device__ __forceinline__ void seg_ctas(const StreamMap& mp, int C, int cta, int seg, int* first, int* last) {
    const int s0 = seg * mp.len, s1 = s0 + mp.len;
    int f = cta, l = cta;
    while (f > 0 && mp.start[f] > s0) --f;
    while (l + 1 < C && mp.start[l + 1] < s1) ++l;
    *first = f;
    *last = l;
}

// Scratch slot of CTA cc's partial of segment seg: 2cc if seg is cc's first segment, else 2cc + 1.
__device__ __forceinline__ int seg_slot(const StreamMap& mp, int cc, int seg) {
    return 2 * cc + (mp.start[cc] >= seg * mp.len ? 0 : 1);
}

// Finishes the (at most two) segments this CTA shares with other CTAs: the
// partials are already in scratch; the last CTA to arrive at a segment calls
// finish(seg, first, last) with every partial visible. One thread publishes
// the CTA's stores (barrier, then a device-scope fence, which is cumulative
// over the stores the barrier ordered before it) and takes the arrival ticket.
template <class Finish>
__device__ __forceinline__ void finish_shared_segments(const GemvArgs& a, const StreamMap& mp, int cta, int seg_lo,
                                                       int seg_hi, bool lo_shared, bool hi_shared, int* s_last,
                                                       Finish finish) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last[0] = s_last[1] = 0;
        int f, l;
        if (lo_shared) {
            seg_ctas(mp, gridDim.x, cta, seg_lo, &f, &l);
            s_last[0] = atomicAdd(&a.counters[seg_lo], 1u) == (unsigned)(l - f);
        }
        if (hi_shared && !(lo_shared && seg_hi == seg_lo)) {
            seg_ctas(mp, gridDim.x, cta, seg_hi, &f, &l);
            s_last[1] = atomicAdd(&a.counters[seg_hi], 1u) == (unsigned)(l - f);
        }
        if (s_last[0] | s_last[1]) __threadfence();
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        if (s_last[k]) {
            const int seg = k ? seg_hi : seg_lo;
            int f, l;
            seg_ctas(mp, gridDim.x, cta, seg, &f, &l);
            finish(seg, f, l);
            if (threadIdx.x == 0) a.counters[seg] = 0u;
        }
    }
}

// Stages x (Pro::Plain) or (xin + yin) * gamma (Pro::AddNorm) for all nb
// blocks of B rows into shared memory (natural order, XPAD floats per block),
// eight float4 loads in flight per thread. For AddNorm it also returns this
// thread's sums of (xin + yin)^2 per row: the RMSNorm scale 1/rms multiplies
// the finished dot products instead of every staged element, so the staging
// needs no prior reduction pass.
// The CTA's slice of the normed residual stream (AddNorm), float4 [i0, i0 + len)
// of every row (the split of write_xout_slice). When B * len <= kXoutStash
// the staging pass parks t = xin + yin and gamma of the slice in shared memory
// and the kernel writes (t * inv) * gamma once 1/rms is known, with no second
// load at its end; longer slices are written by write_xout_slice.
constexpr int kXoutStash = 16;
struct XoutStash {
    float4 t[kXoutStash];
    float4 g[kXoutStash];
};
__device__ __forceinline__ void xout_slice(int d, int c, int C, int* i0, int* len) {
    const int n4 = d / 4;
    *i0 = (int)((int64_t)c * n4 / C);
    *len = (int)((int64_t)(c + 1) * n4 / C) - *i0;
}
template <int B, int NT>
__device__ __forceinline__ void stash_put(XoutStash* st, int i0, int len, int bb, int r, float4 t, float4 g) {
    if (B * len <= kXoutStash && r >= i0 && r < i0 + len) {
        st->t[bb * len + r - i0] = t;
        st->g[bb * len + r - i0] = g;
    }
}
// Writes the stashed slice (barrier between stash_put and this call), or the
// slice from global memory when it was too long to stash.
template <int B, int NT>
__device__ __forceinline__ void write_xout_stashed(const GemvArgs& a, int d, const float* s_inv, int c, int C,
                                                   const XoutStash* st) {
    int i0, len;
    xout_slice(d, c, C, &i0, &len);
    if (B * len > kXoutStash) {
        write_xout_slice<B, NT>(a, d, s_inv, c, C);
        return;
    }
    const int tid = threadIdx.x;
    if (tid < B * len) {
        const int bb = tid / len, i4 = i0 + tid - bb * len;
        const float4 t = st->t[tid], g = st->g[tid];
        const float inv = s_inv[bb];
        *reinterpret_cast<float4*>(a.xout + (size_t)bb * a.x_stride + (size_t)i4 * 4) = make_float4(
            norm_apply(t.x, inv, g.x), norm_apply(t.y, inv, g.y), norm_apply(t.z, inv, g.z), norm_apply(t.w, inv, g.w));
    }
}

template <int QT, int B, Pro PRO, int NT>
__device__ __forceinline__ void stage_x_fold(float* xs, const GemvArgs& a, int nb, float* ss, XoutStash* st,
                                             int st_i0, int st_len) {
    const int nf4 = nb * 8;
    const int total = B * nf4;
#pragma unroll
    for (int b = 0; b < B; ++b) ss[b] = 0.f;
    for (int base = 0; base < total; base += NT * 8) {
        float4 v[8], g[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int idx = base + k * NT + threadIdx.x;
            if (idx < total) {
                const int bb = idx / nf4, r = idx - bb * nf4;
                const size_t off = (size_t)bb * a.x_stride + 4 * (size_t)r;
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
                    g[k] = *reinterpret_cast<const float4*>(a.gamma + 4 * (size_t)r);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int idx = base + k * NT + threadIdx.x;
            if (idx < total) {
                const int bb = idx / nf4, r = idx - bb * nf4;
                float4 o = v[k];
                if constexpr (PRO == Pro::AddNorm) {
                    float q = fmaf(o.x, o.x, fmaf(o.y, o.y, fmaf(o.z, o.z, __fmul_rn(o.w, o.w))));
#pragma unroll
                    for (int b = 0; b < B; ++b)
                        if (b == bb) ss[b] += q;
                    stash_put<B, NT>(st, st_i0, st_len, bb, r, o, g[k]);
                    o = make_float4(__fmul_rn(o.x, g[k].x), __fmul_rn(o.y, g[k].y), __fmul_rn(o.z, g[k].z),
                                    __fmul_rn(o.w, g[k].w));
                }
                v[k] = o;
            }
        }
        // Block sums (the 8 float4 of a block sit in 8 consecutive lanes: the
        // row length and the index bases are multiples of 8), then the
        // subnormal-form scaling of dot32_dn.
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int idx = base + k * NT + threadIdx.x;
            const bool in = idx < total;
            float bs = in ? (v[k].x + v[k].y) + (v[k].z + v[k].w) : 0.f;
            bs += __shfl_xor_sync(0xffffffffu, bs, 1);
            bs += __shfl_xor_sync(0xffffffffu, bs, 2);
            bs += __shfl_xor_sync(0xffffffffu, bs, 4);
            if (in) {
                const int bb = idx / nf4, r = idx - bb * nf4;
                const int e0 = (r & 7) * 4;  // element of the block
                float* dst = xs + ((size_t)bb * nb + (r >> 3)) * XPAD;
                const float4 o = v[k];
                *reinterpret_cast<float4*>(dst + e0) =
                    make_float4(__fmul_rn(o.x, exp2_i(kXExp - x_shift_dn<QT>(e0))),
                                __fmul_rn(o.y, exp2_i(kXExp - x_shift_dn<QT>(e0 + 1))),
                                __fmul_rn(o.z, exp2_i(kXExp - x_shift_dn<QT>(e0 + 2))),
                                __fmul_rn(o.w, exp2_i(kXExp - x_shift_dn<QT>(e0 + 3))));
                if ((r & 7) == 0) dst[32] = __fmul_rn(bs, exp2_i(kXExp - 149));
            }
        }
    }
}

// RMSNorm scales of the B rows from the per-warp sums of squares s_ss[warp][b]
// (fixed summation order: every CTA computes the same values).
template <int B, int NW>
__device__ __forceinline__ void rms_scales(const float* s_ss, int d, float eps, float* inv) {
#pragma unroll
    for (int b = 0; b < B; ++b) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) t += s_ss[w * B + b];
        inv[b] = rms_inv(t, d, eps);
    }
}

struct NSParams {
    const uint8_t* tiles[2];
    int rows, nb, nsteps;
    int slots;     // partial slots per warp (row groups one warp can touch)
    int red_off;   // byte offsets in dynamic shared memory: partial slots, weight rings
    int ring_off;
    int pre;       // ring slots copied before waiting on the previous kernel
    StreamMap map;
    GemvArgs a;
};

template <int QT, int B, Pro PRO, Epi EPI, int NST>
__global__ void __launch_bounds__(S_THREADS, 1) gemv_ns_kernel(const NSParams p) {
    static_assert((NST & (NST - 1)) == 0, "ring depth is a power of two");
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    using TL = NTile<QT>;
    constexpr int SLOT = NM * TL::BYTES;
    constexpr int NV = QTraits<QT>::NV;
    constexpr int VPG = NM * 4 * B;  // partial values per row group
    extern __shared__ __align__(16) float xs[];
    __shared__ float s_ss[S_WARPS * B];  // AddNorm: per-warp sums of squares
    __shared__ float s_inv[B];
    __shared__ int s_last[2];
    __shared__ XoutStash s_xo;  // AddNorm: this CTA's slice of the normed x

    pdl_trigger();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x;
    const int L = p.nsteps;
    const int u_lo = p.map.start[cta], u_hi = p.map.start[cta + 1], n = u_hi - u_lo;
    const int w_lo = u_lo + ((warp * n) >> 4);
    const int T = u_lo + (((warp + 1) * n) >> 4) - w_lo;
    int g = w_lo / L, s = w_lo - g * L;
    const int g_first = g;
    // row groups of this CTA; the first / last may be shared with neighbours
    const int g_lo = u_lo / L, g_hi = (u_hi - 1) / L;
    const bool lo_shared = g_lo * L < u_lo, hi_shared = (g_hi + 1) * L > u_hi;
    float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + p.red_off);
    const uint8_t* ring_ptr = reinterpret_cast<const uint8_t*>(xs) + p.ring_off + warp * NST * SLOT;
    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(ring_ptr);

    const uint8_t* src = p.tiles[0] + (size_t)w_lo * TL::BYTES;
    const uint8_t* src2 = p.tiles[1] + (size_t)w_lo * TL::BYTES;
    int issued = 0;
    auto issue_next = [&]() {
        const uint32_t slot = ring + (issued & (NST - 1)) * SLOT;
        if (issued < T) {
            copy_unit<TL::CHUNKS>(slot, src, lane);
            if constexpr (NM == 2) copy_unit<TL::CHUNKS>(slot + TL::BYTES, src2, lane);
            src += TL::BYTES;
            src2 += TL::BYTES;
        }
        cp_commit();
        ++issued;
    };
    // Weights are never written by earlier kernels: `pre` slots are copied
    // before waiting on them; the ring fills up inside the main loop, after
    // the activation loads.
    for (int k = 0; k < p.pre; ++k) issue_next();
    for (int i = tid; i < S_WARPS * p.slots * VPG; i += S_THREADS) red[i] = 0.f;
    pdl_wait();

    const int d_model = p.nb * 32;
    int st_i0 = 0, st_len = 0;
    xout_slice(d_model, cta, gridDim.x, &st_i0, &st_len);
    {
        float ss[B];
        stage_x_fold<QT, B, PRO, S_THREADS>(xs, p.a, p.nb, ss, &s_xo, st_i0, st_len);
        if constexpr (PRO == Pro::AddNorm) {
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float t = warp_sum(ss[b]);
                if (lane == 0) s_ss[warp * B + b] = t;
            }
        }
    }
    __syncthreads();

    float acc[NM * 4][B];
#pragma unroll
    for (int i = 0; i < NM * 4; ++i)
#pragma unroll
        for (int b = 0; b < B; ++b) acc[i][b] = 0.f;

    for (int t = 0; t < T; ++t) {
        while (issued < t + NST) issue_next();  // NST groups after this one are committed
        cp_wait<NST - 1>();
        __syncwarp();  // every lane's 16-byte pieces of this slot have landed
        const uint8_t* sp = ring_ptr + (t & (NST - 1)) * SLOT;
        const int j = s * 32 + lane;  // this lane's block
        if (j < p.nb) {
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
                    dsc[m * 4 + r] = __fmul_rn(
                        fp16_ftz_fast(*reinterpret_cast<const uint16_t*>(tb + (r * 32 + lane) * 2)), kDnUnscale);
                }
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float4* xv = reinterpret_cast<const float4*>(xs + ((size_t)b * p.nb + j) * XPAD);
                float4 xr[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) xr[k] = xv[k];
                const float sx = xs[((size_t)b * p.nb + j) * XPAD + 32];
#pragma unroll
                for (int i = 0; i < NM * 4; ++i) acc[i][b] = fmaf(dsc[i], dot32_dn<QT>(q[i], xr, sx), acc[i][b]);
            }
        }
        __syncwarp();  // every lane is done with this slot before it is refilled
        int s_next = s + 1, g_next = g;
        if (s_next == L) { s_next = 0; ++g_next; }
        if (t == T - 1 || g_next != g) {
            // row group done (or range end): lane sums into this warp's slot
            float* dst = red + ((size_t)warp * p.slots + (g - g_first)) * VPG;
#pragma unroll
            for (int i = 0; i < NM * 4; ++i)
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float v = warp_sum(acc[i][b]);
                    if (lane == 0) dst[i * B + b] = v;
                    acc[i][b] = 0.f;
                }
        }
        g = g_next;
        s = s_next;
    }
    cp_wait<0>();
    if (tid < B) {
        if constexpr (PRO == Pro::AddNorm) {
            float inv[B];
            rms_scales<B, S_WARPS>(s_ss, d_model, p.a.eps, inv);
            s_inv[tid] = inv[tid];
        } else {
            s_inv[tid] = 1.f;
        }
    }
    __syncthreads();
    if constexpr (PRO == Pro::AddNorm) {
        write_xout_stashed<B, S_THREADS>(p.a, d_model, s_inv, cta, gridDim.x, &s_xo);
    }

    // Row groups of this CTA: sum over warps in warp order, times the RMSNorm scale.
    const int ngc = g_hi - g_lo + 1;
    for (int it = tid; it < ngc * 4 * B; it += S_THREADS) {
        const int gi = it / (4 * B), rb = it - gi * (4 * B);
        const int r = rb / B, b = rb - (rb / B) * B;
        const int gg = g_lo + gi;
        const int s0 = max(gg * L, u_lo) - u_lo, s1 = min((gg + 1) * L, u_hi) - u_lo;
        float v[NM];
#pragma unroll
        for (int m = 0; m < NM; ++m)
            v[m] = sum_warp_partials(red, p.slots, VPG, gg, s0, s1, n, u_lo, L, (m * 4 + r) * B + b);
        if (!((gi == 0 && lo_shared) || (gi == ngc - 1 && hi_shared))) {
            const int row = gg * 4 + r;
            const float inv = s_inv[b];
            if (row < p.rows)
                p.a.y[(size_t)b * p.a.y_stride + row] = n_epilogue<EPI>(__fmul_rn(v[0], inv), __fmul_rn(v[NM - 1], inv));
        } else {
            float* dst = p.a.scratch + (2 * (size_t)cta + (gi == 0 ? 0 : 1)) * VPG;
#pragma unroll
            for (int m = 0; m < NM; ++m) dst[(m * 4 + r) * B + b] = v[m];
        }
    }
    if (lo_shared || hi_shared) {
        finish_shared_segments(p.a, p.map, cta, g_lo, g_hi, lo_shared, hi_shared, s_last, [&](int seg, int f, int l) {
            for (int it = tid; it < 4 * B; it += S_THREADS) {
                const int r = it / B, b = it - (it / B) * B;
                float v[NM];
#pragma unroll
                for (int m = 0; m < NM; ++m) v[m] = 0.f;
                for (int cc = f; cc <= l; ++cc) {
                    const float* part = p.a.scratch + (size_t)seg_slot(p.map, cc, seg) * VPG;
#pragma unroll
                    for (int m = 0; m < NM; ++m) v[m] += __ldcg(part + (m * 4 + r) * B + b);
                }
                const int row = seg * 4 + r;
                const float inv = s_inv[b];
                if (row < p.rows)
                    p.a.y[(size_t)b * p.a.y_stride + row] =
                        n_epilogue<EPI>(__fmul_rn(v[0], inv), __fmul_rn(v[NM - 1], inv));
            }
        });
    }
}

// ---------------------------------------------------------------------------
// Orientation N, batch 3..8: split K into 32-block steps
// ---------------------------------------------------------------------------
// CTA (p, q) stages the 1024 x values of step q for all batch rows and
// streams the tiles (g, q) of the row groups g of part p through per-warp
// cp.async rings, two tiles per unit: the gate and up tiles of one group
// (SiLU epilogue) or two consecutive groups. Lane l owns block 32q + l of
// the unit's 8 rows. x is staged per block as [32 elements][8 batch rows]
// in the subnormal-scaled form of the stream kernel (plus the block sums of
// each batch row), so each weight is decoded once (one mask per weight) and
// applied to the batch by FFMA2 over pairs of batch rows, and every x value
// read serves 8 rows. A group's 4 x B sums per matrix are combined over the
// lanes by a butterfly reduce-scatter (lane l ends with value l) and stored
// as the step's partial. A second kernel sums the steps' partials in step
// order (deterministic) and applies the epilogue. Folded RMSNorm as in the
// stream kernel: each CTA also stores its step's sums of (xin + yin)^2.
constexpr int Q_THREADS = 256;
constexpr int Q_WARPS = Q_THREADS / 32;
constexpr int Q_NST = 2;
constexpr int QX = 268;  // floats per staged block: 32 x 8 values, 8 block sums, 4 padding

struct NQParams {
    const uint8_t* tiles[2];
    int rows, nb, ngroups, nsteps;
    int P;          // row parts (gridDim.x); the steps are gridDim.y
    float* part;    // [nsteps][ngroups][VPAD] partial sums
    float* ssq;     // [P][nsteps][B] sums of squares (AddNorm)
    GemvArgs a;
};

// Sum over the 32 lanes of 32 values per lane: after the butterfly, lane l
// holds the total of value l.
__device__ __forceinline__ float lane_transpose_sum(float* v, int lane) {
    int nn = 32;
#pragma unroll
    for (int bit = 16; bit >= 1; bit >>= 1) {
        const bool upper = (lane & bit) != 0;
        nn >>= 1;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if (k < nn) {
                const float send = upper ? v[k] : v[k + nn];
                const float keep = upper ? v[k + nn] : v[k];
                v[k] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
            }
        }
    }
    return v[0];
}

// Values per row in a group partial: the batch, 7 padded to 8.
__host__ __device__ constexpr int nq_stride(int b) { return b == 7 ? 8 : b; }

// The subnormal-scaled fields of elements 4 kc .. 4 kc + 3 of a block (see
// dot32_dn): Q4_0 from 32-bit word kc / 2 of the block's 16 quant bytes,
// Q8_0 from word kc of its 32.
template <int QT>
__device__ __forceinline__ void q4_fields_dn(uint32_t w, int kc, float* f) {
    if constexpr (QT == AT_GGML_Q4_0) {
        if ((kc & 1) == 0) {
            f[0] = bits_f(w & 0xFu); f[1] = bits_f(w & 0xF0u); f[2] = bits_f(w & 0xF00u); f[3] = bits_f(w & 0xF000u);
        } else {
            const uint32_t t = w >> 24;
            f[0] = bits_f(w & 0xF0000u); f[1] = bits_f(w & 0xF00000u); f[2] = bits_f(t & 0xFu); f[3] = bits_f(t & 0xF0u);
        }
    } else {
        f[0] = bits_f((w ^ 0x80u) & 0xFFu);
        f[1] = bits_f((w ^ 0x8000u) & 0xFF00u);
        f[2] = bits_f((w ^ 0x800000u) & 0xFF0000u);
        f[3] = bits_f((w >> 24) ^ 0x80u);
    }
}

template <int QT, int B, Pro PRO, Epi EPI>
__global__ void __launch_bounds__(Q_THREADS, 1) gemv_nq_kernel(const NQParams p) {
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    using TL = NTile<QT>;
    constexpr int SLOT = 2 * TL::BYTES;  // two tiles per unit
    constexpr int QB = QTraits<QT>::QB;
    constexpr int BP = (B + 1) / 2;      // pairs of batch rows
    static_assert(4 * B <= 32, "one 32-value partial per matrix and group");
    extern __shared__ __align__(16) float xs[];  // [32 blocks][QX], then the rings
    pdl_trigger();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pp = blockIdx.x, q = blockIdx.y;
    const int g0 = (int)((int64_t)pp * p.ngroups / p.P), g1 = (int)((int64_t)(pp + 1) * p.ngroups / p.P);
    // unit i of this warp: SiLU: group g0 + warp + Q_WARPS i (gate, up); else
    // groups ga = g0 + 2 (warp + Q_WARPS i) and ga + 1 (when below g1)
    const int ng = g1 - g0;
    const int nmine = (NM == 2) ? (ng - warp + Q_WARPS - 1) / Q_WARPS
                                : ((ng + 1) / 2 - warp + Q_WARPS - 1) / Q_WARPS;
    const uint8_t* ring_ptr = reinterpret_cast<const uint8_t*>(xs) + 32 * QX * 4 + warp * Q_NST * SLOT;
    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(ring_ptr);
    auto unit_groups = [&](int i, int* ga, int* gb) {
        if constexpr (NM == 2) {
            *ga = *gb = g0 + warp + Q_WARPS * i;
        } else {
            *ga = g0 + 2 * (warp + Q_WARPS * i);
            *gb = *ga + 1 < g1 ? *ga + 1 : -1;
        }
    };
    int issued = 0;
    auto issue_next = [&]() {
        const uint32_t slot = ring + (issued & (Q_NST - 1)) * SLOT;
        if (issued < nmine) {
            int ga, gb;
            unit_groups(issued, &ga, &gb);
            copy_unit<TL::CHUNKS>(slot, p.tiles[0] + ((size_t)ga * p.nsteps + q) * TL::BYTES, lane);
            if (gb >= 0)
                copy_unit<TL::CHUNKS>(slot + TL::BYTES, p.tiles[NM - 1] + ((size_t)gb * p.nsteps + q) * TL::BYTES, lane);
        }
        cp_commit();
        ++issued;
    };
    issue_next();  // weights are never written by earlier kernels
    pdl_wait();

    // stage x (or (xin + yin) * gamma) for blocks 32q .. 32q + 31 of the B rows
    const int jb = q * 32, nbl = min(32, p.nb - jb);
    float ss[B];
#pragma unroll
    for (int b = 0; b < B; ++b) ss[b] = 0.f;
    for (int idx = tid; idx < 8 * 32 * 8; idx += Q_THREADS) {
        // 8 consecutive lanes hold the 8 float4 of one (batch row, block)
        const int b = idx >> 8, r = idx & 255, jl = r >> 3, q4 = r & 7;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (b < B && jl < nbl) {
            const size_t off = (size_t)b * p.a.x_stride + (size_t)(jb + jl) * 32 + q4 * 4;
            if constexpr (PRO == Pro::Plain) {
                o = *reinterpret_cast<const float4*>(p.a.x + off);
            } else {
                float4 t = *reinterpret_cast<const float4*>(p.a.xin + off);
                if (p.a.yin) {
                    const float4 u = *reinterpret_cast<const float4*>(p.a.yin + off);
                    t.x = __fadd_rn(t.x, u.x); t.y = __fadd_rn(t.y, u.y); t.z = __fadd_rn(t.z, u.z); t.w = __fadd_rn(t.w, u.w);
                }
                const float qsum = fmaf(t.x, t.x, fmaf(t.y, t.y, fmaf(t.z, t.z, __fmul_rn(t.w, t.w))));
#pragma unroll
                for (int bb = 0; bb < B; ++bb)
                    if (bb == b) ss[bb] += qsum;
                const float4 g = *reinterpret_cast<const float4*>(p.a.gamma + (size_t)(jb + jl) * 32 + q4 * 4);
                o = make_float4(__fmul_rn(t.x, g.x), __fmul_rn(t.y, g.y), __fmul_rn(t.z, g.z), __fmul_rn(t.w, g.w));
            }
        }
        float bs = (o.x + o.y) + (o.z + o.w);
        bs += __shfl_xor_sync(0xffffffffu, bs, 1);
        bs += __shfl_xor_sync(0xffffffffu, bs, 2);
        bs += __shfl_xor_sync(0xffffffffu, bs, 4);
        float* dst = xs + (size_t)jl * QX + q4 * 4 * 8 + b;
        const int e0 = q4 * 4;
        dst[0] = __fmul_rn(o.x, exp2_i(kXExp - x_shift_dn<QT>(e0)));
        dst[8] = __fmul_rn(o.y, exp2_i(kXExp - x_shift_dn<QT>(e0 + 1)));
        dst[16] = __fmul_rn(o.z, exp2_i(kXExp - x_shift_dn<QT>(e0 + 2)));
        dst[24] = __fmul_rn(o.w, exp2_i(kXExp - x_shift_dn<QT>(e0 + 3)));
        if (q4 == 0) xs[(size_t)jl * QX + 256 + b] = __fmul_rn(bs, exp2_i(kXExp - 149));
    }
    if constexpr (PRO == Pro::AddNorm) {
        __shared__ float s_ss[Q_WARPS][B];
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const float t = warp_sum(ss[b]);
            if (lane == 0) s_ss[warp][b] = t;
        }
        __syncthreads();
        if (tid < B) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < Q_WARPS; ++w) t += s_ss[w][tid];
            p.ssq[((size_t)pp * p.nsteps + q) * B + tid] = t;
        }
    }
    __syncthreads();

    const float* xj = xs + (size_t)lane * QX;  // this lane's block
    const float offs = (QT == AT_GGML_Q4_0) ? -8.f : -128.f;
    for (int t = 0; t < nmine; ++t) {
        while (issued < t + Q_NST) issue_next();
        cp_wait<Q_NST - 1>();
        __syncwarp();
        const uint8_t* sp = ring_ptr + (t & (Q_NST - 1)) * SLOT;
        int ga, gb;
        unit_groups(t, &ga, &gb);
        float2 acc[8][BP];
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int k = 0; k < BP; ++k) acc[r][k] = f2(0.f, 0.f);
        float dsc[8];
        if (lane < nbl) {
            // row r: tile r / 4, row r % 4 of it
            const uint8_t* qlane = sp + 256 + lane * QB;
            const uint8_t* dlane = sp + lane * 2;
#pragma unroll
            for (int r = 0; r < 8; ++r)
                dsc[r] = __fmul_rn(fp16_ftz_fast(*reinterpret_cast<const uint16_t*>(
                                       dlane + (r >> 2) * TL::BYTES + (r & 3) * 64)),
                                   kDnUnscale);
            uint4 qv[8];  // Q4_0: a row's 16 quant bytes; Q8_0: 16 of its 32
#pragma unroll
            for (int kc = 0; kc < 8; ++kc) {
                if (kc == 0 || (QT == AT_GGML_Q8_0 && kc == 4)) {
#pragma unroll
                    for (int r = 0; r < 8; ++r)
                        qv[r] = *reinterpret_cast<const uint4*>(qlane + (r >> 2) * TL::BYTES + (r & 3) * 32 * QB +
                                                                (kc == 4 ? 16 : 0));
                }
                float2 xp[4][BP];
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const float4 x0 = *reinterpret_cast<const float4*>(xj + (4 * kc + kk) * 8);
                    xp[kk][0] = f2(x0.x, x0.y);
                    if constexpr (BP > 1) xp[kk][1] = f2(x0.z, x0.w);
                    if constexpr (BP > 2) {
                        const float4 x1 = *reinterpret_cast<const float4*>(xj + (4 * kc + kk) * 8 + 4);
                        xp[kk][2] = f2(x1.x, x1.y);
                        if constexpr (BP > 3) xp[kk][3] = f2(x1.z, x1.w);
                    }
                }
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const int word = (QT == AT_GGML_Q4_0) ? (kc >> 1) : (kc & 3);
                    const uint32_t w = word == 0 ? qv[r].x : word == 1 ? qv[r].y : word == 2 ? qv[r].z : qv[r].w;
                    float f[4];
                    q4_fields_dn<QT>(w, kc, f);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const float2 w2 = f2(f[kk], f[kk]);
#pragma unroll
                        for (int k = 0; k < BP; ++k) acc[r][k] = __ffma2_rn(w2, xp[kk][k], acc[r][k]);
                    }
                }
            }
        }
        // block results: d * (sum - offset * block sum of x), per matrix / group tile
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;
            if (lane < nbl) {
                const float4 sxa = *reinterpret_cast<const float4*>(xj + 256);
                const float4 sxb = *reinterpret_cast<const float4*>(xj + 260);
                const float sx[8] = {sxa.x, sxa.y, sxa.z, sxa.w, sxb.x, sxb.y, sxb.z, sxb.w};
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int b = 0; b < B; ++b) {
                        const float2 a2 = acc[4 * m + r][b >> 1];
                        v[r * nq_stride(B) + b] = __fmul_rn(dsc[4 * m + r], fmaf(offs, sx[b], (b & 1) ? a2.y : a2.x));
                    }
            }
            const float tot = lane_transpose_sum(v, lane);
            if constexpr (NM == 2) {
                p.part[((size_t)q * p.ngroups + ga) * 64 + 32 * m + lane] = tot;
            } else {
                const int g = m ? gb : ga;
                if (g >= 0) p.part[((size_t)q * p.ngroups + g) * 32 + lane] = tot;
            }
        }
        __syncwarp();  // every lane is done with this slot before it is refilled
    }
    cp_wait<0>();
}

// y from the steps' partials (step order), with the folded RMSNorm scale and
// the epilogue; CTA c also writes its slice of the normed residual stream.
template <int B, Pro PRO, Epi EPI>
__global__ void __launch_bounds__(256) gemv_nq_reduce_kernel(const NQParams p) {
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    __shared__ float s_inv[B];
    pdl_trigger();
    pdl_wait();
    const int d_model = p.nb * 32;
    if (threadIdx.x < B) {
        float inv = 1.f;
        if constexpr (PRO == Pro::AddNorm) {
            float t = 0.f;
            for (int q = 0; q < p.nsteps; ++q) t += p.ssq[(size_t)q * B + threadIdx.x];  // part 0's sums
            inv = rms_inv(t, d_model, p.a.eps);
        }
        s_inv[threadIdx.x] = inv;
    }
    __syncthreads();
    if constexpr (PRO == Pro::AddNorm) write_xout_slice<B, 256>(p.a, d_model, s_inv, blockIdx.x, gridDim.x);
    const int64_t total = (int64_t)p.rows * B;
    for (int64_t it = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; it < total; it += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(it / B), b = (int)(it - (it / B) * B);
        const int g = row >> 2, r = row & 3;
        float v[NM];
#pragma unroll
        for (int m = 0; m < NM; ++m) v[m] = 0.f;
        for (int q = 0; q < p.nsteps; ++q) {
            const float* src = p.part + ((size_t)q * p.ngroups + g) * (32 * NM);
#pragma unroll
            for (int m = 0; m < NM; ++m) v[m] += src[32 * m + r * nq_stride(B) + b];
        }
        const float inv = s_inv[b];
        p.a.y[(size_t)b * p.a.y_stride + row] = n_epilogue<EPI>(__fmul_rn(v[0], inv), __fmul_rn(v[NM - 1], inv));
    }
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
constexpr int TR = 8;  // per-thread cp.async ring depth of the batch <= 2 T kernel (steps)

struct TParams {
    const uint8_t* tiles;
    int64_t tile_bytes;
    int ring_off;      // byte offset of the weight ring in dynamic shared memory
    int E;             // input rows
    int ngroups;       // 32-row groups
    int n_bc;          // block columns (outputs / 32)
    int S;             // CTAs splitting the rows of a block column
    int e_per_split;   // rows per CTA (multiple of the CTA row step)
    int cluster;       // S > 1 launched as clusters of S CTAs: partials combined through DSMEM
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

// Stores output column j of batch row b. Every lane of the warp calls it (the
// RoPE pair partner of column j is column j ^ 1, held by the neighbouring lane).
// RoPE coefficients (cos, sin) of output column j of batch row b (QKV epilogue;
// columns past q and k get (1, 0)). Positions and tables are not written by
// the step's kernels, so this may run before pdl_wait().
__device__ __forceinline__ float2 rope_coef(const GemvArgs& a, int j, int b) {
    const int hd = a.head_dim, nq = a.n_q_cols, nkv = a.n_kv_cols;
    if (j >= nq + nkv) return f2(1.f, 0.f);
    const int64_t pos = a.pos[b];
    const int dd = (j < nq ? j : j - nq) % hd;
    return f2(a.rope_cos[pos * hd + dd], a.rope_sin[pos * hd + dd]);
}

template <Epi EPI>
__device__ __forceinline__ void t_store(const GemvArgs& a, float val, int j, int b, float2 cs_sn) {
    if constexpr (EPI == Epi::Plain) {
        a.y[(size_t)b * a.y_stride + j] = val;
    } else {
        // QKV epilogue: RoPE on q and k (core/Kernels.java:296-309 vector path:
        // a' = fma(a, c, b * -s), b' = fma(b, c, a * s)), then the KV-cache
        // append of k and v (inference/KVCache.java:79-95).
        const int hd = a.head_dim;
        const int nq = a.n_q_cols, nkv = a.n_kv_cols;
        const int64_t pos = a.pos[b];
        const float partner = __shfl_xor_sync(0xffffffffu, val, 1);
        float out = val;
        if (j < nq + nkv) {
            const int dd = (j < nq ? j : j - nq) % hd;
            const float cs = cs_sn.x, sn = cs_sn.y;
            if ((dd & 1) == 0) out = fmaf(val, cs, __fmul_rn(partner, -sn));
            else out = fmaf(val, cs, __fmul_rn(partner, sn));
        }
        if (j < nq) {
            a.y[(size_t)b * a.y_stride + j] = out;
        } else {
            const bool is_k = j < nq + nkv;
            const int jj = is_k ? j - nq : j - nq - nkv;
            const int kvh = jj / hd, dd = jj - kvh * hd;
            const size_t e = (size_t)b * a.kv_slot_stride + ((size_t)kvh * a.ctx_len + pos) * hd + dd;
            if (a.kq) {  // the warp holds one 32-column block (the k / v boundary is block aligned)
                kv_store_q8(is_k ? a.kq : a.vq, is_k ? a.ksc : a.vsc, e, out);
            } else {
                float* cache = is_k ? a.kcache : a.vcache;
                cache[e] = out;
            }
        }
    }
}

// The common end of the T kernels: the RMSNorm scale of a folded AddNorm
// (per-warp sums of squares in s_red), the normed residual slice, the CTA's
// partial per (batch row, column) from red[warp][b][col], the combine over the
// CTAs splitting the rows (cluster shared memory or scratch and counters),
// and the epilogue store.
template <int B, Epi EPI>
__device__ __forceinline__ void t_tail(const TParams& p, float (*red)[B][32], const float* s_red, float* s_inv,
                                       bool fold, int* s_last, const XoutStash* s_xo, int c, int s) {
    if (fold && threadIdx.x < B) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) t += s_red[w * B + threadIdx.x];
        s_inv[threadIdx.x] = rms_inv(t, p.E, p.a.eps);
    }
    __syncthreads();
    if (fold) write_xout_stashed<B, THREADS>(p.a, p.E, s_inv, blockIdx.x, gridDim.x, s_xo);

    // CTA partial for (block column c, rows [e_lo, e_hi)): thread (b = warp, col = lane)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float val = 0.f;
    const int b_me = warp, cl = lane;
    if (b_me < B) {
#pragma unroll
        for (int w = 0; w < 8; ++w) val += red[w][b_me][cl];
    }
    if (p.S > 1 && p.cluster) {
        // The S CTAs of block column c form one cluster (rank = s): rank 0
        // sums the partials in split order from its peers' shared memory.
        namespace cg = cooperative_groups;
        cg::cluster_group cluster = cg::this_cluster();
        if (b_me < B) red[0][b_me][cl] = val;  // each (b_me, cl) slot is read above only by this thread
        cluster.sync();
        if (s == 0 && b_me < B) {
            val = 0.f;
            for (int k = 0; k < p.S; ++k) val += cluster.map_shared_rank(&red[0][0][0], k)[b_me * 32 + cl];
        }
        cluster.sync();  // peers keep their shared memory until rank 0 has read it
        if (s != 0) return;
    } else if (p.S > 1) {
        if (b_me < B) p.a.scratch[(((size_t)c * p.S + s) * B + b_me) * 32 + cl] = val;
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const unsigned prev = atomicAdd(&p.a.counters[c], 1u);
            *s_last = (prev == (unsigned)(p.S - 1));
        }
        __syncthreads();
        if (!*s_last) return;
        __threadfence();
        if (b_me < B) {
            val = 0.f;
            for (int k = 0; k < p.S; ++k)
                val += __ldcg(&p.a.scratch[(((size_t)c * p.S + k) * B + b_me) * 32 + cl]);
        }
        if (tid == 0) p.a.counters[c] = 0u;
    }
    if (b_me >= B) return;
    if (fold) val = __fmul_rn(val, s_inv[b_me]);

    const int j = c * 32 + cl;
    t_store<EPI>(p.a, val, j, b_me, EPI == Epi::QkvRope ? rope_coef(p.a, j, b_me) : f2(1.f, 0.f));
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
    __shared__ XoutStash s_xo;  // AddNorm fold: this CTA's slice of the normed x

    pdl_trigger();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x / p.S, s = blockIdx.x - (blockIdx.x / p.S) * p.S;
    const int e_lo = s * p.e_per_split;
    const int e_hi = min(p.E, e_lo + p.e_per_split);
    const int ne = e_hi - e_lo;
    const int quarter = (LPB == 1) ? 0 : (lane & (LPB - 1));
    const int row_in_warp = lane / LPB;
    const uint8_t* col = p.tiles + (size_t)c * p.ngroups * p.tile_bytes;

    // Batch <= 2 (a lane owns whole rows): every thread copies its own rows'
    // quant bytes and scale word into a per-thread cp.async ring, TR steps
    // deep; larger batches keep U steps in registers. Weights are never
    // written by earlier kernels, so the first steps start before the wait.
    constexpr int NVQ = QTraits<QT>::NV;
    uint4* ringq = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(xs) + p.ring_off);  // [TR][NVQ][THREADS]
    uint32_t* rings = reinterpret_cast<uint32_t*>(ringq + TR * NVQ * THREADS);              // [TR][THREADS]
    int t_issued = 0;
    auto t_issue = [&]() {
        if constexpr (CPL == 32) {
            const int i = t_issued * C::STEP + warp * C::ROWS_PER_WARP + row_in_warp;
            if (i < ne) {
                const int e = e_lo + i;
                const uint8_t* tile = col + (int64_t)(e >> 5) * p.tile_bytes;
                const int l = e & 31, k = t_issued & (TR - 1);
#pragma unroll
                for (int v = 0; v < NVQ; ++v)
                    cp_async16((uint32_t)__cvta_generic_to_shared(ringq + (k * NVQ + v) * THREADS + tid),
                               tile + 64 + l * QTraits<QT>::QB + 16 * v);
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                                 (uint32_t)__cvta_generic_to_shared(rings + k * THREADS + tid)),
                             "l"(tile + 4 * (l >> 1))
                             : "memory");
            }
            cp_commit();
            ++t_issued;
        }
    };
    uint4 q[U][2];
    float dsc[U];
    if constexpr (CPL == 32) {
#pragma unroll
        for (int k = 0; k < TR; ++k) t_issue();
    } else {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = u * C::STEP + warp * C::ROWS_PER_WARP + row_in_warp;
            if (i < ne) t_load<QT, CPL>(q[u], dsc[u], col, p.tile_bytes, e_lo + i, quarter);
        }
    }
    pdl_wait();

    // AddNorm with 16-byte rows folds the RMSNorm: one pass over the full
    // rows sums the squares of t = xin + yin and stages t * gamma for this
    // CTA's rows; 1/rms multiplies the finished column sums (every CTA sums
    // in the same order, so all get the same scale), and each CTA writes its
    // slice of the normed residual stream at the end.
    const bool aligned = (p.a.x_stride & 3) == 0 && (ne & 3) == 0 && (p.E & 3) == 0;
    const bool fold = PRO == Pro::AddNorm && aligned;
    int st_i0 = 0, st_len = 0;
    xout_slice(p.E, blockIdx.x, gridDim.x, &st_i0, &st_len);
    if (fold) {
        const int n4 = p.E >> 2;
        float ss[B];
#pragma unroll
        for (int b = 0; b < B; ++b) ss[b] = 0.f;
        for (int base = 0; base < B * n4; base += THREADS * 4) {
            // x, y and gamma in one round of loads (gamma of rows this CTA
            // stages or writes back)
            float4 v[4], gv[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int idx = base + k * THREADS + tid;
                if (idx < B * n4) {
                    const int bb = idx / n4, i4 = idx - bb * n4;
                    const size_t off = (size_t)bb * p.a.x_stride + 4 * (size_t)i4;
                    float4 t = *reinterpret_cast<const float4*>(p.a.xin + off);
                    if (p.a.yin) {
                        const float4 u = *reinterpret_cast<const float4*>(p.a.yin + off);
                        t.x = __fadd_rn(t.x, u.x); t.y = __fadd_rn(t.y, u.y);
                        t.z = __fadd_rn(t.z, u.z); t.w = __fadd_rn(t.w, u.w);
                    }
                    v[k] = t;
                    const int e = 4 * i4;
                    const bool need = (e >= e_lo && e < e_hi) || (i4 >= st_i0 && i4 < st_i0 + st_len);
                    if (need) gv[k] = *reinterpret_cast<const float4*>(p.a.gamma + e);
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int idx = base + k * THREADS + tid;
                if (idx < B * n4) {
                    const int bb = idx / n4, e = 4 * (idx - bb * n4);
                    const float4 o = v[k];
                    const float q = fmaf(o.x, o.x, fmaf(o.y, o.y, fmaf(o.z, o.z, __fmul_rn(o.w, o.w))));
#pragma unroll
                    for (int b = 0; b < B; ++b)
                        if (b == bb) ss[b] += q;
                    if (B * st_len <= kXoutStash && (e >> 2) >= st_i0 && (e >> 2) < st_i0 + st_len)
                        stash_put<B, THREADS>(&s_xo, st_i0, st_len, bb, e >> 2, o, gv[k]);
                    if (e >= e_lo && e < e_hi) {
                        const float4 g = gv[k];
                        *reinterpret_cast<float4*>(xs + bb * p.e_per_split + (e - e_lo)) =
                            make_float4(__fmul_rn(o.x, g.x), __fmul_rn(o.y, g.y), __fmul_rn(o.z, g.z),
                                        __fmul_rn(o.w, g.w));
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const float t = warp_sum(ss[b]);
            if (lane == 0) s_red[warp * B + b] = t;
        }
    } else if constexpr (PRO == Pro::AddNorm) {
        block_rms_inv<B>(p.a.xin, p.a.yin, p.a.x_stride, p.E, p.a.eps, s_red, s_inv);
        if (blockIdx.x == 0) write_xout<B>(p.a, p.E, s_inv);
    }
    if (fold) {
        // staged above
    } else if (!aligned) {
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
    float dsum[B];  // CPL == 32: this lane's sum of d * x (offset correction)
#pragma unroll
    for (int b = 0; b < B; ++b) {
        dsum[b] = 0.f;
#pragma unroll
        for (int k = 0; k < NPAIR; ++k) acc[b][k] = f2(0.f, 0.f);
    }

    if constexpr (CPL == 32) {
        const int n_u = (ne + C::STEP - 1) / C::STEP;
        for (int u = 0; u < n_u; ++u) {
            cp_wait<TR - 1>();  // this thread's copies of step u have landed (it reads only its own)
            const int i = u * C::STEP + warp * C::ROWS_PER_WARP + row_in_warp;
            if (i < ne) {
                const int k = u & (TR - 1);
                uint4 qq[2];
#pragma unroll
                for (int v = 0; v < NVQ; ++v) qq[v] = ringq[(k * NVQ + v) * THREADS + tid];
                const uint32_t sw = rings[k * THREADS + tid];
                const float d = fp16_ftz_fast(((e_lo + i) & 1) ? (sw >> 16) : (sw & 0xFFFFu));
                float2 wv[NPAIR];
                t_decode_dn<QT>(qq, wv);
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float sv = __fmul_rn(d, xs[b * p.e_per_split + i]);
                    dsum[b] += sv;
                    const float svs = __fmul_rn(sv, exp2_i(kXExp));
                    const float2 s2 = f2(svs, svs);
#pragma unroll
                    for (int kk = 0; kk < NPAIR; ++kk) acc[b][kk] = __ffma2_rn(wv[kk], s2, acc[b][kk]);
                }
            }
            t_issue();  // refills slot u % TR with step u + TR
        }
        cp_wait<0>();
    } else {
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
    }

    // Butterfly reduce-scatter across the lanes sharing a block column.
#pragma unroll
    for (int b = 0; b < B; ++b) {
        float v[CPL];
        if constexpr (CPL == 32) {
            // back from the subnormal-scaled sums of t_decode_dn
            const float corr = __fmul_rn(QT == AT_GGML_Q4_0 ? -8.f : -128.f, dsum[b]);
#pragma unroll
            for (int k = 0; k < NPAIR; ++k) {
                v[2 * k] = fmaf(acc[b][k].x, exp2_i(149 - kXExp - x_shift_dn<QT>(2 * k)), corr);
                v[2 * k + 1] = fmaf(acc[b][k].y, exp2_i(149 - kXExp - x_shift_dn<QT>(2 * k + 1)), corr);
            }
        } else {
#pragma unroll
            for (int k = 0; k < NPAIR; ++k) {
                v[2 * k] = acc[b][k].x;
                v[2 * k + 1] = acc[b][k].y;
            }
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
    t_tail<B, EPI>(p, red, s_red, s_inv, fold, &s_last, &s_xo, c, s);
}

// ---------------------------------------------------------------------------
// Orientation T, batch 3..8
// ---------------------------------------------------------------------------
// CTA (block column c, rows [e_lo, e_hi)) stages x of its rows as [row][8]
// (batch rows b < B, times 2^kXExp; padding zero) and its 8 warps stream the
// column's 32-row tiles round robin through per-warp cp.async rings of whole
// tiles (576 or 1088 contiguous bytes, TB_NST deep). Lane (rs = lane / 4,
// quarter = lane % 4) takes rows rs, rs + 8, rs + 16, rs + 24 of a tile and
// columns 8 quarter .. 8 quarter + 7: each row's 8 weights are decoded once in
// the subnormal-scaled form (one mask per weight) and applied to all B rows of
// x by FFMA2 with d * x broadcast into a pair, so the decode is shared by the
// batch and every staged x value read serves 8 columns. The offset (8 or
// 128) times the lane's sum of d * x and the per-column power of two are
// applied once per column; the 8 lanes sharing a quarter combine by a
// butterfly reduce-scatter, the warps and the row splits as in the batch <= 2
// kernel (t_tail).
constexpr int TB_NST = 4;

template <int QT>
__device__ __forceinline__ void tq_decode_dn(const uint8_t* qp, float2* wv) {
    if constexpr (QT == AT_GGML_Q4_0) {
        const uint32_t w = *reinterpret_cast<const uint32_t*>(qp), t = w >> 24;  // columns 0..7 of the quarter
        wv[0] = f2(bits_f(w & 0xFu), bits_f(w & 0xF0u));
        wv[1] = f2(bits_f(w & 0xF00u), bits_f(w & 0xF000u));
        wv[2] = f2(bits_f(w & 0xF0000u), bits_f(w & 0xF00000u));
        wv[3] = f2(bits_f(t & 0xFu), bits_f(t & 0xF0u));
    } else {
        const uint2 u = *reinterpret_cast<const uint2*>(qp);
        wv[0] = f2(bits_f((u.x ^ 0x80u) & 0xFFu), bits_f((u.x ^ 0x8000u) & 0xFF00u));
        wv[1] = f2(bits_f((u.x ^ 0x800000u) & 0xFF0000u), bits_f((u.x >> 24) ^ 0x80u));
        wv[2] = f2(bits_f((u.y ^ 0x80u) & 0xFFu), bits_f((u.y ^ 0x8000u) & 0xFF00u));
        wv[3] = f2(bits_f((u.y ^ 0x800000u) & 0xFF0000u), bits_f((u.y >> 24) ^ 0x80u));
    }
}

// tq_decode_dn from the quarter's bytes already in registers (Q4_0: w.x).
template <int QT>
__device__ __forceinline__ void tq_decode_dn_w(uint2 w2, float2* wv) {
    if constexpr (QT == AT_GGML_Q4_0) {
        const uint32_t w = w2.x, t = w >> 24;
        wv[0] = f2(bits_f(w & 0xFu), bits_f(w & 0xF0u));
        wv[1] = f2(bits_f(w & 0xF00u), bits_f(w & 0xF000u));
        wv[2] = f2(bits_f(w & 0xF0000u), bits_f(w & 0xF00000u));
        wv[3] = f2(bits_f(t & 0xFu), bits_f(t & 0xF0u));
    } else {
        const uint2 u = w2;
        wv[0] = f2(bits_f((u.x ^ 0x80u) & 0xFFu), bits_f((u.x ^ 0x8000u) & 0xFF00u));
        wv[1] = f2(bits_f((u.x ^ 0x800000u) & 0xFF0000u), bits_f((u.x >> 24) ^ 0x80u));
        wv[2] = f2(bits_f((u.y ^ 0x80u) & 0xFFu), bits_f((u.y ^ 0x8000u) & 0xFF00u));
        wv[3] = f2(bits_f((u.y ^ 0x800000u) & 0xFF0000u), bits_f((u.y >> 24) ^ 0x80u));
    }
}

template <int QT, int B, Pro PRO, Epi EPI>
__global__ void __launch_bounds__(THREADS, 2) gemv_tb_kernel(const TParams p) {
    constexpr int QB = QTraits<QT>::QB;
    constexpr int TBYTES = 64 + 32 * QB;
    constexpr int TCH = TBYTES / 16;
    constexpr bool fold = PRO == Pro::AddNorm;
    static_assert(B >= 3 && B <= 8, "batch 3..8");
    extern __shared__ __align__(16) float xs[];  // [rows of the split, padded to tiles][8], then the rings
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
    const int nt = (ne + 31) >> 5;
    const int nmine = (nt - warp + 7) >> 3;  // this warp's tiles: warp + 8 i
    const uint8_t* col = p.tiles + ((size_t)c * p.ngroups + (e_lo >> 5)) * TBYTES;
    const uint8_t* ring_ptr = reinterpret_cast<const uint8_t*>(xs) + p.ring_off + warp * TB_NST * TBYTES;
    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(ring_ptr);
    int issued = 0;
    auto issue_next = [&]() {
        if (issued < nmine)
            copy_unit<TCH>(ring + (issued & (TB_NST - 1)) * TBYTES, col + (size_t)(warp + 8 * issued) * TBYTES, lane);
        cp_commit();
        ++issued;
    };
    // weights are never written by earlier kernels: the first tiles start before the wait
    for (int k = 0; k < TB_NST - 1; ++k) issue_next();
    pdl_wait();

    // The split's rows of x (Plain) or of t * gamma, t = xin + yin (AddNorm:
    // the RMSNorm is folded, 1/rms multiplies the finished column sums; this
    // CTA's sums of t^2 over its rows are combined over the splits at the
    // end), times 2^kXExp; the padding (rows past the split, b >= B) is zero.
    const float xsc = exp2_i(kXExp);
    if constexpr (B < 8) {
        for (int idx = tid; idx < ne * (8 - B); idx += THREADS) xs[(idx / (8 - B)) * 8 + B + idx % (8 - B)] = 0.f;
    }
    for (int idx = tid; idx < (nt * 32 - ne) * 8; idx += THREADS) xs[(size_t)ne * 8 + idx] = 0.f;
    {
        const int n4 = ne >> 2;
        float ss[B];
#pragma unroll
        for (int b = 0; b < B; ++b) ss[b] = 0.f;
        // item idx = (4-row group i4, batch row bb), bb fastest: B consecutive
        // threads fill the 8-float rows of one group
        for (int base = 0; base < B * n4; base += THREADS * 4) {
            float4 v[4], gv[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int idx = base + k * THREADS + tid;
                if (idx < B * n4) {
                    const int bb = idx % B, e = e_lo + 4 * (idx / B);
                    const size_t off = (size_t)bb * p.a.x_stride + e;
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
                        gv[k] = *reinterpret_cast<const float4*>(p.a.gamma + e);
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int idx = base + k * THREADS + tid;
                if (idx < B * n4) {
                    const int bb = idx % B, i = 4 * (idx / B);
                    float4 o = v[k];
                    if constexpr (fold) {
                        const float q = fmaf(o.x, o.x, fmaf(o.y, o.y, fmaf(o.z, o.z, __fmul_rn(o.w, o.w))));
#pragma unroll
                        for (int b = 0; b < B; ++b)
                            if (b == bb) ss[b] += q;
                        const float4 g = gv[k];
                        o = make_float4(__fmul_rn(o.x, g.x), __fmul_rn(o.y, g.y), __fmul_rn(o.z, g.z),
                                        __fmul_rn(o.w, g.w));
                    }
                    float* dst = xs + (size_t)i * 8 + bb;
                    dst[0] = __fmul_rn(o.x, xsc);
                    dst[8] = __fmul_rn(o.y, xsc);
                    dst[16] = __fmul_rn(o.z, xsc);
                    dst[24] = __fmul_rn(o.w, xsc);
                }
            }
        }
        if constexpr (fold) {
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float t = warp_sum(ss[b]);
                if (lane == 0) s_red[warp * B + b] = t;
            }
        }
    }
    __syncthreads();

    const int qtr = lane & 3, rs = lane >> 2;
    // d * x of a tile's rows, computed once per row (lane l: row l) into this
    // warp's [32 rows][8] buffer; every quarter-lane of a row reads it
    // d * x of a tile's rows, computed once per row (lane l: row l) into this
    // warp's [32 rows][8] buffer; every quarter-lane of a row reads it
    float* svw = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + p.ring_off + 8 * TB_NST * TBYTES) +
                 warp * 32 * 8;
    float2 acc[B][4];
    float dsum[B];  // sum of d * x * 2^kXExp over row `lane` of this warp's tiles (offset correction)
#pragma unroll
    for (int b = 0; b < B; ++b) {
        dsum[b] = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[b][k] = f2(0.f, 0.f);
    }
    for (int t = 0; t < nmine; ++t) {
        issue_next();  // refills the slot read in step t - 1 with tile t + TB_NST - 1
        cp_wait<TB_NST - 1>();
        __syncwarp();  // every lane's pieces of tile t have landed
        const uint8_t* sp = ring_ptr + (t & (TB_NST - 1)) * TBYTES;
        const int row0 = (warp + 8 * t) * 32;
        {
            const int ir = row0 + lane;
            float sv[8];
            if (ir < ne) {
                const float d = fp16_ftz_fast(*reinterpret_cast<const uint16_t*>(sp + 2 * lane));
                const float4 xa = *reinterpret_cast<const float4*>(xs + (size_t)ir * 8);
                const float4 xb = *reinterpret_cast<const float4*>(xs + (size_t)ir * 8 + 4);
                sv[0] = __fmul_rn(d, xa.x); sv[1] = __fmul_rn(d, xa.y); sv[2] = __fmul_rn(d, xa.z); sv[3] = __fmul_rn(d, xa.w);
                sv[4] = __fmul_rn(d, xb.x); sv[5] = __fmul_rn(d, xb.y); sv[6] = __fmul_rn(d, xb.z); sv[7] = __fmul_rn(d, xb.w);
            } else {
#pragma unroll
                for (int b = 0; b < 8; ++b) sv[b] = 0.f;
            }
#pragma unroll
            for (int b = 0; b < B; ++b) dsum[b] += sv[b];
            *reinterpret_cast<float4*>(svw + lane * 8) = make_float4(sv[0], sv[1], sv[2], sv[3]);
            *reinterpret_cast<float4*>(svw + lane * 8 + 4) = make_float4(sv[4], sv[5], sv[6], sv[7]);
        }
        __syncwarp();  // the tile's d * x are visible to the warp
        // the lane's 4 rows: quant words and d * x loaded together, then the products
        uint2 qw[4];
        float4 sa[4], sb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int l = rs + 8 * i;
            const uint8_t* qp = sp + 64 + l * QB + qtr * (QB / 4);
            if constexpr (QT == AT_GGML_Q4_0) qw[i] = make_uint2(*reinterpret_cast<const uint32_t*>(qp), 0u);
            else qw[i] = *reinterpret_cast<const uint2*>(qp);
            sa[i] = *reinterpret_cast<const float4*>(svw + l * 8);
            sb[i] = *reinterpret_cast<const float4*>(svw + l * 8 + 4);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            // rows past the split have d * x = 0: their products add nothing
            float2 wv[4];
            tq_decode_dn_w<QT>(qw[i], wv);
            const float svr[8] = {sa[i].x, sa[i].y, sa[i].z, sa[i].w, sb[i].x, sb[i].y, sb[i].z, sb[i].w};
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float2 s2 = f2(svr[b], svr[b]);
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[b][k] = __ffma2_rn(wv[k], s2, acc[b][k]);
            }
        }
        __syncwarp();  // every lane is done with this slot (and the d * x buffer) before they are refilled
    }
    cp_wait<0>();

    const float offs = (QT == AT_GGML_Q4_0) ? -8.f : -128.f;
#pragma unroll
    for (int b = 0; b < B; ++b) {
        // the offset times the sum of d * x over every row of this warp's tiles (all lanes)
        const float corr = __fmul_rn(offs, __fmul_rn(warp_sum(dsum[b]), exp2_i(-kXExp)));
        float v[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            v[2 * k] = __fmul_rn(acc[b][k].x, exp2_i(149 - kXExp - x_shift_dn<QT>(2 * k)));
            v[2 * k + 1] = __fmul_rn(acc[b][k].y, exp2_i(149 - kXExp - x_shift_dn<QT>(2 * k + 1)));
        }
        // reduce-scatter over the lanes of a quarter (lane bits 4, 8, 16): lane
        // (rs, quarter) ends with column 8 quarter + rs
        int n = 8;
#pragma unroll
        for (int bit = 16; bit >= 4; bit >>= 1) {
            const bool upper = (lane & bit) != 0;
            n >>= 1;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                if (t < n) {
                    const float send = upper ? v[t] : v[t + n];
                    const float keep = upper ? v[t + n] : v[t];
                    v[t] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
                }
            }
        }
        red[warp][b][8 * qtr + rs] = v[0] + corr;
    }
    __syncthreads();

    // CTA partial for (block column c, rows [e_lo, e_hi)): thread (b = warp,
    // col = lane), plus (lane 0) the CTA's sum of t^2 of batch row b
    const int b_me = warp, cl = lane;
    float val = 0.f, ssq = 0.f;
    if (b_me < B) {
#pragma unroll
        for (int w = 0; w < 8; ++w) val += red[w][b_me][cl];
        if (fold) {
#pragma unroll
            for (int w = 0; w < 8; ++w) ssq += s_red[w * B + b_me];
        }
    }
    if (p.S > 1) {
        // splits in scratch [c][S][B][33] (32 column values, then the sum of
        // squares); the last CTA to arrive sums them in split order
        float* part = p.a.scratch + (size_t)c * p.S * B * 33;
        if (b_me < B) {
            part[((size_t)s * B + b_me) * 33 + cl] = val;
            if (cl == 0) part[((size_t)s * B + b_me) * 33 + 32] = ssq;
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(&p.a.counters[c], 1u) == (unsigned)(p.S - 1);
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (b_me < B) {
            val = 0.f;
            ssq = 0.f;
            for (int k = 0; k < p.S; ++k) {
                val += __ldcg(&part[((size_t)k * B + b_me) * 33 + cl]);
                ssq += __ldcg(&part[((size_t)k * B + b_me) * 33 + 32]);
            }
        }
        if (tid == 0) p.a.counters[c] = 0u;
    }
    if (fold) {
        if (b_me < B && cl == 0) s_inv[b_me] = rms_inv(ssq, p.E, p.a.eps);
        __syncthreads();
        // the normed residual stream: rows [c E / n_bc, (c + 1) E / n_bc) of every batch row
        const int n4 = p.E >> 2;
        const int i0 = (int)((int64_t)c * n4 / p.n_bc), i1 = (int)((int64_t)(c + 1) * n4 / p.n_bc);
        for (int idx = tid; idx < B * (i1 - i0); idx += THREADS) {
            const int bb = idx / (i1 - i0), i4 = i0 + idx - bb * (i1 - i0);
            const size_t off = (size_t)bb * p.a.x_stride + (size_t)i4 * 4;
            float4 t = *reinterpret_cast<const float4*>(p.a.xin + off);
            if (p.a.yin) {
                const float4 u = *reinterpret_cast<const float4*>(p.a.yin + off);
                t.x = __fadd_rn(t.x, u.x); t.y = __fadd_rn(t.y, u.y); t.z = __fadd_rn(t.z, u.z); t.w = __fadd_rn(t.w, u.w);
            }
            const float4 g = *reinterpret_cast<const float4*>(p.a.gamma + (size_t)i4 * 4);
            const float inv = s_inv[bb];
            *reinterpret_cast<float4*>(p.a.xout + off) = make_float4(
                norm_apply(t.x, inv, g.x), norm_apply(t.y, inv, g.y), norm_apply(t.z, inv, g.z), norm_apply(t.w, inv, g.w));
        }
        if (b_me < B) val = __fmul_rn(val, s_inv[b_me]);
    }
    if (b_me >= B) return;
    const int j = c * 32 + cl;
    t_store<EPI>(p.a, val, j, b_me, EPI == Epi::QkvRope ? rope_coef(p.a, j, b_me) : f2(1.f, 0.f));
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
void launch(const void* fn, int grid, int smem, cudaStream_t s, bool pdl, const P& params, int threads = THREADS,
            int cluster = 1) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (cluster > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = (unsigned)cluster;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    void* args[] = {const_cast<P*>(&params)};
    AT_CUDA(cudaLaunchKernelExC(&cfg, fn, args));
}

// Stream plan: one CTA per SM (never more CTAs than units), the CTA unit
// map, and the number of shared-memory partial slots per warp (segments one
// warp's units can touch).
struct StreamPlan {
    int grid = 1, slots = 1, nst = 0;  // nst = ring depth, 0 = the stream kernel does not fit
    bool aligned = false;              // CTA ranges are whole segments (nothing shared between CTAs)
    int xbytes = 0, red_bytes = 0, smem = 0;
    StreamMap map{};
};
constexpr int kStreamSmem = 220 * 1024;  // dynamic shared memory budget of the stream kernels
// Segment-aligned CTA ranges are taken when the busiest CTA streams at most
// kAlignSlack x the mean: they need no cross-CTA combine at the end.
constexpr double kAlignSlack = 1.08;
// Ring depth (units per warp in flight). Two 2304-byte units per warp keep
// 74 KB per SM in flight; deeper rings measured slower in the decode step.
constexpr int kMaxNst = 2;

StreamPlan stream_plan(int64_t U, int64_t seg_len, int num_sms, int xbytes, int vals_per_seg, int slot_bytes,
                       int max_nst, double slack) {
    StreamPlan sp;
    AT_REQUIRE(U < (int64_t(1) << 27), AT_ERR_INVALID_ARG, "matrix too large for the stream GEMV");
    const int sms = std::min(num_sms, kMaxStreamCtas);
    const int64_t nseg = U / seg_len;
    // whole segments per CTA when the busiest CTA streams at most kAlignSlack x the mean
    const int64_t ga = std::min<int64_t>(sms, nseg);
    const double mean = (double)U / (double)std::max<int64_t>(1, std::min<int64_t>(sms, U));
    sp.aligned = ga >= 1 && (double)((nseg + ga - 1) / ga * seg_len) <= slack * mean;
    sp.grid = sp.aligned ? (int)ga : (int)std::max<int64_t>(1, std::min<int64_t>(sms, U));
    sp.map.len = (int)seg_len;
    for (int c = 0; c <= sp.grid; ++c)
        sp.map.start[c] = sp.aligned ? (int)((int64_t)c * nseg / sp.grid * seg_len) : (int)((int64_t)c * U / sp.grid);
    int64_t per_cta = 0;
    for (int c = 0; c < sp.grid; ++c) per_cta = std::max<int64_t>(per_cta, sp.map.start[c + 1] - sp.map.start[c]);
    const int64_t per_warp = (per_cta + S_WARPS - 1) / S_WARPS;
    sp.slots = (int)((per_warp + seg_len - 1) / seg_len + 1);
    sp.xbytes = (xbytes + 15) / 16 * 16;
    sp.red_bytes = (S_WARPS * sp.slots * vals_per_seg * 4 + 15) / 16 * 16;
    for (int nst = max_nst; nst >= 2; nst /= 2) {
        const int smem = sp.xbytes + sp.red_bytes + S_WARPS * nst * slot_bytes;
        if (smem <= kStreamSmem) {
            sp.nst = nst;
            sp.smem = smem;
            break;
        }
    }
    return sp;
}

template <int QT, int B, Epi EPI>
StreamPlan n_stream_plan(const at_qmat* m, int num_sms) {
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    const int nb = (int)(m->cols / QK);
    return stream_plan(m->ngroups * m->nsteps, m->nsteps, num_sms, B * nb * XPAD * 4, NM * 4 * B,
                       NM * NTile<QT>::BYTES, kMaxNst, kAlignSlack);
}

template <int QT, int B, Pro PRO, Epi EPI, int NST>
void run_ns(const at_qmat* m, const GemvArgs& a, const StreamPlan& sp, cudaStream_t s, bool pdl) {
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    NSParams p{};
    p.tiles[0] = m->tiles;
    p.tiles[1] = (NM == 2) ? a.m2->tiles : m->tiles;
    p.rows = (int)m->rows;
    p.nb = (int)(m->cols / QK);
    p.nsteps = (int)m->nsteps;
    p.slots = sp.slots;
    p.red_off = sp.xbytes;
    p.ring_off = sp.xbytes + sp.red_bytes;
    p.pre = pdl ? 2 : 1;
    p.map = sp.map;
    p.a = a;
    if (!sp.aligned && sp.grid > 1) AT_REQUIRE(a.scratch && a.counters, AT_ERR_STATE, "N GEMV needs split scratch");
    const void* fn = reinterpret_cast<const void*>(&gemv_ns_kernel<QT, B, PRO, EPI, NST>);
    ensure_smem(fn, sp.smem);
    launch(fn, sp.grid, sp.smem, s, pdl, p, S_THREADS);
}

// Layout of the batch 3..8 split-K scratch: partials then sums of squares.
struct NQLayout {
    int P = 1;
    size_t part_floats = 0, ssq_floats = 0;
};
NQLayout nq_layout(const at_qmat* m, int batch, int num_sms, int nm) {
    NQLayout l;
    const int64_t steps = m->nsteps;
    // CTAs per SM from the shared memory (x of one step + two-tile rings)
    const int smem = 32 * QX * 4 + Q_WARPS * Q_NST * 2 * (4 * 32 * (2 + quant_bytes(m->type)));
    const int occ = std::max(1, std::min(2, (227 * 1024) / (smem + 4 * 1024)));
    // whole waves: P parts x steps CTAs within the SM slots (a second, mostly
    // empty wave doubled the time of 4096 x 14336)
    l.P = (int)std::max<int64_t>(1, std::min<int64_t>(m->ngroups, (int64_t)occ * num_sms / steps));
    l.part_floats = (size_t)steps * m->ngroups * 32 * nm;  // one 32-value partial per matrix and group
    l.ssq_floats = (size_t)l.P * steps * batch;
    return l;
}

template <int QT, int B, Pro PRO, Epi EPI>
void run_nq(const at_qmat* m, const GemvArgs& a, int num_sms, cudaStream_t s, bool pdl) {
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    const NQLayout l = nq_layout(m, B, num_sms, NM);
    NQParams p{};
    p.tiles[0] = m->tiles;
    p.tiles[1] = (NM == 2) ? a.m2->tiles : m->tiles;
    p.rows = (int)m->rows;
    p.nb = (int)(m->cols / QK);
    p.ngroups = (int)m->ngroups;
    p.nsteps = (int)m->nsteps;
    p.P = l.P;
    p.part = a.scratch;
    p.ssq = a.scratch + l.part_floats;
    p.a = a;
    const int smem = 32 * QX * 4 + Q_WARPS * Q_NST * 2 * NTile<QT>::BYTES;
    const void* fn = reinterpret_cast<const void*>(&gemv_nq_kernel<QT, B, PRO, EPI>);
    ensure_smem(fn, smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.P, p.nsteps);
    cfg.blockDim = dim3(Q_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    void* args[] = {&p};
    AT_CUDA(cudaLaunchKernelExC(&cfg, fn, args));
    const int rgrid = (int)std::min<int64_t>(((int64_t)p.rows * B + 255) / 256, (int64_t)num_sms * 4);
    launch(reinterpret_cast<const void*>(&gemv_nq_reduce_kernel<B, PRO, EPI>), std::max(1, rgrid), 0, s, pdl, p, 256);
}

template <int QT, int B, Pro PRO, Epi EPI>
void run_n(const at_qmat* m, const GemvArgs& a, int num_sms, cudaStream_t s, bool pdl) {
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    const int nb = (int)(m->cols / QK);
    if constexpr (B <= 2) {
        const StreamPlan sp = n_stream_plan<QT, B, EPI>(m, num_sms);
        if (sp.nst == 4) { run_ns<QT, B, PRO, EPI, 4>(m, a, sp, s, pdl); return; }
        if (sp.nst == 2) { run_ns<QT, B, PRO, EPI, 2>(m, a, sp, s, pdl); return; }
    } else {
        if (a.scratch) { run_nq<QT, B, PRO, EPI>(m, a, num_sms, s, pdl); return; }
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

// Row splits of the batch 3..8 T kernel: the S that keeps the most SM slots
// busy over whole waves (ties: the fewer CTAs), each split at least one tile
// per warp. CTAs per SM from the shared memory (two at most: 256 threads of
// up to 128 registers).
constexpr int kTbMaxSplits = 16;
bool tb_plan(int qtype, int64_t E, int64_t n_bc, int num_sms, int* S_out, int* rows_out) {
    const int tbytes = 64 + 32 * quant_bytes(qtype);
    const int ring_bytes = 8 * TB_NST * tbytes + 8 * 32 * 8 * 4;  // rings + the warps' d * x buffers
    const int ntiles = (int)((E + 31) / 32);
    int best_S = 0, best_rows = 0;
    double best_eff = -1.0;
    for (int S = 1; S <= kTbMaxSplits; ++S) {
        const int tiles_per = (ntiles + S - 1) / S;
        if (S > 1 && tiles_per < 8) break;
        const int rows = tiles_per * 32;
        const int smem = rows * 32 + ring_bytes;
        if (smem > 200 * 1024) continue;
        const int occ = std::max(1, std::min(2, (227 * 1024) / (smem + 12 * 1024)));
        const int slots = num_sms * occ;
        const int Sx = (ntiles + tiles_per - 1) / tiles_per;
        const int64_t ctas = n_bc * Sx;
        const int64_t waves = (ctas + slots - 1) / slots;
        const double eff = (double)ctas / ((double)waves * slots);
        if (eff > best_eff + 0.02) {
            best_eff = eff;
            best_S = Sx;
            best_rows = rows;
        }
    }
    *S_out = best_S;
    *rows_out = best_rows;
    return best_S > 0;
}

// The batch 3..8 T kernel applies when the rows are 16-byte aligned.
bool tb_applies(const at_qmat* m, int x_stride) {
    return m->tile_bytes == 64 + 32 * quant_bytes(m->type) && (m->rows & 3) == 0 && (x_stride & 3) == 0;
}

template <int QT, int B, Pro PRO, Epi EPI>
bool run_tb(const at_qmat* m, const GemvArgs& a, int num_sms, cudaStream_t s, bool pdl) {
    constexpr int TBYTES = 64 + 32 * QTraits<QT>::QB;
    if (!tb_applies(m, a.x_stride)) return false;
    TParams p{};
    if (!tb_plan(m->type, m->rows, m->cols / QK, num_sms, &p.S, &p.e_per_split)) return false;
    p.tiles = m->tiles;
    p.tile_bytes = m->tile_bytes;
    p.E = (int)m->rows;
    p.ngroups = (int)m->ngroups;
    p.n_bc = (int)(m->cols / QK);
    p.cluster = 0;
    p.a = a;
    if (p.S > 1) AT_REQUIRE(a.scratch && a.counters, AT_ERR_STATE, "T GEMV needs split scratch");
    p.ring_off = p.e_per_split * 32;
    const int smem = p.ring_off + 8 * TB_NST * TBYTES + 8 * 32 * 8 * 4;  // + the warps' d * x buffers
    const void* fn = reinterpret_cast<const void*>(&gemv_tb_kernel<QT, B, PRO, EPI>);
    ensure_smem(fn, smem);
    launch(fn, p.n_bc * p.S, smem, s, pdl, p, THREADS, 1);
    return true;
}

template <int QT, int B, Pro PRO, Epi EPI>
void run_t(const at_qmat* m, const GemvArgs& a, int num_sms, cudaStream_t s, bool pdl) {
    if constexpr (B >= 3) {
        if (run_tb<QT, B, PRO, EPI>(m, a, num_sms, s, pdl)) return;
    }
    TParams p{};
    p.tiles = m->tiles;
    p.tile_bytes = m->tile_bytes;
    p.E = (int)m->rows;
    p.ngroups = (int)m->ngroups;
    p.n_bc = (int)(m->cols / QK);
    t_config(m, B, num_sms, &p.S, &p.e_per_split);
    p.a = a;
    // batch <= 2 splits of up to 8 CTAs combine through cluster shared memory;
    // others through the scratch partials and per-column counters (at batch 8
    // a split's short CTA would hold its SM at the cluster barrier while the
    // grid needs several waves: 4096 x 6144 took 80 instead of 57 us)
    p.cluster = (B <= 2 && p.S > 1 && p.S <= 8) ? 1 : 0;
    if (p.S > 1 && !p.cluster) AT_REQUIRE(a.scratch && a.counters, AT_ERR_STATE, "T GEMV needs split scratch");
    p.ring_off = (B * p.e_per_split * 4 + 15) / 16 * 16;
    const int ring_bytes = (TCfg<B>::CPL == 32) ? TR * THREADS * (16 * QTraits<QT>::NV + 4) : 0;
    const int smem = p.ring_off + ring_bytes;
    const void* fn = reinterpret_cast<const void*>(&gemv_t_kernel<QT, B, PRO, EPI>);
    ensure_smem(fn, smem);
    launch(fn, p.n_bc * p.S, smem, s, pdl, p, THREADS, p.cluster ? p.S : 1);
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
    // see run_t: only a real split (S > 1) touches scratch, and splits of up
    // to 8 CTAs at batch <= 2 combine in cluster shared memory instead
    const bool global_split = S > 1 && (S > 8 || batch > 2);
    *floats = global_split ? n_bc * S * batch * 32 : 0;
    *counters = global_split ? n_bc : 0;
    // batch 3..8 with row-aligned x runs the tile-ring kernel, whose split may differ
    int S2 = 0, per2 = 0;
    if (batch > 2 && tb_plan(m->type, m->rows, m->cols / QK, num_sms, &S2, &per2) && S2 > 1) {
        *floats = std::max(*floats, n_bc * S2 * batch * 33);
        *counters = n_bc;
    }
}

void gemv_n_scratch_need(const at_qmat* m, int batch, int num_sms, size_t* floats, size_t* counters) {
    if (m->type == AT_GGML_Q6_K) {  // one warp per row: no split
        *floats = 0;
        *counters = 0;
        return;
    }
    // upper bound over the epilogues (gate/up pairs carry two partials per row)
    if (batch > 2) {
        const NQLayout l = nq_layout(m, batch, num_sms, 2);
        *floats = l.part_floats + l.ssq_floats;
        *counters = 0;
        return;
    }
    const int64_t U = m->ngroups * m->nsteps;
    const size_t grid = (size_t)std::max<int64_t>(1, std::min<int64_t>(num_sms, U));
    *floats = (grid > 1) ? 2 * grid * 2 * 4 * batch : 0;
    *counters = (grid > 1) ? (size_t)m->ngroups : 0;
}

void launch_gemv_n(const at_qmat* m, int batch, Pro pro, Epi epi, const GemvArgs& a, int num_sms,
                   cudaStream_t s, bool pdl) {
    AT_REQUIRE(m->cols % QK == 0, AT_ERR_INVALID_ARG, "cols must be a multiple of 32");
    AT_REQUIRE(m->orient == AT_ORIENT_N, AT_ERR_INVALID_ARG, "matrix is not stored for orientation N");
    if (m->type == AT_GGML_Q6_K) {
        AT_REQUIRE(epi == Epi::Plain, AT_ERR_UNSUPPORTED, "Q6_K matrices take the plain epilogue only");
        launch_gemv_q6k(m, batch, pro, a, num_sms, s);
        return;
    }
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
// the per-column arrival counters of the orientation-T GEMV (batch above 2 or
// splits of more than 8 CTAs; the others combine in cluster shared memory) live in one
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
