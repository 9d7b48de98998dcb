// Fused-dequant Q4_0 / Q8_0 matrix-vector kernels for sm_100a.
//
// Replaces Kernels.sgemv over load-time dequantized FP32 weights
// (core/Kernels.java:350-371 fed by inference/Weights.java:185-203): the raw
// GGUF blocks stay resident in HBM and are dequantized in registers.
//
// Dequant: Q4_0 w = (q - 8) * d with the interleaved nibble order of
// quant/Q4_0.java:39-42 (element 2k = low nibble of byte k); Q8_0 w = q * d
// (quant/Q8_0.java:130-132); d decoded by Fp16.toFloat with flush-to-zero.
// A nibble/byte becomes the exact float (q - 8) through one byte permute into
// the mantissa of 2^23 plus one packed f32x2 subtraction; products and sums are
// FP32 (packed f32x2 FMA), so (q - 8) * x is formed exactly as the reference's
// dequantized weight times x, only the summation order differs.
//
// Orientation N (rows = outputs, blocks along the row): each warp streams R
// rows with 128-bit loads, lanes stride over blocks, x staged in shared
// memory (per block: even elements then odd elements, padded to 36 floats so
// a quarter-warp of 128-bit reads hits 32 distinct banks).
// Orientation T (rows = inputs, blocks along the outputs, stored
// block-column-major): each lane owns input rows of one block column and
// accumulates the 32 (or 8) outputs of that block; lanes are combined by a
// butterfly reduce-scatter, warps through shared memory, and CTAs that split
// the rows through a deterministic ordered reduction by the last CTA to arrive.
#include <cuda_fp16.h>

#include <map>
#include <mutex>

#include "at_internal.h"
#include "dev_common.cuh"

namespace at {

namespace {

constexpr int THREADS = 256;
constexpr int XPAD = 36;  // floats per staged 32-element block

// ---------------------------------------------------------------------------
// Per-block dot products on staged x.
// ---------------------------------------------------------------------------
// Q4_0: xr[0..3] hold the 16 even elements, xr[4..7] the 16 odd elements.
__device__ __forceinline__ float dot_q4(const uint4 q, const float4* xr) {
    const float2 moff = f2(-8388616.f, -8388616.f);  // -(2^23 + 8)
    float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t lo = w[i] & 0x0F0F0F0Fu, hi = (w[i] >> 4) & 0x0F0F0F0Fu;
        const float2 e01 = __fadd2_rn(f2(magic_byte(lo, 0), magic_byte(lo, 1)), moff);
        const float2 e23 = __fadd2_rn(f2(magic_byte(lo, 2), magic_byte(lo, 3)), moff);
        const float2 o01 = __fadd2_rn(f2(magic_byte(hi, 0), magic_byte(hi, 1)), moff);
        const float2 o23 = __fadd2_rn(f2(magic_byte(hi, 2), magic_byte(hi, 3)), moff);
        a0 = __ffma2_rn(e01, f2(xr[i].x, xr[i].y), a0);
        a1 = __ffma2_rn(e23, f2(xr[i].z, xr[i].w), a1);
        a0 = __ffma2_rn(o01, f2(xr[4 + i].x, xr[4 + i].y), a0);
        a1 = __ffma2_rn(o23, f2(xr[4 + i].z, xr[4 + i].w), a1);
    }
    return (a0.x + a0.y) + (a1.x + a1.y);
}

// Q8_0: xr[0..7] hold the 32 elements in order.
__device__ __forceinline__ float dot_q8(const uint4 q0, const uint4 q1, const float4* xr) {
    const float2 moff = f2(-8388736.f, -8388736.f);  // -(2^23 + 128)
    float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t u = w[i] ^ 0x80808080u;  // int8 q -> unsigned q + 128
        const float2 v01 = __fadd2_rn(f2(magic_byte(u, 0), magic_byte(u, 1)), moff);
        const float2 v23 = __fadd2_rn(f2(magic_byte(u, 2), magic_byte(u, 3)), moff);
        a0 = __ffma2_rn(v01, f2(xr[i].x, xr[i].y), a0);
        a1 = __ffma2_rn(v23, f2(xr[i].z, xr[i].w), a1);
    }
    return (a0.x + a0.y) + (a1.x + a1.y);
}

template <int QT>
struct QTraits;
template <>
struct QTraits<AT_GGML_Q4_0> { static constexpr int QB = 16; static constexpr int NV = 1; };
template <>
struct QTraits<AT_GGML_Q8_0> { static constexpr int QB = 32; static constexpr int NV = 2; };

// Slot of element w (0..31) of a block in the staged x layout.
template <int QT>
__device__ __forceinline__ int x_slot(int w) {
    if constexpr (QT == AT_GGML_Q4_0) return (w & 1) ? 16 + (w >> 1) : (w >> 1);
    else return w;
}

// ---------------------------------------------------------------------------
// Orientation N
// ---------------------------------------------------------------------------
struct NParams {
    const uint8_t* qs[2];
    const uint16_t* d[2];
    int rows, nb;
    int chunk_blocks, nchunks;
    int wk;        // warps splitting the blocks of a row (1, 2, 4, 8)
    int n_tiles;   // row tiles of (8 / wk) * R rows
    GemvArgs a;
};

template <int QT, int B, Pro PRO>
__device__ __forceinline__ void fill_x_n(float* xs, const NParams& p, int b0, int nbc, const float* s_inv) {
    const int n = nbc * 32;
    const int cols = p.nb * 32;
    for (int idx = threadIdx.x; idx < B * n; idx += THREADS) {
        const int bb = idx / n, e = idx - bb * n;
        const int col = b0 * 32 + e;
        float v;
        if constexpr (PRO == Pro::Plain) {
            v = p.a.x[(size_t)bb * p.a.x_stride + col];
        } else {
            float t = p.a.xin[(size_t)bb * p.a.x_stride + col];
            if (p.a.yin) t = __fadd_rn(t, p.a.yin[(size_t)bb * p.a.x_stride + col]);
            v = norm_apply(t, s_inv[bb], p.a.gamma[col]);
        }
        (void)cols;
        xs[(bb * p.chunk_blocks + (e >> 5)) * XPAD + x_slot<QT>(e & 31)] = v;
    }
}

template <int QT, int B, Pro PRO, Epi EPI>
__global__ void __launch_bounds__(THREADS) gemv_n_kernel(const NParams p) {
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    constexpr int R = (NM == 2) ? 2 : 4;
    constexpr int QB = QTraits<QT>::QB;
    constexpr int NV = QTraits<QT>::NV;
    constexpr int NVAL = NM * R * B;

    extern __shared__ __align__(16) float xs[];
    __shared__ float red[8][NVAL];
    __shared__ float s_red[8 * B];
    __shared__ float s_inv[B];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wk = p.wk, wrn = 8 / wk;
    const int wr = warp / wk, wki = warp - wr * wk;
    const int d_model = p.nb * 32;

    if constexpr (PRO == Pro::AddNorm) {
        block_rms_inv<B>(p.a.xin, p.a.yin, p.a.x_stride, d_model, p.a.eps, s_red, s_inv);
        if (blockIdx.x == 0) {
            for (int idx = tid; idx < B * d_model; idx += THREADS) {
                const int bb = idx / d_model, i = idx - bb * d_model;
                float t = p.a.xin[(size_t)bb * p.a.x_stride + i];
                if (p.a.yin) t = __fadd_rn(t, p.a.yin[(size_t)bb * p.a.x_stride + i]);
                p.a.xout[(size_t)bb * p.a.x_stride + i] = norm_apply(t, s_inv[bb], p.a.gamma[i]);
            }
        }
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
                fill_x_n<QT, B, PRO>(xs, p, b0, nbc, s_inv);
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
                            const size_t blk = (size_t)row * p.nb + b0 + j;
                            const uint8_t* src = p.qs[m] + blk * QB;
#pragma unroll
                            for (int v = 0; v < NV; ++v) q[m][r][v] = ld_stream_u4(src + 16 * v);
                            dsc[m][r] = fp16_ftz(ld_stream_u16(p.d[m] + blk));
                        } else {
#pragma unroll
                            for (int v = 0; v < NV; ++v) q[m][r][v] = make_uint4(0, 0, 0, 0);
                            dsc[m][r] = 0.f;
                        }
                    }
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float4* xv = reinterpret_cast<const float4*>(xs + (b * p.chunk_blocks + j) * XPAD);
                    float4 xr[8];
#pragma unroll
                    for (int t = 0; t < 8; ++t) xr[t] = xv[t];
#pragma unroll
                    for (int m = 0; m < NM; ++m)
#pragma unroll
                        for (int r = 0; r < R; ++r) {
                            float dv;
                            if constexpr (QT == AT_GGML_Q4_0) dv = dot_q4(q[m][r][0], xr);
                            else dv = dot_q8(q[m][r][0], q[m][r][NV - 1], xr);
                            acc[m][r][b] = fmaf(dsc[m][r], dv, acc[m][r][b]);
                        }
                }
            }
        }
        // warp reduction, then ordered reduction across the wk warps of a row tile
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
                float out = v0;
                if constexpr (EPI == Epi::SiluMul) {
                    // Kernels.siluInPlace then elementwiseMul (core/Kernels.java:86-87,
                    // inference/LlamaModel.java:372-380): g / (1 + exp(-g)) * u
                    const float sg = __fdiv_rn(v0, __fadd_rn(1.0f, expf(-v0)));
                    out = __fmul_rn(sg, v1);
                }
                p.a.y[(size_t)b * p.a.y_stride + row] = out;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Orientation T (block-column-major planes)
// ---------------------------------------------------------------------------
struct TParams {
    const uint8_t* qs;
    const uint16_t* d;
    int E;             // input rows
    int n_bc;          // block columns (outputs / 32)
    int S;             // CTAs splitting the rows of a block column
    int e_per_split;   // rows per CTA
    GemvArgs a;
};

// Columns per lane: 32 (a whole block) for B <= 2, else 8 (a quarter block).
template <int B>
struct TCfg {
    static constexpr int CPL = (B <= 2) ? 32 : 8;
    static constexpr int LPB = 32 / CPL;           // lanes per block
    static constexpr int ROWS_PER_WARP = 32 / LPB; // rows a warp covers per step
    static constexpr int STEP = 8 * ROWS_PER_WARP; // rows a CTA covers per step
};

// Decodes the CPL weights this lane owns into float pairs (q - 8 or q), in the
// column order given by col_of_pair().
template <int QT, int CPL>
__device__ __forceinline__ void decode_t(const uint4* q, int quarter, float2* wv) {
    if constexpr (QT == AT_GGML_Q4_0) {
        const float2 moff = f2(-8388616.f, -8388616.f);
        uint32_t w[CPL / 8];
        if constexpr (CPL == 32) { w[0] = q[0].x; w[1] = q[0].y; w[2] = q[0].z; w[3] = q[0].w; }
        else {
            const uint32_t a[4] = {q[0].x, q[0].y, q[0].z, q[0].w};
            w[0] = a[quarter];
        }
#pragma unroll
        for (int i = 0; i < CPL / 8; ++i) {
            const uint32_t lo = w[i] & 0x0F0F0F0Fu, hi = (w[i] >> 4) & 0x0F0F0F0Fu;
            wv[4 * i + 0] = __fadd2_rn(f2(magic_byte(lo, 0), magic_byte(lo, 1)), moff);  // cols 8i+0, 8i+2
            wv[4 * i + 1] = __fadd2_rn(f2(magic_byte(lo, 2), magic_byte(lo, 3)), moff);  // cols 8i+4, 8i+6
            wv[4 * i + 2] = __fadd2_rn(f2(magic_byte(hi, 0), magic_byte(hi, 1)), moff);  // cols 8i+1, 8i+3
            wv[4 * i + 3] = __fadd2_rn(f2(magic_byte(hi, 2), magic_byte(hi, 3)), moff);  // cols 8i+5, 8i+7
        }
    } else {
        const float2 moff = f2(-8388736.f, -8388736.f);
        uint32_t w[CPL / 4];
        if constexpr (CPL == 32) {
            w[0] = q[0].x; w[1] = q[0].y; w[2] = q[0].z; w[3] = q[0].w;
            w[4] = q[1].x; w[5] = q[1].y; w[6] = q[1].z; w[7] = q[1].w;
        } else {
            const uint32_t a[8] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w};
            w[0] = a[2 * quarter];
            w[1] = a[2 * quarter + 1];
        }
#pragma unroll
        for (int i = 0; i < CPL / 4; ++i) {
            const uint32_t u = w[i] ^ 0x80808080u;
            wv[2 * i + 0] = __fadd2_rn(f2(magic_byte(u, 0), magic_byte(u, 1)), moff);  // cols 4i, 4i+1
            wv[2 * i + 1] = __fadd2_rn(f2(magic_byte(u, 2), magic_byte(u, 3)), moff);  // cols 4i+2, 4i+3
        }
    }
}

// Column (within the lane's CPL columns) of element h (0/1) of pair k.
template <int QT>
__device__ __forceinline__ int col_of_pair(int k, int h) {
    if constexpr (QT == AT_GGML_Q4_0) {
        const int i = k >> 2, s = k & 3;
        return 8 * i + ((s & 1) ? 4 : 0) + ((s & 2) ? 1 : 0) + 2 * h;
    } else {
        return 2 * k + h;
    }
}

template <int QT, int B, Pro PRO, Epi EPI>
__global__ void __launch_bounds__(THREADS) gemv_t_kernel(const TParams p) {
    using C = TCfg<B>;
    constexpr int CPL = C::CPL, LPB = C::LPB;
    constexpr int QB = QTraits<QT>::QB;
    constexpr int NPAIR = CPL / 2;
    constexpr int NLOAD = (QT == AT_GGML_Q8_0 && CPL == 32) ? 2 : 1;

    extern __shared__ __align__(16) float xs[];  // [B][e_per_split]
    __shared__ float red[8][B][32];
    __shared__ float s_red[8 * B];
    __shared__ float s_inv[B];
    __shared__ int s_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x / p.S, s = blockIdx.x - (blockIdx.x / p.S) * p.S;
    const int e_lo = s * p.e_per_split;
    const int e_hi = min(p.E, e_lo + p.e_per_split);
    const int ne = e_hi - e_lo;

    if constexpr (PRO == Pro::AddNorm) {
        block_rms_inv<B>(p.a.xin, p.a.yin, p.a.x_stride, p.E, p.a.eps, s_red, s_inv);
        if (blockIdx.x == 0) {
            for (int idx = tid; idx < B * p.E; idx += THREADS) {
                const int bb = idx / p.E, i = idx - bb * p.E;
                float t = p.a.xin[(size_t)bb * p.a.x_stride + i];
                if (p.a.yin) t = __fadd_rn(t, p.a.yin[(size_t)bb * p.a.x_stride + i]);
                p.a.xout[(size_t)bb * p.a.x_stride + i] = norm_apply(t, s_inv[bb], p.a.gamma[i]);
            }
        }
    }
    for (int idx = tid; idx < B * ne; idx += THREADS) {
        const int bb = idx / ne, i = idx - bb * ne;
        const int e = e_lo + i;
        float v;
        if constexpr (PRO == Pro::Plain) {
            v = p.a.x[(size_t)bb * p.a.x_stride + e];
        } else {
            float t = p.a.xin[(size_t)bb * p.a.x_stride + e];
            if (p.a.yin) t = __fadd_rn(t, p.a.yin[(size_t)bb * p.a.x_stride + e]);
            v = norm_apply(t, s_inv[bb], p.a.gamma[e]);
        }
        xs[bb * p.e_per_split + i] = v;
    }
    __syncthreads();

    const int quarter = (LPB == 1) ? 0 : (lane & (LPB - 1));
    const int row_in_warp = lane / LPB;
    float2 acc[B][NPAIR];
#pragma unroll
    for (int b = 0; b < B; ++b)
#pragma unroll
        for (int k = 0; k < NPAIR; ++k) acc[b][k] = f2(0.f, 0.f);

    const uint8_t* colq = p.qs + (size_t)c * p.E * QB;
    const uint16_t* cold = p.d + (size_t)c * p.E;
    constexpr int U = 4;  // rows in flight per lane
    for (int base = 0; base < ne; base += C::STEP * U) {
        uint4 q[U][2];
        float dsc[U];
        int iu[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = base + u * C::STEP + warp * C::ROWS_PER_WARP + row_in_warp;
            iu[u] = i;
            if (i < ne) {
                const int e = e_lo + i;
                if constexpr (CPL == 32) {
#pragma unroll
                    for (int v = 0; v < NLOAD; ++v) q[u][v] = ld_stream_u4(colq + (size_t)e * QB + 16 * v);
                } else {
                    // a quarter block: 4 (Q4_0) or 8 (Q8_0) bytes, taken from the
                    // 16-byte vector that holds them (selected in decode_t)
                    q[u][0] = ld_stream_u4(colq + (size_t)e * QB + (QT == AT_GGML_Q8_0 ? 16 * (quarter >> 1) : 0));
                    q[u][1] = q[u][0];
                }
                dsc[u] = fp16_ftz(ld_stream_u16(cold + e));
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (iu[u] < ne) {
                float2 wv[NPAIR];
                if constexpr (QT == AT_GGML_Q8_0 && CPL == 8) decode_t<QT, CPL>(q[u], quarter & 1, wv);
                else decode_t<QT, CPL>(q[u], quarter, wv);
#pragma unroll
                for (int b = 0; b < B; ++b) {
                    const float sv = __fmul_rn(dsc[u], xs[b * p.e_per_split + iu[u]]);
                    const float2 s2 = f2(sv, sv);
#pragma unroll
                    for (int k = 0; k < NPAIR; ++k) acc[b][k] = __ffma2_rn(wv[k], s2, acc[b][k]);
                }
            }
        }
    }

    // Butterfly reduce-scatter across the lanes sharing a block column.
#pragma unroll
    for (int b = 0; b < B; ++b) {
        float v[CPL];
#pragma unroll
        for (int k = 0; k < NPAIR; ++k) {
            v[col_of_pair<QT>(k, 0)] = acc[b][k].x;
            v[col_of_pair<QT>(k, 1)] = acc[b][k].y;
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
        // v[0] is column: CPL==32 -> lane; CPL==8 -> 8*quarter + (lane >> 2)
        const int col = (CPL == 32) ? lane : (8 * quarter + (lane >> 2));
        red[warp][b][col] = v[0];
    }
    __syncthreads();

    // CTA partial for (block column c, rows [e_lo, e_hi)): thread (b = warp, col = lane)
    float val = 0.f;
    const int b_me = warp, col = lane;
    if (b_me < B) {
#pragma unroll
        for (int w = 0; w < 8; ++w) val += red[w][b_me][col];
    }
    if (p.S > 1) {
        if (b_me < B) p.a.scratch[(((size_t)c * p.S + s) * B + b_me) * 32 + col] = val;
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
                val += __ldcg(&p.a.scratch[(((size_t)c * p.S + k) * B + b_me) * 32 + col]);
        }
        if (tid == 0) p.a.counters[c] = 0u;
    }
    if (b_me >= B) return;

    const int j = c * 32 + col;  // output column
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

void ensure_smem(const void* fn, int smem) {
    std::lock_guard<std::mutex> lk(g_attr_mu);
    auto it = g_smem_set.find(fn);
    if (it != g_smem_set.end() && it->second >= smem) return;
    AT_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    g_smem_set[fn] = smem;
}

int occupancy(const void* fn, int smem) {
    int n = 0;
    AT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, THREADS, smem));
    return n < 1 ? 1 : n;
}

constexpr int kMaxXSmem = 96 * 1024;

template <int QT, int B, Pro PRO, Epi EPI>
void run_n(const at_qmat* m, const GemvArgs& a, int num_sms, cudaStream_t s) {
    constexpr int NM = (EPI == Epi::SiluMul) ? 2 : 1;
    constexpr int R = (NM == 2) ? 2 : 4;
    NParams p{};
    p.qs[0] = m->qs; p.d[0] = m->d;
    if constexpr (NM == 2) { p.qs[1] = a.m2->qs; p.d[1] = a.m2->d; }
    else { p.qs[1] = m->qs; p.d[1] = m->d; }
    p.rows = (int)m->rows;
    p.nb = (int)(m->cols / QK);
    p.chunk_blocks = std::min(p.nb, std::max(32, kMaxXSmem / (B * XPAD * 4)));
    p.nchunks = (p.nb + p.chunk_blocks - 1) / p.chunk_blocks;
    p.a = a;
    const int smem = B * p.chunk_blocks * XPAD * 4;
    const void* fn = reinterpret_cast<const void*>(&gemv_n_kernel<QT, B, PRO, EPI>);
    ensure_smem(fn, smem);
    const int occ = occupancy(fn, smem);
    int wk = 1;
    auto tiles = [&](int w) { return (p.rows + (8 / w) * R - 1) / ((8 / w) * R); };
    while (wk < 8 && tiles(wk) < 2 * num_sms && p.chunk_blocks >= 64 * wk) wk *= 2;
    p.wk = wk;
    p.n_tiles = tiles(wk);
    const int grid = std::max(1, std::min(p.n_tiles, num_sms * occ));
    gemv_n_kernel<QT, B, PRO, EPI><<<grid, THREADS, smem, s>>>(p);
    AT_CUDA(cudaGetLastError());
}

void t_config(const at_qmat* m, int batch, int num_sms, int* S, int* eps_rows) {
    const int step = (batch <= 2) ? 256 : 64;
    const int E = (int)m->rows;
    const int n_bc = (int)(m->cols / QK);
    int s = std::max(1, (2 * num_sms + n_bc - 1) / n_bc);
    s = std::min(s, std::max(1, E / (2 * step)));
    int per = (E + s - 1) / s;
    per = ((per + step - 1) / step) * step;
    // the staged x slice must fit the shared-memory budget
    const int cap = std::max(step, (kMaxXSmem / (4 * batch)) / step * step);
    per = std::min(per, cap);
    *eps_rows = per;
    *S = (E + per - 1) / per;
}

template <int QT, int B, Pro PRO, Epi EPI>
void run_t(const at_qmat* m, const GemvArgs& a, int num_sms, cudaStream_t s) {
    TParams p{};
    p.qs = m->qs; p.d = m->d;
    p.E = (int)m->rows;
    p.n_bc = (int)(m->cols / QK);
    t_config(m, B, num_sms, &p.S, &p.e_per_split);
    p.a = a;
    if (p.S > 1) AT_REQUIRE(a.scratch && a.counters, AT_ERR_STATE, "T GEMV needs split scratch");
    const int smem = B * p.e_per_split * 4;
    const void* fn = reinterpret_cast<const void*>(&gemv_t_kernel<QT, B, PRO, EPI>);
    ensure_smem(fn, smem);
    gemv_t_kernel<QT, B, PRO, EPI><<<p.n_bc * p.S, THREADS, smem, s>>>(p);
    AT_CUDA(cudaGetLastError());
}

template <int QT, Pro PRO, Epi EPI, bool IS_T>
void dispatch_b(const at_qmat* m, int batch, const GemvArgs& a, int num_sms, cudaStream_t s) {
#define AT_CASE(BB)                                                      \
    case BB:                                                             \
        if constexpr (IS_T) run_t<QT, BB, PRO, EPI>(m, a, num_sms, s);   \
        else run_n<QT, BB, PRO, EPI>(m, a, num_sms, s);                  \
        break;
    switch (batch) {
        AT_CASE(1) AT_CASE(2) AT_CASE(3) AT_CASE(4) AT_CASE(5) AT_CASE(6) AT_CASE(7) AT_CASE(8)
        default: fail(AT_ERR_INVALID_ARG, "batch must be in [1, 8]");
    }
#undef AT_CASE
}

template <Pro PRO, Epi EPI, bool IS_T>
void dispatch_q(const at_qmat* m, int batch, const GemvArgs& a, int num_sms, cudaStream_t s) {
    if (m->type == AT_GGML_Q4_0) dispatch_b<AT_GGML_Q4_0, PRO, EPI, IS_T>(m, batch, a, num_sms, s);
    else if (m->type == AT_GGML_Q8_0) dispatch_b<AT_GGML_Q8_0, PRO, EPI, IS_T>(m, batch, a, num_sms, s);
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
                   cudaStream_t s) {
    AT_REQUIRE(m->cols % QK == 0, AT_ERR_INVALID_ARG, "cols must be a multiple of 32");
    if (pro == Pro::Plain && epi == Epi::Plain) dispatch_q<Pro::Plain, Epi::Plain, false>(m, batch, a, num_sms, s);
    else if (pro == Pro::AddNorm && epi == Epi::Plain) dispatch_q<Pro::AddNorm, Epi::Plain, false>(m, batch, a, num_sms, s);
    else if (pro == Pro::AddNorm && epi == Epi::SiluMul) {
        AT_REQUIRE(a.m2 && a.m2->type == m->type && a.m2->rows == m->rows && a.m2->cols == m->cols,
                   AT_ERR_INVALID_ARG, "gate/up matrices must match");
        dispatch_q<Pro::AddNorm, Epi::SiluMul, false>(m, batch, a, num_sms, s);
    } else fail(AT_ERR_UNSUPPORTED, "unsupported N prologue/epilogue combination");
}

void launch_gemv_t(const at_qmat* m, int batch, Pro pro, Epi epi, const GemvArgs& a, int num_sms,
                   cudaStream_t s) {
    AT_REQUIRE(m->cols % QK == 0, AT_ERR_INVALID_ARG, "cols must be a multiple of 32");
    if (pro == Pro::Plain && epi == Epi::Plain) dispatch_q<Pro::Plain, Epi::Plain, true>(m, batch, a, num_sms, s);
    else if (pro == Pro::AddNorm && epi == Epi::QkvRope) dispatch_q<Pro::AddNorm, Epi::QkvRope, true>(m, batch, a, num_sms, s);
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

}  // namespace at
