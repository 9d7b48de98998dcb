// Q6_K matrices (256 elements per 210-byte block, quant/Q6_K.java) for the
// token embedding and the lm_head of llama.cpp exports, on sm_100a.
//
// Device layout: a lossless re-layout of whole blocks, orientation N only
// (blocks along the rows): block (row, b) sits at (row * nsteps + b) * 224,
// its 210 bytes copied unchanged (ql[128], qh[64], int8 scales[16], fp16 d)
// and padded to 224 so every block starts on a 16-byte boundary.
//
// Dequant (Q6_K.dequantToFloat, quant/Q6_K.java:54-102, the published
// llama.cpp dequantize_row_q6_K): element n + 32 j + l of a block (half
// n = 0 or 128, group j = 0..3, l = 0..31) is
//   (d * scale[n/16 + l/16 + 2 j]) * (q - 32),  q = 4 bits of ql | 2 bits of qh << 4,
// with the low nibble of ql[n/2 + l] (j = 0), of ql[n/2 + l + 32] (j = 1),
// their high nibbles (j = 2, 3), and qh[n/4 + l] bits 2j..2j+1; d decoded by
// Fp16.toFloat with flush-to-zero. The products are rounded in that order,
// as the reference does in float.
#include <algorithm>
#include <string>

#include "at_internal.h"
#include "dev_common.cuh"

namespace at {

namespace {

constexpr int Q6_BLOCK = 256;
constexpr int Q6_BYTES = 210;
constexpr int Q6_STRIDE = 224;

__device__ __forceinline__ float q6_weight(const uint8_t* blk, int e, float d) {
    const int n = e >> 7, j = (e >> 5) & 3, l = e & 31;
    const uint32_t ql = blk[64 * n + l + ((j & 1) ? 32 : 0)];
    const uint32_t qh = blk[128 + 32 * n + l];
    const int q = (int)(((j >= 2) ? (ql >> 4) : (ql & 0xF)) | (((qh >> (2 * j)) & 3u) << 4)) - 32;
    const float s = (float)(int8_t)blk[192 + 8 * n + (l >> 4) + 2 * j];
    return __fmul_rn(__fmul_rn(d, s), (float)q);
}

__device__ __forceinline__ float q6_d(const uint8_t* blk) {
    return fp16_ftz((uint32_t)blk[208] | ((uint32_t)blk[209] << 8));
}

// Raw blocks (row-major, src_nb blocks per row) -> padded device blocks.
__global__ void q6k_repack_kernel(const uint8_t* __restrict__ src, int64_t src_nb, int64_t r0, int64_t n_rows,
                                  int64_t nb, int64_t dr0, uint8_t* __restrict__ tiles) {
    const int64_t total = n_rows * nb * Q6_STRIDE;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = t / Q6_STRIDE, k = t - blk * Q6_STRIDE;
        const int64_t r = blk / nb, b = blk - r * nb;
        tiles[((dr0 + r) * nb + b) * Q6_STRIDE + k] = (k < Q6_BYTES) ? src[((r0 + r) * src_nb + b) * Q6_BYTES + k] : 0;
    }
}

__global__ void q6k_unpack_kernel(const uint8_t* __restrict__ tiles, int64_t nblocks, uint8_t* __restrict__ dst) {
    const int64_t total = nblocks * Q6_BYTES;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = t / Q6_BYTES, k = t - blk * Q6_BYTES;
        dst[t] = tiles[blk * Q6_STRIDE + k];
    }
}

// Raw row-major blocks -> FP32 (the codec entry point).
__global__ void q6k_dequant_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint8_t* blk = src + (i / Q6_BLOCK) * Q6_BYTES;
        dst[i] = q6_weight(blk, (int)(i % Q6_BLOCK), q6_d(blk));
    }
}

// writeTokenEmbedding (inference/LlamaModel.java:181-186) from a Q6_K table;
// the same side effects as the Q4_0 / Q8_0 embedding kernel (y <- 0, argmax
// keys cleared, step sequence advanced).
__global__ void q6k_embed_kernel(const uint8_t* __restrict__ tiles, int64_t nb, const int* __restrict__ tokens, int d,
                                 float* __restrict__ xa, float* __restrict__ y, unsigned long long* __restrict__ argkeys,
                                 unsigned* __restrict__ step) {
    const int b = blockIdx.x;
    if (threadIdx.x == 0 && argkeys) argkeys[b] = 0ull;
    if (b == 0 && threadIdx.x == 0 && step) *step += 1u;
    const uint8_t* row = tiles + (int64_t)tokens[b] * nb * Q6_STRIDE;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const uint8_t* blk = row + (int64_t)(i / Q6_BLOCK) * Q6_STRIDE;
        xa[(size_t)b * d + i] = q6_weight(blk, i % Q6_BLOCK, q6_d(blk));
        if (y) y[(size_t)b * d + i] = 0.f;
    }
}

// y[b][row] = sum_c W[row][c] x[b][c] over Q6_K rows: one warp per row at a
// time, lane l takes elements n + 32 j + l of every block (its 8 weights per
// block read 4 ql bytes, 2 qh bytes and 8 scales; consecutive lanes read
// consecutive bytes and consecutive x). x (or the normed x + y of an AddNorm
// prologue, the reference's rounding) is staged once per CTA in shared memory.
template <int B, bool ADDNORM>
__global__ void __launch_bounds__(256) gemv_q6k_kernel(const uint8_t* __restrict__ tiles, int rows, int nb,
                                                       GemvArgs a) {
    extern __shared__ __align__(16) float xs[];  // [B][cols]
    __shared__ float s_red[8 * B];
    __shared__ float s_inv[B];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cols = nb * Q6_BLOCK;
    if constexpr (ADDNORM) {
        block_rms_inv<B>(a.xin, a.yin, a.x_stride, cols, a.eps, s_red, s_inv);
        for (int i = tid; i < B * cols; i += 256) {
            const int bb = i / cols, c = i - bb * cols;
            const size_t off = (size_t)bb * a.x_stride + c;
            const float t = a.yin ? __fadd_rn(a.xin[off], a.yin[off]) : a.xin[off];
            const float xn = norm_apply(t, s_inv[bb], a.gamma[c]);
            xs[i] = xn;
            if (blockIdx.x == 0 && a.xout) a.xout[off] = xn;
        }
    } else {
        for (int i = tid; i < B * cols; i += 256) {
            const int bb = i / cols, c = i - bb * cols;
            xs[i] = a.x[(size_t)bb * a.x_stride + c];
        }
    }
    __syncthreads();
    const int nwarps = gridDim.x * 8;
    for (int row = blockIdx.x * 8 + warp; row < rows; row += nwarps) {
        const uint8_t* rp = tiles + (int64_t)row * nb * Q6_STRIDE;
        float acc[B];
#pragma unroll
        for (int bb = 0; bb < B; ++bb) acc[bb] = 0.f;
        for (int blk = 0; blk < nb; ++blk) {
            const uint8_t* bp = rp + (int64_t)blk * Q6_STRIDE;
            const float d = q6_d(bp);
#pragma unroll
            for (int n = 0; n < 2; ++n) {
                const uint32_t lo = bp[64 * n + lane], hi = bp[64 * n + 32 + lane], qh = bp[128 + 32 * n + lane];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t ql = (j & 1) ? hi : lo;
                    const int q = (int)(((j >= 2) ? (ql >> 4) : (ql & 0xF)) | (((qh >> (2 * j)) & 3u) << 4)) - 32;
                    const float s = (float)(int8_t)bp[192 + 8 * n + (lane >> 4) + 2 * j];
                    const float w = __fmul_rn(__fmul_rn(d, s), (float)q);
                    const int c = blk * Q6_BLOCK + 128 * n + 32 * j + lane;
#pragma unroll
                    for (int bb = 0; bb < B; ++bb) acc[bb] = fmaf(w, xs[bb * cols + c], acc[bb]);
                }
            }
        }
#pragma unroll
        for (int bb = 0; bb < B; ++bb) {
            const float v = warp_sum(acc[bb]);
            if (lane == 0) a.y[(size_t)bb * a.y_stride + row] = v;
        }
    }
}

int grid_for(int64_t n) { return (int)std::min<int64_t>(4096, std::max<int64_t>(1, (n + 255) / 256)); }

template <int B, bool ADDNORM>
void run_q6k(const at_qmat* m, const GemvArgs& a, int num_sms, cudaStream_t s) {
    const int nb = (int)(m->cols / Q6_BLOCK);
    const size_t smem = (size_t)B * m->cols * 4;
    const void* fn = reinterpret_cast<const void*>(&gemv_q6k_kernel<B, ADDNORM>);
    AT_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int grid = std::max(1, std::min<int>(2 * num_sms, (int)((m->rows + 7) / 8)));
    gemv_q6k_kernel<B, ADDNORM><<<grid, 256, smem, s>>>(m->tiles, (int)m->rows, nb, a);
    AT_CUDA(cudaGetLastError());
}

}  // namespace

void q6k_alloc(at_qmat* m) {
    AT_REQUIRE(m->orient == AT_ORIENT_N, AT_ERR_UNSUPPORTED, "Q6_K matrices are stored for orientation N only");
    AT_REQUIRE(m->cols % Q6_BLOCK == 0, AT_ERR_INVALID_ARG, "Q6_K matrix cols must be a multiple of 256");
    m->tile_bytes = Q6_STRIDE;
    m->nsteps = m->cols / Q6_BLOCK;
    m->ngroups = m->rows;
    m->bytes = (size_t)(m->rows * m->nsteps * Q6_STRIDE);
    AT_CUDA(cudaMalloc(&m->tiles, m->bytes));
    AT_CUDA(cudaMemset(m->tiles, 0, m->bytes));
}

void q6k_fill_rows(at_qmat* m, const uint8_t* src_dev, int64_t src_cols, int64_t src_r0, int64_t n_rows,
                   int64_t dst_r0, cudaStream_t s) {
    AT_REQUIRE(src_cols == m->cols, AT_ERR_INVALID_ARG, "Q6_K rows are copied whole");
    AT_REQUIRE(dst_r0 + n_rows <= m->rows, AT_ERR_INVALID_ARG, "region exceeds the destination matrix");
    if (n_rows <= 0) return;
    const int64_t nb = m->nsteps;
    q6k_repack_kernel<<<grid_for(n_rows * nb * Q6_STRIDE), 256, 0, s>>>(src_dev, nb, src_r0, n_rows, nb, dst_r0,
                                                                        m->tiles);
    AT_CUDA(cudaGetLastError());
}

void q6k_export(const at_qmat* m, uint8_t* dst_dev, cudaStream_t s) {
    const int64_t nblocks = m->rows * m->nsteps;
    q6k_unpack_kernel<<<grid_for(nblocks * Q6_BYTES), 256, 0, s>>>(m->tiles, nblocks, dst_dev);
    AT_CUDA(cudaGetLastError());
}

void launch_q6k_dequant(const uint8_t* src_dev, float* dst_dev, int64_t n, cudaStream_t s) {
    q6k_dequant_kernel<<<grid_for(n), 256, 0, s>>>(src_dev, dst_dev, n);
    AT_CUDA(cudaGetLastError());
}

void launch_q6k_embed(const at_qmat* tok, const int* tokens, int B, int d, float* xa, float* y,
                      unsigned long long* argkeys, unsigned* step, cudaStream_t s) {
    q6k_embed_kernel<<<B, 256, 0, s>>>(tok->tiles, tok->nsteps, tokens, d, xa, y, argkeys, step);
    AT_CUDA(cudaGetLastError());
}

void launch_gemv_q6k(const at_qmat* m, int batch, Pro pro, const GemvArgs& a, int num_sms, cudaStream_t s) {
    AT_REQUIRE((size_t)batch * m->cols * 4 <= 200 * 1024, AT_ERR_UNSUPPORTED,
               "Q6_K GEMV stages batch x cols floats in shared memory (at most 200 KiB)");
#define AT_Q6(BB)                                                                      \
    case BB:                                                                           \
        if (pro == Pro::AddNorm) run_q6k<BB, true>(m, a, num_sms, s);                  \
        else run_q6k<BB, false>(m, a, num_sms, s);                                     \
        break;
    switch (batch) {
        AT_Q6(1) AT_Q6(2) AT_Q6(3) AT_Q6(4) AT_Q6(5) AT_Q6(6) AT_Q6(7) AT_Q6(8)
        default: fail(AT_ERR_INVALID_ARG, "batch must be in [1, 8]");
    }
#undef AT_Q6
}

}  // namespace at
