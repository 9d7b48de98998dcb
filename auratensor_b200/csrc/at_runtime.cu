// Runtime, memory, block codecs, planar re-layout and the core.Kernels ops of
// libauratensor_cuda.so.
#include <cstring>
#include <mutex>
#include <string>

#include "at_internal.h"
#include "dev_common.cuh"

namespace at {

namespace {
thread_local std::string g_last_error;
constexpr int TPB = 256;

inline int grid_for(int64_t n, int tpb = TPB) {
    int64_t g = (n + tpb - 1) / tpb;
    if (g > (1 << 30)) g = 1 << 30;
    return (int)(g < 1 ? 1 : g);
}
}  // namespace

void set_last_error(const std::string& msg) { g_last_error = msg; }

// ---------------------------------------------------------------------------
// Codecs
// ---------------------------------------------------------------------------
__global__ void fp16_to_f32_kernel(const uint16_t* __restrict__ src, float* __restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = fp16_ftz(src[i]);
}

__device__ __forceinline__ float block_scale(const uint8_t* blk) {
    return fp16_ftz((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
}

// Q4_0.dequantToFloat (quant/Q4_0.java:32-45): element i of block b is
// ((i even ? lo : hi) nibble of byte i/2) - 8, times the block scale.
__device__ __forceinline__ float q4_0_elem(const uint8_t* src, int64_t i) {
    const uint8_t* blk = src + (i >> 5) * 18;
    const int w = (int)(i & 31);
    const uint32_t pack = blk[2 + (w >> 1)];
    const int q = (w & 1) ? (int)((pack >> 4) & 0xF) : (int)(pack & 0xF);
    return __fmul_rn((float)(q - 8), block_scale(blk));
}
// Q8_0.dequantToFloat (quant/Q8_0.java:32-44): int8 q times the block scale.
__device__ __forceinline__ float q8_0_elem(const uint8_t* src, int64_t i) {
    const uint8_t* blk = src + (i >> 5) * 34;
    const int q = (int)(int8_t)blk[2 + (i & 31)];
    return __fmul_rn((float)q, block_scale(blk));
}

template <int QT>
__global__ void dequant_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = (QT == AT_GGML_Q4_0) ? q4_0_elem(src, i) : q8_0_elem(src, i);
}

// dot = sum_i dequant(i) * x[i] over all elements (dequantToFloat semantics).
template <int QT>
__global__ void __launch_bounds__(1024) qdot_kernel(const uint8_t* __restrict__ src, const float* __restrict__ x,
                                                    int64_t n, float* __restrict__ out) {
    __shared__ float red[32];
    float acc = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float w = (QT == AT_GGML_Q4_0) ? q4_0_elem(src, i) : q8_0_elem(src, i);
        acc = fmaf(w, x[i], acc);
    }
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) *out = v;
    }
}

// ---------------------------------------------------------------------------
// Planar re-layout of raw GGUF blocks (lossless: bytes are moved, never
// re-quantized).
// ---------------------------------------------------------------------------
__global__ void repack_kernel(const uint8_t* __restrict__ src, int bb /*18|34*/, int qb /*16|32*/,
                              int64_t src_nb, int64_t r0, int64_t cb0, int64_t n_rows, int64_t n_cb,
                              int64_t dr0, int64_t dcb0, QTileMap map, uint8_t* __restrict__ tiles, int nib_split) {
    const int64_t total = n_rows * n_cb;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / n_cb, b = t - (t / n_cb) * n_cb;
        const uint8_t* s = src + ((r0 + r) * src_nb + cb0 + b) * bb;
        int64_t d_off, q_off;
        map.offsets(dr0 + r, dcb0 + b, &d_off, &q_off);
        tiles[d_off] = s[0];
        tiles[d_off + 1] = s[1];
        uint8_t* q = tiles + q_off;
        if (nib_split) {
            // llama.cpp order in: element e is the low nibble of byte e (e < 16)
            // or the high nibble of byte e - 16; interleaved out: byte k holds
            // elements 2k (low) and 2k + 1 (high)
            for (int k = 0; k < 16; ++k) {
                const int e0 = 2 * k, e1 = 2 * k + 1;
                const uint32_t q0 = (e0 < 16) ? (s[2 + e0] & 0xFu) : (s[2 + e0 - 16] >> 4);
                const uint32_t q1 = (e1 < 16) ? (s[2 + e1] & 0xFu) : (s[2 + e1 - 16] >> 4);
                q[k] = (uint8_t)(q0 | (q1 << 4));
            }
        } else {
            for (int k = 0; k < qb; ++k) q[k] = s[2 + k];
        }
    }
}

__global__ void unpack_kernel(const uint8_t* __restrict__ tiles, QTileMap map, int bb, int qb, int64_t rows,
                              int64_t nb, uint8_t* __restrict__ out) {
    const int64_t total = rows * nb;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / nb, b = t - (t / nb) * nb;
        int64_t d_off, q_off;
        map.offsets(r, b, &d_off, &q_off);
        uint8_t* o = out + (r * nb + b) * bb;
        o[0] = tiles[d_off];
        o[1] = tiles[d_off + 1];
        for (int k = 0; k < qb; ++k) o[2 + k] = tiles[q_off + k];
    }
}

__global__ void float_slice_kernel(const void* __restrict__ src, int src_type, int64_t src_cols, int64_t r0,
                                   int64_t c0, int64_t rows, int64_t cols, float* __restrict__ dst) {
    const int64_t total = rows * cols;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / cols, c = t - (t / cols) * cols;
        const int64_t i = (r0 + r) * src_cols + c0 + c;
        dst[t] = (src_type == AT_GGML_F32) ? static_cast<const float*>(src)[i]
                                           : fp16_ftz(static_cast<const uint16_t*>(src)[i]);
    }
}

void qmat_alloc(at_qmat* m) {
    if (m->type == AT_GGML_Q6_K) {
        q6k_alloc(m);
        return;
    }
    if (m->type == AT_GGML_F32 || m->type == AT_GGML_F16) {
        m->type = AT_GGML_F32;
        AT_CUDA(cudaMalloc(&m->f32, (size_t)(m->rows * m->cols) * 4));
        return;
    }
    AT_REQUIRE(m->type == AT_GGML_Q4_0 || m->type == AT_GGML_Q8_0, AT_ERR_UNSUPPORTED,
               "unsupported tensor type " + std::to_string(m->type));
    AT_REQUIRE(m->cols % QK == 0, AT_ERR_INVALID_ARG, "quantized matrix cols must be a multiple of 32");
    const int64_t nb = m->cols / QK;
    const int64_t qb = quant_bytes(m->type);
    if (m->orient == AT_ORIENT_N) {
        m->tile_bytes = 4 * 32 * (2 + qb);
        m->nsteps = (nb + 31) / 32;
        m->ngroups = (m->rows + 3) / 4;
        m->bytes = (size_t)(m->ngroups * m->nsteps * m->tile_bytes);
    } else {
        m->tile_bytes = 32 * (2 + qb);
        m->nsteps = 0;
        m->ngroups = (m->rows + 31) / 32;
        m->bytes = (size_t)(nb * m->ngroups * m->tile_bytes);
    }
    AT_CUDA(cudaMalloc(&m->tiles, m->bytes));
    AT_CUDA(cudaMemset(m->tiles, 0, m->bytes));
}

void qmat_free(at_qmat* m) {
    if (!m->owns) return;
    if (m->tiles) cudaFree(m->tiles);
    if (m->f32) cudaFree(m->f32);
    m->tiles = nullptr; m->f32 = nullptr;
}

void qmat_fill_region(at_qmat* m, const uint8_t* src_dev, int64_t src_cols, int64_t src_r0, int64_t src_c0,
                      int64_t n_rows, int64_t n_cols, int64_t dst_r0, int64_t dst_c0, cudaStream_t s, int nib_split) {
    if (m->type == AT_GGML_Q6_K) {
        AT_REQUIRE(src_c0 == 0 && dst_c0 == 0 && n_cols == m->cols, AT_ERR_INVALID_ARG, "Q6_K rows are copied whole");
        q6k_fill_rows(m, src_dev, src_cols, src_r0, n_rows, dst_r0, s);
        return;
    }
    AT_REQUIRE(src_cols % QK == 0 && src_c0 % QK == 0 && n_cols % QK == 0 && dst_c0 % QK == 0, AT_ERR_INVALID_ARG,
               "block-matrix regions must be aligned to 32 columns");
    AT_REQUIRE(dst_r0 + n_rows <= m->rows && dst_c0 + n_cols <= m->cols, AT_ERR_INVALID_ARG,
               "region exceeds the destination matrix");
    if (n_rows <= 0 || n_cols <= 0) return;
    const int64_t n_cb = n_cols / QK;
    repack_kernel<<<grid_for(n_rows * n_cb), TPB, 0, s>>>(src_dev, block_bytes(m->type), quant_bytes(m->type),
                                                          src_cols / QK, src_r0, src_c0 / QK, n_rows, n_cb, dst_r0,
                                                          dst_c0 / QK, tile_map(m), m->tiles,
                                                          (nib_split && m->type == AT_GGML_Q4_0) ? 1 : 0);
    AT_CUDA(cudaGetLastError());
}

void qmat_fill_from_blocks(at_qmat* m, const uint8_t* src_dev, int64_t src_cols, int64_t r0, int64_t c0,
                           cudaStream_t s) {
    qmat_fill_region(m, src_dev, src_cols, r0, c0, m->rows, m->cols, 0, 0, s);
}

void qmat_fill_from_float(at_qmat* m, const void* src_dev, int src_type, int64_t src_cols, int64_t r0,
                          int64_t c0, cudaStream_t s) {
    float_slice_kernel<<<grid_for(m->rows * m->cols), TPB, 0, s>>>(src_dev, src_type, src_cols, r0, c0, m->rows,
                                                                   m->cols, m->f32);
    AT_CUDA(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// core.Kernels ops on FP32 device buffers
// ---------------------------------------------------------------------------
// (float) Math.exp(v) of the reference: exponential in double, rounded to float.
__device__ __forceinline__ float exp_as_ref(float v) { return (float)exp((double)v); }

__global__ void sgemm_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C,
                             int M, int K, int N) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x, i = blockIdx.y;
    if (j >= N || i >= M) return;
    float acc = 0.f;
    for (int k = 0; k < K; ++k) acc = fmaf(A[(size_t)i * K + k], B[(size_t)k * N + j], acc);
    C[(size_t)i * N + j] = acc;
}

__global__ void sgemv_t_f32_kernel(const float* __restrict__ W, const float* __restrict__ x, float* __restrict__ y,
                                   int rows, int cols, int batch) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    for (int b = 0; b < batch; ++b) {
        float acc = 0.f;
        for (int r = 0; r < rows; ++r) acc = fmaf(W[(size_t)r * cols + c], x[(size_t)b * rows + r], acc);
        y[(size_t)b * cols + c] = acc;
    }
}

__global__ void __launch_bounds__(256) rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ w, float eps,
                                                      int d) {
    __shared__ float s_red[8];
    __shared__ float s_inv;
    float* row = x + (size_t)blockIdx.x * d;
    float acc = 0.f;
    for (int i = threadIdx.x; i < d; i += 256) acc = fmaf(row[i], row[i], acc);
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int k = 0; k < 8; ++k) t += s_red[k];
        s_inv = rms_inv(t, d, eps);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < d; i += 256) row[i] = norm_apply(row[i], s_inv, w[i]);
}

// Kernels.softmaxInPlaceSegment (core/Kernels.java:181-232): max, exp(x - max),
// sum, then multiply by inv = 1 / sum.
__global__ void __launch_bounds__(256) softmax_kernel(float* __restrict__ x, int n) {
    __shared__ float red[8];
    __shared__ float s_val;
    float* row = x + (size_t)blockIdx.x * n;
    const int tid = threadIdx.x;
    float m = -INFINITY;
    for (int i = tid; i < n; i += 256) m = fmaxf(m, row[i]);
    m = warp_max(m);
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
        float t = red[0];
        for (int k = 1; k < 8; ++k) t = fmaxf(t, red[k]);
        s_val = t;
    }
    __syncthreads();
    const float mx = s_val;
    float sum = 0.f;
    for (int i = tid; i < n; i += 256) {
        const float e = exp_as_ref(__fsub_rn(row[i], mx));
        row[i] = e;
        sum += e;
    }
    sum = warp_sum(sum);
    __syncthreads();
    if ((tid & 31) == 0) red[tid >> 5] = sum;
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int k = 0; k < 8; ++k) t += red[k];
        s_val = __fdiv_rn(1.0f, t);
    }
    __syncthreads();
    const float inv = s_val;
    for (int i = tid; i < n; i += 256) row[i] = __fmul_rn(row[i], inv);
}

// Kernels.ropeInPlaceSegment vector path (core/Kernels.java:296-309).
__global__ void rope_kernel(float* __restrict__ qk, const float* __restrict__ cs, const float* __restrict__ sn,
                            int head_dim, int n) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;  // pair index
    if (2 * t >= n) return;
    const int dd = (2 * t) % head_dim;
    const float a = qk[2 * t], b = qk[2 * t + 1];
    const float c = cs[dd], s = sn[dd];
    qk[2 * t] = fmaf(a, c, __fmul_rn(b, -s));
    qk[2 * t + 1] = fmaf(b, cs[dd + 1], __fmul_rn(a, sn[dd + 1]));
}

// Kernels.siluInPlaceSegment (core/Kernels.java:61-90): x / (1 + (float) exp(-x)).
__global__ void silu_kernel(float* __restrict__ x, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        x[i] = __fdiv_rn(v, __fadd_rn(1.0f, exp_as_ref(-v)));
    }
}

}  // namespace at

using namespace at;

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char* at_version(void) { return "auratensor-b200 0.1 (sm_100a)"; }

int at_last_error(char* buf, size_t len) {
    const std::string& e = g_last_error;
    if (buf && len) {
        const size_t n = e.size() < len - 1 ? e.size() : len - 1;
        memcpy(buf, e.data(), n);
        buf[n] = 0;
    }
    return (int)e.size();
}

int at_device_count(int* n) {
    return guard([&] {
        AT_REQUIRE(n, AT_ERR_INVALID_ARG, "null output");
        AT_CUDA(cudaGetDeviceCount(n));
    });
}

int at_ctx_create(int device, at_ctx** out) {
    return guard([&] {
        AT_REQUIRE(out, AT_ERR_INVALID_ARG, "null output");
        AT_CUDA(cudaSetDevice(device));
        auto* c = new at_ctx();
        c->device = device;
        // A blocking stream: it orders itself after work on the legacy default
        // stream (where host frameworks enqueue by default) and vice versa.
        AT_CUDA(cudaStreamCreateWithFlags(&c->own_stream, cudaStreamDefault));
        c->stream = c->own_stream;
        AT_CUDA(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device));
        *out = c;
    });
}

int at_ctx_synchronize(at_ctx* ctx) {
    return guard([&] {
        AT_REQUIRE(ctx, AT_ERR_INVALID_ARG, "null context");
        AT_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int at_ctx_stream(at_ctx* ctx, void** stream) {
    return guard([&] {
        AT_REQUIRE(ctx && stream, AT_ERR_INVALID_ARG, "null argument");
        *stream = ctx->stream;
    });
}

int at_ctx_set_stream(at_ctx* ctx, void* stream) {
    return guard([&] {
        AT_REQUIRE(ctx, AT_ERR_INVALID_ARG, "null context");
        ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
    });
}

int at_alloc(at_ctx* ctx, size_t bytes, void** dptr) {
    return guard([&] {
        AT_REQUIRE(ctx && dptr, AT_ERR_INVALID_ARG, "null argument");
        AT_CUDA(cudaSetDevice(ctx->device));
        AT_CUDA(cudaMalloc(dptr, bytes ? bytes : 16));
    });
}

int at_free(at_ctx* ctx, void* dptr) {
    return guard([&] {
        AT_REQUIRE(ctx, AT_ERR_INVALID_ARG, "null context");
        if (dptr) AT_CUDA(cudaFree(dptr));
    });
}

int at_memcpy_h2d(at_ctx* ctx, void* dst, const void* src, size_t bytes) {
    return guard([&] {
        AT_REQUIRE(ctx && (bytes == 0 || (dst && src)), AT_ERR_INVALID_ARG, "null argument");
        AT_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
        AT_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int at_memcpy_d2h(at_ctx* ctx, void* dst, const void* src, size_t bytes) {
    return guard([&] {
        AT_REQUIRE(ctx && (bytes == 0 || (dst && src)), AT_ERR_INVALID_ARG, "null argument");
        AT_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
        AT_CUDA(cudaStreamSynchronize(ctx->stream));
    });
}

int at_memset_zero(at_ctx* ctx, void* dst, size_t bytes) {
    return guard([&] {
        AT_REQUIRE(ctx && (bytes == 0 || dst), AT_ERR_INVALID_ARG, "null argument");
        AT_CUDA(cudaMemsetAsync(dst, 0, bytes, ctx->stream));
    });
}

int at_fp16_to_f32(at_ctx* ctx, const uint16_t* src, float* dst, int64_t n) {
    return guard([&] {
        AT_REQUIRE(ctx && n >= 0 && (n == 0 || (src && dst)), AT_ERR_INVALID_ARG, "bad argument");
        if (n == 0) return;
        fp16_to_f32_kernel<<<grid_for(n), TPB, 0, ctx->stream>>>(src, dst, n);
        AT_CUDA(cudaGetLastError());
    });
}

static void check_blocks(at_ctx* ctx, const void* src, const void* dst, int64_t n) {
    AT_REQUIRE(ctx, AT_ERR_INVALID_ARG, "null context");
    AT_REQUIRE(n >= 0, AT_ERR_INVALID_ARG, "negative element count");
    AT_REQUIRE(n % QK == 0, AT_ERR_INVALID_ARG, "element count must be a multiple of 32");
    AT_REQUIRE(n == 0 || (src && dst), AT_ERR_INVALID_ARG, "null buffer");
}

int at_q4_0_dequant(at_ctx* ctx, const void* src, float* dst, int64_t n) {
    return guard([&] {
        check_blocks(ctx, src, dst, n);
        if (!n) return;
        dequant_kernel<AT_GGML_Q4_0><<<grid_for(n), TPB, 0, ctx->stream>>>((const uint8_t*)src, dst, n);
        AT_CUDA(cudaGetLastError());
    });
}

int at_q8_0_dequant(at_ctx* ctx, const void* src, float* dst, int64_t n) {
    return guard([&] {
        check_blocks(ctx, src, dst, n);
        if (!n) return;
        dequant_kernel<AT_GGML_Q8_0><<<grid_for(n), TPB, 0, ctx->stream>>>((const uint8_t*)src, dst, n);
        AT_CUDA(cudaGetLastError());
    });
}

int at_q6_k_dequant(at_ctx* ctx, const void* src, float* dst, int64_t n) {
    return guard([&] {
        AT_REQUIRE(ctx, AT_ERR_INVALID_ARG, "null context");
        AT_REQUIRE(n >= 0 && n % 256 == 0, AT_ERR_INVALID_ARG, "element count must be a multiple of 256");
        AT_REQUIRE(n == 0 || (src && dst), AT_ERR_INVALID_ARG, "null buffer");
        if (!n) return;
        launch_q6k_dequant((const uint8_t*)src, dst, n, ctx->stream);
    });
}
int at_q4_0_dot(at_ctx* ctx, const void* q4, const float* x, int64_t n, float* out) {
    return guard([&] {
        check_blocks(ctx, q4, out, n);
        AT_REQUIRE(n == 0 || x, AT_ERR_INVALID_ARG, "null x");
        qdot_kernel<AT_GGML_Q4_0><<<1, 1024, 0, ctx->stream>>>((const uint8_t*)q4, x, n, out);
        AT_CUDA(cudaGetLastError());
    });
}

int at_q8_0_dot(at_ctx* ctx, const void* q8, const float* x, int64_t n, float* out) {
    return guard([&] {
        check_blocks(ctx, q8, out, n);
        AT_REQUIRE(n == 0 || x, AT_ERR_INVALID_ARG, "null x");
        qdot_kernel<AT_GGML_Q8_0><<<1, 1024, 0, ctx->stream>>>((const uint8_t*)q8, x, n, out);
        AT_CUDA(cudaGetLastError());
    });
}

int at_qmat_create(at_ctx* ctx, int type, int orient, int64_t rows, int64_t cols, const void* blocks,
                   int on_device, at_qmat** out) {
    return at_qmat_create_ex(ctx, type, orient, 0, rows, cols, blocks, on_device, out);
}
int at_qmat_create_ex(at_ctx* ctx, int type, int orient, int layout, int64_t rows, int64_t cols, const void* blocks,
                      int on_device, at_qmat** out) {
    at_qmat* m = nullptr;
    void* staging = nullptr;
    const int rc = guard([&] {
        AT_REQUIRE(ctx && out && blocks, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(rows > 0 && cols > 0, AT_ERR_INVALID_ARG, "dims must be positive");
        AT_REQUIRE(orient == AT_ORIENT_N || orient == AT_ORIENT_T, AT_ERR_INVALID_ARG, "bad orientation");
        AT_REQUIRE((layout & ~AT_LAYOUT_LLAMA_CPP) == 0, AT_ERR_INVALID_ARG, "unknown layout bits");
        AT_CUDA(cudaSetDevice(ctx->device));
        m = new at_qmat();
        m->ctx = ctx;
        m->type = type;
        m->orient = orient;
        m->rows = rows;
        m->cols = cols;
        const int src_type = type;
        qmat_alloc(m);
        size_t bytes;
        if (src_type == AT_GGML_F32) bytes = (size_t)(rows * cols) * 4;
        else if (src_type == AT_GGML_F16) bytes = (size_t)(rows * cols) * 2;
        else bytes = (size_t)(rows * raw_bytes(type, cols));
        const void* src = blocks;
        if (!on_device) {
            AT_CUDA(cudaMalloc(&staging, bytes));
            AT_CUDA(cudaMemcpyAsync(staging, blocks, bytes, cudaMemcpyHostToDevice, ctx->stream));
            src = staging;
        }
        if (m->type == AT_GGML_F32) qmat_fill_from_float(m, src, src_type, cols, 0, 0, ctx->stream);
        else qmat_fill_region(m, (const uint8_t*)src, cols, 0, 0, rows, cols, 0, 0, ctx->stream,
                              layout & AT_LAYOUT_Q4_SPLIT_HALVES);
        AT_CUDA(cudaStreamSynchronize(ctx->stream));
        *out = m;
    });
    if (staging) cudaFree(staging);
    if (rc != AT_OK && m) {
        qmat_free(m);
        delete m;
    }
    return rc;
}

int at_qmat_destroy(at_qmat* m) {
    return guard([&] {
        if (!m) return;
        qmat_free(m);
        delete m;
    });
}

int at_qmat_export(at_ctx* ctx, const at_qmat* m, void* dst) {
    return guard([&] {
        AT_REQUIRE(ctx && m && dst, AT_ERR_INVALID_ARG, "null argument");
        if (m->type == AT_GGML_F32) {
            AT_CUDA(cudaMemcpyAsync(dst, m->f32, (size_t)(m->rows * m->cols) * 4, cudaMemcpyDeviceToDevice,
                                    ctx->stream));
            return;
        }
        if (m->type == AT_GGML_Q6_K) {
            q6k_export(m, (uint8_t*)dst, ctx->stream);
            return;
        }
        const int64_t nb = m->cols / QK;
        unpack_kernel<<<grid_for(m->rows * nb), TPB, 0, ctx->stream>>>(
            m->tiles, tile_map(m), block_bytes(m->type), quant_bytes(m->type), m->rows, nb, (uint8_t*)dst);
        AT_CUDA(cudaGetLastError());
    });
}

// Scratch buffer for split launches made through at_gemv.
struct GemvScratch {
    float* buf = nullptr;
    unsigned* counters = nullptr;
    size_t floats = 0, ncounters = 0;
};
static std::mutex g_scratch_mu;

int at_gemv(at_ctx* ctx, const at_qmat* m, const float* x, float* y, int batch) {
    return guard([&] {
        AT_REQUIRE(ctx && m && x && y, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(batch >= 1 && batch <= 8, AT_ERR_INVALID_ARG, "batch must be in [1, 8]");
        AT_REQUIRE(((uintptr_t)x & 15) == 0, AT_ERR_INVALID_ARG, "x must be 16-byte aligned");
        const int64_t in = (m->orient == AT_ORIENT_N) ? m->cols : m->rows;
        const int64_t outn = (m->orient == AT_ORIENT_N) ? m->rows : m->cols;
        if (m->type == AT_GGML_F32) {
            if (m->orient == AT_ORIENT_N) {
                launch_sgemv_f32(m->f32, x, y, (int)m->rows, (int)m->cols, batch, (int)m->cols, ctx->stream);
            } else {
                sgemv_t_f32_kernel<<<grid_for(m->cols), TPB, 0, ctx->stream>>>(m->f32, x, y, (int)m->rows,
                                                                                (int)m->cols, batch);
                AT_CUDA(cudaGetLastError());
            }
            return;
        }
        GemvArgs a;
        a.x = x;
        a.y = y;
        a.x_stride = (int)in;
        a.y_stride = (int)outn;
        static GemvScratch sc;  // shared by at_gemv calls; calls are serialized by the stream
        size_t nf = 0, nc = 0;
        if (m->orient == AT_ORIENT_N) gemv_n_scratch_need(m, batch, ctx->num_sms, &nf, &nc);
        else gemv_t_scratch_need(m, batch, ctx->num_sms, &nf, &nc);
        {
            std::lock_guard<std::mutex> lk(g_scratch_mu);
            if (nf > sc.floats) {
                AT_CUDA(cudaStreamSynchronize(ctx->stream));
                if (sc.buf) cudaFree(sc.buf);
                AT_CUDA(cudaMalloc(&sc.buf, nf * 4));
                sc.floats = nf;
            }
            if (nc > sc.ncounters) {
                AT_CUDA(cudaStreamSynchronize(ctx->stream));
                if (sc.counters) cudaFree(sc.counters);
                AT_CUDA(cudaMalloc(&sc.counters, nc * 4));
                AT_CUDA(cudaMemset(sc.counters, 0, nc * 4));
                sc.ncounters = nc;
            }
        }
        a.scratch = sc.buf;
        a.counters = sc.counters;
        if (m->orient == AT_ORIENT_N) launch_gemv_n(m, batch, Pro::Plain, Epi::Plain, a, ctx->num_sms, ctx->stream);
        else launch_gemv_t(m, batch, Pro::Plain, Epi::Plain, a, ctx->num_sms, ctx->stream);
    });
}

int at_gemm_tc(at_ctx* ctx, const at_qmat* m, const float* x, float* y, int tokens) {
    return guard([&] {
        AT_REQUIRE(ctx && m && x && y, AT_ERR_INVALID_ARG, "null argument");
        AT_REQUIRE(tokens >= 1, AT_ERR_INVALID_ARG, "tokens must be positive");
        AT_REQUIRE(m->type == AT_GGML_Q4_0 || m->type == AT_GGML_Q8_0, AT_ERR_UNSUPPORTED,
                   "tensor-core GEMM supports Q4_0 and Q8_0");
        const int64_t in = (m->orient == AT_ORIENT_N) ? m->cols : m->rows;
        const int64_t outn = (m->orient == AT_ORIENT_N) ? m->rows : m->cols;
        AT_CUDA(cudaSetDevice(ctx->device));
        // per-device error word and bf16 staging buffer, grown on demand (calls are stream-serialized)
        static std::mutex mu;
        static int* d_err[64] = {};
        static void* xbf[64] = {};
        static size_t xbf_bytes[64] = {};
        static float* ws[64] = {};
        static size_t ws_bytes[64] = {};
        AT_REQUIRE(ctx->device < 64, AT_ERR_INVALID_ARG, "device index");
        const size_t need = (size_t)tokens * in * 2;
        {
            std::lock_guard<std::mutex> lk(mu);
            if (!d_err[ctx->device]) {
                AT_CUDA(cudaMalloc(&d_err[ctx->device], sizeof(int)));
                AT_CUDA(cudaMemset(d_err[ctx->device], 0, sizeof(int)));
            }
            if (xbf_bytes[ctx->device] < need) {
                AT_CUDA(cudaStreamSynchronize(ctx->stream));
                if (xbf[ctx->device]) cudaFree(xbf[ctx->device]);
                AT_CUDA(cudaMalloc(&xbf[ctx->device], need));
                xbf_bytes[ctx->device] = need;
            }
            const size_t wneed = (size_t)gemm_tc_splits(m, tokens, ctx->num_sms) * tokens * outn * 4;
            if (ws_bytes[ctx->device] < wneed) {
                AT_CUDA(cudaStreamSynchronize(ctx->stream));
                if (ws[ctx->device]) cudaFree(ws[ctx->device]);
                AT_CUDA(cudaMalloc(&ws[ctx->device], wneed));
                ws_bytes[ctx->device] = wneed;
            }
        }
        launch_gemm_tc(m, x, (int)in, y, (int)outn, tokens, xbf[ctx->device], xbf_bytes[ctx->device],
                       ws[ctx->device], ws_bytes[ctx->device], ctx->num_sms, d_err[ctx->device], ctx->stream);
        int err = 0;
        AT_CUDA(cudaMemcpyAsync(&err, d_err[ctx->device], sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
        AT_CUDA(cudaStreamSynchronize(ctx->stream));
        AT_REQUIRE(err == 0, AT_ERR_CUDA, "tensor-core GEMM: an mbarrier wait ran out");
    });
}

int at_sgemv(at_ctx* ctx, const float* A, const float* x, float* y, int M, int K) {
    return guard([&] {
        AT_REQUIRE(ctx && A && x && y, AT_ERR_INVALID_ARG, "sgemv: null argument");
        AT_REQUIRE(M > 0 && K > 0, AT_ERR_INVALID_ARG, "sgemv: dim mismatch");
        launch_sgemv_f32(A, x, y, M, K, 1, K, ctx->stream);
    });
}

int at_sgemm(at_ctx* ctx, const float* A, const float* B, float* C, int M, int K, int N) {
    return guard([&] {
        AT_REQUIRE(ctx && A && B && C, AT_ERR_INVALID_ARG, "sgemm: null argument");
        AT_REQUIRE(M > 0 && K > 0 && N > 0, AT_ERR_INVALID_ARG, "sgemm: dim mismatch");
        dim3 grid((N + 127) / 128, M);
        sgemm_kernel<<<grid, 128, 0, ctx->stream>>>(A, B, C, M, K, N);
        AT_CUDA(cudaGetLastError());
    });
}

int at_rmsnorm(at_ctx* ctx, float* x, const float* w, float eps, int rows, int d) {
    return guard([&] {
        AT_REQUIRE(ctx && x && w, AT_ERR_INVALID_ARG, "rmsNorm: null argument");
        AT_REQUIRE(rows > 0 && d > 0, AT_ERR_INVALID_ARG, "rmsNorm requires positive dims");
        rmsnorm_kernel<<<rows, 256, 0, ctx->stream>>>(x, w, eps, d);
        AT_CUDA(cudaGetLastError());
    });
}

int at_softmax(at_ctx* ctx, float* x, int rows, int n) {
    return guard([&] {
        AT_REQUIRE(ctx && x, AT_ERR_INVALID_ARG, "softmax: null argument");
        AT_REQUIRE(rows > 0 && n > 0, AT_ERR_INVALID_ARG, "softmax requires positive dims");
        softmax_kernel<<<rows, 256, 0, ctx->stream>>>(x, n);
        AT_CUDA(cudaGetLastError());
    });
}

int at_rope(at_ctx* ctx, float* qk, const float* cs, const float* sn, int head_dim, int n) {
    return guard([&] {
        AT_REQUIRE(ctx && qk && cs && sn, AT_ERR_INVALID_ARG, "rope: null argument");
        AT_REQUIRE(head_dim > 0 && head_dim % 2 == 0, AT_ERR_INVALID_ARG, "rope: headDim must be even");
        AT_REQUIRE(n % head_dim == 0, AT_ERR_INVALID_ARG,
                   "ropeInPlaceSegment: n " + std::to_string(n) + " is not a multiple of headDim " +
                       std::to_string(head_dim));
        if (n == 0) return;
        rope_kernel<<<grid_for(n / 2), TPB, 0, ctx->stream>>>(qk, cs, sn, head_dim, n);
        AT_CUDA(cudaGetLastError());
    });
}

int at_silu(at_ctx* ctx, float* x, int64_t n) {
    return guard([&] {
        AT_REQUIRE(ctx && (n == 0 || x), AT_ERR_INVALID_ARG, "silu: null argument");
        AT_REQUIRE(n >= 0, AT_ERR_INVALID_ARG, "silu: negative length");
        if (n == 0) return;
        silu_kernel<<<grid_for(n), TPB, 0, ctx->stream>>>(x, n);
        AT_CUDA(cudaGetLastError());
    });
}

}  // extern "C"
