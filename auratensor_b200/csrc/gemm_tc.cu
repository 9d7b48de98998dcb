// Batched fused-dequant GEMM on the 5th-generation tensor cores (tcgen05),
// for prompt processing: Y[t][o] = sum_k X[t][k] * W[o][k] over T tokens.
//
// The reference processes a prompt one token at a time (forwardPrompt,
// inference/LlamaModel.java:166-175, each token a forwardStep over FP32
// weights). Here every projection of a chunk of up to 128 tokens is one GEMM
// whose operands are bf16 (the prompt path's tolerance is 2e-2 of the logit
// range): the weight tile is dequantized from the resident Q4_0 / Q8_0 tiles
// ((q - 8) * d, or q * d, rounded once to bf16) straight into shared memory,
// the activations are rounded to bf16 on the way in, and products are summed
// in FP32 in tensor memory.
//
// CTA tile: 128 outputs (MMA M) x 128 tokens (MMA N), K in steps of 64.
// Both operands are K-major in the canonical 128-byte-swizzled layout: row r
// of a tile is 128 bytes (64 bf16) at (r / 8) * 1024 + (r % 8) * 128, and
// its 16-byte chunk c is stored at chunk position c ^ (r % 8). One elected
// thread issues four tcgen05.mma (K = 16 each) per step and commits them to
// the stage's mbarrier; two stages let the warps dequantize step s + 1 while
// the tensor core works on step s. The 128 x 128 FP32 accumulator lives in
// 128 TMEM columns; the epilogue reads it with tcgen05.ld (warp w reads TMEM
// lanes 32 (w % 4) ..) and stores FP32 rows of Y.
//
// Every wait on an mbarrier is bounded; a wait that runs out records an error
// code, stops issuing, and the CTA still frees its TMEM before returning.
#include <cuda_bf16.h>

#include <cstdint>

#include "at_internal.h"
#include "dev_common.cuh"

namespace at {

namespace {

constexpr int TC_M = 128;        // outputs per CTA (MMA M)
constexpr int TC_N = 128;        // tokens per CTA (MMA N)
constexpr int TC_K = 64;         // K per pipeline step (one 128-byte swizzle row)
constexpr int TC_THREADS = 256;  // 8 warps
constexpr int TC_TILE_BYTES = TC_M * TC_K * 2;  // 16 KB per operand tile (TC_N == TC_M)
constexpr int TC_STAGES = 2;
constexpr int TC_SMEM = TC_STAGES * 2 * TC_TILE_BYTES + 1024;  // + alignment slack
constexpr uint32_t TC_TMEM_COLS = 128;
constexpr int kTcSpinLimit = 1 << 26;

// Instruction descriptor of tcgen05.mma kind::f16: D f32 (bits 4-5 = 1),
// A and B bf16 (bits 7-9 = 1, 10-12 = 1), both K-major (bits 15, 16 = 0),
// N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t make_idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
static_assert(make_idesc_bf16(128, 128) == 0x08200490u, "tcgen05 instruction descriptor");

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: start address
// >> 4 (bits 0-13), leading byte offset 16 B (encoded 1, unused for this
// layout), stride byte offset 1024 B between 8-row groups (encoded 64, bits
// 32-45), version 1 (bit 46), layout type 2 = SWIZZLE_128B (bits 61-63). The
// tile base is 1024-byte aligned (base offset 0).
__host__ __device__ constexpr uint64_t make_sdesc_sw128(uint32_t smem_addr) {
    return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
static_assert(make_sdesc_sw128(0) == 0x4000404000010000ull, "tcgen05 shared-memory descriptor");

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Byte offset of the 16-byte chunk c (0..7) of row r in a swizzled tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait; false when the limit ran out.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (int it = 0; it < kTcSpinLimit; ++it)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 consecutive FP32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float* v) {
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

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);  // a -> low half (lower address)
    return *reinterpret_cast<const uint32_t*>(&h);
}

struct TcParams {
    const uint8_t* tiles;
    QTileMap map;
    int qtype, orient;
    int M;        // outputs
    int K;        // inputs (multiple of 64)
    int T;        // tokens
    const float* x;  // [T][x_stride]
    int x_stride;
    float* y;        // [T][y_stride]
    int y_stride;
    int* err;
};

// Dequantizes W[m0 .. m0+127][k0 .. k0+63] into a swizzled bf16 tile.
__device__ __forceinline__ void fill_a(uint8_t* tile, const TcParams& p, int m0, int k0) {
    const int tid = threadIdx.x;
    if (p.orient == AT_ORIENT_N) {
        // thread = (row r, half j): 32 weights of block (m0 + r, k0/32 + j), 4 chunks of 8
        const int r = tid >> 1, j = tid & 1;
        const int m = m0 + r;
        uint32_t w[16];
        if (m < p.M) {
            int64_t d_off, q_off;
            p.map.offsets(m, (k0 >> 5) + j, &d_off, &q_off);
            const float d = fp16_ftz((uint32_t)p.tiles[d_off] | ((uint32_t)p.tiles[d_off + 1] << 8));
            if (p.qtype == AT_GGML_Q4_0) {
                const uint4 q = *reinterpret_cast<const uint4*>(p.tiles + q_off);
                const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int i = 0; i < 16; ++i) {  // byte i: elements 2i (low nibble), 2i + 1 (high nibble)
                    const uint32_t byte = (qw[i >> 2] >> (8 * (i & 3))) & 0xFFu;
                    w[i] = pack_bf16(__fmul_rn((float)((int)(byte & 15u) - 8), d), __fmul_rn((float)((int)(byte >> 4) - 8), d));
                }
            } else {
                const uint4 q0 = *reinterpret_cast<const uint4*>(p.tiles + q_off);
                const uint4 q1 = *reinterpret_cast<const uint4*>(p.tiles + q_off + 16);
                const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (int i = 0; i < 16; ++i) {  // elements 2i, 2i + 1
                    const uint32_t word = qw[i >> 1];
                    const int sh = 16 * (i & 1);
                    const float a = (float)(int8_t)((word >> sh) & 0xFFu), b = (float)(int8_t)((word >> (sh + 8)) & 0xFFu);
                    w[i] = pack_bf16(__fmul_rn(a, d), __fmul_rn(b, d));
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = 0u;
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(tile + sw128_off(r, 4 * j + c)) =
                make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
    } else {
        // orientation T: stored rows are inputs k, blocks run along the outputs.
        // thread = (k, output block cb): 32 outputs m0 + 32 cb .. at input k0 + k
        const int k = tid & 63, cb = tid >> 6;
        const int kk = k0 + k;
        const int mb = (m0 >> 5) + cb;
        float v[32];
        if (mb * 32 < p.M && kk < p.K) {
            int64_t d_off, q_off;
            p.map.offsets(kk, mb, &d_off, &q_off);
            const float d = fp16_ftz((uint32_t)p.tiles[d_off] | ((uint32_t)p.tiles[d_off + 1] << 8));
            if (p.qtype == AT_GGML_Q4_0) {
                const uint4 q = *reinterpret_cast<const uint4*>(p.tiles + q_off);
                const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const uint32_t byte = (qw[i >> 2] >> (8 * (i & 3))) & 0xFFu;
                    v[2 * i] = __fmul_rn((float)((int)(byte & 15u) - 8), d);
                    v[2 * i + 1] = __fmul_rn((float)((int)(byte >> 4) - 8), d);
                }
            } else {
                const uint4 q0 = *reinterpret_cast<const uint4*>(p.tiles + q_off);
                const uint4 q1 = *reinterpret_cast<const uint4*>(p.tiles + q_off + 16);
                const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __fmul_rn((float)(int8_t)((qw[i >> 2] >> (8 * (i & 3))) & 0xFFu), d);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
        const int c = k >> 3, e = k & 7;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const int r = 32 * cb + i;
            *reinterpret_cast<__nv_bfloat16*>(tile + sw128_off(r, c) + 2 * e) = __float2bfloat16_rn(v[i]);
        }
    }
}

// Rounds X[t0 .. t0+127][k0 .. k0+63] to bf16 into a swizzled tile (zero rows past T).
__device__ __forceinline__ void fill_b(uint8_t* tile, const TcParams& p, int t0, int k0) {
    const int tid = threadIdx.x;
    const int r = tid >> 1, j = tid & 1;  // token row, 32-element half
    const int t = t0 + r;
    uint32_t w[16];
    if (t < p.T) {
        const float4* xs = reinterpret_cast<const float4*>(p.x + (size_t)t * p.x_stride + k0 + 32 * j);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 f = xs[i];
            w[2 * i] = pack_bf16(f.x, f.y);
            w[2 * i + 1] = pack_bf16(f.z, f.w);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = 0u;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(tile + sw128_off(r, 4 * j + c)) =
            make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

__global__ void __launch_bounds__(TC_THREADS, 1) gemm_tc_kernel(const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t s_bar[TC_STAGES];
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * TC_M, t0 = blockIdx.y * TC_N;
    // 1024-byte aligned stage buffers: [stage][A tile | B tile]
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int s = 0; s < TC_STAGES; ++s) mbar_init(smem_u32(&s_bar[s]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_fail = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    constexpr uint32_t idesc = make_idesc_bf16(TC_M, TC_N);

    const int nk = p.K / TC_K;
    bool ok = true;
    for (int ks = 0; ks < nk; ++ks) {
        const int st = ks & 1;
        uint8_t* a_tile = base + st * 2 * TC_TILE_BYTES;
        uint8_t* b_tile = a_tile + TC_TILE_BYTES;
        if (ks >= TC_STAGES) {
            // the MMAs that read this stage two steps ago are complete
            if (!mbar_wait(smem_u32(&s_bar[st]), ((ks - TC_STAGES) / TC_STAGES) & 1)) {
                ok = false;
                if (tid == 0) atomicExch(p.err, 2);
            }
        }
        if (__syncthreads_or(!ok)) { ok = false; break; }
        fill_a(a_tile, p, m0, ks * TC_K);
        fill_b(b_tile, p, t0, ks * TC_K);
        // generic-proxy stores -> visible to the tensor core's async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t a_addr = smem_u32(a_tile), b_addr = smem_u32(b_tile);
#pragma unroll
            for (int kk = 0; kk < TC_K / 16; ++kk)  // 16 bf16 = 32 bytes per MMA along K
                tc_mma(tmem, make_sdesc_sw128(a_addr + 32 * kk), make_sdesc_sw128(b_addr + 32 * kk), idesc,
                       (ks > 0 || kk > 0) ? 1u : 0u);
            tc_commit(smem_u32(&s_bar[st]));
        }
    }
    // all MMAs complete (the last commit covers every earlier one)
    if (ok && nk > 0) {
        const int last = nk - 1;
        if (!mbar_wait(smem_u32(&s_bar[last & 1]), (last / TC_STAGES) & 1)) {
            ok = false;
            if (tid == 0) atomicExch(p.err, 2);
        }
    }
    if (__syncthreads_or(!ok)) ok = false;
    tc_fence_after();

    if (ok) {
        // warp w reads TMEM lanes 32 (w % 4) .. + 31 (outputs), columns 64 (w / 4) .. + 63 (tokens)
        const int quarter = warp & 3, half = warp >> 2;
        const int m = m0 + 32 * quarter + lane;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            const int col = 64 * half + 32 * cc;
            float v[32];
            tc_ld32(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)col, v);
            if (m < p.M) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int t = t0 + col + i;
                    if (t < p.T) p.y[(size_t)t * p.y_stride + m] = v[i];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS) : "memory");
}

}  // namespace

void launch_gemm_tc(const at_qmat* m, const float* x, int x_stride, float* y, int y_stride, int T, int* err,
                    cudaStream_t s) {
    AT_REQUIRE(m->type == AT_GGML_Q4_0 || m->type == AT_GGML_Q8_0, AT_ERR_UNSUPPORTED,
               "tensor-core GEMM supports Q4_0 and Q8_0");
    const int64_t M = (m->orient == AT_ORIENT_N) ? m->rows : m->cols;
    const int64_t K = (m->orient == AT_ORIENT_N) ? m->cols : m->rows;
    AT_REQUIRE(K % TC_K == 0, AT_ERR_INVALID_ARG, "tensor-core GEMM needs K a multiple of 64");
    AT_REQUIRE(T >= 1 && x_stride % 4 == 0 && ((uintptr_t)x & 15) == 0, AT_ERR_INVALID_ARG,
               "tensor-core GEMM: bad activation layout");
    TcParams p{};
    p.tiles = m->tiles;
    p.map = tile_map(m);
    p.qtype = m->type;
    p.orient = m->orient;
    p.M = (int)M;
    p.K = (int)K;
    p.T = T;
    p.x = x;
    p.x_stride = x_stride;
    p.y = y;
    p.y_stride = y_stride;
    p.err = err;
    static bool attr_set = false;
    if (!attr_set) {
        AT_CUDA(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM));
        attr_set = true;
    }
    dim3 grid((unsigned)((M + TC_M - 1) / TC_M), (unsigned)((T + TC_N - 1) / TC_N));
    gemm_tc_kernel<<<grid, TC_THREADS, TC_SMEM, s>>>(p);
    AT_CUDA(cudaGetLastError());
}

}  // namespace at
