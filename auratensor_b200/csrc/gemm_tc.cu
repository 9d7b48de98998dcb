// Batched fused-dequant GEMM on the 5th-generation tensor cores (tcgen05),
// for prompt processing: Y[t][o] = sum_k X[t][k] * W[o][k] over T tokens.
//
// The reference processes a prompt one token at a time (forwardPrompt,
// inference/LlamaModel.java:166-175, each token a forwardStep over FP32
// weights). Here every projection of a chunk of up to 512 tokens is one GEMM
// whose operands are bf16 (the prompt path's tolerance is 2e-2 of the logit
// range): the weight tile is dequantized from the resident Q4_0 / Q8_0 tiles
// ((q - 8) * d, or q * d, rounded once to bf16) straight into shared memory,
// the activations are rounded to bf16 on the way in, and products are summed
// in FP32 in tensor memory.
//
// CTA tile: 128 outputs (MMA M) x 256 or 512 tokens (NB token tiles of MMA
// N = 256, one TMEM accumulator each), K in steps of 64, so a dequantized
// weight tile feeds up to 512 tokens: the dequant warps, not the tensor pipe,
// bound the 256-token form.
// The token tile and the orientation-N weight tile are K-major in the
// canonical 128-byte-swizzled layout: row r of a tile is 128 bytes (64 bf16)
// at (r / 8) * 1024 + (r % 8) * 128, and its 16-byte chunk c is stored at
// chunk position c ^ (r % 8). An orientation-T block holds 32 consecutive
// outputs of one input, so that weight tile is M-major (the same swizzle with
// the roles of outputs and inputs exchanged) and every thread still stores
// 16-byte chunks. The token
// tile (bf16 activations) arrives by TMA (cp.async.bulk.tensor with the
// 128-byte swizzle, rows past the last token zero-filled), one step ahead,
// completing on the stage's "full" mbarrier; the weight tile is dequantized
// by one of two groups of 8 warps (alternate steps) from raw block bytes
// loaded into registers three (Q8_0: two) of the group's steps ahead.
// One thread issues four tcgen05.mma (K = 16 each) per token tile and step
// and commits them to the stages' "empty" mbarriers. The weight tiles and the
// token tiles have rings of their own: four weight stages, and four 32 KB
// (NB = 1) or two 64 KB (NB = 2) token stages, so the TMA, the dequant and
// the tensor core work on different steps within 192 KB of shared memory.
// The 128 x 256 NB FP32 accumulator lives in 256 NB TMEM columns; the
// epilogue reads it with tcgen05.ld (warp w reads TMEM lanes 32 (w % 4) ..)
// and stores FP32 rows of Y.
//
// Every wait on an mbarrier is bounded; a wait that runs out records an error
// code, stops issuing, drains the token-tile copies still in flight, and the
// CTA still frees its TMEM before returning.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>

#include "at_internal.h"
#include "dev_common.cuh"

namespace at {

namespace {

constexpr int TC_M = 128;        // outputs per CTA (MMA M)
constexpr int TC_N = 256;        // tokens per CTA (MMA N)
constexpr int TC_K = 64;         // K per pipeline step (one 128-byte swizzle row)
constexpr int TC_DQ_WARPS = 8;   // warps that dequantize one weight tile (256 threads, one block each)
constexpr int TC_DQ_GROUPS = 2;  // such groups, taking alternate K steps
constexpr int TC_THREADS_WS = 64 + 32 * TC_DQ_WARPS * TC_DQ_GROUPS;  // + a TMA warp and an MMA warp
constexpr int TC_TILE_BYTES = TC_M * TC_K * 2;  // 16 KB weight tile
constexpr int TC_B_BYTES = TC_N * TC_K * 2;     // 32 KB token tile
constexpr int TC_A_STAGES = 4;                  // weight-tile ring
// token-tile ring of NB tiles per stage, and the dynamic shared memory
template <int NB>
constexpr int tc_b_stages() { return NB == 1 ? 4 : 2; }
template <int NB>
constexpr int tc_smem() { return TC_A_STAGES * TC_TILE_BYTES + tc_b_stages<NB>() * NB * TC_B_BYTES + 1024; }
static_assert(tc_smem<1>() <= 227 * 1024 && tc_smem<2>() <= 227 * 1024, "shared memory per CTA");
constexpr int kTcSpinLimit = 1 << 22;
constexpr int kTcMaxSplits = 4;

// Instruction descriptor of tcgen05.mma kind::f16: D f32 (bits 4-5 = 1),
// A and B bf16 (bits 7-9 = 1, 10-12 = 1), both K-major (bits 15, 16 = 0),
// N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t make_idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
static_assert(make_idesc_bf16(128, 128) == 0x08200490u, "tcgen05 instruction descriptor");
static_assert(make_idesc_bf16(TC_M, TC_N) == 0x08400490u, "tcgen05 instruction descriptor, N = 256");

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: start address
// >> 4 (bits 0-13), leading byte offset 16 B (encoded 1, unused for this
// layout), stride byte offset 1024 B between 8-row groups (encoded 64, bits
// 32-45), version 1 (bit 46), layout type 2 = SWIZZLE_128B (bits 61-63). The
// tile base is 1024-byte aligned (base offset 0).
__host__ __device__ constexpr uint64_t make_sdesc_sw128(uint32_t smem_addr) {
    return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
static_assert(make_sdesc_sw128(0) == 0x4000404000010000ull, "tcgen05 shared-memory descriptor");

// The same for an M-major (MN-major) A tile, 128-byte swizzle: a swizzle atom
// is 8 k-rows of 64 consecutive outputs (128 B each, 1024 B); the leading byte
// offset is the stride between the two 64-output atoms along M (1024 B,
// encoded 64, bits 16-29), the stride byte offset the stride between 8-row
// groups along K (2048 B, encoded 128). Used by orientation T, whose blocks
// run along the outputs.
__host__ __device__ constexpr uint64_t make_sdesc_sw128_mn(uint32_t smem_addr) {
    return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | (64ull << 16) | (128ull << 32) | (1ull << 46) | (2ull << 61);
}
static_assert(make_sdesc_sw128_mn(0) == 0x4000408000400000ull, "tcgen05 shared-memory descriptor, MN-major");
constexpr uint32_t kIdescTransposeA = 1u << 15;  // A is MN-major
constexpr uint32_t kIdesc = make_idesc_bf16(TC_M, TC_N);

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
    float* y;     // [T][y_stride], or with split K the partials [split][T][y_stride]
    int y_stride;
    int splits;   // CTAs along K (blockIdx.z); split z covers steps [z nk / splits, (z+1) nk / splits)
    int* err;
};

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// TMA: box {64 k, 256 tokens} at (k0, t0) of the bf16 activations -> swizzled smem tile.
__device__ __forceinline__ void tma_load_x(uint32_t dst, const CUtensorMap* map, int k0, int t0, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(k0), "r"(t0), "r"(bar)
        : "memory");
}

// Raw bytes of the one block a thread dequantizes per step (scale + 16 or 32 quant bytes).
struct RawBlock {
    uint4 q0, q1;
    uint32_t d;
};

// Step k0: N orientation, thread (row r = tid / 2, half j = tid % 2) owns block
// (m0 + r, k0/32 + j); T orientation, thread (k = tid % 64, cb = tid / 64) owns
// block (input row k0 + k, output block m0/32 + cb).
template <int QT, int OR>
__device__ __forceinline__ void load_block(RawBlock& rb, const TcParams& p, int m0, int k0, int tid) {
    int64_t row, blk;
    bool valid;
    if (OR == AT_ORIENT_N) {
        row = m0 + (tid >> 1);
        blk = (k0 >> 5) + (tid & 1);
        valid = row < p.M;
    } else {
        row = k0 + (tid & 63);
        blk = (m0 >> 5) + (tid >> 6);
        valid = blk * 32 < p.M;
    }
    if (!valid) {
        rb.d = 0u;
        rb.q0 = rb.q1 = make_uint4(0, 0, 0, 0);
        return;
    }
    int64_t d_off, q_off;
    p.map.offsets(row, blk, &d_off, &q_off);
    rb.d = *reinterpret_cast<const uint16_t*>(p.tiles + d_off);  // tiles keep each fp16 scale 2-byte aligned
    rb.q0 = *reinterpret_cast<const uint4*>(p.tiles + q_off);
    if (QT == AT_GGML_Q8_0) rb.q1 = *reinterpret_cast<const uint4*>(p.tiles + q_off + 16);
}

// The 32 weights of a raw block, (q - 8) * d or q * d in FP32, rounded to
// bf16 and packed in pairs in element order (pk[i] = elements 2i, 2i + 1). A
// nibble (byte) becomes the exact float q - 8 (q) by one byte permute into
// the mantissa of 2^23 and a packed f32x2 subtraction; then one rounding in
// the multiply by d and one to bf16.
template <int QT>
__device__ __forceinline__ void decode_block(const RawBlock& rb, uint32_t* pk) {
    const float d = fp16_ftz(rb.d);
    const float2 dd = f2(d, d);
    if (QT == AT_GGML_Q4_0) {
        const float2 moff = f2(-8388616.f, -8388616.f);  // -(2^23 + 8)
        const uint32_t qw[4] = {rb.q0.x, rb.q0.y, rb.q0.z, rb.q0.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = qw[i] & 0x0F0F0F0Fu, hi = (qw[i] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int k = 0; k < 4; ++k) {  // byte k of word i: elements 8i + 2k (low), 8i + 2k + 1 (high)
                const float2 w = __fmul2_rn(__fadd2_rn(f2(magic_byte(lo, k), magic_byte(hi, k)), moff), dd);
                pk[4 * i + k] = pack_bf16(w.x, w.y);
            }
        }
    } else {
        const float2 moff = f2(-8388736.f, -8388736.f);  // -(2^23 + 128)
        const uint32_t qw[8] = {rb.q0.x, rb.q0.y, rb.q0.z, rb.q0.w, rb.q1.x, rb.q1.y, rb.q1.z, rb.q1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t u = qw[i] ^ 0x80808080u;  // int8 q -> unsigned q + 128
            const float2 w01 = __fmul2_rn(__fadd2_rn(f2(magic_byte(u, 0), magic_byte(u, 1)), moff), dd);
            const float2 w23 = __fmul2_rn(__fadd2_rn(f2(magic_byte(u, 2), magic_byte(u, 3)), moff), dd);
            pk[2 * i] = pack_bf16(w01.x, w01.y);
            pk[2 * i + 1] = pack_bf16(w23.x, w23.y);
        }
    }
}

// Writes this thread's 32 dequantized weights (16 packed bf16 pairs) into the
// swizzled weight tile.
template <int OR>
__device__ __forceinline__ void store_block(uint8_t* tile, const uint32_t* pk, int tid) {
    if (OR == AT_ORIENT_N) {
        const int r = tid >> 1, j = tid & 1;  // 32 consecutive k of row r: chunks 4j .. 4j + 3
#pragma unroll
        for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(tile + sw128_off(r, 4 * j + c)) =
                make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
    } else {
        // 32 consecutive outputs (32 cb ..) at input k: half of k-row (k & 7) of
        // the M-major atom (k >> 3, cb >> 1), chunks 4 (cb & 1) .. + 3
        const int k = tid & 63, cb = tid >> 6, r = k & 7;
        uint8_t* row = tile + (k >> 3) * 2048 + (cb >> 1) * 1024 + r * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(row + (((4 * (cb & 1) + c) ^ r) << 4)) =
                make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
    }
}

// Steps of weight bytes in flight per dequant thread (registers): 3 Q4_0
// blocks (18 B each) or 2 Q8_0 blocks (34 B) within the register budget.
template <int QT>
constexpr int tc_pf() { return QT == AT_GGML_Q8_0 ? 2 : 3; }

// Warp roles: warp 0 issues the token tiles' TMA, warp 1 owns TMEM and issues
// the MMAs, warps 2-9 dequantize the weight tiles of even steps and warps
// 10-17 those of odd steps (256 threads, one block of 32 weights each per
// step). Per weight stage: full_a (8 warp arrivals after each warp's stores
// and proxy fence; the group's first warp arrives only after the step's
// full_b, so full_a alone gates the MMAs) and empty_a; per token stage:
// full_b (TMA bytes) and empty_b; both empties are the MMAs' commits. No
// CTA-wide barrier inside the K loop.
template <int QT, int OR, int NB>
// 18 warps put 5 on one of the SM's four 16,384-register partitions: at
// most 96 registers a thread. Templated on the quant type and orientation so
// that each instance holds only the registers it uses.
__global__ void __launch_bounds__(TC_THREADS_WS, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                   const TcParams p) {
    constexpr int AS = TC_A_STAGES, BS = tc_b_stages<NB>();
    constexpr uint32_t TMEM_COLS = TC_N * NB;  // FP32 accumulator columns
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t s_fa[AS], s_ea[AS], s_fb[BS], s_eb[BS], s_done;
    __shared__ uint32_t s_tmem;
    __shared__ int s_bad;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * TC_M, t0 = blockIdx.y * TC_N * NB;
    // token tiles of this CTA that hold tokens (the last CTA row may have one)
    const int nbv = (NB == 2 && t0 + TC_N < p.T) ? 2 : 1;
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    auto a_tile = [&](int st) { return base + st * TC_TILE_BYTES; };
    auto b_tile = [&](int st) { return base + AS * TC_TILE_BYTES + st * NB * TC_B_BYTES; };
    const int nk_all = p.K / TC_K;
    const int ks0 = (int)((int64_t)blockIdx.z * nk_all / p.splits);
    const int nk = (int)((int64_t)(blockIdx.z + 1) * nk_all / p.splits) - ks0;  // steps of this split
    const int kbase = ks0 * TC_K;
    float* yout = p.y + (size_t)blockIdx.z * p.T * p.y_stride;

    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int st = 0; st < AS; ++st) {
            mbar_init(smem_u32(&s_fa[st]), TC_DQ_WARPS);
            mbar_init(smem_u32(&s_ea[st]), 1);
        }
        for (int st = 0; st < BS; ++st) {
            mbar_init(smem_u32(&s_fb[st]), 1);
            mbar_init(smem_u32(&s_eb[st]), 1);
        }
        mbar_init(smem_u32(&s_done), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
        s_bad = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    auto fail = [&]() { atomicExch(p.err, 2); s_bad = 1; };
    int tma_issued = 0;  // token-tile loads issued (warp 0, lane 0)

    if (warp == 0) {
        // ---- token tiles by TMA ----
        if (lane == 0) {
            for (int ks = 0; ks < nk; ++ks) {
                const int st = ks % BS;
                if (ks >= BS && !mbar_wait(smem_u32(&s_eb[st]), ((ks - BS) / BS) & 1)) {
                    fail();
                    break;
                }
                mbar_expect_tx(smem_u32(&s_fb[st]), TC_B_BYTES * nbv);
                for (int nb = 0; nb < nbv; ++nb)
                    tma_load_x(smem_u32(b_tile(st) + nb * TC_B_BYTES), &xmap, kbase + ks * TC_K, t0 + nb * TC_N,
                               smem_u32(&s_fb[st]));
                ++tma_issued;
            }
        }
        __syncwarp();  // lanes 1-31 park here instead of spinning beside lane 0
    } else if (warp == 1) {
        // ---- MMA issue ----
        if (lane == 0) {
            constexpr bool mn = OR != AT_ORIENT_N;
            const uint32_t idesc = kIdesc | (mn ? kIdescTransposeA : 0u);
            for (int ks = 0; ks < nk; ++ks) {
                const int sa = ks % AS, sb = ks % BS;
                if (!mbar_wait(smem_u32(&s_fa[sa]), (ks / AS) & 1)) {  // full_a completes after full_b
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(a_tile(sa)), b_addr = smem_u32(b_tile(sb));
#pragma unroll
                for (int kk = 0; kk < TC_K / 16; ++kk) {  // 16 k per MMA: 32 B of a K-major row, 2 M-major row groups
                    const uint64_t ad =
                        mn ? make_sdesc_sw128_mn(a_addr + 4096 * kk) : make_sdesc_sw128(a_addr + 32 * kk);
                    for (int nb = 0; nb < nbv; ++nb)  // accumulator nb: tokens t0 + 256 nb ..
                        tc_mma(tmem + (uint32_t)(nb * TC_N), ad, make_sdesc_sw128(b_addr + nb * TC_B_BYTES + 32 * kk),
                               idesc, (ks > 0 || kk > 0) ? 1u : 0u);
                }
                tc_commit(smem_u32(&s_ea[sa]));
                tc_commit(smem_u32(&s_eb[sb]));
            }
            tc_commit(smem_u32(&s_done));  // arrives when every MMA above is complete
        }
        __syncwarp();
    } else {
        // ---- weight tiles: dequantize into swizzled bf16 ----
        // Group g (warps 2 + 8 g ..) takes steps g, g + 2, ...; with two
        // warps of each group per scheduler, one group's load and FP
        // latencies hide behind the other's work. The loop is unrolled by
        // PF so that slot j always holds the bytes of the same step
        // sequence: no register copy of a load still in flight (which would
        // wait for it) between issue and use.
        constexpr int G = TC_DQ_GROUPS, PF = tc_pf<QT>();
        const int grp = (warp - 2) / TC_DQ_WARPS, dt = (tid - 64) % (32 * TC_DQ_WARPS);
        RawBlock rb[PF];
#pragma unroll
        for (int i = 0; i < PF; ++i)
            if (grp + G * i < nk) load_block<QT, OR>(rb[i], p, m0, kbase + (grp + G * i) * TC_K, dt);
        bool stop = false;
        for (int kq = grp; kq < nk && !stop; kq += G * PF) {
#pragma unroll
            for (int j = 0; j < PF; ++j) {
                const int ks = kq + G * j;
                if (ks >= nk) break;
                const int st = ks % AS;
                uint32_t pk[16];
                decode_block<QT>(rb[j], pk);
                if (ks + G * PF < nk) load_block<QT, OR>(rb[j], p, m0, kbase + (ks + G * PF) * TC_K, dt);
                if (ks >= AS && !mbar_wait(smem_u32(&s_ea[st]), ((ks - AS) / AS) & 1)) {
                    if (lane == 0) fail();
                    stop = true;
                    break;
                }
                store_block<OR>(a_tile(st), pk, dt);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> async proxy
                __syncwarp();
                // The group's first warp also waits for the stage's token tile
                // before it arrives, so that the MMA thread waits on full_a
                // alone (one barrier round trip per step on its path).
                int bad = 0;
                if (lane == 0) {
                    if (dt < 32) bad = !mbar_wait(smem_u32(&s_fb[ks % BS]), (ks / BS) & 1);
                    if (bad) fail();
                    else asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&s_fa[st])) : "memory");
                }
                if (__shfl_sync(0xffffffffu, bad, 0)) {
                    stop = true;
                    break;
                }
            }
        }
    }

    // ---- epilogue: the accumulator (dequant warps 2-17: lanes 32 (w % 4) .., columns 64 ((w - 2) / 4) ..) ----
    bool ok = mbar_wait(smem_u32(&s_done), 0);
    if (!ok && tid == 0) atomicExch(p.err, 2);
    __syncthreads();
    ok = ok && (s_bad == 0);
    // After a failed wait the MMAs may not have consumed every token tile:
    // drain the loads still in flight (the latest one of each stage, bounded
    // waits) so that no copy lands in shared memory after the CTA exits.
    if (!ok && tid == 0)
        for (int ks = max(0, tma_issued - BS); ks < tma_issued; ++ks)
            mbar_wait(smem_u32(&s_fb[ks % BS]), (ks / BS) & 1);
    tc_fence_after();
    if (ok && warp >= 2) {
        constexpr int parts = TC_DQ_WARPS * TC_DQ_GROUPS / 4;  // warps sharing one TMEM lane quarter
        const int quarter = warp & 3, part = (warp - 2) >> 2;
        const int m = m0 + 32 * quarter + lane;
#pragma unroll 1
        for (int cc = 0; cc < TC_N * NB / (32 * parts); ++cc) {
            const int col = (TC_N * NB / parts) * part + 32 * cc;
            if (t0 + col >= p.T) break;  // the part's later columns hold no tokens either
            float v[32];
            tc_ld32(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)col, v);
            if (m < p.M) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int t = t0 + col + i;
                    if (t < p.T) yout[(size_t)t * p.y_stride + m] = v[i];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

// y[t][m] = sum over splits z (in order) of ws[z][t][m]; block row t,
// thread 4 consecutive m (VEC) or one.
template <bool VEC>
__global__ void splitk_sum_kernel(const float* __restrict__ ws, int splits, int T, int M, float* __restrict__ y,
                                  int y_stride) {
    const int t = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const size_t n = (size_t)T * M, r = (size_t)t * M;
    if constexpr (VEC) {
        if (4 * i >= M) return;
        float4 acc = *reinterpret_cast<const float4*>(ws + r + 4 * i);
        for (int z = 1; z < splits; ++z) {
            const float4 v = *reinterpret_cast<const float4*>(ws + z * n + r + 4 * i);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        *reinterpret_cast<float4*>(y + (size_t)t * y_stride + 4 * i) = acc;
    } else {
        if (i >= M) return;
        float acc = ws[r + i];
        for (int z = 1; z < splits; ++z) acc += ws[z * n + r + i];
        y[(size_t)t * y_stride + i] = acc;
    }
}

// FP32 activations -> bf16 (the GEMM's token operand), row-major [T][K].
__global__ void to_bf16_kernel(const float* __restrict__ x, int x_stride, __nv_bfloat16* __restrict__ out, int K,
                               int T) {
    const int64_t n4 = (int64_t)T * K / 4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t e = 4 * i;
        const int t = (int)(e / K), k = (int)(e - (int64_t)t * K);
        const float4 f = *reinterpret_cast<const float4*>(x + (size_t)t * x_stride + k);
        uint2 o;
        o.x = pack_bf16(f.x, f.y);
        o.y = pack_bf16(f.z, f.w);
        *reinterpret_cast<uint2*>(out + e) = o;
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    AT_REQUIRE(fn, AT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    return fn;
}

}  // namespace

// Token tiles per CTA: two (512 tokens, every dequantized weight tile feeds
// twice the tokens) once a chunk has more than 256 tokens.
int gemm_tc_nb(int T) { return T > TC_N ? 2 : 1; }

int gemm_tc_splits(const at_qmat* m, int T, int num_sms) {
    const int64_t M = (m->orient == AT_ORIENT_N) ? m->rows : m->cols;
    const int64_t K = (m->orient == AT_ORIENT_N) ? m->cols : m->rows;
    const int64_t tn = (int64_t)TC_N * gemm_tc_nb(T);
    const int64_t tiles = ((M + TC_M - 1) / TC_M) * ((T + tn - 1) / tn);
    // enough CTAs for most SMs, each split keeping at least 8 K-steps
    int64_t sp = std::max<int64_t>(1, (num_sms + tiles / 2) / tiles);
    sp = std::min<int64_t>(sp, std::max<int64_t>(1, (K / TC_K) / 8));
    return (int)std::min<int64_t>(sp, kTcMaxSplits);
}

void launch_gemm_tc(const at_qmat* m, const float* x, int x_stride, float* y, int y_stride, int T, void* xbf,
                    size_t xbf_bytes, float* ws, size_t ws_bytes, int num_sms, int* err, cudaStream_t s,
                    const GemmTcOut& opt) {
    AT_REQUIRE(m->type == AT_GGML_Q4_0 || m->type == AT_GGML_Q8_0, AT_ERR_UNSUPPORTED,
               "tensor-core GEMM supports Q4_0 and Q8_0");
    const int64_t M = (m->orient == AT_ORIENT_N) ? m->rows : m->cols;
    const int64_t K = (m->orient == AT_ORIENT_N) ? m->cols : m->rows;
    AT_REQUIRE(K % TC_K == 0, AT_ERR_INVALID_ARG, "tensor-core GEMM needs K a multiple of 64");
    AT_REQUIRE(T >= 1 && (!x || (x_stride % 4 == 0 && ((uintptr_t)x & 15) == 0)), AT_ERR_INVALID_ARG,
               "tensor-core GEMM: bad activation layout");
    AT_REQUIRE(xbf && ((uintptr_t)xbf & 127) == 0 && xbf_bytes >= (size_t)T * K * 2, AT_ERR_INVALID_ARG,
               "tensor-core GEMM: bf16 staging buffer too small or misaligned");
    // activations -> bf16 [T][K] (x null: the caller staged them in xbf), described to the
    // TMA unit (128-byte swizzle, zero fill past T)
    if (x) {
        const int64_t n4 = (int64_t)T * K / 4;
        const int grid = (int)std::min<int64_t>((n4 + 255) / 256, 148 * 8);
        to_bf16_kernel<<<grid, 256, 0, s>>>(x, x_stride, static_cast<__nv_bfloat16*>(xbf), (int)K, T);
        AT_CUDA(cudaGetLastError());
    }
    CUtensorMap xmap;
    const cuuint64_t gdim[2] = {(cuuint64_t)K, (cuuint64_t)T};
    const cuuint64_t gstride[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)TC_K, (cuuint32_t)TC_N};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = encode_fn()(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xbf, gdim, gstride, box, estride,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    AT_REQUIRE(r == CUDA_SUCCESS, AT_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    TcParams p{};
    p.tiles = m->tiles;
    p.map = tile_map(m);
    p.qtype = m->type;
    p.orient = m->orient;
    p.M = (int)M;
    p.K = (int)K;
    p.T = T;
    const int splits = gemm_tc_splits(m, T, num_sms);
    const bool split = splits > 1 && ws && ws_bytes >= (size_t)splits * T * M * 4;
    p.splits = split ? splits : 1;
    p.y = split ? ws : y;
    p.y_stride = split ? (int)M : y_stride;
    p.err = err;
    if (opt.defer) *opt.defer = p.splits;
    const int nb = gemm_tc_nb(T);
    const bool q4 = m->type == AT_GGML_Q4_0, on = m->orient == AT_ORIENT_N;
    auto kern = nb == 1 ? (q4 ? (on ? gemm_tc_kernel<AT_GGML_Q4_0, AT_ORIENT_N, 1> : gemm_tc_kernel<AT_GGML_Q4_0, AT_ORIENT_T, 1>)
                              : (on ? gemm_tc_kernel<AT_GGML_Q8_0, AT_ORIENT_N, 1> : gemm_tc_kernel<AT_GGML_Q8_0, AT_ORIENT_T, 1>))
                        : (q4 ? (on ? gemm_tc_kernel<AT_GGML_Q4_0, AT_ORIENT_N, 2> : gemm_tc_kernel<AT_GGML_Q4_0, AT_ORIENT_T, 2>)
                              : (on ? gemm_tc_kernel<AT_GGML_Q8_0, AT_ORIENT_N, 2> : gemm_tc_kernel<AT_GGML_Q8_0, AT_ORIENT_T, 2>));
    static std::once_flag attr_once;
    std::call_once(attr_once, [] {
        for (auto k : {gemm_tc_kernel<AT_GGML_Q4_0, AT_ORIENT_N, 1>, gemm_tc_kernel<AT_GGML_Q4_0, AT_ORIENT_T, 1>,
                       gemm_tc_kernel<AT_GGML_Q8_0, AT_ORIENT_N, 1>, gemm_tc_kernel<AT_GGML_Q8_0, AT_ORIENT_T, 1>})
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, tc_smem<1>());
        for (auto k : {gemm_tc_kernel<AT_GGML_Q4_0, AT_ORIENT_N, 2>, gemm_tc_kernel<AT_GGML_Q4_0, AT_ORIENT_T, 2>,
                       gemm_tc_kernel<AT_GGML_Q8_0, AT_ORIENT_N, 2>, gemm_tc_kernel<AT_GGML_Q8_0, AT_ORIENT_T, 2>})
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, tc_smem<2>());
    });
    const int tn = TC_N * nb;
    dim3 grid((unsigned)((M + TC_M - 1) / TC_M), (unsigned)((T + tn - 1) / tn), (unsigned)p.splits);
    kern<<<grid, TC_THREADS_WS, nb == 1 ? tc_smem<1>() : tc_smem<2>(), s>>>(xmap, p);
    AT_CUDA(cudaGetLastError());
    if (p.splits > 1 && !opt.defer) {
        const bool vec = M % 4 == 0 && y_stride % 4 == 0 && ((uintptr_t)y & 15) == 0 && ((uintptr_t)ws & 15) == 0;
        const int per = vec ? (int)((M / 4 + 127) / 128) : (int)((M + 127) / 128);
        if (vec)
            splitk_sum_kernel<true><<<dim3(per, T), 128, 0, s>>>(ws, p.splits, T, (int)M, y, y_stride);
        else
            splitk_sum_kernel<false><<<dim3(per, T), 128, 0, s>>>(ws, p.splits, T, (int)M, y, y_stride);
        AT_CUDA(cudaGetLastError());
    }
}

}  // namespace at
