// Block decoders shared by the fused-dequant kernels (gemv.cu and the
// persistent decode step, decode_step.cu): Q4_0 / Q8_0 traits and the
// subnormal-scaled dequant (a quant field masked in place and read as a float
// is exactly field * 2^-149), for sm_100a.
#pragma once

#include <cstdint>

#include "at_internal.h"
#include "dev_common.cuh"

namespace at {

template <int QT>
struct QTraits;
template <>
struct QTraits<AT_GGML_Q4_0> { static constexpr int QB = 16; static constexpr int NV = 1; };
template <>
struct QTraits<AT_GGML_Q8_0> { static constexpr int QB = 32; static constexpr int NV = 2; };

// Subnormal-scaled form of dot32 (the batch <= 2 stream kernel).
// A quant field masked in place and read as a float is exactly
// field * 2^-149: the bit patterns 0 .. 2^24 - 1 (subnormals and the first
// normal binade) encode the integers N as N * 2^-149. So one LOP3 per weight
// gives q * 2^(s_k) * 2^-149, s_k the field's bit offset: Q4_0 nibble j of a
// 32-bit word at offset 4j (j < 6; nibbles 6 and 7 after one shift by 24, at
// offsets 0 and 4), Q8_0 byte j (sign bit flipped: q + 128) at 8j (j < 3;
// byte 3 after the shift, at 0). The staged x of element k carries the
// matching power of two 2^(kXExp - s_k) (x_scale_dn), so every product is
// exactly q_k * x_k * 2^(kXExp - 149), one FFMA2 per two weights, no
// subtraction. The offset (8 or 128) times the block's sum of x, staged with
// the block as sx = (sum x_k) * 2^(kXExp - 149), is taken off once per
// block, and kDnUnscale = 2^(149 - kXExp) goes into the block scale.
// Products are exact; only the FP32 summation differs from dot32 (the
// offset is subtracted from the block sum instead of from each weight).
// Requires |x| < 2^(128 - kXExp) = 2^48 for the staged values.
constexpr int kXExp = 80;
constexpr float kDnUnscale = 590295810358705651712.f;  // 2^69 = 2^(149 - kXExp)
static_assert(149 - kXExp == 69, "kDnUnscale is 2^69");

// Power of two that element k (k % 8 for Q4_0, k % 4 for Q8_0) of a block is
// staged with.
template <int QT>
__host__ __device__ constexpr int x_shift_dn(int k) {
    if constexpr (QT == AT_GGML_Q4_0) {
        const int j = k & 7;
        return j < 6 ? 4 * j : 4 * (j - 6);
    } else {
        const int j = k & 3;
        return j < 3 ? 8 * j : 0;
    }
}

__device__ __forceinline__ float bits_f(uint32_t u) { return __uint_as_float(u); }
// 2^n for -126 <= n <= 127.
__device__ __forceinline__ float exp2_i(int n) { return __uint_as_float((uint32_t)(n + 127) << 23); }

template <int QT>
__device__ __forceinline__ float dot32_dn(const uint4* q, const float4* xr, float sx) {
    float2 a0 = f2(0.f, 0.f), a1 = f2(0.f, 0.f);
    if constexpr (QT == AT_GGML_Q4_0) {
        const uint32_t ws[4] = {q[0].x, q[0].y, q[0].z, q[0].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w = ws[i], t = w >> 24;  // word i: elements 8i .. 8i + 7
            a0 = __ffma2_rn(f2(bits_f(w & 0xFu), bits_f(w & 0xF0u)), f2(xr[2 * i].x, xr[2 * i].y), a0);
            a1 = __ffma2_rn(f2(bits_f(w & 0xF00u), bits_f(w & 0xF000u)), f2(xr[2 * i].z, xr[2 * i].w), a1);
            a0 = __ffma2_rn(f2(bits_f(w & 0xF0000u), bits_f(w & 0xF00000u)), f2(xr[2 * i + 1].x, xr[2 * i + 1].y), a0);
            a1 = __ffma2_rn(f2(bits_f(t & 0xFu), bits_f(t & 0xF0u)), f2(xr[2 * i + 1].z, xr[2 * i + 1].w), a1);
        }
        return fmaf(-8.f, sx, (a0.x + a0.y) + (a1.x + a1.y));
    } else {
        const uint32_t ws[8] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t w = ws[i];  // word i: elements 4i .. 4i + 3
            a0 = __ffma2_rn(f2(bits_f((w ^ 0x80u) & 0xFFu), bits_f((w ^ 0x8000u) & 0xFF00u)), f2(xr[i].x, xr[i].y),
                            a0);
            a1 = __ffma2_rn(f2(bits_f((w ^ 0x800000u) & 0xFF0000u), bits_f((w >> 24) ^ 0x80u)), f2(xr[i].z, xr[i].w),
                            a1);
        }
        return fmaf(-128.f, sx, (a0.x + a0.y) + (a1.x + a1.y));
    }
}

// Subnormal-scaled decode of a lane's 32 weights (see dot32_dn): pair k holds
// the fields of columns 2k, 2k+1 masked in place, q * 2^(x_shift_dn(col) - 149)
// (Q8_0: q + 128). The T kernel multiplies them by d * x * 2^kXExp and, per
// column, scales the sums back by 2^(149 - kXExp - x_shift_dn(col)) and takes
// off the offset (8 or 128) times the lane's sum of d * x.
template <int QT>
__device__ __forceinline__ void t_decode_dn(const uint4* q, float2* wv) {
    if constexpr (QT == AT_GGML_Q4_0) {
        const uint32_t ws[4] = {q[0].x, q[0].y, q[0].z, q[0].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w = ws[i], t = w >> 24;
            wv[4 * i + 0] = f2(bits_f(w & 0xFu), bits_f(w & 0xF0u));
            wv[4 * i + 1] = f2(bits_f(w & 0xF00u), bits_f(w & 0xF000u));
            wv[4 * i + 2] = f2(bits_f(w & 0xF0000u), bits_f(w & 0xF00000u));
            wv[4 * i + 3] = f2(bits_f(t & 0xFu), bits_f(t & 0xF0u));
        }
    } else {
        const uint32_t ws[8] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t w = ws[i];
            wv[2 * i + 0] = f2(bits_f((w ^ 0x80u) & 0xFFu), bits_f((w ^ 0x8000u) & 0xFF00u));
            wv[2 * i + 1] = f2(bits_f((w ^ 0x800000u) & 0xFF0000u), bits_f((w >> 24) ^ 0x80u));
        }
    }
}

}  // namespace at
