// Device helpers shared by the kernels of libauratensor_cuda.so (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

namespace at {

// Fp16.toFloat (core/Fp16.java:19-37): subnormals flush to signed zero,
// e == 31 gives +-inf or the canonical NaN 0x7FC00000, otherwise rebias.
__device__ __forceinline__ float fp16_ftz(uint32_t h) {
    const uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t bits = (s << 31) | ((e + 112u) << 23) | (m << 13);
    bits = (e == 0u) ? (s << 31) : bits;
    bits = (e == 31u) ? (m ? 0x7FC00000u : ((s << 31) | 0x7F800000u)) : bits;
    return __uint_as_float(bits);
}

// Float with value 2^23 + byte k of w: byte k becomes the low mantissa byte
// of 0x4B000000 (one PRMT). Subtracting 2^23 + offset is then exact.
__device__ __forceinline__ float magic_byte(uint32_t w, int k) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)k));
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// Read-only streaming 128-bit load of weight bytes (not reused by this kernel).
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ld_stream_u16(const uint16_t* p) {
    unsigned short r;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return (uint32_t)r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// RMSNorm scale of Kernels.rmsNormInPlace (core/Kernels.java:137):
// invRms = (float)(1.0 / Math.sqrt(sumSq / (float) d + eps)), division and eps
// add in float, square root and reciprocal in double.
__device__ __forceinline__ float rms_inv(float sum_sq, int d, float eps) {
    const float mean = __fadd_rn(__fdiv_rn(sum_sq, (float)d), eps);
    return (float)(1.0 / sqrt((double)mean));
}

// Block-wide sum of squares of (xin + yin) for each of B rows of length d,
// returning the RMSNorm scale per row in s_inv[B]. Requires blockDim.x == 256.
template <int B>
__device__ __forceinline__ void block_rms_inv(const float* __restrict__ xin, const float* __restrict__ yin,
                                              int stride, int d, float eps, float* s_red /*[8*B]*/,
                                              float* s_inv /*[B]*/) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float ss[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
        float acc = 0.f;
        const float* xr = xin + (size_t)b * stride;
        const float* yr = yin ? yin + (size_t)b * stride : nullptr;
        for (int i = tid; i < d; i += 256) {
            float v = xr[i];
            if (yr) v = __fadd_rn(v, yr[i]);
            acc = fmaf(v, v, acc);
        }
        ss[b] = warp_sum(acc);
    }
    if (lane == 0) {
#pragma unroll
        for (int b = 0; b < B; ++b) s_red[warp * B + b] = ss[b];
    }
    __syncthreads();
    if (tid < B) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) t += s_red[w * B + tid];
        s_inv[tid] = rms_inv(t, d, eps);
    }
    __syncthreads();
}

// (x * invRms) * gamma, in that rounding order (core/Kernels.java:145).
__device__ __forceinline__ float norm_apply(float x, float inv, float g) {
    return __fmul_rn(__fmul_rn(x, inv), g);
}

}  // namespace at
