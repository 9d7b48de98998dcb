// Device helpers shared by the kernels of libauratensor_cuda.so (sm_100a).
#pragma once

#include <cuda_fp16.h>

#include <cuda_runtime.h>
#include <cstdint>

namespace at {

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start before the previous kernel in the stream ends.
// pdl_wait() blocks until that kernel has completed and its writes are
// visible; everything before it may only touch memory no earlier kernel of
// the step writes. pdl_trigger() lets the next kernel start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Fp16.toFloat (core/Fp16.java:19-37): subnormals flush to signed zero,
// e == 31 gives +-inf or the canonical NaN 0x7FC00000, otherwise rebias.
__device__ __forceinline__ float fp16_ftz(uint32_t h) {
    const uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t bits = (s << 31) | ((e + 112u) << 23) | (m << 13);
    bits = (e == 0u) ? (s << 31) : bits;
    bits = (e == 31u) ? (m ? 0x7FC00000u : ((s << 31) | 0x7F800000u)) : bits;
    return __uint_as_float(bits);
}

// Fp16.toFloat with the same results as fp16_ftz, using the hardware f16->f32
// conversion: subnormal inputs are scaled by zero (keeping the sign), so they
// flush to signed zero; NaN stays NaN.
__device__ __forceinline__ float fp16_ftz_fast(uint32_t h) {
    float f;
    asm("{\n\t.reg .f16 t;\n\tmov.b16 t, %1;\n\tcvt.f32.f16 %0, t;\n\t}" : "=f"(f) : "h"((unsigned short)h));
    return (h & 0x7C00u) ? f : __fmul_rn(f, 0.0f);
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
// returning the RMSNorm scale per row in s_inv[B]. Requires blockDim.x == NT,
// d % 4 == 0 and 16-byte aligned rows. Loads are issued 8 float4 at a time
// before any of them is used.
template <int B, int NT = 256>
__device__ __forceinline__ void block_rms_inv(const float* __restrict__ xin, const float* __restrict__ yin,
                                              int stride, int d, float eps, float* s_red /*[NT/32*B]*/,
                                              float* s_inv /*[B]*/) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n4 = d >> 2;
    float ss[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
        const float4* xr = reinterpret_cast<const float4*>(xin + (size_t)b * stride);
        const float4* yr = yin ? reinterpret_cast<const float4*>(yin + (size_t)b * stride) : nullptr;
        float acc = 0.f;
        for (int base = 0; base < n4; base += NT * 8) {
            float4 xv[8], yv[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int i = base + k * NT + tid;
                xv[k] = (i < n4) ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                yv[k] = (yr && i < n4) ? yr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float a0 = __fadd_rn(xv[k].x, yv[k].x), a1 = __fadd_rn(xv[k].y, yv[k].y);
                const float a2 = __fadd_rn(xv[k].z, yv[k].z), a3 = __fadd_rn(xv[k].w, yv[k].w);
                acc = fmaf(a0, a0, acc);
                acc = fmaf(a1, a1, acc);
                acc = fmaf(a2, a2, acc);
                acc = fmaf(a3, a3, acc);
            }
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
        for (int w = 0; w < NT / 32; ++w) t += s_red[w * B + tid];
        s_inv[tid] = rms_inv(t, d, eps);
    }
    __syncthreads();
}

// Kernels.siluInPlace then elementwiseMul (core/Kernels.java:86-87,
// inference/LlamaModel.java:372-380): g / (1 + exp(-g)) * u.
__device__ __forceinline__ float silu_mul(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// (x * invRms) * gamma, in that rounding order (core/Kernels.java:145).
// Q8_0 KV-cache append of one value per lane: the 32 lanes of the (fully
// active) warp hold the 32 consecutive elements of one block (elem % 32 ==
// lane). d = max|x| / 127 (fp16, stored once), q = round-half-away(x / d)
// computed as x * (1 / d) with the fp32 d.
__device__ __forceinline__ void kv_store_q8(int8_t* q, uint16_t* sc, size_t elem, float v) {
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.f);
    const float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
    const float r = roundf(__fmul_rn(v, id));
    q[elem] = (int8_t)fmaxf(-127.f, fminf(127.f, r));
    if ((threadIdx.x & 31) == 0) sc[elem >> 5] = __half_as_ushort(__float2half_rn(d));
}

__device__ __forceinline__ float norm_apply(float x, float inv, float g) {
    return __fmul_rn(__fmul_rn(x, inv), g);
}

// Order-preserving bits of a float for packed (value, ~index) argmax keys;
// NaN maps to -inf.
__device__ __forceinline__ uint32_t ordered_bits(float v) {
    if (v != v) v = -INFINITY;
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Index of a packed argmax key (the all-ones key marks a NaN at index 0).
__device__ __forceinline__ int key_index(unsigned long long k) {
    return (k == ~0ull) ? 0 : (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
}

}  // namespace at
