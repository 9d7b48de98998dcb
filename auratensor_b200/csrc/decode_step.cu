// Persistent batch-1 decode step for sm_100a: LlamaModel.forwardStep
// (inference/LlamaModel.java:141-308) as ONE kernel launch.
//
// One CTA per SM (cooperative launch). The step is a fixed sequence of jobs:
// per layer QKV (orientation-T GEMV with the attention RMSNorm in its
// prologue), attention (split over positions), wo (T), gate/up
// (orientation-N GEMV, FFN RMSNorm prologue, SiLU * up epilogue) and down (N);
// then the lm_head (N, output norm prologue) and the greedy argmax. Jobs are
// separated by grid barriers (an arrival counter in global memory).
//
// Weight bytes (and the K/V rows of earlier positions) are never written
// during the step, so every warp streams them through its own ring of
// shared-memory slots ahead of the computation, across job boundaries: lane 0
// issues cp.async.bulk copies (global -> shared, completing on the slot's
// mbarrier) as soon as a slot frees up, so while a warp waits at a grid
// barrier its next job's first units are already in flight. A unit is a
// 4-row x 32-block N tile (gate/up: the w1 and the w3 tile of one row group
// and step), 4 row tiles of one T block column, or a few positions of K and
// V rows.
//
// Each job is one out-of-line function and the per-warp ring state lives in
// shared memory, so a job's unit loop is one compact stretch of code (the
// instruction cache, not HBM, limited a fully inlined version).
//
// Work split (fixed per shape, so results do not depend on timing):
//  - N jobs: whole 4-row groups per CTA (balanced split), the CTA's units
//    split evenly over its warps; a warp accumulates a row group's partial
//    sums in registers and writes the finished rows, row groups shared with
//    a neighbouring warp are summed in warp order after a CTA barrier.
//  - T jobs: each block column is cut into S parts of whole units; CTAs take
//    whole parts; a part's sum (over its warps, in warp order) goes to a
//    global part buffer and the consumer of the output sums the S parts in
//    order (S = 1 for wo: its output is final).
//  - attention: a KV head's positions are split over up to 32 CTAs; each
//    warp keeps an online softmax (m, l, o) over its positions; the CTA merges
//    its warps, and the last CTA of the head (arrival ticket) merges the
//    CTAs' partials in CTA order into the attention output.
// Activations are staged in shared memory already normed with the
// reference's rounding ((x * invRms) * gamma, core/Kernels.java:145).
//
// Every wait is bounded (a slot's mbarrier, a grid barrier): a wait that
// runs out sets the error word, the CTA skips the rest of its work (every
// barrier is still reached), each warp waits for its copies in flight, and
// the host sees the error after the launch.
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>

#include "at_internal.h"
#include "dev_common.cuh"
#include "qdecode.cuh"

namespace at {

namespace {

constexpr int DS_THREADS = 512;
constexpr int DS_WARPS = DS_THREADS / 32;
constexpr int DS_RT = 4;           // T row tiles per unit
constexpr int DS_G_MAX = 8;        // query heads per KV head
constexpr int DS_HD_MAX = 128;
constexpr int DS_MAXWP = 4;        // T parts one warp's units may touch
constexpr int DS_MAX_NST = 8;      // ring slots per warp
constexpr int DS_ATT_MAX = 32;     // CTAs per KV head in the attention
constexpr int XP = 36;             // staged floats per 32-element block (N jobs)
constexpr int DS_TV = (8192 + 4 * DS_THREADS - 1) / (4 * DS_THREADS);  // float4 per thread of a d <= 8192 row
constexpr unsigned long long kWaitNs = 200ull * 1000ull * 1000ull;  // bounded waits: 200 ms
constexpr int kStaticSmem = 20 * 1024;  // upper bound of the kernel's static shared memory

enum Kind { K_QKV = 0, K_ATT = 1, K_WO = 2, K_GU = 3, K_DN = 4, K_HEAD = 5 };

__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Global -> shared bulk copy (no multicast) completing on an mbarrier.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ float exp_ref(float v) { return (float)exp((double)v); }

// Error codes in the error word.
constexpr int kErrSlot = 1;     // a ring slot's copy did not complete
constexpr int kErrBarrier = 2;  // a grid barrier did not complete

// ---------------------------------------------------------------------------
// Work split
// ---------------------------------------------------------------------------
struct AttMap {
    int active;          // this CTA works on the attention
    int h, j, nh;        // KV head, CTA index within the head, CTAs of the head
    int p_lo, p_hi;      // positions [p_lo, p_hi) (p_hi = pos + 1 for the last CTA)
    int pend;            // streamed positions [p_lo, pend): the current position comes from QKV
    int up;              // positions per unit (a power of two, up * G <= 32)
    int nunits;
};

__device__ __forceinline__ AttMap att_map(const DsParams& p, int cta, int C, int pos) {
    AttMap a{};
    const int A = min(C, p.Hkvl * DS_ATT_MAX);
    const int G = p.Hl / p.Hkvl;
    int up = min(p.slot_bytes / (2 * p.hd * 4), 32 / G);
    a.up = 1;
    while (2 * a.up <= up) a.up *= 2;
    if (cta >= A) return a;
    a.active = 1;
    a.h = (int)((int64_t)cta * p.Hkvl / A);
    const int f0 = (int)(((int64_t)a.h * A + p.Hkvl - 1) / p.Hkvl);
    const int f1 = (int)(((int64_t)(a.h + 1) * A + p.Hkvl - 1) / p.Hkvl);
    a.nh = f1 - f0;
    a.j = cta - f0;
    const int P = pos + 1;
    a.p_lo = (int)((int64_t)a.j * P / a.nh);
    a.p_hi = (int)((int64_t)(a.j + 1) * P / a.nh);
    a.pend = min(a.p_hi, pos);
    const int npast = max(0, a.pend - a.p_lo);
    a.nunits = (npast + a.up - 1) / a.up;
    return a;
}

// This CTA's unit range of a job.
__device__ __forceinline__ void cta_units(const DsParams& p, int kind, int cta, int C, const AttMap& am, int* u0,
                                          int* u1) {
    if (kind == K_QKV || kind == K_WO) {
        const DsT& t = (kind == K_QKV) ? p.qkv : p.wo;
        const int P = t.ncols * t.S, pu = t.nu / t.S;
        *u0 = (int)((int64_t)cta * P / C) * pu;
        *u1 = (int)((int64_t)(cta + 1) * P / C) * pu;
    } else if (kind == K_ATT) {
        *u0 = 0;
        *u1 = am.active ? am.nunits : 0;
    } else {
        const DsN& n = (kind == K_GU) ? p.gu : (kind == K_DN ? p.dn : p.head);
        const int per = n.nsteps * ((kind == K_GU && !p.gu_pair) ? 2 : 1);
        *u0 = (int)((int64_t)cta * n.ngroups / C) * per;
        *u1 = (int)((int64_t)(cta + 1) * n.ngroups / C) * per;
    }
}

__device__ __forceinline__ void warp_split(int u0, int u1, int warp, int* w0, int* w1) {
    const int n = u1 - u0;
    *w0 = u0 + (warp * n) / DS_WARPS;
    *w1 = u0 + ((warp + 1) * n) / DS_WARPS;
}
// Warp holding unit x (relative to the CTA's first unit) of a CTA range of n units.
__device__ __forceinline__ int warp_of(int x, int n) {
    const int w = (DS_WARPS * x + DS_WARPS - 1) / n;
    return w < DS_WARPS - 1 ? w : DS_WARPS - 1;
}

__device__ __forceinline__ int job_kind(int job) { return job % 5; }
__device__ __forceinline__ int job_layer(int job) { return job / 5; }

// ---------------------------------------------------------------------------
// Shared state
// ---------------------------------------------------------------------------
// Issue cursor of one warp's ring (used by its lane 0): units of a job are
// consecutive in memory for the warp, so unit k's source is base + k * stride
// (gate/up: the w1 and the w3 tile at the same offset, or alternating tiles;
// attention: `up` positions of K rows and of V rows).
struct Cursor {
    int issued;            // units issued
    int job, kind, k, kend;
    const uint8_t* ta;     // the job's matrix (gate/up: w1; attention: K rows of the CTA's first position)
    const uint8_t* tb;     // gate/up: w3; attention: V rows
    long long stride;      // bytes between consecutive units
    int ubytes;            // bytes per copy (attention: one position's row)
    int npos;              // attention: positions this CTA streams
};

struct Shared {
    alignas(8) unsigned long long bars[DS_WARPS * DS_MAX_NST];
    Cursor cur[DS_WARPS];
    int consumed[DS_WARPS];                   // units each warp has consumed
    AttMap am;
    float wpart[DS_WARPS][DS_MAXWP][32];      // T: per-warp part sums
    float npart[DS_WARPS][2][8];              // N: per-warp sums of row groups shared with neighbours
    alignas(16) float qs[DS_G_MAX * DS_HD_MAX];  // attention: roped q of this CTA's head group
    alignas(16) float kn[DS_HD_MAX];          // attention: k and v of the current position
    alignas(16) float vn[DS_HD_MAX];
    float aw[DS_G_MAX][DS_ATT_MAX];           // attention merge weights
    float al[DS_G_MAX];
    float red[DS_WARPS * 2];
    float inv;
    volatile int abort;
    int last;
    unsigned long long best[DS_WARPS];
    unsigned target;                          // grid-barrier target (thread 0)
};

// Per-warp view of the ring, for the unit loops.
struct WarpCtx {
    const DsParams* p;
    Shared* sh;
    const uint8_t* ring;   // this warp's slot 0 (generic address)
    uint32_t slots, bars;  // shared addresses of slot 0 and mbarrier 0
    int warp, lane, cta, C, njobs;
};

// ---------------------------------------------------------------------------
// Per-warp weight ring
// ---------------------------------------------------------------------------
// Moves a warp's issue cursor to its next job with units (once per job and
// warp, out of line).
__device__ __noinline__ void cursor_next_job(const DsParams& p, Shared& sh, int warp, int cta, int C, int njobs) {
    Cursor& c = sh.cur[warp];
    const AttMap& am = sh.am;
    while (c.k >= c.kend) {
        if (c.job + 1 >= njobs) {
            c.job = njobs;
            return;
        }
        ++c.job;
        c.kind = (c.job == njobs - 1) ? K_HEAD : job_kind(c.job);
        int u0, u1;
        cta_units(p, c.kind, cta, C, am, &u0, &u1);
        warp_split(u0, u1, warp, &c.k, &c.kend);
        const DsLayer* ly = p.layers + (c.kind == K_HEAD ? 0 : job_layer(c.job));
        switch (c.kind) {
            case K_QKV:
                c.ta = ly->qkv;
                c.stride = c.ubytes = DS_RT * (int)p.tile_t;
                break;
            case K_WO:
                c.ta = ly->wo;
                c.stride = c.ubytes = DS_RT * (int)p.tile_t;
                break;
            case K_ATT: {
                const int64_t off = (((int64_t)am.h * p.ctx + am.p_lo) * p.hd) * 4;
                c.ta = reinterpret_cast<const uint8_t*>(ly->kc) + off;
                c.tb = reinterpret_cast<const uint8_t*>(ly->vc) + off;
                c.ubytes = p.hd * 4;
                c.stride = (long long)am.up * c.ubytes;
                c.npos = am.pend - am.p_lo;
                break;
            }
            case K_GU:
                c.ta = ly->w1;
                c.tb = ly->w3;
                c.stride = c.ubytes = (int)p.tile_n;
                break;
            case K_DN:
                c.ta = ly->w2;
                c.stride = c.ubytes = (int)p.tile_n;
                break;
            default:
                c.ta = p.out_tiles;
                c.stride = c.ubytes = (int)p.tile_n;
                break;
        }
    }
}

// Lane 0 issues units into free slots until the ring is full or the step's
// units run out.
__device__ __forceinline__ void ring_fill(const WarpCtx& w, int consumed) {
    if (w.lane != 0 || w.sh->abort) return;
    const DsParams& p = *w.p;
    Cursor& c = w.sh->cur[w.warp];
    while (c.issued - consumed < p.nst) {
        if (c.k >= c.kend) {
            cursor_next_job(p, *w.sh, w.warp, w.cta, w.C, w.njobs);
            if (c.job >= w.njobs) return;
        }
        const int slot = c.issued & (p.nst - 1);
        const uint32_t bar = w.bars + slot * 8;
        const uint32_t dst = w.slots + slot * p.slot_bytes;
        if (c.kind == K_ATT) {
            const int ps = c.k * w.sh->am.up;
            const uint32_t n = (uint32_t)(min(w.sh->am.up, c.npos - ps) * c.ubytes);
            mbar_expect_tx(bar, 2 * n);
            bulk_g2s(dst, c.ta + (long long)ps * c.ubytes, n, bar);
            bulk_g2s(dst + n, c.tb + (long long)ps * c.ubytes, n, bar);
        } else if (c.kind == K_GU && p.gu_pair) {
            mbar_expect_tx(bar, 2 * c.ubytes);
            bulk_g2s(dst, c.ta + c.k * c.stride, c.ubytes, bar);
            bulk_g2s(dst + c.ubytes, c.tb + c.k * c.stride, c.ubytes, bar);
        } else {
            const uint8_t* src = (c.kind == K_GU) ? ((c.k & 1) ? c.tb : c.ta) + (c.k >> 1) * c.stride
                                                  : c.ta + c.k * c.stride;
            mbar_expect_tx(bar, c.ubytes);
            bulk_g2s(dst, src, c.ubytes, bar);
        }
        ++c.issued;
        ++c.k;
    }
}

// Waits for unit `consumed` of this warp; false if the wait ran out (sets the error word).
__device__ __forceinline__ bool ring_wait(const WarpCtx& w, int consumed) {
    const int slot = consumed & (w.p->nst - 1);
    const uint32_t bar = w.bars + slot * 8, par = (uint32_t)(consumed / w.p->nst) & 1u;
    if (mbar_try(bar, par)) return true;
    const unsigned long long t0 = gtimer();
    for (int it = 0;; ++it) {
        if (mbar_try(bar, par)) return true;
        if ((it & 63) == 63 && (gtimer() - t0 > kWaitNs || ld_volatile(w.p->err) != 0)) {
            atomicCAS(w.p->err, 0, kErrSlot);
            return false;
        }
    }
}
__device__ __forceinline__ const uint8_t* ring_slot(const WarpCtx& w, int consumed) {
    return w.ring + (size_t)(consumed & (w.p->nst - 1)) * w.p->slot_bytes;
}

// Grid barrier: every CTA arrives once per call; thread 0 spins (bounded) on
// the arrival counter. The CTA's writes are ordered before the arrival by the
// CTA barrier and a device-scope fence; reads of other CTAs' data after it go
// through L2 (__ldcg).
__device__ __noinline__ void grid_barrier(const DsParams& p, Shared& sh) {
    __syncthreads();
    if (threadIdx.x == 0) {
        sh.target += gridDim.x;
        if (!sh.abort) {
            __threadfence();
            atomicAdd(p.bar, 1u);
            const unsigned long long t0 = gtimer();
            for (int it = 0;; ++it) {
                if ((int)(ld_acquire(p.bar) - sh.target) >= 0) break;
                if ((it & 63) == 63 && (ld_volatile(p.err) != 0 || gtimer() - t0 > kWaitNs)) {
                    atomicCAS(p.err, 0, kErrBarrier);
                    sh.abort = 1;
                    break;
                }
            }
            __threadfence();
        }
    }
    __syncthreads();
}

// Optional timeline: stamps [CTA][job][4] = job start (after the grid
// barrier), activations staged, units done, job end.
__device__ __forceinline__ void stamp(const DsParams& p, int job, int which) {
    if (p.stamps && threadIdx.x == 0)
        p.stamps[((size_t)blockIdx.x * (5 * p.L + 1) + job) * 4 + which] = gtimer();
}

// ---------------------------------------------------------------------------
// Prologues: activation staging
// ---------------------------------------------------------------------------
// t = a + b (b may be null; emb_token >= 0 takes the token's embedding row
// instead) over d elements in registers (d <= 8192: DS_TV float4 per thread),
// RMSNorm scale from the CTA-wide sum of squares (fixed order), then
// xn = (t * inv) * gamma: this CTA's slice of xn goes to res_out (if given),
// and xn is staged either plain (T jobs) or in the N layout (N jobs).
template <int QT>
__device__ __forceinline__ void stage_normed(const DsParams& p, Shared& sh, float* xs, const float* a, const float* b,
                                             int bS, int emb_token, const float* gamma, float* res_out, bool n_layout,
                                             int pad_to) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int d = p.d, n4 = d >> 2;
    float4 tv[DS_TV];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < DS_TV; ++k) {
        const int i4 = tid + k * DS_THREADS;
        float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i4 < n4) {
            if (emb_token >= 0) {
                const int blk = (4 * i4) >> 5, w0 = (4 * i4) & 31;
                int64_t d_off, q_off;
                p.tok_map.offsets(emb_token, blk, &d_off, &q_off);
                const float dsc = fp16_ftz(
                    (uint32_t)__ldg(p.tok_tiles + d_off) | ((uint32_t)__ldg(p.tok_tiles + d_off + 1) << 8));
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int w = w0 + e;
                    int q;
                    if constexpr (QT == AT_GGML_Q4_0) {
                        const uint32_t pk = __ldg(p.tok_tiles + q_off + (w >> 1));
                        q = ((w & 1) ? (int)(pk >> 4) : (int)(pk & 0xF)) - 8;
                    } else {
                        q = (int)(int8_t)__ldg(p.tok_tiles + q_off + w);
                    }
                    v[e] = __fmul_rn((float)q, dsc);
                }
                t = make_float4(v[0], v[1], v[2], v[3]);
            } else {
                t = ldcg4(a + 4 * i4);
                if (b) {
                    float4 u;
                    if (bS == 1) {
                        u = ldcg4(b + 4 * i4);
                    } else {
                        // sum of the S part sums of the T output (column c = i / 32)
                        const int e0 = 4 * i4, col = e0 >> 5, j = e0 & 31;
                        u = ldcg4(b + ((size_t)col * bS) * 32 + j);
                        for (int s2 = 1; s2 < bS; ++s2) {
                            const float4 w = ldcg4(b + ((size_t)col * bS + s2) * 32 + j);
                            u.x += w.x; u.y += w.y; u.z += w.z; u.w += w.w;
                        }
                    }
                    t.x = __fadd_rn(t.x, u.x); t.y = __fadd_rn(t.y, u.y);
                    t.z = __fadd_rn(t.z, u.z); t.w = __fadd_rn(t.w, u.w);
                }
            }
            ss = fmaf(t.x, t.x, fmaf(t.y, t.y, fmaf(t.z, t.z, fmaf(t.w, t.w, ss))));
        }
        tv[k] = t;
    }
    ss = warp_sum(ss);
    if (lane == 0) sh.red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        float tot = 0.f;
        for (int w = 0; w < DS_WARPS; ++w) tot += sh.red[w];
        sh.inv = rms_inv(tot, d, p.eps);
    }
    __syncthreads();
    const float inv = sh.inv;
    const int C = gridDim.x;
    const int s0 = (int)((int64_t)blockIdx.x * n4 / C), s1 = (int)((int64_t)(blockIdx.x + 1) * n4 / C);
#pragma unroll
    for (int k = 0; k < DS_TV; ++k) {
        const int i4 = tid + k * DS_THREADS;
        const bool in = i4 < n4;
        float4 xn = make_float4(0.f, 0.f, 0.f, 0.f);
        if (in) {
            const float4 g = __ldg(reinterpret_cast<const float4*>(gamma) + i4);
            const float4 t = tv[k];
            xn = make_float4(norm_apply(t.x, inv, g.x), norm_apply(t.y, inv, g.y), norm_apply(t.z, inv, g.z),
                             norm_apply(t.w, inv, g.w));
            if (res_out && i4 >= s0 && i4 < s1) *reinterpret_cast<float4*>(res_out + 4 * i4) = xn;
        }
        if (!n_layout) {
            if (in) *reinterpret_cast<float4*>(xs + 4 * i4) = xn;
        } else {
            // block sums over the 8 consecutive lanes holding a block (d % 32 == 0)
            float bs = (xn.x + xn.y) + (xn.z + xn.w);
            bs += __shfl_xor_sync(0xffffffffu, bs, 1);
            bs += __shfl_xor_sync(0xffffffffu, bs, 2);
            bs += __shfl_xor_sync(0xffffffffu, bs, 4);
            if (in) {
                const int e0 = (4 * i4) & 31;
                float* dst = xs + (size_t)((4 * i4) >> 5) * XP;
                *reinterpret_cast<float4*>(dst + e0) =
                    make_float4(__fmul_rn(xn.x, exp2_i(kXExp - x_shift_dn<QT>(e0))),
                                __fmul_rn(xn.y, exp2_i(kXExp - x_shift_dn<QT>(e0 + 1))),
                                __fmul_rn(xn.z, exp2_i(kXExp - x_shift_dn<QT>(e0 + 2))),
                                __fmul_rn(xn.w, exp2_i(kXExp - x_shift_dn<QT>(e0 + 3))));
                if (e0 == 0) dst[32] = __fmul_rn(bs, exp2_i(kXExp - 149));
            }
        }
    }
    if (!n_layout)
        for (int e = d + tid; e < pad_to; e += DS_THREADS) xs[e] = 0.f;  // padding rows of the T tiles
}

// Plain staging of n floats (T job input: the attention output).
__device__ __forceinline__ void stage_plain(float* xs, const float* src, int n, int pad_to) {
    for (int i4 = threadIdx.x; i4 < n / 4; i4 += DS_THREADS)
        *reinterpret_cast<float4*>(xs + 4 * i4) = ldcg4(src + 4 * i4);
    for (int e = n + threadIdx.x; e < pad_to; e += DS_THREADS) xs[e] = 0.f;
}

// N-layout staging of n floats (the down projection's input h), no norm.
template <int QT>
__device__ __forceinline__ void stage_n_plain(float* xs, const float* src, int n) {
    const int n4 = n >> 2;
    for (int base = 0; base < n4; base += DS_THREADS * 4) {
        float4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i4 = base + k * DS_THREADS + threadIdx.x;
            v[k] = (i4 < n4) ? ldcg4(src + 4 * i4) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i4 = base + k * DS_THREADS + threadIdx.x;
            const float4 xn = v[k];
            float bs = (xn.x + xn.y) + (xn.z + xn.w);
            bs += __shfl_xor_sync(0xffffffffu, bs, 1);
            bs += __shfl_xor_sync(0xffffffffu, bs, 2);
            bs += __shfl_xor_sync(0xffffffffu, bs, 4);
            if (i4 < n4) {
                const int e0 = (4 * i4) & 31;
                float* dst = xs + (size_t)((4 * i4) >> 5) * XP;
                *reinterpret_cast<float4*>(dst + e0) =
                    make_float4(__fmul_rn(xn.x, exp2_i(kXExp - x_shift_dn<QT>(e0))),
                                __fmul_rn(xn.y, exp2_i(kXExp - x_shift_dn<QT>(e0 + 1))),
                                __fmul_rn(xn.z, exp2_i(kXExp - x_shift_dn<QT>(e0 + 2))),
                                __fmul_rn(xn.w, exp2_i(kXExp - x_shift_dn<QT>(e0 + 3))));
                if (e0 == 0) dst[32] = __fmul_rn(bs, exp2_i(kXExp - 149));
            }
        }
    }
}

// ---------------------------------------------------------------------------
// T job (QKV, wo): lane = input row of a 32-row tile, 32 output columns
// ---------------------------------------------------------------------------
template <int QT>
__device__ __forceinline__ void t_flush(float2 (&acc)[16], float& dsum, float* dst, int lane) {
    const float corr = __fmul_rn(QT == AT_GGML_Q4_0 ? -8.f : -128.f, dsum);
    float v[32];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        v[2 * k] = fmaf(acc[k].x, exp2_i(149 - kXExp - x_shift_dn<QT>(2 * k)), corr);
        v[2 * k + 1] = fmaf(acc[k].y, exp2_i(149 - kXExp - x_shift_dn<QT>(2 * k + 1)), corr);
        acc[k] = f2(0.f, 0.f);
    }
    dsum = 0.f;
    int n = 32;
#pragma unroll
    for (int bit = 16; bit >= 1; bit >>= 1) {
        const bool upper = (lane & bit) != 0;
        n >>= 1;
#pragma unroll
        for (int t = 0; t < 16; ++t) {
            if (t < n) {
                const float send = upper ? v[t] : v[t + n];
                const float keep = upper ? v[t + n] : v[t];
                v[t] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
            }
        }
    }
    dst[lane] = v[0];  // lane holds column `lane`
}

template <int QT>
__device__ __noinline__ void job_t(const DsParams& p, Shared& sh, uint8_t* smem, int kind, int layer, int job,
                                   int token, int njobs) {
    constexpr int QB = QTraits<QT>::QB;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, cta = blockIdx.x, C = gridDim.x;
    float* xs = reinterpret_cast<float*>(smem);
    const DsT& t = (kind == K_QKV) ? p.qkv : p.wo;
    float* part_out = (kind == K_QKV) ? p.qkv_part : p.wo_part;
    if (!sh.abort) {
        if (kind == K_QKV)  // x = norm(res0 + ydown) (layer 0: the token's embedding row), res1 <- x
            stage_normed<QT>(p, sh, xs, p.res0, layer == 0 ? nullptr : p.ydown, 1, layer == 0 ? token : -1,
                             p.layers[layer].attn_norm, p.res1, false, t.ngroups * 32);
        else
            stage_plain(xs, p.att, t.E, t.ngroups * 32);
    }
    __syncthreads();
    stamp(p, job, 1);
    WarpCtx w{&p, &sh, smem + p.xs_bytes + (size_t)warp * p.nst * p.slot_bytes,
              smem_addr(smem + p.xs_bytes) + (uint32_t)(warp * p.nst * p.slot_bytes),
              smem_addr(&sh.bars[warp * DS_MAX_NST]), warp, lane, cta, C, njobs};
    int u0, u1, w0, w1;
    cta_units(p, kind, cta, C, sh.am, &u0, &u1);
    warp_split(u0, u1, warp, &w0, &w1);
    const int pu = t.nu / t.S;
    const int p_first_w = w0 / pu;  // first part of this warp
    for (int i = lane; i < DS_MAXWP * 32; i += 32) (&sh.wpart[warp][0][0])[i] = 0.f;
    float2 acc[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) acc[k] = f2(0.f, 0.f);
    float dsum = 0.f;
    int cur = -1;
    int consumed = sh.consumed[warp];
    int part = w0 / pu, in_part = w0 - part * pu;  // tracked without divisions
    int g = (w0 - (w0 / t.nu) * t.nu) * DS_RT;      // first row tile of the unit
    for (int k = w0; k < w1; ++k) {
        if (sh.abort) break;
        if (!ring_wait(w, consumed)) { sh.abort = 1; break; }
        if (part != cur) {
            if (cur >= 0) t_flush<QT>(acc, dsum, sh.wpart[warp][cur - p_first_w], lane);
            cur = part;
        }
        const uint8_t* slot = ring_slot(w, consumed);
#pragma unroll
        for (int ti = 0; ti < DS_RT; ++ti) {
            const uint8_t* tile = slot + ti * p.tile_t;
            uint4 q[2];
            q[0] = *reinterpret_cast<const uint4*>(tile + 64 + lane * QB);
            if constexpr (QT == AT_GGML_Q8_0) q[1] = *reinterpret_cast<const uint4*>(tile + 64 + lane * QB + 16);
            const float dsc = fp16_ftz_fast(*reinterpret_cast<const uint16_t*>(tile + 2 * lane));
            const float sv = __fmul_rn(dsc, xs[(g + ti) * 32 + lane]);
            dsum += sv;
            const float svs = __fmul_rn(sv, exp2_i(kXExp));
            float2 wv[16];
            t_decode_dn<QT>(q, wv);
#pragma unroll
            for (int kk = 0; kk < 16; ++kk) acc[kk] = __ffma2_rn(wv[kk], f2(svs, svs), acc[kk]);
        }
        __syncwarp();
        ++consumed;
        ring_fill(w, consumed);
        g += DS_RT;
        if (g == t.ngroups) g = 0;
        if (++in_part == pu) { in_part = 0; ++part; }
    }
    if (cur >= 0 && !sh.abort) t_flush<QT>(acc, dsum, sh.wpart[warp][cur - p_first_w], lane);
    if (lane == 0) sh.consumed[warp] = consumed;
    __syncthreads();
    stamp(p, job, 2);
    // part sums over the warps in warp order
    const int n = u1 - u0;
    const int pa = u0 / pu, pb = u1 / pu;
    for (int it = tid; it < (pb - pa) * 32; it += DS_THREADS) {
        const int pi = pa + it / 32, j = it & 31;
        const int x0 = pi * pu - u0, x1 = x0 + pu - 1;
        const int wa = warp_of(x0, n), wb = warp_of(x1, n);
        float v = 0.f;
        for (int ww = wa; ww <= wb; ++ww) {
            int lo, hi;
            warp_split(u0, u1, ww, &lo, &hi);
            if (hi > lo) v += sh.wpart[ww][pi - lo / pu][j];
        }
        if (!sh.abort) part_out[(size_t)pi * 32 + j] = v;
    }
}

// ---------------------------------------------------------------------------
// N job (gate/up, down, lm_head): lane = block of a 4-row x 32-block tile
// ---------------------------------------------------------------------------
// One N tile of 4 rows into a4: lane = block of the tile's step.
template <int QT>
__device__ __forceinline__ void n_tile_dot(const uint8_t* tile, const float4 (&xr)[8], float sx, float (&a4)[4],
                                           int lane) {
    constexpr int QB = QTraits<QT>::QB;
    constexpr int NV = QTraits<QT>::NV;
    uint4 q[4][NV];
    float dsc[4];
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
#pragma unroll
        for (int v = 0; v < NV; ++v)
            q[rr][v] = *reinterpret_cast<const uint4*>(tile + 256 + (rr * 32 + lane) * QB + 16 * v);
        dsc[rr] = __fmul_rn(fp16_ftz_fast(*reinterpret_cast<const uint16_t*>(tile + (rr * 32 + lane) * 2)),
                            kDnUnscale);
    }
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) a4[rr] = fmaf(dsc[rr], dot32_dn<QT>(q[rr], xr, sx), a4[rr]);
}

template <int QT, int KIND>
__device__ __noinline__ void job_n(const DsParams& p, Shared& sh, uint8_t* smem, int layer, int job, int njobs,
                                   unsigned long long* best) {
    constexpr int NM = (KIND == K_GU) ? 2 : 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, cta = blockIdx.x, C = gridDim.x;
    float* xs = reinterpret_cast<float*>(smem);
    const DsN& nm = (KIND == K_GU) ? p.gu : (KIND == K_DN ? p.dn : p.head);
    if (!sh.abort) {
        if constexpr (KIND == K_GU)  // x = norm(res1 + wo output), res0 <- x
            stage_normed<QT>(p, sh, xs, p.res1, p.wo_part, p.wo.S, -1, p.layers[layer].ffn_norm, p.res0, true, 0);
        else if constexpr (KIND == K_DN)
            stage_n_plain<QT>(xs, p.h, p.Fl);
        else  // lm_head: x = norm(res0 + ydown) with the output norm
            stage_normed<QT>(p, sh, xs, p.res0, p.ydown, 1, -1, p.out_norm, nullptr, true, 0);
    }
    __syncthreads();
    stamp(p, job, 1);
    WarpCtx w{&p, &sh, smem + p.xs_bytes + (size_t)warp * p.nst * p.slot_bytes,
              smem_addr(smem + p.xs_bytes) + (uint32_t)(warp * p.nst * p.slot_bytes),
              smem_addr(&sh.bars[warp * DS_MAX_NST]), warp, lane, cta, C, njobs};
    const bool alt = NM == 2 && !p.gu_pair;  // gate/up tiles in alternating units
    int u0, u1, w0, w1;
    cta_units(p, KIND, cta, C, sh.am, &u0, &u1);
    warp_split(u0, u1, warp, &w0, &w1);
    const int per = nm.nsteps * (alt ? 2 : 1);  // units per row group
    const int g_first = w0 / per;
    float acc[NM][4];
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) acc[m][rr] = 0.f;
    auto emit = [&](int row, float v0, float v1) {
        if (row >= nm.rows) return;
        if constexpr (KIND == K_GU) {
            p.h[row] = silu_mul(v0, v1);
        } else if constexpr (KIND == K_DN) {
            p.ydown[row] = v0;
        } else {
            p.logits[row] = v0;
            const unsigned long long key =
                ((unsigned long long)ordered_bits(v0) << 32) | (0xFFFFFFFFu - (uint32_t)row);
            *best = key > *best ? key : *best;
            if (row == 0 && v0 != v0) *best = ~0ull;  // NaN at index 0 wins (greedy Sampler)
        }
    };
    auto flush = [&](int rg) {
        float v[NM][4];
#pragma unroll
        for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
                v[m][rr] = warp_sum(acc[m][rr]);
                acc[m][rr] = 0.f;
            }
        const bool whole = rg * per >= w0 && (rg + 1) * per <= w1;
        if (whole) {
            if (lane < 4) {
                float a = v[0][0], bb = v[NM - 1][0];
#pragma unroll
                for (int rr = 1; rr < 4; ++rr)
                    if (lane == rr) { a = v[0][rr]; bb = v[NM - 1][rr]; }
                emit(rg * 4 + lane, a, bb);
            }
        } else if (lane == 0) {
            float* dst = sh.npart[warp][rg == g_first ? 0 : 1];
#pragma unroll
            for (int m = 0; m < NM; ++m)
#pragma unroll
                for (int rr = 0; rr < 4; ++rr) dst[m * 4 + rr] = v[m][rr];
        }
    };
    int cur = -1;
    int consumed = sh.consumed[warp];
    // unit k = (row group rg, step s[, matrix m when alternating]), tracked without divisions
    int m = alt ? (w0 & 1) : 0;
    int rg = (alt ? (w0 >> 1) : w0) / nm.nsteps;
    int s = (alt ? (w0 >> 1) : w0) - rg * nm.nsteps;
    const int ntile = (NM == 2 && !alt) ? 2 : 1;  // tiles in a unit
    for (int k = w0; k < w1; ++k) {
        if (sh.abort) break;
        if (!ring_wait(w, consumed)) { sh.abort = 1; break; }
        if (rg != cur) {
            if (cur >= 0) flush(cur);
            cur = rg;
        }
        const uint8_t* slot = ring_slot(w, consumed);
        const int j = s * 32 + lane;
        if (j < nm.nb) {
            const float4* xv = reinterpret_cast<const float4*>(xs + (size_t)j * XP);
            float4 xr[8];
#pragma unroll
            for (int tt = 0; tt < 8; ++tt) xr[tt] = xv[tt];
            const float sx = xs[(size_t)j * XP + 32];
#pragma unroll 1
            for (int ti = 0; ti < ntile; ++ti) {
                float a4[4] = {0.f, 0.f, 0.f, 0.f};
                n_tile_dot<QT>(slot + ti * p.tile_n, xr, sx, a4, lane);
                const int which = alt ? m : ti;
#pragma unroll
                for (int rr = 0; rr < 4; ++rr) {
                    if (NM == 1 || which == 0) acc[0][rr] += a4[rr];
                    else acc[NM - 1][rr] += a4[rr];
                }
            }
        }
        __syncwarp();
        ++consumed;
        ring_fill(w, consumed);
        if (!alt || m == 1) {
            if (++s == nm.nsteps) { s = 0; ++rg; }
        }
        if (alt) m ^= 1;
    }
    if (cur >= 0 && !sh.abort) flush(cur);
    if (lane == 0) sh.consumed[warp] = consumed;
    __syncthreads();
    stamp(p, job, 2);
    // row groups shared by neighbouring warps: sum in warp order
    const int n = u1 - u0;
    if (n > 0 && !sh.abort) {
        const int ga = u0 / per, gb = (u1 - 1) / per;
        for (int it = tid; it < (gb - ga + 1) * 4; it += DS_THREADS) {
            const int rg2 = ga + it / 4, rr = it & 3;
            const int x0 = rg2 * per - u0, x1 = x0 + per - 1;
            const int wa = warp_of(x0, n), wb = warp_of(x1, n);
            if (wa == wb) continue;  // written by its warp
            float v0 = 0.f, v1 = 0.f;
            for (int ww = wa; ww <= wb; ++ww) {
                int lo, hi;
                warp_split(u0, u1, ww, &lo, &hi);
                if (hi <= lo) continue;
                const float* src = sh.npart[ww][rg2 == lo / per ? 0 : 1];
                v0 += src[rr];
                if (NM == 2) v1 += src[4 + rr];
            }
            emit(rg2 * 4 + rr, v0, v1);
        }
    }
}

// ---------------------------------------------------------------------------
// Attention (LlamaModel.attention, inference/LlamaModel.java:255-297)
// ---------------------------------------------------------------------------
// Sum over the 32 lanes of 32 values per lane: afterwards lane l holds the
// total of value l (butterfly reduce-scatter, 31 shuffles).
__device__ __forceinline__ float lane_transpose_sum(float (&v)[32], int lane) {
    int n = 32;
#pragma unroll
    for (int bit = 16; bit >= 1; bit >>= 1) {
        const bool upper = (lane & bit) != 0;
        n >>= 1;
#pragma unroll
        for (int t = 0; t < 16; ++t) {
            if (t < n) {
                const float send = upper ? v[t] : v[t + n];
                const float keep = upper ? v[t + n] : v[t];
                v[t] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
            }
        }
    }
    return v[0];
}

// One warp's online softmax over the positions of its units. Lanes own PL
// consecutive dims of every head (q, o); the UPC = 32 / G scores of a unit
// per head are reduced with one butterfly (lane g * UPC + i ends with the
// score of head g, position i), so each lane takes at most two exps.
template <int HD, int G>
struct AttWarp {
    static constexpr int PL = HD / 32;
    static constexpr int UPC = 32 / G;
    float q[G][PL], o[G][PL];
    float m_grp, l_grp;  // running max / sum of this lane's head group (g = lane / UPC)

    __device__ __forceinline__ void init(const float* qs, int lane) {
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < PL; ++e) {
                q[g][e] = qs[g * HD + lane * PL + e];
                o[g][e] = 0.f;
            }
        m_grp = -INFINITY;
        l_grp = 0.f;
    }

    // np <= UPC positions: K rows kr[i * HD], V rows vr[i * HD].
    __device__ __forceinline__ void unit(const float* kr, const float* vr, int np, float scale, int lane) {
        float sp[32];
#pragma unroll
        for (int v = 0; v < 32; ++v) sp[v] = 0.f;
#pragma unroll
        for (int i = 0; i < UPC; ++i) {
            if (i < np) {
                float kv[PL];
#pragma unroll
                for (int e = 0; e < PL; ++e) kv[e] = kr[i * HD + lane * PL + e];
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float dot = 0.f;
#pragma unroll
                    for (int e = 0; e < PL; ++e) dot = fmaf(kv[e], q[g][e], dot);
                    sp[g * UPC + i] = dot;
                }
            }
        }
        const float dot = lane_transpose_sum(sp, lane);
        const int i_l = lane % UPC;
        const bool valid = i_l < np;
        const float s = valid ? __fmul_rn(dot, scale) : -INFINITY;
        float mx = s;
#pragma unroll
        for (int off = UPC / 2; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float mn = fmaxf(m_grp, mx);  // finite: position 0 of the unit is valid
        const float corr = exp_ref(__fsub_rn(m_grp, mn));
        const float pe = valid ? exp_ref(__fsub_rn(s, mn)) : 0.f;
        float ps = pe;
#pragma unroll
        for (int off = UPC / 2; off >= 1; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        l_grp = fmaf(l_grp, corr, ps);
        m_grp = mn;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float cg = __shfl_sync(0xffffffffu, corr, g * UPC);
#pragma unroll
            for (int e = 0; e < PL; ++e) o[g][e] = __fmul_rn(o[g][e], cg);
        }
#pragma unroll
        for (int i = 0; i < UPC; ++i) {
            if (i < np) {
                float vv[PL];
#pragma unroll
                for (int e = 0; e < PL; ++e) vv[e] = vr[i * HD + lane * PL + e];
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float pg = __shfl_sync(0xffffffffu, pe, g * UPC + i);
#pragma unroll
                    for (int e = 0; e < PL; ++e) o[g][e] = fmaf(pg, vv[e], o[g][e]);
                }
            }
        }
    }
};

template <int HD, int G>
__device__ __noinline__ void job_att(const DsParams& p, Shared& sh, uint8_t* smem, int layer, int job, int pos,
                                     int njobs) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, cta = blockIdx.x, C = gridDim.x;
    float* xs = reinterpret_cast<float*>(smem);
    const AttMap am = sh.am;
    // ---- q, k, v of this head from the QKV part sums; RoPE ----
    if (am.active && !sh.abort) {
        const int nq = p.Hl * HD, nkv = p.Hkvl * HD;
        const int S = p.qkv.S;
        constexpr int nout = (G + 2) * HD;  // q heads of the group, then k, then v
        for (int i2 = tid; i2 < nout / 2; i2 += DS_THREADS) {
            const int o = 2 * i2;
            int c;
            if (o < G * HD) c = am.h * G * HD + o;
            else if (o < (G + 1) * HD) c = nq + am.h * HD + (o - G * HD);
            else c = nq + nkv + am.h * HD + (o - (G + 1) * HD);
            const int col = c >> 5, jj = c & 31;
            float a = 0.f, b = 0.f;
            for (int s = 0; s < S; ++s) {
                const float2 v = __ldcg(reinterpret_cast<const float2*>(p.qkv_part + ((size_t)col * S + s) * 32 + jj));
                a += v.x;
                b += v.y;
            }
            const int dd = o % HD;
            if (o < (G + 1) * HD) {
                // RoPE (core/Kernels.java:296-309): a' = fma(a, c, b * -s), b' = fma(b, c, a * s)
                const float cs = __ldg(p.rope_cos + (size_t)pos * HD + dd), sn = __ldg(p.rope_sin + (size_t)pos * HD + dd);
                const float a2 = fmaf(a, cs, __fmul_rn(b, -sn));
                const float b2 = fmaf(b, cs, __fmul_rn(a, sn));
                a = a2;
                b = b2;
            }
            if (o < G * HD) {
                sh.qs[o] = a;
                sh.qs[o + 1] = b;
            } else if (o < (G + 1) * HD) {
                sh.kn[dd] = a;
                sh.kn[dd + 1] = b;
            } else {
                sh.vn[dd] = a;
                sh.vn[dd + 1] = b;
            }
        }
    }
    __syncthreads();
    stamp(p, job, 1);
    const bool owner = am.active && am.j == am.nh - 1;
    if (owner && !sh.abort && tid < HD) {
        // KVCache.append (inference/KVCache.java:79-95) of the current position
        const DsLayer* ly = p.layers + layer;
        const size_t off = ((size_t)am.h * p.ctx + pos) * HD + tid;
        ly->kc[off] = sh.kn[tid];
        ly->vc[off] = sh.vn[tid];
    }
    // ---- per-warp online softmax over the warp's positions ----
    WarpCtx w{&p, &sh, smem + p.xs_bytes + (size_t)warp * p.nst * p.slot_bytes,
              smem_addr(smem + p.xs_bytes) + (uint32_t)(warp * p.nst * p.slot_bytes),
              smem_addr(&sh.bars[warp * DS_MAX_NST]), warp, lane, cta, C, njobs};
    AttWarp<HD, G> aw;
    aw.init(sh.qs, lane);
    int u0, u1, w0, w1;
    cta_units(p, K_ATT, cta, C, am, &u0, &u1);
    warp_split(u0, u1, warp, &w0, &w1);
    int consumed = sh.consumed[warp];
    for (int k = w0; k < w1; ++k) {
        if (sh.abort) break;
        if (!ring_wait(w, consumed)) { sh.abort = 1; break; }
        const int ps = am.p_lo + k * am.up;
        const int np = min(am.up, am.pend - ps);
        const float* slot = reinterpret_cast<const float*>(ring_slot(w, consumed));
        aw.unit(slot, slot + np * HD, np, p.scale, lane);
        __syncwarp();
        ++consumed;
        ring_fill(w, consumed);
    }
    if (lane == 0) sh.consumed[warp] = consumed;
    if (owner && warp == DS_WARPS - 1 && !sh.abort) aw.unit(sh.kn, sh.vn, 1, p.scale, lane);
    // ---- warp partials -> CTA partial (xs: [warps][G] m, [warps][G] l, [warps][G][HD] o) ----
    float* wm = xs;
    float* wl = xs + DS_WARPS * DS_G_MAX;
    float* wo = xs + 2 * DS_WARPS * DS_G_MAX;
    constexpr int UPC = 32 / G;
    if (am.active) {
        if (lane % UPC == 0) {
            wm[warp * DS_G_MAX + lane / UPC] = aw.m_grp;
            wl[warp * DS_G_MAX + lane / UPC] = aw.l_grp;
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < AttWarp<HD, G>::PL; ++e)
                wo[((size_t)warp * G + g) * HD + lane * AttWarp<HD, G>::PL + e] = aw.o[g][e];
    }
    __syncthreads();
    stamp(p, job, 2);
    if (am.active && !sh.abort) {
        if (warp < G) {
            const int g = warp;
            const float mw = lane < DS_WARPS ? wm[lane * DS_G_MAX + g] : -INFINITY;
            const float M = warp_max(mw);
            const float wgt = (lane < DS_WARPS && mw != -INFINITY) ? exp_ref(__fsub_rn(mw, M)) : 0.f;
            const float L = warp_sum(lane < DS_WARPS ? wl[lane * DS_G_MAX + g] * wgt : 0.f);
            if (lane < DS_WARPS) sh.aw[g][lane] = wgt;
            if (lane == 0) { sh.red[g] = M; sh.al[g] = L; }
        }
        __syncthreads();
        float* dst = p.apart + ((size_t)am.h * p.att_max_ctas + am.j) * G * (HD + 2);
        for (int i = tid; i < G * HD; i += DS_THREADS) {
            const int g = i / HD, dd = i - g * HD;
            float acc = 0.f;
            for (int ww = 0; ww < DS_WARPS; ++ww) acc = fmaf(wo[((size_t)ww * G + g) * HD + dd], sh.aw[g][ww], acc);
            dst[g * (HD + 2) + dd] = acc;
            if (dd == 0) {
                dst[g * (HD + 2) + HD] = sh.red[g];
                dst[g * (HD + 2) + HD + 1] = sh.al[g];
            }
        }
    } else {
        __syncthreads();
    }
    // ---- the last CTA of the head merges the CTA partials in CTA order ----
    __syncthreads();
    if (tid == 0) {
        sh.last = 0;
        if (am.active && !sh.abort) {
            __threadfence();
            const unsigned t = atomicAdd(&p.tickets[am.h], 1u);
            if (t == (unsigned)(am.nh - 1)) {
                sh.last = 1;
                p.tickets[am.h] = 0u;
                __threadfence();
            }
        }
    }
    __syncthreads();
    if (sh.last) {
        const float* base = p.apart + (size_t)am.h * p.att_max_ctas * G * (HD + 2);
        if (warp < G) {
            const int g = warp;
            const float mj = lane < am.nh ? __ldcg(base + ((size_t)lane * G + g) * (HD + 2) + HD) : -INFINITY;
            const float lj = lane < am.nh ? __ldcg(base + ((size_t)lane * G + g) * (HD + 2) + HD + 1) : 0.f;
            const float M = warp_max(mj);
            const float wgt = (lane < am.nh && mj != -INFINITY) ? exp_ref(__fsub_rn(mj, M)) : 0.f;
            const float L = warp_sum(lj * wgt);
            if (lane < DS_ATT_MAX) sh.aw[g][lane] = wgt;
            if (lane == 0) sh.al[g] = L;
        }
        __syncthreads();
        for (int i = tid; i < G * HD; i += DS_THREADS) {
            const int g = i / HD, dd = i - g * HD;
            float acc = 0.f;
            for (int jj = 0; jj < am.nh; ++jj)
                acc = fmaf(__ldcg(base + ((size_t)jj * G + g) * (HD + 2) + dd), sh.aw[g][jj], acc);
            p.att[((size_t)am.h * G + g) * HD + dd] = __fdiv_rn(acc, sh.al[g]);
        }
    }
}

// ---------------------------------------------------------------------------
// The step kernel
// ---------------------------------------------------------------------------
template <int QT, int HD>
__global__ void __launch_bounds__(DS_THREADS, 1) decode_step_kernel(const __grid_constant__ DsParams p) {
    extern __shared__ __align__(128) uint8_t ds_smem[];
    __shared__ Shared sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x, C = gridDim.x;
    const int njobs = 5 * p.L + 1;
    const int pos = (int)p.pos[0];
    const int token = p.tokens[0];
    const int G = p.Hl / p.Hkvl;

    if (tid == 0) {
        sh.abort = 0;
        sh.target = *reinterpret_cast<const volatile unsigned*>(p.bar + 1);  // epoch of this launch
        sh.am = att_map(p, cta, C, pos);
    }
    if (lane == 0) {
        for (int s = 0; s < p.nst; ++s) mbar_init(smem_addr(&sh.bars[warp * DS_MAX_NST + s]), 1);
        Cursor& c = sh.cur[warp];
        c.issued = 0;
        c.job = -1;
        c.kind = 0;
        c.k = c.kend = 0;
        c.ta = c.tb = nullptr;
        c.stride = 0;
        c.ubytes = c.npos = 0;
        sh.consumed[warp] = 0;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    {
        WarpCtx w{&p, &sh, ds_smem + p.xs_bytes + (size_t)warp * p.nst * p.slot_bytes,
                  smem_addr(ds_smem + p.xs_bytes) + (uint32_t)(warp * p.nst * p.slot_bytes),
                  smem_addr(&sh.bars[warp * DS_MAX_NST]), warp, lane, cta, C, njobs};
        ring_fill(w, 0);
    }

    unsigned long long best = 0ull;
    for (int job = 0; job < njobs; ++job) {
        const bool head = job == njobs - 1;
        const int kind = head ? K_HEAD : job % 5;
        const int layer = head ? p.L - 1 : job / 5;
        if (job > 0) grid_barrier(p, sh);
        stamp(p, job, 0);
        switch (kind) {
            case K_QKV: job_t<QT>(p, sh, ds_smem, K_QKV, layer, job, token, njobs); break;
            case K_ATT:
                if (G == 8) job_att<HD, 8>(p, sh, ds_smem, layer, job, pos, njobs);
                else if (G == 4) job_att<HD, 4>(p, sh, ds_smem, layer, job, pos, njobs);
                else if (G == 2) job_att<HD, 2>(p, sh, ds_smem, layer, job, pos, njobs);
                else job_att<HD, 1>(p, sh, ds_smem, layer, job, pos, njobs);
                break;
            case K_WO: job_t<QT>(p, sh, ds_smem, K_WO, layer, job, token, njobs); break;
            case K_GU: job_n<QT, K_GU>(p, sh, ds_smem, layer, job, njobs, &best); break;
            case K_DN: job_n<QT, K_DN>(p, sh, ds_smem, layer, job, njobs, &best); break;
            default: job_n<QT, K_HEAD>(p, sh, ds_smem, layer, job, njobs, &best); break;
        }
        stamp(p, job, 3);
        __syncthreads();
    }

    // ---- greedy argmax (Sampler.sample's greedy path, inference/Sampler.java:56-67) ----
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if (lane == 0) sh.best[warp] = best;
    __syncthreads();
    if (tid == 0) {
        sh.last = 0;
        if (!sh.abort) {
            for (int ww = 1; ww < DS_WARPS; ++ww) best = sh.best[ww] > best ? sh.best[ww] : best;
            best = sh.best[0] > best ? sh.best[0] : best;
            atomicMax(p.argkey, best);
            __threadfence();
            const unsigned t = atomicAdd(&p.tickets[p.Hkvl], 1u);
            if (t == (unsigned)(C - 1)) {
                __threadfence();
                const int tok = key_index(__ldcg(p.argkey));
                p.argmax_out[0] = tok;
                if (p.greedy) {
                    const int n = p.gen_count[0];
                    p.gen_out[n] = tok;
                    p.gen_count[0] = n + 1;
                    p.tokens[0] = tok;
                    p.pos[0] = pos + 1;
                }
                *p.argkey = 0ull;
                p.tickets[p.Hkvl] = 0u;
                // every CTA has passed every grid barrier: the next launch starts from here
                p.bar[1] = sh.target;
            }
        }
    }
    // drain: this warp's copies still in flight (only after an abort)
    if (lane == 0) {
        int consumed = sh.consumed[warp];
        const int issued = sh.cur[warp].issued;
        const uint32_t bars = smem_addr(&sh.bars[warp * DS_MAX_NST]);
        while (consumed < issued) {
            const unsigned long long t0 = gtimer();
            const int slot = consumed & (p.nst - 1);
            const uint32_t bar = bars + slot * 8, par = (uint32_t)(consumed / p.nst) & 1u;
            while (!mbar_try(bar, par) && gtimer() - t0 < kWaitNs) {
            }
            ++consumed;
        }
    }
}

template <int QT, int HD>
const void* kernel_ptr() {
    return reinterpret_cast<const void*>(&decode_step_kernel<QT, HD>);
}

const void* pick_kernel(int qtype, int hd) {
    if (qtype == AT_GGML_Q4_0) return hd == 128 ? kernel_ptr<AT_GGML_Q4_0, 128>() : kernel_ptr<AT_GGML_Q4_0, 64>();
    return hd == 128 ? kernel_ptr<AT_GGML_Q8_0, 128>() : kernel_ptr<AT_GGML_Q8_0, 64>();
}

std::mutex g_ds_mu;

}  // namespace

bool decode_step_configure(DsParams* p, int C) {
    if (p->qtype != AT_GGML_Q4_0 && p->qtype != AT_GGML_Q8_0) return false;
    if (p->hd != 64 && p->hd != 128) return false;
    if (p->Hkvl <= 0 || p->Hl % p->Hkvl != 0 || p->Hl / p->Hkvl > DS_G_MAX) return false;
    if (p->d % 32 != 0 || p->d > 4 * DS_TV * DS_THREADS || p->Fl % 32 != 0) return false;
    const int qb = p->qtype == AT_GGML_Q4_0 ? 16 : 32;
    p->tile_t = 32 * (2 + qb);
    p->tile_n = 4 * 32 * (2 + qb);
    // T matrices: S parts per block column minimizing the largest CTA's units
    auto setup_t = [&](DsT& t, int E, int outs, bool final_out) {
        t.E = E;
        t.ngroups = (E + 31) / 32;
        t.ncols = outs / 32;
        t.nu = (t.ngroups + DS_RT - 1) / DS_RT;
        int best_s = 1;
        int64_t best = INT64_MAX;
        for (int S = 1; S <= (final_out ? 1 : 8); ++S) {
            if (t.nu % S) continue;
            const int64_t P = (int64_t)t.ncols * S, pu = t.nu / S;
            const int64_t worst = (P + C - 1) / C * pu;
            if (worst < best) { best = worst; best_s = S; }
        }
        t.S = best_s;
        // parts one warp's units can touch
        const int64_t P = (int64_t)t.ncols * t.S, pu = t.nu / t.S;
        const int64_t per_warp = ((P + C - 1) / C * pu + DS_WARPS - 1) / DS_WARPS;
        return (per_warp + pu - 1) / pu + 1 <= DS_MAXWP;
    };
    if (!setup_t(p->qkv, p->d, (p->Hl + 2 * p->Hkvl) * p->hd, false)) return false;
    if (!setup_t(p->wo, p->Hl * p->hd, p->d, true)) return false;
    auto setup_n = [](DsN& n, int rows, int cols) {
        n.rows = rows;
        n.nb = cols / 32;
        n.ngroups = (rows + 3) / 4;
        n.nsteps = (n.nb + 31) / 32;
    };
    setup_n(p->gu, p->Fl, p->d);
    setup_n(p->dn, p->d, p->Fl);
    setup_n(p->head, p->Vl, p->d);
    if (p->qkv.ngroups % DS_RT || p->wo.ngroups % DS_RT) return false;  // T units contiguous in memory
    p->att_max_ctas = (std::min(C, p->Hkvl * DS_ATT_MAX) + p->Hkvl - 1) / p->Hkvl;
    const int G = p->Hl / p->Hkvl;
    size_t xs = 0;
    xs = std::max(xs, (size_t)p->qkv.ngroups * 32 * 4);
    xs = std::max(xs, (size_t)p->wo.ngroups * 32 * 4);
    xs = std::max(xs, (size_t)(p->d / 32) * XP * 4);
    xs = std::max(xs, (size_t)(p->Fl / 32) * XP * 4);
    xs = std::max(xs, (size_t)(2 * DS_WARPS * DS_G_MAX + DS_WARPS * G * p->hd) * 4);
    xs = (xs + 127) / 128 * 128;
    p->xs_bytes = (int)xs;
    const size_t budget = 232448 - kStaticSmem;
    // gate/up units pair the w1 and w3 tiles of one (row group, step) when two
    // slots of that size per warp fit; otherwise the tiles alternate
    for (int pair = 1; pair >= 0; --pair) {
        const int slot = (int)std::max<int64_t>(p->tile_n * (pair ? 2 : 1), DS_RT * p->tile_t);
        int nst = 0;
        for (int s = DS_MAX_NST; s >= 2; s >>= 1)
            if (xs + (size_t)DS_WARPS * s * slot <= budget) { nst = s; break; }
        if (nst) {
            p->gu_pair = pair;
            p->slot_bytes = slot;
            p->nst = nst;
            return true;
        }
    }
    return false;
}

size_t decode_step_smem(const DsParams& p) { return (size_t)p.xs_bytes + (size_t)DS_WARPS * p.nst * p.slot_bytes; }

void launch_decode_step(const DsParams& p, int num_ctas, cudaStream_t s) {
    const void* fn = pick_kernel(p.qtype, p.hd);
    const size_t smem = decode_step_smem(p);
    {
        std::lock_guard<std::mutex> lk(g_ds_mu);
        AT_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_ctas);
    cfg.blockDim = dim3(DS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {const_cast<DsParams*>(&p)};
    AT_CUDA(cudaLaunchKernelExC(&cfg, fn, args));
}

}  // namespace at
