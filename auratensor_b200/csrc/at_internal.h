// Internal declarations shared by the translation units of libauratensor_cuda.so.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

#include "../../include/auratensor.h"

namespace at {

// Error carrying an AT_ERR_* status; every C-ABI entry point converts it to
// a return code and stores the message for at_last_error().
struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void set_last_error(const std::string& msg);

[[noreturn]] inline void fail(int code, const std::string& msg) { throw Error(code, msg); }

inline void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        int code = (e == cudaErrorMemoryAllocation) ? AT_ERR_OOM : AT_ERR_CUDA;
        fail(code, std::string(what) + ": " + cudaGetErrorString(e));
    }
}
#define AT_CUDA(x) ::at::cuda_check((x), #x)
#define AT_REQUIRE(cond, code, msg) do { if (!(cond)) ::at::fail((code), (msg)); } while (0)

// Runs `body` and converts exceptions into status codes.
template <class F>
int guard(F&& body) {
    try {
        body();
        return AT_OK;
    } catch (const Error& e) {
        set_last_error(e.what());
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("host allocation failed");
        return AT_ERR_OOM;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return AT_ERR_CUDA;
    }
}

struct NcclApi;  // dlopen'd NCCL entry points

}  // namespace at

struct at_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;      // stream every launch of this context uses
    cudaStream_t own_stream = nullptr;  // stream created with the context
    int num_sms = 148;
    // tensor parallelism
    int rank = 0;
    int world = 1;
    void* nccl_comm = nullptr;  // ncclComm_t
};

// Tiled device layout of one quantized matrix: a lossless re-layout of whole
// GGUF blocks (the fp16 scale and the quant bytes of every block are moved,
// never re-quantized) so that the bytes one warp step consumes are contiguous.
//  Orientation N (blocks along the rows): tiles of 4 rows x 32 blocks;
//    tile (g, s) = rows 4g..4g+3, blocks 32s..32s+31, at (g * nsteps + s) * tile_bytes;
//    inside: scales [4][32] u16, then quant bytes [4][32][QB].
//  Orientation T (blocks along the columns): tiles of 32 rows x 1 block column;
//    tile (c, g) = block column c, rows 32g..32g+31, at (c * ngroups + g) * tile_bytes;
//    inside: scales [32] u16, then quant bytes [32][QB].
// QB = 16 (Q4_0) or 32 (Q8_0). Padding rows/blocks are zero (scale 0 -> weight 0).
// F32 matrices keep row-major floats in `f32`.
struct at_qmat {
    at_ctx* ctx = nullptr;
    int type = AT_GGML_Q4_0;
    int orient = AT_ORIENT_N;
    int64_t rows = 0, cols = 0;
    uint8_t* tiles = nullptr;
    int64_t tile_bytes = 0;
    int64_t nsteps = 0;    // N: 32-block steps per row group
    int64_t ngroups = 0;   // N: 4-row groups; T: 32-row groups
    size_t bytes = 0;
    float* f32 = nullptr;
    bool owns = true;
};

namespace at {

constexpr int QK = 32;
inline int quant_bytes(int type) { return type == AT_GGML_Q4_0 ? 16 : 32; }
inline int block_bytes(int type) { return type == AT_GGML_Q4_0 ? 18 : 34; }
// Bytes of n elements of raw GGUF blocks (Q4_0, Q8_0, Q6_K), -1 for other types.
inline int64_t raw_bytes(int type, int64_t n) {
    if (type == AT_GGML_Q4_0) return n / 32 * 18;
    if (type == AT_GGML_Q8_0) return n / 32 * 34;
    if (type == AT_GGML_Q6_K) return n / 256 * 210;
    return -1;
}

// Byte offsets of the scale and of the quant bytes of block (row, b) (b in
// units of 32-element blocks) inside the tiles of a matrix.
struct QTileMap {
    int orient, qb;
    int64_t tile_bytes, nsteps, ngroups;
    __host__ __device__ __forceinline__ void offsets(int64_t row, int64_t b, int64_t* d_off, int64_t* q_off) const {
        if (orient == AT_ORIENT_N) {
            const int64_t g = row >> 2, r = row & 3, s = b >> 5, l = b & 31;
            const int64_t t = (g * nsteps + s) * tile_bytes;
            *d_off = t + (r * 32 + l) * 2;
            *q_off = t + 256 + (r * 32 + l) * qb;
        } else {
            const int64_t g = row >> 5, l = row & 31;
            const int64_t t = (b * ngroups + g) * tile_bytes;
            *d_off = t + l * 2;
            *q_off = t + 64 + l * qb;
        }
    }
};
inline QTileMap tile_map(const at_qmat* m) {
    return QTileMap{m->orient, quant_bytes(m->type), m->tile_bytes, m->nsteps, m->ngroups};
}

// Allocates (zeroed) the tiles of `m` (type/orient/rows/cols already set).
void qmat_alloc(at_qmat* m);
void qmat_free(at_qmat* m);
// Repack raw GGUF blocks (row-major stream, device memory) into the tiles of
// `m`, taking rows [r0, r0+m->rows) and block-columns [c0/32, ...) of a source
// matrix with `src_cols` columns.
void qmat_fill_from_blocks(at_qmat* m, const uint8_t* src_dev, int64_t src_cols, int64_t r0, int64_t c0,
                           cudaStream_t s);
// Copies rows [src_r0, +n_rows) x cols [src_c0, +n_cols) of a raw row-major
// block matrix with src_cols columns into `m` at (dst_r0, dst_c0).
// nib_split: the source Q4_0 blocks hold llama.cpp's split-halves nibble
// order (element k low, k + 16 high nibble of byte k); they are stored in the
// interleaved order (a lossless permutation inside each block).
void qmat_fill_region(at_qmat* m, const uint8_t* src_dev, int64_t src_cols, int64_t src_r0, int64_t src_c0,
                      int64_t n_rows, int64_t n_cols, int64_t dst_r0, int64_t dst_c0, cudaStream_t s,
                      int nib_split = 0);
// F32 / F16 source into an f32 matrix.
void qmat_fill_from_float(at_qmat* m, const void* src_dev, int src_type, int64_t src_cols, int64_t r0,
                          int64_t c0, cudaStream_t s);

// Q6_K matrices (q6k.cu): orientation N, whole blocks padded to 224 bytes.
void q6k_alloc(at_qmat* m);
void q6k_fill_rows(at_qmat* m, const uint8_t* src_dev, int64_t src_cols, int64_t src_r0, int64_t n_rows,
                   int64_t dst_r0, cudaStream_t s);
void q6k_export(const at_qmat* m, uint8_t* dst_dev, cudaStream_t s);
void launch_q6k_dequant(const uint8_t* src_dev, float* dst_dev, int64_t n, cudaStream_t s);
void launch_q6k_embed(const at_qmat* tok, const int* tokens, int B, int d, float* xa, float* y,
                      unsigned long long* argkeys, unsigned* step, cudaStream_t s);

// Prologue/epilogue variants of the fused GEMV kernels.
enum class Pro { Plain, AddNorm };         // x from global, or x = norm(xin + yin) (F7 residual)
enum class Epi { Plain, SiluMul, QkvRope }; // y; silu(g)*u; RoPE + KV append

struct GemvArgs {
    const float* x = nullptr;     // Pro::Plain input [B][in]
    const float* xin = nullptr;   // Pro::AddNorm: residual stream (normed, F7)
    const float* yin = nullptr;   // Pro::AddNorm: projection output to add (may be null)
    const float* gamma = nullptr; // Pro::AddNorm: norm weight
    float* xout = nullptr;        // Pro::AddNorm: normed x written by CTA 0
    float eps = 1e-5f;
    float* y = nullptr;           // output [B][out]
    int x_stride = 0;             // floats between batch rows of x / xin / yin / xout
    int y_stride = 0;             // floats between batch rows of y
    // Epi::SiluMul
    const at_qmat* m2 = nullptr;
    // Epi::QkvRope
    const float* rope_cos = nullptr;   // [ctx][hd]
    const float* rope_sin = nullptr;
    const int64_t* pos = nullptr;      // [B] device
    float* kcache = nullptr;           // [B][L][Hkv][ctx][hd] base of this layer slice
    float* vcache = nullptr;
    int8_t* kq = nullptr;              // Q8_0 KV cache (kq non-null): quants at the fp32 element
    int8_t* vq = nullptr;              // index, one fp16 scale per 32 elements
    uint16_t* ksc = nullptr;
    uint16_t* vsc = nullptr;
    int64_t kv_slot_stride = 0;        // floats between sequence slots
    int head_dim = 0, n_q_cols = 0, n_kv_cols = 0, ctx_len = 0;
    // T split-K scratch (partials + tile counters)
    float* scratch = nullptr;
    unsigned* counters = nullptr;
};

// pdl: launch with programmatic stream serialization (the kernel prefetches
// its weights before waiting on the previous kernel in the stream).
void launch_gemv_n(const at_qmat* m, int batch, Pro pro, Epi epi, const GemvArgs& a, int num_sms,
                   cudaStream_t s, bool pdl = false);
void launch_gemv_t(const at_qmat* m, int batch, Pro pro, Epi epi, const GemvArgs& a, int num_sms,
                   cudaStream_t s, bool pdl = false);
// Scratch floats / counters a T or N launch needs for (m, batch); the N
// figure covers every epilogue.
void gemv_t_scratch_need(const at_qmat* m, int batch, int num_sms, size_t* floats, size_t* counters);
void gemv_n_scratch_need(const at_qmat* m, int batch, int num_sms, size_t* floats, size_t* counters);
// Q6_K orientation-N GEMV (q6k.cu): Pro::Plain or Pro::AddNorm, Epi::Plain.
void launch_gemv_q6k(const at_qmat* m, int batch, Pro pro, const GemvArgs& a, int num_sms, cudaStream_t s);
// Tensor-core prompt GEMM (gemm_tc.cu): y[t][:] = W x[t][:], bf16 operands,
// FP32 sums; xbf is a 128-byte aligned device buffer of at least T x in bf16
// (the activations are converted into it; with x null it already holds them,
// rows of `in` elements); ws (FP32, may be null) holds the
// partials when K is split across CTAs (gemm_tc_splits(m, T) x T x out
// floats); *err records a bounded wait that ran out (2). With opt.defer,
// split partials stay in ws ([split][T][out], rows of `out` floats) for the
// consumer to sum in split order, and the split count is returned there (1:
// y holds the result).
// Causal prompt attention on the tensor cores (prompt_attn_tc.cu): q [T][Hl
// x hd] after RoPE, the layer's KV cache of one slot (kc / vc FP32, or Q8_0
// quants with ksc / vsc scales when kvq), att [T][Hl x hd]; false (nothing
// launched) for head_dim other than 64 / 128 or G = Hl / Hkvl not in 1, 2, 4,
// 8. *err records a bounded wait that ran out (2).
// With att_bf non-null the output is written there in bf16 (the wo GEMM's
// staged operand, rounded as its conversion would) instead of att.
bool launch_prompt_attn_tc(int hd, int G, bool kvq, int Hkvl, int T, cudaStream_t s, const float* q, const float* kc,
                           const float* vc, const uint16_t* ksc, const uint16_t* vsc, float* att, int64_t p0, int Hl,
                           int ctx, float scale, int* err, __nv_bfloat16* att_bf = nullptr);
struct GemmTcOut {
    int* defer = nullptr;  // split count out; partials left in ws
};
int gemm_tc_splits(const at_qmat* m, int T, int num_sms);
void launch_gemm_tc(const at_qmat* m, const float* x, int x_stride, float* y, int y_stride, int T, void* xbf,
                    size_t xbf_bytes, float* ws, size_t ws_bytes, int num_sms, int* err, cudaStream_t s,
                    const GemmTcOut& opt = GemmTcOut{});
void launch_sgemv_f32(const float* A, const float* x, float* y, int M, int K, int batch, int a_ld,
                      cudaStream_t s);

// ---------------------------------------------------------------------------
// Persistent decode step (decode_step.cu): one launch runs a whole batch-1
// forwardStep (every layer, the lm_head and the argmax) on one CTA per SM,
// phases separated by grid barriers.
// ---------------------------------------------------------------------------
struct DsLayer {  // device table, one entry per layer
    const uint8_t* qkv;    // orientation-T tiles, inputs d, outputs (Hl + 2 Hkvl) hd
    const uint8_t* wo;     // orientation-T tiles, inputs Hl hd, outputs d
    const uint8_t* w1;     // orientation-N tiles [Fl][d]
    const uint8_t* w3;
    const uint8_t* w2;     // orientation-N tiles [d][Fl]
    const float* attn_norm;
    const float* ffn_norm;
    float* kc;             // this layer's K cache of slot 0: [Hkvl][ctx][hd]
    float* vc;
};

struct DsT {               // an orientation-T matrix in the step
    int E;                 // inputs (rows)
    int ngroups;           // 32-row tile groups per block column
    int ncols;             // block columns (outputs / 32)
    int nu;                // units (4 row tiles) per block column
    int S;                 // parts per block column (nu % S == 0); output = sum of the S part sums
};

struct DsN {               // an orientation-N matrix in the step
    int rows, nb;          // outputs, 32-element blocks per row
    int ngroups, nsteps;   // 4-row groups, 32-block steps per group
};

struct DsParams {
    const DsLayer* layers;
    int L;
    int qtype, hd;
    int d, Hl, Hkvl, Fl, Vl, ctx;
    float eps, scale;
    int64_t tile_t, tile_n; // bytes per T tile / N tile
    DsT qkv, wo;
    DsN gu, dn, head;
    const uint8_t* tok_tiles;
    QTileMap tok_map;
    const uint8_t* out_tiles;
    const float* out_norm;
    const float* rope_cos;  // [ctx][hd]
    const float* rope_sin;
    int* tokens;            // [1]
    int64_t* pos;           // [1]
    // activations and exchange buffers
    float* res0;            // normed residual stream (ping-pong)
    float* res1;
    float* ydown;           // down projection output [d]
    float* qkv_part;        // [qkv.ncols * qkv.S][32]
    float* wo_part;         // [wo.ncols * wo.S][32]
    float* h;               // silu(gate) * up [Fl]
    float* att;             // attention output [Hl * hd]
    float* apart;           // attention partials [Hkvl][att_max_ctas][G][hd + 2]
    float* logits;          // [Vl]
    int att_max_ctas;       // CTAs per KV head at most
    int nst;                // weight-ring slots per warp (power of two)
    int slot_bytes;         // bytes per ring slot
    int gu_pair;            // gate/up units hold the w1 and the w3 tile of one (row group, step)
    int xs_bytes;           // activation staging bytes
    unsigned* tickets;      // [Hkvl] attention merge tickets, then one for the argmax
    unsigned* bar;          // [2]: grid-barrier arrivals, epoch
    int* err;               // error word (0 = ok)
    unsigned long long* argkey;
    int* argmax_out;
    int greedy;             // advance token / position and append to gen_out
    int* gen_out;
    int* gen_count;
    unsigned long long* stamps;  // optional [gridDim][5 L + 1][4] globaltimer per job
};

// Device sampler (sample.cu): Sampler.sample per logits row.
struct SampleRow {
    float temperature;
    int top_k;
    float top_p;
    float penalty;             // repetition penalty (1: none)
    float r;                   // the row's uniform draw in [0, 1) when rng is null
    unsigned long long* rng;   // device: java.util.Random state advanced per call (unseeded rows), or null
    const int* hist;           // device: penalty history (may be null)
    const int* hist_len;       // device: its length (may be null: empty)
    int* cnt;                  // device: [V] occurrence counts, zero between calls (needed with a penalty)
};
void launch_sample(float* logits_dev, int B, int V, int stride, const SampleRow* rows_dev, int* out_dev,
                   cudaStream_t s);
// picked -> tokens, pos + 1, seq[b][*step] (seq may be null; *step advances
// when step is not null), and the penalty history append of the rows whose
// append flag is set (append null: every row).
void launch_sample_advance(const int* picked, int B, int* tokens, int64_t* pos, int* seq, int seq_stride, int* step,
                           int* hist, int hist_stride, int* hist_len, const int* append, cudaStream_t s);
int sample_k_max();

// Model hooks of the request scheduler (sched.cpp); defined in model.cu.
int model_max_batch(const at_model* m);
int64_t model_ctx_len(const at_model* m);
int model_vocab(const at_model* m);
bool model_slot_prompt(const at_model* m);  // prompts can run into any KV slot
// Row `slot`'s sampler settings and penalty history (cfg null: an idle greedy row).
void sched_set_row(at_model* m, int slot, const at_sampler_config* cfg, const int* history, int n);
void sched_step(at_model* m, int B, const int* tokens, const int64_t* positions, const int* append, int* picked);
void sched_prompt(at_model* m, int slot, const int* tokens, int n);
void sched_reset_slot(at_model* m, int slot);
// The reference's r: a fresh java.util.Random(seed).nextFloat() (seed 0: an unseeded generator).
float sampler_r(int64_t seed);

// Shared memory the step kernel needs (dynamic bytes) and its launch.
size_t decode_step_smem(const DsParams& p);
void launch_decode_step(const DsParams& p, int num_ctas, cudaStream_t s);
// Picks the part counts of the T matrices, the ring depth and the staging
// size for num_ctas CTAs; false when the shapes fall outside the kernel.
bool decode_step_configure(DsParams* p, int num_ctas);

}  // namespace at
