/*
 * auratensor.h — C ABI of libauratensor_cuda.so, the B200 (sm_100a) engine for
 * AuraTensor's quantized-matvec decode path.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, and
 * returns an int status (AT_OK = 0, negative = error class). The message of
 * the last failure on the calling thread is returned by at_last_error().
 * Device pointers are CUDA device addresses on the context's device.
 *
 * The comment above each declaration names the reference interface it
 * replaces (paths relative to src/main/java/io/auratensor/ in AuraTensor).
 * The Java side binds these through java.lang.foreign downcall handles.
 */
#ifndef AURATENSOR_H
#define AURATENSOR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The Java shim maps them to the exception classes the
 * reference throws for the same condition. */
#define AT_OK                 0
#define AT_ERR_INVALID_ARG   -1  /* IllegalArgumentException  (core/Kernels.java:55-57,101-113,332-340) */
#define AT_ERR_STATE         -2  /* IllegalStateException     (inference/KVCache.java:83-85)           */
#define AT_ERR_UNSUPPORTED   -3  /* UnsupportedOperationException (format/GgufFile.java:157-163)       */
#define AT_ERR_IO            -4  /* IOException               (format/GgufFile.java:105-117)           */
#define AT_ERR_CUDA          -5  /* CUDA runtime failure                                                */
#define AT_ERR_NCCL          -6  /* NCCL failure                                                        */
#define AT_ERR_OOM           -7  /* device allocation failed                                            */
#define AT_ERR_TIMEOUT       -8  /* a bounded wait ran out                                              */

/* GGUF tensor type codes (format/GgufTensorType.java:15-27). Q6_K (256
 * elements per 210-byte block, quant/Q6_K.java) is taken for token_embd and
 * output only, as real llama.cpp exports store them. */
#define AT_GGML_F32   0
#define AT_GGML_F16   1
#define AT_GGML_Q4_0  2
#define AT_GGML_Q8_0  8
#define AT_GGML_Q6_K 14

/* Byte layouts of a model's tensors. 0 is the reference's: Q4_0 nibbles
 * interleaved (element 2k = low nibble of byte k, quant/Q4_0.java:21-22) and
 * attention weights read as [in][out] (inference/LlamaModel.java:326-369).
 * llama.cpp exports use split-halves Q4_0 nibbles (element k = low nibble,
 * element k + 16 = high nibble of byte k) and [out][in] attention weights
 * like every other matrix. Split-halves blocks are re-ordered to the
 * interleaved order at upload (a lossless nibble permutation inside each
 * block); [out][in] attention weights run through the orientation-N GEMV. */
#define AT_LAYOUT_Q4_SPLIT_HALVES 1
#define AT_LAYOUT_ATTN_OUT_IN     2
#define AT_LAYOUT_LLAMA_CPP       (AT_LAYOUT_Q4_SPLIT_HALVES | AT_LAYOUT_ATTN_OUT_IN)

/* GEMV orientations of a row-major block matrix W[rows][cols] whose
 * quantization blocks run along cols (inference/LlamaModel.java:326-369).
 *   AT_ORIENT_N: y[b][r] = sum_c W[r][c] * x[b][c]   (ffn, lm_head: [out][in])
 *   AT_ORIENT_T: y[b][c] = sum_r W[r][c] * x[b][r]   (wq/wk/wv/wo: [in][out]) */
#define AT_ORIENT_N 0
#define AT_ORIENT_T 1

typedef struct at_ctx   at_ctx;    /* one device, one stream, optional NCCL communicator */
typedef struct at_qmat  at_qmat;   /* device-resident quantized matrix (planar re-layout) */
typedef struct at_model at_model;  /* device-resident Llama model + KV cache              */

/* ---- runtime ------------------------------------------------------------ */
const char* at_version(void);
/* Copies the calling thread's last error message into buf; returns its length. */
int at_last_error(char* buf, size_t len);
int at_device_count(int* n);
/* New: device context (the reference runs on the calling Java thread). */
int at_ctx_create(int device, at_ctx** out);
int at_ctx_destroy(at_ctx* ctx);
int at_ctx_synchronize(at_ctx* ctx);
/* Returns the cudaStream_t the context launches on. */
int at_ctx_stream(at_ctx* ctx, void** stream);
/* Makes the context launch on `stream` (a cudaStream_t of the same device, for
 * example the host framework's current stream); NULL restores its own stream. */
int at_ctx_set_stream(at_ctx* ctx, void* stream);

/* ---- memory: Tensor.allocate / wrap / close (core/Tensor.java:88-120,234-239) */
int at_alloc(at_ctx* ctx, size_t bytes, void** dptr);
int at_free(at_ctx* ctx, void* dptr);
int at_memcpy_h2d(at_ctx* ctx, void* dst_dev, const void* src_host, size_t bytes);
int at_memcpy_d2h(at_ctx* ctx, void* dst_host, const void* src_dev, size_t bytes);
int at_memset_zero(at_ctx* ctx, void* dst_dev, size_t bytes);

/* ---- fp16: Fp16.toFloat (core/Fp16.java:19-37), subnormals flush to zero -- */
int at_fp16_to_f32(at_ctx* ctx, const uint16_t* src_dev, float* dst_dev, int64_t n);

/* ---- block codecs ----------------------------------------------------------
 * src_dev holds raw GGUF blocks (fp16 d first, then qs). n % 32 == 0.       */
/* Q4_0.dequantToFloat (quant/Q4_0.java:32-45), interleaved nibble order. */
int at_q4_0_dequant(at_ctx* ctx, const void* src_dev, float* dst_dev, int64_t n);
/* Q8_0.dequantToFloat (quant/Q8_0.java:32-44). */
int at_q8_0_dequant(at_ctx* ctx, const void* src_dev, float* dst_dev, int64_t n);
/* Q6_K.dequantToFloat (quant/Q6_K.java:54-102): x = d * scale[i / 16] * (q - 32),
 * d fp16 with flush-to-zero, 256 elements per 210-byte block; n % 256 == 0. */
int at_q6_k_dequant(at_ctx* ctx, const void* src_dev, float* dst_dev, int64_t n);
/* Q4_0.dot (quant/Q4_0.java:51-90) with dequantToFloat semantics over all 32
 * elements of every block; result written to *out_dev. */
int at_q4_0_dot(at_ctx* ctx, const void* q4_dev, const float* x_dev, int64_t n, float* out_dev);
/* Q8_0.dot (quant/Q8_0.java:54-93), same convention. */
int at_q8_0_dot(at_ctx* ctx, const void* q8_dev, const float* x_dev, int64_t n, float* out_dev);

/* ---- quantized matrices ------------------------------------------------------
 * Uploads rows*cols elements of raw GGUF blocks (Q4_0, Q8_0, or F32/F16 which
 * are kept as f32) and re-lays them out losslessly for the given orientation:
 * scales and quant bytes in separate 16-byte-aligned planes; orientation T is
 * stored block-column-major. The raw bytes are never re-quantized.
 * Replaces the load-time dequant of Weights.wrapByName (inference/Weights.java:185-203)
 * and the transposes of LlamaModel (inference/LlamaModel.java:326-369).  */
int at_qmat_create(at_ctx* ctx, int ggml_type, int orient, int64_t rows, int64_t cols,
                   const void* blocks, int blocks_on_device, at_qmat** out);
/* at_qmat_create for blocks in another byte layout: layout
 * AT_LAYOUT_Q4_SPLIT_HALVES reads Q4_0 blocks in llama.cpp's nibble order
 * (stored, and exported, in the interleaved order); AT_GGML_Q6_K matrices
 * take orientation N. No counterpart in the reference (which reads the
 * interleaved order only and dequantizes Q6_K at load). */
int at_qmat_create_ex(at_ctx* ctx, int ggml_type, int orient, int layout, int64_t rows, int64_t cols,
                      const void* blocks, int blocks_on_device, at_qmat** out);
int at_qmat_destroy(at_qmat* m);
/* Writes the matrix back as raw GGUF blocks (row-major) to dst_dev. */
int at_qmat_export(at_ctx* ctx, const at_qmat* m, void* dst_dev);
/* Fused dequant GEMV on the stored orientation; x_dev [batch][in], y_dev
 * [batch][out], 1 <= batch <= 8. Replaces Kernels.sgemv over the dequantized
 * FP32 weights (core/Kernels.java:331-371) on the model path. */
int at_gemv(at_ctx* ctx, const at_qmat* m, const float* x_dev, float* y_dev, int batch);
/* Same orientation-T GEMV as at_gemv (same kernel, same results), for callers
 * that cannot allocate device memory: callers whose device memory belongs to
 * another allocator (a framework's caching allocator, or an arena sized up
 * front) and callers that cannot take cudaMalloc's device-wide
 * synchronisation in the middle of a decode loop. at_gemv grows its split-K
 * scratch with cudaMalloc the first time a larger shape needs it; this entry
 * point allocates nothing: the split partials and arrival counters (at
 * batch above 2, or of splits over more than 8 CTAs; the other splits
 * combine in thread-block cluster shared memory and need none) live in one
 * static device array of
 * 256 KiB (61440 partial floats + 4096 counters),
 * held by every GPU that loads the library until exit. Shapes whose split
 * needs more are rejected with AT_ERR_INVALID_ARG. The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress, with that device
 * current). Every call shares
 * the array and zeroes the counters first: calls that overlap on the GPU
 * (other streams or contexts of the same device) race. No counterpart in the
 * reference. m must be stored for AT_ORIENT_T. */
int at_gemv_t_static_scratch(at_ctx* ctx, const at_qmat* m, const float* x_dev, float* y_dev, int batch);

/* Prompt-chunk GEMM on the tensor cores: y[t][:] = W x[t][:] for t < tokens,
 * with the weights dequantized to bf16 and x rounded to bf16, FP32 sums
 * (the forwardPrompt path, inference/LlamaModel.java:166-175, whose
 * tolerance is 2e-2 of the logit range). x: [tokens][in], y: [tokens][out],
 * device FP32; in must be a multiple of 64; any orientation, Q4_0 or Q8_0. */
int at_gemm_tc(at_ctx* ctx, const at_qmat* m, const float* x_dev, float* y_dev, int tokens);

/* ---- Kernels (core/Kernels.java), FP32 device buffers ----------------------- */
/* Kernels.sgemv(MemorySegment a,x,y,int M,int K)  (core/Kernels.java:350-371) */
int at_sgemv(at_ctx* ctx, const float* a_dev, const float* x_dev, float* y_dev, int M, int K);
/* Kernels.sgemm(a,b,c,int M,int K,int N)          (core/Kernels.java:395-452) */
int at_sgemm(at_ctx* ctx, const float* a_dev, const float* b_dev, float* c_dev, int M, int K, int N);
/* Kernels.rmsNormInPlace(x, weight, eps) over `rows` rows of length d (core/Kernels.java:100-154) */
int at_rmsnorm(at_ctx* ctx, float* x_dev, const float* w_dev, float eps, int rows, int d);
/* Kernels.softmaxInPlace / softmaxInPlaceSegment, per row of length n (core/Kernels.java:161-232) */
int at_softmax(at_ctx* ctx, float* x_dev, int rows, int n);
/* Kernels.ropeInPlaceSegment(qk, cos, sin, headDim, n) (core/Kernels.java:274-321) */
int at_rope(at_ctx* ctx, float* qk_dev, const float* cos_dev, const float* sin_dev, int head_dim, int n);
/* Kernels.siluInPlaceSegment(seg, n) (core/Kernels.java:61-90) */
int at_silu(at_ctx* ctx, float* x_dev, int64_t n);

/* ---- model: LlamaConfig / Weights / LlamaModel / KVCache ------------------- */
typedef struct at_model_config {
    int64_t context_length;       /* inference/LlamaConfig.java:30 */
    int64_t embedding_length;
    int64_t block_count;
    int64_t head_count;
    int64_t head_count_kv;
    int64_t feed_forward_length;
    int64_t vocab_size;
    float   rope_freq_base;
    float   rms_norm_eps;
    int32_t max_batch;            /* independent sequences (KV slots), 1..8 */
    int32_t layout;               /* AT_LAYOUT_* bits of the tensors' bytes (0: the reference's) */
    int32_t kv_type;              /* KV cache storage: AT_GGML_F32 (0, the reference's KVCache) or
                                     AT_GGML_Q8_0 (blocks of 32 along head_dim, see below) */
    int32_t reserved;
} at_model_config;
/* A Q8_0 KV cache (the reference keeps K and V in FP32, KVCache.java:56-61;
 * its README lists quantized KV as missing) stores each appended K/V head
 * vector as blocks of 32 elements: d = max|x| / 127 rounded to fp16 once,
 * q = round-half-away(x * (1 / d)) in int8, read back as q * d (fp16 with
 * flush-to-zero). Logits then differ from the FP32-KV model by the KV
 * rounding (stated and tested tolerance: 2e-2 of the logit range); against
 * the oracle run with the same KV rounding they match within 1e-3. */

/* new LlamaModel(cfg, weights, tok) (inference/LlamaModel.java:79-129) without
 * weights yet; then at_model_set_tensor per GGUF tensor; then at_model_finalize. */
int at_model_create(at_ctx* ctx, const at_model_config* cfg, at_model** out);
/* Weights.wrapByName for one tensor (inference/Weights.java:117-203): name is
 * the GGUF tensor name ("blk.3.attn_q.weight", ...); data is that tensor's raw
 * bytes (host, or device when data_on_device != 0), uploaded once. Under
 * tensor parallelism the rank's shard is cut out on the device. */
int at_model_set_tensor(at_model* m, const char* name, int ggml_type, const void* data,
                        size_t bytes, int data_on_device);
/* Missing tensors become zeros (inference/Weights.java:131-135); builds the
 * RoPE table (inference/RopeCache.java:154-177), the KV cache and the step graph. */
int at_model_finalize(at_model* m);
/* GgufFile.open + LlamaConfig.fromGguf + Weights.load (format/GgufFile.java:97-143,
 * inference/LlamaConfig.java:30-53, inference/Weights.java:83-115): mmap, parse,
 * upload raw blocks once. */
int at_model_load_gguf(at_ctx* ctx, const char* path, int max_batch, at_model** out);
/* at_model_load_gguf for files in another byte layout (AT_LAYOUT_*; for
 * example AT_LAYOUT_LLAMA_CPP for llama.cpp exports). No counterpart in the
 * reference. */
int at_model_load_gguf_ex(at_ctx* ctx, const char* path, int max_batch, int layout, int kv_type, at_model** out);
int at_model_get_config(const at_model* m, at_model_config* out);
int at_model_destroy(at_model* m);
/* LlamaModel.forwardStep(tokenId, position) (inference/LlamaModel.java:141-158):
 * logits_host receives vocab floats (may be NULL to keep them on device). */
int at_model_forward_step(at_model* m, int token, int64_t position, float* logits_host);
/* LlamaModel.forwardPrompt (inference/LlamaModel.java:166-175). */
int at_model_forward_prompt(at_model* m, const int* tokens, int n);
/* Batched decode of `batch` independent sequences: sequence b uses KV slot b,
 * token tokens[b] at positions[b]. logits_host: [batch][vocab] or NULL. */
int at_model_forward_batch(at_model* m, const int* tokens, const int64_t* positions, int batch,
                           float* logits_host);
/* Device address of the last step's logits [max_batch][vocab] (full vocab on every rank). */
int at_model_logits_device(at_model* m, float** logits_dev);
/* Greedy token of each of the last step's `batch` rows (Sampler greedy path,
 * inference/Sampler.java:56-67: first index of the maximum). */
int at_model_argmax(at_model* m, int batch, int* tokens_host);
/* Which implementation serves batch-1 forwardStep and the greedy loop:
 * *persistent = 1 for the one-launch persistent step kernel (every layer,
 * the lm_head and the argmax in one kernel, one CTA per SM; chosen at load
 * when the environment sets AT_DECODE_STEP=1), 0 for the per-kernel step
 * graph (the default). Diagnostics; no counterpart in the reference. */
int at_model_step_kernel(const at_model* m, int* persistent);
/* One batch-1 step of the persistent step kernel with a %globaltimer stamp
 * at four points of every job on every CTA (start, activations staged,
 * units done, end): stamps_host receives [n_ctas][5 * layers + 1][4]
 * nanosecond values (jobs per layer: QKV, attention, wo, gate/up, down; then
 * the lm_head); *n_ctas is set. n is the
 * capacity of stamps_host in values. Diagnostics; no counterpart in the
 * reference. Fails (AT_ERR_STATE) when the model does not use that kernel. */
int at_model_step_stamps(at_model* m, int token, int64_t position, unsigned long long* stamps_host, int64_t n,
                         int* n_ctas);
/* Greedy decode loop resident on the device (the decode loop of the
 * reference's TokenThroughputBenchmark.decodeLoop, benchmarks/TokenThroughputBenchmark.java:147-158:
 * forwardStep then greedy Sampler.sample, repeated): n_steps steps of slot 0,
 * step i at position start_pos + i, whose token is first_token for i = 0 and
 * the previous step's argmax after that. No host round trip between steps.
 * tokens_out_host receives the n_steps generated tokens; when it is NULL the
 * steps are only enqueued on the context's stream (the call does not wait). */
int at_model_generate(at_model* m, int first_token, int64_t start_pos, int n_steps, int* tokens_out_host);

/* ---- sampling on the device and batched requests -------------------------
 * Sampler.Config (inference/Sampler.java:20-30) of one sequence. history is a
 * host array of previously emitted ids for the repetition penalty. */
typedef struct at_sampler_config {
    float temperature;
    int32_t top_k;
    float top_p;
    float repetition_penalty;
    int64_t seed;                 /* 0: an unseeded generator, as the reference */
    const int32_t* history;       /* host, may be NULL */
    int32_t history_len;
    int32_t reserved;
} at_sampler_config;
/* Sampler.sample (inference/Sampler.java:37-121) on the device for each of the
 * last step's `batch` logits rows, row b with cfgs[b]: the same repetition
 * penalty (applied to the device logits in place, as the reference mutates
 * its array), greedy path, stable top-k/top-p and CDF scan with r drawn from
 * a fresh java.util.Random(seed). top_k above 1024 (outside the greedy path)
 * is refused with AT_ERR_UNSUPPORTED; use at_sample on host logits then. */
int at_model_sample(at_model* m, int batch, const at_sampler_config* cfgs, int* tokens_host);
/* Batched sampled decoding on the device: `batch` sequences (KV slots
 * 0..batch-1), slot b starting from first_tokens[b] at start_pos[b]; each of
 * n_steps steps runs the step graph, samples every row with cfgs[b] and feeds
 * the tokens back without a host round trip (each step's tokens are appended
 * to the row's penalty history). tokens_out_host: [batch][n_steps]. The
 * reference samples one sequence per call (inference/Sampler.java:37,
 * server/InferenceServer.java:112-174). */
int at_model_generate_sampled(at_model* m, int batch, const int* first_tokens, const int64_t* start_pos, int n_steps,
                              const at_sampler_config* cfgs, int* tokens_out_host);
/* LlamaModel.forwardPrompt (inference/LlamaModel.java:166-175) into KV slot
 * `slot` (the reference has one sequence per model). One GPU. */
int at_model_forward_prompt_slot(at_model* m, int slot, const int* tokens, int n);

/* Continuous batching over the model's KV slots (one GPU). Requests wait
 * until a slot is free; at_sched_step admits waiting requests (their prompt
 * runs into the slot), runs one batched decode step for every active request
 * with device sampling, and retires requests that reached max_new tokens.
 * The reference's server runs one request at a time on a shared model
 * (server/InferenceServer.java:112-174). */
typedef struct at_sched at_sched;
int at_sched_create(at_model* m, at_sched** out);
int at_sched_destroy(at_sched* s);
/* prompt: n >= 1 ids (host; copied), n + max_new <= the model's context.
 * Generation stops after max_new tokens or at eos_token (not emitted; < 0:
 * none), as the server's loop (server/InferenceServer.java:124-134). The
 * penalty history is the prompt followed by the generated tokens; cfg's own
 * history fields are ignored. *request_id is set. */
int at_sched_submit(at_sched* s, const int* prompt, int n, int max_new, int eos_token, const at_sampler_config* cfg,
                    int* request_id);
/* One scheduling step; *n_active = requests still running or waiting. */
int at_sched_step(at_sched* s, int* n_active);
/* Tokens generated so far for a request (up to cap) and whether it is done. */
int at_sched_result(at_sched* s, int request_id, int* tokens_host, int cap, int* n_tokens, int* done);
/* Per-kernel-class device time of one forward step of slot 0, run as a graph
 * with a CUDA event pair around every launch (and no programmatic overlap):
 * class_ms[AT_PROF_CLASSES] milliseconds and class_launches[AT_PROF_CLASSES]
 * launch counts. New (the reference has only wall-clock prints). */
#define AT_PROF_EMBED    0
#define AT_PROF_QKV      1  /* QKV GEMV + RMSNorm + RoPE + KV append   */
#define AT_PROF_ATTN     2  /* split-KV attention + combine            */
#define AT_PROF_WO       3  /* attention output GEMV                   */
#define AT_PROF_FFN_UP   4  /* gate/up GEMV + RMSNorm + SiLU*up        */
#define AT_PROF_FFN_DOWN 5  /* down GEMV                               */
#define AT_PROF_LM_HEAD  6  /* output norm + lm_head GEMV              */
#define AT_PROF_ARGMAX   7
#define AT_PROF_COMM     8  /* NCCL all-reduce / all-gather            */
#define AT_PROF_CLASSES  9
int at_model_profile_step(at_model* m, int token, int64_t position, float* class_ms, int* class_launches);
/* The same for one batched step of slots 0..batch-1. */
int at_model_profile_batch(at_model* m, int batch, const int* tokens, const int64_t* positions, float* class_ms,
                           int* class_launches);
/* KVCache.size / offsetOf / keys() / values() (inference/KVCache.java:70-104):
 * copies head_dim floats of K and V for (slot, layer, kv_head, position). */
int at_model_kv_size(const at_model* m, int slot, int64_t* size);
int at_model_kv_read(at_model* m, int slot, int layer, int kv_head, int64_t position,
                     float* k_host, float* v_host);
/* Rewinds a sequence slot to empty (the reference builds a new KVCache). */
int at_model_kv_reset(at_model* m, int slot);
/* KVCache.append(layer, position, kSlice, vSlice) (inference/KVCache.java:79-95)
 * into KV slot `slot`: k_host / v_host hold head_count_kv (rank-local) x
 * head_dim floats. Layer out of range: AT_ERR_INVALID_ARG; position at or
 * past maxContext: AT_ERR_STATE. A Q8_0 cache quantizes on the way in. */
int at_model_kv_append(at_model* m, int slot, int64_t layer, int64_t position, const float* k_host,
                       const float* v_host);
/* KVCache.offsetOf(layer, kvHead, position, dim) (inference/KVCache.java:70-76):
 * the byte offset of that element in one slot's K (or V) array of the FP32
 * layout [layer][kvHead][maxContext][headDim], with the reference's checks
 * (layer, kvHead, position out of range or dim >= headDim: AT_ERR_INVALID_ARG).
 * For a Q8_0 cache offset / 4 indexes the quants and offset / 128 the scales. */
int at_model_kv_offset(const at_model* m, int64_t layer, int64_t kv_head, int64_t position, int64_t dim,
                       int64_t* byte_offset);

/* ---- sampler: Sampler.sample (inference/Sampler.java:37-121), host -------- */
int at_sample(float* logits, int vocab, const int* history, int n_history, float temperature,
              int top_k, float top_p, float repetition_penalty, int64_t seed, int* out_token);

/* ---- tensor parallelism over NCCL (new: the reference is single-process) --- */
/* 128-byte ncclUniqueId for rank 0 to broadcast to the other ranks. */
int at_tp_unique_id(uint8_t out_id[128]);
/* Context whose models shard weights Megatron-style over `world` ranks and
 * all-reduce after each attention block and each MLP block. */
int at_ctx_create_tp(int device, int rank, int world, const uint8_t id[128], at_ctx** out);

/* The shard of one GGUF weight tensor that rank `rank` of `world` keeps, as
 * at_model_set_tensor cuts it (host-only query, no device work). The tensor's
 * shape follows Weights.wrapByName (inference/Weights.java:84-112); the cut is
 * Megatron's: wq/wk/wv by heads into the rank's fused [q|k|v] matrix, wo by
 * its head rows (input), w1/w3 by output rows, w2 by input columns, lm_head
 * by vocabulary rows (the last rank's share may be short or empty); norms and
 * the token embedding stay whole. With cfg->layout & AT_LAYOUT_ATTN_OUT_IN
 * the attention tensors are [out][in] and the same heads are rows/columns
 * swapped. Tensors the decode path does not read give target AT_SHARD_NONE.
 * Fails like at_model_create when the heads or the FFN do not divide. */
#define AT_SHARD_NONE        -1
#define AT_SHARD_TOKEN_EMBD   0
#define AT_SHARD_OUTPUT       1
#define AT_SHARD_QKV          2
#define AT_SHARD_WO           3
#define AT_SHARD_W1           4
#define AT_SHARD_W3           5
#define AT_SHARD_W2           6
#define AT_SHARD_NORM         7
typedef struct at_shard_region {
    int32_t target;                 /* AT_SHARD_*: the rank's device matrix the bytes go to */
    int32_t orient;                 /* AT_ORIENT_N / AT_ORIENT_T of that matrix */
    int64_t rows, cols;             /* the whole tensor as its bytes are laid out: [rows][cols] */
    int64_t local_rows, local_cols; /* the rank's device matrix */
    int64_t src_row0, src_col0;     /* first row / column of the tensor this rank keeps */
    int64_t n_rows, n_cols;         /* extent of that part (0 rows: nothing) */
    int64_t dst_row0, dst_col0;     /* where the part starts in the device matrix */
} at_shard_region;
int at_tp_shard_region(const at_model_config* cfg, int world, int rank, const char* tensor_name,
                       at_shard_region* out);

#ifdef __cplusplus
}
#endif
#endif /* AURATENSOR_H */
