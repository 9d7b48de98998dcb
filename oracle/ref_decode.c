/*
 * ref_decode.c — C restatement of the reference decode path (ORACLE / CPU
 * baseline only; test infrastructure, never linked into the product library).
 *
 * Follows the reference algorithm step by step (paths relative to
 * src/main/java/io/auratensor/):
 *   - load time: every Q4_0 / Q8_0 / F16 tensor dequantized to FP32
 *     (inference/Weights.java:167-203, quant/Q4_0.java:32-45,
 *     quant/Q8_0.java:32-44, core/Fp16.java:19-37); attention weights
 *     transposed once (inference/LlamaModel.java:326-369);
 *   - per step: LlamaModel.forwardStep / layerStep / attention
 *     (inference/LlamaModel.java:141-308) with Kernels.sgemv, rmsNormInPlace,
 *     ropeInPlaceSegment, softmaxInPlaceSegment, siluInPlace
 *     (core/Kernels.java:61-371) and the RopeCache tables
 *     (inference/RopeCache.java:154-177).
 * The SIMD lane accumulation of Kernels.sgemv is restated with 16 partial
 * sums per row. The only deviation: the token embedding row is dequantized
 * at lookup instead of dequantizing the whole table at load (a row copy in
 * the reference; it does not change any value).
 * Threads: OpenMP over output rows of each matvec and over the query heads
 * of the attention (1 thread = the
 * reference's single-threaded loop).
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

typedef struct {
    int dim, ffn, n_heads, n_kv, vocab, ctx, n_layers;
    float rope_base, eps;
    int layout; /* bit 0: llama.cpp split-halves Q4_0 nibbles; bit 1: attention bytes [out][in] */
    int kv_q8;  /* 1: K/V rounded as the device's Q8_0 KV cache stores them (no reference counterpart) */
} rd_cfg;

typedef struct {
    float *qT, *kT, *vT, *oT, *gate, *up, *down, *attn_norm, *ffn_norm;
} rd_layer;

typedef struct {
    rd_cfg c;
    int hd, threads;
    rd_layer* L;
    const uint8_t* emb_raw; /* caller-owned raw token_embd blocks */
    int emb_type;
    float *out_norm, *out_w;
    float *kc, *vc, *rcos, *rsin;
    float *x, *q, *k, *v, *att, *proj, *g, *u, *ff, *logits, *scores;
    double t_embed, t_layers, t_head;
} rd_model;

static float fp16_ftz(uint16_t h) {
    uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, b;
    if (e == 0) b = s << 31;
    else if (e == 31) b = m ? 0x7FC00000u : ((s << 31) | 0x7F800000u);
    else b = (s << 31) | ((e + 112u) << 23) | (m << 13);
    float f;
    memcpy(&f, &b, 4);
    return f;
}

/* Q6_K.dequantToFloat (quant/Q6_K.java:54-102, the published llama.cpp
 * dequantize_row_q6_K) of one 210-byte block into 256 floats. */
/* float -> fp16 bits, round to nearest even (IEEE conversion). */
static uint16_t f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds past 65504 */
    if (ax < 0x38800000u) {                                   /* below 2^-14: subnormal (or zero) */
        float a;
        memcpy(&a, &ax, 4);
        const double q = nearbyint((double)a * 16777216.0);   /* units of 2^-24, ties to even */
        return (uint16_t)(sign | (uint32_t)q);
    }
    uint32_t h = (((ax >> 23) - 112u) << 10) | ((ax & 0x7FFFFFu) >> 13);
    const uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
}

static float fp16_ftz(uint16_t h);

/* The device's Q8_0 KV rounding of n values (blocks of 32): d = max|x| / 127
 * stored as fp16, q = roundf(x * (1 / d)) clamped to +-127, x <- q * d. */
static void kv_q8_round(float* x, int n) {
    for (int b = 0; b < n; b += 32) {
        float amax = 0.f;
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[b + i]));
        const float d = amax / 127.f;
        const float id = d != 0.f ? 1.f / d : 0.f;
        const float dd = fp16_ftz(f32_to_f16(d));
        for (int i = 0; i < 32; ++i) {
            float q = roundf(x[b + i] * id);
            q = q > 127.f ? 127.f : (q < -127.f ? -127.f : q);
            x[b + i] = q * dd;
        }
    }
}

static void dequant_q6_k_block(const uint8_t* p, float* y) {
    const float d = fp16_ftz((uint16_t)(p[208] | (p[209] << 8)));
    for (int n = 0; n < 256; n += 128) {
        const uint8_t* ql = p + n / 2;
        const uint8_t* qh = p + 128 + n / 4;
        const int8_t* sc = (const int8_t*)(p + 192 + n / 16);
        for (int l = 0; l < 32; ++l) {
            const int is = l / 16;
            const int q1 = ((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
            const int q2 = ((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
            const int q3 = (((ql[l] >> 4) & 0x0F) | (((qh[l] >> 4) & 3) << 4)) - 32;
            const int q4 = (((ql[l + 32] >> 4) & 0x0F) | (((qh[l] >> 6) & 3) << 4)) - 32;
            y[n + l] = d * (float)sc[is] * (float)q1;
            y[n + l + 32] = d * (float)sc[is + 2] * (float)q2;
            y[n + l + 64] = d * (float)sc[is + 4] * (float)q3;
            y[n + l + 96] = d * (float)sc[is + 6] * (float)q4;
        }
    }
}

/* split != 0: Q4_0 blocks in llama.cpp's nibble order (element k = low
 * nibble of byte k, element k + 16 = its high nibble). */
static void dequant_ex(int type, const uint8_t* src, float* dst, int64_t n, int split) {
    if (type == 0) { memcpy(dst, src, (size_t)n * 4); return; }
    if (type == 1) { for (int64_t i = 0; i < n; ++i) dst[i] = fp16_ftz((uint16_t)(src[2*i] | (src[2*i+1] << 8))); return; }
    if (type == 14) {
#pragma omp parallel for schedule(static)
        for (int64_t b = 0; b < n / 256; ++b) dequant_q6_k_block(src + b * 210, dst + b * 256);
        return;
    }
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < n / 32; ++b) {
        if (type == 2) {
            const uint8_t* p = src + b * 18;
            const float d = fp16_ftz((uint16_t)(p[0] | (p[1] << 8)));
            for (int i = 0; i < 32; ++i) {
                int q;
                if (split) {
                    q = (i < 16) ? (p[2 + i] & 0x0F) : ((p[2 + i - 16] >> 4) & 0x0F);
                } else {
                    const int pk = p[2 + i / 2];
                    q = (i % 2 == 0) ? (pk & 0x0F) : ((pk >> 4) & 0x0F);
                }
                dst[b * 32 + i] = (float)(q - 8) * d;
            }
        } else {
            const uint8_t* p = src + b * 34;
            const float d = fp16_ftz((uint16_t)(p[0] | (p[1] << 8)));
            for (int i = 0; i < 32; ++i) dst[b * 32 + i] = (float)(int8_t)p[2 + i] * d;
        }
    }
}

static int g_split; /* split-halves order of the model being loaded (single-threaded set_tensor) */
static void dequant(int type, const uint8_t* src, float* dst, int64_t n) { dequant_ex(type, src, dst, n, g_split); }

/* One row of Kernels.sgemv: 16 lane-wise partial sums then a reduce. */
static float sgemv_row(const float* a, const float* x, int K) {
    float acc[16] = {0};
    int k = 0;
    for (; k + 16 <= K; k += 16)
        for (int l = 0; l < 16; ++l) acc[l] = fmaf(a[k + l], x[k + l], acc[l]);
    float s = 0.f;
    for (int l = 0; l < 16; ++l) s += acc[l];
    for (; k < K; ++k) s += a[k] * x[k];
    return s;
}

/* Kernels.sgemv: y[M] = A[M,K] x[K], rows over the threads. */
static void sgemv(const float* A, const float* x, float* y, int M, int K) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < M; ++i) y[i] = sgemv_row(A + (size_t)i * K, x, K);
}

/* The same on the calling thread only (inside a parallel region). */
static void sgemv_rows(const float* A, const float* x, float* y, int M, int K) {
    for (int i = 0; i < M; ++i) y[i] = sgemv_row(A + (size_t)i * K, x, K);
}

static void rmsnorm(float* x, const float* w, int d, float eps) {
    float acc[16] = {0};
    int i = 0;
    for (; i + 16 <= d; i += 16)
        for (int l = 0; l < 16; ++l) acc[l] = fmaf(x[i + l], x[i + l], acc[l]);
    float ss = 0.f;
    for (int l = 0; l < 16; ++l) ss += acc[l];
    for (; i < d; ++i) ss += x[i] * x[i];
    const float inv = (float)(1.0 / sqrt((double)(ss / (float)d + eps)));
    for (i = 0; i < d; ++i) x[i] = (x[i] * inv) * w[i];
}

static void rope(float* qk, const float* c, const float* s, int hd, int n) {
    for (int h = 0; h < n / hd; ++h) {
        float* v = qk + (size_t)h * hd;
        for (int i = 0; i < hd; i += 2) {
            const float a = v[i], b = v[i + 1];
            v[i] = fmaf(a, c[i], b * -s[i]);
            v[i + 1] = fmaf(b, c[i + 1], a * s[i + 1]);
        }
    }
}

static void softmax(float* x, int n) {
    float m = -INFINITY;
    for (int i = 0; i < n; ++i) if (x[i] > m) m = x[i];
    float sum = 0.f;
    for (int i = 0; i < n; ++i) { x[i] = (float)exp((double)(x[i] - m)); sum += x[i]; }
    const float inv = 1.0f / sum;
    for (int i = 0; i < n; ++i) x[i] *= inv;
}

static double now(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec + 1e-9 * t.tv_nsec;
}

static float* falloc(size_t n) { return (float*)calloc(n ? n : 1, 4); }

rd_model* rd_create(const rd_cfg* c, int threads) {
    rd_model* m = (rd_model*)calloc(1, sizeof(rd_model));
    m->c = *c;
    m->hd = c->dim / c->n_heads;
    m->threads = threads > 0 ? threads : 1;
    omp_set_num_threads(m->threads);
    const int hd = m->hd, d = c->dim;
    m->L = (rd_layer*)calloc(c->n_layers, sizeof(rd_layer));
    for (int l = 0; l < c->n_layers; ++l) {
        rd_layer* L = &m->L[l];
        L->qT = falloc((size_t)c->n_heads * hd * d); L->kT = falloc((size_t)c->n_kv * hd * d);
        L->vT = falloc((size_t)c->n_kv * hd * d); L->oT = falloc((size_t)d * c->n_heads * hd);
        L->gate = falloc((size_t)c->ffn * d); L->up = falloc((size_t)c->ffn * d); L->down = falloc((size_t)d * c->ffn);
        L->attn_norm = falloc(d); L->ffn_norm = falloc(d);
    }
    m->out_norm = falloc(d);
    m->out_w = falloc((size_t)c->vocab * d);
    const size_t kv = (size_t)c->n_layers * c->n_kv * c->ctx * hd;
    m->kc = falloc(kv); m->vc = falloc(kv);
    m->rcos = falloc((size_t)c->ctx * hd); m->rsin = falloc((size_t)c->ctx * hd);
    for (int p = 0; p < c->ctx; ++p)
        for (int i = 0; i < hd / 2; ++i) {
            const float freq = (float)pow((double)c->rope_base, -2.0 * i / (double)hd);
            const float ang = (float)p * freq;
            const float cv = (float)cos((double)ang), sv = (float)sin((double)ang);
            m->rcos[(size_t)p * hd + 2 * i] = m->rcos[(size_t)p * hd + 2 * i + 1] = cv;
            m->rsin[(size_t)p * hd + 2 * i] = m->rsin[(size_t)p * hd + 2 * i + 1] = sv;
        }
    m->x = falloc(d); m->q = falloc((size_t)c->n_heads * hd); m->k = falloc((size_t)c->n_kv * hd);
    m->v = falloc((size_t)c->n_kv * hd); m->att = falloc((size_t)c->n_heads * hd); m->proj = falloc(d);
    m->g = falloc(c->ffn); m->u = falloc(c->ffn); m->ff = falloc(d); m->logits = falloc(c->vocab);
    m->scores = falloc((size_t)c->n_heads * c->ctx);  /* one row per head */
    return m;
}

/* Weights.wrapByName + LlamaModel transposes for one tensor. Returns 0 on success. */
int rd_set_tensor(rd_model* m, const char* name, int type, const void* data, int64_t numel) {
    const rd_cfg* c = &m->c;
    const int hd = m->hd, d = c->dim;
    omp_set_num_threads(m->threads);
    g_split = c->layout & 1;
    if (!strcmp(name, "token_embd.weight")) { m->emb_raw = (const uint8_t*)data; m->emb_type = type; return 0; }
    if (!strcmp(name, "output_norm.weight")) { dequant(type, data, m->out_norm, d); return 0; }
    if (!strcmp(name, "output.weight")) { dequant(type, data, m->out_w, numel); return 0; }
    int l = -1;
    char leaf[64];
    if (sscanf(name, "blk.%d.%63s", &l, leaf) != 2 || l < 0 || l >= c->n_layers) return -1;
    rd_layer* L = &m->L[l];
    float* tmp = falloc(numel);
    dequant(type, data, tmp, numel);
    int rc = 0;
    const int out_in = (c->layout & 2) != 0; /* llama.cpp: attention bytes already [out][in] */
    if (!strcmp(leaf, "attn_q.weight") || !strcmp(leaf, "attn_k.weight") || !strcmp(leaf, "attn_v.weight")) {
        /* transposeAttnProj: bytes [emb][out] -> [out][emb] */
        const int out = (int)(numel / d);
        float* dst = leaf[5] == 'q' ? L->qT : (leaf[5] == 'k' ? L->kT : L->vT);
        if (out_in) memcpy(dst, tmp, (size_t)numel * 4);
        else
            for (int e = 0; e < d; ++e)
                for (int k = 0; k < out; ++k) dst[(size_t)k * d + e] = tmp[(size_t)e * out + k];
    } else if (!strcmp(leaf, "attn_output.weight")) {
        /* transposeAttnOut: bytes [H*hd][emb] -> [emb][H*hd] */
        const int tk = c->n_heads * hd;
        if (out_in) memcpy(L->oT, tmp, (size_t)numel * 4);
        else
            for (int k = 0; k < tk; ++k)
                for (int e = 0; e < d; ++e) L->oT[(size_t)e * tk + k] = tmp[(size_t)k * d + e];
    } else if (!strcmp(leaf, "ffn_gate.weight")) memcpy(L->gate, tmp, (size_t)numel * 4);
    else if (!strcmp(leaf, "ffn_up.weight")) memcpy(L->up, tmp, (size_t)numel * 4);
    else if (!strcmp(leaf, "ffn_down.weight")) memcpy(L->down, tmp, (size_t)numel * 4);
    else if (!strcmp(leaf, "attn_norm.weight")) memcpy(L->attn_norm, tmp, (size_t)d * 4);
    else if (!strcmp(leaf, "ffn_norm.weight")) memcpy(L->ffn_norm, tmp, (size_t)d * 4);
    else rc = -1;
    free(tmp);
    return rc;
}

static void layer_step(rd_model* m, int l, int pos) {
    const rd_cfg* c = &m->c;
    const int hd = m->hd, d = c->dim, H = c->n_heads, Hkv = c->n_kv, ctx = c->ctx;
    rd_layer* L = &m->L[l];
    rmsnorm(m->x, L->attn_norm, d, c->eps);
    sgemv(L->qT, m->x, m->q, H * hd, d);
    sgemv(L->kT, m->x, m->k, Hkv * hd, d);
    sgemv(L->vT, m->x, m->v, Hkv * hd, d);
    const float* cr = m->rcos + (size_t)pos * hd;
    const float* sr = m->rsin + (size_t)pos * hd;
    rope(m->q, cr, sr, hd, H * hd);
    rope(m->k, cr, sr, hd, Hkv * hd);
    if (c->kv_q8) {
        kv_q8_round(m->k, Hkv * hd);
        kv_q8_round(m->v, Hkv * hd);
    }
    for (int h = 0; h < Hkv; ++h) {
        const size_t off = (((size_t)l * Hkv + h) * ctx + pos) * hd;
        memcpy(m->kc + off, m->k + (size_t)h * hd, hd * 4);
        memcpy(m->vc + off, m->v + (size_t)h * hd, hd * 4);
    }
    const float scale = (float)(1.0 / sqrt((double)hd));
    const int M = pos + 1;
    /* Heads are independent (each one's arithmetic is sequential), so they
     * run on separate threads with a scores row each. */
#pragma omp parallel for schedule(static)
    for (int h = 0; h < H; ++h) {
        const int kvh = (Hkv == H) ? h : (int)((int64_t)h * Hkv / H);
        const size_t base = ((size_t)l * Hkv + kvh) * ctx * hd;
        float* sc = m->scores + (size_t)h * ctx;
        sgemv_rows(m->kc + base, m->q + (size_t)h * hd, sc, M, hd);
        for (int p = 0; p < M; ++p) sc[p] *= scale;
        softmax(sc, M);
        float* o = m->att + (size_t)h * hd;
        for (int j = 0; j < hd; ++j) {
            float acc = 0.f;
            for (int p = 0; p < M; ++p) acc = fmaf(m->vc[base + (size_t)p * hd + j], sc[p], acc);
            o[j] = acc;
        }
    }
    sgemv(L->oT, m->att, m->proj, d, H * hd);
    for (int i = 0; i < d; ++i) m->x[i] += m->proj[i];
    rmsnorm(m->x, L->ffn_norm, d, c->eps);
    sgemv(L->gate, m->x, m->g, c->ffn, d);
    sgemv(L->up, m->x, m->u, c->ffn, d);
    for (int i = 0; i < c->ffn; ++i) m->g[i] = m->g[i] / (1.0f + (float)exp(-(double)m->g[i]));
    for (int i = 0; i < c->ffn; ++i) m->g[i] *= m->u[i];
    sgemv(L->down, m->g, m->ff, d, c->ffn);
    for (int i = 0; i < d; ++i) m->x[i] += m->ff[i];
}

static const float* forward(rd_model* m, int token, int pos, int with_logits);

/* LlamaModel.forwardStep: returns the logits buffer (vocab floats). */
const float* rd_forward_step(rd_model* m, int token, int pos) { return forward(m, token, pos, 1); }

/* The same step without the output norm and lm_head (fills the KV cache only;
 * the logits of such a step are never looked at). */
void rd_forward_layers(rd_model* m, int token, int pos) { forward(m, token, pos, 0); }

/* K and V of (layer, kv head, position): hd floats each. */
void rd_kv(const rd_model* m, int layer, int kv_head, int pos, float* k, float* v) {
    const size_t off = (((size_t)layer * m->c.n_kv + kv_head) * m->c.ctx + pos) * m->hd;
    memcpy(k, m->kc + off, (size_t)m->hd * 4);
    memcpy(v, m->vc + off, (size_t)m->hd * 4);
}

static const float* forward(rd_model* m, int token, int pos, int with_logits) {
    const rd_cfg* c = &m->c;
    const int d = c->dim;
    omp_set_num_threads(m->threads);
    double t0 = now();
    if (m->emb_raw) {
        g_split = c->layout & 1;
        const int bpb = m->emb_type == 2 ? 18 : (m->emb_type == 8 ? 34 : 0);
        if (m->emb_type == 14) dequant(14, m->emb_raw + (size_t)token * (d / 256) * 210, m->x, d);
        else if (bpb) dequant(m->emb_type, m->emb_raw + (size_t)token * (d / 32) * bpb, m->x, d);
        else dequant(m->emb_type, m->emb_raw + (size_t)token * d * (m->emb_type == 0 ? 4 : 2), m->x, d);
    } else {
        memset(m->x, 0, (size_t)d * 4);
    }
    double t1 = now();
    for (int l = 0; l < c->n_layers; ++l) layer_step(m, l, pos);
    double t2 = now();
    if (with_logits) {
        rmsnorm(m->x, m->out_norm, d, c->eps);
        sgemv(m->out_w, m->x, m->logits, c->vocab, d);
    }
    double t3 = now();
    m->t_embed += t1 - t0;
    m->t_layers += t2 - t1;
    m->t_head += t3 - t2;
    return m->logits;
}

void rd_times(rd_model* m, double* t_embed, double* t_layers, double* t_head) {
    *t_embed = m->t_embed; *t_layers = m->t_layers; *t_head = m->t_head;
    m->t_embed = m->t_layers = m->t_head = 0;
}

void rd_destroy(rd_model* m) {
    if (!m) return;
    for (int l = 0; l < m->c.n_layers; ++l) {
        rd_layer* L = &m->L[l];
        free(L->qT); free(L->kT); free(L->vT); free(L->oT); free(L->gate); free(L->up); free(L->down);
        free(L->attn_norm); free(L->ffn_norm);
    }
    free(m->L);
    free(m->out_norm); free(m->out_w); free(m->kc); free(m->vc); free(m->rcos); free(m->rsin);
    free(m->x); free(m->q); free(m->k); free(m->v); free(m->att); free(m->proj); free(m->g); free(m->u);
    free(m->ff); free(m->logits); free(m->scores);
    free(m);
}
