/*
 * qdec_oracle.c - CPU restatement of the reference Qwen3 decoder step and
 * prefill (qwen_asr_decoder.c + the decoder subset of qwen_asr_kernels*.c).
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA library, never part of
 * the product path. Activations, accumulators and the KV cache are f32 and
 * weights are bf16 widened by a 16-bit shift, exactly as in the reference.
 * Loops are plain C; a fork/join helper splits rows/heads across threads the
 * way the reference's pthread pool does (qwen_asr_kernels.c:38-153), which
 * does not change any per-row arithmetic.
 */
#include "qdec_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define ORC_TOKEN_ENDOFTEXT 151643
#define ORC_TOKEN_IM_END 151645

typedef struct {
    const uint16_t *wq, *wk, *wv, *wo, *gate, *up, *down;
    const float *q_norm, *k_norm, *input_norm, *post_attn_norm;
} orc_layer;

struct orc_model {
    orc_config cfg;
    const uint16_t *embed;
    const float *final_norm;
    orc_layer *layers;
};

struct orc_state {
    orc_model *m;
    float *k_cache, *v_cache; /* [layers][max_pos][kv_heads*head_dim] */
    int len, max_pos;
    int kv_round; /* 0: f32 as the reference; 1: round stored K/V to bf16; 2: to fp16 */
};

void orc_state_set_kv_round(orc_state *s, int mode) { s->kv_round = mode; }

static float round_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    memcpy(&f, &u, 4);
    return f;
}

static void round_kv(float *v, int n, int mode) {
    if (mode == 1)
        for (int i = 0; i < n; i++) v[i] = round_bf16(v[i]);
    else if (mode == 2)
        for (int i = 0; i < n; i++) v[i] = (float)(_Float16)v[i];
}

static int g_threads = 1;

void orc_set_threads(int n) { g_threads = n > 0 ? (n > 64 ? 64 : n) : 1; }

typedef void (*range_fn)(int begin, int end, void *arg);
typedef struct { range_fn fn; void *arg; int begin, end; } range_job;

static void *range_trampoline(void *p) {
    range_job *j = (range_job *)p;
    if (j->begin < j->end) j->fn(j->begin, j->end, j->arg);
    return NULL;
}

/* Split [0, n) into contiguous chunks, one per thread, and join. */
static void par_range(int n, range_fn fn, void *arg) {
    int t = g_threads;
    if (t <= 1 || n < 2) { fn(0, n, arg); return; }
    if (t > n) t = n;
    pthread_t th[64];
    range_job jobs[64];
    int chunk = (n + t - 1) / t;
    for (int i = 0; i < t; i++) {
        jobs[i].fn = fn; jobs[i].arg = arg;
        jobs[i].begin = i * chunk;
        jobs[i].end = (i + 1) * chunk < n ? (i + 1) * chunk : n;
    }
    for (int i = 1; i < t; i++) pthread_create(&th[i], NULL, range_trampoline, &jobs[i]);
    range_trampoline(&jobs[0]);
    for (int i = 1; i < t; i++) pthread_join(th[i], NULL);
}

static inline float bf16_to_f32(uint16_t v) {
    uint32_t bits = ((uint32_t)v) << 16;
    float f;
    memcpy(&f, &bits, sizeof(f));
    return f;
}

/* Y[s,o] = sum_k bf16(W[o,k]) * X[s,k] for s < seq, f32 accumulation per
 * (s, o) in ascending k. Each weight row is widened once and reused for all
 * seq rows. Follows qwen_bf16_matvec_fused_generic
 * (qwen_asr_kernels_generic.c:9-22) for seq == 1 and the f32 GEMM after
 * bf16_get_f32_view (qwen_asr_kernels.c:211-222, :322-330) for seq > 1. */
typedef struct { float *Y; const float *X; const uint16_t *W; int in, out, seq; } mm_args;

static void mm_range(int o0, int o1, void *p) {
    mm_args *a = (mm_args *)p;
    float *wrow = (float *)malloc(sizeof(float) * (size_t)a->in);
    for (int o = o0; o < o1; o++) {
        const uint16_t *row = a->W + (size_t)o * a->in;
        for (int k = 0; k < a->in; k++) wrow[k] = bf16_to_f32(row[k]);
        for (int s = 0; s < a->seq; s++) {
            const float *x = a->X + (size_t)s * a->in;
            float sum = 0.0f;
            for (int k = 0; k < a->in; k++) sum += wrow[k] * x[k];
            a->Y[(size_t)s * a->out + o] = sum;
        }
    }
    free(wrow);
}

static void matmul_bf16(float *Y, const float *X, const uint16_t *W, int seq, int in_dim, int out_dim) {
    mm_args a = { Y, X, W, in_dim, out_dim, seq };
    par_range(out_dim, mm_range, &a);
}

void orc_matvec_bf16(float *y, const float *x, const uint16_t *W, int in_dim, int out_dim) {
    matmul_bf16(y, x, W, 1, in_dim, out_dim);
}

/* Greedy argmax over W @ x without keeping logits; strict '>' from the lowest
 * row within a range, ranges merged in ascending order with strict '>', so an
 * exact tie resolves to the lowest index. Follows
 * qwen_argmax_bf16_range_generic (qwen_asr_kernels_generic.c:24-47) and the
 * in-thread-order merge of qwen_argmax_matvec_bf16 (qwen_asr_kernels.c:518-543).
 * mask_eos skips the two end-of-sequence ids (benchmark switch; the reference
 * has no such switch and never masks). */
typedef struct { const float *x; const uint16_t *W; int in, out, mask; int bi[64]; float bv[64]; int chunk; } am_args;

static void am_range(int t0, int t1, void *p) {
    am_args *a = (am_args *)p;
    for (int t = t0; t < t1; t++) {
        int s = t * a->chunk, e = s + a->chunk;
        if (e > a->out) e = a->out;
        int best = s < a->out ? s : 0;
        float best_val = -1e30f;
        for (int o = s; o < e; o++) {
            if (a->mask && (o == ORC_TOKEN_ENDOFTEXT || o == ORC_TOKEN_IM_END)) continue;
            const uint16_t *row = a->W + (size_t)o * a->in;
            float sum = 0.0f;
            for (int k = 0; k < a->in; k++) sum += bf16_to_f32(row[k]) * a->x[k];
            if (sum > best_val) { best_val = sum; best = o; }
        }
        a->bi[t] = best;
        a->bv[t] = best_val;
    }
}

int orc_argmax_matvec_bf16(const float *x, const uint16_t *W, int in_dim, int out_dim,
                           int mask_eos) {
    am_args a;
    a.x = x; a.W = W; a.in = in_dim; a.out = out_dim; a.mask = mask_eos;
    int nt = g_threads;
    a.chunk = (out_dim + nt - 1) / nt;
    par_range(nt, am_range, &a);
    int best = a.bi[0];
    float best_val = a.bv[0];
    for (int t = 1; t < nt; t++)
        if (a.bv[t] > best_val) { best_val = a.bv[t]; best = a.bi[t]; }
    return best;
}

/* out = x * (1/sqrtf(mean(x^2) + eps)) * w per row.
 * Follows qwen_rms_norm (qwen_asr_kernels.c:750-809). */
void orc_rms_norm(float *out, const float *x, const float *w, int seq, int hidden, float eps) {
    for (int s = 0; s < seq; s++) {
        const float *xr = x + (size_t)s * hidden;
        float *orow = out + (size_t)s * hidden;
        float ss = 0.0f;
        for (int i = 0; i < hidden; i++) ss += xr[i] * xr[i];
        float inv = 1.0f / sqrtf(ss / hidden + eps);
        for (int i = 0; i < hidden; i++) orow[i] = xr[i] * inv * w[i];
    }
}

/* In-place per-head RMSNorm with a shared [head_dim] weight.
 * Follows qwen_rms_norm_per_head (qwen_asr_kernels.c:811-873). */
static void rms_norm_per_head(float *x, const float *w, int seq, int n_heads, int hd, float eps) {
    for (int s = 0; s < seq; s++)
        for (int h = 0; h < n_heads; h++) {
            float *v = x + ((size_t)s * n_heads + h) * hd;
            float ss = 0.0f;
            for (int d = 0; d < hd; d++) ss += v[d] * v[d];
            float inv = 1.0f / sqrtf(ss / hd + eps);
            for (int d = 0; d < hd; d++) v[d] = v[d] * inv * w[d];
        }
}

/* cos/sin for one absolute position. inv_freq[d] = 1/powf(theta, 2d/hd) and
 * angle = (float)pos * inv_freq[d] in f32, as ensure_rope_inv_freq /
 * ensure_rope_cache (qwen_asr_decoder.c:207-256). */
static void rope_row(float *c, float *s, int pos, int hd, float theta) {
    int half = hd / 2;
    for (int d = 0; d < half; d++) {
        float inv = 1.0f / powf(theta, (float)(2 * d) / (float)hd);
        float angle = (float)pos * inv;
        c[d] = cosf(angle);
        s[d] = sinf(angle);
    }
}

/* NeoX split-half rotation: x1' = x1 c - x2 s, x2' = x2 c + x1 s.
 * Follows qwen_apply_rope_neox (qwen_asr_kernels.c:1182-1247). */
static void apply_rope(float *x, const float *c, const float *s, int n_heads, int hd) {
    int half = hd / 2;
    for (int h = 0; h < n_heads; h++) {
        float *v = x + (size_t)h * hd;
        for (int d = 0; d < half; d++) {
            float x1 = v[d], x2 = v[half + d];
            v[d] = x1 * c[d] - x2 * s[d];
            v[half + d] = x2 * c[d] + x1 * s[d];
        }
    }
}

typedef struct {
    float *out; const float *Q, *K, *V;
    int seq_q, seq_k, n_heads, n_kv, hd, q_offset; float scale;
} att_args;

static void att_range(int h0, int h1, void *p) {
    att_args *a = (att_args *)p;
    int per_kv = a->n_heads / a->n_kv, hd = a->hd;
    int qh = a->n_heads * hd, kvh = a->n_kv * hd;
    for (int h = h0; h < h1; h++) {
        int g = h / per_kv;
        for (int i = 0; i < a->seq_q; i++) {
            const float *q = a->Q + (size_t)i * qh + (size_t)h * hd;
            float *o = a->out + (size_t)i * qh + (size_t)h * hd;
            int k_end = a->q_offset + i + 1;
            if (k_end > a->seq_k) k_end = a->seq_k;
            float m = -1e30f, l = 0.0f;
            for (int d = 0; d < hd; d++) o[d] = 0.0f;
            for (int j = 0; j < k_end; j++) {
                const float *k = a->K + (size_t)j * kvh + (size_t)g * hd;
                const float *v = a->V + (size_t)j * kvh + (size_t)g * hd;
                float sc = 0.0f;
                for (int d = 0; d < hd; d++) sc += q[d] * k[d];
                sc *= a->scale;
                if (sc > m) {
                    float corr = expf(m - sc);
                    l = l * corr + 1.0f;
                    for (int d = 0; d < hd; d++) o[d] = o[d] * corr + v[d];
                    m = sc;
                } else {
                    float w = expf(sc - m);
                    l += w;
                    for (int d = 0; d < hd; d++) o[d] += w * v[d];
                }
            }
            if (l > 0.0f) {
                float inv = 1.0f / l;
                for (int d = 0; d < hd; d++) o[d] *= inv;
            }
        }
    }
}

/* Causal GQA attention with per-key online softmax (rescale the running sum
 * and output whenever a new maximum appears), f32 throughout, heads split
 * across threads. Follows qwen_causal_attention_heads and
 * qwen_causal_attention (qwen_asr_kernels.c:1050-1141). */
static void causal_attention(float *out, const float *Q, const float *K, const float *V,
                             int seq_q, int seq_k, int n_heads, int n_kv, int hd,
                             float scale, int q_offset) {
    att_args a = { out, Q, K, V, seq_q, seq_k, n_heads, n_kv, hd, q_offset, scale };
    par_range(n_heads, att_range, &a);
}

orc_model *orc_model_create(const orc_config *cfg, const uint16_t *embed, const float *final_norm) {
    if (!cfg || cfg->layers <= 0 || cfg->heads % cfg->kv_heads) return NULL;
    orc_model *m = (orc_model *)calloc(1, sizeof(*m));
    m->cfg = *cfg;
    m->embed = embed;
    m->final_norm = final_norm;
    m->layers = (orc_layer *)calloc((size_t)cfg->layers, sizeof(orc_layer));
    return m;
}

int orc_model_set_layer(orc_model *m, int i, const uint16_t *wq, const uint16_t *wk,
                        const uint16_t *wv, const uint16_t *wo, const uint16_t *gate,
                        const uint16_t *up, const uint16_t *down, const float *q_norm,
                        const float *k_norm, const float *input_norm,
                        const float *post_attn_norm) {
    if (!m || i < 0 || i >= m->cfg.layers) return -1;
    orc_layer *l = &m->layers[i];
    l->wq = wq; l->wk = wk; l->wv = wv; l->wo = wo;
    l->gate = gate; l->up = up; l->down = down;
    l->q_norm = q_norm; l->k_norm = k_norm;
    l->input_norm = input_norm; l->post_attn_norm = post_attn_norm;
    return 0;
}

void orc_model_free(orc_model *m) {
    if (!m) return;
    free(m->layers);
    free(m);
}

orc_state *orc_state_create(orc_model *m, int max_pos) {
    orc_state *s = (orc_state *)calloc(1, sizeof(*s));
    size_t kvd = (size_t)m->cfg.kv_heads * m->cfg.head_dim;
    size_t n = (size_t)m->cfg.layers * max_pos * kvd;
    s->m = m;
    s->max_pos = max_pos;
    s->k_cache = (float *)calloc(n, sizeof(float));
    s->v_cache = (float *)calloc(n, sizeof(float));
    if (!s->k_cache || !s->v_cache) { orc_state_free(s); return NULL; }
    return s;
}

void orc_state_free(orc_state *s) {
    if (!s) return;
    free(s->k_cache);
    free(s->v_cache);
    free(s);
}

int orc_state_len(const orc_state *s) { return s->len; }
void orc_state_set_len(orc_state *s, int len) { s->len = len; }

static float *kv_at(orc_state *s, float *base, int layer, int pos) {
    size_t kvd = (size_t)s->m->cfg.kv_heads * s->m->cfg.head_dim;
    return base + ((size_t)layer * s->max_pos + pos) * kvd;
}

/* One transformer block over `seq` rows starting at absolute position
 * `start` (qwen_asr_decoder.c:304-356 for prefill, :428-469 for one token;
 * both run the same op sequence). x is updated in place. */
static void run_layers(orc_state *s, float *x, int seq, int start) {
    const orc_config *c = &s->m->cfg;
    int h = c->hidden, hd = c->head_dim;
    int qd = c->heads * hd, kvd = c->kv_heads * hd, I = c->intermediate;
    float *xn = (float *)malloc(sizeof(float) * (size_t)seq * h);
    float *q = (float *)malloc(sizeof(float) * (size_t)seq * qd);
    float *k = (float *)malloc(sizeof(float) * (size_t)seq * kvd);
    float *v = (float *)malloc(sizeof(float) * (size_t)seq * kvd);
    float *att = (float *)malloc(sizeof(float) * (size_t)seq * qd);
    float *proj = (float *)malloc(sizeof(float) * (size_t)seq * h);
    float *g = (float *)malloc(sizeof(float) * (size_t)seq * I);
    float *u = (float *)malloc(sizeof(float) * (size_t)seq * I);
    float *rc = (float *)malloc(sizeof(float) * (size_t)seq * hd);
    float *rs = (float *)malloc(sizeof(float) * (size_t)seq * hd);
    for (int r = 0; r < seq; r++) rope_row(rc + (size_t)r * hd, rs + (size_t)r * hd, start + r, hd, c->theta);
    float scale = 1.0f / sqrtf((float)hd);

    for (int li = 0; li < c->layers; li++) {
        const orc_layer *L = &s->m->layers[li];
        orc_rms_norm(xn, x, L->input_norm, seq, h, c->eps);
        matmul_bf16(q, xn, L->wq, seq, h, qd);
        matmul_bf16(k, xn, L->wk, seq, h, kvd);
        matmul_bf16(v, xn, L->wv, seq, h, kvd);
        rms_norm_per_head(q, L->q_norm, seq, c->heads, hd, c->eps);
        rms_norm_per_head(k, L->k_norm, seq, c->kv_heads, hd, c->eps);
        for (int r = 0; r < seq; r++) {
            apply_rope(q + (size_t)r * qd, rc + (size_t)r * hd, rs + (size_t)r * hd, c->heads, hd);
            apply_rope(k + (size_t)r * kvd, rc + (size_t)r * hd, rs + (size_t)r * hd, c->kv_heads, hd);
            memcpy(kv_at(s, s->k_cache, li, start + r), k + (size_t)r * kvd, sizeof(float) * kvd);
            memcpy(kv_at(s, s->v_cache, li, start + r), v + (size_t)r * kvd, sizeof(float) * kvd);
            round_kv(kv_at(s, s->k_cache, li, start + r), kvd, s->kv_round);
            round_kv(kv_at(s, s->v_cache, li, start + r), kvd, s->kv_round);
        }
        causal_attention(att, q, kv_at(s, s->k_cache, li, 0), kv_at(s, s->v_cache, li, 0),
                         seq, start + seq, c->heads, c->kv_heads, hd, scale, start);
        matmul_bf16(proj, att, L->wo, seq, qd, h);
        for (size_t i = 0; i < (size_t)seq * h; i++) x[i] += proj[i];
        orc_rms_norm(xn, x, L->post_attn_norm, seq, h, c->eps);
        matmul_bf16(g, xn, L->gate, seq, h, I);
        matmul_bf16(u, xn, L->up, seq, h, I);
        /* SwiGLU: silu(g) * u, qwen_swiglu_multiply (qwen_asr_kernels.c:895-959) */
        for (size_t j = 0; j < (size_t)seq * I; j++) g[j] = g[j] / (1.0f + expf(-g[j])) * u[j];
        matmul_bf16(proj, g, L->down, seq, I, h);
        for (size_t i = 0; i < (size_t)seq * h; i++) x[i] += proj[i];
    }
    free(xn); free(q); free(k); free(v); free(att); free(proj);
    free(g); free(u); free(rc); free(rs);
}

/* qwen_decoder_prefill (qwen_asr_decoder.c:262-359): append seq_len positions,
 * no logits. */
int orc_prefill(orc_state *s, const float *embeds, int seq_len) {
    if (seq_len <= 0) return 0;
    if (s->len + seq_len > s->max_pos) return -1;
    size_t n = (size_t)seq_len * s->m->cfg.hidden;
    float *x = (float *)malloc(sizeof(float) * n);
    memcpy(x, embeds, sizeof(float) * n);
    run_layers(s, x, seq_len, s->len);
    s->len += seq_len;
    free(x);
    return 0;
}

/* qwen_decoder_forward (qwen_asr_decoder.c:388-476): one position, final
 * RMSNorm in place, streaming argmax over the tied embedding. */
int orc_forward(orc_state *s, const float *embed, int mask_eos, float *logits_out,
                float *hidden_out) {
    const orc_config *c = &s->m->cfg;
    if (s->len >= s->max_pos) return ORC_TOKEN_IM_END;
    float *x = (float *)malloc(sizeof(float) * c->hidden);
    memcpy(x, embed, sizeof(float) * c->hidden);
    run_layers(s, x, 1, s->len);
    s->len += 1;
    orc_rms_norm(x, x, s->m->final_norm, 1, c->hidden, c->eps);
    if (hidden_out) memcpy(hidden_out, x, sizeof(float) * c->hidden);
    if (logits_out) orc_matvec_bf16(logits_out, x, s->m->embed, c->hidden, c->vocab);
    int tok = orc_argmax_matvec_bf16(x, s->m->embed, c->hidden, c->vocab, mask_eos);
    free(x);
    return tok;
}
