/*
 * ref_harness.c - drives the UNMODIFIED reference decoder (qwen_asr_decoder.c,
 * qwen_asr_kernels*.c, qwen_asr_safetensors.c, compiled from the reference
 * tree by oracle/Makefile into oracle/_ref/) on weights held in memory.
 *
 * TEST INFRASTRUCTURE ONLY: used to pin the oracle restatement, to make the
 * golden vectors and as bench.py's reference CPU arm. Never part of the
 * product library.
 *
 * - Weights: one host blob plus a tensor table is presented to the reference
 *   loader as a single in-memory safetensors file (the loader only reads
 *   `data`, `header_size` and the table; qwen_asr_safetensors.c:249-287).
 *   qwen_decoder_load (qwen_asr_decoder.c:45-116) then runs unchanged.
 * - EOS masking: the library is linked with -Wl,--wrap=qwen_argmax_matvec_bf16
 *   so the reference decoder's call (qwen_asr_decoder.c:475) lands in
 *   __wrap_qwen_argmax_matvec_bf16 below, which re-runs the reference argmax on
 *   the row ranges either side of the two EOS ids. The reference has no such
 *   switch; this is the benchmark's fixed-length-decode convention.
 * - Logits: after each step ctx->dec_x holds the final-normed hidden state
 *   (qwen_asr_decoder.c:474); logits are that vector times the tied embedding.
 * - Audio encoder (refh_encoder_*): qwen_encoder_load / qwen_encoder_forward
 *   (qwen_asr_encoder.c) over a tensor table of the same kind.
 */
#include "qwen_asr.h"
#include "qwen_asr_kernels.h"
#include "qwen_asr_safetensors.h"

#include <stdlib.h>
#include <string.h>
#include <sys/time.h>

int qwen_verbose = 0;
int qwen_monitor = 0;

static int g_mask_eos = 0;

int __real_qwen_argmax_matvec_bf16(const float *x, const uint16_t *W, int in_dim, int out_dim);

static float row_dot(const float *x, const uint16_t *row, int n) {
    float s = 0.0f;
    for (int k = 0; k < n; k++) {
        uint32_t b = ((uint32_t)row[k]) << 16;
        float w;
        memcpy(&w, &b, sizeof(w));
        s += w * x[k];
    }
    return s;
}

int __wrap_qwen_argmax_matvec_bf16(const float *x, const uint16_t *W, int in_dim, int out_dim) {
    if (!g_mask_eos || out_dim <= QWEN_TOKEN_ENDOFTEXT)
        return __real_qwen_argmax_matvec_bf16(x, W, in_dim, out_dim);
    /* Candidate ranges: [0, 151643), [151644, 151645), [151646, out_dim). */
    int cand[3];
    int nc = 0;
    cand[nc++] = __real_qwen_argmax_matvec_bf16(x, W, in_dim, QWEN_TOKEN_ENDOFTEXT);
    cand[nc++] = QWEN_TOKEN_ENDOFTEXT + 1;
    if (out_dim > QWEN_TOKEN_IM_END + 1)
        cand[nc++] = QWEN_TOKEN_IM_END + 1 +
            __real_qwen_argmax_matvec_bf16(x, W + (size_t)(QWEN_TOKEN_IM_END + 1) * in_dim,
                                           in_dim, out_dim - QWEN_TOKEN_IM_END - 1);
    int best = cand[0];
    float bv = row_dot(x, W + (size_t)best * in_dim, in_dim);
    for (int i = 1; i < nc; i++) {
        float v = row_dot(x, W + (size_t)cand[i] * in_dim, in_dim);
        if (v > bv) { bv = v; best = cand[i]; }
    }
    return best;
}

typedef struct {
    qwen_ctx_t *ctx;
    safetensors_file_t *sf;
    multi_safetensors_t *ms;
} refh_t;

/* In-memory tensor table over one blob (the loaders read tensors by name
 * through multi_safetensors_find). Shapes are [n][2]; tensors of more
 * dimensions are passed flattened to two (the loaders use only the element
 * count). */
static refh_t *table_create(const uint8_t *blob, int n_tensors, const char *names, const int64_t *offsets,
                            const int64_t *nbytes, const int *dtypes, const int *ndims, const int64_t *shapes) {
    if (n_tensors > SAFETENSORS_MAX_TENSORS) return NULL;
    refh_t *h = (refh_t *)calloc(1, sizeof(*h));
    h->sf = (safetensors_file_t *)calloc(1, sizeof(safetensors_file_t));
    h->ms = (multi_safetensors_t *)calloc(1, sizeof(multi_safetensors_t));
    h->ctx = (qwen_ctx_t *)calloc(1, sizeof(qwen_ctx_t));
    /* safetensors_data() adds 8 + header_size to `data`. */
    h->sf->data = (void *)((uintptr_t)blob - 8);
    h->sf->header_size = 0;
    h->sf->num_tensors = n_tensors;
    const char *p = names;
    for (int i = 0; i < n_tensors; i++) {
        safetensor_t *t = &h->sf->tensors[i];
        snprintf(t->name, sizeof(t->name), "%s", p);
        p += strlen(p) + 1;
        t->dtype = (safetensor_dtype_t)dtypes[i];
        t->ndim = ndims[i];
        t->shape[0] = shapes[2 * i];
        t->shape[1] = shapes[2 * i + 1];
        t->data_offset = (size_t)offsets[i];
        t->data_size = (size_t)nbytes[i];
    }
    h->ms->shards[0] = h->sf;
    h->ms->num_shards = 1;
    return h;
}

/* cfg = {hidden, layers, heads, kv_heads, head_dim, intermediate, vocab}.
 * names: n_tensors NUL-terminated strings back to back. offsets are byte
 * offsets into blob; dtypes use safetensor_dtype_t; shapes are [n][2]. */
void *refh_create(const int *cfg, float eps, float theta, const uint8_t *blob,
                  int n_tensors, const char *names, const int64_t *offsets,
                  const int64_t *nbytes, const int *dtypes, const int *ndims,
                  const int64_t *shapes, int n_threads) {
    refh_t *h = table_create(blob, n_tensors, names, offsets, nbytes, dtypes, ndims, shapes);
    if (!h) return NULL;

    qwen_config_t *c = &h->ctx->config;
    c->dec_hidden = cfg[0];
    c->dec_layers = cfg[1];
    c->dec_heads = cfg[2];
    c->dec_kv_heads = cfg[3];
    c->dec_head_dim = cfg[4];
    c->dec_intermediate = cfg[5];
    c->vocab_size = cfg[6];
    c->dec_rms_norm_eps = eps;
    c->dec_rope_theta = theta;
    h->ctx->safetensors = h->ms;

    qwen_set_threads(n_threads > 0 ? n_threads : 1);
    if (qwen_decoder_load(&h->ctx->decoder, h->ms, c) != 0) {
        free(h->ctx); free(h->ms); free(h->sf); free(h);
        return NULL;
    }
    return h;
}

int refh_len(void *hp) { return ((refh_t *)hp)->ctx->kv_cache_len; }
void refh_set_len(void *hp, int len) { ((refh_t *)hp)->ctx->kv_cache_len = len; }

double refh_now_ms(void) {
    struct timeval tv;
    gettimeofday(&tv, NULL);
    return tv.tv_sec * 1000.0 + tv.tv_usec / 1000.0;
}

void refh_prefill(void *hp, const float *embeds, int seq_len) {
    qwen_decoder_prefill(((refh_t *)hp)->ctx, embeds, seq_len);
}

int refh_forward(void *hp, const float *embed, int mask_eos, float *logits_out,
                 float *hidden_out) {
    refh_t *h = (refh_t *)hp;
    g_mask_eos = mask_eos;
    int tok = qwen_decoder_forward(h->ctx, embed);
    g_mask_eos = 0;
    const qwen_config_t *c = &h->ctx->config;
    if (hidden_out) memcpy(hidden_out, h->ctx->dec_x, sizeof(float) * c->dec_hidden);
    if (logits_out)
        for (int v = 0; v < c->vocab_size; v++)
            logits_out[v] = row_dot(h->ctx->dec_x,
                                    h->ctx->decoder.tok_embeddings_bf16 + (size_t)v * c->dec_hidden,
                                    c->dec_hidden);
    return tok;
}

/* Greedy loop of the reference caller (qwen_asr.c:729-759) with the host
 * embedding lookup (qwen_asr.c:353-360), n_steps tokens, no tokenizer.
 * Returns elapsed wall ms (gettimeofday, as the reference's own timers). */
double refh_decode_loop(void *hp, int first_token, int n_steps, int mask_eos, int *tokens_out) {
    refh_t *h = (refh_t *)hp;
    int dim = h->ctx->config.dec_hidden;
    float *e = (float *)malloc(sizeof(float) * dim);
    int tok = first_token;
    double t0 = refh_now_ms();
    for (int i = 0; i < n_steps; i++) {
        const uint16_t *src = h->ctx->decoder.tok_embeddings_bf16 + (size_t)tok * dim;
        for (int d = 0; d < dim; d++) {
            uint32_t b = ((uint32_t)src[d]) << 16;
            memcpy(&e[d], &b, sizeof(float));
        }
        g_mask_eos = mask_eos;
        tok = qwen_decoder_forward(h->ctx, e);
        g_mask_eos = 0;
        if (tokens_out) tokens_out[i] = tok;
    }
    double ms = refh_now_ms() - t0;
    free(e);
    return ms;
}

/* Defined only by the drop-in decoder (qwen-asr_b200/dropin); absent when the
 * reference's own qwen_asr_decoder.c is linked. */
void qwen_decoder_release(qwen_ctx_t *ctx) __attribute__((weak));

void refh_free(void *hp) {
    refh_t *h = (refh_t *)hp;
    if (!h) return;
    qwen_ctx_t *ctx = h->ctx;
    if (qwen_decoder_release) qwen_decoder_release(ctx);
    for (int i = 0; i < ctx->config.dec_layers; i++) {
        qwen_dec_layer_t *l = &ctx->decoder.layers[i];
        free(l->q_norm_weight); free(l->k_norm_weight);
        free(l->input_norm); free(l->post_attn_norm);
        free(l->gate_up_fused_bf16);
    }
    free(ctx->decoder.norm);
    free(ctx->kv_cache_k); free(ctx->kv_cache_v);
    free(ctx->dec_x); free(ctx->dec_x_norm); free(ctx->dec_q); free(ctx->dec_k);
    free(ctx->dec_v); free(ctx->dec_attn_out); free(ctx->dec_proj_out);
    free(ctx->dec_gate); free(ctx->dec_up); free(ctx->dec_ffn_out);
    free(ctx->dec_rope_cos); free(ctx->dec_rope_sin);
    free(ctx->pref_x); free(ctx->pref_x_norm); free(ctx->pref_q); free(ctx->pref_k);
    free(ctx->pref_v); free(ctx->pref_attn_out); free(ctx->pref_proj_out);
    free(ctx->pref_ffn_out); free(ctx->pref_gate); free(ctx->pref_gate_up);
    free(ctx->rope_cache_cos); free(ctx->rope_cache_sin); free(ctx->rope_inv_freq);
    free(ctx);
    free(h->ms);
    free(h->sf);
    free(h);
}

/* ---- Audio encoder: the reference's qwen_encoder_load / qwen_encoder_forward
 * (qwen_asr_encoder.c:66-168, :171-372) over the same kind of tensor table.
 * ecfg = {d_model, layers, heads, head_dim, ffn_dim, output_dim}; the window
 * settings are the reference's defaults (qwen_asr.c:183 and the config
 * detection: n_window 50, n_window_infer 800, chunk 100). */
void *refh_encoder_create(const int *ecfg, const uint8_t *blob, int n_tensors, const char *names,
                          const int64_t *offsets, const int64_t *nbytes, const int *dtypes, const int *ndims,
                          const int64_t *shapes, int n_threads) {
    refh_t *h = table_create(blob, n_tensors, names, offsets, nbytes, dtypes, ndims, shapes);
    if (!h) return NULL;
    qwen_config_t *c = &h->ctx->config;
    c->enc_d_model = ecfg[0];
    c->enc_layers = ecfg[1];
    c->enc_heads = ecfg[2];
    c->enc_head_dim = ecfg[3];
    c->enc_ffn_dim = ecfg[4];
    c->enc_output_dim = ecfg[5];
    c->enc_n_window = 50;
    c->enc_n_window_infer = 800;
    c->enc_chunk_size = 100;
    c->enc_conv_proj_dim = QWEN_CONV_HIDDEN * 16;
    h->ctx->safetensors = h->ms;
    qwen_set_threads(n_threads > 0 ? n_threads : 1);
    if (qwen_encoder_load(&h->ctx->encoder, h->ms, c) != 0) {
        free(h->ctx); free(h->ms); free(h->sf); free(h);
        return NULL;
    }
    return h;
}

/* mel [128, frames] -> out [seq_len, output_dim] (up to cap_rows rows);
 * returns seq_len, or -1. */
int refh_encoder_forward(void *hp, const float *mel, int frames, float *out, int cap_rows) {
    refh_t *h = (refh_t *)hp;
    int seq = 0;
    float *e = qwen_encoder_forward(h->ctx, mel, frames, &seq);
    if (!e) return -1;
    int n = seq < cap_rows ? seq : cap_rows;
    if (out) memcpy(out, e, sizeof(float) * (size_t)n * h->ctx->config.enc_output_dim);
    free(e);
    return seq;
}

/* Defined only by the drop-in encoder (qwen-asr_b200/dropin). */
void qwen_encoder_release(qwen_ctx_t *ctx) __attribute__((weak));

void refh_encoder_free(void *hp) {
    refh_t *h = (refh_t *)hp;
    if (!h) return;
    if (qwen_encoder_release) qwen_encoder_release(h->ctx);
    qwen_encoder_t *enc = &h->ctx->encoder;
    free(enc->conv1_weight); free(enc->conv1_bias); free(enc->conv2_weight); free(enc->conv2_bias);
    free(enc->conv3_weight); free(enc->conv3_bias); free(enc->conv_out_weight);
    for (int i = 0; i < h->ctx->config.enc_layers; i++) {
        qwen_enc_layer_t *l = &enc->layers[i];
        free(l->wq_weight); free(l->wq_bias); free(l->wk_weight); free(l->wk_bias);
        free(l->wv_weight); free(l->wv_bias); free(l->wo_weight); free(l->wo_bias);
        free(l->attn_norm_weight); free(l->attn_norm_bias);
        free(l->fc1_weight); free(l->fc1_bias); free(l->fc2_weight); free(l->fc2_bias);
        free(l->ffn_norm_weight); free(l->ffn_norm_bias);
    }
    free(enc->ln_post_weight); free(enc->ln_post_bias);
    free(enc->proj1_weight); free(enc->proj1_bias); free(enc->proj2_weight); free(enc->proj2_bias);
    free(h->ctx); free(h->ms); free(h->sf); free(h);
}
