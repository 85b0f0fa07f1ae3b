/*
 * qwen_asr_decoder_b200.c - drop-in replacement of the reference's
 * qwen_asr_decoder.c: the same three symbols, the same signatures, the same
 * ctx->kv_cache_len contract, backed by libqwen_asr_b200.so (B200 CUDA).
 *
 * Build it INSTEAD of qwen_asr_decoder.c, against the reference's own
 * headers (qwen_asr.h, qwen_asr_safetensors.h), and link
 * libqwen_asr_b200.so. main.c, the encoder, audio, tokenizer and safetensors
 * code are unchanged; qwen_asr.c needs one added line, a call of
 * qwen_decoder_release(ctx) at the top of qwen_free (qwen_asr.c:253). Without
 * that call every qwen_load / qwen_free cycle leaks the context's device model
 * (about 1.2 GB at 0.6B, 3.4 GB at 1.7B) and one of the 16 binding slots;
 * after 16 such cycles qwen_decoder_load fails ("too many live contexts").
 *
 *  qwen_decoder_load    (qwen_asr_decoder.c:45-116)  weights -> device once
 *  qwen_decoder_prefill (qwen_asr_decoder.c:262-359) appends at kv_cache_len
 *  qwen_decoder_forward (qwen_asr_decoder.c:388-476) one position, greedy token
 *  qwen_decoder_release (new)                        frees the device state
 *
 * Host pointers the reference leaves in qwen_decoder_t are kept compatible
 * with qwen_free (qwen_asr.c:281-287): the norm vectors are heap f32 as in the
 * reference, the matrix pointers point into the mmap, gate_up_fused_bf16 is
 * NULL (the library keeps its own fused layout on the device). After every
 * forward ctx->dec_x holds the final-normed hidden state, as in the reference
 * (qwen_asr_decoder.c:474); set QWEN_B200_SKIP_HIDDEN=1 to skip that 4-8 KB
 * copy. QWEN_B200_MASK_EOS=1 masks the two end-of-sequence ids (fixed-length
 * benchmarking; the reference has no such switch). QWEN_B200_DEVICE selects
 * the CUDA device (default 0).
 */
#include "qwen_asr.h"
#include "qwen_asr_safetensors.h"
#include "qwen_asr_b200.h"

#include <stddef.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define MAX_BINDINGS 16

typedef struct {
    qwen_ctx_t *ctx;
    qdb_model *model;
    qdb_session *session;
    int keep_hidden;
} b200_binding;

static b200_binding g_bind[MAX_BINDINGS];

static qwen_ctx_t *ctx_of_decoder(qwen_decoder_t *dec) {
    return (qwen_ctx_t *)((char *)dec - offsetof(qwen_ctx_t, decoder));
}

static b200_binding *find_binding(const qwen_ctx_t *ctx) {
    for (int i = 0; i < MAX_BINDINGS; i++)
        if (g_bind[i].ctx == ctx) return &g_bind[i];
    return NULL;
}

static const safetensor_t *find(multi_safetensors_t *ms, const char *name, safetensors_file_t **sf) {
    const safetensor_t *t = multi_safetensors_find(ms, name, sf);
    if (!t) fprintf(stderr, "decoder: weight not found: %s\n", name);
    return t;
}

static uint16_t *bf16_ptr(multi_safetensors_t *ms, const char *name) {
    safetensors_file_t *sf = NULL;
    const safetensor_t *t = find(ms, name, &sf);
    return t ? safetensors_get_bf16_direct(sf, t) : NULL;
}

static float *f32_copy(multi_safetensors_t *ms, const char *name) {
    safetensors_file_t *sf = NULL;
    const safetensor_t *t = find(ms, name, &sf);
    return t ? safetensors_get_f32(sf, t) : NULL;
}

static int env_flag(const char *name) {
    const char *v = getenv(name);
    return v && v[0] && strcmp(v, "0") != 0;
}

void qwen_decoder_release(qwen_ctx_t *ctx) {
    b200_binding *b = find_binding(ctx);
    if (!b) return;
    qdb_session_free(b->session);
    qdb_model_free(b->model);
    memset(b, 0, sizeof(*b));
}

int qwen_decoder_load(qwen_decoder_t *dec, multi_safetensors_t *ms, const qwen_config_t *cfg) {
    qwen_ctx_t *ctx = ctx_of_decoder(dec);
    qwen_decoder_release(ctx);
    b200_binding *b = find_binding(NULL);
    if (!b) {
        fprintf(stderr, "decoder: too many live contexts (max %d)\n", MAX_BINDINGS);
        return -1;
    }
    qdb_config c = {cfg->dec_hidden, cfg->dec_layers, cfg->dec_heads, cfg->dec_kv_heads, cfg->dec_head_dim,
                    cfg->dec_intermediate, cfg->vocab_size, cfg->dec_rms_norm_eps, cfg->dec_rope_theta};
    const char *dv = getenv("QWEN_B200_DEVICE");
    qdb_model *m = qdb_model_create(&c, dv ? atoi(dv) : 0);
    if (!m) {
        fprintf(stderr, "decoder: %s\n", qdb_last_error());
        return -1;
    }
    char name[512];
    dec->tok_embeddings_bf16 = bf16_ptr(ms, "thinker.model.embed_tokens.weight");
    dec->norm = f32_copy(ms, "thinker.model.norm.weight");
    int ok = dec->tok_embeddings_bf16 && dec->norm &&
             qdb_model_set_embed(m, dec->tok_embeddings_bf16, dec->norm) == 0;
    for (int i = 0; ok && i < cfg->dec_layers; i++) {
        qwen_dec_layer_t *l = &dec->layers[i];
#define BF(field, suffix)                                                                  \
    snprintf(name, sizeof(name), "thinker.model.layers.%d." suffix, i);                     \
    l->field = bf16_ptr(ms, name)
#define F32(field, suffix)                                                                 \
    snprintf(name, sizeof(name), "thinker.model.layers.%d." suffix, i);                     \
    l->field = f32_copy(ms, name)
        BF(wq_weight_bf16, "self_attn.q_proj.weight");
        BF(wk_weight_bf16, "self_attn.k_proj.weight");
        BF(wv_weight_bf16, "self_attn.v_proj.weight");
        BF(wo_weight_bf16, "self_attn.o_proj.weight");
        F32(q_norm_weight, "self_attn.q_norm.weight");
        F32(k_norm_weight, "self_attn.k_norm.weight");
        F32(input_norm, "input_layernorm.weight");
        F32(post_attn_norm, "post_attention_layernorm.weight");
        BF(gate_weight_bf16, "mlp.gate_proj.weight");
        BF(up_weight_bf16, "mlp.up_proj.weight");
        BF(down_weight_bf16, "mlp.down_proj.weight");
#undef BF
#undef F32
        l->gate_up_fused_bf16 = NULL;
        ok = l->wq_weight_bf16 && l->wk_weight_bf16 && l->wv_weight_bf16 && l->wo_weight_bf16 &&
             l->gate_weight_bf16 && l->up_weight_bf16 && l->down_weight_bf16 && l->q_norm_weight &&
             l->k_norm_weight && l->input_norm && l->post_attn_norm &&
             qdb_model_set_layer(m, i, l->wq_weight_bf16, l->wk_weight_bf16, l->wv_weight_bf16,
                                 l->wo_weight_bf16, l->gate_weight_bf16, l->up_weight_bf16,
                                 l->down_weight_bf16, l->q_norm_weight, l->k_norm_weight, l->input_norm,
                                 l->post_attn_norm) == 0;
        if (!ok) fprintf(stderr, "decoder: failed to load layer %d: %s\n", i, qdb_last_error());
    }
    if (ok) ok = qdb_model_finalize(m) == 0;
    qdb_session *s = ok ? qdb_session_create(m, 2048) : NULL;
    if (!s) {
        fprintf(stderr, "decoder: %s\n", qdb_last_error());
        qdb_model_free(m);
        return -1;
    }
    qdb_model_set_mask_eos(m, env_flag("QWEN_B200_MASK_EOS"));
    b->ctx = ctx;
    b->model = m;
    b->session = s;
    b->keep_hidden = !env_flag("QWEN_B200_SKIP_HIDDEN");
    return 0;
}

void qwen_decoder_prefill(qwen_ctx_t *ctx, const float *input_embeds, int seq_len) {
    b200_binding *b = find_binding(ctx);
    if (!b || seq_len <= 0) return;
    if (qdb_prefill(b->session, input_embeds, seq_len, ctx->kv_cache_len) != 0) {
        if (qwen_verbose >= 1) fprintf(stderr, "decoder: prefill failed: %s\n", qdb_last_error());
        return; /* kv_cache_len unchanged, as the reference on failure */
    }
    ctx->kv_cache_len += seq_len;
}

int qwen_decoder_forward(qwen_ctx_t *ctx, const float *input_embed) {
    b200_binding *b = find_binding(ctx);
    if (!b) return QWEN_TOKEN_IM_END;
    float *hidden = NULL;
    if (b->keep_hidden) {
        if (!ctx->dec_x) ctx->dec_x = (float *)malloc(sizeof(float) * ctx->config.dec_hidden);
        hidden = ctx->dec_x;
    }
    const int tok = qdb_forward(b->session, input_embed, ctx->kv_cache_len, hidden, NULL);
    if (tok < 0) {
        if (qwen_verbose >= 1) fprintf(stderr, "decoder: forward failed: %s\n", qdb_last_error());
        return QWEN_TOKEN_IM_END;
    }
    ctx->kv_cache_len += 1;
    return tok;
}
