/*
 * qwen_asr_encoder_b200.c - drop-in replacement of the reference's
 * qwen_asr_encoder.c: the same two symbols and signatures, backed by
 * libqwen_asr_b200.so (the audio encoder on the B200).
 *
 *  qwen_encoder_load    (qwen_asr_encoder.c:66-168)  weights -> device once
 *  qwen_encoder_forward (qwen_asr_encoder.c:171-372) mel -> malloc'd
 *                        [tokens, output_dim], freed by the caller as before
 *  qwen_encoder_release (new)                        frees the device state
 *
 * Build it INSTEAD of qwen_asr_encoder.c against the reference's headers and
 * link libqwen_asr_b200.so. The tensors are read through the reference's own
 * safetensors API by the same names: conv kernels, biases and norms as f32
 * copies (safetensors_get_f32, as load_f32 does; freed after the upload),
 * matrices as bf16 pointers into the mapped file (the dtype the reference's
 * load_bf16_as_f32 requires). The fields of qwen_encoder_t stay NULL, so
 * qwen_free's free() calls on them are no-ops; call qwen_encoder_release(ctx)
 * in qwen_free to return the device memory before process exit.
 * QWEN_B200_DEVICE selects the CUDA device (default 0).
 */
#include "qwen_asr.h"
#include "qwen_asr_safetensors.h"
#include "qwen_asr_b200.h"

#include <stddef.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define MAX_ENC_BINDINGS 16
#define P "thinker.audio_tower."

typedef struct {
    qwen_ctx_t *ctx;
    qdb_encoder *enc;
} enc_binding;

static enc_binding g_enc[MAX_ENC_BINDINGS];

static qwen_ctx_t *ctx_of_encoder(qwen_encoder_t *enc) {
    return (qwen_ctx_t *)((char *)enc - offsetof(qwen_ctx_t, encoder));
}

static enc_binding *find_enc(const qwen_ctx_t *ctx) {
    for (int i = 0; i < MAX_ENC_BINDINGS; i++)
        if (g_enc[i].ctx == ctx) return &g_enc[i];
    return NULL;
}

/* f32 copy of a tensor (any dtype the reference's loader accepts) */
static float *f32_of(multi_safetensors_t *ms, const char *name) {
    safetensors_file_t *sf = NULL;
    const safetensor_t *t = multi_safetensors_find(ms, name, &sf);
    if (!t) {
        fprintf(stderr, "encoder: weight not found: %s\n", name);
        return NULL;
    }
    return safetensors_get_f32(sf, t);
}

static const uint16_t *bf16_of(multi_safetensors_t *ms, const char *name) {
    safetensors_file_t *sf = NULL;
    const safetensor_t *t = multi_safetensors_find(ms, name, &sf);
    if (!t) {
        fprintf(stderr, "encoder: weight not found: %s\n", name);
        return NULL;
    }
    return safetensors_get_bf16_direct(sf, t);
}

void qwen_encoder_release(qwen_ctx_t *ctx) {
    enc_binding *b = find_enc(ctx);
    if (!b) return;
    qdb_encoder_free(b->enc);
    memset(b, 0, sizeof(*b));
}

#define NF32 16
int qwen_encoder_load(qwen_encoder_t *enc, multi_safetensors_t *ms, const qwen_config_t *cfg) {
    qwen_ctx_t *ctx = ctx_of_encoder(enc);
    qwen_encoder_release(ctx);
    enc_binding *b = find_enc(NULL);
    if (!b) {
        fprintf(stderr, "encoder: too many live contexts (max %d)\n", MAX_ENC_BINDINGS);
        return -1;
    }
    const char *dv = getenv("QWEN_B200_DEVICE");
    qdb_encoder_config c = {cfg->enc_d_model, cfg->enc_layers, cfg->enc_heads, cfg->enc_head_dim,
                            cfg->enc_ffn_dim, cfg->enc_output_dim};
    qdb_encoder *e = qdb_encoder_create(&c, dv ? atoi(dv) : 0);
    if (!e) {
        fprintf(stderr, "encoder: %s\n", qdb_last_error());
        return -1;
    }
    char name[512];
    float *f[NF32] = {0};
    int rc = 0;
    /* conv stem (f32 kernels and biases, bf16 projection) */
    const char *stem[6] = {P "conv2d1.weight", P "conv2d1.bias", P "conv2d2.weight",
                           P "conv2d2.bias",   P "conv2d3.weight", P "conv2d3.bias"};
    for (int i = 0; i < 6; i++) f[i] = f32_of(ms, stem[i]);
    const uint16_t *cout = bf16_of(ms, P "conv_out.weight");
    if (!f[0] || !f[1] || !f[2] || !f[3] || !f[4] || !f[5] || !cout ||
        qdb_encoder_set_stem(e, f[0], f[1], f[2], f[3], f[4], f[5], cout))
        rc = -1;
    for (int i = 0; i < 6; i++) free(f[i]), f[i] = NULL;
    for (int l = 0; rc == 0 && l < cfg->enc_layers; l++) {
        const uint16_t *w[6];
        const char *mats[6] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                               "self_attn.out_proj", "fc1", "fc2"};
        const char *vecs[10] = {"self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias",
                                "self_attn.out_proj.bias", "self_attn_layer_norm.weight",
                                "self_attn_layer_norm.bias", "fc1.bias", "fc2.bias",
                                "final_layer_norm.weight", "final_layer_norm.bias"};
        for (int i = 0; i < 6; i++) {
            snprintf(name, sizeof(name), P "layers.%d.%s.weight", l, mats[i]);
            w[i] = bf16_of(ms, name);
            if (!w[i]) rc = -1;
        }
        for (int i = 0; i < 10; i++) {
            snprintf(name, sizeof(name), P "layers.%d.%s", l, vecs[i]);
            f[i] = f32_of(ms, name);
            if (!f[i]) rc = -1;
        }
        if (rc == 0 && qdb_encoder_set_layer(e, l, w[0], f[0], w[1], f[1], w[2], f[2], w[3], f[3], f[4], f[5], w[4],
                                             f[6], w[5], f[7], f[8], f[9]))
            rc = -1;
        for (int i = 0; i < 10; i++) free(f[i]), f[i] = NULL;
    }
    if (rc == 0) {
        f[0] = f32_of(ms, P "ln_post.weight");
        f[1] = f32_of(ms, P "ln_post.bias");
        f[2] = f32_of(ms, P "proj1.bias");
        f[3] = f32_of(ms, P "proj2.bias");
        const uint16_t *p1 = bf16_of(ms, P "proj1.weight"), *p2 = bf16_of(ms, P "proj2.weight");
        if (!f[0] || !f[1] || !f[2] || !f[3] || !p1 || !p2 ||
            qdb_encoder_set_post(e, f[0], f[1], p1, f[2], p2, f[3]) || qdb_encoder_finalize(e))
            rc = -1;
        for (int i = 0; i < 4; i++) free(f[i]);
    }
    if (rc) {
        fprintf(stderr, "encoder: load failed: %s\n", qdb_last_error());
        qdb_encoder_free(e);
        return -1;
    }
    b->ctx = ctx;
    b->enc = e;
    return 0;
}

float *qwen_encoder_forward(qwen_ctx_t *ctx, const float *mel, int mel_frames, int *out_seq_len) {
    enc_binding *b = find_enc(ctx);
    if (!b) {
        fprintf(stderr, "encoder: not loaded\n");
        return NULL;
    }
    float *out = qdb_encoder_forward(b->enc, mel, mel_frames, out_seq_len);
    if (!out) fprintf(stderr, "encoder: %s\n", qdb_last_error());
    return out;
}
