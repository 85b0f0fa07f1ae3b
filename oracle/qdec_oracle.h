/*
 * qdec_oracle.h - CPU restatement of the reference Qwen3 decoder hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA path is compared with;
 * it is never linked into, called by, or shipped with the product library.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it.
 *
 * Parity of this restatement is pinned against the reference itself: the
 * reference's own decoder sources are compiled by oracle/Makefile into
 * oracle/_ref/ and driven on the same inputs (tests/test_oracle.py), and the
 * reference's outputs on a small configuration are committed as golden vectors
 * under tests/golden/.
 */
#ifndef QDEC_ORACLE_H
#define QDEC_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int hidden;        /* dec_hidden */
    int layers;        /* dec_layers */
    int heads;         /* dec_heads (query heads) */
    int kv_heads;      /* dec_kv_heads */
    int head_dim;      /* dec_head_dim */
    int intermediate;  /* dec_intermediate */
    int vocab;         /* vocab_size */
    float eps;         /* dec_rms_norm_eps */
    float theta;       /* dec_rope_theta */
} orc_config;

typedef struct orc_model orc_model;
typedef struct orc_state orc_state;

/* Weight pointers are borrowed (caller keeps them alive), same as the
 * reference's mmap'd BF16 pointers. Matrices are row-major [out, in] bf16. */
orc_model *orc_model_create(const orc_config *cfg, const uint16_t *embed,
                            const float *final_norm);
int orc_model_set_layer(orc_model *m, int layer,
                        const uint16_t *wq, const uint16_t *wk,
                        const uint16_t *wv, const uint16_t *wo,
                        const uint16_t *gate, const uint16_t *up,
                        const uint16_t *down,
                        const float *q_norm, const float *k_norm,
                        const float *input_norm, const float *post_attn_norm);
void orc_model_free(orc_model *m);

/* f32 KV cache, same as the reference. */
orc_state *orc_state_create(orc_model *m, int max_pos);
void orc_state_free(orc_state *s);
int orc_state_len(const orc_state *s);
void orc_state_set_len(orc_state *s, int len);
/* Test-only: round the stored K/V (0 = f32 as the reference, 1 = bf16,
 * 2 = fp16) to measure what a 16-bit device cache costs in parity. */
void orc_state_set_kv_round(orc_state *s, int mode);

/* Appends seq_len positions at the current length; returns 0 / -1. */
int orc_prefill(orc_state *s, const float *embeds, int seq_len);

/* One position at the current length. Returns the greedy token. When
 * mask_eos is set, tokens 151643 and 151645 are never chosen. logits_out
 * (nullable) receives [vocab] f32 final-layer logits, hidden_out (nullable)
 * the final-normed hidden state [hidden]. */
int orc_forward(orc_state *s, const float *embed, int mask_eos,
                float *logits_out, float *hidden_out);

/* Stand-alone restatements of the per-op kernels, for unit parity. */
void orc_matvec_bf16(float *y, const float *x, const uint16_t *W, int in_dim, int out_dim);
int orc_argmax_matvec_bf16(const float *x, const uint16_t *W, int in_dim, int out_dim,
                           int mask_eos);
void orc_rms_norm(float *out, const float *x, const float *w, int seq, int hidden, float eps);

void orc_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
