/*
 * qwen_asr_b200.h - C ABI of the B200 decoder library (libqwen_asr_b200.so).
 *
 * This library replaces, for the Qwen3 decoder, the reference's
 * qwen_asr_decoder.c and the decoder-used kernels of qwen_asr_kernels*.c
 * (dispatch in qwen_asr_kernels_impl.h). Plain pointers and sizes only.
 * Host code of the reference (qwen_asr.c) keeps calling
 * qwen_decoder_load / qwen_decoder_prefill / qwen_decoder_forward; the thin C
 * adapter in qwen-asr_b200/dropin/qwen_asr_decoder_b200.c implements those
 * three symbols on top of the functions below.
 *
 * Conventions
 *  - Weights: bf16 (uint16_t bit patterns) row-major [out, in] matrices and
 *    f32 norm vectors, given as HOST pointers; each is copied to the device
 *    once. The caller may free or unmap them after qdb_model_finalize().
 *  - Activations at the boundary are f32, as in the reference.
 *  - Return codes: 0 = ok, -1 = error (message via qdb_last_error()).
 *    Token-returning calls return the token id (>= 0) or -1.
 *  - All work of a model runs on one CUDA stream owned by the model; every
 *    host-pointer call is synchronous like the reference's CPU functions.
 *  - Not thread-safe per model (the reference API is single-caller).
 */
#ifndef QWEN_ASR_B200_H
#define QWEN_ASR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QDB_TOKEN_ENDOFTEXT 151643
#define QDB_TOKEN_IM_END    151645

/* Decoder shape. Mirrors the decoder fields of qwen_config_t
 * (qwen_asr.h:59-68). head_dim must be 128; hidden and intermediate must be
 * multiples of 256; heads must be a multiple of kv_heads. */
typedef struct {
    int hidden;
    int layers;
    int heads;
    int kv_heads;
    int head_dim;
    int intermediate;
    int vocab;
    float eps;
    float theta;
} qdb_config;

typedef struct qdb_model qdb_model;
typedef struct qdb_session qdb_session;

/* Last error message of the calling thread ("" if none). */
const char *qdb_last_error(void);

/* Number of CUDA devices visible (0 when no GPU/driver). Never fails. */
int qdb_device_count(void);

/* ---- Model (weights), replaces qwen_decoder_load (qwen_asr_decoder.c:45-116) ---- */

/* Creates an empty model on `device` and allocates device storage for all
 * weights. Returns NULL on error. */
qdb_model *qdb_model_create(const qdb_config *cfg, int device);

/* Token embedding / tied lm_head [vocab, hidden] bf16 and final norm [hidden]
 * f32 (thinker.model.embed_tokens.weight, thinker.model.norm.weight). */
int qdb_model_set_embed(qdb_model *m, const uint16_t *embed, const float *final_norm);

/* One decoder layer (thinker.model.layers.{i}.*): q/k/v/o, gate/up/down bf16
 * matrices, q_norm/k_norm [head_dim] and input/post-attention norms [hidden]
 * f32. gate and up are separate [intermediate, hidden] matrices; the library
 * builds its own fused layout (the reference's gate_up interleave,
 * qwen_asr_decoder.c:95-107). */
int qdb_model_set_layer(qdb_model *m, int layer,
                        const uint16_t *wq, const uint16_t *wk, const uint16_t *wv,
                        const uint16_t *wo, const uint16_t *gate, const uint16_t *up,
                        const uint16_t *down,
                        const float *q_norm, const float *k_norm,
                        const float *input_norm, const float *post_attn_norm);

/* Checks every weight was set and waits for the uploads. */
int qdb_model_finalize(qdb_model *m);
void qdb_model_free(qdb_model *m);

/* Benchmark switch: when set, greedy selection never returns 151643 or
 * 151645 (fixed-length decoding). The reference has no such switch. */
int qdb_model_set_mask_eos(qdb_model *m, int enable);

/* ---- Session: one utterance's device KV cache (qwen_ctx_t KV fields,
 * qwen_asr.h:187-191; kv_cache_init / kv_cache_grow, qwen_asr_decoder.c:122-160).
 * K/V are stored fp16 [layer][kv_head][pos][head_dim]; the cache grows
 * (doubling, contents kept) when a call needs more positions than it holds. */
qdb_session *qdb_session_create(qdb_model *m, int initial_capacity);
void qdb_session_free(qdb_session *s);
int qdb_session_capacity(const qdb_session *s);
int qdb_session_reserve(qdb_session *s, int positions);

/* ---- Prefill, replaces qwen_decoder_prefill (qwen_asr_decoder.c:262-359) ----
 * Appends seq_len positions starting at absolute position start_pos (the
 * caller's kv_cache_len, which stays authoritative on the host: the caller may
 * rewind it, as the streaming loop does at qwen_asr.c:1764). embeds: host f32
 * [seq_len, hidden]. seq_len == 0 is a no-op. */
int qdb_prefill(qdb_session *s, const float *embeds, int seq_len, int start_pos);

/* Same with a DEVICE pointer to the embeddings (no host copy). */
int qdb_prefill_device(qdb_session *s, const float *embeds_dev, int seq_len, int start_pos);

/* Prefill of n independent sessions of one model in ONE row batch (no
 * reference counterpart: the reference prefills one utterance per process):
 * session i appends seq_lens[i] positions at start_pos[i]; embeds holds the
 * rows of all sessions back to back (host f32 [sum(seq_lens), hidden]). The
 * projections run as one tensor-core GEMM over every row; attention stays
 * causal within each session. Equivalent to n qdb_prefill calls. */
int qdb_prefill_batch(qdb_session *const *sessions, int n, const float *embeds,
                      const int *seq_lens, const int *start_pos);

/* Same with a DEVICE pointer to the embeddings. */
int qdb_prefill_batch_device(qdb_session *const *sessions, int n, const float *embeds_dev,
                             const int *seq_lens, const int *start_pos);

/* ---- One decode step, replaces qwen_decoder_forward (qwen_asr_decoder.c:388-476) ----
 * Runs position `pos` with the host f32 embedding [hidden]; returns the greedy
 * token. hidden_out (nullable, host, [hidden]) receives the final-normed hidden
 * state the reference leaves in ctx->dec_x; logits_out (nullable, host,
 * [vocab]) the final-layer logits. */
int qdb_forward(qdb_session *s, const float *embed, int pos, float *hidden_out,
                float *logits_out);

/* ---- Device-resident greedy loop (embedding lookup on the device, the
 * caller loop of qwen_asr.c:729-759 without the tokenizer). Starts from
 * `first_token` at position `pos` and runs n_steps steps back to back;
 * tokens_out (host, [n_steps]) receives the greedy tokens. */
int qdb_decode_greedy(qdb_session *s, int first_token, int pos, int n_steps, int *tokens_out);

/* ---- Batched decode of independent utterances (no reference counterpart:
 * the reference decodes one utterance per process). Row b runs session
 * sessions[b] at position pos[b] with embedding row b of embeds (host f32
 * [n, hidden]); tokens_out[b] receives its greedy token and logits_out
 * (nullable, host f32 [n, vocab]) its final-layer logits. The model keeps a
 * CUDA graph of this step and replays it while n, its scratch, the RoPE table
 * and the EOS mask are unchanged; sessions and positions may differ from call
 * to call. The projections accumulate split-K partials with atomics, so
 * logits may differ between runs in the last bits (about 1e-6 relative). */
int qdb_forward_batch(qdb_session *const *sessions, int n, const float *embeds,
                      const int *pos, int *tokens_out, float *logits_out);

/* Batched device-resident greedy loop over n sessions: row b starts from
 * first_tokens[b] at pos[b]; tokens_out is [n_steps, n] (host). Steps after
 * the first replay a CUDA graph captured on the model's stream. */
int qdb_decode_greedy_batch(qdb_session *const *sessions, int n, const int *first_tokens,
                            const int *pos, int n_steps, int *tokens_out);

/* Profiling: runs one greedy step (token at position pos) with per-phase
 * timestamps. trace_out receives [ctas][events] globaltimer values (ns); the
 * events of each CTA are: start, then per layer {A entered, A data ready,
 * B entered, C entered, C ready, D entered, D ready, E entered, E ready},
 * then {F entered, F ready, end} (A = input norm + QKV, B = attention,
 * C = O-proj, D = post-norm + gate/up, E = down, F = lm_head + argmax).
 * Returns the number of events per CTA, or -1 (e.g. when max_words is too
 * small). Stands in for the reference's per-stage timers
 * (qwen_asr.c:606-607, :714-715) at the granularity of one step. */
int qdb_trace_step(qdb_session *s, int token, int pos, unsigned long long *trace_out, int max_words);

/* Profiling of the persistent batched step (qdb_bstep.cu: up to 64 rows in
 * one cooperative launch; qdb_forward_batch and qdb_decode_greedy_batch use
 * it when QWEN_ASR_B200_BATCH=persistent, and the captured per-kernel graph
 * otherwise): runs one step like qdb_forward_batch (its tokens are dropped)
 * with globaltimer stamps. trace_out receives [ctas][events] values (ns); the
 * events of each CTA are, per layer: QKV inputs ready, QKV X tiles built,
 * attention start, attention end, O inputs ready, QKV drained, O drained,
 * DOWN drained; then lm_head inputs ready, lm_head drained, end. After those
 * [ctas][events] words come [ctas][256] detail stamps of layer 1 (per CTA:
 * 0..63 MMA item start, 64..127 X tile build start, 128..191 X tile built,
 * 192..223 epilogue segment ready, 224..255 segment drained; 0 = unused), so
 * max_words must hold ctas * (events + 256). Returns the number of events per
 * CTA, or -1. */
int qdb_trace_batch_step(qdb_session *const *sessions, int n, const float *embeds, const int *pos,
                         unsigned long long *trace_out, int max_words);

/* One decode step that allocates nothing. No counterpart in the reference.
 *
 * For callers that must not allocate GPU memory while decoding: code running
 * under a memory budget enforced by a pool or arena they do not own, real-time
 * loops where a cudaMalloc could stall on a device-wide synchronisation, or
 * hosts that forbid allocation after start-up. It runs the same persistent
 * step as qdb_forward, but the step's scratch (its inter-CTA vectors and the
 * argmax / error words) lives in one fixed array inside the library instead
 * of the model's own buffers: 512 KiB per GPU, held from library load to
 * process exit, enough for both reference decoder shapes; larger models are
 * refused with an error.
 *
 * embed_dev: DEVICE f32 [hidden] embedding of position pos; token_dev: DEVICE
 * int receiving the greedy token. The session must already hold pos (use
 * qdb_session_reserve beforehand): nothing is grown here. The call is
 * synchronous on the model's stream. The first call on a device looks up the
 * array's device address and clears it, so make that first call before any
 * stream capture. Every call on a device shares the one array and leaves its
 * contents behind; calls that overlap on the GPU (e.g. from two models on the
 * same device driven concurrently) race and must not be issued. */
int qdb_forward_noalloc(qdb_session *s, const float *embed_dev, int pos, int *token_dev);

/* Bound on the kernels' data waits, in SM clock cycles (default about one
 * second; cycles < 0 restores it). A kernel whose wait runs out records an
 * error, stops and returns; the call then fails with "a bounded wait ... ran
 * out" and the model stays usable. It applies to the waits of the persistent
 * decode step (one CTA waiting for another CTA's results or for its weight
 * copies) and of the tensor-core GEMMs (a stage's copies, a free stage); the
 * waits that drain a CTA's own copies or MMAs before it exits keep the fixed
 * one-second bound. The setting is per device (every model on the device of
 * m), so it exists for tests of the error path and for callers that want a
 * stuck step reported sooner. cycles = 0 makes a wait give up at its first
 * unsuccessful check.
 *
 * Host-side failure injection, for tests of the callers' error handling: the
 * environment variable QWEN_ASR_B200_FAULT (read at each call) holds a comma
 * list of "alloc" (every device allocation of the library fails) and "launch"
 * (every prefill / decode call fails before its first kernel launch). */
int qdb_model_set_wait_limit(qdb_model *m, long long cycles);

/* ---- Streaming scheduler: many concurrent streams of one model, the
 * decoder side of the streaming mode (stream_impl, qwen_asr.c:1214-2152).
 * Each call processes chunk k of every stream together: prompt rebuild with
 * the rolled-back text prefix, KV rewind to the longest unchanged prompt
 * prefix, ONE row-batched prefill of all deltas, ONE device greedy loop over
 * all streams, then the reference's commit rules on token ids (repeat-run
 * suppression, fixed frontier, overlap de-duplication, degeneration /
 * stagnation recovery, periodic re-anchoring). The encoder and its window
 * cache stay with the caller, which clears that cache when a stream reports
 * a reset. Emitted pieces are token ids. ---- */
typedef struct qdb_streams qdb_streams;

typedef struct {
    int max_new_tokens;  /* decode steps per chunk (ctx->stream_max_new_tokens, 32) */
    int rollback;        /* ctx->stream_rollback (5) */
    int unfixed_chunks;  /* ctx->stream_unfixed_chunks (2) */
    int past_text;       /* ctx->past_text_conditioning (0 by default in the reference) */
    /* prompt template; a NULL pointer selects the reference's ids
     * (PROMPT_PREFIX_HEAD / _TAIL / PROMPT_SUFFIX_BASE, qwen_asr.c:339-347) */
    const int *head_tokens; int n_head_tokens;
    const int *tail_tokens; int n_tail_tokens;
    const int *suffix_tokens; int n_suffix_tokens;
    const int *prompt_tokens; int n_prompt_tokens; /* ctx->prompt_tokens (NULL = none) */
    const int *force_tokens; int n_force_tokens;   /* ctx->force_prompt_tokens (NULL = none) */
    int asr_text_token;  /* <asr_text> id (<= 0: 151704) */
} qdb_stream_config;

/* n_streams sessions on model m; cfg NULL = the reference defaults
 * (qwen_asr.c:238-242). NULL on error. */
qdb_streams *qdb_streams_create(qdb_model *m, int n_streams, const qdb_stream_config *cfg);
void qdb_streams_free(qdb_streams *s);

/* One chunk of every stream. audio[i]: host f32 [audio_len[i], hidden], the
 * encoder output this chunk's prompt carries (cached windows + re-encoded
 * tail); audio_len[i] == 0 is the reference's "no encoder output" path (the
 * chunk counts but decodes nothing); audio_len[i] < 0 leaves stream i out of
 * this call untouched. is_final[i]: last chunk of stream i.
 * Outputs (optional): n_emitted[i] text tokens committed this chunk (read
 * them with qdb_streams_tokens), reset[i] 1 = recovery reset, 2 = periodic
 * re-anchor (the caller clears its encoder window cache). 0 = ok. */
int qdb_streams_chunk(qdb_streams *s, const float *const *audio, const int *audio_len, const int *is_final,
                      int *n_emitted, int *reset);

/* Token history of stream i: which 0 = emitted text tokens, 1 = raw history
 * (prefix + generated, qwen_asr.c raw_tokens), 2 = stable candidate. Copies
 * up to cap ids into buf (may be NULL) and returns the full count, or -1. */
int qdb_streams_tokens(const qdb_streams *s, int stream, int which, int *buf, int cap);

/* Counters of stream i into out[8]: chunk index, chunks decoded, prefill rows
 * (total), prefill rows reused, decode steps counted as the reference counts
 * n_generated, the last chunk's n_generated, its reused prefix, its prefill
 * length. 0 = ok. */
int qdb_streams_stats(const qdb_streams *s, int stream, long long *out);

/* Restarts stream i as a new stream (empty history, chunk 0, no prefix to
 * reuse); its KV storage is kept. 0 = ok. */
int qdb_streams_reset(qdb_streams *s, int stream);

/* Device time of the last qdb_streams_chunk call: ms[0] the batched prefill
 * (with the prompt rows' upload), ms[1] the greedy loop; counts[0] streams that
 * ran, counts[1] prompt rows prefilled. Either pointer may be NULL. 0 = ok. */
int qdb_streams_last_chunk(const qdb_streams *s, float *ms, int *counts);

/* Prompt rows on the device (the offline path's input embeddings,
 * qwen_asr.c:626-700): desc[r] >= 0 is a token id (its embedding row),
 * desc[r] < 0 is row -(desc[r] + 1) of audio_dev [*, hidden] (the encoder
 * output); out_dev [n_rows, hidden] f32. Enqueued on the model's stream;
 * desc is host memory and may be reused on return. 0 = ok. */
int qdb_build_prompt_device(qdb_model *m, const int *desc, int n_rows, const float *audio_dev, float *out_dev);

/* ---- Audio encoder, replaces qwen_encoder_load / qwen_encoder_forward
 * (qwen_asr_encoder.c:66-168, :171-372). Conv2D stem per 100-frame chunk,
 * transformer layers with windowed bidirectional attention, projection to the
 * decoder width, all on the GPU. ---- */
typedef struct qdb_encoder qdb_encoder;

typedef struct {
    int d_model, layers, heads, head_dim, ffn_dim, output_dim; /* qwen_config_t enc_* (qwen_asr.h:48-53) */
} qdb_encoder_config;

/* Empty encoder on `device` (head_dim 64, heads * 64 = d_model, d_model and
 * ffn_dim multiples of 64). NULL on error. */
qdb_encoder *qdb_encoder_create(const qdb_encoder_config *cfg, int device);
void qdb_encoder_free(qdb_encoder *e);

/* Weights in the reference loader's forms: conv kernels and all biases /
 * norms f32 (load_f32), matrices bf16 (load_bf16_as_f32's source).
 * conv1 [480, 1, 3, 3], conv2 / conv3 [480, 480, 3, 3], biases [480];
 * conv_out [d_model, 7680]. */
int qdb_encoder_set_stem(qdb_encoder *e, const float *conv1_w, const float *conv1_b, const float *conv2_w,
                         const float *conv2_b, const float *conv3_w, const float *conv3_b,
                         const uint16_t *conv_out_w);
/* Layer i: q/k/v/out [d, d] + biases, attention LayerNorm, fc1 [ffn, d],
 * fc2 [d, ffn] + biases, FFN LayerNorm. */
int qdb_encoder_set_layer(qdb_encoder *e, int i, const uint16_t *wq, const float *bq, const uint16_t *wk,
                          const float *bk, const uint16_t *wv, const float *bv, const uint16_t *wo, const float *bo,
                          const float *ln1_w, const float *ln1_b, const uint16_t *fc1_w, const float *fc1_b,
                          const uint16_t *fc2_w, const float *fc2_b, const float *ln2_w, const float *ln2_b);
/* ln_post, proj1 [d, d], proj2 [output_dim, d] with biases. */
int qdb_encoder_set_post(qdb_encoder *e, const float *ln_w, const float *ln_b, const uint16_t *proj1_w,
                         const float *proj1_b, const uint16_t *proj2_w, const float *proj2_b);
/* Checks every weight was set. */
int qdb_encoder_finalize(qdb_encoder *e);

/* Output rows for mel_frames (13 per full 100-frame chunk). */
int qdb_encoder_tokens(int mel_frames);

/* Same contract as qwen_encoder_forward: host mel [128, mel_frames] ->
 * malloc'd host [tokens, output_dim] (caller frees), token count in
 * *out_seq_len; NULL on error. Synchronous. */
float *qdb_encoder_forward(qdb_encoder *e, const float *mel, int mel_frames, int *out_seq_len);

/* Device form on the encoder's stream (qdb_encoder_stream): mel_dev
 * [128, mel_frames] -> out_dev [qdb_encoder_tokens(mel_frames), output_dim].
 * Returns the token count, or -1. */
int qdb_encoder_forward_device(qdb_encoder *e, const float *mel_dev, int mel_frames, float *out_dev);

/* Many utterances in one pass (no reference counterpart: the reference
 * encodes one utterance per call): mel_dev[u] [128, mel_frames[u]] (device)
 * -> out_dev [sum of tokens, output_dim], utterance u's rows after those of
 * 0..u-1. The row-wise stages (convolutions, projections, norms) run once
 * over all utterances; attention windows restart at each utterance, so each
 * utterance's rows equal its own qdb_encoder_forward_device. Returns the total
 * token count, or -1. */
int qdb_encoder_forward_batch_device(qdb_encoder *e, int n_utt, const float *const *mel_dev, const int *mel_frames,
                                     float *out_dev);
void *qdb_encoder_stream(qdb_encoder *e);

/* ---- Log-mel front end, replaces qwen_mel_spectrogram (qwen_asr_audio.c:293-390,
 * declared at qwen_asr_audio.h:32). 16 kHz mono f32 samples -> [128, n_frames]
 * f32 log-mel (reflect pad 200, periodic Hann 400, 201-bin DFT power, hop 160
 * with the last frame dropped, Slaney filter bank, log10, clamp to the global
 * max - 8, (v + 4) / 4). Runs on the current CUDA device. ---- */

/* n_frames the spectrogram of n_samples has (<= 0: too short). */
int qdb_mel_frames(int n_samples);

/* Same contract as the reference: returns a malloc'd [128, *out_frames] host
 * array the caller frees with free(), or NULL (audio too short, or an error;
 * the message is in qdb_last_error). Synchronous. */
float *qdb_mel_spectrogram(const float *samples, int n_samples, int *out_frames);

/* Device form: samples_dev f32 [n_samples] -> mel_dev f32 [128, n_frames]
 * (n_frames = qdb_mel_frames(n_samples)), enqueued on `stream` (a
 * cudaStream_t as void*, NULL = the legacy default stream). 0 = ok. */
int qdb_mel_spectrogram_device(const float *samples_dev, int n_samples, float *mel_dev, void *stream);

/* Waits for all queued work of the model's stream. */
int qdb_model_sync(qdb_model *m);

/* The cudaStream_t (as void*) every call of this model runs on, for callers
 * that time or order work against it. */
void *qdb_model_stream(qdb_model *m);

#ifdef __cplusplus
}
#endif
#endif
