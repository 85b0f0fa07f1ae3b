// qdb_kernels.h - device-side data layout and kernel entry points shared by
// the host runtime (qdb_runtime.cu) and the kernel files.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

// One decoder layer's device weights. Matrices are bf16 row-major [out, in].
//   qkv : [Hq*128 + 2*Hkv*128, h]  rows of q_proj, then k_proj, then v_proj
//   o   : [h, Hq*128]
//   gu  : [2*I, h]  gate row j at 2j, up row j at 2j+1 (the reference's
//                   interleave, qwen_asr_decoder.c:95-107)
//   down: [h, I]
struct QdbLayerW {
    const uint16_t *qkv, *o, *gu, *down;
    const float *q_norm, *k_norm, *in_norm, *post_norm;
};

struct QdbDims {
    int h, L, Hq, Hkv, I, V;
    float eps;
};

// Arguments of the persistent single-utterance decode step. Inter-CTA
// vectors are tagged 64-bit words (epoch << 32 | f32 bits); all must be zero
// before the first launch and epochs start at 1.
struct QdbStepArgs {
    QdbDims d;
    const QdbLayerW *layers;      // device [L]
    const uint16_t *embed;        // [V, h]
    const float *final_norm;      // [h]
    const float2 *rope;           // [rope_cap][64] (cos, sin)
    uint16_t *kc, *vc;            // [L][Hkv][cap][128] fp16
    int cap;
    int pos;                      // absolute position of this step
    const int *token_in;          // device token (embedding gathered on device) or null
    const float *x_in;            // [h] input embedding when token_in is null
    int *token_out;               // device [1]
    unsigned long long *tx;       // [h] residual stream
    unsigned long long *tqkv;     // [Hq*128 + 2*Hkv*128]
    unsigned long long *tattn;    // [Hq*128]
    unsigned long long *tact;     // [I]
    unsigned long long *tpart;    // [Hq][splits][2 + 128] attention partials
    int splits;                   // attention splits per kv head (Hkv * splits <= grid)
    float *hidden_out;            // nullable [h]
    float *logits_out;            // nullable [V]
    unsigned long long *best;     // argmax key, zero between steps
    unsigned *done;               // CTA completion counter, zero between steps
    unsigned epoch;               // first epoch of this launch
    int *err;                     // [4]: error code, then details of the first failed check
    int mask_eos;
    // extents for the kernel's own bounds checks
    const uint16_t *w_lo, *w_hi;  // all layer matrices
    int rope_cap;
    int part_len;                 // words in tpart
    unsigned long long *trace;    // nullable [grid][qdb_step_trace_events(L)] globaltimer stamps (ns)
};

// Trace events of one step per CTA: start, then per layer A entered, A data
// ready, B entered, C entered, C ready, D entered, D ready, E entered,
// E ready; then F entered, F ready, end.
__host__ __device__ static inline int qdb_step_trace_events(int layers) { return 1 + 9 * layers + 3; }

// Epochs one decode step consumes (host advances the base by this much).
__host__ __device__ static inline unsigned qdb_step_epochs(int layers) { return 5u * (unsigned)layers + 1u; }

// One compiled build of the persistent step (qdb_step.cu is built twice:
// consumer-warp count and ring-stage size are compile-time constants).
struct QdbStepKernel {
    const char *name;
    int consumer_warps;  // also sets the attention split size: 8 keys per warp
    int stage_bytes;     // bytes of one weight stage of the shared-memory ring
    int max_vector;      // longest activation vector (h, heads*head_dim, I) it loads
    int (*smem_bytes)(const QdbDims &d);
    // Launches one persistent step. grid = co-resident CTAs (one per SM).
    cudaError_t (*launch)(const QdbStepArgs &a, int grid, cudaStream_t st);
    // Sets this build's bound on data waits (cycles) on the current device.
    cudaError_t (*set_wait_limit)(long long cycles);
};

extern "C" {
// 6 consumer warps, 16 KB stages (even row counts for hidden 2048)
const QdbStepKernel *qdb_step_kernel_w6(void);
// 7 consumer warps, 12 KB stages (hidden 1024)
const QdbStepKernel *qdb_step_kernel_w7(void);
int qdb_step_max_grid(int device);
int qdb_step_max_splits(int grid, int kv_heads);

// RoPE table: tab[p][i] = (cos, sin) of (float)p * inv_freq[i], p < n_pos.
cudaError_t qdb_launch_rope_table(float2 *tab, int n_pos, float theta, cudaStream_t st);

// ---- row-batched path (prefill and multi-utterance decode) ----
// Per-row KV target: the row's cache base pointers, capacity and position.
struct QdbRowKV {
    uint16_t *kc, *vc;
    int cap, pos;
};

// RMSNorm rows written as the bf16 hi/lo split consumed by the tensor-core GEMM.
// zero (optional): [n, zero_len] f32 target of the next split-K GEMM, cleared row by row.
cudaError_t qdb_launch_rmsnorm_rows(const float *x, const float *w, uint16_t *hi, uint16_t *lo, int n, int h,
                                    float eps, cudaStream_t st, float *zero = nullptr, int zero_len = 0);
// Per-row targets: row b writes position rows[b].pos + row_pos_offset.
cudaError_t qdb_launch_qk_rope_append(const float *qkv, float *q_out, const QdbRowKV *rows,
                                      int row_pos_offset, int layer, int n, int Hq, int Hkv,
                                      const float *q_norm, const float *k_norm, const float2 *rope,
                                      float eps, cudaStream_t st, const int *step = nullptr);
// One session: row i writes position row0->pos + i.
cudaError_t qdb_launch_qk_rope_append_single(const float *qkv, float *q_out, const QdbRowKV *row0,
                                             int layer, int n, int Hq, int Hkv, const float *q_norm,
                                             const float *k_norm, const float2 *rope, float eps,
                                             cudaStream_t st);
// Causal prefill attention on the tensor cores (tcgen05) for several sessions
// at once (qdb_attn_tc.cu). Segment = one session's prompt rows.
struct QdbAttnSeg {
    int row0;       // first row of the segment in q / out
    int start_pos;  // position of that row
    int n;          // rows
    int cap;        // the session's KV capacity
};
// K or V cache map of one session over all layers (host memory, 128 bytes).
int qdb_attn_kv_map(void *map, const uint16_t *cache, int L, int Hkv, int cap);
// maps: device [2 * nseg] (K, V per segment); max_n: longest segment.
// hi/lo (optional): write the output as its bf16 split [rows, Hq*128] instead of f32 out.
cudaError_t qdb_launch_attn_prefill_tc(const void *maps, const QdbAttnSeg *segs, int nseg, int max_n, int layer,
                                       int Hq, int Hkv, const float *q, float *out, int *err, cudaStream_t st,
                                       uint16_t *hi = nullptr, uint16_t *lo = nullptr);
// Independent rows (one query each) over per-row caches. cnt (optional,
// [n * Hkv], all zero and left at zero): the last split of each unit merges
// the partials itself; without it a merge launch follows when splits > 1.
cudaError_t qdb_launch_attn_rows(const float *q, const QdbRowKV *rows, int row_pos_offset, int layer,
                                 int n, int Hq, int Hkv, int splits, float *part, float *out,
                                 cudaStream_t st, int *err = nullptr, const int *step = nullptr,
                                 uint16_t *hi = nullptr, uint16_t *lo = nullptr, unsigned *cnt = nullptr);
// Fused form of qdb_launch_qk_rope_append + qdb_launch_attn_rows (qkv: the
// raw [n, (Hq + 2 Hkv) * 128] QKV rows; cnt required). cudaErrorNotSupported
// when the fused form is built out: launch the two instead.
cudaError_t qdb_launch_attn_rows_rope(const float *qkv, const QdbRowKV *rows, int row_pos_offset, int layer, int n,
                                      int Hq, int Hkv, int S, const float *q_norm, const float *k_norm,
                                      const float2 *rope, float eps, float *part, float *out, cudaStream_t st,
                                      int *err, const int *step, uint16_t *hi, uint16_t *lo, unsigned *cnt);
// ---- persistent batched decode step (qdb_bstep.cu) ----
// One decode position of B <= 64 independent utterances in one cooperative
// launch. Activation buffers are [feature][Bp] f32 (utterance = column).
struct QdbBatchArgs {
    QdbDims d;
    int B, Bp;                    // utterances, and tile columns (16, 32 or 64)
    int nsw;                      // weight-ring stages (qdb_bstep_ring_stages)
    int splits;                   // key splits per (utterance, KV head), <= 8
    const QdbLayerW *layers;      // device [L]
    const uint16_t *wt;           // pre-tiled weights (qdb_bstep_tile_weights): qkv, o, gu, down per layer, then embed
    const uint16_t *embed;        // [V, h]
    const float *final_norm;      // [h]
    const float2 *rope;
    int rope_cap;
    const QdbRowKV *rows;         // device [B]: KV target and position (+ step_base) of each utterance
    const int *tok_in;            // device tokens at tok_in[step_base * B + b], or null
    const float *x_in;            // [B, h] embeddings when tok_in is null
    int *tok_out;                 // device, written at tok_out[step_base * B + b]
    float *logits_out;            // nullable [B, V]
    int mask_eos;
    int step_base;                // added to every position; selects the token slots
    float *x, *qkv, *gu, *attn;   // [h][Bp], [qkvd][Bp], [2I][Bp], [Hq*128][Bp] (merged attention output)
    float *part;                  // attention partials (splits > 1): o [splits][Hq*128][Bp], then (m, l) [splits][Hq][2][Bp]
    unsigned *acnt;               // [64 * Hkv] finished splits per (utterance, KV head), zero between layers
    unsigned long long *stats;    // [(3L + 3) * 64] epoch-tagged 1/rms words
    unsigned long long *best;     // [64] argmax keys, zero between launches
    unsigned *cnt;                // [n_cnt] phase counters, zero between launches
    int n_cnt;
    unsigned *done;               // zero between launches
    unsigned epoch;               // tag of this launch's statistics (never 0)
    int *err;                     // [4]
    unsigned *prog;               // nullable [grid][17]: progress of each role (read after a failed wait)
    unsigned long long *trace;    // nullable [grid][qdb_bstep_trace_events(L)] globaltimer stamps (ns)
    unsigned long long *detail;   // nullable [grid][256]: layer-1 item stamps (profiling)
};
// Trace events of one batched step per CTA: per layer {QKV inputs ready, QKV X
// tiles built, attention start, attention end, O inputs ready, QKV drained, O
// drained, DOWN drained}, then {LM inputs ready, LM drained, end}.
__host__ __device__ static inline int qdb_bstep_trace_events(int layers) { return 8 * layers + 3; }
int qdb_bstep_ring_stages(int Bp, int R);
size_t qdb_bstep_tiled_elems(int N, int K);
cudaError_t qdb_bstep_tile_weights(const uint16_t *w, int N, int K, uint16_t *out, int lm_order, cudaStream_t st);
size_t qdb_bstep_smem(int Bp, int R);
int qdb_bstep_counters(int layers);
cudaError_t qdb_launch_bstep(const QdbBatchArgs *args, int grid, cudaStream_t st);
cudaError_t qdb_set_wait_limit_bstep(long long cycles);

// Tensor-core GEMM (qdb_tcgemm.cu): Y (op)= X W^T with X given as bf16 hi/lo.
cudaError_t qdb_launch_split_bf16(const float *x, uint16_t *hi, uint16_t *lo, size_t count, cudaStream_t st);
cudaError_t qdb_launch_gemm_tc(const uint16_t *W, const uint16_t *Xh, const uint16_t *Xl, float *Y, int n, int N, int K,
                               int mode, int splits, int *err, cudaStream_t st);
cudaError_t qdb_launch_swiglu_split(const float *gu, uint16_t *hi, uint16_t *lo, size_t count, cudaStream_t st);
int qdb_gemm_tc_splits(int n, int N, int K, int sms);
// Prefill gate/up + SwiGLU written as the bf16 split [n, N/2] (n > 64).
extern "C" cudaError_t qdb_launch_gemm_tc_swiglu_split(const uint16_t *W, const uint16_t *Xh, const uint16_t *Xl,
                                                       uint16_t *yhi, uint16_t *ylo, int n, int N, int K, int *err,
                                                       cudaStream_t st);
// Same with an optional f32 bias [N] added to every output (once, also under split-K).
extern "C" cudaError_t qdb_launch_gemm_tc_bias(const uint16_t *W, const uint16_t *Xh, const uint16_t *Xl, float *Y,
                                               int n, int N, int K, int mode, int splits, int *err, cudaStream_t st,
                                               const float *bias);
// Bound (cycles) on the tensor-core GEMMs' data waits, current device.
cudaError_t qdb_set_wait_limit_tcgemm(long long cycles);
// Writes (host memory, 128 bytes) the tensor map of a bf16 [rows, cols]
// weight matrix for 128 x 64 tiles, 128-byte swizzle. 0 = ok.
int qdb_make_weight_map(void *map, const uint16_t *base, int rows, int cols);

// Sets the calling thread's qdb_last_error message; returns -1.
int qdb_set_error(const char *msg);

// What the host-side modules (stream scheduler) need of a finalized model.
struct qdb_model;
struct QdbModelInfo {
    const uint16_t *embed;  // device bf16 [vocab, hidden]
    int hidden, vocab, device;
    cudaStream_t stream;
};
int qdb_model_internals(qdb_model *m, QdbModelInfo *out);
// prompt rows: desc_dev[r] >= 0 token id, < 0 audio row -(desc+1) (qdb_stream.cu)
cudaError_t qdb_launch_prompt_rows(const uint16_t *embed, const int *desc_dev, const float *audio_dev, float *out_dev,
                                   int n_rows, int hidden, cudaStream_t st);
// step (optional, device): the rows' tokens are read at tokens + *step * n
// (embed) / written at tokens + *step * n (argmax), and positions advance by
// *step (qk_rope_append, attn_rows): the form a captured decode step replays.
// keys (optional, device, [2n] zeros): the vocabulary is split over several
// CTAs per row, combined through keys (left at zero again).
cudaError_t qdb_launch_argmax_rows(const float *logits, int n, int V, int mask_eos, int *tokens,
                                   cudaStream_t st, const int *step = nullptr, unsigned long long *keys = nullptr);
cudaError_t qdb_launch_embed_rows(const uint16_t *embed, const int *tokens, float *x, int n, int h, int V,
                                  cudaStream_t st, const int *step = nullptr);
cudaError_t qdb_launch_step_advance(int *step, cudaStream_t st);
}
