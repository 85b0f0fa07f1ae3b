// qdb_runtime.cu - host runtime behind the C ABI in include/qwen_asr_b200.h:
// device weight upload, per-utterance KV sessions, launch sequencing on the
// model's stream. Replaces the decoder's host-side state handling of the
// reference (qwen_asr_decoder.c: load :45-116, KV cache :122-170, prefill
// :262-359, forward :388-476).
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#ifndef QDB_AR_ITERS
#define QDB_AR_ITERS 8  // 8-key steps per warp of a batched-decode attention unit
#endif
#ifndef QDB_ATT_ITERS
#define QDB_ATT_ITERS 1  // key-loop iterations per decode attention unit
#endif
#include <string>
#include <vector>

#include "../../include/qwen_asr_b200.h"
#include "qdb_kernels.h"

#define QDB_HD 128  // head_dim (the kernels support only this)

static thread_local std::string g_err;

static int fail(const char *fmt, ...) __attribute__((format(printf, 1, 2)));
static int fail(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return -1;
}

// Records msg as the calling thread's last error (for the other translation
// units' entry points) and returns -1.
int qdb_set_error(const char *msg) { return fail("%s", msg); }

#define CK(call)                                                                              \
    do {                                                                                      \
        cudaError_t e_ = (call);                                                              \
        if (e_ != cudaSuccess) return fail("%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                           __FILE__, __LINE__);                              \
    } while (0)

// Host-side failure injection (tests of the error paths; no GPU fault is
// involved): QWEN_ASR_B200_FAULT holds a comma list of "alloc" (every device
// allocation of the library fails) and "launch" (every decode / prefill call
// fails before its first kernel launch). Read at each call.
static bool injected(const char *kind) {
    const char *v = getenv("QWEN_ASR_B200_FAULT");
    if (!v || !*v) return false;
    const size_t n = strlen(kind);
    for (const char *p = v; (p = strstr(p, kind)) != nullptr; p += n)
        if ((p == v || p[-1] == ',') && (p[n] == 0 || p[n] == ',')) return true;
    return false;
}

static int launch_gate() {
    if (injected("launch")) return fail("injected launch failure (QWEN_ASR_B200_FAULT)");
    return 0;
}

template <typename T>
static int dev_alloc(T **p, size_t count) {
    *p = nullptr;
    if (injected("alloc")) return fail("injected allocation failure (QWEN_ASR_B200_FAULT)");
    if (count == 0) count = 1;
    cudaError_t e = cudaMalloc((void **)p, count * sizeof(T));
    if (e != cudaSuccess) return fail("cudaMalloc(%zu bytes): %s", count * sizeof(T), cudaGetErrorString(e));
    return 0;
}

struct RowScratch {
    int cap = 0;
    float *X = nullptr, *QKV = nullptr, *Q = nullptr, *ATT = nullptr, *ACT = nullptr;
    uint16_t *XH = nullptr, *XL = nullptr;  // bf16 hi/lo of the current GEMM input [cap, max(h, qd, I)]
    uint16_t *XH2 = nullptr, *XL2 = nullptr;  // [cap, I]: the SwiGLU split written by the gate/up GEMM (rows > 64)
    float *GU = nullptr;                    // [64, 2I] gate/up sums of split-K decode GEMMs
    int *err = nullptr;                     // [4] device error words of the tensor-core GEMMs
    int *step = nullptr;                    // [1] step counter of a captured batched decode step
    float *LOG = nullptr;  // [cap, V] only for batched decode
    int log_cap = 0;
    unsigned long long *amax = nullptr;  // [2 * log_cap] sliced-argmax keys and counters (kept at zero)
    float *part = nullptr;
    size_t part_cap = 0;
    unsigned *acnt = nullptr;  // [acnt_cap] split counters of the decode attention units (kept at zero)
    int acnt_cap = 0;
    QdbRowKV *rowkv = nullptr;
    int rowkv_cap = 0;
    void *amaps = nullptr;         // device CUtensorMap [2 * aseg_cap]: K, V map of each prefill segment
    QdbAttnSeg *asegs = nullptr;   // device [aseg_cap]
    int aseg_cap = 0;
    int *tok = nullptr;
    size_t tok_cap = 0;
};

// Scratch of the persistent batched decode step (qdb_bstep.cu), sized for its
// largest batch (64 utterances, 8 key splits); allocated on first use.
struct BatchScratch {
    float *x = nullptr, *qkv = nullptr, *gu = nullptr, *part = nullptr, *attn = nullptr;
    unsigned *acnt = nullptr;
    unsigned long long *stats = nullptr, *best = nullptr;
    unsigned *cnt = nullptr, *done = nullptr;
    int *err = nullptr;
    unsigned *prog = nullptr;  // [sms][8] progress words (diagnostics)
    uint16_t *wt = nullptr;  // pre-tiled weights: every 128 x 64 tile one contiguous 16 KB block
    int n_cnt = 0;
    unsigned epoch = 1;
};

struct qdb_model {
    qdb_config cfg;
    // captured step of qdb_forward_batch, valid while its key (row count,
    // split count and every scratch pointer it uses) is unchanged
    cudaGraphExec_t fb_exec = nullptr;
    std::vector<const void *> fb_key;
    QdbDims d;
    int device = 0;
    int sms = 0;
    cudaStream_t st = nullptr;
    int qd = 0, kvd = 0;

    uint16_t *w = nullptr;  // all layer matrices
    size_t layer_elems = 0, off_qkv = 0, off_o = 0, off_gu = 0, off_down = 0;
    float *norms = nullptr;  // per layer: in[h], post[h], q[128], k[128]
    size_t norm_stride = 0;
    uint16_t *embed = nullptr;
    float *final_norm = nullptr;
    QdbLayerW *layers_dev = nullptr;
    std::vector<QdbLayerW> layers_host;
    std::vector<char> layer_set;
    bool embed_set = false;
    bool finalized = false;
    int mask_eos = 0;

    float2 *rope = nullptr;
    int rope_cap = 0;

    // single-utterance step scratch (tagged inter-CTA vectors, see qdb_step.cu)
    int grid = 0;                    // CTAs of the persistent step
    unsigned long long *tags = nullptr;  // one allocation: tx | tqkv | tattn | tact | tpart
    size_t tags_len = 0;
    unsigned long long *tx = nullptr, *tqkv = nullptr, *tattn = nullptr, *tact = nullptr, *tpart = nullptr;
    unsigned epoch = 1;
    float *x_in = nullptr;
    float *hidden_dev = nullptr, *logits_dev = nullptr;
    unsigned *done = nullptr;
    unsigned long long *best = nullptr;
    int *err = nullptr;
    int *tok_dev = nullptr;
    int tok_cap = 0;
    int max_splits = 1;
    const QdbStepKernel *step_k = nullptr;  // the step build this model uses
    float *h_stage = nullptr;  // pinned [max(h, V)]
    int *h_tok = nullptr;      // pinned
    RowScratch rs;
    BatchScratch bs;
    // prompt-row descriptors: pinned host staging + device copy (grow-only)
    int *pdesc_host = nullptr, *pdesc_dev = nullptr;
    int pdesc_cap = 0;
    cudaEvent_t pdesc_ev = nullptr;
    // weight upload staging (two pinned buffers; freed at finalize)
    unsigned char *up_buf[2] = {nullptr, nullptr};
    cudaEvent_t up_ev[2] = {nullptr, nullptr};
    int up_next = 0;
    double up_bytes = 0;
    std::vector<qdb_session *> sessions;  // live sessions (detached when the model is freed)
};

struct qdb_session {
    qdb_model *m;  // null once the model has been freed (session detached)
    uint16_t *kc = nullptr, *vc = nullptr;
    int cap = 0;
};

extern "C" const char *qdb_last_error(void) { return g_err.c_str(); }

// Prompt rows on the device for the offline path (qwen_asr.c:626-700 builds
// them on the host): desc[r] >= 0 is a token id (its embedding row), desc[r] < 0
// is audio row -(desc[r] + 1) of audio_dev. The descriptors go through a
// pinned buffer of the model (no allocation or pageable copy per call).
extern "C" int qdb_build_prompt_device(qdb_model *m, const int *desc, int n_rows, const float *audio_dev,
                                       float *out_dev) {
    g_err.clear();
    if (!m || !m->finalized) return fail("qdb_build_prompt_device: model not finalized");
    if (!desc || n_rows <= 0 || !out_dev) return fail("qdb_build_prompt_device: bad arguments");
    for (int r = 0; r < n_rows; r++) {
        if (desc[r] >= m->cfg.vocab) return fail("qdb_build_prompt_device: token %d out of range", desc[r]);
        if (desc[r] < 0 && !audio_dev) return fail("qdb_build_prompt_device: audio rows without audio");
    }
    CK(cudaSetDevice(m->device));
    if (!m->pdesc_ev) CK(cudaEventCreateWithFlags(&m->pdesc_ev, cudaEventDisableTiming));
    CK(cudaEventSynchronize(m->pdesc_ev));  // the previous call's copy has left the pinned buffer
    if (n_rows > m->pdesc_cap) {
        if (m->pdesc_host) cudaFreeHost(m->pdesc_host);
        if (m->pdesc_dev) cudaFree(m->pdesc_dev);
        m->pdesc_host = nullptr;
        m->pdesc_dev = nullptr;
        m->pdesc_cap = 0;
        const int cap = std::max(n_rows, 4096);
        CK(cudaMallocHost((void **)&m->pdesc_host, sizeof(int) * cap));
        if (dev_alloc(&m->pdesc_dev, (size_t)cap)) return -1;
        m->pdesc_cap = cap;
    }
    memcpy(m->pdesc_host, desc, sizeof(int) * n_rows);
    CK(cudaMemcpyAsync(m->pdesc_dev, m->pdesc_host, sizeof(int) * n_rows, cudaMemcpyHostToDevice, m->st));
    CK(cudaEventRecord(m->pdesc_ev, m->st));
    CK(qdb_launch_prompt_rows(m->embed, m->pdesc_dev, audio_dev, out_dev, n_rows, m->cfg.hidden, m->st));
    return 0;
}

int qdb_model_internals(qdb_model *m, QdbModelInfo *out) {
    if (!m || !out) return fail("null model");
    if (!m->finalized) return fail("model not finalized");
    out->embed = m->embed;
    out->hidden = m->cfg.hidden;
    out->vocab = m->cfg.vocab;
    out->device = m->device;
    out->stream = m->st;
    return 0;
}

extern "C" int qdb_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

static int set_dev(qdb_model *m) {
    CK(cudaSetDevice(m->device));
    return 0;
}

static int ensure_rope(qdb_model *m, int n_pos) {
    if (n_pos <= m->rope_cap) return 0;
    int cap = m->rope_cap ? m->rope_cap : 4096;
    while (cap < n_pos) cap *= 2;
    float2 *t = nullptr;
    if (dev_alloc(&t, (size_t)cap * (QDB_HD / 2))) return -1;
    CK(qdb_launch_rope_table(t, cap, m->cfg.theta, m->st));
    CK(cudaStreamSynchronize(m->st));
    if (m->rope) cudaFree(m->rope);
    m->rope = t;
    m->rope_cap = cap;
    return 0;
}

extern "C" qdb_model *qdb_model_create(const qdb_config *cfg, int device) {
    g_err.clear();
    if (!cfg) { fail("null config"); return nullptr; }
    if (cfg->head_dim != QDB_HD) { fail("head_dim must be %d (got %d)", QDB_HD, cfg->head_dim); return nullptr; }
    if (cfg->hidden <= 0 || cfg->hidden % 256 || cfg->intermediate <= 0 || cfg->intermediate % 256) {
        fail("hidden and intermediate must be positive multiples of 256");
        return nullptr;
    }
    if (cfg->kv_heads <= 0 || cfg->heads % cfg->kv_heads) { fail("heads must be a multiple of kv_heads"); return nullptr; }
    const int R = cfg->heads / cfg->kv_heads;
    if (R != 1 && R != 2 && R != 4 && R != 8) { fail("heads/kv_heads must be 1, 2, 4 or 8"); return nullptr; }
    if (cfg->layers <= 0 || cfg->layers > 32 || cfg->vocab <= 0) { fail("layers must be 1..32 and vocab > 0"); return nullptr; }
    if (cfg->heads * QDB_HD % 256) { fail("heads*head_dim must be a multiple of 256"); return nullptr; }
    // Step build: 16 KB stages for hidden >= 2048 (even rows per item), the
    // 7-warp 12 KB build below that; either one if the other cannot hold the
    // model. A ring stage must hold a gate/up row pair and one row of the
    // longest K, and the step loads vectors of at most max_vector floats.
    const QdbStepKernel *step_k = nullptr;
    {
        const long long kmax = std::max<long long>(std::max<long long>(2LL * cfg->hidden, cfg->intermediate),
                                                   (long long)cfg->heads * QDB_HD);
        const int vmax = std::max(cfg->hidden, std::max(cfg->intermediate, cfg->heads * QDB_HD));
        const QdbStepKernel *pref[2] = {qdb_step_kernel_w6(), qdb_step_kernel_w7()};
        if (cfg->hidden < 2048) std::swap(pref[0], pref[1]);
        // QWEN_ASR_B200_STEP=w6|w7 forces a build (tuning; falls back if it cannot hold the model)
        if (const char *ov = getenv("QWEN_ASR_B200_STEP"))  // "w6" / "w7": leading part of a build name
            if (ov[0] && !strncmp(ov, pref[1]->name, strlen(ov))) std::swap(pref[0], pref[1]);
        for (const QdbStepKernel *k : pref)
            if (!step_k && kmax * 2 <= k->stage_bytes && vmax <= k->max_vector) step_k = k;
        if (!step_k) {
            fail("rows of %lld bf16 / vectors of %d floats exceed the decode step's stages", kmax, vmax);
            return nullptr;
        }
    }
    int ndev = qdb_device_count();
    if (device < 0 || device >= ndev) { fail("CUDA device %d not available (%d visible)", device, ndev); return nullptr; }

    qdb_model *m = new qdb_model();
    m->cfg = *cfg;
    m->step_k = step_k;
    m->device = device;
    m->d = QdbDims{cfg->hidden, cfg->layers, cfg->heads, cfg->kv_heads, cfg->intermediate, cfg->vocab, cfg->eps};
    m->qd = cfg->heads * QDB_HD;
    m->kvd = cfg->kv_heads * QDB_HD;
    auto bad = [&]() { qdb_model_free(m); return (qdb_model *)nullptr; };
    if (set_dev(m)) return bad();
    if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess) { fail("stream create"); return bad(); }
    m->sms = qdb_step_max_grid(device);

    const size_t h = cfg->hidden, I = cfg->intermediate;
    auto al = [](size_t e) { return (e + 127) & ~(size_t)127; };  // 256-byte aligned offsets
    m->off_qkv = 0;
    m->off_o = m->off_qkv + al((m->qd + 2 * m->kvd) * h);
    m->off_gu = m->off_o + al(h * m->qd);
    m->off_down = m->off_gu + al(2 * I * h);
    m->layer_elems = m->off_down + al(h * I);
    if (dev_alloc(&m->w, m->layer_elems * cfg->layers)) return bad();
    m->norm_stride = al(2 * h + 2 * QDB_HD);
    if (dev_alloc(&m->norms, m->norm_stride * cfg->layers)) return bad();
    if (dev_alloc(&m->embed, (size_t)cfg->vocab * h)) return bad();
    if (dev_alloc(&m->final_norm, h)) return bad();
    m->layers_host.resize(cfg->layers);
    m->layer_set.assign(cfg->layers, 0);
    for (int l = 0; l < cfg->layers; l++) {
        uint16_t *b = m->w + m->layer_elems * l;
        float *nb = m->norms + m->norm_stride * l;
        m->layers_host[l] = QdbLayerW{b + m->off_qkv, b + m->off_o, b + m->off_gu, b + m->off_down,
                                      nb + 2 * h, nb + 2 * h + QDB_HD, nb, nb + h};
    }
    if (dev_alloc(&m->layers_dev, cfg->layers)) return bad();
    if (cudaMemcpy(m->layers_dev, m->layers_host.data(), sizeof(QdbLayerW) * cfg->layers,
                   cudaMemcpyHostToDevice) != cudaSuccess) { fail("layer table upload"); return bad(); }

    // step scratch. Every CTA of the persistent step must own at least one row
    // of every phase (the tagged-data ordering argument in qdb_step.cu), so the
    // grid is capped by the smallest phase.
    m->grid = m->sms;
    const int min_rows = (int)std::min<size_t>(std::min<size_t>(h, I), (size_t)(m->qd + 2 * m->kvd));
    if (m->grid > min_rows) m->grid = min_rows;
    if (m->grid < cfg->kv_heads) { fail("GPU too small for the persistent step"); return bad(); }
    m->max_splits = qdb_step_max_splits(m->grid, cfg->kv_heads);
    {
        const size_t n_x = h, n_qkv = m->qd + 2 * m->kvd, n_attn = m->qd, n_act = I;
        const size_t n_part = (size_t)cfg->heads * m->max_splits * (2 + QDB_HD);
        m->tags_len = n_x + n_qkv + n_attn + n_act + n_part;
        if (dev_alloc(&m->tags, m->tags_len)) return bad();
        m->tx = m->tags;
        m->tqkv = m->tx + n_x;
        m->tattn = m->tqkv + n_qkv;
        m->tact = m->tattn + n_attn;
        m->tpart = m->tact + n_act;
    }
    if (dev_alloc(&m->x_in, h) || dev_alloc(&m->hidden_dev, h) || dev_alloc(&m->logits_dev, cfg->vocab) ||
        dev_alloc(&m->done, 1) || dev_alloc(&m->best, 1) || dev_alloc(&m->err, 4))
        return bad();
    if (cudaMemset(m->tags, 0, m->tags_len * 8) != cudaSuccess || cudaMemset(m->done, 0, sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(m->best, 0, sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemset(m->err, 0, 4 * sizeof(int)) != cudaSuccess) { fail("scratch memset"); return bad(); }
    size_t stage = h > (size_t)cfg->vocab ? h : (size_t)cfg->vocab;
    if (cudaMallocHost((void **)&m->h_stage, stage * sizeof(float)) != cudaSuccess ||
        cudaMallocHost((void **)&m->h_tok, sizeof(int) * 4096) != cudaSuccess) { fail("pinned alloc"); return bad(); }
    if (ensure_rope(m, 4096)) return bad();
    return m;
}

extern "C" void qdb_model_free(qdb_model *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->st) cudaStreamSynchronize(m->st);
    if (m->fb_exec) cudaGraphExecDestroy(m->fb_exec);
    // Sessions still alive are detached: their device KV is released here and
    // a later qdb_session_free only deletes the handle.
    for (qdb_session *s : m->sessions) {
        cudaFree(s->kc);
        cudaFree(s->vc);
        s->kc = s->vc = nullptr;
        s->cap = 0;
        s->m = nullptr;
    }
    m->sessions.clear();
    cudaFree(m->w); cudaFree(m->norms); cudaFree(m->embed); cudaFree(m->final_norm); cudaFree(m->layers_dev);
    cudaFree(m->rope); cudaFree(m->tags); cudaFree(m->x_in);
    cudaFree(m->hidden_dev); cudaFree(m->logits_dev); cudaFree(m->done); cudaFree(m->best);
    cudaFree(m->err); cudaFree(m->tok_dev);
    RowScratch &r = m->rs;
    cudaFree(r.X); cudaFree(r.XH); cudaFree(r.XL); cudaFree(r.QKV); cudaFree(r.Q); cudaFree(r.ATT); cudaFree(r.ACT);
    cudaFree(r.XH2); cudaFree(r.XL2); cudaFree(r.LOG); cudaFree(r.amax); cudaFree(r.part); cudaFree(r.acnt); cudaFree(r.rowkv); cudaFree(r.tok); cudaFree(r.err); cudaFree(r.GU); cudaFree(r.step);
    cudaFree(r.amaps); cudaFree(r.asegs);
    BatchScratch &b = m->bs;
    cudaFree(b.x); cudaFree(b.qkv); cudaFree(b.gu); cudaFree(b.part); cudaFree(b.stats); cudaFree(b.best);
    cudaFree(b.cnt); cudaFree(b.done); cudaFree(b.err); cudaFree(b.wt); cudaFree(b.prog); cudaFree(b.attn);
    cudaFree(b.acnt);
    for (int i = 0; i < 2; i++) {
        if (m->up_buf[i]) cudaFreeHost(m->up_buf[i]);
        if (m->up_ev[i]) cudaEventDestroy(m->up_ev[i]);
    }
    if (m->pdesc_host) cudaFreeHost(m->pdesc_host);
    if (m->pdesc_dev) cudaFree(m->pdesc_dev);
    if (m->pdesc_ev) cudaEventDestroy(m->pdesc_ev);
    if (m->h_stage) cudaFreeHost(m->h_stage);
    if (m->h_tok) cudaFreeHost(m->h_tok);
    if (m->st) cudaStreamDestroy(m->st);
    delete m;
}

// ---- weight upload: pinned double-buffered staging (the reference loader
// maps the safetensors file and reads the bf16 matrices in place,
// qwen_asr_safetensors.c:194-228; here they cross PCIe once). A chunk is
// copied into one pinned buffer by the host while the other one's DMA runs;
// sources that are already pinned go straight to the device.
constexpr size_t UP_CHUNK = 32u << 20;

static bool host_pinned(const void *p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

static int up_ready(qdb_model *m) {
    for (int i = 0; i < 2; i++) {
        if (!m->up_buf[i]) CK(cudaMallocHost((void **)&m->up_buf[i], UP_CHUNK));
        if (!m->up_ev[i]) CK(cudaEventCreateWithFlags(&m->up_ev[i], cudaEventDisableTiming));
    }
    return 0;
}

// rows rows of row_bytes each, source row r at src + r * src_pitch, to
// dst + r * dst_pitch (device); contiguous when both pitches equal row_bytes.
static int upload_rows(qdb_model *m, void *dst, size_t dst_pitch, const void *src, size_t src_pitch, size_t row_bytes,
                       size_t rows) {
    m->up_bytes += (double)row_bytes * rows;
    if (host_pinned(src)) {
        CK(cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, row_bytes, rows, cudaMemcpyHostToDevice, m->st));
        return 0;
    }
    if (up_ready(m)) return -1;
    const size_t per = std::max<size_t>(1, UP_CHUNK / row_bytes);
    for (size_t r0 = 0; r0 < rows; r0 += per) {
        const size_t n = std::min(per, rows - r0);
        const int b = m->up_next;
        m->up_next ^= 1;
        CK(cudaEventSynchronize(m->up_ev[b]));  // this buffer's previous DMA is done
        unsigned char *st = m->up_buf[b];
        const unsigned char *s0 = (const unsigned char *)src + r0 * src_pitch;
        if (src_pitch == row_bytes) {
            memcpy(st, s0, n * row_bytes);
        } else {
            for (size_t r = 0; r < n; r++) memcpy(st + r * row_bytes, s0 + r * src_pitch, row_bytes);
        }
        CK(cudaMemcpy2DAsync((unsigned char *)dst + r0 * dst_pitch, dst_pitch, st, row_bytes, row_bytes, n,
                             cudaMemcpyHostToDevice, m->st));
        CK(cudaEventRecord(m->up_ev[b], m->st));
    }
    return 0;
}

static int upload(qdb_model *m, void *dst, const void *src, size_t bytes) {
    // contiguous: as rows of 1 MiB plus a tail
    const size_t rb = 1u << 20, full = bytes / rb, tail = bytes % rb;
    if (full && upload_rows(m, dst, rb, src, rb, rb, full)) return -1;
    if (tail && upload_rows(m, (unsigned char *)dst + full * rb, tail, (const unsigned char *)src + full * rb, tail,
                            tail, 1))
        return -1;
    return 0;
}

extern "C" int qdb_model_set_embed(qdb_model *m, const uint16_t *embed, const float *final_norm) {
    g_err.clear();
    if (!m || !embed || !final_norm) return fail("null argument");
    if (set_dev(m)) return -1;
    const size_t h = m->cfg.hidden;
    if (upload(m, m->embed, embed, (size_t)m->cfg.vocab * h * 2) || upload(m, m->final_norm, final_norm, h * 4))
        return -1;
    CK(cudaStreamSynchronize(m->st));  // the caller's buffers are free to go on return
    m->embed_set = true;
    return 0;
}

extern "C" int qdb_model_set_layer(qdb_model *m, int layer, const uint16_t *wq, const uint16_t *wk,
                                   const uint16_t *wv, const uint16_t *wo, const uint16_t *gate,
                                   const uint16_t *up, const uint16_t *down, const float *q_norm,
                                   const float *k_norm, const float *input_norm, const float *post_attn_norm) {
    g_err.clear();
    if (!m) return fail("null model");
    if (layer < 0 || layer >= m->cfg.layers) return fail("layer %d out of range", layer);
    if (!wq || !wk || !wv || !wo || !gate || !up || !down || !q_norm || !k_norm || !input_norm || !post_attn_norm)
        return fail("null weight pointer for layer %d", layer);
    if (set_dev(m)) return -1;
    const size_t h = m->cfg.hidden, I = m->cfg.intermediate, qd = m->qd, kvd = m->kvd;
    uint16_t *b = m->w + m->layer_elems * layer;
    // gate row j -> fused row 2j, up row j -> fused row 2j+1
    float *nb = m->norms + m->norm_stride * layer;
    if (upload(m, b + m->off_qkv, wq, qd * h * 2) || upload(m, b + m->off_qkv + qd * h, wk, kvd * h * 2) ||
        upload(m, b + m->off_qkv + (qd + kvd) * h, wv, kvd * h * 2) || upload(m, b + m->off_o, wo, h * qd * 2) ||
        upload_rows(m, b + m->off_gu, 4 * h, gate, 2 * h, 2 * h, I) ||
        upload_rows(m, b + m->off_gu + h, 4 * h, up, 2 * h, 2 * h, I) || upload(m, b + m->off_down, down, h * I * 2) ||
        upload(m, nb, input_norm, h * 4) || upload(m, nb + h, post_attn_norm, h * 4) ||
        upload(m, nb + 2 * h, q_norm, QDB_HD * 4) || upload(m, nb + 2 * h + QDB_HD, k_norm, QDB_HD * 4))
        return -1;
    CK(cudaStreamSynchronize(m->st));  // the caller's buffers are free to go on return
    m->layer_set[layer] = 1;
    return 0;
}

extern "C" int qdb_model_finalize(qdb_model *m) {
    g_err.clear();
    if (!m) return fail("null model");
    if (!m->embed_set) return fail("embedding / final norm not set");
    for (int l = 0; l < m->cfg.layers; l++)
        if (!m->layer_set[l]) return fail("layer %d not set", l);
    if (set_dev(m)) return -1;
    CK(cudaStreamSynchronize(m->st));
    CK(cudaDeviceSynchronize());
    for (int i = 0; i < 2; i++) {
        if (m->up_buf[i]) cudaFreeHost(m->up_buf[i]);
        if (m->up_ev[i]) cudaEventDestroy(m->up_ev[i]);
        m->up_buf[i] = nullptr;
        m->up_ev[i] = nullptr;
    }
    m->finalized = true;
    return 0;
}

extern "C" int qdb_model_set_mask_eos(qdb_model *m, int enable) {
    if (!m) return fail("null model");
    m->mask_eos = enable ? 1 : 0;
    return 0;
}

extern "C" int qdb_model_set_wait_limit(qdb_model *m, long long cycles) {
    g_err.clear();
    if (!m) return fail("null model");
    if (set_dev(m)) return -1;
    if (cycles < 0) cycles = 2000000000LL;  // the default: about one second of SM clock
    CK(qdb_step_kernel_w6()->set_wait_limit(cycles));
    CK(qdb_step_kernel_w7()->set_wait_limit(cycles));
    CK(qdb_set_wait_limit_tcgemm(cycles));
    CK(qdb_set_wait_limit_bstep(cycles));
    return 0;
}

extern "C" void *qdb_model_stream(qdb_model *m) { return m ? (void *)m->st : nullptr; }

extern "C" int qdb_model_sync(qdb_model *m) {
    if (!m) return fail("null model");
    if (set_dev(m)) return -1;
    CK(cudaStreamSynchronize(m->st));
    return 0;
}

// ------------------------------------------------------------------ sessions
extern "C" qdb_session *qdb_session_create(qdb_model *m, int initial_capacity) {
    g_err.clear();
    if (!m || !m->finalized) { fail("model missing or not finalized"); return nullptr; }
    qdb_session *s = new qdb_session();
    s->m = m;
    if (qdb_session_reserve(s, initial_capacity > 0 ? initial_capacity : 1024)) {
        delete s;
        return nullptr;
    }
    m->sessions.push_back(s);
    return s;
}

extern "C" void qdb_session_free(qdb_session *s) {
    if (!s) return;
    if (qdb_model *m = s->m) {
        cudaSetDevice(m->device);
        cudaStreamSynchronize(m->st);
        cudaFree(s->kc);
        cudaFree(s->vc);
        for (size_t i = 0; i < m->sessions.size(); i++)
            if (m->sessions[i] == s) {
                m->sessions.erase(m->sessions.begin() + i);
                break;
            }
    }
    delete s;
}

extern "C" int qdb_session_capacity(const qdb_session *s) { return s ? s->cap : 0; }

// Grows the cache (doubling, like kv_cache_grow, qwen_asr_decoder.c:133-160)
// and keeps the first `cap` positions of every (layer, kv head) block.
extern "C" int qdb_session_reserve(qdb_session *s, int positions) {
    if (!s) return fail("null session");
    if (!s->m) return fail("session's model has been freed");
    if (positions <= s->cap) return 0;
    qdb_model *m = s->m;
    if (set_dev(m)) return -1;
    int cap = s->cap ? s->cap : 256;
    while (cap < positions) cap *= 2;
    const size_t blocks = (size_t)m->cfg.layers * m->cfg.kv_heads;
    const size_t row = QDB_HD * 2;
    uint16_t *kc = nullptr, *vc = nullptr;
    if (dev_alloc(&kc, blocks * cap * QDB_HD)) return -1;
    if (dev_alloc(&vc, blocks * cap * QDB_HD)) { cudaFree(kc); return -1; }
    if (s->cap) {
        CK(cudaMemcpy2DAsync(kc, cap * row, s->kc, s->cap * row, s->cap * row, blocks, cudaMemcpyDeviceToDevice, m->st));
        CK(cudaMemcpy2DAsync(vc, cap * row, s->vc, s->cap * row, s->cap * row, blocks, cudaMemcpyDeviceToDevice, m->st));
        CK(cudaStreamSynchronize(m->st));
        cudaFree(s->kc);
        cudaFree(s->vc);
    }
    s->kc = kc;
    s->vc = vc;
    s->cap = cap;
    return ensure_rope(m, cap);
}

// ------------------------------------------------------------------ single-utterance step
// fetched: the error words already copied to the host (after the caller's
// stream sync), or null to read them here.
static int check_err(qdb_model *m, const int *fetched = nullptr) {
    int ev[4] = {0, 0, 0, 0};
    if (fetched) memcpy(ev, fetched, sizeof(ev));
    else CK(cudaMemcpy(ev, m->err, sizeof(ev), cudaMemcpyDeviceToHost));
    const int e = ev[0];
    if (e) {
        // A bounded wait ran out or a check refused an access: reset the
        // step's device state.
        cudaMemset(m->err, 0, 4 * sizeof(int));
        cudaMemset(m->tags, 0, m->tags_len * 8);
        cudaMemset(m->done, 0, sizeof(unsigned));
        cudaMemset(m->best, 0, sizeof(unsigned long long));
        cudaDeviceSynchronize();
        m->epoch = 1;
        return fail("device error code %d (%s; check %d: %d %d)", e,
                    e == 1   ? "a bounded wait in the decode step ran out"
                    : e == 2 ? "invalid token in the decode step"
                             : "an access refused by a bounds check",
                    ev[1], ev[2], ev[3]);
    }
    return 0;
}

static QdbStepArgs step_args(qdb_session *s, int pos) {
    qdb_model *m = s->m;
    QdbStepArgs a;
    memset(&a, 0, sizeof(a));
    a.d = m->d;
    a.layers = m->layers_dev;
    a.embed = m->embed;
    a.final_norm = m->final_norm;
    a.rope = m->rope;
    a.kc = s->kc;
    a.vc = s->vc;
    a.cap = s->cap;
    a.pos = pos;
    a.x_in = m->x_in;
    a.tx = m->tx;
    a.tqkv = m->tqkv;
    a.tattn = m->tattn;
    a.tact = m->tact;
    a.tpart = m->tpart;
    // attention splits: one key-loop iteration per unit (8 keys per consumer
    // warp), at most grid / Hkv units per head
    const int ctx = pos + 1;
    const int keys_per_unit = m->step_k->consumer_warps * 8 * QDB_ATT_ITERS;
    int S = (ctx + keys_per_unit - 1) / keys_per_unit;
    if (S > m->max_splits) S = m->max_splits;
    if (S < 1) S = 1;
    a.splits = S;
    a.best = m->best;
    a.done = m->done;
    a.err = m->err;
    a.mask_eos = m->mask_eos;
    a.w_lo = m->w;
    a.w_hi = m->w + m->layer_elems * m->cfg.layers;
    a.rope_cap = m->rope_cap;
    a.part_len = (int)((size_t)m->cfg.heads * m->max_splits * (2 + QDB_HD));
    return a;
}

static int launch_step(qdb_model *m, QdbStepArgs &a) {
    if (launch_gate()) return -1;
    const unsigned span = qdb_step_epochs(m->cfg.layers);
    if (m->epoch > 0xffffffffu - 2 * span) {  // epoch wrap: clear the tags and restart
        CK(cudaMemsetAsync(m->tags, 0, m->tags_len * 8, m->st));
        m->epoch = 1;
    }
    a.epoch = m->epoch;
    CK(m->step_k->launch(a, m->grid, m->st));
    m->epoch += span;
    return 0;
}

static int prep_pos(qdb_session *s, int last_pos) {
    if (qdb_session_reserve(s, last_pos + 1)) return -1;
    return ensure_rope(s->m, last_pos + 1);
}

extern "C" int qdb_forward(qdb_session *s, const float *embed, int pos, float *hidden_out, float *logits_out) {
    g_err.clear();
    if (!s || !embed) return fail("null argument");
    if (!s->m) return fail("session's model has been freed");
    if (pos < 0) return fail("negative position");
    qdb_model *m = s->m;
    if (set_dev(m) || prep_pos(s, pos)) return -1;
    const size_t h = m->cfg.hidden;
    memcpy(m->h_stage, embed, h * 4);
    CK(cudaMemcpyAsync(m->x_in, m->h_stage, h * 4, cudaMemcpyHostToDevice, m->st));
    if (m->tok_cap < 2) {
        cudaFree(m->tok_dev);
        if (dev_alloc(&m->tok_dev, 4096)) return -1;
        m->tok_cap = 4096;
    }
    QdbStepArgs a = step_args(s, pos);
    a.token_out = m->tok_dev;
    a.hidden_out = hidden_out ? m->hidden_dev : nullptr;
    a.logits_out = logits_out ? m->logits_dev : nullptr;
    if (launch_step(m, a)) return -1;
    // token and error words into pinned memory with the outputs: one stream
    // sync per call, no second round trip for the error check
    CK(cudaMemcpyAsync(m->h_tok, m->tok_dev, sizeof(int), cudaMemcpyDeviceToHost, m->st));
    CK(cudaMemcpyAsync(m->h_tok + 8, m->err, 4 * sizeof(int), cudaMemcpyDeviceToHost, m->st));
    if (hidden_out) CK(cudaMemcpyAsync(hidden_out, m->hidden_dev, h * 4, cudaMemcpyDeviceToHost, m->st));
    if (logits_out)
        CK(cudaMemcpyAsync(logits_out, m->logits_dev, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost, m->st));
    CK(cudaStreamSynchronize(m->st));
    if (check_err(m, m->h_tok + 8)) return -1;
    return m->h_tok[0];
}

extern "C" int qdb_decode_greedy(qdb_session *s, int first_token, int pos, int n_steps, int *tokens_out) {
    g_err.clear();
    if (!s || (n_steps > 0 && !tokens_out)) return fail("null argument");
    if (!s->m) return fail("session's model has been freed");
    if (n_steps <= 0) return 0;
    qdb_model *m = s->m;
    if (first_token < 0 || first_token >= m->cfg.vocab) return fail("token %d out of range", first_token);
    if (pos < 0) return fail("negative position");
    if (set_dev(m) || prep_pos(s, pos + n_steps - 1)) return -1;
    if (m->tok_cap < n_steps + 1) {
        cudaFree(m->tok_dev);
        m->tok_cap = 0;
        if (dev_alloc(&m->tok_dev, (size_t)n_steps + 1)) return -1;
        m->tok_cap = n_steps + 1;
    }
    m->h_tok[0] = first_token;
    CK(cudaMemcpyAsync(m->tok_dev, m->h_tok, sizeof(int), cudaMemcpyHostToDevice, m->st));
    for (int i = 0; i < n_steps; i++) {
        QdbStepArgs a = step_args(s, pos + i);
        a.token_in = m->tok_dev + i;
        a.token_out = m->tok_dev + i + 1;
        if (launch_step(m, a)) return -1;
    }
    CK(cudaMemcpyAsync(tokens_out, m->tok_dev + 1, sizeof(int) * n_steps, cudaMemcpyDeviceToHost, m->st));
    CK(cudaStreamSynchronize(m->st));
    return check_err(m);
}

extern "C" int qdb_trace_step(qdb_session *s, int token, int pos, unsigned long long *trace_out, int max_words) {
    g_err.clear();
    if (!s || !trace_out) return fail("null argument");
    if (!s->m) return fail("session's model has been freed");
    qdb_model *m = s->m;
    if (token < 0 || token >= m->cfg.vocab || pos < 0) return fail("bad token or position");
    const int ev = qdb_step_trace_events(m->cfg.layers);
    const size_t words = (size_t)m->grid * ev;
    if ((size_t)max_words < words) return fail("trace buffer needs %zu words", words);
    if (set_dev(m) || prep_pos(s, pos)) return -1;
    unsigned long long *tr = nullptr;
    if (dev_alloc(&tr, words)) return -1;
    if (m->tok_cap < 2) {
        cudaFree(m->tok_dev);
        m->tok_cap = 0;
        if (dev_alloc(&m->tok_dev, 4096)) { cudaFree(tr); return -1; }
        m->tok_cap = 4096;
    }
    m->h_tok[0] = token;
    int rc = 0;
    QdbStepArgs a = step_args(s, pos);
    a.token_in = m->tok_dev;
    a.token_out = m->tok_dev + 1;
    a.trace = tr;
    if (cudaMemcpyAsync(m->tok_dev, m->h_tok, sizeof(int), cudaMemcpyHostToDevice, m->st) != cudaSuccess ||
        launch_step(m, a) ||
        cudaMemcpyAsync(trace_out, tr, words * 8, cudaMemcpyDeviceToHost, m->st) != cudaSuccess ||
        cudaStreamSynchronize(m->st) != cudaSuccess)
        rc = fail("trace step failed: %s", cudaGetErrorString(cudaGetLastError()));
    cudaFree(tr);
    if (rc == 0 && check_err(m)) return -1;
    return rc ? -1 : ev;
}

// ------------------------------------------------------------------ row-batched path
static int ensure_rows(qdb_model *m, int n, bool logits) {
    RowScratch &r = m->rs;
    const size_t h = m->cfg.hidden, I = m->cfg.intermediate;
    if (n > r.cap) {
        int cap = r.cap ? r.cap : 64;
        while (cap < n) cap *= 2;
        cudaFree(r.X); cudaFree(r.XH); cudaFree(r.XL); cudaFree(r.QKV); cudaFree(r.Q); cudaFree(r.ATT); cudaFree(r.ACT);
        cudaFree(r.XH2); cudaFree(r.XL2);
        r.X = r.QKV = r.Q = r.ATT = r.ACT = nullptr;
        r.XH = r.XL = r.XH2 = r.XL2 = nullptr;
        r.cap = 0;
        const size_t kmax = std::max<size_t>(std::max<size_t>(h, (size_t)m->qd), I);
        if (dev_alloc(&r.X, cap * h) || dev_alloc(&r.XH, cap * kmax) || dev_alloc(&r.XL, cap * kmax) ||
            dev_alloc(&r.QKV, cap * (size_t)(m->qd + 2 * m->kvd)) || dev_alloc(&r.Q, cap * (size_t)m->qd) ||
            dev_alloc(&r.ATT, cap * (size_t)m->qd) || dev_alloc(&r.ACT, cap * I) || dev_alloc(&r.XH2, cap * I) ||
            dev_alloc(&r.XL2, cap * I))
            return -1;
        r.cap = cap;
    }
    if (logits && n > r.log_cap) {
        cudaFree(r.LOG);
        cudaFree(r.amax);
        r.LOG = nullptr;
        r.amax = nullptr;
        r.log_cap = 0;
        if (dev_alloc(&r.LOG, (size_t)n * m->cfg.vocab) || dev_alloc(&r.amax, (size_t)2 * n)) return -1;
        CK(cudaMemset(r.amax, 0, sizeof(unsigned long long) * 2 * n));
        r.log_cap = n;
    }
    if (n <= 64 && !r.GU && dev_alloc(&r.GU, (size_t)64 * 2 * I)) return -1;
    if (!r.err) {
        if (dev_alloc(&r.err, 4)) return -1;
        CK(cudaMemset(r.err, 0, 4 * sizeof(int)));
    }
    if (!r.step && dev_alloc(&r.step, 1)) return -1;
    if (n > r.rowkv_cap) {
        cudaFree(r.rowkv);
        r.rowkv = nullptr;
        r.rowkv_cap = 0;
        if (dev_alloc(&r.rowkv, n)) return -1;
        r.rowkv_cap = n;
    }
    return 0;
}

// Prompt rows of a prefill: nseg sessions whose K/V maps and segments are in
// rs.amaps / rs.asegs. per_row: rs.rowkv holds one entry per row (several
// sessions); otherwise one entry for a single session whose row i is at
// position rowkv[0].pos + i.
struct PrefillPlan {
    int nseg, max_n;
    bool per_row;
};

// One transformer stack over the rows already in rs.X. pf: prefill rows
// (causal attention over each session's cache, tensor cores); null: decode
// rows, row b uses rowkv[b] at position rowkv[b].pos + pos_off (+ *step).
static int run_rows(qdb_model *m, int n, const PrefillPlan *pf, const QdbRowKV *row0_dev, int pos_off, int max_ctx = 1,
                    const int *step = nullptr) {
    const bool single = pf != nullptr;
    if (launch_gate()) return -1;
    RowScratch &r = m->rs;
    const int h = m->cfg.hidden, I = m->cfg.intermediate, Hq = m->cfg.heads, Hkv = m->cfg.kv_heads;
    const int qkvd = m->qd + 2 * m->kvd;
    int S = 1;
    if (!single) {
        // one attention unit per QDB_AR_ITERS x 64 keys of the longest row
        // (8-key steps per warp, double-buffered)
        S = (max_ctx + 64 * QDB_AR_ITERS - 1) / (64 * QDB_AR_ITERS);
        if (S > 64) S = 64;
        if (S < 1) S = 1;
        const size_t need = (size_t)n * Hq * S * (2 + QDB_HD);
        if (need > r.part_cap) {
            cudaFree(r.part);
            r.part = nullptr;
            r.part_cap = 0;
            if (dev_alloc(&r.part, need)) return -1;
            r.part_cap = need;
        }
        if (n * Hkv > r.acnt_cap) {
            cudaFree(r.acnt);
            r.acnt = nullptr;
            r.acnt_cap = 0;
            if (dev_alloc(&r.acnt, (size_t)n * Hkv)) return -1;
            CK(cudaMemsetAsync(r.acnt, 0, sizeof(unsigned) * (size_t)n * Hkv, m->st));
            r.acnt_cap = n * Hkv;
        }
    }
    // Y (op)= X W^T from the bf16 split in XH/XL. Skinny problems (decode
    // batches of <= 64 rows) use split-K with atomic accumulation: mode 0
    // targets are zeroed first, mode 1 targets already hold the residual.
    // (the norm before a mode-0 split GEMM clears its target: zeroed = true)
    auto splits_of = [&](int N, int K) { return n <= 64 ? qdb_gemm_tc_splits(n, N, K, m->sms) : 1; };
    auto gemm = [&](const uint16_t *W, float *Y, int N, int K, int mode, bool zeroed = false) -> int {
        const int sp = splits_of(N, K);
        if (sp > 1) {
            if (mode == 0 && !zeroed) CK(cudaMemsetAsync(Y, 0, sizeof(float) * (size_t)n * N, m->st));
            CK(qdb_launch_gemm_tc(W, r.XH, r.XL, Y, n, N, K, 3, sp, r.err, m->st));
        } else {
            CK(qdb_launch_gemm_tc(W, r.XH, r.XL, Y, n, N, K, mode, 1, r.err, m->st));
        }
        return 0;
    };
    for (int l = 0; l < m->cfg.layers; l++) {
        const QdbLayerW &lw = m->layers_host[l];
        const bool qkv_split = splits_of(qkvd, h) > 1;
        CK(qdb_launch_rmsnorm_rows(r.X, lw.in_norm, r.XH, r.XL, n, h, m->cfg.eps, m->st, qkv_split ? r.QKV : nullptr,
                                   qkvd));
        if (gemm(lw.qkv, r.QKV, qkvd, h, 0, qkv_split)) return -1;
        if (single) {
            if (pf->per_row)
                CK(qdb_launch_qk_rope_append(r.QKV, r.Q, row0_dev, 0, l, n, Hq, Hkv, lw.q_norm, lw.k_norm, m->rope,
                                             m->cfg.eps, m->st));
            else
                CK(qdb_launch_qk_rope_append_single(r.QKV, r.Q, row0_dev, l, n, Hq, Hkv, lw.q_norm, lw.k_norm,
                                                    m->rope, m->cfg.eps, m->st));
            CK(qdb_launch_attn_prefill_tc(r.amaps, r.asegs, pf->nseg, pf->max_n, l, Hq, Hkv, r.Q, r.ATT, r.err, m->st,
                                          r.XH, r.XL));
        } else {
            const cudaError_t fe =
                qdb_launch_attn_rows_rope(r.QKV, row0_dev, pos_off, l, n, Hq, Hkv, S, lw.q_norm, lw.k_norm, m->rope,
                                          m->cfg.eps, r.part, r.ATT, m->st, r.err, step, r.XH, r.XL, r.acnt);
            if (fe == cudaErrorNotSupported) {
                CK(qdb_launch_qk_rope_append(r.QKV, r.Q, row0_dev, pos_off, l, n, Hq, Hkv, lw.q_norm, lw.k_norm,
                                             m->rope, m->cfg.eps, m->st, step));
                CK(qdb_launch_attn_rows(r.Q, row0_dev, pos_off, l, n, Hq, Hkv, S, r.part, r.ATT, m->st, r.err, step,
                                        r.XH, r.XL, r.acnt));
            } else {
                CK(fe);
            }
        }
        // (both attention paths write the O-projection's bf16 split directly)
        if (gemm(lw.o, r.X, h, m->qd, 1)) return -1;
        const bool gu_split = splits_of(2 * I, h) > 1;
        CK(qdb_launch_rmsnorm_rows(r.X, lw.post_norm, r.XH, r.XL, n, h, m->cfg.eps, m->st, gu_split ? r.GU : nullptr,
                                   2 * I));
        if (gu_split) {
            // split-K: gate/up sums into GU, then SwiGLU straight into the bf16 split
            if (gemm(lw.gu, r.GU, 2 * I, h, 0, true)) return -1;
            CK(qdb_launch_swiglu_split(r.GU, r.XH, r.XL, (size_t)n * I, m->st));
        } else if (n > 64) {
            // gate/up, SwiGLU and the bf16 split in one GEMM epilogue (into the
            // second split buffers: the GEMM still reads its input from the first)
            CK(qdb_launch_gemm_tc_swiglu_split(lw.gu, r.XH, r.XL, r.XH2, r.XL2, n, 2 * I, h, r.err, m->st));
            CK(qdb_launch_gemm_tc(lw.down, r.XH2, r.XL2, r.X, n, h, I, 1, 1, r.err, m->st));
            continue;
        } else {
            CK(qdb_launch_gemm_tc(lw.gu, r.XH, r.XL, r.ACT, n, 2 * I, h, 2, 1, r.err, m->st));
            CK(qdb_launch_split_bf16(r.ACT, r.XH, r.XL, (size_t)n * I, m->st));
        }
        if (gemm(lw.down, r.X, h, I, 1)) return -1;
    }
    return 0;
}

// Reads (and clears) the tensor-core GEMMs' device error words after a sync.
static int check_rows_err(qdb_model *m) {
    int ev[4] = {0, 0, 0, 0};
    CK(cudaMemcpy(ev, m->rs.err, sizeof(ev), cudaMemcpyDeviceToHost));
    if (ev[0]) {
        cudaMemset(m->rs.err, 0, sizeof(ev));
        return fail("device error code %d in a tensor-core GEMM (a bounded wait ran out)", ev[0]);
    }
    return 0;
}

// Prefill of nsess sessions in one row batch: session i appends lens[i]
// positions at starts[i]; embeds holds all rows back to back (host or device).
static int prefill_rows(qdb_session *const *ss, int nsess, const int *lens, const int *starts, const float *embeds,
                        bool device_ptr) {
    g_err.clear();
    if (!ss || nsess <= 0 || !lens || !starts) return fail("bad prefill arguments");
    if (!ss[0]) return fail("null session");
    qdb_model *m = ss[0]->m;
    if (!m) return fail("session's model has been freed");
    long long total = 0;
    int max_n = 0;
    for (int i = 0; i < nsess; i++) {
        if (!ss[i]) return fail("null session %d", i);
        if (ss[i]->m != m) return fail("session %d: sessions must share one (live) model", i);
        if (lens[i] < 0 || starts[i] < 0) return fail("session %d: negative length or position", i);
        total += lens[i];
        max_n = std::max(max_n, lens[i]);
    }
    if (total == 0) return 0;
    if (!embeds) return fail("null embeddings");
    if (total > (1 << 22)) return fail("prefill of %lld rows exceeds the 4M-row limit", total);
    const int T = (int)total;
    if (set_dev(m)) return -1;
    for (int i = 0; i < nsess; i++)
        if (lens[i] && prep_pos(ss[i], starts[i] + lens[i] - 1)) return -1;
    if (ensure_rows(m, T, false)) return -1;
    RowScratch &r = m->rs;
    if (nsess > r.aseg_cap) {
        cudaFree(r.amaps);
        cudaFree(r.asegs);
        r.amaps = nullptr;
        r.asegs = nullptr;
        r.aseg_cap = 0;
        unsigned char *mp = nullptr;
        if (dev_alloc(&mp, (size_t)nsess * 256) || dev_alloc(&r.asegs, (size_t)nsess)) {
            cudaFree(mp);
            return -1;
        }
        r.amaps = mp;
        r.aseg_cap = nsess;
    }
    const size_t h = m->cfg.hidden;
    CK(cudaMemcpyAsync(r.X, embeds, (size_t)T * h * 4, device_ptr ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                       m->st));
    // segments (empty ones dropped), their K/V maps, and the per-row KV targets
    std::vector<unsigned char> maps;
    std::vector<QdbAttnSeg> segs;
    std::vector<QdbRowKV> rk;
    int row = 0;
    for (int i = 0; i < nsess; i++) {
        if (!lens[i]) continue;
        qdb_session *s = ss[i];
        segs.push_back(QdbAttnSeg{row, starts[i], lens[i], s->cap});
        const size_t at = maps.size();
        maps.resize(at + 256);
        if (qdb_attn_kv_map(maps.data() + at, s->kc, m->cfg.layers, m->cfg.kv_heads, s->cap) ||
            qdb_attn_kv_map(maps.data() + at + 128, s->vc, m->cfg.layers, m->cfg.kv_heads, s->cap))
            return fail("KV tensor map of session %d", i);
        if (nsess > 1)
            for (int j = 0; j < lens[i]; j++) rk.push_back(QdbRowKV{s->kc, s->vc, s->cap, starts[i] + j});
        else
            rk.push_back(QdbRowKV{s->kc, s->vc, s->cap, starts[i]});
        row += lens[i];
    }
    CK(cudaMemcpyAsync(r.amaps, maps.data(), maps.size(), cudaMemcpyHostToDevice, m->st));
    CK(cudaMemcpyAsync(r.asegs, segs.data(), sizeof(QdbAttnSeg) * segs.size(), cudaMemcpyHostToDevice, m->st));
    CK(cudaMemcpyAsync(r.rowkv, rk.data(), sizeof(QdbRowKV) * rk.size(), cudaMemcpyHostToDevice, m->st));
    const PrefillPlan pf{(int)segs.size(), max_n, nsess > 1};
    const int rc = run_rows(m, T, &pf, r.rowkv, 0);
    cudaError_t e = cudaStreamSynchronize(m->st);  // (the staging vectors outlive the copies)
    if (rc) return -1;
    if (e != cudaSuccess) return fail("prefill: %s", cudaGetErrorString(e));
    return check_rows_err(m);
}

static int prefill_impl(qdb_session *s, const float *embeds, bool device_ptr, int seq_len, int start_pos) {
    g_err.clear();
    if (!s) return fail("null session");
    if (!s->m) return fail("session's model has been freed");
    if (seq_len < 0 || start_pos < 0) return fail("negative length or position");
    if (seq_len == 0) return 0;
    return prefill_rows(&s, 1, &seq_len, &start_pos, embeds, device_ptr);
}

extern "C" int qdb_prefill(qdb_session *s, const float *embeds, int seq_len, int start_pos) {
    return prefill_impl(s, embeds, false, seq_len, start_pos);
}

extern "C" int qdb_prefill_device(qdb_session *s, const float *embeds_dev, int seq_len, int start_pos) {
    return prefill_impl(s, embeds_dev, true, seq_len, start_pos);
}

extern "C" int qdb_prefill_batch(qdb_session *const *sessions, int n, const float *embeds, const int *seq_lens,
                                 const int *start_pos) {
    return prefill_rows(sessions, n, seq_lens, start_pos, embeds, false);
}

extern "C" int qdb_prefill_batch_device(qdb_session *const *sessions, int n, const float *embeds_dev,
                                        const int *seq_lens, const int *start_pos) {
    return prefill_rows(sessions, n, seq_lens, start_pos, embeds_dev, true);
}

static int batch_setup(qdb_session *const *ss, int n, const int *pos, int extra_steps, qdb_model **mo,
                       int *max_pos = nullptr) {
    if (!ss || n <= 0 || !pos) return fail("bad batch arguments");
    qdb_model *m = ss[0] ? ss[0]->m : nullptr;
    if (!m) return fail("null session or session's model has been freed");
    for (int b = 0; b < n; b++) {
        if (!ss[b] || ss[b]->m != m) return fail("row %d: sessions must share one model", b);
        if (pos[b] < 0) return fail("row %d: negative position", b);
    }
    if (set_dev(m) || ensure_rows(m, n, true)) return -1;
    std::vector<QdbRowKV> rk(n);
    for (int b = 0; b < n; b++) {
        if (prep_pos(ss[b], pos[b] + extra_steps)) return -1;
    }
    for (int b = 0; b < n; b++) rk[b] = QdbRowKV{ss[b]->kc, ss[b]->vc, ss[b]->cap, pos[b]};
    if (max_pos) {
        *max_pos = 0;
        for (int b = 0; b < n; b++) *max_pos = std::max(*max_pos, pos[b]);
    }
    CK(cudaMemcpyAsync(m->rs.rowkv, rk.data(), sizeof(QdbRowKV) * n, cudaMemcpyHostToDevice, m->st));
    CK(cudaStreamSynchronize(m->st));  // rk is a stack vector
    *mo = m;
    return 0;
}

static int batch_tail(qdb_model *m, int n, int *tok_dev, const int *step = nullptr) {
    RowScratch &r = m->rs;
    CK(qdb_launch_rmsnorm_rows(r.X, m->final_norm, r.XH, r.XL, n, m->cfg.hidden, m->cfg.eps, m->st));
    CK(qdb_launch_gemm_tc(m->embed, r.XH, r.XL, r.LOG, n, m->cfg.vocab, m->cfg.hidden, 0, 1, r.err, m->st));
    CK(qdb_launch_argmax_rows(r.LOG, n, m->cfg.vocab, m->mask_eos, tok_dev, m->st, step, r.amax));
    return 0;
}

static int ensure_tok(qdb_model *m, size_t count) {
    RowScratch &r = m->rs;
    if (count <= r.tok_cap) return 0;
    cudaFree(r.tok);
    r.tok = nullptr;
    r.tok_cap = 0;
    if (dev_alloc(&r.tok, count)) return -1;
    r.tok_cap = count;
    return 0;
}

// ------------------------------------------------------------------ persistent batched step
static constexpr int BSTEP_MAX_B = 64, BSTEP_MAX_SPLITS = 8;

// Utterance columns of the step's tiles: 16, 32 or 64.
static int bstep_cols(int n) { return n <= 16 ? 16 : (n <= 32 ? 32 : 64); }

// Batched decode runs as the captured launch-per-kernel graph by default. The
// persistent batched step (qdb_bstep.cu, up to 64 utterances) is selected with
// QWEN_ASR_B200_BATCH=persistent: it computes the same step, but is measured
// slower on this hardware (per-instruction tcgen05 MMA and commit costs at
// N = 2 x batch columns, split-K reduction traffic, shallow attention staging).
static bool bstep_fits(qdb_model *m, int n) {
    if (n < 1 || n > BSTEP_MAX_B) return false;
    int dev_smem = 0;
    cudaDeviceGetAttribute(&dev_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device);
    const int R = m->cfg.heads / m->cfg.kv_heads;
    return qdb_bstep_ring_stages(bstep_cols(n), R) >= 8 && qdb_bstep_smem(bstep_cols(n), R) + 2048 <= (size_t)dev_smem;
}

static bool bstep_usable(qdb_model *m, int n) {
    const char *v = getenv("QWEN_ASR_B200_BATCH");
    return v && !strcmp(v, "persistent") && bstep_fits(m, n);
}

static void free_bstep(BatchScratch &b) {
    cudaFree(b.x); cudaFree(b.qkv); cudaFree(b.gu); cudaFree(b.part); cudaFree(b.stats); cudaFree(b.best);
    cudaFree(b.cnt); cudaFree(b.done); cudaFree(b.err); cudaFree(b.prog); cudaFree(b.attn); cudaFree(b.acnt);
    cudaFree(b.wt);
    b = BatchScratch();
}

static int ensure_bstep(qdb_model *m) {
    BatchScratch &b = m->bs;
    if (b.wt) return 0;  // allocated last: everything else is in place
    free_bstep(b);
    const size_t h = m->cfg.hidden, I = m->cfg.intermediate, L = m->cfg.layers;
    const size_t qkvd = (size_t)m->qd + 2 * m->kvd;
    b.n_cnt = qdb_bstep_counters((int)L);
    if (dev_alloc(&b.x, h * BSTEP_MAX_B) || dev_alloc(&b.qkv, qkvd * BSTEP_MAX_B) ||
        dev_alloc(&b.gu, 2 * I * BSTEP_MAX_B) ||
        dev_alloc(&b.part, (size_t)BSTEP_MAX_B * m->cfg.heads * BSTEP_MAX_SPLITS * (2 + QDB_HD)) ||
        dev_alloc(&b.stats, (3 * L + 3) * 64) || dev_alloc(&b.best, 64) || dev_alloc(&b.cnt, (size_t)b.n_cnt) ||
        dev_alloc(&b.done, 1) || dev_alloc(&b.err, 4) || dev_alloc(&b.prog, (size_t)m->sms * 17) ||
        dev_alloc(&b.attn, (size_t)m->qd * BSTEP_MAX_B) || dev_alloc(&b.acnt, (size_t)BSTEP_MAX_B * m->cfg.kv_heads)) {
        std::string e = g_err;
        free_bstep(b);
        g_err = e;
        return -1;
    }
    CK(cudaMemset(b.gu, 0, 2 * I * BSTEP_MAX_B * 4));
    CK(cudaMemset(b.qkv, 0, qkvd * BSTEP_MAX_B * 4));
    CK(cudaMemset(b.stats, 0, (3 * L + 3) * 64 * 8));
    CK(cudaMemset(b.best, 0, 64 * 8));
    CK(cudaMemset(b.cnt, 0, (size_t)b.n_cnt * 4));
    CK(cudaMemset(b.done, 0, 4));
    CK(cudaMemset(b.err, 0, 16));
    CK(cudaMemset(b.prog, 0, (size_t)m->sms * 17 * 4));
    CK(cudaMemset(b.acnt, 0, (size_t)BSTEP_MAX_B * m->cfg.kv_heads * 4));
    // pre-tiled weights, in the order the step streams them
    size_t total = 0;
    const size_t per_layer = qdb_bstep_tiled_elems((int)qkvd, (int)h) + qdb_bstep_tiled_elems((int)h, m->qd) +
                             qdb_bstep_tiled_elems((int)(2 * I), (int)h) + qdb_bstep_tiled_elems((int)h, (int)I);
    total = per_layer * L + qdb_bstep_tiled_elems(m->cfg.vocab, (int)h);
    uint16_t *wt = nullptr;
    if (dev_alloc(&wt, total)) {
        std::string e = g_err;
        free_bstep(b);
        g_err = e;
        return -1;
    }
    uint16_t *o = wt;
    for (size_t l = 0; l < L; l++) {
        const QdbLayerW &lw = m->layers_host[l];
        CK(qdb_bstep_tile_weights(lw.qkv, (int)qkvd, (int)h, o, 0, m->st));
        o += qdb_bstep_tiled_elems((int)qkvd, (int)h);
        CK(qdb_bstep_tile_weights(lw.o, (int)h, m->qd, o, 0, m->st));
        o += qdb_bstep_tiled_elems((int)h, m->qd);
        CK(qdb_bstep_tile_weights(lw.gu, (int)(2 * I), (int)h, o, 0, m->st));
        o += qdb_bstep_tiled_elems((int)(2 * I), (int)h);
        CK(qdb_bstep_tile_weights(lw.down, (int)h, (int)I, o, 0, m->st));
        o += qdb_bstep_tiled_elems((int)h, (int)I);
    }
    CK(qdb_bstep_tile_weights(m->embed, m->cfg.vocab, (int)h, o, 1, m->st));
    CK(cudaStreamSynchronize(m->st));
    b.wt = wt;
    return 0;
}

// Key splits per (utterance, KV head): enough attention units to occupy the
// grid evenly (at least 32 keys per split).
static int bstep_splits(qdb_model *m, int n, int max_ctx) {
    const int base = n * m->cfg.kv_heads, G = m->sms;
    int best = 1;
    double best_eff = 0.0;
    for (int s = 1; s <= BSTEP_MAX_SPLITS; s++) {
        if (s > 1 && (max_ctx + s - 1) / s < 32) break;
        const int units = base * s;
        const double eff = (double)units / ((double)G * ((units + G - 1) / G));
        if (eff > best_eff + 0.05) {
            best_eff = eff;
            best = s;
        }
        if (eff >= 0.9) break;
    }
    return best;
}

// One launch of the persistent step over the n rows whose QdbRowKV entries are
// in rs.rowkv. tok_in / x_in: device tokens (slots step_base * n + b) or f32
// embeddings [n, h]; tok_out slots step_base * n + b.
static int launch_bstep(qdb_model *m, int n, int max_ctx, const int *tok_in, const float *x_in, int *tok_out,
                        float *logits, int step_base, int splits, unsigned long long *trace = nullptr,
                        unsigned long long *detail = nullptr) {
    if (launch_gate()) return -1;
    BatchScratch &b = m->bs;
    QdbBatchArgs a;
    memset(&a, 0, sizeof(a));
    a.d = m->d;
    a.B = n;
    a.Bp = bstep_cols(n);
    a.nsw = qdb_bstep_ring_stages(a.Bp, m->cfg.heads / m->cfg.kv_heads);

    a.splits = splits;
    a.layers = m->layers_dev;
    a.wt = b.wt;
    a.embed = m->embed;
    a.final_norm = m->final_norm;
    a.rope = m->rope;
    a.rope_cap = m->rope_cap;
    a.rows = m->rs.rowkv;
    a.tok_in = tok_in;
    a.x_in = x_in;
    a.tok_out = tok_out;
    a.logits_out = logits;
    a.mask_eos = m->mask_eos;
    a.step_base = step_base;
    a.x = b.x;
    a.qkv = b.qkv;
    a.gu = b.gu;
    a.part = b.part;
    a.attn = b.attn;
    a.acnt = b.acnt;
    a.stats = b.stats;
    a.best = b.best;
    a.cnt = b.cnt;
    a.n_cnt = b.n_cnt;
    a.done = b.done;
    if (++b.epoch == 0) b.epoch = 1;
    a.epoch = b.epoch;
    a.err = b.err;
    a.prog = b.prog;
    a.trace = trace;
    a.detail = detail;
    (void)max_ctx;
    CK(qdb_launch_bstep(&a, m->sms, m->st));
    return 0;
}

static int check_bstep_err(qdb_model *m) {
    int ev[4] = {0, 0, 0, 0};
    CK(cudaMemcpy(ev, m->bs.err, sizeof(ev), cudaMemcpyDeviceToHost));
    if (ev[0]) {
        // progress of the CTA that gave up, and the slowest / fastest of each word over all CTAs
        constexpr int PW = 17;
        std::vector<unsigned> pg((size_t)m->sms * PW);
        std::string prog;
        if (cudaMemcpy(pg.data(), m->bs.prog, pg.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess) {
            char buf[1024];
            const int c = (ev[2] >= 0 && ev[2] < m->sms) ? ev[2] : 0;
            int o = snprintf(buf, sizeof(buf), "; progress of CTA %d:", c);
            for (int w = 0; w < PW; w++) o += snprintf(buf + o, sizeof(buf) - o, " %x", pg[(size_t)c * PW + w]);
            o += snprintf(buf + o, sizeof(buf) - o, "; min/max:");
            for (int w = 0; w < 9 && o < (int)sizeof(buf) - 24; w++) {
                unsigned lo = ~0u, hi = 0;
                for (int k = 0; k < m->sms; k++) {
                    lo = std::min(lo, pg[(size_t)k * PW + w]);
                    hi = std::max(hi, pg[(size_t)k * PW + w]);
                }
                o += snprintf(buf + o, sizeof(buf) - o, " %u/%u", lo, hi);
            }
            prog = buf;
        }
        cudaMemset(m->bs.err, 0, sizeof(ev));
        cudaMemset(m->bs.prog, 0, pg.size() * 4);
        cudaDeviceSynchronize();
        return fail("device error code %d in the batched decode step (%s; check %d: %d %d%s)", ev[0],
                    ev[0] == 1   ? "a bounded wait ran out"
                    : ev[0] == 2 ? "invalid token or no argmax candidate"
                                 : "an access refused by a bounds check",
                    ev[1], ev[2], ev[3], prog.c_str());
    }
    return 0;
}

extern "C" int qdb_forward_batch(qdb_session *const *sessions, int n, const float *embeds, const int *pos,
                                 int *tokens_out, float *logits_out) {
    g_err.clear();
    qdb_model *m = nullptr;
    if (!embeds || !tokens_out) return fail("null argument");
    int maxp = 0;
    if (batch_setup(sessions, n, pos, 0, &m, &maxp) || ensure_tok(m, n)) return -1;
    CK(cudaMemcpyAsync(m->rs.X, embeds, (size_t)n * m->cfg.hidden * 4, cudaMemcpyHostToDevice, m->st));
    RowScratch &r = m->rs;
    if (bstep_usable(m, n)) {
        if (ensure_bstep(m) ||
            launch_bstep(m, n, maxp + 1, nullptr, r.X, r.tok, logits_out ? r.LOG : nullptr, 0,
                         bstep_splits(m, n, maxp + 1)))
            return -1;
        CK(cudaMemcpyAsync(tokens_out, r.tok, sizeof(int) * n, cudaMemcpyDeviceToHost, m->st));
        if (logits_out)
            CK(cudaMemcpyAsync(logits_out, r.LOG, sizeof(float) * (size_t)n * m->cfg.vocab, cudaMemcpyDeviceToHost,
                               m->st));
        CK(cudaStreamSynchronize(m->st));
        return check_bstep_err(m);
    }
    auto step = [&]() { return run_rows(m, n, nullptr, r.rowkv, 0, maxp + 1) || batch_tail(m, n, r.tok); };
    const int S = std::min(64, std::max(1, (maxp + 1 + 64 * QDB_AR_ITERS - 1) / (64 * QDB_AR_ITERS)));
    // the captured launches bake in the row count, the split count, every
    // scratch pointer, the RoPE table (reallocated when a session grows past
    // it) and the EOS mask
    auto graph_key = [&]() {
        return std::vector<const void *>{(const void *)(intptr_t)n, (const void *)(intptr_t)S,
                                         (const void *)(intptr_t)m->mask_eos, m->rope, r.X, r.XH, r.XL, r.QKV, r.Q,
                                         r.ATT, r.ACT, r.LOG, r.part, r.acnt, r.GU, r.tok, r.err, r.rowkv, r.amax};
    };
    const std::vector<const void *> key = graph_key();
    if (m->fb_exec && key == m->fb_key) {
        CK(cudaGraphLaunch(m->fb_exec, m->st));
    } else {
        // run directly (this sizes the scratch), then capture the same launch
        // sequence for the calls that follow
        if (step()) return -1;
        if (m->fb_exec) cudaGraphExecDestroy(m->fb_exec);
        m->fb_exec = nullptr;
        m->fb_key.clear();
        const std::vector<const void *> key2 = graph_key();
        cudaGraph_t graph = nullptr;
        if (cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const bool bad = step();
            if (cudaStreamEndCapture(m->st, &graph) == cudaSuccess && !bad && graph &&
                cudaGraphInstantiate(&m->fb_exec, graph, 0) == cudaSuccess)
                m->fb_key = key2;
            else
                m->fb_exec = nullptr;
            if (graph) cudaGraphDestroy(graph);
            if (!m->fb_exec) {  // a failed capture only means no graph: the step above already ran
                cudaGetLastError();
                g_err.clear();
            }
        }
    }
    CK(cudaMemcpyAsync(tokens_out, m->rs.tok, sizeof(int) * n, cudaMemcpyDeviceToHost, m->st));
    if (logits_out)
        CK(cudaMemcpyAsync(logits_out, m->rs.LOG, sizeof(float) * (size_t)n * m->cfg.vocab, cudaMemcpyDeviceToHost,
                           m->st));
    CK(cudaStreamSynchronize(m->st));
    return check_rows_err(m);
}

extern "C" int qdb_trace_batch_step(qdb_session *const *sessions, int n, const float *embeds, const int *pos,
                                    unsigned long long *trace_out, int max_words) {
    g_err.clear();
    qdb_model *m = nullptr;
    if (!embeds || !trace_out) return fail("null argument");
    int maxp = 0;
    if (batch_setup(sessions, n, pos, 0, &m, &maxp) || ensure_tok(m, n)) return -1;
    if (!bstep_fits(m, n)) return fail("the persistent batched step does not serve %d rows", n);
    const int ev = qdb_bstep_trace_events(m->cfg.layers);
    const size_t words = (size_t)m->sms * (ev + 512);  // phase stamps, then layer-1 detail stamps
    if ((size_t)max_words < words) return fail("trace buffer needs %zu words", words);
    unsigned long long *tr = nullptr;
    if (ensure_bstep(m) || dev_alloc(&tr, words)) return -1;
    int rc = 0;
    if (cudaMemsetAsync(tr, 0, words * 8, m->st) != cudaSuccess ||
        cudaMemcpyAsync(m->rs.X, embeds, (size_t)n * m->cfg.hidden * 4, cudaMemcpyHostToDevice, m->st) != cudaSuccess ||
        launch_bstep(m, n, maxp + 1, nullptr, m->rs.X, m->rs.tok, nullptr, 0, bstep_splits(m, n, maxp + 1), tr,
                     tr + (size_t)m->sms * ev) ||
        cudaMemcpyAsync(trace_out, tr, words * 8, cudaMemcpyDeviceToHost, m->st) != cudaSuccess ||
        cudaStreamSynchronize(m->st) != cudaSuccess)
        rc = -1;
    cudaFree(tr);
    if (rc) return g_err.empty() ? fail("batched trace step failed") : -1;
    return check_bstep_err(m) ? -1 : ev;
}

extern "C" int qdb_decode_greedy_batch(qdb_session *const *sessions, int n, const int *first_tokens, const int *pos,
                                       int n_steps, int *tokens_out) {
    g_err.clear();
    qdb_model *m = nullptr;
    if (!first_tokens || (n_steps > 0 && !tokens_out)) return fail("null argument");
    if (n_steps <= 0) return 0;
    int maxp = 0;
    if (batch_setup(sessions, n, pos, n_steps - 1, &m, &maxp) || ensure_tok(m, (size_t)n * (n_steps + 1))) return -1;
    for (int b = 0; b < n; b++)
        if (first_tokens[b] < 0 || first_tokens[b] >= m->cfg.vocab) return fail("row %d: token out of range", b);
    CK(cudaMemcpyAsync(m->rs.tok, first_tokens, sizeof(int) * n, cudaMemcpyHostToDevice, m->st));
    if (bstep_usable(m, n)) {
        if (ensure_bstep(m)) return -1;
        const int S = bstep_splits(m, n, maxp + n_steps);
        for (int i = 0; i < n_steps; i++)
            if (launch_bstep(m, n, maxp + 1 + i, m->rs.tok, nullptr, m->rs.tok + n, nullptr, i, S)) return -1;
        CK(cudaMemcpyAsync(tokens_out, m->rs.tok + n, sizeof(int) * (size_t)n * n_steps, cudaMemcpyDeviceToHost,
                           m->st));
        CK(cudaStreamSynchronize(m->st));
        return check_bstep_err(m);
    }
    // One step reads its tokens and position offset from the device step
    // counter, so the same launch sequence serves every step: step 0 runs
    // directly (it also sizes the scratch), the rest replay a CUDA graph of
    // one step (~11 launches per layer), which removes the launch gaps. The
    // attention split count is fixed for the call (sized for its last step).
    RowScratch &r = m->rs;
    const int ctx_last = maxp + n_steps;
    CK(cudaMemsetAsync(r.step, 0, sizeof(int), m->st));
    auto one_step = [&]() -> int {
        CK(qdb_launch_embed_rows(m->embed, r.tok, r.X, n, m->cfg.hidden, m->cfg.vocab, m->st, r.step));
        if (run_rows(m, n, nullptr, r.rowkv, 0, ctx_last, r.step) || batch_tail(m, n, r.tok + n, r.step))
            return -1;
        CK(qdb_launch_step_advance(r.step, m->st));
        return 0;
    };
    if (one_step()) return -1;
    if (n_steps > 1) {
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
        CK(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
        const int rc = one_step();
        const cudaError_t ce = cudaStreamEndCapture(m->st, &graph);
        if (rc || ce != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            return rc ? -1 : fail("decode step capture: %s", cudaGetErrorString(ce));
        }
        cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return fail("decode step graph: %s", cudaGetErrorString(e));
        for (int i = 1; i < n_steps && e == cudaSuccess; i++) e = cudaGraphLaunch(exec, m->st);
        cudaGraphExecDestroy(exec);
        if (e != cudaSuccess) return fail("decode step graph launch: %s", cudaGetErrorString(e));
    }
    CK(cudaMemcpyAsync(tokens_out, m->rs.tok + n, sizeof(int) * (size_t)n * n_steps, cudaMemcpyDeviceToHost, m->st));
    CK(cudaStreamSynchronize(m->st));
    return check_rows_err(m);
}

// ------------------------------------------------------------------ decode step without allocation
// Scratch of qdb_forward_noalloc: the persistent step's tagged inter-CTA
// vectors, followed by its argmax key, completion counter and error words.
// Sized for the largest decoder this library runs (the 1.7B shape needs about
// 52k words), 512 KiB in all; every GPU that loads the library holds it.
#define QDB_NOALLOC_TAG_WORDS 65536
static __device__ __align__(256) unsigned long long g_noalloc_scratch[QDB_NOALLOC_TAG_WORDS + 4];

static unsigned long long *g_noalloc_ptr[64];  // device address of the array, per device
static unsigned g_noalloc_epoch[64];           // next epoch for the array, per device

extern "C" int qdb_forward_noalloc(qdb_session *s, const float *embed_dev, int pos, int *token_dev) {
    g_err.clear();
    if (!s || !embed_dev || !token_dev) return fail("null argument");
    if (!s->m) return fail("session's model has been freed");
    qdb_model *m = s->m;
    if (m->device < 0 || m->device >= 64) return fail("device index %d out of range", m->device);
    if (pos < 0) return fail("negative position");
    // Nothing may grow here (growing allocates): the session and the RoPE
    // table must already cover pos.
    if (pos >= s->cap) return fail("position %d needs KV capacity %d (have %d); reserve it first", pos, pos + 1, s->cap);
    if (pos >= m->rope_cap) return fail("position %d beyond the RoPE table (%d)", pos, m->rope_cap);
    const size_t need = m->tags_len;
    if (need > QDB_NOALLOC_TAG_WORDS)
        return fail("model needs %zu scratch words, the no-allocation scratch holds %d", need, QDB_NOALLOC_TAG_WORDS);
    if (set_dev(m)) return -1;
    unsigned long long *base = g_noalloc_ptr[m->device];
    if (!base) {  // set-up, once per device, with that device current
        CK(cudaGetSymbolAddress((void **)&base, g_noalloc_scratch));
        g_noalloc_ptr[m->device] = base;
        g_noalloc_epoch[m->device] = 1;
        CK(cudaMemsetAsync(base, 0, sizeof(unsigned long long) * (QDB_NOALLOC_TAG_WORDS + 4), m->st));
    }
    const unsigned span = qdb_step_epochs(m->cfg.layers);
    unsigned &epoch = g_noalloc_epoch[m->device];
    if (epoch > 0xffffffffu - 2 * span) {
        CK(cudaMemsetAsync(base, 0, sizeof(unsigned long long) * QDB_NOALLOC_TAG_WORDS, m->st));
        epoch = 1;
    }
    unsigned long long *tail = base + QDB_NOALLOC_TAG_WORDS;  // best | done, err[4]
    // the argmax key, the completion counter and the error words start at zero
    CK(cudaMemsetAsync(tail, 0, 4 * sizeof(unsigned long long), m->st));

    if (launch_gate()) return -1;
    QdbStepArgs a = step_args(s, pos);
    const size_t n_x = m->cfg.hidden, n_qkv = m->qd + 2 * m->kvd, n_attn = m->qd, n_act = m->cfg.intermediate;
    a.tx = base;
    a.tqkv = a.tx + n_x;
    a.tattn = a.tqkv + n_qkv;
    a.tact = a.tattn + n_attn;
    a.tpart = a.tact + n_act;
    a.best = tail;
    a.done = reinterpret_cast<unsigned *>(tail + 1);
    a.err = reinterpret_cast<int *>(tail + 2);
    a.x_in = embed_dev;
    a.token_in = nullptr;
    a.token_out = token_dev;
    a.hidden_out = nullptr;
    a.logits_out = nullptr;
    a.epoch = epoch;
    CK(m->step_k->launch(a, m->grid, m->st));
    epoch += span;
    int ev[4] = {0, 0, 0, 0};
    CK(cudaMemcpyAsync(ev, a.err, sizeof(ev), cudaMemcpyDeviceToHost, m->st));
    CK(cudaStreamSynchronize(m->st));
    if (ev[0]) {
        // a bounded wait ran out: forget the array's contents (epochs restart)
        CK(cudaMemsetAsync(base, 0, sizeof(unsigned long long) * (QDB_NOALLOC_TAG_WORDS + 4), m->st));
        CK(cudaStreamSynchronize(m->st));
        epoch = 1;
        return fail("device error code %d in the no-allocation step (check %d: %d %d)", ev[0], ev[1], ev[2], ev[3]);
    }
    return 0;
}
