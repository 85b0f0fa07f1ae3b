// qdb_stream.cu - streaming scheduler for many concurrent streams of one
// model (the streaming mode's decoder side, stream_impl in qwen_asr.c).
//
// The reference runs one stream per context, one chunk at a time, one token
// per qwen_decoder_forward call. Here every stream's chunk k is processed in
// lockstep, so the device work of a chunk becomes two batched calls:
//   1. one row-batched prefill of every stream's prompt delta (the rows after
//      the longest unchanged prefix of its previous prompt; the KV cache is
//      rewound there, qwen_asr.c:1750-1770),
//   2. one device-resident greedy loop over all streams (first token from the
//      last prompt row, then the chunk's decode steps, qwen_asr.c:1775, :1821-1829).
// Everything else is host bookkeeping on token ids, restated from stream_impl:
//   prefix rollback (:1676-1690), prompt layout (:1692-1746), repeat-run
//   suppression (:1850-1884), raw history update (:1886-1906), text region
//   (:1908-1922), fixed frontier (:1924-1941), degeneration / stagnation
//   recovery (:1943-1992, stream_tail_repeat_blocks :1078-1111), commit with
//   overlap de-duplication (:1993-2054), periodic re-anchoring (:2057-2085,
//   stream_reanchor_text_state :1135-1182).
// Emitted pieces are token ids (the tokenizer is outside this library). The
// encoder output of each chunk is the caller's (it owns the window cache,
// :1506-1674, and clears it when a chunk reports a reset).
//
// Prefix comparison: the reference memcmp's f32 prompt rows. Token rows are
// compared here by token id and audio rows bytewise, which gives the same
// prefix unless two different token ids have bitwise-equal embedding rows or
// an audio row equals a token row bitwise.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "../../include/qwen_asr_b200.h"
#include "qdb_kernels.h"

namespace {

// reference constants (qwen_asr.c:1310-1319, qwen_asr.h:33-36)
constexpr int MAX_PREFIX_TOKENS = 150;
constexpr int MAX_REPEAT_TOKEN_RUN = 12;
constexpr int OVERLAP_MAX_TOKENS = 48;
constexpr int OVERLAP_MIN_TOKENS = 4;
constexpr int DEGEN_MAX_PERIOD = 6;
constexpr int DEGEN_MIN_REPEATS = 4;
constexpr int STALE_CHUNKS = 4;
constexpr int RESET_INTERVAL_CHUNKS = 45;
constexpr int RESET_CARRY_TOKENS = 24;
constexpr int TOKEN_ENDOFTEXT = 151643, TOKEN_IM_END = 151645, TOKEN_ASR_TEXT = 151704;
const int HEAD_DEFAULT[] = {151644, 8948, 198};
const int TAIL_DEFAULT[] = {151645, 198, 151644, 872, 198, 151669};
const int SUFFIX_DEFAULT[] = {151670, 151645, 198, 151644, 77091, 198};

// prompt rows: token id >= 0, audio row r as -(r + 1)
__global__ void prompt_rows_kernel(const uint16_t *__restrict__ embed, const int *__restrict__ desc,
                                   const float *__restrict__ audio, float *__restrict__ out, int h) {
    const int r = blockIdx.x, d = desc[r];
    float *o = out + (size_t)r * h;
    if (d >= 0) {
        const uint16_t *e = embed + (size_t)d * h;
        for (int i = threadIdx.x; i < h; i += blockDim.x) o[i] = __uint_as_float((uint32_t)e[i] << 16);
    } else {
        const float *a = audio + (size_t)(-d - 1) * h;
        for (int i = threadIdx.x; i < h; i += blockDim.x) o[i] = a[i];
    }
}

struct Stream {
    qdb_session *sess = nullptr;
    int chunk_idx = 0;
    std::vector<int> raw, stable, emitted;
    int stagnant = 0;
    // previous prefill prompt (prev_prefill_embeds): row descriptors and
    // the audio rows they index
    std::vector<int> prev_desc;
    std::vector<float> prev_audio;
    int prev_len = 0;
    long long prefill_total = 0, prefill_reused = 0, decoded = 0, chunks_done = 0;
    int last_reset = 0, last_emitted = 0, last_generated = 0;
    // per-chunk scratch
    std::vector<int> desc;
    int n_prefix_full = 0, reused = 0, prefill_len = 0, audio_rows = 0;
};

int tail_repeat_blocks(const int *t, int n, int max_period, int *out_period) {
    *out_period = 0;
    if (n < 2) return 1;
    int best = 1, best_p = 0;
    int cap = n / 2;
    if (max_period > 0 && cap > max_period) cap = max_period;
    for (int p = 1; p <= cap; p++) {
        int reps = 1;
        while ((reps + 1) * p <= n && memcmp(t + n - (reps + 1) * p, t + n - reps * p, sizeof(int) * p) == 0) reps++;
        if (reps > best) {
            best = reps;
            best_p = p;
        }
    }
    *out_period = best_p;
    return best;
}

}  // namespace

struct qdb_streams {
    qdb_model *m = nullptr;
    QdbModelInfo info{};
    qdb_stream_config cfg{};
    std::vector<int> head, prompt, tail, suffix, force;
    int asr_text = TOKEN_ASR_TEXT;
    std::vector<Stream> st;
    // device scratch, grown on demand
    int *d_desc = nullptr;
    float *d_audio = nullptr, *d_rows = nullptr;
    size_t desc_cap = 0, audio_cap = 0, rows_cap = 0;
    float *h_audio = nullptr;  // pinned staging of the chunk's uploaded audio rows
    size_t h_audio_cap = 0;
    std::vector<int> h_tokens;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};  // chunk start, prefill done, decode done
    float last_ms[2] = {0.f, 0.f};
    int last_rows = 0, last_active = 0;
};

namespace {

// Runs fn(j) for j in [0, n) on up to 16 host threads (the per-stream host
// work of a chunk: prefix comparison and the copies of audio rows, about a
// megabyte per stream, is independent across streams).
template <typename F>
void parallel_for(int n, F fn) {
    const int hw = (int)std::max(1u, std::thread::hardware_concurrency());
    const int T = std::min({16, hw, (n + 7) / 8});
    if (T <= 1) {
        for (int j = 0; j < n; j++) fn(j);
        return;
    }
    std::vector<std::thread> th;
    th.reserve(T);
    for (int t = 0; t < T; t++)
        th.emplace_back([&, t] {
            for (int j = t; j < n; j += T) fn(j);
        });
    for (auto &x : th) x.join();
}

template <typename T>
int grow_dev(T **p, size_t *cap, size_t need) {
    if (need <= *cap) return 0;
    size_t c = std::max<size_t>(need, *cap * 2);
    cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMalloc((void **)p, c * sizeof(T)) != cudaSuccess) return qdb_set_error("stream scheduler: out of device memory");
    *cap = c;
    return 0;
}

void reanchor(qdb_streams *S, Stream &s) {
    // stream_reanchor_text_state (qwen_asr.c:1135-1182)
    int carry = (int)s.emitted.size();
    if (carry > RESET_CARRY_TOKENS) carry = RESET_CARRY_TOKENS;
    const int lead = S->force.empty() ? 1 : 0;
    const int off = (int)s.emitted.size() - carry;
    s.raw.assign(lead, S->asr_text);
    s.raw.insert(s.raw.end(), s.emitted.begin() + off, s.emitted.end());
    s.stable.assign(s.emitted.begin() + off, s.emitted.end());
    s.prev_len = 0;
}

// Token bookkeeping of one finished chunk (qwen_asr.c:1850-2085).
void commit_chunk(qdb_streams *S, Stream &s, const int *gen, int n_gen_raw, bool is_final) {
    const qdb_stream_config &c = S->cfg;
    // chunk tokens: up to the first end token
    std::vector<int> chunk;
    int n_generated = 0;
    for (int i = 0; i < c.max_new_tokens; i++) {
        n_generated++;
        const int t = i < n_gen_raw ? gen[i] : TOKEN_IM_END;
        if (t == TOKEN_ENDOFTEXT || t == TOKEN_IM_END) break;
        chunk.push_back(t);
    }
    s.last_generated = n_generated;
    // repeat-run suppression
    int dropped = 0;
    if (!chunk.empty()) {
        int prev_tok = -1, prev_run = 0;
        if (s.n_prefix_full > 0) {
            prev_tok = s.raw[s.n_prefix_full - 1];
            prev_run = 1;
            for (int j = s.n_prefix_full - 2; j >= 0; j--) {
                if (s.raw[j] != prev_tok) break;
                prev_run++;
                if (prev_run >= MAX_REPEAT_TOKEN_RUN) break;
            }
        }
        size_t out = 0;
        for (size_t i = 0; i < chunk.size(); i++) {
            const int t = chunk[i];
            if (t == prev_tok) {
                if (++prev_run > MAX_REPEAT_TOKEN_RUN) {
                    dropped++;
                    continue;
                }
            } else {
                prev_tok = t;
                prev_run = 1;
            }
            chunk[out++] = t;
        }
        chunk.resize(out);
    }
    s.raw.resize(s.n_prefix_full);
    s.raw.insert(s.raw.end(), chunk.begin(), chunk.end());
    const int n_raw = (int)s.raw.size();
    // text region
    int text_start = 0;
    if (S->force.empty()) {
        int at = -1;
        for (int i = 0; i < n_raw; i++)
            if (s.raw[i] == S->asr_text) {
                at = i;
                break;
            }
        text_start = at >= 0 ? at + 1 : 0;
    }
    text_start = std::min(std::max(text_start, 0), n_raw);
    const int n_text = n_raw - text_start;
    int cand = 0;
    if (is_final) {
        cand = n_text;
    } else if (s.chunk_idx >= c.unfixed_chunks) {
        cand = n_text - c.rollback;
        if (cand <= 0 && n_text > 0) cand = n_text - 1;
        if (cand < 0) cand = 0;
    }
    const int *cand_tok = s.raw.data() + text_start;
    int period = 0;
    const int reps = tail_repeat_blocks(cand_tok, cand, DEGEN_MAX_PERIOD, &period);
    const int advance = cand - (int)s.stable.size();
    if (!is_final && n_generated >= c.max_new_tokens && advance <= 1)
        s.stagnant++;
    else
        s.stagnant = 0;
    bool recovery = (period > 0 && reps >= DEGEN_MIN_REPEATS) || s.stagnant >= STALE_CHUNKS || dropped >= 8;
    s.last_reset = 0;
    s.last_emitted = 0;
    if (recovery) {
        reanchor(S, s);
        s.stagnant = 0;
        s.last_reset = 1;
        return;
    }
    int lcp = 0;
    const int n_stable = (int)s.stable.size();
    while (lcp < n_stable && lcp < cand && s.stable[lcp] == cand_tok[lcp]) lcp++;
    s.stable.resize(std::max(n_stable, cand));
    for (int i = lcp; i < cand; i++) s.stable[i] = cand_tok[i];
    int emit_start = lcp;
    const int n_emitted = (int)s.emitted.size();
    if (emit_start < cand && n_emitted > 0) {
        int max_ov = std::min(cand - emit_start, n_emitted);
        if (max_ov > OVERLAP_MAX_TOKENS) max_ov = OVERLAP_MAX_TOKENS;
        for (int k = max_ov; k >= OVERLAP_MIN_TOKENS; k--)
            if (memcmp(s.emitted.data() + (n_emitted - k), cand_tok + emit_start, sizeof(int) * k) == 0) {
                emit_start += k;
                break;
            }
    }
    for (int i = emit_start; i < cand; i++) s.emitted.push_back(s.stable[i]);
    s.last_emitted = std::max(0, cand - emit_start);
    s.stable.resize(cand);
    const bool periodic = !is_final && c.past_text && s.chunk_idx >= c.unfixed_chunks &&
                          (s.chunk_idx + 1) % RESET_INTERVAL_CHUNKS == 0;
    if (periodic) {
        reanchor(S, s);
        s.last_reset = 2;
    }
}

}  // namespace

extern "C" qdb_streams *qdb_streams_create(qdb_model *m, int n_streams, const qdb_stream_config *cfg) {
    if (!m || n_streams <= 0) {
        qdb_set_error("qdb_streams_create: null model or no streams");
        return nullptr;
    }
    qdb_streams *S = new qdb_streams();
    S->m = m;
    if (qdb_model_internals(m, &S->info)) {
        delete S;
        return nullptr;
    }
    qdb_stream_config c{};
    c.max_new_tokens = 32;
    c.rollback = 5;
    c.unfixed_chunks = 2;
    if (cfg) c = *cfg;
    if (c.max_new_tokens <= 0) c.max_new_tokens = 32;
    if (c.rollback < 0 || c.unfixed_chunks < 0) {
        delete S;
        qdb_set_error("qdb_streams_create: negative rollback or unfixed_chunks");
        return nullptr;
    }
    auto take = [](const int *p, int n, const int *def, int ndef) {
        return p ? std::vector<int>(p, p + std::max(n, 0)) : std::vector<int>(def, def + ndef);
    };
    S->head = take(c.head_tokens, c.n_head_tokens, HEAD_DEFAULT, 3);
    S->tail = take(c.tail_tokens, c.n_tail_tokens, TAIL_DEFAULT, 6);
    S->suffix = take(c.suffix_tokens, c.n_suffix_tokens, SUFFIX_DEFAULT, 6);
    S->prompt = take(c.prompt_tokens, c.n_prompt_tokens, nullptr, 0);
    S->force = take(c.force_tokens, c.n_force_tokens, nullptr, 0);
    if (c.asr_text_token > 0) S->asr_text = c.asr_text_token;
    c.head_tokens = c.tail_tokens = c.suffix_tokens = c.prompt_tokens = c.force_tokens = nullptr;
    S->cfg = c;
    if (S->suffix.empty() && S->force.empty()) {
        delete S;
        qdb_set_error("qdb_streams_create: the prompt must end in a token row (suffix or forced tokens)");
        return nullptr;
    }
    for (const auto *v : {&S->head, &S->tail, &S->suffix, &S->prompt, &S->force})
        for (int t : *v)
            if (t < 0 || t >= S->info.vocab) {
                delete S;
                qdb_set_error("qdb_streams_create: prompt token out of the model's vocabulary");
                return nullptr;
            }
    S->st.resize(n_streams);
    for (auto &e : S->ev)
        if (cudaEventCreate(&e) != cudaSuccess) {
            qdb_streams_free(S);
            qdb_set_error("qdb_streams_create: cudaEventCreate failed");
            return nullptr;
        }
    for (auto &s : S->st) {
        s.sess = qdb_session_create(m, 512);
        if (!s.sess) {
            qdb_streams_free(S);
            return nullptr;
        }
    }
    return S;
}

extern "C" void qdb_streams_free(qdb_streams *S) {
    if (!S) return;
    for (auto &s : S->st)
        if (s.sess) qdb_session_free(s.sess);
    for (auto &e : S->ev)
        if (e) cudaEventDestroy(e);
    cudaFree(S->d_desc);
    cudaFree(S->d_audio);
    cudaFree(S->d_rows);
    cudaFreeHost(S->h_audio);
    delete S;
}

extern "C" int qdb_streams_chunk(qdb_streams *S, const float *const *audio, const int *audio_len,
                                 const int *is_final, int *n_emitted, int *reset) {
    if (!S || !audio || !audio_len || !is_final) return qdb_set_error("qdb_streams_chunk: null argument");
    const int n = (int)S->st.size(), h = S->info.hidden;
    const qdb_stream_config &c = S->cfg;
    if (cudaSetDevice(S->info.device) != cudaSuccess) return qdb_set_error("qdb_streams_chunk: cudaSetDevice failed");
    // ---- prompts (host, serial: small integer work and validation)
    std::vector<int> act;  // streams with audio this chunk
    for (int i = 0; i < n; i++) {
        Stream &s = S->st[i];
        if (n_emitted) n_emitted[i] = 0;
        if (reset) reset[i] = 0;
        if (audio_len[i] < 0) continue;  // not part of this call
        if (audio_len[i] == 0) {  // no encoder output: the chunk is skipped (qwen_asr.c:1649-1654)
            s.chunk_idx++;
            continue;
        }
        if (!audio[i]) return qdb_set_error("qdb_streams_chunk: null audio rows");
        act.push_back(i);
        // prefix rollback (qwen_asr.c:1676-1690)
        int n_full = 0, n_pref = 0, off = 0;
        const int n_raw = (int)s.raw.size();
        if (c.past_text && s.chunk_idx >= c.unfixed_chunks && n_raw > 0) {
            n_full = std::max(0, n_raw - c.rollback);
            n_pref = std::min(n_full, MAX_PREFIX_TOKENS);
            off = n_full - n_pref;
        }
        s.n_prefix_full = n_full;
        // [head] [prompt] [tail] [audio] [suffix] [force] [prefix tokens]
        s.desc.clear();
        for (const auto *v : {&S->head, &S->prompt, &S->tail}) s.desc.insert(s.desc.end(), v->begin(), v->end());
        for (int r = 0; r < audio_len[i]; r++) s.desc.push_back(-(r + 1));
        s.desc.insert(s.desc.end(), S->suffix.begin(), S->suffix.end());
        s.desc.insert(s.desc.end(), S->force.begin(), S->force.end());
        s.desc.insert(s.desc.end(), s.raw.begin() + off, s.raw.begin() + off + n_pref);
        for (int k = off; k < off + n_pref; k++)
            if (s.raw[k] < 0 || s.raw[k] >= S->info.vocab) return qdb_set_error("qdb_streams_chunk: token out of range");
        s.prefill_len = (int)s.desc.size() - 1;
        s.audio_rows = audio_len[i];
    }
    // ---- longest unchanged prefix of the previous prefill (qwen_asr.c:1750-1762), per stream in parallel
    parallel_for((int)act.size(), [&](int j) {
        Stream &s = S->st[act[j]];
        int reused = 0;
        if (s.prev_len > 0) {
            const int cmp = std::min(s.prefill_len, s.prev_len);
            const float *a_new = audio[act[j]];
            while (reused < cmp) {
                const int dn = s.desc[reused], dp = s.prev_desc[reused];
                bool same;
                if (dn >= 0 || dp >= 0)
                    same = dn == dp;
                else
                    same = memcmp(a_new + (size_t)(-dn - 1) * h, s.prev_audio.data() + (size_t)(-dp - 1) * h,
                                  sizeof(float) * h) == 0;
                if (!same) break;
                reused++;
            }
        }
        s.reused = reused;
    });
    // ---- deltas: KV capacity, row descriptors, staging offsets (serial)
    std::vector<qdb_session *> pf_sess;
    std::vector<int> pf_len, pf_start, all_desc;
    std::vector<size_t> stage_off(act.size(), 0);
    size_t up_rows = 0;
    for (size_t j = 0; j < act.size(); j++) {
        Stream &s = S->st[act[j]];
        if (qdb_session_reserve(s.sess, s.prefill_len + c.max_new_tokens + 1)) return -1;
        stage_off[j] = up_rows;
        if (s.prefill_len > s.reused) {
            pf_sess.push_back(s.sess);
            pf_len.push_back(s.prefill_len - s.reused);
            pf_start.push_back(s.reused);
            for (int r = s.reused; r < s.prefill_len; r++) {
                const int d = s.desc[r];
                all_desc.push_back(d >= 0 ? d : -(int)(++up_rows));  // staged audio row up_rows - 1
            }
        }
        s.prefill_total += s.prefill_len;
        s.prefill_reused += s.reused;
    }
    S->last_ms[0] = S->last_ms[1] = 0.f;
    S->last_rows = (int)all_desc.size();
    S->last_active = (int)act.size();
    if (act.empty()) return 0;
    cudaStream_t st = S->info.stream;
    cudaEventRecord(S->ev[0], st);
    // ---- stage the delta rows' audio, build the rows on the device, prefill
    if (!pf_sess.empty()) {
        // the previous chunk's uploads from h_audio are complete (its greedy
        // loop returned tokens to the host); this only catches stray work
        if (cudaStreamSynchronize(st) != cudaSuccess) return qdb_set_error("qdb_streams_chunk: stream error");
        if (up_rows * h > S->h_audio_cap) {
            const size_t cap = std::max(up_rows * h, S->h_audio_cap * 2);
            cudaFreeHost(S->h_audio);
            S->h_audio = nullptr;
            S->h_audio_cap = 0;
            if (cudaMallocHost((void **)&S->h_audio, cap * sizeof(float)) != cudaSuccess)
                return qdb_set_error("qdb_streams_chunk: out of pinned host memory");
            S->h_audio_cap = cap;
        }
        parallel_for((int)act.size(), [&](int j) {
            const Stream &s = S->st[act[j]];
            size_t k = stage_off[j];
            for (int r = s.reused; r < s.prefill_len; r++)
                if (s.desc[r] < 0)
                    memcpy(S->h_audio + (k++) * h, audio[act[j]] + (size_t)(-s.desc[r] - 1) * h, sizeof(float) * h);
        });
        if (grow_dev(&S->d_desc, &S->desc_cap, all_desc.size()) ||
            grow_dev(&S->d_audio, &S->audio_cap, std::max<size_t>(up_rows * h, 1)) ||
            grow_dev(&S->d_rows, &S->rows_cap, all_desc.size() * h))
            return -1;
        if (cudaMemcpyAsync(S->d_desc, all_desc.data(), sizeof(int) * all_desc.size(), cudaMemcpyHostToDevice, st) !=
                cudaSuccess ||
            (up_rows && cudaMemcpyAsync(S->d_audio, S->h_audio, sizeof(float) * up_rows * h, cudaMemcpyHostToDevice,
                                        st) != cudaSuccess))
            return qdb_set_error("qdb_streams_chunk: upload failed");
        prompt_rows_kernel<<<(unsigned)all_desc.size(), 256, 0, st>>>(S->info.embed, S->d_desc, S->d_audio, S->d_rows, h);
        if (cudaGetLastError() != cudaSuccess) return qdb_set_error("qdb_streams_chunk: prompt rows launch failed");
        if (qdb_prefill_batch_device(pf_sess.data(), (int)pf_sess.size(), S->d_rows, pf_len.data(), pf_start.data()))
            return -1;
    }
    cudaEventRecord(S->ev[1], st);
    // ---- first token + decode steps of every active stream in one greedy loop
    const int na = (int)act.size(), steps = c.max_new_tokens;
    std::vector<qdb_session *> ds(na);
    std::vector<int> first(na), pos(na);
    for (int j = 0; j < na; j++) {
        Stream &s = S->st[act[j]];
        ds[j] = s.sess;
        first[j] = s.desc[s.prefill_len];  // the last prompt row is a token row
        pos[j] = s.prefill_len;
    }
    S->h_tokens.resize((size_t)na * steps);
    // Keep this prompt for the next chunk's prefix comparison: host copies of
    // the rows (hundreds of MB per call at 256 streams) that depend only on
    // this call's inputs, made on a host thread while the GPU runs the greedy
    // loop (nothing reads prev_* until the next call).
    std::thread saver([&] {
        parallel_for(na, [&](int j) {
            Stream &s = S->st[act[j]];
            s.prev_desc.assign(s.desc.begin(), s.desc.begin() + s.prefill_len);
            s.prev_audio.assign(audio[act[j]], audio[act[j]] + (size_t)s.audio_rows * h);
            s.prev_len = s.prefill_len;
        });
    });
    const int grc = qdb_decode_greedy_batch(ds.data(), na, first.data(), pos.data(), steps, S->h_tokens.data());
    saver.join();
    if (grc) return -1;
    cudaEventRecord(S->ev[2], st);
    if (cudaEventSynchronize(S->ev[2]) == cudaSuccess) {
        cudaEventElapsedTime(&S->last_ms[0], S->ev[0], S->ev[1]);
        cudaEventElapsedTime(&S->last_ms[1], S->ev[1], S->ev[2]);
    }
    // ---- bookkeeping
    parallel_for(na, [&](int j) {
        const int i = act[j];
        Stream &s = S->st[i];
        std::vector<int> gen(steps);
        for (int t = 0; t < steps; t++) gen[t] = S->h_tokens[(size_t)t * na + j];
        commit_chunk(S, s, gen.data(), steps, is_final[i] != 0);
        s.decoded += s.last_generated;
        s.chunks_done++;
        if (n_emitted) n_emitted[i] = s.last_emitted;
        if (reset) reset[i] = s.last_reset;
        s.chunk_idx++;
    });
    return 0;
}

extern "C" int qdb_streams_tokens(const qdb_streams *S, int stream, int which, int *buf, int cap) {
    if (!S || stream < 0 || stream >= (int)S->st.size()) return qdb_set_error("qdb_streams_tokens: bad stream");
    const Stream &s = S->st[stream];
    const std::vector<int> *v = which == 0 ? &s.emitted : which == 1 ? &s.raw : which == 2 ? &s.stable : nullptr;
    if (!v) return qdb_set_error("qdb_streams_tokens: which must be 0 (emitted), 1 (raw) or 2 (stable)");
    if (buf) memcpy(buf, v->data(), sizeof(int) * std::min<size_t>(v->size(), (size_t)std::max(cap, 0)));
    return (int)v->size();
}

extern "C" int qdb_streams_stats(const qdb_streams *S, int stream, long long *out) {
    if (!S || !out || stream < 0 || stream >= (int)S->st.size()) return qdb_set_error("qdb_streams_stats: bad stream");
    const Stream &s = S->st[stream];
    out[0] = s.chunk_idx;
    out[1] = s.chunks_done;
    out[2] = s.prefill_total;
    out[3] = s.prefill_reused;
    out[4] = s.decoded;
    out[5] = s.last_generated;
    out[6] = s.reused;
    out[7] = s.prefill_len;
    return 0;
}

extern "C" int qdb_streams_reset(qdb_streams *S, int stream) {
    if (!S || stream < 0 || stream >= (int)S->st.size()) return qdb_set_error("qdb_streams_reset: bad stream");
    Stream &s = S->st[stream];
    qdb_session *keep = s.sess;
    s = Stream();
    s.sess = keep;
    return 0;
}

extern "C" int qdb_streams_last_chunk(const qdb_streams *S, float *ms, int *counts) {
    if (!S) return qdb_set_error("qdb_streams_last_chunk: null scheduler");
    if (ms) {
        ms[0] = S->last_ms[0];
        ms[1] = S->last_ms[1];
    }
    if (counts) {
        counts[0] = S->last_active;
        counts[1] = S->last_rows;
    }
    return 0;
}

// Launcher for the prompt-row builder (qdb_build_prompt_device, qdb_runtime.cu).
cudaError_t qdb_launch_prompt_rows(const uint16_t *embed, const int *desc_dev, const float *audio_dev, float *out_dev,
                                   int n_rows, int hidden, cudaStream_t st) {
    if (n_rows <= 0) return cudaSuccess;
    prompt_rows_kernel<<<n_rows, 256, 0, st>>>(embed, desc_dev, audio_dev, out_dev, hidden);
    return cudaGetLastError();
}
