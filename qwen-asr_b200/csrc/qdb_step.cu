// qdb_step.cu - persistent single-utterance decode step (batch 1).
//
// One cooperative launch runs one decode position end to end: 28 layers, the
// tied lm_head and the greedy argmax (qwen_decoder_forward,
// qwen_asr_decoder.c:388-476). One CTA per SM, two roles:
//
//  * producer warp: streams this CTA's slice of EVERY weight matrix of the
//    step (layer by layer, then the lm_head rows) into a ring of shared-memory
//    stages with cp.async.bulk + mbarrier transaction counts. It never waits
//    for activations, so weight traffic runs ahead across phase boundaries
//    and the whole step is one continuous HBM stream.
//  * 8 consumer warps: per layer
//      A  input RMSNorm (each CTA, from the full residual) -> QKV rows
//      B  per-head QK RMSNorm + NeoX RoPE + fp16 KV append + split-K
//         attention (one unit per (KV head, key range) CTA; split 0 merges)
//      C  O-proj rows + residual
//      D  post-attention RMSNorm -> gate/up row pairs + SwiGLU
//      E  down rows + residual
//    then F: final RMSNorm, lm_head rows, (value, lowest index) argmax.
//
// Inter-CTA data are "tagged" 64-bit words: high 32 bits = epoch of the
// phase that wrote it, low 32 bits = the f32 value. One 64-bit store is
// single-copy atomic, so a reader polls the data itself until the epoch
// matches: no grid barrier, no fence, one L2 round trip per dependency, and
// attention units wait only for the q/k/v rows of their own KV head.
//
// Every wait is bounded (about one second of SM clock). A wait that runs out
// records an error code, raises a CTA-local abort flag and returns; all
// consumer warps still pass every named barrier, the producer stops issuing
// and waits (bounded) for its copies in flight, and the kernel returns.
#include "qdb_common.cuh"
#include "qdb_kernels.h"

// Build constants (qdb_step_w7.cu includes this file with its own).
#ifndef QDB_NCW
#define QDB_NCW 6
#endif
#ifndef QDB_STAGE_BYTES
#define QDB_STAGE_BYTES 16384
#endif
#ifndef QDB_STEP_ENTRY
#define QDB_STEP_ENTRY qdb_step_kernel_w6
#define QDB_STEP_NAME "w6s16"
#define QDB_STEP_COMMON 1  // this build also defines the variant-independent helpers
#endif

namespace {

constexpr int NCW = QDB_NCW;              // consumer warps
constexpr int NCT = NCW * 32;             // consumer threads
constexpr int NTHREADS = NCT + 32;        // + producer warp
#ifndef QDB_STAGES_PER_WARP
#define QDB_STAGES_PER_WARP 2
#endif
constexpr int STAGE_BYTES = QDB_STAGE_BYTES;
// Ring stages are owned by warps: item `it` goes to warp it % NCW and stage
// it % NSTAGE with NSTAGE a multiple of NCW, so a stage is only ever reused
// by the warp that consumed its previous item. (Otherwise a fast warp could
// wait on a stage two mbarrier phases ahead, which a parity wait cannot tell
// from "complete".)
constexpr int NSTAGE = NCW * QDB_STAGES_PER_WARP;
constexpr int OWN_ROWS = 64;              // residual rows one CTA may own
constexpr int MAX_LAYERS = 32;             // layer table kept in shared memory
constexpr int ATT_KEYS = 8;               // keys per warp iteration
constexpr int POLL = (6144 + NCT - 1) / NCT;  // tagged words per consumer thread per vector load

static_assert(NSTAGE % NCW == 0, "a ring stage must belong to exactly one consumer warp");

typedef unsigned long long u64;

struct Ctl {
    volatile int *abort;  // CTA-local
    int *err;             // global
};

__device__ __forceinline__ void st_tag(u64 *p, float v, unsigned ep) {
    const u64 w = ((u64)ep << 32) | (u64)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ u64 ld_tag(const u64 *p) {
    u64 w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ unsigned tag_ep(u64 w) { return (unsigned)(w >> 32); }
__device__ __forceinline__ float tag_val(u64 w) { return __uint_as_float((unsigned)w); }

__device__ __forceinline__ bool timed_out(long long t0) { return clock64() - t0 > qdb_wait_limit_c; }
// Drain waits (the producer's own copies in flight) keep the fixed bound.
__device__ __forceinline__ bool drain_timed_out(long long t0) { return clock64() - t0 > QDB_SPIN_LIMIT_CYCLES; }

// A wait ran out: raise the CTA abort flag and record the first failure with
// its location (err[1] = wait site, err[2] = CTA, err[3] = warp).
__device__ __forceinline__ void abort_now(const Ctl &c, int site = 0) {
    *c.abort = 1;
    if (c.err && atomicCAS(c.err, 0, QDB_ERR_BARRIER_TIMEOUT) == 0) {
        c.err[1] = site;
        c.err[2] = blockIdx.x;
        c.err[3] = threadIdx.x >> 5;
    }
}

// Abort flag as one decision for the whole warp (lane 0's view), so no warp
// ever splits between a collective and an early exit.
__device__ __forceinline__ bool warp_aborted(const Ctl &c) {
    int v = 0;
    if ((threadIdx.x & 31) == 0) v = *c.abort;
    return __shfl_sync(0xffffffffu, v, 0) != 0;
}

// Checks the CTA flag and, every so often, the global error word (so one
// CTA's failure stops the others quickly).
__device__ __forceinline__ bool should_stop(const Ctl &c, int iter) {
    if (*c.abort) return true;
    if ((iter & 255) == 255 && *(volatile int *)c.err) {
        *c.abort = 1;
        return true;
    }
    return false;
}

__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }

// ---------------------------------------------------------------- mbarriers
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(u64 *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(u64 *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(u64 *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(u64 *bar, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait by ONE thread (the producer); `check` = honour the abort flag
// and the run-time wait limit (a drain passes false: it ignores the abort flag
// and waits up to the fixed bound).
__device__ bool mbar_wait(u64 *bar, unsigned parity, const Ctl &c, bool check, int site) {
    const long long t0 = clock64();
    for (int it = 0;; it++) {
        if (mbar_try(bar, parity)) return true;
        if (check && should_stop(c, it)) return false;
        if (check ? timed_out(t0) : drain_timed_out(t0)) {
            abort_now(c, site);
            return false;
        }
    }
}

// Bounded wait by a whole warp: every lane observes the phase completion
// (so the bulk-copied bytes are visible to it) and the result is uniform.
__device__ bool mbar_wait_warp(u64 *bar, unsigned parity, const Ctl &c, int site) {
    const long long t0 = clock64();
    for (int it = 0;; it++) {
        const bool done = mbar_try(bar, parity);
        if (__all_sync(0xffffffffu, done)) return true;
        int stop = 0;
        if ((threadIdx.x & 31) == 0) {
            stop = should_stop(c, it) ? 1 : 0;
            if (!stop && timed_out(t0)) {
                abort_now(c, site);
                stop = 1;
            }
        }
        if (__shfl_sync(0xffffffffu, stop, 0)) return false;
    }
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, u64 *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

#ifndef QDB_W_EVICT_FIRST
#define QDB_W_EVICT_FIRST 1  // weights stream through L2 with an evict-first policy
#endif
// Same copy with an L2 cache policy (createpolicy) on the global reads.
__device__ __forceinline__ void bulk_g2s_pol(void *dst, const void *src, unsigned bytes, u64 *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}


// Asynchronous 16-byte global -> shared copies (no registers held while the
// thread goes on polling); completed with cp_async_wait().
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Consumer threads start copying n floats (n % 4 == 0, 16-byte aligned) to smem.
__device__ __forceinline__ void prefetch_f32(float *dst, const float *src, int n) {
    for (int i = threadIdx.x * 4; i < n; i += NCT * 4) cp_async16(dst + i, src + i);
    cp_async_commit();
}

// ---------------------------------------------------------------- schedule
// A phase's matrix slice for CTA `c` of `G`: rows [r0, r1) of a [R, K] matrix,
// processed in items of `ipr` rows (an item fits one ring stage).
struct Slice {
    const uint16_t *w;
    int r0, r1, K, ipr;
    __device__ int items() const { return r1 > r0 ? (r1 - r0 + ipr - 1) / ipr : 0; }
};

__device__ __forceinline__ Slice make_slice(const uint16_t *w, int R, int K, int c, int G, bool pairs) {
    Slice s;
    s.w = w;
    s.K = K;
    const int units = pairs ? R / 2 : R;
    const int u0 = (int)((long long)units * c / G), u1 = (int)((long long)units * (c + 1) / G);
    s.r0 = pairs ? 2 * u0 : u0;
    s.r1 = pairs ? 2 * u1 : u1;
    int ipr = STAGE_BYTES / (K * 2);
    if (ipr > 32) ipr = 32;  // one output row per lane
    if (pairs) ipr &= ~1;
    s.ipr = ipr < 1 ? 1 : ipr;
    return s;
}

// Phase p (0..3 = QKV, O, GU, DOWN) of a layer, or the lm_head (p = 4).
__device__ __forceinline__ Slice phase_slice(const QdbStepArgs &a, const QdbLayerW *layers, int layer, int p) {
    const QdbDims &d = a.d;
    const int qd = d.Hq * QDB_HD, kvd = d.Hkv * QDB_HD;
    const int c = blockIdx.x, G = gridDim.x;
    if (p == 4) return make_slice(a.embed, d.V, d.h, c, G, false);
    const QdbLayerW &lw = layers[layer];
    switch (p) {
        case 0: return make_slice(lw.qkv, qd + 2 * kvd, d.h, c, G, false);
        case 1: return make_slice(lw.o, d.h, qd, c, G, false);
        case 2: return make_slice(lw.gu, 2 * d.I, d.h, c, G, true);
        default: return make_slice(lw.down, d.h, d.I, c, G, false);
    }
}

// ---------------------------------------------------------------- producer
// Walks the step's weight schedule: layers 0..L-1 phases 0..3, then the
// lm_head (layer L, phase 4), one item (<= ipr rows) at a time.
struct Cursor {
    int layer, p, r;
    Slice s;
    bool done;
};

__device__ __forceinline__ void cursor_settle(const QdbStepArgs &a, const QdbLayerW *layers, Cursor &q) {
    while (!q.done && q.r >= q.s.r1) {
        if (q.layer == a.d.L) {
            q.done = true;
            break;
        }
        if (++q.p == 4) {
            q.layer++;
            q.p = q.layer < a.d.L ? 0 : 4;
        }
        q.s = phase_slice(a, layers, q.layer, q.p);
        q.r = q.s.r0;
    }
}

__device__ __forceinline__ void cursor_init(const QdbStepArgs &a, const QdbLayerW *layers, Cursor &q) {
    q.layer = 0;
    q.p = 0;
    q.done = false;
    q.s = phase_slice(a, layers, 0, 0);
    q.r = q.s.r0;
    cursor_settle(a, layers, q);
}

__device__ __forceinline__ void cursor_next(const QdbStepArgs &a, const QdbLayerW *layers, Cursor &q) {
    q.r += q.s.ipr;
    cursor_settle(a, layers, q);
}

__device__ __noinline__ void producer(const QdbStepArgs &a, const QdbLayerW *layers, unsigned char *ring, u64 *full,
                                      u64 *empty, const Ctl &c) {
    if ((threadIdx.x & 31) != 0) return;
    uint64_t pol_w = 0;
    if (QDB_W_EVICT_FIRST) asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_w));
    Cursor ld;
    cursor_init(a, layers, ld);
    unsigned it = 0;
    bool ok = true;
    for (; !ld.done && ok; cursor_next(a, layers, ld), it++) {
        const int nr = min(ld.s.ipr, ld.s.r1 - ld.r);
        const unsigned st = it % NSTAGE;
        if (it >= NSTAGE && !mbar_wait(&empty[st], ((it / NSTAGE) - 1) & 1, c, true, 1)) {
            ok = false;
            break;
        }
        const unsigned bytes = (unsigned)(nr * ld.s.K * 2);
        const uint16_t *src = ld.s.w + (size_t)ld.r * ld.s.K;
        const bool in_w = (src >= a.w_lo && src + (size_t)bytes / 2 <= a.w_hi);
        const bool in_e = (src >= a.embed && src + (size_t)bytes / 2 <= a.embed + (size_t)a.d.V * a.d.h);
        if (!check_or_record(((uintptr_t)src & 15) == 0 && (bytes & 15) == 0 && bytes <= STAGE_BYTES && bytes > 0 &&
                                 (in_w || in_e),
                             a.err, 1, (long long)ld.r, (long long)bytes)) {
            *c.abort = 1;
            ok = false;
            break;
        }
        mbar_expect_tx(&full[st], bytes);
        if (QDB_W_EVICT_FIRST)
            // each weight byte is read once per step: keep it from evicting the
            // KV cache and the small per-layer vectors the latency chain reads
            bulk_g2s_pol(ring + (size_t)st * STAGE_BYTES, src, bytes, &full[st], pol_w);
        else
            bulk_g2s(ring + (size_t)st * STAGE_BYTES, src, bytes, &full[st]);
    }
    if (!ok) {
        // Drain: wait (bounded, ignoring the abort flag) for the copies in
        // flight, i.e. the latest item issued into each stage.
        for (unsigned k = 0; k < NSTAGE && k < it; k++) {
            const unsigned i = it - 1 - k;
            mbar_wait(&full[i % NSTAGE], (i / NSTAGE) & 1, c, false, 2);
        }
    }
}

// ---------------------------------------------------------------- consumer helpers
// Fills dst[0..n) from tagged words src expecting epoch ep (n <= POLL*NCT).
// All still-missing words are re-read together each round.
__device__ __noinline__ bool load_tagged(const u64 *src, int n, unsigned ep, float *dst, const Ctl &c, int site) {
    const int t = threadIdx.x;
    uint32_t pending = 0;
    u64 w[POLL];
#pragma unroll
    for (int j = 0; j < POLL; j++) {
        const int i = t + j * NCT;
        if (i < n) {
            pending |= 1u << j;
            w[j] = ld_tag(src + i);
        }
    }
    const long long t0 = clock64();
    for (int iter = 0;; iter++) {
#pragma unroll
        for (int j = 0; j < POLL; j++)
            if ((pending >> j) & 1u) {
                if (tag_ep(w[j]) == ep) {
                    dst[t + j * NCT] = tag_val(w[j]);
                    pending &= ~(1u << j);
                }
            }
        if (!pending) return true;
        if (should_stop(c, iter)) return false;
        if (timed_out(t0)) {
            abort_now(c, site);
            return false;
        }
#pragma unroll
        for (int j = 0; j < POLL; j++)
            if ((pending >> j) & 1u) w[j] = ld_tag(src + t + j * NCT);
    }
}

// Consumer-wide sum; red has NCW floats.
__device__ float consumer_sum(float v, float *red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = v;
    consumer_sync();
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NCW; i++) s += red[i];
    consumer_sync();
    return s;
}

// In place: x[i] = x[i] * (1/sqrtf(mean(x^2)+eps)) * w[i]  (qwen_rms_norm,
// qwen_asr_kernels.c:750-809); x (raw) and w (prefetched) in smem. The raw
// values of this CTA's residual rows [own0, own0+nown) are kept in xown first.
__device__ void rmsnorm_smem(float *x, const float *w, int h, float eps, float *red, float *xown, int own0,
                             int nown) {
    cp_async_wait();
    consumer_sync();
    for (int i = threadIdx.x; i < nown; i += NCT) xown[i] = x[own0 + i];
    float ss = 0.f;
    for (int i = threadIdx.x; i < h; i += NCT) ss += x[i] * x[i];
    ss = consumer_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)h + eps);
    for (int i = threadIdx.x; i < h; i += NCT) x[i] = x[i] * inv * w[i];
    consumer_sync();
}

// Dot products of nr rows (bf16, row length K, in smem) with act (smem f32).
// out[r] for r < nr (nr <= 32). Two dot streams at a time, lanes stride 8
// elements: row pairs share the activation loads; an odd last row is split
// into its two halves (when K is a multiple of 512) instead of being paired
// with a duplicate of itself.
typedef unsigned long long f32x2_t;  // two f32 in one 64-bit register pair
__device__ __forceinline__ f32x2_t pk2(float lo, float hi) {
    f32x2_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void fma2(f32x2_t &acc, f32x2_t a, f32x2_t b) {
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}
__device__ __forceinline__ float sum2(f32x2_t v) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
    return lo + hi;
}
// bf16 pair (low half = even column) -> f32 pair
__device__ __forceinline__ f32x2_t bf2(uint32_t w) { return pk2(bf16lo(w), bf16hi(w)); }

// HALVES: the second stream reads act at +x1off (a half row); otherwise both
// streams share one activation load.
template <bool HALVES>
__device__ __forceinline__ void dots2(const uint4 *p0, const uint4 *p1, const float *x0, int x1off, int nv,
                                      float &s0, float &s1) {
    const int lane = threadIdx.x & 31;
    // two independent packed chains per stream (each FMA2 = two columns)
    f32x2_t a[2] = {0ull, 0ull}, b[2] = {0ull, 0ull};
#pragma unroll 4
    for (int j = 0; j < nv; j++) {
        const int e = (j * 32 + lane);
        const uint4 w0 = p0[e];
        const uint4 w1 = p1[e];
        const ulonglong2 xa = *reinterpret_cast<const ulonglong2 *>(x0 + e * 8);
        const ulonglong2 xb = *reinterpret_cast<const ulonglong2 *>(x0 + e * 8 + 4);
        const ulonglong2 ya = HALVES ? *reinterpret_cast<const ulonglong2 *>(x0 + x1off + e * 8) : xa;
        const ulonglong2 yb = HALVES ? *reinterpret_cast<const ulonglong2 *>(x0 + x1off + e * 8 + 4) : xb;
        fma2(a[0], bf2(w0.x), xa.x); fma2(a[1], bf2(w0.y), xa.y);
        fma2(a[0], bf2(w0.z), xb.x); fma2(a[1], bf2(w0.w), xb.y);
        fma2(b[0], bf2(w1.x), ya.x); fma2(b[1], bf2(w1.y), ya.y);
        fma2(b[0], bf2(w1.z), yb.x); fma2(b[1], bf2(w1.w), yb.y);
    }
    s0 = sum2(a[0]) + sum2(a[1]);
    s1 = sum2(b[0]) + sum2(b[1]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        s0 += __shfl_xor_sync(0xffffffffu, s0, o);
        s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
}

constexpr int DOT_GROUP = 4;  // rows per pass over K (activation loads are shared by the group)
// Dot products of NR consecutive rows (stride K) with act, all lanes end
// with the sums in out[0..NR). One f32x2 chain per row, lanes stride 8.
template <int NR>
__device__ __forceinline__ void dots_rows(const uint16_t *w, int K, const float *act, float *out) {
    const int lane = threadIdx.x & 31;
    const int nv = K >> 8;
    f32x2_t acc[NR][2];
#pragma unroll
    for (int r = 0; r < NR; r++) acc[r][0] = acc[r][1] = 0ull;
#pragma unroll 2
    for (int j = 0; j < nv; j++) {
        const int e = (j * 32 + lane);
        const ulonglong2 xa = *reinterpret_cast<const ulonglong2 *>(act + e * 8);
        const ulonglong2 xb = *reinterpret_cast<const ulonglong2 *>(act + e * 8 + 4);
#pragma unroll
        for (int r = 0; r < NR; r++) {
            const uint4 wv = reinterpret_cast<const uint4 *>(w + (size_t)r * K)[e];
            fma2(acc[r][0], bf2(wv.x), xa.x);
            fma2(acc[r][1], bf2(wv.y), xa.y);
            fma2(acc[r][0], bf2(wv.z), xb.x);
            fma2(acc[r][1], bf2(wv.w), xb.y);
        }
    }
#pragma unroll
    for (int r = 0; r < NR; r++) {
        float v = sum2(acc[r][0]) + sum2(acc[r][1]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        out[r] = v;
    }
}

__device__ __forceinline__ void stage_dots(const uint16_t *wst, int nr, int K, const float *act, float *out) {
    int r = 0;
    for (; r + DOT_GROUP <= nr; r += DOT_GROUP) dots_rows<DOT_GROUP>(wst + (size_t)r * K, K, act, out + r);
    if (r + 2 <= nr) {
        dots_rows<2>(wst + (size_t)r * K, K, act, out + r);
        r += 2;
    }
    if (r < nr) {
        const uint4 *p0 = reinterpret_cast<const uint4 *>(wst + (size_t)r * K);
        const int nv = K >> 8;
        float s0, s1;
        if ((nv & 1) == 0) {  // an odd last row: its two halves as two streams
            dots2<true>(p0, p0 + (K >> 4), act, K >> 1, nv >> 1, s0, s1);
            out[r] = s0 + s1;
        } else {
            dots2<false>(p0, p0, act, 0, nv, s0, s1);
            out[r] = s0;
        }
    }
}

// ---------------------------------------------------------------- attention
template <int R>
struct AttnSmem {
    float q[R][QDB_HD];
    float knew[QDB_HD];
    float vnew[QDB_HD];
    float qn[QDB_HD], kn[QDB_HD];   // q_norm / k_norm weights (prefetched)
    float2 rope[QDB_HD / 2];        // this position's (cos, sin) row (prefetched)
    float m[NCW][R];
    float l[NCW][R];
    float o[NCW][R][QDB_HD];
    float wq[R][64];                // split-0 merge: weight of each split's partial
    float invl[R];                  //   and 1 / the merged softmax denominator
};

// Per-head RMSNorm then NeoX rotation of one 128-float head in smem, one warp
// (qwen_rms_norm_per_head :811-873, qwen_apply_rope_neox :1182-1247).
__device__ __forceinline__ void head_norm_rope(float *v, const float *w, const float2 *rope_row, float eps) {
    const int lane = threadIdx.x & 31;
    float e[4];
#pragma unroll
    for (int i = 0; i < 4; i++) e[i] = v[lane + 32 * i];
    const float ss = warp_sum(e[0] * e[0] + e[1] * e[1] + e[2] * e[2] + e[3] * e[3]);
    const float inv = 1.0f / sqrtf(ss / (float)QDB_HD + eps);
#pragma unroll
    for (int i = 0; i < 4; i++) e[i] = e[i] * inv * w[lane + 32 * i];
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const float2 cs = rope_row[lane + 32 * i];
        const float x1 = e[i], x2 = e[i + 2];
        e[i] = x1 * cs.x - x2 * cs.y;
        e[i + 2] = x2 * cs.x + x1 * cs.y;
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; i++) v[lane + 32 * i] = e[i];
    __syncwarp();
}

// Polls one 128-word head (4 words per lane, all in flight) with one warp;
// the result is the same for every lane.
__device__ __forceinline__ bool warp_load_head(const u64 *src, unsigned ep, float *dst, const Ctl &c, int site) {
    const int lane = threadIdx.x & 31;
    u64 w[4];
    uint32_t pending = 0xfu;
#pragma unroll
    for (int j = 0; j < 4; j++) w[j] = ld_tag(src + lane + 32 * j);
    const long long t0 = clock64();
    for (int iter = 0;; iter++) {
#pragma unroll
        for (int j = 0; j < 4; j++)
            if (((pending >> j) & 1u) && tag_ep(w[j]) == ep) {
                dst[lane + 32 * j] = tag_val(w[j]);
                pending &= ~(1u << j);
            }
        if (!__any_sync(0xffffffffu, pending != 0)) break;
        int stop = 0;
        if (lane == 0) {
            stop = should_stop(c, iter) ? 1 : 0;
            if (!stop && timed_out(t0)) {
                abort_now(c, site);
                stop = 1;
            }
        }
        if (__shfl_sync(0xffffffffu, stop, 0)) return false;
#pragma unroll
        for (int j = 0; j < 4; j++)
            if ((pending >> j) & 1u) w[j] = ld_tag(src + lane + 32 * j);
    }
    __syncwarp();
    return true;
}

// Attention unit (KV head g, split s of S) for this step's position. Reads
// q/k/v tagged ep_in (phase A); partials and the merged output are tagged
// ep_in + 1. Everything that does not depend on this step's q/k/v (the
// q/k norm weights, the RoPE row and the first cached K/V rows of each warp)
// is requested before the q/k/v poll.
template <int R>
__device__ __noinline__ void attn_unit(const QdbStepArgs &a, const QdbLayerW &lw, int layer, int g, int s, int S,
                                       unsigned ep_in, AttnSmem<R> *sm, const Ctl &c) {
    const unsigned ep = ep_in + 1;
    const QdbDims &d = a.d;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ctx = a.pos + 1;
    const int per = (ctx + S - 1) / S;
    const int p0 = s * per;
    const int p1 = min(ctx, p0 + per);
    const int qd = d.Hq * QDB_HD, kvd = d.Hkv * QDB_HD;
    const size_t head_base = ((size_t)layer * d.Hkv + g) * (size_t)a.cap * QDB_HD;
    uint16_t *kc = a.kc + head_base;
    uint16_t *vc = a.vc + head_base;
    const bool owns_new = (p0 <= a.pos && a.pos < p1);
    if (!check_or_record(a.pos < a.cap && a.pos < a.rope_cap &&
                             (size_t)(d.Hq * S) * (2 + QDB_HD) <= (size_t)a.part_len,
                         a.err, 2, a.pos, a.cap)) {
        *c.abort = 1;
        return;
    }
    // prefetch: norm weights + rope row to smem, first K/V rows to registers
    if (threadIdx.x < 32) cp_async16(sm->qn + threadIdx.x * 4, lw.q_norm + threadIdx.x * 4);
    else if (threadIdx.x < 64) cp_async16(sm->kn + (threadIdx.x - 32) * 4, lw.k_norm + (threadIdx.x - 32) * 4);
    else if (threadIdx.x < 96)
        cp_async16(&sm->rope[(threadIdx.x - 64) * 2], a.rope + (size_t)a.pos * (QDB_HD / 2) + (threadIdx.x - 64) * 2);
    cp_async_commit();
    const int sub = lane & 3, kk = lane >> 2;
    const int base0 = p0 + warp * ATT_KEYS;
    uint4 kv4[4];
    uint2 vv[ATT_KEYS];
    {
        const int j = base0 + kk;
        if (j < p1 && j != a.pos) {
            const uint4 *kp = reinterpret_cast<const uint4 *>(kc + (size_t)j * QDB_HD + sub * 32);
#pragma unroll
            for (int u = 0; u < 4; u++) kv4[u] = __ldcg(kp + u);
        }
#pragma unroll
        for (int t = 0; t < ATT_KEYS; t++) {
            const int jt = base0 + t;
            if (jt < p1 && jt != a.pos)
                vv[t] = __ldcg(reinterpret_cast<const uint2 *>(vc + (size_t)jt * QDB_HD + lane * 4));
        }
    }
    cp_async_wait();
    consumer_sync();

    // q heads of this group (and the new K/V row for the owner), one warp each
    for (int h = warp; h < R + (owns_new ? 2 : 0); h += NCW) {
        if (h < R) {
            if (warp_load_head(a.tqkv + (size_t)(g * R + h) * QDB_HD, ep_in, sm->q[h], c, 10))
                head_norm_rope(sm->q[h], sm->qn, sm->rope, d.eps);
        } else if (h == R) {
            if (warp_load_head(a.tqkv + qd + (size_t)g * QDB_HD, ep_in, sm->knew, c, 11)) {
                head_norm_rope(sm->knew, sm->kn, sm->rope, d.eps);
                for (int i = lane; i < QDB_HD; i += 32)
                    kc[(size_t)a.pos * QDB_HD + i] = f32_to_kv(sm->knew[i]);
            }
        } else {
            if (warp_load_head(a.tqkv + qd + kvd + (size_t)g * QDB_HD, ep_in, sm->vnew, c, 12))
                for (int i = lane; i < QDB_HD; i += 32)
                    vc[(size_t)a.pos * QDB_HD + i] = f32_to_kv(sm->vnew[i]);
        }
    }
    consumer_sync();  // new K/V row stored (global writes by this CTA are visible to it)

    const float scale = 1.0f / sqrtf((float)QDB_HD);
    float m[R], l[R], o[R][4];
#pragma unroll
    for (int h = 0; h < R; h++) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int e = 0; e < 4; e++) o[h][e] = 0.f;
    }
    if (!warp_aborted(c)) {
        for (int base = base0; base < p1; base += NCW * ATT_KEYS) {
            const int j = base + kk;
            const bool valid = j < p1;
            const bool first = (base == base0);
            if (valid && !first) {
                const uint4 *kp = reinterpret_cast<const uint4 *>(kc + (size_t)j * QDB_HD + sub * 32);
#pragma unroll
                for (int u = 0; u < 4; u++) kv4[u] = __ldcg(kp + u);
            }
            if (first && j == a.pos) {  // this step's row: the rounded values stored above, from smem
                const float *kn = sm->knew + sub * 32;
#pragma unroll
                for (int u = 0; u < 4; u++)
                    kv4[u] = make_uint4(kv_pack2(kn[u * 8 + 0], kn[u * 8 + 1]), kv_pack2(kn[u * 8 + 2], kn[u * 8 + 3]),
                                        kv_pack2(kn[u * 8 + 4], kn[u * 8 + 5]), kv_pack2(kn[u * 8 + 6], kn[u * 8 + 7]));
            }
#pragma unroll
            for (int t = 0; t < ATT_KEYS; t++) {
                const int jt = base + t;
                if (jt >= p1) vv[t] = make_uint2(0u, 0u);
                else if (!first)
                    vv[t] = __ldcg(reinterpret_cast<const uint2 *>(vc + (size_t)jt * QDB_HD + lane * 4));
                else if (jt == a.pos)
                    vv[t] = make_uint2(kv_pack2(sm->vnew[lane * 4], sm->vnew[lane * 4 + 1]),
                                       kv_pack2(sm->vnew[lane * 4 + 2], sm->vnew[lane * 4 + 3]));
            }
            float sc[R];
#pragma unroll
            for (int h = 0; h < R; h++) {
                float acc = 0.f;
                if (valid) {
                    const float *qv = sm->q[h] + sub * 32;
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const float4 qa = *reinterpret_cast<const float4 *>(qv + u * 8);
                        const float4 qb = *reinterpret_cast<const float4 *>(qv + u * 8 + 4);
                        acc = dot8_kv(kv4[u], qa, qb, acc);
                    }
                }
                acc += __shfl_xor_sync(0xffffffffu, acc, 1);
                acc += __shfl_xor_sync(0xffffffffu, acc, 2);
                sc[h] = valid ? acc * scale : -INFINITY;
            }
#pragma unroll
            for (int h = 0; h < R; h++) {
                float cm = sc[h];
                cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 4));
                cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 8));
                cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 16));
                const float mn = fmaxf(m[h], cm);
                const float corr = expf(m[h] - mn);
                const float p = valid ? expf(sc[h] - mn) : 0.f;
                float ps = p;
                ps += __shfl_xor_sync(0xffffffffu, ps, 4);
                ps += __shfl_xor_sync(0xffffffffu, ps, 8);
                ps += __shfl_xor_sync(0xffffffffu, ps, 16);
                l[h] = l[h] * corr + ps;
#pragma unroll
                for (int e = 0; e < 4; e++) o[h][e] *= corr;
#pragma unroll
                for (int t = 0; t < ATT_KEYS; t++) {
                    const float pt = __shfl_sync(0xffffffffu, p, t * 4);
                    o[h][0] = fmaf(pt, kvlo(vv[t].x), o[h][0]);
                    o[h][1] = fmaf(pt, kvhi(vv[t].x), o[h][1]);
                    o[h][2] = fmaf(pt, kvlo(vv[t].y), o[h][2]);
                    o[h][3] = fmaf(pt, kvhi(vv[t].y), o[h][3]);
                }
                m[h] = mn;
            }
        }
    }
#pragma unroll
    for (int h = 0; h < R; h++) {
        if (lane == 0) {
            sm->m[warp][h] = m[h];
            sm->l[warp][h] = l[h];
        }
#pragma unroll
        for (int e = 0; e < 4; e++) sm->o[warp][h][lane * 4 + e] = o[h][e];
    }
    consumer_sync();
    // merge the warps; write the unit partial (m, l, o) tagged
    for (int t = threadIdx.x; t < R * QDB_HD; t += NCT) {
        const int h = t / QDB_HD, dd = t % QDB_HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NCW; w++) M = fmaxf(M, sm->m[w][h]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < NCW; w++) {
                const float f = expf(sm->m[w][h] - M);
                L += sm->l[w][h] * f;
                O += sm->o[w][h][dd] * f;
            }
        }
        u64 *dst = a.tpart + ((size_t)(g * R + h) * S + s) * (2 + QDB_HD);
        if (dd == 0) {
            st_tag(dst, M, ep);
            st_tag(dst + 1, L, ep);
        }
        st_tag(dst + 2 + dd, O, ep);
    }
    if (s != 0) return;
    // Split 0 merges all S partials of its KV head into attn. First one warp
    // per head polls every split's (m, l) at once and turns them into
    // weights; then each thread merges its output elements with the O words
    // of MERGE_CHUNK splits in flight per round trip.
    for (int h = warp; h < R; h += NCW) {
        const u64 *src = a.tpart + (size_t)(g * R + h) * S * (2 + QDB_HD);
        float mq[2], lq[2];
        uint32_t pending = 0;
        u64 w[4];
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int q = lane + 32 * k;
            mq[k] = -INFINITY;
            lq[k] = 0.f;
            if (q < S) {
                pending |= 3u << (2 * k);
                w[2 * k] = ld_tag(src + (size_t)q * (2 + QDB_HD));
                w[2 * k + 1] = ld_tag(src + (size_t)q * (2 + QDB_HD) + 1);
            }
        }
        const long long t0 = clock64();
        bool ok = true;
        for (int iter = 0;; iter++) {
#pragma unroll
            for (int b = 0; b < 4; b++)
                if (((pending >> b) & 1u) && tag_ep(w[b]) == ep) pending &= ~(1u << b);
            const bool stop = should_stop(c, iter);
            const bool late = !stop && timed_out(t0);
            if (__all_sync(0xffffffffu, pending == 0)) break;
            if (__any_sync(0xffffffffu, stop || late)) {
                if (__any_sync(0xffffffffu, late) && lane == 0) abort_now(c, 13);
                ok = false;
                break;
            }
#pragma unroll
            for (int b = 0; b < 4; b++)
                if ((pending >> b) & 1u)
                    w[b] = ld_tag(src + (size_t)(lane + 32 * (b >> 1)) * (2 + QDB_HD) + (b & 1));
        }
        if (!ok) continue;
#pragma unroll
        for (int k = 0; k < 2; k++)
            if (lane + 32 * k < S) {
                mq[k] = tag_val(w[2 * k]);
                lq[k] = tag_val(w[2 * k + 1]);
            }
        float M = fmaxf(mq[0], mq[1]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float f[2], L = 0.f;
#pragma unroll
        for (int k = 0; k < 2; k++) {
            f[k] = (M == -INFINITY || mq[k] == -INFINITY) ? 0.f : expf(mq[k] - M);
            L += lq[k] * f[k];
        }
        L = warp_sum(L);
#pragma unroll
        for (int k = 0; k < 2; k++)
            if (lane + 32 * k < 64) sm->wq[h][lane + 32 * k] = f[k];
        if (lane == 0) sm->invl[h] = L > 0.f ? 1.0f / L : 0.f;
    }
    consumer_sync();
    if (warp_aborted(c)) return;
    constexpr int MERGE_CHUNK = 16;
    for (int t = threadIdx.x; t < R * QDB_HD; t += NCT) {
        const int h = t / QDB_HD, dd = t % QDB_HD;
        const u64 *src = a.tpart + (size_t)(g * R + h) * S * (2 + QDB_HD) + 2 + dd;
        float O = 0.f;
        for (int q0 = 0; q0 < S; q0 += MERGE_CHUNK) {
            u64 w[MERGE_CHUNK];
            uint32_t pending = 0;
#pragma unroll
            for (int k = 0; k < MERGE_CHUNK; k++)
                if (q0 + k < S) {
                    pending |= 1u << k;
                    w[k] = ld_tag(src + (size_t)(q0 + k) * (2 + QDB_HD));
                }
            const long long t0 = clock64();
            for (int iter = 0;; iter++) {
#pragma unroll
                for (int k = 0; k < MERGE_CHUNK; k++)
                    if (((pending >> k) & 1u) && tag_ep(w[k]) == ep) pending &= ~(1u << k);
                if (!pending) break;
                if (should_stop(c, iter)) return;
                if (timed_out(t0)) {
                    abort_now(c, 14);
                    return;
                }
#pragma unroll
                for (int k = 0; k < MERGE_CHUNK; k++)
                    if ((pending >> k) & 1u) w[k] = ld_tag(src + (size_t)(q0 + k) * (2 + QDB_HD));
            }
#pragma unroll
            for (int k = 0; k < MERGE_CHUNK; k++)
                if (q0 + k < S) O = fmaf(sm->wq[h][q0 + k], tag_val(w[k]), O);
        }
        st_tag(a.tattn + (size_t)(g * R + h) * QDB_HD + dd, O * sm->invl[h], ep);
    }
}

// One phase's ring items for this warp (items it % NCW == warp): row dots,
// then the phase's epilogue. mode 0: QKV store, 1: O + residual, 2: gate/up
// SwiGLU, 3: down + residual, 4: lm_head + running argmax. One out-of-line
// copy serves every phase, which keeps the kernel's code small.
__device__ __forceinline__ void items_phase(const QdbStepArgs &a, const Slice &s, int mode, unsigned ep, u64 &best, unsigned &it,
                 unsigned char *ring, u64 *full, u64 *empty, const float *act, const float *xown, int own0,
                 float *outw, const Ctl &c) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = s.items();
    for (int k = 0; k < n; k++, it++) {
        if ((int)(it % NCW) != warp) continue;
        const unsigned st = it % NSTAGE;
        if (warp_aborted(c) || !mbar_wait_warp(&full[st], (it / NSTAGE) & 1, c, 3)) continue;
        const int r = s.r0 + k * s.ipr;
        const int nr = min(s.ipr, s.r1 - r);
        const uint16_t *wst = reinterpret_cast<const uint16_t *>(ring + (size_t)st * STAGE_BYTES);
        stage_dots(wst, nr, s.K, act, outw);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        if (mode == 4) {
            if (lane < nr) {
                const int row = r + lane;
                const float v = outw[lane];
                if (a.logits_out) a.logits_out[row] = v;
                if (!(a.mask_eos && (row == QDB_ENDOFTEXT || row == QDB_IM_END)) && !isnan(v)) {
                    const u64 key = argmax_key(v, row);
                    best = key > best ? key : best;
                }
            }
        } else if (mode == 2) {
            if (lane < nr / 2) {
                const int pr = r / 2 + lane;
                st_tag(a.tact + pr, silu_mul(outw[2 * lane], outw[2 * lane + 1]), ep);
            }
        } else if (lane < nr) {
            const int row = r + lane;
            const float v = outw[lane];
            if (mode == 0) st_tag(a.tqkv + row, v, ep);
            else st_tag(a.tx + row, xown[row - own0] + v, ep);
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------- the kernel
// Dynamic shared memory: ring | act. act holds the phase's input vector
// (x while it is normalised in place with the norm weights at act[h..2h),
// attn, or the SwiGLU activations) and, in attention CTAs, the attention
// scratch.
template <int R>
__host__ __device__ constexpr int act_region_floats(int h, int qd, int I) {
    int n = 2 * h > qd ? 2 * h : qd;
    n = n > I ? n : I;
    const int att = (int)(sizeof(AttnSmem<R>) / sizeof(float));
    return n > att ? n : att;
}

template <int R>
__global__ void __launch_bounds__(NTHREADS, 1) step_kernel(const QdbStepArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ __align__(8) u64 full[NSTAGE], empty[NSTAGE];
    __shared__ __align__(16) QdbLayerW layers[MAX_LAYERS];
    __shared__ float red[NCW];
    __shared__ float outs[NCW][32];
    __shared__ u64 wbest[NCW];
    __shared__ volatile int s_abort;

    const QdbDims &d = a.d;
    // residual rows owned by this CTA in phases C and E (same slice of h rows)
    const int own0 = (int)((long long)d.h * blockIdx.x / gridDim.x);
    const int nown = (int)((long long)d.h * (blockIdx.x + 1) / gridDim.x) - own0;
    const int h = d.h, qd = d.Hq * QDB_HD, I = d.I;
    unsigned char *ring = smem_raw;
    float *act = reinterpret_cast<float *>(smem_raw + (size_t)NSTAGE * STAGE_BYTES);
    float *wn = act + h;
    __shared__ float xown[OWN_ROWS];  // raw residual of this CTA's O/down rows
    AttnSmem<R> *asm_ = reinterpret_cast<AttnSmem<R> *>(act);

    if (threadIdx.x == 0) {
        s_abort = 0;
        for (int i = 0; i < NSTAGE; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    {  // layer table -> shared memory (no dependent global load per phase)
        const int words = d.L * (int)(sizeof(QdbLayerW) / 8);
        const u64 *src = reinterpret_cast<const u64 *>(a.layers);
        u64 *dst = reinterpret_cast<u64 *>(layers);
        for (int i = threadIdx.x; i < words; i += NTHREADS) dst[i] = src[i];
    }
    __syncthreads();
    Ctl c{&s_abort, a.err};
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == NCW) {
        producer(a, layers, ring, full, empty, c);
        return;
    }

    const int tstride = qdb_step_trace_events(d.L);
    auto mark = [&](int idx) {
        if (a.trace && threadIdx.x == 0) {
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            a.trace[(size_t)blockIdx.x * tstride + idx] = t;
        }
    };
    mark(0);
    unsigned it = 0;  // ring item counter (same sequence as the producer)
    auto run_items = [&](const Slice &s, int mode, unsigned ep, u64 &best) {
        items_phase(a, s, mode, ep, best, it, ring, full, empty, act, xown, own0, outs[warp], c);
    };

    u64 best = 0ull;
    for (int layer = 0; layer < d.L; layer++) {
        const unsigned epA = a.epoch + 5u * layer;
        const QdbLayerW &lw = layers[layer];
        const int tb = 1 + 9 * layer;
        // ---- A: residual -> act (own rows kept), input norm in place, QKV rows
        consumer_sync();
        mark(tb + 0);
        prefetch_f32(wn, lw.in_norm, h);
        if (layer == 0) {
            if (a.token_in) {
                int tok = *a.token_in;
                if (tok < 0 || tok >= d.V) {  // never gather outside the table
                    set_error(a.err, QDB_ERR_BAD_ARG);
                    tok = 0;
                }
                const uint16_t *e = a.embed + (size_t)tok * h;
                for (int i = threadIdx.x; i < h; i += NCT) act[i] = __uint_as_float(((uint32_t)e[i]) << 16);
            } else {
                for (int i = threadIdx.x; i < h; i += NCT) act[i] = a.x_in[i];
            }
        } else if (!*c.abort) {
            load_tagged(a.tx, h, epA - 1, act, c, 4);  // written by E of the previous layer
        }
        rmsnorm_smem(act, wn, h, d.eps, red, xown, own0, nown);
        mark(tb + 1);
        run_items(phase_slice(a, layers, layer, 0), 0, epA, best);

        // ---- B: attention units
        const int S = a.splits;
        if ((int)blockIdx.x < d.Hkv * S) {
            consumer_sync();
            mark(tb + 2);
            const int u = blockIdx.x;
            attn_unit<R>(a, lw, layer, u / S, u % S, S, epA, asm_, c);
        }

        // ---- C: O-proj + residual
        consumer_sync();
        mark(tb + 3);
        if (!*c.abort) load_tagged(a.tattn, qd, epA + 1, act, c, 5);
        consumer_sync();
        mark(tb + 4);
        run_items(phase_slice(a, layers, layer, 1), 1, epA + 2, best);

        // ---- D: post-attention norm + gate/up + SwiGLU
        consumer_sync();
        mark(tb + 5);
        prefetch_f32(wn, lw.post_norm, h);
        if (!*c.abort) load_tagged(a.tx, h, epA + 2, act, c, 6);
        rmsnorm_smem(act, wn, h, d.eps, red, xown, own0, nown);
        mark(tb + 6);
        run_items(phase_slice(a, layers, layer, 2), 2, epA + 3, best);

        // ---- E: down + residual
        consumer_sync();
        mark(tb + 7);
        if (!*c.abort) load_tagged(a.tact, I, epA + 3, act, c, 7);
        consumer_sync();
        mark(tb + 8);
        run_items(phase_slice(a, layers, layer, 3), 3, epA + 4, best);
    }
    // ---- F: final norm + lm_head + argmax
    const unsigned epF = a.epoch + 5u * d.L;
    const int tf = 1 + 9 * d.L;
    consumer_sync();
    mark(tf);
    prefetch_f32(wn, a.final_norm, h);
    if (!*c.abort) load_tagged(a.tx, h, epF - 1, act, c, 8);
    rmsnorm_smem(act, wn, h, d.eps, red, xown, own0, nown);
    mark(tf + 1);
    if (blockIdx.x == 0 && a.hidden_out)
        for (int i = threadIdx.x; i < h; i += NCT) a.hidden_out[i] = act[i];
    run_items(phase_slice(a, layers, 0, 4), 4, epF, best);
    // reduce this CTA's best, publish, elect the last CTA
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const u64 t = __shfl_xor_sync(0xffffffffu, best, o);
        best = t > best ? t : best;
    }
    if (lane == 0) wbest[warp] = best;
    consumer_sync();
    mark(tf + 2);
    if (threadIdx.x == 0) {
        u64 b = 0ull;
        for (int w = 0; w < NCW; w++) b = wbest[w] > b ? wbest[w] : b;
        if (b) atomicMax(a.best, b);
        __threadfence();
        const unsigned prev = atomicAdd(a.done, 1u);
        if (prev == gridDim.x - 1) {
            __threadfence();
            const u64 fin = atomicMax(a.best, 0ull);
            if (fin == 0ull) set_error(a.err, QDB_ERR_BAD_ARG);  // no candidate (aborted step)
            *a.token_out = fin ? argmax_key_index(fin) : 0;
            atomicExch(a.best, 0ull);
            atomicExch(a.done, 0u);
        }
    }
}

__global__ void rope_table_kernel(float2 *tab, int n_pos, float theta) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_pos * (QDB_HD / 2)) return;
    const int p = i / (QDB_HD / 2), dd = i % (QDB_HD / 2);
    // inv_freq = 1/powf(theta, 2d/hd) and angle = (float)p * inv_freq in f32,
    // as the reference (qwen_asr_decoder.c:216, :244); pow/cos/sin evaluated
    // in double and rounded once.
    const float e = (float)(2 * dd) / (float)QDB_HD;
    const float pw = (float)pow((double)theta, (double)e);
    const float inv = 1.0f / pw;
    const float angle = (float)p * inv;
    tab[i] = make_float2((float)cos((double)angle), (float)sin((double)angle));
}


int step_smem_bytes(const QdbDims &d) {
    const int qd = d.Hq * QDB_HD;
    int act = 0;
    switch (d.Hq / d.Hkv) {
        case 1: act = act_region_floats<1>(d.h, qd, d.I); break;
        case 2: act = act_region_floats<2>(d.h, qd, d.I); break;
        case 4: act = act_region_floats<4>(d.h, qd, d.I); break;
        default: act = act_region_floats<8>(d.h, qd, d.I); break;
    }
    return NSTAGE * STAGE_BYTES + act * (int)sizeof(float);
}

template <int R>
cudaError_t launch_r(const QdbStepArgs &a, int grid, cudaStream_t st) {
    const int smem = step_smem_bytes(a.d);
    cudaError_t e = cudaFuncSetAttribute(step_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    void *args[] = {const_cast<QdbStepArgs *>(&a)};
    return cudaLaunchCooperativeKernel((const void *)step_kernel<R>, dim3(grid), dim3(NTHREADS), args,
                                       (size_t)smem, st);
}

cudaError_t launch_step(const QdbStepArgs &a, int grid, cudaStream_t st) {
    if (a.d.h > POLL * NCT || a.d.I > POLL * NCT || a.d.Hq * QDB_HD > POLL * NCT) return cudaErrorInvalidValue;
    if (a.d.L > MAX_LAYERS) return cudaErrorInvalidValue;
    if ((a.d.h + grid - 1) / grid > OWN_ROWS) return cudaErrorInvalidValue;
    if (a.splits < 1 || a.splits > 64 || a.d.Hkv * a.splits > grid) return cudaErrorInvalidValue;
    switch (a.d.Hq / a.d.Hkv) {
        case 1: return launch_r<1>(a, grid, st);
        case 2: return launch_r<2>(a, grid, st);
        case 4: return launch_r<4>(a, grid, st);
        case 8: return launch_r<8>(a, grid, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t set_wait_limit(long long cycles) {
    return cudaMemcpyToSymbol(qdb_wait_limit_c, &cycles, sizeof(cycles));
}

const QdbStepKernel k_entry = {QDB_STEP_NAME, NCW, STAGE_BYTES, POLL * NCT, step_smem_bytes, launch_step,
                               set_wait_limit};

}  // namespace

extern "C" const QdbStepKernel *QDB_STEP_ENTRY(void) { return &k_entry; }

#if QDB_STEP_COMMON
extern "C" int qdb_step_max_splits(int grid, int kv_heads) {
    int s = grid / kv_heads;
    return s < 1 ? 1 : (s > 64 ? 64 : s);
}

extern "C" int qdb_step_max_grid(int device) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    return sms;
}

extern "C" cudaError_t qdb_launch_rope_table(float2 *tab, int n_pos, float theta, cudaStream_t st) {
    const int n = n_pos * (QDB_HD / 2);
    rope_table_kernel<<<(n + 255) / 256, 256, 0, st>>>(tab, n_pos, theta);
    return cudaGetLastError();
}
#endif
