// qdb_bstep.cu - persistent batched decode step: one decode position of B
// independent utterances (B <= 64) in ONE cooperative launch, the row dots on
// the 5th-generation tensor cores. Per utterance it computes what
// qwen_decoder_forward does (qwen_asr_decoder.c:388-476): 28 layers of
// RMSNorm -> QKV -> per-head QK-norm + NeoX RoPE + KV append -> causal GQA
// attention -> O + residual -> RMSNorm -> gate/up + SwiGLU -> down + residual,
// then the final norm, the tied lm_head and the greedy argmax (lowest index
// on exact ties, qwen_asr_kernels.c:518-543).
//
// One CTA per SM (cooperative: all CTAs co-resident). Warp roles:
//   warp 0       producer: streams this CTA's slice of every weight matrix of
//                the step (128-row x 64-column bf16 tiles, TMA with 128-byte
//                swizzle, L2 evict-first) through a ring of W stages. It never
//                waits for activations, so weights run ahead across phases.
//   warp 1       allocates TMEM; one thread issues tcgen05.mma: D[128 weight
//                rows, Bp utterances] += W[128, 64] . X[Bp, 64]^T, twice per
//                k-step (X as bf16 hi + lo: ~16 mantissa bits of the f32
//                activation), f32 accumulators in TMEM (8 slots of Bp columns).
//   warps 2..5   epilogue: tcgen05.ld of a finished accumulator (warp q holds
//                TMEM lanes 32q..32q+31 = weight rows), red.global.add.v4 of the
//                split-K partial into the phase output (layout [row][Bp], so a
//                thread's utterances are consecutive addresses), or, for the
//                lm_head, scaled logits and a running (value, index) argmax.
//                They also compute the per-utterance RMS statistics.
//   warps 6..13  builders: turn the phase's f32 activations into the X tiles
//                of the ring (bf16 hi/lo, 128-byte swizzle, written by threads,
//                fence.proxy.async before the MMA reads them), and run the
//                attention units between the QKV and O phases.
//
// Phases of a layer (each CTA takes an equal contiguous share of every
// matrix's (tile, k-block) items; split-K partials meet in red.add targets):
//   QKV   X = x * w_in (the 1/rms factor of the input norm is applied by the
//         attention units: the projections are linear in it) -> qkv [qkvd][Bp]
//   ATT   unit = (utterance, KV head, key split): q/k/v scaled by 1/rms, q/k
//         RMSNorm + RoPE, fp16 K/V append at the position, online-softmax
//         partial (m, l, o) over the split's keys
//   O     X = merged attention output -> red.add into the residual x [h][Bp]
//   GU    X = x * w_post -> gu [2I][Bp]
//   DOWN  X = silu(r g) * (r u) (r = 1/rms of x after O) -> red.add into x
// then LM: X = x * w_final, whole 128-row vocabulary tiles per CTA (no
// split-K, kb-outer so one X tile serves up to 8 accumulators), logits scaled
// by the final 1/rms, argmax per utterance.
//
// Phase completion is a counter per (phase, layer) that every CTA increments
// once after its part (fence first); a reader polls it until it reaches the
// grid size. RMS statistics are epoch-tagged 64-bit words. The last CTA to
// finish clears the counters and the argmax keys and advances the step
// counter, so the next launch (or graph replay) starts clean.
//
// Every wait is bounded (run-time limit); a wait that runs out records an
// error, raises the CTA abort flag, and every role winds down: the producer
// drains its copies in flight, the MMA thread waits for its MMAs before TMEM
// is released (fixed bound), and the kernel returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "qdb_common.cuh"
#include "qdb_kernels.h"

namespace {

typedef unsigned long long u64;

constexpr int NWARPS = 14;
constexpr int NTHREADS = NWARPS * 32;
constexpr int EPI0 = 2, NEPI = 4;      // epilogue warps 2..5
constexpr int BLD0 = 6, NBLD = 8;      // builder warps 6..13
constexpr int NACC = 4;                // lm_head tiles per round (one TMEM accumulator each)
constexpr int NSLOT = 2;               // projection segments in flight (double-buffered TMEM slots)
// An MMA multiplies a weight tile (M = 128 rows) with the X tile's hi AND lo
// rows at once (N = 2 * Bp: hi rows 0..Bp-1, lo rows Bp..2Bp-1), so an
// accumulator is 2 * Bp columns; the epilogue adds the two halves. The k-steps
// of a tile alternate over nchain(Bp) independent accumulators (an MMA costs
// about the same for any N; dependent MMAs wait for each other).
__host__ __device__ constexpr int nchain(int Bp) { return Bp >= 64 ? 2 : 4; }
constexpr int W_TILE = 128 * 64 * 2;   // one weight tile (16 KB)
constexpr int MAX_NSW = 8;             // W ring stages (at most)
constexpr int NGRP = 4, GRP_WARPS = 2;  // builder groups: group g builds X tiles xi % 4 == g
constexpr int GRP_T = GRP_WARPS * 32;
constexpr int NSX = NGRP;              // X ring stages (stage g belongs to group g)
constexpr int AK = 64;                 // keys per attention chunk
constexpr int ACHUNK = AK * QDB_HD * 2 * 2;  // K + V of one chunk (32 KB)
constexpr int XRING_MIN = 2 * ACHUNK;  // the X ring doubles as the attention K/V staging (2 chunks)
constexpr int MAX_LAYERS = 32;
constexpr int ATT_KEYS = 8;            // keys per builder warp per attention step

// ---------------------------------------------------------------- small helpers
__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

struct Ctl {
    volatile int *abort;  // CTA-local
    int *err;             // global [4]
};

__device__ __forceinline__ bool timed_out(long long t0) { return clock64() - t0 > qdb_wait_limit_c; }

__device__ __forceinline__ void abort_now(const Ctl &c, int site) {
    *c.abort = 1;
    if (atomicCAS(c.err, 0, QDB_ERR_BARRIER_TIMEOUT) == 0) {
        c.err[1] = site;
        c.err[2] = blockIdx.x;
        c.err[3] = threadIdx.x >> 5;
    }
}

__device__ __forceinline__ bool should_stop(const Ctl &c, int iter) {
    if (*c.abort) return true;
    if ((iter & 255) == 255 && *(volatile int *)c.err) {
        *c.abort = 1;
        return true;
    }
    return false;
}

__device__ __forceinline__ bool warp_aborted(const Ctl &c) {
    int v = 0;
    if ((threadIdx.x & 31) == 0) v = *c.abort;
    return __shfl_sync(0xffffffffu, v, 0) != 0;
}

__device__ __forceinline__ void mb_init(u64 *b, unsigned n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mb_arrive(u64 *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void mb_expect(u64 *b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mb_try(u64 *b, unsigned par) {
    uint32_t ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok)
                 : "r"(su32(b)), "r"(par)
                 : "memory");
    return ok != 0;
}
// One thread. check: honour the abort flag and the run-time limit; otherwise
// (drains) wait up to the fixed bound.
__device__ bool mb_wait(u64 *b, unsigned par, const Ctl &c, bool check, int site) {
    const long long t0 = clock64();
    for (int it = 0;; it++) {
        if (mb_try(b, par)) return true;
        if (check && should_stop(c, it)) return false;
        if (check ? timed_out(t0) : (clock64() - t0 > QDB_SPIN_LIMIT_CYCLES)) {
            abort_now(c, site);
            return false;
        }
    }
}
// Whole warp, uniform result; every lane observes the phase.
__device__ bool mb_wait_warp(u64 *b, unsigned par, const Ctl &c, int site) {
    const long long t0 = clock64();
    for (int it = 0;; it++) {
        const bool done = mb_try(b, par);
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

// Progress word w of this CTA (diagnostics of a wait that ran out): 0 W tiles
// issued, 1 W tiles consumed by the MMA, 2 X tiles consumed, 3 accumulator
// segments issued, 4 segments drained by the epilogue, 5 epilogue phase
// (layer * 8 + matrix), 6 X tiles built, 7 builder phase, 8 the MMA's current
// wait (3 W tile, 4 X tile, 5 accumulator slot, 0 none), 9..16 per builder
// warp: X tile it works on (bit 31 set while it waits for the stage).
constexpr int PROG_WORDS = 17;
__device__ __forceinline__ void progress(const QdbBatchArgs &a, int w, unsigned v) {
    if (a.prog) *(volatile unsigned *)(a.prog + blockIdx.x * PROG_WORDS + w) = v;
}

__device__ __forceinline__ void stamp(const QdbBatchArgs &a, int idx) {
    if (a.trace) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.trace[(size_t)blockIdx.x * qdb_bstep_trace_events(a.d.L) + idx] = t;
    }
}

// Detail stamps of layer 1 (profiling): slot = 0..63 MMA item start (both
// operands ready), 64..127 X tile build start, 128..191 X tile built, 192..223
// epilogue segment ready, 224..255 segment drained; index within the layer.
__device__ __forceinline__ void dstamp(const QdbBatchArgs &a, int slot) {
    if (a.detail && slot >= 0 && slot < 512) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.detail[(size_t)blockIdx.x * 512 + slot] = t;
    }
}

// Phase counter: this CTA's part is done (the caller fenced its writes).
__device__ __forceinline__ void signal(unsigned *cnt) { atomicAdd(cnt, 1u); }

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Warp-uniform bounded wait until *cnt >= target (lane 0 polls).
__device__ bool wait_count_warp(const unsigned *cnt, unsigned target, const Ctl &c, int site) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) {
        const long long t0 = clock64();
        for (int it = 0;; it++) {
            if (ld_acquire(cnt) >= target) break;
            if (should_stop(c, it) || (timed_out(t0) && (abort_now(c, site), true))) {
                ok = 0;
                break;
            }
        }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}

__device__ __forceinline__ void st_tag(u64 *p, float v, unsigned ep) {
    const u64 w = ((u64)ep << 32) | (u64)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ u64 ld_tag(const u64 *p) {
    u64 w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// One lane polls one tagged word (bounded); returns the value, or 0 with the
// abort flag raised.
__device__ float poll_tag(const u64 *p, unsigned ep, const Ctl &c, int site) {
    const long long t0 = clock64();
    for (int it = 0;; it++) {
        const u64 w = ld_tag(p);
        if ((unsigned)(w >> 32) == ep) return __uint_as_float((unsigned)w);
        if (should_stop(c, it)) return 0.f;
        if (timed_out(t0)) {
            abort_now(c, site);
            return 0.f;
        }
    }
}

__device__ __forceinline__ void red_add_v4(float *p, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

// ---------------------------------------------------------------- tcgen05 pieces

__device__ __forceinline__ void bulk_g2s_pol(void *dst, const void *src, unsigned bytes, u64 *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            su32(dst)),
        "l"(src), "r"(bytes), "r"(su32(bar)), "l"(pol)
        : "memory");
}

// K-major operand, rows of 128 bytes in 1024-byte 8-row atoms, 128-byte
// swizzle (the layout the TMA writes for W and the builders write for X).
__device__ __forceinline__ u64 sm_desc(uint32_t saddr) {
    u64 d = 0;
    d |= (u64)((saddr >> 4) & 0x3fffu);
    d |= (u64)1 << 16;
    d |= (u64)(1024 >> 4) << 32;
    d |= (u64)1 << 46;
    d |= (u64)2 << 61;
    return d;
}
// kind::f16 instruction descriptor: D f32, A and B bf16, both K-major, N>>3 at
// bit 17, M>>4 at bit 24.
__device__ __forceinline__ uint32_t instr_desc(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void mma_bf16(uint32_t tmem, u64 a, u64 b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit(u64 *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 16 consecutive accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float *v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- the work schedule
// Matrix m of the step: 0..3 = QKV, O, GU, DOWN of a layer, 4 = lm_head.
struct Mat {
    int N, K, T, KB;
};

__device__ __forceinline__ Mat mat_of(const QdbDims &d, int m) {
    const int qd = d.Hq * QDB_HD, kvd = d.Hkv * QDB_HD;
    Mat r;
    switch (m) {
        case 0: r.N = qd + 2 * kvd; r.K = d.h; break;
        case 1: r.N = d.h; r.K = qd; break;
        case 2: r.N = 2 * d.I; r.K = d.h; break;
        case 3: r.N = d.h; r.K = d.I; break;
        default: r.N = d.V; r.K = d.h; break;
    }
    r.T = (r.N + 127) / 128;
    r.KB = r.K / 64;
    return r;
}

// This CTA's share of a split-K matrix: items [i0, i1) of T*KB (tile-major).
__device__ __forceinline__ void share(const Mat &M, int &i0, int &i1) {
    const long long n = (long long)M.T * M.KB;
    i0 = (int)(n * blockIdx.x / gridDim.x);
    i1 = (int)(n * (blockIdx.x + 1) / gridDim.x);
}
// lm_head: whole tiles in groups of NACC consecutive tiles (the last group
// may be shorter); CTA c takes groups c, c + G, ... A group is one round: its
// tiles share every X tile (kb-outer order) and are accumulated together.
__device__ __forceinline__ int lm_groups(const Mat &M) { return (M.T + NACC - 1) / NACC; }

// Counter index of (layer, phase); phase 0..4 = QKV, ATT, O, GU, DOWN. Slot 0
// is the set-up phase (embedding + clears).
__device__ __forceinline__ int cidx(int layer, int ph) { return 1 + layer * 5 + ph; }

struct Smem {
    u64 wfull[MAX_NSW], wempty[MAX_NSW];
    u64 xfull[NSX], xempty[NSX];
    u64 accfull[NSLOT], accempty[NSLOT];
    u64 lmfull, lmempty;  // lm_head rounds (all of a round's tiles complete together)
    u64 afull[2];  // attention K/V chunks (staged in the X ring)
    u64 mma_done;
    uint32_t tmem;
    int abort;
};

// ---------------------------------------------------------------- builders: X tiles
// L2 load (activations are written by other SMs during the launch: never
// through L1).
__device__ __forceinline__ float ld_l2(const float *p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

// Two f32 as bf16 hi = rn(v) and lo = rn(v - hi), each pair packed (even
// column in the low half): hardware conversions, three instructions per value.
__device__ __forceinline__ void split_bf16x2(float v0, float v1, uint32_t &hi, uint32_t &lo) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(v1), "f"(v0));
    const float r0 = v0 - __uint_as_float(hi << 16), r1 = v1 - __uint_as_float(hi & 0xffff0000u);
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(r1), "f"(r0));
}

// X tile sources: the tile's value at (utterance b, column k0 + k) is
//   XW      src[(k0+k)*Bp + b] * w[k0+k]                  (norm weight)
//   PLAIN   src[(k0+k)*Bp + b]
//   SWIGLU  silu(r g) * (r u), g = src[2(k0+k)*Bp + b], u = src[(2(k0+k)+1)*Bp + b]
enum { SRC_XW = 0, SRC_PLAIN = 1, SRC_SWIGLU = 2 };

// Writes the X tile (Bp rows = utterances, 64 columns = k0..k0+63) into the
// stage as bf16 hi and lo with the 128-byte swizzle: element (b, k) at byte
// (b/8)*1024 + (b%8)*128 + (((k/8) ^ (b%8)) * 16) + (k%8)*2. A group of 2
// builder warps builds a tile: thread gt takes utterance b = gt % Bp and the
// 8-column chunks gt / Bp + i * (64 / Bp); for a fixed column consecutive
// threads read consecutive utterances, which the [feature][Bp] layout of every
// activation buffer makes one coalesced access. All loads of a round (4 chunks,
// 2 for SwiGLU) are issued before the first value is used.
template <int MODE>
__device__ __forceinline__ void build_tile(unsigned char *xs, int Bp, int B, int gt, const float *src,
                                           const float *w, float r, int k0, const QdbBatchArgs &a, int dslot) {
    constexpr int TPR = MODE == SRC_SWIGLU ? 2 : 4;  // chunks per round
    unsigned char *hi = xs, *lo = xs + Bp * 128;
    const int b = gt % Bp, c0 = gt / Bp, cstep = GRP_T / Bp, ntask = 8 / cstep;
    const uint32_t rb = (uint32_t)(b >> 3) * 1024u + (uint32_t)(b & 7) * 128u;
    for (int t0 = 0; t0 < ntask; t0 += TPR) {
        float v[TPR][8], u[MODE == SRC_SWIGLU ? TPR : 1][8];
#pragma unroll
        for (int t = 0; t < TPR; t++) {
            const int k = k0 + (c0 + (t0 + t) * cstep) * 8;
            const bool live = t0 + t < ntask && b < B;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                if (MODE == SRC_SWIGLU) {
                    v[t][i] = live ? ld_l2(src + (size_t)(2 * (k + i)) * Bp + b) : 0.f;
                    u[t][i] = live ? ld_l2(src + (size_t)(2 * (k + i) + 1) * Bp + b) : 0.f;
                } else {
                    v[t][i] = live ? ld_l2(src + (size_t)(k + i) * Bp + b) : 0.f;
                }
            }
        }
#pragma unroll
        for (int t = 0; t < TPR; t++) {
            if (t0 + t >= ntask) break;
            const int cc = c0 + (t0 + t) * cstep;
            if (MODE == SRC_XW) {
                const float4 wa = __ldg(reinterpret_cast<const float4 *>(w + k0 + cc * 8));
                const float4 wb = __ldg(reinterpret_cast<const float4 *>(w + k0 + cc * 8 + 4));
                v[t][0] *= wa.x; v[t][1] *= wa.y; v[t][2] *= wa.z; v[t][3] *= wa.w;
                v[t][4] *= wb.x; v[t][5] *= wb.y; v[t][6] *= wb.z; v[t][7] *= wb.w;
            } else if (MODE == SRC_SWIGLU) {
#pragma unroll
                for (int i = 0; i < 8; i++) v[t][i] = silu_mul(v[t][i] * r, u[t][i] * r);
            }
            uint32_t h[4], l[4];
#pragma unroll
            for (int i = 0; i < 4; i++) split_bf16x2(v[t][2 * i], v[t][2 * i + 1], h[i], l[i]);
            const uint32_t off = rb + (uint32_t)((cc ^ (b & 7)) * 16);
            *reinterpret_cast<uint4 *>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<uint4 *>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
        }
    }
    // generic-proxy writes -> visible to the tensor core's async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
}

// ---------------------------------------------------------------- attention scratch
struct AttnSm {
    float q[8][QDB_HD];      // up to R = 8 query heads of the group
    float knew[QDB_HD], vnew[QDB_HD];
    float qn[QDB_HD], kn[QDB_HD];
    float2 rope[QDB_HD / 2];
    float m[NBLD][8], l[NBLD][8];
    float r1;
    int last;  // this unit merges the splits of its (utterance, KV head)
};

// Per-head RMSNorm then NeoX rotation of one 128-float head in smem, one warp
// (qwen_rms_norm_per_head, qwen_asr_kernels.c:811-873; qwen_apply_rope_neox,
// :1182-1247).
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

__device__ __forceinline__ void bld_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NBLD * 32) : "memory"); }
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 2, %0;" ::"n"(NEPI * 32) : "memory"); }
__device__ __forceinline__ void work_sync() {  // builders + epilogue
    asm volatile("bar.sync 3, %0;" ::"n"((NBLD + NEPI) * 32) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, u64 *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32(dst)),
        "l"(src), "r"(bytes), "r"(su32(bar))
        : "memory");
}

// One attention unit (utterance b, KV head g, split s of S) by the 8 builder
// warps: partial (m, l, o[128]) of each of the R query heads. The unit's keys
// [p0, p1) are contiguous in the cache: thread 0 streams them in 64-key
// chunks (K and V, 32 KB) with cp.async.bulk into two stages of the X ring
// (idle between the QKV and O phases); the first two chunks are requested
// before q/k/v are read. Each warp takes 8 keys of a chunk: 4 lanes per key
// over 32 dims for q.k (16-byte pieces rotated per lane against bank
// conflicts), then 4 dims per lane for p.V; the R query heads share every K/V
// read. This step's own row (position pos) comes from smem, rounded like the
// cache. ach: chunks streamed so far by this CTA (stage / parity of the next).
// Partials go to part in [feature][Bp] layout: o at ((s*qd + head*128 + d) *
// Bp + b), then (m, l) at (qd*S*Bp + ((s*Hq + head)*2 + {0,1}) * Bp + b).
template <int R>
__device__ void attn_unit(const QdbBatchArgs &a, const QdbLayerW &lw, int layer, int b, int g, int s, int S,
                          float r1, AttnSm *sm, float *obuf, unsigned char *stg, u64 *afull, unsigned &ach,
                          const Ctl &c) {
    const QdbDims &d = a.d;
    const int lane = threadIdx.x & 31, warp = (threadIdx.x >> 5) - BLD0, t = threadIdx.x - BLD0 * 32;
    const QdbRowKV rk = a.rows[b];
    const int pos = rk.pos + a.step_base;
    const int ctx = pos + 1;
    const int per = (ctx + S - 1) / S;
    const int p0 = s * per, p1 = min(ctx, p0 + per);
    const int qd = d.Hq * QDB_HD, kvd = d.Hkv * QDB_HD;
    const int Bp = a.Bp;
    const size_t head_base = ((size_t)layer * d.Hkv + g) * (size_t)rk.cap * QDB_HD;
    uint16_t *kc = rk.kc + head_base;
    uint16_t *vc = rk.vc + head_base;
    const bool owns_new = (p0 <= pos && pos < p1);
    const int nch = p1 > p0 ? (p1 - p0 + AK - 1) / AK : 0;
    auto issue = [&](int ci) {
        const unsigned it = ach + (unsigned)ci;
        unsigned char *st = stg + (size_t)(it & 1) * ACHUNK;
        const int k0 = p0 + ci * AK;
        const unsigned bytes = (unsigned)(min(AK, p1 - k0) * QDB_HD * 2);
        mb_expect(&afull[it & 1], 2 * bytes);
        bulk_g2s(st, kc + (size_t)k0 * QDB_HD, bytes, &afull[it & 1]);
        bulk_g2s(st + AK * QDB_HD * 2, vc + (size_t)k0 * QDB_HD, bytes, &afull[it & 1]);
    };
    int issued = 0;  // (thread 0)
    if (t == 0)
        for (; issued < nch && issued < 2; issued++) issue(issued);
    // q/k/v of this utterance (column b of qkv), times the input-norm factor
    for (int i = t; i < (R + 2) * QDB_HD; i += NBLD * 32) {
        const int hh = i / QDB_HD, dd = i % QDB_HD;
        int row;
        float *dst;
        if (hh < R) {
            row = (g * R + hh) * QDB_HD + dd;
            dst = &sm->q[hh][dd];
        } else if (hh == R) {
            row = qd + g * QDB_HD + dd;
            dst = &sm->knew[dd];
        } else {
            row = qd + kvd + g * QDB_HD + dd;
            dst = &sm->vnew[dd];
        }
        *dst = __ldcg(a.qkv + (size_t)row * Bp + b) * r1;
    }
    for (int i = t; i < QDB_HD; i += NBLD * 32) {
        sm->qn[i] = lw.q_norm[i];
        sm->kn[i] = lw.k_norm[i];
    }
    for (int i = t; i < QDB_HD / 2; i += NBLD * 32) sm->rope[i] = a.rope[(size_t)pos * (QDB_HD / 2) + i];
    bld_sync();
    for (int hh = warp; hh < R + 1; hh += NBLD) {
        if (hh < R) head_norm_rope(sm->q[hh], sm->qn, sm->rope, d.eps);
        else head_norm_rope(sm->knew, sm->kn, sm->rope, d.eps);
    }
    bld_sync();
    if (owns_new) {  // the new K/V row, rounded to the cache format
        for (int i = t; i < QDB_HD; i += NBLD * 32) {
            kc[(size_t)pos * QDB_HD + i] = f32_to_kv(sm->knew[i]);
            vc[(size_t)pos * QDB_HD + i] = f32_to_kv(sm->vnew[i]);
        }
    }
    const float scale = 1.0f / sqrtf((float)QDB_HD);
    const int sub = lane & 3, kk = lane >> 2;
    float m[R], l[R], o[R][4];
#pragma unroll
    for (int h = 0; h < R; h++) {
        m[h] = -INFINITY;
        l[h] = 0.f;
#pragma unroll
        for (int e = 0; e < 4; e++) o[h][e] = 0.f;
    }
    for (int ci = 0; ci < nch; ci++) {
        const unsigned it = ach + (unsigned)ci;
        const unsigned char *st = stg + (size_t)(it & 1) * ACHUNK;
        const bool ok = !warp_aborted(c) && mb_wait_warp(&afull[it & 1], (it >> 1) & 1, c, 40);
        if (ok) {
            const int base = p0 + ci * AK + warp * ATT_KEYS;  // this warp's 8 keys
            const int j = base + kk;
            const bool valid = j < p1;
            uint4 kv4[4];
            const int rot = (sub + kk) & 3;
            if (valid) {
                if (j == pos) {
                    const float *kn = sm->knew + sub * 32;
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int uu = (u + rot) & 3;
                        kv4[u] = make_uint4(kv_pack2(kn[uu * 8 + 0], kn[uu * 8 + 1]), kv_pack2(kn[uu * 8 + 2], kn[uu * 8 + 3]),
                                            kv_pack2(kn[uu * 8 + 4], kn[uu * 8 + 5]), kv_pack2(kn[uu * 8 + 6], kn[uu * 8 + 7]));
                    }
                } else {
                    const uint4 *kp = reinterpret_cast<const uint4 *>(st + (size_t)(warp * ATT_KEYS + kk) * QDB_HD * 2) +
                                      sub * 4;
#pragma unroll
                    for (int u = 0; u < 4; u++) kv4[u] = kp[(u + rot) & 3];
                }
            }
            uint2 vv[ATT_KEYS];
#pragma unroll
            for (int tt = 0; tt < ATT_KEYS; tt++) {
                const int jt = base + tt;
                if (jt >= p1) vv[tt] = make_uint2(0u, 0u);
                else if (jt == pos)
                    vv[tt] = make_uint2(kv_pack2(sm->vnew[lane * 4], sm->vnew[lane * 4 + 1]),
                                        kv_pack2(sm->vnew[lane * 4 + 2], sm->vnew[lane * 4 + 3]));
                else
                    vv[tt] = *reinterpret_cast<const uint2 *>(st + AK * QDB_HD * 2 +
                                                              (size_t)(warp * ATT_KEYS + tt) * QDB_HD * 2 + lane * 8);
            }
            float sc[R];
#pragma unroll
            for (int h = 0; h < R; h++) {
                float a0 = 0.f, a1 = 0.f;
                if (valid) {
                    const float *qv = sm->q[h] + sub * 32;
#pragma unroll
                    for (int u = 0; u < 4; u += 2) {
                        const int ua = (u + rot) & 3, ub = (u + 1 + rot) & 3;
                        a0 = dot8_kv(kv4[u], *reinterpret_cast<const float4 *>(qv + ua * 8),
                                     *reinterpret_cast<const float4 *>(qv + ua * 8 + 4), a0);
                        a1 = dot8_kv(kv4[u + 1], *reinterpret_cast<const float4 *>(qv + ub * 8),
                                     *reinterpret_cast<const float4 *>(qv + ub * 8 + 4), a1);
                    }
                }
                float acc = a0 + a1;
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
                const float corr = (mn == -INFINITY) ? 1.f : expf(m[h] - mn);
                const float p = valid ? expf(sc[h] - mn) : 0.f;
                float ps = p;
                ps += __shfl_xor_sync(0xffffffffu, ps, 4);
                ps += __shfl_xor_sync(0xffffffffu, ps, 8);
                ps += __shfl_xor_sync(0xffffffffu, ps, 16);
                l[h] = l[h] * corr + ps;
#pragma unroll
                for (int e = 0; e < 4; e++) o[h][e] *= corr;
#pragma unroll
                for (int tt = 0; tt < ATT_KEYS; tt++) {
                    const float pt = __shfl_sync(0xffffffffu, p, tt * 4);
                    o[h][0] = fmaf(pt, kvlo(vv[tt].x), o[h][0]);
                    o[h][1] = fmaf(pt, kvhi(vv[tt].x), o[h][1]);
                    o[h][2] = fmaf(pt, kvlo(vv[tt].y), o[h][2]);
                    o[h][3] = fmaf(pt, kvhi(vv[tt].y), o[h][3]);
                }
                m[h] = mn;
            }
        }
        bld_sync();  // every warp is done with this stage
        if (t == 0 && ci + 2 < nch && !*c.abort) issue(issued++);
    }
    if (t == 0)  // after an abort, the copies still in flight land before the stage is reused or the CTA exits
        for (int ci = issued > 2 ? issued - 2 : 0; ci < issued; ci++) {
            const unsigned it = ach + (unsigned)ci;
            mb_wait(&afull[it & 1], (it >> 1) & 1, c, false, 41);
        }
    ach += (unsigned)nch;
    // merge the warps' partials; write the unit's partial of each query head
#pragma unroll
    for (int h = 0; h < R; h++) {
        if (lane == 0) {
            sm->m[warp][h] = m[h];
            sm->l[warp][h] = l[h];
        }
#pragma unroll
        for (int e = 0; e < 4; e++) obuf[((size_t)warp * R + h) * QDB_HD + lane * 4 + e] = o[h][e];
    }
    bld_sync();
    // One split: the normalised output goes straight to attn [qd][Bp]. Several:
    // each unit writes its partial; the last of the S units of (b, g) to
    // finish (a counter per (b, g), reset by that unit) merges them.
    float *part_ml = a.part + (size_t)qd * S * Bp;
    for (int i = t; i < R * QDB_HD; i += NBLD * 32) {
        const int h = i / QDB_HD, dd = i % QDB_HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NBLD; w++) M = fmaxf(M, sm->m[w][h]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < NBLD; w++) {
                const float f = expf(sm->m[w][h] - M);
                L += sm->l[w][h] * f;
                O += obuf[((size_t)w * R + h) * QDB_HD + dd] * f;
            }
        }
        const int head = g * R + h;
        if (S == 1) {
            a.attn[((size_t)head * QDB_HD + dd) * Bp + b] = L > 0.f ? O / L : 0.f;
        } else {
            a.part[((size_t)s * qd + head * QDB_HD + dd) * Bp + b] = O;
            if (dd == 0) {
                part_ml[(((size_t)s * d.Hq + head) * 2 + 0) * Bp + b] = M;
                part_ml[(((size_t)s * d.Hq + head) * 2 + 1) * Bp + b] = L;
            }
        }
    }
    if (S > 1) {
        __threadfence();
        bld_sync();
        if (t == 0) {
            unsigned *cnt = a.acnt + (size_t)b * d.Hkv + g;
            const unsigned prev = atomicAdd(cnt, 1u);
            sm->last = prev == (unsigned)(S - 1);
            if (sm->last) atomicExch(cnt, 0u);
            __threadfence();
        }
        bld_sync();
        if (sm->last) {
            for (int i = t; i < R * QDB_HD; i += NBLD * 32) {
                const int h = i / QDB_HD, dd = i % QDB_HD, head = g * R + h;
                float M = -INFINITY;
                for (int q = 0; q < S; q++) M = fmaxf(M, ld_l2(part_ml + (((size_t)q * d.Hq + head) * 2) * Bp + b));
                float L = 0.f, O = 0.f;
                if (M != -INFINITY)
                    for (int q = 0; q < S; q++) {
                        const float mq = ld_l2(part_ml + (((size_t)q * d.Hq + head) * 2) * Bp + b);
                        const float f = mq == -INFINITY ? 0.f : expf(mq - M);
                        L += ld_l2(part_ml + (((size_t)q * d.Hq + head) * 2 + 1) * Bp + b) * f;
                        O += ld_l2(a.part + ((size_t)q * qd + head * QDB_HD + dd) * Bp + b) * f;
                    }
                a.attn[((size_t)head * QDB_HD + dd) * Bp + b] = L > 0.f ? O / L : 0.f;
            }
        }
    }
    bld_sync();  // smem reused by the next unit
}

// 1/rms of utterance b's residual column (h values, stride Bp), by one warp.
__device__ float row_inv_rms(const float *x, int h, int Bp, int b, float eps) {
    const int lane = threadIdx.x & 31;
    float ss = 0.f;
    for (int k = lane; k < h; k += 32) {
        const float v = __ldcg(x + (size_t)k * Bp + b);
        ss += v * v;
    }
    ss = warp_sum(ss);
    return 1.0f / sqrtf(ss / (float)h + eps);
}

// ---------------------------------------------------------------- the kernel
template <int R>
__global__ void __launch_bounds__(NTHREADS, 1) bstep_kernel(const QdbBatchArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_dyn[];
    __shared__ Smem S_;
    __shared__ __align__(16) QdbLayerW layers[MAX_LAYERS];
    __shared__ u64 lm_best[NEPI][64];  // per epilogue warp: best key per utterance (lm_head)
    __shared__ float lm_r3[64];

    const QdbDims &d = a.d;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int Bp = a.Bp, B = a.B, G = gridDim.x;
    const int NSW = a.nsw;
    unsigned char *smem = smem_dyn + ((1024u - (su32(smem_dyn) & 1023u)) & 1023u);
    unsigned char *wring = smem;
    unsigned char *xring = wring + (size_t)NSW * W_TILE;
    const int XST = 2 * Bp * 128;  // one X stage: hi + lo
    const int xring_bytes = NSX * XST > XRING_MIN ? NSX * XST : XRING_MIN;
    AttnSm *asm_ = reinterpret_cast<AttnSm *>(xring + (size_t)xring_bytes);
    float *obuf = reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(asm_) + sizeof(AttnSm));
    const Ctl c{&S_.abort, a.err};
    const unsigned ep = a.epoch;
    const int step = a.step_base;

    if (threadIdx.x == 0) {
        S_.abort = 0;
        for (int i = 0; i < NSW; i++) {
            mb_init(&S_.wfull[i], 1);
            mb_init(&S_.wempty[i], 1);
        }
        for (int i = 0; i < NSX; i++) {
            mb_init(&S_.xfull[i], GRP_WARPS);  // both warps of the owning builder group write the tile
            mb_init(&S_.xempty[i], 1);
        }
        for (int i = 0; i < 2; i++) mb_init(&S_.afull[i], 1);
        for (int i = 0; i < NSLOT; i++) {
            mb_init(&S_.accfull[i], 1);
            mb_init(&S_.accempty[i], NEPI);
        }
        mb_init(&S_.lmfull, 1);
        mb_init(&S_.lmempty, NEPI);
        mb_init(&S_.mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    {
        const int words = d.L * (int)(sizeof(QdbLayerW) / 8);
        const u64 *src = reinterpret_cast<const u64 *>(a.layers);
        u64 *dst = reinterpret_cast<u64 *>(layers);
        for (int i = threadIdx.x; i < words; i += NTHREADS) dst[i] = src[i];
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(su32(&S_.tmem))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S_.tmem;
    const int L = d.L;

    if (warp == 0) {
        // ================================================================ producer
        if (lane == 0) {
            uint64_t pol = 0;
            asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
            unsigned wi = 0;
            bool ok = true;
            // weight tile blk of the pre-tiled copy: 16 KB, contiguous, already in
            // the swizzled shared-memory layout -> one 1D bulk copy
            auto issue = [&](size_t blk) -> bool {
                const int s = wi % NSW;
                if (wi >= (unsigned)NSW && !mb_wait(&S_.wempty[s], ((wi / NSW) - 1) & 1, c, true, 1)) return false;
                mb_expect(&S_.wfull[s], W_TILE);
                bulk_g2s_pol(wring + (size_t)s * W_TILE, a.wt + blk * (W_TILE / 2), W_TILE, &S_.wfull[s], pol);
                wi++;
                progress(a, 0, wi);
                return true;
            };
            size_t base = 0;
            for (int layer = 0; layer < L && ok; layer++)
                for (int m = 0; m < 4 && ok; m++) {
                    const Mat M = mat_of(d, m);
                    int i0, i1;
                    share(M, i0, i1);
                    for (int i = i0; i < i1 && ok; i++) ok = issue(base + (size_t)i);
                    base += (size_t)M.T * M.KB;
                }
            if (ok) {
                const Mat M = mat_of(d, 4);
                for (int grp = blockIdx.x; grp < lm_groups(M) && ok; grp += G) {
                    const int nt = min(NACC, M.T - grp * NACC);
                    for (int kb = 0; kb < M.KB && ok; kb++)
                        for (int j = 0; j < nt && ok; j++)
                            ok = issue(base + (size_t)grp * NACC * M.KB + (size_t)kb * nt + j);
                }
            }
            // drain: the latest copy issued into each stage lands before exit
            for (unsigned k = 0; k < (unsigned)NSW && k < wi; k++) {
                const unsigned i = wi - 1 - k;
                mb_wait(&S_.wfull[i % NSW], (i / NSW) & 1, c, false, 2);
            }
        }
    } else if (warp == 1) {
        // ================================================================ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = instr_desc(128, 2 * Bp);
            unsigned wi = 0, xi = 0, seg = 0;
            int l1_item = -1000;  // item index within layer 1 (detail stamps)
            bool ok = true;
            // One projection item: W stage wi x X stage xi into the segment's slot:
            // 4 MMAs (k-steps) over NCH accumulator chains at slot + chain * 2Bp.
            const int NCH = nchain(Bp);
            auto item = [&](uint32_t slot_base, bool first) -> bool {
                const int ws = wi % NSW, xs = xi % NSX;
                progress(a, 8, 3);
                if (l1_item >= 0 && l1_item < 64) dstamp(a, 256 + l1_item);  // W wait begins
                if (!mb_wait(&S_.wfull[ws], (wi / NSW) & 1, c, true, 3)) return false;
                if (l1_item >= 0 && l1_item < 64) dstamp(a, 320 + l1_item);  // W ready
                progress(a, 8, 4);
                if (!mb_wait(&S_.xfull[xs], (xi / NSX) & 1, c, true, 4)) return false;
                progress(a, 8, 0);
                dstamp(a, l1_item++);
                tc_fence_after();
                const uint32_t wb = su32(wring + (size_t)ws * W_TILE);
                const uint32_t xb = su32(xring + (size_t)xs * XST);
#pragma unroll
                for (int k = 0; k < 4; k++)
                    mma_bf16(slot_base + (uint32_t)((k % NCH) * 2 * Bp), sm_desc(wb + k * 32), sm_desc(xb + k * 32), idesc,
                             (first && k < NCH) ? 0u : 1u);
                mma_commit(&S_.wempty[ws]);
                mma_commit(&S_.xempty[xs]);
                wi++;
                xi++;
                progress(a, 1, wi);
                progress(a, 2, xi);
                return true;
            };
            auto begin_seg = [&](unsigned sg) -> bool {
                const int slot = sg % NSLOT;
                progress(a, 8, 5);
                if (sg >= (unsigned)NSLOT && !mb_wait(&S_.accempty[slot], ((sg / NSLOT) - 1) & 1, c, true, 5))
                    return false;
                tc_fence_after();
                progress(a, 3, sg + 1);
                return true;
            };
            for (int layer = 0; layer < L && ok; layer++)
                for (int m = 0; m < 4 && ok; m++) {
                    if (layer == 1 && m == 0) l1_item = 0;
                    if (layer == 2 && m == 0) l1_item = -1000;
                    const Mat M = mat_of(d, m);
                    int i0, i1;
                    share(M, i0, i1);
                    for (int i = i0; i < i1 && ok;) {
                        const int tile = i / M.KB;
                        const int iend = min(i1, (tile + 1) * M.KB);
                        if (!(ok = begin_seg(seg))) break;
                        const uint32_t sb = tmem + (uint32_t)((seg % NSLOT) * NCH * 2 * Bp);
                        for (int k = i; k < iend && ok; k++) ok = item(sb, k == i);
                        if (ok) mma_commit(&S_.accfull[seg % NSLOT]);
                        seg++;
                        i = iend;
                    }
                }
            // lm_head rounds reuse all of TMEM: the projection slots drain first
            for (unsigned sg = seg > NSLOT ? seg - NSLOT : 0; sg < seg && ok; sg++)
                ok = mb_wait(&S_.accempty[sg % NSLOT], (sg / NSLOT) & 1, c, true, 5);
            if (ok) {
                tc_fence_after();
                const Mat M = mat_of(d, 4);
                l1_item = 384;  // detail stamps of the lm_head k-blocks
                unsigned rnd = 0;
                for (int grp = blockIdx.x; grp < lm_groups(M) && ok; grp += G, rnd++) {
                    const int nt = min(NACC, M.T - grp * NACC);
                    if (rnd > 0 && !(ok = mb_wait(&S_.lmempty, (rnd - 1) & 1, c, true, 5))) break;
                    tc_fence_after();
                    // per k-block: the round's nt weight tiles and one X tile; MMAs
                    // interleaved over the nt tiles (independent accumulators)
                    for (int kb = 0; kb < M.KB && ok; kb++) {
                        for (int j = 0; j < nt && ok; j++)
                            ok = mb_wait(&S_.wfull[(wi + j) % NSW], ((wi + j) / NSW) & 1, c, true, 3);
                        if (ok) ok = mb_wait(&S_.xfull[xi % NSX], (xi / NSX) & 1, c, true, 4);
                        if (!ok) break;
                        dstamp(a, l1_item++);
                        tc_fence_after();
                        const uint32_t xb = su32(xring + (size_t)(xi % NSX) * XST);
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            for (int j = 0; j < nt; j++) {
                                const uint32_t wb = su32(wring + (size_t)((wi + j) % NSW) * W_TILE);
                                mma_bf16(tmem + (uint32_t)(j * 2 * Bp), sm_desc(wb + k * 32), sm_desc(xb + k * 32),
                                         idesc, (kb == 0 && k == 0) ? 0u : 1u);
                            }
                        for (int j = 0; j < nt; j++) mma_commit(&S_.wempty[(wi + j) % NSW]);
                        mma_commit(&S_.xempty[xi % NSX]);
                        wi += nt;
                        xi++;
                        progress(a, 1, wi);
                        progress(a, 2, xi);
                    }
                    if (ok) mma_commit(&S_.lmfull);
                }
            }
            // every MMA issued by this thread completes before TMEM is released
            mma_commit(&S_.mma_done);
            mb_wait(&S_.mma_done, 0, c, false, 6);
        }
    } else if (warp < BLD0) {
        // ================================================================ epilogue
        const int q = warp & 3;  // TMEM lanes 32q..32q+31
        const int et = threadIdx.x - EPI0 * 32;
        unsigned seg = 0;
        int l1_seg = -1000;
        bool ok = true;
        // waits for accumulator slot of segment sg; uniform over the warp
        auto acc_ready = [&](unsigned sg) -> bool {
            if (!ok || warp_aborted(c)) return false;
            if (!mb_wait_warp(&S_.accfull[sg % NSLOT], (sg / NSLOT) & 1, c, 7)) return false;
            tc_fence_after();
            return true;
        };
        auto acc_release = [&](unsigned sg) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mb_arrive(&S_.accempty[sg % NSLOT]);
            if (warp == EPI0 && lane == 0) progress(a, 4, sg + 1);
        };
        auto phase_done = [&](int idx) {
            __threadfence();
            epi_sync();
            if (et == 0) signal(a.cnt + idx);
        };
        auto epi_stamp = [&](int idx) {
            if (et == 0) stamp(a, idx);
        };
        // ---- set-up: clear the accumulation targets of layer 0 (qkv, gu)
        {
            const size_t nq = (size_t)(d.Hq + 2 * d.Hkv) * QDB_HD * Bp, ng = (size_t)2 * d.I * Bp;
            const size_t q0 = nq * blockIdx.x / G, q1 = nq * (blockIdx.x + 1) / G;
            const size_t g0 = ng * blockIdx.x / G, g1 = ng * (blockIdx.x + 1) / G;
            for (size_t i = q0 + et; i < q1; i += NEPI * 32) a.qkv[i] = 0.f;
            for (size_t i = g0 + et; i < g1; i += NEPI * 32) a.gu[i] = 0.f;
        }
        __threadfence();
        work_sync();  // with the builders' embedding writes: then one signal
        for (int layer = 0; layer < L; layer++) {
            for (int m = 0; m < 4; m++) {
                const Mat M = mat_of(d, m);
                float *out = m == 0 ? a.qkv : (m == 2 ? a.gu : a.x);
                if (warp == EPI0 && lane == 0) progress(a, 5, (unsigned)(layer * 8 + m + 1));
                if (m == 0 && (int)blockIdx.x < B) {
                    // input-norm statistic of utterance blockIdx.x (after the previous layer)
                    if (warp == EPI0 && wait_count_warp(a.cnt + (layer ? cidx(layer - 1, 4) : 0), G, c, 20)) {
                        const float r = row_inv_rms(a.x, d.h, Bp, blockIdx.x, d.eps);
                        if (lane == 0) st_tag(a.stats + ((size_t)layer * 3 + 0) * 64 + blockIdx.x, r, ep);
                    }
                }
                if (m == 1) {
                    // attention of this layer is complete everywhere: qkv is free, and so is gu
                    // (read by the previous layer's down builders): clear this CTA's slices
                    if (wait_count_warp(a.cnt + cidx(layer, 1), G, c, 21)) {
                        const size_t nq = (size_t)(d.Hq + 2 * d.Hkv) * QDB_HD * Bp, ng = (size_t)2 * d.I * Bp;
                        const size_t q0 = nq * blockIdx.x / G, q1 = nq * (blockIdx.x + 1) / G;
                        const size_t g0 = ng * blockIdx.x / G, g1 = ng * (blockIdx.x + 1) / G;
                        for (size_t i = q0 + et; i < q1; i += NEPI * 32) a.qkv[i] = 0.f;
                        if (layer > 0)
                            for (size_t i = g0 + et; i < g1; i += NEPI * 32) a.gu[i] = 0.f;
                    }
                }
                if (m == 2 && (int)blockIdx.x < B) {
                    // post-attention-norm statistic (x after this layer's O)
                    if (warp == EPI0 && wait_count_warp(a.cnt + cidx(layer, 2), G, c, 22)) {
                        const float r = row_inv_rms(a.x, d.h, Bp, blockIdx.x, d.eps);
                        if (lane == 0) st_tag(a.stats + ((size_t)layer * 3 + 1) * 64 + blockIdx.x, r, ep);
                    }
                }
                int i0, i1;
                share(M, i0, i1);
                if (layer == 1 && m == 0) l1_seg = 0;
                if (layer == 2) l1_seg = -1000;
                for (int i = i0; i < i1;) {
                    const int tile = i / M.KB;
                    const int iend = min(i1, (tile + 1) * M.KB);
                    const bool rdy = acc_ready(seg);
                    if (et == 0) dstamp(a, 192 + l1_seg);
                    if (rdy) {
                        const int NCH = nchain(Bp);
                        const uint32_t tbase =
                            tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)((seg % NSLOT) * NCH * 2 * Bp);
                        const int row = tile * 128 + 32 * q + lane;
                        float *dst = out + (size_t)row * Bp;
                        for (int c0 = 0; c0 < Bp; c0 += 16) {
                            float v[16], w[16];
                            tmem_ld16(tbase + (uint32_t)c0, v);
                            // the lo half, then the other chains (both halves)
                            for (int k = 0; k < NCH; k++)
                                for (int hl = (k == 0); hl < 2; hl++) {
                                    tmem_ld16(tbase + (uint32_t)(k * 2 * Bp + hl * Bp + c0), w);
#pragma unroll
                                    for (int j = 0; j < 16; j++) v[j] += w[j];
                                }
                            if (row < M.N)
#pragma unroll
                                for (int j = 0; j < 16; j += 4) red_add_v4(dst + c0 + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
                        }
                    } else {
                        ok = false;
                    }
                    acc_release(seg);
                    if (et == 0) dstamp(a, 224 + l1_seg);
                    l1_seg++;
                    seg++;
                    i = iend;
                }
                phase_done(cidx(layer, m == 0 ? 0 : m + 1));
                if (m == 0) epi_stamp(layer * 8 + 5);
                if (m == 1) epi_stamp(layer * 8 + 6);
                if (m == 3) epi_stamp(layer * 8 + 7);
            }
        }
        // ---- lm_head: scaled logits, running argmax per utterance
        const Mat M = mat_of(d, 4);
        if (warp == EPI0 && lane == 0) progress(a, 5, (unsigned)(L * 8 + 5));
        if ((int)blockIdx.x < B && warp == EPI0 && wait_count_warp(a.cnt + cidx(L - 1, 4), G, c, 23)) {
            const float r = row_inv_rms(a.x, d.h, Bp, blockIdx.x, d.eps);
            if (lane == 0) st_tag(a.stats + ((size_t)L * 3 + 2) * 64 + blockIdx.x, r, ep);
        }
        for (int b = et; b < Bp; b += NEPI * 32)
            lm_r3[b] = b < B ? poll_tag(a.stats + ((size_t)L * 3 + 2) * 64 + b, ep, c, 24) : 0.f;
        // Per 16-column chunk of a tile: the warp's 32 rows x 16 logits go
        // through a padded smem buffer; lanes l and l + 16 scan rows 0-15 /
        // 16-31 of column l in increasing row order (strict >: the lowest row
        // wins an exact tie) and merge with one shuffle. Lane l (< 16) keeps
        // the best key of columns c0 + l, c0 in {0, 16, 32, 48}.
        float *tbuf = reinterpret_cast<float *>(asm_) + (size_t)q * 32 * 17;  // attention scratch is idle now
        u64 best[4] = {0ull, 0ull, 0ull, 0ull};
        epi_sync();
        unsigned rnd = 0;
        for (int grp = blockIdx.x; grp < lm_groups(M); grp += G, rnd++) {
            const int r0 = grp * NACC, nt = min(NACC, M.T - r0);
            bool rdy = ok && !warp_aborted(c) && mb_wait_warp(&S_.lmfull, rnd & 1, c, 7);
            if (!rdy) ok = false;
            tc_fence_after();
            for (int j = 0; j < nt && rdy; j++) {
                const int tile = r0 + j;
                const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(j * 2 * Bp);
                const int row = tile * 128 + 32 * q + lane;
                const bool live = row < M.N && !(a.mask_eos && (row == QDB_ENDOFTEXT || row == QDB_IM_END));
#pragma unroll
                for (int cq = 0; cq < 4; cq++) {
                    const int c0 = cq * 16;
                    if (c0 >= Bp) break;
                    float v[16], w[16];
                    tmem_ld16(tbase + (uint32_t)c0, v);
                    tmem_ld16(tbase + (uint32_t)(Bp + c0), w);  // lo half
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) v[jj] += w[jj];
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) {
                        const int b = c0 + jj;
                        const float lg = v[jj] * lm_r3[b];
                        if (a.logits_out && row < M.N && b < B) a.logits_out[(size_t)b * M.N + row] = lg;
                        tbuf[lane * 17 + jj] = (live && b < B && !isnan(lg)) ? lg : -INFINITY;
                    }
                    __syncwarp();
                    const int col = lane & 15, rbase = (lane >> 4) * 16;
                    float bv = -INFINITY;
                    int br = -1;
#pragma unroll
                    for (int rr = 0; rr < 16; rr++) {
                        const float x = tbuf[(rbase + rr) * 17 + col];
                        if (x > bv) {
                            bv = x;
                            br = rbase + rr;
                        }
                    }
                    u64 key = br >= 0 ? argmax_key(bv, tile * 128 + 32 * q + br) : 0ull;
                    const u64 other = __shfl_xor_sync(0xffffffffu, key, 16);
                    key = other > key ? other : key;
                    best[cq] = key > best[cq] ? key : best[cq];
                    __syncwarp();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mb_arrive(&S_.lmempty);
        }
        epi_stamp(8 * L + 1);
        // combine the 4 epilogue warps, then the CTA's candidates go to the global keys
        if (lane < 16)
#pragma unroll
            for (int cq = 0; cq < 4; cq++) lm_best[q][cq * 16 + lane] = best[cq];
        epi_sync();
        for (int b = et; b < B; b += NEPI * 32) {
            u64 k = 0ull;
#pragma unroll
            for (int w = 0; w < NEPI; w++) k = lm_best[w][b] > k ? lm_best[w][b] : k;
            if (k) atomicMax(a.best + b, k);
        }
    } else {
        // ================================================================ builders
        const int bw = warp - BLD0;  // builder warp 0..7
        const int bt = threadIdx.x - BLD0 * 32;
        unsigned xi = 0;
        // ---- set-up: residual x = embedding rows (column b), [h][Bp]
        {
            const size_t n = (size_t)d.h * Bp;
            const size_t i0 = n * blockIdx.x / G, i1 = n * (blockIdx.x + 1) / G;
            for (size_t i = i0 + bt; i < i1; i += NBLD * 32) {
                const int k = (int)(i / Bp), b = (int)(i % Bp);
                float v = 0.f;
                if (b < B) {
                    if (a.tok_in) {
                        int tok = a.tok_in[(size_t)step * B + b];
                        if (tok < 0 || tok >= d.V) {
                            set_error(a.err, QDB_ERR_BAD_ARG);
                            tok = 0;
                        }
                        v = __uint_as_float(((uint32_t)a.embed[(size_t)tok * d.h + k]) << 16);
                    } else {
                        v = a.x_in[(size_t)b * d.h + k];
                    }
                }
                a.x[i] = v;
            }
        }
        __threadfence();
        work_sync();
        if (bt == 0) {
            __threadfence();
            signal(a.cnt + 0);
        }
        // X tile xi is built by builder group xi % NGRP (2 warps) into stage
        // xi % NSX, which only that group ever writes: a group waits for its
        // own stage's previous tile, so its parity wait cannot alias an older
        // phase. Up to NGRP tiles are built at once.
        const int grp = bw / GRP_WARPS, gt = bt % GRP_T;
        int l1_tile = -1000;  // X tile index within layer 1 (detail stamps)
        const int my_b = gt % Bp;  // the utterance this thread fills in every tile
        auto x_tile = [&](int mode, const float *src, const float *w, float r, int k0) {
            const int s = xi % NSX;
            if ((int)(xi % NGRP) == grp && !warp_aborted(c)) {
                if (lane == 0) progress(a, 9 + bw, xi | 0x80000000u);
                const bool ok = xi < (unsigned)NSX || mb_wait_warp(&S_.xempty[s], ((xi / NSX) - 1) & 1, c, 8);
                if (lane == 0) progress(a, 9 + bw, xi);
                if (ok) {
                    if (gt == 0) dstamp(a, 64 + l1_tile);
                    unsigned char *xs = xring + (size_t)s * XST;
                    const int ds = 256 + l1_tile;
                    if (mode == SRC_XW) build_tile<SRC_XW>(xs, Bp, B, gt, src, w, r, k0, a, ds);
                    else if (mode == SRC_PLAIN) build_tile<SRC_PLAIN>(xs, Bp, B, gt, src, w, r, k0, a, ds);
                    else build_tile<SRC_SWIGLU>(xs, Bp, B, gt, src, w, r, k0, a, ds);
                    if (gt == 0) dstamp(a, 128 + l1_tile);
                    if (lane == 0) {
                        mb_arrive(&S_.xfull[s]);
                        if ((bw & 1) == 0) progress(a, 6, xi + 1);
                    }
                }
            }
            xi++;
            l1_tile++;
        };
        // phase start: one warp polls the counter, the builders then move together
        auto phase_wait = [&](int idx, int site) {
            if (bw == 0) wait_count_warp(a.cnt + idx, G, c, site);
            bld_sync();
        };
        unsigned ach = 0;  // attention chunks streamed by this CTA
        for (int layer = 0; layer < L; layer++) {
            const QdbLayerW &lw = layers[layer];
            l1_tile = layer == 1 ? 0 : -1000;
            // ---- QKV: X = x * w_in
            if (bt == 0) progress(a, 7, (unsigned)(layer * 8 + 1));
            {
                const Mat M = mat_of(d, 0);
                int i0, i1;
                share(M, i0, i1);
                phase_wait(layer ? cidx(layer - 1, 4) : 0, 30);
                if (bt == 0) stamp(a, layer * 8 + 0);
                for (int i = i0; i < i1; i++) {
                    const int k0 = (i % M.KB) * 64;
                    x_tile(SRC_XW, a.x, lw.in_norm, 0.f, k0);
                }
                if (bt == 0) stamp(a, layer * 8 + 1);
            }
            // ---- attention units
            if (bt == 0) progress(a, 7, (unsigned)(layer * 8 + 2));
            {
                const int Sp = a.splits;
                const int units = B * d.Hkv * Sp;
                phase_wait(cidx(layer, 0), 31);
                if (bt == 0) stamp(a, layer * 8 + 2);
                for (int u = blockIdx.x; u < units; u += G) {
                    const int b = u / (d.Hkv * Sp), g = (u / Sp) % d.Hkv, s = u % Sp;
                    if (bt == 0) asm_->r1 = poll_tag(a.stats + ((size_t)layer * 3 + 0) * 64 + b, ep, c, 32);
                    bld_sync();
                    const float r1 = asm_->r1;
                    const QdbRowKV rk = a.rows[b];
                    const int pos = rk.pos + step;
                    if (!check_or_record(pos < rk.cap && pos < a.rope_cap, a.err, 2, pos, rk.cap)) {
                        *c.abort = 1;
                        break;
                    }
                    attn_unit<R>(a, lw, layer, b, g, s, Sp, r1, asm_, obuf, xring, S_.afull, ach, c);
                }
                __threadfence();
                bld_sync();
                if (bt == 0) {
                    stamp(a, layer * 8 + 3);
                    signal(a.cnt + cidx(layer, 1));
                }
            }
            // ---- O: X = merged attention output (splits combined per utterance)
            if (bt == 0) progress(a, 7, (unsigned)(layer * 8 + 3));
            {
                const Mat M = mat_of(d, 1);
                int i0, i1;
                share(M, i0, i1);
                phase_wait(cidx(layer, 1), 33);
                if (bt == 0) stamp(a, layer * 8 + 4);
                for (int i = i0; i < i1; i++) {
                    const int k0 = (i % M.KB) * 64;
                    x_tile(SRC_PLAIN, a.attn, nullptr, 0.f, k0);
                }
            }
            // ---- GU: X = x * w_post (after this layer's O)
            if (bt == 0) progress(a, 7, (unsigned)(layer * 8 + 4));
            {
                const Mat M = mat_of(d, 2);
                int i0, i1;
                share(M, i0, i1);
                phase_wait(cidx(layer, 2), 34);
                for (int i = i0; i < i1; i++) {
                    const int k0 = (i % M.KB) * 64;
                    x_tile(SRC_XW, a.x, lw.post_norm, 0.f, k0);
                }
            }
            // ---- DOWN: X = silu(r g) * (r u)
            if (bt == 0) progress(a, 7, (unsigned)(layer * 8 + 5));
            {
                const Mat M = mat_of(d, 3);
                int i0, i1;
                share(M, i0, i1);
                float r2 = 0.f;  // post-attention-norm factor of this thread's utterance
                phase_wait(cidx(layer, 3), 35);
                if (i1 > i0 && my_b < B) r2 = poll_tag(a.stats + ((size_t)layer * 3 + 1) * 64 + my_b, ep, c, 36);
                for (int i = i0; i < i1; i++) {
                    const int k0 = (i % M.KB) * 64;
                    x_tile(SRC_SWIGLU, a.gu, nullptr, r2, k0);
                }
            }
        }
        // ---- lm_head: X = x * w_final (the 1/rms factor scales the logits)
        if (bt == 0) progress(a, 7, (unsigned)(L * 8 + 6));
        {
            const Mat M = mat_of(d, 4);
            phase_wait(cidx(L - 1, 4), 37);
            if (bt == 0) stamp(a, 8 * L + 0);
            for (int grp = blockIdx.x; grp < lm_groups(M); grp += G)
                for (int kb = 0; kb < M.KB; kb++) {
                    const int k0 = kb * 64;
                    x_tile(SRC_XW, a.x, a.final_norm, 0.f, k0);
                }
        }
    }

    // ---------------------------------------------------------------- wind-down
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
    if (threadIdx.x == 0) {
        stamp(a, 8 * L + 2);
        __threadfence();
        const unsigned prev = atomicAdd(a.done, 1u);
        if (prev == gridDim.x - 1) {
            // every CTA has passed all of its waits: publish the tokens, clear the state
            __threadfence();
            for (int b = 0; b < B; b++) {
                const u64 k = atomicExch(a.best + b, 0ull);
                if (k == 0ull) set_error(a.err, QDB_ERR_BAD_ARG);  // no candidate (aborted step)
                a.tok_out[(size_t)step * B + b] = k ? argmax_key_index(k) : 0;
            }
            for (int i = 0; i < a.n_cnt; i++) a.cnt[i] = 0u;
            __threadfence();
            atomicExch(a.done, 0u);
        }
    }
}

// Pre-tiled weight copy: block blk = one 128-row x 64-column tile in the
// shared-memory layout the MMA reads (K-major, 128-byte swizzle: row r,
// 16-byte chunk c at (r/8)*1024 + (r%8)*128 + ((c ^ (r%8)) * 16)); rows past
// the matrix are zero. One thread per 16-byte chunk.
__global__ void tile_weights_kernel(const uint16_t *__restrict__ w, int N, int K, uint16_t *__restrict__ out,
                                    int lm_order) {
    const int T = (N + 127) / 128, KB = K / 64;
    const size_t nchunks = (size_t)T * KB * 1024;  // 1024 chunks of 16 bytes per tile
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nchunks; i += (size_t)gridDim.x * blockDim.x) {
        const size_t blk = i >> 10;
        const int r = (int)((i >> 3) & 127), cc = (int)(i & 7);
        int tile, kb;
        if (!lm_order) {
            tile = (int)(blk / KB);
            kb = (int)(blk % KB);
        } else {  // groups of NACC tiles, kb-outer inside a group
            const int grp = (int)(blk / ((size_t)NACC * KB));
            const int nt = min(NACC, T - grp * NACC);
            const int in = (int)(blk - (size_t)grp * NACC * KB);
            kb = in / nt;
            tile = grp * NACC + in % nt;
        }
        const int row = tile * 128 + r;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (row < N) v = *reinterpret_cast<const uint4 *>(w + (size_t)row * K + kb * 64 + cc * 8);
        unsigned char *dst = reinterpret_cast<unsigned char *>(out + blk * (W_TILE / 2));
        *reinterpret_cast<uint4 *>(dst + (r >> 3) * 1024 + (r & 7) * 128 + ((cc ^ (r & 7)) << 4)) = v;
    }
}

}  // namespace

extern "C" size_t qdb_bstep_tiled_elems(int N, int K) { return (size_t)((N + 127) / 128) * (K / 64) * (W_TILE / 2); }

// Writes the pre-tiled copy of one bf16 [N, K] matrix (K % 64 == 0) to out.
// lm_order: the lm_head's group order; otherwise tile-major, k-blocks inner.
extern "C" cudaError_t qdb_bstep_tile_weights(const uint16_t *w, int N, int K, uint16_t *out, int lm_order,
                                              cudaStream_t st) {
    if (K % 64 || N <= 0) return cudaErrorInvalidValue;
    tile_weights_kernel<<<1184, 256, 0, st>>>(w, N, K, out, lm_order);
    return cudaGetLastError();
}

static_assert(sizeof(AttnSm) + NBLD * 1 * QDB_HD * 4 >= NEPI * 32 * 17 * 4,
              "the lm_head transpose buffers live in the attention scratch");

// Layout of the step's dynamic shared memory for Bp utterance columns and
// group size R: W ring, X ring, attention scratch (+ 1 KB alignment slack).
static int smem_for(int Bp, int R, int nsw) {
    const int att = (int)sizeof(AttnSm) + NBLD * R * QDB_HD * 4;
    const int xr = NSX * 2 * Bp * 128 > XRING_MIN ? NSX * 2 * Bp * 128 : XRING_MIN;
    return 1024 + nsw * W_TILE + xr + att;
}

extern "C" int qdb_bstep_ring_stages(int Bp, int R) {
    int nsw = MAX_NSW;
    while (nsw > 2 && smem_for(Bp, R, nsw) > 227 * 1024 - 8 * 1024) nsw--;
    return nsw;
}

extern "C" size_t qdb_bstep_smem(int Bp, int R) { return (size_t)smem_for(Bp, R, qdb_bstep_ring_stages(Bp, R)); }

extern "C" int qdb_bstep_counters(int layers) { return 1 + 5 * layers; }

extern "C" cudaError_t qdb_launch_bstep(const QdbBatchArgs *args, int grid, cudaStream_t st) {
    const QdbBatchArgs &a = *args;
    if (a.B < 1 || a.B > 64 || a.Bp < a.B || (a.Bp != 16 && a.Bp != 32 && a.Bp != 64)) return cudaErrorInvalidValue;
    if (a.nsw < NACC) return cudaErrorInvalidValue;  // an lm_head k-block holds NACC weight stages at once
    if (a.d.L > MAX_LAYERS || a.d.h % 64 || a.d.I % 64 || a.splits < 1) return cudaErrorInvalidValue;
    const int R = a.d.Hq / a.d.Hkv;
    const int smem = smem_for(a.Bp, R, a.nsw);
    void *kargs[] = {const_cast<QdbBatchArgs *>(&a)};
    cudaError_t e;
#define QDB_BSTEP_CASE(RR)                                                                                    \
    case RR:                                                                                                  \
        e = cudaFuncSetAttribute(bstep_kernel<RR>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);        \
        if (e != cudaSuccess) return e;                                                                       \
        return cudaLaunchCooperativeKernel((const void *)bstep_kernel<RR>, dim3(grid), dim3(NTHREADS), kargs, \
                                           (size_t)smem, st);
    switch (R) {
        QDB_BSTEP_CASE(1)
        QDB_BSTEP_CASE(2)
        QDB_BSTEP_CASE(4)
        QDB_BSTEP_CASE(8)
        default: return cudaErrorInvalidValue;
    }
#undef QDB_BSTEP_CASE
}

QDB_WAIT_LIMIT_SETTER(qdb_set_wait_limit_bstep)
