// qdb_rows.cu - row-batched decoder kernels around the tensor-core GEMM
// (qdb_tcgemm.cu): prefill of one utterance (qwen_decoder_prefill,
// qwen_asr_decoder.c:262-359) and one decode step of many independent
// utterances. Every row is one position.
#include "qdb_common.cuh"
#include "qdb_kernels.h"

namespace {

// ---------------------------------------------------------------- RMSNorm
// Per row: y = x * (1/sqrtf(mean(x^2)+eps)) * w (qwen_rms_norm,
// qwen_asr_kernels.c:750-809), written as the bf16 hi/lo split the
// tensor-core GEMM consumes (hi + lo ~= y to ~16 mantissa bits).
// The row is read once into registers (up to RN_VEC float4 per thread).
// zero/zero_len: optionally clears this row of the next split-K GEMM's
// target (zero_len floats per row), which saves a memset launch.
constexpr int RN_THREADS = 256, RN_VEC = 8;  // h <= 8192
__global__ void __launch_bounds__(RN_THREADS) rmsnorm_rows_kernel(const float *x, const float *w, uint16_t *hi,
                                                                 uint16_t *lo, int h, float eps, float *zero,
                                                                 int zero_len) {
    __shared__ float red[RN_THREADS / 32];
    pdl_enter();
    const int t = threadIdx.x;

    const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)blockIdx.x * h);
    const int h4 = h >> 2;
    float4 v[RN_VEC];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < RN_VEC; k++) {
        const int i = t + k * RN_THREADS;
        if (i < h4) {
            v[k] = xr[i];
            ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
        }
    }
    if (zero) {
        float4 *zr = reinterpret_cast<float4 *>(zero + (size_t)blockIdx.x * zero_len);
        for (int i = t; i < (zero_len >> 2); i += RN_THREADS) zr[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    ss = warp_sum(ss);
    if ((t & 31) == 0) red[t >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < RN_THREADS / 32; k++) tot += red[k];
    const float inv = 1.0f / sqrtf(tot / (float)h + eps);
    uint2 *hr = reinterpret_cast<uint2 *>(hi + (size_t)blockIdx.x * h);
    uint2 *lr = reinterpret_cast<uint2 *>(lo + (size_t)blockIdx.x * h);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
#pragma unroll
    for (int k = 0; k < RN_VEC; k++) {
        const int i = t + k * RN_THREADS;
        if (i < h4) {
            const float4 ww = w4[i];
            const float y[4] = {v[k].x * inv * ww.x, v[k].y * inv * ww.y, v[k].z * inv * ww.z, v[k].w * inv * ww.w};
            uint16_t b[4], c[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                b[e] = f32_to_bf16_rn(y[e]);
                c[e] = f32_to_bf16_rn(y[e] - __uint_as_float((uint32_t)b[e] << 16));
            }
            hr[i] = make_uint2((uint32_t)b[0] | ((uint32_t)b[1] << 16), (uint32_t)b[2] | ((uint32_t)b[3] << 16));
            lr[i] = make_uint2((uint32_t)c[0] | ((uint32_t)c[1] << 16), (uint32_t)c[2] | ((uint32_t)c[3] << 16));
        }
    }
}

// ---------------------------------------------------------------- Q/K norm, RoPE, KV append
// One warp per (row, head slot). Slots: [0, Hq) query heads -> q_out,
// [Hq, Hq+Hkv) key heads -> cache K, [Hq+Hkv, Hq+2Hkv) value heads -> cache V.
__global__ void qk_rope_append_kernel(const float *qkv, float *q_out, const QdbRowKV *rows, int n_rowkv,
                                      int row_pos_offset, int layer, int n, int Hq, int Hkv,
                                      const float *q_norm, const float *k_norm, const float2 *rope, float eps,
                                      const int *step) {
    pdl_enter();
    const int lane = threadIdx.x & 31;
    const int slot = blockIdx.y * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int row = blockIdx.x;
    if (slot >= Hq + 2 * Hkv || row >= n) return;
    const bool single = (n_rowkv == 1);
    const QdbRowKV rk = rows[single ? 0 : row];
    const int pos = rk.pos + (single ? row : 0) + row_pos_offset + (step ? *step : 0);
    const int width = (Hq + 2 * Hkv) * QDB_HD;
    const float *src = qkv + (size_t)row * width + (size_t)slot * QDB_HD;
    float e[4];
#pragma unroll
    for (int i = 0; i < 4; i++) e[i] = src[lane + 32 * i];
    if (slot < Hq + Hkv) {
        const float *w = slot < Hq ? q_norm : k_norm;
        float ss = warp_sum(e[0] * e[0] + e[1] * e[1] + e[2] * e[2] + e[3] * e[3]);
        const float inv = 1.0f / sqrtf(ss / (float)QDB_HD + eps);
#pragma unroll
        for (int i = 0; i < 4; i++) e[i] = e[i] * inv * w[lane + 32 * i];
        const float2 *rr = rope + (size_t)pos * (QDB_HD / 2);
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const float2 cs = rr[lane + 32 * i];
            const float x1 = e[i], x2 = e[i + 2];
            e[i] = x1 * cs.x - x2 * cs.y;
            e[i + 2] = x2 * cs.x + x1 * cs.y;
        }
    }
    if (slot < Hq) {
        float *dst = q_out + (size_t)row * Hq * QDB_HD + (size_t)slot * QDB_HD;
#pragma unroll
        for (int i = 0; i < 4; i++) dst[lane + 32 * i] = e[i];
    } else {
        const bool is_k = slot < Hq + Hkv;
        const int g = is_k ? slot - Hq : slot - Hq - Hkv;
        uint16_t *base = is_k ? rk.kc : rk.vc;
        uint16_t *dst = base + (((size_t)layer * Hkv + g) * (size_t)rk.cap + pos) * QDB_HD;
#pragma unroll
        for (int i = 0; i < 4; i++) dst[lane + 32 * i] = f32_to_kv(e[i]);
    }
}

// ---------------------------------------------------------------- independent-row attention
// Unit = (row, KV head g, split s) = one CTA of 8 warps over keys [p0, p1)
// of ctx = pos + 1. Lanes: 4 per key over 32 dims for q.k, then 4 dims per
// lane for p.V; the R query heads of the group share each K/V load. Writes
// the unnormalised partial (m, l, o[128]) of each query head; the merge
// kernel combines the splits (same online-softmax algebra as
// qwen_causal_attention, qwen_asr_kernels.c:1050-1141).
#ifndef QDB_AR_WARPS
#define QDB_AR_WARPS 8  // warps per unit CTA (each takes AR_KEYS keys of a chunk)
#endif
constexpr int AR_WARPS = QDB_AR_WARPS, AR_KEYS = 8;

// The unit is computed from a shared-memory ring: the unit's K and V rows are
// contiguous in the cache, so thread 0 streams them in 64-key chunks with
// cp.async.bulk (3 stages x 32 KB, 2 CTAs per SM: ~190 KB in flight per SM)
// and the 8 warps take 8 keys each per chunk. K chunks are read with the
// 16-byte piece order rotated per lane, which keeps the quarter-warp
// LDS.128 phases free of bank conflicts.
#ifndef QDB_AR_STAGES
#define QDB_AR_STAGES 2  // bulk-copy ring stages (32 KB each); 2 x 3 CTAs per SM measured best
#endif
#ifndef QDB_AR_MINB
#define QDB_AR_MINB 3  // CTAs per SM the register budget is sized for
#endif
constexpr int AB_STAGES = QDB_AR_STAGES, AB_KEYS = AR_WARPS * AR_KEYS, AB_HALF = AB_KEYS * QDB_HD * 2, AB_STAGE = 2 * AB_HALF;
typedef unsigned long long u64r;
__device__ __forceinline__ uint32_t su32r(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Combines the S unnormalised partials (m, l, o[128]) of one query head at
// dimension dd (L2 reads: other CTAs wrote them) and stores the normalised
// output as f32 or as the bf16 hi/lo split of the O-projection input.
__device__ __forceinline__ void attn_merge_store(const float *src, int S, int dd, size_t at, float *out, uint16_t *hi,
                                                 uint16_t *lo) {
    float M = -INFINITY;
    for (int s = 0; s < S; s++) M = fmaxf(M, __ldcg(src + s * (2 + QDB_HD)));
    float L = 0.f, O = 0.f;
    for (int s = 0; s < S; s++) {
        const float ms = __ldcg(src + s * (2 + QDB_HD));
        if (ms == -INFINITY) continue;
        const float f = expf(ms - M);
        L += __ldcg(src + s * (2 + QDB_HD) + 1) * f;
        O += __ldcg(src + s * (2 + QDB_HD) + 2 + dd) * f;
    }
    const float v = L > 0.f ? O / L : 0.f;
    if (hi) {
        const uint16_t b = f32_to_bf16_rn(v);
        hi[at] = b;
        lo[at] = f32_to_bf16_rn(v - __uint_as_float((uint32_t)b << 16));
    } else {
        out[at] = v;
    }
}

template <int R>
__global__ void __launch_bounds__(AR_WARPS * 32, QDB_AR_MINB) attn_rows_bulk_kernel(const float *q, const QdbRowKV *rows,
                                                                         int row_pos_offset, int layer, int Hq,
                                                                         int Hkv, int S, float *part, int *err,
                                                                         const int *step, float *out, uint16_t *hi,
                                                                         uint16_t *lo, unsigned *cnt) {
    pdl_enter();
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ __align__(16) float qs[R][QDB_HD];
    __shared__ float sm_m[AR_WARPS][R], sm_l[AR_WARPS][R];
    __shared__ __align__(16) float sm_o[AR_WARPS][R][QDB_HD];
    __shared__ __align__(8) u64r full[AB_STAGES];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x / Hkv, g = blockIdx.x % Hkv, s = blockIdx.y;
    const QdbRowKV rk = rows[row];
    const int pos = rk.pos + row_pos_offset + (step ? *step : 0);
    const int ctx = pos + 1;
    const int per = (ctx + S - 1) / S;
    const int p0 = s * per, p1 = min(ctx, p0 + per);
    const int nch = p1 > p0 ? (p1 - p0 + AB_KEYS - 1) / AB_KEYS : 0;
    const size_t head_base = ((size_t)layer * Hkv + g) * (size_t)rk.cap * QDB_HD;
    const uint16_t *kc = rk.kc + head_base, *vc = rk.vc + head_base;
    auto issue = [&](int c) {
        const int k0 = p0 + c * AB_KEYS;
        const unsigned bytes = (unsigned)(min(AB_KEYS, p1 - k0) * QDB_HD * 2);
        unsigned char *st = ring + (size_t)(c % AB_STAGES) * AB_STAGE;
        u64r *bar = &full[c % AB_STAGES];
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32r(bar)), "r"(2 * bytes)
                     : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32r(st)),
            "l"(kc + (size_t)k0 * QDB_HD), "r"(bytes), "r"(su32r(bar))
            : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                su32r(st + AB_HALF)),
            "l"(vc + (size_t)k0 * QDB_HD), "r"(bytes), "r"(su32r(bar))
            : "memory");
    };
    if (threadIdx.x == 0) {
        for (int i = 0; i < AB_STAGES; i++)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32r(&full[i])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int c = 0; c < nch && c < AB_STAGES; c++) issue(c);
    }
    for (int t = threadIdx.x; t < R * QDB_HD; t += blockDim.x)
        qs[t / QDB_HD][t % QDB_HD] = q[(size_t)row * Hq * QDB_HD + (size_t)(g * R) * QDB_HD + t];
    __syncthreads();
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
    for (int c = 0; c < nch; c++) {
        const unsigned char *st = ring + (size_t)(c % AB_STAGES) * AB_STAGE;
        {  // bounded wait for this chunk (every thread observes the phase)
            const unsigned par = (unsigned)(c / AB_STAGES) & 1u;
            const long long t0 = clock64();
            for (;;) {
                uint32_t ok;
                asm volatile(
                    "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                    : "=r"(ok)
                    : "r"(su32r(&full[c % AB_STAGES])), "r"(par)
                    : "memory");
                if (ok) break;
                if (clock64() - t0 > QDB_SPIN_LIMIT_CYCLES) {
                    set_error(err, QDB_ERR_BARRIER_TIMEOUT);
                    break;
                }
            }
        }
        const int base = p0 + c * AB_KEYS + warp * AR_KEYS;  // this warp's 8 keys
        const int j = base + kk;
        const bool valid = j < p1;
        uint4 kv4[4];
        const int rot = (sub + kk) & 3;
        if (valid) {
            const uint4 *kp = reinterpret_cast<const uint4 *>(st + (size_t)(warp * AR_KEYS + kk) * QDB_HD * 2) + sub * 4;
#pragma unroll
            for (int u = 0; u < 4; u++) kv4[u] = kp[(u + rot) & 3];
        }
        uint2 vv[AR_KEYS];
#pragma unroll
        for (int t = 0; t < AR_KEYS; t++)
            vv[t] = base + t < p1
                        ? *reinterpret_cast<const uint2 *>(st + AB_HALF + (size_t)(warp * AR_KEYS + t) * QDB_HD * 2 + lane * 8)
                        : make_uint2(0u, 0u);
#pragma unroll
        for (int h = 0; h < R; h++) {
            float a0 = 0.f, a1 = 0.f;
            if (valid) {
                const float *qv = qs[h] + sub * 32;
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
            const float sc = valid ? acc * scale : -INFINITY;
            float cm = sc;
            cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 4));
            cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 8));
            cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 16));
            const float mn = fmaxf(m[h], cm);
            const float corr = (mn == -INFINITY) ? 1.f : expf(m[h] - mn);
            const float p = valid ? expf(sc - mn) : 0.f;
            float ps = p;
            ps += __shfl_xor_sync(0xffffffffu, ps, 4);
            ps += __shfl_xor_sync(0xffffffffu, ps, 8);
            ps += __shfl_xor_sync(0xffffffffu, ps, 16);
            l[h] = l[h] * corr + ps;
#pragma unroll
            for (int e = 0; e < 4; e++) o[h][e] *= corr;
#pragma unroll
            for (int t = 0; t < AR_KEYS; t++) {
                const float pt = __shfl_sync(0xffffffffu, p, t * 4);
                o[h][0] = fmaf(pt, kvlo(vv[t].x), o[h][0]);
                o[h][1] = fmaf(pt, kvhi(vv[t].x), o[h][1]);
                o[h][2] = fmaf(pt, kvlo(vv[t].y), o[h][2]);
                o[h][3] = fmaf(pt, kvhi(vv[t].y), o[h][3]);
            }
            m[h] = mn;
        }
        __syncthreads();  // every warp is done with this stage
        if (threadIdx.x == 0 && c + AB_STAGES < nch) issue(c + AB_STAGES);
    }
#pragma unroll
    for (int h = 0; h < R; h++) {
        if (lane == 0) {
            sm_m[warp][h] = m[h];
            sm_l[warp][h] = l[h];
        }
#pragma unroll
        for (int e = 0; e < 4; e++) sm_o[warp][h][lane * 4 + e] = o[h][e];
    }
    __syncthreads();
    for (int t = threadIdx.x; t < R * QDB_HD; t += blockDim.x) {
        const int h = t / QDB_HD, dd = t % QDB_HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < AR_WARPS; w++) M = fmaxf(M, sm_m[w][h]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < AR_WARPS; w++) {
                const float f = expf(sm_m[w][h] - M);
                L += sm_l[w][h] * f;
                O += sm_o[w][h][dd] * f;
            }
        }
        if (S == 1) {
            // one unit holds every key: the normalised output directly (no merge launch)
            const float v = L > 0.f ? O / L : 0.f;
            const size_t at = (size_t)row * Hq * QDB_HD + (size_t)(g * R + h) * QDB_HD + dd;
            if (hi) {
                const uint16_t b = f32_to_bf16_rn(v);
                hi[at] = b;
                lo[at] = f32_to_bf16_rn(v - __uint_as_float((uint32_t)b << 16));
            } else {
                out[at] = v;
            }
            continue;
        }
        float *dst = part + (((size_t)row * Hq + g * R + h) * S + s) * (2 + QDB_HD);
        if (dd == 0) {
            dst[0] = M;
            dst[1] = L;
        }
        dst[2 + dd] = O;
    }
    if (S == 1 || !cnt) return;
    // The unit's last split to finish (counter cnt[row * Hkv + g], left at
    // zero) merges the S partials: no separate merge launch.
    __shared__ int last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        last = atomicAdd(&cnt[blockIdx.x], 1u) == (unsigned)(S - 1);
        if (last) cnt[blockIdx.x] = 0u;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int t = threadIdx.x; t < R * QDB_HD; t += blockDim.x) {
        const int h = t / QDB_HD, dd = t % QDB_HD;
        attn_merge_store(part + ((size_t)row * Hq + g * R + h) * S * (2 + QDB_HD), S, dd,
                         (size_t)row * Hq * QDB_HD + (size_t)(g * R + h) * QDB_HD + dd, out, hi, lo);
    }
}

// QK-norm / RoPE inputs of the fused form (qkv == nullptr: q is read as is)
struct AttnRope {
    const float *qkv, *q_norm, *k_norm;
    const float2 *rope;
    float eps;
};

// ---------------------------------------------------------------- fragment (MMA) form
// The same unit (row, KV head g, split s) on the tensor cores' warp-level
// MMA (m16n8k16, f16 in, f32 accumulate): the unit is bound by instruction
// issue in the lane-dot form above (~160 instructions per KB of K/V), and
// fragments do the q.K and p.V products in a few instructions per 8 x 16
// tile. Precision: K and V are the cache's fp16 values exactly; q is carried
// as an fp16 hi + lo pair (two MMAs, ~22 significant bits), so the scores
// match the f32 form to ~1e-6 relative; p in [0, 1] is rounded to fp16
// (relative error <= 2^-11 per weight, averaging out over the keys: the
// same order as the fp16 cache rounding of V itself), f32 accumulation.
// Layout: each chunk's 64 K and V rows are copied in 16-byte pieces
// (cp.async) into a 272-byte row stride (conflict-free ldmatrix); warp w scores keys [8w, 8w + 8) with the R
// query heads as MMA rows, every warp runs the same softmax over the chunk's
// 64 x R scores (shared memory), and warp w accumulates output dims
// [16w, 16w + 16) (p as the A operand, V through ldmatrix.trans).
#ifndef QDB_AR_MMA
#define QDB_AR_MMA 1  // fragment form for the batched-decode attention units
#endif
#ifndef QDB_AM_MINB
#define QDB_AM_MINB 3  // CTAs per SM the fragment form's register budget is sized for
#endif
#ifndef QDB_AM_EARLY
#define QDB_AM_EARLY 0  // copy chunks of earlier steps' keys before the dependency wait (measured slower)
#endif
#ifndef QDB_AM_PLO
#define QDB_AM_PLO 0  // 1: p carried as fp16 hi + lo in p.V (twice the p.V MMAs); 0: fp16 p
#endif
#ifndef QDB_AM_CHAINS
#define QDB_AM_CHAINS 0  // independent MMA accumulation chains (hi / lo, even / odd k-steps): measured slower
#endif
#ifndef QDB_AR_FUSED_ROPE
#define QDB_AR_FUSED_ROPE 0  // QK-norm, RoPE and the K/V append inside the decode attention units (measured: no gain)
#endif
#ifndef QDB_AM_BAR3
#define QDB_AM_BAR3 0  // three block barriers per chunk (the refill moves after the next chunk's first): no gain measured
#endif
#ifndef QDB_AM_STAGES
#define QDB_AM_STAGES 2  // chunk slots of the fragment form (34 KB each)
#endif
constexpr int AM_STAGES = QDB_AM_STAGES;
constexpr int AM_LDB = (QDB_HD + 8) * 2;             // padded row stride in bytes (272)
constexpr int AM_HALF = AB_KEYS * AM_LDB, AM_STAGE = 2 * AM_HALF;

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    // rows 8..15 of A are zero (a1 = a3 = 0): only rows 0..7 carry query heads
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// (x, y) as packed fp16 hi and the fp16 residual lo: x ~ hi.x + lo.x
__device__ __forceinline__ void split_h2(float x, float y, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

template <int R>
__global__ void __launch_bounds__(AR_WARPS * 32, QDB_AM_MINB) attn_rows_mma_kernel(const float *q, const QdbRowKV *rows,
                                                                        int row_pos_offset, int layer, int Hq,
                                                                        int Hkv, int S, float *part, int *err,
                                                                        const int *step, float *out, uint16_t *hi,
                                                                        uint16_t *lo, unsigned *cnt, AttnRope rp) {
    static_assert(AR_WARPS * 16 == QDB_HD && AR_WARPS * 8 == AB_KEYS && R <= 8, "fragment form shape");
    constexpr int PLD = AB_KEYS + 8;  // p row stride in halves (144 bytes: conflict-free ldmatrix)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ __align__(128) unsigned char ring[];
    constexpr int QLD = QDB_HD + 8;  // q row stride in halves (272 bytes)
    // q and p of the chunk as fp16 hi / lo rows; row R is zeros, and the
    // ldmatrix lanes of MMA rows R..7 all point at it
    __shared__ __align__(16) uint16_t qsm[2][R + 1][QLD];
    __shared__ __align__(16) uint16_t ps[2][R + 1][PLD];
    __shared__ float smax[AR_WARPS][R], ssum[AR_WARPS][R];
    __shared__ int last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g4 = lane >> 2, t4 = lane & 3;
    const int row = blockIdx.x / Hkv, g = blockIdx.x % Hkv, s = blockIdx.y;
    const QdbRowKV rk = rows[row];  // written by the host before the launch
    const size_t head_base = ((size_t)layer * Hkv + g) * (size_t)rk.cap * QDB_HD;
    // this thread's 16-byte pieces: piece tp of keys tk, tk + 16, tk + 32, tk + 48
    constexpr int PIECES = QDB_HD * 2 / 16, KSTEP = AR_WARPS * 32 / PIECES;
    const int tk = threadIdx.x / PIECES, tp = threadIdx.x % PIECES;
    const uint16_t *kc = rk.kc + head_base + (size_t)tk * QDB_HD + tp * 8;
    const uint16_t *vc = rk.vc + head_base + (size_t)tk * QDB_HD + tp * 8;
    const uint32_t sdst = su32r(ring) + tk * AM_LDB + tp * 16;
    auto copy_chunk = [&](int c, int k0, int nk) {
        const uint32_t d = sdst + (uint32_t)(c % AM_STAGES) * AM_STAGE;
#pragma unroll
        for (int j = 0; j < AB_KEYS / KSTEP; j++) {
            if (tk + j * KSTEP < nk) {
                const size_t src = (size_t)(k0 + j * KSTEP) * QDB_HD;
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d + j * KSTEP * AM_LDB), "l"(kc + src)
                             : "memory");
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d + AM_HALF + j * KSTEP * AM_LDB),
                             "l"(vc + src)
                             : "memory");
            }
        }
    };
    // Before waiting on the previous kernel: whole chunks of keys written by
    // earlier steps. Only the current position's key is written by this
    // step's RoPE kernel; the step counter read here may still lag the
    // step's own increment by one, which only lowers the bound.
    int early = 0;
    if (S == 1 && QDB_AM_EARLY) {
        const int old_keys = rk.pos + row_pos_offset + (step ? *(volatile const int *)step : 0);
        while (early < AM_STAGES && (early + 1) * AB_KEYS <= old_keys) {
            copy_chunk(early, early * AB_KEYS, AB_KEYS);
            asm volatile("cp.async.commit_group;" ::: "memory");
            early++;
        }
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int pos = rk.pos + row_pos_offset + (step ? *step : 0);
    const int ctx = pos + 1;
    const int per = (ctx + S - 1) / S;
    const int p0 = s * per, p1 = min(ctx, p0 + per);
    const int nch = p1 > p0 ? (p1 - p0 + AB_KEYS - 1) / AB_KEYS : 0;
    auto issue = [&](int c) {  // one cp.async commit group per chunk slot (empty past the last chunk)
        if (c < nch) {
            const int k0 = p0 + c * AB_KEYS;
            copy_chunk(c, k0, min(AB_KEYS, p1 - k0));
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // With rp.qkv the unit also does the QK-norm, RoPE and cache append of
    // its own heads (the work of qk_rope_append_kernel): the split holding
    // key pos writes K/V row pos, and that chunk is copied only after the
    // block barrier that follows the write.
    const bool own_kv = rp.qkv && p0 <= pos && pos < p1;
    int pro = AM_STAGES;  // prologue chunks issued before the append
    if (own_kv)
        for (int c = early; c < AM_STAGES; c++)
            if (c < nch && p0 + (c + 1) * AB_KEYS > pos) {
                pro = c;
                break;
            }
    for (int c = early; c < pro; c++) issue(c);
    for (int i = threadIdx.x; i < 2 * (R + 1) * PLD; i += blockDim.x) (&ps[0][0][0])[i] = 0;
    if (rp.qkv) {
        if (threadIdx.x < QDB_HD) {  // the zero row
            qsm[0][R][threadIdx.x] = 0;
            qsm[1][R][threadIdx.x] = 0;
        }
        // warp w < R: query head g R + w; warp R: key head g; warp R + 1: value head g
        if (warp < R + 2 && (warp < R || own_kv)) {
            const int slot = warp < R ? g * R + warp : (warp == R ? Hq + g : Hq + Hkv + g);
            const float *src = rp.qkv + (size_t)row * (Hq + 2 * Hkv) * QDB_HD + (size_t)slot * QDB_HD;
            float e[4];
#pragma unroll
            for (int i = 0; i < 4; i++) e[i] = src[lane + 32 * i];
            if (warp <= R) {
                const float *w = warp < R ? rp.q_norm : rp.k_norm;
                const float ss = warp_sum(e[0] * e[0] + e[1] * e[1] + e[2] * e[2] + e[3] * e[3]);
                const float inv = 1.0f / sqrtf(ss / (float)QDB_HD + rp.eps);
#pragma unroll
                for (int i = 0; i < 4; i++) e[i] = e[i] * inv * w[lane + 32 * i];
                const float2 *rr = rp.rope + (size_t)pos * (QDB_HD / 2);
#pragma unroll
                for (int i = 0; i < 2; i++) {
                    const float2 cs = rr[lane + 32 * i];
                    const float x1 = e[i], x2 = e[i + 2];
                    e[i] = x1 * cs.x - x2 * cs.y;
                    e[i + 2] = x2 * cs.x + x1 * cs.y;
                }
            }
            if (warp < R) {
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const __half h = __float2half_rn(e[i]);
                    qsm[0][warp][lane + 32 * i] = __half_as_ushort(h);
                    qsm[1][warp][lane + 32 * i] = __half_as_ushort(__float2half_rn(e[i] - __half2float(h)));
                }
            } else {
                uint16_t *dst = (warp == R ? rk.kc : rk.vc) + head_base + (size_t)pos * QDB_HD;
#pragma unroll
                for (int i = 0; i < 4; i++) dst[lane + 32 * i] = f32_to_kv(e[i]);
            }
        }
        __syncthreads();  // q in shared memory; row pos in the cache for this CTA's copies
        for (int c = pro; c < AM_STAGES; c++) issue(c);
    } else {
        for (int i = threadIdx.x; i < (R + 1) * QDB_HD / 2; i += blockDim.x) {  // q as hi / lo pairs
            const int h = i / (QDB_HD / 2), d = (i % (QDB_HD / 2)) * 2;
            uint32_t qh = 0u, ql = 0u;
            if (h < R) {
                const float2 v = *reinterpret_cast<const float2 *>(q + (size_t)row * Hq * QDB_HD +
                                                                   (size_t)(g * R + h) * QDB_HD + d);
                split_h2(v.x, v.y, qh, ql);
            }
            *reinterpret_cast<uint32_t *>(&qsm[0][h][d]) = qh;
            *reinterpret_cast<uint32_t *>(&qsm[1][h][d]) = ql;
        }
    }
    // scores in log2 units: p = 2^(s' - m'), s' = q.k / sqrt(128) x log2(e)
    const float scale2 = 1.4426950408889634f / sqrtf((float)QDB_HD);
    float m = -INFINITY, l = 0.f;
    float o[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#if QDB_AM_CHAINS
    float ol[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#endif
    const int mi = lane >> 3;
    const uint32_t kb = su32r(ring) + (warp * 8 + (lane & 7)) * AM_LDB + mi * 16;
    const uint32_t vb = su32r(ring) + AM_HALF + ((mi & 1) * 8 + (lane & 7)) * AM_LDB + (warp * 16 + (mi >> 1) * 8) * 2;
    const int arow = (lane & 7) < R ? (lane & 7) : R;  // MMA row of this ldmatrix lane (R: the zero row)
    const uint32_t pb = su32r(&ps[0][arow][(mi & 1) * 8]);  // x2: cols +0 (lanes 0-7) / +8 (lanes 8-15)
    const uint32_t qb = su32r(&qsm[0][arow][mi * 8]);       // x4: cols +0, +8 of k-step 2 k2 and of 2 k2 + 1
    for (int c = 0; c < nch; c++) {
        const uint32_t so = (uint32_t)(c % AM_STAGES) * AM_STAGE;
        const int k0 = p0 + c * AB_KEYS, nk = min(AB_KEYS, p1 - k0);
        if (nk < AB_KEYS) {  // rows past the last key: zero V (p = 0 must not meet stale non-finite values)
            unsigned char *st = ring + so;
            for (int i = threadIdx.x; i < (AB_KEYS - nk) * PIECES; i += blockDim.x)
                *reinterpret_cast<uint4 *>(st + AM_HALF + (size_t)(nk + i / PIECES) * AM_LDB + (i % PIECES) * 16) =
                    make_uint4(0u, 0u, 0u, 0u);
        }
        // this thread's copies of chunk c are done (later slots may still be
        // in flight); the barrier makes every thread's copies visible
        if (QDB_AM_BAR3 && c > 0)
            asm volatile("cp.async.wait_group %0;" ::"n"(AM_STAGES - 2) : "memory");
        else
            asm volatile("cp.async.wait_group %0;" ::"n"(AM_STAGES - 1) : "memory");
        __syncthreads();
        // with QDB_AM_BAR3 the slot of chunk c - 1 is refilled here: the
        // barrier above is the proof that every warp is done with it
        if (QDB_AM_BAR3 && c > 0) issue(c + AM_STAGES - 1);
        // 1. scores of keys [8 warp, 8 warp + 8) and their max per head
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
#if QDB_AM_CHAINS
        {  // four independent accumulation chains of four MMAs each
            float c1[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f}, c3[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k2 = 0; k2 < 4; k2++) {
                uint32_t b[4], ah[4], al[4];
                ldsm_x4(b, kb + so + k2 * 64);
                ldsm_x4(ah, qb + k2 * 64);
                ldsm_x4(al, qb + k2 * 64 + (R + 1) * QLD * 2);
                mma16816(sc, ah[0], ah[1], b[0], b[1]);
                mma16816(c1, al[0], al[1], b[0], b[1]);
                mma16816(c2, ah[2], ah[3], b[2], b[3]);
                mma16816(c3, al[2], al[3], b[2], b[3]);
            }
#pragma unroll
            for (int e = 0; e < 4; e++) sc[e] = (sc[e] + c2[e]) + (c1[e] + c3[e]);
        }
#else
#pragma unroll
        for (int k2 = 0; k2 < 4; k2++) {
            uint32_t b[4], ah[4], al[4];
            ldsm_x4(b, kb + so + k2 * 64);
            ldsm_x4(ah, qb + k2 * 64);
            ldsm_x4(al, qb + k2 * 64 + (R + 1) * QLD * 2);
            mma16816(sc, ah[0], ah[1], b[0], b[1]);
            mma16816(sc, al[0], al[1], b[0], b[1]);
            mma16816(sc, ah[2], ah[3], b[2], b[3]);
            mma16816(sc, al[2], al[3], b[2], b[3]);
        }
#endif
        const int kl = warp * 8 + t4 * 2;
        const float s0 = kl < nk ? sc[0] * scale2 : -INFINITY, s1 = kl + 1 < nk ? sc[1] * scale2 : -INFINITY;
        float lm = fmaxf(s0, s1);
        lm = fmaxf(lm, __shfl_xor_sync(0xffffffffu, lm, 1));
        lm = fmaxf(lm, __shfl_xor_sync(0xffffffffu, lm, 2));
        if (g4 < R && t4 == 0) smax[warp][g4] = lm;
        __syncthreads();
        // 2. p of these keys under the chunk's running max; partial sums
        float corr = 1.f;
        if (g4 < R) {
            float mc = smax[0][g4];
#pragma unroll
            for (int w = 1; w < AR_WARPS; w++) mc = fmaxf(mc, smax[w][g4]);
            const float mn = fmaxf(m, mc);  // finite: every chunk holds a key
            corr = exp2f(m - mn);
            m = mn;
            const float e0 = exp2f(s0 - mn), e1 = exp2f(s1 - mn);
            float sum = e0 + e1;
            sum += __shfl_xor_sync(0xfu << (lane & 28), sum, 1);
            sum += __shfl_xor_sync(0xfu << (lane & 28), sum, 2);
            if (t4 == 0) ssum[warp][g4] = sum;
            uint32_t h2, l2;
            split_h2(e0, e1, h2, l2);
            *reinterpret_cast<uint32_t *>(&ps[0][g4][kl]) = h2;
            *reinterpret_cast<uint32_t *>(&ps[1][g4][kl]) = l2;
        }
        __syncthreads();
        // 3. o[:, 16 warp .. 16 warp + 16) = corr o + p V
        if (g4 < R) {
            float sum = ssum[0][g4];
#pragma unroll
            for (int w = 1; w < AR_WARPS; w++) sum += ssum[w][g4];
            l = l * corr + sum;
        }
#pragma unroll
        for (int nt = 0; nt < 2; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                o[nt][e] *= corr;
#if QDB_AM_CHAINS
                ol[nt][e] *= corr;
#endif
            }
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
            uint32_t b[4], ah[2], al[2];
            ldsm_x4_t(b, vb + so + ks * 16 * AM_LDB);
            asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                         : "=r"(ah[0]), "=r"(ah[1])
                         : "r"(pb + ks * 32));
            asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                         : "=r"(al[0]), "=r"(al[1])
                         : "r"(pb + ks * 32 + (R + 1) * PLD * 2));
            mma16816(o[0], ah[0], ah[1], b[0], b[1]);
            mma16816(o[1], ah[0], ah[1], b[2], b[3]);
#if QDB_AM_CHAINS
            mma16816(ol[0], al[0], al[1], b[0], b[1]);  // the p lo products: their own chains
            mma16816(ol[1], al[0], al[1], b[2], b[3]);
#else
            if (QDB_AM_PLO) {
                mma16816(o[0], al[0], al[1], b[0], b[1]);
                mma16816(o[1], al[0], al[1], b[2], b[3]);
            }
#endif
        }
        if (!QDB_AM_BAR3) {
            __syncthreads();  // the stage, p and the partial maxima / sums are free
            issue(c + AM_STAGES);
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
#if QDB_AM_CHAINS
#pragma unroll
    for (int nt = 0; nt < 2; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) o[nt][e] += ol[nt][e];
#endif
    // lane (g4 < R) holds head g4 at dims 16 warp + 8 nt + 2 t4 + {0, 1}
    if (g4 < R) {
        const int h = g4;
#pragma unroll
        for (int nt = 0; nt < 2; nt++) {
            const int dd = warp * 16 + nt * 8 + t4 * 2;
            if (S == 1) {
                const float inv = l > 0.f ? 1.f / l : 0.f;
                const size_t at = (size_t)row * Hq * QDB_HD + (size_t)(g * R + h) * QDB_HD + dd;
                const float v0 = o[nt][0] * inv, v1 = o[nt][1] * inv;
                if (hi) {
                    const uint16_t b0 = f32_to_bf16_rn(v0), b1 = f32_to_bf16_rn(v1);
                    hi[at] = b0;
                    hi[at + 1] = b1;
                    lo[at] = f32_to_bf16_rn(v0 - __uint_as_float((uint32_t)b0 << 16));
                    lo[at + 1] = f32_to_bf16_rn(v1 - __uint_as_float((uint32_t)b1 << 16));
                } else {
                    out[at] = v0;
                    out[at + 1] = v1;
                }
            } else {
                // partial in natural-log units, as the merge expects
                float *dst = part + (((size_t)row * Hq + g * R + h) * S + s) * (2 + QDB_HD);
                if (warp == 0 && nt == 0 && t4 == 0) {
                    dst[0] = m * 0.6931471805599453f;
                    dst[1] = l;
                }
                dst[2 + dd] = o[nt][0];
                dst[3 + dd] = o[nt][1];
            }
        }
    }
    if (S == 1 || !cnt) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        last = atomicAdd(&cnt[blockIdx.x], 1u) == (unsigned)(S - 1);
        if (last) cnt[blockIdx.x] = 0u;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int t = threadIdx.x; t < R * QDB_HD; t += blockDim.x) {
        const int h = t / QDB_HD, dd = t % QDB_HD;
        attn_merge_store(part + ((size_t)row * Hq + g * R + h) * S * (2 + QDB_HD), S, dd,
                         (size_t)row * Hq * QDB_HD + (size_t)(g * R + h) * QDB_HD + dd, out, hi, lo);
    }
}

// hi/lo (optional): write the bf16 split the O-projection GEMM reads instead of f32 out.
__global__ void attn_rows_merge_kernel(const float *part, int S, int Hq, float *out, uint16_t *hi, uint16_t *lo) {
    pdl_enter();
    const int row = blockIdx.x, h = blockIdx.y, dd = threadIdx.x;
    attn_merge_store(part + ((size_t)row * Hq + h) * S * (2 + QDB_HD), S, dd,
                     (size_t)row * Hq * QDB_HD + (size_t)h * QDB_HD + dd, out, hi, lo);
}

// ---------------------------------------------------------------- argmax / embed
// Sliced form: gridDim.y CTAs per row each take a slice of the vocabulary and
// fold its best (value, lowest index) key into keys[row] with a 64-bit
// atomicMax; the row's last CTA (counter keys[n + row]) writes the token and
// leaves both words at zero for the next call. Same key, so the same token.
constexpr int AM_SLICES = 16, AM_THREADS = 256;
__global__ void __launch_bounds__(AM_THREADS) argmax_rows_sliced_kernel(const float *logits, int V, int mask_eos,
                                                                         int *tokens, const int *step,
                                                                         unsigned long long *keys) {
    pdl_enter();
    __shared__ unsigned long long red[AM_THREADS / 32];
    __shared__ bool last;
    const int row = blockIdx.x, n = gridDim.x;
    const float *lr = logits + (size_t)row * V;
    const int per = (V + gridDim.y - 1) / gridDim.y, i0 = blockIdx.y * per, i1 = min(V, i0 + per);
    unsigned long long best = 0ull;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        if (mask_eos && (i == QDB_ENDOFTEXT || i == QDB_IM_END)) continue;
        const float v = lr[i];
        if (isnan(v)) continue;
        const unsigned long long k = argmax_key(v, i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
        best = t > best ? t : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < AM_THREADS / 32; w++) best = red[w] > best ? red[w] : best;
        if (best) atomicMax(&keys[row], best);
        __threadfence();
        last = atomicAdd(&keys[n + row], 1ull) == (unsigned long long)(gridDim.y - 1);
        if (last) {
            __threadfence();
            const unsigned long long k = atomicExch(&keys[row], 0ull);
            keys[n + row] = 0ull;
            tokens[(step ? (size_t)*step * n : 0) + row] = k ? argmax_key_index(k) : 0;
        }
    }
}

__global__ void argmax_rows_kernel(const float *logits, int V, int mask_eos, int *tokens, const int *step) {
    pdl_enter();
    __shared__ unsigned long long red[32];
    const float *lr = logits + (size_t)blockIdx.x * V;
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        if (mask_eos && (i == QDB_ENDOFTEXT || i == QDB_IM_END)) continue;
        const float v = lr[i];
        if (isnan(v)) continue;
        const unsigned long long k = argmax_key(v, i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
        best = t > best ? t : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        best = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
            best = t > best ? t : best;
        }
        if (threadIdx.x == 0) tokens[(step ? (size_t)*step * gridDim.x : 0) + blockIdx.x] = best ? argmax_key_index(best) : 0;
    }
}

__global__ void embed_rows_kernel(const uint16_t *embed, const int *tokens, float *x, int h, int V, const int *step) {
    pdl_enter();
    const int row = blockIdx.x;
    int tok = tokens[(step ? (size_t)*step * gridDim.x : 0) + row];
    if (tok < 0 || tok >= V) tok = 0;  // never gather outside the table
    const uint16_t *src = embed + (size_t)tok * h;
    for (int i = threadIdx.x; i < h; i += blockDim.x) x[(size_t)row * h + i] = __uint_as_float(((uint32_t)src[i]) << 16);
}

// One thread: the device-side step counter of a captured decode step.
__global__ void step_advance_kernel(int *step) {
    pdl_enter();
    *step += 1;
}

}  // namespace

extern "C" cudaError_t qdb_launch_step_advance(int *step, cudaStream_t st) {
    return pdl_launch(step_advance_kernel, dim3(1), dim3(1), 0, st, step);
}

extern "C" cudaError_t qdb_launch_rmsnorm_rows(const float *x, const float *w, uint16_t *hi, uint16_t *lo, int n, int h,
                                               float eps, cudaStream_t st, float *zero, int zero_len) {
    if (n <= 0) return cudaSuccess;
    if (h % 4 || h > 4 * RN_VEC * RN_THREADS || (zero && zero_len % 4)) return cudaErrorInvalidValue;
    return pdl_launch(rmsnorm_rows_kernel, dim3(n), dim3(RN_THREADS), 0, st, x, w, hi, lo, h, eps, zero, zero_len);
}

extern "C" cudaError_t qdb_launch_qk_rope_append(const float *qkv, float *q_out, const QdbRowKV *rows, int row_pos_offset,
                                                 int layer, int n, int Hq, int Hkv, const float *q_norm,
                                                 const float *k_norm, const float2 *rope, float eps,
                                                 cudaStream_t st, const int *step) {
    if (n <= 0) return cudaSuccess;
    const int slots = Hq + 2 * Hkv;
    dim3 grid(n, (slots + 3) / 4);
    // n_rowkv: callers pass a single-entry array for one session (rows[0].pos is the first row's position)
    return pdl_launch(qk_rope_append_kernel, grid, dim3(128), 0, st, qkv, q_out, rows, 0, row_pos_offset, layer, n, Hq,
                      Hkv, q_norm, k_norm, rope, eps, step);
}

extern "C" cudaError_t qdb_launch_qk_rope_append_single(const float *qkv, float *q_out, const QdbRowKV *row0,
                                                        int layer, int n, int Hq, int Hkv, const float *q_norm,
                                                        const float *k_norm, const float2 *rope, float eps,
                                                        cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    const int slots = Hq + 2 * Hkv;
    dim3 grid(n, (slots + 3) / 4);
    qk_rope_append_kernel<<<grid, 128, 0, st>>>(qkv, q_out, row0, 1, 0, layer, n, Hq, Hkv, q_norm, k_norm, rope,
                                                eps, nullptr);
    return cudaGetLastError();
}

template <int R>
static cudaError_t attn_rows_launch(dim3 grid, const float *q, const QdbRowKV *rows, int row_pos_offset, int layer,
                                    int Hq, int Hkv, int S, float *part, int *err, cudaStream_t st, const int *step,
                                    float *out, uint16_t *hi, uint16_t *lo, unsigned *cnt,
                                    AttnRope rp = AttnRope{nullptr, nullptr, nullptr, nullptr, 0.f}) {
    if (QDB_AR_MMA && (S == 1 || cnt)) {
        const int smem = AM_STAGES * AM_STAGE;
        cudaError_t e =
            cudaFuncSetAttribute(attn_rows_mma_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        return pdl_launch(attn_rows_mma_kernel<R>, grid, dim3(AR_WARPS * 32), (size_t)smem, st, q, rows,
                          row_pos_offset, layer, Hq, Hkv, S, part, err, step, out, hi, lo, cnt, rp);
    }
    const int smem = AB_STAGES * AB_STAGE;
    cudaError_t e = cudaFuncSetAttribute(attn_rows_bulk_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    return pdl_launch(attn_rows_bulk_kernel<R>, grid, dim3(AR_WARPS * 32), (size_t)smem, st, q, rows, row_pos_offset,
                      layer, Hq, Hkv, S, part, err, step, out, hi, lo, cnt);
}

extern "C" cudaError_t qdb_launch_attn_rows(const float *q, const QdbRowKV *rows, int row_pos_offset, int layer,
                                            int n, int Hq, int Hkv, int S, float *part, float *out,
                                            cudaStream_t st, int *err, const int *step, uint16_t *hi,
                                            uint16_t *lo, unsigned *cnt) {
    if (n <= 0) return cudaSuccess;
    cudaError_t e0;
    dim3 grid(n * Hkv, S);
    switch (Hq / Hkv) {
        case 1: e0 = attn_rows_launch<1>(grid, q, rows, row_pos_offset, layer, Hq, Hkv, S, part, err, st, step, out, hi, lo, cnt); break;
        case 2: e0 = attn_rows_launch<2>(grid, q, rows, row_pos_offset, layer, Hq, Hkv, S, part, err, st, step, out, hi, lo, cnt); break;
        case 4: e0 = attn_rows_launch<4>(grid, q, rows, row_pos_offset, layer, Hq, Hkv, S, part, err, st, step, out, hi, lo, cnt); break;
        case 8: e0 = attn_rows_launch<8>(grid, q, rows, row_pos_offset, layer, Hq, Hkv, S, part, err, st, step, out, hi, lo, cnt); break;
        default: return cudaErrorInvalidValue;
    }
    if (e0 != cudaSuccess) return e0;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || S == 1 || cnt) return e;  // S == 1 or cnt: the units wrote the output
    return pdl_launch(attn_rows_merge_kernel, dim3(n, Hq), dim3(QDB_HD), 0, st, part, S, Hq, out, hi, lo);
}

// Fused form: QK-norm, RoPE and the K/V append of the decode rows inside the
// attention units (replaces qdb_launch_qk_rope_append + qdb_launch_attn_rows).
// cudaErrorNotSupported: the fused form is built out; the caller launches the two.
extern "C" cudaError_t qdb_launch_attn_rows_rope(const float *qkv, const QdbRowKV *rows, int row_pos_offset,
                                                 int layer, int n, int Hq, int Hkv, int S, const float *q_norm,
                                                 const float *k_norm, const float2 *rope, float eps, float *part,
                                                 float *out, cudaStream_t st, int *err, const int *step,
                                                 uint16_t *hi, uint16_t *lo, unsigned *cnt) {
    if (!QDB_AR_MMA || !QDB_AR_FUSED_ROPE || !cnt) return cudaErrorNotSupported;
    if (n <= 0) return cudaSuccess;
    const AttnRope rp{qkv, q_norm, k_norm, rope, eps};
    dim3 grid(n * Hkv, S);
    cudaError_t e0;
    switch (Hq / Hkv) {
        case 1: e0 = attn_rows_launch<1>(grid, nullptr, rows, row_pos_offset, layer, Hq, Hkv, S, part, err, st, step, out, hi, lo, cnt, rp); break;
        case 2: e0 = attn_rows_launch<2>(grid, nullptr, rows, row_pos_offset, layer, Hq, Hkv, S, part, err, st, step, out, hi, lo, cnt, rp); break;
        case 4: e0 = attn_rows_launch<4>(grid, nullptr, rows, row_pos_offset, layer, Hq, Hkv, S, part, err, st, step, out, hi, lo, cnt, rp); break;
        case 8: e0 = attn_rows_launch<8>(grid, nullptr, rows, row_pos_offset, layer, Hq, Hkv, S, part, err, st, step, out, hi, lo, cnt, rp); break;
        default: return cudaErrorInvalidValue;
    }
    if (e0 != cudaSuccess) return e0;
    return cudaGetLastError();
}

extern "C" cudaError_t qdb_launch_argmax_rows(const float *logits, int n, int V, int mask_eos, int *tokens,
                                              cudaStream_t st, const int *step, unsigned long long *keys) {
    if (n <= 0) return cudaSuccess;
    if (keys)
        return pdl_launch(argmax_rows_sliced_kernel, dim3(n, AM_SLICES), dim3(AM_THREADS), 0, st, logits, V, mask_eos,
                          tokens, step, keys);
    return pdl_launch(argmax_rows_kernel, dim3(n), dim3(1024), 0, st, logits, V, mask_eos, tokens, step);
}

extern "C" cudaError_t qdb_launch_embed_rows(const uint16_t *embed, const int *tokens, float *x, int n, int h,
                                             int V, cudaStream_t st, const int *step) {
    if (n <= 0) return cudaSuccess;
    return pdl_launch(embed_rows_kernel, dim3(n), dim3(256), 0, st, embed, tokens, x, h, V, step);
}
