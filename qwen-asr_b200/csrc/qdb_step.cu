// qdb_step.cu - persistent single-utterance decode step (batch 1).
//
// One cooperative launch runs a whole decode position: 28 layers plus the
// tied lm_head and greedy argmax (qwen_decoder_forward,
// qwen_asr_decoder.c:388-476). One CTA per SM; phases are separated by a
// grid barrier whose spin is bounded (error word + early return, never a
// trap). Per layer:
//   A  input RMSNorm (every CTA, redundantly) -> QKV matvec rows
//   B  per-head Q/K RMSNorm + NeoX RoPE + bf16 KV append + split-K attention;
//      the last CTA of each KV head merges the splits
//   C  O-proj matvec rows + residual
//   D  post-attention RMSNorm -> gate/up row pairs + SwiGLU
//   E  down matvec rows + residual
// then F: final RMSNorm, lm_head rows with a (value, lowest index) argmax.
//
// Weights are streamed once per step with 16-byte non-allocating loads; all
// data that other CTAs write during the launch is read with ld.global.cg so
// a stale L1 line is never used.
#include "qdb_common.cuh"
#include "qdb_kernels.h"

namespace {

constexpr int WPB = QDB_STEP_THREADS / 32;  // warps per CTA
constexpr int ATT_KEYS = 8;                 // keys per warp iteration
constexpr int MAX_GQA = 8;                  // query heads per KV head supported

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier on a monotonically increasing counter. Returns false when the
// wait ran out (error recorded); callers then return from the kernel.
__device__ bool grid_barrier(unsigned *bar, unsigned target, int *err, volatile int *s_ok) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(bar, 1u);
        long long t0 = clock64();
        int ok = 1;
        while ((int)(ld_acquire_u32(bar) - target) < 0) {
            if (clock64() - t0 > QDB_SPIN_LIMIT_CYCLES) {
                ok = 0;
                set_error(err, QDB_ERR_BARRIER_TIMEOUT);
                break;
            }
        }
        __threadfence();
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

// Block-wide sum (all threads get the result). red: >= WPB floats of smem.
__device__ float block_sum(float v, float *red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < WPB ? red[lane] : 0.f;
    return warp_sum(t);
}

// xs[i] = x[i] * (1/sqrtf(mean(x^2)+eps)) * w[i] into shared memory
// (qwen_rms_norm, qwen_asr_kernels.c:750-809). x is either global f32
// (read through L2) or, when emb != null, a bf16 embedding row.
__device__ void norm_to_smem(const float *x, const uint16_t *emb, const float *w, int h, float eps,
                             float *xs, float *red) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < h; i += blockDim.x) {
        float v = emb ? __uint_as_float(((uint32_t)emb[i]) << 16) : __ldcg(x + i);
        xs[i] = v;
        ss += v * v;
    }
    ss = block_sum(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)h + eps);
    for (int i = threadIdx.x; i < h; i += blockDim.x) xs[i] = xs[i] * inv * w[i];
    __syncthreads();
}

__device__ void load_to_smem(const float *src, int n, float *xs) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = __ldcg(src + i);
    __syncthreads();
}

// Dot of one bf16 weight row (K elements, K % 256 == 0) with xs (smem), one
// warp; every lane gets the sum. Up to 8 16-byte loads per lane in flight.
__device__ __forceinline__ float row_dot(const uint16_t *wrow, const float *xs, int K) {
    const int lane = threadIdx.x & 31;
    const uint4 *wp = reinterpret_cast<const uint4 *>(wrow);
    const int nv = K >> 8;
    float acc = 0.f;
    for (int i0 = 0; i0 < nv; i0 += 8) {
        uint4 w[8];
#pragma unroll
        for (int u = 0; u < 8; u++)
            if (i0 + u < nv) w[u] = ldg_stream(wp + (i0 + u) * 32 + lane);
#pragma unroll
        for (int u = 0; u < 8; u++)
            if (i0 + u < nv) {
                const float4 *xp = reinterpret_cast<const float4 *>(xs + ((i0 + u) * 32 + lane) * 8);
                acc = dot8(w[u], xp[0], xp[1], acc);
            }
    }
    return warp_sum(acc);
}

// Two rows at once (independent loads in flight for both).
__device__ __forceinline__ void row_dot2(const uint16_t *r0, const uint16_t *r1, const float *xs, int K,
                                         float &s0, float &s1) {
    const int lane = threadIdx.x & 31;
    const uint4 *p0 = reinterpret_cast<const uint4 *>(r0);
    const uint4 *p1 = reinterpret_cast<const uint4 *>(r1);
    const int nv = K >> 8;
    float a0 = 0.f, a1 = 0.f;
    for (int i0 = 0; i0 < nv; i0 += 4) {
        uint4 w0[4], w1[4];
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (i0 + u < nv) {
                w0[u] = ldg_stream(p0 + (i0 + u) * 32 + lane);
                w1[u] = ldg_stream(p1 + (i0 + u) * 32 + lane);
            }
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (i0 + u < nv) {
                const float4 *xp = reinterpret_cast<const float4 *>(xs + ((i0 + u) * 32 + lane) * 8);
                const float4 xa = xp[0], xb = xp[1];
                a0 = dot8(w0[u], xa, xb, a0);
                a1 = dot8(w1[u], xa, xb, a1);
            }
    }
    s0 = warp_sum(a0);
    s1 = warp_sum(a1);
}

// Per-head RMSNorm then NeoX rotation of one 128-float head held in smem,
// one warp (qwen_rms_norm_per_head :811-873, qwen_apply_rope_neox :1182-1247).
__device__ void head_norm_rope(float *v, const float *w, const float2 *rope_row, float eps) {
    const int lane = threadIdx.x & 31;
    float e[4];
#pragma unroll
    for (int i = 0; i < 4; i++) e[i] = v[lane + 32 * i];
    float ss = e[0] * e[0] + e[1] * e[1] + e[2] * e[2] + e[3] * e[3];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)QDB_HD + eps);
#pragma unroll
    for (int i = 0; i < 4; i++) e[i] = e[i] * inv * w[lane + 32 * i];
    // lane + 32*i: i = 0,1 first half (d = lane, lane+32); i = 2,3 second half.
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

struct AttnSmem {
    float q[MAX_GQA][QDB_HD];
    float knew[QDB_HD];
    float m[WPB][MAX_GQA];
    float l[WPB][MAX_GQA];
    float o[WPB][MAX_GQA][QDB_HD];
};

// One attention work unit: KV head g, keys [p0, p1) of ctx = pos + 1.
// Writes the unnormalised partial (m, l, o[128]) for its query heads.
template <int R>
__device__ void attn_unit(const QdbStepArgs &a, int layer, int g, int s, int S, AttnSmem *sm) {
    const QdbDims &d = a.d;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ctx = a.pos + 1;
    const int per = (ctx + S - 1) / S;
    const int p0 = s * per;
    const int p1 = min(ctx, p0 + per);
    const int qd = d.Hq * QDB_HD, kvd = d.Hkv * QDB_HD;
    const QdbLayerW &lw = a.layers[layer];
    const float2 *rope_row = a.rope + (size_t)a.pos * (QDB_HD / 2);
    const size_t head_base = ((size_t)layer * d.Hkv + g) * (size_t)a.cap * QDB_HD;
    const uint16_t *kc = a.kc + head_base;
    const uint16_t *vc = a.vc + head_base;

    // Query heads of this group: normalise + rotate (one warp per head).
    for (int h = warp; h < R; h += WPB) {
        for (int i = lane; i < QDB_HD; i += 32) sm->q[h][i] = __ldcg(a.qkv + (g * R + h) * QDB_HD + i);
        __syncwarp();
        head_norm_rope(sm->q[h], lw.q_norm, rope_row, d.eps);
    }
    // The unit holding position pos appends the new K/V row (bf16).
    const bool owns_new = (p0 <= a.pos && a.pos < p1);
    if (owns_new && warp == WPB - 1) {
        for (int i = lane; i < QDB_HD; i += 32) sm->knew[i] = __ldcg(a.qkv + qd + g * QDB_HD + i);
        __syncwarp();
        head_norm_rope(sm->knew, lw.k_norm, rope_row, d.eps);
        uint16_t *kdst = const_cast<uint16_t *>(kc) + (size_t)a.pos * QDB_HD;
        uint16_t *vdst = const_cast<uint16_t *>(vc) + (size_t)a.pos * QDB_HD;
        for (int i = lane; i < QDB_HD; i += 32) {
            kdst[i] = f32_to_bf16_rn(sm->knew[i]);
            vdst[i] = f32_to_bf16_rn(__ldcg(a.qkv + qd + kvd + g * QDB_HD + i));
        }
    }
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
    for (int base = p0 + warp * ATT_KEYS; base < p1; base += WPB * ATT_KEYS) {
        const int j = base + kk;
        const bool valid = j < p1;
        uint4 kv4[4];
        if (valid) {
            const uint4 *kp = reinterpret_cast<const uint4 *>(kc + (size_t)j * QDB_HD + sub * 32);
#pragma unroll
            for (int u = 0; u < 4; u++) kv4[u] = __ldcg(kp + u);
        }
        uint2 vv[ATT_KEYS];
#pragma unroll
        for (int t = 0; t < ATT_KEYS; t++) {
            const int jt = base + t;
            if (jt < p1) vv[t] = __ldcg(reinterpret_cast<const uint2 *>(vc + (size_t)jt * QDB_HD + lane * 4));
            else vv[t] = make_uint2(0u, 0u);
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
                    acc = dot8(kv4[u], qa, qb, acc);
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
            l[h] = l[h] * corr + ps;  // xor 4/8/16 sums the 8 keys once each
#pragma unroll
            for (int e = 0; e < 4; e++) o[h][e] *= corr;
#pragma unroll
            for (int t = 0; t < ATT_KEYS; t++) {
                const float pt = __shfl_sync(0xffffffffu, p, t * 4);
                o[h][0] = fmaf(pt, bf16lo(vv[t].x), o[h][0]);
                o[h][1] = fmaf(pt, bf16hi(vv[t].x), o[h][1]);
                o[h][2] = fmaf(pt, bf16lo(vv[t].y), o[h][2]);
                o[h][3] = fmaf(pt, bf16hi(vv[t].y), o[h][3]);
            }
            m[h] = mn;
        }
    }
    // Merge the warps of this CTA.
#pragma unroll
    for (int h = 0; h < R; h++) {
        if (lane == 0) {
            sm->m[warp][h] = m[h];
            sm->l[warp][h] = l[h];
        }
#pragma unroll
        for (int e = 0; e < 4; e++) sm->o[warp][h][lane * 4 + e] = o[h][e];
    }
    __syncthreads();
    for (int t = threadIdx.x; t < R * QDB_HD; t += blockDim.x) {
        const int h = t / QDB_HD, dd = t % QDB_HD;
        float M = -INFINITY;
        for (int w = 0; w < WPB; w++) M = fmaxf(M, sm->m[w][h]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
            for (int w = 0; w < WPB; w++) {
                const float f = expf(sm->m[w][h] - M);
                L += sm->l[w][h] * f;
                O += sm->o[w][h][dd] * f;
            }
        }
        float *dst = a.part + ((size_t)(g * R + h) * S + s) * (2 + QDB_HD);
        if (dd == 0) {
            dst[0] = M;
            dst[1] = L;
        }
        dst[2 + dd] = O;
    }
}

// Last unit of KV head g: merge the S split partials into attn.
template <int R>
__device__ void attn_merge(const QdbStepArgs &a, int g, int S) {
    for (int t = threadIdx.x; t < R * QDB_HD; t += blockDim.x) {
        const int h = t / QDB_HD, dd = t % QDB_HD;
        const float *src = a.part + (size_t)(g * R + h) * S * (2 + QDB_HD);
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
        a.attn[(g * R + h) * QDB_HD + dd] = L > 0.f ? O / L : 0.f;
    }
}

template <int R>
__device__ void phase_attention(const QdbStepArgs &a, int layer, AttnSmem *sm, volatile int *s_last) {
    const int S = a.splits;
    const int units = a.d.Hkv * S;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int g = u / S, s = u % S;
        attn_unit<R>(a, layer, g, s, S, sm);
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            const unsigned old = atomicAdd(a.cnt + g, 1u);
            *s_last = (old == (unsigned)S - 1u);
            __threadfence();
        }
        __syncthreads();
        if (*s_last) {
            attn_merge<R>(a, g, S);
            __syncthreads();
            if (threadIdx.x == 0) a.cnt[g] = 0u;
        }
        __syncthreads();
    }
}

template <int R>
__global__ void __launch_bounds__(QDB_STEP_THREADS, 1) step_kernel(const QdbStepArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ float red[32];
    __shared__ volatile int s_flag;
    float *xs = reinterpret_cast<float *>(smem_raw);
    AttnSmem *asm_ = reinterpret_cast<AttnSmem *>(smem_raw);

    const QdbDims &d = a.d;
    const int h = d.h, qd = d.Hq * QDB_HD, kvd = d.Hkv * QDB_HD, I = d.I;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = blockIdx.x * WPB + warp, TW = gridDim.x * WPB;
    unsigned target = a.bar_base;

    const uint16_t *emb_row = nullptr;
    if (a.token_in) emb_row = a.embed + (size_t)__ldcg(a.token_in) * h;

    for (int layer = 0; layer < d.L; layer++) {
        const QdbLayerW &lw = a.layers[layer];
        // ---- A: input norm + QKV rows ----
        const bool first = (layer == 0 && emb_row != nullptr);
        norm_to_smem(a.x, first ? emb_row : nullptr, lw.in_norm, h, d.eps, xs, red);
        if (first && blockIdx.x == 0)
            for (int i = threadIdx.x; i < h; i += blockDim.x) a.x[i] = __uint_as_float(((uint32_t)emb_row[i]) << 16);
        {
            const int R3 = qd + 2 * kvd;
            for (int r = gw; r < R3; r += 2 * TW) {
                const int r1 = r + TW;
                if (r1 < R3) {
                    float s0, s1;
                    row_dot2(lw.qkv + (size_t)r * h, lw.qkv + (size_t)r1 * h, xs, h, s0, s1);
                    if (lane == 0) { a.qkv[r] = s0; a.qkv[r1] = s1; }
                } else {
                    const float s0 = row_dot(lw.qkv + (size_t)r * h, xs, h);
                    if (lane == 0) a.qkv[r] = s0;
                }
            }
        }
        target += gridDim.x;
        if (!grid_barrier(a.bar, target, a.err, &s_flag)) return;

        // ---- B: QK norm, RoPE, KV append, attention ----
        phase_attention<R>(a, layer, asm_, &s_flag);
        target += gridDim.x;
        if (!grid_barrier(a.bar, target, a.err, &s_flag)) return;

        // ---- C: O-proj + residual ----
        load_to_smem(a.attn, qd, xs);
        for (int r = gw; r < h; r += TW) {
            const float s0 = row_dot(lw.o + (size_t)r * qd, xs, qd);
            if (lane == 0) a.x[r] = __ldcg(a.x + r) + s0;
        }
        target += gridDim.x;
        if (!grid_barrier(a.bar, target, a.err, &s_flag)) return;

        // ---- D: post-attention norm + gate/up pairs + SwiGLU ----
        norm_to_smem(a.x, nullptr, lw.post_norm, h, d.eps, xs, red);
        for (int j = gw; j < I; j += TW) {
            float g, u;
            row_dot2(lw.gu + (size_t)(2 * j) * h, lw.gu + (size_t)(2 * j + 1) * h, xs, h, g, u);
            if (lane == 0) a.act[j] = silu_mul(g, u);
        }
        target += gridDim.x;
        if (!grid_barrier(a.bar, target, a.err, &s_flag)) return;

        // ---- E: down + residual ----
        load_to_smem(a.act, I, xs);
        for (int r = gw; r < h; r += TW) {
            const float s0 = row_dot(lw.down + (size_t)r * I, xs, I);
            if (lane == 0) a.x[r] = __ldcg(a.x + r) + s0;
        }
        target += gridDim.x;
        if (!grid_barrier(a.bar, target, a.err, &s_flag)) return;
    }

    // ---- F: final norm + tied lm_head + greedy argmax ----
    norm_to_smem(a.x, nullptr, a.final_norm, h, d.eps, xs, red);
    if (blockIdx.x == 0 && a.hidden_out)
        for (int i = threadIdx.x; i < h; i += blockDim.x) a.hidden_out[i] = xs[i];
    unsigned long long best = 0ull;
    for (int r = gw; r < d.V; r += 2 * TW) {
        const int r1 = r + TW;
        float s0, s1 = 0.f;
        if (r1 < d.V) row_dot2(a.embed + (size_t)r * h, a.embed + (size_t)r1 * h, xs, h, s0, s1);
        else s0 = row_dot(a.embed + (size_t)r * h, xs, h);
        if (lane == 0) {
            if (a.logits_out) {
                a.logits_out[r] = s0;
                if (r1 < d.V) a.logits_out[r1] = s1;
            }
            if (!(a.mask_eos && (r == QDB_ENDOFTEXT || r == QDB_IM_END)) && !isnan(s0)) {
                const unsigned long long k = argmax_key(s0, r);
                best = k > best ? k : best;
            }
            if (r1 < d.V && !(a.mask_eos && (r1 == QDB_ENDOFTEXT || r1 == QDB_IM_END)) && !isnan(s1)) {
                const unsigned long long k = argmax_key(s1, r1);
                best = k > best ? k : best;
            }
        }
    }
    if (lane == 0 && best) atomicMax(a.best, best);
    target += gridDim.x;
    if (!grid_barrier(a.bar, target, a.err, &s_flag)) return;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        const unsigned long long b = __ldcg(a.best);
        *a.token_out = argmax_key_index(b);
        *a.best = 0ull;
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

}  // namespace

extern "C" int qdb_step_smem_bytes(const QdbDims &d) {
    const int qd = d.Hq * QDB_HD;
    int n = d.h;
    if (qd > n) n = qd;
    if (d.I > n) n = d.I;
    int bytes = n * (int)sizeof(float);
    if ((int)sizeof(AttnSmem) > bytes) bytes = (int)sizeof(AttnSmem);
    return bytes;
}

template <int R>
static cudaError_t launch_r(const QdbStepArgs &a, int grid, cudaStream_t st) {
    const int smem = qdb_step_smem_bytes(a.d);
    cudaError_t e = cudaFuncSetAttribute(step_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    void *args[] = {const_cast<QdbStepArgs *>(&a)};
    return cudaLaunchCooperativeKernel((const void *)step_kernel<R>, dim3(grid), dim3(QDB_STEP_THREADS), args,
                                       (size_t)smem, st);
}

extern "C" cudaError_t qdb_launch_step(const QdbStepArgs &a, int grid, cudaStream_t st) {
    const int R = a.d.Hq / a.d.Hkv;
    switch (R) {
        case 1: return launch_r<1>(a, grid, st);
        case 2: return launch_r<2>(a, grid, st);
        case 4: return launch_r<4>(a, grid, st);
        case 8: return launch_r<8>(a, grid, st);
        default: return cudaErrorInvalidValue;
    }
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
