// qdb_attn_tc.cu - causal GQA prefill attention on the 5th-generation tensor
// cores (tcgen05), replacing the CUDA-core flash attention for the prompt of
// qwen_decoder_prefill (qwen_asr_decoder.c:262-359; per-position math of
// qwen_causal_attention, qwen_asr_kernels.c:1117-1180: scores scaled by
// 1/sqrt(head_dim), softmax over keys <= the query position, weighted V sum).
//
// One CTA = one KV head g x one query tile of QT positions, all R query heads
// of the group: 128 MMA rows (row r = position r / R, head r % R). 128
// threads, thread = row = TMEM lane. TMEM: S (128 columns) and O (128 columns).
//
//   S = Q K^T      A = Q rows (fp16 hi + lo of the f32 q, written by threads),
//                  B = 128 cached keys (fp16, TMA 2D with 128-byte swizzle)
//   per key tile  online softmax: row max of S, P = exp(s - m) as fp16
//                  (threads), the running max raised (O rescaled in
//                  TMEM) only when it grows by more than 8; O += P V in TMEM
//                  with V straight from its TMA tile as an MN-major B operand
//                  (keys along K, dims along N); O / l in the epilogue
//
// All operands are K-major with 128-byte swizzle (the layout the TMA writes
// for the K tile and the threads write for Q and P). The q halves keep ~22
// mantissa bits of the f32 q; P in [0, 1] is rounded to fp16 (relative error
// <= 2^-11 per weight, the order of the fp16 cache rounding of V; the hi + lo
// form is QDB_AT_PLO=1); K and V are the cache's own fp16 values; f32
// accumulation.
// Every mbarrier wait is bounded (error word + early exit); TMEM is always
// released.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include "qdb_common.cuh"
#include "qdb_kernels.h"

namespace {

constexpr int AT_THREADS = 256;  // two threads per MMA row: warps w and w + 4 share TMEM lanes, split the columns
constexpr int AT_M = 128;          // MMA rows per CTA (query vectors)
constexpr int AT_N = 128;          // keys per tile
constexpr int AT_TILE = 128 * 128; // bytes of one 128-row x 64-column fp16 swizzled tile (16 KB)

typedef unsigned long long u64;

__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mb_init(u64 *b, unsigned n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
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
// Bounded wait of one thread; false = ran out (error recorded).
__device__ bool mb_wait(u64 *b, unsigned par, int *err) {
    const long long t0 = clock64();
    while (!mb_try(b, par)) {
        if (clock64() - t0 > QDB_SPIN_LIMIT_CYCLES) {
            set_error(err, QDB_ERR_BARRIER_TIMEOUT);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, u64 *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(su32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(su32(bar))
        : "memory");
}

// K-major operand descriptor, 128-byte swizzle: rows of 128 bytes in
// 1024-byte 8-row atoms (start >> 4 in bits 0-13, leading offset 16 B in
// 16-29, 8-row-group stride 1024 B in 32-45, version 1 at bit 46, layout 2 =
// 128-byte swizzle in bits 61-63).
__device__ __forceinline__ u64 sm_desc(uint32_t saddr) {
    u64 d = 0;
    d |= (u64)((saddr >> 4) & 0x3fffu);
    d |= (u64)1 << 16;
    d |= (u64)(1024 >> 4) << 32;
    d |= (u64)1 << 46;
    d |= (u64)2 << 61;
    return d;
}

// MN-major operand descriptor, 128-byte swizzle: rows of 128 bytes (64 fp16
// of the N dimension) along K, 8-row atoms 1024 B apart (stride offset), the
// next 64 N-elements lbo bytes away (leading offset).
__device__ __forceinline__ u64 sm_desc_mn(uint32_t saddr, uint32_t lbo) {
    u64 d = 0;
    d |= (u64)((saddr >> 4) & 0x3fffu);
    d |= (u64)((lbo >> 4) & 0x3fffu) << 16;
    d |= (u64)(1024 >> 4) << 32;
    d |= (u64)1 << 46;
    d |= (u64)2 << 61;
    return d;
}

// Instruction descriptor, kind::f16 with fp16 A and B (format 0 in bits 7-9
// and 10-12), f32 D (bits 4-5 = 1), both K-major, N >> 3 at bit 17, M >> 4 at 24.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem, u64 a, u64 b, uint32_t idesc, uint32_t acc) {
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
// Generic-proxy shared-memory writes become visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
        "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

// Byte offset of 16-byte chunk c (8 fp16 columns) of row r in a 128-row x
// 64-column swizzled tile: 8-row atoms of 1024 B, chunk index XOR (r & 7).
__device__ __forceinline__ uint32_t swz(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t h2u(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

#ifndef QDB_AT_PLO
#define QDB_AT_PLO 0  // 1: P as fp16 hi + lo tiles (two P.V MMAs per step); 0: P as fp16
#endif

// Writes 8 f32 values as fp16 (tile hi), chunk c of row r.
__device__ __forceinline__ void put8_hi(unsigned char *hi, int r, int c, const float *v) {
    __half h[8];
#pragma unroll
    for (int i = 0; i < 8; i++) h[i] = __float2half_rn(v[i]);
    *reinterpret_cast<uint4 *>(hi + swz(r, c)) =
        make_uint4(h2u(h[0], h[1]), h2u(h[2], h[3]), h2u(h[4], h[5]), h2u(h[6], h[7]));
}

// Writes 8 f32 values as fp16 hi (tile hi) and lo = fp16(v - hi) (tile lo),
// chunk c of row r.
__device__ __forceinline__ void put8_split(unsigned char *hi, unsigned char *lo, int r, int c, const float *v) {
    __half h[8], l[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        h[i] = __float2half_rn(v[i]);
        l[i] = __float2half_rn(v[i] - __half2float(h[i]));
    }
    const uint32_t off = swz(r, c);
    *reinterpret_cast<uint4 *>(hi + off) = make_uint4(h2u(h[0], h[1]), h2u(h[2], h[3]), h2u(h[4], h[5]), h2u(h[6], h[7]));
    *reinterpret_cast<uint4 *>(lo + off) = make_uint4(h2u(l[0], l[1]), h2u(l[2], l[3]), h2u(l[4], l[5]), h2u(l[6], l[7]));
}

template <int R>
__global__ void __launch_bounds__(AT_THREADS, 1)
    attn_tc_kernel(const CUtensorMap *__restrict__ maps, const QdbAttnSeg *__restrict__ segs, int layer, int Hkv,
                   const float *__restrict__ q, int Hq, float *__restrict__ out, int *err, uint16_t *hi,
                   uint16_t *lo) {
    constexpr int QT = AT_M / R;  // query positions per CTA
    extern __shared__ __align__(1024) unsigned char smem_dyn[];
    __shared__ __align__(8) u64 barK, barS, barO;
    __shared__ uint32_t tmem_slot;
    __shared__ int s_ok;
    unsigned char *sm = smem_dyn + ((1024u - (su32(smem_dyn) & 1023u)) & 1023u);
    unsigned char *Qh = sm, *Ql = sm + 2 * AT_TILE;              // [2 dim blocks] each
    unsigned char *Kt = sm + 4 * AT_TILE;                         // [2 dim blocks] (TMA)
    unsigned char *Ph = sm + 6 * AT_TILE, *Pl = sm + 8 * AT_TILE; // [2 key blocks] each

    // segment = one session's prompt rows; its K/V maps cover all layers
    const QdbAttnSeg sg = segs[blockIdx.z];
    const int cap = sg.cap, start_pos = sg.start_pos, n = sg.n;
    const int i0 = blockIdx.x * QT;
    if (i0 >= n) return;  // shorter segment than the grid's longest (uniform per CTA)
    const CUtensorMap *tmK = maps + 2 * blockIdx.z, *tmV = tmK + 1;
    q += (size_t)sg.row0 * Hq * QDB_HD;
    out += (size_t)sg.row0 * Hq * QDB_HD;
    if (hi) {
        hi += (size_t)sg.row0 * Hq * QDB_HD;
        lo += (size_t)sg.row0 * Hq * QDB_HD;
    }
    const int t = threadIdx.x, warp = t >> 5;
    const int g = blockIdx.y;
    const int kv_row0 = (layer * Hkv + g) * cap;  // this layer's KV head g in the all-layer map
    const int half = warp >> 2;                     // this thread's half of the row's columns
    const int r = 32 * (warp & 3) + (t & 31), p = r / R, h = r % R;  // MMA row: position i0 + p, head g*R + h
    const bool row_ok = i0 + p < n;
    const int qpos = start_pos + i0 + p;
    const int kend = start_pos + min(n, i0 + QT);  // keys this tile needs
    const int ntiles = (kend + AT_N - 1) / AT_N;
    const float scale = 1.0f / sqrtf((float)QDB_HD);

    if (t == 0) {
        mb_init(&barK, 1);
        mb_init(&barS, 1);
        mb_init(&barO, 1);
        s_ok = 1;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_slot)),
                     "r"(256)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // Q rows -> fp16 hi/lo swizzled tiles (zeros past the prompt)
    {
        const float *src = q + (size_t)(i0 + p) * Hq * QDB_HD + (size_t)(g * R + h) * QDB_HD;
#pragma unroll 1
        for (int c = half * 8; c < half * 8 + 8; c++) {
            float v[8];
            if (row_ok) {
                const float4 a = *reinterpret_cast<const float4 *>(src + c * 8);
                const float4 b = *reinterpret_cast<const float4 *>(src + c * 8 + 4);
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] = 0.f;
            }
            put8_split(Qh + (c >> 3) * AT_TILE, Ql + (c >> 3) * AT_TILE, r, c & 7, v);
        }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot, tS = tmem, tO = tmem + 128;
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    constexpr uint32_t idesc = idesc_f16(AT_M, AT_N);
    unsigned phK = 0, phS = 0, phO = 0;

    // thread 0: K tile k0 by TMA, then S = Q K^T into TMEM; false = a wait ran out
    auto s_tile = [&](int k0) -> bool {
        mb_expect(&barK, 2 * AT_TILE);
        tma_load_2d(Kt, tmK, 0, kv_row0 + k0, &barK);
        tma_load_2d(Kt + AT_TILE, tmK, 64, kv_row0 + k0, &barK);
        if (!mb_wait(&barK, phK, err)) return false;
        phK ^= 1;
        tc_fence_after();
#pragma unroll
        for (int kb = 0; kb < 2; kb++)
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const u64 bk = sm_desc(su32(Kt + kb * AT_TILE) + k * 32);
                mma_f16(tS, sm_desc(su32(Qh + kb * AT_TILE) + k * 32), bk, idesc, (kb | k) ? 1u : 0u);
                mma_f16(tS, sm_desc(su32(Ql + kb * AT_TILE) + k * 32), bk, idesc, 1u);
            }
        mma_commit(&barS);
        if (!mb_wait(&barS, phS, err)) return false;
        phS ^= 1;
        return true;
    };

    // ---- one pass over the key tiles (online softmax): per tile the row max
    // of S, then P = exp(s - m) with the row's running max m, O += P V. m is
    // raised (and O, l rescaled by exp(m_old - m_new) in TMEM) only when a
    // tile's max exceeds it by more than RESCALE, so P <= e^RESCALE: numerator
    // and denominator always share one m, and the rescale is rare after the
    // first tiles. The epilogue divides by l.
    constexpr float RESCALE = 8.0f;
    __shared__ float xch[AT_THREADS];  // the two column halves' tile maxima
    float m = -INFINITY, l = 0.f;      // running max (same in both halves of a row), this half's sum
#pragma unroll 1
    for (int kt = 0; kt < ntiles && s_ok; kt++) {
        const int k0 = kt * AT_N;
        if (t == 0) {
            if (!s_tile(k0)) {
                s_ok = 0;
            } else {  // the K buffer is free once S is done: V of this tile into it
                mb_expect(&barK, 2 * AT_TILE);
                tma_load_2d(Kt, tmV, 0, kv_row0 + k0, &barK);
                tma_load_2d(Kt + AT_TILE, tmV, 64, kv_row0 + k0, &barK);
            }
        }
        __syncthreads();
        if (!s_ok) break;
        tc_fence_after();
        float v[64];
        tmem_ld32(tS + lane_base + half * 64, v);
        tmem_ld32(tS + lane_base + half * 64 + 32, v + 32);
        float cm = -INFINITY;
#pragma unroll
        for (int j = 0; j < 64; j++) {
            const bool ok = row_ok && k0 + half * 64 + j <= qpos;
            v[j] = ok ? v[j] * scale : -INFINITY;
            cm = fmaxf(cm, v[j]);
        }
        xch[t] = cm;
        __syncthreads();
        cm = fmaxf(cm, xch[t ^ 128]);
        if (cm > m + RESCALE || (m == -INFINITY && cm != -INFINITY)) {
            if (m != -INFINITY) {  // O holds earlier tiles: rescale this half of the row
                const float f = expf(m - cm);
                l *= f;
                float o[32];
#pragma unroll 1
                for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 32) {
                    tmem_ld32(tO + lane_base + c0, o);
#pragma unroll
                    for (int j = 0; j < 32; j++) o[j] *= f;
                    tmem_st32(tO + lane_base + c0, o);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            }
            m = cm;
        }
#pragma unroll
        for (int j = 0; j < 64; j++) {
            v[j] = v[j] == -INFINITY ? 0.f : expf(v[j] - m);
            l += v[j];
        }
#pragma unroll
        for (int q8 = 0; q8 < 8; q8++) {
            const int col = half * 64 + q8 * 8;  // key column within the tile
            if (QDB_AT_PLO)
                put8_split(Ph + (col >> 6) * AT_TILE, Pl + (col >> 6) * AT_TILE, r, (col & 63) >> 3, v + q8 * 8);
            else
                put8_hi(Ph + (col >> 6) * AT_TILE, r, (col & 63) >> 3, v + q8 * 8);
        }
        // V: wait for its tile
        if (t == 0 && s_ok) {
            if (!mb_wait(&barK, phK, err)) s_ok = 0;
            phK ^= 1;
        }
        tc_fence_before();
        __syncthreads();
        if (s_ok) {
            // V as loaded is the MN-major B operand already; only the rows past
            // the last valid key (stale cache memory) are cleared
            const int nvalid = kend - k0;
            if (nvalid < AT_N) {
                for (int i = t; i < (AT_N - nvalid) * 16; i += AT_THREADS) {
                    const int key = nvalid + (i >> 4), chunk = i & 15;  // 16 chunks of 16 B: 2 dim halves x 8
                    *reinterpret_cast<uint4 *>(Kt + (chunk >> 3) * AT_TILE + swz(key, chunk & 7)) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
            }
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (t == 0 && s_ok) {
            tc_fence_after();
#pragma unroll
            for (int kb = 0; kb < 2; kb++)
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    // B = V as loaded: keys along K, dims along N (MN-major)
                    const u64 bv = sm_desc_mn(su32(Kt) + (kb * 64 + k * 16) * 128, AT_TILE);
                    const uint32_t id = idesc | (1u << 16);  // bit 16: B is MN-major
                    mma_f16(tO, sm_desc(su32(Ph + kb * AT_TILE) + k * 32), bv, id, (kt | kb | k) ? 1u : 0u);
                    if (QDB_AT_PLO) mma_f16(tO, sm_desc(su32(Pl + kb * AT_TILE) + k * 32), bv, id, 1u);
                }
            mma_commit(&barO);
            if (!mb_wait(&barO, phO, err)) s_ok = 0;
            phO ^= 1;
        }
        __syncthreads();
    }
    // the row's denominator: both halves' sums (same m)
    xch[t] = l;
    __syncthreads();
    l += xch[t ^ 128];
    const float inv_l = l > 0.f ? 1.0f / l : 0.f;
    // ---- epilogue: O row -> out
    if (s_ok && ntiles > 0) {
        tc_fence_after();
        const size_t at = (size_t)(i0 + p) * Hq * QDB_HD + (size_t)(g * R + h) * QDB_HD;
        float *dst = out + at;
#pragma unroll 1
        for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 32) {
            float v[32];
            tmem_ld32(tO + lane_base + c0, v);
            if (!row_ok) continue;
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] *= inv_l;
            if (hi) {  // the bf16 split the O-projection GEMM reads
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const uint16_t b0 = f32_to_bf16_rn(v[j]), b1 = f32_to_bf16_rn(v[j + 1]);
                    const uint16_t l0 = f32_to_bf16_rn(v[j] - __uint_as_float((uint32_t)b0 << 16));
                    const uint16_t l1 = f32_to_bf16_rn(v[j + 1] - __uint_as_float((uint32_t)b1 << 16));
                    *reinterpret_cast<uint32_t *>(hi + at + c0 + j) = (uint32_t)b0 | ((uint32_t)b1 << 16);
                    *reinterpret_cast<uint32_t *>(lo + at + c0 + j) = (uint32_t)l0 | ((uint32_t)l1 << 16);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4 *>(dst + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn_at() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

template <int R>
cudaError_t launch_at(const CUtensorMap *maps, const QdbAttnSeg *segs, int nseg, int max_n, int layer, int Hq, int Hkv,
                      const float *q, float *out, int *err, cudaStream_t st, uint16_t *hi, uint16_t *lo) {
    const int smem = 10 * AT_TILE + 1024;  // Q hi/lo, K (then V), P hi/lo + alignment slack
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    constexpr int QT = AT_M / R;
    dim3 grid((max_n + QT - 1) / QT, Hkv, nseg);
    attn_tc_kernel<R><<<grid, AT_THREADS, smem, st>>>(maps, segs, layer, Hkv, q, Hq, out, err, hi, lo);
    return cudaGetLastError();
}

}  // namespace

// Tensor map (written to host memory, 128 bytes) of one session's fp16 K or V
// cache [L][Hkv][cap][128] as [L * Hkv * cap rows][128]: 64-column x 128-row
// boxes, 128-byte swizzle. 0 = ok.
extern "C" int qdb_attn_kv_map(void *map, const uint16_t *cache, int L, int Hkv, int cap) {
    auto fn = encode_fn_at();
    if (!fn || ((uintptr_t)cache & 15)) return -1;
    cuuint64_t dims[2] = {(cuuint64_t)QDB_HD, (cuuint64_t)L * Hkv * (cuuint64_t)cap};
    cuuint64_t strides[1] = {(cuuint64_t)QDB_HD * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)AT_N};
    cuuint32_t es[2] = {1, 1};
    return fn(reinterpret_cast<CUtensorMap *>(map), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t *>(cache),
              dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
               ? 0
               : -1;
}

// Causal prefill attention of one layer for nseg sessions at once on the
// tensor cores. Segment i: prompt rows [row0, row0 + n) of q / out are the
// session's positions [start_pos, start_pos + n); its K and V maps
// (qdb_attn_kv_map) are maps[2i] and maps[2i + 1] (device memory); the caches
// already hold keys [0, start_pos + n) of this layer. q: f32 [rows, Hq*128]
// (normed, rotated); out: f32 [rows, Hq*128], or its bf16 split into hi/lo.
extern "C" cudaError_t qdb_launch_attn_prefill_tc(const void *maps, const QdbAttnSeg *segs, int nseg, int max_n,
                                                  int layer, int Hq, int Hkv, const float *q, float *out, int *err,
                                                  cudaStream_t st, uint16_t *hi, uint16_t *lo) {
    if (nseg <= 0 || max_n <= 0) return cudaSuccess;
    if (Hkv <= 0 || Hq % Hkv || !maps || !segs) return cudaErrorInvalidValue;
    if (((uintptr_t)q | (uintptr_t)out | (uintptr_t)maps) & 15) return cudaErrorInvalidValue;
    const CUtensorMap *m = reinterpret_cast<const CUtensorMap *>(maps);
    switch (Hq / Hkv) {
        case 1: return launch_at<1>(m, segs, nseg, max_n, layer, Hq, Hkv, q, out, err, st, hi, lo);
        case 2: return launch_at<2>(m, segs, nseg, max_n, layer, Hq, Hkv, q, out, err, st, hi, lo);
        case 4: return launch_at<4>(m, segs, nseg, max_n, layer, Hq, Hkv, q, out, err, st, hi, lo);
        case 8: return launch_at<8>(m, segs, nseg, max_n, layer, Hq, Hkv, q, out, err, st, hi, lo);
        default: return cudaErrorInvalidValue;
    }
}
