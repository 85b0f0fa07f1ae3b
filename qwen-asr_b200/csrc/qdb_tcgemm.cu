// qdb_tcgemm.cu - tcgen05 (5th-generation tensor core) GEMM for the
// row-batched path: prefill of one utterance (qwen_decoder_prefill,
// qwen_asr_decoder.c:262-359, whose projections the reference runs as
// cblas_sgemm after a bf16->f32 copy of the weight, qwen_asr_kernels.c:462-472)
// and one decode step of many utterances.
//
//   Y[n, N] (op)= X[n, K] * W[N, K]^T     X f32 (given as bf16 hi + lo), W bf16
//
// The f32 activations are split as X = Xhi + Xlo (both bf16, Xlo = bf16 of
// the residual); both halves are multiplied into the SAME f32 TMEM
// accumulator, so the product keeps ~16 mantissa bits of X instead of bf16's 8
// and stays within the f32 reference's tolerance.
//
// One CTA per 128 weight rows x BN activation rows. Warp roles:
//   warp 0       TMA producer: W / Xhi / Xlo K-slices (64 bf16 = 128 B, 128B
//                swizzle) into an S-stage shared-memory ring (each CTA loads its own tiles)
//   warp 1       allocates TMEM; one thread issues tcgen05.mma (M=128, N=BN,
//                K=16, kind::f16 bf16 x bf16 -> f32), commits stages back
//   warps 2..5   epilogue: tcgen05.ld of the accumulator (each warp its 32
//                TMEM lanes = 32 weight rows), store / add / SwiGLU to Y
// Every wait is bounded (error word + skip); TMEM is always released.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "qdb_common.cuh"
#include "qdb_kernels.h"

namespace {

constexpr int TC_BM = 128;  // weight rows per tile (MMA M)
constexpr int TC_BK = 64;   // K per stage (128 bytes of bf16: one swizzle row)
constexpr int TC_THREADS = 192;

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
// Bounded wait of one thread; false = ran out (error recorded). Data waits
// (a stage's copies, a free stage) use the run-time limit; the waits that must
// not be cut short (the accumulator before TMEM is read and released, the
// producer's copies in flight before it exits) pass fixed = true.
__device__ bool mb_wait(u64 *b, unsigned par, int *err, bool fixed = false) {
    const long long t0 = clock64();
    const long long limit = fixed ? QDB_SPIN_LIMIT_CYCLES : qdb_wait_limit_c;
    while (!mb_try(b, par)) {
        if (clock64() - t0 > limit) {
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

// Same load with an L2 cache policy on the global reads.
__device__ __forceinline__ void tma_load_2d_pol(void *dst, const CUtensorMap *map, int x, int y, u64 *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3}], [%4], %5;" ::"r"(su32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(su32(bar)), "l"(pol)
        : "memory");
}

#ifndef QDB_GEMM_PDL
#define QDB_GEMM_PDL 1  // programmatic dependent launch: weight prefetch overlaps the previous kernel
#endif
#ifndef QDB_GEMM_W_EVICT_FIRST
#define QDB_GEMM_W_EVICT_FIRST 1
#endif

// Shared-memory matrix descriptor: K-major operand, rows of 128 bytes in
// 1024-byte 8-row swizzle atoms (128-byte swizzle). start >> 4 in bits 0-13,
// leading offset 16 B (unused for this layout) in 16-29, stride between
// 8-row groups (1024 B) in 32-45, descriptor version 1 in 46-47, layout type
// 2 (128-byte swizzle) in 61-63.
__device__ __forceinline__ u64 sm_desc(uint32_t saddr) {
    u64 d = 0;
    d |= (u64)((saddr >> 4) & 0x3fffu);
    d |= (u64)1 << 16;
    d |= (u64)(1024 >> 4) << 32;
    d |= (u64)1 << 46;
    d |= (u64)2 << 61;
    return d;
}

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A bf16 (7-9 = 1),
// B bf16 (10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t instr_desc(int M, int N) {
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

template <int BN, int S, bool BIAS, int MODE>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmXh,
                   const __grid_constant__ CUtensorMap tmXl, float *__restrict__ Y, int n, int N, int K, int mode,
                   int kb_per, int *err, const float *__restrict__ bias) {
    if (MODE >= 0) mode = MODE;  // fixed-mode instantiations (decode) compile one store path
    constexpr int A_BYTES = TC_BM * TC_BK * 2;  // 16 KB
    constexpr int B_BYTES = BN * TC_BK * 2;
    constexpr int STAGE = A_BYTES + 2 * B_BYTES;
    extern __shared__ __align__(1024) unsigned char smem_dyn[];
    __shared__ __align__(8) u64 full[S], empty[S], accum;
    __shared__ uint32_t tmem_slot;

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // successors may become resident
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * TC_BM, a0 = blockIdx.y * BN;
    // split-K: this CTA takes k-blocks [kb0, kb0 + nk) (gridDim.z splits)
    const int kb0 = blockIdx.z * kb_per;
    const int nk = min(K / TC_BK - kb0, kb_per);
    // 128-byte swizzle atoms need 1024-byte aligned tiles: round the base up
    // (the launch reserves 1 KB of slack for this)
    unsigned char *smem = smem_dyn + ((1024u - (su32(smem_dyn) & 1023u)) & 1023u);
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            mb_init(&full[i], 1);
            mb_init(&empty[i], 1);
        }
        mb_init(&accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_slot)),
                     "r"(BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---- TMA producer. With one activation tile (decode batches) every
        // weight tile is read exactly once: stream it evict-first so the KV
        // caches the attention kernels read stay in L2.
        const bool w_once = QDB_GEMM_W_EVICT_FIRST && gridDim.y == 1;
        uint64_t pol = 0;
        if (w_once) asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
        // Weights do not depend on the kernels before this one: the first S
        // weight tiles are requested before griddepcontrol.wait (launched
        // with programmatic dependent launch, this overlaps the previous
        // kernel); activation tiles only after it.
        const int pre = nk < S ? nk : S;
        for (int kb = 0; kb < pre; kb++) {
            unsigned char *st = smem + (size_t)kb * STAGE;
            mb_expect(&full[kb], STAGE);
            const int kx = (kb0 + kb) * TC_BK;
            if (w_once) tma_load_2d_pol(st, &tmW, kx, m0, &full[kb], pol);
            else tma_load_2d(st, &tmW, kx, m0, &full[kb]);
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");
        int issued = 0;
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % S;
            if (kb >= S && !mb_wait(&empty[s], ((kb / S) - 1) & 1, err)) break;
            unsigned char *st = smem + (size_t)s * STAGE;
            const int kx = (kb0 + kb) * TC_BK;
            if (kb >= pre) {
                mb_expect(&full[s], STAGE);
                if (w_once) tma_load_2d_pol(st, &tmW, kx, m0, &full[s], pol);
                else tma_load_2d(st, &tmW, kx, m0, &full[s]);
            }
            tma_load_2d(st + A_BYTES, &tmXh, kx, a0, &full[s]);
            tma_load_2d(st + A_BYTES + B_BYTES, &tmXl, kx, a0, &full[s]);
            issued = kb + 1;
        }
        // wait for the last copies of every stage to land before leaving
        for (int kb = issued > S ? issued - S : 0; kb < issued; kb++) mb_wait(&full[kb % S], (kb / S) & 1, err, true);
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        constexpr uint32_t idesc = instr_desc(TC_BM, BN);
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % S;
            if (!mb_wait(&full[s], (kb / S) & 1, err)) break;
            tc_fence_after();
            const uint32_t base = su32(smem + (size_t)s * STAGE);
#pragma unroll
            for (int k = 0; k < TC_BK / 16; k++) {
                const u64 ad = sm_desc(base + k * 32);
                const u64 bh = sm_desc(base + A_BYTES + k * 32);
                const u64 bl = sm_desc(base + A_BYTES + B_BYTES + k * 32);
                mma_bf16(tmem, ad, bh, idesc, (kb | k) ? 1u : 0u);
                mma_bf16(tmem, ad, bl, idesc, 1u);
            }
            mma_commit(&empty[s]);  // frees the stage once these MMAs have read it
        }
        mma_commit(&accum);  // completes when every issued MMA is done
    } else if (warp >= 2) {
        // ---- epilogue: warp q reads TMEM lanes [32q, 32q+32) = weight rows
        const int q = warp & 3;
        asm volatile("griddepcontrol.wait;" ::: "memory");  // Y (residual / zeroed target) is the predecessors' output
        bool ok = true;
        if (lane == 0) ok = mb_wait(&accum, 0, err, true);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        tc_fence_after();
        const int wrow = m0 + 32 * q + lane;
        // bias[wrow] is added once, by the first K-split (a separate
        // instantiation: the bias-free kernels compile without it; measured
        // 13% slower on the decode GEMMs when it was a runtime branch)
        float bb = 0.f;
        if (BIAS) bb = (blockIdx.z == 0 && wrow < N) ? bias[wrow] : 0.f;
        if (ok) {
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                float v[32];
                tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
                if (BIAS) {
#pragma unroll
                    for (int j = 0; j < 32; j++) v[j] += bb;
                }
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    const int arow = a0 + c0 + j;
                    if (mode == 2) {
                        const float u = __shfl_down_sync(0xffffffffu, v[j], 1);
                        if (arow < n && (lane & 1) == 0 && wrow + 1 < N)
                            Y[(size_t)arow * (N / 2) + wrow / 2] = silu_mul(v[j], u);
                    } else if (arow < n && wrow < N) {
                        float *dst = Y + (size_t)arow * N + wrow;
                        if (mode == 3) atomicAdd(dst, v[j]);  // split-K partial (compiles to a reduction)
                        else *dst = mode == 1 ? *dst + v[j] : v[j];
                    }
                }
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
    }
}

// SwiGLU of interleaved (gate, up) f32 pairs [n, 2I] -> bf16 hi/lo [n, I]
// (qwen_swiglu_multiply, qwen_asr_kernels.c:895-959, then the GEMM split).
__global__ void swiglu_split_kernel(const float *__restrict__ gu, uint16_t *__restrict__ hi, uint16_t *__restrict__ lo,
                                    size_t count) {
    pdl_enter();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const float2 p = reinterpret_cast<const float2 *>(gu)[i];
    const float v = silu_mul(p.x, p.y);
    const uint16_t h = f32_to_bf16_rn(v);
    hi[i] = h;
    lo[i] = f32_to_bf16_rn(v - __uint_as_float((uint32_t)h << 16));
}

// f32 [n, K] -> bf16 hi [n, K] + bf16 lo [n, K] with hi + lo ~= x
__global__ void split_bf16_kernel(const float *__restrict__ x, uint16_t *__restrict__ hi, uint16_t *__restrict__ lo,
                                  size_t count) {
    pdl_enter();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const float v = x[i];
    const uint16_t h = f32_to_bf16_rn(v);
    hi[i] = h;
    lo[i] = f32_to_bf16_rn(v - __uint_as_float((uint32_t)h << 16));
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

// 2D bf16 [rows, cols] row-major, box [box_rows, 64 cols], 128-byte swizzle.
bool make_map(CUtensorMap *m, const void *base, int rows, int cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Accumulator tile -> Y: warp q of the epilogue reads TMEM lanes [32q, 32q+32)
// (weight rows m0 + 32q + lane), columns [col0, col0 + BN) (activation rows a0..).
template <int BN, bool BIAS>
__device__ __forceinline__ void epilogue_tile(uint32_t tcol, int q, int lane, int m0, int a0, float *__restrict__ Y,
                                              int n, int N, int mode, const float *__restrict__ bias,
                                              uint16_t *__restrict__ ylo) {
    const int wrow = m0 + 32 * q + lane;
    float bb = 0.f;
    if (BIAS) bb = wrow < N ? bias[wrow] : 0.f;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_ld32(tcol + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
        if (BIAS) {
#pragma unroll
            for (int j = 0; j < 32; j++) v[j] += bb;
        }
        if (mode == 1) {  // residual add: all 32 loads in flight before the stores
            float y[32];
#pragma unroll
            for (int j = 0; j < 32; j++) {
                const int arow = a0 + c0 + j;
                y[j] = (arow < n && wrow < N) ? Y[(size_t)arow * N + wrow] : 0.f;
            }
#pragma unroll
            for (int j = 0; j < 32; j++) {
                const int arow = a0 + c0 + j;
                if (arow < n && wrow < N) Y[(size_t)arow * N + wrow] = y[j] + v[j];
            }
            continue;
        }
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const int arow = a0 + c0 + j;
            if (mode == 2 || mode == 4) {
                const float u = __shfl_down_sync(0xffffffffu, v[j], 1);
                if (arow < n && (lane & 1) == 0 && wrow + 1 < N) {
                    const size_t at = (size_t)arow * (N / 2) + wrow / 2;
                    const float g = silu_mul(v[j], u);
                    if (mode == 2) {
                        Y[at] = g;
                    } else {  // the bf16 split the down GEMM reads: hi into Y (as bf16), lo into ylo
                        const uint16_t hb = f32_to_bf16_rn(g);
                        reinterpret_cast<uint16_t *>(Y)[at] = hb;
                        ylo[at] = f32_to_bf16_rn(g - __uint_as_float((uint32_t)hb << 16));
                    }
                }
            } else if (arow < n && wrow < N) {
                float *dst = Y + (size_t)arow * N + wrow;
                if (mode == 3) atomicAdd(dst, v[j]);
                else *dst = mode == 1 ? *dst + v[j] : v[j];
            }
        }
    }
}

// Persistent form for the prefill shapes (no split-K): one CTA per SM walks
// the output tiles (tile t -> weight tile t / ny, activation tile t % ny, so
// the CTAs of a wave share weight tiles in L2). The TMA ring runs on across
// tiles, and the accumulator is double-buffered in TMEM (2 x BN columns):
// the MMA warp fills one buffer while the epilogue warps drain the other.
template <int BN, int S, bool BIAS, int MODE>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_persist_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmXh,
                           const __grid_constant__ CUtensorMap tmXl, float *__restrict__ Y, int n, int N, int K,
                           int mode, int *err, const float *__restrict__ bias, uint16_t *__restrict__ ylo) {
    if (MODE >= 0) mode = MODE;  // fixed-mode instantiations compile one store path
    constexpr int A_BYTES = TC_BM * TC_BK * 2;
    constexpr int B_BYTES = BN * TC_BK * 2;
    constexpr int STAGE = A_BYTES + 2 * B_BYTES;
    extern __shared__ __align__(1024) unsigned char smem_dyn[];
    __shared__ __align__(8) u64 full[S], empty[S], acc_full[2], acc_empty[2];
    __shared__ uint32_t tmem_slot;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nx = (N + TC_BM - 1) / TC_BM, ny = (n + BN - 1) / BN, ntile = nx * ny;
    const int nk = K / TC_BK;
    unsigned char *smem = smem_dyn + ((1024u - (su32(smem_dyn) & 1023u)) & 1023u);
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            mb_init(&full[i], 1);
            mb_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mb_init(&acc_full[i], 1);
            mb_init(&acc_empty[i], 4);  // one arrival per epilogue warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_slot)),
                     "r"(2 * BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---- TMA producer: every k-block of every tile of this CTA, one ring
        asm volatile("griddepcontrol.wait;" ::: "memory");
        unsigned it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntile && ok; tile += gridDim.x) {
            const int m0 = (tile / ny) * TC_BM, a0 = (tile % ny) * BN;
            for (int kb = 0; kb < nk; kb++, it++) {
                const int s = it % S;
                if (it >= (unsigned)S && !mb_wait(&empty[s], ((it / S) - 1) & 1, err)) {
                    ok = false;
                    break;
                }
                unsigned char *st = smem + (size_t)s * STAGE;
                mb_expect(&full[s], STAGE);
                const int kx = kb * TC_BK;
                tma_load_2d(st, &tmW, kx, m0, &full[s]);
                tma_load_2d(st + A_BYTES, &tmXh, kx, a0, &full[s]);
                tma_load_2d(st + A_BYTES + B_BYTES, &tmXl, kx, a0, &full[s]);
            }
        }
        // the copies of the last round of every stage land before leaving
        for (unsigned i = it > (unsigned)S ? it - S : 0; i < it; i++) mb_wait(&full[i % S], (i / S) & 1, err, true);
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        constexpr uint32_t idesc = instr_desc(TC_BM, BN);
        unsigned it = 0, tl = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntile && ok; tile += gridDim.x, tl++) {
            const int b = tl & 1;
            // the epilogue has drained this accumulator buffer (its previous use)
            if (tl >= 2 && !mb_wait(&acc_empty[b], ((tl >> 1) - 1) & 1, err)) break;
            tc_fence_after();
            const uint32_t acc = tmem + (uint32_t)(b * BN);
            for (int kb = 0; kb < nk; kb++, it++) {
                const int s = it % S;
                if (!mb_wait(&full[s], (it / S) & 1, err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t base = su32(smem + (size_t)s * STAGE);
#pragma unroll
                for (int k = 0; k < TC_BK / 16; k++) {
                    const u64 ad = sm_desc(base + k * 32);
                    mma_bf16(acc, ad, sm_desc(base + A_BYTES + k * 32), idesc, (kb | k) ? 1u : 0u);
                    mma_bf16(acc, ad, sm_desc(base + A_BYTES + B_BYTES + k * 32), idesc, 1u);
                }
                mma_commit(&empty[s]);
            }
            mma_commit(&acc_full[b]);
        }
    } else if (warp >= 2) {
        // ---- epilogue (warp q = warp & 3 owns TMEM lanes [32q, 32q+32))
        const int q = warp & 3;
        asm volatile("griddepcontrol.wait;" ::: "memory");
        unsigned tl = 0;
        for (int tile = blockIdx.x; tile < ntile; tile += gridDim.x, tl++) {
            const int b = tl & 1;
            bool ok = true;
            if (lane == 0) ok = mb_wait(&acc_full[b], (tl >> 1) & 1, err, true);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            tc_fence_after();
            epilogue_tile<BN, BIAS>(tmem + (uint32_t)(b * BN), q, lane, (tile / ny) * TC_BM, (tile % ny) * BN, Y, n, N, mode,
                              bias, ylo);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&acc_empty[b])) : "memory");
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN) : "memory");
    }
}

template <int BN, int S, bool BIAS, int MODE = -1>
cudaError_t launch_tc(const uint16_t *W, const uint16_t *Xh, const uint16_t *Xl, float *Y, int n, int N, int K,
                      int mode, int splits, int *err, cudaStream_t st, const float *bias) {
    CUtensorMap mw, mh, ml;
    if (!make_map(&mw, W, N, K, TC_BM) || !make_map(&mh, Xh, n, K, BN) || !make_map(&ml, Xl, n, K, BN))
        return cudaErrorInvalidValue;
    constexpr int STAGE = TC_BM * TC_BK * 2 + 2 * BN * TC_BK * 2;
    const int smem = S * STAGE + 1024;  // + slack to round the base up to 1024 B
    cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<BN, S, BIAS, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((N + TC_BM - 1) / TC_BM, (n + BN - 1) / BN);
    const int nk = K / TC_BK;
    const int kb_per = (nk + splits - 1) / splits;
    grid.z = (nk + kb_per - 1) / kb_per;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = QDB_GEMM_PDL;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BN, S, BIAS, MODE>, mw, mh, ml, Y, n, N, K, mode, kb_per, err, bias);
}


#ifndef QDB_GEMM_PERSIST
#define QDB_GEMM_PERSIST 1  // prefill shapes: persistent CTAs with a double-buffered TMEM accumulator
#endif
template <int BN, int S, bool BIAS, int MODE = -1>
cudaError_t launch_persist(const uint16_t *W, const uint16_t *Xh, const uint16_t *Xl, float *Y, int n, int N, int K,
                           int mode, int *err, cudaStream_t st, const float *bias, uint16_t *ylo = nullptr) {
    CUtensorMap mw, mh, ml;
    if (!make_map(&mw, W, N, K, TC_BM) || !make_map(&mh, Xh, n, K, BN) || !make_map(&ml, Xl, n, K, BN))
        return cudaErrorInvalidValue;
    constexpr int STAGE = TC_BM * TC_BK * 2 + 2 * BN * TC_BK * 2;
    const int smem = S * STAGE + 1024;
    cudaError_t e =
        cudaFuncSetAttribute(tc_gemm_persist_kernel<BN, S, BIAS, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return cudaErrorInvalidValue;
    const int tiles = ((N + TC_BM - 1) / TC_BM) * ((n + BN - 1) / BN);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles < sms ? tiles : sms);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = QDB_GEMM_PDL;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tc_gemm_persist_kernel<BN, S, BIAS, MODE>, mw, mh, ml, Y, n, N, K, mode, err, bias, ylo);
}

}  // namespace

QDB_WAIT_LIMIT_SETTER(qdb_set_wait_limit_tcgemm)

// Tensor map of a bf16 weight matrix [rows, cols] for 128-row x 64-column
// tiles with 128-byte swizzle (the batched decode step's weight stream).
extern "C" int qdb_make_weight_map(void *map, const uint16_t *base, int rows, int cols) {
    return make_map(reinterpret_cast<CUtensorMap *>(map), base, rows, cols, TC_BM) ? 0 : -1;
}

extern "C" cudaError_t qdb_launch_split_bf16(const float *x, uint16_t *hi, uint16_t *lo, size_t count,
                                             cudaStream_t st) {
    if (!count) return cudaSuccess;
    return pdl_launch(split_bf16_kernel, dim3((unsigned)((count + 255) / 256)), dim3(256), 0, st, x, hi, lo, count);
}

extern "C" cudaError_t qdb_launch_swiglu_split(const float *gu, uint16_t *hi, uint16_t *lo, size_t count,
                                               cudaStream_t st) {
    if (!count) return cudaSuccess;
    return pdl_launch(swiglu_split_kernel, dim3((unsigned)((count + 255) / 256)), dim3(256), 0, st, gu, hi, lo, count);
}

// Y (op)= X W^T on tensor cores; X given as its bf16 split (Xh, Xl) [n, K].
// mode: 0 store [n, N], 1 add into Y [n, N], 2 SwiGLU of row pairs -> Y [n, N/2],
// 3 add with atomics (split-K allowed; Y must hold the starting value).
// splits > 1 (mode 3 only) divides K across CTAs so that skinny problems
// (few weight-row tiles) still spread the weight stream over the whole GPU.
// K % 64 == 0; all base pointers 16-byte aligned; N even for mode 2.
#ifndef QDB_PF_BN
#define QDB_PF_BN 128     // activation rows per tile of the persistent (prefill) GEMM
#endif
#ifndef QDB_PF_STAGES
#define QDB_PF_STAGES 4   // its ring stages
#endif
#ifndef QDB_PF_FIXED_MODE
#define QDB_PF_FIXED_MODE 1  // prefill GEMMs as fixed-mode instantiations
#endif
#ifndef QDB_DEC_FIXED_MODE
#define QDB_DEC_FIXED_MODE 1  // decode GEMMs as fixed-mode instantiations
#endif
#ifndef QDB_DEC_STAGES
#define QDB_DEC_STAGES 3  // ring stages of the <= 64-row (decode) GEMM: 97 KB, 2 CTAs per SM
#endif
// bias (optional, f32 [N]) is added to every output (once per element, also
// under split-K).
extern "C" cudaError_t qdb_launch_gemm_tc_bias(const uint16_t *W, const uint16_t *Xh, const uint16_t *Xl, float *Y,
                                               int n, int N, int K, int mode, int splits, int *err, cudaStream_t st,
                                               const float *bias) {
    if (n <= 0) return cudaSuccess;
    if (K % TC_BK || (mode == 2 && (N & 1)) || mode < 0 || mode > 3) return cudaErrorInvalidValue;
    if (splits < 1 || (splits > 1 && mode != 3)) return cudaErrorInvalidValue;
    if (((uintptr_t)W | (uintptr_t)Xh | (uintptr_t)Xl) & 15) return cudaErrorInvalidValue;
    if (bias) {
        if (n <= 64) return launch_tc<64, 6, true>(W, Xh, Xl, Y, n, N, K, mode, splits, err, st, bias);
        if (QDB_GEMM_PERSIST && splits == 1)
            return launch_persist<128, 4, true>(W, Xh, Xl, Y, n, N, K, mode, err, st, bias);
        return launch_tc<128, 4, true>(W, Xh, Xl, Y, n, N, K, mode, splits, err, st, bias);
    }
    if (n <= 64) {
        if (QDB_DEC_FIXED_MODE) {
            switch (mode) {
                case 0: return launch_tc<64, QDB_DEC_STAGES, false, 0>(W, Xh, Xl, Y, n, N, K, 0, splits, err, st, nullptr);
                case 1: return launch_tc<64, QDB_DEC_STAGES, false, 1>(W, Xh, Xl, Y, n, N, K, 1, splits, err, st, nullptr);
                case 3: return launch_tc<64, QDB_DEC_STAGES, false, 3>(W, Xh, Xl, Y, n, N, K, 3, splits, err, st, nullptr);
                default: break;
            }
        }
        return launch_tc<64, QDB_DEC_STAGES, false>(W, Xh, Xl, Y, n, N, K, mode, splits, err, st, nullptr);
    }
    if (QDB_GEMM_PERSIST && splits == 1) {
        // fixed modes only at prefill row counts: the decode-size logits GEMM
        // (n <= 64, mode 0) measured ~0.3% slower on its fixed-mode build
        if (QDB_PF_FIXED_MODE && n > 64 && mode == 0)
            return launch_persist<QDB_PF_BN, QDB_PF_STAGES, false, 0>(W, Xh, Xl, Y, n, N, K, 0, err, st, nullptr);
        if (QDB_PF_FIXED_MODE && n > 64 && mode == 1)
            return launch_persist<QDB_PF_BN, QDB_PF_STAGES, false, 1>(W, Xh, Xl, Y, n, N, K, 1, err, st, nullptr);
        return launch_persist<QDB_PF_BN, QDB_PF_STAGES, false>(W, Xh, Xl, Y, n, N, K, mode, err, st, nullptr);
    }
    return launch_tc<128, 4, false>(W, Xh, Xl, Y, n, N, K, mode, splits, err, st, nullptr);
}

// Prefill gate/up with the SwiGLU and the bf16 split fused into the epilogue:
// interleaved (gate, up) rows of W -> yhi / ylo [n, N/2] bf16 (hi + lo = the
// SwiGLU value), the input of the down GEMM. n > 64 (persistent kernel), N even.
extern "C" cudaError_t qdb_launch_gemm_tc_swiglu_split(const uint16_t *W, const uint16_t *Xh, const uint16_t *Xl,
                                                       uint16_t *yhi, uint16_t *ylo, int n, int N, int K, int *err,
                                                       cudaStream_t st) {
    if (n <= 64 || (N & 1) || K % TC_BK || !yhi || !ylo) return cudaErrorInvalidValue;
    if (((uintptr_t)W | (uintptr_t)Xh | (uintptr_t)Xl) & 15) return cudaErrorInvalidValue;
    if (QDB_PF_FIXED_MODE)
        return launch_persist<QDB_PF_BN, QDB_PF_STAGES, false, 4>(W, Xh, Xl, reinterpret_cast<float *>(yhi), n, N, K, 4,
                                                                 err, st, nullptr, ylo);
    return launch_persist<QDB_PF_BN, QDB_PF_STAGES, false>(W, Xh, Xl, reinterpret_cast<float *>(yhi), n, N, K, 4, err,
                                                          st, nullptr, ylo);
}

extern "C" cudaError_t qdb_launch_gemm_tc(const uint16_t *W, const uint16_t *Xh, const uint16_t *Xl, float *Y, int n,
                                          int N, int K, int mode, int splits, int *err, cudaStream_t st) {
    return qdb_launch_gemm_tc_bias(W, Xh, Xl, Y, n, N, K, mode, splits, err, st, nullptr);
}

#ifndef QDB_SPLIT_WAVES
#define QDB_SPLIT_WAVES 2    // CTAs targeted per SM by split-K (two fit: 3-stage ring)
#endif
#ifndef QDB_SPLIT_MIN_KB
#define QDB_SPLIT_MIN_KB 1   // fewest 64-wide k-blocks one split-K CTA takes
#endif
// Split count for a skinny GEMM: about QDB_SPLIT_WAVES CTAs per SM, each
// with at least QDB_SPLIT_MIN_KB k-blocks (short CTAs are all set-up).
extern "C" int qdb_gemm_tc_splits(int n, int N, int K, int sms) {
    const int tiles = ((N + TC_BM - 1) / TC_BM) * ((n + (n <= 64 ? 63 : 127)) / (n <= 64 ? 64 : 128));
    const int nk = K / TC_BK;
    int s = (QDB_SPLIT_WAVES * sms + tiles - 1) / tiles;
    const int smax = nk / QDB_SPLIT_MIN_KB;
    if (s > smax) s = smax;
    return s < 1 ? 1 : s;
}
