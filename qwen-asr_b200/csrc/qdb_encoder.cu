// qdb_encoder.cu - the audio encoder on the GPU, replacing qwen_encoder_forward
// (qwen_asr_encoder.c:171-372; loader :66-168): log-mel [128, frames] ->
// audio embeddings [tokens, output_dim] that the decoder prefill consumes.
//
// Reference computation (all f32 on the host there):
//   per 100-frame chunk: 3 x (Conv2D 3x3 stride 2 pad 1 + bias, GELU), 480
//   channels; [480, 16, w3] -> [w3, 7680] (column ch * 16 + f); conv_out
//   projection (no bias); + sinusoidal positions restarting at 0 per chunk;
//   L x [LayerNorm -> Q/K/V (+bias) -> bidirectional attention inside windows
//   of 104 tokens -> out_proj (+bias) + residual -> LayerNorm -> fc1 (+bias)
//   -> GELU -> fc2 (+bias) + residual]; LayerNorm; proj1 (+bias) -> GELU ->
//   proj2 (+bias).
//
// B200 layout and kernels:
//   - Every projection and both 480-channel convolutions run on the tcgen05
//     GEMM (qdb_tcgemm.cu) with bf16 weights and f32 activations split into
//     bf16 hi + lo (~16 mantissa bits kept), bias in the GEMM epilogue,
//     residual adds as accumulate-into-output.
//   - Convolutions as im2col GEMMs over channel-last activations: conv output
//     row = (chunk, h, w) position, 480 channels contiguous; the im2col row of
//     an output position is 9 contiguous 480-channel vectors (K order
//     ki, kj, channel; weights re-ordered to match at upload, K padded to
//     4352), GELU of the previous layer applied while gathering. The stem runs
//     over groups of chunks to bound the im2col scratch.
//   - conv1 (1 input channel, K = 9) runs on CUDA cores straight from the mel.
//   - LayerNorm fused with the bf16 split of its output; GELU fused with the
//     split of fc1 / proj1 outputs; the [480,16,w3] -> [w3,7680] reshape fused
//     with GELU and the split (shared-memory transpose).
//   - Windowed attention: one CTA per (window, head), K/V of the window in
//     shared memory, one warp per query row, output written as the bf16 split
//     of the out_proj input.
// Conv kernels that are not exactly bf16 get a second (lo) weight pass.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "../../include/qwen_asr_b200.h"
#include "qdb_common.cuh"
#include "qdb_kernels.h"

namespace {

constexpr int NMEL = 128, CH = 480, CHUNK = 100, WIN_TOK = 13 * (800 / CHUNK);  // 104 tokens per window
constexpr int KC = 9 * CH, KCP = 4352;                                             // conv K, padded to 64
constexpr int KP = CH * 16;                                                        // 7680
constexpr int GROUP = 32;                                                          // chunks per stem group

struct EncChunk {
    const float *mel;       // the chunk's utterance: mel [128, frames]
    int frames;             // its mel row stride
    int f0, w, w1, w2, w3;  // first mel frame, widths after each convolution
    int p1, p2, p3, t0;     // row offsets (within the group) of conv1/2/3 outputs, first token
};

__device__ __forceinline__ float gelu_f(float v) {
    // tanh form of qwen_gelu (qwen_asr_kernels.c:886-893)
    const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
    return 0.5f * v * (1.0f + tanhf(inner));
}

__device__ __forceinline__ void split_store(uint16_t *hi, uint16_t *lo, size_t i, float v) {
    const uint16_t h = f32_to_bf16_rn(v);
    hi[i] = h;
    lo[i] = f32_to_bf16_rn(v - __uint_as_float((uint32_t)h << 16));
}

// conv1: mel [128, frames] -> Y1 [(chunk, oh, ow), 480] pre-GELU (+bias).
// One CTA per (oh, chunk).
__global__ void __launch_bounds__(256) conv1_kernel(const EncChunk *__restrict__ ch, const float *__restrict__ w,
                                                    const float *__restrict__ b, float *__restrict__ Y1) {
    __shared__ float rows[3][CHUNK + 2];
    __shared__ float ws[CH * 9];
    const EncChunk c = ch[blockIdx.y];
    const int oh = blockIdx.x;  // 0..63
    for (int i = threadIdx.x; i < CH * 9; i += blockDim.x) ws[i] = w[i];
    for (int i = threadIdx.x; i < 3 * (CHUNK + 2); i += blockDim.x) {
        const int r = i / (CHUNK + 2), t = i % (CHUNK + 2) - 1;  // t in [-1, CHUNK]
        const int fr = 2 * oh - 1 + r;
        rows[r][t + 1] = (fr >= 0 && fr < NMEL && t >= 0 && t < c.w) ? c.mel[(size_t)fr * c.frames + c.f0 + t] : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < c.w1 * CH; i += blockDim.x) {
        const int ow = i / CH, oc = i % CH;
        const float *k = ws + oc * 9;
        float acc = b[oc];
#pragma unroll
        for (int ki = 0; ki < 3; ki++)
#pragma unroll
            for (int kj = 0; kj < 3; kj++) acc = fmaf(k[ki * 3 + kj], rows[ki][2 * ow + kj], acc);
        Y1[(size_t)(c.p1 + oh * c.w1 + ow) * CH + oc] = acc;
    }
}

// im2col of a stride-2 3x3 convolution over channel-last GELU(Y): X row of
// output (chunk, oh, ow) = [GELU(Y[(chunk, 2oh-1+ki, 2ow-1+kj), :]) for ki, kj]
// (zero outside), bf16 hi/lo, K padded to KCP. stage 2: Y1 -> X2, stage 3: Y2 -> X3.
__global__ void __launch_bounds__(256) im2col_gelu_kernel(const float *__restrict__ Y, const EncChunk *__restrict__ ch,
                                                          int stage, uint16_t *__restrict__ hi,
                                                          uint16_t *__restrict__ lo) {
    const EncChunk c = ch[blockIdx.y];
    const int h_in = stage == 2 ? 64 : 32, h_out = h_in / 2;
    const int w_in = stage == 2 ? c.w1 : c.w2, w_out = stage == 2 ? c.w2 : c.w3;
    const int pin = stage == 2 ? c.p1 : c.p2, pout = stage == 2 ? c.p2 : c.p3;
    const int pos = blockIdx.x;
    if (pos >= h_out * w_out) return;
    const int oh = pos / w_out, ow = pos % w_out;
    const size_t orow = (size_t)(pout + pos) * KCP;
    for (int k = threadIdx.x; k < KCP; k += blockDim.x) {
        float v = 0.f;
        if (k < KC) {
            const int kk = k / CH, ic = k % CH;
            const int ih = 2 * oh - 1 + kk / 3, iw = 2 * ow - 1 + kk % 3;
            if (ih >= 0 && ih < h_in && iw >= 0 && iw < w_in) v = gelu_f(Y[(size_t)(pin + ih * w_in + iw) * CH + ic]);
        }
        split_store(hi, lo, orow + k, v);
    }
}

// GELU of conv3's output Y3 [(chunk, f, t), 480] reshaped to the projection
// input [token, ch * 16 + f] (qwen_asr_encoder.c:262-271), bf16 hi/lo.
// One CTA per (t, chunk); the 16 x 480 block goes through shared memory.
__global__ void __launch_bounds__(256) stem_gather_kernel(const float *__restrict__ Y3, const EncChunk *__restrict__ ch,
                                                          int tok_base, uint16_t *__restrict__ hi,
                                                          uint16_t *__restrict__ lo) {
    __shared__ float blk[16][CH + 1];
    const EncChunk c = ch[blockIdx.y];
    const int t = blockIdx.x;
    if (t >= c.w3) return;
    for (int i = threadIdx.x; i < 16 * CH; i += blockDim.x) {
        const int f = i / CH, cc = i % CH;
        blk[f][cc] = gelu_f(Y3[(size_t)(c.p3 + f * c.w3 + t) * CH + cc]);
    }
    __syncthreads();
    const size_t orow = (size_t)(tok_base + c.t0 + t) * KP;
    for (int k = threadIdx.x; k < KP; k += blockDim.x) split_store(hi, lo, orow + k, blk[k % 16][k / 16]);
}

// x[token] = sinusoidal position of its index inside its chunk
// (qwen_sinusoidal_pe, qwen_asr_kernels.c:1147-1160); the conv_out GEMM then
// accumulates onto it.
__global__ void pe_fill_kernel(const EncChunk *__restrict__ ch, int tok_base, float *__restrict__ x, int d) {
    const EncChunk c = ch[blockIdx.y];
    const int t = blockIdx.x;
    if (t >= c.w3) return;
    const int half = d / 2;
    const float lt = logf(10000.0f) / (float)(half - 1);
    float *row = x + (size_t)(tok_base + c.t0 + t) * d;
    for (int j = threadIdx.x; j < half; j += blockDim.x) {
        const float inv = expf(-(float)j * lt);
        const float a = (float)t * inv;
        row[j] = sinf(a);
        row[half + j] = cosf(a);
    }
}

// LayerNorm (population variance, eps) of x rows -> bf16 hi/lo
// (qwen_layer_norm, qwen_asr_kernels.c:640-748). One CTA per row.
__global__ void __launch_bounds__(256) layernorm_split_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                              const float *__restrict__ b, int d, float eps,
                                                              uint16_t *__restrict__ hi, uint16_t *__restrict__ lo) {
    __shared__ float red[8];
    __shared__ float stat;
    const float *r = x + (size_t)blockIdx.x * d;
    const int t = threadIdx.x, wid = t >> 5, lane = t & 31;
    float s = 0.f;
    for (int i = t; i < d; i += blockDim.x) s += r[i];
    s = warp_sum(s);
    if (lane == 0) red[wid] = s;
    __syncthreads();
    if (t == 0) {
        float a = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) a += red[i];
        stat = a / (float)d;
    }
    __syncthreads();
    const float mean = stat;
    float v = 0.f;
    for (int i = t; i < d; i += blockDim.x) {
        const float q = r[i] - mean;
        v = fmaf(q, q, v);
    }
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    if (t == 0) {
        float a = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) a += red[i];
        stat = 1.0f / sqrtf(a / (float)d + eps);
    }
    __syncthreads();
    const float inv = stat;
    for (int i = t; i < d; i += blockDim.x) split_store(hi, lo, (size_t)blockIdx.x * d + i, (r[i] - mean) * inv * w[i] + b[i]);
}

__global__ void gelu_split_kernel(const float *__restrict__ y, size_t count, uint16_t *__restrict__ hi,
                                  uint16_t *__restrict__ lo) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) split_store(hi, lo, i, gelu_f(y[i]));
}

// Bidirectional attention inside windows of at most WIN_TOK tokens
// (qwen_bidirectional_attention, qwen_asr_kernels.c:1003-1048), head_dim 64;
// the windows restart at each utterance's first token.
// qkv [n, 3d] (q | k | v, each head h at columns h*64); output as the bf16
// split of [n, d]. One CTA per (window, head), one warp per query row.
constexpr int AW = 4;  // warps
__global__ void __launch_bounds__(AW * 32) win_attn_kernel(const float *__restrict__ qkv, const int2 *__restrict__ wins,
                                                           int d, float scale, uint16_t *__restrict__ hi,
                                                           uint16_t *__restrict__ lo) {
    extern __shared__ float sm[];
    float *K = sm;                        // [WIN_TOK][65]
    float *V = K + WIN_TOK * 65;          // [WIN_TOK][64]
    float *Q = V + WIN_TOK * 64;          // [AW][64]
    float *P = Q + AW * 64;               // [AW][WIN_TOK]
    const int2 win = wins[blockIdx.x];  // (first token, tokens) of this window
    const int w0 = win.x, L = win.y, h = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t rs = (size_t)3 * d;
    for (int i = threadIdx.x; i < L * 64; i += blockDim.x) {
        const int j = i >> 6, c = i & 63;
        const float *row = qkv + (size_t)(w0 + j) * rs + h * 64 + c;
        K[j * 65 + c] = row[d];
        V[j * 64 + c] = row[2 * d];
    }
    __syncthreads();
    float *q = Q + warp * 64, *p = P + warp * WIN_TOK;
    // query rows of this window split over gridDim.z CTAs (each loads the window's K/V)
    for (int i = blockIdx.z * AW + warp; i < L; i += AW * gridDim.z) {
        const float *qr = qkv + (size_t)(w0 + i) * rs + h * 64;
        q[lane] = qr[lane];
        q[lane + 32] = qr[lane + 32];
        __syncwarp();
        float s[(WIN_TOK + 31) / 32];
        float mx = -INFINITY;
#pragma unroll
        for (int u = 0; u < (WIN_TOK + 31) / 32; u++) {
            const int j = lane + 32 * u;
            float a = -INFINITY;
            if (j < L) {
                a = 0.f;
#pragma unroll 16
                for (int c = 0; c < 64; c++) a = fmaf(q[c], K[j * 65 + c], a);
                a *= scale;
            }
            s[u] = a;
            mx = fmaxf(mx, a);
        }
        mx = warp_max(mx);
        float sum = 0.f;
#pragma unroll
        for (int u = 0; u < (WIN_TOK + 31) / 32; u++) {
            const int j = lane + 32 * u;
            const float e = j < L ? expf(s[u] - mx) : 0.f;
            if (j < L) p[j] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        __syncwarp();
        float o0 = 0.f, o1 = 0.f;
        for (int j = 0; j < L; j++) {
            const float pj = p[j];
            o0 = fmaf(pj, V[j * 64 + lane], o0);
            o1 = fmaf(pj, V[j * 64 + lane + 32], o1);
        }
        const float inv = 1.0f / sum;
        const size_t o = (size_t)(w0 + i) * d + h * 64;
        split_store(hi, lo, o + lane, o0 * inv);
        split_store(hi, lo, o + lane + 32, o1 * inv);
        __syncwarp();
    }
}

struct EncLayer {
    uint16_t *wqkv = nullptr, *wo = nullptr, *fc1 = nullptr, *fc2 = nullptr;
    float *bqkv = nullptr, *bo = nullptr, *b1 = nullptr, *b2 = nullptr;
    float *ln1w = nullptr, *ln1b = nullptr, *ln2w = nullptr, *ln2b = nullptr;
};

}  // namespace

struct qdb_encoder {
    qdb_encoder_config cfg{};
    int device = 0, sms = 0;
    cudaStream_t st = nullptr;
    std::vector<void *> allocs;
    float *c1w = nullptr, *c1b = nullptr, *c2b = nullptr, *c3b = nullptr;
    uint16_t *c2w = nullptr, *c2lo = nullptr, *c3w = nullptr, *c3lo = nullptr, *cout = nullptr;
    std::vector<EncLayer> layers;
    float *lnpw = nullptr, *lnpb = nullptr, *p1b = nullptr, *p2b = nullptr;
    uint16_t *p1w = nullptr, *p2w = nullptr;
    bool stem_set = false, post_set = false, finalized = false;
    std::vector<char> layer_set;
    // scratch
    size_t cap_tok = 0;
    float *x = nullptr, *big = nullptr;  // x [tok, d]; big: qkv / fc1 / proj1 outputs [tok, max(3d, ffn)]
    uint16_t *xh = nullptr, *xl = nullptr;  // bf16 split [rows, K] of the current GEMM input
    size_t cap_split = 0;
    float *y1 = nullptr, *y2 = nullptr, *y3 = nullptr;  // stem group outputs
    EncChunk *d_chunks_all = nullptr;
    size_t cap_chunks = 0;
    int2 *d_wins = nullptr;
    size_t cap_wins = 0;
    int *err = nullptr;
    float *mel_dev = nullptr, *out_dev = nullptr;
    size_t cap_mel = 0, cap_out = 0;
};

namespace {

template <typename T>
int enc_alloc(qdb_encoder *e, T **p, size_t count) {
    *p = nullptr;
    if (cudaMalloc((void **)p, std::max<size_t>(count, 1) * sizeof(T)) != cudaSuccess) {
        *p = nullptr;
        return qdb_set_error("qdb_encoder: out of device memory");
    }
    e->allocs.push_back(*p);
    return 0;
}

template <typename T>
int upload(qdb_encoder *e, T **dst, const T *src, size_t count) {
    if (!src) return qdb_set_error("qdb_encoder: null weight");
    if (enc_alloc(e, dst, count)) return -1;
    return cudaMemcpy(*dst, src, count * sizeof(T), cudaMemcpyHostToDevice) == cudaSuccess
               ? 0
               : qdb_set_error("qdb_encoder: weight upload failed");
}

uint16_t bf16_rn_host(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // NaN stays NaN
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// f32 conv kernel [480, 480, 3, 3] -> bf16 [480, KCP] with K order
// (ki, kj, channel), zero padded; lo = bf16 of the residual (null when zero)
int upload_conv(qdb_encoder *e, const float *w, uint16_t **hi, uint16_t **lo) {
    if (!w) return qdb_set_error("qdb_encoder: null conv weight");
    std::vector<uint16_t> h((size_t)CH * KCP, 0), l((size_t)CH * KCP, 0);
    bool any_lo = false;
    for (int oc = 0; oc < CH; oc++)
        for (int ic = 0; ic < CH; ic++)
            for (int kk = 0; kk < 9; kk++) {
                const float v = w[((size_t)oc * CH + ic) * 9 + kk];
                const uint16_t b = bf16_rn_host(v);
                uint32_t bu = (uint32_t)b << 16;
                float bv;
                memcpy(&bv, &bu, 4);
                const uint16_t r = bf16_rn_host(v - bv);
                const size_t at = (size_t)oc * KCP + kk * CH + ic;
                h[at] = b;
                l[at] = r;
                any_lo |= (r & 0x7fffu) != 0;
            }
    if (upload(e, hi, h.data(), h.size())) return -1;
    *lo = nullptr;
    return any_lo ? upload(e, lo, l.data(), l.size()) : 0;
}

int grow_scratch(qdb_encoder *e, size_t tok) {
    const int d = e->cfg.d_model;
    const size_t bigw = std::max<size_t>(3 * (size_t)d, std::max<size_t>(e->cfg.ffn_dim, e->cfg.output_dim));
    if (tok > e->cap_tok) {
        cudaFree(e->x);
        cudaFree(e->big);
        e->x = e->big = nullptr;
        e->cap_tok = 0;
        if (cudaMalloc(&e->x, tok * d * sizeof(float)) != cudaSuccess ||
            cudaMalloc(&e->big, tok * bigw * sizeof(float)) != cudaSuccess)
            return qdb_set_error("qdb_encoder: out of device memory (activations)");
        e->cap_tok = tok;
    }
    // GEMM inputs: stem groups [GROUP * 800, KCP], projection [tok, 7680], layers [tok, max(d, ffn)]
    const size_t need = std::max({(size_t)GROUP * 800 * KCP, tok * KP, tok * (size_t)std::max(d, e->cfg.ffn_dim)});
    if (need > e->cap_split) {
        cudaFree(e->xh);
        cudaFree(e->xl);
        e->xh = e->xl = nullptr;
        e->cap_split = 0;
        if (cudaMalloc(&e->xh, need * 2) != cudaSuccess || cudaMalloc(&e->xl, need * 2) != cudaSuccess)
            return qdb_set_error("qdb_encoder: out of device memory (GEMM inputs)");
        e->cap_split = need;
    }
    return 0;
}

int gemm(qdb_encoder *e, const uint16_t *W, float *Y, int n, int N, int K, int mode, const float *bias) {
    // skinny problems (<= 64 rows): split-K with atomic accumulation
    int sp = n <= 64 ? qdb_gemm_tc_splits(n, N, K, e->sms) : 1;
    if (sp > 1) {
        if (mode == 0 && cudaMemsetAsync(Y, 0, sizeof(float) * (size_t)n * N, e->st) != cudaSuccess)
            return qdb_set_error("qdb_encoder: memset failed");
        mode = 3;
    }
    const cudaError_t r = qdb_launch_gemm_tc_bias(W, e->xh, e->xl, Y, n, N, K, mode, sp, e->err, e->st, bias);
    return r == cudaSuccess ? 0 : qdb_set_error(cudaGetErrorString(r));
}

}  // namespace

extern "C" int qdb_encoder_tokens(int mel_frames) {
    int n = 0;
    for (int c0 = 0; c0 < mel_frames; c0 += CHUNK) {
        int w = std::min(CHUNK, mel_frames - c0);
        for (int k = 0; k < 3; k++) w = (w - 1) / 2 + 1;
        n += w;
    }
    return n;
}

extern "C" qdb_encoder *qdb_encoder_create(const qdb_encoder_config *cfg, int device) {
    if (!cfg) {
        qdb_set_error("qdb_encoder_create: null config");
        return nullptr;
    }
    const qdb_encoder_config &c = *cfg;
    if (c.head_dim != 64 || c.heads * c.head_dim != c.d_model || c.d_model % 64 || c.ffn_dim % 64 ||
        c.output_dim <= 0 || c.layers <= 0 || c.d_model > 4096) {
        qdb_set_error("qdb_encoder_create: unsupported shape (head_dim 64, heads * 64 = d_model, d_model and "
                      "ffn_dim multiples of 64)");
        return nullptr;
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        qdb_set_error("qdb_encoder_create: cudaSetDevice failed");
        return nullptr;
    }
    qdb_encoder *e = new qdb_encoder();
    e->cfg = c;
    e->device = device;
    cudaDeviceGetAttribute(&e->sms, cudaDevAttrMultiProcessorCount, device);
    e->layers.resize(c.layers);
    e->layer_set.assign(c.layers, 0);
    if (cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking) != cudaSuccess ||
        enc_alloc(e, &e->err, 4) ||
        cudaMemset(e->err, 0, 16) != cudaSuccess) {
        qdb_encoder_free(e);
        return nullptr;
    }
    return e;
}

extern "C" void qdb_encoder_free(qdb_encoder *e) {
    if (!e) return;
    cudaSetDevice(e->device);
    if (e->st) cudaStreamSynchronize(e->st);
    for (void *p : e->allocs) cudaFree(p);
    for (void *p : {(void *)e->x, (void *)e->big, (void *)e->xh, (void *)e->xl, (void *)e->y1, (void *)e->y2,
                    (void *)e->y3, (void *)e->mel_dev, (void *)e->out_dev, (void *)e->d_chunks_all,
                    (void *)e->d_wins})
        cudaFree(p);
    if (e->st) cudaStreamDestroy(e->st);
    delete e;
}

extern "C" int qdb_encoder_set_stem(qdb_encoder *e, const float *conv1_w, const float *conv1_b, const float *conv2_w,
                                    const float *conv2_b, const float *conv3_w, const float *conv3_b,
                                    const uint16_t *conv_out_w) {
    if (!e) return qdb_set_error("qdb_encoder_set_stem: null encoder");
    if (cudaSetDevice(e->device) != cudaSuccess) return qdb_set_error("qdb_encoder: cudaSetDevice failed");
    if (upload(e, &e->c1w, conv1_w, CH * 9) || upload(e, &e->c1b, conv1_b, CH) ||
        upload_conv(e, conv2_w, &e->c2w, &e->c2lo) || upload(e, &e->c2b, conv2_b, CH) ||
        upload_conv(e, conv3_w, &e->c3w, &e->c3lo) || upload(e, &e->c3b, conv3_b, CH) ||
        upload(e, &e->cout, conv_out_w, (size_t)e->cfg.d_model * KP))
        return -1;
    e->stem_set = true;
    return 0;
}

extern "C" int qdb_encoder_set_layer(qdb_encoder *e, int i, const uint16_t *wq, const float *bq, const uint16_t *wk,
                                     const float *bk, const uint16_t *wv, const float *bv, const uint16_t *wo,
                                     const float *bo, const float *ln1_w, const float *ln1_b, const uint16_t *fc1_w,
                                     const float *fc1_b, const uint16_t *fc2_w, const float *fc2_b,
                                     const float *ln2_w, const float *ln2_b) {
    if (!e || i < 0 || i >= e->cfg.layers) return qdb_set_error("qdb_encoder_set_layer: bad encoder or layer index");
    if (cudaSetDevice(e->device) != cudaSuccess) return qdb_set_error("qdb_encoder: cudaSetDevice failed");
    const size_t d = e->cfg.d_model, f = e->cfg.ffn_dim;
    if (!wq || !wk || !wv || !bq || !bk || !bv) return qdb_set_error("qdb_encoder_set_layer: null weight");
    EncLayer &L = e->layers[i];
    // Q, K, V concatenated into one [3d, d] projection (one GEMM)
    std::vector<uint16_t> w3(3 * d * d);
    memcpy(w3.data(), wq, d * d * 2);
    memcpy(w3.data() + d * d, wk, d * d * 2);
    memcpy(w3.data() + 2 * d * d, wv, d * d * 2);
    std::vector<float> b3(3 * d);
    memcpy(b3.data(), bq, d * 4);
    memcpy(b3.data() + d, bk, d * 4);
    memcpy(b3.data() + 2 * d, bv, d * 4);
    if (upload(e, &L.wqkv, (const uint16_t *)w3.data(), w3.size()) || upload(e, &L.bqkv, (const float *)b3.data(), b3.size()) ||
        upload(e, &L.wo, wo, d * d) || upload(e, &L.bo, bo, d) || upload(e, &L.ln1w, ln1_w, d) ||
        upload(e, &L.ln1b, ln1_b, d) || upload(e, &L.fc1, fc1_w, f * d) || upload(e, &L.b1, fc1_b, f) ||
        upload(e, &L.fc2, fc2_w, d * f) || upload(e, &L.b2, fc2_b, d) || upload(e, &L.ln2w, ln2_w, d) ||
        upload(e, &L.ln2b, ln2_b, d))
        return -1;
    e->layer_set[i] = 1;
    return 0;
}

extern "C" int qdb_encoder_set_post(qdb_encoder *e, const float *ln_w, const float *ln_b, const uint16_t *proj1_w,
                                    const float *proj1_b, const uint16_t *proj2_w, const float *proj2_b) {
    if (!e) return qdb_set_error("qdb_encoder_set_post: null encoder");
    if (cudaSetDevice(e->device) != cudaSuccess) return qdb_set_error("qdb_encoder: cudaSetDevice failed");
    const size_t d = e->cfg.d_model, o = e->cfg.output_dim;
    if (upload(e, &e->lnpw, ln_w, d) || upload(e, &e->lnpb, ln_b, d) || upload(e, &e->p1w, proj1_w, d * d) ||
        upload(e, &e->p1b, proj1_b, d) || upload(e, &e->p2w, proj2_w, o * d) || upload(e, &e->p2b, proj2_b, o))
        return -1;
    e->post_set = true;
    return 0;
}

extern "C" int qdb_encoder_finalize(qdb_encoder *e) {
    if (!e) return qdb_set_error("qdb_encoder_finalize: null encoder");
    if (!e->stem_set || !e->post_set) return qdb_set_error("qdb_encoder_finalize: stem or post weights not set");
    for (int i = 0; i < e->cfg.layers; i++)
        if (!e->layer_set[i]) return qdb_set_error("qdb_encoder_finalize: a layer's weights are not set");
    if (cudaFuncSetAttribute(win_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (WIN_TOK * 129 + AW * (64 + WIN_TOK)) * 4) != cudaSuccess)
        return qdb_set_error("qdb_encoder_finalize: attention kernel attribute");
    e->finalized = true;
    return 0;
}

extern "C" void *qdb_encoder_stream(qdb_encoder *e) { return e ? (void *)e->st : nullptr; }

// n utterances: mel_dev[u] [128, frames[u]] (device) -> out_dev [sum of
// tokens, output_dim] (device), utterance u's rows after those of 0..u-1, on
// the encoder's stream. Every row-wise stage runs once over all utterances'
// tokens; attention windows restart at each utterance. Returns the token
// count, or -1.
extern "C" int qdb_encoder_forward_batch_device(qdb_encoder *e, int n_utt, const float *const *mel_dev,
                                                const int *frames, float *out_dev) {
    if (!e || !e->finalized) return qdb_set_error("qdb_encoder_forward: encoder not finalized");
    if (n_utt <= 0 || !mel_dev || !frames || !out_dev) return qdb_set_error("qdb_encoder_forward: no input");
    for (int u = 0; u < n_utt; u++)
        if (!mel_dev[u] || frames[u] <= 0) return qdb_set_error("qdb_encoder_forward: empty utterance");
    if (cudaSetDevice(e->device) != cudaSuccess) return qdb_set_error("qdb_encoder: cudaSetDevice failed");
    const int d = e->cfg.d_model;
    // chunks of every utterance, windows of every utterance
    std::vector<EncChunk> all;
    std::vector<int2> wins;
    int ntok = 0;
    for (int u = 0; u < n_utt; u++) {
        const int t_u = qdb_encoder_tokens(frames[u]);
        for (int f0 = 0; f0 < frames[u]; f0 += CHUNK) {
            EncChunk k{};
            k.mel = mel_dev[u];
            k.frames = frames[u];
            k.f0 = f0;
            k.w = std::min(CHUNK, frames[u] - f0);
            k.w1 = (k.w - 1) / 2 + 1;
            k.w2 = (k.w1 - 1) / 2 + 1;
            k.w3 = (k.w2 - 1) / 2 + 1;
            all.push_back(k);
        }
        for (int w0 = 0; w0 < t_u; w0 += WIN_TOK) wins.push_back(make_int2(ntok + w0, std::min(WIN_TOK, t_u - w0)));
        ntok += t_u;
    }
    if (grow_scratch(e, ntok)) return -1;
    if (!e->y1 && (cudaMalloc(&e->y1, (size_t)GROUP * 3200 * CH * 4) != cudaSuccess ||
                   cudaMalloc(&e->y2, (size_t)GROUP * 800 * CH * 4) != cudaSuccess ||
                   cudaMalloc(&e->y3, (size_t)GROUP * 208 * CH * 4) != cudaSuccess))
        return qdb_set_error("qdb_encoder: out of device memory (stem)");
    if (wins.size() > e->cap_wins) {
        cudaFree(e->d_wins);
        e->d_wins = nullptr;
        e->cap_wins = 0;
        if (cudaMalloc(&e->d_wins, wins.size() * sizeof(int2)) != cudaSuccess)
            return qdb_set_error("qdb_encoder: out of device memory (windows)");
        e->cap_wins = wins.size();
    }
    cudaStream_t st = e->st;
    if (cudaMemcpyAsync(e->d_wins, wins.data(), wins.size() * sizeof(int2), cudaMemcpyHostToDevice, st) != cudaSuccess)
        return qdb_set_error("qdb_encoder: window table upload failed");
    // ---- convolution stem, GROUP chunks at a time (any mix of utterances)
    const int nchunks = (int)all.size();
    if ((size_t)nchunks > e->cap_chunks) {
        cudaFree(e->d_chunks_all);
        e->d_chunks_all = nullptr;
        e->cap_chunks = 0;
        if (cudaMalloc(&e->d_chunks_all, sizeof(EncChunk) * nchunks) != cudaSuccess)
            return qdb_set_error("qdb_encoder: out of device memory (chunk table)");
        e->cap_chunks = nchunks;
    }
    int tok = 0;
    for (int g0 = 0; g0 < nchunks; g0 += GROUP) {
        const int ng = std::min(GROUP, nchunks - g0);
        int p1 = 0, p2 = 0, p3 = 0, t0 = 0;
        for (int c = g0; c < g0 + ng; c++) {
            EncChunk &k = all[c];
            k.p1 = p1;
            k.p2 = p2;
            k.p3 = p3;
            k.t0 = t0;
            p1 += 64 * k.w1;
            p2 += 32 * k.w2;
            p3 += 16 * k.w3;
            t0 += k.w3;
        }
        EncChunk *tab = e->d_chunks_all + g0;
        if (cudaMemcpyAsync(tab, all.data() + g0, sizeof(EncChunk) * ng, cudaMemcpyHostToDevice, st) != cudaSuccess)
            return qdb_set_error("qdb_encoder: chunk table upload failed");
        conv1_kernel<<<dim3(64, ng), 256, 0, st>>>(tab, e->c1w, e->c1b, e->y1);
        im2col_gelu_kernel<<<dim3(32 * 25, ng), 256, 0, st>>>(e->y1, tab, 2, e->xh, e->xl);
        if (gemm(e, e->c2w, e->y2, p2, CH, KCP, 0, e->c2b) || (e->c2lo && gemm(e, e->c2lo, e->y2, p2, CH, KCP, 1, nullptr)))
            return -1;
        im2col_gelu_kernel<<<dim3(16 * 13, ng), 256, 0, st>>>(e->y2, tab, 3, e->xh, e->xl);
        if (gemm(e, e->c3w, e->y3, p3, CH, KCP, 0, e->c3b) || (e->c3lo && gemm(e, e->c3lo, e->y3, p3, CH, KCP, 1, nullptr)))
            return -1;
        // this group's projection input rows, then its projection (the stem
        // scratch is reused by the next group)
        stem_gather_kernel<<<dim3(13, ng), 256, 0, st>>>(e->y3, tab, 0, e->xh, e->xl);
        pe_fill_kernel<<<dim3(13, ng), 256, 0, st>>>(tab, tok, e->x, d);
        if (gemm(e, e->cout, e->x + (size_t)tok * d, t0, d, KP, 1, nullptr)) return -1;
        tok += t0;
    }
    // ---- transformer layers over all tokens
    const int n = ntok, nwin = (int)wins.size();
    const size_t asmem = (size_t)(WIN_TOK * 129 + AW * (64 + WIN_TOK)) * 4;
    // few windows (one short utterance) leave most SMs idle: split the
    // windows' query rows over more CTAs until there are ~2 per SM
    int qsplit = 1;
    while (qsplit < 8 && nwin * e->cfg.heads * qsplit < 2 * e->sms) qsplit *= 2;
    for (int l = 0; l < e->cfg.layers; l++) {
        const EncLayer &L = e->layers[l];
        layernorm_split_kernel<<<n, 256, 0, st>>>(e->x, L.ln1w, L.ln1b, d, 1e-5f, e->xh, e->xl);
        if (gemm(e, L.wqkv, e->big, n, 3 * d, d, 0, L.bqkv)) return -1;
        win_attn_kernel<<<dim3(nwin, e->cfg.heads, qsplit), AW * 32, asmem, st>>>(e->big, e->d_wins, d,
                                                                         1.0f / sqrtf((float)e->cfg.head_dim), e->xh,
                                                                         e->xl);
        if (gemm(e, L.wo, e->x, n, d, d, 1, L.bo)) return -1;
        layernorm_split_kernel<<<n, 256, 0, st>>>(e->x, L.ln2w, L.ln2b, d, 1e-5f, e->xh, e->xl);
        if (gemm(e, L.fc1, e->big, n, e->cfg.ffn_dim, d, 0, L.b1)) return -1;
        const size_t cnt = (size_t)n * e->cfg.ffn_dim;
        gelu_split_kernel<<<(unsigned)((cnt + 255) / 256), 256, 0, st>>>(e->big, cnt, e->xh, e->xl);
        if (gemm(e, L.fc2, e->x, n, d, e->cfg.ffn_dim, 1, L.b2)) return -1;
    }
    layernorm_split_kernel<<<n, 256, 0, st>>>(e->x, e->lnpw, e->lnpb, d, 1e-5f, e->xh, e->xl);
    if (gemm(e, e->p1w, e->big, n, d, d, 0, e->p1b)) return -1;
    const size_t cnt = (size_t)n * d;
    gelu_split_kernel<<<(unsigned)((cnt + 255) / 256), 256, 0, st>>>(e->big, cnt, e->xh, e->xl);
    if (gemm(e, e->p2w, out_dev, n, e->cfg.output_dim, d, 0, e->p2b)) return -1;
    const cudaError_t le = cudaGetLastError();
    if (le != cudaSuccess) return qdb_set_error(cudaGetErrorString(le));
    return n;
}

// One utterance: mel_dev [128, frames] (device) -> out_dev [tokens,
// output_dim] (device), on the encoder's stream. Returns the token count, or -1.
extern "C" int qdb_encoder_forward_device(qdb_encoder *e, const float *mel_dev, int frames, float *out_dev) {
    return qdb_encoder_forward_batch_device(e, 1, &mel_dev, &frames, out_dev);
}

// Drop-in for qwen_encoder_forward (qwen_asr_encoder.c:171): host mel
// [128, frames] -> malloc'd host [tokens, output_dim] (caller frees), NULL on
// error. Synchronous.
extern "C" float *qdb_encoder_forward(qdb_encoder *e, const float *mel, int frames, int *out_seq_len) {
    if (!e || !mel || frames <= 0 || !out_seq_len) {
        qdb_set_error("qdb_encoder_forward: bad arguments");
        return nullptr;
    }
    if (cudaSetDevice(e->device) != cudaSuccess) {
        qdb_set_error("qdb_encoder: cudaSetDevice failed");
        return nullptr;
    }
    const int ntok = qdb_encoder_tokens(frames);
    const size_t mel_n = (size_t)NMEL * frames, out_n = (size_t)ntok * e->cfg.output_dim;
    if (mel_n > e->cap_mel) {
        cudaFree(e->mel_dev);
        e->mel_dev = nullptr;
        e->cap_mel = 0;
        if (cudaMalloc(&e->mel_dev, mel_n * 4) != cudaSuccess) {
            qdb_set_error("qdb_encoder: out of device memory");
            return nullptr;
        }
        e->cap_mel = mel_n;
    }
    if (out_n > e->cap_out) {
        cudaFree(e->out_dev);
        e->out_dev = nullptr;
        e->cap_out = 0;
        if (cudaMalloc(&e->out_dev, out_n * 4) != cudaSuccess) {
            qdb_set_error("qdb_encoder: out of device memory");
            return nullptr;
        }
        e->cap_out = out_n;
    }
    if (cudaMemcpyAsync(e->mel_dev, mel, mel_n * 4, cudaMemcpyHostToDevice, e->st) != cudaSuccess) {
        qdb_set_error("qdb_encoder: mel upload failed");
        return nullptr;
    }
    if (qdb_encoder_forward_device(e, e->mel_dev, frames, e->out_dev) < 0) return nullptr;
    float *host = (float *)malloc(out_n * 4);
    if (!host) {
        qdb_set_error("qdb_encoder: out of host memory");
        return nullptr;
    }
    int ev[4] = {0, 0, 0, 0};
    if (cudaMemcpyAsync(host, e->out_dev, out_n * 4, cudaMemcpyDeviceToHost, e->st) != cudaSuccess ||
        cudaMemcpyAsync(ev, e->err, sizeof(ev), cudaMemcpyDeviceToHost, e->st) != cudaSuccess ||
        cudaStreamSynchronize(e->st) != cudaSuccess) {
        free(host);
        qdb_set_error("qdb_encoder: forward failed on the device");
        return nullptr;
    }
    if (ev[0]) {
        free(host);
        cudaMemset(e->err, 0, sizeof(ev));
        qdb_set_error("qdb_encoder: a tensor-core GEMM's bounded wait ran out");
        return nullptr;
    }
    *out_seq_len = ntok;
    return host;
}
