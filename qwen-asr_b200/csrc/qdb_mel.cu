// qdb_mel.cu - log-mel spectrogram on the GPU, replacing qwen_mel_spectrogram
// (qwen_asr_audio.c:293-390; filter bank :254-291): 16 kHz mono f32 samples
// -> [128 mel bins, n_frames] with
//   center reflect padding of 200 samples, periodic Hann window of 400,
//   400-point DFT power of 201 bins (hop 160, the last frame dropped),
//   Slaney mel filter bank (128 x 201), log10(max(., 1e-10)), then the
//   dynamic clamp max(v, global_max - 8) and (v + 4) / 4.
//
// The window, DFT and filter tables are computed on the host with the same
// f32 expressions the reference evaluates (so they hold the same values) and
// uploaded once per device. The per-frame sums run in f32 on CUDA cores in
// the reference's order (n = 0..399, k = 0..200): the spectrogram is f32
// arithmetic of ~0.5 MFLOP per frame, far from any roofline that tensor
// cores would change, and a bf16 DFT would not hold the reference's values.
//
//   mel_frames_kernel  one CTA per 16 frames: windowed frames in smem, thread
//                      k computes the 16 frames' bin-k power from its cos/sin
//                      table rows, then thread m the 16 frames' mel bin m and
//                      the block's max (atomicMax on the ordered bits)
//   mel_norm_kernel    clamp, scale, transpose to [128, n_frames]
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "qdb_kernels.h"

namespace {

constexpr int SAMPLE_RATE = 16000, N_MEL = 128, HOP = 160, WIN = 400, N_FFT = 400, N_FREQ = N_FFT / 2 + 1;
constexpr int FB = 16;  // frames per CTA
constexpr float kPi = 3.14159265358979323846f;

// f32 ordered as unsigned (larger float -> larger key), for atomicMax
__device__ __forceinline__ unsigned ord(float f) {
    const unsigned u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unord(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// padded: [n_samples + 400] reflect-padded signal; tables: window [400],
// cos / sin [201][400], filters [128][201]; mel_tmp [n_frames][128].
__global__ void __launch_bounds__(256) mel_frames_kernel(const float *__restrict__ padded, int n_frames,
                                                         const float *__restrict__ window,
                                                         const float *__restrict__ dcos,
                                                         const float *__restrict__ dsin,
                                                         const float *__restrict__ filters, float *__restrict__ mel_tmp,
                                                         unsigned *__restrict__ gmax) {
    __shared__ float win[FB][N_FFT];
    __shared__ float pw[FB][N_FREQ + 3];
    __shared__ unsigned bmax;
    const int f0 = blockIdx.x * FB, t = threadIdx.x;
    const int nf = min(FB, n_frames - f0);
    if (t == 0) bmax = 0u;
    for (int i = t; i < FB * N_FFT; i += blockDim.x) {
        const int f = i / N_FFT, n = i % N_FFT;
        win[f][n] = f < nf ? padded[(size_t)(f0 + f) * HOP + n] * window[n] : 0.f;
    }
    __syncthreads();
    if (t < N_FREQ) {
        float re[FB], im[FB];
#pragma unroll
        for (int f = 0; f < FB; f++) re[f] = im[f] = 0.f;
        const float *cr = dcos + (size_t)t * N_FFT, *sr = dsin + (size_t)t * N_FFT;
        for (int n = 0; n < N_FFT; n++) {
            const float c = __ldg(cr + n), s = __ldg(sr + n);
#pragma unroll
            for (int f = 0; f < FB; f++) {
                re[f] = fmaf(win[f][n], c, re[f]);
                im[f] = fmaf(win[f][n], s, im[f]);
            }
        }
#pragma unroll
        for (int f = 0; f < FB; f++) pw[f][t] = re[f] * re[f] + im[f] * im[f];
    }
    __syncthreads();
    if (t < N_MEL) {
        float acc[FB];
#pragma unroll
        for (int f = 0; f < FB; f++) acc[f] = 0.f;
        const float *fr = filters + (size_t)t * N_FREQ;
        for (int k = 0; k < N_FREQ; k++) {
            const float w = __ldg(fr + k);
#pragma unroll
            for (int f = 0; f < FB; f++) acc[f] = fmaf(w, pw[f][k], acc[f]);
        }
        unsigned m = 0u;
#pragma unroll
        for (int f = 0; f < FB; f++) {
            if (f < nf) {
                const float v = log10f(fmaxf(acc[f], 1e-10f));
                mel_tmp[(size_t)(f0 + f) * N_MEL + t] = v;
                m = max(m, ord(v));
            }
        }
        atomicMax(&bmax, m);
    }
    __syncthreads();
    if (t == 0) atomicMax(gmax, bmax);
}

__global__ void mel_norm_kernel(const float *__restrict__ mel_tmp, int n_frames, const unsigned *__restrict__ gmax,
                                float *__restrict__ mel) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)n_frames * N_MEL) return;
    const int m = (int)(i / n_frames), t = (int)(i % n_frames);
    const float lo = unord(*gmax) - 8.0f;
    const float v = fmaxf(mel_tmp[(size_t)t * N_MEL + m], lo);
    mel[i] = (v + 4.0f) / 4.0f;
}

// Reflect padding of the reference (center = true): out[i] for i < 200 is
// samples[200 - i] (0 past the end), then the samples, then samples[n - 2 - i].
__global__ void mel_pad_kernel(const float *__restrict__ s, int n, float *__restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int pad = N_FFT / 2;
    if (i >= n + 2 * pad) return;
    float v;
    if (i < pad) {
        const int src = pad - i;
        v = src < n ? s[src] : 0.f;
    } else if (i < pad + n) {
        v = s[i - pad];
    } else {
        const int src = n - 2 - (i - pad - n);
        v = src >= 0 ? s[src] : 0.f;
    }
    out[i] = v;
}

// ---------------------------------------------------------------- host tables
float hertz_to_mel(float freq) {
    const float min_log_hertz = 1000.0f, min_log_mel = 15.0f;
    const float logstep = 27.0f / logf(6.4f);
    float mels = 3.0f * freq / 200.0f;
    if (freq >= min_log_hertz) mels = min_log_mel + logf(freq / min_log_hertz) * logstep;
    return mels;
}

float mel_to_hertz(float mels) {
    const float min_log_hertz = 1000.0f, min_log_mel = 15.0f;
    const float logstep = logf(6.4f) / 27.0f;
    float freq = 200.0f * mels / 3.0f;
    if (mels >= min_log_mel) freq = min_log_hertz * expf(logstep * (mels - min_log_mel));
    return freq;
}

struct MelTables {
    float *window = nullptr, *dcos = nullptr, *dsin = nullptr, *filters = nullptr;
    // per-device scratch, grown on demand
    float *padded = nullptr, *tmp = nullptr, *out = nullptr;
    unsigned *gmax = nullptr;
    size_t cap_samples = 0, cap_frames = 0;
    bool ready = false;
};

MelTables g_mel[64];
std::mutex g_mel_mu;

int upload_tables(MelTables &t) {
    std::vector<float> win(WIN), dc((size_t)N_FREQ * N_FFT), ds((size_t)N_FREQ * N_FFT), fl((size_t)N_MEL * N_FREQ);
    for (int i = 0; i < WIN; i++) win[i] = 0.5f * (1.0f - cosf(2.0f * kPi * (float)i / (float)WIN));
    for (int k = 0; k < N_FREQ; k++)
        for (int n = 0; n < N_FFT; n++) {
            const float angle = 2.0f * kPi * (float)k * (float)n / (float)N_FFT;
            dc[(size_t)k * N_FFT + n] = cosf(angle);
            ds[(size_t)k * N_FFT + n] = sinf(angle);
        }
    // Slaney filter bank (qwen_asr_audio.c:254-291)
    float fft_freqs[N_FREQ];
    for (int i = 0; i < N_FREQ; i++) fft_freqs[i] = (float)i * ((float)SAMPLE_RATE / 2.0f) / (float)(N_FREQ - 1);
    const float mel_min = hertz_to_mel(0.0f), mel_max = hertz_to_mel((float)SAMPLE_RATE / 2.0f);
    float ff[N_MEL + 2], fd[N_MEL + 1];
    for (int i = 0; i < N_MEL + 2; i++) ff[i] = mel_to_hertz(mel_min + (mel_max - mel_min) * (float)i / (float)(N_MEL + 1));
    for (int i = 0; i < N_MEL + 1; i++) {
        fd[i] = ff[i + 1] - ff[i];
        if (fd[i] == 0.0f) fd[i] = 1e-6f;
    }
    for (int m = 0; m < N_MEL; m++) {
        const float enorm = 2.0f / (ff[m + 2] - ff[m]);
        for (int f = 0; f < N_FREQ; f++) {
            const float down = (fft_freqs[f] - ff[m]) / fd[m];
            const float up = (ff[m + 2] - fft_freqs[f]) / fd[m + 1];
            float val = fminf(down, up);
            if (val < 0.0f) val = 0.0f;
            fl[(size_t)m * N_FREQ + f] = val * enorm;
        }
    }
    if (cudaMalloc(&t.window, WIN * 4) != cudaSuccess || cudaMalloc(&t.dcos, dc.size() * 4) != cudaSuccess ||
        cudaMalloc(&t.dsin, ds.size() * 4) != cudaSuccess || cudaMalloc(&t.filters, fl.size() * 4) != cudaSuccess ||
        cudaMalloc(&t.gmax, sizeof(unsigned)) != cudaSuccess)
        return -1;
    if (cudaMemcpy(t.window, win.data(), WIN * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(t.dcos, dc.data(), dc.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(t.dsin, ds.data(), ds.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(t.filters, fl.data(), fl.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return -1;
    t.ready = true;
    return 0;
}

}  // namespace

// Frames the reference produces for n_samples (<= 0: too short).
extern "C" int qdb_mel_frames(int n_samples) {
    const int padded = n_samples + N_FFT;
    return (padded - N_FFT) / HOP + 1 - 1;
}

// Device-side spectrogram on the current device: samples_dev f32 [n_samples]
// -> mel_dev f32 [128, n_frames] (n_frames = qdb_mel_frames(n_samples)), all on
// `stream`. Returns 0, or -1 (too short, or a CUDA error).
extern "C" int qdb_mel_spectrogram_device(const float *samples_dev, int n_samples, float *mel_dev,
                                          void *stream_) {
    cudaStream_t stream = (cudaStream_t)stream_;
    const int n_frames = qdb_mel_frames(n_samples);
    if (n_samples <= 0 || n_frames <= 0) return qdb_set_error("qdb_mel_spectrogram: audio too short");
    if (!samples_dev || !mel_dev) return qdb_set_error("qdb_mel_spectrogram: null buffer");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return qdb_set_error("qdb_mel_spectrogram: no usable CUDA device");
    MelTables &t = g_mel[dev];
    {
        std::lock_guard<std::mutex> lk(g_mel_mu);
        if (!t.ready && upload_tables(t)) return qdb_set_error("qdb_mel_spectrogram: table upload failed");
        const size_t ns = (size_t)n_samples + N_FFT;
        if (ns > t.cap_samples) {
            cudaFree(t.padded);
            t.padded = nullptr;
            t.cap_samples = 0;
            if (cudaMalloc(&t.padded, ns * 4) != cudaSuccess) return qdb_set_error("qdb_mel_spectrogram: out of device memory");
            t.cap_samples = ns;
        }
        if ((size_t)n_frames > t.cap_frames) {
            cudaFree(t.tmp);
            t.tmp = nullptr;
            t.cap_frames = 0;
            if (cudaMalloc(&t.tmp, (size_t)n_frames * N_MEL * 4) != cudaSuccess)
                return qdb_set_error("qdb_mel_spectrogram: out of device memory");
            t.cap_frames = n_frames;
        }
    }
    const int np = n_samples + N_FFT;
    mel_pad_kernel<<<(np + 255) / 256, 256, 0, stream>>>(samples_dev, n_samples, t.padded);
    if (cudaMemsetAsync(t.gmax, 0, sizeof(unsigned), stream) != cudaSuccess)
        return qdb_set_error("qdb_mel_spectrogram: cudaMemsetAsync failed");
    mel_frames_kernel<<<(n_frames + FB - 1) / FB, 256, 0, stream>>>(t.padded, n_frames, t.window, t.dcos, t.dsin,
                                                                   t.filters, t.tmp, t.gmax);
    const size_t total = (size_t)n_frames * N_MEL;
    mel_norm_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(t.tmp, n_frames, t.gmax, mel_dev);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : qdb_set_error(cudaGetErrorString(e));
}

// Drop-in for qwen_mel_spectrogram (qwen_asr_audio.c:293): host samples in,
// malloc'd host [128, n_frames] out (the caller frees it), NULL when the audio
// is too short or on error. Runs on the current device; synchronous.
extern "C" float *qdb_mel_spectrogram(const float *samples, int n_samples, int *out_frames) {
    const int n_frames = qdb_mel_frames(n_samples);
    if (n_samples <= 0 || n_frames <= 0) {
        qdb_set_error("qdb_mel_spectrogram: audio too short");
        return nullptr;
    }
    if (!samples || !out_frames) {
        qdb_set_error("qdb_mel_spectrogram: null buffer");
        return nullptr;
    }
    float *s_dev = nullptr, *m_dev = nullptr, *host = nullptr;
    const size_t mel_bytes = (size_t)n_frames * N_MEL * 4;
    if (cudaMalloc(&s_dev, (size_t)n_samples * 4) != cudaSuccess || cudaMalloc(&m_dev, mel_bytes) != cudaSuccess ||
        cudaMemcpy(s_dev, samples, (size_t)n_samples * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        qdb_set_error("qdb_mel_spectrogram: device allocation or upload failed");
    } else if (qdb_mel_spectrogram_device(s_dev, n_samples, m_dev, 0) == 0) {
        host = (float *)malloc(mel_bytes);
        if (!host) {
            qdb_set_error("qdb_mel_spectrogram: out of host memory");
        } else if (cudaMemcpy(host, m_dev, mel_bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
            free(host);
            host = nullptr;
            qdb_set_error("qdb_mel_spectrogram: device to host copy failed");
        }
    }
    cudaFree(s_dev);
    cudaFree(m_dev);
    if (host) *out_frames = n_frames;
    return host;
}
