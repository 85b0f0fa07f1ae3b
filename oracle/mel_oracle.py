"""CPU restatement of the reference's log-mel front end - TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline may import
this module; it is the checker for the GPU spectrogram, never the product.

Restates qwen_asr_audio.c (reference project):
  hertz_to_mel / mel_to_hertz     :236-252  (Slaney scale, log above 1 kHz)
  build_mel_filters               :254-291  (triangular filters, Slaney norm)
  qwen_mel_spectrogram            :293-390  (reflect pad 200, periodic Hann 400,
                                             400-point DFT power of 201 bins,
                                             hop 160 with the last frame dropped,
                                             log10(max(., 1e-10)), clamp to
                                             global max - 8, (v + 4) / 4,
                                             output [128, n_frames])
Tables are built in float32 by the same expressions (cos/sin of a float32
angle); the sums run in numpy float32 matrix products, so results agree with
the reference to float32 rounding of different summation orders.

Pinned against the reference's own qwen_mel_spectrogram compiled from its
sources (oracle/_ref, tests/test_mel.py) and the fixtures it wrote
(tests/golden/mel_ref.npz, made by tests/golden/make_golden.py).
"""
from __future__ import annotations

import numpy as np

SAMPLE_RATE = 16000
N_MEL = 128
HOP = 160
WIN = 400
N_FFT = 400
N_FREQ = N_FFT // 2 + 1

_f = np.float32


def _hz_to_mel(freq):
    freq = _f(freq)
    logstep = _f(27.0) / np.log(_f(6.4))
    if freq >= _f(1000.0):
        return _f(15.0) + np.log(freq / _f(1000.0)) * logstep
    return _f(3.0) * freq / _f(200.0)


def _mel_to_hz(mels):
    mels = _f(mels)
    logstep = np.log(_f(6.4)) / _f(27.0)
    if mels >= _f(15.0):
        return _f(1000.0) * np.exp(logstep * (mels - _f(15.0)))
    return _f(200.0) * mels / _f(3.0)


def mel_filters() -> np.ndarray:
    """[128, 201] float32 filter bank (qwen_asr_audio.c:254-291)."""
    fft_freqs = np.array([_f(i) * (_f(SAMPLE_RATE) / _f(2.0)) / _f(N_FREQ - 1) for i in range(N_FREQ)], _f)
    mmin, mmax = _hz_to_mel(0.0), _hz_to_mel(SAMPLE_RATE / 2.0)
    ff = np.array([_mel_to_hz(mmin + (mmax - mmin) * _f(i) / _f(N_MEL + 1)) for i in range(N_MEL + 2)], _f)
    fd = (ff[1:] - ff[:-1]).astype(_f)
    fd[fd == 0] = _f(1e-6)
    out = np.zeros((N_MEL, N_FREQ), _f)
    for m in range(N_MEL):
        enorm = _f(2.0) / (ff[m + 2] - ff[m])
        down = (fft_freqs - ff[m]) / fd[m]
        up = (ff[m + 2] - fft_freqs) / fd[m + 1]
        out[m] = np.maximum(np.minimum(down, up), _f(0.0)) * enorm
    return out


def tables():
    """(window [400], cos [201, 400], sin [201, 400]) in float32."""
    i = np.arange(WIN, dtype=_f)
    window = (_f(0.5) * (_f(1.0) - np.cos(_f(2.0) * _f(np.pi) * i / _f(WIN)))).astype(_f)
    k = np.arange(N_FREQ, dtype=_f)[:, None]
    n = np.arange(N_FFT, dtype=_f)[None, :]
    angle = (_f(2.0) * _f(np.pi) * k * n / _f(N_FFT)).astype(_f)
    return window, np.cos(angle).astype(_f), np.sin(angle).astype(_f)


def n_frames(n_samples: int) -> int:
    return (n_samples + N_FFT - N_FFT) // HOP + 1 - 1


def reflect_pad(samples: np.ndarray) -> np.ndarray:
    """Center padding of qwen_asr_audio.c:298-308 (0 where the source is out of range)."""
    n = len(samples)
    pad = N_FFT // 2
    out = np.zeros(n + 2 * pad, _f)
    for i in range(pad):
        src = pad - i
        out[i] = samples[src] if src < n else 0.0
        src = n - 2 - i
        out[pad + n + i] = samples[src] if src >= 0 else 0.0
    out[pad:pad + n] = samples
    return out


def mel_spectrogram(samples: np.ndarray):
    """[128, n_frames] float32 log-mel, or None when the audio is too short."""
    samples = np.ascontiguousarray(samples, dtype=_f)
    nf = n_frames(len(samples))
    if len(samples) <= 0 or nf <= 0:
        return None
    padded = reflect_pad(samples)
    window, dcos, dsin = tables()
    idx = np.arange(nf)[:, None] * HOP + np.arange(N_FFT)[None, :]
    frames = padded[idx] * window[None, :]
    re = frames @ dcos.T
    im = frames @ dsin.T
    power = (re * re + im * im).astype(_f)
    mel = power @ mel_filters().T
    mel = np.log10(np.maximum(mel, _f(1e-10))).astype(_f)
    mel = np.maximum(mel, mel.max() - _f(8.0))
    return ((mel + _f(4.0)) / _f(4.0)).T.copy()
