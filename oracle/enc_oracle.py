"""CPU restatement of the reference's audio encoder - TEST INFRASTRUCTURE.

Only tests/ and __graft_entry__.smoke() may import this module; it checks the
CUDA encoder (qwen-asr_b200/csrc/qdb_encoder.cu) and is never the product.

Restates qwen_encoder_forward (qwen_asr_encoder.c:171-372, reference project)
in numpy float64 (the reference computes in float32; float64 here makes the
oracle the more exact of the two):
  per 100-frame chunk (:186-211): three Conv2D 3x3 stride 2 pad 1 + GELU
    (qwen_conv2d via im2col, qwen_asr_kernels.c:560-634; qwen_gelu tanh form
    :886-893), reshape [480, 16, w3] -> [w3, 7680] with column ch*16 + f
    (:262-271), conv_out projection without bias, per-chunk sinusoidal
    positions (qwen_sinusoidal_pe :1147-1160: sin half then cos half,
    log-timescale ln(10000)/(half-1));
  windows of 13 * (800 / 100) = 104 tokens (:288-296);
  per layer (:311-351): LayerNorm (eps 1e-5, population variance,
    qwen_layer_norm :640-748) -> Q/K/V with bias -> bidirectional softmax
    attention inside each window, scale 1/sqrt(head_dim)
    (qwen_bidirectional_attention :1003-1048) -> out_proj with bias + residual;
    LayerNorm -> fc1 + bias -> GELU -> fc2 + bias + residual;
  final LayerNorm, proj1 + bias -> GELU -> proj2 + bias (:353-365).
Pinned to the reference's own qwen_encoder_forward (oracle/_ref) in
tests/test_encoder.py and by the fixtures in tests/golden/enc_ref.npz.
"""
from __future__ import annotations

import numpy as np

CONV_HIDDEN = 480
CHUNK = 100
WINDOW_INFER = 800


def gelu(x):
    return 0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


def layer_norm(x, w, b, eps=1e-5):
    m = x.mean(axis=-1, keepdims=True)
    v = ((x - m) ** 2).mean(axis=-1, keepdims=True)
    return (x - m) / np.sqrt(v + eps) * w + b


def conv2d_s2(x, w, b):
    """x [C, H, W], w [O, C, 3, 3] -> [O, H', W'] (stride 2, pad 1)."""
    C, H, W = x.shape
    Ho, Wo = (H - 1) // 2 + 1, (W - 1) // 2 + 1
    xp = np.zeros((C, H + 2, W + 2), x.dtype)
    xp[:, 1:H + 1, 1:W + 1] = x
    cols = np.empty((C, 3, 3, Ho, Wo), x.dtype)
    for ki in range(3):
        for kj in range(3):
            cols[:, ki, kj] = xp[:, ki:ki + 2 * Ho:2, kj:kj + 2 * Wo:2]
    out = np.tensordot(w, cols, axes=([1, 2, 3], [0, 1, 2]))
    return out + b[:, None, None]


def sinusoidal_pe(n, d):
    half = d // 2
    lt = np.log(10000.0) / (half - 1)
    inv = np.exp(-np.arange(half) * lt)
    ang = np.arange(n)[:, None] * inv[None, :]
    return np.concatenate([np.sin(ang), np.cos(ang)], axis=1)


def encoder_forward(ews, mel):
    """mel f32 [128, frames] -> float64 [seq, output_dim]"""
    ec = ews.cfg
    p = "thinker.audio_tower."
    f = lambda n: ews.f32(p + n).astype(np.float64)
    mel = np.asarray(mel, np.float64)
    frames = mel.shape[1]
    toks = []
    for c0 in range(0, frames, CHUNK):
        x = mel[None, :, c0:min(c0 + CHUNK, frames)]
        for k in (1, 2, 3):
            x = gelu(conv2d_s2(x, f(f"conv2d{k}.weight"), f(f"conv2d{k}.bias")))
        C, F, T = x.shape  # [480, 16, w3]
        r = x.transpose(2, 0, 1).reshape(T, C * F)  # column ch * 16 + f
        y = r @ f("conv_out.weight").T
        toks.append(y + sinusoidal_pe(T, ec.d_model))
    x = np.concatenate(toks, axis=0)
    n = x.shape[0]
    win = 13 * (WINDOW_INFER // CHUNK)
    H, hd = ec.heads, ec.head_dim
    for i in range(ec.layers):
        q = f"layers.{i}."
        h = layer_norm(x, f(q + "self_attn_layer_norm.weight"), f(q + "self_attn_layer_norm.bias"))
        Q = h @ f(q + "self_attn.q_proj.weight").T + f(q + "self_attn.q_proj.bias")
        K = h @ f(q + "self_attn.k_proj.weight").T + f(q + "self_attn.k_proj.bias")
        V = h @ f(q + "self_attn.v_proj.weight").T + f(q + "self_attn.v_proj.bias")
        att = np.empty_like(Q)
        for w0 in range(0, n, win):
            w1 = min(w0 + win, n)
            for hh in range(H):
                sl = slice(hh * hd, (hh + 1) * hd)
                s = Q[w0:w1, sl] @ K[w0:w1, sl].T / np.sqrt(hd)
                s = np.exp(s - s.max(axis=1, keepdims=True))
                att[w0:w1, sl] = (s / s.sum(axis=1, keepdims=True)) @ V[w0:w1, sl]
        x = x + att @ f(q + "self_attn.out_proj.weight").T + f(q + "self_attn.out_proj.bias")
        h = layer_norm(x, f(q + "final_layer_norm.weight"), f(q + "final_layer_norm.bias"))
        m = gelu(h @ f(q + "fc1.weight").T + f(q + "fc1.bias"))
        x = x + m @ f(q + "fc2.weight").T + f(q + "fc2.bias")
    x = layer_norm(x, f("ln_post.weight"), f("ln_post.bias"))
    x = gelu(x @ f("proj1.weight").T + f("proj1.bias"))
    return x @ f("proj2.weight").T + f("proj2.bias")
