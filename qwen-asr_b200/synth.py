"""Seeded synthetic decoder weights and inputs in the reference's tensor layout.

No checkpoints or datasets are available offline, so parity tests and the
benchmark use random-init weights of the real architectures:

* Decoder shapes follow the reference's hard-coded variants
  (qwen_asr.c:135-191): 0.6B = hidden 1024 / intermediate 3072, 1.7B = hidden
  2048 / intermediate 6144; 28 layers, 16 query / 8 KV heads, head_dim 128,
  vocab 151936, RMSNorm eps 1e-6, RoPE theta 1e6.
* Tensor names are the reference's (qwen_asr_decoder.c:45-116), all bf16.
  Matrices are N(0, 0.02) drawn from one torch.Generator(seed) in sorted
  tensor-name order; norm weights are 1 (optionally jittered for tests so the
  norm weights are exercised).
* Every tensor lives inside one contiguous uint16 host blob (256-byte aligned
  slots) so the same bytes can be handed to the CUDA library, the CPU oracle
  and the reference's own loader without copies.
"""
from __future__ import annotations

import dataclasses

import numpy as np

# Prompt template ids of the reference (qwen_asr.c:339-350): 9 prefix ids
# before the audio embeddings and 6 suffix ids after them.
PROMPT_PREFIX = (151644, 8948, 198, 151645, 198, 151644, 872, 198, 151669)
PROMPT_SUFFIX = (151670, 151645, 198, 151644, 77091, 198)
ENC_TOKENS_PER_SECOND = 13  # 13 encoder tokens per 100 mel frames (1 s)


@dataclasses.dataclass(frozen=True)
class Config:
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    eps: float = 1e-6
    theta: float = 1e6

    def as_tuple(self):
        return (self.hidden, self.layers, self.heads, self.kv_heads, self.head_dim,
                self.intermediate, self.vocab)


PRESETS = {
    "0.6b": Config(1024, 28, 16, 8, 128, 3072, 151936),
    "1.7b": Config(2048, 28, 16, 8, 128, 6144, 151936),
    # Small shapes for parity tests (the oracle finishes them in seconds).
    "tiny": Config(256, 2, 4, 2, 128, 512, 1000),
    "small": Config(512, 3, 8, 4, 128, 768, 4099),
    "gqa4": Config(256, 2, 8, 2, 128, 512, 777),
}

BF16 = 2  # safetensor_dtype_t DTYPE_BF16 in the reference loader


def tensor_specs(cfg: Config):
    """(name, shape) of every decoder tensor, reference naming."""
    h, hd, I = cfg.hidden, cfg.head_dim, cfg.intermediate
    qd, kvd = cfg.heads * hd, cfg.kv_heads * hd
    specs = [("thinker.model.embed_tokens.weight", (cfg.vocab, h)),
             ("thinker.model.norm.weight", (h,))]
    for i in range(cfg.layers):
        p = f"thinker.model.layers.{i}."
        specs += [
            (p + "self_attn.q_proj.weight", (qd, h)),
            (p + "self_attn.k_proj.weight", (kvd, h)),
            (p + "self_attn.v_proj.weight", (kvd, h)),
            (p + "self_attn.o_proj.weight", (h, qd)),
            (p + "self_attn.q_norm.weight", (hd,)),
            (p + "self_attn.k_norm.weight", (hd,)),
            (p + "input_layernorm.weight", (h,)),
            (p + "post_attention_layernorm.weight", (h,)),
            (p + "mlp.gate_proj.weight", (I, h)),
            (p + "mlp.up_proj.weight", (I, h)),
            (p + "mlp.down_proj.weight", (h, I)),
        ]
    return specs


def _is_norm(name: str) -> bool:
    return "norm" in name


class WeightSet:
    """All decoder tensors of one synthetic model in one bf16 host blob."""

    def __init__(self, cfg: Config, seed: int = 0, norm_jitter: float = 0.0, pin: bool = False):
        import torch

        self.cfg = cfg
        specs = tensor_specs(cfg)
        self.offsets = {}
        self.shapes = {}
        off = 0
        for name, shape in specs:
            n = int(np.prod(shape))
            self.offsets[name] = off
            self.shapes[name] = shape
            off += (n + 127) // 128 * 128  # 256-byte slots
        self.n_elems = off
        if pin:
            self._blob_t = torch.empty(off, dtype=torch.int16).pin_memory()
            self.blob = self._blob_t.numpy().view(np.uint16)
        else:
            self.blob = np.empty(off, dtype=np.uint16)
        g = torch.Generator().manual_seed(seed)
        for name in sorted(self.offsets):
            shape = self.shapes[name]
            view = self.view(name)
            if _is_norm(name):
                t = torch.ones(shape)
                if norm_jitter:
                    t = t + norm_jitter * torch.randn(shape, generator=g)
            else:
                t = torch.randn(shape, generator=g) * 0.02
            view[...] = t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        self._f32 = {}

    def view(self, name):
        off = self.offsets[name]
        shape = self.shapes[name]
        return self.blob[off:off + int(np.prod(shape))].reshape(shape)

    def f32(self, name):
        """bf16 tensor widened to f32 (what the reference's load_f32 returns)."""
        if name not in self._f32:
            self._f32[name] = bf16_to_f32(self.view(name))
        return self._f32[name]

    def table(self):
        """(names, byte offsets, byte sizes, shapes) for the reference loader."""
        names, offs, sizes, shapes = [], [], [], []
        for name, _ in tensor_specs(self.cfg):
            names.append(name)
            offs.append(self.offsets[name] * 2)
            sizes.append(int(np.prod(self.shapes[name])) * 2)
            s = self.shapes[name]
            shapes.append((s[0], s[1] if len(s) > 1 else 0))
        return names, offs, sizes, shapes

    def layer(self, i):
        p = f"thinker.model.layers.{i}."
        return dict(
            wq=self.view(p + "self_attn.q_proj.weight"),
            wk=self.view(p + "self_attn.k_proj.weight"),
            wv=self.view(p + "self_attn.v_proj.weight"),
            wo=self.view(p + "self_attn.o_proj.weight"),
            gate=self.view(p + "mlp.gate_proj.weight"),
            up=self.view(p + "mlp.up_proj.weight"),
            down=self.view(p + "mlp.down_proj.weight"),
            q_norm=self.f32(p + "self_attn.q_norm.weight"),
            k_norm=self.f32(p + "self_attn.k_norm.weight"),
            input_norm=self.f32(p + "input_layernorm.weight"),
            post_attn_norm=self.f32(p + "post_attention_layernorm.weight"),
        )

    @property
    def embed(self):
        return self.view("thinker.model.embed_tokens.weight")

    @property
    def final_norm(self):
        return self.f32("thinker.model.norm.weight")


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def embed_rows(ws: WeightSet, ids) -> np.ndarray:
    """Host token embedding, bf16 -> f32 (tok_embed_bf16_to_f32, qwen_asr.c:353-360)."""
    return bf16_to_f32(ws.embed[np.asarray(ids, dtype=np.int64)])


def audio_embeddings(cfg: Config, n_tokens: int, seed: int) -> np.ndarray:
    """Stand-in for the encoder output (the encoder is outside this library):
    seeded N(0, 1) f32 rows of the decoder width."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((n_tokens, cfg.hidden), dtype=np.float32)


def prompt_embeddings(ws: WeightSet, audio: np.ndarray) -> np.ndarray:
    """[prefix ids][audio rows][suffix ids], the reference's input_embeds
    layout without a system prompt or forced language (qwen_asr.c:626-700).
    Small test vocabularies take the ids modulo their size."""
    V = ws.cfg.vocab
    pre = embed_rows(ws, [t % V for t in PROMPT_PREFIX])
    suf = embed_rows(ws, [t % V for t in PROMPT_SUFFIX])
    return np.ascontiguousarray(np.concatenate([pre, audio, suf], axis=0), dtype=np.float32)


def utterance(ws: WeightSet, seconds: float, seed: int) -> np.ndarray:
    n = int(round(seconds * ENC_TOKENS_PER_SECOND))
    return prompt_embeddings(ws, audio_embeddings(ws.cfg, n, seed))


SAMPLE_RATE = 16000


def speech_audio(n_samples: int, seed: int) -> np.ndarray:
    """Seeded synthetic 16 kHz mono float32 audio with speech-like structure:
    a gliding harmonic voice (100-250 Hz fundamental, 8 harmonics with a
    formant-shaped envelope) gated into 80-400 ms syllables, plus low-level
    noise, peak about 0.5. Stands in for recorded utterances (none ship)."""
    rng = np.random.default_rng(seed)
    t = np.arange(n_samples, dtype=np.float64) / SAMPLE_RATE
    f0 = 100.0 + 150.0 * rng.random() + 30.0 * np.sin(2 * np.pi * (0.3 + 0.5 * rng.random()) * t)
    phase = 2 * np.pi * np.cumsum(f0) / SAMPLE_RATE
    formant = 500.0 + 1500.0 * rng.random()
    voice = np.zeros(n_samples)
    for h in range(1, 9):
        voice += np.exp(-((h * f0 - formant) / 800.0) ** 2) * np.sin(h * phase) / h
    gate = np.zeros(n_samples)
    i = 0
    while i < n_samples:
        on = int(SAMPLE_RATE * (0.08 + 0.32 * rng.random()))
        off = int(SAMPLE_RATE * 0.15 * rng.random())
        gate[i:i + on] = np.hanning(max(on, 2))[:max(0, min(on, n_samples - i))]
        i += on + off
    x = voice * gate + 0.01 * rng.standard_normal(n_samples)
    peak = np.abs(x).max() if n_samples else 1.0
    return (0.5 * x / max(peak, 1e-9)).astype(np.float32)


class SyntheticEncoder:
    """Stand-in for one stream's encoder and its window cache (qwen_asr.c:1506-1674):
    completed windows of `window_s` seconds keep fixed rows (seeded per window
    index), the partial tail window is re-encoded each chunk (rows seeded by
    its length), at most `max_windows` completed windows stay (eviction), and
    clear() drops the cache like stream_clear_enc_cache. Rows per second
    follow the encoder's 13 tokens per 100 mel frames (qwen_asr_encoder.c:186-211).
    Synthetic data for the streaming scheduler's tests and benchmark."""

    def __init__(self, hidden, seed, chunk_s=2.0, window_s=8.0, max_windows=4, scale=1.0, bank=None):
        # bank: optional f32 [rows, hidden]; rows are then seeded picks from it
        # (cheap enough for hundreds of streams) instead of fresh draws
        self.h, self.seed, self.scale, self.bank = hidden, seed, scale, bank
        self.chunk, self.window, self.max_windows = chunk_s, window_s, max_windows
        self.cursor = 0.0
        self.next_window = 0.0
        self.cache = []  # (start_s, rows)

    @staticmethod
    def rows_for(seconds):
        frames = int(round(seconds * 100))
        full, rem = divmod(frames, 100)
        n = full * 13
        if rem:
            w = rem
            for _ in range(3):
                w = (w - 1) // 2 + 1
            n += w
        return n

    def _rows(self, key, n):
        rng = np.random.default_rng([self.seed, *key])
        if self.bank is not None:
            return self.bank[rng.integers(0, len(self.bank), n)]
        return (self.scale * rng.standard_normal((n, self.h))).astype(np.float32)

    def advance(self, total_s):
        """Audio rows of the next chunk (None when the stream has ended)."""
        if self.cursor >= total_s:
            return None, True
        self.cursor = min(self.cursor + self.chunk, total_s)
        full_end = int(self.cursor / self.window) * self.window
        while self.next_window < full_end:
            self.cache.append((self.next_window, self._rows((int(self.next_window * 1000), 0),
                                                             self.rows_for(self.window))))
            self.next_window += self.window
        parts = []
        if full_end < self.cursor:
            tail_s = self.cursor - full_end
            parts.append(self._rows((int(full_end * 1000), int(tail_s * 1000)), self.rows_for(tail_s)))
        while len(self.cache) > self.max_windows:
            self.cache.pop(0)
        rows = [r for _, r in self.cache] + parts
        audio = np.concatenate(rows) if rows else np.zeros((0, self.h), np.float32)
        return audio, self.cursor >= total_s

    def clear(self):
        self.cache = []
        self.next_window = int(self.cursor / self.window) * self.window


# ---------------------------------------------------------------- audio encoder
CONV_HIDDEN = 480  # QWEN_CONV_HIDDEN (qwen_asr.h:39)


@dataclasses.dataclass(frozen=True)
class EncoderConfig:
    d_model: int
    layers: int
    heads: int
    head_dim: int
    ffn: int
    output_dim: int

    def as_tuple(self):
        return (self.d_model, self.layers, self.heads, self.head_dim, self.ffn, self.output_dim)


# encoder shapes (qwen_asr.h:48-53); the small ones feed the small decoder presets
ENC_PRESETS = {
    "0.6b": EncoderConfig(896, 18, 14, 64, 3584, 1024),
    "1.7b": EncoderConfig(1024, 24, 16, 64, 4096, 2048),
    "tiny": EncoderConfig(128, 2, 2, 64, 256, 256),
    "small": EncoderConfig(256, 2, 4, 64, 512, 512),
}


def encoder_tensor_specs(ec: EncoderConfig):
    """(name, shape) of every encoder tensor, reference naming (qwen_asr_encoder.c:66-168)."""
    p = "thinker.audio_tower."
    d = ec.d_model
    specs = [(p + "conv2d1.weight", (CONV_HIDDEN, 1, 3, 3)), (p + "conv2d1.bias", (CONV_HIDDEN,)),
             (p + "conv2d2.weight", (CONV_HIDDEN, CONV_HIDDEN, 3, 3)), (p + "conv2d2.bias", (CONV_HIDDEN,)),
             (p + "conv2d3.weight", (CONV_HIDDEN, CONV_HIDDEN, 3, 3)), (p + "conv2d3.bias", (CONV_HIDDEN,)),
             (p + "conv_out.weight", (d, CONV_HIDDEN * 16))]
    for i in range(ec.layers):
        q = f"{p}layers.{i}."
        specs += [(q + "self_attn.q_proj.weight", (d, d)), (q + "self_attn.q_proj.bias", (d,)),
                  (q + "self_attn.k_proj.weight", (d, d)), (q + "self_attn.k_proj.bias", (d,)),
                  (q + "self_attn.v_proj.weight", (d, d)), (q + "self_attn.v_proj.bias", (d,)),
                  (q + "self_attn.out_proj.weight", (d, d)), (q + "self_attn.out_proj.bias", (d,)),
                  (q + "self_attn_layer_norm.weight", (d,)), (q + "self_attn_layer_norm.bias", (d,)),
                  (q + "fc1.weight", (ec.ffn, d)), (q + "fc1.bias", (ec.ffn,)),
                  (q + "fc2.weight", (d, ec.ffn)), (q + "fc2.bias", (d,)),
                  (q + "final_layer_norm.weight", (d,)), (q + "final_layer_norm.bias", (d,))]
    specs += [(p + "ln_post.weight", (d,)), (p + "ln_post.bias", (d,)),
              (p + "proj1.weight", (d, d)), (p + "proj1.bias", (d,)),
              (p + "proj2.weight", (ec.output_dim, d)), (p + "proj2.bias", (ec.output_dim,))]
    return specs


class EncoderWeightSet:
    """All encoder tensors of one synthetic model in one bf16 host blob:
    matrices, conv kernels and biases N(0, std) (std 0.02 by default), LayerNorm
    weights 1 and biases 0 (plus optional jitter). `scale_by_fan_in` draws
    matrices and conv kernels with std 1/sqrt(fan_in) instead, which keeps
    activations O(1) through the stack (parity tests use it so that every
    stage contributes)."""

    def __init__(self, ec: EncoderConfig, seed: int = 0, std: float = 0.02, norm_jitter: float = 0.0,
                 scale_by_fan_in: bool = False):
        import torch

        self.cfg = ec
        self.specs = encoder_tensor_specs(ec)
        self.offsets, self.shapes = {}, {}
        off = 0
        for name, shape in self.specs:
            n = int(np.prod(shape))
            self.offsets[name] = off
            self.shapes[name] = shape
            off += (n + 127) // 128 * 128
        self.blob = np.empty(off, dtype=np.uint16)
        g = torch.Generator().manual_seed(seed)
        for name, shape in self.specs:
            if "norm" in name or "ln_post" in name:
                base = torch.ones(shape) if name.endswith("weight") else torch.zeros(shape)
                t = base + (norm_jitter * torch.randn(shape, generator=g) if norm_jitter else 0)
            elif name.endswith("bias"):
                t = torch.randn(shape, generator=g) * std
            else:
                fan_in = int(np.prod(shape[1:]))
                s = 1.0 / np.sqrt(fan_in) if scale_by_fan_in else std
                t = torch.randn(shape, generator=g) * s
            self.view(name)[...] = t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).reshape(shape)

    def view(self, name):
        off = self.offsets[name]
        shape = self.shapes[name]
        return self.blob[off:off + int(np.prod(shape))].reshape(shape)

    def f32(self, name):
        return bf16_to_f32(self.view(name))

    def table(self):
        """(names, byte offsets, byte sizes, shapes flattened to 2-D) for the reference loader."""
        names, offs, sizes, shapes = [], [], [], []
        for name, s in self.specs:
            names.append(name)
            offs.append(self.offsets[name] * 2)
            sizes.append(int(np.prod(s)) * 2)
            shapes.append((s[0], int(np.prod(s[1:])) if len(s) > 1 else 0))
        return names, offs, sizes, shapes


def encoder_tokens(mel_frames: int, chunk: int = 100) -> int:
    """Encoder output rows for mel_frames (qwen_asr_encoder.c:186-211): per
    100-frame chunk, three stride-2 convolutions."""
    n = 0
    for c0 in range(0, mel_frames, chunk):
        w = min(chunk, mel_frames - c0)
        for _ in range(3):
            w = (w - 1) // 2 + 1
        n += w
    return n


def bench_pcm(seconds: float, seed: int, freq: float = 440.0, noise: float = 0.1, tone: float = 0.05) -> np.ndarray:
    """The benchmark configurations' synthetic audio: seeded white noise (sigma
    `noise` of full scale) plus a `freq` Hz sine of amplitude `tone`, quantised
    to 16-bit PCM and read back as the reference's WAV loader does (s16 / 32768)."""
    n = int(round(seconds * SAMPLE_RATE))
    rng = np.random.default_rng(seed)
    t = np.arange(n, dtype=np.float64) / SAMPLE_RATE
    x = noise * rng.standard_normal(n) + tone * np.sin(2 * np.pi * freq * t)
    pcm = np.clip(np.round(x * 32768.0), -32768, 32767).astype(np.int16)
    return (pcm.astype(np.float32) / 32768.0).astype(np.float32)


def bench_tone_hz(seed: int) -> float:
    """c2's per-utterance sine frequency, uniform in 100-2000 Hz from the seed."""
    return float(np.random.default_rng(seed + 1_000_000).uniform(100.0, 2000.0))
