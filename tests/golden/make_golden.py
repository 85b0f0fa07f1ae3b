"""Generates the golden vectors in this directory from the REFERENCE itself.

The reference's own decoder sources (qwen_asr_decoder.c, qwen_asr_kernels*.c,
qwen_asr_safetensors.c) are compiled unmodified into oracle/_ref/ by
oracle/Makefile and driven through qwen_decoder_load / qwen_decoder_prefill /
qwen_decoder_forward (oracle/ref_harness.c). This script runs them on seeded
synthetic weights and inputs and stores tokens and logits, so the parity tests
can pin both the oracle restatement and the CUDA path on a machine without the
reference tree.

Run here (needs oracle/_ref built):  python tests/golden/make_golden.py
  --small-only        only the three small shapes
  --bench=c0,c1,...   only the named benchmark-length cases (c0 c1 c3 c2set)
  --enc               only enc_ref.npz: the reference's qwen_encoder_forward
                      (qwen_asr_encoder.c, compiled unmodified into oracle/_ref)
                      on synthetic encoder weights and the log-mel of seeded
                      synthetic audio (mel by oracle/mel_oracle.py)
  --mel               only mel_ref.npz: the reference's qwen_mel_spectrogram
                      (qwen_asr_audio.c, compiled unmodified into oracle/_ref)
                      on seeded synthetic audio (synth.speech_audio)

The benchmark-length cases record the reference's own prefill time
(ref_prefill_s, with ref_threads threads): c3's 3914-position 1.7B prefill is
the long one.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import __graft_entry__ as ge  # noqa: E402
from oracle.pyoracle import RefDecoder, RefEncoder, margin_top2, ref_mel_spectrogram  # noqa: E402
from oracle import mel_oracle  # noqa: E402

synth = ge.load_synth()

# Small configurations: full logits of every step.
SMALL_CASES = [
    # (preset, norm_jitter, n_audio_tokens, audio_seed, steps)
    ("tiny", 0.1, 20, 1, 10),
    ("gqa4", 0.1, 33, 2, 10),
    ("small", 0.1, 57, 3, 10),
]
# Full-size shapes: tokens, top-64 logits and checksums of every step.
FULL_CASES = [
    ("0.6b", 0.0, 40, 1, 4),
    ("1.7b", 0.0, 24, 1, 3),
]
TOPK = 64
# The benchmark configurations at their own prompt lengths (bench.py CONFIGS):
# c0 = 0.6B, 10 s (130 audio rows); c1 = 1.7B, 30 s (390 rows); c3 = 1.7B,
# 300 s (3900 rows). Tokens, top-64 logits and checksums of every step.
BENCH_CASES = [
    ("c0", "0.6b", 130, 1, 16),
    ("c1", "1.7b", 390, 1, 16),
    ("c3", "1.7b", 3900, 1, 4),
]
# A c2-shaped set: 8 independent 0.6B utterances of different lengths
# (audio seeds 100..107, as bench.py's c2 seeds), 8 steps each.
C2SET_AUDIO = [260, 200, 130, 65, 240, 100, 180, 30]
C2SET_STEPS = 8


def run_case(preset, jitter, n_audio, seed, steps, full_logits, threads):
    cfg = synth.PRESETS[preset]
    ws = synth.WeightSet(cfg, seed=0, norm_jitter=jitter)
    emb = synth.prompt_embeddings(ws, synth.audio_embeddings(cfg, n_audio, seed))
    ref = RefDecoder(ws, threads=threads)
    ref.kv_cache_len = 0
    ref.prefill(emb[:-1])
    e = emb[-1]
    toks, logits, tops, topi, sums, sqs, margins = [], [], [], [], [], [], []
    for _ in range(steps):
        tok, _, lg = ref.forward(e, mask_eos=True)
        toks.append(tok)
        margins.append(margin_top2(lg, mask_eos=True))
        if full_logits:
            logits.append(lg.copy())
        idx = np.argsort(-lg, kind="stable")[:TOPK]
        topi.append(idx.astype(np.int32))
        tops.append(lg[idx])
        sums.append(float(lg.astype(np.float64).sum()))
        sqs.append(float((lg.astype(np.float64) ** 2).sum()))
        e = synth.embed_rows(ws, [tok])[0]
    # Rewind (the streaming caller's prefix reuse, qwen_asr.c:1764): back to
    # the prefill length + 2 and re-run 3 steps from there.
    rew = emb.shape[0] - 1 + 2
    ref.kv_cache_len = rew
    e = synth.embed_rows(ws, [toks[1]])[0]
    rew_toks, rew_logits = [], []
    for _ in range(3):
        tok, _, lg = ref.forward(e, mask_eos=True)
        rew_toks.append(tok)
        if full_logits:
            rew_logits.append(lg.copy())
        e = synth.embed_rows(ws, [tok])[0]
    out = dict(preset=preset, norm_jitter=jitter, n_audio=n_audio, audio_seed=seed, weight_seed=0,
               prefill_len=emb.shape[0] - 1, tokens=np.array(toks, np.int32), margins=np.array(margins),
               top_idx=np.array(topi), top_val=np.array(tops, np.float32), logit_sum=np.array(sums),
               logit_sumsq=np.array(sqs), rewind_pos=rew, rewind_tokens=np.array(rew_toks, np.int32))
    if full_logits:
        out["logits"] = np.array(logits, np.float32)
        out["rewind_logits"] = np.array(rew_logits, np.float32)
    ref.close()
    return out


def summarize_steps(ref, ws, e, steps):
    toks, tops, topi, sums, sqs, margins = [], [], [], [], [], []
    for _ in range(steps):
        tok, _, lg = ref.forward(e, mask_eos=True)
        toks.append(tok)
        margins.append(margin_top2(lg, mask_eos=True))
        idx = np.argsort(-lg, kind="stable")[:TOPK]
        topi.append(idx.astype(np.int32))
        tops.append(lg[idx])
        sums.append(float(lg.astype(np.float64).sum()))
        sqs.append(float((lg.astype(np.float64) ** 2).sum()))
        e = synth.embed_rows(ws, [tok])[0]
    return dict(tokens=np.array(toks, np.int32), margins=np.array(margins), top_idx=np.array(topi),
                top_val=np.array(tops, np.float32), logit_sum=np.array(sums), logit_sumsq=np.array(sqs))


def run_bench_case(name, preset, n_audio, seed, steps, threads):
    import time
    cfg = synth.PRESETS[preset]
    ws = synth.WeightSet(cfg, seed=0)
    emb = synth.prompt_embeddings(ws, synth.audio_embeddings(cfg, n_audio, seed))
    ref = RefDecoder(ws, threads=threads)
    ref.kv_cache_len = 0
    t0 = time.perf_counter()
    ref.prefill(emb[:-1])
    prefill_s = time.perf_counter() - t0
    out = summarize_steps(ref, ws, emb[-1], steps)
    ref.close()
    out.update(preset=preset, norm_jitter=0.0, n_audio=n_audio, audio_seed=seed, weight_seed=0,
               prefill_len=emb.shape[0] - 1, ref_prefill_s=prefill_s, ref_threads=threads)
    return out


def run_c2set(threads):
    cfg = synth.PRESETS["0.6b"]
    ws = synth.WeightSet(cfg, seed=0)
    ref = RefDecoder(ws, threads=threads)
    per = []
    for b, n_audio in enumerate(C2SET_AUDIO):
        emb = synth.prompt_embeddings(ws, synth.audio_embeddings(cfg, n_audio, 100 + b))
        ref.kv_cache_len = 0
        ref.prefill(emb[:-1])
        per.append(summarize_steps(ref, ws, emb[-1], C2SET_STEPS))
    ref.close()
    out = {k: np.stack([p[k] for p in per]) for k in per[0]}
    out.update(preset="0.6b", weight_seed=0, n_audio=np.array(C2SET_AUDIO, np.int32),
               audio_seed=np.arange(100, 100 + len(C2SET_AUDIO), dtype=np.int32))
    return out


# Log-mel cases: (name, n_samples, audio seed; seed < 0 = silence). Short
# ones store the whole [128, frames] output; long ones per-bin and per-frame
# sums plus the first 64 frames.
MEL_FULL = [("m_short", 161, 1), ("m_two_frames", 400, 2), ("m_ragged", 4007, 3), ("m_silence", 16000, -1)]
MEL_SUMS = [("m_2s", 32033, 4), ("m_10s", 160000, 5), ("m_30s", 480000, 6)]
MEL_TOO_SHORT = [0, 1, 100, 159]


def mel_audio(n, seed):
    return np.zeros(n, np.float32) if seed < 0 else synth.speech_audio(n, seed)


def run_mel():
    out = {"too_short": np.array(MEL_TOO_SHORT, np.int32)}
    for n in MEL_TOO_SHORT:
        assert ref_mel_spectrogram(mel_audio(n, 0)) is None
    for name, n, seed in MEL_FULL + MEL_SUMS:
        m = ref_mel_spectrogram(mel_audio(n, seed))
        out[name + "_args"] = np.array([n, seed], np.int64)
        if (name, n, seed) in MEL_FULL:
            out[name] = m
        else:
            out[name + "_bins"] = m.sum(axis=1, dtype=np.float64)
            out[name + "_frames"] = m.sum(axis=0, dtype=np.float64)
            out[name + "_head"] = m[:, :64].copy()
    return out


# Encoder cases: (name, preset, weight std or "fan_in", norm jitter, audio samples, audio seed, full output?)
ENC_CASES = [
    ("e_tiny", "tiny", "fan_in", 0.1, 69333, 21, True),         # 433 frames: a partial last chunk
    ("e_tiny_long", "tiny", "fan_in", 0.1, 321000, 22, False),  # 2006 frames: 3 attention windows
    ("e_06b", "0.6b", 0.02, 0.0, 48000, 23, True),              # real 0.6B shape, 3 s
    ("e_17b", "1.7b", 0.02, 0.0, 32000, 24, False),             # real 1.7B shape, 2 s
]


def enc_weights(preset, std, jitter):
    ec = synth.ENC_PRESETS[preset]
    if std == "fan_in":
        return synth.EncoderWeightSet(ec, seed=0, norm_jitter=jitter, scale_by_fan_in=True)
    return synth.EncoderWeightSet(ec, seed=0, std=std, norm_jitter=jitter)


def enc_mel(n, seed):
    return mel_oracle.mel_spectrogram(synth.speech_audio(n, seed))


def run_enc(threads):
    out = {}
    for name, preset, std, jit, n, seed, full in ENC_CASES:
        ews = enc_weights(preset, std, jit)
        ref = RefEncoder(ews, threads=threads)
        y = ref.forward(enc_mel(n, seed))
        ref.close()
        out[name + "_args"] = np.array([n, seed], np.int64)
        out[name + "_shape"] = np.array(y.shape, np.int64)
        if full:
            out[name] = y
        else:
            out[name + "_head"] = y[:8].copy()
            out[name + "_rowsum"] = y.sum(axis=1, dtype=np.float64)
            out[name + "_rowsq"] = (y.astype(np.float64) ** 2).sum(axis=1)
        print("encoder", name, y.shape, float(np.abs(y).max()))
    return out


def main():
    if "--enc" in sys.argv:
        np.savez_compressed(os.path.join(HERE, "enc_ref.npz"), **run_enc(min(os.cpu_count() or 1, 16)))
        print("wrote enc_ref.npz")
        return
    if "--mel" in sys.argv:
        np.savez_compressed(os.path.join(HERE, "mel_ref.npz"), **run_mel())
        print("wrote mel_ref.npz")
        return
    threads = min(os.cpu_count() or 1, 16)
    for case in ([] if any(a.startswith("--bench=") for a in sys.argv) else SMALL_CASES):
        d = run_case(*case, full_logits=True, threads=threads)
        np.savez_compressed(os.path.join(HERE, f"ref_{case[0]}.npz"), **d)
        print("wrote", case[0], d["tokens"], d["margins"].round(4))
    if "--small-only" in sys.argv:
        return
    only = [x for a in sys.argv if a.startswith("--bench=") for x in a.split("=", 1)[1].split(",")]
    for case in ([] if only else FULL_CASES):
        d = run_case(*case, full_logits=False, threads=threads)
        np.savez_compressed(os.path.join(HERE, f"ref_{case[0]}.npz"), **d)
        print("wrote", case[0], d["tokens"], d["margins"].round(4))
    if "--full-only" in sys.argv:
        return
    for case in BENCH_CASES:
        if only and case[0] not in only:
            continue
        d = run_bench_case(*case, threads=threads)
        np.savez_compressed(os.path.join(HERE, f"ref_{case[0]}.npz"), **d)
        print("wrote", case[0], d["tokens"], d["margins"].round(4), "prefill %.1f s" % d["ref_prefill_s"])
    if not only or "c2set" in only:
        d = run_c2set(threads)
        np.savez_compressed(os.path.join(HERE, "ref_c2set.npz"), **d)
        print("wrote c2set", d["tokens"][:, :4])


if __name__ == "__main__":
    main()
