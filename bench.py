"""Benchmark of the B200 decoder hot path (qwen-asr decoder token loop + prefill).

Metric: decode tok/s per GPU (b=1 and batched) as a fraction of
the HBM roofline, plus end-to-end x-realtime of the decoder stage.

Default workload = config c2: the 0.6B-shaped decoder, 64 independent
utterances of 20 s (274-position prompts), 200 greedy tokens each with EOS
masked, decoded as one batch and sharded evenly over the ranks (strong
scaling: 64/N utterances per GPU, no collective on the data path). At N=1 the
same JSON line carries a `b1` object with the batch-1 configs c0 (0.6B, 10 s,
128 tokens) and c1 (1.7B, 30 s, 256 tokens) measured in the same run.
`--config c0|c1|c3` makes a batch-1 config the headline instead (replicas on
N>1, weak scaling).

One timed step = this rank's utterances: one batched prefill of every prompt
(qdb_prefill_batch: all rows in one row batch) followed by the greedy decode
loop (b=1: one persistent kernel launch per position; batches: a CUDA graph of
one step replayed per position). `value` = decoded tokens (all ranks) / decode time
(max over ranks), inputs resident in HBM (device embedding lookup, device
greedy loop). `e2e` = the same metric through the reference-facing C ABI with
host buffers: host f32 prompt embeddings (pinned) through qdb_prefill(_batch), then
one host embedding row in and one token out per utterance per decode step
(the qwen_asr.c:729-759 caller loop; qdb_forward_batch for batches).

Weights and inputs are seeded synthetic data of the real shapes (no
checkpoints offline). Weights (1.2 / 3.4 GB) exceed the 126 MB L2, so every
step streams them from HBM; no flush is needed.

--impl reference times the reference's own CPU decoder (oracle/_ref, built
from the reference sources) on this host for the same config: the decode of
one utterance (the reference decodes utterances one after another), sampled
evenly over the whole decode context range of the config at every step. This
arm never loads the CUDA library.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import socket
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

CONFIGS = {
    # name: (preset, seconds of audio, decode tokens, utterances)
    "c0": ("0.6b", 10.0, 128, 1),
    "c1": ("1.7b", 30.0, 256, 1),
    "c2": ("0.6b", 20.0, 200, 64),
    "c3": ("1.7b", 300.0, 1024, 1),
    # streaming: 256 streams of 120 s, 2 s chunks, <= 32 tokens per chunk (run_streams_*)
    "c4": ("0.6b", 120.0, 32, 256),
}
C4_CHUNK_S = 2.0
C4_METRIC = "streaming decode tok/s (all streams) and x-realtime of the decoder side"
KV_BYTES_PER_POS = 28 * 8 * 128 * 2 * 2  # fp16 K and V per cached position (all layers; 0.6B and 1.7B alike)
METRIC = "decode tok/s/GPU (b=1, b=64) as % of 8 TB/s HBM; end-to-end x-realtime"
REF_WINDOWS = 8  # reference sample: windows spread evenly over the decode range


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def load_synth_standalone():
    """synth.py by file path: the seeded weights and inputs without importing
    the package (which loads the CUDA library)."""
    name = "qdb_bench_synth"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(REPO, "qwen-asr_b200", "synth.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples during the timed region (clocks and throttle reasons)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def step_traffic_from_profile(kernel, workload):
    """dram bytes per launch recorded from an ncu capture in profiles/ (or None)."""
    p = os.path.join(REPO, "profiles", f"{kernel}_{workload}.txt")
    if not os.path.exists(p):
        return None
    for ln in open(p):
        if ln.startswith("traffic_bytes_per_launch:"):
            return float(ln.split(":", 1)[1])
    return None


def utterance_seed(cfg_name, u):
    return 1 if CONFIGS[cfg_name][3] == 1 else 100 + u


def config_block(cfg_name, world, n_local, P):
    preset, seconds, n_dec, n_utt = CONFIGS[cfg_name]
    if n_utt > 1:
        par = f"dp{world}: {n_utt} utterances split into contiguous blocks, no collective" if world > 1 else \
            "single GPU"
    else:
        par = f"{world} independent replicas (one utterance does not shard)" if world > 1 else "single GPU"
    return {"workload": f"{cfg_name}: {preset} decoder, {n_utt} utterance(s) of {seconds:g} s "
                        f"-> prefill {P} positions + {n_dec} greedy tokens each (EOS masked)",
            "global_batch": n_utt if n_utt > 1 else world, "per_gpu_batch": n_local, "prefill_len": P,
            "decode_tokens": n_dec, "parallelism": par,
            "l2": "weights (> 1 GB) exceed the 126 MB L2; no flush needed"}


def weight_bytes(cfg):
    h, L, V, I = cfg.hidden, cfg.layers, cfg.vocab, cfg.intermediate
    qd, kvd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    return 2 * (L * ((qd + 2 * kvd) * h + h * qd + 2 * I * h + h * I) + V * h)


def measure(pkg, synth, cfg_name, world, rank, local, steps, warmup, clocks=None, e2e_steps=3):
    """Times `steps` steps of cfg_name on this rank; returns a dict of device
    times (ms, this rank) and what the JSON line needs."""
    import torch

    preset, seconds, n_dec, n_utt = CONFIGS[cfg_name]
    cfg = synth.PRESETS[preset]
    if n_utt > 1:
        import importlib
        shard = importlib.import_module("qwen_asr_b200.shard")
        first, n_local = shard.shard_range(n_utt, world, rank)
    else:
        first, n_local = 0, 1
    t0 = time.time()
    ws = synth.WeightSet(cfg, seed=0)
    embs = [synth.utterance(ws, seconds, utterance_seed(cfg_name, u)) for u in range(first, first + n_local)]
    P = embs[0].shape[0] - 1  # prefill length; the last prompt position is token 198
    last_tok = synth.PROMPT_SUFFIX[-1]
    t_up = time.perf_counter()
    model = pkg.Model(ws, device=local, mask_eos=True)  # weight upload: staged through pinned buffers
    upload_s = time.perf_counter() - t_up
    setup_s = time.time() - t0
    stream = torch.cuda.ExternalStream(model.stream_handle, device=torch.device("cuda", local))
    cap = P + n_dec + 8
    sessions = [model.session(cap) for _ in range(n_local)]
    # every prompt of this rank back to back: one batched prefill
    emb_dev = torch.from_numpy(np.concatenate([e[:-1] for e in embs])).to(f"cuda:{local}")
    torch.cuda.synchronize()

    def one_step(timing):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(stream)
        if n_local == 1:
            sessions[0].prefill_device(emb_dev.data_ptr(), P, 0)
        else:
            pkg.prefill_batch_device(sessions, emb_dev.data_ptr(), [P] * n_local, [0] * n_local)
        ev[1].record(stream)
        if n_local == 1:
            toks = sessions[0].decode_greedy(last_tok, P, n_dec)
        else:
            toks = pkg.decode_greedy_batch(sessions, [last_tok] * n_local, [P] * n_local, n_dec)
        ev[2].record(stream)
        timing.append(ev)
        return toks

    for _ in range(warmup):
        one_step([])
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    if clocks:
        clocks.start()
    timing = []
    t_wall = time.time()
    for _ in range(steps):
        one_step(timing)
    torch.cuda.synchronize()
    wall = time.time() - t_wall
    clk = clocks.stop() if clocks else None
    pre_ms = sum(e[0].elapsed_time(e[1]) for e in timing)
    dec_ms = sum(e[1].elapsed_time(e[2]) for e in timing)
    tot_ms = sum(e[0].elapsed_time(e[2]) for e in timing)

    # e2e through the reference-facing ABI with host buffers (pinned inputs)
    pinned = [torch.from_numpy(e).pin_memory() for e in embs]
    prompts = torch.from_numpy(np.concatenate([e[:-1] for e in embs])).pin_memory()
    emb_tab = ws.embed  # host bf16 table, the caller's mmap
    e2e_ev = []

    def e2e_step():
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(stream)
        if n_local == 1:
            sessions[0].prefill(prompts.numpy(), 0)
        else:
            pkg.prefill_batch(sessions, prompts.numpy(), [0] * n_local, lens=[P] * n_local)
        ev[1].record(stream)
        if n_local == 1:
            s = sessions[0]
            x = pinned[0].numpy()[-1]
            for i in range(n_dec):
                t, _, _ = s.forward(x, P + i)
                x = synth.bf16_to_f32(emb_tab[t])
        else:
            x = np.stack([p.numpy()[-1] for p in pinned])
            for i in range(n_dec):
                t = pkg.forward_batch(sessions, x, [P + i] * n_local)
                x = synth.bf16_to_f32(emb_tab[t])
        ev[2].record(stream)
        e2e_ev.append(ev)

    e2e_step()  # warm
    e2e_ev.clear()
    for _ in range(e2e_steps):
        e2e_step()
    torch.cuda.synchronize()
    e2e_dec_ms = sum(e[1].elapsed_time(e[2]) for e in e2e_ev)
    e2e_tot_ms = sum(e[0].elapsed_time(e[2]) for e in e2e_ev)
    h = cfg.hidden
    h2d = sum(e.numel() * 4 for e in pinned) - n_local * h * 4 + n_dec * n_local * h * 4
    d2h = n_dec * n_local * 4
    for s in sessions:
        s.close()
    model.close()
    del emb_dev
    torch.cuda.synchronize()
    return dict(cfg=cfg, ws=ws, embs=embs, P=P, n_dec=n_dec, n_utt=n_utt, n_local=n_local, seconds=seconds,
                pre_ms=pre_ms, dec_ms=dec_ms, tot_ms=tot_ms, e2e_dec_ms=e2e_dec_ms, e2e_tot_ms=e2e_tot_ms,
                e2e_steps=e2e_steps, h2d=h2d, d2h=d2h, clk=clk, wall=wall, setup_s=setup_s, upload_s=upload_s)


def measure_pipeline(pkg, synth, cfg_name, first, n_local, local, steps, warmup=1):
    """Whole offline pipeline on the GPU for this rank's utterances of cfg_name:
    PCM (pinned host) -> log-mel (qdb_mel) -> encoder (qdb_encoder) -> prompt rows
    (qdb_build_prompt_device) -> one batched prefill -> greedy decode, tokens back
    to the host. Returns per-stage device ms per step and the step total."""
    import torch

    preset, seconds, n_dec, n_utt = CONFIGS[cfg_name]
    cfg, ecfg = synth.PRESETS[preset], synth.ENC_PRESETS[preset]
    ws = synth.WeightSet(cfg, seed=0)
    ews = synth.EncoderWeightSet(ecfg, seed=0)
    model = pkg.Model(ws, device=local, mask_eos=True)
    enc = pkg.Encoder(ews, device=local)
    dev = torch.device("cuda", local)
    seeds = [utterance_seed(cfg_name, u) for u in range(first, first + n_local)]
    freqs = [synth.bench_tone_hz(sd) if n_utt > 1 else 440.0 for sd in seeds]
    pcm = [torch.from_numpy(synth.bench_pcm(seconds, sd, f)).pin_memory() for sd, f in zip(seeds, freqs)]
    ns = [p.numel() for p in pcm]
    frames = [pkg.mel_frames(n) for n in ns]
    toks = [pkg.Encoder.tokens(f) for f in frames]
    samples_dev = torch.empty(sum(ns), dtype=torch.float32, device=dev)
    mel_dev = torch.empty(128 * sum(frames), dtype=torch.float32, device=dev)
    audio_dev = torch.empty((sum(toks), cfg.hidden), dtype=torch.float32, device=dev)
    pre = [t % cfg.vocab for t in synth.PROMPT_PREFIX]
    suf = [t % cfg.vocab for t in synth.PROMPT_SUFFIX]
    desc, lens, a0 = [], [], 0
    for t in toks:
        rows = pre + [-(a0 + r + 1) for r in range(t)] + suf
        desc += rows[:-1]  # the prefill takes all rows but the last (a token, fed to the first step)
        lens.append(len(rows) - 1)
        a0 += t
    emb_dev = torch.empty((len(desc), cfg.hidden), dtype=torch.float32, device=dev)
    mel_ptrs = [int(mel_dev.data_ptr() + 4 * o) for o in np.cumsum([0] + [128 * f for f in frames[:-1]])]
    sessions = [model.session(max(lens) + n_dec + 8) for _ in range(n_local)]
    es = torch.cuda.ExternalStream(enc.stream_handle, device=dev)
    ms_ = torch.cuda.ExternalStream(model.stream_handle, device=dev)
    # The PCM copies run on a torch-owned stream: torch's pinned-memory pool
    # records an event on every stream a pinned block was used on when the
    # block is freed, so that stream must outlive the tensors (the library's
    # streams die with their objects).
    cs = torch.cuda.Stream(device=dev)

    def step(rec):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
        ev[0].record(cs)
        so = 0
        with torch.cuda.stream(cs):
            for p, n in zip(pcm, ns):
                samples_dev[so:so + n].copy_(p, non_blocking=True)
                so += n
        ev[1].record(cs)
        es.wait_event(ev[1])
        so = mo = 0
        for n, f in zip(ns, frames):
            pkg.mel_spectrogram_device(samples_dev.data_ptr() + 4 * so, n, mel_dev.data_ptr() + 4 * mo,
                                       enc.stream_handle)
            so += n
            mo += 128 * f
        ev[2].record(es)
        enc.forward_batch_device(mel_ptrs, frames, audio_dev.data_ptr())  # every utterance in one pass
        ev[3].record(es)
        ms_.wait_event(ev[3])
        model.build_prompt_device(desc, audio_dev.data_ptr(), emb_dev.data_ptr())
        ev[4].record(ms_)
        if n_local == 1:
            sessions[0].prefill_device(emb_dev.data_ptr(), lens[0], 0)
        else:
            pkg.prefill_batch_device(sessions, emb_dev.data_ptr(), lens, [0] * n_local)
        ev[5].record(ms_)
        if n_local == 1:
            out = sessions[0].decode_greedy(suf[-1], lens[0], n_dec)
        else:
            out = pkg.decode_greedy_batch(sessions, [suf[-1]] * n_local, lens, n_dec)
        ev[6].record(ms_)
        if rec is not None:
            rec.append(ev)
        return out

    for _ in range(warmup):
        step(None)
    torch.cuda.synchronize()
    rec = []
    for _ in range(steps):
        step(rec)
    torch.cuda.synchronize()
    names = ("h2d", "mel", "encoder", "prompt", "prefill", "decode")
    # the median step: the stages are separate host calls, and a host stall
    # between two calls (the GPU box's host is shared) idles the GPU inside an
    # interval; the median step is the steady state, the mean is reported too
    totals = [r[0].elapsed_time(r[6]) for r in rec]
    med = rec[sorted(range(len(rec)), key=lambda i: totals[i])[len(rec) // 2]]
    stage = {k: med[i].elapsed_time(med[i + 1]) for i, k in enumerate(names)}
    total = med[0].elapsed_time(med[6])
    mean_total = sum(totals) / len(totals)
    torch.cuda.synchronize()
    del pcm, rec
    for s_ in sessions:
        s_.close()
    enc.close()
    model.close()
    return {"stage_ms": {k: round(v, 3) for k, v in stage.items()}, "total_ms": total, "mean_total_ms": mean_total,
            "audio_s": seconds * n_local, "tokens": n_dec * n_local, "encoder_tokens": sum(toks),
            "ews": ews, "mel_frames": frames[0]}


def cpu_pipeline_sample(synth, ws, ews, cfg_name, dec_tok_s):
    """The reference's CPU stages for one utterance of cfg_name on this host:
    qwen_mel_spectrogram and qwen_encoder_forward (oracle/_ref), prefill, and
    the greedy decode at the per-token rate measured by the CPU baseline."""
    from oracle.pyoracle import RefDecoder, RefEncoder, ref_mel_spectrogram
    preset, seconds, n_dec, n_utt = CONFIGS[cfg_name]
    th = ref_threads()
    sd = utterance_seed(cfg_name, 0)
    x = synth.bench_pcm(seconds, sd, synth.bench_tone_hz(sd) if n_utt > 1 else 440.0)
    t0 = time.perf_counter()
    mel = ref_mel_spectrogram(x)
    t1 = time.perf_counter()
    re_ = RefEncoder(ews, threads=th)
    t2 = time.perf_counter()
    audio = re_.forward(mel)
    t3 = time.perf_counter()
    re_.close()
    emb = synth.prompt_embeddings(ws, audio)
    rd = RefDecoder(ws, threads=th)
    t4 = time.perf_counter()
    rd.prefill(emb[:-1])
    t5 = time.perf_counter()
    rd.close()
    dec_s = n_dec / dec_tok_s
    total = (t1 - t0) + (t3 - t2) + (t5 - t4) + dec_s
    return {"stage_s": {"mel": round(t1 - t0, 3), "encoder": round(t3 - t2, 3), "prefill": round(t5 - t4, 3),
                        "decode": round(dec_s, 3)},
            "x_realtime": round(seconds / total, 3), "cores": th, "kind": "reference",
            "sample": f"one utterance ({seconds:g} s): reference mel, encoder and prefill timed once; decode = "
                      f"{n_dec} tokens at the CPU baseline's measured {dec_tok_s:.2f} tok/s"}


def summarize(m, cfg_name, world, steps):
    """Rates and roofline of one measure() result whose times are already the
    max over ranks."""
    n_dec, n_utt, n_local, P = m["n_dec"], m["n_utt"], m["n_local"], m["P"]
    per_step_tokens = n_dec * (n_utt if n_utt > 1 else world)
    value = steps * per_step_tokens / (m["dec_ms"] / 1e3)
    e2e_value = m["e2e_steps"] * per_step_tokens / (m["e2e_dec_ms"] / 1e3)
    ctx_avg = P + (n_dec + 1) / 2.0
    bytes_per_step = weight_bytes(m["cfg"]) + n_local * KV_BYTES_PER_POS * ctx_avg
    launch_s = (m["dec_ms"] / 1e3) / (steps * n_dec)
    achieved = bytes_per_step / launch_s / 1e9
    peak, peak_kind = measured_peaks()
    # b=1: one persistent step kernel per token; batches: the CUDA graph of one
    # step (9 kernels per layer + 5), whose weight + KV bytes are counted once
    kernel = "step_kernel" if n_local == 1 else "rows_decode"
    return dict(value=value, e2e_value=e2e_value, achieved=achieved, peak=peak, peak_kind=peak_kind,
                frac=achieved / peak, kernel=kernel, bytes_per_step=bytes_per_step,
                traffic=step_traffic_from_profile(kernel, cfg_name))


def launches_per_step(cfg, n_local, n_dec):
    # prefill (all of the rank's prompts in one row batch), per layer: 2 norms, 4 GEMMs, q/k RoPE +
    # KV append, attention, bf16 split of the SwiGLU output. Decode, b=1: one persistent step kernel
    # per token (qdb_step.cu). Decode, batches: a graph-replayed step of the same 9 kernels per layer
    # plus embedding lookup, final norm, lm_head GEMM, argmax and the step counter.
    if n_local == 1:
        return cfg.layers * 9 + n_dec
    return cfg.layers * 9 + n_dec * (cfg.layers * 9 + 5)


def run_ours(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    import __graft_entry__ as ge
    pkg = ge.load_package()
    synth = ge.load_synth()
    import importlib
    shard = importlib.import_module("qwen_asr_b200.shard")

    m = measure(pkg, synth, args.config, world, rank, local, args.steps, args.warmup, clocks=ClockSampler(local))
    keys = ["dec_ms", "pre_ms", "tot_ms", "e2e_dec_ms", "e2e_tot_ms"]
    for k, v in zip(keys, shard.max_over_ranks([m[k] for k in keys], device=f"cuda:{local}")):
        m[k] = v
    r = summarize(m, args.config, world, args.steps)
    n_local, seconds, steps = m["n_local"], m["seconds"], args.steps
    n_utt = m["n_utt"]
    result = {
        "metric": METRIC,
        "value": round(r["value"], 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(m["tot_ms"] / steps, 3),
        "higher_is_better": True,
        "scaling": "strong" if n_utt > 1 else "weak",
        "vs_baseline": None,
        "dtype": "bf16 weights x f32 activations (f32 accumulate), fp16 KV cache",
        "data": "synthetic: seeded random-init weights of the real shape, seeded prompt embeddings",
        "config": config_block(args.config, world, n_local, m["P"]),
        "prefill_ms": round(m["pre_ms"] / steps, 3),
        "decode_ms": round(m["dec_ms"] / steps, 3),
        "decoder_x_realtime": round(seconds * (n_utt if n_utt > 1 else world) * steps / (m["tot_ms"] / 1e3), 2),
        "e2e": {"value": round(r["e2e_value"], 2), "unit": "tok/s", "h2d_bytes_per_step": int(m["h2d"]),
                "d2h_bytes_per_step": int(m["d2h"]),
                "decoder_x_realtime": round(seconds * (n_utt if n_utt > 1 else world) * m["e2e_steps"]
                                            / (m["e2e_tot_ms"] / 1e3), 2),
                "path": "qdb_prefill + qdb_forward (b=1) / qdb_forward_batch (batches) with host buffers"},
        "roofline": {"bound": "hbm", "achieved": round(r["achieved"], 1), "peak": r["peak"], "unit": "GB/s",
                     "frac": round(r["frac"], 4), "traffic": r["traffic"], "kernel": r["kernel"],
                     "peak_kind": f"{r['peak_kind']} (MEASURED_PEAKS.json hbm_gbs)",
                     "bytes_per_launch": int(r["bytes_per_step"])},
        "gpu_launches": int(launches_per_step(m["cfg"], n_local, m["n_dec"]) * steps),
        "clocks": m["clk"],
        "wall_s": round(m["wall"], 3),
        "setup_s": round(m["setup_s"], 1),
        "weight_upload": {"s": round(m["upload_s"], 3), "bytes": int(weight_bytes(m["cfg"])),
                          "gb_s": round(weight_bytes(m["cfg"]) / m["upload_s"] / 1e9, 2),
                          "path": "qdb_model_set_* from pageable host memory (the reference's mmap case), "
                                  "double-buffered pinned staging"},
    }
    if rank == 0 and world == 1 and not args.no_b1 and args.config == "c2":
        b1 = {}
        for name in ("c0", "c1"):
            mb = measure(pkg, synth, name, 1, 0, local, min(steps, 5), args.warmup, e2e_steps=2)
            rb = summarize(mb, name, 1, min(steps, 5))
            b1[name] = {"value": round(rb["value"], 2), "unit": "tok/s", "roofline_frac": round(rb["frac"], 4),
                        "achieved_gbs": round(rb["achieved"], 1), "e2e": round(rb["e2e_value"], 2),
                        "prefill_ms": round(mb["pre_ms"] / min(steps, 5), 3),
                        "steps": min(steps, 5), "workload": config_block(name, 1, 1, mb["P"])["workload"]}
        result["b1"] = b1
    if not args.no_pipeline:
        first, n_local_p = shard.shard_range(n_utt, world, rank) if n_utt > 1 else (0, 1)
        pl = measure_pipeline(pkg, synth, args.config, first, n_local_p, local, 5)
        tot = shard.max_over_ranks([pl["total_ms"]] + list(pl["stage_ms"].values()) + [pl["mean_total_ms"]],
                                   device=f"cuda:{local}")
        audio_all = seconds * (n_utt if n_utt > 1 else world)
        result["pipeline"] = {
            "x_realtime": round(audio_all / (tot[0] / 1e3), 2),
            "tok_s": round((m["n_dec"] * (n_utt if n_utt > 1 else world)) / (tot[0] / 1e3), 2),
            "ms_per_step": round(tot[0], 3),
            "stage_ms": dict(zip(pl["stage_ms"].keys(), [round(v, 3) for v in tot[1:-1]])),
            "steps": "median of 5 steps (stages of that step); mean step "
                     f"{tot[-1]:.1f} ms",
            "path": "pinned PCM -> qdb_mel_spectrogram_device -> qdb_encoder_forward_batch_device -> "
                    "qdb_build_prompt_device -> batched prefill -> device greedy loop -> tokens on the host",
            "stages_on_gpu": "all (mel, encoder, prefill, decode)",
            "encoder_tokens_per_step": pl["encoder_tokens"]}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(synth, m["ws"], m["embs"][0], args.config)
        if "pipeline" in result:
            result["cpu_baseline"]["pipeline"] = cpu_pipeline_sample(
                synth, m["ws"], pl["ews"], args.config, result["cpu_baseline"]["value"])
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def stream_encoders(synth, cfg, seeds, bank):
    return [synth.SyntheticEncoder(cfg.hidden, sd, chunk_s=C4_CHUNK_S, bank=bank) for sd in seeds]


def c4_config(world, n_local):
    return {"workload": f"c4: 0.6b decoder, 256 streams of 120 s in 2 s chunks, prefix-rollback re-prefill "
                        f"(past-text conditioning on), <= 32 greedy tokens per chunk (EOS masked)",
            "global_batch": 256, "per_gpu_batch": n_local, "chunk_s": C4_CHUNK_S,
            "parallelism": f"dp{world}: streams split into contiguous blocks, no collective" if world > 1
            else "single GPU",
            "phases": "streams staggered over the 60 chunks of a stream before timing; a finished stream "
                      "restarts as a new one",
            "l2": "weights (> 1 GB) exceed the 126 MB L2; no flush needed"}


def run_streams_ours(args):
    """c4: every timed step is one chunk of every stream of this rank through
    qdb_streams_chunk (host encoder rows in, tokens out)."""
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    import __graft_entry__ as ge
    pkg = ge.load_package()
    synth = ge.load_synth()
    import importlib
    shard = importlib.import_module("qwen_asr_b200.shard")
    preset, seconds, max_new, n_streams = CONFIGS["c4"]
    cfg = synth.PRESETS[preset]
    first, n_local = shard.shard_range(n_streams, world, rank)
    t0 = time.time()
    ws = synth.WeightSet(cfg, seed=0)
    model = pkg.Model(ws, device=local, mask_eos=True)
    S = pkg.Streams(model, n_local, max_new_tokens=max_new, past_text=True,
                    head=[t % cfg.vocab for t in synth.PROMPT_PREFIX[:3]],
                    tail=[t % cfg.vocab for t in synth.PROMPT_PREFIX[3:]],
                    suffix=[t % cfg.vocab for t in synth.PROMPT_SUFFIX])
    bank = np.random.default_rng(4242).standard_normal((16384, cfg.hidden), dtype=np.float32)
    next_seed = [1000 + first + i for i in range(n_local)]
    encs = stream_encoders(synth, cfg, next_seed, bank)
    chunks_per_stream = int(seconds / C4_CHUNK_S)

    def round_inputs(only=None):
        audio, fin = [], []
        for i, e in enumerate(encs):
            if only is not None and not only[i]:
                audio.append(None)
                fin.append(False)
                continue
            a, f = e.advance(seconds)
            audio.append(a)
            fin.append(f)
        return audio, fin

    def after_round(rs, fin):
        for i in range(n_local):
            if fin[i]:  # a new stream takes the slot
                next_seed[i] += n_streams
                encs[i] = stream_encoders(synth, cfg, [next_seed[i]], bank)[0]
                S.reset(i)
            elif rs[i]:
                encs[i].clear()

    # stagger: stream i starts (i * 60 / n) chunks ahead, so every phase of a stream is in flight
    target = [(i * chunks_per_stream) // n_local for i in range(n_local)]
    for k in range(max(target)):
        only = [target[i] > k for i in range(n_local)]
        audio, fin = round_inputs(only)
        _, rs = S.chunk(audio, fin)
        after_round(rs, fin)
    setup_s = time.time() - t0
    stream = torch.cuda.ExternalStream(model.stream_handle, device=torch.device("cuda", local))

    def one(record):
        audio, fin = round_inputs()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        h2d = sum(a.nbytes for a in audio if a is not None)
        w0 = time.perf_counter()
        ev[0].record(stream)
        _, rs = S.chunk(audio, fin)
        ev[1].record(stream)
        wall = time.perf_counter() - w0
        lc = S.last_chunk()
        toks = sum(S.stats(i)["last_generated"] for i in range(n_local))
        pls = [S.stats(i)["last_prefill_len"] for i in range(n_local)]
        ctx = np.mean(pls)
        ctx_max = max(pls) + max_new
        after_round(rs, fin)
        if record is not None:
            record.append(dict(ev=ev, wall=wall, toks=toks, ctx=ctx, ctx_max=ctx_max, h2d=h2d, lc=lc,
                               audio_s=C4_CHUNK_S * sum(a is not None for a in audio)))

    for _ in range(args.warmup):
        one(None)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    rec = []
    for _ in range(args.steps):
        one(rec)
    torch.cuda.synchronize()
    clk = clocks.stop()
    dev_ms = sum(r["ev"][0].elapsed_time(r["ev"][1]) for r in rec)
    wall_ms = sum(r["wall"] for r in rec) * 1e3
    pre_ms = sum(r["lc"]["prefill_ms"] for r in rec)
    dec_ms = sum(r["lc"]["decode_ms"] for r in rec)
    toks = sum(r["toks"] for r in rec)
    audio_s = sum(r["audio_s"] for r in rec)
    rows = sum(r["lc"]["rows"] for r in rec)
    ctx = float(np.mean([r["ctx"] for r in rec]))
    mx = shard.max_over_ranks([dev_ms, wall_ms, pre_ms, dec_ms], device=f"cuda:{local}")
    dev_ms, wall_ms, pre_ms, dec_ms = mx
    tot = shard.sum_over_ranks([toks, audio_s, rows], device=f"cuda:{local}")
    toks, audio_s, rows = tot
    bytes_step = weight_bytes(cfg) + n_local * KV_BYTES_PER_POS * (ctx + (max_new + 1) / 2.0)
    achieved = bytes_step * max_new * args.steps / (dec_ms / 1e3) / 1e9
    peak, peak_kind = measured_peaks()
    nparams = weight_bytes(cfg) / 2 - cfg.vocab * cfg.hidden
    pre_tflops = 2 * nparams * rows / (pre_ms / 1e3) / 1e12 / world if pre_ms > 0 else None
    result = {
        "metric": C4_METRIC, "value": round(toks / (dev_ms / 1e3), 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 weights x f32 activations (f32 accumulate), fp16 KV cache",
        "data": "synthetic: seeded random-init weights of the real shape; seeded encoder-output stand-in "
                "(stable rows per completed 8 s window, re-drawn partial tail, 4-window eviction)",
        "config": c4_config(world, n_local),
        "x_realtime": round(audio_s / (dev_ms / 1e3), 1),
        "prefill_ms": round(pre_ms / args.steps, 3), "decode_ms": round(dec_ms / args.steps, 3),
        "prefill_rows_per_step": round(rows / args.steps, 1),
        "prefill_tflops": round(pre_tflops, 1) if pre_tflops else None,
        "e2e": {"value": round(toks / (wall_ms / 1e3), 2), "unit": "tok/s",
                "h2d_bytes_per_step": int(sum(r["h2d"] for r in rec) / args.steps),
                "d2h_bytes_per_step": int(4 * max_new * n_local),
                "x_realtime": round(audio_s / (wall_ms / 1e3), 1),
                "path": "qdb_streams_chunk with host encoder rows (memcmp prefix reuse, staging, upload, "
                        "batched prefill, greedy loop, token bookkeeping)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "kernel": "rows_decode",
                     "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "bytes_per_launch": int(bytes_step)},
        # prefill: 9 kernels per layer + prompt rows; greedy step: 9 per layer, +1 (the split
        # merge) when a row holds more than 512 keys, + embedding, final norm, lm_head, argmax, counter
        "gpu_launches": int(sum(cfg.layers * 9 + 1 + max_new * (cfg.layers * (9 + (r["ctx_max"] > 512)) + 5)
                                for r in rec)),
        "clocks": clk, "setup_s": round(setup_s, 1),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = stream_cpu_sample(synth, ws, budget_s=20.0)
    S.close()
    model.close()
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def stream_cpu_sample(synth, ws, budget_s=20.0, warm_chunks=0):
    """The reference's streaming decoder side on the host: stream_impl's policy
    (oracle/stream_oracle.py) over the reference's own decoder (oracle/_ref),
    one stream (seed 1000) chunk by chunk from its start until budget_s of
    chunk time has passed."""
    from oracle.pyoracle import RefDecoder
    from oracle import stream_oracle as so
    cfg = ws.cfg
    th = ref_threads()
    d = RefDecoder(ws, threads=th)

    class Adapter:
        def prefill(self, e, start):
            d.kv_cache_len = start
            d.prefill(e)

        def forward(self, row, pos):
            d.kv_cache_len = pos
            tok, _, _ = d.forward(row, mask_eos=True, want_logits=False)
            return tok, None

    emb = lambda t: synth.bf16_to_f32(ws.embed[t]).astype(np.float32)
    o = so.StreamOracle(Adapter(), emb, max_new_tokens=CONFIGS["c4"][2], past_text=True,
                        head=[t % cfg.vocab for t in synth.PROMPT_PREFIX[:3]],
                        tail=[t % cfg.vocab for t in synth.PROMPT_PREFIX[3:]],
                        suffix=[t % cfg.vocab for t in synth.PROMPT_SUFFIX])
    bank = np.random.default_rng(4242).standard_normal((16384, cfg.hidden), dtype=np.float32)
    enc = stream_encoders(synth, cfg, [1000], bank)[0]
    spent, chunks, toks = 0.0, 0, 0
    while spent < budget_s:
        a, fin = enc.advance(CONFIGS["c4"][1])
        if a is None:
            break
        t0 = time.perf_counter()
        _, rs = o.chunk(a, fin)
        spent += time.perf_counter() - t0
        chunks += 1
        toks += o.last.get("generated", 0)
        if rs:
            enc.clear()
    d.close()
    return {"value": round(toks / spent, 3), "unit": "tok/s", "cores": th, "kind": "reference",
            "x_realtime": round(chunks * C4_CHUNK_S / spent, 3),
            "sample": f"one stream (seed 1000) from its start, {chunks} chunks of 2 s ({spent:.1f} s): the "
                      f"reference's decoder (oracle/_ref) driven by a restatement of stream_impl's decoder-side "
                      f"policy, prefill reuse as the reference; value = generated tokens / chunk wall time"}


def run_streams_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    synth = load_synth_standalone()
    cfg = synth.PRESETS[CONFIGS["c4"][0]]
    ws = synth.WeightSet(cfg, seed=0)
    budget = max(10.0, 2.0 * args.steps)
    cb = stream_cpu_sample(synth, ws, budget_s=budget)
    n_local = -(-CONFIGS["c4"][3] // world)
    res = {"impl": "reference", "metric": C4_METRIC, "value": cb["value"], "unit": "tok/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "f32 activations x bf16 weights (reference CPU path)",
           "data": "synthetic: seeded random-init weights of the real shape; seeded encoder-output stand-in",
           "config": c4_config(world, n_local), "x_realtime": cb["x_realtime"],
           "cpu_baseline": cb,
           "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


def ref_threads():
    return max(1, min(os.cpu_count() or 1, 16))


class RefSampler:
    """The reference's own CPU decoder (oracle/_ref) on one utterance of the
    config. Set-up (untimed): prefill, then the full greedy decode, which
    fills the KV cache over the whole decode range and records the tokens.
    A sample then re-decodes REF_WINDOWS windows of `per_window` tokens spread
    evenly over that range (kv_cache_len rewound to each window's start, fed
    the token the full decode produced there), so every timed token repeats a
    step of the real run at its real context length."""

    def __init__(self, synth, ws, emb, n_dec, threads):
        from oracle.pyoracle import Oracle, RefDecoder
        try:
            self.ref = RefDecoder(ws, threads=threads)
            self.kind = "reference"
        except (FileNotFoundError, OSError):
            self.ref = Oracle(ws, max_pos=emb.shape[0] + n_dec + 8, threads=threads)
            self.kind = "port"
        self.ws, self.n_dec = ws, n_dec
        self.P = emb.shape[0] - 1
        t0 = time.perf_counter()
        self.ref.prefill(emb[:-1])
        self.prefill_s = time.perf_counter() - t0
        self.first = int(synth.PROMPT_SUFFIX[-1])
        t0 = time.perf_counter()
        self.tokens = self._decode(self.first, n_dec)
        self.full_decode_s = time.perf_counter() - t0

    def _decode(self, first, n):
        if self.kind == "reference":
            out, _ = self.ref.decode_loop(first, n, mask_eos=True)
            return [int(t) for t in out]
        out, tok = [], first
        for _ in range(n):
            x = (self.ws.embed[tok].astype(np.uint32) << 16).view(np.float32)
            tok, _, _ = self.ref.forward(x, mask_eos=True, want_logits=False)
            out.append(int(tok))
        return out

    def sample(self, per_window):
        """Seconds for REF_WINDOWS x per_window decode tokens."""
        total = 0.0
        for w in range(REF_WINDOWS):
            start = (w * self.n_dec) // REF_WINDOWS
            self.ref.kv_cache_len = self.P + start
            first = self.first if start == 0 else self.tokens[start - 1]
            if self.kind == "reference":
                _, ms = self.ref.decode_loop(first, per_window, mask_eos=True)
                total += ms / 1e3
            else:
                t0 = time.perf_counter()
                self._decode(first, per_window)
                total += time.perf_counter() - t0
        return total

    def describe(self, steps, per_window):
        return (f"one utterance (prefill {self.P} positions, {self.prefill_s:.2f} s, then the full {self.n_dec}-token "
                f"greedy decode untimed); each step re-decodes {REF_WINDOWS} windows x {per_window} tokens spread "
                f"evenly over decode positions {self.P}..{self.P + self.n_dec - 1}; {steps} steps timed")

    def close(self):
        self.ref.close()


def cpu_baseline(synth, ws, emb, cfg_name, steps=2, per_window=3):
    """Reference CPU decoder on this host: a bounded sample of the config."""
    th = ref_threads()
    n_dec = CONFIGS[cfg_name][2]
    rs = RefSampler(synth, ws, emb, n_dec, th)
    secs = sum(rs.sample(per_window) for _ in range(steps))
    value = steps * REF_WINDOWS * per_window / secs
    out = {"value": round(value, 3), "unit": "tok/s", "cores": th, "kind": rs.kind,
           "sample": rs.describe(steps, per_window) + "; value = timed tokens / their decode wall time "
                                                      "(one utterance at a time, the reference's mode)",
           "prefill_s": round(rs.prefill_s, 3), "host_nproc": os.cpu_count()}
    rs.close()
    return out


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    synth = load_synth_standalone()
    preset, seconds, n_dec, n_utt = CONFIGS[args.config]
    cfg = synth.PRESETS[preset]
    ws = synth.WeightSet(cfg, seed=0)
    # same per-GPU block as the GPU arm's rank 0 at this world size
    n_local = -(-n_utt // world) if n_utt > 1 else 1
    emb = synth.utterance(ws, seconds, utterance_seed(args.config, 0))
    th = ref_threads()
    per_window = 3
    rs = RefSampler(synth, ws, emb, n_dec, th)
    for _ in range(args.warmup):
        rs.sample(per_window)
    times = [rs.sample(per_window) for _ in range(args.steps)]
    dec_s = sum(times)
    value = args.steps * REF_WINDOWS * per_window / dec_s
    res = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dec_s / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if n_utt > 1 else "weak",
        "vs_baseline": None, "dtype": "f32 activations x bf16 weights (reference CPU path)",
        "data": "synthetic: seeded random-init weights of the real shape, seeded prompt embeddings",
        "config": config_block(args.config, world, n_local, rs.P),
        "prefill_ms": round(rs.prefill_s * 1e3, 1),
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": th, "kind": rs.kind,
                         "sample": rs.describe(args.steps, per_window)},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    rs.close()
    print(json.dumps(res), flush=True)


def profile_step(args):
    """Small fixed case for ncu captures of the decode step: the config's
    model, a prefill of the config's prompt, then 3 device greedy steps."""
    import __graft_entry__ as ge
    pkg = ge.load_package()
    synth = ge.load_synth()
    preset, seconds, n_dec, n_utt = CONFIGS[args.config]
    ws = synth.WeightSet(synth.PRESETS[preset], seed=0)
    emb = synth.utterance(ws, seconds, 1)
    P = emb.shape[0] - 1
    model = pkg.Model(ws, device=0, mask_eos=True)
    s = model.session(P + 8)
    s.prefill(emb[:-1], 0)
    print(list(s.decode_greedy(synth.PROMPT_SUFFIX[-1], P, 3)))


def profile_batch(args):
    """Fixed case for ncu captures of the batched decode kernels: 64 sessions
    of the 0.6B synthetic model, a 270-position batched prefill, then three
    forward_batch steps; the third (a replay of the cached step graph) runs
    inside the NVTX range "decode" (ncu --nvtx --nvtx-include "decode/")."""
    import torch
    import __graft_entry__ as ge
    pkg = ge.load_package()
    synth = ge.load_synth()
    cfg = synth.PRESETS["0.6b"]
    ws = synth.WeightSet(cfg, seed=0)
    B, P = 64, 270
    model = pkg.Model(ws, device=0, mask_eos=True)
    sess = [model.session(P + 16) for _ in range(B)]
    emb = synth.audio_embeddings(cfg, P, seed=1)
    pkg.prefill_batch(sess, np.tile(emb, (B, 1)), [0] * B, lens=[P] * B)
    x = np.tile(emb[:1], (B, 1))
    for i in range(3):
        torch.cuda.synchronize()
        if i == 2:
            torch.cuda.nvtx.range_push("decode")
        toks = pkg.forward_batch(sess, x, np.full(B, P + i, np.int32))
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(toks[:4].tolist())


def profile_encoder(args):
    """Fixed case for ncu captures of the audio front end: log-mel and encoder
    of one 30 s 0.6B utterance (seeded PCM), run twice, the second time inside
    the NVTX range "frontend" (ncu --nvtx --nvtx-include "frontend/")."""
    import torch
    import __graft_entry__ as ge
    pkg = ge.load_package()
    synth = ge.load_synth()
    ews = synth.EncoderWeightSet(synth.ENC_PRESETS["0.6b"], seed=0)
    enc = pkg.Encoder(ews)
    x = torch.from_numpy(synth.bench_pcm(30.0, 1)).cuda()
    f = pkg.mel_frames(x.numel())
    mel = torch.empty(128 * f, device="cuda")
    out = torch.empty((pkg.Encoder.tokens(f), ews.cfg.output_dim), device="cuda")
    es = torch.cuda.ExternalStream(enc.stream_handle)
    for i in range(2):
        torch.cuda.synchronize()
        if i == 1:
            torch.cuda.nvtx.range_push("frontend")
        pkg.mel_spectrogram_device(x.data_ptr(), x.numel(), mel.data_ptr(), enc.stream_handle)
        enc.forward_device(mel.data_ptr(), f, out.data_ptr())
        es.synchronize()
    torch.cuda.nvtx.range_pop()
    print(out.shape, float(out.abs().max()))
    enc.close()


def profile_prefill(args):
    """Fixed case for ncu captures of the prefill kernels: one 2048-position
    prefill of the 1.7B synthetic model (seeded rows), run twice, the second
    time inside the NVTX range "prefill" (ncu --nvtx --nvtx-include "prefill/")."""
    import torch
    import __graft_entry__ as ge
    pkg = ge.load_package()
    synth = ge.load_synth()
    cfg = synth.PRESETS["1.7b"]
    ws = synth.WeightSet(cfg, seed=0)
    model = pkg.Model(ws, device=0, mask_eos=True)
    s = model.session(2048 + 8)
    emb = torch.from_numpy(synth.audio_embeddings(cfg, 2048, seed=1)).cuda()
    for i in range(2):
        torch.cuda.synchronize()
        if i == 1:
            torch.cuda.nvtx.range_push("prefill")
        s.prefill_device(emb.data_ptr(), 2048, 0)
        model.sync()
    torch.cuda.nvtx.range_pop()
    s.close()
    model.close()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-b1", action="store_true", help="skip the in-line batch-1 (c0, c1) measurements")
    ap.add_argument("--no-pipeline", action="store_true", help="skip the audio -> tokens pipeline measurement")
    ap.add_argument("--profile-step", action="store_true", help="small fixed case for ncu (no timing)")
    ap.add_argument("--profile-batch", action="store_true", help="batched-decode case for ncu (no timing)")
    ap.add_argument("--profile-encoder", action="store_true", help="mel + encoder case for ncu (no timing)")
    ap.add_argument("--profile-prefill", action="store_true", help="1.7B 2048-position prefill for ncu (no timing)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "0"))
    if args.gpus > 1 and world == 0:
        # --gpus N without a launcher: start one rank per GPU on this node
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={args.gpus}",
               "--master-addr=127.0.0.1", f"--master-port={free_port()}", os.path.abspath(__file__)] + sys.argv[1:]
        sys.exit(subprocess.call(cmd))
    if world and world != args.gpus:
        print(f"bench.py: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE", file=sys.stderr)
    if args.profile_batch:
        profile_batch(args)
        return
    if args.profile_encoder:
        profile_encoder(args)
        return
    if args.profile_prefill:
        profile_prefill(args)
        return
    if args.profile_step:
        profile_step(args)
    elif args.impl == "reference":
        run_streams_reference(args) if args.config == "c4" else run_reference(args)
    else:
        run_streams_ours(args) if args.config == "c4" else run_ours(args)


if __name__ == "__main__":
    main()
