"""Benchmark of the B200 decoder hot path (qwen-asr decoder token loop + prefill).

Metric: decode tok/s per GPU as a fraction of the HBM roofline, plus
end-to-end x-realtime of the decoder stage. Default workload = config c1
(1.7B-shaped, batch 1, 30 s utterance -> 404-position prefill, 256 greedy
tokens with EOS masked); --config c0 / c2 / c3 select the 0.6B batch-1, the
0.6B 64-utterance and the 1.7B long-context (300 s) configurations.

One timed step = one utterance per rank (c2: this rank's shard of the 64
utterances): prefill over the prompt embeddings followed by the greedy decode
loop. `value` = decoded tokens / decode time, inputs resident in HBM (device
embedding lookup, device greedy loop). `e2e` = the same metric through the
reference-facing C ABI with host buffers: host f32 prompt embeddings (pinned),
one host embedding in and one token out per decode step, exactly the
qwen_asr.c:729-759 caller loop.

Weights and inputs are seeded synthetic data of the real shapes (no
checkpoints offline). Weights (1.2 / 3.4 GB) exceed the 126 MB L2, so every
step streams them from HBM; no flush is needed.

--impl reference times the reference's own CPU decoder (oracle/_ref, built
from the reference sources) on this host, bounded samples of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
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
}
KV_BYTES_PER_POS = 28 * 8 * 128 * 2 * 2  # bf16 K and V per cached position (all layers)


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


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


def build_inputs(synth, ws, cfg_name, rank, n_local, first_utt):
    preset, seconds, steps, n_utt = CONFIGS[cfg_name]
    embs = []
    for u in range(first_utt, first_utt + n_local):
        seed = 1 if n_utt == 1 else 100 + u
        embs.append(synth.utterance(ws, seconds, seed))
    return embs


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

    preset, seconds, n_dec, n_utt = CONFIGS[args.config]
    cfg = synth.PRESETS[preset]
    if n_utt > 1:
        import importlib
        shard = importlib.import_module("qwen_asr_b200.shard")
        first, n_local = shard.shard_range(n_utt, world, rank)
        scaling = "strong"
    else:
        n_local, first = 1, 0
        scaling = "weak"  # batch-1 configs run one replica per GPU
    t0 = time.time()
    ws = synth.WeightSet(cfg, seed=0)
    embs = build_inputs(synth, ws, args.config, rank, n_local, first)
    P = embs[0].shape[0] - 1  # prefill length; the last prompt position is token 198
    last_tok = synth.PROMPT_SUFFIX[-1]
    model = pkg.Model(ws, device=local, mask_eos=True)
    gen_s = time.time() - t0
    stream = torch.cuda.ExternalStream(model.stream_handle, device=torch.device("cuda", local))
    cap = P + n_dec + 8
    sessions = [model.session(cap) for _ in range(n_local)]
    emb_dev = [torch.from_numpy(e[:-1]).to(f"cuda:{local}") for e in embs]
    torch.cuda.synchronize()

    def one_step(timing):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(stream)
        for s, e in zip(sessions, emb_dev):
            s.prefill_device(e.data_ptr(), P, 0)
        ev[1].record(stream)
        if n_local == 1:
            toks = sessions[0].decode_greedy(last_tok, P, n_dec)
        else:
            toks = pkg.decode_greedy_batch(sessions, [last_tok] * n_local, [P] * n_local, n_dec)
        ev[2].record(stream)
        timing.append(ev)
        return toks

    for _ in range(args.warmup):
        one_step([])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    timing = []
    t_wall = time.time()
    for _ in range(args.steps):
        one_step(timing)
    torch.cuda.synchronize()
    wall = time.time() - t_wall
    clk = clocks.stop()
    pre_ms = sum(e[0].elapsed_time(e[1]) for e in timing)
    dec_ms = sum(e[1].elapsed_time(e[2]) for e in timing)
    tot_ms = sum(e[0].elapsed_time(e[2]) for e in timing)

    # e2e through the reference-facing ABI with host buffers (pinned inputs)
    pinned = [torch.from_numpy(e).pin_memory() for e in embs]
    emb_tab = ws.embed  # host bf16 table, the caller's mmap
    e2e_ev = []

    def e2e_step():
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(stream)
        toks_all = []
        for s, e in zip(sessions, pinned):
            s.prefill(e.numpy()[:-1], 0)
        ev[1].record(stream)
        if n_local == 1:
            s = sessions[0]
            x = pinned[0].numpy()[-1]
            out = []
            for i in range(n_dec):
                t, _, _ = s.forward(x, P + i)
                out.append(t)
                x = synth.bf16_to_f32(emb_tab[t])
            toks_all.append(out)
        else:
            x = np.stack([p.numpy()[-1] for p in pinned])
            for i in range(n_dec):
                t = pkg.forward_batch(sessions, x, [P + i] * n_local)
                x = synth.bf16_to_f32(emb_tab[t])
        ev[2].record(stream)
        e2e_ev.append(ev)

    e2e_step()  # warm
    e2e_ev.clear()
    n_e2e = max(1, min(args.steps, 3))
    for _ in range(n_e2e):
        e2e_step()
    torch.cuda.synchronize()
    e2e_dec_ms = sum(e[1].elapsed_time(e[2]) for e in e2e_ev)
    e2e_tot_ms = sum(e[0].elapsed_time(e[2]) for e in e2e_ev)

    # max over ranks
    import importlib
    shard = importlib.import_module("qwen_asr_b200.shard")
    dec_ms, pre_ms, tot_ms, e2e_dec_ms, e2e_tot_ms = shard.max_over_ranks(
        [dec_ms, pre_ms, tot_ms, e2e_dec_ms, e2e_tot_ms], device=f"cuda:{local}")

    tokens_total = args.steps * n_dec * (n_utt if n_utt > 1 else world)
    value = tokens_total / (dec_ms / 1e3)
    e2e_value = (n_e2e * n_dec * (n_utt if n_utt > 1 else world)) / (e2e_dec_ms / 1e3)
    # roofline of the dominant kernel (the persistent decode step at b=1; the
    # batched decode step for c2): algorithmic bytes per launch / launch time
    h, L, V, I = cfg.hidden, cfg.layers, cfg.vocab, cfg.intermediate
    qd, kvd = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    w_bytes = 2 * (L * ((qd + 2 * kvd) * h + h * qd + 2 * I * h + h * I) + V * h)
    ctx_avg = P + (n_dec + 1) / 2.0
    bytes_per_step = w_bytes + n_local * KV_BYTES_PER_POS * ctx_avg
    launch_s = (dec_ms / 1e3) / (args.steps * n_dec)
    achieved = bytes_per_step / launch_s / 1e9
    peak, peak_kind = measured_peaks()
    kernel = "step_kernel" if n_local == 1 else "rows_decode"
    traffic = step_traffic_from_profile(kernel, args.config)
    # per prefill, per layer: 2 norms, 4 GEMMs, q/k RoPE + KV append, attention, bf16 split of the
    # SwiGLU output; per batched decode step: embed, 10 per layer (2 norms, 4 GEMMs, RoPE/append,
    # attention units, split merge, SwiGLU split), final norm, lm_head GEMM, argmax, step advance;
    # b=1 decode: one persistent step kernel per token
    launches_per_step = (L * 9) * n_local + (n_dec if n_local == 1 else n_dec * (L * 10 + 5))
    h2d = sum(e.numel() * 4 for e in pinned) - n_local * h * 4 + n_dec * n_local * h * 4
    d2h = n_dec * n_local * 4
    result = {
        "metric": "decode tok/s/GPU (b=1, b=64) as % of HBM; end-to-end x-realtime",
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(tot_ms / args.steps, 3),
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": "bf16 weights x f32 activations (f32 accumulate), fp16 KV cache",
        "data": "synthetic: seeded random-init weights of the real shape, seeded prompt embeddings",
        "config": {"workload": f"{args.config}: {preset} decoder, {n_utt} utterance(s) of {seconds:g} s "
                               f"-> prefill {P} positions + {n_dec} greedy tokens (EOS masked)",
                   "global_batch": n_utt, "per_gpu_batch": n_local, "prefill_len": P, "decode_tokens": n_dec,
                   "parallelism": f"dp{world} (independent utterances, no collective)" if world > 1 else "single GPU",
                   "l2": "weights (> 1 GB) exceed the 126 MB L2; no flush needed"},
        "prefill_ms": round(pre_ms / args.steps, 3),
        "decode_ms": round(dec_ms / args.steps, 3),
        "decoder_x_realtime": round(seconds * n_local * args.steps / (tot_ms / 1e3), 2),
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h),
                "decoder_x_realtime": round(seconds * n_local * n_e2e / (e2e_tot_ms / 1e3), 2),
                "path": "qdb_prefill + qdb_forward/qdb_forward_batch with host buffers"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": kernel, "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "bytes_per_launch": int(bytes_per_step)},
        "gpu_launches": int(launches_per_step * args.steps),
        "clocks": clk,
        "wall_s": round(wall, 3),
        "setup_s": round(gen_s, 1),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(ws, embs[0], n_dec, args.config)
    if rank == 0:
        print(json.dumps(result), flush=True)
    for s in sessions:
        s.close()
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def ref_threads():
    return max(1, min(os.cpu_count() or 1, 16))


def cpu_baseline(ws, emb, n_dec, cfg_name, sample_tokens=24):
    """Reference CPU decoder on this host: prefill + a bounded decode sample."""
    from oracle.pyoracle import RefDecoder, Oracle
    th = ref_threads()
    try:
        ref = RefDecoder(ws, threads=th)
        kind = "reference"
    except (FileNotFoundError, OSError):
        ref = Oracle(ws, max_pos=emb.shape[0] + sample_tokens + 8, threads=th)
        kind = "port"
    P = emb.shape[0] - 1
    t0 = time.perf_counter()
    ref.prefill(emb[:-1])
    pre_s = time.perf_counter() - t0
    if kind == "reference":
        _, ms = ref.decode_loop(198, sample_tokens, mask_eos=True)
        dec_s = ms / 1e3
    else:
        t0 = time.perf_counter()
        x = emb[-1]
        for _ in range(sample_tokens):
            t, _, _ = ref.forward(x, mask_eos=True, want_logits=False)
            x = (ws.embed[t].astype(np.uint32) << 16).view(np.float32)
        dec_s = time.perf_counter() - t0
    ref.close()
    return {"value": round(sample_tokens / dec_s, 3), "unit": "tok/s", "cores": th, "kind": kind,
            "sample": f"{cfg_name}: prefill {P} positions ({pre_s:.2f} s) then {sample_tokens} greedy decode "
                      f"tokens from position {P}; value = decode tokens / decode wall time",
            "prefill_s": round(pre_s, 3), "host_nproc": os.cpu_count()}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    import __graft_entry__ as ge
    synth = ge.load_synth()
    from oracle.pyoracle import RefDecoder, Oracle
    preset, seconds, n_dec, n_utt = CONFIGS[args.config]
    cfg = synth.PRESETS[preset]
    ws = synth.WeightSet(cfg, seed=0)
    emb = synth.utterance(ws, seconds, 1 if n_utt == 1 else 100)
    th = ref_threads()
    try:
        ref = RefDecoder(ws, threads=th)
        kind = "reference"
    except (FileNotFoundError, OSError) as ex:
        ref = Oracle(ws, max_pos=emb.shape[0] + 4096, threads=th)
        kind = "port"
    P = emb.shape[0] - 1
    t0 = time.perf_counter()
    ref.prefill(emb[:-1])
    pre_s = time.perf_counter() - t0
    per_step = 8  # decode tokens per timed step (bounded sample)
    tok = 198
    pos = P

    def step():
        nonlocal tok, pos
        if kind == "reference":
            ref.kv_cache_len = pos
            out, ms = ref.decode_loop(tok, per_step, mask_eos=True)
            return ms / 1e3
        t0 = time.perf_counter()
        x = (ws.embed[tok].astype(np.uint32) << 16).view(np.float32)
        for _ in range(per_step):
            t, _, _ = ref.forward(x, mask_eos=True, want_logits=False)
            x = (ws.embed[t].astype(np.uint32) << 16).view(np.float32)
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        step()
    times = [step() for _ in range(args.steps)]
    dec_s = sum(times)
    value = args.steps * per_step / dec_s
    res = {
        "impl": "reference",
        "metric": "decode tok/s/GPU (b=1, b=64) as % of HBM; end-to-end x-realtime",
        "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dec_s / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 activations x bf16 weights (reference CPU path)",
        "data": "synthetic: seeded random-init weights of the real shape, seeded prompt embeddings",
        "config": {"workload": f"{args.config}: {preset} decoder, reference CPU path, each step = {per_step} "
                               f"greedy decode tokens continuing after a {P}-position prefill",
                   "global_batch": 1, "prefill_len": P},
        "prefill_ms": round(pre_s * 1e3, 1),
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": th, "kind": kind,
                         "sample": f"{args.steps} steps x {per_step} tokens after a {P}-position prefill"},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    ref.close()
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
    of the 0.6B synthetic model, a 270-position prefill each, then one
    forward_batch step inside the NVTX range "decode" (ncu --nvtx
    --nvtx-include "decode/")."""
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
    for s in sess:
        s.prefill(emb, 0)
    pos = np.full(B, P, np.int32)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("decode")
    toks = pkg.forward_batch(sess, np.tile(emb[:1], (B, 1)), pos)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(toks[:4].tolist())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c1", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-step", action="store_true", help="small fixed case for ncu (no timing)")
    ap.add_argument("--profile-batch", action="store_true", help="batched-decode case for ncu (no timing)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_batch:
        profile_batch(args)
        return
    if args.profile_step:
        profile_step(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
