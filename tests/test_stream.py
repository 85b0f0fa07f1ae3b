"""Streaming scheduler (qdb_streams_*, qdb_stream.cu) against the per-stream
restatement of the reference's stream_impl (oracle/stream_oracle.py).

CPU: the restatement driven by the reference's own decoder (oracle/_ref):
  - stream-cache equivalence, the property the reference's regression harness
    checks (asr_regression.py stream-cache-check): prefill-KV reuse must give the
    same tokens as re-prefilling every prompt from scratch;
  - the policy rules on scripted token streams (repeat-run suppression,
    degeneration reset, stagnation reset, periodic re-anchor, overlap de-dup).
GPU: many streams batched through qdb_streams_chunk against the restatement
run stream by stream over the b=1 C-ABI path (qdb_prefill / qdb_forward, the
drop-in for qwen_decoder_prefill / _forward) and over the reference decoder:
identical raw / emitted token ids and prefix-reuse counts per chunk. A
decision whose top-2 logit margin is below 1e-3 may flip between the batched
and b=1 arithmetic; such cases are reported, not failed.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)

import __graft_entry__ as ge  # noqa: E402
from oracle import stream_oracle as so  # noqa: E402

synth = ge.load_synth()
CFG = synth.PRESETS["tiny"]
V = CFG.vocab


def template():
    return dict(head=[t % V for t in so.HEAD], tail=[t % V for t in so.TAIL], suffix=[t % V for t in so.SUFFIX],
                asr_text_token=so.TOKEN_ASR_TEXT % V)


@pytest.fixture(scope="module")
def ws():
    return synth.WeightSet(CFG, seed=0, norm_jitter=0.1)


def embed_fn(ws):
    return lambda t: synth.bf16_to_f32(ws.embed[t]).astype(np.float32)


class RefAdapter:
    """reference decoder (oracle/_ref) with explicit positions"""

    def __init__(self, ws):
        from oracle.pyoracle import RefDecoder
        self.d = RefDecoder(ws)

    def prefill(self, e, start):
        self.d.kv_cache_len = start
        self.d.prefill(e)

    def forward(self, row, pos):
        self.d.kv_cache_len = pos
        tok, _, log = self.d.forward(row, mask_eos=True, want_logits=True)
        return tok, log


class NoReuse:
    """wraps an oracle so every chunk re-prefills its whole prompt"""

    def __init__(self, o):
        self.o = o

    def chunk(self, audio, fin):
        self.o.prev = None
        return self.o.chunk(audio, fin)


def run_streams(oracles, encoders, total_s):
    """chunk loop over several oracle streams; returns per-chunk (emit, reset) lists"""
    log = [[] for _ in oracles]
    done = [False] * len(oracles)
    while not all(done):
        for i, (o, e) in enumerate(zip(oracles, encoders)):
            if done[i]:
                continue
            audio, fin = e.advance(total_s[i])
            if audio is None:
                done[i] = True
                continue
            ne, rs = o.chunk(audio, fin)
            if rs:
                e.clear()
            log[i].append((ne, rs, dict(getattr(o, "last", {}) or getattr(o, "o", o).last)))
            done[i] = fin
    return log


def ref_available():
    from oracle.pyoracle import ref_so_path
    return ref_so_path() is not None


# --------------------------------------------------------------------- CPU
@pytest.mark.parametrize("past_text", [False, True])
def test_stream_cache_equivalence_reference_decoder(ws, past_text):
    if not ref_available():
        pytest.skip("oracle/_ref not built")
    total = 14.0  # 7 chunks, one window eviction boundary crossed at 8 s
    a = so.StreamOracle(RefAdapter(ws), embed_fn(ws), max_new_tokens=8, past_text=past_text, **template())
    b = so.StreamOracle(RefAdapter(ws), embed_fn(ws), max_new_tokens=8, past_text=past_text, **template())
    run_streams([a], [synth.SyntheticEncoder(CFG.hidden, 7, window_s=4.0, max_windows=2)], [total])
    run_streams([NoReuse(b)], [synth.SyntheticEncoder(CFG.hidden, 7, window_s=4.0, max_windows=2)], [total])
    assert a.prefill_reused > 0 and b.prefill_reused == 0
    assert a.raw == b.raw and a.emitted == b.emitted, (a.min_margin, b.min_margin)
    assert a.emitted, "nothing committed"


class Scripted:
    """decoder whose forward returns a scripted token sequence per chunk, then
    an end token"""

    def __init__(self, script):
        self.script, self.chunk, self.i = script, -1, 0

    def prefill(self, e, start):
        pass

    def forward(self, row, pos):
        seq = self.script[self.chunk]
        t = seq[self.i] if self.i < len(seq) else so.TOKEN_IM_END  # the script ends with an end token
        self.i += 1
        return t, None


def scripted_oracle(chunks, **kw):
    dec = Scripted(chunks)
    o = so.StreamOracle(dec, lambda t: np.full(4, t, np.float32), head=[1], tail=[2], suffix=[3],
                        asr_text_token=9, **kw)
    out = []
    for k in range(len(chunks)):
        dec.chunk, dec.i = k, 0
        out.append(o.chunk(np.full((2, 4), 0.5 + k, np.float32), k == len(chunks) - 1))
    return o, out


def test_policy_commit_frontier_and_final_flush():
    # <asr_text>=9 then text; chunks 0-1 are cold (nothing fixed), rollback 5 holds the tail back
    text = [9] + list(range(100, 140))
    o, out = scripted_oracle([text[:12], text[:20], text[:30], text[:41]], max_new_tokens=64)
    assert [e for e, _ in out[:2]] == [0, 0]
    assert out[2] == (30 - 1 - 5, 0)
    assert o.emitted == text[1:]  # the final chunk emits the rest


def test_policy_repeat_run_suppression_and_recovery():
    # 20 copies of one token: 12 kept, 8 dropped -> recovery reset
    o, out = scripted_oracle([[9] + [50] * 20 + [51]], max_new_tokens=32)
    assert out[0][1] == 1
    assert o.raw == [9]  # re-anchored on nothing emitted


def test_policy_degeneration_period_reset():
    # a period-3 block repeated 4 times at the candidate tail triggers a reset
    o, out = scripted_oracle([[9, 1, 2], [9, 1, 2, 3] + [60, 61, 62] * 4 + [7, 7, 7, 7, 7]], max_new_tokens=64)
    assert out[1][1] == 1


def test_policy_periodic_reanchor_with_past_text():
    chunks = [[9] + list(range(200, 200 + 3 + k)) for k in range(46)]
    o, out = scripted_oracle(chunks, max_new_tokens=64, past_text=True)
    resets = [k for k, (_, r) in enumerate(out) if r == 2]
    assert resets == [44]
    assert len(o.raw) >= 1 and o.raw[0] == 9


def test_synthetic_encoder_window_cache():
    e = synth.SyntheticEncoder(16, 3, window_s=8.0, max_windows=4)
    rows = []
    for k in range(25):
        a, fin = e.advance(50.0)
        rows.append(a)
    assert synth.SyntheticEncoder.rows_for(8.0) == 104 and synth.SyntheticEncoder.rows_for(2.0) == 26
    assert len(rows[3]) == 104  # 8 s: one completed window, no tail
    assert np.array_equal(rows[4][:104], rows[3][:104])  # completed window rows are stable
    assert len(rows[-1]) <= 4 * 104 + 26  # at most 4 windows plus the tail
    assert fin


# --------------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def pkg():
    p = ge.load_package()
    if p.device_count() < 1:
        pytest.skip("no CUDA device")
    return p


class AbiAdapter:
    """b=1 C-ABI path (qdb_prefill / qdb_forward)"""

    def __init__(self, model):
        self.s = model.session(256)

    def prefill(self, e, start):
        self.s.prefill(e, start)

    def forward(self, row, pos):
        tok, _, log = self.s.forward(row, pos, want_logits=True)
        return tok, log


def compare(pkg, ws, n, total_s, past_text, oracle_of, max_new=12, window_s=4.0):
    model = pkg.Model(ws, device=0, mask_eos=True)
    S = pkg.Streams(model, n, max_new_tokens=max_new, past_text=past_text, **template())
    enc_g = [synth.SyntheticEncoder(CFG.hidden, 50 + i, window_s=window_s, max_windows=2) for i in range(n)]
    enc_o = [synth.SyntheticEncoder(CFG.hidden, 50 + i, window_s=window_s, max_windows=2) for i in range(n)]
    orc = [so.StreamOracle(oracle_of(model), embed_fn(ws), max_new_tokens=max_new, past_text=past_text,
                           **template()) for _ in range(n)]
    flips = []
    active = [True] * n
    k = 0
    while any(active):
        audio, fins = [], []
        for i in range(n):
            a, fin = enc_g[i].advance(total_s[i]) if active[i] else (None, True)
            audio.append(a)
            fins.append(fin)
        ne, rs = S.chunk(audio, fins)
        for i in range(n):
            if audio[i] is None:
                active[i] = False
                continue
            a2, _ = enc_o[i].advance(total_s[i])
            ne2, rs2 = orc[i].chunk(a2, fins[i])
            st = S.stats(i)
            same = (list(S.tokens(i, "raw")) == orc[i].raw and list(S.tokens(i, "emitted")) == orc[i].emitted
                    and (ne[i], rs[i]) == (ne2, rs2) and st["last_reused"] == orc[i].last["reused"]
                    and st["last_prefill_len"] == orc[i].last["prefill_len"])
            if not same:
                flips.append((i, k, orc[i].min_margin))
                assert orc[i].min_margin < 1e-3, f"stream {i} chunk {k}: scheduler differs from the oracle"
                active[i] = False  # past a near-tie flip the streams legitimately diverge
                continue
            if rs[i]:
                enc_g[i].clear()
                enc_o[i].clear()
            if fins[i]:
                active[i] = False
        k += 1
    reused = sum(S.stats(i)["prefill_reused"] for i in range(n))
    S.close()
    model.close()
    return flips, reused


@pytest.mark.gpu
@pytest.mark.parametrize("past_text", [False, True])
def test_streams_match_oracle_over_b1_path(pkg, ws, past_text):
    n = 6
    total = [10.0, 14.0, 6.0, 12.0, 9.0, 16.0]
    flips, reused = compare(pkg, ws, n, total, past_text, lambda m: AbiAdapter(m))
    assert reused > 0
    assert len(flips) <= 1, flips


@pytest.mark.gpu
def test_streams_match_reference_decoder(pkg, ws):
    if not ref_available():
        pytest.skip("oracle/_ref not built")
    flips, reused = compare(pkg, ws, 2, [10.0, 12.0], True, lambda m: RefAdapter(ws))
    assert reused > 0
    assert not flips or all(f[2] < 1e-3 for f in flips)


@pytest.mark.gpu
def test_streams_skip_chunk_and_config_errors(pkg, ws):
    model = pkg.Model(ws, device=0, mask_eos=True)
    S = pkg.Streams(model, 2, max_new_tokens=4, **template())
    e = synth.SyntheticEncoder(CFG.hidden, 1)
    a, _ = e.advance(4.0)
    empty = np.zeros((0, CFG.hidden), np.float32)
    ne, rs = S.chunk([a, empty], [False, False])  # stream 1 has no encoder output: the chunk is skipped
    assert S.stats(1)["chunk_idx"] == 1 and S.stats(1)["chunks"] == 0
    assert S.stats(0)["chunks"] == 1 and S.stats(0)["last_generated"] == 4
    ne, rs = S.chunk([None, a], [False, False])  # stream 0 not in this call: untouched
    assert S.stats(0)["chunk_idx"] == 1 and S.stats(1)["chunk_idx"] == 2 and S.stats(1)["chunks"] == 1
    S.reset(1)
    assert S.stats(1)["chunk_idx"] == 0 and len(S.tokens(1, "raw")) == 0
    assert S.last_chunk()["active"] == 1
    S.close()
    with pytest.raises(pkg.QdbError):
        pkg.Streams(model, 2)  # the reference's template ids exceed the tiny vocabulary
    model.close()
