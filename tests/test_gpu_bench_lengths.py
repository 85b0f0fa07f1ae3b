"""GPU parity at the benchmark configurations' own lengths, against golden
vectors the reference itself produced (tests/golden/make_golden.py):

* c0: 0.6B, 144-position prompt, 16 steps;  c1: 1.7B, 404 positions, 16 steps;
* c3: 1.7B, 3914-position prompt (tcgen05 prefill attention over 31 key tiles,
  fp16 KV), 4 steps;
* c2set: 8 independent 0.6B utterances of different lengths decoded as one
  batch (the batched path of config c2), 8 steps.

Bar (conftest): tokens equal wherever the reference's top-2 margin > 1e-2;
logits within 2e-2 max-abs on the reference's top-64 and the sum of squares of
all logits within 2e-2 relative. Teacher-forced on the reference's tokens; the
free-running device loops must reproduce the reference's tokens up to the
first exempt (small-margin) step.
"""
import numpy as np
import pytest

from conftest import MARGIN, MAX_ABS, golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def weights(synth):
    cache = {}

    def get(preset):
        if preset not in cache:
            cache.clear()  # one full-size weight set at a time
            cache[preset] = synth.WeightSet(synth.PRESETS[preset], seed=0)
        return cache[preset]
    return get


def _check_step(logits, g, step, what, row=None):
    sel = (lambda k: g[k][row][step]) if row is not None else (lambda k: g[k][step])
    d = np.abs(logits[sel("top_idx")] - sel("top_val")).max()
    assert d <= MAX_ABS, f"{what} step {step}: top-64 max|d| {d:.3g}"
    ss = float((logits.astype(np.float64) ** 2).sum())
    want = float(sel("logit_sumsq"))
    assert abs(ss - want) <= 2e-2 * want, f"{what} step {step}: sum of squares {ss:.6g} vs {want:.6g}"


def _agreeing_prefix(tokens, margins):
    """Steps up to (excluding) the first one the margin rule exempts."""
    n = 0
    for m in margins:
        if m <= MARGIN:
            break
        n += 1
    return n


@pytest.mark.parametrize("name", ["c0", "c1", "c3"])
def test_bench_config_against_reference(pkg, synth, weights, name):
    g = golden(name)
    ws = weights(str(g["preset"]))
    cfg = ws.cfg
    emb = synth.prompt_embeddings(ws, synth.audio_embeddings(cfg, int(g["n_audio"]), int(g["audio_seed"])))
    P = int(g["prefill_len"])
    steps = len(g["tokens"])
    model = pkg.Model(ws, device=0, mask_eos=True)
    ctx = pkg.Decoder(model, capacity=P + steps + 8)
    ctx.prefill(emb[:-1])
    assert ctx.last_error == "" and ctx.kv_cache_len == P
    e = emb[-1]
    for step, want in enumerate(g["tokens"]):
        tok = ctx.forward(e, want_logits=True)
        assert ctx.last_error == "", ctx.last_error
        _check_step(ctx.logits, g, step, name)
        if g["margins"][step] > MARGIN:
            assert tok == want, (name, step, tok, want)
        e = synth.embed_rows(ws, [int(want)])[0]
    # free-running device greedy loop from a fresh prefill
    s = model.session(P + steps + 8)
    s.prefill(emb[:-1], 0)
    got = s.decode_greedy(synth.PROMPT_SUFFIX[-1], P, steps)
    n = _agreeing_prefix(g["tokens"], g["margins"])
    assert list(got[:n]) == list(g["tokens"][:n]), (name, got[:n], g["tokens"][:n])
    s.close()
    ctx.session.close()
    model.close()


def _c2set_sessions(pkg, synth, ws, model, g):
    cfg = ws.cfg
    embs = [synth.prompt_embeddings(ws, synth.audio_embeddings(cfg, int(n), int(sd)))
            for n, sd in zip(g["n_audio"], g["audio_seed"])]
    steps = g["tokens"].shape[1]
    sess = []
    for e in embs:
        s = model.session(e.shape[0] + steps + 8)
        s.prefill(e[:-1], 0)
        sess.append(s)
    return embs, sess


def test_c2set_batched_against_reference(pkg, synth, weights):
    """qdb_forward_batch (tokens and logits) over 8 utterances of different
    lengths, teacher-forced, against the reference's per-utterance runs; then
    the same step repeated: the split-K atomics may reorder additions, so
    logits agree to 1e-3 max-abs between runs (tokens identical unless the
    margin rule exempts them)."""
    g = golden("c2set")
    ws = weights("0.6b")
    model = pkg.Model(ws, device=0, mask_eos=True)
    embs, sess = _c2set_sessions(pkg, synth, ws, model, g)
    B, steps = g["tokens"].shape
    pos = np.array([e.shape[0] - 1 for e in embs], np.int32)
    x = np.stack([e[-1] for e in embs])
    for step in range(steps):
        toks, logits = pkg.forward_batch(sess, x, pos + step, want_logits=True)
        for b in range(B):
            _check_step(logits[b], g, step, f"c2set row {b}", row=b)
            if g["margins"][b][step] > MARGIN:
                assert toks[b] == g["tokens"][b][step], (b, step, toks[b], g["tokens"][b][step])
        if step == steps - 1:
            toks2, logits2 = pkg.forward_batch(sess, x, pos + step, want_logits=True)
            d = np.abs(logits2 - logits).max()
            assert d <= 1e-3, f"run-to-run logits differ by {d:.3g}"
            for b in range(B):
                assert toks2[b] == toks[b] or g["margins"][b][step] <= MARGIN
        x = synth.embed_rows(ws, g["tokens"][:, step])
    for s in sess:
        s.close()
    model.close()


def test_c2set_device_batch_loop_against_reference(pkg, synth, weights):
    """qdb_decode_greedy_batch (device embedding lookup, captured step) over
    the same 8 utterances: each row reproduces the reference's tokens up to its
    first exempt step."""
    g = golden("c2set")
    ws = weights("0.6b")
    model = pkg.Model(ws, device=0, mask_eos=True)
    embs, sess = _c2set_sessions(pkg, synth, ws, model, g)
    B, steps = g["tokens"].shape
    pos = [e.shape[0] - 1 for e in embs]
    got = pkg.decode_greedy_batch(sess, [synth.PROMPT_SUFFIX[-1]] * B, pos, steps)
    for b in range(B):
        n = _agreeing_prefix(g["tokens"][b], g["margins"][b])
        assert list(got[:n, b]) == list(g["tokens"][b][:n]), (b, got[:n, b], g["tokens"][b][:n])
    for s in sess:
        s.close()
    model.close()
