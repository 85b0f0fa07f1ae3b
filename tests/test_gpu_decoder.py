"""GPU parity of the CUDA decoder against the reference (golden vectors made by
the reference's own code) and the CPU oracle, through the C ABI.

Bar: greedy tokens identical wherever the reference's top-2 margin > 1e-2;
final-layer logits within 2e-2 max-abs and 1e-2 relative L2 (conftest).
Comparisons are teacher-forced on the reference's tokens so that one exempt
near-tie cannot cascade.
"""
import numpy as np
import pytest

from conftest import MARGIN, MAX_ABS, assert_logits_close, golden
from oracle.pyoracle import Oracle, margin_top2

pytestmark = pytest.mark.gpu

SMALL = ["tiny", "gqa4", "small"]


def _setup(synth, g):
    cfg = synth.PRESETS[str(g["preset"])]
    ws = synth.WeightSet(cfg, seed=int(g["weight_seed"]), norm_jitter=float(g["norm_jitter"]))
    emb = synth.prompt_embeddings(ws, synth.audio_embeddings(cfg, int(g["n_audio"]), int(g["audio_seed"])))
    return cfg, ws, emb


@pytest.fixture(scope="module")
def models(pkg, synth):
    cache = {}

    def get(name):
        if name not in cache:
            g = golden(name)
            cfg, ws, emb = _setup(synth, g)
            cache[name] = (g, ws, emb, pkg.Model(ws, device=0, mask_eos=True))
        return cache[name]
    return get


@pytest.mark.parametrize("name", SMALL)
def test_forward_matches_reference_golden(pkg, synth, models, name):
    g, ws, emb, model = models(name)
    ctx = pkg.Decoder(model, capacity=64)
    ctx.prefill(emb[:-1])
    assert ctx.kv_cache_len == int(g["prefill_len"])
    e = emb[-1]
    for step, want in enumerate(g["tokens"]):
        tok = ctx.forward(e, want_logits=True)
        assert ctx.last_error == ""
        assert_logits_close(ctx.logits, g["logits"][step], f"{name} step {step}")
        if g["margins"][step] > MARGIN:
            assert tok == want, (name, step, tok, want)
        e = synth.embed_rows(ws, [int(want)])[0]
    # rewind of the host-owned length (stream prefix reuse) then continue
    ctx.kv_cache_len = int(g["rewind_pos"])
    e = synth.embed_rows(ws, [int(g["tokens"][1])])[0]
    for step, want in enumerate(g["rewind_tokens"]):
        tok = ctx.forward(e, want_logits=True)
        assert_logits_close(ctx.logits, g["rewind_logits"][step], f"{name} rewind {step}")
        e = synth.embed_rows(ws, [int(want)])[0]


@pytest.mark.parametrize("name", SMALL)
def test_device_greedy_loop_matches_host_loop(pkg, synth, models, name):
    """qdb_decode_greedy (embedding lookup on the device) == host loop of
    qdb_forward calls with host embeddings."""
    g, ws, emb, model = models(name)
    a, b = model.session(64), model.session(64)
    P = emb.shape[0] - 1
    a.prefill(emb[:-1], 0)
    b.prefill(emb[:-1], 0)
    t0, _, _ = a.forward(emb[-1], P)
    tb, _, _ = b.forward(emb[-1], P)
    assert t0 == tb
    dev = a.decode_greedy(t0, P + 1, 12)
    host, t = [], t0
    for i in range(12):
        t, _, _ = b.forward(synth.embed_rows(ws, [t])[0], P + 1 + i)
        host.append(t)
    assert list(dev) == host


def test_hidden_state_matches_oracle(pkg, synth, models):
    """ctx->dec_x equivalent (final-normed hidden) against the oracle."""
    g, ws, emb, model = models("small")
    s = model.session(64)
    o = Oracle(ws, max_pos=128)
    s.prefill(emb[:-1], 0)
    o.prefill(emb[:-1])
    _, hid, _ = s.forward(emb[-1], emb.shape[0] - 1, want_hidden=True)
    _, ohid, _ = o.forward(emb[-1])
    # bf16 KV cache: ~0.5% elementwise noise on a unit-RMS vector
    rel = np.linalg.norm(hid - ohid) / np.linalg.norm(ohid)
    assert rel <= 1e-2 and np.abs(hid - ohid).max() <= 3e-2, rel


@pytest.mark.parametrize("chunks", [[1], [1, 1, 1], [7, 1, 30], [64], [3, 0, 5]])
def test_chunked_prefill_and_edges(pkg, synth, chunks):
    """Prefill in several calls (1-position calls, an empty call) at growing
    start positions equals the oracle."""
    cfg = synth.PRESETS["tiny"]
    ws = synth.WeightSet(cfg, seed=4, norm_jitter=0.1)
    emb = synth.audio_embeddings(cfg, sum(chunks) + 1, seed=11)
    model = pkg.Model(ws, device=0)
    s = model.session(8)  # small capacity: forces KV growth with content kept
    o = Oracle(ws, max_pos=256)
    at = 0
    for c in chunks:
        s.prefill(emb[at:at + c], at)
        o.prefill(emb[at:at + c])
        at += c
    assert s.capacity >= at + 1
    tok, _, lg = s.forward(emb[at], at, want_logits=True)
    otok, _, olg = o.forward(emb[at])
    assert_logits_close(lg, olg, f"chunks {chunks}")
    assert tok == otok or margin_top2(olg) <= MARGIN


def test_long_context_split_attention(pkg, synth):
    """Context longer than every split threshold (attention over ~1.1k keys,
    many splits) against the oracle, decode steps past a KV growth."""
    cfg = synth.PRESETS["tiny"]
    ws = synth.WeightSet(cfg, seed=6, norm_jitter=0.1)
    emb = synth.audio_embeddings(cfg, 1100, seed=12)
    model = pkg.Model(ws, device=0)
    s = model.session(512)
    o = Oracle(ws, max_pos=1200)
    s.prefill(emb[:1090], 0)
    o.prefill(emb[:1090])
    for i in range(1090, 1100):
        tok, _, lg = s.forward(emb[i], i, want_logits=True)
        otok, _, olg = o.forward(emb[i])
        assert_logits_close(lg, olg, f"pos {i}")
        assert tok == otok or margin_top2(olg) <= MARGIN


def test_session_outlives_model(pkg, synth):
    """Freeing the model first detaches its sessions; later calls fail cleanly."""
    ws = synth.WeightSet(synth.PRESETS["tiny"], seed=1)
    model = pkg.Model(ws, device=0)
    s = model.session(16)
    model.close()
    with pytest.raises(pkg.QdbError, match="freed"):
        s.forward(np.zeros(ws.cfg.hidden, np.float32), 0)
    s.close()


def test_batched_decode_matches_single(pkg, synth):
    """qdb_forward_batch over independent sessions at different positions ==
    per-session qdb_forward (the row-batched path vs the persistent step)."""
    cfg = synth.PRESETS["small"]
    ws = synth.WeightSet(cfg, seed=7, norm_jitter=0.1)
    model = pkg.Model(ws, device=0, mask_eos=True)
    n = 5
    lens = [9, 30, 17, 64, 3]
    embs = [synth.audio_embeddings(cfg, L + 3, seed=100 + b) for b, L in enumerate(lens)]
    sb = [model.session(32) for _ in range(n)]
    ss = [model.session(32) for _ in range(n)]
    for b in range(n):
        sb[b].prefill(embs[b][:lens[b]], 0)
        ss[b].prefill(embs[b][:lens[b]], 0)
    for step in range(3):
        x = np.stack([embs[b][lens[b] + step] for b in range(n)])
        pos = [lens[b] + step for b in range(n)]
        got = pkg.forward_batch(sb, x, pos)
        for b in range(n):
            want, _, lg = ss[b].forward(x[b], pos[b], want_logits=True)
            assert got[b] == want or margin_top2(lg, mask_eos=True) <= MARGIN, (step, b)


def test_forward_batch_graph_reuse_across_session_groups(pkg, synth):
    """qdb_forward_batch replays one captured step for every call with the same
    row count: two disjoint groups of sessions (other KV caches, other
    positions) alternate through it, and each step still equals per-session
    qdb_forward."""
    cfg = synth.PRESETS["small"]
    ws = synth.WeightSet(cfg, seed=8, norm_jitter=0.1)
    model = pkg.Model(ws, device=0, mask_eos=True)
    n = 4
    groups = []
    for gi, lens in enumerate([[5, 21, 40, 12], [33, 2, 17, 60]]):
        embs = [synth.audio_embeddings(cfg, L + 4, seed=300 + 10 * gi + b) for b, L in enumerate(lens)]
        sb = [model.session(80) for _ in range(n)]
        ss = [model.session(80) for _ in range(n)]
        for b in range(n):
            sb[b].prefill(embs[b][:lens[b]], 0)
            ss[b].prefill(embs[b][:lens[b]], 0)
        groups.append((lens, embs, sb, ss))
    for step in range(3):
        for gi, (lens, embs, sb, ss) in enumerate(groups):
            x = np.stack([embs[b][lens[b] + step] for b in range(n)])
            pos = [lens[b] + step for b in range(n)]
            got = pkg.forward_batch(sb, x, pos)
            for b in range(n):
                want, _, lg = ss[b].forward(x[b], pos[b], want_logits=True)
                assert got[b] == want or margin_top2(lg, mask_eos=True) <= MARGIN, (step, gi, b)


def test_batched_greedy_loop_matches_oracle(pkg, synth):
    cfg = synth.PRESETS["tiny"]
    ws = synth.WeightSet(cfg, seed=8, norm_jitter=0.1)
    model = pkg.Model(ws, device=0)
    n, steps = 3, 6
    embs = [synth.audio_embeddings(cfg, 12 + 5 * b, seed=200 + b) for b in range(n)]
    sess = [model.session(16) for _ in range(n)]
    first, pos = [], []
    for b in range(n):
        sess[b].prefill(embs[b][:-1], 0)
        t, _, _ = sess[b].forward(embs[b][-1], embs[b].shape[0] - 1)
        first.append(t)
        pos.append(embs[b].shape[0])
    got = pkg.decode_greedy_batch(sess, first, pos, steps)
    for b in range(n):
        o = Oracle(ws, max_pos=64)
        o.prefill(embs[b][:-1])
        t, _, lg = o.forward(embs[b][-1])
        for i in range(steps):
            t_prev = int(got[i - 1, b]) if i else first[b]
            t, _, lg = o.forward(synth.embed_rows(ws, [t_prev])[0])
            assert got[i, b] == t or margin_top2(lg) <= MARGIN, (b, i)


@pytest.mark.parametrize("name", ["0.6b", "1.7b"])
def test_full_size_against_reference_golden(pkg, synth, name):
    """Real 0.6B / 1.7B shapes: tokens and the reference's top-64 logits."""
    g = golden(name)
    cfg, ws, emb = _setup(synth, g)
    model = pkg.Model(ws, device=0, mask_eos=True)
    ctx = pkg.Decoder(model, capacity=256)
    ctx.prefill(emb[:-1])
    e = emb[-1]
    for step, want in enumerate(g["tokens"]):
        tok = ctx.forward(e, want_logits=True)
        assert ctx.last_error == ""
        d = np.abs(ctx.logits[g["top_idx"][step]] - g["top_val"][step]).max()
        assert d <= MAX_ABS, (step, d)
        ss = float((ctx.logits.astype(np.float64) ** 2).sum())
        assert abs(ss - g["logit_sumsq"][step]) <= 2e-2 * g["logit_sumsq"][step]
        if g["margins"][step] > MARGIN:
            assert tok == want, (step, tok, want)
        e = synth.embed_rows(ws, [int(want)])[0]
    model.close()


def _dropin_so():
    import os
    from conftest import REPO
    p = os.path.join(REPO, "oracle", "_ref", "dropin", "libqwen_dropin.so")
    return p if os.path.exists(p) else None


@pytest.mark.skipif(_dropin_so() is None, reason="drop-in harness not built (needs the reference tree)")
@pytest.mark.parametrize("name", SMALL)
def test_dropin_reference_api_matches_golden(synth, name, monkeypatch):
    """The CUDA library behind the reference's own qwen_decoder_load /
    qwen_decoder_prefill / qwen_decoder_forward (qwen-asr_b200/dropin), loaded
    by the reference's safetensors loader, against the reference's golden
    tokens and logits (logits from ctx->dec_x, as for the reference)."""
    from oracle.pyoracle import RefDecoder
    monkeypatch.setenv("QWEN_B200_MASK_EOS", "1")
    g = golden(name)
    cfg, ws, emb = _setup(synth, g)
    d = RefDecoder(ws, so_path=_dropin_so())
    d.kv_cache_len = 0
    d.prefill(emb[:-1])
    assert d.kv_cache_len == int(g["prefill_len"])
    e = emb[-1]
    for step, want in enumerate(g["tokens"]):
        tok, _, lg = d.forward(e, mask_eos=True)
        assert_logits_close(lg, g["logits"][step], f"dropin {name} step {step}")
        if g["margins"][step] > MARGIN:
            assert tok == want, (step, tok, want)
        e = synth.embed_rows(ws, [int(want)])[0]
    d.kv_cache_len = int(g["rewind_pos"])  # the streaming caller's rewind
    e = synth.embed_rows(ws, [int(g["tokens"][1])])[0]
    for step, want in enumerate(g["rewind_tokens"]):
        tok, _, lg = d.forward(e, mask_eos=True)
        assert_logits_close(lg, g["rewind_logits"][step], f"dropin {name} rewind {step}")
        e = synth.embed_rows(ws, [int(want)])[0]
    d.close()


@pytest.mark.parametrize("heads,kv_heads,chunks", [(4, 4, [200, 150]), (8, 1, [130, 1, 97]), (8, 2, [300])])
def test_prefill_attention_groupings(pkg, synth, heads, kv_heads, chunks):
    """Prefill attention for every GQA grouping the tensor-core kernel is
    built for (1, 8 and 4 query heads per KV head here; 2 in the tests
    above), over several 128-key tiles and query tiles, with prefill calls
    that start mid-tile, against the oracle."""
    cfg = synth.Config(256, 2, heads, kv_heads, 128, 512, 600)
    ws = synth.WeightSet(cfg, seed=9, norm_jitter=0.1)
    n = sum(chunks)
    emb = synth.audio_embeddings(cfg, n + 2, seed=13)
    model = pkg.Model(ws, device=0)
    s = model.session(n + 8)
    o = Oracle(ws, max_pos=n + 8)
    at = 0
    for c in chunks:
        s.prefill(emb[at:at + c], at)
        o.prefill(emb[at:at + c])
        at += c
    for i in range(at, at + 2):
        tok, _, lg = s.forward(emb[i], i, want_logits=True)
        otok, _, olg = o.forward(emb[i])
        assert_logits_close(lg, olg, f"R={heads // kv_heads} pos {i}")
        assert tok == otok or margin_top2(olg) <= MARGIN


@pytest.mark.parametrize("n", [1, 17, 64])
def test_persistent_batch_step_matches_graph_path(pkg, synth, monkeypatch, n):
    """The persistent batched step (one cooperative launch, n <= 64, selected
    with QWEN_ASR_B200_BATCH=persistent) against the default launch-per-kernel
    graph path on the same sessions: tokens equal under the margin rule and
    logits within the parity bar, at 1, 17 (padded to 32 columns) and 64 rows,
    with several key splits."""
    cfg = synth.PRESETS["small"]
    ws = synth.WeightSet(cfg, seed=31, norm_jitter=0.1)
    model = pkg.Model(ws, device=0, mask_eos=True)
    lens = [5 + (37 * b) % 300 for b in range(n)]
    embs = [synth.audio_embeddings(cfg, L + 2, seed=500 + b) for b, L in enumerate(lens)]
    sa = [model.session(320) for _ in range(n)]
    sg = [model.session(320) for _ in range(n)]
    for b in range(n):
        sa[b].prefill(embs[b][:lens[b]], 0)
        sg[b].prefill(embs[b][:lens[b]], 0)
    for step in range(2):
        x = np.stack([embs[b][lens[b] + step] for b in range(n)])
        pos = [lens[b] + step for b in range(n)]
        monkeypatch.setenv("QWEN_ASR_B200_BATCH", "persistent")
        ta, la = pkg.forward_batch(sa, x, pos, want_logits=True)
        monkeypatch.delenv("QWEN_ASR_B200_BATCH")
        tg, lg = pkg.forward_batch(sg, x, pos, want_logits=True)
        for b in range(n):
            assert_logits_close(la[b], lg[b], f"n={n} step {step} row {b}")
            assert ta[b] == tg[b] or margin_top2(lg[b], mask_eos=True) <= MARGIN


def test_batch_above_64_rows_uses_graph_path(pkg, synth):
    """More than 64 rows: the graph path serves the call; rows agree with the
    per-session step."""
    cfg = synth.PRESETS["tiny"]
    ws = synth.WeightSet(cfg, seed=32, norm_jitter=0.1)
    model = pkg.Model(ws, device=0, mask_eos=True)
    n = 70
    emb = synth.audio_embeddings(cfg, 12, seed=9)
    sess = [model.session(16) for _ in range(n)]
    for s in sess:
        s.prefill(emb[:10], 0)
    got = pkg.forward_batch(sess, np.stack([emb[10]] * n), [10] * n)
    ref = model.session(16)
    ref.prefill(emb[:10], 0)
    want, _, lg = ref.forward(emb[10], 10, want_logits=True)
    assert all(t == want for t in got) or margin_top2(lg, mask_eos=True) <= MARGIN


def test_prefill_batch_equals_separate_prefills(pkg, synth):
    """qdb_prefill_batch over sessions of different lengths and start
    positions (one row batch, segmented tensor-core attention) leaves every
    cache as separate qdb_prefill calls do: the next step's logits agree."""
    cfg = synth.PRESETS["small"]
    ws = synth.WeightSet(cfg, seed=33, norm_jitter=0.1)
    model = pkg.Model(ws, device=0)
    lens = [37, 1, 130, 0, 64]
    starts = [0, 5, 12, 0, 0]
    emb = [synth.audio_embeddings(cfg, st + L + 1, seed=600 + i) for i, (st, L) in enumerate(zip(starts, lens))]
    sa = [model.session(8) for _ in lens]
    sb = [model.session(256) for _ in lens]
    for i, st in enumerate(starts):  # shared history before the batched part
        if st:
            sa[i].prefill(emb[i][:st], 0)
            sb[i].prefill(emb[i][:st], 0)
    pkg.prefill_batch(sa, [emb[i][starts[i]:starts[i] + lens[i]] for i in range(len(lens))], starts)
    for i in range(len(lens)):
        if lens[i]:
            sb[i].prefill(emb[i][starts[i]:starts[i] + lens[i]], starts[i])
    for i in range(len(lens)):
        p = starts[i] + lens[i]
        ta, _, la = sa[i].forward(emb[i][p], p, want_logits=True)
        tb, _, lb = sb[i].forward(emb[i][p], p, want_logits=True)
        assert_logits_close(la, lb, f"session {i}")
        assert ta == tb or margin_top2(lb) <= MARGIN


def test_persistent_batch_greedy_loop_matches_graph_path(pkg, synth, monkeypatch):
    """qdb_decode_greedy_batch through the persistent step (one launch per
    position) equals the default graph loop, token for token, at the 0.6B
    shape with 8 utterances of different lengths."""
    cfg = synth.PRESETS["0.6b"]
    ws = synth.WeightSet(cfg, seed=0)
    model = pkg.Model(ws, device=0, mask_eos=True)
    lens = [40, 75, 13, 120, 64, 90, 27, 101]
    embs = [synth.audio_embeddings(cfg, L, seed=700 + b) for b, L in enumerate(lens)]
    sa = [model.session(160) for _ in lens]
    sg = [model.session(160) for _ in lens]
    pkg.prefill_batch(sa, embs, [0] * len(lens))
    pkg.prefill_batch(sg, embs, [0] * len(lens))
    monkeypatch.setenv("QWEN_ASR_B200_BATCH", "persistent")
    ta = pkg.decode_greedy_batch(sa, [198] * len(lens), lens, 12)
    monkeypatch.delenv("QWEN_ASR_B200_BATCH")
    tg = pkg.decode_greedy_batch(sg, [198] * len(lens), lens, 12)
    assert (ta == tg).mean() >= 0.9, (ta, tg)  # exact except where a near-tie flips


@pytest.mark.parametrize("heads,kv_heads", [(4, 4), (4, 2), (8, 2), (8, 1)])
def test_batched_decode_long_contexts_groupings(pkg, synth, heads, kv_heads):
    """qdb_forward_batch with contexts past one 512-key attention unit (the
    rows' keys split over up to 3 units whose last finisher merges the
    partials inside the attention kernel; a 40-key row leaves units empty),
    for 1, 2, 4 and 8 query heads per KV head, against per-session
    qdb_forward (the b=1 step kernel)."""
    cfg = synth.Config(256, 2, heads, kv_heads, 128, 512, 600)
    ws = synth.WeightSet(cfg, seed=10, norm_jitter=0.1)
    model = pkg.Model(ws, device=0, mask_eos=True)
    lens = [1100, 40, 530, 700]
    embs = [synth.audio_embeddings(cfg, L + 3, seed=800 + b) for b, L in enumerate(lens)]
    sb = [model.session(L + 8) for L in lens]
    ss = [model.session(L + 8) for L in lens]
    for b, L in enumerate(lens):
        sb[b].prefill(embs[b][:L], 0)
        ss[b].prefill(embs[b][:L], 0)
    for step in range(3):
        x = np.stack([embs[b][L + step] for b, L in enumerate(lens)])
        pos = [L + step for L in lens]
        got, logits = pkg.forward_batch(sb, x, pos, want_logits=True)
        for b in range(len(lens)):
            want, _, lg = ss[b].forward(x[b], pos[b], want_logits=True)
            assert_logits_close(logits[b], lg, f"R={heads // kv_heads} row {b} step {step}")
            assert got[b] == want or margin_top2(lg, mask_eos=True) <= MARGIN, (step, b)
