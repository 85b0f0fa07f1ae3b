"""GPU: the error paths, exercised without faulting the GPU.

* Host-side injection (QWEN_ASR_B200_FAULT=alloc|launch): a failing call must
  follow the reference's conventions - qwen_decoder_prefill returns silently
  with kv_cache_len unchanged (qwen_asr_decoder.c:276-282) and
  qwen_decoder_forward returns QWEN_TOKEN_IM_END (qwen_asr_decoder.c:417,
  :421) - both in the Python mirror and through the drop-in C decoder driven
  by the reference's own harness; once the fault is lifted the same context
  decodes correctly.
* Bounded device waits: with the wait limit set to 0 cycles, the persistent
  decode step's first unsatisfied wait (a CTA polling another CTA's q/k/v)
  runs out; the kernel records the error, drains its own copies and returns,
  the call reports "a bounded wait ... ran out", and after the limit is
  restored the model decodes the same tokens as an untouched session.
"""
import os

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu


def _tiny(pkg, synth, mask=False):
    cfg = synth.PRESETS["tiny"]
    ws = synth.WeightSet(cfg, seed=12, norm_jitter=0.1)
    emb = synth.audio_embeddings(cfg, 30, seed=4)
    return ws, emb, pkg.Model(ws, device=0, mask_eos=mask)


def test_injected_launch_failure_keeps_reference_conventions(pkg, synth, monkeypatch):
    ws, emb, model = _tiny(pkg, synth)
    ctx = pkg.Decoder(model, capacity=64)
    clean = model.session(64)
    clean.prefill(emb[:20], 0)
    want, _, _ = clean.forward(emb[20], 20)
    monkeypatch.setenv("QWEN_ASR_B200_FAULT", "launch")
    ctx.prefill(emb[:20])
    assert ctx.kv_cache_len == 0 and "injected launch failure" in ctx.last_error
    monkeypatch.delenv("QWEN_ASR_B200_FAULT")
    ctx.last_error = ""
    ctx.prefill(emb[:20])
    assert ctx.kv_cache_len == 20 and ctx.last_error == ""
    monkeypatch.setenv("QWEN_ASR_B200_FAULT", "alloc,launch")
    assert ctx.forward(emb[20]) == pkg.QWEN_TOKEN_IM_END
    assert ctx.kv_cache_len == 20 and "injected" in ctx.last_error
    monkeypatch.delenv("QWEN_ASR_B200_FAULT")
    assert ctx.forward(emb[20]) == want
    assert ctx.kv_cache_len == 21


def test_injected_allocation_failure(pkg, synth, monkeypatch):
    """A prefill that must grow the KV cache fails cleanly when allocation
    fails; the cache keeps its contents and the call succeeds afterwards."""
    ws, emb, model = _tiny(pkg, synth)
    ctx = pkg.Decoder(model, capacity=8)
    ctx.prefill(emb[:6])
    assert ctx.kv_cache_len == 6
    monkeypatch.setenv("QWEN_ASR_B200_FAULT", "alloc")
    ctx.prefill(emb[6:26])  # needs 26 positions > capacity 8: growth allocates
    assert ctx.kv_cache_len == 6 and "injected allocation failure" in ctx.last_error
    with pytest.raises(pkg.QdbError, match="injected allocation failure"):
        model.session(16)
    monkeypatch.delenv("QWEN_ASR_B200_FAULT")
    ctx.prefill(emb[6:26])
    assert ctx.kv_cache_len == 26
    clean = model.session(64)
    clean.prefill(emb[:26], 0)
    assert ctx.forward(emb[26]) == clean.forward(emb[26], 26)[0]


def _dropin_so():
    p = os.path.join(REPO, "oracle", "_ref", "dropin", "libqwen_dropin.so")
    return p if os.path.exists(p) else None


@pytest.mark.skipif(_dropin_so() is None, reason="drop-in harness not built (needs the reference tree)")
def test_dropin_error_conventions(synth, monkeypatch):
    """Through the reference's own qwen_decoder_prefill / qwen_decoder_forward
    (drop-in decoder + reference harness)."""
    from oracle.pyoracle import RefDecoder
    cfg = synth.PRESETS["tiny"]
    ws = synth.WeightSet(cfg, seed=12, norm_jitter=0.1)
    emb = synth.audio_embeddings(cfg, 30, seed=4)
    d = RefDecoder(ws, so_path=_dropin_so())
    d.kv_cache_len = 0
    monkeypatch.setenv("QWEN_ASR_B200_FAULT", "launch")
    d.prefill(emb[:20])
    assert d.kv_cache_len == 0  # silent return, length unchanged
    monkeypatch.delenv("QWEN_ASR_B200_FAULT")
    d.prefill(emb[:20])
    assert d.kv_cache_len == 20
    monkeypatch.setenv("QWEN_ASR_B200_FAULT", "launch")
    tok, _, _ = d.forward(emb[20], want_logits=False)
    assert tok == 151645 and d.kv_cache_len == 20  # QWEN_TOKEN_IM_END, no position consumed
    monkeypatch.delenv("QWEN_ASR_B200_FAULT")
    tok, _, _ = d.forward(emb[20], want_logits=False)
    assert d.kv_cache_len == 21 and 0 <= tok < cfg.vocab
    d.close()


def test_bounded_wait_runs_out_and_the_model_recovers(pkg, synth):
    ws, emb, model = _tiny(pkg, synth)
    a, clean = model.session(64), model.session(64)
    a.prefill(emb[:20], 0)
    clean.prefill(emb[:20], 0)
    ctx = pkg.Decoder(model, capacity=64)
    ctx.prefill(emb[:20])
    try:
        model.set_wait_limit(0)
        with pytest.raises(pkg.QdbError, match="bounded wait"):
            a.forward(emb[20], 20)
        # the mirror turns it into the reference's error token
        assert ctx.forward(emb[20]) == pkg.QWEN_TOKEN_IM_END and ctx.kv_cache_len == 20
        assert "bounded wait" in ctx.last_error
    finally:
        model.set_wait_limit(-1)
    want = [clean.forward(emb[20 + i], 20 + i)[0] for i in range(3)]
    got = [a.forward(emb[20 + i], 20 + i)[0] for i in range(3)]
    assert got == want
    assert ctx.forward(emb[20]) == want[0] and ctx.kv_cache_len == 21


def test_bounded_wait_in_the_batched_path(pkg, synth):
    """The tensor-core GEMMs of the batched step honour the same limit."""
    ws, emb, model = _tiny(pkg, synth)
    sess = [model.session(64) for _ in range(3)]
    for s in sess:
        s.prefill(emb[:20], 0)
    x = np.stack([emb[20]] * 3)
    try:
        model.set_wait_limit(0)
        with pytest.raises(pkg.QdbError, match="bounded wait"):
            pkg.forward_batch(sess, x, [20] * 3)
    finally:
        model.set_wait_limit(-1)
    got = pkg.forward_batch(sess, x, [20] * 3)
    clean = model.session(64)
    clean.prefill(emb[:20], 0)
    want = clean.forward(emb[20], 20)[0]
    assert list(got) == [want] * 3
