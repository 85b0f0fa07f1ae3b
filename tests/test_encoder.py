"""Audio encoder: the numpy restatement (oracle/enc_oracle.py) pinned to the
reference's qwen_encoder_forward (qwen_asr_encoder.c:171-372) through the
committed fixtures (tests/golden/enc_ref.npz, made by
tests/golden/make_golden.py --enc from oracle/_ref), and the CUDA encoder
(qdb_encoder.cu via the C ABI) checked against both.

Tolerance: the reference computes in f32 with BLAS sums; the CUDA encoder
multiplies bf16 weights with bf16 hi + lo splits of the f32 activations
(~16 mantissa bits) on tensor cores. Outputs agree to max-abs 2e-3 x the
largest |output| and 1e-3 relative L2 (measured ~1e-5 relative)."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(HERE, "golden"))

import __graft_entry__ as ge  # noqa: E402
from oracle import enc_oracle, mel_oracle  # noqa: E402

synth = ge.load_synth()
GOLD = np.load(os.path.join(HERE, "golden", "enc_ref.npz"))
import make_golden as mg  # noqa: E402  (case table and weight recipes)

CASES = {c[0]: c for c in mg.ENC_CASES}


def case_inputs(name):
    _, preset, std, jit, n, seed, _ = CASES[name]
    return mg.enc_weights(preset, std, jit), mg.enc_mel(n, seed)


def close(a, b, tol_abs=2e-3, tol_rel=1e-3):
    scale = float(np.abs(b).max())
    err = float(np.abs(a - b).max())
    rel = float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))
    assert err <= tol_abs * scale and rel <= tol_rel, (err, scale, rel)


def check_against_gold(name, y):
    assert tuple(y.shape) == tuple(GOLD[name + "_shape"])
    if name in GOLD.files:
        close(y, GOLD[name])
    else:
        close(y[:8], GOLD[name + "_head"])
        np.testing.assert_allclose(y.astype(np.float64).sum(axis=1), GOLD[name + "_rowsum"],
                                   atol=2e-3 * np.abs(GOLD[name + "_head"]).max() * y.shape[1] ** 0.5)
        np.testing.assert_allclose((y.astype(np.float64) ** 2).sum(axis=1), GOLD[name + "_rowsq"], rtol=2e-3)


# --------------------------------------------------------------------- CPU
def test_token_count_rule():
    for f in (1, 7, 8, 9, 99, 100, 101, 433, 800, 2006, 3000):
        x = np.zeros((128, f), np.float32)
        # oracle chunk walk vs the closed-form count
        assert synth.encoder_tokens(f) == sum(((((min(100, f - c) - 1) // 2) // 2) // 2) + 1
                                              for c in range(0, f, 100)), f
        del x


@pytest.mark.parametrize("name", ["e_tiny", "e_tiny_long"])
def test_oracle_matches_reference_fixture(name):
    ews, mel = case_inputs(name)
    check_against_gold(name, enc_oracle.encoder_forward(ews, mel).astype(np.float32))


def test_oracle_matches_live_reference():
    from oracle.pyoracle import RefEncoder, ref_so_path
    if not ref_so_path():
        pytest.skip("oracle/_ref not built")
    ews = synth.EncoderWeightSet(synth.ENC_PRESETS["tiny"], seed=3, norm_jitter=0.2, scale_by_fan_in=True)
    mel = mel_oracle.mel_spectrogram(synth.speech_audio(16000 * 9 + 123, 31))  # 9 s: a window boundary at 8 s
    ref = RefEncoder(ews, threads=4)
    close(enc_oracle.encoder_forward(ews, mel), ref.forward(mel), 1e-5, 1e-5)
    ref.close()


# --------------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def pkg():
    p = ge.load_package()
    if p.device_count() < 1:
        pytest.skip("no CUDA device")
    return p


@pytest.mark.gpu
@pytest.mark.parametrize("name", [c[0] for c in mg.ENC_CASES])
def test_gpu_encoder_matches_reference_fixture(pkg, name):
    ews, mel = case_inputs(name)
    enc = pkg.Encoder(ews)
    y = enc.forward(mel)
    enc.close()
    check_against_gold(name, y)


@pytest.mark.gpu
@pytest.mark.parametrize("frames", [1, 8, 9, 100, 101, 250, 899, 1700])
def test_gpu_encoder_ragged_lengths_match_oracle(pkg, frames):
    ews = synth.EncoderWeightSet(synth.ENC_PRESETS["tiny"], seed=5, norm_jitter=0.1, scale_by_fan_in=True)
    mel = np.random.default_rng(frames).uniform(-1.0, 1.5, (128, frames)).astype(np.float32)
    enc = pkg.Encoder(ews)
    y = enc.forward(mel)
    assert y.shape == (pkg.Encoder.tokens(frames), ews.cfg.output_dim) == (synth.encoder_tokens(frames), 256)
    close(y, enc_oracle.encoder_forward(ews, mel))
    enc.close()


@pytest.mark.gpu
def test_gpu_encoder_non_bf16_conv_weights(pkg):
    """f32 conv kernels that bf16 cannot hold take the second (lo) weight pass."""
    ews = synth.EncoderWeightSet(synth.ENC_PRESETS["tiny"], seed=6, scale_by_fan_in=True)

    class F32Conv:
        cfg = ews.cfg

        def __init__(self):
            rng = np.random.default_rng(0)
            self.extra = {}
            for k in (2, 3):
                nm = f"thinker.audio_tower.conv2d{k}.weight"
                w = ews.f32(nm)
                self.extra[nm] = (w * (1 + 1e-3 * rng.standard_normal(w.shape))).astype(np.float32)

        def view(self, name):
            return ews.view(name)

        def f32(self, name):
            return self.extra.get(name, ews.f32(name))

    w = F32Conv()
    mel = np.random.default_rng(7).uniform(-1.0, 1.5, (128, 333)).astype(np.float32)
    enc = pkg.Encoder(w)
    y = enc.forward(mel)
    enc.close()
    close(y, enc_oracle.encoder_forward(w, mel))


@pytest.mark.gpu
def test_gpu_encoder_device_form_and_reuse(pkg):
    import torch
    ews, mel = case_inputs("e_tiny")
    enc = pkg.Encoder(ews)
    m = torch.from_numpy(mel).cuda()
    n = pkg.Encoder.tokens(mel.shape[1])
    out = torch.empty((n, ews.cfg.output_dim), dtype=torch.float32, device="cuda")
    assert enc.forward_device(m.data_ptr(), mel.shape[1], out.data_ptr()) == n
    torch.cuda.synchronize()
    torch.cuda.ExternalStream(enc.stream_handle).synchronize()
    check_against_gold("e_tiny", out.cpu().numpy())
    # a longer then a shorter call on the same encoder (scratch growth)
    _ = enc.forward(np.tile(mel, (1, 5)))
    check_against_gold("e_tiny", enc.forward(mel))
    enc.close()


def _dropin_so():
    p = os.path.join(REPO, "oracle", "_ref", "dropin", "libqwen_dropin.so")
    return p if os.path.exists(p) else None


@pytest.mark.gpu
@pytest.mark.skipif(_dropin_so() is None, reason="drop-in harness not built (needs the reference tree)")
@pytest.mark.parametrize("name", ["e_tiny", "e_06b"])
def test_dropin_encoder_through_reference_loader(name):
    """qwen_encoder_load / qwen_encoder_forward of the drop-in adapter
    (qwen-asr_b200/dropin/qwen_asr_encoder_b200.c), driven by the same harness
    and the reference's own safetensors loader as the reference encoder."""
    from oracle.pyoracle import RefEncoder
    ews, mel = case_inputs(name)
    enc = RefEncoder(ews, so_path=_dropin_so())
    check_against_gold(name, enc.forward(mel))
    enc.close()


@pytest.mark.gpu
def test_gpu_encoder_batch_equals_separate_calls(pkg):
    """Utterances of different lengths in one pass: each one's rows equal its
    own forward (windows restart per utterance)."""
    import torch
    ews = synth.EncoderWeightSet(synth.ENC_PRESETS["tiny"], seed=8, norm_jitter=0.1, scale_by_fan_in=True)
    frames = [1500, 37, 900, 1, 260, 2150]  # windows cut mid-utterance, a 1-frame utterance
    mels = [np.random.default_rng(f).uniform(-1.0, 1.5, (128, f)).astype(np.float32) for f in frames]
    enc = pkg.Encoder(ews)
    sep = [enc.forward(m) for m in mels]
    dm = [torch.from_numpy(m).cuda() for m in mels]
    n = sum(pkg.Encoder.tokens(f) for f in frames)
    out = torch.empty((n, ews.cfg.output_dim), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    assert enc.forward_batch_device([t.data_ptr() for t in dm], frames, out.data_ptr()) == n
    torch.cuda.ExternalStream(enc.stream_handle).synchronize()
    got = out.cpu().numpy()
    r = 0
    for y, m in zip(sep, mels):
        close(got[r:r + len(y)], y, 1e-4, 1e-4)  # split-K vs persistent GEMM tiling only
        close(y, enc_oracle.encoder_forward(ews, m))
        r += len(y)
    enc.close()
