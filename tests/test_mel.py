"""Log-mel front end: the CPU restatement (oracle/mel_oracle.py) pinned to the
reference's qwen_mel_spectrogram (qwen_asr_audio.c:293-390) through the
committed fixtures, and the CUDA spectrogram (qdb_mel.cu, via the C ABI)
checked against both.

Tolerance: the log-mel values lie in about [-1, 2]; float32 sums in a
different order differ by ~2e-4 at most on these inputs, so every comparison
allows 1e-3 absolute per element (the sums of 128 or ~3000 elements 0.05 and 0.5).
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
from oracle import mel_oracle  # noqa: E402

synth = ge.load_synth()
GOLD = np.load(os.path.join(HERE, "golden", "mel_ref.npz"))
TOL = 1e-3


def names(suffix):
    return sorted(k[:-len(suffix)] for k in GOLD.files if k.endswith(suffix))


def audio(name):
    n, seed = (int(v) for v in GOLD[name + "_args"])
    return np.zeros(n, np.float32) if seed < 0 else synth.speech_audio(n, seed)


FULL = [k for k in names("_args") if k in GOLD.files]
SUMS = names("_bins")


def check_sums(name, m):
    assert m.shape == (128, GOLD[name + "_frames"].shape[0])
    np.testing.assert_allclose(m[:, :64], GOLD[name + "_head"], atol=TOL, rtol=0)
    np.testing.assert_allclose(m.sum(axis=0, dtype=np.float64), GOLD[name + "_frames"], atol=0.05, rtol=0)
    np.testing.assert_allclose(m.sum(axis=1, dtype=np.float64), GOLD[name + "_bins"], atol=0.5, rtol=0)


# --------------------------------------------------------------- CPU (oracle)
def test_frame_count_rule():
    for n in [0, 1, 159, 160, 161, 400, 4007, 480000]:
        assert mel_oracle.n_frames(n) == (n // 160 if n > 0 else 0)
    for n in GOLD["too_short"]:
        assert mel_oracle.mel_spectrogram(np.zeros(int(n), np.float32)) is None


@pytest.mark.parametrize("name", FULL)
def test_oracle_matches_reference_fixture(name):
    m = mel_oracle.mel_spectrogram(audio(name))
    assert m.shape == GOLD[name].shape
    np.testing.assert_allclose(m, GOLD[name], atol=TOL, rtol=0)


@pytest.mark.parametrize("name", SUMS)
def test_oracle_matches_reference_sums(name):
    check_sums(name, mel_oracle.mel_spectrogram(audio(name)))


def test_silence_clamps_to_floor():
    # all power below 1e-10: every value is log10(1e-10) = -10 -> (-10 + 4) / 4
    np.testing.assert_allclose(GOLD["m_silence"], -1.5, atol=1e-6)


def test_reflect_pad_rule():
    x = np.arange(1, 11, dtype=np.float32)  # shorter than the 200-sample pad
    p = mel_oracle.reflect_pad(x)
    assert p.shape == (410,)
    assert p[199] == 2 and p[191] == 10 and p[190] == 0  # samples[200 - i], 0 past the end
    assert p[210] == 9 and p[218] == 1 and p[219] == 0  # samples[n - 2 - i], 0 below 0


def test_oracle_matches_live_reference():
    from oracle.pyoracle import ref_mel_spectrogram, ref_so_path
    if not ref_so_path():
        pytest.skip("oracle/_ref not built")
    for n, seed in [(161, 11), (3333, 12), (20000, 13)]:
        x = synth.speech_audio(n, seed)
        np.testing.assert_allclose(mel_oracle.mel_spectrogram(x), ref_mel_spectrogram(x), atol=TOL, rtol=0)


# ------------------------------------------------------------ GPU (C ABI)
@pytest.fixture(scope="module")
def pkg():
    p = ge.load_package()
    if p.device_count() < 1:
        pytest.skip("no CUDA device")
    return p


@pytest.mark.gpu
@pytest.mark.parametrize("name", FULL)
def test_gpu_matches_reference_fixture(pkg, name):
    m = pkg.mel_spectrogram(audio(name))
    assert m.shape == GOLD[name].shape
    np.testing.assert_allclose(m, GOLD[name], atol=TOL, rtol=0)


@pytest.mark.gpu
@pytest.mark.parametrize("name", SUMS)
def test_gpu_matches_reference_sums(pkg, name):
    x = audio(name)
    m = pkg.mel_spectrogram(x)
    check_sums(name, m)
    np.testing.assert_allclose(m, mel_oracle.mel_spectrogram(x), atol=TOL, rtol=0)


@pytest.mark.gpu
def test_gpu_too_short_returns_none(pkg):
    for n in GOLD["too_short"]:
        if n > 0:
            assert pkg.mel_spectrogram(np.ones(int(n), np.float32)) is None
        assert pkg.mel_frames(int(n)) <= 0


@pytest.mark.gpu
@pytest.mark.parametrize("n", [160, 161, 319, 320, 16 * 160 + 1, 17 * 160, 33 * 160 + 7])
def test_gpu_ragged_frame_blocks(pkg, n):
    # frame counts around the kernel's 16-frame blocks
    x = synth.speech_audio(n, 40 + n % 7)
    np.testing.assert_allclose(pkg.mel_spectrogram(x), mel_oracle.mel_spectrogram(x), atol=TOL, rtol=0)


@pytest.mark.gpu
def test_gpu_device_form_on_stream(pkg):
    import torch
    x = synth.speech_audio(48000 + 123, 77)
    xs = torch.from_numpy(x).cuda()
    nf = pkg.mel_frames(len(x))
    out = torch.empty((128, nf), dtype=torch.float32, device="cuda")
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        pkg.mel_spectrogram_device(xs.data_ptr(), len(x), out.data_ptr(), st.cuda_stream)
    st.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), mel_oracle.mel_spectrogram(x), atol=TOL, rtol=0)
    # a second, shorter call reuses the grown scratch
    y = x[:5000].copy()
    np.testing.assert_allclose(pkg.mel_spectrogram(y), mel_oracle.mel_spectrogram(y), atol=TOL, rtol=0)


def _dropin_so():
    p = os.path.join(REPO, "oracle", "_ref", "dropin", "libqwen_dropin.so")
    return p if os.path.exists(p) else None


@pytest.mark.gpu
@pytest.mark.skipif(_dropin_so() is None, reason="drop-in harness not built (needs the reference tree)")
def test_dropin_mel_replaces_reference_symbol():
    """qwen_mel_spectrogram of the drop-in adapter (qwen-asr_b200/dropin/
    qwen_asr_mel_b200.c), resolved by symbol like the reference's caller does."""
    from oracle.pyoracle import ref_mel_spectrogram
    for name in FULL:
        np.testing.assert_allclose(ref_mel_spectrogram(audio(name), so_path=_dropin_so()), GOLD[name], atol=TOL, rtol=0)
    assert ref_mel_spectrogram(np.ones(100, np.float32), so_path=_dropin_so()) is None
