"""CPU: the C-ABI library loads, exports every declared symbol, and fails
loudly (no CPU fallback) when no GPU is present."""
import ctypes
import os
import re

import pytest

from conftest import REPO, has_gpu

HEADER = os.path.join(REPO, "include", "qwen_asr_b200.h")
LIB = os.path.join(REPO, "qwen-asr_b200", "libqwen_asr_b200.so")


def declared_symbols(path):
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qdb_[a-z0-9_]+)\s*\(", text)))


def test_header_symbols_exported_and_bound(pkg):
    syms = declared_symbols(HEADER)
    assert len(syms) >= 20
    lib = ctypes.CDLL(LIB)
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in the header but not exported"
    # the Python mirror binds exactly the header's symbols
    assert sorted(pkg.ABI) == syms


def test_no_cpu_fallback_without_gpu(pkg, synth):
    if has_gpu():
        pytest.skip("a GPU is present")
    assert pkg.device_count() == 0
    ws = synth.WeightSet(synth.PRESETS["tiny"], seed=0)
    with pytest.raises(pkg.QdbError, match="not available"):
        pkg.Model(ws, device=0)


def test_config_validation_messages(pkg):
    c = pkg.QdbConfig(256, 2, 4, 2, 64, 512, 1000, 1e-6, 1e6)  # head_dim 64 unsupported
    assert not pkg.lib.qdb_model_create(ctypes.byref(c), 0)
    assert b"head_dim" in pkg.lib.qdb_last_error()
    c = pkg.QdbConfig(200, 2, 4, 2, 128, 512, 1000, 1e-6, 1e6)  # hidden not a multiple of 256
    assert not pkg.lib.qdb_model_create(ctypes.byref(c), 0)
    assert b"multiples of 256" in pkg.lib.qdb_last_error()
    c = pkg.QdbConfig(256, 2, 6, 4, 128, 512, 1000, 1e-6, 1e6)  # 6 heads over 4 kv heads
    assert not pkg.lib.qdb_model_create(ctypes.byref(c), 0)
    assert b"kv_heads" in pkg.lib.qdb_last_error()


def test_null_arguments_rejected(pkg):
    assert pkg.lib.qdb_forward(None, None, 0, None, None) == -1
    assert b"null" in pkg.lib.qdb_last_error()
    assert pkg.lib.qdb_prefill(None, None, 4, 0) == -1
    assert pkg.lib.qdb_session_create(None, 16) is None


def test_library_is_sm100a_only():
    """The fat binary carries sm_100a code only (names read with cuobjdump
    --list-elf, which prints ELF names, not code)."""
    import shutil
    import subprocess
    tool = shutil.which("cuobjdump") or "/usr/local/cuda/bin/cuobjdump"
    if not os.path.exists(tool):
        pytest.skip("cuobjdump not available")
    out = subprocess.run([tool, "--list-elf", LIB], capture_output=True, text=True).stdout
    archs = set(re.findall(r"sm_\d+a?", out))
    assert archs == {"sm_100a"}, archs


def test_dropin_adapter_exports_reference_symbols(pkg, synth):
    """The drop-in adapters export the reference's decoder, encoder and mel
    symbols (the reference's own qwen_mel_spectrogram renamed away) and,
    with no GPU, fails loudly inside the reference's qwen_decoder_load."""
    from oracle.pyoracle import RefDecoder
    p = os.path.join(REPO, "oracle", "_ref", "dropin", "libqwen_dropin.so")
    if not os.path.exists(p):
        pytest.skip("drop-in harness not built (needs the reference tree)")
    lib = ctypes.CDLL(p)
    for sym in ("qwen_decoder_load", "qwen_decoder_prefill", "qwen_decoder_forward", "qwen_decoder_release",
                "qwen_encoder_load", "qwen_encoder_forward", "qwen_encoder_release", "qwen_mel_spectrogram"):
        assert hasattr(lib, sym)
    if has_gpu():
        return
    ws = synth.WeightSet(synth.PRESETS["tiny"], seed=0)
    with pytest.raises(RuntimeError, match="qwen_decoder_load failed"):
        RefDecoder(ws, so_path=p)
