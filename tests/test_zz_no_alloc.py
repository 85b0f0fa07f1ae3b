"""GPU: qdb_forward_noalloc, the decode step for callers that may not allocate
GPU memory while decoding (a fixed memory budget they do not control, a
real-time loop that cannot risk the device-wide stall of a cudaMalloc, or a
host that forbids allocation after start-up). It runs the same step kernel as
qdb_forward with its scratch in one fixed array inside the library, so its
greedy tokens must equal qdb_forward's on the same inputs, call after call.

Kept in a file of its own that is collected last.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_noalloc_step_matches_forward_twice(pkg, synth, monkeypatch):
    import torch

    cfg = synth.PRESETS["small"]
    ws = synth.WeightSet(cfg, seed=21, norm_jitter=0.1)
    emb = synth.audio_embeddings(cfg, 40, seed=5)
    model = pkg.Model(ws, device=0, mask_eos=True)
    ref, nal = model.session(64), model.session(64)
    P = 36
    ref.prefill(emb[:P], 0)
    nal.prefill(emb[:P], 0)
    tok_dev = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    wants = [ref.forward(emb[pos], pos)[0] for pos in (P, P + 1, P + 2)]
    e_devs = [torch.from_numpy(np.ascontiguousarray(emb[pos])).to("cuda:0") for pos in (P, P + 1, P + 2)]
    torch.cuda.synchronize()
    for i, pos in enumerate((P, P + 1, P + 2)):  # calls in a row: the shared scratch is reused
        free_before = torch.cuda.mem_get_info(0)[0]
        if i:  # after the first call (its one-time set-up): any library allocation would now fail
            monkeypatch.setenv("QWEN_ASR_B200_FAULT", "alloc")
        rc = pkg.lib.qdb_forward_noalloc(nal.h, ctypes.c_void_p(e_devs[i].data_ptr()), pos,
                                         ctypes.c_void_p(tok_dev.data_ptr()))
        monkeypatch.delenv("QWEN_ASR_B200_FAULT", raising=False)
        assert rc == 0, pkg.lib.qdb_last_error()
        if i:
            assert torch.cuda.mem_get_info(0)[0] == free_before, "device memory changed across the call"
        assert int(tok_dev.item()) == wants[i], (pos, int(tok_dev.item()), wants[i])
    e_dev = e_devs[0]
    # sizes the array cannot serve are refused with a clear error, not run
    rc = pkg.lib.qdb_forward_noalloc(nal.h, ctypes.c_void_p(e_dev.data_ptr()), 10_000,
                                     ctypes.c_void_p(tok_dev.data_ptr()))
    assert rc == -1 and b"capacity" in pkg.lib.qdb_last_error()
