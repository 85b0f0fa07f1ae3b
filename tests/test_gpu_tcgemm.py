"""GPU: the tcgen05 tensor-core GEMM of the row-batched path against an f64
reference. The activations are f32 split into bf16 hi + lo, so the product
must match the f32 computation of the reference's prefill GEMM (cblas_sgemm
after bf16->f32 widening, qwen_asr_kernels.c:462-472) to ~1e-5 relative."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(pkg, W, X, mode, Y0=None, splits=1):
    import torch
    dev = "cuda:0"
    n, K = X.shape
    N = W.shape[0]
    Wt = torch.from_numpy(W).to(dev)                      # bf16 bits as int16
    Xt = torch.from_numpy(X).to(dev)
    Xh = Xt.to(torch.bfloat16)
    Xl = (Xt - Xh.float()).to(torch.bfloat16)
    out_cols = N // 2 if mode == 2 else N
    Y = torch.from_numpy(Y0.copy()).to(dev) if Y0 is not None else torch.zeros(n, out_cols, device=dev)
    err = torch.zeros(4, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    f = pkg.lib.qdb_launch_gemm_tc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [ctypes.c_void_p, ctypes.c_void_p]
    rc = f(Wt.data_ptr(), Xh.data_ptr(), Xl.data_ptr(), Y.data_ptr(), n, N, K, mode, splits, err.data_ptr(), st)
    assert rc == 0, rc
    torch.cuda.synchronize()
    assert int(err[0].item()) == 0
    return Y.cpu().numpy()


def _ref(W, X, mode, Y0=None):
    Wf = (W.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    P = X.astype(np.float64) @ Wf.T
    if mode in (1, 3):
        return Y0.astype(np.float64) + P
    if mode == 2:
        g, u = P[:, 0::2], P[:, 1::2]
        return g / (1.0 + np.exp(-g)) * u
    return P


@pytest.mark.parametrize("n,N,K,mode", [
    (37, 256, 256, 0), (64, 384, 1024, 0), (200, 4096, 1024, 0), (130, 1000, 512, 0),
    (77, 512, 768, 1), (404, 1024, 2048, 1), (19, 1024, 256, 2), (150, 6144, 1024, 2)])
def test_tc_gemm_matches_f64(pkg, n, N, K, mode):
    import torch
    rng = np.random.default_rng(n * 7 + N + K + mode)
    W = torch.from_numpy((rng.standard_normal((N, K)) * 0.02).astype(np.float32)).to(torch.bfloat16).view(torch.int16).numpy()
    X = rng.standard_normal((n, K)).astype(np.float32)
    Y0 = rng.standard_normal((n, N)).astype(np.float32) if mode == 1 else None
    got = _run(pkg, W, X, mode, Y0)
    want = _ref(W, X, mode, Y0)
    err = np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)
    assert err < 2e-5, err


@pytest.mark.parametrize("n,N,K,splits", [(64, 4096, 1024, 8), (5, 1024, 3072, 12), (64, 12288, 2048, 3), (33, 256, 256, 4)])
def test_tc_gemm_split_k_matches_f64(pkg, n, N, K, splits):
    """Split-K with atomic accumulation (the skinny decode-batch GEMMs)."""
    import torch
    rng = np.random.default_rng(n + N + K + splits)
    W = torch.from_numpy((rng.standard_normal((N, K)) * 0.02).astype(np.float32)).to(torch.bfloat16).view(torch.int16).numpy()
    X = rng.standard_normal((n, K)).astype(np.float32)
    Y0 = rng.standard_normal((n, N)).astype(np.float32)
    got = _run(pkg, W, X, 3, Y0, splits)
    want = _ref(W, X, 3, Y0)
    err = np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)
    assert err < 2e-5, err
