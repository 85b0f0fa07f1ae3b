import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(REPO, "tests", "golden")
sys.path.insert(0, REPO)

import __graft_entry__ as ge  # noqa: E402

# Parity bar (from the benchmark contract): greedy tokens identical wherever the
# reference's top-2 margin exceeds MARGIN; final-layer logits within MAX_ABS
# max-abs and REL_L2 relative L2.
MARGIN = 1e-2
MAX_ABS = 2e-2
REL_L2 = 1e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: long-running (full-size shapes)")


@pytest.fixture(scope="session")
def pkg():
    return ge.load_package()


@pytest.fixture(scope="session")
def synth():
    return ge.load_synth()


def golden(name):
    return dict(np.load(os.path.join(GOLDEN, f"ref_{name}.npz")))


def has_gpu():
    try:
        return ge.load_package().device_count() > 0
    except Exception:
        return False


def assert_logits_close(got, want, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    d = np.abs(got - want).max()
    rel = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    assert d <= MAX_ABS and rel <= REL_L2, f"{what}: max|d|={d:.3g} rel_l2={rel:.3g}"
    return d, rel
