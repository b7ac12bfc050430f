import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libb2e.so")
    config.addinivalue_line("markers", "slow: long-running check")


def pytest_collection_modifyitems(config, items):
    """GPU tests skip (not fail) on a host without CUDA; on a GPU host they run and
    a missing libb2e.so is an error, never a fallback."""
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device on this host")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def load_golden(name):
    g = np.load(GOLDEN / f"{name}.npz")
    return g, json.loads(str(g["meta"]))


def assert_close(got, want, rtol, atol, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    same = (got == want) | (np.isnan(got) & np.isnan(want))
    with np.errstate(invalid="ignore"):
        err = np.where(same, 0.0, np.abs(got - want))
    bound = atol + rtol * np.abs(want)
    bad = ~(err <= bound)
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(bad, err - bound, -np.inf)), err.shape)
        raise AssertionError(f"{what}: {int(bad.sum())} of {err.size} outside rtol={rtol} atol={atol}; "
                             f"worst at {i}: got {got[i]!r} want {want[i]!r} (max abs err {err.max():.3g})")


@pytest.fixture(scope="session")
def golden():
    return load_golden
