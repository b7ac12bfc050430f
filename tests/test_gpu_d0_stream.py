"""BASELINE config 1 on the GPU at the default dims (hidden 2048, proj 4096, depth
12): 10,000 requests, one per process_batch call, symbols SYM_001..SYM_016
round-robin, fp32 weights, against the reference's own outputs
(tests/golden/d0stream.npz, made by make_golden.py d0stream from the reference
model with the same seeded weights): every prediction, and a summary (sum, sum of
squares, 32 samples) of every state leaf of every symbol at the end.
"""

import numpy as np
import pytest

from hackathon_b200 import config as C
from hackathon_b200 import weights as Wt
from hackathon_b200.engine import EnsembleEngine
from tests.conftest import load_golden
from tests.golden import streams

pytestmark = pytest.mark.gpu

# fp32 at depth 12 with K = 2048/4096 dot products: summation order (torch CPU
# BLAS in the reference, tensor-free fp32 kernels here) moves predictions by a few
# 1e-4 relative. The numpy oracle, another fp32 restatement, already differs from
# the reference by 1.6e-4 (absolute, on a prediction of 0.544) at the stream's
# first request; the engine's worst over the 10,000 requests measures 4.6e-4.
RTOL, ATOL = 2e-3, 2e-3


def test_d0_stream_matches_reference():
    g, meta = load_golden("d0stream")
    n = meta["n_requests"]
    sd = Wt.generate_model(C.D0, seed=meta["weight_seed"])
    eng = EnsembleEngine(C.D0, sd, linear_dtype="fp32", capacity=streams.D0_SYMBOLS, max_batch=1)
    del sd
    feats = streams.d0_features(n)
    assert abs(float(feats.astype(np.float64).sum()) - meta["input_sum"]) < 1e-6 * max(1.0, abs(meta["input_sum"]))
    preds = np.empty((n, 4), np.float32)
    for i in range(n):
        preds[i] = eng.step(np.array([i % streams.D0_SYMBOLS], np.int32), feats[i:i + 1])[0]
    assert eng.device_error() == 0
    want = g["preds"]
    err = np.abs(preds.astype(np.float64) - want) / (np.abs(want) + ATOL / RTOL)
    assert np.all(np.isfinite(preds))
    print(f"d0 stream: max relative prediction error {float(err.max()):.3g}")
    assert float(err.max()) <= RTOL, f"worst prediction error {float(err.max()):.3g} at {np.unravel_index(err.argmax(), err.shape)}"
    for s in range(streams.D0_SYMBOLS):
        leaves = eng.read_slot(s)
        for j, leaf in enumerate(leaves):
            got = streams.leaf_summary(np.asarray(leaf, dtype=np.float32))
            ref = g[f"sym{s}_leaf{j}"]
            assert got.shape == ref.shape
            # sums over a leaf: relative to the leaf's scale (sqrt of its sum of squares times its size)
            scale = np.sqrt(max(ref[1], 1e-30) * max(leaf.size, 1))
            assert abs(got[0] - ref[0]) <= RTOL * scale + ATOL, f"sym {s} leaf {j} sum"
            assert abs(got[1] - ref[1]) <= RTOL * abs(ref[1]) + ATOL, f"sym {s} leaf {j} sum of squares"
            np.testing.assert_allclose(got[2:], ref[2:], rtol=RTOL, atol=ATOL, err_msg=f"sym {s} leaf {j} samples")
    eng.close()
