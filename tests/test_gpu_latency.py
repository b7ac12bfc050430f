"""The latency path (one kernel per step, one thread-block cluster per tower)
against the oracle.

Host steps of at most four rows run as a single kernel instead of the batch
graph (hackathon_b200/csrc/latency.cu). These tests step engines through runs
of 1-4-row steps over recurring slots - and, in one case, a 6-row step on the
batch graph in between, since both paths share the state table - and check the
predictions and every state leaf against the oracle with the float64 arbiter of
tests/arbiter.py: fp32 weights within twice the fp32 oracle's own distance from
float64, bf16 weights tracking the exact CastLinear emulation. Dims: the small
test model, the benchmark's D2, the north-star target's D1 (depth 12), and odd
sizes (hidden 48, Mamba2 head 32 and B/C width 24).
"""

import numpy as np
import pytest

from hackathon_b200 import _lib
from hackathon_b200 import config as C
from hackathon_b200 import weights as Wt
from hackathon_b200.engine import EnsembleEngine
from oracle import model as O
from tests import arbiter as A

pytestmark = pytest.mark.gpu

ODD = C.ModelConfig(hidden_size=48, proj_size=96, tower_depth=1, num_heads=4, num_features=79,
                    mamba_head_size=32, mamba_bc_size=24)
CASES = {"small": C.SMALL, "d2": C.D2, "d1": C.D1, "odd": ODD}
SIZES = (1, 2, 4, 3, 1, 4, 2, 1, 3, 4)


def _steps(capacity, sizes, rng, big=None):
    out = [rng.choice(capacity, n, replace=False).astype(np.int32) for n in sizes]
    if big is not None:  # a step on the batch graph in the middle
        out.insert(len(out) // 2, rng.permutation(capacity)[:big].astype(np.int32))
    return out


def _run(cfg, lp, capacity=6, big=None, seed=7):
    sd = Wt.generate_model(cfg, seed=0)
    rng = np.random.default_rng(seed)
    eng = EnsembleEngine(cfg, sd, device=0, linear_dtype=lp, capacity=capacity, max_batch=8)
    rows, cl = eng.latency_rows()
    # shared memory holds 4 rows at small dims; fewer at hidden 256 (1 row with fp32 weights)
    assert 1 <= rows <= 4 and cl in (8, 16), (rows, cl)
    steps = _steps(capacity, [min(n, rows) for n in SIZES], rng, big)
    feats = [rng.standard_normal((len(s), cfg.num_features), dtype=np.float32) for s in steps]
    got = np.concatenate([eng.step(s, f) for s, f in zip(steps, feats)]).astype(np.float64)
    assert eng.device_error() == 0
    tracked = np.arange(capacity, dtype=np.int32)
    got_s = A.slot_leaves(eng, tracked)
    eng.close()
    return sd, steps, feats, tracked, got, got_s


@pytest.mark.parametrize("case", sorted(CASES))
def test_latency_path_fp32_within_fp32_noise_of_float64(case):
    cfg = CASES[case]
    big = 6 if case == "small" else None
    sd, steps, feats, tracked, got, got_s = _run(cfg, "fp32", big=big)
    o32, o32_s = A.oracle_run(O, cfg, sd, None, steps, tracked, feats)
    o64, o64_s = A.oracle_run(A.O64, cfg, sd, None, steps, tracked, feats)
    A.check_fp32(f"latency {case} fp32", got, got_s, o32, o32_s, o64, o64_s)


@pytest.mark.parametrize("case", sorted(CASES))
def test_latency_path_bf16_follows_castlinear_rounding(case):
    cfg = CASES[case]
    big = 6 if case == "small" else None
    sd, steps, feats, tracked, got, got_s = _run(cfg, "bf16", big=big)
    emu, emu_s = A.oracle_run(O, cfg, sd, "bf16", steps, tracked, feats)
    o32, o32_s = A.oracle_run(O, cfg, sd, None, steps, tracked, feats)
    A.check_bf16(f"latency {case} bf16", got, got_s, emu, emu_s, o32, o32_s)


def test_latency_path_is_one_launch_and_can_be_turned_off():
    cfg = C.SMALL
    sd = Wt.generate_model(cfg, seed=0)
    on = EnsembleEngine(cfg, sd, capacity=4, max_batch=4)
    off = EnsembleEngine(cfg, sd, capacity=4, max_batch=4, flags=_lib.FLAG_NO_LATENCY_PATH)
    assert on.latency_rows()[0] == 4 and on.launches_per_step(1) == 1
    assert off.latency_rows() == (0, 0) and off.launches_per_step(1) > 50
    f = np.random.default_rng(0).standard_normal((2, cfg.num_features), dtype=np.float32)
    a, b = on.step([1, 3], f), off.step([1, 3], f)
    np.testing.assert_allclose(a, b, rtol=1e-4, atol=1e-5)
    on.close()
    off.close()
