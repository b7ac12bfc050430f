"""Seeded input streams shared by the fixture generator and the tests.

Both sides regenerate the inputs from these functions (numpy PCG64), so the
fixtures only store what the reference computed plus a checksum of the inputs.
"""

from __future__ import annotations

from typing import Dict, Iterator, List, Tuple

import numpy as np

from hackathon_b200 import config as C

F32 = np.float32

# check_kernels.py:142-158 shapes: (batch, (heads, size_h, size_k)); the ragged
# ones are off every power-of-two tile.
CELL_CASES = {
    "mlstm": [(6, (4, 32, 32)), (5, (3, 48, 80)), (3, (2, 64, 64))],
    "retnet": [(6, (4, 32, 32)), (6, (4, 16, 16)), (5, (3, 48, 80))],
    "mamba2": [(6, (8, 16, 32)), (6, (8, 16, 24)), (6, (2, 64, 128)), (5, (5, 40, 96))],
}


def _rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def cell_masks(batch: int, rng) -> Dict[str, object]:
    """check_kernels.py:161-168: mixed (first live, last idle), all-true, all-false, none."""
    mixed = rng.random(batch) < 0.5
    mixed[0], mixed[-1] = True, False
    return {"mixed": mixed, "alltrue": np.ones(batch, bool), "allfalse": np.zeros(batch, bool), "none": None}


def cell_inputs(tag: str, batch: int, dims, seed: int):
    """check_kernels.py:96-135: states N(0,1), gates/decays U(0,1), k scaled by h^-1/2."""
    rng = _rng(seed)
    n, sh, sk = dims
    rnd = lambda *s: rng.standard_normal(s, dtype=F32)  # noqa: E731
    uni = lambda *s: rng.random(s, dtype=F32)  # noqa: E731
    state = rnd(batch, n, sh, sk)
    if tag == "mlstm":  # q, k, v, i_gate, f_gate
        rest = (rnd(batch, n, sh), (rnd(batch, n, sh) * F32(sh ** -0.5)).astype(F32), rnd(batch, n, sk),
                uni(batch, n), uni(batch, n))
    elif tag == "retnet":  # k_rope, v, q_scaled, decay
        rest = ((rnd(batch, n, sh) * F32(sh ** -0.5)).astype(F32), rnd(batch, n, sk), rnd(batch, n, sh), uni(n))
    elif tag == "mamba2":  # x, b, c, dt, decay
        rest = (rnd(batch, n, sh), rnd(batch, sk), rnd(batch, sk), uni(batch, n), uni(batch, n))
    else:
        raise ValueError(tag)
    return state, rest, cell_masks(batch, rng)


# Layer cases of check_cell_rewrite.py:272-278: hidden 64; xLSTM with 4 mLSTM
# and 2 sLSTM heads, Mamba2(64, head_size=16, bc_head_size=24), RetNet 4 heads.
LAYER_CFG = C.ModelConfig(hidden_size=64, proj_size=128, tower_depth=1, num_heads=4, num_features=7,
                          mamba_head_size=16, mamba_bc_size=24)
LAYER_CASES = {tag: (LAYER_CFG, 12, 6) for tag in ("xlstm", "mamba2", "retnet", "hawk")}


def step_masks(steps: int, batch: int, rng) -> np.ndarray:
    """check_cell_rewrite.py:171-174: random, row 0 live and row 1 idle."""
    m = rng.random((steps, batch)) < 0.5
    m[:, 0], m[:, 1] = True, False
    return m


def layer_stream(tag: str, cfg: C.ModelConfig, steps: int, batch: int, seed: int):
    rng = _rng(seed)
    xs = rng.standard_normal((steps, batch, cfg.hidden_size), dtype=F32)
    return xs, step_masks(steps, batch, rng)


MODEL_CASE = (C.SMALL, 8, 6)  # check_cell_rewrite.py:265-269, 6 steps there


def model_stream(cfg: C.ModelConfig, steps: int, batch: int, seed: int):
    rng = _rng(seed)
    feats = rng.standard_normal((steps, batch, cfg.num_features), dtype=F32)
    return feats, step_masks(steps, batch, rng)


LONG_CASE = (C.ModelConfig(hidden_size=64, proj_size=128, tower_depth=2, num_heads=4, num_features=79),
             10_000, 4)


def long_features(cfg: C.ModelConfig, batch: int, seed: int) -> Iterator[np.ndarray]:
    rng = _rng(seed)
    while True:
        yield rng.standard_normal((batch, cfg.num_features), dtype=F32)


API_CFG = C.ModelConfig(hidden_size=64, proj_size=128, tower_depth=2, num_heads=4, num_features=79)
API_CAPACITY = 4


def api_calls(cfg: C.ModelConfig) -> List[List[Tuple[str, List[Tuple[int, list]]]]]:
    """process_batch inputs: several symbols, queued requests of unequal length,
    an empty list, and more distinct symbols than the capacity (overflow)."""
    rng = _rng(21)
    uid = [0]

    def reqs(n):
        out = []
        for _ in range(n):
            out.append((uid[0], rng.standard_normal(cfg.num_features, dtype=F32).astype(float).tolist()))
            uid[0] += 1
        return out

    return [
        [("SYM_002", reqs(1))],
        [("SYM_007", reqs(3)), ("SYM_002", reqs(2)), ("SYM_001", [])],
        [("SYM_001", reqs(1)), ("SYM_009", reqs(2)), ("SYM_011", reqs(1)), ("SYM_007", reqs(1))],
        [("SYM_011", reqs(2)), ("SYM_002", reqs(1))],
    ]


D0_SYMBOLS = 16


def d0_features(n: int) -> np.ndarray:
    """BASELINE config 1 features: n x 79 N(0,1) float32, seed 0."""
    return _rng(0).standard_normal((n, 79), dtype=F32)


def d0_symbol(i: int) -> str:
    return f"SYM_{i % D0_SYMBOLS + 1:03d}"


SAMPLES = 32


def sample_index(n: int) -> np.ndarray:
    return np.unique(np.linspace(0, n - 1, num=min(SAMPLES, n)).astype(np.int64))


def leaf_summary(a: np.ndarray) -> np.ndarray:
    """float64 [sum, sum of squares, then SAMPLES evenly spaced elements]."""
    a = a.reshape(-1)
    fin = np.isfinite(a)
    s = np.array([np.sum(a[fin], dtype=np.float64), np.sum(np.square(a[fin], dtype=np.float64))])
    return np.concatenate([s, a[sample_index(a.size)].astype(np.float64)])


# BASELINE configs 2 and 3 (single-layer micro-benchmarks, hackathon_b200.weights.micro_layer):
# all rows active, layer inputs N(0,1)
MICRO_STEPS, MICRO_BATCH, MICRO_SEED = 24, 4, 31


def micro_inputs(kind: str, steps: int = MICRO_STEPS, batch: int = MICRO_BATCH, seed: int = MICRO_SEED) -> np.ndarray:
    from hackathon_b200.weights import MICRO_CONFIGS

    h = MICRO_CONFIGS[kind].hidden_size
    return _rng(seed).standard_normal((steps, batch, h), dtype=F32)


# default dims, 256 symbols, one N(0,1) request each per step
D0_BATCH = 256
D0_BATCH_ROWS = 16  # rows the fixture follows (rows are independent)
D0_BATCH_ARBITER = 4  # of those, rows also run in float64


def d0_batch_features(step: int) -> np.ndarray:
    """Config 4's features of one step: 256 x 79 N(0,1) float32, seed (4, step)."""
    return np.random.default_rng([4, step]).standard_normal((D0_BATCH, 79), dtype=F32)
