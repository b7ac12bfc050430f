"""BASELINE configs 2 and 3 on the GPU: the Mamba2 layer at d_state 64 with its
stated a / dt fills, RetNet with four 64-wide heads and gamma_h = 1 - 2^(-5-h),
and the xLSTM layer whose mLSTM cell has four 64-wide heads
(hackathon_b200.weights.micro_layer).

* Against the reference itself (tests/golden/micro.npz: the reference's layers
  in float32 and float64 over 24 steps of 4 rows): with fp32 weights the
  engine's worst row error against float64 is within twice the reference fp32's
  (never required below 1e-4), on every output row and final state leaf.
* At the micro-benchmark's own shape (4096 symbols, the batch the state kernels
  stream in bulk): three steps, a sample of rows against the oracle in float32
  and float64 (fp32 weights), and against the oracle's exact CastLinear
  emulation (bf16 weights: the MSE to it at most a quarter of the MSE bf16
  weights make against fp32).
"""

import numpy as np
import pytest
import torch

from hackathon_b200 import weights as Wt
from hackathon_b200.engine import LayerEngine
from oracle import model as O
from tests import arbiter as A
from tests.conftest import load_golden
from tests.golden import streams

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
KINDS = ["mamba2", "retnet", "xlstm"]


def _engine_run(kind, cfg, sd, lp, xs, slots):
    """Layer outputs of `slots` rows per step, and every slot's final leaves."""
    n = len(slots)
    eng = LayerEngine(kind, cfg, sd, linear_dtype=lp, capacity=int(slots.max()) + 1, max_batch=n)
    st = torch.from_numpy(slots.astype(np.int32)).to(DEV)
    y = torch.empty(n, cfg.hidden_size, device=DEV)
    ys = []
    for s in range(xs.shape[0]):
        eng.step_device(st, torch.from_numpy(xs[s]).to(DEV), y)
        torch.cuda.synchronize()
        ys.append(y.cpu().numpy().copy())
    return eng, np.stack(ys)


@pytest.mark.parametrize("kind", KINDS)
def test_micro_layer_against_the_reference_with_float64_arbiter(kind):
    g, meta = load_golden("micro")
    cfg, sd = Wt.micro_layer(kind, seed=0)
    xs = streams.micro_inputs(kind)
    eng, ys = _engine_run(kind, cfg, sd, "fp32", xs, np.arange(xs.shape[1]))
    e, o = A.check_fp32_rows(f"{kind} outputs", ys, g[f"{kind}_f32_y"], g[f"{kind}_f64_y"])
    print(f"{kind}: worst row error against float64 {e:.3g} (reference fp32 {o:.3g})")
    leaves = A.slot_leaves(eng, range(xs.shape[1]))
    nl = len(leaves)
    A.check_fp32_leaves(kind, leaves, [g[f"{kind}_f32_state{i}"] for i in range(nl)],
                        [g[f"{kind}_f64_state{i}"] for i in range(nl)])
    eng.close()


def _oracle_rows(mod, kind, cfg, sd, lp, xs, rows):
    W = mod.Weights(sd, lp=lp)
    st = mod.init_block_state(kind, cfg, len(rows))
    ys = []
    for s in range(xs.shape[0]):
        y, st = mod.layer_step(kind, W, xs[s][rows], st, cfg)
        ys.append(y)
    return np.stack(ys).astype(np.float64), [leaf.astype(np.float64) for leaf in st]


@pytest.mark.parametrize("kind", KINDS)
def test_micro_layer_at_4096_symbols(kind):
    cfg, sd = Wt.micro_layer(kind, seed=0)
    rng = np.random.default_rng(5)
    xs = rng.standard_normal((3, 4096, cfg.hidden_size), dtype=np.float32)
    slots = rng.permutation(4096).astype(np.int32)
    rows = np.r_[0, 1, 31, 32, 127, 128, 4095, rng.choice(4096, 25, replace=False)]
    rows = np.unique(rows)
    o32, o32_s = _oracle_rows(O, kind, cfg, sd, None, xs, rows)
    o64, o64_s = _oracle_rows(A.O64, kind, cfg, sd, None, xs, rows)
    eng, ys = _engine_run(kind, cfg, sd, "fp32", xs, slots)
    A.check_fp32_rows(f"{kind} 4096 fp32", ys[:, rows], o32, o64)
    got_s = A.slot_leaves(eng, slots[rows])
    A.check_fp32_leaves(f"{kind} 4096 fp32", got_s, o32_s, o64_s)
    eng.close()
    emu, emu_s = _oracle_rows(O, kind, cfg, sd, "bf16", xs, rows)
    eng, ys = _engine_run(kind, cfg, sd, "bf16", xs, slots)
    got = ys[:, rows].astype(np.float64)
    dev = float(np.mean((got - emu) ** 2))
    quant = float(np.mean((emu - o32) ** 2))
    print(f"{kind} 4096 bf16: MSE to the emulation {dev:.3g}, bf16 vs fp32 {quant:.3g}")
    assert dev <= max(0.25 * quant, float(np.mean(emu ** 2)) * A.FLOOR ** 2)
    got_s = A.slot_leaves(eng, slots[rows])
    for li, want in enumerate(emu_s):
        gl = np.asarray(got_s[li])
        if not np.issubdtype(gl.dtype, np.floating):
            assert np.array_equal(gl.astype(np.float64), want), f"{kind} integer leaf {li}"
            continue
        d = float(np.mean((gl.astype(np.float64) - want) ** 2))
        q = float(np.mean((want - o32_s[li]) ** 2))
        assert d <= max(0.5 * q, float(np.mean(want ** 2)) * A.FLOOR ** 2), f"{kind} leaf {li}: {d:.3g} vs {q:.3g}"
    eng.close()
