"""Each layer at the bench's dims (hidden 256, 8 heads: Mamba2 head 64 with state
128, mLSTM head 64, sLSTM 4 blocks of 64, RetNet head 32) and at odd dims (hidden
48, 4 heads: head sizes 24, 12, Mamba2 state 24, sLSTM blocks of 24) against the
oracle: fp32 weights, a random non-zero start state, masked steps over 40 rows
(so the 16-row tiles of the fused kernels end ragged). The golden layer fixtures
run at hidden 64; the bench's dims select the fused and bulk-streaming kernels at
their real tile shapes, the odd dims every fallback (sLSTM in three kernels,
register-streaming state steps, the one-CTA-per-row mLSTM and Mamba2 post)."""

import numpy as np
import pytest
import torch

from hackathon_b200 import config as C
from hackathon_b200 import weights as Wt
from hackathon_b200.engine import LayerEngine
from oracle import model as O
from tests.conftest import assert_close
from tests.golden import streams

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
CFGS = {"bench": C.ModelConfig(hidden_size=256, proj_size=512, tower_depth=1, num_heads=8, num_features=79),
        "odd": C.ModelConfig(hidden_size=48, proj_size=96, tower_depth=1, num_heads=4, num_features=79,
                             mamba_head_size=32, mamba_bc_size=24)}
RTOL, ATOL = 1e-4, 1e-5  # check_kernels.py:78


def _start_state(tag, CFG, batch, rng):
    st = O.init_block_state(tag, CFG, batch)
    for i, leaf in enumerate(st):
        if leaf.dtype != np.float32:
            leaf[...] = rng.integers(0, 50, leaf.shape)
        elif tag == "retnet" and i == 1:  # decay-normaliser scales stay positive
            leaf[...] = 1.0 + rng.random(leaf.shape).astype(np.float32)
        else:
            leaf[...] = rng.standard_normal(leaf.shape).astype(np.float32) * np.float32(0.5)
    return st


@pytest.mark.parametrize("dims", sorted(CFGS))
@pytest.mark.parametrize("tag", ["xlstm", "mamba2", "retnet", "hawk"])
def test_layer_at_bench_dims_matches_oracle(tag, dims):
    CFG = CFGS[dims]
    batch, steps = 40, 4
    sd = Wt.generate(Wt.layer_specs(tag, "", CFG), seed=3)
    eng = LayerEngine(tag, CFG, sd, capacity=batch, max_batch=batch)
    W = O.Weights(sd)
    rng = np.random.default_rng(9)
    st = _start_state(tag, CFG, batch, rng)
    for row in range(batch):
        eng.write_slot(row, [leaf[row] for leaf in st])
    xs = rng.standard_normal((steps, batch, CFG.hidden_size), dtype=np.float32)
    masks = streams.step_masks(steps, batch, rng)
    y = torch.empty(batch, CFG.hidden_size, device=DEV)
    for s in range(steps):
        rows = np.nonzero(masks[s])[0]
        slots = torch.from_numpy(rows.astype(np.int32)).to(DEV)
        eng.step_device(slots, torch.from_numpy(xs[s][rows]).to(DEV), y)
        torch.cuda.synchronize()
        want, new = O.layer_step(tag, W, xs[s][rows], [leaf[rows] for leaf in st], CFG)
        for leaf, nl in zip(st, new):
            leaf[rows] = nl
        assert_close(y[:len(rows)].cpu().numpy(), want, RTOL, ATOL, f"{tag} y step {s}")
    for row in range(batch):
        for i, (got, want) in enumerate(zip(eng.read_slot(row), st)):
            assert_close(got, want[row], RTOL, ATOL, f"{tag} slot {row} leaf {i}")
    eng.close()
