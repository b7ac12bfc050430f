"""Pipelined steps (a tower's chain waits only for the same tower's previous step,
so consecutive steps overlap) against the same steps run one at a time.

The pipelined engine and an engine with B2E_FLAG_NO_PIPELINE run the same kernels
on the same inputs, so predictions and state must agree bit for bit. The steps
share most of their slots - a symbol stepped by two consecutive steps is the case
the per-tower ordering must get right - change batch bucket, and (host path) put
one-kernel latency steps between pipelined ones. Dims: the benchmark's D2 with
bf16 weights, and the small test model with fp32 weights.
"""

import numpy as np
import pytest

from hackathon_b200 import _lib
from hackathon_b200 import config as C
from hackathon_b200 import weights as Wt
from hackathon_b200.engine import EnsembleEngine

pytestmark = pytest.mark.gpu

CASES = {"d2-bf16": (C.D2, "bf16", 1024), "small-fp32": (C.SMALL, "fp32", 256)}


def _plan(rows, seed, with_small):
    """Step sizes and slots: full, ragged and smaller buckets over a pool only
    1.5x the batch, so consecutive steps share most of their slots."""
    rng = np.random.default_rng(seed)
    pool = rows + rows // 2
    sizes = [rows, rows, rows - 24, rows // 2 - 7, rows, 3 if with_small else rows // 4, rows, rows - 1, 2 if with_small else 5, rows]
    return pool, [rng.permutation(pool)[:n].astype(np.int32) for n in sizes]


def _engines(cfg, lp, rows, pool):
    sd = Wt.generate_model(cfg, seed=0)
    kw = dict(device=0, linear_dtype=lp, capacity=pool, max_batch=rows)
    return EnsembleEngine(cfg, sd, **kw), EnsembleEngine(cfg, sd, flags=_lib.FLAG_NO_PIPELINE, **kw)


def _state(eng, slots):
    return [np.concatenate([np.asarray(leaf).reshape(-1) for leaf in eng.read_slot(int(s))]) for s in slots]


def _same_state(a, b, pool, rng):
    check = rng.choice(pool, 24, replace=False)
    for s, x, y in zip(check, _state(a, check), _state(b, check)):
        assert np.array_equal(x.view(np.uint8), y.view(np.uint8)), f"slot {s}: state differs"


@pytest.mark.parametrize("case", sorted(CASES))
def test_host_steps_two_in_flight_match_one_by_one(case):
    cfg, lp, rows = CASES[case]
    pool, plan = _plan(rows, 11, with_small=True)
    pipe, ref = _engines(cfg, lp, rows, pool)
    rng = np.random.default_rng(5)
    feats = [rng.standard_normal((len(s), cfg.num_features), dtype=np.float32) for s in plan]
    want = [ref.step(s, f) for s, f in zip(plan, feats)]
    got = []
    pipe.submit(plan[0], feats[0])
    for s, f in zip(plan[1:], feats[1:]):
        pipe.submit(s, f)  # two steps in flight: this one's towers start beside the last one's
        got.append(pipe.wait())
    got.append(pipe.wait())
    for i, (g, w) in enumerate(zip(got, want)):
        assert np.array_equal(g, w), f"step {i} ({len(plan[i])} rows): predictions differ"
    assert pipe.device_error() == 0 and ref.device_error() == 0
    _same_state(pipe, ref, pool, rng)
    pipe.close()
    ref.close()


@pytest.mark.parametrize("case", sorted(CASES))
def test_device_submits_match_step_device(case):
    import torch

    cfg, lp, rows = CASES[case]
    pool, plan = _plan(rows, 12, with_small=False)
    pipe, ref = _engines(cfg, lp, rows, pool)
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(6)
    slots = [torch.from_numpy(s).to(dev) for s in plan]
    feats = [torch.from_numpy(rng.standard_normal((len(s), cfg.num_features), dtype=np.float32)).to(dev) for s in plan]
    out_p = [torch.full((len(s), 4), float("nan"), device=dev) for s in plan]
    out_r = [torch.full((len(s), 4), float("nan"), device=dev) for s in plan]
    st = torch.cuda.current_stream(dev)
    for s, f, o in zip(slots, feats, out_p):
        pipe.submit_device(s, f, o, len(s), stream=st)
    pipe.join_device(stream=st)
    for s, f, o in zip(slots, feats, out_r):
        ref.step_device(s, f, o, len(s), stream=st)
    torch.cuda.synchronize()
    for i, (g, w) in enumerate(zip(out_p, out_r)):
        assert torch.equal(g, w), f"step {i}: predictions differ"
    assert pipe.device_error() == 0 and ref.device_error() == 0
    _same_state(pipe, ref, pool, rng)
    pipe.close()
    ref.close()


def test_device_submit_refuses_bad_slots_on_the_device():
    import torch

    cfg = C.SMALL
    sd = Wt.generate_model(cfg, seed=0)
    eng = EnsembleEngine(cfg, sd, capacity=16, max_batch=8)
    dev = torch.device("cuda:0")
    before = eng.read_slot(3)
    slots = torch.tensor([3, 99], dtype=torch.int32, device=dev)  # 99 is outside the table
    feats = torch.ones(2, cfg.num_features, device=dev)
    preds = torch.empty(2, 4, device=dev)
    eng.submit_device(slots, feats, preds, 2)
    eng.join_device()
    assert eng.device_error() == 1
    after = eng.read_slot(3)
    assert all(np.array_equal(a, b) for a, b in zip(before, after)), "a refused step changed state"
    eng.close()
