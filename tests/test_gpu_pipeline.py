"""Two host steps in flight on one engine (b2e_engine_submit twice, then
b2e_engine_wait): the second step's input copies overlap the first step, and the
results equal one-step-at-a-time stepping bit for bit, also when consecutive
steps share symbols (the state dependency that orders them)."""

import numpy as np
import pytest

from hackathon_b200 import _lib
from hackathon_b200 import config as C
from hackathon_b200 import weights as Wt
from hackathon_b200.engine import EnsembleEngine

pytestmark = pytest.mark.gpu
CFG = C.ModelConfig(hidden_size=64, proj_size=128, tower_depth=2, num_heads=4, num_features=79)
CAP = 400


def _workload(steps, seed=6):
    rng = np.random.default_rng(seed)
    out = []
    for k in range(steps):
        n = int(rng.integers(200, 320)) if k % 3 else int(rng.integers(1, 40))
        slots = rng.choice(330 if k % 2 else CAP, n, replace=False).astype(np.int32)  # symbols recur
        out.append((slots, rng.standard_normal((n, CFG.num_features), dtype=np.float32)))
    return out


def test_two_host_steps_in_flight_equal_sequential_steps():
    sd = Wt.generate_model(CFG, seed=3)
    a = EnsembleEngine(CFG, sd, capacity=CAP, max_batch=512)
    b = EnsembleEngine(CFG, sd, capacity=CAP, max_batch=512)
    work = _workload(6, seed=8)
    want = [a.step(s, f) for s, f in work]
    got = []
    b.submit(*work[0])
    for k in range(1, len(work)):
        b.submit(*work[k])
        if k == 1:
            with pytest.raises(_lib.B2EError):
                b.submit(*work[0])  # a third step in flight is refused
        got.append(b.wait())
    got.append(b.wait())
    for k, (x, y) in enumerate(zip(want, got)):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32)), f"step {k}"
    with pytest.raises(_lib.B2EError):
        b.wait()  # nothing in flight
    a.close()
    b.close()


@pytest.mark.parametrize("lanes", [1, 2])
def test_device_and_host_steps_interleave_in_step_order(lanes):
    """Device-buffer steps (on a torch stream) between host steps: each step sees
    the state the one before it left, whichever path either took."""
    import torch

    dev = torch.device("cuda", 0)
    sd = Wt.generate_model(CFG, seed=3)
    a = EnsembleEngine(CFG, sd, capacity=CAP, max_batch=512, lanes=lanes)
    b = EnsembleEngine(CFG, sd, capacity=CAP, max_batch=512, lanes=lanes)
    work = _workload(8, seed=9)
    want = [a.step(s, f) for s, f in work]
    got = []
    for k, (s, f) in enumerate(work):
        if k % 3 == 1:
            p = torch.empty(len(s), 4, device=dev)
            b.step_device(torch.from_numpy(s).to(dev), torch.from_numpy(f).to(dev), p, len(s))
            got.append(p.cpu().numpy())
        else:
            b.submit(s, f)
            got.append(b.wait())
    for k, (x, y) in enumerate(zip(want, got)):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32)), f"step {k}"
    a.close()
    b.close()
