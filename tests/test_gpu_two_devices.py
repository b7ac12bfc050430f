"""process_batch over two GPUs (symbols hashed to their owner device, each
device stepping its own rows, answers merged in the reference's order) against
the same calls on one GPU: same answer order, same predictions. Needs two
visible GPUs; skipped otherwise."""

import numpy as np
import pytest
import torch

from hackathon_b200 import client as CL
from hackathon_b200 import weights as Wt
from tests.conftest import assert_close
from tests.golden import streams

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_devices_answer_like_one():
    cfg = streams.API_CFG
    sd = Wt.generate_model(cfg, seed=0)
    one = CL.B200InferenceClient(num_symbols=24, config=cfg, weights=sd, linear_dtype="fp32", devices=[0])
    two = CL.B200InferenceClient(num_symbols=24, config=cfg, weights=sd, linear_dtype="fp32", devices=[0, 1])
    rng = np.random.default_rng(3)
    uid = 0
    for call in range(4):
        batch = {}
        for s in rng.choice(20, 12, replace=False):
            reqs = []
            for _ in range(int(rng.integers(1, 4))):
                reqs.append(CL.PendingRequest(uid, f"SYM_{int(s):03d}",
                                              rng.standard_normal(cfg.num_features, dtype=np.float32).tolist(), 0.0))
                uid += 1
            batch[f"SYM_{int(s):03d}"] = reqs
        a, b = one.process_batch(batch), two.process_batch(batch)
        assert list(a.unique_ids) == list(b.unique_ids), f"call {call}: answer order"
        assert_close(np.asarray(b.predictions, np.float32), np.asarray(a.predictions, np.float32), 1e-4, 1e-5,
                     f"call {call}")
    assert {e for e, _ in two.symbol_to_idx.values()} == {0, 1}, "both devices own symbols"
    one.close()
    two.close()
