"""The parquet accuracy harness end to end on the GPU: a synthetic requests
parquet through B200InferenceClient.process_batch at batch sizes 1 and 8; the
per-tower errors equal those of the oracle's predictions for the same requests
(each symbol's requests in row order, whatever the batching)."""

import numpy as np
import pytest

from hackathon_b200 import client as CL
from hackathon_b200 import evaluate as EV
from hackathon_b200 import weights as Wt
from oracle import model as O
from tests.golden import streams
from tests.test_evaluate import write_requests

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch_size", [1, 8])
def test_harness_metrics_equal_the_oracle_predictions(tmp_path, batch_size):
    cfg = streams.API_CFG
    path = tmp_path / "req.parquet"
    write_requests(path, n=40, F=cfg.num_features, n_sym=5, seed=2)
    req = EV.Requests(str(path))
    sd = Wt.generate_model(cfg, seed=0)
    client = CL.B200InferenceClient(num_symbols=req.num_symbols, config=cfg, weights=sd, linear_dtype="fp32")
    got = EV.evaluate(req, client.process_batch, batch_size=batch_size)
    client.close()
    orc = O.Oracle(cfg, sd)
    state = {}
    preds = {}
    for i in range(req.n):
        s = req.symbols[i]
        st = state.get(s, O.init_state(cfg, 1))
        p, state[s] = orc.step(req.features[i:i + 1], st)
        preds[i] = [float(x) for x in p[0]]
    want = EV.metrics(req, preds, {i: 0.0 for i in preds})
    assert got["total_responses"] == req.n and got["response_rate"] == 1.0
    for t in range(4):
        np.testing.assert_allclose(got[f"tower_{t}"], want[f"tower_{t}"], rtol=1e-4, atol=1e-5)


def test_command_line_reports_like_the_reference(tmp_path, capsys):
    """`python -m hackathon_b200.evaluate` at the reference's default dims with
    seeded weights: every request answered, the reference's report layout."""
    path = tmp_path / "req.parquet"
    write_requests(path, n=12, F=79, n_sym=3, seed=5)
    EV.main(["--requests-parquet-file", str(path), "--batch-size", "4", "--seeded-weights"])
    out = capsys.readouterr().out
    assert "Total requests: 12" in out and "Total responses: 12" in out and "Response rate: 100.00%" in out
    for name in EV.TOWER_NAMES:
        assert f"{name}: max_error = " in out
