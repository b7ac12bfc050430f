"""The parquet accuracy harness (hackathon_b200/evaluate.py) on the CPU: the
reference LocalEvaluator's batching and metrics (local_evaluator.py:26-105) on a
synthetic requests parquet of the same schema, with a stand-in process_batch."""

import numpy as np
import pyarrow as pa
import pyarrow.parquet as pq

from hackathon_b200 import evaluate as EV


def write_requests(path, n=37, F=79, n_sym=5, seed=0):
    rng = np.random.default_rng(seed)
    cols = {f"feature_{i:02d}": rng.standard_normal(n).astype(np.float32) for i in range(F)}
    cols["delay_ms"] = rng.random(n)
    for t in range(4):
        cols[f"target_{t:02d}"] = rng.standard_normal(n)
    cols["symbol"] = [f"SYM_{int(s):03d}" for s in rng.integers(1, n_sym + 1, n)]
    pq.write_table(pa.table(cols), path)
    return cols


class _Resp:
    def __init__(self, u, p):
        self.unique_ids, self.predictions = u, p


def test_batches_group_by_symbol_in_first_seen_order_and_metrics_match(tmp_path):
    path = tmp_path / "req.parquet"
    cols = write_requests(path)
    req = EV.Requests(str(path))
    assert req.n == 37 and req.features.shape == (37, 79)
    assert req.num_symbols == max(int(s[-3:]) for s in set(cols["symbol"])) + 1
    seen = []

    def pb(by_symbol):
        seen.append([(s, [r.unique_id for r in rs]) for s, rs in by_symbol.items()])
        uids, preds = [], []
        for s, rs in by_symbol.items():
            for r in rs:
                if r.unique_id % 11 == 5:  # a request left unanswered
                    continue
                uids.append(r.unique_id)
                preds.append([float(np.sum(r.features)) * k for k in (1.0, -0.5, 0.25, 2.0)])
        return _Resp(uids, preds)

    m = EV.evaluate(req, pb, batch_size=6)
    # batches of 6 consecutive rows, symbols in first-seen order within each
    for b, batch in enumerate(seen):
        rows = list(range(6 * b, min(6 * b + 6, 37)))
        want = {}
        for i in rows:
            want.setdefault(cols["symbol"][i], []).append(i)
        assert batch == list(want.items())
    answered = [i for i in range(37) if i % 11 != 5]
    assert m["total_requests"] == 37 and m["total_responses"] == len(answered)
    assert m["response_rate"] == len(answered) / 37
    feats = np.stack([cols[f"feature_{i:02d}"] for i in range(79)], 1).astype(np.float32)
    for t, k in enumerate((1.0, -0.5, 0.25, 2.0)):
        e = [abs(float(np.sum(feats[i])) * k - float(cols[f"target_{t:02d}"][i])) for i in answered]
        assert m[f"tower_{t}"] == (max(e), float(np.mean(e)))
    text = EV.report(m)
    assert "Response rate:" in text and "XLSTM: max_error = " in text and "Hawk: max_error = " in text
