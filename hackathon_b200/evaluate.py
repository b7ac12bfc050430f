"""Accuracy harness over a requests parquet: the reference's LocalEvaluator
(local_evaluator.py:19-105) on the B200 client.

The parquet holds one request per row: columns ``feature_*`` (the model inputs,
in column order), ``target_*`` (one per tower), ``symbol`` and ``delay_ms``.
Requests get the row index as unique id and are answered in batches of
``batch_size`` consecutive rows, each batch grouped by symbol in first-seen
order and passed to ``process_batch`` (local_evaluator.py:26-57). The report is
the reference's: response rate, the mean per-batch wall time in ms charged to
each request of the batch, and per tower the max and mean absolute error
against its target (local_evaluator.py:62-93).

Columns are read with pyarrow as whole arrays (no per-row pandas access), and
the feature rows reach ``process_batch`` as float32 rows, which
``B200InferenceClient`` takes as they are.

    python -m hackathon_b200.evaluate --requests-parquet-file tiny.parquet --batch-size 1
"""

from __future__ import annotations

import argparse
import time
from typing import Callable, Dict, List, Optional

import numpy as np

TOWER_NAMES = ("XLSTM", "Mamba2", "RetNet", "Hawk")


class Requests:
    """A requests parquet as arrays: features [n, F] f32, targets [n, T] f64, symbols."""

    def __init__(self, path: str):
        import pyarrow.parquet as pq

        t = pq.read_table(path)
        names = t.schema.names
        fcols = [c for c in names if c.startswith("feature")]
        tcols = [c for c in names if c.startswith("target")]
        # float(row[col]) (local_evaluator.py:31-32), then process_batch's float32
        self.features = np.stack([t.column(c).to_numpy(zero_copy_only=False).astype(np.float64) for c in fcols],
                                 axis=1).astype(np.float32) if fcols else np.zeros((t.num_rows, 0), np.float32)
        self.targets = np.stack([t.column(c).to_numpy(zero_copy_only=False).astype(np.float64) for c in tcols],
                                axis=1) if tcols else np.zeros((t.num_rows, 0))
        self.symbols: List[str] = [str(s) for s in t.column("symbol").to_pylist()]
        self.n = t.num_rows
        # local_evaluator.py:22-23: the symbol names end in a three-digit index
        self.num_symbols = max(int(s[-3:]) for s in set(self.symbols)) + 1 if self.n else 0


def evaluate(req: Requests, process_batch: Callable, batch_size: int = 1, pending_cls=None) -> Dict[str, object]:
    """LocalEvaluator.evaluate_model + _calculate_metrics over `req`."""
    if pending_cls is None:
        from .client import PendingRequest as pending_cls
    predictions: Dict[int, list] = {}
    latency: Dict[int, float] = {}
    now = time.time()
    for i in range(0, req.n, batch_size):
        by_symbol: Dict[str, list] = {}
        for idx in range(i, min(i + batch_size, req.n)):
            by_symbol.setdefault(req.symbols[idx], []).append(
                pending_cls(unique_id=idx, symbol=req.symbols[idx], features=req.features[idx], received_time=now))
        t0 = time.perf_counter()
        resp = process_batch(by_symbol)
        ms = (time.perf_counter() - t0) * 1000
        for uid, pred in zip(resp.unique_ids, resp.predictions):
            predictions[uid] = pred
            latency[uid] = ms
    return metrics(req, predictions, latency)


def metrics(req: Requests, predictions: Dict[int, list], latency: Dict[int, float]) -> Dict[str, object]:
    """_calculate_metrics (local_evaluator.py:62-93)."""
    errs: Dict[int, list] = {}
    lat = []
    for idx in range(req.n):
        if idx not in predictions:
            continue
        p = predictions[idx]
        if len(p) != req.targets.shape[1]:
            raise ValueError(f"request {idx}: {len(p)} predictions for {req.targets.shape[1]} targets")
        for t, (pv, tv) in enumerate(zip(p, req.targets[idx])):
            errs.setdefault(t, []).append(abs(float(pv) - float(tv)))
        lat.append(latency[idx])
    out: Dict[str, object] = {
        "total_requests": req.n,
        "total_responses": len(predictions),
        "response_rate": len(predictions) / req.n if req.n else 0.0,
        "avg_latency_ms": float(np.mean(lat)) if lat else 0,
    }
    for t, e in errs.items():
        out[f"tower_{t}"] = (max(e), float(np.mean(e)))
    return out


def report(m: Dict[str, object]) -> str:
    """LocalEvaluator.print_report's text (local_evaluator.py:95-105)."""
    lines = [f"\nTotal requests: {m['total_requests']:,}", f"Total responses: {m['total_responses']:,}",
             f"Response rate: {m['response_rate']:.2%}", f"Average latency: {m['avg_latency_ms']:.1f} ms",
             "Tower Accuracies:"]
    for t, name in enumerate(TOWER_NAMES):
        if f"tower_{t}" in m:
            mx, mean = m[f"tower_{t}"]
            lines.append(f"{name}: max_error = {mx:.4f}, mean_error = {mean:.4f}")
    return "\n".join(lines)


def main(argv: Optional[List[str]] = None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--requests-parquet-file", type=str, default="tiny.parquet")
    ap.add_argument("--batch-size", type=int, default=1)
    ap.add_argument("--token", type=str, default=None)
    ap.add_argument("--seeded-weights", action="store_true",
                    help="seed-0 weights instead of the reference's checkpoint (no download)")
    a = ap.parse_args(argv)
    from .client import B200InferenceClient
    from .config import D0
    from .weights import generate_model

    req = Requests(a.requests_parquet_file)
    weights = generate_model(D0, seed=0) if a.seeded_weights else None
    client = B200InferenceClient(num_symbols=req.num_symbols, token=a.token, weights=weights)
    print(report(evaluate(req, client.process_batch, a.batch_size)))
    client.close()


if __name__ == "__main__":
    main()
