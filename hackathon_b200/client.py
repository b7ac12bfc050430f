"""Drop-in inference client: the reference's ``process_batch`` on the B200 engine.

``B200InferenceClient`` replaces ``NnInferenceClient`` (example_model.py:248-949)
behind the same constructor and the same ``process_batch(requests_by_symbol) ->
InferenceResponse`` (client.py:88-92). Its semantics are the reference's:

* Requests are answered in rounds: round k takes the k-th queued request of every
  symbol that has one, so each symbol appears at most once per round and its
  requests reach the model in list order (example_model.py:885-899). Answers
  come out round by round, in the dict's symbol order within a round.
* A symbol gets a state slot on first sight and keeps it for the life of the
  process (example_model.py:724-767). When the slots run out, that symbol's
  requests are answered with four zeros and a warning prints once
  (example_model.py:750-764, 831-838).
* Every prediction is a list of 4 Python floats, one per tower in the order
  xLSTM, Mamba2, RetNet, Hawk (model/inference_model.py:107-112, 142-143).

What changes is underneath: rows are stepped on the GPU by libb2e.so against a
slot-indexed state table, so a round costs the live rows only (no masked pass
over all rows, no state blend), and symbols can be spread over several GPUs by
a stable hash of the symbol name, each GPU holding its own symbols' state (a
symbol whose home GPU is full takes a slot on another one).
"""

from __future__ import annotations

import importlib
import itertools
import math
import os
import time
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import batcher as B
from .config import D0, TOWER_KINDS, ModelConfig


def _reference_module(name: str, attr: str):
    """The reference's own module (client / protocol) when it is importable."""
    try:
        mod = importlib.import_module(name)
    except Exception:
        return None
    return mod if hasattr(mod, attr) else None


_rclient = _reference_module("client", "BaseInferenceClient")
_rproto = _reference_module("protocol", "InferenceResponse")

if _rproto is not None:
    InferenceResponse = _rproto.InferenceResponse
else:

    @dataclass
    class InferenceResponse:  # protocol.py:38-44
        unique_ids: list
        predictions: list
        client_timestamp: float
        message_type: str = "inference_response"


if _rclient is not None:
    PendingRequest = _rclient.PendingRequest
    _Base = _rclient.BaseInferenceClient
else:

    @dataclass
    class PendingRequest:  # client.py:28-39
        unique_id: int
        symbol: str
        features: List[float]
        received_time: float

        def age_ms(self) -> float:
            return (time.time() - self.received_time) * 1000

    class _Base:
        """Stands in for client.BaseInferenceClient when the reference client is
        not on the path: same constructor fields, no networking."""

        def __init__(self, num_symbols: int, server_host: str = "localhost", server_port: int = 8080,
                     max_queue_size: int = 100):
            self.num_symbols = num_symbols
            self.server_host = server_host
            self.server_port = server_port
            self.max_queue_size = max_queue_size

        def run(self):
            raise NotImplementedError("the reference's client.py provides the socket loop")


LINEAR_DTYPES = ("bf16", "fp16", "fp32")  # example_model.py:151-156
DEFAULT_LINEAR_DTYPE = "fp16"            # example_model.py:157


def owner_device(symbol: str, n_devices: int) -> int:
    """Home device of a symbol name: the bench's sharding rule (splitmix64 mod
    the device count) over the name's crc32 key."""
    if n_devices <= 1:
        return 0
    return int(B.owner(np.asarray([B.symbol_key(symbol)], np.int64), n_devices)[0])


def load_reference_weights(token: Optional[str] = None) -> Dict[str, np.ndarray]:
    """The reference's checkpoint (example_model.py:296-302), as float32 arrays."""
    from huggingface_hub import hf_hub_download  # imported only when asked for
    import torch

    path = hf_hub_download(repo_id="jane-street-gpu-mode/hackathon", filename="state_dict.pt", token=token)
    sd = torch.load(path, weights_only=True, map_location="cpu")
    return {k: v.float().numpy() for k, v in sd.items()}


def _load_rows():
    """lib/_b2e_rows (csrc/rows.c, built beside libb2e.so), or None if absent."""
    import importlib.util
    import sysconfig
    from pathlib import Path

    path = Path(__file__).resolve().parent / "lib" / ("_b2e_rows" + sysconfig.get_config_var("EXT_SUFFIX"))
    if not path.exists():
        return None
    spec = importlib.util.spec_from_file_location("_b2e_rows", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


_ROWS = _load_rows()


def _feature_rows(feats, nf: int) -> np.ndarray:
    """np.asarray(feats, float32) of rows of nf values (example_model.py:854-855):
    the same float32 values. The native helper walks the Python lists in ~1 ms
    for 4096 rows of 79; without it (or for input it refuses) np.fromiter over
    the chained lists, ~10 ms, or numpy's own conversion, which raises for a row
    of another length as the reference's reshape does."""
    if _ROWS is not None:
        out = np.empty((len(feats), nf), dtype=np.float32)
        try:
            _ROWS.rows_f32(feats, nf, out)
            return out
        except (TypeError, ValueError):
            pass  # numpy's path below gives the reference's behaviour for this input
    if all(len(f) == nf for f in feats):
        return np.fromiter(itertools.chain.from_iterable(feats), dtype=np.float32,
                           count=len(feats) * nf).reshape(len(feats), nf)
    return np.asarray(feats, dtype=np.float32).reshape(len(feats), nf)


class B200InferenceClient(_Base):
    """process_batch on libb2e.so; see the module docstring."""

    _overflow_warned = False  # once per process, like the reference

    def __init__(self, num_symbols: int, server_host: str = "localhost", server_port: int = 8080,
                 device: Optional[str] = None, token: Optional[str] = None, *, config: ModelConfig = D0,
                 weights: Optional[Dict[str, np.ndarray]] = None, linear_dtype: Optional[str] = None,
                 devices: Optional[Sequence[int]] = None, per_device_capacity: Optional[int] = None,
                 max_batch: Optional[int] = None, graphs: bool = True):
        super().__init__(num_symbols, server_host, server_port)
        if linear_dtype is None:
            linear_dtype = os.environ.get("LINEAR_DTYPE", DEFAULT_LINEAR_DTYPE).strip().lower()
            if linear_dtype not in LINEAR_DTYPES:
                print(f"LINEAR_DTYPE={linear_dtype!r} is not one of {sorted(LINEAR_DTYPES)}; "
                      f"falling back to {DEFAULT_LINEAR_DTYPE}")
                linear_dtype = DEFAULT_LINEAR_DTYPE
        if devices is None:
            dev = 0
            if device is not None and ":" in str(device):
                dev = int(str(device).split(":")[1])
            devices = [dev]
        self.devices = list(devices)
        self.config = config
        self.capacity = int(num_symbols)
        nd = len(self.devices)
        if per_device_capacity is None:
            per_device_capacity = self.capacity if nd == 1 else int(math.ceil(self.capacity * 1.25 / nd)) + 4
        if per_device_capacity * nd < self.capacity:
            raise ValueError(f"{nd} devices x {per_device_capacity} slots hold fewer than num_symbols="
                             f"{self.capacity} symbols")
        self.per_device_capacity = per_device_capacity
        if max_batch is None:
            max_batch = max(1, min(per_device_capacity, 4096))
        self.max_batch = max_batch
        if weights is None:
            weights = load_reference_weights(token)
        self.engines = [self._make_engine(config, weights, d, linear_dtype, per_device_capacity, max_batch, graphs)
                        for d in self.devices]
        self.num_outputs = len(TOWER_KINDS)
        self.num_features = config.num_features
        self.symbol_to_idx: Dict[str, tuple] = {}  # symbol -> (engine index, slot)
        self._used = [0] * nd
        print(f"Ready: {self.capacity} symbol slots over {nd} device(s), weights {linear_dtype}")

    @staticmethod
    def _make_engine(config, weights, device, linear_dtype, capacity, max_batch, graphs):
        from .engine import EnsembleEngine

        return EnsembleEngine(config, weights, device=device, linear_dtype=linear_dtype, capacity=capacity,
                              max_batch=max_batch, graphs=graphs)

    def _row_for(self, symbol: str):
        """(engine, slot) that `symbol` owns, taking the next free slot on first sight.

        A new symbol goes to its home device (``owner_device``); when that device's
        slots are all taken it goes to the device with the most free slots, so, as
        in the reference (example_model.py:750-764), requests are answered with
        zeros only once `num_symbols` distinct symbols hold every slot."""
        loc = self.symbol_to_idx.get(symbol)
        if loc is not None:
            return loc
        e = owner_device(symbol, len(self.engines))
        if self._used[e] >= self.per_device_capacity:
            e = min(range(len(self.engines)), key=lambda d: (self._used[d], d))
        if len(self.symbol_to_idx) >= self.capacity or self._used[e] >= self.per_device_capacity:
            if not B200InferenceClient._overflow_warned:
                B200InferenceClient._overflow_warned = True
                print(f"WARNING: out of state rows ({self.capacity} of them, all owned); {symbol!r} and every "
                      f"later new symbol are being answered with zeros, which is wrong but keeps the rest of the "
                      f"batch alive. Raise --num-symbols above the size of the live universe. This prints once.")
            return None
        loc = (e, self._used[e])
        self._used[e] += 1
        self.symbol_to_idx[symbol] = loc
        return loc

    def _run_round(self, locs: List[tuple], feats: np.ndarray) -> np.ndarray:
        """Step one round's rows (distinct symbols) on their engines; preds in row order."""
        return self._run_rounds([(locs, feats)])[0]

    def _run_rounds(self, rounds: List[tuple]) -> List[np.ndarray]:
        """Step rounds of (locs, feats) in order; preds per round in row order.
        Each engine's steps are its chunks of each round, in round order, with
        up to two in flight (b2e_engine_submit / b2e_engine_wait): a symbol's
        next round runs after its previous one on the GPU (same engine, same
        order), and the devices run side by side."""
        out = [np.empty((len(locs), self.num_outputs), np.float32) for locs, _ in rounds]
        queue: Dict[int, List[tuple]] = {}
        for k, (locs, feats) in enumerate(rounds):
            by_engine: Dict[int, List[int]] = {}
            for i, (e, _) in enumerate(locs):
                by_engine.setdefault(e, []).append(i)
            for e, rows in by_engine.items():
                rows_a = np.asarray(rows, np.int64)
                for c0 in range(0, len(rows_a), self.max_batch):
                    chunk = rows_a[c0:c0 + self.max_batch]
                    slots = np.asarray([locs[i][1] for i in chunk], np.int32)
                    queue.setdefault(e, []).append((k, chunk, slots, feats[chunk]))
        depth = 2
        inflight: Dict[int, List[tuple]] = {e: [] for e in queue}
        pos = {e: 0 for e in queue}
        try:
            while any(pos[e] < len(queue[e]) or inflight[e] for e in queue):
                for e in queue:  # top every engine up, then drain the oldest of each
                    while pos[e] < len(queue[e]) and len(inflight[e]) < depth:
                        k, chunk, slots, f = queue[e][pos[e]]
                        self.engines[e].submit(slots, f)
                        inflight[e].append((k, chunk))
                        pos[e] += 1
                for e in queue:
                    if inflight[e]:
                        k, chunk = inflight[e].pop(0)
                        out[k][chunk] = self.engines[e].wait()
        except BaseException:
            # an engine refused or reported a device error: collect every step
            # still in flight, so each engine is idle again, then re-raise
            for e in queue:
                while inflight[e]:
                    inflight[e].pop(0)
                    try:
                        self.engines[e].wait()
                    except Exception:  # noqa: BLE001  (the first error is the one raised)
                        pass
            raise
        return out

    def process_batch(self, requests_by_symbol: Dict[str, List["PendingRequest"]]) -> "InferenceResponse":
        """Answer every pending request, batching horizontally across symbols
        (example_model.py:769-905)."""
        all_unique_ids: List[int] = []
        all_predictions: List[List[float]] = []
        symbol_items = []
        for symbol, reqs in requests_by_symbol.items():
            if not reqs:
                continue
            loc = self._row_for(symbol)
            if loc is None:
                for req in reqs:
                    all_unique_ids.append(req.unique_id)
                    all_predictions.append([0.0] * self.num_outputs)
                continue
            symbol_items.append((loc, reqs))
        if symbol_items:
            rounds, reqs_of = [], []
            for k in range(max(len(reqs) for _, reqs in symbol_items)):
                locs, feats, batch_requests = [], [], []
                for loc, reqs in symbol_items:
                    if len(reqs) > k:
                        locs.append(loc)
                        feats.append(reqs[k].features)
                        batch_requests.append(reqs[k])
                rows = _feature_rows(feats, self.num_features)
                rounds.append((locs, rows))
                reqs_of.append(batch_requests)
            for batch_requests, preds in zip(reqs_of, self._run_rounds(rounds)):
                # one conversion a round: the same Python floats, row by row
                all_unique_ids.extend(req.unique_id for req in batch_requests)
                all_predictions.extend(preds.astype(float).tolist())
        return InferenceResponse(unique_ids=all_unique_ids, predictions=all_predictions,
                                 client_timestamp=time.time())

    def close(self):
        for e in self.engines:
            e.close()
        self.engines = []
