"""Request ingest on libb2e's native decoder: the client's receive path and
response encoding without a Python object per request or per float.

The reference client reads newline-delimited JSON from its socket
(protocol.py:134-160), decodes each line with json.loads into a dataclass
(protocol.py:86-103), queues one ``PendingRequest`` per request in a per-symbol
``queue.Queue(maxsize=max_queue_size)`` (client.py:156-173), drains every queue
at once (client.py:202-220) and lets ``process_batch`` build rounds from the
Python float lists (example_model.py:885-899); responses go out through
``json.dumps`` (protocol.py:80-84).

``RequestIngest`` keeps the queues in native memory: well-typed
``inference_request`` lines are parsed straight into them, and every other line
comes back whole, in order, to be decoded by the reference's own
``ProtocolHandler`` (``IngestClient.receive``), so no line is read differently.
``take()`` returns the drained requests as flat arrays in round order.
``encode_response`` writes the bytes ``ProtocolHandler.encode`` would.
``IngestClient`` is ``B200InferenceClient`` wired to both; its process loop
either answers micro-batches as they form (continuous batching, the default)
or drains every queue into the reference's rounds.
"""

from __future__ import annotations

import ctypes as C
import json
import select
import threading
import time
from dataclasses import dataclass
from typing import Dict, List, NamedTuple, Optional

import numpy as np

from . import _lib
from .client import B200InferenceClient, _reference_module

_rproto = _reference_module("protocol", "ProtocolHandler")


class IngestRows(NamedTuple):
    """Drained requests, round by round (round k: the k-th queued request of every
    symbol that has one, symbols in first-seen order)."""

    symbols: np.ndarray     # int32 [n] symbol ids (dense, first-seen order)
    unique_ids: np.ndarray  # int64 [n]
    features: np.ndarray    # float32 [n, num_features]
    round_rows: np.ndarray  # int32 [rounds]


class RequestIngest:
    """Native queues of pending requests; see the module docstring."""

    def __init__(self, num_features: int, max_queue_size: int = 100, threads: Optional[int] = None):
        self.num_features = int(num_features)
        self._L = _lib.lib()
        h = C.c_void_p()
        _lib.check(self._L.b2e_ingest_create(self.num_features, int(max_queue_size), C.byref(h)))
        self._h = h
        self._names: List[str] = []
        # guards the name cache: a receive thread (drops) and a process thread
        # (take, then names) both grow it; the native handle has its own lock
        self._names_lock = threading.Lock()
        if threads is not None:
            _lib.check(self._L.b2e_ingest_set_threads(self._h, int(threads)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.b2e_ingest_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def feed(self, data: bytes = b"") -> int:
        """Append socket bytes and queue the complete request lines; stops after
        the first line kept for ``next_other``. Returns the requests queued."""
        nr, no = C.c_int32(), C.c_int32()
        buf = C.c_char_p(data) if data else None
        _lib.check(self._L.b2e_ingest_feed(self._h, buf, len(data), C.byref(nr), C.byref(no)))
        return nr.value

    def _bytes(self, fn, *args) -> Optional[bytes]:
        n = C.c_int64()
        _lib.check(fn(self._h, *args, None, 0, C.byref(n)))
        if n.value < 0:
            return None
        out = C.create_string_buffer(max(1, n.value))
        _lib.check(fn(self._h, *args, out, n.value, C.byref(n)))
        return out.raw[:n.value]

    def next_other(self) -> Optional[bytes]:
        """The oldest line the native decoder left to the caller, or None."""
        return self._bytes(self._L.b2e_ingest_next_other)

    def push(self, unique_id: int, symbol: str, features) -> bool:
        """Queue one request decoded elsewhere; False when its queue was full."""
        f = np.ascontiguousarray(np.asarray(features, dtype=np.float32).reshape(self.num_features))
        s = symbol.encode("utf-8")
        q = C.c_int32()
        _lib.check(self._L.b2e_ingest_push(self._h, int(unique_id), s, len(s), f.ctypes.data, C.byref(q)))
        return bool(q.value)

    def symbol_name(self, sid: int) -> str:
        with self._names_lock:
            while len(self._names) <= sid:
                b = self._bytes(self._L.b2e_ingest_symbol_name, C.c_int32(len(self._names)))
                self._names.append(b.decode("utf-8"))
            return self._names[sid]

    def drops(self) -> List[str]:
        """Symbols of the requests dropped on a full queue since the last call, in order."""
        out = []
        sid = C.c_int32()
        while True:
            _lib.check(self._L.b2e_ingest_next_drop(self._h, C.byref(sid)))
            if sid.value < 0:
                return out
            out.append(self.symbol_name(sid.value))

    def pending(self) -> int:
        n = C.c_int64()
        _lib.check(self._L.b2e_ingest_pending(self._h, C.byref(n)))
        return n.value

    def take(self) -> IngestRows:
        """Drain every queue (client.py:202-220) into round order."""
        n = self.pending()
        sym = np.empty(n, np.int32)
        uid = np.empty(n, np.int64)
        feats = np.empty((n, self.num_features), np.float32)
        rr = np.empty(max(n, 1), np.int32)
        nr, nrows = C.c_int32(), C.c_int64()
        _lib.check(self._L.b2e_ingest_take(self._h, n, sym.ctypes.data, uid.ctypes.data, feats.ctypes.data,
                                           rr.ctypes.data, C.byref(nr), C.byref(nrows)))
        return IngestRows(sym, uid, feats, rr[:nr.value].copy())


    def take_batch(self, max_rows: int) -> IngestRows:
        """One micro-batch (continuous batching): the oldest queued request of up
        to `max_rows` distinct symbols, in the arrival order of those requests;
        later requests of those symbols stay queued (b2e_ingest_take_batch)."""
        m = max(0, int(max_rows))
        sym = np.empty(m, np.int32)
        uid = np.empty(m, np.int64)
        feats = np.empty((m, self.num_features), np.float32)
        n = C.c_int32()
        _lib.check(self._L.b2e_ingest_take_batch(self._h, m, sym.ctypes.data, uid.ctypes.data, feats.ctypes.data,
                                                 C.byref(n)))
        k = n.value
        return IngestRows(sym[:k], uid[:k], feats[:k], np.asarray([k], np.int32) if k else np.zeros(0, np.int32))


def encode_response(unique_ids, predictions, client_timestamp: float) -> bytes:
    """ProtocolHandler.encode(InferenceResponse(unique_ids, predictions,
    client_timestamp)) for float32 predictions [n, n_out]."""
    L = _lib.lib()
    u = np.ascontiguousarray(np.asarray(unique_ids, dtype=np.int64))
    p = np.ascontiguousarray(np.asarray(predictions, dtype=np.float32))
    n = len(u)
    n_out = p.shape[1] if p.ndim == 2 else 0
    need = C.c_int64()
    guess = 160 + n * (24 + 26 * max(n_out, 1))
    out = C.create_string_buffer(guess)
    _lib.check(L.b2e_encode_response(u.ctypes.data, p.ctypes.data, n, n_out, float(client_timestamp), out, guess,
                                     C.byref(need)))
    if need.value > guess:
        out = C.create_string_buffer(need.value)
        _lib.check(L.b2e_encode_response(u.ctypes.data, p.ctypes.data, n, n_out, float(client_timestamp), out,
                                         need.value, C.byref(need)))
    return out.raw[:need.value]


@dataclass
class _Decoded:
    kind: str
    msg: object


def _decode(line: bytes) -> _Decoded:
    """The reference's ProtocolHandler.decode when it is importable; else the
    same steps (protocol.py:86-103) on plain dicts."""
    if _rproto is not None:
        msg = _rproto.ProtocolHandler.decode(line)
        return _Decoded(getattr(msg, "message_type", "error"), msg)
    try:
        d = json.loads(line.decode("utf-8").strip())
        mt = d.get("message_type")
        known = {"register": set(), "inference_request": {"unique_ids", "symbols", "features", "timestamp"},
                 "inference_response": {"unique_ids", "predictions", "client_timestamp"},
                 "score_update": {"unique_ids", "trade_pnls", "accuracies", "latencies_ms"},
                 "heartbeat": {"timestamp"}, "error": {"error", "details"}}
        if mt not in known:
            raise ValueError(f"Unknown message type: {mt}")
        d.pop("message_type", None)
        need = known[mt] - ({"details"} if mt == "error" else set())
        if not need <= set(d) <= known[mt]:
            raise TypeError(f"fields {sorted(d)} do not match {mt}")
        return _Decoded(mt, d)
    except Exception as e:  # noqa: BLE001  (the reference turns every failure into an ErrorMessage)
        return _Decoded("error", {"error": str(e)})


class IngestClient(B200InferenceClient):
    """B200InferenceClient whose receive path queues requests natively and whose
    process loop answers them as process_batch would, with the response bytes
    written natively. ``receive(bytes)`` and ``process_ingested()`` are the two
    halves; ``run()`` drives them from the socket like the reference's threads."""

    def __init__(self, *args, max_queue_size: int = 100, clock=time.time, batching: str = "continuous", **kw):
        super().__init__(*args, **kw)
        if batching not in ("continuous", "rounds"):
            raise ValueError(f"batching must be 'continuous' or 'rounds', got {batching!r}")
        self.batching = batching
        self.max_queue_size = max_queue_size
        if not hasattr(self, "queue_lock"):
            self.queue_lock = threading.RLock()
        self.ingest = RequestIngest(self.num_features, max_queue_size)
        self.clock = clock
        self._send_lock = threading.Lock()  # heartbeats and responses never interleave on the socket

    def _send(self, data: bytes) -> None:
        with self._send_lock:
            self.socket.sendall(data)

    def _fields(self, msg):
        return msg if isinstance(msg, dict) else vars(msg)

    def receive(self, data: bytes) -> None:
        """_receive_loop + _handle_request for one socket read (client.py:125-173)."""
        with self.queue_lock:
            self.ingest.feed(data)
            while True:
                line = self.ingest.next_other()
                if line is None:
                    break
                d = _decode(line)
                if d.kind == "inference_request":
                    f = self._fields(d.msg)
                    for uid, sym, feats in zip(f["unique_ids"], f["symbols"], f["features"]):
                        try:
                            self.ingest.push(int(uid), str(sym), feats)
                        except Exception as e:  # noqa: BLE001
                            print(f"Dropping request {uid!r} for {sym!r}: {e}")
                elif d.kind == "score_update":
                    self._handle_score(d.msg)
                elif d.kind == "error":
                    print(f"Server error: {self._fields(d.msg).get('error')}")
                self.ingest.feed(b"")
            for sym in self.ingest.drops():
                print(f"Queue full for symbol {sym}, dropping request")

    def _handle_score(self, score) -> None:
        pass

    def process_ingested(self) -> Optional[bytes]:
        """Answer every queued request like process_batch (example_model.py:769-905):
        overflow symbols' requests as zeros first (symbol order, then request
        order), then the rounds; returns the response line, or None when idle."""
        with self.queue_lock:
            rows = self.ingest.take()
            sids = np.unique(rows.symbols)  # ascending ids = first-seen = dict order
            names = {s: self.ingest.symbol_name(s) for s in sids.tolist()}
        n = len(rows.unique_ids)
        if n == 0:
            return None
        loc_of: Dict[int, Optional[tuple]] = {}
        for s in sids.tolist():
            loc_of[s] = self._row_for(names[s])
        over = np.asarray([s for s in sids.tolist() if loc_of[s] is None], np.int32)
        uids_out, preds_out = [], []
        live = np.ones(n, bool)
        if len(over):
            is_over = np.isin(rows.symbols, over)
            live = ~is_over
            idx = np.nonzero(is_over)[0]
            idx = idx[np.argsort(rows.symbols[idx], kind="stable")]
            uids_out.append(rows.unique_ids[idx])
            preds_out.append(np.zeros((len(idx), self.num_outputs), np.float32))
        start = 0
        rounds = []
        for cnt in rows.round_rows.tolist():
            sel = np.arange(start, start + cnt)
            start += cnt
            sel = sel[live[sel]]
            if len(sel) == 0:
                continue
            rounds.append(([loc_of[s] for s in rows.symbols[sel].tolist()], rows.features[sel]))
            uids_out.append(rows.unique_ids[sel])
        preds_out += self._run_rounds(rounds)
        return encode_response(np.concatenate(uids_out), np.concatenate(preds_out), self.clock())

    def process_continuous(self) -> Optional[bytes]:
        """Continuous batching: answer one micro-batch formed from whatever is
        queued now - the oldest request of up to max_batch distinct symbols, in
        arrival order (RequestIngest.take_batch) - and return its response line,
        or None when idle. A symbol's requests still reach the model one per
        step and in order; a micro-batch does not wait for a whole drain, so a
        request's answer never waits behind a deep backlog's later rounds.
        Symbols without a state slot are answered with zeros (example_model.py:
        750-764)."""
        with self.queue_lock:
            rows = self.ingest.take_batch(self.max_batch)
            names = {s: self.ingest.symbol_name(s) for s in np.unique(rows.symbols).tolist()}
        n = len(rows.unique_ids)
        if n == 0:
            return None
        locs = [self._row_for(names[s]) for s in rows.symbols.tolist()]
        live = np.asarray([loc is not None for loc in locs], bool)
        preds = np.zeros((n, self.num_outputs), np.float32)
        if live.any():
            idx = np.nonzero(live)[0]
            preds[idx] = self._run_rounds([([locs[i] for i in idx.tolist()], rows.features[idx])])[0]
        return encode_response(rows.unique_ids, preds, self.clock())

    # ---- socket driving (client.py:125-200); the reference's connect() and
    # run() start these two threads
    def _receive_loop(self):
        last_hb = 0
        while self.running:
            try:
                readable, _, _ = select.select([self.socket], [], [], 0.001)
                if readable:
                    data = self.socket.recv(1 << 16)
                    if not data:
                        break  # connection closed
                    self.receive(data)
                now = int(time.time())
                if now % 5 == 0 and now - last_hb >= 5:
                    # Heartbeat(timestamp) as ProtocolHandler.encode writes it
                    self._send((json.dumps({"timestamp": time.time(), "message_type": "heartbeat"})
                                + "\n").encode("utf-8"))
                    last_hb = now
            except Exception as e:  # noqa: BLE001
                if self.running:
                    print(f"Receive error: {e}")
                    break

    def _process_loop(self):
        step = self.process_continuous if self.batching == "continuous" else self.process_ingested
        while self.running:
            try:
                out = step()
                if out is None:
                    time.sleep(0.001)
                    continue
                self._send(out)
            except Exception as e:  # noqa: BLE001
                print(f"Process error: {e}")
                time.sleep(0.1)

    def close(self):
        self.ingest.close()
        super().close()
