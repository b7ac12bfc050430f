"""IngestClient's two socket loops on the CPU (the engine replaced by the CPU
oracle, as in test_client_host.py): request lines written to one end of a
socket pair, in pieces and mixed with other message types, come back as
response lines on it. Whatever batching the two threads happen to form, every
request is answered exactly once, with the prediction the reference path gives
it (each symbol's requests in arrival order), within the fp32 tolerance: the
oracle's sums follow the batch size."""

import json
import socket
import threading
import time

import numpy as np
import pytest

from hackathon_b200 import client as CL
from hackathon_b200 import ingest as IG
from hackathon_b200 import weights as Wt
from tests.conftest import assert_close
from tests.golden import streams
from tests.test_client_host import OracleEngine


def _client(monkeypatch, cls, cfg, sd, **kw):
    monkeypatch.setattr(CL.B200InferenceClient, "_make_engine",
                        staticmethod(lambda config, weights, device, lp, cap, mb, graphs: OracleEngine(config, weights, cap)))
    return cls(num_symbols=6, config=cfg, weights=sd, linear_dtype="fp32", **kw)


@pytest.mark.parametrize("batching", ["continuous", "rounds"])
def test_socket_loops_answer_every_request_like_the_reference_path(monkeypatch, batching):
    cfg = streams.API_CFG
    sd = Wt.generate_model(cfg, seed=0)
    rng = np.random.default_rng(12)
    reqs = []
    for uid in range(60):
        sym = f"SYM_{int(rng.integers(1, 6)):03d}"
        reqs.append((uid, sym, rng.standard_normal(cfg.num_features, dtype=np.float32).astype(float).tolist()))
    lines = b""
    for i in range(0, len(reqs), 7):
        chunk = reqs[i:i + 7]
        lines += (json.dumps({"unique_ids": [u for u, _, _ in chunk], "symbols": [s for _, s, _ in chunk],
                              "features": [f for _, _, f in chunk], "timestamp": 1.0,
                              "message_type": "inference_request"}) + "\n").encode()
        lines += b'{"timestamp": 2.0, "message_type": "heartbeat"}\n'
    lines += b"not json\n"

    # the reference path: the same requests, each symbol in arrival order
    ref = _client(monkeypatch, CL.B200InferenceClient, cfg, sd)
    by_sym = {}
    for u, s, f in reqs:
        by_sym.setdefault(s, []).append(CL.PendingRequest(u, s, f, 0.0))
    r = ref.process_batch(by_sym)
    want = dict(zip(r.unique_ids, r.predictions))

    ing = _client(monkeypatch, IG.IngestClient, cfg, sd, max_queue_size=100, batching=batching)
    a, b = socket.socketpair()
    ing.socket = a
    ing.running = True
    threads = [threading.Thread(target=ing._receive_loop, daemon=True),
               threading.Thread(target=ing._process_loop, daemon=True)]
    for t in threads:
        t.start()
    for i in range(0, len(lines), 997):  # arbitrary pieces
        b.sendall(lines[i:i + 997])
        time.sleep(0.002)
    got, buf = {}, b""
    b.settimeout(0.2)
    deadline = time.time() + 20
    while len(got) < len(reqs) and time.time() < deadline:
        try:
            buf += b.recv(1 << 16)
        except socket.timeout:
            continue
        while b"\n" in buf:
            line, buf = buf.split(b"\n", 1)
            d = json.loads(line)
            if d["message_type"] != "inference_response":
                assert d["message_type"] == "heartbeat"
                continue
            for u, p in zip(d["unique_ids"], d["predictions"]):
                assert u not in got, f"request {u} answered twice"
                got[u] = p
    ing.running = False
    for t in threads:
        t.join(timeout=5)
    a.close()
    b.close()
    assert sorted(got) == sorted(want)
    assert_close(np.asarray([got[u] for u in sorted(got)], np.float32),
                 np.asarray([want[u] for u in sorted(got)], np.float32), 1e-4, 1e-5, "predictions")


class SlotEchoEngine:
    """Test double that answers each row with (its slot, its first feature, 0, 0),
    so a response shows which state slot a request was stepped on."""

    def __init__(self):
        self._pending = []

    def submit(self, slots, feats):
        slots = np.asarray(slots, np.int32).reshape(-1)
        feats = np.asarray(feats, np.float32)
        out = np.zeros((len(slots), 4), np.float32)
        out[:, 0] = slots
        out[:, 1] = feats[:, 0]
        self._pending.append(out)

    def wait(self):
        return self._pending.pop(0)

    def close(self):
        pass


def test_new_symbols_arriving_while_the_process_loop_runs_keep_their_own_slots(monkeypatch):
    """A receive thread keeps feeding lines that introduce new symbols while a
    process thread drains and names them: every request is answered once, and
    every symbol's requests land on one slot that no other symbol shares."""
    cfg = streams.API_CFG
    monkeypatch.setattr(CL.B200InferenceClient, "_make_engine",
                        staticmethod(lambda config, weights, device, lp, cap, mb, graphs: SlotEchoEngine()))
    n_sym, per_msg, n_msg = 3000, 16, 400
    ing = IG.IngestClient(num_symbols=n_sym, config=cfg, weights={}, linear_dtype="fp32", max_queue_size=1000)
    rng = np.random.default_rng(5)
    sym_of, feat0 = {}, {}
    msgs = []
    uid = 0
    for m in range(n_msg):
        hi = min(n_sym, 8 * (m + 1))  # the symbol universe keeps growing
        syms = [f"S{int(x)}" for x in rng.integers(0, hi, per_msg)]
        feats = rng.standard_normal((per_msg, cfg.num_features), dtype=np.float32)
        ids = list(range(uid, uid + per_msg))
        uid += per_msg
        for u, s, f in zip(ids, syms, feats):
            sym_of[u], feat0[u] = s, float(f[0])
        msgs.append((json.dumps({"unique_ids": ids, "symbols": syms, "features": feats.astype(float).tolist(),
                                 "timestamp": 1.0, "message_type": "inference_request"}) + "\n").encode())
    answers = []
    done = threading.Event()

    def receiver():
        for b in msgs:
            ing.receive(b)
        done.set()

    def processor():
        while True:
            finished = done.is_set()
            out = ing.process_ingested()
            if out is not None:
                answers.append(out)
            elif finished:
                return

    threads = [threading.Thread(target=receiver), threading.Thread(target=processor)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    got = {}
    for line in answers:
        d = json.loads(line)
        for u, p in zip(d["unique_ids"], d["predictions"]):
            assert u not in got, f"request {u} answered twice"
            got[u] = p
    assert sorted(got) == list(range(uid))
    slot_of = {}
    for u, p in got.items():
        assert np.float32(p[1]) == np.float32(feat0[u]), "a request was answered with another's features"
        assert slot_of.setdefault(sym_of[u], p[0]) == p[0], f"symbol {sym_of[u]} stepped on two slots"
    assert len(set(slot_of.values())) == len(slot_of), "two symbols share a slot"
    ing.close()
