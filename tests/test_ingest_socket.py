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


def test_socket_loops_answer_every_request_like_the_reference_path(monkeypatch):
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

    ing = _client(monkeypatch, IG.IngestClient, cfg, sd, max_queue_size=100)
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
