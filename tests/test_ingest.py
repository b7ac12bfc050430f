"""Native request ingest (b2e_ingest_*, b2e_encode_response) against the
reference's own codec and queue logic, on the CPU.

The reference decodes each line with json.loads (protocol.py:86-103), queues
requests per symbol in a dict of bounded queues (client.py:156-173), drains
them all (client.py:202-220) and answers in rounds (example_model.py:885-899);
it encodes with json.dumps (protocol.py:80-84). `_reference_rounds` restates
those steps in Python over json.loads' own output; features must match bit for
bit after the float32 conversion process_batch applies."""

import json
import math
import struct

import numpy as np
import pytest

from hackathon_b200 import _lib
from hackathon_b200.ingest import RequestIngest, encode_response

F = 5


def _request(uids, syms, feats, ts=1.5, **dump_kw):
    d = {"unique_ids": uids, "symbols": syms, "features": feats, "timestamp": ts,
         "message_type": "inference_request"}  # dataclasses.asdict order (protocol.py:28-34)
    return (json.dumps(d, **dump_kw) + "\n").encode()


def _reference_rounds(lines, max_queue):
    """json.loads + _handle_request + _gather_requests + process_batch rounds."""
    queues, drops = {}, []
    for ln in lines:
        d = json.loads(ln.decode("utf-8").strip())
        for uid, sym, f in zip(d["unique_ids"], d["symbols"], d["features"]):
            q = queues.setdefault(sym, [])
            if max_queue > 0 and len(q) >= max_queue:
                drops.append(sym)
                continue
            with np.errstate(over="ignore"):
                q.append((uid, np.asarray(f, dtype=np.float32)))
    order = list(queues)
    rows, rounds = [], []
    depth = max((len(q) for q in queues.values()), default=0)
    for k in range(depth):
        r = [(order.index(s), q[k][0], q[k][1]) for s, q in queues.items() if len(q) > k]
        rows += r
        rounds.append(len(r))
    return order, rows, rounds, drops


def _same_f32(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def _check_take(ing, lines, max_queue):
    order, rows, rounds, drops = _reference_rounds(lines, max_queue)
    got = ing.take()
    assert [ing.symbol_name(i) for i in range(len(order))] == order
    assert got.round_rows.tolist() == rounds
    assert got.symbols.tolist() == [r[0] for r in rows]
    assert got.unique_ids.tolist() == [r[1] for r in rows]
    want = np.stack([r[2] for r in rows]) if rows else np.zeros((0, F), np.float32)
    assert _same_f32(got.features, want)
    assert ing.drops() == drops
    assert ing.pending() == 0


def test_library_exports_the_ingest_entry_points():
    L = _lib.lib()
    for name in ("b2e_ingest_create", "b2e_ingest_feed", "b2e_ingest_take", "b2e_encode_response"):
        assert hasattr(L, name)


def test_requests_decode_into_rounds_like_the_reference():
    rng = np.random.default_rng(0)
    syms = [f"SYM_{i:03d}" for i in range(7)]
    lines, uid = [], 0
    for m in range(40):
        n = int(rng.integers(0, 6))
        s = [syms[int(rng.integers(0, len(syms)))] for _ in range(n)]
        f = rng.standard_normal((n, F)).astype(np.float32).astype(float).tolist()
        lines.append(_request(list(range(uid, uid + n)), s, f, ts=float(m)))
        uid += n
    ing = RequestIngest(F, max_queue_size=100)
    blob = b"".join(lines)
    # arbitrary socket chunking: lines split across feeds
    cuts = sorted(rng.integers(0, len(blob), 25).tolist())
    prev = 0
    for c in cuts + [len(blob)]:
        ing.feed(blob[prev:c])
        prev = c
    assert ing.next_other() is None
    _check_take(ing, lines, 100)
    assert ing.take().unique_ids.size == 0


def test_numbers_convert_like_float_then_float32():
    vals = ["0", "-0", "0.0", "-0.0", "1", "-17", "123456789012345", "1.5", "-2.25e-3", "1E5", "1e+2", "3.4e38",
            "3.5e38", "1e39", "1e-45", "7e-46", "1e-400", "-1e-400", "1e400", "-1e400", "5e-324",
            "0.1000000000000000055511151231257827", "16777217", "NaN", "Infinity", "-Infinity",
            "2.718281828459045235360287", "340282356779733661637539395458142568448.0"]
    rows = [vals[i:i + F] for i in range(0, len(vals) - F + 1, 2)]
    body = ", ".join("[" + ", ".join(r) + "]" for r in rows)
    line = ('{"unique_ids": [' + ", ".join(str(i) for i in range(len(rows))) + '], "symbols": ['
            + ", ".join(f'"S{i % 3}"' for i in range(len(rows))) + '], "features": [' + body
            + '], "timestamp": 0, "message_type": "inference_request"}\n').encode()
    ing = RequestIngest(F)
    assert ing.feed(line) == len(rows)
    _check_take(ing, [line], 100)


def test_formatting_variants_and_repeated_keys():
    f = [[0.5, -1.0, 2.0, 3.0, 4.0]]
    lines = [
        _request([1], ["A"], f, separators=(",", ":")),
        _request([2], ["A"], f, indent=None, separators=(" ,  ", " :\t")),
        (b'  {"message_type":"inference_request","timestamp":"not a number","features":[[1,2,3,4,5]],'
         b'"symbols":["B"],"unique_ids":[3]}\r\n'),
        # a repeated key keeps its last value (json.loads)
        (b'{"unique_ids": [9], "unique_ids": [4], "symbols": ["x"], "symbols": ["C"], '
         b'"features": [[1,1,1,1,1]], "timestamp": 1, "message_type": "heartbeat", '
         b'"message_type": "inference_request"}\n'),
        # escapes in a symbol
        _request([5], ["café \"q\" \\ / \t \U0001f600"], f),
        # zip() stops at the shortest list
        _request([6, 7, 8], ["D", "D"], [[0, 0, 0, 0, 0]] * 3),
    ]
    ing = RequestIngest(F)
    for ln in lines:
        ing.feed(ln)
    assert ing.next_other() is None
    _check_take(ing, lines, 100)


def test_every_other_line_comes_back_whole_and_in_order():
    good = _request([1], ["A"], [[1, 2, 3, 4, 5]])
    others = [
        b'{"timestamp": 12.5, "message_type": "heartbeat"}',
        b'{"unique_ids": [1], "trade_pnls": [0.1], "accuracies": [1.0], "latencies_ms": [2.0], '
        b'"message_type": "score_update"}',
        b'{"error": "boom", "details": null, "message_type": "error"}',
        b'{"unique_ids": [1], "symbols": ["A"], "features": [[1,2,3,4,5]], "message_type": "inference_request"}',
        b'{"unique_ids": [1], "symbols": ["A"], "features": [[1,2,3,4,5]], "timestamp": 1, "extra": 0, '
        b'"message_type": "inference_request"}',
        b'{"unique_ids": [1.0], "symbols": ["A"], "features": [[1,2,3,4,5]], "timestamp": 1, '
        b'"message_type": "inference_request"}',
        b'{"unique_ids": [99999999999999999999], "symbols": ["A"], "features": [[1,2,3,4,5]], "timestamp": 1, '
        b'"message_type": "inference_request"}',
        b'{"unique_ids": [1], "symbols": [7], "features": [[1,2,3,4,5]], "timestamp": 1, '
        b'"message_type": "inference_request"}',
        b'{"unique_ids": [1], "symbols": ["A"], "features": [[1,2,3,4]], "timestamp": 1, '
        b'"message_type": "inference_request"}',
        b'{"unique_ids": [1], "symbols": ["A"], "features": [[1,2,3,4,"5"]], "timestamp": 1, '
        b'"message_type": "inference_request"}',
        '{"unique_ids": [1], "symbols": ["é"], "features": [[1,2,3,4,5]], "timestamp": 1, '
        '"message_type": "inference_request"}'.encode("utf-8"),
        b'{"unique_ids": [1], "symbols": ["\\ud800"], "features": [[1,2,3,4,5]], "timestamp": 1, '
        b'"message_type": "inference_request"}',
        b'{"unique_ids": [01], "symbols": ["A"], "features": [[1,2,3,4,5]], "timestamp": 1, '
        b'"message_type": "inference_request"}',
        b'{"unique_ids": [1], "symbols": ["A"], "features": [[1,2,3,4,5.]], "timestamp": 1, '
        b'"message_type": "inference_request"}',
        b'{"unique_ids": [1], "symbols": ["A"], "features": [[1,2,3,4,5]], "timestamp": 1, '
        b'"message_type": "inference_request"} x',
        b'[1, 2]',
        b'not json',
        b'\r',
        b'\x0c{"timestamp": 1, "message_type": "heartbeat"}',
        b'{"symbols": ["tab\there"], "unique_ids": [1], "features": [[1,2,3,4,5]], "timestamp": 1, '
        b'"message_type": "inference_request"}',
    ]
    blob = good + b"\n".join(others) + b"\n\n" + good
    ing = RequestIngest(F)
    got = []
    ing.feed(blob)
    while True:
        ln = ing.next_other()
        if ln is None:
            break
        got.append(ln)
        assert ing.next_other() is None  # the feed stopped right after it
        ing.feed(b"")
    assert got == others
    rows = ing.take()
    assert rows.unique_ids.tolist() == [1, 1]
    # every kept line is one json.loads or ProtocolHandler.decode would not turn
    # into a well-typed request: either it raises, or it is another type, or a field
    # has a type outside the protocol's
    for ln in others:
        try:
            d = json.loads(ln.decode("utf-8").strip())
        except Exception:
            continue
        ok_types = (isinstance(d, dict) and d.get("message_type") == "inference_request"
                    and set(d) == {"unique_ids", "symbols", "features", "timestamp", "message_type"}
                    and all(type(u) is int and -2**63 <= u < 2**63 for u in d["unique_ids"])
                    and all(type(s) is str and s.isascii() and s.isprintable() for s in d["symbols"])
                    and all(isinstance(r, list) and len(r) == F and all(type(x) in (int, float) for x in r)
                            for r in d["features"])
                    and ln.isascii() and b"\\ud8" not in ln and b"\x0c" not in ln)
        assert not ok_types, ln


def test_push_keeps_order_and_queue_limit_drops_like_queue_full():
    ing = RequestIngest(F, max_queue_size=2)
    lines = [_request([i], ["A"], [[float(i)] * F]) for i in range(3)]
    ing.feed(lines[0])
    assert ing.push(100, "B", [1.0] * F)
    ing.feed(lines[1] + lines[2])
    assert not ing.push(101, "A", [2.0] * F)
    assert ing.drops() == ["A", "A"]
    rows = ing.take()
    assert [ing.symbol_name(s) for s in rows.symbols.tolist()] == ["A", "B", "A"]
    assert rows.unique_ids.tolist() == [0, 100, 1]
    assert rows.round_rows.tolist() == [2, 1]


def test_unbounded_queue_when_max_queue_is_not_positive():
    ing = RequestIngest(F, max_queue_size=0)
    lines = [_request(list(range(300)), ["A"] * 300, [[0.0] * F] * 300)]
    ing.feed(lines[0])
    _check_take(ing, lines, 0)


def _dumps_response(uids, preds, ts):
    with np.errstate(invalid="ignore"):
        p = np.asarray(preds, np.float32).astype(float).tolist()
    d = {"unique_ids": [int(u) for u in uids], "predictions": p,
         "client_timestamp": ts, "message_type": "inference_response"}
    return (json.dumps(d) + "\n").encode("utf-8")


def test_response_bytes_equal_json_dumps():
    rng = np.random.default_rng(1)
    specials = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 3.4028235e38, 1e-5, 1e-4, 9.999999e-5,
                         1e16, 1e15, 123456.789, 0.1, 1.0, -2.0, 65504.0, 1.17549435e-38, 16777216.0, 1e17],
                        np.float32)
    bits = rng.integers(0, 2**32, 4000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    vals = np.concatenate([specials, bits, rng.standard_normal(400).astype(np.float32),
                           (rng.standard_normal(400) * 10.0 ** rng.integers(-30, 30, 400)).astype(np.float32)])
    vals = vals[: len(vals) // 4 * 4].reshape(-1, 4)
    uids = rng.integers(-2**62, 2**62, len(vals))
    for ts in (0.0, 1765432101.123456, 1e-7, 12345678901234567890.0, -3.5):
        assert encode_response(uids, vals, ts) == _dumps_response(uids, vals, ts)
    assert encode_response([], np.zeros((0, 4), np.float32), 2.0) == _dumps_response([], [], 2.0)


def test_float_repr_matches_python_on_random_doubles():
    rng = np.random.default_rng(2)
    raw = rng.integers(0, 2**63, 3000, dtype=np.int64).view(np.float64)
    ts = [float(x) for x in raw if math.isfinite(x)][:2000]
    for t in ts:
        got = encode_response([], np.zeros((0, 4), np.float32), t)
        assert got == _dumps_response([], [], t), (t, got)


def test_feed_rejects_bad_arguments():
    ing = RequestIngest(F)
    L = _lib.lib()
    rc = L.b2e_ingest_feed(ing._h, None, 5, None, None)
    assert rc == _lib.B2E_OK - 1  # B2E_ERR_INVALID
    with pytest.raises(_lib.B2EError):
        RequestIngest(0)
    assert struct.calcsize("q") == 8


def test_parallel_parsing_queues_exactly_what_one_thread_does():
    rng = np.random.default_rng(3)
    lines = []
    for m in range(300):
        n = int(rng.integers(1, 40))
        syms = [f"S{int(x)}" for x in rng.integers(0, 50, n)]
        f = rng.standard_normal((n, F)).astype(np.float32).astype(float).tolist()
        lines.append(_request(list(range(m * 100, m * 100 + n)), syms, f))
        if m % 37 == 5:
            lines.append(b'{"timestamp": 1, "message_type": "heartbeat"}\n')
    blob = b"".join(lines)
    assert len(blob) > 256 << 10
    out = []
    for threads in (1, 8):
        ing = RequestIngest(F, max_queue_size=0, threads=threads)
        others = []
        ing.feed(blob)
        while (ln := ing.next_other()) is not None:
            others.append(ln)
            ing.feed(b"")
        r = ing.take()
        out.append((others, r.symbols.tolist(), r.unique_ids.tolist(), r.features.copy(), r.round_rows.tolist(),
                    [ing.symbol_name(i) for i in range(int(r.symbols.max()) + 1)]))
    a, b = out
    assert a[0] == b[0] and len(a[0]) == sum(1 for m in range(300) if m % 37 == 5)
    assert a[1] == b[1] and a[2] == b[2] and a[4] == b[4] and a[5] == b[5]
    assert _same_f32(a[3], b[3])


def test_take_batch_is_the_continuous_batching_rule():
    """b2e_ingest_take_batch picks, batch after batch, exactly the requests
    hackathon_b200.batcher.continuous_batches picks from the same arrivals (the
    oldest head request of up to k distinct symbols, oldest first), also when
    new arrivals land between batches, and every request comes out once with
    its own features."""
    from hackathon_b200 import batcher as B
    from hackathon_b200 import ingest as IG

    rng = np.random.default_rng(4)
    stream = B.zipf_stream(40, 600, 1.1, seed=2)
    feats = rng.standard_normal((len(stream), 5), dtype=np.float32)
    ing = IG.RequestIngest(5, max_queue_size=0)
    for i, sym in enumerate(stream):
        assert ing.push(i, f"S{int(sym)}", feats[i])
    got = []
    while True:
        rows = ing.take_batch(7)
        if len(rows.unique_ids) == 0:
            break
        assert len(set(rows.symbols.tolist())) == len(rows.symbols), "a symbol twice in one batch"
        assert np.array_equal(rows.features, feats[rows.unique_ids])
        got.append(rows.unique_ids.tolist())
    want = [b.tolist() for b in B.continuous_batches(stream, 7)]
    assert got == want
    assert ing.pending() == 0

    # arrivals between batches: a second stream after the first batch
    ing2 = IG.RequestIngest(5, max_queue_size=0)
    for i in range(100):
        ing2.push(i, f"S{int(stream[i])}", feats[i])
    first = ing2.take_batch(7).unique_ids.tolist()
    for i in range(100, 200):
        ing2.push(i, f"S{int(stream[i])}", feats[i])
    rest = []
    while True:
        rows = ing2.take_batch(7)
        if len(rows.unique_ids) == 0:
            break
        rest.append(rows.unique_ids.tolist())
    order = {}
    for u in first + [u for b in rest for u in b]:
        order.setdefault(int(stream[u]), []).append(u)
    assert all(v == sorted(v) for v in order.values()), "a symbol's requests out of order"
    assert sorted(first + [u for b in rest for u in b]) == list(range(200))
    ing.close()
    ing2.close()
