"""Host logic of process_batch on CPU: rounds, answer order, first-sight slots,
overflow answered with zeros - checked against the reference's own
process_batch (tests/golden/api.npz). The engine underneath is replaced by the
CPU oracle here; the GPU tests run the same calls through libb2e.so."""

import numpy as np

from hackathon_b200 import client as CL
from hackathon_b200 import weights as Wt
from oracle import model as O
from tests.conftest import assert_close, load_golden
from tests.golden import streams


class OracleEngine:
    """Engine-shaped wrapper of the CPU oracle (test double): steps run in
    submit order, up to two in flight, wait() returns the oldest."""

    def __init__(self, cfg, sd, capacity):
        self.orc = O.Oracle(cfg, sd)
        self.state = O.init_state(cfg, capacity)
        self.calls = []
        self._pending = []

    def submit(self, slots, feats):
        assert len(self._pending) < 2, "more than two steps in flight"
        slots = list(np.asarray(slots).reshape(-1))
        assert len(set(slots)) == len(slots), "a symbol appears twice in one round"
        self.calls.append(slots)
        p, new = self.orc.step(np.asarray(feats, np.float32), O.gather_rows(self.state, slots))
        O.scatter_rows(self.state, slots, new)
        self._pending.append(p)

    def wait(self):
        return self._pending.pop(0)

    def close(self):
        pass


def make_client(monkeypatch, cfg, sd, capacity, devices=None):
    made = []

    def fake(config, weights, device, linear_dtype, cap, max_batch, graphs):
        e = OracleEngine(config, weights, cap)
        made.append(e)
        return e

    monkeypatch.setattr(CL.B200InferenceClient, "_make_engine", staticmethod(fake))
    monkeypatch.setattr(CL.B200InferenceClient, "_overflow_warned", False)
    c = CL.B200InferenceClient(num_symbols=capacity, config=cfg, weights=sd, linear_dtype="fp32", devices=devices)
    return c, made


def run_api_calls(client, cfg):
    uids, preds = [], []
    for call in streams.api_calls(cfg):
        batch = {sym: [CL.PendingRequest(unique_id=u, symbol=sym, features=f, received_time=0.0) for (u, f) in reqs]
                 for sym, reqs in call}
        r = client.process_batch(batch)
        assert len(r.unique_ids) == len(r.predictions)
        assert all(isinstance(p, list) and len(p) == 4 and all(isinstance(v, float) for v in p)
                   for p in r.predictions)
        uids += list(r.unique_ids)
        preds += r.predictions
    return uids, np.asarray(preds, np.float32)


def test_process_batch_matches_reference(monkeypatch, capsys):
    g, meta = load_golden("api")
    cfg = streams.API_CFG
    sd = Wt.generate_model(cfg, seed=0)
    client, _ = make_client(monkeypatch, cfg, sd, meta["capacity"])
    uids, preds = run_api_calls(client, cfg)
    assert uids == list(g["unique_ids"]), "answer order must be the reference's"
    assert_close(preds, g["predictions"], 1e-4, 1e-5, "predictions")
    assert {k: v[1] for k, v in client.symbol_to_idx.items()} == meta["symbol_rows"], "first-sight slots"
    out = capsys.readouterr().out
    assert out.count("WARNING: out of state rows") == 1


def test_rounds_keep_one_request_per_symbol(monkeypatch):
    cfg = streams.API_CFG
    sd = Wt.generate_model(cfg, seed=0)
    client, made = make_client(monkeypatch, cfg, sd, 8)
    rng = np.random.default_rng(0)
    batch = {f"S{i}": [CL.PendingRequest(100 * i + j, f"S{i}", rng.standard_normal(79).tolist(), 0.0)
                       for j in range(n)] for i, n in enumerate([3, 1, 0, 2])}
    r = client.process_batch(batch)
    assert r.unique_ids == [0, 100, 300, 1, 301, 2]
    assert made[0].calls == [[0, 1, 2], [0, 2], [0]]


def test_sharded_client_routes_by_symbol_hash(monkeypatch):
    """Two devices: each symbol's rows go to crc32(name) % 2, and the answers equal
    the single-device client's."""
    cfg = streams.API_CFG
    sd = Wt.generate_model(cfg, seed=0)
    one, _ = make_client(monkeypatch, cfg, sd, 16)
    two, made = make_client(monkeypatch, cfg, sd, 16, devices=[0, 1])
    rng = np.random.default_rng(3)
    for step in range(3):
        batch = {f"SYM_{i:03d}": [CL.PendingRequest(1000 * step + 10 * i + j, f"SYM_{i:03d}",
                                                    rng.standard_normal(79).tolist(), 0.0) for j in range(1 + i % 2)]
                 for i in range(10)}
        r1, r2 = one.process_batch(batch), two.process_batch(batch)
        assert r1.unique_ids == r2.unique_ids
        assert_close(r2.predictions, r1.predictions, 1e-4, 1e-5, "sharded vs single")
    for sym, (e, _) in two.symbol_to_idx.items():
        assert e == CL.owner_device(sym, 2)
    assert made[0].calls and made[1].calls


def test_full_home_device_spills_and_zeros_start_only_at_global_capacity(monkeypatch, capsys):
    """Three devices of two slots each, six symbols allowed: a symbol whose home
    device is full takes a slot elsewhere, and only the seventh distinct symbol
    is answered with zeros (the reference's rule, example_model.py:750-764)."""
    cfg = streams.API_CFG
    sd = Wt.generate_model(cfg, seed=0)
    made = []
    monkeypatch.setattr(CL.B200InferenceClient, "_make_engine", staticmethod(
        lambda config, weights, device, lp, cap, mb, graphs: made.append(OracleEngine(config, weights, cap)) or made[-1]))
    monkeypatch.setattr(CL.B200InferenceClient, "_overflow_warned", False)
    c = CL.B200InferenceClient(num_symbols=6, config=cfg, weights=sd, linear_dtype="fp32", devices=[0, 1, 2],
                               per_device_capacity=2)
    # pick names whose home device is 0, so devices 1 and 2 only fill by spilling
    names = [n for n in (f"SYM_{i:03d}" for i in range(500)) if CL.owner_device(n, 3) == 0][:7]
    rng = np.random.default_rng(1)
    batch = {n: [CL.PendingRequest(i, n, rng.standard_normal(79).tolist(), 0.0)] for i, n in enumerate(names)}
    r = c.process_batch(batch)
    placed = [c.symbol_to_idx[n] for n in names[:6]]
    assert sorted(placed) == [(0, 0), (0, 1), (1, 0), (1, 1), (2, 0), (2, 1)]
    assert names[6] not in c.symbol_to_idx
    zeros = [p for u, p in zip(r.unique_ids, r.predictions) if u == 6]
    assert zeros == [[0.0] * 4]
    assert all(any(v != 0.0 for v in p) for u, p in zip(r.unique_ids, r.predictions) if u != 6)
    assert capsys.readouterr().out.count("WARNING: out of state rows") == 1


def test_device_error_from_an_engine_raises_from_process_batch_and_drains_the_rest(monkeypatch):
    """An engine whose wait() reports a device error (B2E_ERR_DEVICE) makes
    process_batch raise; every other step in flight is collected first, so the
    engines are idle and the next call runs."""
    from hackathon_b200 import _lib

    cfg = streams.API_CFG
    sd = Wt.generate_model(cfg, seed=0)
    client, made = make_client(monkeypatch, cfg, sd, 8, devices=[0, 1])
    fail = {"on": True}
    real_wait = OracleEngine.wait

    def wait(self):
        out = real_wait(self)
        if self is made[1] and fail["on"]:
            raise _lib.B2EError(-6, "device error word 101 after this step")
        return out

    monkeypatch.setattr(OracleEngine, "wait", wait)
    rng = np.random.default_rng(2)
    names = [f"SYM_{i:03d}" for i in range(6)]
    assert {CL.owner_device(n, 2) for n in names} == {0, 1}
    batch = {n: [CL.PendingRequest(10 * i + j, n, rng.standard_normal(79).tolist(), 0.0) for j in range(3)]
             for i, n in enumerate(names)}
    try:
        client.process_batch(batch)
        raise AssertionError("process_batch returned despite a device error")
    except _lib.B2EError as e:
        assert e.code == -6
    assert not made[0]._pending and not made[1]._pending, "steps left in flight"
    fail["on"] = False
    r = client.process_batch(batch)
    assert len(r.unique_ids) == 18


def test_feature_rows_native_helper_matches_numpy_bit_for_bit():
    """The native row writer (csrc/rows.c) gives numpy's float32 values for float64
    values that round, ints, bools, numpy scalars, tuples, inf and nan."""
    assert CL._ROWS is not None, "lib/_b2e_rows is not built (python -m hackathon_b200.build)"
    rng = np.random.default_rng(7)
    feats = [rng.standard_normal(79).tolist() for _ in range(300)]  # float64 values: rounding matters
    feats[3][5] = 7
    feats[4][0] = True
    feats[5][1] = np.float64(1e-40)
    feats[6][2] = np.float32(3.25)
    feats[7][3] = float("inf")
    feats[8] = tuple(feats[8])
    feats[9][4] = 3.4028235677973366e38  # rounds past float32's largest finite value
    got = CL._feature_rows(feats, 79)
    with np.errstate(over="ignore"):  # numpy warns on the value that rounds to inf
        want = np.asarray(feats, dtype=np.float32)
    assert got.dtype == np.float32 and got.shape == (300, 79)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    nan_row = [[float("nan")] * 3]
    assert np.isnan(CL._feature_rows(nan_row, 3)).all()


def test_feature_rows_refusals_follow_numpy():
    """A row of another length or a value that is not a number takes numpy's
    path, which raises as the reference's conversion does."""
    import pytest

    with pytest.raises(ValueError):
        CL._feature_rows([[1.0, 2.0], [1.0]], 2)
    with pytest.raises(ValueError):
        CL._feature_rows([[1.0, "x"]], 2)
    out = np.empty((1, 2), np.float32)
    with pytest.raises(ValueError):
        CL._ROWS.rows_f32([[1.0, 2.0, 3.0]], 2, out)
    with pytest.raises(TypeError):
        CL._ROWS.rows_f32([[1.0, None]], 2, out)


def test_feature_rows_without_the_native_helper(monkeypatch):
    """Without lib/_b2e_rows the client converts with numpy: the same values."""
    rng = np.random.default_rng(8)
    feats = [rng.standard_normal(79).tolist() for _ in range(64)]
    with_helper = CL._feature_rows(feats, 79)
    monkeypatch.setattr(CL, "_ROWS", None)
    without = CL._feature_rows(feats, 79)
    assert np.array_equal(with_helper.view(np.uint32), without.view(np.uint32))
