"""The CUDA engine against the reference's own outputs (tests/golden) and the
oracle: single layers, the whole ensemble (fp32 and bf16 weights), a 10,000-step
stream, process_batch end to end, and the error paths of the C-ABI."""

import numpy as np
import pytest
import torch

from hackathon_b200 import _lib
from hackathon_b200 import client as CL
from hackathon_b200 import config as C
from hackathon_b200 import weights as Wt
from hackathon_b200.engine import EnsembleEngine, LayerEngine
from oracle import model as O
from tests.conftest import assert_close, load_golden
from tests.golden import streams

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
# fp32 path: the reference's own kernel-checker tolerance (check_kernels.py:78)
RTOL, ATOL = 1e-4, 1e-5


def _leaf_rows(golden, key_fmt, n_leaves, row):
    return [golden[key_fmt.format(i)][row] for i in range(n_leaves)]


@pytest.mark.parametrize("tag", ["xlstm", "mamba2", "retnet", "hawk"])
def test_layer_matches_reference(tag):
    g, meta = load_golden("layers")
    (c,) = [m for m in meta["cases"] if m["tag"] == tag]
    cfg = streams.LAYER_CFG
    sd = Wt.generate(Wt.layer_specs(tag, "", cfg), seed=c["weight_seed"])
    eng = LayerEngine(tag, cfg, sd, capacity=c["batch"], max_batch=c["batch"])
    xs, masks = streams.layer_stream(tag, cfg, c["steps"], c["batch"], seed=c["input_seed"])
    y = torch.empty(c["batch"], cfg.hidden_size, device=DEV)
    for s in range(c["steps"]):
        rows = np.nonzero(masks[s])[0]
        slots = torch.from_numpy(rows.astype(np.int32)).to(DEV)
        eng.step_device(slots, torch.from_numpy(xs[s][rows]).to(DEV), y)
        torch.cuda.synchronize()
        assert_close(y[:len(rows)].cpu().numpy(), g[f"{tag}_y"][s][rows], RTOL, ATOL, f"{tag} y step {s}")
    nl = len(eng.layout)
    for row in range(c["batch"]):
        for i, (got, want) in enumerate(zip(eng.read_slot(row), _leaf_rows(g, tag + "_state{}", nl, row))):
            assert_close(got, want, RTOL, ATOL, f"{tag} slot {row} leaf {i}")
    eng.close()


def _engine_masked_run(cfg, sd, lp, feats, masks, graphs=True):
    batch = feats.shape[1]
    eng = EnsembleEngine(cfg, sd, linear_dtype=lp, capacity=batch, max_batch=batch, graphs=graphs)
    preds = []
    for s in range(len(feats)):
        rows = np.nonzero(masks[s])[0]
        preds.append((rows, eng.step(rows, feats[s][rows])))
    return eng, preds


def test_model_fp32_matches_reference():
    g, meta = load_golden("model")
    cfg, steps, batch = streams.MODEL_CASE
    sd = Wt.generate_model(cfg, seed=meta["weight_seed"])
    feats, masks = streams.model_stream(cfg, steps, batch, seed=meta["input_seed"])
    eng, preds = _engine_masked_run(cfg, sd, "fp32", feats, masks)
    for s, (rows, p) in enumerate(preds):
        assert_close(p, g["fp32_preds"][s][rows], RTOL, ATOL, f"preds step {s}")
    n = len(eng.layout)
    for row in range(batch):
        for i, (got, want) in enumerate(zip(eng.read_slot(row), _leaf_rows(g, "fp32_state{}", n, row))):
            assert_close(got, want, RTOL, ATOL, f"slot {row} leaf {i}")


def test_graph_replay_equals_eager_bit_for_bit():
    cfg, steps, batch = streams.MODEL_CASE
    sd = Wt.generate_model(cfg, seed=0)
    feats, masks = streams.model_stream(cfg, steps, batch, seed=3)
    e1, p1 = _engine_masked_run(cfg, sd, "fp32", feats, masks, graphs=True)
    e2, p2 = _engine_masked_run(cfg, sd, "fp32", feats, masks, graphs=False)
    for (r1, a), (r2, b) in zip(p1, p2):
        assert np.array_equal(a, b)
    for row in range(batch):
        for x, y in zip(e1.read_slot(row), e2.read_slot(row)):
            assert np.array_equal(x, y)


def test_model_bf16_weights_mse_bound():
    """bf16 CastLinear variant: against the oracle's exact emulation of the same
    rounding, and against the fp32 reference with the MSE bound of the bf16
    weights (relative MSE <= 1e-3 of the prediction power)."""
    g, meta = load_golden("model")
    cfg, steps, batch = streams.MODEL_CASE
    sd = Wt.generate_model(cfg, seed=meta["weight_seed"])
    feats, masks = streams.model_stream(cfg, steps, batch, seed=meta["input_seed"])
    _, preds = _engine_masked_run(cfg, sd, "bf16", feats, masks)
    got = np.concatenate([p for _, p in preds])
    ref32 = np.concatenate([g["fp32_preds"][s][r] for s, (r, _) in enumerate(preds)])
    refbf = np.concatenate([g["bf16_preds"][s][r] for s, (r, _) in enumerate(preds)])
    power = float(np.mean(ref32 ** 2))
    assert float(np.mean((got - refbf) ** 2)) <= 1e-5 * power, "bf16 engine vs reference bf16 CastLinear"
    assert float(np.mean((got - ref32) ** 2)) <= 1e-3 * power, "bf16 engine vs fp32 reference"


def test_long_stream_10k_steps_matches_reference():
    """4 rows, all active, 10,000 consecutive steps: per-prediction and final-state
    error against the reference's fp32 run."""
    g, meta = load_golden("long")
    cfg, steps, batch = streams.LONG_CASE
    sd = Wt.generate_model(cfg, seed=meta["weight_seed"])
    eng = EnsembleEngine(cfg, sd, capacity=batch, max_batch=batch)
    gen = streams.long_features(cfg, batch, seed=meta["input_seed"])
    slots = np.arange(batch, dtype=np.int32)
    preds = np.empty((steps, batch, 4), np.float32)
    for s in range(steps):
        preds[s] = eng.step(slots, next(gen))
    scale = float(np.sqrt(np.mean(g["preds"].astype(np.float64) ** 2)))
    assert_close(preds, g["preds"], 1e-4, 1e-5 * scale, "predictions over 10k steps")
    n = len(eng.layout)
    for row in range(batch):
        for i, (got, want) in enumerate(zip(eng.read_slot(row), _leaf_rows(g, "state{}", n, row))):
            lscale = float(np.sqrt(np.mean(np.square(want[np.isfinite(want)], dtype=np.float64)))) if want.size else 0
            assert_close(got, want, 1e-4, 1e-5 * max(lscale, 1e-3), f"slot {row} leaf {i} after 10k steps")


def test_batch_composition_does_not_change_a_row():
    """Rows are independent (no op mixes rows, example_model.py:422-427): a row
    stepped alone or among 40 others at other slots gives the same answer."""
    cfg = C.ModelConfig(hidden_size=64, proj_size=128, tower_depth=2, num_heads=4, num_features=79)
    sd = Wt.generate_model(cfg, seed=1)
    eng = EnsembleEngine(cfg, sd, capacity=64, max_batch=64)
    rng = np.random.default_rng(0)
    feats = rng.standard_normal((41, 79), dtype=np.float32)
    alone = eng.step([40], feats[40:41])
    eng.reset_slots([40])
    slots = np.arange(41, dtype=np.int32)
    together = eng.step(slots[::-1].copy(), feats[::-1].copy())[0:1]
    assert_close(together, alone, RTOL, ATOL, "row 40 alone vs in a batch of 41")


def test_state_table_roundtrip_and_reset():
    cfg = C.SMALL
    sd = Wt.generate_model(cfg, seed=0)
    eng = EnsembleEngine(cfg, sd, capacity=8, max_batch=8)
    init = eng.read_slot(3)
    ref = O.flat_leaves(O.init_state(cfg, 1))
    for a, b in zip(init, ref):
        assert np.array_equal(a, b[0]), "fresh slot = init_state"
    rng = np.random.default_rng(0)
    eng.step([3, 5], rng.standard_normal((2, cfg.num_features), dtype=np.float32))
    moved = eng.read_slot(3)
    assert any(not np.array_equal(a, b) for a, b in zip(moved, init))
    untouched = eng.read_slot(4)
    for a, b in zip(untouched, init):
        assert np.array_equal(a, b), "a slot outside the step is never written"
    leaves = [np.asarray(rng.standard_normal(a.shape), a.dtype) if a.dtype == np.float32 else a for a in moved]
    eng.write_slot(6, leaves)
    for a, b in zip(eng.read_slot(6), leaves):
        assert np.array_equal(a, b)
    eng.reset_slots([3, 6])
    for s in (3, 6):
        for a, b in zip(eng.read_slot(s), init):
            assert np.array_equal(a, b)


def test_engine_steps_from_injected_state_like_the_oracle():
    """Random (non-zero) state written into slots, then one step: the engine and the
    oracle agree, so every leaf is read with the reference's layout."""
    cfg = C.SMALL
    sd = Wt.generate_model(cfg, seed=0)
    eng = EnsembleEngine(cfg, sd, capacity=4, max_batch=4)
    rng = np.random.default_rng(5)
    st = O.init_state(cfg, 2)
    for tower in st:
        for blk in tower:
            for leaf in blk:
                if leaf.dtype == np.float32:
                    leaf[...] = rng.standard_normal(leaf.shape).astype(np.float32) * np.float32(0.5)
                else:
                    leaf[...] = rng.integers(0, 50, leaf.shape)
    flat = O.flat_leaves(st)
    for row, slot in enumerate((1, 3)):
        eng.write_slot(slot, [leaf[row] for leaf in flat])
    feats = rng.standard_normal((2, cfg.num_features), dtype=np.float32)
    want, new = O.Oracle(cfg, sd).step(feats, st)
    got = eng.step([1, 3], feats)
    assert_close(got, want, RTOL, ATOL, "preds from injected state")
    for row, slot in enumerate((1, 3)):
        for i, (a, b) in enumerate(zip(eng.read_slot(slot), O.flat_leaves(new))):
            assert_close(a, b[row], RTOL, ATOL, f"slot {slot} leaf {i}")


def test_error_paths_refuse_without_touching_state():
    cfg = C.SMALL
    sd = Wt.generate_model(cfg, seed=0)
    eng = EnsembleEngine(cfg, sd, capacity=4, max_batch=4)
    f = np.zeros((2, cfg.num_features), np.float32)
    with pytest.raises(_lib.B2EError, match="twice"):
        eng.step([1, 1], f)
    with pytest.raises(_lib.B2EError, match="outside"):
        eng.step([0, 4], f)
    with pytest.raises(_lib.B2EError):
        eng.step(np.arange(5), np.zeros((5, cfg.num_features), np.float32))
    bad = dict(sd)
    bad.pop("output_proj.bias")
    with pytest.raises(_lib.B2EError, match="missing weight"):
        EnsembleEngine(cfg, bad, capacity=2, max_batch=2)
    extra = dict(sd)
    extra["towers.0.bogus"] = np.zeros(3, np.float32)
    with pytest.raises(_lib.B2EError, match="unexpected weight"):
        EnsembleEngine(cfg, extra, capacity=2, max_batch=2)
    # device path: an out-of-range slot steps no row and raises the device flag
    before = eng.read_slot(0)
    slots = torch.tensor([0, 99], dtype=torch.int32, device=DEV)
    feats = torch.zeros(2, cfg.num_features, device=DEV)
    preds = torch.zeros(2, 4, device=DEV)
    eng.step_device(slots, feats, preds, 2)
    assert eng.device_error() == 1
    assert eng.device_error() == 0, "the flag clears once read"
    for a, b in zip(eng.read_slot(0), before):
        assert np.array_equal(a, b)


def test_device_error_word_fails_host_steps_until_cleared():
    """A code in the engine's device error word (here the out-of-table slot flag
    of a device step; a tensor-core timeout writes the same word) makes every
    host step fail with B2E_ERR_DEVICE, through the engine and process_batch,
    until device_error() reads and clears it; then steps answer again."""
    cfg = C.SMALL
    sd = Wt.generate_model(cfg, seed=0)
    eng = EnsembleEngine(cfg, sd, capacity=4, max_batch=4)
    f = np.random.default_rng(0).standard_normal((2, cfg.num_features), dtype=np.float32)
    good = eng.step([0, 1], f)
    eng.step_device(torch.tensor([0, 99], dtype=torch.int32, device=DEV), torch.zeros(2, cfg.num_features, device=DEV),
                    torch.zeros(2, 4, device=DEV), 2)
    for _ in range(2):
        with pytest.raises(_lib.B2EError, match="device error word 1") as ei:
            eng.step([2, 3], f)
        assert ei.value.code == -6
    assert eng.device_error() == 1
    eng.reset_slots([0, 1])
    assert np.array_equal(eng.step([0, 1], f), good), "after clearing, steps answer as before"
    eng.close()

    client = CL.B200InferenceClient(num_symbols=4, config=cfg, weights=sd, linear_dtype="fp32")
    e = client.engines[0]
    e.step_device(torch.tensor([99], dtype=torch.int32, device=DEV), torch.zeros(1, cfg.num_features, device=DEV),
                  torch.zeros(1, 4, device=DEV), 1)
    batch = {"SYM_001": [CL.PendingRequest(1, "SYM_001", f[0].tolist(), 0.0)]}
    with pytest.raises(_lib.B2EError):
        client.process_batch(batch)
    assert e.device_error() == 1
    assert len(client.process_batch(batch).predictions) == 1
    client.close()


def test_device_step_equals_host_step():
    cfg = C.SMALL
    sd = Wt.generate_model(cfg, seed=0)
    e1 = EnsembleEngine(cfg, sd, capacity=8, max_batch=8)
    e2 = EnsembleEngine(cfg, sd, capacity=8, max_batch=8)
    rng = np.random.default_rng(1)
    for _ in range(3):
        slots = rng.permutation(8)[:5].astype(np.int32)
        feats = rng.standard_normal((5, cfg.num_features), dtype=np.float32)
        a = e1.step(slots, feats)
        p = torch.empty(5, 4, device=DEV)
        e2.step_device(torch.from_numpy(slots).to(DEV), torch.from_numpy(feats).to(DEV), p, 5)
        torch.cuda.synchronize()
        assert np.array_equal(a, p.cpu().numpy())


def test_launch_count_is_reported():
    cfg = C.SMALL
    eng = EnsembleEngine(cfg, Wt.generate_model(cfg, 0), capacity=4, max_batch=4, flags=_lib.FLAG_NO_LATENCY_PATH)
    k = eng.launches_per_step(4)
    assert 50 < k < 400, k
    lat = EnsembleEngine(cfg, Wt.generate_model(cfg, 0), capacity=4, max_batch=4)
    assert lat.launches_per_step(4) == 1  # the latency path: one kernel


def test_process_batch_on_gpu_matches_reference(capsys):
    g, meta = load_golden("api")
    cfg = streams.API_CFG
    sd = Wt.generate_model(cfg, seed=0)
    CL.B200InferenceClient._overflow_warned = False
    client = CL.B200InferenceClient(num_symbols=meta["capacity"], config=cfg, weights=sd, linear_dtype="fp32")
    uids, preds = [], []
    for call in streams.api_calls(cfg):
        batch = {s: [CL.PendingRequest(u, s, f, 0.0) for (u, f) in reqs] for s, reqs in call}
        r = client.process_batch(batch)
        uids += list(r.unique_ids)
        preds += r.predictions
    assert uids == list(g["unique_ids"])
    assert_close(np.asarray(preds, np.float32), g["predictions"], RTOL, ATOL, "process_batch predictions")
    assert capsys.readouterr().out.count("WARNING: out of state rows") == 1
    client.close()


@pytest.mark.parametrize("lane_towers", [0, 0b0011, 0b0100])
def test_large_batch_split_into_lanes_matches_oracle(lane_towers):
    """300 rows: the 512-row bucket runs as two lanes of 256 (the second with 44
    live rows) for the towers in lane_towers (0: all), one chain over all rows
    for the others; every row still equals the oracle, and two steps in a row
    keep the state consistent."""
    cfg = C.ModelConfig(hidden_size=64, proj_size=128, tower_depth=2, num_heads=4, num_features=79)
    sd = Wt.generate_model(cfg, seed=3)
    eng = EnsembleEngine(cfg, sd, capacity=400, max_batch=512, lanes=2, lane_towers=lane_towers)
    orc = O.Oracle(cfg, sd)
    rng = np.random.default_rng(8)
    slots = rng.permutation(400)[:300].astype(np.int32)
    state = O.init_state(cfg, 300)
    for _ in range(2):
        feats = rng.standard_normal((300, 79), dtype=np.float32)
        got = eng.step(slots, feats)
        want, state = orc.step(feats, state)
        assert_close(got, want, RTOL, ATOL, "preds of a two-lane step")
    for i in (0, 255, 256, 299):
        for a, b in zip(eng.read_slot(int(slots[i])), O.flat_leaves(state)):
            assert_close(a, b[i], RTOL, ATOL, f"state of row {i}")
