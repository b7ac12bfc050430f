"""Pin the CPU oracle to the reference: every fixture under tests/golden was made
by the reference's own torch code (tests/golden/make_golden.py)."""

import numpy as np
import pytest

from hackathon_b200 import config as C
from hackathon_b200 import weights as Wt
from oracle import cells as OC
from oracle import model as O
from tests.conftest import assert_close, load_golden
from tests.golden import streams

# The oracle restates the reference's fp32 arithmetic; the only differences are
# summation order inside numpy's BLAS / reductions.
RTOL, ATOL = 1e-4, 1e-5


def test_cells_match_reference_kernels():
    g, meta = load_golden("cells")
    for c in meta["cases"]:
        state0, rest, masks = streams.cell_inputs(c["tag"], c["batch"], tuple(c["dims"]), c["seed"])
        st = state0.copy()
        out = getattr(OC, f"{c['tag']}_step")(st, *rest, masks[c["mask"]])
        assert_close(out, g[c["key"] + "_out"], RTOL, ATOL, c["key"] + " out")
        if c["mask"] == "mixed":
            assert_close(st, g[c["key"] + "_state"], RTOL, ATOL, c["key"] + " state")
            idle = ~masks["mixed"]
            assert np.array_equal(st[idle], state0[idle]), "idle rows must stay bit for bit"
        if c["mask"] == "allfalse":
            assert np.array_equal(st, state0)
            assert not out.any()


@pytest.mark.parametrize("tag", ["xlstm", "mamba2", "retnet", "hawk"])
def test_layers_match_reference(tag):
    g, meta = load_golden("layers")
    (c,) = [m for m in meta["cases"] if m["tag"] == tag]
    cfg = streams.LAYER_CFG
    sd = Wt.generate(Wt.layer_specs(tag, "", cfg), seed=c["weight_seed"])
    xs, masks = streams.layer_stream(tag, cfg, c["steps"], c["batch"], seed=c["input_seed"])
    assert np.isclose(float(np.sum(xs, dtype=np.float64)), c["input_sum"]), "input stream drifted"
    state = O.init_block_state(tag, cfg, c["batch"])
    W = O.Weights(sd)
    for s in range(c["steps"]):
        rows = np.nonzero(masks[s])[0]
        y, new = O.layer_step(tag, W, xs[s][rows], [leaf[rows] for leaf in state], cfg)
        for leaf, nl in zip(state, new):
            leaf[rows] = nl
        assert_close(y, g[f"{tag}_y"][s][rows], RTOL, ATOL, f"{tag} y step {s}")
    for i, leaf in enumerate(state):
        assert_close(leaf, g[f"{tag}_state{i}"], RTOL, ATOL, f"{tag} state leaf {i}")


def _run_model(cfg, sd, lp, feats, masks):
    orc = O.Oracle(cfg, sd, lp)
    state = O.init_state(cfg, feats.shape[1])
    preds = []
    for s in range(len(feats)):
        rows = np.nonzero(masks[s])[0]
        p, new = orc.step(feats[s][rows], O.gather_rows(state, rows))
        O.scatter_rows(state, rows, new)
        preds.append((rows, p))
    return preds, state


def test_model_fp32_matches_reference():
    g, meta = load_golden("model")
    cfg, steps, batch = streams.MODEL_CASE
    sd = Wt.generate_model(cfg, seed=meta["weight_seed"])
    feats, masks = streams.model_stream(cfg, steps, batch, seed=meta["input_seed"])
    assert np.isclose(float(np.sum(feats, dtype=np.float64)), meta["input_sum"])
    preds, state = _run_model(cfg, sd, None, feats, masks)
    for s, (rows, p) in enumerate(preds):
        assert_close(p, g["fp32_preds"][s][rows], RTOL, ATOL, f"preds step {s}")
    for i, leaf in enumerate(O.flat_leaves(state)):
        assert_close(leaf, g[f"fp32_state{i}"], RTOL, ATOL, f"state leaf {i}")


def test_model_bf16_emulation_tracks_reference():
    """CastLinear in bf16 (example_model.py:68-106): the oracle's emulation rounds
    exactly like torch (single rounding of acc + bias, checked bit for bit on one
    linear in make_golden's probe); across the model, accumulation-order ulp flips
    are amplified, so the bound is on the mean squared error, not per element."""
    g, meta = load_golden("model")
    cfg, steps, batch = streams.MODEL_CASE
    sd = Wt.generate_model(cfg, seed=meta["weight_seed"])
    feats, masks = streams.model_stream(cfg, steps, batch, seed=meta["input_seed"])
    preds, _ = _run_model(cfg, sd, "bf16", feats, masks)
    err = np.concatenate([(p - g["bf16_preds"][s][rows]).ravel() for s, (rows, p) in enumerate(preds)])
    ref = np.concatenate([g["bf16_preds"][s][rows].ravel() for s, (rows, p) in enumerate(preds)])
    assert np.mean(err ** 2) <= 1e-5 * max(1.0, float(np.mean(ref ** 2)))


def test_linear_bf16_rounding_is_single():
    x = np.random.default_rng(0).standard_normal((3, 16), dtype=np.float32)
    w = np.random.default_rng(1).standard_normal((5, 16), dtype=np.float32)
    b = np.random.default_rng(2).standard_normal(5, dtype=np.float32)
    y = O.linear(x, w, b, "bf16")
    assert np.array_equal(y, O.round_bf16(y)), "CastLinear output is a bf16 value"
    assert np.array_equal(O.round_bf16(np.float32([1.0 + 2 ** -8])), np.float32([1.0])), "ties to even"


def test_long_stream_prefix_matches_reference():
    """First 300 steps of the 10,000-step stream (the GPU test runs all of it)."""
    g, meta = load_golden("long")
    cfg, steps, batch = streams.LONG_CASE
    sd = Wt.generate_model(cfg, seed=meta["weight_seed"])
    orc = O.Oracle(cfg, sd)
    state = O.init_state(cfg, batch)
    gen = streams.long_features(cfg, batch, seed=meta["input_seed"])
    for s in range(300):
        p, state = orc.step(next(gen), state)
        assert_close(p, g["preds"][s], RTOL, ATOL, f"step {s}")


def test_d0_stream_first_requests_match_reference():
    """BASELINE config 1 at the default dims: the first requests of the stream."""
    from tests.conftest import GOLDEN

    g, meta = load_golden("d0stream")
    sd = Wt.generate_model(C.D0, seed=meta["weight_seed"])
    orc = O.Oracle(C.D0, sd)
    feats = streams.d0_features(3)
    for i in range(2):  # SYM_001 then SYM_002: fresh state each
        p, _ = orc.step(feats[i:i + 1], O.init_state(C.D0, 1))
        # 12 blocks of K=2048/4096 float32 dot products: numpy's and torch's BLAS
        # sum in different orders, which moves the predictions by ~3e-4 relative.
        assert_close(p[0], g["preds"][i], 1e-3, 1e-3, f"request {i}")


@pytest.mark.parametrize("kind", ["mamba2", "retnet", "xlstm"])
def test_micro_layers_within_fp32_noise_of_the_reference_in_float64(kind):
    """BASELINE configs 2 and 3 (tests/golden/micro.npz, the reference's layers
    in float32 and float64): the oracle, another fp32 evaluation, is within twice
    the reference fp32's distance from float64 (never required below 1e-4), on
    every step's output rows and on every final state leaf."""
    from tests import arbiter as A

    g, meta = load_golden("micro")
    (c,) = [m for m in meta["cases"] if m["kind"] == kind]
    cfg, sd = Wt.micro_layer(kind, seed=0)
    xs = streams.micro_inputs(kind)
    assert np.isclose(float(np.sum(xs, dtype=np.float64)), c["input_sum"]), "input stream drifted"
    W = O.Weights(sd)
    state = O.init_block_state(kind, cfg, xs.shape[1])
    ys = []
    for s in range(xs.shape[0]):
        y, state = O.layer_step(kind, W, xs[s], state, cfg)
        ys.append(y)
    A.check_fp32_rows(f"{kind} outputs", np.stack(ys), g[f"{kind}_f32_y"], g[f"{kind}_f64_y"])
    nl = len(state)
    A.check_fp32_leaves(kind, state, [g[f"{kind}_f32_state{i}"] for i in range(nl)],
                        [g[f"{kind}_f64_state{i}"] for i in range(nl)])


def test_micro_fills_are_the_stated_ones():
    """Config 2: a = -exp(U(0, ln 16)) in [-16, -1], softplus(dt bias) in
    [1e-3, 0.1]; config 3: gamma_h = 1 - 2^(-5-h), 64-wide heads."""
    cfg, sd = Wt.micro_layer("mamba2")
    assert cfg.mamba_bc_size == 64 and 2 * cfg.hidden_size // cfg.mamba_head_size == 8
    assert np.all((sd["a"] <= -1.0) & (sd["a"] >= -16.0))
    sp = np.log1p(np.exp(sd["dt_proj.bias"].astype(np.float64)))
    assert np.all((sp >= 1e-3 - 1e-9) & (sp <= 0.1 + 1e-9))
    cfg, sd = Wt.micro_layer("retnet")
    assert cfg.hidden_size // cfg.num_heads == 64
    np.testing.assert_allclose(sd["decay"], 1.0 - 2.0 ** (-5.0 - np.arange(4)), rtol=0, atol=1e-7)
    cfg, _ = Wt.micro_layer("xlstm")
    assert 2 * cfg.hidden_size // cfg.num_heads == 64


def test_config4_fixtures_agree_with_each_other():
    """BASELINE config 4's fixtures (make_golden.py d0batch, d0emu): the
    reference's float64 run is within 1e-3 (normwise) of its float32 run per
    tower, and the oracle's exact bf16 emulation is closer to the reference's bf16
    run than bf16 weights move the answer (on the same rows and steps)."""
    g, meta = load_golden("d0batch")
    e, em = load_golden("d0batch_emu")
    ra, steps = meta["arbiter_rows"], meta["steps"]
    assert em["rows"] == ra and em["steps"] == steps
    assert g["fp32_preds"].shape == g["bf16_preds"].shape == (steps, meta["rows"], 4)
    assert g["f64_preds"].shape == e["emu_preds"].shape == (steps, ra, 4)
    r32 = g["fp32_preds"][:, :ra].astype(np.float64)
    rbf = g["bf16_preds"][:, :ra].astype(np.float64)
    f64 = g["f64_preds"].astype(np.float64)
    emu = e["emu_preds"].astype(np.float64)
    for c in range(4):
        assert np.linalg.norm(r32[..., c] - f64[..., c]) <= 1e-3 * np.linalg.norm(f64[..., c]), c
        assert np.mean((emu[..., c] - rbf[..., c]) ** 2) < np.mean((rbf[..., c] - r32[..., c]) ** 2), c
