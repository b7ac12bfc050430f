"""The three fused state steps on the GPU against the reference's torch kernels
(tests/golden/cells.npz) and the oracle, with the checks of the reference's own
kernel checker (check_kernels.py:174-293): idle rows bit for bit, zero outputs
on idle rows, contiguous fp32 output, strided operands, refusals."""

import numpy as np
import pytest
import torch

from hackathon_b200 import kernels as K
from oracle import cells as OC
from tests.conftest import assert_close, load_golden
from tests.golden import streams

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
RTOL, ATOL = 1e-4, 1e-5  # check_kernels.py:78


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _mask(m):
    return None if m is None else torch.from_numpy(m).to(DEV)


def test_cells_match_reference_fixtures():
    g, meta = load_golden("cells")
    for c in meta["cases"]:
        state0, rest, masks = streams.cell_inputs(c["tag"], c["batch"], tuple(c["dims"]), c["seed"])
        st = _t(state0)
        out = getattr(K, f"{c['tag']}_step")(st, *[_t(a) for a in rest], _mask(masks[c["mask"]]))
        torch.cuda.synchronize()
        assert out.dtype == torch.float32 and out.is_contiguous() and out.device == DEV
        want = g[c["key"] + "_out"]
        assert tuple(out.shape) == want.shape
        m = masks[c["mask"]]
        live = np.ones(c["batch"], bool) if m is None else m
        assert_close(out.cpu().numpy()[live], want[live], RTOL, ATOL, c["key"] + " out")
        assert not out.cpu().numpy()[~live].any(), "idle rows must output zeros"
        got_state = st.cpu().numpy()
        assert np.array_equal(got_state[~live], state0[~live]), "idle rows must stay bit for bit"
        if c["mask"] == "mixed":
            assert_close(got_state, g[c["key"] + "_state"], RTOL, ATOL, c["key"] + " state")


@pytest.mark.parametrize("tag,dims,batch", [
    ("mlstm", (8, 512, 512), 3), ("mlstm", (8, 64, 64), 64), ("retnet", (8, 256, 256), 3),
    ("retnet", (8, 32, 32), 64), ("mamba2", (64, 64, 128), 3), ("mamba2", (8, 64, 128), 64),
    ("mamba2", (8, 64, 64), 33),
    # ragged head sizes through the vectorised kernels
    ("mamba2", (3, 17, 64), 5), ("mamba2", (2, 300, 32), 3), ("mamba2", (4, 7, 128), 4),
    ("mlstm", (3, 40, 64), 5), ("mlstm", (2, 33, 128), 3), ("retnet", (4, 16, 32), 7),
])
def test_cells_model_shapes_match_oracle(tag, dims, batch):
    """The shapes the model runs at (default and reduced dims), against the oracle."""
    state0, rest, masks = streams.cell_inputs(tag, batch, dims, seed=5)
    for mname in ("mixed", "none"):
        st_ref = state0.copy()
        want = getattr(OC, f"{tag}_step")(st_ref, *rest, masks[mname])
        st = _t(state0)
        out = getattr(K, f"{tag}_step")(st, *[_t(a) for a in rest], _mask(masks[mname]))
        assert_close(out.cpu().numpy(), want, RTOL, 2e-5, f"{tag} {dims} out")
        assert_close(st.cpu().numpy(), st_ref, RTOL, ATOL, f"{tag} {dims} state")


@pytest.mark.parametrize("tag", ["mlstm", "retnet", "mamba2"])
def test_strided_operands_are_packed(tag):
    """check_kernels.py:201-236: operands interleaved with NaN must not leak."""
    batch, dims = 5, {"mlstm": (3, 48, 80), "retnet": (3, 48, 80), "mamba2": (5, 40, 96)}[tag]
    state0, rest, masks = streams.cell_inputs(tag, batch, dims, seed=9)
    mask = masks["mixed"]
    strided = []
    for a in rest:
        t = _t(a)
        wide = torch.stack([torch.full_like(t, float("nan")), t], dim=-1)
        strided.append(wide[..., 1])
        assert not strided[-1].is_contiguous()
    wide_mask = torch.zeros(batch, 2, dtype=torch.bool, device=DEV)
    wide_mask[:, 1] = _mask(mask)
    st_ref = state0.copy()
    want = getattr(OC, f"{tag}_step")(st_ref, *rest, mask)
    st = _t(state0)
    out = getattr(K, f"{tag}_step")(st, *strided, wide_mask[:, 1])
    assert_close(out.cpu().numpy(), want, RTOL, ATOL, "out")
    assert_close(st.cpu().numpy(), st_ref, RTOL, ATOL, "state")
    assert np.array_equal(st.cpu().numpy()[~mask], state0[~mask])


def test_wrappers_refuse_like_the_reference():
    """check_kernels.py:272-293: refuse rather than repair."""
    state0, rest, masks = streams.cell_inputs("mlstm", 4, (2, 16, 16), seed=1)
    st = _t(state0)
    args = [_t(a) for a in rest]
    with pytest.raises(AssertionError):  # non-contiguous state
        K.mlstm_step(st.transpose(2, 3), *args, None)
    with pytest.raises(AssertionError):  # non-fp32 state
        K.mlstm_step(st.double(), *args, None)
    with pytest.raises(AssertionError):  # non-fp32 operand
        K.mlstm_step(st, args[0].double(), *args[1:], None)
    with pytest.raises(AssertionError):  # short mask
        K.mlstm_step(st, *args, torch.ones(3, dtype=torch.bool, device=DEV))
    with pytest.raises(AssertionError):  # mask on the wrong device
        K.mlstm_step(st, *args, torch.ones(4, dtype=torch.bool))
    with pytest.raises(AssertionError):  # wrong-shaped operand
        K.mlstm_step(st, args[0][:, :1], *args[1:], None)


def test_state_advances_over_repeated_steps():
    """The same state stepped 50 times stays equal to the oracle stepped 50 times."""
    state0, rest, masks = streams.cell_inputs("retnet", 6, (4, 32, 32), seed=2)
    st_ref = state0.copy()
    st = _t(state0)
    for _ in range(50):
        want = OC.retnet_step(st_ref, *rest, masks["mixed"])
        out = K.retnet_step(st, *[_t(a) for a in rest], _mask(masks["mixed"]))
    assert_close(st.cpu().numpy(), st_ref, 1e-4, 1e-4, "state after 50 steps")
    assert_close(out.cpu().numpy(), want, 1e-4, 1e-4, "out after 50 steps")


@pytest.mark.parametrize("tag,dims,batch", [
    ("mamba2", (8, 64, 128), 300), ("mlstm", (8, 64, 64), 300), ("retnet", (8, 32, 32), 300),
    ("mamba2", (3, 17, 64), 37), ("mlstm", (3, 40, 64), 29),
])
def test_state_kernel_grids_agree_bit_for_bit(tag, dims, batch):
    """The persistent grid (the ensemble step's) and the short-CTA grids (alone)
    run the same per-item arithmetic: outputs and state agree bit for bit, idle
    rows included, for several wave counts and a ragged last CTA."""
    state0, rest, masks = streams.cell_inputs(tag, batch, dims, seed=9)
    results = []
    prev = K.set_state_kernel_waves(0)
    try:
        for waves in (0, 1, 8, 64):
            K.set_state_kernel_waves(waves)
            st = _t(state0)
            out = getattr(K, f"{tag}_step")(st, *[_t(a) for a in rest], _mask(masks["mixed"]))
            torch.cuda.synchronize()
            results.append((waves, out.cpu().numpy(), st.cpu().numpy()))
    finally:
        K.set_state_kernel_waves(prev)
    w0, out0, st0 = results[0]
    for waves, out, st in results[1:]:
        assert np.array_equal(out.view(np.uint32), out0.view(np.uint32)), f"waves {waves}: outputs differ"
        assert np.array_equal(st.view(np.uint32), st0.view(np.uint32)), f"waves {waves}: state differs"
