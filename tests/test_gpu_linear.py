"""CastLinear / nn.Linear on the GPU (b2e_linear): the tcgen05 tensor-core kernel
and the SIMT kernels against a float64 restatement of CastLinear.forward
(example_model.py:92-95): x and W rounded to bf16, exact products, the bias in
bf16, one rounding of the result to bf16."""

import numpy as np
import pytest
import torch

from hackathon_b200 import config as C
from hackathon_b200 import kernels as K
from hackathon_b200 import weights as Wt
from hackathon_b200.engine import EnsembleEngine
from oracle import model as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def reference(x, w, b, relu, dt):
    """(rounded CastLinear result, unrounded float64 value, f32 accumulation bound)."""
    xr = x.to(dt).double()
    wd = w.double()
    y = xr @ wd.T
    if b is not None:
        y = y + b.double()
    k = x.shape[1]
    # f32 accumulation of k products: a few sqrt(k) roundings of the running sum,
    # bounded by the sum of |x w|.
    acc = 4.0 * k ** 0.5 * 2.0 ** -24 * (xr.abs() @ wd.abs().T)
    rounded = y.to(dt).float()
    if relu:
        rounded, y = torch.relu(rounded), torch.relu(y)
    return rounded, y, acc


def half_ulp(v, dt):
    mant = 8 if dt == torch.bfloat16 else 11
    scale = torch.clamp(v.abs(), min=2.0 ** -100)
    return 0.5 * 2.0 ** (torch.floor(torch.log2(scale)) - (mant - 1))


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,k,n,bias,relu", [
    (200, 512, 1280, False, False),   # ragged M, the Mamba2 x|z|b|c projection at D2
    (4096, 256, 256, True, False),    # a full batch, out_proj-like
    (129, 80, 512, True, True),       # K not a multiple of the 64-wide K tile; fc1-like
    (33, 2048, 128, False, False),    # long K
    (512, 512, 1024, True, False),
])
@pytest.mark.parametrize("tensor_cores", [True, False])
def test_cast_linear_matches_castlinear(dt, m, k, n, bias, relu, tensor_cores):
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n)
    x = torch.randn(m, k, device=DEV, generator=g)
    w = (torch.rand(n, k, device=DEV, generator=g) * 2 - 1).mul_(k ** -0.5).to(dt)
    b = (torch.rand(n, device=DEV, generator=g) * 0.1 - 0.05).to(dt) if bias else None
    err = torch.zeros(1, dtype=torch.int32, device=DEV) if tensor_cores else None
    want, exact, acc = reference(x, w, b, relu, dt)
    for xin in (x, x.to(dt)):  # f32 input (rounded inside) and an already-rounded input
        got = K.cast_linear(xin, w, b, relu=relu, err=err)
        torch.cuda.synchronize()
        # one rounding of a value within the f32 accumulation bound of the exact one
        excess = (got.double() - exact).abs() - (half_ulp(exact, dt) * 1.0001 + acc) * 2
        assert float(excess.max()) <= 0.0, f"worst excess {float(excess.max()):.3g}"
        mismatch = float((got != want).float().mean())
        assert mismatch < 0.02, f"{mismatch:.3%} differ from the rounded reference"
    if err is not None:
        assert int(err.item()) == 0


def test_fp32_linear_is_exact_fp32():
    g = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn(64, 256, device=DEV, generator=g)
    w = torch.randn(96, 256, device=DEV, generator=g) * 0.05
    b = torch.randn(96, device=DEV, generator=g) * 0.05
    got = K.cast_linear(x, w, b)
    want = (x.double() @ w.double().T + b.double()).float()
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)


def test_engine_bf16_dense_batch_tracks_oracle_emulation():
    """A batch of 96 rows routes every CastLinear projection through tcgen05; the
    engine must track the oracle's exact bf16 emulation (MSE bound: bf16 rounding
    flips are amplified by the model, so not per element)."""
    cfg = C.ModelConfig(hidden_size=64, proj_size=128, tower_depth=2, num_heads=4, num_features=79)
    sd = Wt.generate_model(cfg, seed=2)
    eng = EnsembleEngine(cfg, sd, linear_dtype="bf16", capacity=96, max_batch=96)
    orc = O.Oracle(cfg, sd, "bf16")
    state = O.init_state(cfg, 96)
    rng = np.random.default_rng(4)
    slots = np.arange(96, dtype=np.int32)
    for _ in range(3):
        feats = rng.standard_normal((96, 79), dtype=np.float32)
        got = eng.step(slots, feats)
        want, state = orc.step(feats, state)
        power = float(np.mean(want.astype(np.float64) ** 2))
        assert float(np.mean((got - want) ** 2)) <= 1e-4 * power
    assert eng.device_error() == 0
