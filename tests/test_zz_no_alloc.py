"""b2e_linear_static, the projection for callers that cannot allocate device
memory (a host whose device memory all belongs to its own pool, or a loop that
must not allocate after start-up): its scratch is a static array inside the
library. Checked through the C-ABI against b2e_linear on the same operands, two
calls in a row, so the second call runs on the scratch the first one left.

This file is named to be collected last: a failure here stops a `-x` run only
after every other test has run.
"""

import ctypes as C

import pytest
import torch

from hackathon_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def _p(t):
    return C.c_void_p(t.data_ptr() if t is not None else 0)


def _stream():
    return C.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)


def linear(x, w, b, relu):
    """The existing entry point, tensor cores allowed (a caller-allocated error word)."""
    y = torch.empty(x.shape[0], w.shape[0], device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    _lib.check(_lib.lib().b2e_linear(_p(x), DT[x.dtype], x.shape[0], x.shape[1], _p(w), DT[w.dtype], _p(b),
                                     w.shape[0], int(relu), _p(y), _p(err), _stream()))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return y


def linear_static(x, w, b, relu):
    y = torch.empty(x.shape[0], w.shape[0], device=DEV)
    h_err = C.c_int32(-1)
    _lib.check(_lib.lib().b2e_linear_static(_p(x), DT[x.dtype], x.shape[0], x.shape[1], _p(w), DT[w.dtype], _p(b),
                                            w.shape[0], int(relu), _p(y), C.byref(h_err), _stream()))
    assert h_err.value == 0
    return y


def bound(x, w, dt):
    """Two CastLinear results may differ by the rounding of each plus the f32
    accumulation-order bound (the tolerance of the b2e_linear tests)."""
    xr, wd = x.to(dt).double(), w.double()
    y = xr @ wd.T
    mant = 8 if dt == torch.bfloat16 else 11
    half_ulp = 0.5 * 2.0 ** (torch.floor(torch.log2(torch.clamp(y.abs(), min=2.0 ** -100))) - (mant - 1))
    acc = 4.0 * x.shape[1] ** 0.5 * 2.0 ** -24 * (xr.abs() @ wd.abs().T)
    return 4 * (half_ulp * 1.0001 + acc)


def operands(m, k, n, dt, x_dt, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(m, k, device=DEV, generator=g)
    w = ((torch.rand(n, k, device=DEV, generator=g) * 2 - 1) * k ** -0.5).to(dt)
    b = (torch.rand(n, device=DEV, generator=g) * 0.1 - 0.05).to(dt)
    return x.to(x_dt), w, b


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_static_scratch_matches_linear_on_two_calls_in_a_row(dt):
    # call 1: f32 x, rounded into the static buffer (b2e_linear runs it on SIMT)
    x1, w1, b1 = operands(640, 512, 384, dt, torch.float32, 11)
    got1 = linear_static(x1, w1, b1, relu=True)
    # call 2: a smaller f32 x over the first call's leftover scratch
    x2, w2, b2 = operands(200, 256, 512, dt, torch.float32, 12)
    got2 = linear_static(x2, w2, b2, relu=False)
    torch.cuda.synchronize()
    for x, w, b, relu, got in ((x1, w1, b1, True, got1), (x2, w2, b2, False, got2)):
        want = linear(x, w, b, relu)
        excess = (got.double() - want.double()).abs() - bound(x, w, dt)
        assert float(excess.max()) <= 0.0, f"worst excess {float(excess.max()):.3g}"
        assert float((got != want).float().mean()) < 0.02

    # x already in the weight's type: both entry points run the same tensor-core
    # kernel, so the results are identical bit for bit
    x3, w3, b3 = operands(300, 512, 256, dt, dt, 13)
    for _ in range(2):
        assert torch.equal(linear_static(x3, w3, b3, relu=False), linear(x3, w3, b3, relu=False))


def test_static_scratch_f32_input_within_one_rounding_of_float64():
    """The f32-input result (x rounded into the static buffer) against a float64
    restatement of CastLinear: x and the weight in the weight's type, exact
    products and sums, bias added, ReLU, within the rounding bound above."""
    for dt in (torch.bfloat16, torch.float16):
        x, w, b = operands(512, 384, 320, dt, torch.float32, 21)
        got = linear_static(x, w, b, relu=True)
        want = torch.relu(x.to(dt).double() @ w.double().T + b.double())
        excess = (got.double() - want).abs() - bound(x, w, dt)
        assert float(excess.max()) <= 0.0, f"{dt}: worst excess {float(excess.max()):.3g}"


def test_static_scratch_calls_allocate_no_device_memory():
    """Repeated calls (after one warm-up round, which loads the kernels) leave
    the device's free memory exactly where it was: no allocation on the path."""
    dt = torch.bfloat16
    ops = [operands(640, 512, 384, dt, torch.float32, 31), operands(300, 512, 256, dt, dt, 32)]
    ys = [torch.empty(x.shape[0], w.shape[0], device=DEV) for x, w, _ in ops]
    h_err = C.c_int32(-1)

    def run(with_err):
        for (x, w, b), y in zip(ops, ys):
            _lib.check(_lib.lib().b2e_linear_static(_p(x), DT[x.dtype], x.shape[0], x.shape[1], _p(w), DT[w.dtype],
                                                    _p(b), w.shape[0], 0, _p(y),
                                                    C.byref(h_err) if with_err else None, _stream()))
        torch.cuda.synchronize()

    run(True)
    run(False)
    free0 = torch.cuda.mem_get_info(DEV)[0]
    for i in range(5):
        run(i % 2 == 0)
    assert torch.cuda.mem_get_info(DEV)[0] == free0
    assert h_err.value == 0


def test_static_scratch_refuses_inputs_beyond_its_size():
    x = torch.zeros(4097, 2048, device=DEV)  # m * k = 8390656 > 8388608
    w = torch.zeros(16, 2048, dtype=torch.bfloat16, device=DEV)
    y = torch.empty(4097, 16, device=DEV)
    rc = _lib.lib().b2e_linear_static(_p(x), 0, 4097, 2048, _p(w), 1, None, 16, 0, _p(y), None, _stream())
    assert rc == -1  # B2E_ERR_INVALID
    assert b"8388608" in _lib.lib().b2e_last_error()
