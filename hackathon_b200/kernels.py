"""The fused state steps, with the reference's operator API.

Drop-in for model/kernels.py's ``mlstm_step``, ``retnet_step`` and
``mamba2_step`` (model/kernels.py:346-401): same arguments, same semantics, same
refusals. The state is updated IN PLACE on active rows (idle rows stay bit
for bit), the returned output is a fresh contiguous float32 tensor with zeros on
idle rows, and ``mask=None`` means every row is active. Operands may be strided
views (they are made contiguous); the state may not, because it is written in
place. Errors raise AssertionError, like the reference's wrappers
(model/kernels.py:85-122). The computation is libb2e.so's CUDA kernels on the
current torch stream; there is no CPU path.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib


def _small(t: torch.Tensor, shape: tuple, name: str, device) -> torch.Tensor:
    # model/kernels.py:85-98: fp32 asserted, never cast; shape and device checked.
    assert t.dtype == torch.float32, f"{name} must be fp32, got {t.dtype}"
    assert tuple(t.shape) == shape, f"{name} must be {shape}, got {tuple(t.shape)}"
    assert t.device == device, f"{name} must be on {device}, it is on {t.device}"
    return t.contiguous()


def _mask_u8(mask, batch: int, device):
    # model/kernels.py:101-113; the contiguous copy also packs a strided mask.
    if mask is None:
        return None
    assert mask.dtype == torch.bool, f"mask must be bool, got {mask.dtype}"
    assert tuple(mask.shape) == (batch,), f"mask must be ({batch},), got {tuple(mask.shape)}"
    assert mask.device == device, f"mask must be on {device}, it is on {mask.device}"
    return mask.to(torch.uint8).contiguous()


def _state_ok(state: torch.Tensor, name: str) -> None:
    # model/kernels.py:116-121: written in place, so never copied.
    assert state.dtype == torch.float32, f"{name} must be fp32, got {state.dtype}"
    assert state.is_contiguous(), f"{name} must be contiguous, it is written in place"
    assert state.dim() == 4, f"{name} must be 4-D, got {tuple(state.shape)}"
    assert state.is_cuda, f"{name} must be a CUDA tensor (there is no CPU path)"


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(device) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def mlstm_step(cell, q, k, v, i_gate, f_gate, mask):
    """cell <- f*cell + i*(k outer v) on active rows; return sum_h q*cell_new."""
    _state_ok(cell, "cell")
    b, n, sh, sk = cell.shape
    dev = cell.device
    q = _small(q, (b, n, sh), "q", dev)
    k = _small(k, (b, n, sh), "k", dev)
    v = _small(v, (b, n, sk), "v", dev)
    i_gate = _small(i_gate, (b, n), "i_gate", dev)
    f_gate = _small(f_gate, (b, n), "f_gate", dev)
    m = _mask_u8(mask, b, dev)
    out = torch.empty(b, n, sk, dtype=torch.float32, device=dev)
    if b:
        _lib.check(_lib.lib().b2e_mlstm_step(_ptr(cell), _ptr(q), _ptr(k), _ptr(v), _ptr(i_gate), _ptr(f_gate),
                                             _ptr(m), b, n, sh, sk, _ptr(out), _stream(dev)))
    return out


def retnet_step(state, k_rope, v, q_scaled, decay, mask):
    """state <- decay*state + (k outer v) on active rows; return sum_h q_scaled*state_new."""
    _state_ok(state, "state")
    b, n, sh, sk = state.shape
    dev = state.device
    k_rope = _small(k_rope, (b, n, sh), "k_rope", dev)
    v = _small(v, (b, n, sk), "v", dev)
    q_scaled = _small(q_scaled, (b, n, sh), "q_scaled", dev)
    decay = _small(decay, (n,), "decay", dev)
    m = _mask_u8(mask, b, dev)
    out = torch.empty(b, n, sk, dtype=torch.float32, device=dev)
    if b:
        _lib.check(_lib.lib().b2e_retnet_step(_ptr(state), _ptr(k_rope), _ptr(v), _ptr(q_scaled), _ptr(decay),
                                              _ptr(m), b, n, sh, sk, _ptr(out), _stream(dev)))
    return out


def mamba2_step(ssm, x, b, c, dt, decay, mask):
    """ssm <- decay*ssm + dt*(b outer x) on active rows; return sum_c c*ssm_new."""
    _state_ok(ssm, "ssm")
    bs, n, sh, sc = ssm.shape
    dev = ssm.device
    x = _small(x, (bs, n, sh), "x", dev)
    b = _small(b, (bs, sc), "b", dev)
    c = _small(c, (bs, sc), "c", dev)
    dt = _small(dt, (bs, n), "dt", dev)
    decay = _small(decay, (bs, n), "decay", dev)
    m = _mask_u8(mask, bs, dev)
    out = torch.empty(bs, n, sh, dtype=torch.float32, device=dev)
    if bs:
        _lib.check(_lib.lib().b2e_mamba2_step(_ptr(ssm), _ptr(x), _ptr(b), _ptr(c), _ptr(dt), _ptr(decay),
                                              _ptr(m), bs, n, sh, sc, _ptr(out), _stream(dev)))
    return out


_TORCH_DTYPES = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def set_state_kernel_waves(waves: int) -> int:
    """Grid of the state kernels when they stream alone (this module's three steps
    and the layer engine): waves > 0 short CTAs of a few items, ~waves waves of two
    CTAs per SM (default 8, the fastest alone); 0 one persistent CTA per SM, the
    grid the ensemble engine's step uses. Results are identical bit for bit.
    Process-wide; returns the previous value (b2e_set_state_kernel_waves)."""
    prev = C.c_int32()
    _lib.check(_lib.lib().b2e_set_state_kernel_waves(int(waves), C.byref(prev)))
    return prev.value


def cast_linear(x, weight, bias=None, relu: bool = False, err=None):
    """CastLinear.forward (example_model.py:92-95) / nn.Linear on the GPU.

    ``weight`` (out, in) is float32, bfloat16 or float16. With a low-precision
    weight, x is rounded to its type, products accumulate in float32, the bias
    (same type as the weight) is added and the result is rounded to the weight's
    type before widening: exactly CastLinear. Returns a new float32 tensor.
    ``err`` is an optional int32 CUDA tensor of one element that receives an error
    code if the tensor-core kernel times out; without it the tensor-core kernel
    is not used.
    """
    assert weight.is_cuda and weight.dim() == 2 and weight.is_contiguous()
    wt = _TORCH_DTYPES[weight.dtype]
    assert x.dtype in (torch.float32, weight.dtype), f"x must be fp32 or {weight.dtype}, got {x.dtype}"
    assert x.device == weight.device and x.dim() == 2 and x.shape[1] == weight.shape[1]
    x = x.contiguous()
    if bias is not None:
        assert bias.dtype == weight.dtype and bias.shape == (weight.shape[0],)
        bias = bias.contiguous()
    y = torch.empty(x.shape[0], weight.shape[0], dtype=torch.float32, device=x.device)
    _lib.check(_lib.lib().b2e_linear(_ptr(x), _TORCH_DTYPES[x.dtype], x.shape[0], x.shape[1], _ptr(weight), wt,
                                     _ptr(bias), weight.shape[0], int(relu), _ptr(y), _ptr(err), _stream(x.device)))
    return y
