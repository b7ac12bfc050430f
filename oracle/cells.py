"""CPU oracle for the three fused state steps of the reference.

TEST INFRASTRUCTURE ONLY (see oracle/model.py's header for who may use it).

Restates model/kernels.py's torch references and their masked write-back:
  mlstm_step_reference  (model/kernels.py:143-151)
  retnet_step_reference (model/kernels.py:154-160)
  mamba2_step_reference (model/kernels.py:163-171)
  _write_back           (model/kernels.py:124-137)
Semantics: the state is updated in place on active rows only, idle rows keep
their old value bit for bit, and the returned output is zero on idle rows;
mask None means every row is active.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def _write_back(state, new, out, mask):
    if mask is None:
        state[...] = new
        return out
    m = np.asarray(mask, dtype=bool)
    state[m] = new[m]
    out = out.copy()
    out[~m] = 0.0
    return out


def mlstm_step(cell, q, k, v, i_gate, f_gate, mask):
    """cell <- f*cell + i*(k outer v); return sum_h q*cell_new (kernels.py:143-151)."""
    new = (f_gate[:, :, None, None] * cell + (i_gate[:, :, None, None] * k[:, :, :, None]) * v[:, :, None, :]).astype(F32)
    num = np.sum(q[:, :, :, None] * new, axis=2, dtype=F32)
    return _write_back(cell, new, num, mask)


def retnet_step(state, k_rope, v, q_scaled, decay, mask):
    """state <- decay*state + (k outer v); return sum_h q_scaled*state_new (kernels.py:154-160)."""
    new = (state * decay[None, :, None, None] + k_rope[:, :, :, None] * v[:, :, None, :]).astype(F32)
    out = np.sum(q_scaled[:, :, :, None] * new, axis=2, dtype=F32)
    return _write_back(state, new, out, mask)


def mamba2_step(ssm, x, b, c, dt, decay, mask):
    """ssm <- decay*ssm + dt*(b outer x); return sum_c c*ssm_new (kernels.py:163-171)."""
    new = (decay[:, :, None, None] * ssm + (dt[:, :, None, None] * b[:, None, None, :]) * x[:, :, :, None]).astype(F32)
    y = np.sum(c[:, None, None, :] * new, axis=-1, dtype=F32)
    return _write_back(ssm, new, y, mask)
