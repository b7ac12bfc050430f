"""CPU oracle: numpy float32 restatement of the reference's recurrent step.

TEST INFRASTRUCTURE ONLY. This file is the checker the CUDA engine is compared
against; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
may import it, and never as the thing measured or shipped.

It restates, operation for operation, the per-row recurrent step of the
reference's MultiTowerModel (model/inference_model.py:55-146) and its four layers
(model/xlstm.py, model/mamba2.py, model/retnet.py, model/hawk.py, model/modules.py)
in numpy float32. Only the active rows are passed in, so the reference's mask is
implicit: no operator of the model mixes rows (example_model.py:422-427), which
makes stepping a subset of rows identical to the reference's masked step over
all rows.

Parity is pinned against the reference itself: tests/golden/make_golden.py
imports the reference's torch modules, loads the same seeded weights, and
records predictions and state, which tests/test_oracle_golden.py replays here.

`lp` selects the weight storage of CastLinear (example_model.py:68-106): None
is the fp32 path, "bf16"/"fp16" emulate it exactly - the input and the weights
rounded to the low type, a float32 accumulation, the output rounded to the low
type and widened back - for every nn.Linear except the four names kept fp32
(example_model.py:106). BlockLinear, convs and norms stay fp32 either way.

State layout (per block, a flat list of leaves in the reference's init_state
order; see leaf_shapes()):
  xlstm : s_conv (B,H,3) s_h s_c s_n s_m (B,H) m_conv (B,2H,3) m_C (B,nh,hs,hs) m_n (B,nh,hs) m_m (B,nh)
  mamba2: x_conv (B,2H,3) b_conv (B,bc,3) c_conv (B,bc,3) ssm (B,nh,hs,bc)
  retnet: pos int32 (B,) scales (B,nh) S (B,nh,hs,hs)
  hawk  : conv (B,H,3) h (B,H)
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
from scipy.special import erf as _erf

from hackathon_b200.config import CONV_K, TOWER_KINDS, ModelConfig

F32 = np.float32
FP32_LINEAR_NAMES = ("dt_proj", "igate_proj", "fgate_proj", "output_proj")  # example_model.py:106
F32_EPS = float(np.finfo(np.float32).eps)  # nn.RMSNorm(eps=None) uses finfo(float32).eps


def float64_twin():
    """This restatement again, with every operation that runs in float32 here
    carried out in float64 instead (the module's F32 rebound to float64): the
    arbiter that measures how far an fp32 implementation - this one, the
    reference's torch path, the CUDA engine - is from the exact answer of the
    same arithmetic. Weights and inputs widen exactly; the reference's epsilon
    constants keep their values. fp32 weights only (no CastLinear emulation)."""
    import importlib.util

    spec = importlib.util.spec_from_file_location(__name__ + "_float64", __file__)
    twin = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(twin)
    twin.F32 = np.float64
    return twin


# --------------------------------------------------------------- precision


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bfloat16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=F32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(F32).copy()
    out[nan] = np.nan
    return out


def round_fp16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=F32).astype(np.float16).astype(F32)


def lowp(x: np.ndarray, lp: Optional[str]) -> np.ndarray:
    if lp is None:
        return np.asarray(x, dtype=F32)
    if lp == "bf16":
        return round_bf16(x)
    if lp == "fp16":
        return round_fp16(x)
    raise ValueError(lp)


# ------------------------------------------------------------ primitives


def linear(x, w, b=None, lp: Optional[str] = None):
    """nn.Linear / CastLinear.forward (example_model.py:92-95)."""
    if lp is None:
        y = x.astype(F32) @ w.T.astype(F32)
        if b is not None:
            y = y + b.astype(F32)
        return y.astype(F32)
    y = lowp(x, lp) @ lowp(w, lp).T
    if b is not None:
        y = y + lowp(b, lp)
    return lowp(y, lp)


def relu(x):
    return np.maximum(x, F32(0)).astype(F32)


def sigmoid(x):
    return (F32(1) / (F32(1) + np.exp(-x))).astype(F32)


def silu(x):
    return (x * sigmoid(x)).astype(F32)


def softplus(x):
    """F.softplus with beta 1, threshold 20 (model/mamba2.py:92)."""
    return np.where(x > F32(20), x, np.log1p(np.exp(np.minimum(x, F32(20))))).astype(F32)


def logsigmoid(x):
    """F.logsigmoid = min(x,0) - log1p(exp(-|x|)) (model/xlstm.py:40,249)."""
    return (np.minimum(x, F32(0)) - np.log1p(np.exp(-np.abs(x)))).astype(F32)


def gelu(x):
    """F.gelu, exact erf form (model/hawk.py:77)."""
    return (F32(0.5) * x * (F32(1) + _erf(x / F32(math.sqrt(2.0))).astype(F32))).astype(F32)


def rmsnorm(x, w, eps):
    """nn.RMSNorm over the last axis."""
    ms = np.mean(x.astype(F32) * x, axis=-1, keepdims=True, dtype=F32)
    y = x * (F32(1) / np.sqrt(ms + F32(eps)))
    if w is not None:
        y = y * w
    return y.astype(F32)


def layernorm(x, w, b=None, eps=1e-5):
    """nn.LayerNorm(bias=False) over the last axis, biased variance."""
    mu = np.mean(x, axis=-1, keepdims=True, dtype=F32)
    d = x - mu
    var = np.mean(d * d, axis=-1, keepdims=True, dtype=F32)
    y = d / np.sqrt(var + F32(eps)) * w
    if b is not None:
        y = y + b
    return y.astype(F32)


def groupnorm(x, groups, w, b, eps=1e-5):
    """nn.GroupNorm on (B, C): normalise each of `groups` channel groups."""
    bsz, c = x.shape
    g = x.reshape(bsz, groups, c // groups)
    mu = np.mean(g, axis=-1, keepdims=True, dtype=F32)
    d = g - mu
    var = np.mean(d * d, axis=-1, keepdims=True, dtype=F32)
    y = (d / np.sqrt(var + F32(eps))).reshape(bsz, c)
    return (y * w + b).astype(F32)


def conv_step(x, state, w, b):
    """CausalConv1d.forward (model/modules.py:37-41): depthwise k=4 on [state, x]."""
    win = np.concatenate([state, x[:, :, None]], axis=-1)  # (B, C, 4)
    out = np.sum(win * w[None, :, 0, :], axis=-1, dtype=F32) + b
    return out.astype(F32), np.ascontiguousarray(win[:, :, 1:])


def block_linear(x, w, b=None):
    """BlockLinear.forward (model/modules.py:71-79): einsum bnh,nkh->bnk (+bias)."""
    bsz = x.shape[0]
    nb, bs, _ = w.shape
    xv = x.reshape(bsz, nb, bs)
    out = np.einsum("bnh,nkh->bnk", xv, w, optimize=True).astype(F32).reshape(bsz, nb * bs)
    if b is not None:
        out = out + b
    return out.astype(F32)


# ----------------------------------------------------------------- layers


class Weights:
    """Prefix-scoped view of a state_dict with the CastLinear precision rule."""

    def __init__(self, sd: Dict[str, np.ndarray], prefix: str = "", lp: Optional[str] = None):
        self.sd, self.prefix, self.lp = sd, prefix, lp

    def __getitem__(self, key):
        return self.sd[self.prefix + key]

    def get(self, key):
        return self.sd.get(self.prefix + key)

    def sub(self, p: str) -> "Weights":
        return Weights(self.sd, self.prefix + p, self.lp)

    def lin(self, name, x):
        """Apply the nn.Linear stored under `name` with the CastLinear rule."""
        leaf = name.rsplit(".", 1)[-1]
        lp = None if leaf in FP32_LINEAR_NAMES else self.lp
        return linear(x, self[f"{name}.weight"], self.get(f"{name}.bias"), lp)


def mamba2_step(W: Weights, t, st, head_size=64, bc=128):
    """Mamba2.forward (model/mamba2.py:62-168), torch branch (:128-165)."""
    x_conv, b_conv, c_conv, ssm = st
    bsz = t.shape[0]
    x = W.lin("input_proj", t)
    z = W.lin("z_proj", t)
    b = W.lin("b_proj", t)
    c = W.lin("c_proj", t)
    dt = W.lin("dt_proj", t)
    x, x_conv = conv_step(x, x_conv, W["input_conv.conv.weight"], W["input_conv.conv.bias"])
    b, b_conv = conv_step(b, b_conv, W["b_conv.conv.weight"], W["b_conv.conv.bias"])
    c, c_conv = conv_step(c, c_conv, W["c_conv.conv.weight"], W["c_conv.conv.bias"])
    x, b, c = silu(x), silu(b), silu(c)
    nh = x.shape[1] // head_size
    xh = x.reshape(bsz, nh, head_size)
    dt = softplus(dt)
    decay = np.exp(W["a"][None] * dt).astype(F32)
    ssm_new = (decay[:, :, None, None] * ssm + (dt[:, :, None, None] * b[:, None, None, :]) * xh[:, :, :, None]).astype(F32)
    y = np.sum(c[:, None, None, :] * ssm_new, axis=-1, dtype=F32)
    y = (y + W["d"][None, :, None] * xh).reshape(bsz, nh * head_size)
    y = y * silu(z)
    y = rmsnorm(y, W["norm.weight"], 1e-5)
    return W.lin("out_proj", y), [x_conv, b_conv, c_conv, ssm_new]


def rotate_every_two(x):
    """model/retnet.py:9-13."""
    x1, x2 = x[..., ::2], x[..., 1::2]
    return np.stack((-x2, x1), axis=-1).reshape(x.shape)


def retnet_step(W: Weights, x, st, heads):
    """RetNet.forward (model/retnet.py:38-172), torch branch (:124-170)."""
    pos, scales, S = st
    bsz, hidden = x.shape
    hs = hidden // heads
    q = W.lin("q_proj", x)
    k = W.lin("k_proj", x)
    v = W.lin("v_proj", x)
    g = W.lin("g_proj", x)
    k = (k * F32(hs ** -0.5)).astype(F32)
    qh, kh, vh = (a.reshape(bsz, heads, hs) for a in (q, k, v))
    arg = (pos.astype(F32)[:, None, None] * W["angle"][None, None, :]).astype(F32)
    sin, cos = np.sin(arg).astype(F32), np.cos(arg).astype(F32)
    q_rope = (qh * cos + rotate_every_two(qh) * sin).astype(F32)
    k_rope = (kh * cos + rotate_every_two(kh) * sin).astype(F32)
    new_scales = (scales * W["decay"] + F32(1)).astype(F32)
    q_scaled = (q_rope * (F32(1) / np.sqrt(new_scales))[:, :, None]).astype(F32)
    S_new = (S * W["decay"][None, :, None, None] + k_rope[:, :, :, None] * vh[:, :, None, :]).astype(F32)
    out = np.sum(q_scaled[:, :, :, None] * S_new, axis=2, dtype=F32)
    out = rmsnorm(out, None, 1e-6).reshape(bsz, hidden)
    out = silu(g) * out
    return W.lin("out_proj", out), [(pos + 1).astype(np.int32), new_scales, S_new]


def hawk_step(W: Weights, x, st):
    """Hawk.forward + RGLRU.forward (model/hawk.py:60-87, 19-37)."""
    conv, h = st
    gate = gelu(W.lin("gate_proj", x))
    xr = W.lin("recurrent_proj", x)
    xr, conv = conv_step(xr, conv, W["conv.conv.weight"], W["conv.conv.bias"])
    i_t = sigmoid(block_linear(xr, W["rglru.input_gate.weight"]))
    r_t = sigmoid(block_linear(xr, W["rglru.recurrence_gate.weight"]))
    a_t = np.power(W["rglru.a"], F32(8.0) * r_t).astype(F32)
    mult = np.sqrt(F32(1) - a_t * a_t).astype(F32)
    h_new = (h * a_t + mult * (i_t * xr)).astype(F32)
    return W.lin("out_proj", gate * h_new), [conv, h_new]


def slstm_block_step(W: Weights, x, st, heads):
    """SLSTMBlock.forward + SLSTMCell.forward (model/xlstm.py:304-318, 247-274)."""
    conv, h, c, n, m = st
    skip = x
    xn = layernorm(x, W["norm.weight"])
    xc, conv = conv_step(xn, conv, W["conv1d.conv.weight"], W["conv1d.conv.bias"])
    xca = silu(xc)

    def bl(name, a):
        return block_linear(a, W[f"{name}.weight"], W.get(f"{name}.bias"))

    i = bl("igate_input", xca) + bl("igate_state", h)
    f = bl("fgate_input", xca) + bl("fgate_state", h)
    z = bl("zgate_input", xn) + bl("zgate_state", h)
    o = bl("ogate_input", xn) + bl("ogate_state", h)
    with np.errstate(invalid="ignore", over="ignore"):
        lfm = (m + logsigmoid(f)).astype(F32)
        m_new = np.maximum(i, lfm).astype(F32)
        o_g = sigmoid(o)
        i_g = np.exp(i - m_new).astype(F32)
        f_g = np.exp(lfm - m_new).astype(F32)
        c_new = (f_g * c + i_g * np.tanh(z)).astype(F32)
        n_new = (f_g * n + i_g).astype(F32)
        y = (o_g * c_new / (n_new + F32(1e-6))).astype(F32)
    out = groupnorm(y, heads, W["group_norm.weight"], W["group_norm.bias"])
    return (out + skip).astype(F32), [conv, y, c_new, n_new, m_new]


def mlstm_cell_step(W: Weights, q, k, v, st, heads):
    """MLSTMCell.forward (model/xlstm.py:33-154), torch branch (:144-154)."""
    C, n, m = st
    bsz, inner = q.shape
    hs = inner // heads
    qkv = np.concatenate([q, k, v], axis=-1)
    ig = W.lin("igate_proj", qkv)
    fg = W.lin("fgate_proj", qkv)
    qh, kh, vh = (a.reshape(bsz, heads, hs) for a in (q, k, v))
    log_f = logsigmoid(fg)
    m_new = np.maximum(ig, m + log_f).astype(F32)
    i_g = np.exp(ig - m_new).astype(F32)
    f_g = np.exp(log_f + m - m_new).astype(F32)
    kh = (kh / F32(math.sqrt(hs))).astype(F32)
    n_new = (f_g[:, :, None] * n + i_g[:, :, None] * kh).astype(F32)
    C_new = (f_g[:, :, None, None] * C + (i_g[:, :, None, None] * kh[:, :, :, None]) * vh[:, :, None, :]).astype(F32)
    num = np.sum(qh[:, :, :, None] * C_new, axis=2, dtype=F32)
    qn = np.sum(qh * n_new, axis=-1, dtype=F32)
    den = (np.maximum(np.abs(qn), np.exp(-m_new)) + F32(1e-6)).astype(F32)
    out = (num / den[:, :, None]).reshape(bsz, inner)
    out = groupnorm(out, heads, W["outnorm.weight"], W["outnorm.bias"])
    return out, [C_new, n_new, m_new]


def mlstm_block_step(W: Weights, x, st, heads):
    """MLSTMBlock.forward (model/xlstm.py:198-225)."""
    conv, C, n, m = st
    skip = x
    xn = layernorm(x, W["norm.weight"])
    x_m = W.lin("x_proj", xn)
    x_g = W.lin("gate_proj", xn)
    xc, conv = conv_step(x_m, conv, W["conv1d.conv.weight"], W["conv1d.conv.bias"])
    xca = silu(xc)
    q = block_linear(xca, W["q_proj.weight"])
    k = block_linear(xca, W["k_proj.weight"])
    v = block_linear(x_m, W["v_proj.weight"])
    out, (C, n, m) = mlstm_cell_step(W.sub("mlstm_cell."), q, k, v, (C, n, m), heads)
    h = (out + W["learnable_skip"] * xca) * silu(x_g)
    y = W.lin("proj_down", h)
    return (y + skip).astype(F32), [conv, C, n, m]


def xlstm_step(W: Weights, x, st, cfg: ModelConfig):
    """XLSTM.forward (model/xlstm.py:355-367)."""
    x, s_st = slstm_block_step(W.sub("slstm."), x, st[:5], cfg.slstm_heads)
    x, m_st = mlstm_block_step(W.sub("mlstm."), x, st[5:], cfg.mlstm_heads)
    return layernorm(x, W["final_norm.weight"]), s_st + m_st


def layer_step(kind: str, W: Weights, x, st, cfg: ModelConfig):
    if kind == "xlstm":
        return xlstm_step(W, x, st, cfg)
    if kind == "mamba2":
        return mamba2_step(W, x, st, cfg.mamba_head_size, cfg.mamba_bc_size)
    if kind == "retnet":
        return retnet_step(W, x, st, cfg.num_heads)
    if kind == "hawk":
        return hawk_step(W, x, st)
    raise ValueError(kind)


# ----------------------------------------------------------------- model


def leaf_shapes(kind: str, cfg: ModelConfig) -> List[Tuple[Tuple[int, ...], type]]:
    """Per-row shapes and dtypes of one block's state leaves, init_state order."""
    h = cfg.hidden_size
    if kind == "xlstm":
        inner, nh, hs = cfg.mlstm_inner, cfg.mlstm_heads, cfg.mlstm_head_size
        return [((h, CONV_K - 1), F32), ((h,), F32), ((h,), F32), ((h,), F32), ((h,), F32),
                ((inner, CONV_K - 1), F32), ((nh, hs, hs), F32), ((nh, hs), F32), ((nh,), F32)]
    if kind == "mamba2":
        inner, nh, hs, bc = cfg.mamba_inner, cfg.mamba_heads, cfg.mamba_head_size, cfg.mamba_bc_size
        return [((inner, CONV_K - 1), F32), ((bc, CONV_K - 1), F32), ((bc, CONV_K - 1), F32),
                ((nh, hs, bc), F32)]
    if kind == "retnet":
        nh, hs = cfg.num_heads, cfg.retnet_head_size
        return [((), np.int32), ((nh,), F32), ((nh, hs, hs), F32)]
    if kind == "hawk":
        return [((h, CONV_K - 1), F32), ((h,), F32)]
    raise ValueError(kind)


def init_block_state(kind: str, cfg: ModelConfig, bsz: int) -> List[np.ndarray]:
    """Layer init_state (model/xlstm.py:232-236,331-336,369-379; mamba2.py:48-60;
    retnet.py:174-189; hawk.py:89-95). sLSTM's running max starts at -inf (xlstm.py:280)."""
    leaves = [np.zeros((bsz,) + shp, dtype=dt) for shp, dt in leaf_shapes(kind, cfg)]
    if kind == "xlstm":
        leaves[4][:] = -np.inf
    return leaves


def init_state(cfg: ModelConfig, bsz: int) -> List[List[List[np.ndarray]]]:
    return [[init_block_state(kind, cfg, bsz) for _ in range(cfg.tower_depth)] for kind in TOWER_KINDS]


def flat_leaves(state) -> List[np.ndarray]:
    """Leaves in the reference's iter_state_tensors order (example_model.py:160-176)."""
    return [leaf for tower in state for block in tower for leaf in block]


class Oracle:
    """The whole ensemble step on CPU: `step(features, state) -> (preds, state)`."""

    def __init__(self, cfg: ModelConfig, sd: Dict[str, np.ndarray], lp: Optional[str] = None):
        cfg.validate()
        if lp is not None and F32 is not np.float32:
            raise ValueError("the float64 twin has no CastLinear emulation (lp must be None)")
        self.cfg, self.lp = cfg, lp
        self.sd = {k: np.ascontiguousarray(v, dtype=F32) for k, v in sd.items()}

    def tower_step(self, t: int, feats, tower_state):
        """Tower.forward (model/inference_model.py:85-95) + Block.forward (:63-68)."""
        cfg, kind = self.cfg, TOWER_KINDS[t]
        W = Weights(self.sd, f"towers.{t}.", self.lp)
        x = relu(W.lin("input_up", feats))
        x = W.lin("input_down", x)
        new_state = []
        for b in range(cfg.tower_depth):
            B = W.sub(f"blocks.{b}.")
            y, st = layer_step(kind, B.sub("layer."), rmsnorm(x, B["norm1.weight"], F32_EPS), tower_state[b], cfg)
            x = (y + x).astype(F32)
            h = relu(B.lin("mlp.fc1", rmsnorm(x, B["norm2.weight"], F32_EPS)))
            x = (x + B.lin("mlp.fc2", h)).astype(F32)
            new_state.append(st)
        return x, new_state

    def step(self, feats: np.ndarray, state):
        """MultiTowerModel.forward (model/inference_model.py:119-143) on the given rows."""
        feats = np.ascontiguousarray(feats, dtype=F32)
        W = Weights(self.sd, "", self.lp)
        cols, new_state = [], []
        for t in range(len(TOWER_KINDS)):
            x, st = self.tower_step(t, feats, state[t])
            cols.append(W.lin("output_proj", x))
            new_state.append(st)
        return np.concatenate(cols, axis=1).astype(F32), new_state


def gather_rows(state, rows: Sequence[int]):
    idx = np.asarray(rows, dtype=np.int64)
    return [[[leaf[idx] for leaf in blk] for blk in tower] for tower in state]


def scatter_rows(state, rows: Sequence[int], sub) -> None:
    idx = np.asarray(rows, dtype=np.int64)
    for tower, stower in zip(state, sub):
        for blk, sblk in zip(tower, stower):
            for leaf, sleaf in zip(blk, sblk):
                leaf[idx] = sleaf
