"""Seeded synthetic weights in the reference's state_dict layout.

The reference ships several parameters as ``torch.empty`` that only its Hugging
Face checkpoint fills (BlockLinear weights model/modules.py:63-69, RetNet
``decay``/``angle`` model/retnet.py:35-36, RG-LRU ``a`` model/hawk.py:16), and
that checkpoint is not available offline. Its own equivalence checker fills
every parameter and buffer with ``randomize_`` (check_cell_rewrite.py:177-210),
whose value ranges keep gates and decays where a trained model puts them. This
module draws weights from exactly those ranges, under exactly the reference's
key names and shapes, from a deterministic per-tensor stream:

    values(name) = lo + (hi - lo) * U[0,1)   (float32),
    U drawn by numpy PCG64 seeded with (seed, crc32(name)).

Seeding per name makes the draw independent of iteration order and cheap to
reproduce on any host (the 1.99 B-parameter default model regenerates in about
twenty seconds), so a multi-gigabyte weight file never has to be shipped: the
engine, the CPU oracle and the reference itself all load the same dict.
"""

from __future__ import annotations

import math
import zlib
from dataclasses import dataclass
from typing import Dict, Iterable, List, Tuple

import numpy as np

from .config import CONV_K, ModelConfig, TOWER_KINDS


@dataclass(frozen=True)
class ParamSpec:
    name: str
    shape: Tuple[int, ...]
    lo: float
    hi: float
    linear: bool = False  # an nn.Linear weight/bias (CastLinear converts these)


def _fan(shape: Tuple[int, ...]) -> Tuple[float, float]:
    # randomize_'s default branch: U(-s, s), s = 1/sqrt(shape[-1])
    # (check_cell_rewrite.py:208-210).
    s = 1.0 / math.sqrt(shape[-1])
    return -s, s


NORM_W = (0.9, 1.1)  # norm weights (check_cell_rewrite.py:204-205)
BIAS = (-0.05, 0.05)  # biases and other norm params (check_cell_rewrite.py:206-207)


def _linear(name: str, out_f: int, in_f: int, bias: bool) -> List[ParamSpec]:
    specs = [ParamSpec(f"{name}.weight", (out_f, in_f), *_fan((out_f, in_f)), linear=True)]
    if bias:
        specs.append(ParamSpec(f"{name}.bias", (out_f,), *BIAS, linear=True))
    return specs


def _conv(name: str, channels: int) -> List[ParamSpec]:
    # CausalConv1d wraps nn.Conv1d as `.conv` (model/modules.py:34-36).
    shape = (channels, 1, CONV_K)
    return [
        ParamSpec(f"{name}.conv.weight", shape, *_fan(shape)),
        ParamSpec(f"{name}.conv.bias", (channels,), *BIAS),
    ]


def _block_linear(name: str, blocks: int, size: int, bias: bool) -> List[ParamSpec]:
    bs = size // blocks
    shape = (blocks, bs, bs)
    specs = [ParamSpec(f"{name}.weight", shape, *_fan(shape))]
    if bias:
        specs.append(ParamSpec(f"{name}.bias", (size,), *BIAS))
    return specs


def _norm(name: str, size: int, bias: bool = False) -> List[ParamSpec]:
    specs = [ParamSpec(f"{name}.weight", (size,), *NORM_W)]
    if bias:
        specs.append(ParamSpec(f"{name}.bias", (size,), *BIAS))
    return specs


def xlstm_specs(p: str, cfg: ModelConfig) -> List[ParamSpec]:
    """XLSTM layer (model/xlstm.py:339-379): sLSTM block, mLSTM block, final norm."""
    h, nh_s, inner, nh_m = cfg.hidden_size, cfg.slstm_heads, cfg.mlstm_inner, cfg.mlstm_heads
    s: List[ParamSpec] = []
    s += _norm(f"{p}slstm.norm", h)
    s += _conv(f"{p}slstm.conv1d", h)
    for g in "ifzo":
        s += _block_linear(f"{p}slstm.{g}gate_input", nh_s, h, bias=False)
    for g in "ifzo":
        s += _block_linear(f"{p}slstm.{g}gate_state", nh_s, h, bias=True)
    s += _norm(f"{p}slstm.group_norm", h, bias=True)
    s.append(ParamSpec(f"{p}mlstm.learnable_skip", (inner,), 0.9, 1.1))
    s += _norm(f"{p}mlstm.norm", h)
    s += _linear(f"{p}mlstm.x_proj", inner, h, bias=False)
    s += _linear(f"{p}mlstm.gate_proj", inner, h, bias=False)
    for g in "qkv":
        s += _block_linear(f"{p}mlstm.{g}_proj", inner // 4, inner, bias=False)
    s += _conv(f"{p}mlstm.conv1d", inner)
    s += mlstm_cell_specs(f"{p}mlstm.mlstm_cell.", inner, nh_m)
    s += _linear(f"{p}mlstm.proj_down", h, inner, bias=False)
    s += _norm(f"{p}final_norm", h)
    return s


def mlstm_cell_specs(p: str, inner: int, heads: int) -> List[ParamSpec]:
    """MLSTMCell (model/xlstm.py:21-31): fp32 gate projections and GroupNorm."""
    s: List[ParamSpec] = []
    s += _linear(f"{p}igate_proj", heads, 3 * inner, bias=True)
    s += _linear(f"{p}fgate_proj", heads, 3 * inner, bias=True)
    s += _norm(f"{p}outnorm", inner, bias=True)
    return s


def mamba2_specs(p: str, hidden: int, head_size: int = 64, bc: int = 128) -> List[ParamSpec]:
    """Mamba2 layer (model/mamba2.py:9-46)."""
    inner = 2 * hidden
    nh = inner // head_size
    s: List[ParamSpec] = [
        ParamSpec(f"{p}a", (nh,), -16.0, -1.0),  # check_cell_rewrite.py:194-195
        ParamSpec(f"{p}d", (nh,), 0.5, 1.5),  # check_cell_rewrite.py:196-197
    ]
    s += _linear(f"{p}input_proj", inner, hidden, bias=False)
    s += _linear(f"{p}z_proj", inner, hidden, bias=False)
    s += _linear(f"{p}b_proj", bc, hidden, bias=False)
    s += _linear(f"{p}c_proj", bc, hidden, bias=False)
    s += _linear(f"{p}dt_proj", nh, hidden, bias=True)
    s += _conv(f"{p}input_conv", inner)
    s += _conv(f"{p}b_conv", bc)
    s += _conv(f"{p}c_conv", bc)
    s += _norm(f"{p}norm", inner)
    s += _linear(f"{p}out_proj", hidden, inner, bias=False)
    return s


def retnet_specs(p: str, hidden: int, heads: int) -> List[ParamSpec]:
    """RetNet layer (model/retnet.py:16-36); decay/angle are buffers."""
    hs = hidden // heads
    s: List[ParamSpec] = [
        ParamSpec(f"{p}decay", (heads,), 0.85, 0.99),  # check_cell_rewrite.py:198-199
        ParamSpec(f"{p}angle", (hs,), 0.01, 0.2),  # check_cell_rewrite.py:200-201
    ]
    for g in "qkvg":
        s += _linear(f"{p}{g}_proj", hidden, hidden, bias=False)
    s += _linear(f"{p}out_proj", hidden, hidden, bias=False)
    return s


def hawk_specs(p: str, hidden: int) -> List[ParamSpec]:
    """Hawk layer + RG-LRU (model/hawk.py:8-66)."""
    s: List[ParamSpec] = []
    s += _linear(f"{p}gate_proj", hidden, hidden, bias=False)
    s += _linear(f"{p}recurrent_proj", hidden, hidden, bias=False)
    s += _conv(f"{p}conv", hidden)
    s.append(ParamSpec(f"{p}rglru.a", (hidden,), 0.1, 0.9))  # check_cell_rewrite.py:192-193
    s += _block_linear(f"{p}rglru.input_gate", 4, hidden, bias=False)
    s += _block_linear(f"{p}rglru.recurrence_gate", 4, hidden, bias=False)
    s += _linear(f"{p}out_proj", hidden, hidden, bias=False)
    return s


def layer_specs(kind: str, p: str, cfg: ModelConfig) -> List[ParamSpec]:
    if kind == "xlstm":
        return xlstm_specs(p, cfg)
    if kind == "mamba2":
        return mamba2_specs(p, cfg.hidden_size, cfg.mamba_head_size, cfg.mamba_bc_size)
    if kind == "retnet":
        return retnet_specs(p, cfg.hidden_size, cfg.num_heads)
    if kind == "hawk":
        return hawk_specs(p, cfg.hidden_size)
    raise ValueError(f"unknown layer kind {kind!r}")


def param_specs(cfg: ModelConfig) -> List[ParamSpec]:
    """Every tensor of MultiTowerModel.state_dict() (model/inference_model.py:55-146)."""
    cfg.validate()
    h, pj, f = cfg.hidden_size, cfg.proj_size, cfg.num_features
    specs: List[ParamSpec] = []
    for t, kind in enumerate(TOWER_KINDS):
        tp = f"towers.{t}."
        specs += _linear(f"{tp}input_up", pj, f, bias=True)
        specs += _linear(f"{tp}input_down", h, pj, bias=True)
        for b in range(cfg.tower_depth):
            bp = f"{tp}blocks.{b}."
            specs += _norm(f"{bp}norm1", h)
            specs += layer_specs(kind, f"{bp}layer.", cfg)
            specs += _norm(f"{bp}norm2", h)
            specs += _linear(f"{bp}mlp.fc1", pj, h, bias=True)
            specs += _linear(f"{bp}mlp.fc2", h, pj, bias=True)
    specs += _linear("output_proj", 1, h, bias=True)
    return specs


def draw(spec: ParamSpec, seed: int) -> np.ndarray:
    """One tensor of the seeded stream (see the module docstring)."""
    key = zlib.crc32(spec.name.encode("utf-8"))
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([int(seed), key])))
    n = int(np.prod(spec.shape))
    out = np.empty(n, dtype=np.float32)
    rng.random(out=out, dtype=np.float32)
    lo, hi = np.float32(spec.lo), np.float32(spec.hi)
    # lo + (hi - lo) * u, evaluated in float32 in place
    out *= hi - lo
    out += lo
    return out.reshape(spec.shape)


def generate(specs: Iterable[ParamSpec], seed: int = 0, threads: int = 8) -> Dict[str, np.ndarray]:
    """Draw every spec. numpy's generators release the GIL while filling, so the
    tensors are drawn on a thread pool; each tensor's values depend only on
    (seed, name), never on scheduling."""
    specs = list(specs)
    if threads <= 1 or len(specs) < 8:
        return {s.name: draw(s, seed) for s in specs}
    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=threads) as ex:
        arrays = list(ex.map(lambda s: draw(s, seed), specs))
    return {s.name: a for s, a in zip(specs, arrays)}


def generate_model(cfg: ModelConfig, seed: int = 0) -> Dict[str, np.ndarray]:
    """Seeded weights for MultiTowerModel(cfg), keyed like its state_dict()."""
    return generate(param_specs(cfg), seed)


def param_count(cfg: ModelConfig) -> int:
    return sum(int(np.prod(s.shape)) for s in param_specs(cfg))


FP32_LINEAR_NAMES = ("dt_proj", "igate_proj", "fgate_proj", "output_proj")  # example_model.py:106


def weight_bytes(cfg: ModelConfig, linear_dtype: str) -> int:
    """Bytes of the model's weights as the engine stores them: CastLinear-converted
    nn.Linear parameters in the low type, everything else float32."""
    low = {"fp32": 4, "bf16": 2, "fp16": 2}[linear_dtype]
    total = 0
    for s in param_specs(cfg):
        n = int(np.prod(s.shape))
        lin = s.linear and s.name.split(".")[-2] not in FP32_LINEAR_NAMES
        total += n * (low if lin else 4)
    return total


def layer_weight_bytes(kind: str, cfg: ModelConfig, linear_dtype: str) -> int:
    """Bytes of one layer's weights as the engine stores them (see weight_bytes)."""
    low = {"fp32": 4, "bf16": 2, "fp16": 2}[linear_dtype]
    total = 0
    for s in layer_specs(kind, "", cfg):
        n = int(np.prod(s.shape))
        lin = s.linear and s.name.split(".")[-2] not in FP32_LINEAR_NAMES
        total += n * (low if lin else 4)
    return total


# ---------------------------------------------------------------------------
# BASELINE configs 2 and 3: single-layer micro-benchmarks with stated fills.
#
# config 2: Mamba2(256, head_size=64, bc_head_size=64) - d_inner 512, 8 heads,
#           d_state 64 - with a = -exp(U(0, ln 16)) and the dt bias set so that
#           softplus(dt) lies in [1e-3, 0.1] (bias = softplus^-1(U(1e-3, 0.1)),
#           dt_proj weights U(-1e-4, 1e-4), so W.x moves dt by ~1e-3 at most).
# config 3: RetNet(256, num_heads=4) - heads of 64 - with decay
#           gamma_h = 1 - 2^(-5-h) and angle theta_j = 10000^(-2 floor(j/2) / 64);
#           and the mLSTM cell with 4 heads of 64 (a 64 x 64 matrix memory per
#           head), which is the cell of XLSTM(128, mlstm_num_heads=4): its inner
#           width 2 x 128 = 256 splits into 4 heads of 64.
MICRO_CONFIGS = {
    "mamba2": ModelConfig(hidden_size=256, proj_size=512, tower_depth=1, num_heads=8, num_features=79,
                          mamba_head_size=64, mamba_bc_size=64),
    "retnet": ModelConfig(hidden_size=256, proj_size=512, tower_depth=1, num_heads=4, num_features=79),
    "xlstm": ModelConfig(hidden_size=128, proj_size=256, tower_depth=1, num_heads=4, num_features=79),
}


def micro_layer(kind: str, seed: int = 0) -> Tuple[ModelConfig, Dict[str, np.ndarray]]:
    """(config, layer state_dict) of BASELINE config 2 ("mamba2") or 3
    ("retnet", "xlstm"): the seeded layer weights with the fills stated above."""
    cfg = MICRO_CONFIGS[kind]
    sd = generate(layer_specs(kind, "", cfg), seed=seed)
    rng = np.random.default_rng([seed, zlib.crc32(f"micro.{kind}".encode())])
    if kind == "mamba2":
        nh = 2 * cfg.hidden_size // cfg.mamba_head_size
        sd["a"] = (-np.exp(rng.uniform(0.0, math.log(16.0), nh))).astype(np.float32)
        target = rng.uniform(1e-3, 0.1, nh)
        sd["dt_proj.bias"] = np.log(np.expm1(target)).astype(np.float32)  # softplus^-1
        sd["dt_proj.weight"] = rng.uniform(-1e-4, 1e-4, sd["dt_proj.weight"].shape).astype(np.float32)
    elif kind == "retnet":
        nh, hs = cfg.num_heads, cfg.hidden_size // cfg.num_heads
        sd["decay"] = (1.0 - 2.0 ** (-5.0 - np.arange(nh))).astype(np.float32)
        sd["angle"] = (10000.0 ** (-2.0 * (np.arange(hs) // 2) / hs)).astype(np.float32)
    return cfg, sd
