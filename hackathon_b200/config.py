"""Model dimensions and the named size presets.

`ModelConfig` mirrors the reference's frozen dataclass
(model/inference_model.py:21-27) field for field, so a config built for the
reference can be handed to this package unchanged. The derived sizes below are
the ones the reference's layer constructors compute:

* xLSTM (model/inference_model.py:45-50): mLSTM heads = num_heads, sLSTM heads =
  num_heads // 2; the mLSTM block works at 2*hidden (model/xlstm.py:181,193)
  with q/k/v BlockLinears of 4x4 blocks (model/xlstm.py:189-193); the sLSTM
  BlockLinears have one block per sLSTM head (model/xlstm.py:290-299).
* Mamba2 (model/mamba2.py:10-46): inner = 2*hidden, head_size 64, B/C width
  ("bc") 128, conv kernel 4, num_heads = inner // 64.
* RetNet (model/retnet.py:20-36): head_size = hidden // num_heads.
* Hawk (model/hawk.py:56-66, 8-18): RG-LRU BlockLinears of 4 blocks.
"""

from __future__ import annotations

from dataclasses import dataclass

# Tower order of MultiTowerModel (model/inference_model.py:107-112); the
# prediction columns come out in this order (model/inference_model.py:142-143).
TOWER_KINDS = ("xlstm", "mamba2", "retnet", "hawk")

CONV_K = 4  # CausalConv1d kernel size everywhere in the model


@dataclass(frozen=True, kw_only=True)
class ModelConfig:
    hidden_size: int
    proj_size: int
    tower_depth: int
    num_heads: int
    num_features: int
    # Mamba2 sizes are constructor defaults in the reference, not ModelConfig
    # fields; they are carried here so the single-layer micro-benchmarks can use
    # Mamba2(256, head_size=64, bc_head_size=64) through the same engine.
    mamba_head_size: int = 64
    mamba_bc_size: int = 128

    # ---- derived sizes -------------------------------------------------
    @property
    def mlstm_inner(self) -> int:
        return 2 * self.hidden_size

    @property
    def mlstm_heads(self) -> int:
        return self.num_heads

    @property
    def mlstm_head_size(self) -> int:
        return self.mlstm_inner // self.mlstm_heads

    @property
    def slstm_heads(self) -> int:
        return self.num_heads // 2

    @property
    def slstm_block(self) -> int:
        return self.hidden_size // self.slstm_heads

    @property
    def mamba_inner(self) -> int:
        return 2 * self.hidden_size

    @property
    def mamba_heads(self) -> int:
        return self.mamba_inner // self.mamba_head_size

    @property
    def retnet_head_size(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def hawk_block(self) -> int:
        return self.hidden_size // 4

    def validate(self) -> None:
        h = self.hidden_size
        assert h > 0 and self.proj_size > 0 and self.tower_depth > 0
        assert self.num_heads >= 2 and self.num_heads % 2 == 0, "sLSTM uses num_heads // 2 heads"
        assert h % self.slstm_heads == 0
        assert self.mlstm_inner % self.mlstm_heads == 0
        assert self.mlstm_inner % 4 == 0, "mLSTM q/k/v BlockLinear uses 4x4 blocks"
        assert self.mamba_inner % self.mamba_head_size == 0
        assert h % self.num_heads == 0 and self.retnet_head_size % 2 == 0, "rotary pairs"
        assert h % 4 == 0, "RG-LRU BlockLinear uses 4 blocks"


# Reference default dims (example_model.py:283-289).
D0 = ModelConfig(hidden_size=2048, proj_size=4096, tower_depth=12, num_heads=8, num_features=79)
# Reduced dims for the 4096-symbol batch and single-request latency targets.
D1 = ModelConfig(hidden_size=256, proj_size=512, tower_depth=12, num_heads=8, num_features=79)
# Scale-out dims: 65,536 symbols of state fit one B200 at depth 4.
D2 = ModelConfig(hidden_size=256, proj_size=512, tower_depth=4, num_heads=8, num_features=79)
# The small model of the reference's own equivalence checker
# (check_cell_rewrite.py:265-269).
SMALL = ModelConfig(hidden_size=64, proj_size=128, tower_depth=2, num_heads=4, num_features=7)

PRESETS = {"D0": D0, "D1": D1, "D2": D2, "SMALL": SMALL}
