"""Conv tower stages (ttrl/nets/towers.py)."""

from __future__ import annotations

from dataclasses import dataclass

__all__ = ["ConvStage", "NATURE_CNN"]


@dataclass(frozen=True)
class ConvStage:
    out_channels: int
    kernel: int
    stride: int
    padding: int = 0
    fold: int = 1


#: Mnih et al. 2015: 84x84 -> 20x20 -> 9x9 -> 7x7.
NATURE_CNN = (ConvStage(32, 8, 4), ConvStage(64, 4, 2), ConvStage(64, 3, 1))
