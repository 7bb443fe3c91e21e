"""Engine configuration (ttrl/engine/config.py:10-23), kept for interface
compatibility. `l1_small_size` and `trace_region_size` size Tenstorrent L1
regions and have no B200 meaning; they are accepted and ignored."""

from __future__ import annotations

from dataclasses import dataclass

__all__ = ["EngineConfig", "DEFAULT"]


@dataclass(frozen=True)
class EngineConfig:
    trace_blocking: bool = False
    l1_small_size: int = 0
    trace_region_size: int = 0


DEFAULT = EngineConfig()
