"""Device acquisition (ttrl/engine/device/acquire.py:56-140), B200 edition.

The reference locks a Tenstorrent chip (flock + fuser) and probes its arch;
here a device is a CUDA ordinal. `acquire(chip_id)` returns the torch
device and a small profile; one process drives one GPU (its rank's).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

__all__ = ["DeviceProfile", "NoDeviceAvailable", "acquire"]


class NoDeviceAvailable(RuntimeError):
    pass


@dataclass(frozen=True)
class DeviceProfile:
    arch: str
    name: str
    sm_count: int
    memory_bytes: int

    @property
    def torch_device(self):  # pragma: no cover - convenience
        return None


def acquire(chip_id: int = 0, cfg=None, wait: bool = False, timeout: float | None = None):
    """-> (torch.device, DeviceProfile) for CUDA ordinal `chip_id`."""
    if not torch.cuda.is_available():
        raise NoDeviceAvailable("no CUDA device is visible to this process")
    if not 0 <= int(chip_id) < torch.cuda.device_count():
        raise NoDeviceAvailable(
            f"CUDA device {chip_id} does not exist (have {torch.cuda.device_count()})")
    dev = torch.device("cuda", int(chip_id))
    props = torch.cuda.get_device_properties(dev)
    cap = f"sm_{props.major}{props.minor}"
    return dev, DeviceProfile(arch=cap, name=props.name, sm_count=props.multi_processor_count,
                              memory_bytes=props.total_memory)
