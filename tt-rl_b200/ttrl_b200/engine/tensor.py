"""Fixed-address buffers and in-place copies (ttrl/engine/tensor/{arena,
transfer,precision}.py): the address-stability idiom a captured CUDA graph
needs. Nothing that a graph touches is ever rebound; only contents change.
"""

from __future__ import annotations

import numpy as np
import torch

from ttrl_b200.device import context

__all__ = ["MASTER_DTYPE", "StaticArena", "copy_in_place", "copy_tensor_in_place",
           "restore_in_place", "to_device", "to_host"]

#: Every parameter and all optimizer state is fp32 (ttrl/engine/tensor/precision.py).
MASTER_DTYPE = torch.float32


def _raw(obj):
    return obj if isinstance(obj, torch.Tensor) else obj.data


def copy_in_place(dst, src):
    """Write src's contents into dst's existing buffer (one copy kernel)."""
    dst_t, src_t = _raw(dst), _raw(src)
    if not dst_t.is_cuda:
        raise ValueError("copy_in_place destination must be a device tensor")
    if dst_t.numel() != src_t.numel():
        raise ValueError(f"copy_in_place: {src_t.numel()} elements into {dst_t.numel()}")
    context(dst_t.device).copy_strided(dst_t, src_t.reshape(dst_t.shape))
    return dst


def copy_tensor_in_place(dst, src):
    copy_in_place(dst.data, _raw(src))
    return dst


def to_device(array, device=None, dtype=MASTER_DTYPE, *, layout=None) -> torch.Tensor:
    from ttrl_b200.engine.autograd import as_device
    arr = np.ascontiguousarray(np.asarray(array))
    if dtype == MASTER_DTYPE:
        arr = arr.astype(np.float32, copy=False)
    return torch.from_numpy(arr).to(as_device(device))


def restore_in_place(dst, array):
    """Write a host array into dst's existing device buffer (H2D, same address)."""
    dst_t = _raw(dst)
    arr = np.ascontiguousarray(np.asarray(array, dtype=np.float32))
    if arr.size != dst_t.numel():
        raise ValueError(f"restore_in_place: {arr.size} values into {dst_t.numel()}")
    dst_t.copy_(torch.from_numpy(arr).reshape(dst_t.shape), non_blocking=False)
    return dst


def to_host(tensor) -> np.ndarray:
    t = _raw(tensor)
    out = t.detach().to("cpu").numpy()
    return out.astype(np.float32) if out.dtype.kind == "f" else out


class StaticArena:
    """Named fixed-address device buffers, allocated once."""

    def __init__(self, device):
        self.device = device
        self._buffers: dict[str, torch.Tensor] = {}

    def allocate(self, name: str, like) -> torch.Tensor:
        if name in self._buffers:
            raise ValueError(
                f"arena buffer {name!r} is already allocated; allocate() is "
                "one-shot. Use copy_into() to update its contents in place."
            )
        raw = _raw(like)
        buf = torch.zeros_like(raw)
        self._buffers[name] = buf
        return buf

    def __getitem__(self, name: str) -> torch.Tensor:
        return self._buffers[name]

    def __contains__(self, name: str) -> bool:
        return name in self._buffers

    def names(self):
        return self._buffers.keys()

    def copy_into(self, name: str, src):
        return copy_in_place(self._buffers[name], _raw(src))

    def restore_into_from_numpy(self, name: str, array):
        return restore_in_place(self._buffers[name], array)
