"""`InputBinder` and `input_arena` (ttrl/engine/step/inputs.py): host arrays
into the fixed device buffers a captured update reads, in place."""

from __future__ import annotations

import numpy as np
import torch

from ttrl_b200.engine.autograd import Tensor, as_device

__all__ = ["InputBinder", "input_arena"]


class InputBinder:
    """Copies host arrays into the bound input tensors' existing buffers
    (address stability: the device buffer a graph reads is never rebound),
    through a ring of `STAGES` reusable pinned host buffers.

    Writing stage k waits only for the upload out of stage k - STAGES, so a
    host that enqueues update k+1 while update k runs never blocks on the
    previous update's copies. When the inputs are views of one device buffer
    (`input_arena`), the inputs loaded since the last `flush()` go up in as
    few host-to-device copies as there are contiguous runs of them (one, when
    every input is loaded). With `deferred`, `load` only stages and
    `flush()` (TrainStep calls it before every replay) issues the copies;
    otherwise every `load` uploads at once."""

    STAGES = 3

    def __init__(self, device, inputs: dict, *, deferred: bool = False):
        self.device = as_device(device)
        self.inputs = inputs
        self.deferred = deferred
        self._slots: list = [None] * self.STAGES
        self._events: list = [None] * self.STAGES
        self._slot = 0
        self._dirty: set = set()
        tensors = {k: (t.data if isinstance(t, Tensor) else t) for k, t in inputs.items()}
        self._tensors = tensors
        storages = {t.untyped_storage().data_ptr() for t in tensors.values()}
        self._arena = None
        if len(tensors) > 1 and len(storages) == 1 and all(t.is_contiguous()
                                                           for t in tensors.values()):
            first = next(iter(tensors.values()))
            storage = first.untyped_storage()
            self._arena = torch.empty(0, dtype=torch.uint8, device=first.device).set_(
                storage, 0, (storage.nbytes(),), (1,))
            self._offset = {k: t.storage_offset() * t.element_size() for k, t in tensors.items()}
            self._span = storage.nbytes()
        else:
            self._offset, self._span = {}, 0
            for k, t in tensors.items():
                self._offset[k] = self._span
                self._span += (t.numel() * t.element_size() + 255) // 256 * 256
        self._nbytes = {k: t.numel() * t.element_size() for k, t in tensors.items()}
        self._mirror = None
        self._from_mirror: set = set()
        self.last_upload = None

    def _stage(self):
        """The pinned buffer of the current ring slot, free for writing."""
        buf = self._slots[self._slot]
        if buf is None:
            buf = self._slots[self._slot] = torch.empty(max(self._span, 1), dtype=torch.uint8,
                                                        pin_memory=True)
        ev = self._events[self._slot]
        if ev is not None and not (self._dirty - self._from_mirror):
            ev.synchronize()  # the upload out of this slot, STAGES flushes ago, is done
            self._events[self._slot] = None
        return buf

    def pinned_inputs(self) -> dict:
        """Pinned host tensors laid out like the device inputs (one
        allocation). Loading these uploads straight from them -- no host copy
        -- and, in an input arena, all of them in one transfer. The caller
        owns their contents and must not change them before the upload of
        the step that loaded them has run (`last_upload` records it)."""
        if getattr(self, "_mirror", None) is None:
            buf = torch.empty(max(self._span, 1), dtype=torch.uint8, pin_memory=True)
            self._mirror_buf = buf
            self._mirror = {k: buf[self._offset[k]:self._offset[k] + self._nbytes[k]]
                            .view(t.dtype).view(t.shape) for k, t in self._tensors.items()}
        return self._mirror

    def load(self, name: str, array) -> None:
        dst = self._tensors[name]
        mirror = getattr(self, "_mirror", None)
        if mirror is not None and isinstance(array, torch.Tensor) and \
                array.data_ptr() == mirror[name].data_ptr():
            self._from_mirror.add(name)
            self._dirty.add(name)
            if not self.deferred:
                self.flush()
            return
        self._from_mirror.discard(name)
        arr = np.asarray(array)
        if dst.dtype == torch.uint8:
            arr = np.ascontiguousarray(arr, dtype=np.uint8)
        elif dst.dtype == torch.int32:
            arr = np.ascontiguousarray(arr, dtype=np.int32)
        else:
            arr = np.ascontiguousarray(arr, dtype=np.float32)
        if arr.size != dst.numel():
            raise ValueError(
                f"load_input({name!r}): {arr.size} values for a buffer of {dst.numel()} "
                f"(shape {tuple(dst.shape)})"
            )
        buf = self._stage()
        off = self._offset[name]
        buf.numpy()[off:off + self._nbytes[name]] = arr.reshape(-1).view(np.uint8)
        self._dirty.add(name)
        if not self.deferred:
            self.flush()

    def flush(self) -> None:
        """Upload everything loaded since the last flush, on the current
        stream, and move to the next ring slot."""
        if not self._dirty:
            return
        buf = self._slots[self._slot]
        names = sorted(self._dirty, key=lambda k: self._offset[k])
        mirrored = [k for k in names if k in self._from_mirror]
        staged = [k for k in names if k not in self._from_mirror]
        self._upload(self._mirror_buf if mirrored else None, mirrored)
        self._upload(buf, staged)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.last_upload = ev
        if staged:
            self._events[self._slot] = ev
            self._slot = (self._slot + 1) % self.STAGES
        self._dirty.clear()
        self._from_mirror.clear()

    def _upload(self, buf, names) -> None:
        """Host-to-device copies of `names` (sorted by offset) out of `buf`,
        which holds each at its input offset."""
        if not names:
            return
        if self._arena is not None:
            # Contiguous runs: an input starting where the previous one ends
            # (up to its 256-byte alignment) joins its run.
            start = end = None
            for k in names:
                off, n = self._offset[k], self._nbytes[k]
                if start is not None and off <= (end + 255) // 256 * 256:
                    end = max(end, off + n)
                    continue
                if start is not None:
                    self._arena[start:end].copy_(buf[start:end], non_blocking=True)
                start, end = off, off + n
            self._arena[start:end].copy_(buf[start:end], non_blocking=True)
        else:
            for k in names:
                dst, off = self._tensors[k], self._offset[k]
                src = buf[off:off + self._nbytes[k]].view(dst.dtype).view(dst.shape)
                dst.copy_(src, non_blocking=True)

    def close(self) -> None:
        for ev in self._events + [self.last_upload]:
            if ev is not None:
                ev.synchronize()
        self._mirror = None
        self._mirror_buf = None
        self._slots = [None] * self.STAGES
        self._events = [None] * self.STAGES
        self._dirty.clear()


def input_arena(device, specs: dict) -> dict:
    """Device input buffers as views of ONE allocation, 256-byte aligned:
    `specs` maps name -> (shape, dtype); returns name -> Tensor. An
    InputBinder over them uploads a whole batch in one copy."""
    dev = as_device(device)
    layout, total = {}, 0
    for name, (shape, dtype) in specs.items():
        n = int(np.prod(shape, dtype=np.int64)) * torch.empty(0, dtype=dtype).element_size()
        layout[name] = (total, n, shape, dtype)
        total += (n + 255) // 256 * 256
    raw = torch.zeros(max(total, 256), dtype=torch.uint8, device=dev)
    return {name: Tensor(raw[off:off + n].view(dtype).view(shape))
            for name, (off, n, shape, dtype) in layout.items()}
