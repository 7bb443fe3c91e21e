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
    otherwise every `load` uploads at once.

    A deferred binder over an input arena overlaps the upload with the work
    already queued: the host-to-device copy goes on a copy stream into one
    of two device staging arenas, and the current stream, once that copy is
    in, moves the staged bytes into the bound buffers with one device copy
    per run. The upload of update k+1 thus runs while update k still reads
    the bound buffers; the bound addresses never change."""

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
        # Overlapped uploads (deferred, arena): copy stream, two device
        # staging arenas and, per arena, the event after which it is free.
        self._overlap = deferred and self._arena is not None
        self._copy_stream = None
        self._dev_stage: list = [None, None]
        self._stage_free: list = [None, None]
        self._dslot = 0

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
        cur = torch.cuda.current_stream(self.device)
        if self._overlap and not torch.cuda.is_current_stream_capturing():
            ev = self._flush_overlapped(cur, buf, mirrored, staged)
        else:
            self._upload(self._mirror_buf if mirrored else None, mirrored)
            self._upload(buf, staged)
            ev = torch.cuda.Event()
            ev.record(cur)
        self.last_upload = ev
        if staged:
            self._events[self._slot] = ev
            self._slot = (self._slot + 1) % self.STAGES
        self._dirty.clear()
        self._from_mirror.clear()

    def _runs(self, names):
        """Byte ranges covering `names` (sorted by offset): an input starting
        where the previous one ends (up to its 256-byte alignment) joins its
        run."""
        runs = []
        start = end = None
        for k in names:
            off, n = self._offset[k], self._nbytes[k]
            if start is not None and off <= (end + 255) // 256 * 256:
                end = max(end, off + n)
                continue
            if start is not None:
                runs.append((start, end))
            start, end = off, off + n
        if start is not None:
            runs.append((start, end))
        return runs

    def _flush_overlapped(self, cur, buf, mirrored, staged):
        """Upload on the copy stream into a device staging arena, then move it
        into the bound buffers on `cur` once the upload is in. -> the event
        after which the host sources may be rewritten."""
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(self.device)
        slot = self._dslot
        stage = self._dev_stage[slot]
        if stage is None:
            stage = self._dev_stage[slot] = torch.empty(self._span, dtype=torch.uint8,
                                                        device=self.device)
        cs = self._copy_stream
        if self._stage_free[slot] is not None:
            cs.wait_event(self._stage_free[slot])
        with torch.cuda.stream(cs):
            for src, names in ((self._mirror_buf if mirrored else None, mirrored),
                               (buf, staged)):
                for a, b in self._runs(names):
                    stage[a:b].copy_(src[a:b], non_blocking=True)
        up = torch.cuda.Event()
        up.record(cs)
        cur.wait_event(up)
        for a, b in self._runs(sorted(mirrored + staged, key=lambda k: self._offset[k])):
            self._arena[a:b].copy_(stage[a:b], non_blocking=True)
        free = torch.cuda.Event()
        free.record(cur)
        self._stage_free[slot] = free
        self._dslot = 1 - slot
        return up

    def _upload(self, buf, names) -> None:
        """Host-to-device copies of `names` (sorted by offset) out of `buf`,
        which holds each at its input offset."""
        if not names:
            return
        if self._arena is not None:
            for a, b in self._runs(names):
                self._arena[a:b].copy_(buf[a:b], non_blocking=True)
        else:
            for k in names:
                dst, off = self._tensors[k], self._offset[k]
                src = buf[off:off + self._nbytes[k]].view(dst.dtype).view(dst.shape)
                dst.copy_(src, non_blocking=True)

    def close(self) -> None:
        for ev in self._events + self._stage_free + [self.last_upload]:
            if ev is not None:
                ev.synchronize()
        self._dev_stage = [None, None]
        self._stage_free = [None, None]
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
