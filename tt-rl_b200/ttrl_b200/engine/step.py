"""`TrainStep`, `InputBinder`, `read_metrics`
(ttrl/engine/step/{core,inputs,metrics}.py).

`TrainStep(step_fn, inputs, device, optimizer=..., mode=...)` runs one
training step eagerly or from a CUDA graph. In the traced modes the graph
holds the WHOLE update: forward, backward, the optimizer step (whose bias
correction comes from device step counters) and the packing of the scalar
metrics into one buffer. A replay is one graph launch; reading the metrics
is one device-to-host copy.

The reference captures forward+backward only and runs Adam eagerly after
the replay (ttrl/engine/step/core.py:35-41) because its bias-correction
scalars are host values; here they are not, so Adam joins the graph. The
arithmetic and the order of operations are unchanged.
"""

from __future__ import annotations

import contextlib

from typing import Callable

import numpy as np
import torch

from ttrl_b200.device import context
from ttrl_b200.engine.autograd import Tensor, as_device
from ttrl_b200.engine.config import DEFAULT, EngineConfig
from ttrl_b200.engine.trace import capture

__all__ = ["MODES", "StepFn", "TrainStep", "InputBinder", "read_metrics"]

StepFn = Callable[[dict], dict]

#: "traced_fwd_bwd" keeps the reference's name; on this backend it captures
#: the optimizer too. "graph" is an alias that says so.
MODES = ("eager", "traced_fwd_bwd", "graph")


class InputBinder:
    """Copies host arrays into the bound input tensors' existing buffers
    through reusable pinned staging buffers (address stability: the device
    buffer a graph reads is never rebound)."""

    def __init__(self, device, inputs: dict):
        self.device = as_device(device)
        self.inputs = inputs
        self._staging: dict[str, torch.Tensor] = {}
        self._events: dict[str, torch.cuda.Event] = {}

    def load(self, name: str, array) -> None:
        t = self.inputs[name]
        dst = t.data if isinstance(t, Tensor) else t
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
        stage = self._staging.get(name)
        if stage is None or stage.numel() != dst.numel() or stage.dtype != dst.dtype:
            stage = torch.empty(dst.shape, dtype=dst.dtype, pin_memory=True)
            self._staging[name] = stage
        ev = self._events.get(name)
        if ev is not None:
            ev.synchronize()  # the previous upload from this staging buffer finished
        stage.numpy().reshape(-1)[:] = arr.reshape(-1)
        dst.copy_(stage.reshape(dst.shape), non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._events[name] = ev

    def close(self) -> None:
        self._staging.clear()
        self._events.clear()


def _numel(t) -> int:
    n = 1
    for d in t.shape:
        n *= int(d)
    return n


class MetricPack:
    """Packs the scalar metrics of one step into one device buffer with copy
    kernels, so reading them back is a single device-to-host transfer."""

    def __init__(self, metrics: dict):
        self.scalar_keys = []
        self.vector_keys = []
        self.passthrough = {}
        self.sources = {}
        for k, v in metrics.items():
            if isinstance(v, Tensor):
                if _numel(v) == 1:
                    self.scalar_keys.append(k)
                else:
                    self.vector_keys.append(k)
                self.sources[k] = v
            else:
                self.passthrough[k] = v
        self.buffer = None
        if self.scalar_keys:
            dev = self.sources[self.scalar_keys[0]].data.device
            ctx = context(dev)
            # On side lane 2 (when lanes are on), beside the optimizer step
            # that follows on the current stream; the caller joins.
            lane = ctx.side(2) if ctx.concurrent else contextlib.nullcontext()
            with lane:
                self.buffer = torch.empty(len(self.scalar_keys), dtype=torch.float32,
                                          device=dev)
                for i, k in enumerate(self.scalar_keys):
                    src = self.sources[k].data.reshape(1)
                    if src.dtype != torch.float32:
                        src = src.float()
                    ctx.copy_strided(self.buffer[i:i + 1], src)

    def read(self) -> dict:
        out = dict(self.passthrough)
        if self.buffer is not None:
            context(self.buffer.device).join()
            host = self.buffer.detach().to("cpu").numpy()
            for i, k in enumerate(self.scalar_keys):
                out[k] = host[i:i + 1].reshape(self.sources[k].shape)
        for k in self.vector_keys:
            out[k] = self.sources[k].numpy()
        return out

    def fetch(self):
        """Start copying every metric to pinned host memory on the current
        stream; `result(handle)` waits for those copies only."""
        copies = {}
        dev = None
        if self.buffer is not None:
            dev = self.buffer.device
            context(dev).join()
            copies[None] = torch.empty(self.buffer.shape, dtype=self.buffer.dtype,
                                       pin_memory=True)
            copies[None].copy_(self.buffer, non_blocking=True)
        for k in self.vector_keys:
            src = self.sources[k].data
            dev = src.device
            copies[k] = torch.empty(src.shape, dtype=src.dtype, pin_memory=True)
            copies[k].copy_(src, non_blocking=True)
        done = None
        if dev is not None:
            done = torch.cuda.Event()
            done.record(torch.cuda.current_stream(dev))
        return copies, done

    def result(self, handle) -> dict:
        copies, done = handle
        if done is not None:
            done.synchronize()
        out = dict(self.passthrough)
        if None in copies:
            host = copies[None].numpy()
            for i, k in enumerate(self.scalar_keys):
                out[k] = host[i:i + 1].reshape(self.sources[k].shape)
        for k in self.vector_keys:
            out[k] = copies[k].numpy().reshape(self.sources[k].shape)
        return out


def read_metrics(metrics: dict | None) -> dict:
    """Download every tensor-valued metric; scalars in one transfer."""
    if not metrics:
        return {}
    return MetricPack(metrics).read()


class TrainStep:
    """One training step behind one call API, eager or graph-replayed."""

    def __init__(self, step_fn: StepFn, inputs: dict, device, *, optimizer=None,
                 mode: str = "eager", cfg: EngineConfig = DEFAULT):
        if mode not in MODES:
            raise ValueError(f"TrainStep mode must be one of {list(MODES)}, got {mode!r}")
        self.step_fn = step_fn
        self.inputs = inputs
        self.device = as_device(device)
        self.optimizer = optimizer
        self.mode = mode
        self.cfg = cfg
        self._binder = InputBinder(self.device, inputs)
        self._trace = None
        self._pack: MetricPack | None = None
        self._captured_grads: list = []
        self.launches_per_replay = 0

    def load_input(self, name: str, array) -> None:
        self._binder.load(name, array)

    def run(self) -> dict:
        if self.mode == "eager":
            return self._run_eager()
        return self._run_traced()

    def launch(self) -> None:
        """Replay the captured update without reading metrics back (for
        back-to-back replays; call `run()` or `metrics()` to read)."""
        if self._trace is None:
            self._capture()
            return
        self._trace.replay(cfg=self.cfg)
        self._after_replay()

    def metrics(self) -> dict:
        return self._pack.read() if self._pack is not None else {}

    def fetch_metrics(self):
        """Start the metric read of the last replay without waiting (a handle
        for `metrics_of`), so the next step can be enqueued first."""
        return self._pack.fetch() if self._pack is not None else ({}, None)

    def metrics_of(self, handle) -> dict:
        return self._pack.result(handle) if self._pack is not None else {}

    def _run_eager(self) -> dict:
        if self.optimizer is not None:
            self.optimizer.zero_grad()
        metrics = self.step_fn(self.inputs)
        if self.optimizer is not None:
            self.optimizer.step()
        return read_metrics(metrics)

    def _run_traced(self) -> dict:
        self.launch()
        return self.metrics()

    def _record(self):
        if self.optimizer is not None:
            self.optimizer.zero_grad()
        metrics = self.step_fn(self.inputs)
        # Packed before the optimizer step so that, on a side lane, the
        # metric copies run beside it.
        pack = MetricPack(metrics)
        if self.optimizer is not None:
            self.optimizer.step()
        context(self.device).join()
        return pack

    def _capture(self) -> None:
        # Warm-up pass: real launches (kernel loading, workspace sizing,
        # persistent gradient buffers); its gradients are discarded.
        if self.optimizer is not None:
            self.optimizer.zero_grad()
        self.step_fn(self.inputs)
        if self.optimizer is not None:
            self.optimizer.zero_grad()
        from ttrl_b200._lib import lib
        before = lib().ttrl_launch_count()
        self._trace, self._pack = capture(self.device, self._record)
        self.launches_per_replay = int(lib().ttrl_launch_count() - before)
        if self.optimizer is not None:
            self._captured_grads = [(p, p.grad) for p in self.optimizer.params]
        # Capture only records: run it once so this first call is a real step.
        self._trace.replay(blocking=False)
        self._after_replay()

    def _after_replay(self) -> None:
        for param, grad in self._captured_grads:
            param.grad = grad
        opt = self.optimizer
        if opt is not None and getattr(opt, "captured_indices", None) is not None:
            opt.advance(opt.captured_indices)

    def close(self) -> None:
        trace, self._trace = self._trace, None
        self._pack = None
        self._captured_grads = []
        try:
            if trace is not None:
                trace.close()
        finally:
            self._binder.close()

    def __enter__(self) -> "TrainStep":
        return self

    def __exit__(self, *exc) -> None:
        self.close()
