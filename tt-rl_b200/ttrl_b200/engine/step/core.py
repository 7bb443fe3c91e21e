"""`TrainStep` and `MODES` (ttrl/engine/step/core.py).

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

from typing import Callable

from ttrl_b200.device import context
from ttrl_b200.engine.autograd import as_device
from ttrl_b200.engine.config import DEFAULT, EngineConfig
from ttrl_b200.engine.step.inputs import InputBinder
from ttrl_b200.engine.step.metrics import MetricPack, read_metrics
from ttrl_b200.engine.trace import capture

__all__ = ["MODES", "StepFn", "TrainStep"]

StepFn = Callable[[dict], dict]

#: "traced_fwd_bwd" keeps the reference's name; on this backend it captures
#: the optimizer too. "graph" is an alias that says so.
MODES = ("eager", "traced_fwd_bwd", "graph")


class TrainStep:
    """One training step behind one call API, eager or graph-replayed."""

    def __init__(self, step_fn: StepFn, inputs: dict, device, *, optimizer=None,
                 mode: str = "eager", cfg: EngineConfig = DEFAULT,
                 critical_main: bool = False):
        """`critical_main`: capture at the highest stream priority (see
        `engine.trace.capture`); for steps whose side lanes carry only work
        off the critical path, or whose critical side work runs on the
        equally prioritised forward lanes."""
        if mode not in MODES:
            raise ValueError(f"TrainStep mode must be one of {list(MODES)}, got {mode!r}")
        self.step_fn = step_fn
        self.inputs = inputs
        self.device = as_device(device)
        self.optimizer = optimizer
        self.mode = mode
        self.cfg = cfg
        self._binder = InputBinder(self.device, inputs, deferred=True)
        self._trace = None
        self._pack: MetricPack | None = None
        self._captured_grads: list = []
        self.launches_per_replay = 0
        self.critical_main = bool(critical_main)

    def load_input(self, name: str, array) -> None:
        self._binder.load(name, array)

    def pinned_inputs(self) -> dict:
        """Pinned host tensors shaped like the inputs; `load_input(name,
        pinned_inputs()[name])` uploads straight from them (see
        InputBinder.pinned_inputs for the ownership rule)."""
        return self._binder.pinned_inputs()

    def run(self) -> dict:
        self._binder.flush()
        if self.mode == "eager":
            return self._run_eager()
        return self._run_traced()

    def launch(self) -> None:
        """Replay the captured update without reading metrics back (for
        back-to-back replays; call `run()` or `metrics()` to read)."""
        self._binder.flush()
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
        self._trace, self._pack = capture(self.device, self._record,
                                          critical_main=self.critical_main)
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
