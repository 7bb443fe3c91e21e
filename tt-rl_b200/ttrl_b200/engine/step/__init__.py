"""`ttrl_b200.engine.step`: the training step (ttrl/engine/step/): `TrainStep`
(core), `InputBinder` (inputs) and `read_metrics` (metrics)."""

from ttrl_b200.engine.step.core import MODES, StepFn, TrainStep
from ttrl_b200.engine.step.inputs import InputBinder, input_arena
from ttrl_b200.engine.step.metrics import MetricPack, read_metrics

__all__ = ["MODES", "StepFn", "TrainStep", "InputBinder", "input_arena", "MetricPack",
           "read_metrics"]
