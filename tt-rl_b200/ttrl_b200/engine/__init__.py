"""ttrl_b200.engine: the B200 learner engine with ttrl.engine's interface
(ttrl/engine/__init__.py:15-83).

Lazy: importing this package loads no library and touches no GPU.
"""

from __future__ import annotations

import importlib
from typing import Any

from ttrl_b200.engine.config import DEFAULT, EngineConfig

_LAZY = {
    "DeviceProfile": "device_mgmt",
    "NoDeviceAvailable": "device_mgmt",
    "acquire": "device_mgmt",
    "MASTER_DTYPE": "tensor",
    "StaticArena": "tensor",
    "copy_in_place": "tensor",
    "copy_tensor_in_place": "tensor",
    "to_device": "tensor",
    "to_host": "tensor",
    "restore_in_place": "tensor",
    "Tensor": "autograd",
    "backward": "autograd",
    "no_grad": "autograd",
    "Adam": "optim",
    "Optimizer": "optim",
    "adam_fused_scalars": "optim",
    "TrainStep": "step",
    "read_metrics": "step",
    "InputBinder": "step",
    "ActingCarry": "carry",
    "CapturedTrace": "trace",
    "TraceCaptureError": "trace",
    "capture": "trace",
    "ParamSync": "mesh",
    "ParamSyncError": "mesh",
    "host_all_reduce_sum": "mesh",
    "Module": "nn",
    "ModuleList": "nn",
    "ModuleDict": "nn",
    "Linear": "layers",
    "LayerNorm": "layers",
    "ReLU": "layers",
    "Tanh": "layers",
    "Sequential": "layers",
    "Flatten": "layers",
    "Conv2d": "conv",
    "ConvGeometry": "conv",
    "ConvDoesNotFit": "conv",
    "GRU": "recurrent",
    "GRUCell": "recurrent",
}

_OPS = "ttrl_b200.engine.ops"

__all__ = [
    "DEFAULT",
    "EngineConfig",
    *sorted(_LAZY),
    "add", "div", "mul", "sub",
    "abs_", "exp", "log", "neg", "relu", "sigmoid", "sqrt", "square", "tanh",
    "clamp", "maximum", "minimum",
    "matmul",
    "argmax_dim_detached", "max_dim_detached", "mean_all", "mean_dim",
    "sum_all", "sum_dim",
    "concat", "reshape", "split",
    "apply_done_mask", "entropy", "gather_onehot", "huber", "log_softmax",
    "masks", "non_finite_check", "one_hot_device", "one_hot_gather",
    "one_hot_host",
]


def __getattr__(name: str) -> Any:
    module = _LAZY.get(name)
    if module is not None:
        return getattr(importlib.import_module(f"ttrl_b200.engine.{module}"), name)
    if name in __all__:
        return getattr(importlib.import_module(_OPS), name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


def __dir__() -> list[str]:
    return sorted(__all__)
