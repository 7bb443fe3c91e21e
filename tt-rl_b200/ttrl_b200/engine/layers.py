"""`Linear`, `LayerNorm`, `ReLU`, `Tanh`, `Sequential`, `Flatten`
(ttrl/engine/layers.py), plus `Conv2d` in ttrl_b200.engine.conv.

Parameters are drawn from numpy's global generator in the same order and
with the same bounds as the reference, so a seeded construction yields the
same initial weights on both sides.

`Sequential` fuses a `Linear` or `Conv2d` immediately followed by a `ReLU`
into one node (one GEMM launch with the bias and ReLU in its epilogue); the
module tree, parameter names and results are unchanged.
"""

from __future__ import annotations

import math

import numpy as np

from ttrl_b200.engine.autograd import Tensor, as_device
from ttrl_b200.engine.nn import Module, ModuleList
from ttrl_b200.engine.ops import (add, div, linear, mean_dim, mul, relu, reshape, sqrt, square,
                                  sub, tanh)

__all__ = ["Linear", "LayerNorm", "ReLU", "Tanh", "Sequential", "Flatten"]


class Linear(Module):
    """y = x @ W + b, W stored (in_features, out_features) (layers.py:22-61).

    Init matches PyTorch's nn.Linear default, U(+-1/sqrt(in_features)).
    """

    def __init__(self, in_features: int, out_features: int, device=None, *, bias: bool = True):
        if in_features <= 0 or out_features <= 0:
            raise ValueError(f"Linear({in_features}, {out_features}): both widths have to be "
                             "positive")
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        bound = 1.0 / math.sqrt(in_features)
        dev = as_device(device)
        weight = np.random.uniform(-bound, bound,
                                   (self.in_features, self.out_features)).astype(np.float32)
        self.weight = Tensor.from_numpy(weight, dev, requires_grad=True)
        self.bias = None
        if bias:
            b = np.random.uniform(-bound, bound, (1, self.out_features)).astype(np.float32)
            self.bias = Tensor.from_numpy(b, dev, requires_grad=True)

    def forward(self, x: Tensor) -> Tensor:
        return linear(x, self.weight, self.bias, relu=False)

    def forward_relu(self, x: Tensor) -> Tensor:
        """This layer followed by a ReLU, as one fused GEMM."""
        return linear(x, self.weight, self.bias, relu=True)


class LayerNorm(Module):
    """Composed exactly as ttrl/engine/layers.py:64-115 does."""

    def __init__(self, normalized_shape: int, device=None, *, eps: float = 1e-5):
        if normalized_shape <= 0:
            raise ValueError(f"LayerNorm({normalized_shape}): the normalised width has to be "
                             "positive")
        if eps <= 0.0:
            raise ValueError(f"LayerNorm(eps={eps}): eps has to be positive, since a row of "
                             "equal values has zero variance")
        self.normalized_shape = int(normalized_shape)
        self.eps = float(eps)
        dev = as_device(device)
        self.weight = Tensor.from_numpy(np.ones((1, self.normalized_shape), np.float32), dev,
                                        requires_grad=True)
        self.bias = Tensor.from_numpy(np.zeros((1, self.normalized_shape), np.float32), dev,
                                      requires_grad=True)

    def forward(self, x: Tensor) -> Tensor:
        if int(x.shape[-1]) != self.normalized_shape:
            raise ValueError(f"LayerNorm({self.normalized_shape}) was given an input of shape "
                             f"{tuple(x.shape)}, whose last axis is not {self.normalized_shape} "
                             "wide")
        centred = sub(x, mean_dim(x, dim=-1))
        variance = mean_dim(square(centred), dim=-1)
        return add(mul(div(centred, sqrt(add(variance, self.eps))), self.weight), self.bias)


class ReLU(Module):
    def forward(self, x: Tensor) -> Tensor:
        return relu(x)


class Tanh(Module):
    def forward(self, x: Tensor) -> Tensor:
        return tanh(x)


class Sequential(Module):
    """Chain layers; children named `layers.<i>.<name>`."""

    def __init__(self, *layers):
        self.layers = ModuleList(layers)

    def forward(self, x: Tensor) -> Tensor:
        items = list(self.layers)
        i = 0
        while i < len(items):
            layer = items[i]
            nxt = items[i + 1] if i + 1 < len(items) else None
            if isinstance(nxt, ReLU) and hasattr(layer, "forward_relu") and \
                    type(nxt).forward is ReLU.forward:
                x = layer.forward_relu(x)
                i += 2
                continue
            x = layer(x)
            i += 1
        return x

    def append(self, layer) -> "Sequential":
        self.layers.append(layer)
        return self

    def __len__(self) -> int:
        return len(self.layers)

    def __getitem__(self, index):
        return self.layers[index]


class Flatten(Module):
    """`[1, 1, N*H*W, C]` -> `(N, H*W*C)`, in (h, w, c) order (layers.py:158-200)."""

    def __init__(self, h: int, w: int, channels: int):
        if h <= 0 or w <= 0 or channels <= 0:
            raise ValueError(f"Flatten({h}, {w}, {channels}): every extent has to be positive")
        self.h = int(h)
        self.w = int(w)
        self.channels = int(channels)

    @property
    def out_features(self) -> int:
        return self.h * self.w * self.channels

    def forward(self, x: Tensor) -> Tensor:
        shape = tuple(int(d) for d in x.shape)
        rows = self.h * self.w
        if (len(shape) != 4 or shape[0] != 1 or shape[1] != 1 or shape[3] != self.channels
                or shape[2] % rows != 0):
            raise ValueError(f"Flatten({self.h}, {self.w}, {self.channels}) reads NHWC rows "
                             f"[1, 1, images * {rows}, {self.channels}]; this input is {shape}")
        return reshape(x, (shape[2] // rows, self.out_features))
