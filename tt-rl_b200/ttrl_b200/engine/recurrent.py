"""`GRUCell` and `GRU` (ttrl/engine/recurrent.py), composed from the tape ops
in the reference's order: gates (reset, update, candidate) in PyTorch's
column order, weights stored (features, 3*hidden), the done mask applied to
the state entering each step, and a fixed-length unroll whose backward
accumulates each weight's gradient T times.
"""

from __future__ import annotations

import math

import numpy as np

from ttrl_b200.engine.autograd import Tensor, as_device
from ttrl_b200.engine.nn import Module
from ttrl_b200.engine.ops import (add, apply_done_mask, concat, linear, mul, reshape,
                                  sigmoid, split, sub, tanh)

__all__ = ["GRU", "GRUCell", "GATES"]

GATES = ("reset", "update", "candidate")


class GRUCell(Module):
    """r = sigmoid(xW_ir + b_ir + hW_hr + b_hr); z likewise;
    n = tanh(xW_in + b_in + r * (hW_hn + b_hn)); h' = (1 - z) * n + z * h."""

    def __init__(self, in_features: int, hidden_size: int, device=None):
        if in_features <= 0 or hidden_size <= 0:
            raise ValueError(
                "GRUCell: in_features and hidden_size must be > 0, got "
                f"in_features={in_features}, hidden_size={hidden_size}"
            )
        self.in_features = int(in_features)
        self.hidden_size = int(hidden_size)
        gates = len(GATES) * self.hidden_size
        bound = 1.0 / math.sqrt(self.hidden_size)
        dev = as_device(device)

        def uniform(shape):
            return np.random.uniform(-bound, bound, shape).astype(np.float32)

        self.weight_ih = Tensor.from_numpy(uniform((self.in_features, gates)), dev,
                                           requires_grad=True)
        self.weight_hh = Tensor.from_numpy(uniform((self.hidden_size, gates)), dev,
                                           requires_grad=True)
        self.bias_ih = Tensor.from_numpy(uniform((1, gates)), dev, requires_grad=True)
        self.bias_hh = Tensor.from_numpy(uniform((1, gates)), dev, requires_grad=True)

    def forward(self, x: Tensor, h: Tensor) -> Tensor:
        self._check(x, h)
        widths = (self.hidden_size,) * len(GATES)
        # x @ W + b as one fused GEMM each (the reference's matmul + add).
        gi = split(linear(x, self.weight_ih, self.bias_ih), widths)
        gh = split(linear(h, self.weight_hh, self.bias_hh), widths)
        reset = sigmoid(add(gi[0], gh[0]))
        update = sigmoid(add(gi[1], gh[1]))
        candidate = tanh(add(gi[2], mul(reset, gh[2])))
        return add(mul(sub(1.0, update), candidate), mul(update, h))

    def _check(self, x: Tensor, h: Tensor) -> None:
        xs, hs = tuple(int(d) for d in x.shape), tuple(int(d) for d in h.shape)
        if len(xs) != 2 or xs[1] != self.in_features:
            raise ValueError(
                f"GRUCell({self.in_features}, {self.hidden_size}): expected an input of shape "
                f"(batch, {self.in_features}), got {xs}."
            )
        if len(hs) != 2 or hs[1] != self.hidden_size:
            raise ValueError(
                f"GRUCell({self.in_features}, {self.hidden_size}): expected a state of shape "
                f"(batch, {self.hidden_size}), got {hs}."
            )
        if xs[0] != hs[0]:
            raise ValueError(f"GRUCell: input batch {xs[0]} and state batch {hs[0]} disagree.")


class GRU(Module):
    """A GRUCell unrolled over (T, batch, features) with an optional
    (T, batch, 1) done mask applied to the state entering each step."""

    def __init__(self, in_features: int, hidden_size: int, device=None):
        self.cell = GRUCell(in_features, hidden_size, device)
        self.in_features = self.cell.in_features
        self.hidden_size = self.cell.hidden_size

    def forward(self, x: Tensor, h0: Tensor, done: Tensor | None = None):
        shape = tuple(int(d) for d in x.shape)
        if len(shape) != 3 or shape[2] != self.in_features:
            raise ValueError(
                f"GRU({self.in_features}, {self.hidden_size}): expected a sequence of shape "
                f"(timesteps, batch, {self.in_features}), got {shape}."
            )
        steps, batch, _ = shape
        if done is not None:
            dshape = tuple(int(d) for d in done.shape)
            if dshape != (steps, batch, 1):
                raise ValueError(
                    f"GRU: done must be shaped ({steps}, {batch}, 1), got {dshape}."
                )
            done_steps = split(done, (1,) * steps, dim=0)
        rows = split(x, (1,) * steps, dim=0)
        h = h0
        outputs = []
        for index, row in enumerate(rows):
            if done is not None:
                h = apply_done_mask(h, reshape(done_steps[index], (batch, 1)))
            h = self.cell(reshape(row, (batch, self.in_features)), h)
            outputs.append(reshape(h, (1, batch, self.hidden_size)))
        return concat(outputs, dim=0), h
