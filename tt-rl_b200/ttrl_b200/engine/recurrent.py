"""`GRUCell` and `GRU` (ttrl/engine/recurrent.py), with the reference's
semantics: gates (reset, update, candidate) in PyTorch's column order,
weights stored (features, 3*hidden), the done mask applied to the state
entering each step, and a fixed-length unroll whose backward accumulates each
weight's gradient over all T steps.

The unroll runs as one tape node, `gru_unroll`. Its forward computes the input
projection x @ W_ih + b_ih of every timestep in one GEMM. The recurrence then
runs as one launch over all T steps (one thread-block cluster per slice of
the sequences, W_hh split across its CTAs' shared memory, the state exchanged
through distributed shared memory between steps), and its backward through
time as a second one; dW_hh and db_hh come from a single GEMM over all T
steps, and the tape's ordinary `linear` backward turns the stacked d gi into
dX, dW_ih and db_ih. Shapes the sequence kernels have no plan for (hidden not
a multiple of 4, or slices too large for shared memory) run the same
arithmetic step by step: one recurrent GEMM and one fused gate kernel per step
forward, one gate-backward kernel and one GEMM per step backward.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from ttrl_b200.engine.autograd import Tensor, _detached, _needs, as_device
from ttrl_b200.engine.nn import Module
from ttrl_b200.engine.ops import _ctx, _new, linear, reshape

__all__ = ["GRU", "GRUCell", "GATES", "gru_unroll"]

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
        gi = linear(x, self.weight_ih, self.bias_ih)
        out = gru_unroll(gi, h, None, self.weight_hh, self.bias_hh, steps=1)
        return reshape(out, (int(h.shape[0]), self.hidden_size))

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
        cell = self.cell
        gi = linear(reshape(x, (steps * batch, self.in_features)), cell.weight_ih, cell.bias_ih)
        outputs = gru_unroll(gi, h0, done, cell.weight_hh, cell.bias_hh, steps=steps)
        return outputs, _last_step(outputs)


def _last_step(outputs: Tensor) -> Tensor:
    """outputs[T-1] as a view; its backward (taken only when the final state
    feeds the loss) scatters into a zero gradient of the whole sequence."""
    steps = int(outputs.shape[0])
    data = outputs.data[steps - 1]
    if not _needs(outputs):
        return _detached(data)
    out = Tensor(data, True, (outputs,), "gru_final")

    def _backward(grad):
        if outputs.requires_grad:
            full = _new(outputs.shape, grad)
            ctx = _ctx(grad)
            ctx.ew("fill", None, None, full, 0.0)
            ctx.copy_strided(full[steps - 1], grad.reshape(full[steps - 1].shape))
            outputs._accumulate(full)

    out._backward = _backward
    return out


def gru_unroll(gi: Tensor, h0: Tensor, starts, w_hh: Tensor, b_hh: Tensor, *,
               steps: int, persistent: bool | None = None) -> Tensor:
    """The recurrent half of a GRU over `steps` timesteps, as one tape node.

    gi: x @ W_ih + b_ih for every step, rows time-major [steps * batch, 3H];
    h0: [batch, H]; starts: None or a (steps, batch, 1) {0, 1} mask applied to
    the state entering each step (ttrl/engine/recurrent.py:163-167);
    w_hh [H, 3H], b_hh [1, 3H]. -> outputs (steps, batch, H).
    `persistent` picks the one-launch sequence kernels (None: whenever the
    shape has a plan) or the step-by-step launches.
    """
    batch, hidden = int(h0.shape[0]), int(h0.shape[1])
    g = gi.data if gi.data.is_contiguous() else gi.data.contiguous()
    if tuple(g.shape) != (steps * batch, 3 * hidden):
        raise ValueError(f"gru_unroll: gi has shape {tuple(g.shape)}, expected "
                         f"({steps * batch}, {3 * hidden})")
    g = g.reshape(steps, batch, 3 * hidden)
    hd = h0.data if h0.data.is_contiguous() else h0.data.contiguous()
    sd = None
    if starts is not None:
        sv = starts.data if isinstance(starts, Tensor) else starts
        sd = sv.contiguous().reshape(steps, batch)
    ctx = _ctx(g)
    gh = _new((steps, batch, 3 * hidden), g)
    gates = _new((steps, batch, 3 * hidden), g)
    hm = _new((steps, batch, hidden), g)
    out = _new((steps, batch, hidden), g)
    if persistent is None:
        persistent = ctx.gru_sequence_supported(batch, hidden)
    if persistent:
        ctx.gru_sequence_fwd(g, hd, sd, w_hh.data, b_hh.data, gh, gates, hm, out)
    else:
        ctx.gru_mask(hd, None if sd is None else sd[0], hm[0])
        for t in range(steps):
            ctx.linear_fwd(hm[t], w_hh.data, b_hh.data, gh[t], False)
            nxt = t + 1 < steps
            ctx.gru_gates_fwd(g[t], gh[t], hm[t], sd[t + 1] if (nxt and sd is not None) else None,
                              out[t], gates[t], hm[t + 1] if nxt else None)
    parents = (gi, h0, w_hh, b_hh)
    if not _needs(*parents):
        return _detached(out)
    node = Tensor(out, True, parents, "gru_unroll")

    def _backward(grad):
        dy = grad if grad.is_contiguous() else grad.contiguous()
        dy = dy.reshape(steps, batch, hidden)
        dgi = _new((steps, batch, 3 * hidden), dy)
        dgh = _new((steps, batch, 3 * hidden), dy)
        need_h0 = h0.requires_grad
        if persistent:
            d0 = _new((batch, hidden), dy) if need_h0 else None
            ctx.gru_sequence_bwd(dy, sd, w_hh.data, gates, gh, hm, dgi, dgh, d0)
        else:
            dhm = _new((batch, hidden), dy)
            for t in reversed(range(steps)):
                nxt = t + 1 < steps
                ctx.gru_gates_bwd(dy[t], dhm, sd[t + 1] if (nxt and sd is not None) else None,
                                  nxt, gates[t], gh[t], hm[t], dgi[t], dgh[t])
                if t > 0 or need_h0:
                    ctx.linear_dgrad(dgh[t], w_hh.data, None, dhm, True)
            if need_h0:
                d0 = _new((batch, hidden), dy)
                ctx.gru_mask(dhm, None if sd is None else sd[0], d0)
        if need_h0:
            h0._accumulate(d0)
        wb, bb = w_hh.requires_grad, b_hh.requires_grad
        if wb or bb:
            if wb:
                dw, accw = w_hh._grad_slot()
            else:
                dw, accw = torch.empty_like(w_hh.data), False
            if bb:
                db, accb = b_hh._grad_slot()
            else:
                db, accb = None, False
            ctx.linear_wgrad(hm.reshape(steps * batch, hidden),
                             dgh.reshape(steps * batch, 3 * hidden), dw, db, accw, accb)
            if wb:
                w_hh._set_grad(dw)
            if bb:
                b_hh._set_grad(db)
        if gi.requires_grad:
            gi._accumulate(dgi.reshape(steps * batch, 3 * hidden))

    node._backward = _backward
    return node
