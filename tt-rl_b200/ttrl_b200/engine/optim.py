"""Optimizers: `Optimizer`, `Adam`, `adam_fused_scalars`
(ttrl/engine/optim/{base,adam,scalars,checkpoint}.py).

Adam keeps the reference's stored S = m/(1-b1), V = v/(1-b2) moments and
its per-parameter step counts, and runs as ONE multi-tensor CUDA kernel per
step. The step counts live on the device (the kernel reads and advances
them), so the whole update -- Adam included -- can be captured into a CUDA
graph and replayed with the correct bias correction every time. A host
mirror of the counts backs `state_dict`.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from ttrl_b200.device import context
from ttrl_b200.engine.tensor import MASTER_DTYPE, restore_in_place, to_host

__all__ = ["Optimizer", "Adam", "adam_bias_table", "adam_fused_scalars", "share_launch",
           "step_together"]


def adam_fused_scalars(lr: float, b1: float, b2: float, eps: float, t: int) -> tuple[float, float]:
    """(alpha_t, eps_t) folding the bias correction (ttrl/engine/optim/scalars.py:13-27)."""
    if t < 1:
        raise ValueError(f"adam_fused_scalars: t must be >= 1, got {t}")
    bc1 = 1 - b1 ** t
    bc2 = 1 - b2 ** t
    c = math.sqrt((1 - b2) / bc2)
    return lr * (1 - b1) / bc1 / c, eps / c


#: Longest bias-term table built (steps); betas that converge later fall
#: back to the kernel's own pow().
BIAS_TABLE_MAX_STEPS = 1 << 20

_BIAS_TABLES: dict = {}


def adam_bias_table(b1: float, b2: float, device):
    """(T, 2) float64 device table of (1 - b1^t, sqrt((1 - b2)/(1 - b2^t)))
    for t = 1..T, the terms of adam_fused_scalars from the host's pow(); T
    is the first step at which both have converged to 1 (in double), so the
    kernel reads the last row for every later step. None when that takes
    more than BIAS_TABLE_MAX_STEPS steps. One table per (betas, device)."""
    key = (float(b1), float(b2), str(device))
    if key in _BIAS_TABLES:
        return _BIAS_TABLES[key]
    tiny = math.ldexp(1.0, -54)  # 1 - x == 1 in double once x < 2^-54
    need = 1
    for b in (b1, b2):
        if b > 0.0:
            need = max(need, int(math.ceil(math.log(tiny) / math.log(b))) + 2)
    table = None
    if need <= BIAS_TABLE_MAX_STEPS:
        # Python's own pow (the reference's `b ** t`), not a vectorised one
        # that may round differently.
        rows = []
        for t in range(1, need + 1):
            bc1, bc2 = 1 - b1 ** t, 1 - b2 ** t
            rows.append((bc1, math.sqrt((1 - b2) / bc2)))
            if bc1 == 1.0 and bc2 == 1.0:
                table = torch.tensor(rows, dtype=torch.float64).to(device)
                break
    _BIAS_TABLES[key] = table
    return table


class Optimizer:
    def __init__(self, params):
        self.params = list(params)

    def zero_grad(self) -> None:
        for p in self.params:
            p.zero_grad()

    def step(self) -> None:
        raise NotImplementedError


class Adam(Optimizer):
    """Adam over fp32 parameters, updated in place by one fused kernel."""

    def __init__(self, params, lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0):
        super().__init__(params)
        if not self.params:
            raise ValueError("Adam: params is empty, so there is nothing to optimize")
        if lr <= 0:
            raise ValueError(f"Adam: lr must be > 0, got {lr}")
        b1, b2 = betas
        if not (0.0 <= b1 < 1.0 and 0.0 <= b2 < 1.0):
            raise ValueError(f"Adam: betas must be in [0, 1), got {betas}")
        if eps <= 0:
            raise ValueError(f"Adam: eps must be > 0, got {eps}")
        if weight_decay < 0:
            raise ValueError(f"Adam: weight_decay must be >= 0, got {weight_decay}")
        wrong = [i for i, p in enumerate(self.params) if p.data.dtype != MASTER_DTYPE]
        if wrong:
            raise ValueError(f"Adam: parameters must be {MASTER_DTYPE}; parameters {wrong} are not")
        self.b1, self.b2 = b1, b2
        self.eps = eps
        self.weight_decay = weight_decay
        self.t = 0
        self.steps = [0] * len(self.params)
        dev = self.params[0].data.device
        self._device = dev
        self.m = [torch.zeros_like(p.data) for p in self.params]   # S
        self.v = [torch.zeros_like(p.data) for p in self.params]   # V
        self._dev_steps = torch.zeros(len(self.params), dtype=torch.int32, device=dev)
        self._ticket = torch.zeros(1, dtype=torch.int32, device=dev)
        self._lr_dev = torch.zeros(1, dtype=torch.float64, device=dev)
        self._lr = float(lr)
        self._lr_dev.copy_(torch.tensor([self._lr], dtype=torch.float64))
        # Set by a device-side gradient clip for the next step() (see
        # ttrl_b200.algos.grads.clip_grad_norm_device).
        self.grad_scale = None
        # Indices stepped by the launch recorded inside a graph capture.
        self.captured_indices: list[int] | None = None
        # (group, counter base, rate slot) once share_launch joined it.
        self._shared = None
        self._bias = adam_bias_table(b1, b2, dev)

    # The learning rate lives on the device too, so a replayed graph reads
    # the current value (PPO's annealing, ttrl/algos/ppo/learn.py:54-56).
    @property
    def lr(self) -> float:
        return self._lr

    @lr.setter
    def lr(self, value: float) -> None:
        self._lr = float(value)
        self._lr_dev.copy_(torch.tensor([self._lr], dtype=torch.float64))

    @property
    def _m_scale(self) -> float:
        return 1 - self.b1

    @property
    def _v_scale(self) -> float:
        return 1 - self.b2

    def _pending(self, step_base: int = 0, lr_index: int = 0):
        """(tensors, stepped indices) of the parameters that hold a gradient."""
        tensors = []
        stepped = []
        for i, p in enumerate(self.params):
            if p.grad is None:
                continue
            g = p.grad if p.grad.is_contiguous() else p.grad.contiguous()
            tensors.append((p.data, g.reshape(p.data.shape), self.m[i], self.v[i],
                            step_base + i, lr_index))
            stepped.append(i)
        return tensors, stepped

    def _finish(self, stepped) -> None:
        self.grad_scale = None
        if torch.cuda.is_current_stream_capturing():
            # Recorded, not run: TrainStep advances the host mirror per replay.
            self.captured_indices = stepped
            return
        self.advance(stepped)

    def step(self) -> None:
        """One update of every parameter that holds a gradient."""
        tensors, stepped = self._pending()
        if tensors:
            context(self._device).adam_step(
                tensors, self._dev_steps, self._ticket, self.grad_scale, self._lr, self.b1,
                self.b2, self.eps, self.weight_decay, lr_device=self._lr_dev, bias=self._bias)
        self._finish(stepped)

    def advance(self, stepped) -> None:
        """Advance the host mirror of the device step counters."""
        self.t += 1
        for i in stepped:
            self.steps[i] += 1

    def _step_scalars(self, t: int) -> tuple[float, float]:
        return adam_fused_scalars(self._lr, self.b1, self.b2, self.eps, t)

    # -- checkpoint (ttrl/engine/optim/checkpoint.py) ---------------------

    def state_dict(self) -> dict:
        return {
            "t": self.t,
            "steps": list(self.steps),
            "lr": self._lr,
            "betas": (self.b1, self.b2),
            "eps": self.eps,
            "weight_decay": self.weight_decay,
            "m": [self._portable(i, to_host(m) * self._m_scale) for i, m in enumerate(self.m)],
            "v": [self._portable(i, to_host(v) * self._v_scale) for i, v in enumerate(self.v)],
        }

    def _portable(self, i: int, array: np.ndarray) -> np.ndarray:
        """A moment in its parameter's portable layout (a convolution weight's
        in OIHW, every other parameter's as stored)."""
        layout = getattr(self.params[i], "_layout", None)
        return array if layout is None else layout.to_portable(array)

    def load_state_dict(self, state: dict, device=None) -> None:
        if len(state["m"]) != len(self.m) or len(state["v"]) != len(self.v):
            raise ValueError(
                f"Adam.load_state_dict: checkpoint has {len(state['m'])} m and "
                f"{len(state['v'])} v buffers, expected {len(self.m)} of each."
            )
        device_form = {"m": [], "v": []}
        for key, buffers in (("m", self.m), ("v", self.v)):
            for i, (arr, buf) in enumerate(zip(state[key], buffers)):
                layout = getattr(self.params[i], "_layout", None)
                got = tuple(np.asarray(arr).shape)
                if layout is not None:
                    # Logical OIHW or the reference's prepared matrix; the
                    # stored v fixes the latter's channel stride.
                    try:
                        arr = layout.from_stored(arr, v=state["v"][i])
                    except ValueError as exc:
                        raise ValueError(
                            f"Adam.load_state_dict: {key}[{i}] has shape {got}, which is "
                            f"neither its convolution weight's OIHW shape {layout.oihw} nor "
                            f"a prepared matrix holding it ({exc})") from None
                elif got != tuple(buf.shape):
                    raise ValueError(
                        f"Adam.load_state_dict: {key}[{i}] has shape {got}, which does "
                        f"not match its parameter's shape {tuple(buf.shape)}."
                    )
                device_form[key].append(arr)
        t = int(state["t"])
        steps = [int(s) for s in state.get("steps", [t] * len(self.params))]
        lr = state.get("lr", self._lr)
        b1, b2 = state.get("betas", (self.b1, self.b2))
        eps = state.get("eps", self.eps)
        weight_decay = state.get("weight_decay", self.weight_decay)
        if len(steps) != len(self.params):
            raise ValueError(f"Adam.load_state_dict: checkpoint has {len(steps)} step counters, "
                             f"expected {len(self.params)}.")
        if t < 0 or any(s < 0 for s in steps):
            raise ValueError(f"Adam.load_state_dict: step counts must be >= 0, got t={t}.")
        if not lr > 0:
            raise ValueError(f"Adam.load_state_dict: lr must be > 0, got {lr}.")
        if not (0.0 <= b1 < 1.0 and 0.0 <= b2 < 1.0):
            raise ValueError(f"Adam.load_state_dict: betas must be in [0, 1), got {(b1, b2)}.")
        if not eps > 0:
            raise ValueError(f"Adam.load_state_dict: eps must be > 0, got {eps}.")
        if weight_decay < 0:
            raise ValueError(f"Adam.load_state_dict: weight_decay must be >= 0, got {weight_decay}.")
        self.t = t
        self.steps = steps
        self.lr = lr
        self.b1, self.b2 = b1, b2
        self.eps = eps
        self.weight_decay = weight_decay
        self._bias = adam_bias_table(self.b1, self.b2, self._device)
        ms, vs = self._m_scale, self._v_scale
        for i, arr in enumerate(device_form["m"]):
            restore_in_place(self.m[i], np.asarray(arr) / ms)
        for i, arr in enumerate(device_form["v"]):
            restore_in_place(self.v[i], np.asarray(arr) / vs)
        self._dev_steps.copy_(torch.tensor(steps, dtype=torch.int32))


class _SharedLaunch:
    """Device state that several Adams keep side by side so that one kernel
    launch can step them all: their step counters in one int32 array, their
    learning rates in one float64 array, one ticket."""

    def __init__(self, opts):
        dev = opts[0]._device
        counts = [len(o.params) for o in opts]
        self.steps = torch.zeros(sum(counts), dtype=torch.int32, device=dev)
        self.lrs = torch.zeros(len(opts), dtype=torch.float64, device=dev)
        self.ticket = torch.zeros(1, dtype=torch.int32, device=dev)
        self.opts = list(opts)
        self.bases = []
        base = 0
        for slot, (o, n) in enumerate(zip(opts, counts)):
            self.steps[base:base + n].copy_(o._dev_steps)
            self.lrs[slot:slot + 1].copy_(o._lr_dev)
            # Views: every in-place write of the optimizer (load_state_dict,
            # the lr setter, a restore) lands in the shared arrays.
            o._dev_steps = self.steps[base:base + n]
            o._lr_dev = self.lrs[slot:slot + 1]
            o._shared = (self, base, slot)
            self.bases.append(base)
            base += n


def share_launch(opts) -> None:
    """Let `step_together(opts)` step these Adams in one kernel launch. Each
    keeps its own parameters, moments, step counters, learning rate and
    state_dict; only where the device copies of the counters and the rate
    live changes. All must be on one device."""
    opts = list(opts)
    if len(opts) < 2:
        return
    if any(not isinstance(o, Adam) for o in opts):
        raise TypeError("share_launch: Adam optimizers only")
    if len({o._device for o in opts}) != 1:
        raise ValueError("share_launch: the optimizers live on different devices")
    if sum(len(o.params) for o in opts) > 64:
        raise ValueError("share_launch: more than 64 parameters in all")
    _SharedLaunch(opts)


def step_together(opts) -> None:
    """step() every optimizer of `opts`: one launch when they were joined by
    share_launch and agree on betas, eps and weight decay with no gradient
    scale pending (the math per parameter is unchanged: each reads its own
    counter and rate); otherwise one step() each, in order."""
    opts = list(opts)
    shared = [getattr(o, "_shared", None) for o in opts]
    group = shared[0][0] if shared and shared[0] is not None else None
    joint = (group is not None and all(s is not None and s[0] is group for s in shared)
             and all(o.grad_scale is None for o in opts)
             and len({(o.b1, o.b2, o.eps, o.weight_decay) for o in opts}) == 1
             and len({id(o._bias) for o in opts}) == 1)
    if not joint:
        for o in opts:
            o.step()
        return
    tensors, stepped = [], []
    for o, (_, base, slot) in zip(opts, shared):
        t, s = o._pending(base, slot)
        tensors += t
        stepped.append(s)
    if tensors:
        head = opts[0]
        context(head._device).adam_step(tensors, group.steps, group.ticket, None, head._lr,
                                        head.b1, head.b2, head.eps, head.weight_decay,
                                        lr_device=group.lrs, bias=head._bias)
    for o, s in zip(opts, stepped):
        o._finish(s)

