"""Gradient-norm measurement and clipping (ttrl/algos/grads.py:13-65).

`grad_norm` / `clip_grad_norm` keep the reference's host-read semantics
(float64 sum, clip factor max_norm/(norm + 1e-6)). The `_device` variants do
the same arithmetic in one deterministic kernel (float64 accumulation on the
GPU) and hand the clip factor to the optimizer on the device, so a PPO
minibatch step stays inside one CUDA graph.
"""

from __future__ import annotations

import numpy as np
import torch

from ttrl_b200.device import context

__all__ = ["clip_grad_norm", "clip_grad_norm_device", "grad_norm", "grad_sq_device",
           "param_snapshot"]

_WS: dict = {}


def _grads(params):
    return [p.grad.reshape(-1) if p.grad.is_contiguous() else p.grad.contiguous().reshape(-1)
            for p in params if p.grad is not None]


def _sqnorm(params, max_norm: float):
    grads = _grads(params)
    if not grads:
        return None
    dev = grads[0].device
    ctx = context(dev)
    numels = [g.numel() for g in grads]
    need = ctx.sqnorm_workspace_bytes(numels)
    key = (str(dev), need, ctx._lane)  # one per launch lane: lanes may run at once
    ws = _WS.get(key)
    if ws is None:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("grad-norm workspace must be sized before graph capture "
                               "(run the step once eagerly first)")
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)
        _WS[key] = ws
    out = torch.empty(2, dtype=torch.float32, device=dev)
    for start in range(0, len(grads), 64):
        if start:
            raise ValueError("grad-norm over more than 64 tensors is not supported")
        ctx.grad_sqnorm(grads[start:start + 64], out, max_norm, ws)
    return out


def grad_sq_device(params):
    """Sum of squared gradients as a (1,) device tensor, or None."""
    out = _sqnorm(list(params), 0.0)
    return None if out is None else out[0:1]


def clip_grad_norm_device(params, max_norm: float, optimizer=None):
    """Device-side clip: returns the (2,) device tensor [norm^2, factor] and,
    when `optimizer` is given, makes its next step() scale every gradient by
    the factor (inside the same kernel)."""
    if not max_norm > 0.0:
        raise ValueError(f"clip_grad_norm: max_norm must be > 0, got {max_norm}")
    out = _sqnorm(list(params), float(max_norm))
    if out is not None and optimizer is not None:
        optimizer.grad_scale = out[1:2]
    return out


def grad_norm(params) -> float:
    total = 0.0
    for p in params:
        if p.grad is None:
            continue
        arr = p.grad.detach().to("cpu").numpy().astype(np.float64)
        total += float(np.sum(arr * arr))
    return float(np.sqrt(total))


def clip_grad_norm(params, max_norm: float) -> float:
    """Host-read clip with the reference's semantics; returns the pre-clip norm."""
    if not max_norm > 0.0:
        raise ValueError(f"clip_grad_norm: max_norm must be > 0, got {max_norm}")
    params = list(params)
    total = grad_norm(params)
    if total > max_norm:
        scale = max_norm / (total + 1e-6)
        for p in params:
            if p.grad is not None:
                scaled = torch.empty_like(p.grad)
                context(p.grad.device).ew("mul_s", p.grad, None, scaled, scale)
                p.grad = scaled
                p._grad_owned = True
    return total


def param_snapshot(module) -> dict:
    return {name: p.numpy().copy() for name, p in module.named_parameters()}
