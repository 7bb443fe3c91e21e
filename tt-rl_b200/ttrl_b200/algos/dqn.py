"""DQN's update body and its input buffers (ttrl/algos/dqn/losses.py).

`update_loss` keeps the reference's contract -- reads only the bound inputs,
never reads back to the host, calls backward itself, returns device metrics
{loss, mean_q, grad_sq[, td_abs]} -- so it captures into one CUDA graph. The
three forwards run the fused conv/linear kernels and the whole loss head
(gather, double-DQN argmax, bootstrap, Huber, mean, and dQ) is one kernel.

Observation buffers may be uint8 frames [B, C, H, W] (converted on the
device by one kernel, the 1/255 folded into conv1 as the reference folds
it) or float rows already in the network's input layout.
"""

from __future__ import annotations

import contextlib

import numpy as np
import torch

from ttrl_b200.algos.grads import grad_sq_device
from ttrl_b200.device import context
from ttrl_b200.engine.autograd import Tensor, as_device, no_grad
from ttrl_b200.engine.conv import input_fold
from ttrl_b200.engine.ops import dqn_td_huber

__all__ = ["step_inputs", "update_loss", "obs_to_rows"]


def step_inputs(obs_shape, device, *, batch: int, num_actions: int, mask_n: int = 0,
                prioritized: bool = False, uint8_frames: bool = True) -> dict:
    """The fixed device buffers one update reads (ttrl/algos/dqn/losses.py:44-74)."""
    dev = as_device(device)

    def zeros(*shape, dtype=torch.float32):
        return Tensor(torch.zeros(shape, dtype=dtype, device=dev))

    inputs = {
        "rewards": zeros(batch, 1),
        "dones": zeros(batch, 1),
        "discounts": zeros(batch, 1),
        "actions_onehot": zeros(batch, num_actions),
    }
    shape = tuple(int(v) for v in obs_shape)
    for which in ("obs", "next_obs"):
        if len(shape) == 3 and uint8_frames:
            inputs[which] = zeros(batch, *shape, dtype=torch.uint8)
        elif len(shape) == 3:
            c, h, w = shape
            inputs[which] = zeros(1, 1, batch * h * w, c)
        else:
            inputs[which] = zeros(batch, shape[0])
    if mask_n:
        inputs["next_mask"] = Tensor(torch.ones((batch, mask_n), device=dev))
    if prioritized:
        inputs["is_weights"] = Tensor(torch.ones((batch, 1), device=dev))
    return inputs


def obs_to_rows(obs: Tensor, fold: int = 1) -> Tensor:
    """uint8 [B, C, H, W] frames -> fp32 NHWC rows [1, 1, B*H*W, C] (raw 0..255;
    the 1/255 is conv1's input scale), in the space-to-depth order of `fold`
    when the first convolution reads that (`input_fold(net)`). Float inputs
    pass through."""
    if obs.data.dtype != torch.uint8:
        return obs
    b, c, h, w = obs.shape
    out = torch.empty((1, 1, b * h * w // (fold * fold), c * fold * fold), dtype=torch.float32,
                      device=obs.data.device)
    context(obs.data.device).u8_to_f32(obs.data, None, out.reshape(-1, c * fold * fold), 1.0,
                                       fold=fold)
    rows = Tensor(out, requires_grad=False)
    rows._exact = True  # raw 0..255 values
    rows._fold = fold
    return rows


def update_loss(online, target, inputs: dict, *, num_actions: int, double: bool = True,
                huber_delta: float = 1.0, mask_n: int = 0, prioritized: bool = False,
                leaves=None) -> dict:
    """One DQN update: Huber loss against the (double-)DQN n-step target,
    backward, and device metrics (ttrl/algos/dqn/losses.py:77-140)."""
    fold = input_fold(online)
    next_obs = obs_to_rows(inputs["next_obs"], fold)
    # The two no-grad forwards on s' are independent of the online forward on
    # s: they run on side lanes, concurrently with it (parallel branches of
    # the captured graph), and the loss waits for all three.
    ctx = context(next_obs.data.device)
    main = torch.cuda.current_stream(ctx.device)
    lane = ctx.side if ctx.concurrent else (lambda _k: contextlib.nullcontext())
    with no_grad():
        with lane(1):
            next_target_q = target(next_obs)
            next_target_q.data.record_stream(main)
        if double:
            with lane(2):
                selector = online(next_obs)
                selector.data.record_stream(main)
        else:
            selector = next_target_q
    obs = obs_to_rows(inputs["obs"], fold)
    q = online(obs)
    ctx.join()
    loss, mean_q, td_abs = dqn_td_huber(
        q, selector, next_target_q, inputs["actions_onehot"], inputs["rewards"],
        inputs["dones"], inputs["discounts"], delta=huber_delta,
        next_mask=inputs.get("next_mask") if mask_n else None,
        is_weights=inputs.get("is_weights") if prioritized else None,
        want_td_abs=prioritized)
    loss.backward()
    metrics = {"loss": loss, "mean_q": mean_q}
    if prioritized:
        metrics["td_abs"] = td_abs
    # The gradient norm is a metric only: on side lane 2 it runs beside the
    # optimizer step that follows.
    with lane(2):
        grad_sq = grad_sq_device(online.parameters())
    if grad_sq is not None:
        metrics["grad_sq"] = Tensor(grad_sq.reshape(1, 1), requires_grad=False)
    return metrics
