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
from ttrl_b200.device import FORWARD_LANES, context
from ttrl_b200.engine.autograd import Tensor, as_device, no_grad
from ttrl_b200.engine.conv import input_fold
from ttrl_b200.engine.ops import dqn_td_huber

__all__ = ["DQNLearner", "step_inputs", "update_loss", "obs_to_rows"]


def step_inputs(obs_shape, device, *, batch: int, num_actions: int, mask_n: int = 0,
                prioritized: bool = False, uint8_frames: bool = True) -> dict:
    """The fixed device buffers one update reads (ttrl/algos/dqn/losses.py:44-74),
    laid out in one allocation so that a whole batch uploads in one copy."""
    from ttrl_b200.engine.step import input_arena
    f32 = torch.float32
    specs = {"obs": None, "next_obs": None}
    shape = tuple(int(v) for v in obs_shape)
    for which in ("obs", "next_obs"):
        if len(shape) == 3 and uint8_frames:
            specs[which] = ((batch, *shape), torch.uint8)
        elif len(shape) == 3:
            c, h, w = shape
            specs[which] = ((1, 1, batch * h * w, c), f32)
        else:
            specs[which] = ((batch, shape[0]), f32)
    specs.update(rewards=((batch, 1), f32), dones=((batch, 1), f32),
                 discounts=((batch, 1), f32), actions_onehot=((batch, num_actions), f32))
    if mask_n:
        specs["next_mask"] = ((batch, mask_n), f32)
    if prioritized:
        specs["is_weights"] = ((batch, 1), f32)
    inputs = input_arena(device, specs)
    for name in ("next_mask", "is_weights"):
        if name in inputs:
            inputs[name].data.fill_(1.0)
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
        with lane(FORWARD_LANES[0]):
            next_target_q = target(next_obs)
            next_target_q.data.record_stream(main)
        if double:
            with lane(FORWARD_LANES[1]):
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


class DQNLearner:
    """The learner half of the reference's DQN agent: online and target
    Q-networks, Adam, and the update as one graph replay, with the agent's
    target schedule -- after every `target_sync_interval`-th update the
    target network becomes a bit-for-bit copy of the online one, in place
    and in one launch (ttrl/algos/dqn/agent.py:180-208, which calls
    ttrl/engine/nn/module.py:164-189). Each network's parameters sit in one
    flat arena, so that copy is a single contiguous pair."""

    def __init__(self, online, target, obs_shape, num_actions: int, device=None, *,
                 batch: int = 32, lr: float = 1e-4, eps: float = 1e-8, double: bool = True,
                 huber_delta: float = 1.0, target_sync_interval: int = 8_000,
                 mask_n: int = 0, prioritized: bool = False):
        from ttrl_b200.engine.nn import parameter_arena
        from ttrl_b200.engine.optim import Adam
        from ttrl_b200.engine.step import TrainStep
        if target_sync_interval < 1:
            raise ValueError(f"DQNLearner: target_sync_interval must be at least 1, got "
                             f"{target_sync_interval}")
        self.online, self.target = online, target
        self.device = as_device(device)
        self.online_arena = parameter_arena([online])
        self.target_arena = parameter_arena([target])
        self.target.copy_from(self.online)
        self.target_sync_interval = int(target_sync_interval)
        self.update_count = 0
        self.optimizer = Adam(list(online.parameters()), lr=lr, eps=eps)
        self.inputs = step_inputs(obs_shape, self.device, batch=batch, num_actions=num_actions,
                                  mask_n=mask_n, prioritized=prioritized)
        self.step = TrainStep(
            lambda i: update_loss(online, target, i, num_actions=num_actions, double=double,
                                  huber_delta=huber_delta, mask_n=mask_n,
                                  prioritized=prioritized),
            self.inputs, self.device, optimizer=self.optimizer, mode="traced_fwd_bwd",
            critical_main=True)

    def load(self, **arrays) -> None:
        """Bind one batch of host arrays (obs, next_obs, actions_onehot,
        rewards, dones, discounts, ...) into the update's input buffers."""
        for name, value in arrays.items():
            self.step.load_input(name, value)

    def update(self, **arrays) -> dict:
        """One update on the given batch (bound first when arrays are given),
        then the target schedule; returns the update's metrics."""
        if arrays:
            self.load(**arrays)
        metrics = self.step.run()
        self._after_update()
        return metrics

    def launch(self) -> None:
        """One update on the bound batch without reading metrics back."""
        self.step.launch()
        self._after_update()

    def _after_update(self) -> None:
        self.update_count += 1
        if self.update_count % self.target_sync_interval == 0:
            self.target.copy_from(self.online)

    def close(self) -> None:
        self.step.close()
