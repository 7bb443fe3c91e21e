"""The acting forward (ttrl/nets/acting.py:117-188, ttrl/algos/dqn/agent.py:97-119,
ttrl/algos/ppo/policy.py:36-62): one acting step of every environment lane as
one CUDA-graph replay. The frames go up from pinned host memory, are
converted to the first convolution's row order on the device, run through the
net at the acting width, and the action choice is made by one fused kernel;
only the actions (and for PPO the log-probs and values) come back.

The random numbers are drawn on the host from the caller's generator in the
reference's order (DQN: one uniform per lane, then the exploring actions; PPO:
one uniform per lane), so a run is reproducible from the generator state and
the device makes exactly the choice the reference's host code makes.
"""

from __future__ import annotations

import copy

import numpy as np
import torch

from ttrl_b200.algos.dqn import obs_to_rows
from ttrl_b200.device import context
from ttrl_b200.engine.autograd import Tensor, as_device, no_grad
from ttrl_b200.engine.conv import Conv2d, input_fold
from ttrl_b200.engine.nn import Module
from ttrl_b200.engine.trace import capture

__all__ = ["net_at_batch", "DQNActor", "PPOActor", "draw_legal"]


def net_at_batch(net, batch: int, _seen: dict | None = None):
    """A view of `net` whose convolutions run at activation batch `batch`,
    sharing every parameter (ttrl/nets/acting.py:60-114). A module reachable
    twice (a shared trunk) maps to one view."""
    seen = {} if _seen is None else _seen
    key = id(net)
    if key in seen:
        return seen[key]
    if isinstance(net, Conv2d):
        view = net if net.geom.batch == batch else net.at_batch(batch)
    elif isinstance(net, dict):
        view = {k: net_at_batch(v, batch, seen) for k, v in net.items()}
    elif isinstance(net, (list, tuple)):
        view = type(net)(net_at_batch(v, batch, seen) for v in net)
    elif isinstance(net, Module):
        view = copy.copy(net)
        seen[key] = view
        for name, value in vars(net).items():
            setattr(view, name, net_at_batch(value, batch, seen))
        return view
    else:
        return net
    seen[key] = view
    return view


def draw_legal(rng: np.random.Generator, mask: np.ndarray) -> np.ndarray:
    """One uniformly drawn legal action per row (ttrl/spaces/mask.py:59-66)."""
    return np.argmax(np.where(np.asarray(mask) > 0.5, rng.random(np.shape(mask)), -1.0),
                     axis=-1).astype(np.int64)


class _Actor:
    """Pinned host staging, device buffers and the captured acting graphs."""

    def __init__(self, net, lanes: int, obs_shape, device):
        self.device = as_device(device)
        self.ctx = context(self.device)
        self.lanes = int(lanes)
        self.obs_shape = tuple(int(v) for v in obs_shape)
        self.net = net_at_batch(net, self.lanes)
        self.fold = input_fold(net)
        dev = self.device
        self.frames = torch.zeros((self.lanes,) + self.obs_shape, dtype=torch.uint8, device=dev)
        self.frames_host = torch.zeros(self.frames.shape, dtype=torch.uint8, pin_memory=True)
        self._graphs: dict = {}

    def _pinned(self, shape, dtype):
        return (torch.zeros(shape, dtype=dtype, device=self.device),
                torch.zeros(shape, dtype=dtype, pin_memory=True))

    def _rows(self) -> Tensor:
        frames = Tensor(self.frames, requires_grad=False)
        return obs_to_rows(frames, self.fold)

    def _run(self, key, record) -> None:
        """Replay the graph for `key`, capturing it after one eager run."""
        graph = self._graphs.get(key)
        if graph is None:
            record()  # kernel loading, workspace sizing
            torch.cuda.synchronize(self.device)
            graph, _ = capture(self.device, record)
            self._graphs[key] = graph
        graph.replay()
        torch.cuda.current_stream(self.device).synchronize()

    def close(self) -> None:
        for graph in self._graphs.values():
            graph.close()
        self._graphs.clear()


class DQNActor(_Actor):
    """Epsilon-greedy acting for `lanes` environments (ttrl/algos/dqn/agent.py:97-119)."""

    def __init__(self, net, lanes: int, obs_shape, num_actions: int, device=None, *,
                 masked: bool = False):
        super().__init__(net, lanes, obs_shape, device)
        self.num_actions = int(num_actions)
        self.draws, self.draws_host = self._pinned((self.lanes,), torch.float64)
        self.alt, self.alt_host = self._pinned((self.lanes,), torch.int32)
        self.eps, self.eps_host = self._pinned((1,), torch.float64)
        self.actions, self.actions_host = self._pinned((self.lanes,), torch.int32)
        self.masked = bool(masked)
        if self.masked:
            self.mask, self.mask_host = self._pinned((self.lanes, self.num_actions), torch.float32)

    def _record(self) -> None:
        for dst, src in ((self.frames, self.frames_host), (self.draws, self.draws_host),
                         (self.alt, self.alt_host), (self.eps, self.eps_host)):
            dst.copy_(src, non_blocking=True)
        if self.masked:
            self.mask.copy_(self.mask_host, non_blocking=True)
        with no_grad():
            q = self.net(self._rows())
        self.ctx.epsilon_greedy(q.data, self.mask if self.masked else None, self.draws, self.alt,
                                self.eps, self.actions)
        self.actions_host.copy_(self.actions, non_blocking=True)

    def act(self, obs_u8, eps: float, rng: np.random.Generator, mask=None) -> np.ndarray:
        """One action per lane: with probability eps an exploring action (any
        action, or a uniformly drawn legal one under a mask), else the greedy
        one, the random numbers drawn from `rng` in the reference's order."""
        b = self.lanes
        self.frames_host.numpy()[:] = np.asarray(obs_u8, np.uint8).reshape(self.frames.shape)
        draws = rng.random(b)
        if self.masked:
            if mask is None:
                raise ValueError("DQNActor(masked=True).act needs the legal-action mask")
            legal = np.asarray(mask, np.float32).reshape(b, self.num_actions)
            alt = draw_legal(rng, legal)
            self.mask_host.numpy()[:] = legal
        else:
            alt = rng.integers(0, self.num_actions, size=b)
        self.draws_host.numpy()[:] = draws
        self.alt_host.numpy()[:] = alt.astype(np.int32)
        self.eps_host.numpy()[0] = float(eps)
        self._run("act", self._record)
        return self.actions_host.numpy().astype(np.int64)


class PPOActor(_Actor):
    """Categorical acting for `lanes` environments (ttrl/algos/ppo/policy.py:36-62):
    -> (actions, log-probs, values)."""

    def __init__(self, net, lanes: int, obs_shape, num_actions: int, device=None):
        super().__init__(net, lanes, obs_shape, device)
        self.num_actions = int(num_actions)
        self.uniforms, self.uniforms_host = self._pinned((self.lanes,), torch.float64)
        self.actions, self.actions_host = self._pinned((self.lanes,), torch.int32)
        self.logp, self.logp_host = self._pinned((self.lanes,), torch.float32)
        self.values, self.values_host = self._pinned((self.lanes,), torch.float32)

    def _record(self, deterministic: bool) -> None:
        self.frames.copy_(self.frames_host, non_blocking=True)
        if not deterministic:
            self.uniforms.copy_(self.uniforms_host, non_blocking=True)
        with no_grad():
            logits, value = self.net(self._rows())
        self.ctx.categorical_sample(logits.data, None if deterministic else self.uniforms,
                                    self.actions, self.logp)
        self.ctx.copy_strided(self.values, value.data.reshape(-1))
        for dst, src in ((self.actions_host, self.actions), (self.logp_host, self.logp),
                         (self.values_host, self.values)):
            dst.copy_(src, non_blocking=True)

    def act(self, obs_u8, rng: np.random.Generator | None = None, *, deterministic=False):
        b = self.lanes
        self.frames_host.numpy()[:] = np.asarray(obs_u8, np.uint8).reshape(self.frames.shape)
        if not deterministic:
            self.uniforms_host.numpy()[:] = rng.random(b)
        self._run(("act", bool(deterministic)), lambda: self._record(bool(deterministic)))
        return (self.actions_host.numpy().astype(np.int64), self.logp_host.numpy().copy(),
                self.values_host.numpy().copy())
