"""SAC's learning half on the B200 kernels (ttrl/algos/sac/{losses,step,policy,
targets}.py and ttrl/algos/gaussian.py).

The losses, the tanh-squashed Gaussian and the gaussian helpers keep the
reference's compositions op for op (the same relu-identity `minimum`, the
same stable `log(1 - tanh(u)^2)` form, the same 0.5 on the twin-critic sum),
so the parity vectors of the reference's own code apply unchanged.

`SACLearner` runs one whole update -- critic region, critic Adam, actor and
temperature region, policy and temperature Adams, Polyak averaging of the
targets -- from ONE CUDA graph. The reference captures the two regions and
runs its three Adams eagerly between them (ttrl/algos/sac/step.py:1-13)
because its bias corrections are host scalars; here Adam reads device step
counters, so it joins the graph. The order of the steps is unchanged.

One difference that changes no result: during the actor region the critic
parameters do not request gradients. The reference's actor backward computes
critic weight gradients and then discards them (the region steps only the
policy); skipping those two weight-gradient GEMMs leaves d loss / d action,
and so every policy gradient, as it was.

For nets of `build_sac_nets`'s shape (a Gaussian-head policy, critics that
read concat(obs, action) directly), the learner runs the regions on the fused
heads of engine.ops (`sac_sample`, `sac_critic_loss`, `sac_actor_loss`): the
sample with its log-density and its backward, each loss with its gradient,
one launch each, in place of the reference's elementwise chains; both online
critics read one concat(obs, action) buffer. The composed functions below
stay the reference's op-for-op form (`fused=False` runs the learner on them).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from functools import reduce

import numpy as np
import torch

from ttrl_b200.algos.grads import grad_sq_device
from ttrl_b200.device import FORWARD_LANES, context
from ttrl_b200.engine.autograd import Tensor, as_device, no_grad
from ttrl_b200.engine.ops import (abs_, add, apply_done_mask, div, exp, log, mean_all,
                                  minimum, mul, neg, relu, sac_actor_loss, sac_critic_loss,
                                  sac_sample, square, sub, sum_dim, tanh)
from ttrl_b200.engine.optim import Adam, share_launch, step_together
from ttrl_b200.engine.trace import capture

__all__ = ["LOG_2PI", "softplus", "normal_logp", "log_one_minus_tanh_sq", "squashed_logp",
           "ActionScale", "SquashedGaussian", "min_q", "critic_loss", "actor_loss",
           "alpha_loss", "priority_errors", "critic_region", "actor_region",
           "critic_region_fused", "actor_region_fused", "fused_heads_apply", "SACConfig",
           "SACLearner"]

LOG_2PI = math.log(2.0 * math.pi)
_LOG_2 = math.log(2.0)


# ---------------------------------------------------------------- gaussian

def softplus(x: Tensor) -> Tensor:
    """relu(x) + log(1 + exp(-|x|)) (ttrl/algos/gaussian.py:55-62)."""
    return add(relu(x), log(add(exp(neg(abs_(x))), 1.0)))


def normal_logp(x: Tensor, mean: Tensor, log_std: Tensor) -> Tensor:
    """log N(x; mean, exp(log_std)^2) summed over the action dim, (B, 1)
    (ttrl/algos/gaussian.py:65-70)."""
    dim = int(x.shape[-1])
    z = div(sub(x, mean), exp(log_std))
    per_dim = sub(mul(square(z), -0.5), log_std)
    return sub(sum_dim(per_dim, dim=-1, keepdim=True), 0.5 * dim * LOG_2PI)


def log_one_minus_tanh_sq(u: Tensor) -> Tensor:
    """2 * (log 2 - u - softplus(-2u)) (ttrl/algos/gaussian.py:73-84)."""
    return mul(sub(sub(_LOG_2, u), softplus(mul(u, -2.0))), 2.0)


def squashed_logp(u: Tensor, mean: Tensor, log_std: Tensor) -> Tensor:
    """log density of tanh(u) (ttrl/algos/gaussian.py:87-90), (B, 1)."""
    correction = sum_dim(log_one_minus_tanh_sq(u), dim=-1, keepdim=True)
    return sub(normal_logp(u, mean, log_std), correction)


class ActionScale:
    """Affine map of [-1, 1]^d onto the action bounds
    (ttrl/algos/gaussian.py:120-167)."""

    def __init__(self, low, high, device=None):
        low = np.asarray(low, np.float32).reshape(-1)
        high = np.asarray(high, np.float32).reshape(-1)
        if low.shape != high.shape or np.any(high <= low):
            raise ValueError("ActionScale: every bound must satisfy low < high")
        self.dim = int(low.size)
        self.centre = ((high + low) * 0.5).astype(np.float32)
        self.half_width = ((high - low) * 0.5).astype(np.float32)
        self.log_det = float(np.sum(np.log(self.half_width.astype(np.float64))))
        self._scale = self._centre = None
        if device is not None:
            self._scale = Tensor.from_numpy(self.half_width.reshape(1, self.dim), device)
            self._centre = Tensor.from_numpy(self.centre.reshape(1, self.dim), device)

    def to_env(self, squashed: Tensor) -> Tensor:
        if self._scale is None:
            raise ValueError("ActionScale.to_env needs device bounds: pass a device")
        return add(mul(squashed, self._scale), self._centre)

    def env_logp(self, value: Tensor) -> Tensor:
        return sub(value, self.log_det)

    def to_env_numpy(self, squashed):
        return (self.centre + self.half_width * np.asarray(squashed)).astype(np.float32)


class SquashedGaussian:
    """tanh of a diagonal Gaussian on the action bounds
    (ttrl/algos/sac/policy.py:22-40)."""

    def __init__(self, low, high, device):
        self.scale = ActionScale(low, high, device)
        self.dim = self.scale.dim

    def sample(self, mean: Tensor, log_std: Tensor, noise: Tensor):
        """-> (env_action (B, dim), logp (B, 1)), both differentiable."""
        pre_squash = add(mean, mul(exp(log_std), noise))
        logp = self.scale.env_logp(squashed_logp(pre_squash, mean, log_std))
        return self.scale.to_env(tanh(pre_squash)), logp


# ------------------------------------------------------------------ losses

def min_q(nets, obs, action: Tensor) -> Tensor:
    """Minimum over the critics (ttrl/algos/sac/losses.py:24-26)."""
    return reduce(minimum, [net(obs, action) for net in nets])


def priority_errors(errors) -> Tensor:
    """Mean over critics of |TD error|, detached (losses.py:29-44)."""
    with no_grad():
        total = None
        for error in errors:
            magnitude = abs_(error.detach())
            total = magnitude if total is None else add(total, magnitude)
        return mul(total, 1.0 / len(errors))


def critic_loss(nets, dist, batch, alpha: Tensor, weights: Tensor | None = None):
    """0.5 * sum over critics of mean((Q_i - y)^2) against the soft target
    (ttrl/algos/sac/losses.py:46-79). -> (loss, target, errors)."""
    with no_grad():
        mean, log_std = nets.policy(batch.next_obs)
        next_action, next_logp = dist.sample(mean, log_std, batch["next_noise"])
        soft_value = sub(min_q(nets.targets, batch.next_obs, next_action),
                         mul(next_logp, alpha))
        target = add(batch["rewards"],
                     mul(apply_done_mask(soft_value, batch["dones"]), batch["discounts"]))
    errors = [sub(critic(batch.obs, batch["actions"]), target) for critic in nets.critics]
    squared = [square(error) for error in errors]
    if weights is not None:
        squared = [mul(term, weights) for term in squared]
    loss = reduce(add, [mean_all(term) for term in squared])
    return mul(loss, 0.5), target, errors


def actor_loss(nets, dist, batch, alpha: Tensor):
    """mean(alpha * logp - min_i Q_i(s, a~pi)) (losses.py:82-87). -> (loss, logp)."""
    mean, log_std = nets.policy(batch.obs)
    action, logp = dist.sample(mean, log_std, batch["noise"])
    return mean_all(sub(mul(logp, alpha), min_q(nets.critics, batch.obs, action))), logp


def alpha_loss(log_alpha: Tensor, logp: Tensor, target_entropy: float) -> Tensor:
    """-mean(log_alpha * (logp + target_entropy)), logp detached (losses.py:90-98)."""
    return mul(mean_all(mul(log_alpha, add(logp.detach(), target_entropy))), -1.0)


def _alpha(log_alpha: Tensor) -> Tensor:
    with no_grad():
        return exp(log_alpha)


def critic_region(nets, dist, batch, log_alpha: Tensor, *, prioritized: bool) -> dict:
    """Critic forward, twin-critic loss, backward -> device metrics
    (ttrl/algos/sac/step.py:63-76)."""
    alpha = _alpha(log_alpha)
    weights = batch["is_weights"] if prioritized else None
    loss, target, errors = critic_loss(nets, dist, batch, alpha, weights)
    loss.backward()
    metrics = {"critic_loss": loss, "alpha": alpha, "q_target": target.detach()}
    total = grad_sq_device(nets.critic_parameters())
    if total is not None:
        metrics["critic_grad_sq"] = total
    if prioritized:
        metrics["td_abs"] = priority_errors(errors)
    return metrics


def actor_region(nets, dist, batch, log_alpha: Tensor, target_entropy: float, *,
                 learn_alpha: bool) -> dict:
    """Actor forward, loss, backward, and the temperature's dual
    (ttrl/algos/sac/step.py:79-99)."""
    alpha = _alpha(log_alpha)
    critic_params = nets.critic_parameters()
    flags = [p.requires_grad for p in critic_params]
    for p in critic_params:
        p.requires_grad = False
    try:
        loss, logp = actor_loss(nets, dist, batch, alpha)
        loss.backward()
    finally:
        for p, f in zip(critic_params, flags):
            p.requires_grad = f
    metrics = {"actor_loss": loss, "logp": logp.detach()}
    total = grad_sq_device(nets.policy_parameters())
    if total is not None:
        metrics["actor_grad_sq"] = total
    if learn_alpha:
        dual = alpha_loss(log_alpha, logp, target_entropy)
        dual.backward()
        metrics["alpha_loss"] = dual
    return metrics


# ------------------------------------------------------------ fused regions

def fused_heads_apply(nets) -> bool:
    """True for nets the fused heads serve: a policy that is an encoder and a
    Gaussian head, and critics (and targets) reading concat(obs, action)
    through an encoder without layers."""
    from ttrl_b200.nets.heads import GaussianHead
    from ttrl_b200.nets.models import ConcatEncoder, ContinuousCritic, EncoderHead
    policy = getattr(nets, "policy", None)
    if not isinstance(policy, EncoderHead) or not isinstance(policy.head, GaussianHead):
        return False
    critics, targets = list(nets.critics), list(nets.targets)
    if not critics or len(critics) != len(targets) or len(critics) > 8:
        return False
    for net in critics + targets:
        if not isinstance(net, ContinuousCritic) or not isinstance(net.encoder, ConcatEncoder):
            return False
        if getattr(net.encoder.encoder, "has_parameters", True):
            return False
    return True


def _policy_raw(policy, obs):
    """(mean, log-std before the clamp) of a Gaussian-head policy."""
    features = policy.encoder(obs)
    heads = policy.head.heads
    return heads["mean"](features), heads["log_std"](features)


def _sample(dist, policy, mean, raw, noise, obs, pack=None):
    head = policy.head
    scale = dist.scale
    return sac_sample(mean, raw, noise, scale._scale.data.reshape(-1),
                      scale._centre.data.reshape(-1), scale.log_det,
                      log_std_min=head.log_std_min, log_std_max=head.log_std_max, obs=obs,
                      pack=pack)


def _critics_side_by_side(ctx, critics, joint):
    """Q(s, a) of every critic on `joint`: the first on the current stream,
    the others on the forward lanes beside it (their forwards are
    independent; the tape's backward later runs on the current stream). The
    caller joins the lanes before using the values."""
    critics = list(critics)
    if not ctx.concurrent or len(critics) - 1 > len(FORWARD_LANES):
        return [critic.head(joint) for critic in critics]
    main = torch.cuda.current_stream(ctx.device)
    qs = [None] * len(critics)
    for i, critic in enumerate(critics[1:]):
        with ctx.side(FORWARD_LANES[i]):
            qs[i + 1] = critic.head(joint)
            qs[i + 1].data.record_stream(main)
    qs[0] = critics[0].head(joint)
    return qs


def critic_region_fused(nets, dist, batch, log_alpha: Tensor, *, prioritized: bool) -> dict:
    """critic_region on the fused heads: the next-state sample also packs the
    replayed concat(obs, action) that both online critics read."""
    ctx = context(batch.next_obs.data.device)
    main = torch.cuda.current_stream(ctx.device)
    with no_grad():
        mean, raw = _policy_raw(nets.policy, batch.next_obs)
        joint_next, next_logp, joint = _sample(dist, nets.policy, mean, raw,
                                               batch["next_noise"], batch.next_obs,
                                               pack=(batch.obs, batch["actions"]))
        # The target critics are independent of each other and of the online
        # critics' forward: on the forward lanes, beside it (parallel branches
        # of the captured graph); the loss waits for all of them.
        q_next = []
        for i, net in enumerate(nets.targets):
            if ctx.concurrent and len(nets.targets) <= len(FORWARD_LANES):
                with ctx.side(FORWARD_LANES[i]):
                    q = net.head(joint_next)
                    q.data.record_stream(main)
            else:
                q = net.head(joint_next)
            q_next.append(q)
    qs = _critics_side_by_side(ctx, nets.critics, joint)
    ctx.join()
    loss, alpha, target, td_abs = sac_critic_loss(
        qs, q_next, next_logp, log_alpha, batch["rewards"], batch["dones"],
        batch["discounts"], weights=batch["is_weights"] if prioritized else None,
        want_td_abs=prioritized)
    loss.backward()
    metrics = {"critic_loss": loss, "alpha": alpha, "q_target": target}
    total = grad_sq_device(nets.critic_parameters())
    if total is not None:
        metrics["critic_grad_sq"] = total
    if prioritized:
        metrics["td_abs"] = td_abs
    return metrics


def actor_region_fused(nets, dist, batch, log_alpha: Tensor, target_entropy: float, *,
                       learn_alpha: bool) -> dict:
    """actor_region on the fused heads (critic parameters request no
    gradient, as in actor_region)."""
    critic_params = nets.critic_parameters()
    flags = [p.requires_grad for p in critic_params]
    for p in critic_params:
        p.requires_grad = False
    try:
        mean, raw = _policy_raw(nets.policy, batch.obs)
        joint, logp, _ = _sample(dist, nets.policy, mean, raw, batch["noise"], batch.obs)
        ctx = context(batch.obs.data.device)
        qs = _critics_side_by_side(ctx, nets.critics, joint)
        ctx.join()
        loss, dual = sac_actor_loss(qs, logp, log_alpha, target_entropy,
                                    learn_alpha=learn_alpha)
        loss.backward()
    finally:
        for p, f in zip(critic_params, flags):
            p.requires_grad = f
    metrics = {"actor_loss": loss, "logp": logp.detach()}
    total = grad_sq_device(nets.policy_parameters())
    if total is not None:
        metrics["actor_grad_sq"] = total
    if learn_alpha:
        dual.backward()
        metrics["alpha_loss"] = dual
    return metrics


# ----------------------------------------------------------------- learner

class _Batch(dict):
    """The bound input buffers of one update: named tensors plus `.obs` and
    `.next_obs` (the observation halves the nets read)."""


@dataclass(frozen=True)
class SACConfig:
    """The learner fields of ttrl/algos/sac/config.py this path reads."""
    gamma: float = 0.99
    tau: float = 0.005
    lr: float = 3e-4
    init_alpha: float = 0.2
    learn_alpha: bool = True
    target_entropy: float | None = None  # default: -action_dim


class SACLearner:
    """Graph-replayed SAC update over bound device batch buffers."""

    def __init__(self, nets, low, high, batch_size: int, obs_dim: int, device=None, *,
                 cfg: SACConfig = SACConfig(), prioritized: bool = False,
                 fused: bool | None = None):
        self.nets = nets
        # The fused heads where the nets allow them (fused=None), or as asked.
        if fused is None:
            fused = fused_heads_apply(nets)
        elif fused and not fused_heads_apply(nets):
            raise ValueError("SACLearner(fused=True): the nets are not a Gaussian-head policy "
                             "with critics on concat(obs, action)")
        self.fused = bool(fused)
        self.cfg = cfg
        self.device = as_device(device)
        self.dist = SquashedGaussian(low, high, self.device)
        self.dim = self.dist.dim
        self.prioritized = prioritized
        self.target_entropy = (-float(self.dim) if cfg.target_entropy is None
                               else float(cfg.target_entropy))
        self.log_alpha = Tensor.from_numpy(
            np.array([[math.log(cfg.init_alpha)]], np.float32), self.device, requires_grad=True)
        self.critic_opt = Adam(nets.critic_parameters(), lr=cfg.lr)
        self.policy_opt = Adam(nets.policy_parameters(), lr=cfg.lr)
        self.alpha_opt = Adam([self.log_alpha], lr=cfg.lr)
        # The policy and temperature steps run back to back: one launch.
        share_launch([self.policy_opt, self.alpha_opt])
        B, D = int(batch_size), self.dim
        dev = self.device

        def buf(*shape):
            return Tensor(torch.zeros(shape, dtype=torch.float32, device=dev))

        self.batch = _Batch(actions=buf(B, D), rewards=buf(B, 1), dones=buf(B, 1),
                            discounts=buf(B, 1), noise=buf(B, D), next_noise=buf(B, D))
        if prioritized:
            self.batch["is_weights"] = Tensor(torch.ones((B, 1), device=dev))
        self.batch.obs = buf(B, obs_dim)
        self.batch.next_obs = buf(B, obs_dim)
        self._pairs = [(t, c) for t, c in zip(list(nets.targets.parameters()),
                                              list(nets.critics.parameters()))]
        self._graph = None
        self._metrics = None
        self._pack = None
        self.launches_per_replay = 0

    # -- inputs ----------------------------------------------------------

    def load_batch(self, obs, next_obs, actions, rewards, dones, discounts, noise, next_noise,
                   is_weights=None) -> None:
        """Copy one batch of host arrays into the bound buffers, in place."""
        def put(t, a):
            t.data.copy_(torch.from_numpy(np.ascontiguousarray(a, np.float32)).reshape(t.shape))
        put(self.batch.obs, obs)
        put(self.batch.next_obs, next_obs)
        for key, arr in (("actions", actions), ("rewards", rewards), ("dones", dones),
                         ("discounts", discounts), ("noise", noise), ("next_noise", next_noise)):
            put(self.batch[key], arr)
        if self.prioritized and is_weights is not None:
            put(self.batch["is_weights"], is_weights)

    # -- one update --------------------------------------------------------

    def _polyak(self) -> None:
        """t <- (1 - tau) t + tau c for every target/critic pair, all pairs in
        one launch (ttrl/algos/sac/targets.py:45-96)."""
        context(self.device).blend([(t.data, c.data) for t, c in self._pairs], self.cfg.tau)

    def _update(self) -> dict:
        opts = (self.critic_opt, self.policy_opt, self.alpha_opt)
        for opt in opts:
            opt.zero_grad()
        critic_fn, actor_fn = ((critic_region_fused, actor_region_fused) if self.fused
                               else (critic_region, actor_region))
        critic = critic_fn(self.nets, self.dist, self.batch, self.log_alpha,
                           prioritized=self.prioritized)
        self.critic_opt.step()
        for opt in opts:
            opt.zero_grad()
        actor = actor_fn(self.nets, self.dist, self.batch, self.log_alpha,
                         self.target_entropy, learn_alpha=self.cfg.learn_alpha)
        step_together([self.policy_opt, self.alpha_opt] if self.cfg.learn_alpha
                      else [self.policy_opt])
        self._polyak()
        return {**critic, **actor}

    def update_eager(self) -> dict:
        metrics = self._update()
        for opt in (self.critic_opt, self.policy_opt, self.alpha_opt):
            opt.captured_indices = None
        return metrics

    def capture(self) -> None:
        """Warm up on a copy of the state (kernel loading, gradient buffers),
        restore it, then capture one whole update into a CUDA graph."""
        params = (self.nets.critic_parameters() + self.nets.policy_parameters()
                  + list(self.nets.targets.parameters()) + [self.log_alpha])
        saved = [p.data.clone() for p in params]
        opts = (self.critic_opt, self.policy_opt, self.alpha_opt)
        state = [([m.clone() for m in o.m], [v.clone() for v in o.v], o._dev_steps.clone(),
                  o.t, list(o.steps)) for o in opts]
        self._update()
        torch.cuda.synchronize(self.device)
        for p, s in zip(params, saved):
            p.data.copy_(s)
        for o, (ms, vs, dsteps, t, steps) in zip(opts, state):
            for m, s in zip(o.m, ms):
                m.copy_(s)
            for v, s in zip(o.v, vs):
                v.copy_(s)
            o._dev_steps.copy_(dsteps)
            o.t, o.steps = t, steps
        from ttrl_b200._lib import lib
        before = lib().ttrl_launch_count()
        self._graph, self._metrics = capture(self.device, self._update, critical_main=True)
        self.launches_per_replay = int(lib().ttrl_launch_count() - before)

    def replay(self) -> None:
        if self._graph is None:
            self.capture()
        self._graph.replay()
        for opt in (self.critic_opt, self.policy_opt, self.alpha_opt):
            if opt.captured_indices is not None:
                opt.advance(opt.captured_indices)

    def read_metrics(self) -> dict:
        """Host copies of the last update's scalar metrics."""
        if self._metrics is None:
            return {}
        out = {}
        for k, v in self._metrics.items():
            arr = v.numpy() if isinstance(v, Tensor) else np.asarray(v.detach().cpu())
            out[k] = float(np.asarray(arr, np.float64).mean()) if arr.size > 1 else float(arr.reshape(-1)[0])
        return out

    def close(self) -> None:
        if self._graph is not None:
            self._graph.close()
            self._graph = None
