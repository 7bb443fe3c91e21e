"""Builders (ttrl/nets/build.py) over plain shapes: an image observation is
(C, H, W) and gets the Nature-CNN tower, a vector observation is (D,) and
gets the MLP tower."""

from __future__ import annotations

from ttrl_b200.engine.layers import Linear, ReLU, Sequential
from ttrl_b200.engine.nn import ModuleList
from ttrl_b200.nets.encoders import Encoder, image_encoder, vector_encoder
from ttrl_b200.nets.heads import CategoricalHead, GaussianHead, QHead, ValueHead
from ttrl_b200.nets.models import (ActorCritic, ConcatEncoder, ContinuousCritic, EncoderHead,
                                   SacNets)
from ttrl_b200.nets.multi import MultiEncoder, single_leaf

__all__ = ["build_q_net", "build_actor_critic", "build_sac_nets", "build_encoder"]


def build_encoder(obs_shape, device=None, *, batch: int, hidden=None, scale=None,
                  **kw) -> MultiEncoder:
    """The tower for one observation leaf, wrapped as the reference's
    `MultiEncoder` (ttrl/nets/multi.py:108-145) so parameters are named
    `towers.obs.layers.<i>.*`."""
    shape = tuple(int(v) for v in obs_shape)
    if len(shape) == 3:
        return single_leaf(image_encoder(shape, device, batch=batch, hidden=hidden or 512,
                                         scale=(1.0 / 255.0) if scale is None else scale, **kw))
    if len(shape) == 1:
        return single_leaf(vector_encoder(shape[0], device, hidden=hidden or (256, 256),
                                          scale=1.0 if scale is None else scale))
    raise ValueError(f"observation shape {shape} is neither (C, H, W) nor (D,)")


def build_q_net(obs_shape, n_actions: int, device=None, *, batch: int, **kw) -> EncoderHead:
    tower = build_encoder(obs_shape, device, batch=batch, **kw)
    return EncoderHead(tower, QHead(tower.out_features, n_actions, device))


def build_actor_critic(obs_shape, n_actions: int, device=None, *, batch: int,
                       **kw) -> ActorCritic:
    tower = build_encoder(obs_shape, device, batch=batch, **kw)
    return ActorCritic(tower, tower, CategoricalHead(tower.out_features, n_actions, device),
                       ValueHead(tower.out_features, device))


def build_sac_nets(obs_dim: int, action_dim: int, device=None, *, batch: int,
                   n_critics: int = 2, critic_hidden=(256, 256), policy_hidden=(256, 256)):
    """Gaussian policy MLP plus twin Q(s, a) critics on concat(s, a) and
    their targets (hard-copied from the critics at construction)."""
    if n_critics < 2:
        raise ValueError(f"build_sac_nets: n_critics must be >= 2, got {n_critics}")

    def one_critic():
        joint = ConcatEncoder(single_leaf(Encoder((), obs_dim)), action_dim)
        layers = []
        prev = joint.out_features
        for width in critic_hidden:
            layers += [Linear(prev, width, device), ReLU()]
            prev = width
        layers.append(ValueHead(prev, device))
        return ContinuousCritic(joint, Sequential(*layers))

    policy_tower = single_leaf(vector_encoder(obs_dim, device, hidden=policy_hidden))
    policy = EncoderHead(policy_tower, GaussianHead(policy_tower.out_features, action_dim, device))
    nets = SacNets(policy=policy,
                   critics=ModuleList([one_critic() for _ in range(n_critics)]),
                   targets=ModuleList([one_critic() for _ in range(n_critics)]))
    nets.sync_targets()
    return nets
