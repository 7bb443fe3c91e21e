"""Composed networks (ttrl/nets/models.py). Each takes the observation tensor
directly (the single-leaf case of the reference's ObsPair)."""

from __future__ import annotations

from dataclasses import dataclass

from ttrl_b200.engine.nn import Module, ModuleDict, ModuleList
from ttrl_b200.engine.ops import concat

__all__ = ["EncoderHead", "ActorCritic", "ContinuousCritic", "SacNets"]


def _leaf(obs):
    """Accept a Tensor, or an ObsPair-like object / single-leaf mapping."""
    if hasattr(obs, "actor"):
        obs = obs.actor
    if isinstance(obs, dict):
        if len(obs) != 1:
            raise ValueError("multi-leaf observations are outside this backend's hot path")
        obs = next(iter(obs.values()))
    return obs


class EncoderHead(Module):
    def __init__(self, encoder, head):
        self.encoder = encoder
        self.head = head

    def forward(self, obs):
        return self.head(self.encoder(_leaf(obs)))


class ActorCritic(Module):
    """Shared trunk feeding a policy head and a value head."""

    def __init__(self, actor, critic, policy, value):
        self.encoders = ModuleDict({"actor": actor, "critic": critic})
        self.heads = ModuleDict({"policy": policy, "value": value})

    def forward(self, obs):
        actor, critic = self.encoders["actor"], self.encoders["critic"]
        features = actor(_leaf(obs))
        critic_features = features if critic is actor else critic(_leaf(obs))
        return self.heads["policy"](features), self.heads["value"](critic_features)


class ConcatEncoder(Module):
    """concat(obs features, action) -> one row (ttrl/nets/fusion.py)."""

    def __init__(self, encoder, action_dim: int):
        self.encoder = encoder
        self.action_dim = int(action_dim)
        self.out_features = int(encoder.out_features) + self.action_dim

    def forward(self, obs, action):
        return concat([self.encoder(_leaf(obs)), action], dim=-1)


class ContinuousCritic(Module):
    def __init__(self, encoder, head):
        self.encoder = encoder
        self.head = head

    def forward(self, obs, action):
        return self.head(self.encoder(obs, action))


@dataclass
class SacNets:
    policy: Module
    critics: ModuleList
    targets: ModuleList

    def sync_targets(self) -> None:
        for critic, target in zip(self.critics, self.targets, strict=True):
            target.copy_from(critic)

    def policy_parameters(self):
        return list(self.policy.parameters())

    def critic_parameters(self):
        return list(self.critics.parameters())

    def state_dict(self) -> dict:
        out = {}
        for name, module in (("policy", self.policy), ("critics", self.critics),
                             ("targets", self.targets)):
            for key, array in module.state_dict().items():
                out[f"{name}.{key}"] = array
        return out

    def load_state_dict(self, state: dict) -> None:
        for name, module in (("policy", self.policy), ("critics", self.critics),
                             ("targets", self.targets)):
            prefix = f"{name}."
            module.load_state_dict({k[len(prefix):]: v for k, v in state.items()
                                    if k.startswith(prefix)})
