"""Output heads (ttrl/nets/heads.py)."""

from __future__ import annotations

from ttrl_b200.engine.layers import Linear
from ttrl_b200.engine.nn import Module, ModuleDict
from ttrl_b200.engine.ops import clamp

__all__ = ["QHead", "CategoricalHead", "ValueHead", "GaussianHead", "LOG_STD_MIN",
           "LOG_STD_MAX"]

LOG_STD_MIN = -20.0
LOG_STD_MAX = 2.0


class QHead(Module):
    def __init__(self, in_features: int, n_actions: int, device=None):
        self.q = Linear(in_features, n_actions, device)
        self.n_actions = int(n_actions)

    def forward(self, x):
        return self.q(x)


class CategoricalHead(Module):
    def __init__(self, in_features: int, n_actions: int, device=None):
        self.logits = Linear(in_features, n_actions, device)
        self.n_actions = int(n_actions)

    def forward(self, x):
        return self.logits(x)


class ValueHead(Module):
    def __init__(self, in_features: int, device=None):
        self.value = Linear(in_features, 1, device)

    def forward(self, x):
        return self.value(x)


class GaussianHead(Module):
    """(mean, log_std), log_std clamped to [-20, 2] by the relu-identity clamp."""

    def __init__(self, in_features: int, action_dim: int, device=None, *,
                 log_std_min: float = LOG_STD_MIN, log_std_max: float = LOG_STD_MAX):
        if log_std_min >= log_std_max:
            raise ValueError("GaussianHead: log_std_min must be < log_std_max")
        self.action_dim = int(action_dim)
        self.log_std_min = float(log_std_min)
        self.log_std_max = float(log_std_max)
        self.heads = ModuleDict({
            "mean": Linear(in_features, self.action_dim, device),
            "log_std": Linear(in_features, self.action_dim, device),
        })

    def forward(self, x):
        mean = self.heads["mean"](x)
        log_std = clamp(self.heads["log_std"](x), self.log_std_min, self.log_std_max)
        return mean, log_std
