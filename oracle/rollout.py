"""PPO rollout post-processing restated in numpy. TEST INFRASTRUCTURE ONLY
(see oracle/__init__.py).

* `gae`: ttrl/buffers/rollout.py:195-227, the GAE-lambda recursion over
  `t = T-1 .. 0`, vectorised over lanes, in the same float32 operations.
* `normalize`: ttrl/buffers/rollout.py:269-270 and
  ttrl/buffers/seqbatch.py:86-101, (adv - mean) / (std + 1e-8) with the
  statistics over valid slots.
"""

from __future__ import annotations

import numpy as np

__all__ = ["gae", "normalize"]


def gae(rewards, values, dones, valid, last_values, gamma: float, lam: float):
    """-> (advantages, returns), float32 [T, E]."""
    rewards = np.asarray(rewards, np.float32)
    values = np.asarray(values, np.float32)
    dones = np.asarray(dones, np.float32)
    valid = np.ones_like(values) if valid is None else np.asarray(valid, np.float32)
    steps, envs = values.shape
    adv = np.zeros((steps, envs), np.float32)
    last_gae = np.zeros(envs, np.float32)
    next_values = np.asarray(last_values, np.float32)
    for t in range(steps - 1, -1, -1):
        not_done = 1.0 - dones[t]
        delta = rewards[t] + gamma * next_values * not_done - values[t]
        last_gae = delta + gamma * lam * not_done * last_gae
        last_gae = last_gae * valid[t]
        adv[t] = last_gae
        next_values = values[t]
    return adv, adv + values


def normalize(adv, valid=None):
    """Normalised advantages of the valid slots (flattened, in slot order)."""
    flat = np.asarray(adv, np.float32).reshape(-1)
    if valid is not None:
        flat = flat[np.asarray(valid).reshape(-1) > 0]
    return (flat - flat.mean()) / (flat.std() + 1e-8)
