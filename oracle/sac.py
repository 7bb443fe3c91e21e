"""SAC's losses and the tanh-squashed Gaussian, restated in numpy with their
analytic gradients. TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows ttrl/algos/sac/losses.py:24-98, ttrl/algos/sac/policy.py:30-40 and
ttrl/algos/gaussian.py:55-167. The critics' minimum is the reference's relu
identity min(a, b) = a - relu(a - b), so on a tie the gradient goes to the
first critic.
"""

from __future__ import annotations

import math

import numpy as np

LOG_2PI = math.log(2.0 * math.pi)
_LOG_2 = math.log(2.0)


def softplus(x):
    x = np.asarray(x, np.float64)
    return np.maximum(x, 0.0) + np.log1p(np.exp(-np.abs(x)))


def action_scale(low, high):
    low = np.asarray(low, np.float64).reshape(1, -1)
    high = np.asarray(high, np.float64).reshape(1, -1)
    centre, half = (high + low) * 0.5, (high - low) * 0.5
    return centre, half, float(np.sum(np.log(half)))


def squashed_sample(mean, log_std, noise, low, high):
    """-> (env_action [B, D], logp [B], cache) of
    ttrl/algos/sac/policy.py:30-40 with the stable log(1 - tanh^2) of
    ttrl/algos/gaussian.py:73-90."""
    mean = np.asarray(mean, np.float64)
    log_std = np.asarray(log_std, np.float64)
    noise = np.asarray(noise, np.float64)
    std = np.exp(log_std)
    u = mean + std * noise
    z = (u - mean) / std
    d = u.shape[-1]
    normal = (-0.5 * z * z - log_std).sum(-1) - 0.5 * d * LOG_2PI
    log_1m_tanh2 = 2.0 * (_LOG_2 - u - softplus(-2.0 * u))
    centre, half, log_det = action_scale(low, high)
    logp = normal - log_1m_tanh2.sum(-1) - log_det
    t = np.tanh(u)
    action = centre + half * t
    return action, logp, {"u": u, "z": z, "std": std, "noise": noise, "t": t, "half": half}


def squashed_sample_backward(d_action, d_logp, cache):
    """Gradients of a loss with respect to (mean, log_std) given d loss /
    d env_action [B, D] and d loss / d logp [B]."""
    t, std, noise, half, z = (cache[k] for k in ("t", "std", "noise", "half", "z"))
    dl = np.asarray(d_logp, np.float64).reshape(-1, 1)
    # logp(u, mean, log_std): direct partials and the path through u.
    dlogp_du = -z / std + 2.0 * t
    du = dl * dlogp_du + np.asarray(d_action, np.float64) * half * (1.0 - t * t)
    d_mean = dl * (z / std) + du
    d_log_std = dl * (z * z - 1.0) + du * std * noise
    return d_mean, d_log_std


def min_with_selection(values):
    """min over critics (relu identity, first critic on ties) and the index
    of the critic each sample's gradient reaches."""
    cur = np.asarray(values[0], np.float64)
    sel = np.zeros(cur.shape, np.int64)
    for i, v in enumerate(values[1:], start=1):
        v = np.asarray(v, np.float64)
        take = (cur - v) > 0
        cur = np.where(take, v, cur)
        sel = np.where(take, i, sel)
    return cur, sel


def critic_loss(q, target, weights=None):
    """0.5 * sum_i mean((q_i - y)^2 * w) and d loss / d q_i
    (ttrl/algos/sac/losses.py:46-79). `q` is a list of [B] arrays."""
    b = target.shape[0]
    w = np.ones(b) if weights is None else np.asarray(weights, np.float64).reshape(-1)
    loss = 0.0
    grads = []
    for qi in q:
        e = np.asarray(qi, np.float64) - target
        loss += float(np.mean(e * e * w))
        grads.append(e * w / b)
    return 0.5 * loss, grads


def soft_target(rewards, dones, discounts, q_target_next, next_logp, alpha):
    """y = r + (1 - done) * discount * (min_i Q'_i(s', a') - alpha * logp')."""
    soft = min_with_selection(q_target_next)[0] - alpha * np.asarray(next_logp, np.float64)
    return (np.asarray(rewards, np.float64) + soft * (1.0 - np.asarray(dones, np.float64))
            * np.asarray(discounts, np.float64))


def actor_loss(logp, q_values, alpha):
    """mean(alpha * logp - min_i Q_i) with d/d logp and d/d Q_i
    (ttrl/algos/sac/losses.py:82-87)."""
    b = logp.shape[0]
    qmin, sel = min_with_selection(q_values)
    loss = float(np.mean(alpha * logp - qmin))
    d_logp = np.full(b, alpha / b)
    d_q = [np.where(sel == i, -1.0 / b, 0.0) for i in range(len(q_values))]
    return loss, d_logp, d_q


def alpha_loss(log_alpha, logp, target_entropy):
    """-mean(log_alpha * (logp + H)) and its gradient (losses.py:90-98)."""
    term = np.asarray(logp, np.float64) + target_entropy
    return float(-np.mean(log_alpha * term)), float(-np.mean(term))
