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


# --------------------------------------------------------------------------
# The whole update: networks, regions, Adams and Polyak
# (ttrl/algos/sac/agent.py:218-238, ttrl/algos/sac/step.py:28-96,
# ttrl/algos/sac/targets.py:45-96). Parameters are a dict keyed by the
# reference's state_dict names (Linear weights stored (in, out), biases
# (1, out)); "log_alpha" is the (1, 1) temperature.

LOG_STD_MIN, LOG_STD_MAX = -20.0, 2.0  # ttrl/nets/heads.py:29-30
POLICY_TRUNK = ("policy.encoder.towers.obs.layers.0", "policy.encoder.towers.obs.layers.2")
POLICY_MEAN = "policy.head.heads.mean"
POLICY_LOG_STD = "policy.head.heads.log_std"


def _critic_layers(prefix):
    return (f"{prefix}.head.layers.0", f"{prefix}.head.layers.2", f"{prefix}.head.layers.4.value")


def _affine(p, name, x):
    return x @ p[name + ".weight"] + p[name + ".bias"]


def policy_forward(p, obs):
    """Actor MLP (Linear-ReLU twice) and the Gaussian head; log_std clamped
    to [-20, 2] with no gradient at or beyond a bound (the relu identities of
    ttrl/engine/ops/select.py:39-63)."""
    acts = [np.asarray(obs, np.float64)]
    for name in POLICY_TRUNK:
        acts.append(np.maximum(_affine(p, name, acts[-1]), 0.0))
    mean = _affine(p, POLICY_MEAN, acts[-1])
    raw = _affine(p, POLICY_LOG_STD, acts[-1])
    gate = (raw > LOG_STD_MIN) & (raw < LOG_STD_MAX)
    return mean, np.clip(raw, LOG_STD_MIN, LOG_STD_MAX), {"acts": acts, "gate": gate}


def policy_backward(p, cache, d_mean, d_log_std):
    acts = cache["acts"]
    h = acts[-1]
    d_raw = d_log_std * cache["gate"]
    g = {POLICY_MEAN + ".weight": h.T @ d_mean, POLICY_MEAN + ".bias": d_mean.sum(0, keepdims=True),
         POLICY_LOG_STD + ".weight": h.T @ d_raw,
         POLICY_LOG_STD + ".bias": d_raw.sum(0, keepdims=True)}
    dh = d_mean @ p[POLICY_MEAN + ".weight"].T + d_raw @ p[POLICY_LOG_STD + ".weight"].T
    for i in reversed(range(len(POLICY_TRUNK))):
        dh = dh * (acts[i + 1] > 0.0)
        g[POLICY_TRUNK[i] + ".weight"] = acts[i].T @ dh
        g[POLICY_TRUNK[i] + ".bias"] = dh.sum(0, keepdims=True)
        dh = dh @ p[POLICY_TRUNK[i] + ".weight"].T
    return g


def critic_forward(p, prefix, obs, action):
    """Q(s, a) of one critic: concat(s, a) -> Linear-ReLU twice -> value."""
    layers = _critic_layers(prefix)
    acts = [np.concatenate([np.asarray(obs, np.float64), np.asarray(action, np.float64)], -1)]
    for name in layers[:2]:
        acts.append(np.maximum(_affine(p, name, acts[-1]), 0.0))
    return _affine(p, layers[2], acts[-1])[:, 0], acts


def critic_backward(p, prefix, acts, dq):
    """-> (parameter gradients, d loss / d concat(s, a))."""
    layers = _critic_layers(prefix)
    dy = np.asarray(dq, np.float64).reshape(-1, 1)
    g = {layers[2] + ".weight": acts[2].T @ dy, layers[2] + ".bias": dy.sum(0, keepdims=True)}
    dh = dy @ p[layers[2] + ".weight"].T
    for i in (1, 0):
        dh = dh * (acts[i + 1] > 0.0)
        g[layers[i] + ".weight"] = acts[i].T @ dh
        g[layers[i] + ".bias"] = dh.sum(0, keepdims=True)
        dh = dh @ p[layers[i] + ".weight"].T
    return g, dh


def sac_update(p, adam, steps, batch, *, low, high, n_critics=2, lr=3e-4, eps=1e-8,
               tau=0.005, target_entropy=None):
    """One SAC update in the reference agent's order; returns (new params,
    new Adam state, new step counts, metrics).

    `adam` maps a parameter name to its (S, V) moments; `steps` maps
    "critic" / "policy" / "alpha" to that optimizer's step count so far.
    `batch`: obs, next_obs [B, obs]; actions, noise, next_noise [B, D];
    rewards, dones, discounts [B, 1]."""
    from oracle.layers import adam_step_sv
    p = {k: np.asarray(v, np.float64) for k, v in p.items()}
    adam = dict(adam)
    steps = dict(steps)
    f = {k: np.asarray(v, np.float64) for k, v in batch.items()}
    d = f["actions"].shape[1]
    h_target = -float(d) if target_entropy is None else float(target_entropy)
    obs_dim = f["obs"].shape[1]
    critics = [f"critics.{i}" for i in range(n_critics)]
    targets = [f"targets.{i}" for i in range(n_critics)]

    def step_params(names, grads, which):
        steps[which] = steps.get(which, 0) + 1
        for name in names:
            s, v = adam.get(name, (np.zeros_like(p[name]), np.zeros_like(p[name])))
            p[name], s, v = adam_step_sv(p[name], grads[name], s, v, steps[which], lr=lr, eps=eps)
            adam[name] = (s, v)

    # -- critic region: soft target under no_grad, twin MSE, critic Adam.
    alpha = float(np.exp(p["log_alpha"]).reshape(-1)[0])
    mean_n, ls_n, _ = policy_forward(p, f["next_obs"])
    a_n, logp_n, _ = squashed_sample(mean_n, ls_n, f["next_noise"], low, high)
    q_next = [critic_forward(p, t, f["next_obs"], a_n)[0] for t in targets]
    y = soft_target(f["rewards"][:, 0], f["dones"][:, 0], f["discounts"][:, 0], q_next, logp_n,
                    alpha)
    online = [critic_forward(p, c, f["obs"], f["actions"]) for c in critics]
    c_loss, dq = critic_loss([q for q, _ in online], y)
    grads = {}
    for c, (_, acts), g in zip(critics, online, dq):
        grads.update(critic_backward(p, c, acts, g)[0])
    critic_names = [n for c in critics for n in sorted(grads) if n.startswith(c + ".")]
    step_params(critic_names, grads, "critic")

    # -- actor region: reparameterised actor loss through the updated
    # critics, the temperature's dual on the detached log-prob, then the
    # policy and temperature Adams (alpha is read before either steps).
    mean, log_std, pcache = policy_forward(p, f["obs"])
    action, logp, scache = squashed_sample(mean, log_std, f["noise"], low, high)
    q_pi = [critic_forward(p, c, f["obs"], action) for c in critics]
    a_loss, d_logp, d_q = actor_loss(logp, [q for q, _ in q_pi], alpha)
    d_action = np.zeros_like(action)
    for c, (_, acts), g in zip(critics, q_pi, d_q):
        d_action += critic_backward(p, c, acts, g)[1][:, obs_dim:]
    d_mean, d_log_std = squashed_sample_backward(d_action, d_logp, scache)
    pgrads = policy_backward(p, pcache, d_mean, d_log_std)
    log_alpha = float(p["log_alpha"].reshape(-1)[0])
    al_loss, d_log_alpha = alpha_loss(log_alpha, logp, h_target)
    step_params(sorted(pgrads), pgrads, "policy")
    step_params(["log_alpha"], {"log_alpha": np.full((1, 1), d_log_alpha)}, "alpha")

    # -- Polyak: target <- (1 - tau) target + tau critic, by name.
    for c, t in zip(critics, targets):
        for name in [n for n in p if n.startswith(c + ".")]:
            tn = t + name[len(c):]
            p[tn] = p[tn] * (1.0 - tau) + p[name] * tau
    metrics = {"critic_loss": c_loss, "actor_loss": a_loss, "alpha_loss": al_loss,
               "alpha": alpha, "logp": logp, "q_target": y}
    return p, adam, steps, metrics
