"""Whole learner updates of the reference, restated in numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

* `nature_forward` / `nature_backward`: the Nature-CNN trunk of
  ttrl/nets/encoders.py:70-131 (conv 8x8/4 -> 32, 4x4/2 -> 64, 3x3/1 -> 64,
  each + bias + ReLU, NHWC flatten in (h, w, c) order
  (ttrl/engine/layers.py:158-200), Linear(3136, 512) + ReLU) with optional
  heads, and its reverse pass by the chain rule the tape applies.
* `dqn_update`: ttrl/algos/dqn/losses.py:77-140 -- three forwards, the
  double-DQN bootstrap, Huber (ttrl/engine/ops/functional.py:56-69), mean,
  backward, grad_sq -- followed by Adam (ttrl/engine/optim/adam.py:93-134).
* `ppo_objective_and_grads`: ttrl/algos/ppo/loss.py:42-83 with its gradient,
  and `ppo_minibatch_step`: ttrl/algos/ppo/learn.py:76-112 (backward,
  clip_grad_norm of ttrl/algos/grads.py:29-43, Adam).

Parameters are dicts of numpy arrays: conv weights in OIHW, Linear
weights (in, out), biases flat. Arithmetic runs in the dtype given
(float64 for gradient references, float32 for the CPU baseline).
"""

from __future__ import annotations

import numpy as np

from oracle.layers import (adam_step_sv, conv2d_dgrad, conv2d_nhwc, conv2d_wgrad, relu)

__all__ = ["NATURE", "nature_params", "nature_forward", "nature_backward", "huber_grad",
           "dqn_loss_head", "dqn_update", "ppo_objective_and_grads", "ppo_minibatch_step",
           "log_softmax", "clip_grad_norm_scale", "sigmoid", "gru_cell_forward", "gru_cell_backward"]

#: (out_channels, kernel, stride) of ttrl/nets/towers.py:40.
NATURE = ((32, 8, 4), (64, 4, 2), (64, 3, 1))


def nature_params(rng, in_ch=4, hw=84, hidden=512, heads=(("q", 6),), dtype=np.float32):
    """U(+-1/sqrt(fan_in)) init (PyTorch default, as the reference uses)."""
    p = {}
    c, h = in_ch, hw
    for i, (co, k, s) in enumerate(NATURE):
        bound = 1.0 / np.sqrt(c * k * k)
        p[f"conv{i}.w"] = rng.uniform(-bound, bound, (co, c, k, k)).astype(dtype)
        p[f"conv{i}.b"] = rng.uniform(-bound, bound, (co,)).astype(dtype)
        c, h = co, (h - k) // s + 1
    flat = c * h * h
    bound = 1.0 / np.sqrt(flat)
    p["fc.w"] = rng.uniform(-bound, bound, (flat, hidden)).astype(dtype)
    p["fc.b"] = rng.uniform(-bound, bound, (hidden,)).astype(dtype)
    for name, width in heads:
        bound = 1.0 / np.sqrt(hidden)
        p[f"{name}.w"] = rng.uniform(-bound, bound, (hidden, width)).astype(dtype)
        p[f"{name}.b"] = rng.uniform(-bound, bound, (width,)).astype(dtype)
    return p


def nature_forward(p, x_nhwc, *, input_scale=1.0 / 255.0, heads=("q",)):
    """-> (outputs dict per head, cache). x is [N, H, W, C] (raw 0..255)."""
    cache = {"x": x_nhwc}
    h = x_nhwc
    for i, (co, k, s) in enumerate(NATURE):
        h = conv2d_nhwc(h, p[f"conv{i}.w"], p[f"conv{i}.b"], stride=s,
                        input_scale=input_scale if i == 0 else 1.0, apply_relu=True)
        cache[f"a{i}"] = h
    n = h.shape[0]
    flat = h.reshape(n, -1)
    feat = relu(flat @ p["fc.w"] + p["fc.b"])
    cache["flat"] = flat
    cache["feat"] = feat
    outs = {name: feat @ p[f"{name}.w"] + p[f"{name}.b"] for name in heads}
    return outs, cache


def nature_backward(p, cache, dheads, *, input_scale=1.0 / 255.0, gates=None):
    """Gradients of every parameter given d(output) per head.

    `gates` optionally supplies the ReLU masks {"a0", "a1", "a2", "feat"}
    observed on the device under test, the method of the reference's own
    float64 twins (tests/_fakes/torch_twin.py, `DeviceGates`): where fp32 and
    float64 disagree on the sign of a pre-activation within rounding, the
    comparison follows the device's gate instead of charging the whole
    rank-1 term to the kernel."""
    gates = gates or {}
    g = {}
    feat = cache["feat"]
    dfeat = np.zeros_like(feat)
    for name, d in dheads.items():
        g[f"{name}.w"] = feat.T @ d
        g[f"{name}.b"] = d.sum(0)
        dfeat = dfeat + d @ p[f"{name}.w"].T
    dz = dfeat * gates.get("feat", feat > 0)
    flat = cache["flat"]
    g["fc.w"] = flat.T @ dz
    g["fc.b"] = dz.sum(0)
    dflat = dz @ p["fc.w"].T
    a2 = cache["a2"]
    da = dflat.reshape(a2.shape)
    for i in (2, 1, 0):
        co, k, s = NATURE[i]
        a = cache[f"a{i}"]
        dz = da * gates.get(f"a{i}", a > 0)
        inp = cache["x"] if i == 0 else cache[f"a{i - 1}"]
        scale = input_scale if i == 0 else 1.0
        g[f"conv{i}.w"] = conv2d_wgrad(inp, dz, k, stride=s, input_scale=scale)
        g[f"conv{i}.b"] = dz.reshape(-1, co).sum(0)
        if i > 0:
            da = conv2d_dgrad(dz, p[f"conv{i}.w"], inp.shape, stride=s)
    return g


def huber_grad(e, delta):
    """d huber(e)/d e with the relu-identity composition's values: e inside
    the band, +-delta outside, 0 at e == 0."""
    return np.sign(e) * np.minimum(np.abs(e), delta)


def dqn_loss_head(q, q_sel, q_tgt, actions, rewards, dones, discounts, *, delta=1.0,
                  next_mask=None, is_weights=None):
    """-> (loss, mean_q, dq, td_abs, next_actions) of the DQN loss head."""
    b = q.shape[0]
    pred = q[np.arange(b), actions]
    sel = q_sel if next_mask is None else q_sel + (next_mask - 1.0) * 1.0e4
    nxt = np.argmax(sel, axis=1)
    next_value = q_tgt[np.arange(b), nxt]
    target = rewards + next_value * (1.0 - dones) * discounts
    e = pred - target
    a = np.abs(e)
    quad = np.minimum(a, delta)
    err = 0.5 * quad * quad + delta * (a - quad)
    w = np.ones(b) if is_weights is None else is_weights
    loss = np.mean(err * w)
    dq = np.zeros_like(q)
    dq[np.arange(b), actions] = huber_grad(e, delta) * w / b
    return loss, float(np.mean(pred)), dq, a, nxt


def dqn_update(online, target, obs, next_obs, actions, rewards, dones, discounts, *,
               double=True, delta=1.0, adam_state=None, lr=1e-4, eps=1.5e-4, t=1, gates=None):
    """One DQN update. obs/next_obs are raw NHWC [B, H, W, C]. Returns
    (metrics, grads, new_params, new_adam_state). `gates`: the device's ReLU
    masks of the online forward on obs (see nature_backward)."""
    outs, cache = nature_forward(online, obs)
    q = outs["q"]
    q_tgt = nature_forward(target, next_obs)[0]["q"]
    q_sel = nature_forward(online, next_obs)[0]["q"] if double else q_tgt
    loss, mean_q, dq, _, nxt = dqn_loss_head(q, q_sel, q_tgt, actions, rewards, dones,
                                             discounts, delta=delta)
    grads = nature_backward(online, cache, {"q": dq}, gates=gates)
    grad_sq = sum(float(np.sum(np.asarray(g, np.float64) ** 2)) for g in grads.values())
    new_params, new_state = {}, {}
    for k in online:
        S, V = (adam_state or {}).get(k, (np.zeros_like(online[k]), np.zeros_like(online[k])))
        new_params[k], S, V = adam_step_sv(online[k], grads[k], S, V, t, lr=lr, eps=eps)
        new_state[k] = (S, V)
    metrics = {"loss": loss, "mean_q": mean_q, "grad_sq": grad_sq, "next_actions": nxt}
    return metrics, grads, new_params, new_state


def clip_grad_norm_scale(grads, max_norm):
    """(norm, scale) of ttrl/algos/grads.py:13-43: the f64 global L2 norm,
    and max_norm / (norm + 1e-6) when norm > max_norm, else None."""
    norm = float(np.sqrt(sum(float(np.sum(np.asarray(g, np.float64) ** 2)) for g in grads)))
    return norm, (max_norm / (norm + 1e-6) if norm > max_norm else None)


def log_softmax(x):
    m = x.max(axis=1, keepdims=True)
    sh = x - m
    return sh - np.log(np.exp(sh).sum(axis=1, keepdims=True))


def ppo_objective_and_grads(logits, value, actions, old_logp, adv, returns, old_values, *,
                            clip=0.1, vclip=0.1, vcoef=0.5, entcoef=0.01, valid=None):
    """PPO's loss terms and d loss / d (logits, value)
    (ttrl/algos/ppo/loss.py:42-83). The reduction is the mean, or with
    `valid` the masked mean sum(x * valid) / sum(valid) of
    ttrl/algos/ppo/loss.py:27-39."""
    b = logits.shape[0]
    if valid is None:
        w = np.full(b, 1.0 / b)
    else:
        valid = np.asarray(valid, np.float64).reshape(-1)
        w = valid / valid.sum()
    lsm = log_softmax(logits)
    p = np.exp(lsm)
    new_logp = lsm[np.arange(b), actions]
    ent = -(p * lsm).sum(1)
    ratio = np.exp(new_logp - old_logp)
    s1 = ratio * adv
    cl = np.clip(ratio, 1 - clip, 1 + clip)
    s2 = cl * adv
    surr = np.minimum(s1, s2)
    policy_loss = -(surr * w).sum()
    v = value.reshape(-1)
    vcl = old_values + np.clip(v - old_values, -vclip, vclip)
    ue, ce = v - returns, vcl - returns
    vmax = np.maximum(ue * ue, ce * ce)
    value_loss = 0.5 * (vmax * w).sum()
    entropy = (ent * w).sum()
    loss = policy_loss + vcoef * value_loss - entcoef * entropy
    # gradients; min/max/clamp follow the relu identities: ties go to the
    # first operand, clamp passes strictly inside the band.
    g_s = -w
    take2 = (s1 - s2) > 0
    pass_c = (ratio > 1 - clip) & (ratio < 1 + clip)
    dratio = np.where(take2, 0.0, g_s * adv) + np.where(take2, g_s * adv * pass_c, 0.0)
    dnl = dratio * ratio
    gv = vcoef * 0.5 * w
    takeb = (ce * ce - ue * ue) > 0
    vpass = (v - old_values > -vclip) & (v - old_values < vclip)
    dv = np.where(takeb, 0.0, 2 * gv * ue) + np.where(takeb, 2 * gv * ce * vpass, 0.0)
    ge = (-entcoef * w)[:, None]
    onehot = np.zeros_like(logits)
    onehot[np.arange(b), actions] = 1.0
    dlogits = dnl[:, None] * (onehot - p) + ge * (-p * (lsm + ent[:, None]))
    parts = {"policy_loss": policy_loss, "value_loss": value_loss, "entropy": entropy}
    return loss, parts, new_logp, dlogits, dv.reshape(value.shape)


def ppo_minibatch_step(params, adam_state, t, x_nhwc, actions, old_logp, adv, returns,
                       old_values, *, lr=2.5e-4, eps=1e-8, max_grad_norm=0.5, **loss_kw):
    """One PPO gradient step on the shared-trunk actor-critic."""
    outs, cache = nature_forward(params, x_nhwc, heads=("pi", "v"))
    loss, parts, new_logp, dl, dv = ppo_objective_and_grads(
        outs["pi"], outs["v"], actions, old_logp, adv, returns, old_values, **loss_kw)
    grads = nature_backward(params, cache, {"pi": dl, "v": dv})
    norm = float(np.sqrt(sum(float(np.sum(np.asarray(g, np.float64) ** 2))
                             for g in grads.values())))
    scale = max_grad_norm / (norm + 1e-6) if norm > max_grad_norm else None
    new_params, new_state = {}, {}
    for k in params:
        S, V = adam_state.get(k, (np.zeros_like(params[k]), np.zeros_like(params[k])))
        new_params[k], S, V = adam_step_sv(params[k], grads[k], S, V, t, lr=lr, eps=eps,
                                           grad_scale=scale)
        new_state[k] = (S, V)
    metrics = dict(parts, loss=loss, grad_norm=norm)
    return metrics, grads, new_params, new_state, new_logp


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def gru_cell_forward(x, h, w_ih, w_hh, b_ih, b_hh):
    """One GRU step, gates in (reset, update, candidate) order with W stored
    (in, 3H) (ttrl/engine/recurrent.py:86-94):
        r = sig(x Wr + br + h Ur + cr), z = sig(x Wz + bz + h Uz + cz),
        n = tanh(x Wn + bn + r * (h Un + cn)), h' = (1 - z) n + z h.
    Returns (h', cache)."""
    H = h.shape[1]
    gi = x @ w_ih + b_ih.reshape(1, -1)
    gh = h @ w_hh + b_hh.reshape(1, -1)
    r = sigmoid(gi[:, :H] + gh[:, :H])
    z = sigmoid(gi[:, H:2 * H] + gh[:, H:2 * H])
    n = np.tanh(gi[:, 2 * H:] + r * gh[:, 2 * H:])
    h1 = (1.0 - z) * n + z * h
    return h1, {"x": x, "h": h, "r": r, "z": z, "n": n, "ghn": gh[:, 2 * H:]}


def gru_cell_backward(dh1, cache, w_ih, w_hh):
    """Gradients of one GRU step given d h'. Returns a dict with dx, dh and
    the four parameter gradients (biases as (1, 3H))."""
    x, h, r, z, n, ghn = (cache[k] for k in ("x", "h", "r", "z", "n", "ghn"))
    dn = dh1 * (1.0 - z)
    dz = dh1 * (h - n)
    dh = dh1 * z
    dan = dn * (1.0 - n * n)          # d pre-tanh
    dr = dan * ghn
    dghn = dan * r
    dar = dr * r * (1.0 - r)
    daz = dz * z * (1.0 - z)
    dgi = np.concatenate([dar, daz, dan], axis=1)
    dgh = np.concatenate([dar, daz, dghn], axis=1)
    return {
        "dx": dgi @ w_ih.T, "dh": dh + dgh @ w_hh.T,
        "weight_ih": x.T @ dgi, "weight_hh": h.T @ dgh,
        "bias_ih": dgi.sum(0, keepdims=True), "bias_hh": dgh.sum(0, keepdims=True),
    }
