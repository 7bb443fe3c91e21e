"""Recurrent PPO's minibatch, restated in numpy with its analytic gradients.
TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

* `gru_unroll_forward` / `gru_unroll_backward`: ttrl/engine/recurrent.py:143-168
  -- the cell of :86-94 stepped over (T, batch, features) with the done mask
  h * (1 - start_t) (ttrl/engine/ops/functional.py:40-46) on the state
  entering each step -- and the truncated BPTT that the tape runs through it.
* `recurrent_ppo_minibatch`: ttrl/algos/ppo/recurrent.py:179-227 (invalid
  slots' advantages, returns and old log-probs zeroed; masked mean over
  `valid`) over ttrl/nets/recurrent.py:98-123 (trunk -> GRU over time-major
  rows -> policy and value heads) and ttrl/algos/ppo/loss.py:42-83. Returns
  the loss, its parts, the outputs and every parameter's gradient.
* `recurrent_ppo_step`: that minibatch followed by the grad-norm clip of
  ttrl/algos/grads.py:29-43 and Adam (ttrl/engine/optim/adam.py:93-134), as
  ttrl/algos/ppo/learn.py:76-112 runs them.

Parameters are a dict keyed by the reference's state_dict names; Linear
weights are (in, out) and biases (1, out).
"""

from __future__ import annotations

import numpy as np

from oracle.layers import adam_step_sv
from oracle.learner import (clip_grad_norm_scale, gru_cell_backward, gru_cell_forward,
                            ppo_objective_and_grads)

__all__ = ["gru_unroll_forward", "gru_unroll_backward", "recurrent_ppo_minibatch",
           "recurrent_ppo_step", "mlp_trunk_forward", "mlp_trunk_backward"]


def gru_unroll_forward(x, h0, starts, w_ih, w_hh, b_ih, b_hh):
    """x (T, B, F), h0 (B, H), starts None or (T, B, 1) -> (outputs (T, B, H), caches)."""
    steps = x.shape[0]
    h = h0
    outs, caches = [], []
    for t in range(steps):
        if starts is not None:
            h = h * (1.0 - starts[t])
        h, cache = gru_cell_forward(x[t], h, w_ih, w_hh, b_ih, b_hh)
        outs.append(h)
        caches.append(cache)
    return np.stack(outs), caches


def gru_unroll_backward(dout, caches, starts, w_ih, w_hh):
    """d outputs (T, B, H) -> dict of dx (T, B, F), dh0 and the four weight grads."""
    steps = dout.shape[0]
    carry = np.zeros_like(dout[0])
    dx = [None] * steps
    grads = {k: 0.0 for k in ("weight_ih", "weight_hh", "bias_ih", "bias_hh")}
    for t in reversed(range(steps)):
        g = gru_cell_backward(dout[t] + carry, caches[t], w_ih, w_hh)
        dx[t] = g["dx"]
        for k in grads:
            grads[k] = grads[k] + g[k]
        carry = g["dh"] * (1.0 - starts[t]) if starts is not None else g["dh"]
    grads["dx"] = np.stack(dx)
    grads["dh0"] = carry
    return grads


def mlp_trunk_forward(layers, x):
    """Linear -> ReLU per (weight, bias) pair (ttrl/nets/encoders.py:147-172)."""
    acts = [x]
    for w, b in layers:
        acts.append(np.maximum(acts[-1] @ w + b.reshape(1, -1), 0.0))
    return acts


def mlp_trunk_backward(layers, acts, dy):
    grads = []
    for i in reversed(range(len(layers))):
        w, _ = layers[i]
        dy = dy * (acts[i + 1] > 0.0)
        grads.append((acts[i].T @ dy, dy.sum(0, keepdims=True)))
        dy = dy @ w.T
    return list(reversed(grads)), dy


def recurrent_ppo_minibatch(params, obs, h0, starts, valid, actions, old_logp, values, adv,
                            returns, *, seq_len, clip=0.1, vclip=0.1, vcoef=0.5, entcoef=0.01,
                            trunk="encoders.actor.towers.obs.layers",
                            memory="memories.actor.cell"):
    """One minibatch of whole sequences, rows time-major (row = t * n_seq + s).

    Returns {"loss", "policy_loss", "value_loss", "entropy", "new_logp",
    "logits", "value", "grads": {name: array}}.
    """
    rows = obs.shape[0]
    n_seq = rows // seq_len
    keep = valid.reshape(rows).astype(np.float64)
    adv, returns, old_logp = adv * keep, returns * keep, old_logp * keep
    depth = 0
    while f"{trunk}.{2 * depth}.weight" in params:
        depth += 1
    layers = [(params[f"{trunk}.{2 * i}.weight"], params[f"{trunk}.{2 * i}.bias"])
              for i in range(depth)]
    acts = mlp_trunk_forward(layers, obs)
    feat = acts[-1]
    w_ih, w_hh = params[f"{memory}.weight_ih"], params[f"{memory}.weight_hh"]
    b_ih, b_hh = params[f"{memory}.bias_ih"], params[f"{memory}.bias_hh"]
    seq = feat.reshape(seq_len, n_seq, -1)
    outs, caches = gru_unroll_forward(seq, h0, starts, w_ih, w_hh, b_ih, b_hh)
    state = outs.reshape(rows, -1)
    wp, bp = params["heads.policy.logits.weight"], params["heads.policy.logits.bias"]
    wv, bv = params["heads.value.value.weight"], params["heads.value.value.bias"]
    logits = state @ wp + bp.reshape(1, -1)
    value = state @ wv + bv.reshape(1, -1)
    loss, parts, new_logp, dlogits, dvalue = ppo_objective_and_grads(
        logits, value, actions, old_logp, adv, returns, values, clip=clip, vclip=vclip,
        vcoef=vcoef, entcoef=entcoef, valid=valid)
    dvalue = dvalue.reshape(rows, 1)
    grads = {
        "heads.policy.logits.weight": state.T @ dlogits,
        "heads.policy.logits.bias": dlogits.sum(0, keepdims=True),
        "heads.value.value.weight": state.T @ dvalue,
        "heads.value.value.bias": dvalue.sum(0, keepdims=True),
    }
    dstate = dlogits @ wp.T + dvalue @ wv.T
    g = gru_unroll_backward(dstate.reshape(outs.shape), caches, starts, w_ih, w_hh)
    for k in ("weight_ih", "weight_hh", "bias_ih", "bias_hh"):
        grads[f"{memory}.{k}"] = g[k]
    tg, _ = mlp_trunk_backward(layers, acts, g["dx"].reshape(rows, -1))
    for i, (dw, db) in enumerate(tg):
        grads[f"{trunk}.{2 * i}.weight"] = dw
        grads[f"{trunk}.{2 * i}.bias"] = db
    return {"loss": loss, "new_logp": new_logp, "logits": logits, "value": value,
            "grads": grads, **parts}


def recurrent_ppo_step(params, adam_state, t, *args, lr=2.5e-4, eps=1e-8, max_grad_norm=0.5,
                       **kw):
    """One recurrent PPO gradient step: `recurrent_ppo_minibatch(params,
    *args, **kw)`, clip, Adam at step t. -> (metrics, new params, new state)."""
    out = recurrent_ppo_minibatch(params, *args, **kw)
    names = sorted(params)
    norm, scale = clip_grad_norm_scale([out["grads"][k] for k in names], max_grad_norm)
    new_params, new_state = {}, {}
    for k in names:
        S, V = adam_state.get(k, (np.zeros_like(params[k]), np.zeros_like(params[k])))
        new_params[k], S, V = adam_step_sv(params[k], out["grads"][k], S, V, t, lr=lr, eps=eps,
                                           grad_scale=scale)
        new_state[k] = (S, V)
    metrics = {k: out[k] for k in ("loss", "policy_loss", "value_loss", "entropy")}
    metrics["grad_norm"] = norm
    return metrics, new_params, new_state
