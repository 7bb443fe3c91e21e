"""Shared helpers for the parity tests: seeded synthetic inputs with the
BASELINE configs' shapes, and loading oracle parameters into the B200 nets."""

from __future__ import annotations

import numpy as np

TOL_GRAD = 1e-4   # relative Frobenius, split-TF32 contractions (spec budget 1e-3)
TOL_PARAM = 1e-6  # relative Frobenius of post-Adam parameters (fp32 elementwise)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def nature_state_dict(p, heads=("q",)):
    """Oracle parameter dict -> the state_dict of ttrl_b200's Nature-CNN nets
    (EncoderHead for heads=('q',), ActorCritic for ('pi', 'v'))."""
    enc = ("encoder" if heads == ("q",) else "encoders.actor") + ".towers.obs"
    sd = {}
    for i, layer in enumerate((0, 2, 4)):
        sd[f"{enc}.layers.{layer}.weight"] = p[f"conv{i}.w"]
        sd[f"{enc}.layers.{layer}.bias"] = p[f"conv{i}.b"].reshape(1, 1, 1, -1)
    sd[f"{enc}.layers.7.weight"] = p["fc.w"]
    sd[f"{enc}.layers.7.bias"] = p["fc.b"].reshape(1, -1)
    if heads == ("q",):
        sd["head.q.weight"] = p["q.w"]
        sd["head.q.bias"] = p["q.b"].reshape(1, -1)
    else:
        sd["heads.policy.logits.weight"] = p["pi.w"]
        sd["heads.policy.logits.bias"] = p["pi.b"].reshape(1, -1)
        sd["heads.value.value.weight"] = p["v.w"]
        sd["heads.value.value.bias"] = p["v.b"].reshape(1, -1)
    return sd


def oracle_params_from_state(sd, heads=("q",)):
    """The inverse of nature_state_dict: a Nature-CNN state_dict (portable
    layout) -> the oracle's parameter dict, float64."""
    names = nature_state_dict({k: np.zeros(1) for k in _ORACLE_KEYS[heads]}, heads)
    return {key: np.asarray(sd[name], np.float64).reshape(_oracle_shape(key, sd[name]))
            for key, name in zip(_ORACLE_KEYS[heads], names)}


_ORACLE_KEYS = {
    ("q",): ["conv0.w", "conv0.b", "conv1.w", "conv1.b", "conv2.w", "conv2.b", "fc.w", "fc.b",
             "q.w", "q.b"],
    ("pi", "v"): ["conv0.w", "conv0.b", "conv1.w", "conv1.b", "conv2.w", "conv2.b", "fc.w",
                  "fc.b", "pi.w", "pi.b", "v.w", "v.b"],
}


def _oracle_shape(key, value):
    a = np.asarray(value)
    return (a.size,) if key.endswith(".b") else a.shape


def oracle_grads_to_named(g, heads=("q",)):
    """Oracle gradient dict -> {state_dict name: OIHW/(in,out) array}."""
    return nature_state_dict(g, heads)


def dqn_batch(rng, batch=32, actions=6, hw=84):
    obs = rng.integers(0, 256, (batch, 4, hw, hw), dtype=np.uint8)
    next_obs = rng.integers(0, 256, (batch, 4, hw, hw), dtype=np.uint8)
    act = rng.integers(0, actions, batch)
    rewards = rng.choice(np.array([-1.0, 0.0, 1.0], np.float32), batch)
    dones = (rng.random(batch) < 0.01).astype(np.float32)
    discounts = np.full(batch, 0.99, np.float32)
    return obs, next_obs, act, rewards, dones, discounts


def nchw_to_nhwc(x):
    return np.ascontiguousarray(np.asarray(x).transpose(0, 2, 3, 1))


def device_gates(net, rows_tensor):
    """ReLU masks of the device forward of a Nature-CNN encoder, shaped like
    the oracle's cache entries (NHWC per conv stage, (B, hidden) for fc)."""
    import torch
    from ttrl_b200.engine.autograd import no_grad
    enc = net.encoder if hasattr(net, "encoder") else net.encoders["actor"]
    layers = list(enc["obs"].layers)
    gates = {}
    x = rows_tensor
    with no_grad():
        for i, idx in enumerate((0, 2, 4)):
            conv = layers[idx]
            x = conv.forward_relu(x)
            g = conv.geom
            gates[f"a{i}"] = (x.numpy().reshape(g.batch, g.out_h, g.out_w, g.out_channels) > 0)
        flat = layers[6](x)
        feat = layers[7].forward_relu(flat)
        gates["feat"] = feat.numpy() > 0
    torch.cuda.synchronize()
    return gates


def grads_in_state_layout(net):
    """{parameter name: its gradient in the state_dict layout}: conv weights
    converted from the device's (possibly space-to-depth) KRSC to OIHW."""
    from ttrl_b200.engine.conv import Conv2d
    from ttrl_b200.engine.nn import Module
    convs = {}
    stack = [net]
    seen = set()
    while stack:
        v = stack.pop()
        if id(v) in seen:
            continue
        seen.add(id(v))
        if isinstance(v, Conv2d):
            convs[id(v.weight)] = v
        if isinstance(v, Module):
            stack.extend(val for _, val in v._slot_sources())
        elif isinstance(v, dict):
            stack.extend(v.values())
        elif isinstance(v, (list, tuple)):
            stack.extend(v)
    out = {}
    for name, p in net.named_parameters():
        g = p.grad.detach().cpu().numpy()
        conv = convs.get(id(p))
        out[name] = conv._from_device_layout(g) if conv is not None else g
    return out
