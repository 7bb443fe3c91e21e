"""Generate the golden vectors under tests/golden/ from the reference itself.

Run in a container that has the reference checkout (its path is the first
argument, or TTRL_REFERENCE):

    python tests/golden/make_golden.py /path/to/tt-rl [case ...]

(naming cases regenerates only those).

The reference's device code imports `ttnn` at module scope; this script
installs `ttnn_numpy` (a float32 numpy stand-in) under that name first, so
the reference's OWN autograd tape (ttrl/engine/autograd.py), ops
(ttrl/engine/ops/*), Adam (ttrl/engine/optim/adam.py), Linear
(ttrl/engine/layers.py), GRU (ttrl/engine/recurrent.py), gradient clipping
(ttrl/algos/grads.py), DQN update body (ttrl/algos/dqn/losses.py:77-140), PPO
objective (ttrl/algos/ppo/loss.py:42-83) and ParamSync
(ttrl/engine/mesh/sync.py) run unchanged. Modules that are pure numpy/Python
run as they are: adam_fused_scalars (ttrl/engine/optim/scalars.py:13-27), the
deploy conv tower (ttrl/deploy/conv.py:31-50) and conv geometry
(ttrl/engine/conv/geometry.py).

Outputs (all seeded, small): one .npz per case family plus index.json. The
tests never import the reference; they read these files.
"""

from __future__ import annotations

import json
import os
import sys
from types import SimpleNamespace

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _install(reference: str):
    sys.path.insert(0, HERE)
    import ttnn_numpy
    sys.modules["ttnn"] = ttnn_numpy
    sys.path.insert(0, reference)
    return ttnn_numpy


def _save(name: str, arrays: dict, index: dict, note: str) -> None:
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **{k: np.asarray(v) for k, v in arrays.items()})
    index[name] = {"note": note, "keys": sorted(arrays)}


def adam_scalars(index):
    from ttrl.engine.optim.scalars import adam_fused_scalars
    rows = []
    for lr, b1, b2, eps in [(1e-4, 0.9, 0.999, 1.5e-4), (2.5e-4, 0.9, 0.999, 1e-8),
                            (3e-4, 0.9, 0.999, 1e-8), (1e-3, 0.5, 0.9, 1e-5)]:
        for t in (1, 2, 3, 10, 100, 1000, 8000, 100000):
            a, e = adam_fused_scalars(lr, b1, b2, eps, t)
            rows.append([lr, b1, b2, eps, t, a, e])
    _save("adam_scalars", {"rows": np.array(rows, np.float64)}, index,
          "ttrl/engine/optim/scalars.py:13-27: (lr,b1,b2,eps,t) -> (alpha_t, eps_t)")


def adam_steps(index):
    from ttrl.engine.autograd import Tensor
    from ttrl.engine.optim.adam import Adam
    import ttnn
    out = {}
    for case, (lr, eps, wd) in enumerate([(1e-4, 1.5e-4, 0.0), (2.5e-4, 1e-8, 0.0),
                                          (1e-3, 1e-8, 0.01)]):
        rng = np.random.default_rng(100 + case)
        shapes = [(37,), (5, 7), (64, 3)]
        init = [rng.standard_normal(s).astype(np.float32) for s in shapes]
        params = [Tensor.from_numpy(a, ttnn.DEVICE, requires_grad=True) for a in init]
        opt = Adam(params, lr=lr, eps=eps, weight_decay=wd)
        grads = []
        for step in range(6):
            g_step = [rng.standard_normal(s).astype(np.float32) * (0.1 + step) for s in shapes]
            for i, p in enumerate(params):
                # Parameter 1 gets no gradient on step 2: its own step count lags.
                p.grad = None if (i == 1 and step == 2) else ttnn.Tensor(g_step[i])
            grads.append(g_step)
            opt.step()
        pre = f"c{case}_"
        out[pre + "hyper"] = np.array([lr, eps, wd], np.float64)
        for i in range(len(shapes)):
            out[pre + f"p{i}_init"] = init[i]
            out[pre + f"p{i}_grads"] = np.stack([g[i] for g in grads])
            out[pre + f"p{i}_final"] = params[i].numpy()
            out[pre + f"p{i}_S"] = opt.m[i].to_numpy()
            out[pre + f"p{i}_V"] = opt.v[i].to_numpy()
        out[pre + "steps"] = np.array(opt.steps, np.int64)
    _save("adam_steps", out, index,
          "ttrl/engine/optim/adam.py:93-134 over 6 steps; param 1 has no grad on step 2")


class _FakeQNet:
    """Stands in for a Q network: returns preset Q tensors in call order
    (online(obs), target(next_obs), online(next_obs)) and exposes the
    online(obs) leaf as its only parameter."""

    def __init__(self, outputs):
        self.outputs = list(outputs)
        self.calls = 0

    def __call__(self, obs):
        q = self.outputs[self.calls]
        self.calls += 1
        return q

    def parameters(self):
        return [self.outputs[0]]


def dqn_loss(index):
    from ttrl.algos.dqn.losses import update_loss
    from ttrl.engine.autograd import Tensor
    import ttnn
    out = {}
    variants = [("vanilla", False, 0, False), ("double", True, 0, False),
                ("double_mask", True, 6, False), ("double_per", True, 0, True)]
    for v, (name, double, mask_n, per) in enumerate(variants):
        rng = np.random.default_rng(200 + v)
        B, A = 32, 6
        q = rng.standard_normal((B, A)).astype(np.float32)
        q_next_online = rng.standard_normal((B, A)).astype(np.float32)
        q_next_target = (q_next_online + 0.3 * rng.standard_normal((B, A))).astype(np.float32)
        actions = rng.integers(0, A, B)
        onehot = np.eye(A, dtype=np.float32)[actions]
        rewards = rng.choice([-1.0, 0.0, 1.0], B).astype(np.float32).reshape(B, 1)
        dones = (rng.random(B) < 0.1).astype(np.float32).reshape(B, 1)
        discounts = np.where(rng.random(B) < 0.2, 0.99 ** 2, 0.99).astype(np.float32).reshape(B, 1)
        # Large errors on a few rows exercise Huber's linear branch.
        rewards[:4] *= 5.0
        dev = ttnn.DEVICE
        q_leaf = Tensor.from_numpy(q, dev, requires_grad=True)
        online = _FakeQNet([q_leaf, None])
        qn_online = Tensor.from_numpy(q_next_online, dev)
        qn_target = Tensor.from_numpy(q_next_target, dev)
        # call order inside update_loss: online(obs), target(next), online(next)
        online.outputs[1] = qn_online
        target = _FakeQNet([qn_target])
        inputs = {
            "rewards": Tensor.from_numpy(rewards, dev),
            "dones": Tensor.from_numpy(dones, dev),
            "discounts": Tensor.from_numpy(discounts, dev),
            "actions_onehot": Tensor.from_numpy(onehot, dev),
            "obs.x": Tensor.from_numpy(np.zeros((B, 1), np.float32), dev),
            "next_obs.x": Tensor.from_numpy(np.zeros((B, 1), np.float32), dev),
        }
        mask = np.ones((B, A), np.float32)
        if mask_n:
            mask = (rng.random((B, A)) < 0.7).astype(np.float32)
            mask[np.arange(B), rng.integers(0, A, B)] = 1.0  # at least one legal
            inputs["next_mask"] = Tensor.from_numpy(mask, dev)
        isw = np.ones((B, 1), np.float32)
        if per:
            isw = rng.uniform(0.2, 1.0, (B, 1)).astype(np.float32)
            inputs["is_weights"] = Tensor.from_numpy(isw, dev)
        metrics = update_loss(online, target, inputs, leaves=("x",), num_actions=A,
                              mask_n=mask_n, double=double, huber_delta=1.0, prioritized=per)
        pre = f"{name}_"
        out.update({pre + "q": q, pre + "q_next_online": q_next_online,
                    pre + "q_next_target": q_next_target, pre + "onehot": onehot,
                    pre + "rewards": rewards, pre + "dones": dones,
                    pre + "discounts": discounts, pre + "next_mask": mask,
                    pre + "is_weights": isw,
                    pre + "flags": np.array([int(double), mask_n, int(per)], np.int64),
                    pre + "loss": metrics["loss"].numpy(),
                    pre + "mean_q": metrics["mean_q"].numpy(),
                    pre + "grad_sq": metrics["grad_sq"].numpy(),
                    pre + "dq": q_leaf.grad.to_numpy()})
        if per:
            out[pre + "td_abs"] = metrics["td_abs"].numpy()
    _save("dqn_loss", out, index,
          "ttrl/algos/dqn/losses.py:77-140 with preset Q tensors (B=32, A=6, delta=1)")


def ppo_objective(index):
    from ttrl.algos.ppo.loss import masked_mean, objective
    from ttrl.algos.ppo.policy import CategoricalPolicy
    from ttrl.engine.autograd import Tensor
    from ttrl.engine.ops import mean_all
    import ttnn
    out = {}
    for v, name in enumerate(("mean", "masked")):
        rng = np.random.default_rng(300 + v)
        B, A = 256, 6
        logits = (rng.standard_normal((B, A)) * 1.5).astype(np.float32)
        value = rng.standard_normal((B, 1)).astype(np.float32)
        actions = rng.integers(0, A, B)
        # old log-probs near the current ones, so the ratio hits both clip sides
        lsm = logits - logits.max(1, keepdims=True)
        lsm = lsm - np.log(np.exp(lsm).sum(1, keepdims=True))
        old_logp = (lsm[np.arange(B), actions] + 0.2 * rng.standard_normal(B)).astype(np.float32)
        adv = rng.standard_normal(B).astype(np.float32)
        returns = rng.standard_normal(B).astype(np.float32)
        old_values = (value.reshape(-1) + 0.3 * rng.standard_normal(B)).astype(np.float32)
        valid = np.ones(B, np.float32)
        dev = ttnn.DEVICE
        lg = Tensor.from_numpy(logits, dev, requires_grad=True)
        val = Tensor.from_numpy(value, dev, requires_grad=True)
        batch = SimpleNamespace(old_logp=old_logp, actions=actions, mask=None,
                                advantages=adv, returns=returns, values=old_values)
        cfg = SimpleNamespace(clip_eps=0.1, value_clip_eps=0.1, value_coef=0.5,
                              entropy_coef=0.01)
        if name == "masked":
            valid = (rng.random(B) < 0.8).astype(np.float32)
            reduce = masked_mean(Tensor.from_numpy(valid.reshape(B, 1), dev))
        else:
            reduce = mean_all
        policy = CategoricalPolicy(SimpleNamespace(n=A), dev)
        loss, parts, new_logp = objective(policy, lg, val, batch, cfg, dev, reduce=reduce)
        loss.backward()
        pre = f"{name}_"
        out.update({pre + "logits": logits, pre + "value": value,
                    pre + "actions": actions.astype(np.int64), pre + "old_logp": old_logp,
                    pre + "adv": adv, pre + "returns": returns,
                    pre + "old_values": old_values, pre + "valid": valid,
                    pre + "loss": loss.numpy(),
                    pre + "policy_loss": parts["policy_loss"].numpy(),
                    pre + "value_loss": parts["value_loss"].numpy(),
                    pre + "entropy": parts["entropy"].numpy(),
                    pre + "new_logp": new_logp.numpy(),
                    pre + "dlogits": lg.grad.to_numpy(), pre + "dvalue": val.grad.to_numpy()})
    _save("ppo_objective", out, index,
          "ttrl/algos/ppo/loss.py:42-83 (clip 0.1, vclip 0.1, vf 0.5, ent 0.01), B=256, A=6")


def linear_mlp(index):
    from ttrl.engine.autograd import Tensor
    from ttrl.engine.layers import Flatten, Linear
    from ttrl.engine.ops import mean_all, mul, relu
    import ttnn
    np.random.seed(400)
    dev = ttnn.DEVICE
    B = 4
    fc1 = Linear(3 * 3 * 16, 32, dev)
    fc2 = Linear(32, 6, dev)
    rng = np.random.default_rng(401)
    x_nhwc = rng.uniform(0, 2, (B, 3, 3, 16)).astype(np.float32)
    upstream = rng.standard_normal((B, 6)).astype(np.float32)
    x = Tensor.from_numpy(x_nhwc.reshape(1, 1, B * 9, 16), dev, requires_grad=True)
    flat = Flatten(3, 3, 16)(x)
    h = relu(fc1(flat))
    y = fc2(h)
    # mean(y * G) * B*6 seeds dy = G (the tape's seed is 1.0)
    loss = mul(mean_all(mul(y, Tensor.from_numpy(upstream, dev))), float(B * 6))
    loss.backward()
    _save("linear_mlp", {
        "x_nhwc": x_nhwc, "upstream": upstream,
        "w1": fc1.weight.numpy(), "b1": fc1.bias.numpy(),
        "w2": fc2.weight.numpy(), "b2": fc2.bias.numpy(),
        "y": y.numpy(), "dw1": fc1.weight.grad.to_numpy(), "db1": fc1.bias.grad.to_numpy(),
        "dw2": fc2.weight.grad.to_numpy(), "db2": fc2.bias.grad.to_numpy(),
        "dx": x.grad.to_numpy().reshape(B, 3, 3, 16),
    }, index, "ttrl/engine/layers.py Flatten(3,3,16) -> Linear(144,32) -> relu -> Linear(32,6), "
              "fwd and bwd with upstream gradient G")


def conv_tower(index):
    from ttrl.deploy.conv import conv_features
    from ttrl.engine.conv.geometry import conv_out_size
    rng = np.random.default_rng(500)
    out = {}
    # Nature CNN stages at a reduced width (channels 4->8->16->16) over a
    # full 84x84 frame, and a padded stride-1 stage.
    stages_def = [(4, 8, 8, 4, 0), (8, 16, 4, 2, 0), (16, 16, 3, 1, 0)]
    frames = rng.integers(0, 256, (2, 4, 84, 84)).astype(np.float32)
    stages = []
    for i, (cin, cout, k, s, p) in enumerate(stages_def):
        bound = 1.0 / np.sqrt(cin * k * k)
        w = rng.uniform(-bound, bound, (cout, cin, k, k)).astype(np.float32)
        b = rng.uniform(-bound, bound, (cout,)).astype(np.float32)
        if i == 0:
            w = w / np.float32(255.0)  # ObsSpec.scale folded into the first stage
        stages.append((w, b, s, p))
        out[f"nature_w{i}"] = w
        out[f"nature_b{i}"] = b
    out["nature_frames"] = frames.astype(np.uint8)
    out["nature_features"] = conv_features(frames, stages)
    x = rng.standard_normal((2, 3, 9, 9)).astype(np.float32)
    w = rng.standard_normal((5, 3, 3, 3)).astype(np.float32)
    b = rng.standard_normal(5).astype(np.float32)
    out["pad_x"] = x
    out["pad_w"] = w
    out["pad_b"] = b
    out["pad_features"] = conv_features(x, [(w, b, 1, 1)])
    sizes = []
    # -1 marks a geometry the reference refuses (ragged stride or empty output).
    for size, k, s, p in [(84, 8, 4, 0), (20, 4, 2, 0), (9, 3, 1, 0), (9, 3, 1, 1),
                          (64, 8, 4, 2), (11, 3, 2, 1), (85, 8, 4, 0), (10, 4, 2, 0),
                          (2, 3, 1, 0)]:
        try:
            o = conv_out_size(size, k, s, p, axis="h")
        except ValueError:
            o = -1
        sizes.append([size, k, s, p, o])
    out["geometry"] = np.array(sizes, np.int64)
    _save("conv_tower", out, index,
          "ttrl/deploy/conv.py:31-50 conv_features (ReLU after every stage, NHWC flatten) "
          "and ttrl/engine/conv/geometry.py conv_out_size")


def grad_clip(index):
    from ttrl.algos.grads import clip_grad_norm, grad_sq_device
    from ttrl.engine.autograd import Tensor
    import ttnn
    out = {}
    for v, max_norm in enumerate((0.5, 1e3)):
        rng = np.random.default_rng(600 + v)
        shapes = [(32, 4), (100,), (7, 3)]
        params = [Tensor.from_numpy(np.zeros(s, np.float32), ttnn.DEVICE, requires_grad=True)
                  for s in shapes]
        grads = [rng.standard_normal(s).astype(np.float32) for s in shapes]
        for p, g in zip(params, grads):
            p.grad = ttnn.Tensor(g)
        sq = grad_sq_device(params).to_numpy()
        norm = clip_grad_norm(params, max_norm)
        pre = f"c{v}_"
        out[pre + "max_norm"] = np.float64(max_norm)
        out[pre + "norm"] = np.float64(norm)
        out[pre + "grad_sq"] = sq
        for i, (p, g) in enumerate(zip(params, grads)):
            out[pre + f"g{i}"] = g
            out[pre + f"clipped{i}"] = p.grad.to_numpy()
    _save("grad_clip", out, index,
          "ttrl/algos/grads.py:29-61 clip_grad_norm (f64 host norm) and grad_sq_device")


def gru(index):
    from ttrl.engine.autograd import Tensor
    from ttrl.engine.ops import mean_all, mul
    from ttrl.engine.recurrent import GRUCell
    import ttnn
    np.random.seed(700)
    dev = ttnn.DEVICE
    B, I, H = 4, 10, 8
    cell = GRUCell(I, H, dev)
    rng = np.random.default_rng(701)
    x = rng.standard_normal((B, I)).astype(np.float32)
    h = rng.standard_normal((B, H)).astype(np.float32)
    upstream = rng.standard_normal((B, H)).astype(np.float32)
    xt = Tensor.from_numpy(x, dev, requires_grad=True)
    ht = Tensor.from_numpy(h, dev, requires_grad=True)
    h1 = cell(xt, ht)
    loss = mul(mean_all(mul(h1, Tensor.from_numpy(upstream, dev))), float(B * H))
    loss.backward()
    out = {"x": x, "h": h, "upstream": upstream, "h1": h1.numpy(),
           "dx": xt.grad.to_numpy(), "dh": ht.grad.to_numpy()}
    for name, p in cell.named_parameters():
        out["param." + name] = p.numpy()
        out["grad." + name] = p.grad.to_numpy()
    _save("gru_cell", out, index, "ttrl/engine/recurrent.py GRUCell forward and backward")


def param_sync(index):
    from ttrl.engine.autograd import Tensor
    from ttrl.engine.mesh.sync import ParamSync
    from ttrl.engine.nn import Module
    import ttnn

    class Two(Module):
        def __init__(self, a, b):
            self.w = Tensor.from_numpy(np.array(a, np.float32), ttnn.DEVICE, requires_grad=True)
            self.b = Tensor.from_numpy(np.array(b, np.float32), ttnn.DEVICE, requires_grad=True)

    rng = np.random.default_rng(800)
    out = {}
    for n in (2, 3, 4):
        a = [rng.standard_normal(5).astype(np.float32) for _ in range(n)]
        b = [rng.standard_normal((2, 3)).astype(np.float32) for _ in range(n)]
        mods = [Two(a[i], b[i]) for i in range(n)]
        sync = ParamSync(mods, sync_every=1)
        sync.average()
        out[f"n{n}_w_in"] = np.stack(a)
        out[f"n{n}_b_in"] = np.stack(b)
        out[f"n{n}_w_out"] = np.stack([m.w.numpy() for m in mods])
        out[f"n{n}_b_out"] = np.stack([m.b.numpy() for m in mods])
    _save("param_sync", out, index,
          "ttrl/engine/mesh/sync.py ParamSync.average: exact fp32 sum in replica order, then /N")


class _Batch(dict):
    """Mapping of named device tensors plus .obs / .next_obs, as the SAC
    losses read a loaded batch."""


class _FakePolicy:
    """Returns preset (mean, log_std) leaves for obs and next_obs."""

    def __init__(self, cur, nxt):
        self.cur, self.nxt = cur, nxt

    def __call__(self, obs):
        return self.nxt if obs == "next" else self.cur


class _LinearCritic:
    """Q(s, a) = sum(a * w) + s_feat: linear in the action, so d Q / d a
    carries the actor loss back through the reparameterised sample."""

    def __init__(self, w, s_cur, s_next):
        self.w, self.s_cur, self.s_next = w, s_cur, s_next

    def __call__(self, obs, action):
        from ttrl.engine.ops import add, mul, sum_dim
        feat = self.s_next if obs == "next" else self.s_cur
        return add(sum_dim(mul(action, self.w), dim=-1, keepdim=True), feat)


def sac_losses(index):
    from ttrl.algos.sac.losses import actor_loss, alpha_loss, critic_loss
    from ttrl.algos.sac.policy import SquashedGaussian
    from ttrl.engine.autograd import Tensor
    from ttrl.spaces.action import ActionSpec
    import ttnn
    out = {}
    dev = ttnn.DEVICE
    for v, (name, per) in enumerate((("uniform", False), ("prioritized", True))):
        rng = np.random.default_rng(900 + v)
        B, D = 256, 3
        low, high = (-1.0, -2.0, -0.5), (1.0, 2.0, 1.5)
        spec = ActionSpec(kind="continuous", dim=D, low=low, high=high)
        dist = SquashedGaussian(spec, dev)
        mean = (rng.standard_normal((B, D)) * 0.8).astype(np.float32)
        log_std = rng.uniform(-2.0, 0.5, (B, D)).astype(np.float32)
        mean_n = (rng.standard_normal((B, D)) * 0.8).astype(np.float32)
        log_std_n = rng.uniform(-2.0, 0.5, (B, D)).astype(np.float32)
        noise = rng.standard_normal((B, D)).astype(np.float32)
        next_noise = rng.standard_normal((B, D)).astype(np.float32)
        q_w = [rng.standard_normal((1, D)).astype(np.float32) for _ in range(4)]
        s_feat = [rng.standard_normal((B, 1)).astype(np.float32) for _ in range(8)]
        actions = rng.uniform(-1, 1, (B, D)).astype(np.float32)
        rewards = rng.standard_normal((B, 1)).astype(np.float32)
        dones = (rng.random((B, 1)) < 0.05).astype(np.float32)
        discounts = np.full((B, 1), 0.99, np.float32)
        isw = rng.uniform(0.3, 1.0, (B, 1)).astype(np.float32) if per else None
        log_alpha_v = np.array([[np.log(0.2)]], np.float32)
        T = lambda a, g=False: Tensor.from_numpy(a, dev, requires_grad=g)
        mean_t, log_std_t = T(mean, True), T(log_std, True)
        nets = SimpleNamespace(
            policy=_FakePolicy((mean_t, log_std_t), (T(mean_n), T(log_std_n))),
            critics=[_LinearCritic(T(q_w[i]), T(s_feat[i]), T(s_feat[2 + i])) for i in range(2)],
            targets=[_LinearCritic(T(q_w[2 + i]), T(s_feat[4 + i]), T(s_feat[6 + i]))
                     for i in range(2)])
        batch = _Batch(rewards=T(rewards), dones=T(dones), discounts=T(discounts),
                       actions=T(actions), noise=T(noise), next_noise=T(next_noise))
        batch.obs, batch.next_obs = "cur", "next"
        log_alpha = T(log_alpha_v, True)
        alpha = Tensor(ttnn.exp(log_alpha.data), requires_grad=False)
        # critic loss: gradients reach the critics' outputs (here the action
        # weights of the online critics and their state features)
        for i in range(2):
            nets.critics[i].w.requires_grad = True
            nets.critics[i].s_cur.requires_grad = True
        weights = T(isw) if per else None
        closs, target, errors = critic_loss(nets, dist, batch, alpha, weights)
        closs.backward()
        pre = f"{name}_"
        out.update({pre + "mean": mean, pre + "log_std": log_std, pre + "mean_next": mean_n,
                    pre + "log_std_next": log_std_n, pre + "noise": noise,
                    pre + "next_noise": next_noise, pre + "q_w": np.stack(q_w),
                    pre + "s_feat": np.stack(s_feat), pre + "actions": actions,
                    pre + "rewards": rewards, pre + "dones": dones, pre + "discounts": discounts,
                    pre + "is_weights": isw if per else np.ones((B, 1), np.float32),
                    pre + "log_alpha": log_alpha_v, pre + "low": np.array(low, np.float32),
                    pre + "high": np.array(high, np.float32),
                    pre + "critic_loss": closs.numpy(), pre + "q_target": target.numpy()})
        for i in range(2):
            out[pre + f"d_critic{i}_w"] = nets.critics[i].w.grad.to_numpy()
            out[pre + f"d_critic{i}_s"] = nets.critics[i].s_cur.grad.to_numpy()
        # actor loss (fresh graph; critics' weights now constants again)
        for i in range(2):
            nets.critics[i].w.requires_grad = False
            nets.critics[i].s_cur.requires_grad = False
            nets.critics[i].w.grad = None
        aloss, logp = actor_loss(nets, dist, batch, alpha)
        aloss.backward()
        dual = alpha_loss(log_alpha, logp, -float(D))
        dual.backward()
        out.update({pre + "actor_loss": aloss.numpy(), pre + "logp": logp.numpy(),
                    pre + "d_mean": mean_t.grad.to_numpy(),
                    pre + "d_log_std": log_std_t.grad.to_numpy(),
                    pre + "alpha_loss": dual.numpy(),
                    pre + "d_log_alpha": log_alpha.grad.to_numpy()})
    _save("sac_losses", out, index,
          "ttrl/algos/sac/losses.py:46-94 with SquashedGaussian (ttrl/algos/sac/policy.py:30-40,"
          " ttrl/algos/gaussian.py:55-167) over preset policy outputs and action-linear critics")


def sac_update(index):
    """Three whole SAC updates in the reference agent's order
    (ttrl/algos/sac/agent.py:218-238): critic_region then the critic Adam,
    actor_region (actor and temperature losses) then the policy and
    temperature Adams, then PolyakSync's blend (ttrl/algos/sac/targets.py:
    45-96) -- each region zeroing all three optimizers first, as
    RegionOptimizers does (ttrl/algos/sac/step.py:28-55). The nets are the
    reference's build_sac_nets at BASELINE configs[2]: obs 11, actions 3 in
    [-1, 1], twin critics 14-256-256-1 with targets, actor 11-256-256-(3, 3),
    batch 256, tau 0.005, lr 3e-4, target entropy -3."""
    from ttrl.algos.sac.policy import SquashedGaussian
    from ttrl.algos.sac.step import actor_region, critic_region
    from ttrl.algos.sac.targets import _blend
    from ttrl.engine.autograd import Tensor
    from ttrl.engine.optim import Adam
    from ttrl.nets.build import build_sac_nets
    from ttrl.nets.obs import ObsPair
    from ttrl.spaces import ActionSpec, ObsGroup, ObsSpec
    import ttnn
    dev = ttnn.DEVICE
    B, OBS, D, UPDATES = 256, 11, 3, 3
    np.random.seed(2024)
    spec = ObsGroup.of(ObsSpec.vector(OBS))
    action_spec = ActionSpec.continuous([-1.0] * D, [1.0] * D)
    nets = build_sac_nets(spec, action_spec, dev, batch=B, critic_hidden=(256, 256),
                          encoder_kwargs={"hidden": (256, 256)})
    dist = SquashedGaussian(action_spec, dev)
    log_alpha = Tensor.from_numpy(np.full((1, 1), np.log(0.2), np.float32), dev,
                                  requires_grad=True)
    actor_opt = Adam(nets.policy_parameters(), lr=3e-4)
    critic_opt = Adam(nets.critic_parameters(), lr=3e-4)
    alpha_opt = Adam([log_alpha], lr=3e-4)
    out = {f"init.{k}": v for k, v in nets.state_dict().items()}
    out["init.log_alpha"] = log_alpha.numpy()
    rng = np.random.default_rng(2025)
    T = lambda a: Tensor.from_numpy(np.asarray(a, np.float32), dev)  # noqa: E731
    for u in range(UPDATES):
        b = {"obs": rng.standard_normal((B, OBS)), "next_obs": rng.standard_normal((B, OBS)),
             "actions": np.tanh(rng.standard_normal((B, D))),
             "rewards": rng.standard_normal((B, 1)),
             "dones": (rng.random((B, 1)) < 0.05).astype(np.float64),
             "discounts": np.full((B, 1), 0.99), "noise": rng.standard_normal((B, D)),
             "next_noise": rng.standard_normal((B, D))}
        b = {k: np.asarray(v, np.float32) for k, v in b.items()}
        for k, v in b.items():
            out[f"batch{u}.{k}"] = v
        batch = _Batch(actions=T(b["actions"]), rewards=T(b["rewards"]), dones=T(b["dones"]),
                       discounts=T(b["discounts"]), noise=T(b["noise"]),
                       next_noise=T(b["next_noise"]))
        batch.obs = ObsPair.shared({"obs": T(b["obs"])})
        batch.next_obs = ObsPair.shared({"obs": T(b["next_obs"])})
        for opt in (actor_opt, critic_opt, alpha_opt):
            opt.zero_grad()
        critic = critic_region(nets, dist, batch, log_alpha, prioritized=False)
        critic_opt.step()
        for opt in (actor_opt, critic_opt, alpha_opt):
            opt.zero_grad()
        actor = actor_region(nets, dist, batch, log_alpha, -float(D), learn_alpha=True)
        actor_opt.step()
        alpha_opt.step()
        _blend(nets, 0.005)
        for key in ("critic_loss", "alpha"):
            out[f"update{u}.{key}"] = critic[key].numpy()
        out[f"update{u}.q_target"] = critic["q_target"].numpy()
        for key in ("actor_loss", "alpha_loss", "logp"):
            out[f"update{u}.{key}"] = actor[key].numpy()
    out.update({f"final.{k}": v for k, v in nets.state_dict().items()})
    out["final.log_alpha"] = log_alpha.numpy()
    _save("sac_update", out, index,
          "three SAC updates of build_sac_nets (obs 11, act 3, hidden 256) in the agent's "
          "order: critic_region + critic Adam, actor_region + policy and alpha Adams, "
          "PolyakSync blend tau 0.005 (ttrl/algos/sac/{agent,step,targets}.py)")


def conv_backward(index):
    """The reference's own convolution backward (ttrl/engine/conv/backward.py):
    weight_grad (k*k strided slices of X, concat, one (M, k*k*C)^T @ (M, K)
    matmul, scaled by input_scale, into the prepared layout by
    dw_to_prepared, transform.py:232-254) and input_grad (transpose_weight,
    transform.py:71-100: the master unpadded, mirrored in both kernel axes,
    channel pair swapped and padded into the transposed layout, then one
    conv_transpose2d with mirror_kernel, transform.py:103-129) at the three
    Nature-CNN geometries and conv1's space-to-depth form, batch 2. The
    prepared layouts use the default padding rule (channels to 8, a kernel
    row to 32 rows, outputs to 32 columns)."""
    from ttrl.engine.conv.backward import input_grad, weight_grad
    from ttrl.engine.conv.geometry import ConvGeometry
    from ttrl.engine.conv.packing import PreparedLayout
    from ttrl.engine.conv.transform import TransposeSpec
    import ttnn
    dev = ttnn.DEVICE

    def layout(out_ch, in_ch, k):
        cp = (in_ch + 7) // 8 * 8
        row_block = (k * cp + 31) // 32 * 32
        return PreparedLayout(rows=k * row_block, cols=(out_ch + 31) // 32 * 32, cp=cp,
                              row_block=row_block, out_channels=out_ch, in_channels=in_ch,
                              kernel_h=k, kernel_w=k)

    out = {}
    cases = (("conv1", 84, 4, 32, 8, 4, 1.0 / 255.0), ("conv1s2d", 21, 64, 32, 2, 1, 1.0 / 255.0),
             ("conv2", 20, 32, 64, 4, 2, 1.0), ("conv3", 9, 64, 64, 3, 1, 1.0))
    for i, (name, hw, c, co, k, st, scale) in enumerate(cases):
        rng = np.random.default_rng(700 + i)
        n = 2
        geom = ConvGeometry(batch=n, in_channels=c, in_h=hw, in_w=hw, out_channels=co,
                            kernel=k, stride=st, padding=0)
        oh = geom.out_h
        x = rng.standard_normal((n, hw, hw, c)).astype(np.float32)
        w = (rng.standard_normal((co, c, k, k)) / np.sqrt(c * k * k)).astype(np.float32)
        dy = rng.standard_normal((n, oh, oh, co)).astype(np.float32)
        lay = layout(co, c, k)
        rows = lambda a: ttnn.Tensor(a.reshape(1, 1, -1, a.shape[-1]), _dev=dev)  # noqa: E731
        dw = weight_grad(rows(x), rows(dy), geom, lay, dev, input_scale=scale)
        tspec = TransposeSpec(batch=n, in_channels=co, out_channels=c, in_h=oh, in_w=oh,
                              kernel=k, stride=st, padding=0, layout=layout(c, co, k),
                              shard_layout=None, conv_cfg=None)
        master = ttnn.Tensor(lay.pack(w), _dev=dev)
        dx = input_grad(rows(dy), master, SimpleNamespace(layout=lay), tspec, dev,
                        input_scale=scale)
        out.update({f"{name}.x": x, f"{name}.w": w, f"{name}.dy": dy,
                    f"{name}.scale": np.float32(scale),
                    f"{name}.dw": lay.unpack(dw.to_numpy()),
                    f"{name}.dx": dx.to_numpy().reshape(n, hw, hw, c)})
    _save("conv_backward", out, index,
          "ttrl/engine/conv/backward.py weight_grad and input_grad (with transform.py's "
          "dw_to_prepared / transpose_weight) over the stand-in's conv_transpose2d; "
          "x/dy NHWC, w/dw OIHW, dx NHWC")


def recurrent_ppo(index):
    """One recurrent PPO minibatch through the reference's own pieces:
    build_recurrent_actor_critic (MLP trunk -> GRU -> heads), a
    RolloutSequenceBatch with resets inside the sequences and padding slots,
    RecurrentRuntime.forward (zeroing + masked mean) and objective, then
    backward. Also the unroll's outputs against T acting steps of the cell."""
    from ttrl.algos.ppo.loss import objective
    from ttrl.algos.ppo.policy import CategoricalPolicy
    from ttrl.algos.ppo.recurrent import RecurrentRuntime
    from ttrl.buffers.types import RolloutSequenceBatch
    from ttrl.engine.autograd import Tensor
    from ttrl.nets.obs import ObsPair
    from ttrl.nets.recurrent import ACTOR, build_recurrent_actor_critic
    from ttrl.spaces import ActionSpec, ObsGroup, ObsSpec
    import ttnn
    np.random.seed(950)
    dev = ttnn.DEVICE
    T, S, D, H, A = 6, 4, 9, 8, 5
    spec = ObsGroup.of(ObsSpec.vector(D))
    net = build_recurrent_actor_critic(spec, ActionSpec.discrete(A), dev, batch=T * S,
                                       hidden_size=H, hidden=(16,))
    rng = np.random.default_rng(951)
    rows = T * S
    obs = rng.standard_normal((rows, D)).astype(np.float32)
    h0 = rng.standard_normal((S, H)).astype(np.float32)
    starts = (rng.random((T, S, 1)) < 0.25).astype(np.float32)
    starts[0, 0, 0], starts[3, 1, 0] = 1.0, 1.0
    valid = (rng.random(rows) < 0.85).astype(np.float32)
    actions = rng.integers(0, A, rows)
    old_logp = (np.log(1.0 / A) + 0.3 * rng.standard_normal(rows)).astype(np.float32)
    values = rng.standard_normal(rows).astype(np.float32)
    adv = rng.standard_normal(rows).astype(np.float32)
    returns = rng.standard_normal(rows).astype(np.float32)
    batch = RolloutSequenceBatch(obs=obs, actions=actions, old_logp=old_logp, values=values,
                                 advantages=adv, returns=returns, starts=starts, valid=valid,
                                 h0={ACTOR: h0}, seq_len=T, lanes=np.arange(S))

    def acting(o, h, st, *, seq_len):
        return net(ObsPair.shared({"obs": Tensor.from_numpy(o, dev)}), h, st, seq_len=seq_len)

    runtime = RecurrentRuntime(net, dev, n_envs=S, seq_len=T)
    policy_out, value, reduce, masked = runtime.forward(acting, batch, dev)
    cfg = SimpleNamespace(clip_eps=0.1, value_clip_eps=0.1, value_coef=0.5, entropy_coef=0.01)
    policy = CategoricalPolicy(SimpleNamespace(n=A), dev)
    loss, parts, new_logp = objective(policy, policy_out, value, masked, cfg, dev,
                                      reduce=reduce)
    loss.backward()
    out = {"obs": obs, "h0": h0, "starts": starts, "valid": valid,
           "actions": actions.astype(np.int64), "old_logp": old_logp, "values": values,
           "advantages": adv, "returns": returns, "logits": policy_out.numpy(),
           "value": value.numpy(), "loss": loss.numpy(),
           "policy_loss": parts["policy_loss"].numpy(),
           "value_loss": parts["value_loss"].numpy(), "entropy": parts["entropy"].numpy(),
           "new_logp": new_logp.numpy()}
    for name, p in net.named_parameters():
        out["param." + name] = p.numpy()
        out["grad." + name] = p.grad.to_numpy()
    _save("recurrent_ppo", out, index,
          "ttrl/algos/ppo/recurrent.py:179-227 + ttrl/nets/recurrent.py:98-123 + "
          "ttrl/algos/ppo/loss.py:27-83: T=6 x 4 sequences, MLP(9->16) -> GRU(16->8) -> "
          "(5 logits, value), starts inside sequences, padding slots; loss and every grad")


def rollout_gae(index):
    """ttrl/buffers/rollout.py's compute_gae and the minibatch advantage
    normalisation over valid slots, on a buffer with terminations and
    autoreset padding slots."""
    from ttrl.buffers.rollout import RolloutBuffer
    from ttrl.spaces import ActionSpec, ObsGroup, ObsSpec
    out = {}
    for case, (T, E, gamma, lam) in enumerate([(16, 5, 0.99, 0.95), (9, 3, 0.9, 0.8)]):
        rng = np.random.default_rng(1100 + case)
        buf = RolloutBuffer(ObsGroup.of(ObsSpec.vector(2)), ActionSpec.discrete(3), n_envs=E,
                            n_steps=T, seed=5)
        rewards = rng.standard_normal((T, E)).astype(np.float32)
        values = rng.standard_normal((T, E)).astype(np.float32)
        dones = (rng.random((T, E)) < 0.15).astype(np.float32)
        valid = (rng.random((T, E)) > 0.1).astype(np.float32)
        for t in range(T):
            buf.add({"obs": np.zeros((E, 2), np.float32)}, np.zeros(E, np.int64),
                    np.zeros(E, np.float32), values[t], rewards[t], dones[t], valid[t])
        last = rng.standard_normal(E).astype(np.float32)
        buf.compute_gae(gamma, lam, last)
        keep = valid.reshape(-1) > 0
        adv = buf.advantages.reshape(-1)[keep]
        norm = (adv - adv.mean()) / (adv.std() + 1e-8)
        pre = f"c{case}_"
        out.update({pre + "rewards": rewards, pre + "values": values, pre + "dones": dones,
                    pre + "valid": valid, pre + "last_values": last,
                    pre + "gamma_lam": np.array([gamma, lam]),
                    pre + "advantages": buf.advantages.copy(), pre + "returns": buf.returns.copy(),
                    pre + "normalized_valid": norm})
    _save("rollout_gae", out, index,
          "ttrl/buffers/rollout.py:195-227 compute_gae and :269-270 normalisation over valid")


def priority_replay(index):
    """ttrl/buffers/sampling.py's PrioritySampler (pure numpy) through a
    scripted sequence: fresh columns, two write-backs (one with a column drawn
    twice), and draws over wrapped ring runs."""
    from ttrl.buffers.sampling import PriorityConfig, PrioritySampler
    from ttrl.buffers.window import SampleWindow
    lanes, columns = 3, 40
    cfg = PriorityConfig(alpha=0.6, epsilon=1e-6)
    s = PrioritySampler(cfg, lanes=lanes, columns=columns)
    rng = np.random.default_rng(1200)
    out = {}
    fresh = [(l, c) for l in range(lanes) for c in range(columns)]
    for l, c in fresh:
        s.on_write(l, c)
    for phase in range(2):
        n = 24
        ul = rng.integers(0, lanes, n)
        uc = rng.integers(0, columns, n)
        ul[-1], uc[-1] = ul[0], uc[0]  # one pair twice: the last value wins
        td = (np.abs(rng.standard_normal(n)) * (3.0 if phase else 1.0)).astype(np.float32)
        s.update(ul, uc, td)
        out[f"u{phase}_lanes"], out[f"u{phase}_cols"], out[f"u{phase}_td"] = ul, uc, td
        out[f"u{phase}_weight"] = s._weight.copy()
        out[f"u{phase}_max"] = np.float64(s._max_priority)
    s.on_write(1, 7)
    out["fresh_weight"] = s._weight.copy()
    window = SampleWindow(counts=np.array([40, 25, 31]), start=np.array([0, 30, 12]),
                          capacity=columns)
    for k, beta in enumerate((0.4, 0.9)):
        draw_rng = np.random.default_rng(1300 + k)
        d = s.draw(draw_rng, window, batch_size=64, beta=beta)
        out[f"d{k}_lanes"], out[f"d{k}_offsets"], out[f"d{k}_weights"] = d.lanes, d.offsets, d.weights
        out[f"d{k}_beta"] = np.float64(beta)
    out["window_counts"], out["window_start"] = window.counts, window.start
    _save("priority_replay", out, index,
          "ttrl/buffers/sampling.py PrioritySampler: on_write, update (duplicate pair), draw "
          "(multinomial lane quota, searchsorted, IS weights) over wrapped runs")


#: A small image DQN: the Nature-CNN stages over 4x36x36 frames (36 -> 8 -> 3
#: -> 1), a 16-wide feature layer and 6 actions.
CKPT_OBS = (4, 36, 36)
CKPT_HIDDEN, CKPT_ACTIONS = 16, 6
CKPT_CONV = ((32, 4, 8, 8), (64, 32, 4, 4), (64, 64, 3, 3))


def _ckpt_q_state(rng):
    """The names and shapes `EncoderHead.state_dict()` of the reference's
    build_q_net has for this spec (every encoder a MultiEncoder, Sequential
    numbering ReLUs and the Flatten), values on a 1/1024 grid so the file
    compresses."""
    sd = {}
    grid = lambda shape: (rng.integers(-48, 49, shape) / 1024.0).astype(np.float32)
    for layer, shape in zip((0, 2, 4), CKPT_CONV):
        sd[f"encoder.towers.obs.layers.{layer}.weight"] = grid(shape)
        sd[f"encoder.towers.obs.layers.{layer}.bias"] = grid((1, 1, 1, shape[0]))
    sd["encoder.towers.obs.layers.7.weight"] = grid((64, CKPT_HIDDEN))
    sd["encoder.towers.obs.layers.7.bias"] = grid((1, CKPT_HIDDEN))
    sd["head.q.weight"] = grid((CKPT_HIDDEN, CKPT_ACTIONS))
    sd["head.q.bias"] = grid((1, CKPT_ACTIONS))
    return sd


def _ckpt_layout(shape):
    """The prepared layout the reference's device library gives this conv
    (cp: channels rounded up to 8; the 4-channel 8x8 case is pinned by the
    reference's own tests at (1, 1, 512, 32))."""
    from ttrl.engine.conv.packing import candidate_layouts
    o, c, kh, kw = shape
    cp = (c + 7) // 8 * 8
    rows = kh * ((kw * cp + 31) // 32 * 32)
    cols = (o + 31) // 32 * 32
    return next(lay for lay in candidate_layouts(rows, cols, o, c, kh, kw) if lay.cp == cp)


def checkpoint_dqn(index):
    """A DQN-shaped L1 checkpoint written by the reference's own
    save_checkpoint (ttrl/train/checkpoint/file.py:112-218), with the Adam
    moments of each conv weight in the reference's prepared matrix
    (ttrl/engine/conv/packing.py:24-108) as its optimizer stores them, read
    back by its load_checkpoint and exported by its ttrl.deploy path; then the
    same file rewritten by ttrl_b200.checkpoint with changed weights and
    moments, and THAT file read and exported by the reference too."""
    import tempfile
    from ttrl.algos.dqn.config import DQNConfig
    from ttrl.deploy.export import export_policy
    from ttrl.deploy.read import load_policy
    from ttrl.spaces import ActionSpec, ObsSpec
    from ttrl.train.checkpoint import L1, load_checkpoint, save_checkpoint
    from ttrl.train.config import TrainConfig
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "..", "tt-rl_b200"))
    from ttrl_b200.checkpoint import Checkpoint
    from ttrl_b200.engine.packing import solve_cp

    rng = np.random.default_rng(1500)
    online, target = _ckpt_q_state(rng), _ckpt_q_state(rng)
    names = list(online)
    m, v, layouts = [], [], {}
    for i, name in enumerate(names):
        shape = online[name].shape
        mi = (rng.integers(-32, 33, shape) / 4096.0).astype(np.float32)
        vi = (rng.integers(1, 64, shape) / 2.0 ** 20).astype(np.float32)
        if len(shape) == 4 and shape[2] > 1:  # a conv weight: prepared matrix
            lay = _ckpt_layout(shape)
            layouts[i] = lay
            mi, vi = lay.pack(mi), lay.pack(vi)
        m.append(mi)
        v.append(vi)
    optimizer = {"t": 7, "steps": [7] * len(names), "lr": 1e-4, "betas": (0.9, 0.999),
                 "eps": 1.5e-4, "weight_decay": 0.0, "m": m, "v": v}
    state = {"config": DQNConfig(), "online": online, "target": target,
             "optimizer": optimizer, "frame_count": 2800, "update_count": 7,
             "rng_state": np.random.default_rng(3).bit_generator.state,
             "autoreset": {}, "clock": {}}
    obs = rng.integers(0, 256, (3,) + CKPT_OBS, dtype=np.uint8)
    out = {"obs": obs}
    with tempfile.TemporaryDirectory() as tmp:
        ref_path = os.path.join(tmp, "ref.npz")
        save_checkpoint(ref_path, agent_state=state, obs_spec=ObsSpec.image(*CKPT_OBS),
                        action_spec=ActionSpec.discrete(CKPT_ACTIONS), level=L1, frame=2800,
                        config=TrainConfig(), env_policy_state=[])
        loaded = load_checkpoint(ref_path)["agent_state"]
        assert set(loaded["online"]) == set(names)
        export_policy(ref_path, os.path.join(tmp, "ref_policy.npz"))
        out["deploy_q"] = load_policy(os.path.join(tmp, "ref_policy.npz")).head(obs)

        # Our reader and writer on the reference's file.
        ours = Checkpoint.read(ref_path)
        tree = ours.agent_state()
        for name in names:
            assert np.array_equal(tree["online"][name], loaded["online"][name])
        assert ours.to_bytes() is not None
        for i, lay in layouts.items():
            mine = solve_cp(tree["optimizer"]["m"][i].shape, CKPT_CONV[list(layouts).index(i)],
                            v=tree["optimizer"]["v"][i])
            assert (mine.cp, mine.rows, mine.cols) == (lay.cp, lay.rows, lay.cols)
            assert np.array_equal(mine.unpack(tree["optimizer"]["m"][i]),
                                  lay.unpack(tree["optimizer"]["m"][i]))
        # Changed weights and moments written back in the stored forms.
        upd_online = {k: (a + np.float32(1.0 / 512)).astype(np.float32)
                      for k, a in tree["online"].items()}
        opt = dict(tree["optimizer"])
        opt["t"], opt["steps"] = 8, [8] * len(names)
        opt["m"] = [a * np.float32(0.5) for a in opt["m"]]
        tree["online"] = upd_online
        tree["optimizer"] = opt
        tree["update_count"] = 8
        upd_path = os.path.join(tmp, "ours.npz")
        ours.with_agent_state(tree).write(upd_path)
        back = load_checkpoint(upd_path)
        for name in names:
            assert np.array_equal(back["agent_state"]["online"][name], upd_online[name])
        assert back["agent_state"]["optimizer"]["t"] == 8
        for i, lay in layouts.items():
            got = back["agent_state"]["optimizer"]["m"][i]
            assert got.shape == lay.shape and np.array_equal(got, opt["m"][i])
        export_policy(upd_path, os.path.join(tmp, "ours_policy.npz"))
        out["deploy_q_updated"] = load_policy(os.path.join(tmp, "ours_policy.npz")).head(obs)
        with open(ref_path, "rb") as f:
            out["ref_file"] = np.frombuffer(f.read(), np.uint8)
    out["layouts"] = np.array([[i, lay.rows, lay.cols, lay.cp] for i, lay in layouts.items()],
                              np.int64)
    _save("checkpoint_dqn", out, index,
          "ttrl/train/checkpoint/file.py save_checkpoint (L1) of a 4x36x36 DQN with prepared "
          "conv Adam moments (engine/conv/packing.py); deploy_q: ttrl.deploy export -> head "
          "of that file; deploy_q_updated: the same after ttrl_b200.checkpoint rewrote it")


def state_names(index):
    """state_dict names and shapes of the reference's builders over vector
    observations (ttrl/nets/build.py: build_q_net, build_actor_critic,
    build_sac_nets; ttrl/nets/recurrent.py), built on the numpy stand-in. An
    image net's names are pinned by the checkpoint_dqn file."""
    from ttrl.nets.build import build_actor_critic, build_q_net, build_sac_nets
    from ttrl.nets.recurrent import build_recurrent_actor_critic
    from ttrl.spaces import ActionSpec, ObsGroup, ObsSpec
    import ttnn
    dev = ttnn.DEVICE
    np.random.seed(1600)
    spec = ObsGroup.of(ObsSpec.vector(11))
    nets = {
        "q": build_q_net(spec, ActionSpec.discrete(5), dev, batch=8, hidden=(32, 24)),
        "ac": build_actor_critic(spec, ActionSpec.discrete(5), dev, batch=8, hidden=(32, 24)),
        "sac": build_sac_nets(spec, ActionSpec.continuous([-1.0] * 3, [1.0] * 3), dev, batch=8,
                              critic_hidden=(20, 12), encoder_kwargs={"hidden": (24, 16)}),
        "rec": build_recurrent_actor_critic(spec, ActionSpec.discrete(5), dev, batch=8,
                                            hidden_size=10, hidden=(16,)),
    }
    out = {}
    for family, net in nets.items():
        sd = net.state_dict()
        out[f"{family}.names"] = np.array(list(sd), dtype=np.str_)
        out[f"{family}.shapes"] = np.array(
            [",".join(str(d) for d in np.asarray(a).shape) for a in sd.values()], dtype=np.str_)
    _save("state_names", out, index,
          "state_dict names/shapes of build_q_net, build_actor_critic, build_sac_nets, "
          "build_recurrent_actor_critic over an 11-dim vector observation")


def main() -> None:
    reference = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TTRL_REFERENCE")
    if not reference or not os.path.isdir(os.path.join(reference, "ttrl")):
        raise SystemExit("usage: make_golden.py <reference checkout>")
    _install(reference)
    index_path = os.path.join(HERE, "index.json")
    only = set(sys.argv[2:])
    index: dict = {}
    if only and os.path.exists(index_path):
        with open(index_path) as f:
            index = json.load(f)
    for fn in (adam_scalars, adam_steps, dqn_loss, ppo_objective, linear_mlp, conv_tower,
               grad_clip, gru, param_sync, sac_losses, sac_update, conv_backward,
               recurrent_ppo, rollout_gae,
               priority_replay, checkpoint_dqn, state_names):
        if only and fn.__name__ not in only:
            continue
        fn(index)
        print("wrote", fn.__name__)
    with open(index_path, "w") as f:
        json.dump(index, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
