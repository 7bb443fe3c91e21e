"""The CPU oracle against golden vectors made by the reference's own code
(tests/golden/make_golden.py runs ttrl's tape, ops, Adam, losses, GRU,
ParamSync and deploy conv tower). This pins the oracle; the GPU tests then
compare the CUDA path with the pinned oracle.

Tolerances: fp32 elementwise chains 1e-6 relative (the spec's bar); float64
oracle against float32 reference arithmetic through exp/log/softmax 1e-5;
matmul-bearing chains 1e-5 (both sides are exact fp32/f64 BLAS, no TF32).
"""

import os

import numpy as np
import pytest

from oracle import layers as L
from oracle import learner as R

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def test_adam_scalars():
    for lr, b1, b2, eps, t, alpha, eps_t in load("adam_scalars")["rows"]:
        a, e = L.adam_fused_scalars(lr, b1, b2, eps, int(t))
        assert a == pytest.approx(alpha, rel=1e-14)
        assert e == pytest.approx(eps_t, rel=1e-14)


@pytest.mark.parametrize("case", [0, 1, 2])
def test_adam_steps(case):
    d = load("adam_steps")
    pre = f"c{case}_"
    lr, eps, wd = d[pre + "hyper"]
    for i in range(3):
        p = d[pre + f"p{i}_init"].copy()
        S = np.zeros_like(p)
        V = np.zeros_like(p)
        t = 0
        for step, g in enumerate(d[pre + f"p{i}_grads"]):
            if i == 1 and step == 2:
                continue  # no gradient: no update, no step count
            t += 1
            p, S, V = L.adam_step_sv(p, g, S, V, t, lr=lr, eps=eps, weight_decay=wd)
        assert t == d[pre + "steps"][i]
        assert rel(p, d[pre + f"p{i}_final"]) <= 1e-6
        assert rel(S, d[pre + f"p{i}_S"]) <= 1e-6
        assert rel(V, d[pre + f"p{i}_V"]) <= 1e-6


@pytest.mark.parametrize("name", ["vanilla", "double", "double_mask", "double_per"])
def test_dqn_loss_head(name):
    d = load("dqn_loss")
    g = {k[len(name) + 1:]: d[k] for k in d.files if k.startswith(name + "_")}
    double, mask_n, per = (int(v) for v in g["flags"])
    q = g["q"].astype(np.float64)
    q_tgt = g["q_next_target"].astype(np.float64)
    q_sel = g["q_next_online"].astype(np.float64) if double else q_tgt
    actions = g["onehot"].argmax(1)
    loss, mean_q, dq, td_abs, _ = R.dqn_loss_head(
        q, q_sel, q_tgt, actions, g["rewards"].reshape(-1), g["dones"].reshape(-1),
        g["discounts"].reshape(-1), delta=1.0,
        next_mask=g["next_mask"] if mask_n else None,
        is_weights=g["is_weights"].reshape(-1) if per else None)
    assert rel(loss, g["loss"]) <= 1e-6
    assert abs(mean_q - float(g["mean_q"].reshape(-1)[0])) <= 1e-6
    assert rel(dq, g["dq"]) <= 1e-6
    assert rel(np.sum(dq * dq), g["grad_sq"]) <= 1e-5
    if per:
        assert rel(td_abs, g["td_abs"].reshape(-1)) <= 1e-6


@pytest.mark.parametrize("name", ["mean", "masked"])
def test_ppo_objective(name):
    d = load("ppo_objective")
    g = {k[len(name) + 1:]: d[k] for k in d.files if k.startswith(name + "_")}
    loss, parts, new_logp, dlogits, dvalue = R.ppo_objective_and_grads(
        g["logits"].astype(np.float64), g["value"].astype(np.float64), g["actions"],
        g["old_logp"].astype(np.float64), g["adv"].astype(np.float64),
        g["returns"].astype(np.float64), g["old_values"].astype(np.float64),
        clip=0.1, vclip=0.1, vcoef=0.5, entcoef=0.01,
        valid=g["valid"] if name == "masked" else None)
    assert rel(loss, g["loss"]) <= 1e-5
    for k in ("policy_loss", "value_loss", "entropy"):
        assert rel(parts[k], g[k]) <= 1e-5, k
    assert rel(new_logp, g["new_logp"].reshape(-1)) <= 1e-5
    assert rel(dlogits, g["dlogits"]) <= 1e-5
    assert rel(dvalue, g["dvalue"]) <= 1e-5


def test_linear_mlp():
    d = load("linear_mlp")
    x = d["x_nhwc"].astype(np.float64)
    b = x.shape[0]
    flat = x.reshape(b, -1)  # (h, w, c) flatten order
    h_pre = L.linear(flat, d["w1"].astype(np.float64), d["b1"])
    h = L.relu(h_pre)
    y = L.linear(h, d["w2"].astype(np.float64), d["b2"])
    assert rel(y, d["y"]) <= 1e-5
    dh, dw2, db2 = L.linear_backward(h, d["w2"].astype(np.float64), d["upstream"])
    dz = dh * (h_pre > 0)
    dx, dw1, db1 = L.linear_backward(flat, d["w1"].astype(np.float64), dz)
    assert rel(dw2, d["dw2"]) <= 1e-5
    assert rel(db2, d["db2"]) <= 1e-5
    assert rel(dw1, d["dw1"]) <= 1e-5
    assert rel(db1, d["db1"]) <= 1e-5
    assert rel(dx.reshape(d["dx"].shape), d["dx"]) <= 1e-5


def test_conv_tower_forward():
    d = load("conv_tower")
    x = d["nature_frames"].astype(np.float64).transpose(0, 2, 3, 1)
    for i, s in enumerate((4, 2, 1)):
        x = L.conv2d_nhwc(x, d[f"nature_w{i}"].astype(np.float64), d[f"nature_b{i}"],
                          stride=s, apply_relu=True)
    assert rel(x.reshape(x.shape[0], -1), d["nature_features"]) <= 1e-5
    y = L.conv2d_nhwc(d["pad_x"].astype(np.float64).transpose(0, 2, 3, 1),
                      d["pad_w"].astype(np.float64), d["pad_b"], stride=1, padding=1,
                      apply_relu=True)
    assert rel(y.reshape(y.shape[0], -1), d["pad_features"]) <= 1e-5


def test_conv_geometry():
    for size, k, s, p, want in load("conv_tower")["geometry"]:
        if want < 0:
            with pytest.raises(ValueError):
                L.conv_out(int(size), int(k), int(s), int(p))
        else:
            assert L.conv_out(int(size), int(k), int(s), int(p)) == want


@pytest.mark.parametrize("case", [0, 1])
def test_grad_clip(case):
    d = load("grad_clip")
    pre = f"c{case}_"
    grads = [d[pre + f"g{i}"] for i in range(3)]
    norm, scale = R.clip_grad_norm_scale(grads, float(d[pre + "max_norm"]))
    assert norm == pytest.approx(float(d[pre + "norm"]), rel=1e-12)
    assert rel(sum(np.sum(np.asarray(g, np.float64) ** 2) for g in grads),
               d[pre + "grad_sq"]) <= 1e-6
    for i, g in enumerate(grads):
        want = d[pre + f"clipped{i}"]
        got = g if scale is None else g * np.float32(scale)
        assert rel(got, want) <= 1e-6


def test_gru_cell():
    d = load("gru_cell")
    p = {k[len("param."):]: d[k].astype(np.float64) for k in d.files if k.startswith("param.")}
    h1, cache = R.gru_cell_forward(d["x"].astype(np.float64), d["h"].astype(np.float64),
                                   p["weight_ih"], p["weight_hh"], p["bias_ih"], p["bias_hh"])
    assert rel(h1, d["h1"]) <= 1e-5
    g = R.gru_cell_backward(d["upstream"].astype(np.float64), cache, p["weight_ih"],
                            p["weight_hh"])
    assert rel(g["dx"], d["dx"]) <= 1e-5
    assert rel(g["dh"], d["dh"]) <= 1e-5
    for k in ("weight_ih", "weight_hh", "bias_ih", "bias_hh"):
        assert rel(g[k], d["grad." + k]) <= 1e-5, k


@pytest.mark.parametrize("n,h,c,cout,k,s,p", [
    (2, 84, 4, 8, 8, 4, 0), (2, 20, 8, 16, 4, 2, 0), (2, 9, 16, 16, 3, 1, 0),
    (1, 9, 3, 5, 3, 1, 1),
])
def test_conv_backward_is_the_adjoint_of_the_pinned_forward(n, h, c, cout, k, s, p):
    """The conv forward is pinned by the deploy tower fixture; dX and dW are
    its adjoints: <conv(x, W), dY> = <x, dX(dY)> = <W, dW(x, dY)>, in f64.
    This is the property ttrl/engine/conv/backward.py:33-78 relies on."""
    rng = np.random.default_rng(n * 1000 + h * 10 + k)
    x = rng.standard_normal((n, h, h, c))
    w = rng.standard_normal((cout, c, k, k))
    oh = L.conv_out(h, k, s, p)
    dy = rng.standard_normal((n, oh, oh, cout))
    y = L.conv2d_nhwc(x, w, stride=s, padding=p)
    lhs = float(np.sum(y * dy))
    dx = L.conv2d_dgrad(dy, w, x.shape, stride=s, padding=p)
    dw = L.conv2d_wgrad(x, dy, k, stride=s, padding=p)
    assert float(np.sum(x * dx)) == pytest.approx(lhs, rel=1e-10)
    assert float(np.sum(w * dw)) == pytest.approx(lhs, rel=1e-10)


@pytest.mark.parametrize("name", ["uniform", "prioritized"])
def test_sac_losses(name):
    """SAC critic, actor and temperature losses with their gradients against
    the reference's own ttrl/algos/sac code (preset policy outputs,
    critics linear in the action: Q_i(s, a) = a . w_i + s_i)."""
    from oracle import sac as S
    d = load("sac_losses")
    g = {k[len(name) + 1:]: d[k] for k in d.files if k.startswith(name + "_")}
    w, s = g["q_w"].astype(np.float64), g["s_feat"].astype(np.float64)
    alpha = float(np.exp(g["log_alpha"].astype(np.float32)).reshape(-1)[0])
    low, high = g["low"], g["high"]
    # critic loss against the soft target
    a_n, logp_n, _ = S.squashed_sample(g["mean_next"], g["log_std_next"], g["next_noise"],
                                       low, high)
    q_targ = [(a_n * w[2 + i]).sum(-1) + s[6 + i].reshape(-1) for i in range(2)]
    y = S.soft_target(g["rewards"].reshape(-1), g["dones"].reshape(-1),
                      g["discounts"].reshape(-1), q_targ, logp_n, alpha)
    assert rel(y, g["q_target"].reshape(-1)) <= 1e-5
    acts = g["actions"].astype(np.float64)
    q = [(acts * w[i]).sum(-1) + s[i].reshape(-1) for i in range(2)]
    weights = g["is_weights"].reshape(-1) if name == "prioritized" else None
    loss, dq = S.critic_loss(q, y, weights)
    assert rel(loss, g["critic_loss"]) <= 1e-5
    for i in range(2):
        assert rel((dq[i][:, None] * acts).sum(0), g[f"d_critic{i}_w"].reshape(-1)) <= 1e-5
        assert rel(dq[i], g[f"d_critic{i}_s"].reshape(-1)) <= 1e-5
    # actor loss through the reparameterised sample
    a, logp, cache = S.squashed_sample(g["mean"], g["log_std"], g["noise"], low, high)
    assert rel(logp, g["logp"].reshape(-1)) <= 1e-5
    qa = [(a * w[i]).sum(-1) + s[i].reshape(-1) for i in range(2)]
    aloss, d_logp, d_q = S.actor_loss(logp, qa, alpha)
    assert rel(aloss, g["actor_loss"]) <= 1e-5
    d_action = sum(d_q[i][:, None] * w[i] for i in range(2))
    d_mean, d_log_std = S.squashed_sample_backward(d_action, d_logp, cache)
    assert rel(d_mean, g["d_mean"]) <= 1e-5
    assert rel(d_log_std, g["d_log_std"]) <= 1e-5
    # temperature
    la = float(g["log_alpha"].reshape(-1)[0])
    dual, dla = S.alpha_loss(la, logp, -3.0)
    assert rel(dual, g["alpha_loss"]) <= 1e-5
    assert rel(dla, g["d_log_alpha"]) <= 1e-5


def test_recurrent_ppo_minibatch():
    """The recurrent minibatch (trunk -> GRU with in-sequence resets -> heads,
    zeroed padding fields, masked-mean objective) and every gradient, against
    the reference's own RecurrentRuntime.forward + objective."""
    from oracle.recurrent import recurrent_ppo_minibatch
    d = load("recurrent_ppo")
    p = {k[len("param."):]: d[k].astype(np.float64) for k in d.files if k.startswith("param.")}
    f = lambda k: d[k].astype(np.float64)
    T = d["starts"].shape[0]
    out = recurrent_ppo_minibatch(p, f("obs"), f("h0"), f("starts"), f("valid"), d["actions"],
                                  f("old_logp"), f("values"), f("advantages"), f("returns"),
                                  seq_len=T)
    assert rel(out["logits"], d["logits"]) <= 1e-5
    assert rel(out["value"], d["value"]) <= 1e-5
    for k in ("loss", "policy_loss", "value_loss", "entropy"):
        assert rel(out[k], d[k]) <= 1e-5, k
    for name, g in out["grads"].items():
        assert rel(g, d["grad." + name]) <= 1e-5, name
    assert set(out["grads"]) == {k[len("grad."):] for k in d.files if k.startswith("grad.")}


@pytest.mark.parametrize("case", [0, 1])
def test_rollout_gae(case):
    """GAE-lambda and the valid-slot normalisation, bit-exact against the
    reference's RolloutBuffer (same float32 operations)."""
    from oracle import rollout as ro
    d = load("rollout_gae")
    g = {k[3:]: d[k] for k in d.files if k.startswith(f"c{case}_")}
    gamma, lam = (float(v) for v in g["gamma_lam"])
    adv, ret = ro.gae(g["rewards"], g["values"], g["dones"], g["valid"], g["last_values"],
                      gamma, lam)
    assert np.array_equal(adv, g["advantages"])
    assert np.array_equal(ret, g["returns"])
    assert np.array_equal(ro.normalize(adv, g["valid"]), g["normalized_valid"])


def test_priority_replay():
    """The prioritized-replay restatement against the reference's own
    PrioritySampler on the same scripted sequence."""
    from oracle.priority import PriorityTable
    d = load("priority_replay")
    t = PriorityTable(3, 40, 0.6, 1e-6)
    for l in range(3):
        for c in range(40):
            t.on_write(l, c)
    for phase in range(2):
        t.update(d[f"u{phase}_lanes"], d[f"u{phase}_cols"], d[f"u{phase}_td"])
        assert np.array_equal(t.weight, d[f"u{phase}_weight"])
        assert t.max_priority == float(d[f"u{phase}_max"])
    t.on_write(1, 7)
    assert np.array_equal(t.weight, d["fresh_weight"])
    for k in range(2):
        lanes, offsets, weights = t.draw(np.random.default_rng(1300 + k), d["window_counts"],
                                         d["window_start"], 40, 64, float(d[f"d{k}_beta"]))
        assert np.array_equal(lanes, d[f"d{k}_lanes"])
        assert np.array_equal(offsets, d[f"d{k}_offsets"])
        assert np.array_equal(weights, d[f"d{k}_weights"])


def test_sac_whole_update():
    """The oracle's whole SAC update (critic step, actor and temperature
    steps, Polyak) against three updates of the reference's own
    build_sac_nets / critic_region / actor_region / Adam / PolyakSync blend
    at BASELINE configs[2] shapes. The fixture is float32; the oracle is
    float64: losses to 1e-6, every parameter to 1e-5 relative Frobenius."""
    from oracle import sac
    d = load("sac_update")
    p = {k[len("init."):]: d[k] for k in d.files if k.startswith("init.")}
    adam, steps = {}, {}
    for u in range(3):
        batch = {k.split(".", 1)[1]: d[k] for k in d.files if k.startswith(f"batch{u}.")}
        p, adam, steps, m = sac.sac_update(p, adam, steps, batch, low=-np.ones(3),
                                           high=np.ones(3))
        for key in ("critic_loss", "actor_loss", "alpha_loss", "alpha"):
            want = float(d[f"update{u}.{key}"].reshape(-1)[0])
            assert abs(m[key] - want) <= 1e-6 * max(1.0, abs(want)), (u, key)
        assert np.allclose(m["logp"], d[f"update{u}.logp"][:, 0], rtol=0, atol=5e-5)
    assert steps == {"critic": 3, "policy": 3, "alpha": 3}
    for name, value in p.items():
        want = d["final." + name]
        err = np.linalg.norm(value.reshape(want.shape) - want) / np.linalg.norm(want)
        assert err <= 1e-5, (name, err)


@pytest.mark.parametrize("name,stride", [("conv1", 4), ("conv1s2d", 1), ("conv2", 2),
                                         ("conv3", 1)])
def test_conv_backward_against_the_reference(name, stride):
    """The oracle's conv dW and dX against the reference's own weight_grad
    and input_grad (ttrl/engine/conv/backward.py:33-78 with transform.py's
    weight transforms) run over the stand-in: 1e-5 of the largest entry."""
    d = load("conv_backward")
    x, w, dy = (d[f"{name}.{k}"].astype(np.float64) for k in ("x", "w", "dy"))
    scale = float(d[f"{name}.scale"])
    dw = L.conv2d_wgrad(x, dy, w.shape[2], stride=stride, input_scale=scale)
    dx = L.conv2d_dgrad(dy, w, x.shape, stride=stride, input_scale=scale)
    assert rel(np.asarray(dw).reshape(w.shape), d[f"{name}.dw"]) <= 1e-5
    assert rel(np.asarray(dx).reshape(x.shape), d[f"{name}.dx"]) <= 1e-5
