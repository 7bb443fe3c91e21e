"""The fused SAC heads (engine.ops.sac_sample / sac_critic_loss /
sac_actor_loss) against the composed ops they replace.

The composed ops are pinned to the reference's own SAC code by the golden
vectors of test_sac_gpu.py; here the fused kernels must give the same
forward values and gradients on the same inputs: the joint critic input and
the log-density bit for bit (the same fp32 operations in the same order),
losses to 1e-6 relative, gradients to 1e-5 relative (their sums may be
formed in another order). Inputs put some raw log-stds beyond both clamp
bounds, some Q pairs tied and some dones set, so every branch runs.
"""

import os
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.helpers import rel  # noqa: E402

pytestmark = pytest.mark.gpu

B, D, OBS = 256, 3, 11


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _T(a, grad=False):
    from ttrl_b200.engine.autograd import Tensor
    return Tensor.from_numpy(np.ascontiguousarray(a, np.float32), "cuda", requires_grad=grad)


def _policy_inputs(rng):
    mean = rng.standard_normal((B, D)) * 0.8
    raw = rng.standard_normal((B, D)) * 1.5 - 0.5
    raw[0, 0], raw[1, 1], raw[2, 2] = -25.0, 3.5, 2.0  # below, above, at a bound
    noise = rng.standard_normal((B, D))
    obs = rng.standard_normal((B, OBS))
    return mean, raw, noise, obs


@pytest.mark.parametrize("learn_alpha", [True, False])
def test_fused_sample_and_actor_loss_equal_composed(learn_alpha):
    _need_gpu()
    from functools import reduce
    from ttrl_b200.algos import sac
    from ttrl_b200.engine import ops
    rng = np.random.default_rng(7)
    mean, raw, noise, obs = _policy_inputs(rng)
    low, high = np.array([-1.0, -2.0, 0.0]), np.array([1.0, 0.5, 3.0])
    dist = sac.SquashedGaussian(low, high, "cuda")
    ws = [rng.standard_normal((OBS + D, 1)) * 0.3 for _ in range(2)]
    la0 = np.array([[np.log(0.2)]])
    H = -3.0

    # composed (the reference's op sequence)
    m1, r1, la1 = _T(mean, True), _T(raw, True), _T(la0, True)
    log_std = ops.clamp(r1, -20.0, 2.0)
    action, logp1 = dist.sample(m1, log_std, _T(noise))
    joint1 = ops.concat([_T(obs), action], dim=-1)
    q1 = [ops.linear(joint1, _T(w), None) for w in ws]
    alpha = ops.exp(la1.detach())
    loss1 = ops.mean_all(ops.sub(ops.mul(logp1, alpha), reduce(ops.minimum, q1)))
    loss1.backward()
    if learn_alpha:
        dual1 = sac.alpha_loss(la1, logp1, H)
        dual1.backward()

    # fused
    m2, r2, la2 = _T(mean, True), _T(raw, True), _T(la0, True)
    scale = dist.scale
    joint2, logp2, _ = ops.sac_sample(m2, r2, _T(noise), scale._scale.data.reshape(-1),
                                      scale._centre.data.reshape(-1), scale.log_det,
                                      log_std_min=-20.0, log_std_max=2.0, obs=_T(obs))
    q2 = [ops.linear(joint2, _T(w), None) for w in ws]
    loss2, dual2 = ops.sac_actor_loss(q2, logp2, la2, H, learn_alpha=learn_alpha)
    loss2.backward()
    if learn_alpha:
        dual2.backward()

    assert np.array_equal(joint1.numpy(), joint2.numpy())
    assert np.array_equal(logp1.numpy(), logp2.numpy())
    assert rel(loss2.numpy(), loss1.numpy()) <= 1e-6
    g = lambda t: t.grad.detach().cpu().numpy()
    assert rel(g(m2), g(m1)) <= 1e-5
    assert rel(g(r2), g(r1)) <= 1e-5
    # beyond a bound the raw log-std gets no gradient
    assert g(r2)[0, 0] == 0.0 and g(r2)[1, 1] == 0.0 and g(r2)[2, 2] == 0.0
    if learn_alpha:
        assert rel(dual2.numpy(), dual1.numpy()) <= 1e-6
        assert rel(g(la2), g(la1)) <= 1e-6
    else:
        assert dual2 is None


@pytest.mark.parametrize("prioritized", [False, True])
def test_fused_critic_loss_equals_composed(prioritized):
    _need_gpu()
    from functools import reduce
    from ttrl_b200.algos import sac
    from ttrl_b200.engine import ops
    from ttrl_b200.engine.autograd import no_grad
    rng = np.random.default_rng(11)
    q = [rng.standard_normal((B, 1)) for _ in range(2)]
    qt = [rng.standard_normal((B, 1)) for _ in range(2)]
    qt[1][:8] = qt[0][:8]  # ties in the target minimum
    next_logp = rng.standard_normal((B, 1)) * 2.0
    rewards = rng.standard_normal((B, 1))
    dones = (rng.random((B, 1)) < 0.1).astype(np.float64)
    disc = np.full((B, 1), 0.99)
    w = rng.random((B, 1)) + 0.5
    la = np.array([[np.log(0.3)]])

    # composed (ttrl/algos/sac/losses.py:46-76 through the generic ops)
    qa = [_T(v, True) for v in q]
    with no_grad():
        alpha = ops.exp(_T(la))
        soft = ops.sub(reduce(ops.minimum, [_T(v) for v in qt]), ops.mul(_T(next_logp), alpha))
        target1 = ops.add(_T(rewards), ops.mul(ops.apply_done_mask(soft, _T(dones)), _T(disc)))
    errors = [ops.sub(v, target1) for v in qa]
    squared = [ops.square(e) for e in errors]
    if prioritized:
        squared = [ops.mul(t, _T(w)) for t in squared]
    loss1 = ops.mul(reduce(ops.add, [ops.mean_all(t) for t in squared]), 0.5)
    loss1.backward()
    td1 = sac.priority_errors(errors)

    qb = [_T(v, True) for v in q]
    loss2, alpha2, target2, td2 = ops.sac_critic_loss(
        qb, [_T(v) for v in qt], _T(next_logp), _T(la), _T(rewards), _T(dones), _T(disc),
        weights=_T(w) if prioritized else None, want_td_abs=prioritized)
    loss2.backward()

    assert np.array_equal(alpha2.numpy(), alpha.numpy())
    assert np.array_equal(target2.numpy(), target1.numpy())
    assert rel(loss2.numpy(), loss1.numpy()) <= 1e-6
    for a, b in zip(qa, qb):
        assert np.array_equal(b.grad.cpu().numpy(), a.grad.cpu().numpy())
    if prioritized:
        assert np.array_equal(td2.numpy(), td1.numpy())
    else:
        assert td2 is None


def _learner(seed, fused, obs_dim=11, act_dim=3, batch=256):
    from ttrl_b200.algos.sac import SACLearner
    from ttrl_b200.nets import build_sac_nets
    np.random.seed(seed)
    nets = build_sac_nets(obs_dim, act_dim, "cuda", batch=batch)
    return SACLearner(nets, -np.ones(act_dim), np.ones(act_dim), batch, obs_dim, "cuda",
                      fused=fused)


def _batch(rng, b=256, obs_dim=11, act_dim=3):
    return dict(obs=rng.standard_normal((b, obs_dim)), next_obs=rng.standard_normal((b, obs_dim)),
                actions=np.tanh(rng.standard_normal((b, act_dim))),
                rewards=rng.standard_normal((b, 1)), dones=(rng.random((b, 1)) < 0.05) * 1.0,
                discounts=np.full((b, 1), 0.99), noise=rng.standard_normal((b, act_dim)),
                next_noise=rng.standard_normal((b, act_dim)))


def _params(learner):
    nets = learner.nets
    return [p.data.detach().cpu().numpy().copy()
            for p in (nets.critic_parameters() + nets.policy_parameters()
                      + list(nets.targets.parameters()) + [learner.log_alpha])]


def test_sac_learner_fused_equals_composed():
    """Two whole updates, graph-replayed, on the fused heads and on the
    composed ops from the same weights: metrics to 1e-5, every parameter to
    1e-5 relative; and the fused update's launch count."""
    _need_gpu()
    rng = np.random.default_rng(3)
    batches = [_batch(rng) for _ in range(2)]
    composed, fused = _learner(21, False), _learner(21, True)
    assert fused.fused and not composed.fused
    for b in batches:
        for learner in (composed, fused):
            learner.load_batch(**b)
            learner.replay()
        mc, mf = composed.read_metrics(), fused.read_metrics()
        for key in ("critic_loss", "actor_loss", "alpha_loss", "alpha", "critic_grad_sq",
                    "actor_grad_sq", "q_target", "logp"):
            assert rel(mf[key], mc[key]) <= 1e-5, (key, mf[key], mc[key])
    for pc, pf in zip(_params(composed), _params(fused)):
        assert rel(pf, pc) <= 1e-5
    print(f"launches per update: fused {fused.launches_per_replay}, "
          f"composed {composed.launches_per_replay}", file=sys.stderr)
    assert fused.launches_per_replay <= 60
    assert fused.launches_per_replay * 3 < composed.launches_per_replay
    composed.close()
    fused.close()
