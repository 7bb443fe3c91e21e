"""SAC on the B200 kernels.

* The losses and the squashed Gaussian against golden vectors from the
  reference's own ttrl/algos/sac code (tests/golden/make_golden.py): preset
  policy outputs and critics linear in the action, so the loss algebra and
  every gradient path through the reparameterised sample are pinned.
  Tolerance 1e-5 relative (fp32 exp/log/tanh chains).
* The graph-replayed SACLearner: one whole update (critic region, critic
  Adam, actor + temperature region, two Adams, Polyak) replayed from a CUDA
  graph equals the same update run op by op, and the targets move by the
  Polyak rule.
"""

import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.helpers import rel  # noqa: E402

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


class _Policy:
    def __init__(self, cur, nxt):
        self.cur, self.nxt = cur, nxt

    def __call__(self, obs):
        return self.nxt if obs == "next" else self.cur


class _LinearCritic:
    def __init__(self, w, s_cur, s_next):
        self.w, self.s_cur, self.s_next = w, s_cur, s_next

    def __call__(self, obs, action):
        from ttrl_b200.engine.ops import add, mul, sum_dim
        feat = self.s_next if obs == "next" else self.s_cur
        return add(sum_dim(mul(action, self.w), dim=-1, keepdim=True), feat)


@pytest.mark.parametrize("name", ["uniform", "prioritized"])
def test_sac_losses_match_reference(name):
    _need_gpu()
    from types import SimpleNamespace
    from ttrl_b200.algos import sac
    from ttrl_b200.engine.autograd import Tensor
    from ttrl_b200.engine.ops import exp
    d = np.load(os.path.join(GOLDEN, "sac_losses.npz"))
    g = {k[len(name) + 1:]: d[k] for k in d.files if k.startswith(name + "_")}
    T = lambda a, grad=False: Tensor.from_numpy(np.ascontiguousarray(a), "cuda", requires_grad=grad)
    dist = sac.SquashedGaussian(g["low"], g["high"], "cuda")
    mean, log_std = T(g["mean"], True), T(g["log_std"], True)
    crit = [_LinearCritic(T(g["q_w"][i], True), T(g["s_feat"][i], True), T(g["s_feat"][2 + i]))
            for i in range(2)]
    targ = [_LinearCritic(T(g["q_w"][2 + i]), T(g["s_feat"][4 + i]), T(g["s_feat"][6 + i]))
            for i in range(2)]
    nets = SimpleNamespace(policy=_Policy((mean, log_std), (T(g["mean_next"]),
                                                            T(g["log_std_next"]))),
                           critics=crit, targets=targ)
    batch = sac._Batch(rewards=T(g["rewards"]), dones=T(g["dones"]), discounts=T(g["discounts"]),
                       actions=T(g["actions"]), noise=T(g["noise"]), next_noise=T(g["next_noise"]))
    batch.obs, batch.next_obs = "cur", "next"
    log_alpha = T(g["log_alpha"], True)
    alpha = exp(log_alpha.detach())
    weights = T(g["is_weights"]) if name == "prioritized" else None
    closs, target, _ = sac.critic_loss(nets, dist, batch, alpha, weights)
    closs.backward()
    assert rel(closs.numpy(), g["critic_loss"]) <= 1e-5
    assert rel(target.numpy(), g["q_target"]) <= 1e-5
    for i in range(2):
        assert rel(crit[i].w.grad.detach().cpu().numpy(), g[f"d_critic{i}_w"]) <= 1e-5
        assert rel(crit[i].s_cur.grad.detach().cpu().numpy(), g[f"d_critic{i}_s"]) <= 1e-5
    for c in crit:
        c.w.requires_grad = False
        c.s_cur.requires_grad = False
    aloss, logp = sac.actor_loss(nets, dist, batch, alpha)
    aloss.backward()
    assert rel(aloss.numpy(), g["actor_loss"]) <= 1e-5
    assert rel(logp.numpy(), g["logp"]) <= 1e-5
    assert rel(mean.grad.detach().cpu().numpy(), g["d_mean"]) <= 1e-5
    assert rel(log_std.grad.detach().cpu().numpy(), g["d_log_std"]) <= 1e-5
    dual = sac.alpha_loss(log_alpha, logp, -3.0)
    dual.backward()
    assert rel(dual.numpy(), g["alpha_loss"]) <= 1e-5
    assert rel(log_alpha.grad.detach().cpu().numpy(), g["d_log_alpha"]) <= 1e-5


def _learner(seed, obs_dim=11, act_dim=3, batch=256):
    from ttrl_b200.algos.sac import SACLearner
    from ttrl_b200.nets import build_sac_nets
    np.random.seed(seed)
    nets = build_sac_nets(obs_dim, act_dim, "cuda", batch=batch)
    low, high = -np.ones(act_dim), np.ones(act_dim)
    return SACLearner(nets, low, high, batch, obs_dim, "cuda")


def _batch(rng, b=256, obs_dim=11, act_dim=3):
    return dict(obs=rng.standard_normal((b, obs_dim)), next_obs=rng.standard_normal((b, obs_dim)),
                actions=np.tanh(rng.standard_normal((b, act_dim))),
                rewards=rng.standard_normal((b, 1)), dones=(rng.random((b, 1)) < 0.001) * 1.0,
                discounts=np.full((b, 1), 0.99), noise=rng.standard_normal((b, act_dim)),
                next_noise=rng.standard_normal((b, act_dim)))


def _state(learner):
    nets = learner.nets
    params = (nets.critic_parameters() + nets.policy_parameters()
              + list(nets.targets.parameters()) + [learner.log_alpha])
    return [p.data.detach().cpu().numpy().copy() for p in params]


def test_sac_learner_graph_replay_equals_eager():
    _need_gpu()
    rng = np.random.default_rng(5)
    batches = [_batch(rng) for _ in range(3)]
    eager, graph = _learner(11), _learner(11)
    for s1, s2 in zip(_state(eager), _state(graph)):
        assert np.array_equal(s1, s2)
    targets_before = [p.data.detach().cpu().numpy().copy()
                      for p in eager.nets.targets.parameters()]
    critics_before = [p.data.detach().cpu().numpy().copy()
                      for p in eager.nets.critics.parameters()]
    for b in batches:
        eager.load_batch(**b)
        eager.update_eager()
        graph.load_batch(**b)
        graph.replay()
    torch.cuda.synchronize()
    for s1, s2 in zip(_state(eager), _state(graph)):
        assert np.array_equal(s1, s2)
    m = graph.read_metrics()
    for k in ("critic_loss", "actor_loss", "alpha_loss", "alpha"):
        assert np.isfinite(m[k]), k
    assert graph.launches_per_replay > 0
    # After the first update the targets are (1 - tau) t + tau c of the
    # critics' post-Adam values: check the rule on a fresh learner.
    one = _learner(11)
    one.load_batch(**batches[0])
    one.update_eager()
    torch.cuda.synchronize()
    for t0, c_new, t_new in zip(targets_before, [p.data.cpu().numpy() for p in
                                                 one.nets.critics.parameters()],
                                [p.data.cpu().numpy() for p in one.nets.targets.parameters()]):
        want = 0.995 * t0.astype(np.float64) + 0.005 * c_new.astype(np.float64)
        assert rel(t_new, want) <= 1e-6
    assert any(not np.array_equal(c0, c1.data.cpu().numpy())
               for c0, c1 in zip(critics_before, one.nets.critics.parameters()))
    eager.close()
    graph.close()
    one.close()


def test_sac_learner_matches_the_reference_update():
    """SACLearner at BASELINE configs[2] (obs 11, actions 3, twin critics and
    actor with 256-wide layers, batch 256, tau 0.005, lr 3e-4, learned
    temperature with target entropy -3), three graph-replayed updates,
    against three updates of the reference's own SAC code
    (tests/golden/sac_update.npz: ttrl/algos/sac/agent.py:218-238 order --
    critic step, then actor and temperature steps, then the Polyak blend).

    Losses to 1e-5 relative. Every parameter (policy, critics, targets,
    log alpha) to 1e-4 relative Frobenius after the three Adam steps: the
    contractions are split-TF32 against the fixture's fp32."""
    _need_gpu()
    from ttrl_b200.algos.sac import SACConfig, SACLearner
    from ttrl_b200.nets import build_sac_nets
    d = np.load(os.path.join(GOLDEN, "sac_update.npz"))
    B, OBS, ACT = 256, 11, 3
    nets = build_sac_nets(OBS, ACT, "cuda", batch=B)
    init = {k[len("init."):]: d[k] for k in d.files
            if k.startswith("init.") and k != "init.log_alpha"}
    nets.load_state_dict(init)
    learner = SACLearner(nets, -np.ones(ACT), np.ones(ACT), B, OBS, "cuda",
                         cfg=SACConfig(init_alpha=0.2, target_entropy=-3.0))
    learner.log_alpha.data.copy_(torch.from_numpy(d["init.log_alpha"]))
    for u in range(3):
        batch = {k.split(".", 1)[1]: d[k] for k in d.files if k.startswith(f"batch{u}.")}
        learner.load_batch(**batch)
        learner.replay()
        got = learner.read_metrics()
        for key in ("critic_loss", "actor_loss", "alpha_loss"):
            want = float(d[f"update{u}.{key}"].reshape(-1)[0])
            assert rel(got[key], want) <= 1e-5, (u, key, got[key], want)
    sd = nets.state_dict()
    assert set(sd) == set(init)
    for name, value in sd.items():
        want = d["final." + name]
        err = np.linalg.norm(value.reshape(want.shape) - want) / np.linalg.norm(want)
        assert err <= 1e-4, (name, err)
    la = learner.log_alpha.numpy().reshape(1, 1)
    assert rel(la, d["final.log_alpha"]) <= 1e-5
    assert learner.critic_opt.steps == [3] * len(learner.critic_opt.params)
    learner.close()
