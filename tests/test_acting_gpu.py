"""The acting forward: one graph replay per acting step of every lane.

* `ttrl_epsilon_greedy` against the reference's host rule
  (ttrl/algos/dqn/agent.py:97-119, ttrl/algos/mask.py:95-110): bit-exact
  actions, ties going to the first maximum, masks honoured on both halves.
* `DQNActor` at an acting width different from the training batch: the
  actions equal the reference's rule applied to the Q values of the same net,
  with the random numbers drawn from the same seeded generator.
* `ttrl_categorical_sample` against the reference's inverse-CDF draw on the
  same log-probs (lanes whose uniform sits within 1e-6 of a CDF boundary are
  skipped: exp may differ by an ulp between numpy and CUDA); deterministic
  mode is the first maximum.
* `PPOActor`: the recorded log-prob is the PPO loss kernel's log-prob of the
  chosen action, bit for bit.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _reference_eps_greedy(q, mask, draws, alt, eps):
    if mask is None:
        greedy = np.argmax(q, axis=-1)
    else:
        greedy = np.argmax(np.where(mask > 0.5, q, -np.inf), axis=-1)
    return np.where(draws < eps, alt, greedy).astype(np.int64)


@pytest.mark.parametrize("masked", [False, True])
def test_epsilon_greedy_kernel_is_the_reference_rule(masked):
    _need_gpu()
    from ttrl_b200.device import context
    ctx = context("cuda")
    rng = np.random.default_rng(3)
    B, A = 300, 7
    q = rng.integers(-3, 4, (B, A)).astype(np.float32)  # many ties
    mask = (rng.random((B, A)) < 0.6).astype(np.float32) if masked else None
    if masked:
        mask[np.arange(B), rng.integers(0, A, B)] = 1.0  # every row has a legal action
    draws = rng.random(B)
    alt = rng.integers(0, A, B)
    out = torch.empty(B, dtype=torch.int32, device="cuda")
    cu = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dt)
    eps = torch.tensor([0.3], dtype=torch.float64, device="cuda")
    ctx.epsilon_greedy(cu(q, torch.float32), None if mask is None else cu(mask, torch.float32),
                       cu(draws, torch.float64), cu(alt, torch.int32), eps, out)
    want = _reference_eps_greedy(q, mask, draws, alt, 0.3)
    assert np.array_equal(out.cpu().numpy(), want)


def test_dqn_actor_matches_reference_acting():
    _need_gpu()
    from ttrl_b200.algos.acting import DQNActor, net_at_batch
    from ttrl_b200.algos.dqn import obs_to_rows
    from ttrl_b200.engine.autograd import Tensor, no_grad
    from ttrl_b200.engine.conv import input_fold
    from ttrl_b200.nets import build_q_net
    np.random.seed(5)
    net = build_q_net((4, 84, 84), 6, "cuda", batch=32)
    lanes = 16
    actor = DQNActor(net, lanes, (4, 84, 84), 6, "cuda")
    rng = np.random.default_rng(8)
    for step in range(3):
        obs = rng.integers(0, 256, (lanes, 4, 84, 84), dtype=np.uint8)
        eps = (0.0, 0.5, 1.0)[step]
        got = actor.act(obs, eps, np.random.default_rng(100 + step))
        view = net_at_batch(net, lanes)
        with no_grad():
            frames = Tensor(torch.from_numpy(obs).cuda())
            q = view(obs_to_rows(frames, input_fold(net))).numpy()
        ref_rng = np.random.default_rng(100 + step)
        draws = ref_rng.random(lanes)
        alt = ref_rng.integers(0, 6, size=lanes)
        assert np.array_equal(got, _reference_eps_greedy(q, None, draws, alt, eps)), step
    actor.close()


def test_categorical_sample_kernel_is_the_reference_draw():
    _need_gpu()
    from ttrl_b200.device import context
    from ttrl_b200.engine.autograd import Tensor
    from ttrl_b200.engine.ops import log_softmax
    ctx = context("cuda")
    rng = np.random.default_rng(11)
    B, A = 512, 6
    logits = (rng.standard_normal((B, A)) * 2.0).astype(np.float32)
    u = rng.random(B)
    dl = torch.from_numpy(logits).cuda()
    act = torch.empty(B, dtype=torch.int32, device="cuda")
    logp = torch.empty(B, dtype=torch.float32, device="cuda")
    ctx.categorical_sample(dl, torch.from_numpy(u).cuda(), act, logp)
    lp_all = log_softmax(Tensor(dl), dim=-1).numpy()
    probs = np.exp(lp_all)
    probs = probs / probs.sum(axis=-1, keepdims=True)
    cdf = np.cumsum(probs, axis=-1)
    want = np.clip((u[:, None] > cdf).sum(axis=-1), 0, A - 1)
    clear = np.abs(u[:, None] - cdf).min(axis=-1) > 1e-6
    got = act.cpu().numpy()
    assert clear.sum() > 0.9 * B
    assert np.array_equal(got[clear], want[clear])
    assert np.allclose(logp.cpu().numpy(), lp_all[np.arange(B), got], rtol=0, atol=1e-6)
    ctx.categorical_sample(dl, None, act, logp)
    assert np.array_equal(act.cpu().numpy(), np.argmax(lp_all, axis=-1))


def test_ppo_actor_logp_is_the_loss_logp():
    _need_gpu()
    from ttrl_b200.algos.acting import PPOActor, net_at_batch
    from ttrl_b200.algos.dqn import obs_to_rows
    from ttrl_b200.engine.autograd import Tensor, no_grad
    from ttrl_b200.engine.conv import input_fold
    from ttrl_b200.engine.ops import ppo_objective
    from ttrl_b200.nets import build_actor_critic
    np.random.seed(6)
    net = build_actor_critic((4, 84, 84), 6, "cuda", batch=64)
    lanes = 8
    actor = PPOActor(net, lanes, (4, 84, 84), 6, "cuda")
    rng = np.random.default_rng(2)
    obs = rng.integers(0, 256, (lanes, 4, 84, 84), dtype=np.uint8)
    actions, logp, values = actor.act(obs, np.random.default_rng(5))
    det, _, _ = actor.act(obs, deterministic=True)
    view = net_at_batch(net, lanes)
    with no_grad():
        logits, value = view(obs_to_rows(Tensor(torch.from_numpy(obs).cuda()), input_fold(net)))
    z = torch.zeros(lanes, device="cuda")
    acts = torch.from_numpy(actions.astype(np.int32)).cuda()
    _, _, new_logp = ppo_objective(logits, value, acts, z, z, z, z, clip_eps=0.1,
                                   value_clip_eps=0.1, value_coef=0.5, entropy_coef=0.01)
    assert np.array_equal(logp, new_logp.numpy().reshape(-1))
    assert np.array_equal(values, value.numpy().reshape(-1))
    assert np.array_equal(det, np.argmax(logits.numpy(), axis=-1))
    actor.close()
