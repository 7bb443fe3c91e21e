"""Recurrent PPO on the B200 kernels.

* One minibatch (MLP trunk -> fused GRU unroll with resets inside the
  sequences -> heads, zeroed padding fields, masked-mean objective, BPTT)
  against golden vectors from the reference's own RecurrentRuntime.forward +
  objective (tests/golden/make_golden.py): loss parts and every parameter
  gradient to 1e-4 relative (split-TF32 GEMMs).
* The training unroll against T acting steps of the cell from a carried
  state, with a reset strictly inside the sequence (the property of the
  reference's tests/hardware/test_recurrent_policy.py:43-95).
* The graph-replayed RecurrentPPOLearner: replay equals the same update run op
  by op, bit for bit; and a whole rollout update (two epochs of sequence
  minibatches, clip, Adam) against the oracle's sequence of steps on the same
  sequence permutations: metrics to 1e-4, parameters to 1e-3 (Adam moves
  near-zero-gradient elements by about lr whatever their sign, which
  dominates this measure).
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


def _vector_net(d, a, hidden, trunk=(16,), batch=24, seed=0):
    from ttrl_b200.nets import build_recurrent_actor_critic
    np.random.seed(seed)
    return build_recurrent_actor_critic((d,), a, "cuda", batch=batch, hidden_size=hidden,
                                        hidden=trunk)


def test_recurrent_minibatch_matches_reference_golden():
    _need_gpu()
    from ttrl_b200.engine.autograd import Tensor
    from ttrl_b200.engine.ops import ppo_objective
    from ttrl_b200.nets.recurrent import ACTOR
    g = np.load(os.path.join(GOLDEN, "recurrent_ppo.npz"))
    T, S, _ = g["starts"].shape
    rows, D = g["obs"].shape
    H = g["h0"].shape[1]
    A = g["logits"].shape[1]
    net = _vector_net(D, A, H)
    net.load_state_dict({k[len("param."):]: g[k] for k in g.files
                         if k.startswith("param.")})
    cu = lambda a, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dt)
    keep = g["valid"].astype(np.float32)
    logits, value = net(Tensor(cu(g["obs"])), {ACTOR: Tensor(cu(g["h0"]))},
                        Tensor(cu(g["starts"])), seq_len=T)
    loss, parts, new_logp = ppo_objective(
        logits, value, cu(g["actions"], torch.int32), cu(g["old_logp"] * keep),
        cu(g["advantages"] * keep), cu(g["returns"] * keep), cu(g["values"]),
        clip_eps=0.1, value_clip_eps=0.1, value_coef=0.5, entropy_coef=0.01, valid=cu(keep))
    loss.backward()
    assert rel(logits.numpy(), g["logits"]) <= 1e-4
    assert rel(value.numpy(), g["value"]) <= 1e-4
    assert rel(loss.numpy(), g["loss"]) <= 1e-4
    for k in ("policy_loss", "value_loss", "entropy"):
        assert rel(parts[k].numpy(), g[k]) <= 1e-4, k
    names = set()
    for name, p in net.named_parameters():
        names.add(name)
        assert rel(p.grad.detach().cpu().numpy(), g["grad." + name]) <= 1e-4, name
    assert names == {k[len("grad."):] for k in g.files if k.startswith("grad.")}


def test_unroll_equals_acting_steps_with_a_reset_inside():
    _need_gpu()
    from ttrl_b200.engine.autograd import Tensor, no_grad
    from ttrl_b200.nets.recurrent import ACTOR
    seq_len, hidden, obs_dim, reset_at = 4, 7, 5, 2
    net = _vector_net(obs_dim, 6, hidden, trunk=(32, 32), batch=seq_len, seed=3)
    rng = np.random.default_rng(17)
    rows = rng.normal(size=(seq_len, obs_dim)).astype(np.float32)
    starts = np.zeros(seq_len, np.float32)
    starts[reset_at] = 1.0
    h0 = rng.normal(size=(1, hidden)).astype(np.float32)
    cu = lambda a: Tensor(torch.from_numpy(np.ascontiguousarray(a)).cuda())
    acted = []
    h = cu(h0)
    with no_grad():
        for t in range(seq_len):
            logits, value, nxt = net.step(cu(rows[t:t + 1]), {ACTOR: h},
                                          {ACTOR: cu(starts[t:t + 1].reshape(1, 1))})
            acted.append((logits.numpy()[0].copy(), float(value.numpy().reshape(-1)[0])))
            h = nxt[ACTOR]
        logits, value = net(cu(rows), {ACTOR: cu(h0)}, cu(starts.reshape(seq_len, 1, 1)),
                            seq_len=seq_len)
    ul, uv = logits.numpy(), value.numpy().reshape(-1)
    spread = float(np.abs(np.diff([r for r, _ in acted], axis=0)).max())
    assert spread > 1e-4
    for t, (lr, vr) in enumerate(acted):
        assert np.allclose(lr, ul[t], atol=1e-5, rtol=1e-5), t
        assert abs(uv[t] - vr) <= 1e-5, t


def _vector_rollout(rng, n_steps, n_envs, d, a, hidden, n_chunks):
    from ttrl_b200.algos.recurrent_ppo import shift_to_starts
    shape = (n_steps, n_envs)
    boundary = (rng.random(shape) < 0.1).astype(np.float32)
    return dict(
        obs=rng.standard_normal(shape + (d,)).astype(np.float32),
        actions=rng.integers(0, a, shape),
        old_logp=(np.log(1.0 / a) + 0.2 * rng.standard_normal(shape)).astype(np.float32),
        values=rng.standard_normal(shape).astype(np.float32),
        returns=rng.standard_normal(shape).astype(np.float32),
        advantages=rng.standard_normal(shape).astype(np.float32),
        starts=shift_to_starts(boundary, np.ones(n_envs)),
        hidden=(0.5 * rng.standard_normal((n_chunks, n_envs, hidden))).astype(np.float32),
        valid=(rng.random(shape) < 0.9).astype(np.float32))


def _learner(seed, cfg, n_steps, n_envs, d, a, hidden, seq_len):
    from ttrl_b200.algos.recurrent_ppo import RecurrentPPOLearner
    net = _vector_net(d, a, hidden, batch=cfg.minibatch_size, seed=seed)
    return RecurrentPPOLearner(net, n_steps, n_envs, (d,), "cuda", cfg=cfg, seq_len=seq_len,
                               seed=7)


def test_recurrent_learner_replay_equals_eager_and_oracle():
    _need_gpu()
    from ttrl_b200.algos.ppo import PPOConfig
    from ttrl_b200.algos.recurrent_ppo import normalize_valid_advantages, sequence_rows
    from oracle.recurrent import recurrent_ppo_step
    n_steps, n_envs, d, a, hidden, seq_len = 12, 4, 9, 5, 8, 6
    cfg = PPOConfig(epochs=2, minibatch_size=12)
    rng = np.random.default_rng(31)
    ro = _vector_rollout(rng, n_steps, n_envs, d, a, hidden, n_steps // seq_len)
    eager = _learner(5, cfg, n_steps, n_envs, d, a, hidden, seq_len)
    graph = _learner(5, cfg, n_steps, n_envs, d, a, hidden, seq_len)
    init = {k: v.astype(np.float64) for k, v in eager.net.state_dict().items()}
    for lrn in (eager, graph):
        lrn.load_rollout(**ro)
        lrn.draw_permutations()
    eager.update_eager()
    graph.replay()
    torch.cuda.synchronize()
    assert graph.launches_per_replay > 0
    for (n1, p1), (_, p2) in zip(eager.net.named_parameters(), graph.net.named_parameters()):
        assert np.array_equal(p1.data.cpu().numpy(), p2.data.cpu().numpy()), n1
    got = graph.read_metrics()
    assert got["minibatches"] == 8

    # oracle: the same sequence minibatches in the same order, float64
    valid = ro["valid"].reshape(-1).astype(np.float64)
    adv = normalize_valid_advantages(ro["advantages"], ro["valid"]).reshape(-1)
    flat = {k: np.asarray(ro[k]).reshape((n_steps * n_envs,) + np.shape(ro[k])[2:])
            for k in ("obs", "actions", "old_logp", "values", "returns", "starts")}
    hid = ro["hidden"].reshape(-1, hidden).astype(np.float64)
    params, state, losses = init, {}, []
    for t in range(graph.steps_per_update):
        slots, ids = graph.minibatch_slots(t)
        assert np.array_equal(slots, sequence_rows(ids, n_envs, seq_len))
        m, params, state = recurrent_ppo_step(
            params, state, t + 1, flat["obs"][slots].astype(np.float64), hid[ids],
            flat["starts"][slots].reshape(seq_len, -1, 1).astype(np.float64), valid[slots],
            flat["actions"][slots], flat["old_logp"][slots].astype(np.float64),
            flat["values"][slots].astype(np.float64), adv[slots].astype(np.float64),
            flat["returns"][slots].astype(np.float64), seq_len=seq_len, lr=cfg.lr,
            eps=cfg.eps, max_grad_norm=cfg.max_grad_norm)
        losses.append(m["loss"])
    assert rel(got["loss"], np.mean(losses)) <= 1e-4
    sd = graph.net.state_dict()
    for name in sd:
        assert rel(sd[name], params[name]) <= 1e-3, name
    for lrn in (eager, graph):
        lrn.close()


def test_recurrent_learner_refuses_bad_shapes():
    _need_gpu()
    from ttrl_b200.algos.ppo import PPOConfig
    with pytest.raises(ValueError, match="does not divide"):
        _learner(1, PPOConfig(minibatch_size=12), 10, 4, 3, 2, 4, 6)
    with pytest.raises(ValueError, match="not a multiple of seq_len"):
        _learner(1, PPOConfig(minibatch_size=10), 12, 4, 3, 2, 4, 6)
    with pytest.raises(ValueError, match="zero minibatches"):
        _learner(1, PPOConfig(minibatch_size=60), 12, 4, 3, 2, 4, 6)
