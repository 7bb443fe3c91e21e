"""On-device rollout post-processing (ttrl/buffers/rollout.py:195-283).

* `ttrl_gae` against golden vectors from the reference's own
  RolloutBuffer.compute_gae (terminations and autoreset padding slots):
  bit-exact, the kernel performs the reference's float32 operations in order.
* `ttrl_normalize_advantages` against the reference's normalisation over
  valid slots: 1e-6 relative (statistics in double here, float32 pairwise
  sums in numpy).
* `PPOLearner.load_rollout_raw`: GAE and normalisation on the device feed the
  same minibatches as the host path would, and only valid slots are drawn.
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


@pytest.mark.parametrize("case", [0, 1])
def test_gae_and_normalisation_match_reference(case):
    _need_gpu()
    from ttrl_b200.device import context
    d = np.load(os.path.join(GOLDEN, "rollout_gae.npz"))
    g = {k[3:]: d[k] for k in d.files if k.startswith(f"c{case}_")}
    gamma, lam = (float(v) for v in g["gamma_lam"])
    ctx = context("cuda")
    cu = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    T, E = g["values"].shape
    adv = torch.empty((T, E), device="cuda")
    ret = torch.empty((T, E), device="cuda")
    valid = cu(g["valid"])
    ctx.gae(cu(g["rewards"]), cu(g["values"]), cu(g["dones"]), valid, cu(g["last_values"]),
            adv, ret, gamma, lam)
    assert np.array_equal(adv.cpu().numpy(), g["advantages"])
    assert np.array_equal(ret.cpu().numpy(), g["returns"])
    out = torch.empty_like(adv)
    ctx.normalize_advantages(adv, valid, out)
    ctx.check_status()
    keep = g["valid"].reshape(-1) > 0
    assert rel(out.cpu().numpy().reshape(-1)[keep], g["normalized_valid"]) <= 1e-6


def test_learner_raw_rollout_uses_device_gae_and_valid_slots():
    _need_gpu()
    from oracle import rollout as ro
    from ttrl_b200.algos.ppo import PPOConfig, PPOLearner
    from ttrl_b200.nets import build_actor_critic
    np.random.seed(3)
    T, E, mb = 32, 4, 32
    cfg = PPOConfig(epochs=2, minibatch_size=mb)
    net = build_actor_critic((4, 84, 84), 6, "cuda", batch=mb)
    rng = np.random.default_rng(4)
    valid = (rng.random((T, E)) > 0.05).astype(np.float32)
    kept = int(valid.sum())
    learner = PPOLearner(net, T * E, (4, 84, 84), "cuda", cfg=cfg, seed=9,
                         minibatches=kept // mb)
    obs = rng.integers(0, 256, (T, E, 4, 84, 84), dtype=np.uint8)
    rewards = rng.standard_normal((T, E)).astype(np.float32)
    values = rng.standard_normal((T, E)).astype(np.float32)
    dones = (rng.random((T, E)) < 0.05).astype(np.float32)
    last = rng.standard_normal(E).astype(np.float32)
    learner.load_rollout_raw(obs, rng.integers(0, 6, (T, E)),
                             rng.standard_normal((T, E)).astype(np.float32), values, rewards,
                             dones, last, valid=valid)
    adv, ret = ro.gae(rewards, values, dones, valid, last, cfg.gamma, cfg.lam)
    assert np.array_equal(learner.returns.cpu().numpy().reshape(T, E), ret)
    keep = np.flatnonzero(valid.reshape(-1) > 0)
    got = learner.advantages.cpu().numpy().reshape(-1)[keep]
    assert rel(got, ro.normalize(adv, valid)) <= 1e-6
    learner.draw_permutations()
    slots = learner.perm_host.numpy()
    assert np.isin(slots, keep).all()
    # the draw is the reference's: a permutation of the valid slots per epoch
    rng2 = np.random.default_rng(9)
    want = np.concatenate([keep[rng2.permutation(len(keep))[:learner.minibatches * mb]]
                           for _ in range(cfg.epochs)])
    assert np.array_equal(slots.reshape(-1), want)
    learner.close()
