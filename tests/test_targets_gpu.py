"""Target-network updates on the B200: the multi-tensor blend kernel behind
the DQN hard copy (ttrl/algos/dqn/agent.py:205-208 ->
ttrl/engine/nn/module.py:164-189) and SAC's Polyak averaging
(ttrl/algos/sac/targets.py:45-96), and the DQN learner's
`target_sync_interval` schedule.

The copy is bit-exact by definition. The Polyak blend is checked bit-exact
against the reference's two rounded operations, add(mul(t, 1-tau),
mul(c, tau)), evaluated in float32 by numpy.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

SIZES = (1, 3, 4, 4095, 4097, 10_001, 1_687_206 // 7)


def _pairs(rng, dev, offset):
    dst, src = [], []
    for n in SIZES:
        # An offset of one float leaves the views 4-byte but not 16-byte
        # aligned, so the kernel's scalar path runs too.
        d = torch.from_numpy(rng.standard_normal(n + offset).astype(np.float32)).to(dev)
        s = torch.from_numpy(rng.standard_normal(n + offset).astype(np.float32)).to(dev)
        dst.append(d[offset:])
        src.append(s[offset:])
    return dst, src


@pytest.mark.parametrize("offset", [0, 1])
def test_blend_copy_is_bit_exact(offset):
    from ttrl_b200._lib import lib
    from ttrl_b200.device import context
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(5 + offset)
    dst, src = _pairs(rng, dev, offset)
    # Special values travel unchanged.
    src[3][:4] = torch.tensor([float("nan"), float("inf"), -0.0, -float("inf")], device=dev)
    before = lib().ttrl_launch_count()
    context(dev).blend(list(zip(dst, src)))
    assert lib().ttrl_launch_count() - before == 1
    torch.cuda.synchronize()
    for d, s in zip(dst, src):
        assert np.array_equal(d.cpu().numpy().view(np.uint32), s.cpu().numpy().view(np.uint32))


@pytest.mark.parametrize("offset", [0, 1])
def test_blend_polyak_rounds_like_the_reference(offset):
    from ttrl_b200.device import context
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(17 + offset)
    dst, src = _pairs(rng, dev, offset)
    tau = 0.005
    want = []
    for d, s in zip(dst, src):
        dn, sn = d.cpu().numpy(), s.cpu().numpy()
        want.append(dn * np.float32(1.0 - tau) + sn * np.float32(tau))
    context(dev).blend(list(zip(dst, src)), tau)
    torch.cuda.synchronize()
    for d, w in zip(dst, want):
        assert np.array_equal(d.cpu().numpy(), w)


def test_copy_from_refuses_another_network():
    from ttrl_b200.nets import build_q_net
    np.random.seed(0)
    a = build_q_net((4, 84, 84), 6, "cuda", batch=4)
    b = build_q_net((4, 84, 84), 5, "cuda", batch=4)
    with pytest.raises(ValueError, match="copy_from"):
        a.copy_from(b)


def test_dqn_target_sync_interval_schedule():
    """DQNLearner with target_sync_interval = 3 over 7 updates: after
    updates 3 and 6 the target equals the online network bit for bit; in
    between it keeps the last copy."""
    from ttrl_b200.algos.dqn import DQNLearner
    from ttrl_b200.nets import build_q_net
    np.random.seed(1)
    B = 8
    online = build_q_net((4, 84, 84), 6, "cuda", batch=B)
    target = build_q_net((4, 84, 84), 6, "cuda", batch=B)
    learner = DQNLearner(online, target, (4, 84, 84), 6, "cuda", batch=B, lr=1e-3,
                         eps=1.5e-4, target_sync_interval=3)
    state = lambda m: {k: v.copy() for k, v in m.state_dict().items()}  # noqa: E731
    synced = state(online)
    assert all(np.array_equal(v, state(target)[k]) for k, v in synced.items())
    rng = np.random.default_rng(2)
    for update in range(1, 8):
        act = rng.integers(0, 6, B)
        learner.update(obs=rng.integers(0, 256, (B, 4, 84, 84), dtype=np.uint8),
                       next_obs=rng.integers(0, 256, (B, 4, 84, 84), dtype=np.uint8),
                       actions_onehot=np.eye(6, dtype=np.float32)[act],
                       rewards=rng.choice([-1.0, 0.0, 1.0], (B, 1)).astype(np.float32),
                       dones=(rng.random((B, 1)) < 0.1).astype(np.float32),
                       discounts=np.full((B, 1), 0.99, np.float32))
        on, tg = state(online), state(target)
        if update % 3 == 0:
            synced = on
        for k in on:
            assert np.array_equal(tg[k], synced[k]), (update, k)
        if update % 3 != 0:
            # The online network moved on, the target did not.
            assert any(not np.array_equal(on[k], tg[k]) for k in on), update
    assert learner.update_count == 7
    learner.close()
