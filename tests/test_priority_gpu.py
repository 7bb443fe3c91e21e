"""Prioritized replay with the priority table on the device.

* `DevicePrioritySampler` through the scripted sequence of the reference's
  own PrioritySampler (golden vectors): the table after each write-back
  (including a column drawn twice, where the last value wins) and after a
  fresh write to 1e-15 relative (CUDA's and the C library's pow may differ in
  the last bit), the running maximum exactly, and both draws (lanes, run
  positions, importance-sampling weights) with the same seeded generators.
* The DQN write-back: a prioritized update's |TD| errors go from the loss
  kernel's device output into the table with no host read, and equal the
  priorities written from the host copy of the same errors.
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


def test_device_sampler_matches_reference_sampler():
    _need_gpu()
    from ttrl_b200.algos.priority import DevicePrioritySampler, PriorityConfig, Window
    d = np.load(os.path.join(GOLDEN, "priority_replay.npz"))
    s = DevicePrioritySampler(PriorityConfig(alpha=0.6, epsilon=1e-6), lanes=3, columns=40,
                              device="cuda")
    lanes = np.repeat(np.arange(3), 40)
    cols = np.tile(np.arange(40), 3)
    s.on_write(lanes, cols)
    for phase in range(2):
        s.update(d[f"u{phase}_lanes"], d[f"u{phase}_cols"], d[f"u{phase}_td"])
        st = s.state()
        assert rel(st["weight"], d[f"u{phase}_weight"]) <= 1e-15
        assert st["max_priority"] == float(d[f"u{phase}_max"])
    s.on_write([1], [7])
    assert rel(s.state()["weight"], d["fresh_weight"]) <= 1e-15
    window = Window(counts=d["window_counts"], start=d["window_start"], capacity=40)
    for k in range(2):
        got = s.draw(np.random.default_rng(1300 + k), window, batch_size=64,
                     beta=float(d[f"d{k}_beta"]))
        assert np.array_equal(got.lanes, d[f"d{k}_lanes"])
        assert np.array_equal(got.offsets, d[f"d{k}_offsets"])
        assert rel(got.weights, d[f"d{k}_weights"]) <= 1e-6
    s.ctx.check_status()


def test_dqn_td_errors_write_back_without_a_host_read():
    _need_gpu()
    from tests.helpers import dqn_batch
    from ttrl_b200.algos import dqn
    from ttrl_b200.algos.priority import DevicePrioritySampler, PriorityConfig
    from ttrl_b200.engine.optim import Adam
    from ttrl_b200.engine.step import TrainStep
    from ttrl_b200.nets import build_q_net
    np.random.seed(2)
    online = build_q_net((4, 84, 84), 6, "cuda", batch=32)
    target = build_q_net((4, 84, 84), 6, "cuda", batch=32)
    opt = Adam(list(online.parameters()), lr=1e-4, eps=1.5e-4)
    inputs = dqn.step_inputs((4, 84, 84), "cuda", batch=32, num_actions=6, prioritized=True)
    step = TrainStep(lambda i: dqn.update_loss(online, target, i, num_actions=6,
                                               prioritized=True), inputs, "cuda",
                     optimizer=opt, mode="traced_fwd_bwd")
    rng = np.random.default_rng(6)
    obs, next_obs, act, rewards, dones, discounts = dqn_batch(rng)
    for k, v in (("obs", obs), ("next_obs", next_obs),
                 ("actions_onehot", np.eye(6, dtype=np.float32)[act]),
                 ("rewards", rewards.reshape(-1, 1)), ("dones", dones.reshape(-1, 1)),
                 ("discounts", discounts.reshape(-1, 1)),
                 ("is_weights", rng.random((32, 1)).astype(np.float32))):
        step.load_input(k, v)
    metrics = step.run()
    td_dev = step._pack.sources["td_abs"].data  # the loss kernel's output, on the device
    lanes = rng.integers(0, 2, 32)
    cols = rng.integers(0, 100, 32)
    a = DevicePrioritySampler(PriorityConfig(), lanes=2, columns=100, device="cuda")
    b = DevicePrioritySampler(PriorityConfig(), lanes=2, columns=100, device="cuda")
    a.update(lanes, cols, td_dev)
    b.update(lanes, cols, np.asarray(metrics["td_abs"]).reshape(-1))
    assert np.array_equal(a.state()["weight"], b.state()["weight"])
    assert a.state()["max_priority"] == b.state()["max_priority"]
    step.close()
