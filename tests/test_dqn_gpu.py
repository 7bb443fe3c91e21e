"""Nature-DQN batch-32 learner update on the B200 against the oracle
loss, gradients of every parameter and post-Adam
parameters, eager and CUDA-graph-replayed.

Tolerances: loss / mean_q 1e-5 relative; gradients 1e-4 relative Frobenius
(split-TF32; the spec allows 1e-3); post-Adam parameters 1e-6 relative
Frobenius; double-DQN next-action choice bit-exact.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import learner as ref  # noqa: E402
from tests.helpers import (TOL_GRAD, TOL_PARAM, dqn_batch, grads_in_state_layout,
                           nature_state_dict,  # noqa: E402
                           nchw_to_nhwc, rel)

pytestmark = pytest.mark.gpu

LR, EPS = 1e-4, 1.5e-4


def _setup(seed=0, batch=32):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from ttrl_b200.algos import dqn
    from ttrl_b200.engine.optim import Adam
    from ttrl_b200.nets import build_q_net

    rng = np.random.default_rng(seed)
    online_p = ref.nature_params(rng)
    # A jittered copy as the target, so double and vanilla DQN differ.
    target_p = {k: (v + rng.normal(0, 0.01, v.shape)).astype(np.float32)
                for k, v in online_p.items()}
    online = build_q_net((4, 84, 84), 6, "cuda", batch=batch)
    target = build_q_net((4, 84, 84), 6, "cuda", batch=batch)
    online.load_state_dict(nature_state_dict(online_p))
    target.load_state_dict(nature_state_dict(target_p))
    opt = Adam(list(online.parameters()), lr=LR, eps=EPS)
    inputs = dqn.step_inputs((4, 84, 84), "cuda", batch=batch, num_actions=6)
    return rng, online_p, target_p, online, target, opt, inputs


def _load(step, batch):
    obs, next_obs, act, rewards, dones, discounts = batch
    onehot = np.eye(6, dtype=np.float32)[act]
    step.load_input("obs", obs)
    step.load_input("next_obs", next_obs)
    step.load_input("actions_onehot", onehot)
    step.load_input("rewards", rewards.reshape(-1, 1))
    step.load_input("dones", dones.reshape(-1, 1))
    step.load_input("discounts", discounts.reshape(-1, 1))


def _step_fn(online, target):
    from ttrl_b200.algos import dqn
    return lambda inputs: dqn.update_loss(online, target, inputs, num_actions=6, double=True,
                                          huber_delta=1.0)


@pytest.mark.parametrize("precision,mode", [("tf32x3", "eager"), ("tf32", "traced_fwd_bwd")])
def test_dqn_update_matches_oracle(precision, mode):
    """Split-TF32 eagerly at the tolerances above; one TF32 pass replayed
    from the graph (the bench's configuration) at the spec's 1e-3 for TF32
    GEMM paths, the accuracy class of the reference's own HiFi4 matmuls
    (ttrl/engine/ops/matmul.py:14-20), for loss, gradients and post-Adam
    parameters alike."""
    from ttrl_b200.device import context
    ctx = context("cuda") if torch.cuda.is_available() else None
    saved = ctx.precision if ctx else None
    try:
        if ctx:
            ctx.set_precision(precision)
        _dqn_update_check(mode, *((1e-5, 1e-4, TOL_GRAD, TOL_PARAM) if precision == "tf32x3"
                                  else (1e-3, 1e-3, 1e-3, 1e-3)),
                          device_relu=precision == "tf32")
    finally:
        if ctx:
            ctx.precision = saved


def _dqn_update_check(mode, tol_loss, tol_sq, tol_grad, tol_param, device_relu=False):
    from ttrl_b200.engine.step import TrainStep
    rng, online_p, target_p, online, target, opt, inputs = _setup()
    batch = dqn_batch(rng)
    gates = None
    if device_relu:
        # The device's own ReLU masks (before the update changes the weights):
        # at ~1e-4 forward error a pre-activation within rounding of zero may
        # take the other side than in float64, and the oracle follows the
        # device there instead of charging that rank-1 term to the GEMMs.
        from ttrl_b200.engine.autograd import Tensor
        from tests.helpers import device_gates
        x = nchw_to_nhwc(batch[0]).astype(np.float32)
        gates = device_gates(online, Tensor(torch.from_numpy(x.reshape(1, 1, -1, 4)).cuda()))
    step = TrainStep(_step_fn(online, target), inputs, "cuda", optimizer=opt, mode=mode)
    _load(step, batch)
    grads_before = None
    metrics = step.run()
    obs, next_obs, act, rewards, dones, discounts = batch
    f64 = {k: v.astype(np.float64) for k, v in online_p.items()}
    t64 = {k: v.astype(np.float64) for k, v in target_p.items()}
    m, grads, new_p, _ = ref.dqn_update(
        f64, t64, nchw_to_nhwc(obs).astype(np.float64), nchw_to_nhwc(next_obs).astype(np.float64),
        act, rewards.astype(np.float64), dones.astype(np.float64), discounts.astype(np.float64),
        lr=LR, eps=EPS, gates=gates)
    assert rel(metrics["loss"], m["loss"]) <= tol_loss
    # mean Q sits near zero (a mean of mixed-sign values): compare on the
    # scale of the Q values rather than of their mean.
    assert abs(float(metrics["mean_q"].reshape(-1)[0]) - m["mean_q"]) <= tol_loss * 0.1
    assert rel(metrics["grad_sq"], m["grad_sq"]) <= tol_sq
    named_g = nature_state_dict(grads)
    for name, g in grads_in_state_layout(online).items():
        want = named_g[name]
        assert rel(g.reshape(want.shape), want) <= tol_grad, name
    sd = online.state_dict()
    want_p = nature_state_dict(new_p)
    for name in sd:
        assert rel(sd[name], want_p[name]) <= tol_param, name
    step.close()
    del grads_before


def test_dqn_graph_replay_is_bit_identical_to_eager():
    from ttrl_b200.engine.step import TrainStep
    results = {}
    for mode in ("eager", "traced_fwd_bwd"):
        rng, online_p, target_p, online, target, opt, inputs = _setup(seed=3)
        step = TrainStep(_step_fn(online, target), inputs, "cuda", optimizer=opt, mode=mode)
        losses = []
        for _ in range(3):
            _load(step, dqn_batch(rng))
            losses.append(float(step.run()["loss"].reshape(-1)[0]))
        results[mode] = (losses, online.state_dict(), list(opt.steps))
        step.close()
    le, se, ste = results["eager"]
    lg, sg, stg = results["traced_fwd_bwd"]
    assert le == lg
    assert ste == stg == [3] * len(ste)
    for name in se:
        assert np.array_equal(se[name], sg[name]), name


def test_dqn_replays_are_deterministic():
    from ttrl_b200.engine.step import TrainStep
    finals = []
    for _ in range(2):
        rng, online_p, target_p, online, target, opt, inputs = _setup(seed=5)
        step = TrainStep(_step_fn(online, target), inputs, "cuda", optimizer=opt,
                         mode="traced_fwd_bwd")
        for _ in range(4):
            _load(step, dqn_batch(rng))
            step.run()
        finals.append(online.state_dict())
        step.close()
    for name in finals[0]:
        assert np.array_equal(finals[0][name], finals[1][name]), name


def test_dqn_pipelined_metric_reads_match_run():
    """launch + fetch_metrics / metrics_of, with update k+1 enqueued before
    update k's metrics are waited on, reads the same losses as run()."""
    from ttrl_b200.engine.step import TrainStep
    runs = []
    for pipelined in (False, True):
        rng, online_p, target_p, online, target, opt, inputs = _setup(seed=13)
        step = TrainStep(_step_fn(online, target), inputs, "cuda", optimizer=opt,
                         mode="traced_fwd_bwd")
        batches = [dqn_batch(rng) for _ in range(4)]
        losses = []
        if not pipelined:
            for b in batches:
                _load(step, b)
                losses.append(float(step.run()["loss"].reshape(-1)[0]))
        else:
            _load(step, batches[0])
            step.run()  # capture: the first call is a whole step
            losses.append(float(step.metrics()["loss"].reshape(-1)[0]))
            pending = None
            for b in batches[1:]:
                _load(step, b)
                step.launch()
                handle = step.fetch_metrics()
                if pending is not None:
                    losses.append(float(step.metrics_of(pending)["loss"].reshape(-1)[0]))
                pending = handle
            losses.append(float(step.metrics_of(pending)["loss"].reshape(-1)[0]))
        runs.append((losses, online.state_dict()))
        step.close()
    assert runs[0][0] == runs[1][0]
    for name in runs[0][1]:
        assert np.array_equal(runs[0][1][name], runs[1][1][name]), name
