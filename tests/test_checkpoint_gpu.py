"""Resume from, and write back to, a checkpoint the reference wrote.

The file (tests/golden/checkpoint_dqn.npz, made by the reference's own
save_checkpoint) holds a 4x36x36 DQN's online and target nets in logical
OIHW and its Adam moments with each conv weight's in the reference's
prepared matrix. On the device:

* the B200 nets' state_dict names and shapes are the file's;
* after `load_learner`, the B200 forward of the file's online net matches the
  Q values the reference's `ttrl.deploy` export of the same file computes
  (relative 1e-4: split-TF32 contractions against a float32 numpy forward);
* the optimizer's moments come back in OIHW equal to the unpacked prepared
  matrices (relative 1e-6: one division and one multiplication by 1 - beta);
* after one graph-replayed update, `Checkpoint.update` writes a file whose
  members all keep their stored shapes (conv moments prepared, padding zero),
  whose non-agent members are untouched, and from which a second learner
  resumes to the same weights and moments.
"""

from __future__ import annotations

import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from tests.helpers import rel  # noqa: E402

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
OBS = (4, 36, 36)


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _learner(batch):
    from ttrl_b200.engine.optim import Adam
    from ttrl_b200.nets import build_q_net
    online = build_q_net(OBS, 6, "cuda", batch=batch, hidden=16)
    target = build_q_net(OBS, 6, "cuda", batch=batch, hidden=16)
    opt = Adam(list(online.parameters()), lr=1e-4, eps=1.5e-4)
    return online, target, opt


def _q(net, obs):
    from ttrl_b200.algos.acting import net_at_batch
    from ttrl_b200.algos.dqn import obs_to_rows
    from ttrl_b200.engine.autograd import Tensor, no_grad
    from ttrl_b200.engine.conv import input_fold
    view = net_at_batch(net, obs.shape[0])
    with no_grad():
        rows = obs_to_rows(Tensor(torch.from_numpy(obs).cuda()), input_fold(net))
        return view(rows).numpy()


def test_resume_and_write_back_a_reference_checkpoint(tmp_path):
    _need_gpu()
    from ttrl_b200.algos import dqn
    from ttrl_b200.checkpoint import Checkpoint, load_learner
    from ttrl_b200.engine.packing import solve_cp
    from ttrl_b200.engine.step import TrainStep
    g = np.load(os.path.join(GOLDEN, "checkpoint_dqn.npz"))
    src = tmp_path / "ref.npz"
    src.write_bytes(g["ref_file"].tobytes())
    ck = Checkpoint.read(str(src))
    state = ck.agent_state()

    batch = 4
    online, target, opt = _learner(batch)
    mine = online.state_dict()
    assert sorted(mine) == sorted(state["online"])
    for k, a in mine.items():
        assert a.shape == state["online"][k].shape and a.dtype == np.float32, k
    load_learner(state, online=online, target=target, optimizer=opt)

    q = _q(online, g["obs"])
    assert rel(q, g["deploy_q"]) <= 1e-4

    restored = opt.state_dict()
    assert restored["t"] == 7 and restored["steps"] == [7] * 10
    for i, (m, v) in enumerate(zip(state["optimizer"]["m"], state["optimizer"]["v"])):
        got_m, got_v = restored["m"][i], restored["v"][i]
        if m.shape != got_m.shape:  # prepared in the file, OIHW here
            lay = solve_cp(m.shape, got_m.shape, v=v)
            m, v = lay.unpack(m), lay.unpack(v)
        assert rel(got_m, m) <= 1e-6 and rel(got_v, v) <= 1e-6, i

    rng = np.random.default_rng(4)
    inputs = dqn.step_inputs(OBS, "cuda", batch=batch, num_actions=6)
    step = TrainStep(lambda i: dqn.update_loss(online, target, i, num_actions=6), inputs,
                     "cuda", optimizer=opt, mode="traced_fwd_bwd")
    act = rng.integers(0, 6, batch)
    for k, v in (("obs", rng.integers(0, 256, (batch,) + OBS, dtype=np.uint8)),
                 ("next_obs", rng.integers(0, 256, (batch,) + OBS, dtype=np.uint8)),
                 ("actions_onehot", np.eye(6)[act]),
                 ("rewards", np.array([[1.0], [0.0], [-1.0], [0.0]], np.float32)),
                 ("dones", np.zeros((batch, 1), np.float32)),
                 ("discounts", np.full((batch, 1), 0.99, np.float32))):
        step.load_input(k, v)
    step.run()
    torch.cuda.synchronize()
    step.close()
    assert opt.t == 8

    out = tmp_path / "ours.npz"
    ck.update(online=online, target=target, optimizer=opt, frame=3200).write(str(out))
    with np.load(str(src)) as a, np.load(str(out)) as b:
        assert sorted(a.files) == sorted(b.files)
        for k in a.files:
            if k == "__meta__":
                continue
            assert a[k].shape == b[k].shape and a[k].dtype == b[k].dtype, k
            if not k.startswith("state."):
                assert np.array_equal(a[k], b[k]), k
    back = Checkpoint.read(str(out))
    assert back.meta["frame"] == 3200
    tree = back.agent_state()
    assert tree["optimizer"]["t"] == 8
    names = list(state["online"])
    for i, m in enumerate(tree["optimizer"]["m"]):
        oihw = state["online"][names[i]].shape
        assert m.shape == state["optimizer"]["m"][i].shape, names[i]
        if m.shape != oihw:
            lay = solve_cp(m.shape, oihw, v=tree["optimizer"]["v"][i])
            assert lay.padding_is_zero(m) and lay.padding_is_zero(tree["optimizer"]["v"][i])
    for k, a in online.state_dict().items():
        assert np.array_equal(tree["online"][k], a), k

    online2, target2, opt2 = _learner(batch)
    load_learner(tree, online=online2, target=target2, optimizer=opt2)
    for k, a in online.state_dict().items():
        assert np.array_equal(online2.state_dict()[k], a), k
    s1, s2 = opt.state_dict(), opt2.state_dict()
    assert s1["t"] == s2["t"] and s1["steps"] == s2["steps"]
    for a, b in zip(s1["m"] + s1["v"], s2["m"] + s2["v"]):
        assert rel(b, a) <= 1e-6


def test_state_dict_names_and_shapes_are_the_references():
    """Every vector family's state_dict against the reference builders' own
    (tests/golden/state_names.npz, made on the reference's modules)."""
    _need_gpu()
    from ttrl_b200.nets import (build_actor_critic, build_q_net, build_recurrent_actor_critic,
                                build_sac_nets)
    g = np.load(os.path.join(GOLDEN, "state_names.npz"))
    np.random.seed(0)
    nets = {
        "q": build_q_net((11,), 5, "cuda", batch=8, hidden=(32, 24)),
        "ac": build_actor_critic((11,), 5, "cuda", batch=8, hidden=(32, 24)),
        "sac": build_sac_nets(11, 3, "cuda", batch=8, critic_hidden=(20, 12),
                              policy_hidden=(24, 16)),
        "rec": build_recurrent_actor_critic((11,), 5, "cuda", batch=8, hidden_size=10,
                                            hidden=(16,)),
    }
    for family, net in nets.items():
        sd = net.state_dict()
        assert list(sd) == [str(n) for n in g[f"{family}.names"]], family
        shapes = [",".join(str(d) for d in a.shape) for a in sd.values()]
        assert shapes == [str(s) for s in g[f"{family}.shapes"]], family
