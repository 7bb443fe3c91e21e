"""The checkpoint file layer on the host (no GPU).

`tests/golden/checkpoint_dqn.npz` holds a DQN checkpoint written by the
reference's own save_checkpoint (ttrl/train/checkpoint/file.py:112-218), its
conv Adam moments in the reference's prepared matrix
(ttrl/engine/conv/packing.py:24-108). These tests pin ttrl_b200.checkpoint's
reader, writer and packing against that file:

* reading it gives the tree the reference's load_checkpoint gives (the
  generator asserted the arrays equal); rewriting it unchanged reproduces the
  `__meta__` bytes and every member exactly;
* the prepared layouts are recovered from the stored shapes and second
  moments, and pack/unpack round-trips them bit for bit;
* the candidate set for the reference's pinned case (4-channel 8x8 conv with
  32 outputs, `(1, 1, 512, 32)`) is the reference's (cp 4..8, row_block 64).
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CONV = {0: (32, 4, 8, 8), 2: (64, 32, 4, 4), 4: (64, 64, 3, 3)}


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN, "checkpoint_dqn.npz"))


@pytest.fixture()
def ref_path(golden, tmp_path):
    path = tmp_path / "ref.npz"
    path.write_bytes(golden["ref_file"].tobytes())
    return str(path)


def _members(path):
    with np.load(path, allow_pickle=False) as npz:
        return {k: npz[k] for k in npz.files}


def test_reads_the_reference_file(ref_path):
    from ttrl_b200.checkpoint import Checkpoint, Tagged
    ck = Checkpoint.read(ref_path)
    assert ck.level == "L1"
    state = ck.agent_state()
    assert {"config", "online", "target", "optimizer", "frame_count", "update_count",
            "rng_state"} <= set(state)
    assert isinstance(state["config"], Tagged) and state["config"].path.endswith("DQNConfig")
    opt = state["optimizer"]
    assert opt["t"] == 7 and opt["betas"] == [0.9, 0.999]
    assert len(opt["m"]) == len(state["online"]) == 10
    assert state["online"]["encoder.towers.obs.layers.0.weight"].shape == (32, 4, 8, 8)
    assert state["online"]["head.q.bias"].shape == (1, 6)


def test_unchanged_rewrite_is_byte_identical(ref_path, tmp_path):
    from ttrl_b200.checkpoint import Checkpoint
    ck = Checkpoint.read(ref_path)
    out = tmp_path / "again.npz"
    ck.with_agent_state(ck.agent_state()).write(str(out))
    a, b = _members(ref_path), _members(str(out))
    assert sorted(a) == sorted(b)
    assert a["__meta__"].tobytes() == b["__meta__"].tobytes()
    for k in a:
        assert a[k].dtype == b[k].dtype and np.array_equal(a[k], b[k]), k


def test_prepared_layouts_are_recovered(ref_path, golden):
    from ttrl_b200.checkpoint import Checkpoint
    from ttrl_b200.engine.packing import solve_cp
    opt = Checkpoint.read(ref_path).agent_state()["optimizer"]
    rows = golden["layouts"]
    assert len(rows) == 3
    for (i, r, c, cp), oihw in zip(rows, CONV.values()):
        m, v = opt["m"][i], opt["v"][i]
        lay = solve_cp(m.shape, oihw, v=v)
        assert (lay.rows, lay.cols, lay.cp) == (r, c, cp)
        assert lay.padding_is_zero(m) and lay.padding_is_zero(v)
        assert np.array_equal(lay.pack(lay.unpack(m)), m)
        assert np.all(lay.unpack(v) > 0)


def test_candidate_layouts_match_the_reference_pin():
    from ttrl_b200.engine.packing import candidate_layouts, default_layout
    cands = candidate_layouts(512, 32, 32, 4, 8, 8)
    assert [c.cp for c in cands] == [4, 5, 6, 7, 8]
    assert all(c.row_block == 64 and c.shape == (1, 1, 512, 32) for c in cands)
    w = np.arange(32 * 4 * 8 * 8, dtype=np.float32).reshape(32, 4, 8, 8)
    for c in cands:
        assert np.array_equal(c.unpack(c.pack(w)), w)
    assert default_layout(32, 4, 8, 8).shape == (1, 1, 512, 32)


def test_update_keeps_other_members(ref_path, tmp_path):
    from ttrl_b200.checkpoint import Checkpoint
    ck = Checkpoint.read(ref_path)
    state = ck.agent_state()
    state["update_count"] = 9
    out = tmp_path / "u.npz"
    ck.with_agent_state(state).write(str(out))
    a, b = _members(ref_path), _members(str(out))
    for k in a:
        if not k.startswith("state.") and k != "__meta__":
            assert np.array_equal(a[k], b[k]), k
    ma = json.loads(a["__meta__"].tobytes())
    mb = json.loads(b["__meta__"].tobytes())
    assert mb["agent_state"]["update_count"] == 9
    for key in ma:
        if key != "agent_state":
            assert ma[key] == mb[key], key


def test_refuses_another_format(ref_path, tmp_path):
    from ttrl_b200.checkpoint import Checkpoint
    members = _members(ref_path)
    meta = json.loads(members["__meta__"].tobytes())
    meta["format"] = "something-else"
    members["__meta__"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
    bad = tmp_path / "bad.npz"
    np.savez(str(bad), **members)
    with pytest.raises(ValueError, match="format"):
        Checkpoint.read(str(bad))
    np.savez(str(bad), w=np.zeros(2))
    with pytest.raises(ValueError, match="__meta__"):
        Checkpoint.read(str(bad))


def test_new_checkpoint_round_trips(tmp_path):
    from ttrl_b200.checkpoint import Checkpoint, Tagged
    cfg = Tagged("ttrl.train.config:TrainConfig", {"seed": 3})
    state = {"net": {"a.weight": np.ones((2, 3), np.float32)}, "blob": b"\x00\x01",
             "pair": (1, 2.5)}
    ck = Checkpoint.new(agent_state=state, obs_spec={"leaves": []}, action_spec={"kind": "x"},
                        level="L1", frame=5, config=cfg)
    path = tmp_path / "n.npz"
    ck.write(str(path))
    back = Checkpoint.read(str(path))
    got = back.agent_state()
    assert np.array_equal(got["net"]["a.weight"], state["net"]["a.weight"])
    assert got["blob"] == b"\x00\x01" and got["pair"] == [1, 2.5]
    assert back.meta["frame"] == 5
    with pytest.raises(ValueError, match="L1"):
        Checkpoint.new(agent_state=state, obs_spec={}, action_spec={}, level="L1")


def test_load_learner_names_missing_parts():
    from ttrl_b200.checkpoint import load_learner
    with pytest.raises(KeyError, match="online"):
        load_learner({"net": {}}, online=object())


def test_learner_state_packs_conv_moments_into_the_stored_layout(ref_path):
    """learner_state puts an optimizer's OIHW convolution moments back into
    the prepared matrices the file holds them in (and leaves the others as
    they are), with a host-only stand-in for the B200 Adam."""
    from types import SimpleNamespace
    from ttrl_b200.checkpoint import Checkpoint, learner_state
    from ttrl_b200.engine.packing import solve_cp
    stored = Checkpoint.read(ref_path).agent_state()
    names = list(stored["online"])
    rng = np.random.default_rng(5)
    params, m, v = [], [], []
    for name in names:
        shape = stored["online"][name].shape
        conv = len(shape) == 4 and shape[2] > 1
        params.append(SimpleNamespace(_layout=SimpleNamespace(oihw=shape) if conv else None))
        m.append(rng.standard_normal(shape).astype(np.float32))
        v.append(np.abs(rng.standard_normal(shape)).astype(np.float32) + 1e-3)
    opt = SimpleNamespace(params=params, m=m,
                          state_dict=lambda: {"t": 8, "steps": [8] * len(names), "lr": 1e-4,
                                              "betas": (0.9, 0.999), "eps": 1.5e-4,
                                              "weight_decay": 0.0, "m": list(m), "v": list(v)})
    out = learner_state(like=stored, optimizer=opt)["optimizer"]
    assert out["t"] == 8
    for i, name in enumerate(names):
        want_shape = stored["optimizer"]["m"][i].shape
        assert out["m"][i].shape == want_shape and out["v"][i].shape == want_shape, name
        if want_shape != m[i].shape:
            lay = solve_cp(want_shape, m[i].shape, v=stored["optimizer"]["v"][i])
            assert np.array_equal(lay.unpack(out["m"][i]), m[i])
            assert np.array_equal(lay.unpack(out["v"][i]), v[i])
            assert lay.padding_is_zero(out["m"][i])
        else:
            assert np.array_equal(out["m"][i], m[i])


def test_ambiguous_prepared_layout_is_refused_not_guessed():
    """A prepared matrix wider than the default whose second moment is all
    zero (a weight that never had a gradient) fits several channel strides:
    the strict solver refuses instead of picking one."""
    from ttrl_b200.engine.packing import AmbiguousLayout, candidate_layouts, solve_cp
    oihw = (32, 4, 8, 8)
    shape = (1, 1, 8 * 64, 32)  # row_block 64 holds cp = 4..8 for an 8-wide kernel row
    assert len(candidate_layouts(shape[2], shape[3], *oihw)) > 1
    with pytest.raises(AmbiguousLayout):
        solve_cp(shape, oihw, v=np.zeros(shape, np.float32), strict=True)
    # A trained v (non-zero on every live entry of one layout) resolves it.
    lay = candidate_layouts(shape[2], shape[3], *oihw)[-1]
    v = lay.pack(np.full(oihw, 0.5, np.float32))
    assert solve_cp(shape, oihw, v=v, strict=True) == lay
