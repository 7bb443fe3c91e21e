"""The Python drop-in, end to end: tt-rl's OWN `ttrl.nets.build_q_net` and
`ttrl.algos.dqn.losses.update_loss` (unchanged reference source) run on this
backend through `ttrl_b200.dropin.install()` -- its `ttrl.engine` resolved to
`ttrl_b200.engine` -- and driven by `TrainStep` as the reference's DQN agent
drives them (ttrl/algos/dqn/agent.py:180-208).

The reference package comes from `TTRL_REFERENCE` or the repository's
`baseline/_ref` (the reference installed there with pip). The run happens in
a child process, so the module aliases never touch the test session.

Checks against this repository's own DQN path (its nets, the fused loss
kernel and u8 frame conversion) from the same initial weights on the same
batches: identical state_dict names and shapes, then two graph-replayed
updates with loss and mean Q to 1e-5, gradient norm to 1e-4, and every
parameter after the two Adam steps to 1e-4 relative. The two paths differ
only in how the loss head is composed (the reference's generic ops against
one fused kernel) and in the frames' upload format (fp32 NHWC rows against
uint8 frames converted on the device).
"""

import json
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_CHILD = r"""
import json, os, sys
import numpy as np
import torch
sys.path[:0] = [{root!r}, os.path.join({root!r}, "tt-rl_b200")]
from ttrl_b200 import dropin
dropin.install({ref!r})
from ttrl.algos.dqn.losses import leaf_key, step_inputs as ref_inputs, update_loss as ref_update
from ttrl.nets.build import build_q_net as ref_build
from ttrl.nets.obs import obs_rows
from ttrl.spaces import ActionSpec, ObsGroup, ObsSpec
from ttrl.engine.optim import Adam
from ttrl.engine.step import TrainStep
from ttrl_b200.algos import dqn as own
from ttrl_b200.nets import build_q_net as own_build

B, A = 8, 6
spec = ObsGroup.of(ObsSpec.image(4, 84, 84))
leaves = [name for name, _ in spec.specs()]
np.random.seed(0)
ref_online = ref_build(spec, ActionSpec.discrete(A), "cuda", batch=B)
ref_target = ref_build(spec, ActionSpec.discrete(A), "cuda", batch=B)
ref_target.copy_from(ref_online)
own_online = own_build((4, 84, 84), A, "cuda", batch=B)
own_target = own_build((4, 84, 84), A, "cuda", batch=B)
init = ref_online.state_dict()
names = {{k: list(np.shape(v)) for k, v in init.items()}}
own_names = {{k: list(np.shape(v)) for k, v in own_online.state_dict().items()}}
own_online.load_state_dict(init)
own_target.load_state_dict(init)

ref_opt = Adam(list(ref_online.parameters()), lr=1e-4, eps=1.5e-4)
own_opt = Adam(list(own_online.parameters()), lr=1e-4, eps=1.5e-4)
ri = ref_inputs(spec, "cuda", batch=B, num_actions=A, mask_n=0)
oi = own.step_inputs((4, 84, 84), "cuda", batch=B, num_actions=A)
ref_step = TrainStep(lambda i: ref_update(ref_online, ref_target, i, leaves=leaves,
                                          num_actions=A, mask_n=0, double=True,
                                          huber_delta=1.0),
                     ri, "cuda", optimizer=ref_opt, mode="traced_fwd_bwd")
own_step = TrainStep(lambda i: own.update_loss(own_online, own_target, i, num_actions=A,
                                               double=True, huber_delta=1.0),
                     oi, "cuda", optimizer=own_opt, mode="traced_fwd_bwd")
rng = np.random.default_rng(1)
metrics = []
for u in range(2):
    obs = rng.integers(0, 256, (B, 4, 84, 84), dtype=np.uint8)
    nxt = rng.integers(0, 256, (B, 4, 84, 84), dtype=np.uint8)
    onehot = np.eye(A, dtype=np.float32)[rng.integers(0, A, B)]
    rew = rng.choice([-1.0, 0.0, 1.0], (B, 1)).astype(np.float32)
    done = (rng.random((B, 1)) < 0.2).astype(np.float32)
    disc = np.full((B, 1), 0.99, np.float32)
    for leaf, leaf_spec in spec.specs():
        ref_step.load_input(leaf_key("obs", leaf), obs_rows(obs, leaf_spec))
        ref_step.load_input(leaf_key("next_obs", leaf), obs_rows(nxt, leaf_spec))
    for key, value in (("actions_onehot", onehot), ("rewards", rew), ("dones", done),
                       ("discounts", disc)):
        ref_step.load_input(key, value)
    for key, value in (("obs", obs), ("next_obs", nxt), ("actions_onehot", onehot),
                       ("rewards", rew), ("dones", done), ("discounts", disc)):
        own_step.load_input(key, value)
    r = ref_step.run()
    o = own_step.run()
    scalar = lambda m, k: float(np.asarray(m[k]).reshape(-1)[0])
    metrics.append({{k: [scalar(r, k), scalar(o, k)] for k in ("loss", "mean_q", "grad_sq")}})
ref_sd, own_sd = ref_online.state_dict(), own_online.state_dict()
errs = {{k: float(np.linalg.norm(own_sd[k].astype(np.float64) - ref_sd[k])
                 / max(np.linalg.norm(ref_sd[k].astype(np.float64)), 1e-30)) for k in ref_sd}}
moved = {{k: float(np.abs(ref_sd[k] - init[k]).max()) for k in ref_sd}}
ref_step.close()
own_step.close()
with open({out!r}, "w") as f:
    json.dump({{"names": names, "own_names": own_names, "metrics": metrics, "errs": errs,
               "moved": moved}}, f)
"""


def _reference_checkout():
    for path in (os.environ.get("TTRL_REFERENCE"), os.path.join(ROOT, "baseline", "_ref")):
        if path and os.path.isdir(os.path.join(path, "ttrl")):
            return path
    return None


def test_reference_dqn_runs_unchanged_on_the_b200_engine():
    ref = _reference_checkout()
    if ref is None:
        pytest.skip("no reference checkout (TTRL_REFERENCE or baseline/_ref)")
    with tempfile.TemporaryDirectory() as tmp:
        out = os.path.join(tmp, "result.json")
        script = os.path.join(tmp, "child.py")
        with open(script, "w") as f:
            f.write(_CHILD.format(root=ROOT, ref=ref, out=out))
        proc = subprocess.run([sys.executable, script], capture_output=True, text=True,
                              timeout=600)
        assert proc.returncode == 0, proc.stderr[-4000:]
        with open(out) as f:
            res = json.load(f)
    assert res["names"] == res["own_names"]
    for u, m in enumerate(res["metrics"]):
        for key, tol in (("loss", 1e-5), ("mean_q", 1e-5), ("grad_sq", 2e-4)):
            want, got = m[key]
            assert abs(got - want) <= tol * max(abs(want), 1e-6), (u, key, got, want)
    for name, err in res["errs"].items():
        assert res["moved"][name] > 0.0, name  # Adam moved every parameter
        assert err <= 1e-4, (name, err)
