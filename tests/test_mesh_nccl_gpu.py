"""ParamSync's NCCL path on two GPUs (ttrl/engine/mesh/sync.py:138-177
semantics): one process per GPU, each with its own PPO Nature-CNN
actor-critic and Adam state; `average()` is one in-place all-reduce
(ReduceOp.AVG) of the learner's flat parameter arena.

At two ranks NCCL's average is exact: (a + b) / 2 rounds once, and a
halving is exact, so the averaged parameters must equal the host's
(a + b) / 2 bit for bit. Adam moments must not move. `broadcast(0)` must
leave rank 1 holding rank 0's parameters exactly.

Runs only where two GPUs are visible (skipped on one). NVLS is off and no
kernel of this library waits on another rank, so a failing rank cannot
leave a peer spinning.
"""

import os
import socket
import subprocess
import sys
import tempfile

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_WORKER = r"""
import os, sys, datetime, numpy as np, torch, torch.distributed as dist
sys.path[:0] = [{root!r}, os.path.join({root!r}, "tt-rl_b200")]
rank = int(sys.argv[1])
torch.cuda.set_device(rank)
dev = torch.device("cuda", rank)
dist.init_process_group("nccl", init_method="tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                        timeout=datetime.timedelta(seconds=60), device_id=dev)
from ttrl_b200.algos.ppo import PPOConfig, PPOLearner
from ttrl_b200.engine.mesh import ParamSync
from ttrl_b200.nets import build_actor_critic
np.random.seed(100 + rank)
net = build_actor_critic((4, 84, 84), 6, dev, batch=256)
learner = PPOLearner(net, 512, (4, 84, 84), dev, cfg=PPOConfig(epochs=1, minibatch_size=256),
                     seed=rank)
rng = np.random.default_rng(rank)
learner.load_rollout(rng.integers(0, 256, (512, 4, 84, 84), dtype=np.uint8),
                     rng.integers(0, 6, 512), np.full(512, np.log(1 / 6), np.float32),
                     rng.standard_normal(512).astype(np.float32),
                     rng.standard_normal(512).astype(np.float32),
                     rng.standard_normal(512).astype(np.float32))
learner.draw_permutations()
sync = ParamSync([net], sync_every=1, group=dist.group.WORLD)
assert sync.arena.data_ptr() == learner.param_arena.data_ptr()
learner.replay()  # Adam moments become non-zero and differ between ranks
torch.cuda.synchronize()
host = lambda: np.concatenate([p.numpy().ravel() for p in net.parameters()])
moments = lambda: np.concatenate([m.cpu().numpy().ravel() for m in learner.optimizer.m]
                                 + [v.cpu().numpy().ravel() for v in learner.optimizer.v])
before, m_before = host(), moments()
sync.average()
torch.cuda.synchronize()
after, m_after = host(), moments()
sync.broadcast(0)
torch.cuda.synchronize()
bcast = host()
np.savez(os.path.join({out!r}, f"rank{{rank}}.npz"), before=before, after=after,
         m_before=m_before, m_after=m_after, bcast=bcast)
learner.close()
dist.barrier()
dist.destroy_process_group()
"""


def test_param_sync_nccl_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    with tempfile.TemporaryDirectory() as out:
        script = os.path.join(out, "worker.py")
        with open(script, "w") as f:
            f.write(_WORKER.format(root=ROOT, port=port, out=out))
        procs = [subprocess.Popen([sys.executable, script, str(r)], env=env) for r in range(2)]
        try:
            codes = [p.wait(timeout=300) for p in procs]
        finally:
            for p in procs:
                if p.poll() is None:
                    p.kill()
        assert codes == [0, 0]
        r = [dict(np.load(os.path.join(out, f"rank{i}.npz"))) for i in range(2)]
    a, b = r[0]["before"], r[1]["before"]
    assert not np.array_equal(a, b)
    want = (a + b) / np.float32(2.0)
    for i in range(2):
        assert np.array_equal(r[i]["after"], want), i
        assert np.array_equal(r[i]["m_after"], r[i]["m_before"]), i
        assert np.array_equal(r[i]["bcast"], r[0]["after"]), i
    assert not np.array_equal(r[0]["m_before"], r[1]["m_before"])
