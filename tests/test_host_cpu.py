"""Host-side checks that need no GPU: the C-ABI library loads and exports
every entry point its header declares; ParamSync's averaging, schedule and
error contract (ttrl/engine/mesh/sync.py, tests/engine/test_mesh_sync.py's
known answers); the multi-process averaging path over a world-size-2 gloo
group; and conv geometry validation.
"""

import os
import re
import subprocess
import sys
import tempfile

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ttrl_b200.h")
GOLDEN = os.path.join(ROOT, "tests", "golden")


def header_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ttrl_[a-z0-9_]+)\s*\(", text)))


def _ensure_built():
    from ttrl_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        subprocess.run(["make", "-C", os.path.join(ROOT, "tt-rl_b200", "csrc"), "-j8"],
                       check=True, capture_output=True)
    return _lib


def test_library_exports_every_header_symbol():
    _lib = _ensure_built()
    lib = _lib.lib()  # loads without a GPU: no CUDA call happens at load
    declared = header_symbols()
    assert len(declared) >= 25
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    # ...and the Python binding types every one of them.
    assert sorted(_lib.EXPORTED_SYMBOLS) == declared
    assert lib.ttrl_version() >= 1


def test_library_refuses_bad_arguments_without_a_gpu():
    _lib = _ensure_built()
    lib = _lib.lib()
    # Argument validation happens on the host before any CUDA call.
    rc = lib.ttrl_linear_fwd(None, None, None, None, 0, 4, 4, 0, 0, None, 0, None, None)
    assert rc == 1  # TTRL_EINVAL
    assert b"bad extents" in lib.ttrl_last_error()
    rc = lib.ttrl_gru_gates_fwd(None, None, None, None, None, None, None, 0, 8, None)
    assert rc == 1
    assert b"gru_gates_fwd" in lib.ttrl_last_error()
    rc = lib.ttrl_gru_gates_bwd(None, None, None, 0, None, None, None, None, None, 4, 8, None)
    assert rc == 1
    assert b"null pointer" in lib.ttrl_last_error()


# ------------------------------------------------- recurrent sequence layout

def test_sequence_rows_are_time_major_whole_lanes():
    """Row t * n_seq + s of a minibatch is timestep chunk_s * seq_len + t of
    lane_s (ttrl/buffers/sequences.py:129-177 gather + flatten_time_major)."""
    from ttrl_b200.algos.recurrent_ppo import sequence_rows
    n_steps, n_envs, seq_len = 12, 4, 3
    slot_of = np.arange(n_steps * n_envs).reshape(n_steps, n_envs)  # [t, lane] -> slot
    ids = np.array([5, 0, 14, 9])
    got = sequence_rows(ids, n_envs, seq_len)
    want = []
    for t in range(seq_len):
        for i in ids:
            chunk, lane = divmod(int(i), n_envs)
            want.append(slot_of[chunk * seq_len + t, lane])
    assert got.tolist() == want
    # one sequence is one lane and consecutive timesteps
    rows = got.reshape(seq_len, len(ids))
    assert (rows % n_envs == (ids % n_envs)[None, :]).all()
    assert (np.diff(rows // n_envs, axis=0) == 1).all()


def test_sequence_helpers_follow_the_reference_contract():
    from ttrl_b200.algos.recurrent_ppo import (chunk_count, chunks_per_minibatch,
                                               normalize_valid_advantages, shift_to_starts)
    assert chunk_count(128, 32) == 4
    with pytest.raises(ValueError, match="does not divide"):
        chunk_count(100, 32)
    with pytest.raises(ValueError, match="seq_len must be >= 1"):
        chunk_count(8, 0)
    assert chunks_per_minibatch(512, 32) == 16
    with pytest.raises(ValueError, match="not a multiple"):
        chunks_per_minibatch(500, 32)
    boundary = np.array([[0, 1], [1, 0], [0, 0]], np.float32)
    starts = shift_to_starts(boundary, [1, 0])
    assert starts.tolist() == [[1, 0], [0, 1], [1, 0]]
    with pytest.raises(ValueError, match="carried covers"):
        shift_to_starts(boundary, [1, 0, 0])
    adv = np.array([1.0, 2.0, 100.0, 3.0], np.float32)
    valid = np.array([1, 1, 0, 1], np.float32)
    out = normalize_valid_advantages(adv, valid)
    live = adv[valid > 0]
    assert np.allclose(out, (adv - live.mean()) / (live.std() + 1e-8))
    assert abs(float(out[valid > 0].mean())) < 1e-6
    with pytest.raises(ValueError, match="no valid transitions"):
        normalize_valid_advantages(adv, np.zeros(4))


# ---------------------------------------------------------------- ParamSync

def _module(values):
    from ttrl_b200.engine.autograd import Tensor
    from ttrl_b200.engine.nn import Module

    class Two(Module):
        def __init__(self, w, b):
            self.w = Tensor(torch.tensor(np.asarray(w, np.float32)), requires_grad=True)
            self.b = Tensor(torch.tensor(np.asarray(b, np.float32)), requires_grad=True)

    return Two(*values)


def test_param_sync_known_answers():
    # tests/engine/test_mesh_sync.py:21-46: (1, 3) -> 2 and (10, 20) -> 15.
    from ttrl_b200.engine.mesh import ParamSync
    mods = [_module(([1.0], [10.0])), _module(([3.0], [20.0]))]
    ParamSync(mods, sync_every=1).average()
    for m in mods:
        assert m.w.numpy().tolist() == [2.0]
        assert m.b.numpy().tolist() == [15.0]


@pytest.mark.parametrize("n", [2, 3, 4])
def test_param_sync_matches_reference_golden(n):
    from ttrl_b200.engine.mesh import ParamSync
    d = np.load(os.path.join(GOLDEN, "param_sync.npz"))
    mods = [_module((d[f"n{n}_w_in"][i], d[f"n{n}_b_in"][i])) for i in range(n)]
    ParamSync(mods, sync_every=1).average()
    for i, m in enumerate(mods):
        assert np.array_equal(m.w.numpy(), d[f"n{n}_w_out"][i])
        assert np.array_equal(m.b.numpy(), d[f"n{n}_b_out"][i])


def test_param_sync_schedule():
    from ttrl_b200.engine.mesh import ParamSync
    mods = [_module(([0.0], [0.0])), _module(([2.0], [2.0]))]
    sync = ParamSync(mods, sync_every=3)
    assert [sync.maybe_average() for _ in range(6)] == [False, False, True, False, False, True]
    assert mods[0].w.numpy().tolist() == [1.0]


def test_param_sync_errors():
    from ttrl_b200.engine.mesh import ParamSync, ParamSyncError
    with pytest.raises(ValueError):
        ParamSync([_module(([0.0], [0.0]))], sync_every=0)
    with pytest.raises(ParamSyncError):  # schema mismatch by shape
        ParamSync([_module(([0.0], [0.0])), _module(([0.0, 1.0], [0.0]))])

    def raising(arrays):
        raise RuntimeError("link down")

    mods = [_module(([1.0], [1.0])), _module(([3.0], [3.0]))]
    with pytest.raises(ParamSyncError, match="reduction failed on parameter 0"):
        ParamSync(mods, reduce_fn=raising).average()
    with pytest.raises(ParamSyncError, match="1 result.* for 2 replica"):
        ParamSync(mods, reduce_fn=lambda arrays: arrays[:1]).average()
    # Nothing was written back by the failed calls.
    assert mods[0].w.numpy().tolist() == [1.0]


_GLOO_WORKER = r"""
import os, sys, numpy as np, torch, torch.distributed as dist
sys.path[:0] = [{root!r}, os.path.join({root!r}, "tt-rl_b200")]
from datetime import timedelta
rank = int(sys.argv[1])
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:{port}", rank=rank,
                        world_size=2, timeout=timedelta(seconds=60))
from ttrl_b200.engine.autograd import Tensor
from ttrl_b200.engine.nn import Module
from ttrl_b200.engine.mesh import ParamSync
class Net(Module):
    def __init__(self, r):
        self.w = Tensor(torch.full((3, 4), float(r + 1)), requires_grad=True)
        self.b = Tensor(torch.arange(5, dtype=torch.float32) * (10.0 ** r), requires_grad=True)
net = Net(rank)
sync = ParamSync([net], sync_every=2, group=dist.group.WORLD)
assert sync.maybe_average() is False
assert sync.maybe_average() is True
np.save(os.path.join({out!r}, f"rank{{rank}}.npy"),
        np.concatenate([net.w.numpy().ravel(), net.b.numpy().ravel()]))
dist.destroy_process_group()
"""


def test_param_sync_gloo_world_size_2():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as out:
        script = os.path.join(out, "worker.py")
        with open(script, "w") as f:
            f.write(_GLOO_WORKER.format(root=ROOT, port=port, out=out))
        procs = [subprocess.Popen([sys.executable, script, str(r)]) for r in range(2)]
        codes = [p.wait(timeout=180) for p in procs]
        assert codes == [0, 0]
        r0 = np.load(os.path.join(out, "rank0.npy"))
        r1 = np.load(os.path.join(out, "rank1.npy"))
    want = np.concatenate([np.full(12, 1.5, np.float32),
                           (np.arange(5, dtype=np.float32) * 11.0) / 2.0])
    assert np.array_equal(r0, want) and np.array_equal(r1, want)


# ---------------------------------------------------------------- geometry

def test_conv_geometry_matches_reference():
    from ttrl_b200.engine.conv import conv_out_size
    for size, k, s, p, want in np.load(os.path.join(GOLDEN, "conv_tower.npz"))["geometry"]:
        if want < 0:
            with pytest.raises(ValueError):
                conv_out_size(int(size), int(k), int(s), int(p))
        else:
            assert conv_out_size(int(size), int(k), int(s), int(p)) == want


_GLOO_FAULT_WORKER = r"""
import os, sys, torch, torch.distributed as dist
sys.path[:0] = [{root!r}, os.path.join({root!r}, "tt-rl_b200")]
from datetime import timedelta
rank = int(sys.argv[1])
dist.init_process_group("gloo", init_method="tcp://127.0.0.1:{port}", rank=rank,
                        world_size=2, timeout=timedelta(seconds=30))
from ttrl_b200.engine.autograd import Tensor
from ttrl_b200.engine.nn import Module
from ttrl_b200.engine.mesh import ParamSync, ParamSyncError
class Net(Module):
    def __init__(self, r):
        self.w = Tensor(torch.full((3, 4), float(r + 1)), requires_grad=True)
net = Net(rank)
sync = ParamSync([net], sync_every=1, group=dist.group.WORLD, timeout_s=5.0)
# The arena is what the collective reduces: no packing copies.
assert sync.arena.data_ptr() == net.w.data.data_ptr()
dist.barrier()
if rank == 1:
    # This rank fails between updates and never joins the average.
    os._exit(3)
try:
    sync.average()
    outcome = "averaged"
except ParamSyncError as exc:
    outcome = "ParamSyncError " + str(exc).splitlines()[0][:200]
with open(os.path.join({out!r}, "rank0.txt"), "w") as f:
    f.write(outcome + "\n" + repr(net.w.numpy().ravel().tolist()))
os._exit(0)
"""


def test_param_sync_gloo_rank_that_fails_mid_run():
    """A rank that dies instead of joining an average: the surviving rank's
    average() ends with ParamSyncError within its bound, its parameters
    untouched (tests/engine/test_mesh_sync.py:47-118 holds the in-process
    counterparts)."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as out:
        script = os.path.join(out, "worker.py")
        with open(script, "w") as f:
            f.write(_GLOO_FAULT_WORKER.format(root=ROOT, port=port, out=out))
        procs = [subprocess.Popen([sys.executable, script, str(r)]) for r in range(2)]
        codes = [p.wait(timeout=180) for p in procs]
        assert codes == [0, 3]
        with open(os.path.join(out, "rank0.txt")) as f:
            outcome, values = f.read().splitlines()
    assert outcome.startswith("ParamSyncError"), outcome
    assert "all-reduce over 2 ranks did not complete" in outcome
    assert values == repr([1.0] * 12)


@pytest.mark.parametrize("b1,b2", [(0.9, 0.999), (0.9, 0.99), (0.5, 0.9)])
def test_adam_bias_table_is_the_reference_arithmetic(b1, b2):
    """Adam's bias-term table holds, for every step t, exactly the terms of
    ttrl/engine/optim/scalars.py:13-27 as the host evaluates them (Python's
    own `**`, `math.sqrt`), up to the first step where both have reached 1
    in double; the kernel reads the last row for every later step, so that
    row must equal the terms at any later t."""
    import math
    from ttrl_b200.engine.optim import adam_bias_table, adam_fused_scalars
    table = adam_bias_table(b1, b2, "cpu")
    assert table is not None and table.dtype == torch.float64
    rows = table.numpy()
    T = rows.shape[0]
    for t in list(range(1, 200)) + list(range(max(1, T - 50), T + 1)):
        bc1, bc2 = 1 - b1 ** t, 1 - b2 ** t
        assert rows[t - 1, 0] == bc1
        assert rows[t - 1, 1] == math.sqrt((1 - b2) / bc2)
    for t in (T, T + 1, 10 * T):
        bc1, bc2 = 1 - b1 ** t, 1 - b2 ** t
        assert (bc1, bc2) == (1.0, 1.0)
        assert rows[-1, 1] == math.sqrt((1 - b2) / bc2)
    # The kernel's alpha_t = lr * (1 - b1) / bc1 / c and eps_t = eps / c from
    # the row equal the host's fused scalars.
    for t in (1, 7, T, 3 * T):
        r = rows[min(t, T) - 1]
        alpha, eps_t = adam_fused_scalars(2.5e-4, b1, b2, 1e-8, t)
        assert 2.5e-4 * (1 - b1) / r[0] / r[1] == alpha
        assert 1e-8 / r[1] == eps_t


def _bench_reference_arm(env_extra):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ)
    env.update(env_extra)
    return subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "0"], cwd=root, env=env,
                          capture_output=True, text=True, timeout=600)


def test_bench_reference_arm_line_contract():
    """`bench.py --impl reference` (the CPU port of the reference's path, no
    GPU needed) prints one JSON line with the CUDA arm's metric and workload,
    its own cpu_baseline, and an end-to-end figure with no host-device bytes."""
    import json
    import bench
    r = _bench_reference_arm({"WORLD_SIZE": "1", "RANK": "0", "LOCAL_RANK": "0"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "samples/s"
    assert d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["workload"] == "ppo_nature_cnn_rollout8x128_mb256_epochs4"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "samples/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_bench_reference_arm_other_ranks_exit_without_work():
    """Under torchrun only rank 0 runs the reference arm and prints its line;
    the other ranks exit 0 and print nothing."""
    r = _bench_reference_arm({"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
