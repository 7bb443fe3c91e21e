"""Learner throughput of the B200 backend on BASELINE.json's workload.

Headline (configs[1] at N=1, configs[4] at N>1): PPO Nature-CNN learner
samples/sec. One bench "step" is one PPO rollout update: a rollout of
8 envs x 128 steps (1024 uint8 [4,84,84] frames plus per-sample fields)
resident in HBM, 4 epochs x 4 minibatches of 256, each minibatch step = the
Nature-CNN actor-critic forward, the PPO objective, backward, device-side
grad-norm clip 0.5 and Adam (lr 2.5e-4) -- all 16 gradient steps replayed
from ONE CUDA graph. samples/sec = 256 x minibatch steps / s, summed over
ranks. At N>1 every rank runs its own seed stream and the online
parameters are averaged by an NCCL all-reduce (ReduceOp.AVG) every 50
rollout updates (the reference's sync_every unit).

Also reported: the Nature-DQN batch-32 update (configs[0] shapes; forward x3,
double-DQN Huber loss, backward, Adam) as updates/sec from one graph replay
each, the SAC and recurrent PPO updates, end-to-end numbers through host
buffers (the PPO one the median of three runs), the live per-kernel roofline
(the longest contraction and its next two contenders), the CPU baseline, and
the clocks seen during the timed region. At N>1 the line also names the GPU
each rank ran on.

`--impl reference` times the reference's arithmetic on the host CPU (the
numpy oracle restating it; the reference itself needs ttnn and a
Tenstorrent chip) on the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "tt-rl_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

MB = 256
ROLLOUT = 8 * 128
EPOCHS = 4
STEPS_PER_UPDATE = EPOCHS * (ROLLOUT // MB)
SAMPLES_PER_UPDATE = STEPS_PER_UPDATE * MB
SYNC_EVERY = 50
# Algorithmic work per sample: three times the forward MACs less conv1's
# data gradient (which no layer needs), two FLOP per MAC.
PPO_FLOP_PER_SAMPLE = 2 * 24_762_880
DQN_FLOP_PER_UPDATE = 2 * 43_453_440 * 32
RPPO_FLOP_PER_STEP = 2 * 26_526_976 * 512  # 3F_r - conv1 dX per row, 512 rows

# DRAM bytes (read + write) per launch of the kernels that have been the
# dominant one, from one ncu capture each of `python bench.py --profile-case
# <case> --batch 256` (conv1s2d_wgrad, conv1s2d_fprop, conv2_dgrad,
# conv3_dgrad, fc1_wgrad).
NCU_TRAFFIC_BYTES = {
    "conv_wgrad[2x2/1 64->32]": 42.106624e6 + 512,
    "conv_fprop[2x2/1 64->32]": 29.039872e6,
    "conv_dgrad[4x4/2 32->64]": 18.6368e6,
    "conv_dgrad[3x3/1 64->64]": 8.75648e6,
    "linear_wgrad[256x3136x512]": 3.847168e6,
}

METRIC = "PPO learner samples/sec (Nature-CNN actor-critic, minibatch 256, fwd+bwd+clip+Adam, graph-replayed)"


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-dqn", action="store_true")
    # tf32x3: split-TF32 (~1e-6 relative; gradients within 1e-4 of float64);
    # tf32: one TF32 pass over round-to-nearest operands (the accuracy class
    # of the reference's HiFi4 matmuls; ill-conditioned reductions reach
    # ~1.5e-3 of float64).
    ap.add_argument("--precision", choices=("tf32", "tf32x3"), default="tf32x3")
    # Profiling cases (for ncu): run one kernel family of the Nature-CNN
    # shapes a few times and exit without timing or printing a bench line.
    ap.add_argument("--profile-case", choices=sorted(PROFILE_CASES), default=None)
    ap.add_argument("--batch", type=int, default=256, help="batch of a --profile-case")
    ap.add_argument("--reps", type=int, default=3, help="repetitions of a --profile-case")
    return ap.parse_args()


PRECISION_TEXT = {
    "tf32": "TF32 tensor cores (tcgen05 kind::tf32, one pass), fp32 accumulate and fp32 "
            "elementwise",
    "tf32x3": "split-TF32 tensor cores (tcgen05 kind::tf32 x3), fp32 accumulate and fp32 "
              "elementwise",
}


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        try:
            rows = open(self.path).read().strip().splitlines()
        except OSError:
            rows = []
        for row in rows:
            f = [x.strip() for x in row.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if self.path:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "samples": len(sm),
                "reasons": sorted(reasons)}


# ------------------------------------------------------------ helpers

def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained"), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback"}


def _rollout(rng):
    obs = rng.integers(0, 256, (ROLLOUT, 4, 84, 84), dtype=np.uint8)
    actions = rng.integers(0, 6, ROLLOUT)
    adv = rng.standard_normal(ROLLOUT).astype(np.float32)
    returns = rng.standard_normal(ROLLOUT).astype(np.float32)
    return obs, actions, adv, returns


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


_JSON_OUT = None


def _route_stdout_to_stderr() -> None:
    """Keep a private handle on stdout for the bench line and point file
    descriptor 1 at stderr, so library logs written there stay off it."""
    global _JSON_OUT
    if _JSON_OUT is None:
        sys.stdout.flush()
        _JSON_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def emit(line: dict) -> None:
    """Print the one JSON line of this run on stdout."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def sync_points(k: int) -> set:
    """Indices of the updates (0-based) after which a multi-GPU run averages
    its replicas: every SYNC_EVERY-th update, and the last one."""
    points = {i for i in range(k) if (i + 1) % SYNC_EVERY == 0}
    if k > 0:
        points.add(k - 1)
    return points


# ----------------------------------------------------------- CPU arms

def cpu_ppo_steps(n_steps: int, seed: int = 0):
    """The reference's arithmetic on the host (numpy fp32, all BLAS threads):
    PPO minibatch steps of 256. Returns seconds per step."""
    from oracle import learner as ref
    rng = np.random.default_rng(seed)
    p = ref.nature_params(rng, heads=(("pi", 6), ("v", 1)))
    x = rng.integers(0, 256, (MB, 84, 84, 4)).astype(np.float32)
    acts = rng.integers(0, 6, MB)
    f = lambda: rng.standard_normal(MB).astype(np.float32)  # noqa: E731
    old, adv, ret, val = f() * 0.1 + np.log(1 / 6), f(), f(), f()
    state = {}
    times = []
    for t in range(1, n_steps + 1):
        t0 = time.perf_counter()
        _, _, p, state, _ = ref.ppo_minibatch_step(p, state, t, x, acts, old, adv, ret, val,
                                                   lr=2.5e-4, eps=1e-8, max_grad_norm=0.5)
        times.append(time.perf_counter() - t0)
    return times


def cpu_dqn_updates(n_updates: int, seed: int = 0):
    """The reference's arithmetic on the host (numpy fp32, all BLAS threads):
    Nature-DQN batch-32 double-DQN updates with Adam. Seconds per update."""
    from oracle import learner as ref
    rng = np.random.default_rng(seed)
    online = ref.nature_params(rng, heads=(("q", 6),))
    target = ref.nature_params(rng, heads=(("q", 6),))
    obs = rng.integers(0, 256, (32, 84, 84, 4)).astype(np.float32)
    nxt = rng.integers(0, 256, (32, 84, 84, 4)).astype(np.float32)
    acts = rng.integers(0, 6, 32)
    rew = rng.choice([-1.0, 0.0, 1.0], 32).astype(np.float32)
    dones = np.zeros(32, np.float32)
    disc = np.full(32, 0.99, np.float32)
    state = None
    times = []
    for t in range(1, n_updates + 1):
        t0 = time.perf_counter()
        out = ref.dqn_update(online, target, obs, nxt, acts, rew, dones, disc,
                             adam_state=state, t=t)
        online, state = out[2], out[3]
        times.append(time.perf_counter() - t0)
    return times


def run_reference(args):
    world, rank, _ = _dist()
    if rank != 0:
        return
    warm = min(args.warmup, 1)
    steps = max(1, min(args.steps, 3))
    cpu_ppo_steps(warm)
    times = cpu_ppo_steps(steps, seed=1)
    total = sum(times)
    value = MB * steps / total
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "samples/s",
        "n_gpus": world, "steps": steps, "warmup": warm, "ms_per_step": 1000 * total / steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded uint8 frames, N(0,1) advantages/returns)",
        "config": {"workload": "ppo_nature_cnn_rollout8x128_mb256_epochs4",
                   "global_batch": MB * world, "minibatch": MB, "rollout": ROLLOUT,
                   "epochs": EPOCHS, "parallelism": f"dp{world}",
                   "note": "the same workload and metric as the CUDA arm; each reference "
                           "step is a bounded sample of it, one PPO minibatch step of 256 "
                           "samples, in samples/s"},
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": cores, "kind": "port",
                         "sample": f"{steps} PPO minibatch steps of 256 (numpy fp32 restatement "
                                   "of the reference's tape, objective, clip and Adam)"},
        "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


# ---------------------------------------------------------- GPU arm

def build_ppo(device, seed):
    import torch
    from ttrl_b200.algos.ppo import PPOConfig, PPOLearner, initial_old_logp
    from ttrl_b200.nets import build_actor_critic
    np.random.seed(seed)
    net = build_actor_critic((4, 84, 84), 6, device, batch=MB)
    learner = PPOLearner(net, ROLLOUT, (4, 84, 84), device,
                         cfg=PPOConfig(epochs=EPOCHS, minibatch_size=MB), seed=seed)
    rng = np.random.default_rng(seed)
    obs, actions, adv, returns = _rollout(rng)
    old_logp, values = initial_old_logp(net, obs, actions, device)
    learner.load_rollout(obs, actions, old_logp, values, returns, adv)
    learner.draw_permutations()
    torch.cuda.synchronize(device)
    host = {"obs": obs, "actions": actions.astype(np.int32), "old_logp": old_logp,
            "values": values, "returns": returns, "adv": adv}
    return learner, host


def kernel_profile(learner, device):
    """One eager minibatch step with CUDA events around every kernel-family
    call (on the launching stream): per-call duration and algorithmic FLOPs."""
    import torch
    from ttrl_b200.device import context
    ctx = context(device)
    records = []
    ctx.profile = records
    try:
        learner._minibatch_step(0)
        torch.cuda.synchronize(device)
    finally:
        ctx.profile = None
    # Each pass is one more optimizer step on the learner; the passes run
    # after the timed regions, and nothing after them is timed.
    return [(name, flops, s.elapsed_time(e) * 1e-3, call) for name, flops, s, e, call in records]


def device_time(call, device, reps=20, trials=3):
    """Per-launch device time (s) of one library call: `reps` launches back
    to back in one CUDA graph, the replay bracketed by events on the replay
    stream, median over `trials` replays. No host launch gap enters it (the
    eager events around a single call also hold the host's ctypes time when
    the device is idle waiting for the launch)."""
    import torch
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        call()  # the launch configuration is cached before the capture
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(reps):
                call()
        graph.replay()
        times = []
        for _ in range(trials):
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record(stream)
            graph.replay()
            e.record(stream)
            e.synchronize()
            times.append(s.elapsed_time(e) * 1e-3 / reps)
    torch.cuda.current_stream(device).wait_stream(stream)
    torch.cuda.synchronize(device)
    del graph
    return statistics.median(times)


def run_ours(args):
    import torch
    world, rank, local = _dist()
    if not torch.cuda.is_available():
        print(json.dumps({"error": "no CUDA device"}))
        sys.exit(1)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    group = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        # NCCL's communicator log (ranks, transports, NVLS) goes to stderr:
        # NCCL writes it to file descriptor 1, which now points at stderr,
        # and the one JSON line leaves through a copy of the real stdout. A
        # level that prints no communicator lines (unset, WARN, VERSION) is
        # raised to INFO for the INIT subsystem.
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "WARN", "VERSION", "NONE"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        _route_stdout_to_stderr()
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
        group = dist.group.WORLD
    # Which physical GPU each rank ran on (outside the timed region).
    gpu_ids = [str(torch.cuda.get_device_properties(device).uuid)]
    if group is not None:
        gpu_ids = [None] * world
        dist.all_gather_object(gpu_ids, str(torch.cuda.get_device_properties(device).uuid),
                               group=group)
    from ttrl_b200.device import context
    from ttrl_b200.engine.mesh import ParamSync

    ctx = context(device)
    ctx.set_precision(args.precision)
    seed = 1234 + rank * 1_000_003
    learner, host = build_ppo(device, seed)
    sync = ParamSync([learner.net], sync_every=SYNC_EVERY, group=group)
    # L2 flush buffer (> 126 MB), written by our fill kernel between steps.
    flush = torch.empty(64 << 20, dtype=torch.float32, device=device)

    def do_flush():
        ctx.ew("fill", None, None, flush, 0.0)

    # capture + warm-up
    learner.capture()
    launches_per_step = learner.launches_per_replay
    for _ in range(max(args.warmup, 3)):
        learner.replay()
    if group is not None:
        sync.average()
    torch.cuda.synchronize(device)

    # timed region: K rollout updates, each bracketed by its own events. At
    # N > 1 the parameters are averaged after every 50th update and once more
    # after the last one, so every timed region holds ceil(K / 50) averages
    # (one per update at most 50 -- never fewer than the reference's rate).
    K = args.steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    syncs = 0
    sync_after = sync_points(K) if group is not None else set()
    n_sync = len(sync_after)
    sync_s = [torch.cuda.Event(enable_timing=True) for _ in range(n_sync)]
    sync_e = [torch.cuda.Event(enable_timing=True) for _ in range(n_sync)]
    if group is not None:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        for k in range(K):
            do_flush()
            starts[k].record()
            learner.replay()
            if k in sync_after:
                sync_s[syncs].record()
                sync.average()
                sync_e[syncs].record()
                syncs += 1
            ends[k].record()
        torch.cuda.synchronize(device)
    clock = clocks.summary()
    per_step = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(per_step)
    sync_ms = sum(a.elapsed_time(b) for a, b in zip(sync_s[:syncs], sync_e[:syncs]))
    if group is not None:
        import torch.distributed as dist
        t = torch.tensor([total_ms, sync_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, sync_ms = float(t[0].item()), float(t[1].item())
        dist.barrier()
    value = SAMPLES_PER_UPDATE * K * world / (total_ms * 1e-3)

    # end to end through host buffers: per step the rollout (pinned host ->
    # device), fresh permutations, the graph, and the metric read-back.
    pinned = {k: torch.from_numpy(np.ascontiguousarray(v)).pin_memory()
              for k, v in host.items()}
    # At least 20 and up to 60 steps: a single host hiccup (page faults in
    # the pinned-copy path, scheduler noise) moves a 20-step figure by ~15%.
    E = max(20, min(3 * K, 60))
    h2d = sum(v.numel() * v.element_size() for v in pinned.values()) + \
        learner.perm_host.numel() * 4
    d2h = learner.metric_buf.numel() * 4
    if group is not None:
        dist.barrier()
    torch.cuda.synchronize(device)
    staged = (pinned["obs"], pinned["actions"], pinned["old_logp"], pinned["values"],
              pinned["returns"], pinned["adv"])
    e2e_sync = sync_points(E) if group is not None else set()

    def e2e_run() -> float:
        """Seconds for E updates through host buffers (max over ranks)."""
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        # Each step's rollout crosses host -> device and its metric rows
        # device -> host inside the timed region. The upload of step k+1
        # runs on a copy stream beside the replay of step k, and the host
        # waits for a step's metrics two steps later.
        learner.stage_rollout(*staged)
        pending = []
        for k in range(E):
            learner.commit_staged()
            learner.draw_permutations()
            learner.replay()
            if k in e2e_sync:
                sync.average()
            pending.append(learner.fetch_metrics())
            if k + 1 < E:
                learner.stage_rollout(*staged)
            # The host stays up to two updates ahead of the device: it reads
            # the metrics of update k-2 while k-1 and k are queued, so a host
            # hiccup of a few milliseconds leaves no gap on the device.
            if len(pending) > 2:
                learner.metrics_of(pending.pop(0))
        for handle in pending:
            learner.metrics_of(handle)
        sec = time.perf_counter() - t0
        if group is not None:
            t = torch.tensor([sec], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sec = float(t.item())
        return sec

    # Three runs, the median reported: the host side shares its cores and
    # PCIe with the other jobs on the machine, and one slow run moves a
    # single figure by 10-15%.
    e2e_runs = [SAMPLES_PER_UPDATE * E * world / e2e_run() for _ in range(3)]
    e2e = statistics.median(e2e_runs)

    out = None
    if rank == 0:
        peaks = _peaks()
        # live per-kernel roofline (dominant contraction of one minibatch
        # step): each call's median over three eager passes
        passes = [kernel_profile(learner, device) for _ in range(3)]
        prof = [(name, flops, statistics.median(p[i][2] for p in passes))
                for i, (name, flops, _, _) in enumerate(passes[0])]
        # Device time of every contraction of the step: each call re-issued
        # 20x back to back in one graph (its own inputs and outputs).
        dev = [(name, flops, device_time(call, device))
               for name, flops, _, call in passes[-1] if flops > 0]
        dom = max(dev, key=lambda r: r[2])
        achieved = dom[1] / dom[2] / 1e12
        step_tflops = PPO_FLOP_PER_SAMPLE * SAMPLES_PER_UPDATE * K * world / (total_ms * 1e-3) / 1e12
        out = {
            "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world, "steps": K,
            "warmup": max(args.warmup, 3), "ms_per_step": total_ms / K,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": args.precision,
            "data": "synthetic (seeded uint8 frames U{0..255}, actions U[0,6), advantages and "
                    "returns N(0,1), old log-probs and values from the initial policy)",
            "config": {"workload": "ppo_nature_cnn_rollout8x128_mb256_epochs4",
                       "global_batch": MB * world, "minibatch": MB, "rollout": ROLLOUT,
                       "epochs": EPOCHS, "grad_steps_per_step": STEPS_PER_UPDATE,
                       "parallelism": f"dp{world}", "sync_every_updates": SYNC_EVERY,
                       "syncs_in_timed_region": syncs,
                       "ranks": world,
                       "rank_gpus": gpu_ids,
                       "distinct_gpus": len(set(gpu_ids)),
                       "sync_rule": "after every 50th update and after the last one "
                                    "(ceil(steps / 50) averages)" if world > 1 else "none (N=1)",
                       "allreduce_ms_total": round(sync_ms, 4),
                       "allreduce_bytes": int(sync.arena.numel() * 4) if group is not None
                       else 0,
                       "precision": PRECISION_TEXT[args.precision],
                       "l2": "flushed (256 MB write) before every timed step"},
            "e2e": {"value": e2e, "unit": "samples/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "steps": E,
                    "runs": [round(v, 1) for v in e2e_runs],
                    "reduction": f"median of 3 runs of {E} updates"},
            "gpu_launches": launches_per_step * K,
            "gpu_launches_per_step": launches_per_step,
            "roofline": {
                "bound": "tensor", "kernel": dom[0], "achieved": achieved,
                "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16_tflops"],
                "traffic": NCU_TRAFFIC_BYTES.get(dom[0]),
                "peak_source": f"{peaks['source']} dense bf16 (TF32 dense is half"
                               + ("; split-TF32 issues 3 MMAs per product)"
                                  if args.precision == "tf32x3" else ")"),
                "whole_step_tflops": step_tflops,
                "timing": "per-launch device time of the dominant contraction: 20 launches "
                          "back to back in one CUDA graph, events on the replay stream, "
                          "median of 3 replays; operands L2-resident as inside the step",
                "launch_us": round(dom[2] * 1e6, 3),
                # The next-longest contractions: the first place changes hands
                # between launches a few tenths of a microsecond apart.
                "contenders": [
                    {"kernel": n, "launch_us": round(t * 1e6, 3),
                     "frac": f / t / 1e12 / peaks["bf16_tflops"],
                     "traffic": NCU_TRAFFIC_BYTES.get(n)}
                    for n, f, t in sorted(dev, key=lambda r: -r[2])[:3]],
            },
            "kernel_times_us_device": {f"{n}#{i}": round(t * 1e6, 3)
                                       for i, (n, _, t) in enumerate(dev)},
            # Each call timed alone, eagerly, with its own launch latency: not
            # a share of the graph replay (whose kernels overlap on lanes).
            "kernel_times_us_isolated_eager": {f"{n}#{i}": round(t * 1e6, 2)
                                               for i, (n, _, t) in enumerate(prof)},
            "clocks": clock,
        }
        if world == 1 and not args.no_dqn:
            out["dqn"] = bench_dqn(device, args)
            # The same update at the other contraction precision, for reference.
            other = "tf32x3" if args.precision == "tf32" else "tf32"
            ctx.set_precision(other)
            alt = bench_dqn(device, args)
            ctx.set_precision(args.precision)
            out["dqn"]["precision"] = args.precision
            out["dqn"]["other_precision"] = {"precision": other, "value": alt["value"],
                                             "ms_per_update": alt["ms_per_update"]}
            out["sac"] = bench_sac(device, args)
            out["sac"]["precision"] = args.precision
            out["recurrent_ppo"] = bench_recurrent(device, args)
            out["recurrent_ppo"]["precision"] = args.precision
        if world == 1 and not args.no_cpu_baseline:
            times = cpu_ppo_steps(2, seed=2)
            t = statistics.median(times)
            out["cpu_baseline"] = {
                "value": MB / t, "unit": "samples/s", "cores": os.cpu_count(), "kind": "port",
                "sample": "2 PPO minibatch steps of 256 (numpy fp32 restatement of the "
                          "reference's forward, objective, backward, clip and Adam), median"}
    learner.close()
    if group is not None:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if out is not None:
        emit(out)


def bench_dqn(device, args):
    """Nature-DQN batch-32 update (forward x3, double-DQN Huber, backward,
    grad_sq, Adam) as one graph replay through `DQNLearner` (its
    target_sync_interval of 8,000 updates falls outside the timed region);
    updates/sec, device time."""
    import torch
    from ttrl_b200.algos.dqn import DQNLearner
    from ttrl_b200.device import context
    from ttrl_b200.nets import build_q_net
    np.random.seed(7)
    online = build_q_net((4, 84, 84), 6, device, batch=32)
    target = build_q_net((4, 84, 84), 6, device, batch=32)
    learner = DQNLearner(online, target, (4, 84, 84), 6, device, batch=32, lr=1e-4, eps=1.5e-4,
                         double=True, target_sync_interval=8_000)
    rng = np.random.default_rng(3)
    obs = rng.integers(0, 256, (32, 4, 84, 84), dtype=np.uint8)
    nxt = rng.integers(0, 256, (32, 4, 84, 84), dtype=np.uint8)
    act = rng.integers(0, 6, 32)
    arrays = {"obs": obs, "next_obs": nxt, "actions_onehot": np.eye(6, dtype=np.float32)[act],
              "rewards": rng.choice([-1.0, 0.0, 1.0], (32, 1)).astype(np.float32),
              "dones": (rng.random((32, 1)) < 0.01).astype(np.float32),
              "discounts": np.full((32, 1), 0.99, np.float32)}
    learner.update(**arrays)
    step = learner.step
    launches = step.launches_per_replay
    for _ in range(10):
        learner.launch()
    ctx = context(device)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=device)
    K = max(50, args.steps * 5)
    s = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    e = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    torch.cuda.synchronize(device)
    for k in range(K):
        ctx.ew("fill", None, None, flush, 0.0)
        s[k].record()
        learner.launch()
        e[k].record()
    torch.cuda.synchronize(device)
    ms = sum(a.elapsed_time(b) for a, b in zip(s, e)) / K
    # end to end: the batch sits in pinned host memory laid out like the
    # device inputs (TrainStep.pinned_inputs: where a replay sampler writes
    # its rows), and every update uploads it in ONE host-to-device copy
    # (the inputs share one device allocation), replays, reads the metrics.
    pinned = step.pinned_inputs()
    for k, v in arrays.items():
        pinned[k].copy_(torch.from_numpy(np.ascontiguousarray(v)).reshape(pinned[k].shape))
    # 200 updates (about 40 ms): a 50-update sample moved by 25% with one
    # host hiccup.
    E = 200
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    # Every update's inputs go host -> device and its metrics device -> host
    # inside the timed region; the upload of update k+1 runs on a copy stream
    # beside replay k, and the host reads an update's metrics two updates
    # later.
    pending = []
    for _ in range(E):
        learner.load(**pinned)
        learner.launch()
        pending.append(step.fetch_metrics())
        if len(pending) > 2:  # the host reads update k-2's metrics
            step.metrics_of(pending.pop(0))
    for handle in pending:
        step.metrics_of(handle)
    e2e_ms = (time.perf_counter() - t0) * 1000 / E
    h2d = sum(v.nbytes for v in arrays.values())
    learner.close()
    cpu = {}
    if not args.no_cpu_baseline:
        cpu_dqn_updates(2)  # warm-up (BLAS threads, allocations)
        t = statistics.median(cpu_dqn_updates(20, seed=1))
        cpu = {"cpu_baseline": {"value": 1.0 / t, "unit": "updates/s", "cores": os.cpu_count(),
                                "kind": "port",
                                "sample": "median of 20 double-DQN batch-32 updates with Adam "
                                          "(oracle.learner.dqn_update, numpy fp32)"}}
    return {"metric": "Nature-DQN batch-32 learner updates/sec (fwd x3 + bwd + Adam, one graph "
                      "replay per update)",
            "value": 1000.0 / ms, "unit": "updates/s", "ms_per_update": ms,
            "e2e": {"value": 1000.0 / e2e_ms, "unit": "updates/s", "ms_per_update": e2e_ms,
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 3 * 4},
            "gpu_launches_per_update": launches,
            "achieved_tflops": DQN_FLOP_PER_UPDATE / (ms * 1e-3) / 1e12,
            "target": ">= 5000 updates/s", **cpu}


def bench_sac(device, args):
    """SAC MLP update (batch 256, obs 11, action 3: twin critics 14-256-256-1
    with Polyak targets, actor 11-256-256-(3,3), learned temperature, three
    Adams) as one graph replay; updates/sec, device time."""
    import torch
    from ttrl_b200.algos.sac import SACLearner
    from ttrl_b200.device import context
    from ttrl_b200.nets import build_sac_nets
    B, OBS, ACT = 256, 11, 3
    np.random.seed(9)
    nets = build_sac_nets(OBS, ACT, device, batch=B)
    learner = SACLearner(nets, -np.ones(ACT), np.ones(ACT), B, OBS, device)
    rng = np.random.default_rng(4)
    batch = dict(obs=rng.standard_normal((B, OBS)), next_obs=rng.standard_normal((B, OBS)),
                 actions=np.tanh(rng.standard_normal((B, ACT))), rewards=rng.standard_normal((B, 1)),
                 dones=(rng.random((B, 1)) < 0.001) * 1.0, discounts=np.full((B, 1), 0.99),
                 noise=rng.standard_normal((B, ACT)), next_noise=rng.standard_normal((B, ACT)))
    learner.load_batch(**batch)
    for _ in range(max(args.warmup, 3)):
        learner.replay()
    ctx = context(device)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=device)
    K = max(50, args.steps * 5)
    s = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    e = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    torch.cuda.synchronize(device)
    for k in range(K):
        ctx.ew("fill", None, None, flush, 0.0)
        s[k].record()
        learner.replay()
        e[k].record()
    torch.cuda.synchronize(device)
    ms = sum(a.elapsed_time(b) for a, b in zip(s, e)) / K
    out = {"metric": "SAC MLP batch-256 learner updates/sec (critic + actor + temperature + "
                     "Polyak, one graph replay per update)",
           "value": 1000.0 / ms, "unit": "updates/s", "ms_per_update": ms,
           "gpu_launches_per_update": learner.launches_per_replay,
           "achieved_tflops": 0.635e9 / (ms * 1e-3) / 1e12}
    learner.close()
    return out


def bench_recurrent(device, args):
    """Recurrent PPO rollout update (16 envs x 128 steps, BPTT T=32, GRU 256
    on the Nature-CNN trunk, minibatch 512 rows = 16 sequences, 4 epochs =
    16 minibatch steps) as one graph replay; samples/sec over minibatch steps,
    device time."""
    import torch
    from ttrl_b200.algos.ppo import PPOConfig
    from ttrl_b200.algos.recurrent_ppo import RecurrentPPOLearner, shift_to_starts
    from ttrl_b200.device import context
    from ttrl_b200.nets import build_recurrent_actor_critic
    n_steps, n_envs, T, H, rows = 128, 16, 32, 256, 512
    np.random.seed(11)
    net = build_recurrent_actor_critic((4, 84, 84), 6, device, batch=rows, hidden_size=H)
    learner = RecurrentPPOLearner(net, n_steps, n_envs, (4, 84, 84), device,
                                  cfg=PPOConfig(minibatch_size=rows), seq_len=T, seed=5)
    rng = np.random.default_rng(6)
    shape = (n_steps, n_envs)
    boundary = (rng.random(shape) < 0.01).astype(np.float32)
    learner.load_rollout(
        rng.integers(0, 256, shape + (4, 84, 84), dtype=np.uint8), rng.integers(0, 6, shape),
        (np.log(1 / 6) + 0.05 * rng.standard_normal(shape)).astype(np.float32),
        rng.standard_normal(shape).astype(np.float32), rng.standard_normal(shape).astype(np.float32),
        rng.standard_normal(shape).astype(np.float32),
        starts=shift_to_starts(boundary, np.zeros(n_envs)),
        hidden=(0.1 * rng.standard_normal((n_steps // T, n_envs, H))).astype(np.float32))
    learner.draw_permutations()
    for _ in range(max(args.warmup, 3)):
        learner.replay()
    ctx = context(device)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=device)
    K = max(3, args.steps // 10)
    s = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    e = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    torch.cuda.synchronize(device)
    for k in range(K):
        ctx.ew("fill", None, None, flush, 0.0)
        s[k].record()
        learner.replay()
        e[k].record()
    torch.cuda.synchronize(device)
    ms = sum(a.elapsed_time(b) for a, b in zip(s, e)) / K
    steps = learner.steps_per_update
    ms_step = ms / steps
    out = {"metric": "recurrent PPO samples/sec (GRU 256, T=32, minibatch 512 rows, "
                     "16 minibatch steps per graph replay)",
           "value": rows * 1000.0 / ms_step, "unit": "samples/s", "ms_per_minibatch_step": ms_step,
           "gpu_launches_per_step": learner.launches_per_replay / steps,
           "achieved_tflops": RPPO_FLOP_PER_STEP / (ms_step * 1e-3) / 1e12}
    learner.close()
    return out


# ------------------------------------------------------ profiling cases
#
# `python bench.py --profile-case NAME [--batch B] [--reps R]` runs one kernel
# family of the Nature-CNN shapes R times on seeded inputs and exits; the
# ncu summaries under profiles/ name the exact command they came from.

#: (input extent, in channels, out channels, kernel, stride). conv1s2d is
#: conv1 in the space-to-depth form the nets run it in (fold 4), reading raw
#: 0..255 pixels (exact in tf32) as the first layer does.
PROFILE_CONV = {"conv1": (84, 4, 32, 8, 4), "conv1s2d": (21, 64, 32, 2, 1),
                "conv2": (20, 32, 64, 4, 2), "conv3": (9, 64, 64, 3, 1)}
PROFILE_EXACT = ("conv1", "conv1s2d")

#: The Nature-DQN parameter shapes as the device holds them (conv weights
#: KRSC, conv1 folded): 1,687,206 floats.
DQN_PARAM_SHAPES = ((32, 2, 2, 64), (32,), (64, 4, 4, 32), (64,), (64, 3, 3, 64), (64,),
                    (3136, 512), (512,), (512, 6), (6,))


def _profile_conv(layer: str, kind: str):
    def run(args):
        import torch
        from ttrl_b200.device import context, conv_geom
        hw, c, co, k, st = PROFILE_CONV[layer]
        exact = layer in PROFILE_EXACT
        g = conv_geom(args.batch, hw, hw, c, co, k, k, st, 0).with_exact_input(exact)
        rng = np.random.default_rng(0)
        dev = torch.device("cuda", 0)
        x = (rng.integers(0, 256, (args.batch * hw * hw, c)) if exact
             else rng.standard_normal((args.batch * hw * hw, c)))
        x = torch.from_numpy(x.astype(np.float32)).to(dev)
        w = torch.from_numpy(rng.standard_normal((co, k, k, c)).astype(np.float32)).to(dev)
        b = torch.zeros(co, device=dev)
        y = torch.empty((args.batch * g.oh * g.ow, co), device=dev)
        ctx = context(dev)
        for _ in range(args.reps):
            if kind == "fprop":
                ctx.conv_fprop(x, w, b, y, g, 1.0, True)
            elif kind == "dgrad":
                ctx.conv_dgrad(y, w, x, torch.empty_like(x), g, False)
            else:
                ctx.conv_wgrad(x, y, torch.empty_like(w), b, g, 1.0, False, False)
        torch.cuda.synchronize()
    return run


def _profile_fc1(kind: str):
    """The Nature-CNN hidden layer (3136 -> 512) at --batch rows: forward,
    data gradient (ReLU mask fused) or weight gradient (with the bias)."""
    def run(args):
        import torch
        from ttrl_b200.device import context
        dev = torch.device("cuda", 0)
        rng = np.random.default_rng(0)
        x = torch.from_numpy(rng.standard_normal((args.batch, 3136)).astype(np.float32)).to(dev)
        w = torch.from_numpy(rng.standard_normal((3136, 512)).astype(np.float32)).to(dev)
        b = torch.zeros(512, device=dev)
        y = torch.empty((args.batch, 512), device=dev)
        ctx = context(dev)
        for _ in range(args.reps):
            if kind == "fwd":
                ctx.linear_fwd(x, w, b, y, True)
            elif kind == "dgrad":
                ctx.linear_dgrad(y, w, x, torch.empty_like(x), False)
            else:
                ctx.linear_wgrad(x, y, torch.empty_like(w), b, False, False)
        torch.cuda.synchronize()
    return run


def _dqn_param_tensors(sets: int):
    """`sets` copies of the Nature-DQN parameter list with seeded gradients."""
    import torch
    from ttrl_b200.engine.autograd import Tensor
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(0)
    params = []
    for _ in range(sets):
        for shape in DQN_PARAM_SHAPES:
            p = Tensor(torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(dev),
                       requires_grad=True)
            p.grad = torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(dev)
            params.append(p)
    return params


def _profile_adam(sets: int):
    def run(args):
        import torch
        from ttrl_b200.engine.optim import Adam
        params = _dqn_param_tensors(sets)
        opt = Adam(params, lr=1e-4, eps=1.5e-4)
        for _ in range(args.reps):
            opt.step()
        torch.cuda.synchronize()
    return run


def _profile_sqnorm(sets: int):
    def run(args):
        import torch
        from ttrl_b200.algos.grads import grad_sq_device
        params = _dqn_param_tensors(sets)
        for _ in range(args.reps):
            grad_sq_device(params)
        torch.cuda.synchronize()
    return run


def _profile_u8_s2d(args):
    import torch
    from ttrl_b200.device import context
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(0)
    frames = torch.from_numpy(rng.integers(0, 256, (args.batch, 4, 84, 84),
                                           dtype=np.uint8)).to(dev)
    out = torch.empty((args.batch * 21 * 21, 64), device=dev)
    ctx = context(dev)
    for _ in range(args.reps):
        ctx.u8_to_f32(frames, None, out, 1.0, fold=4)
    torch.cuda.synchronize()


def _profile_dqn(args):
    import torch
    from ttrl_b200.algos import dqn
    from ttrl_b200.engine.optim import Adam
    from ttrl_b200.engine.step import TrainStep
    from ttrl_b200.nets import build_q_net
    np.random.seed(0)
    online = build_q_net((4, 84, 84), 6, "cuda", batch=32)
    target = build_q_net((4, 84, 84), 6, "cuda", batch=32)
    opt = Adam(list(online.parameters()), lr=1e-4, eps=1.5e-4)
    inputs = dqn.step_inputs((4, 84, 84), "cuda", batch=32, num_actions=6)
    step = TrainStep(lambda i: dqn.update_loss(online, target, i, num_actions=6), inputs,
                     "cuda", optimizer=opt, mode="traced_fwd_bwd")
    rng = np.random.default_rng(1)
    step.load_input("obs", rng.integers(0, 256, (32, 4, 84, 84), dtype=np.uint8))
    step.load_input("next_obs", rng.integers(0, 256, (32, 4, 84, 84), dtype=np.uint8))
    step.load_input("actions_onehot", np.eye(6, dtype=np.float32)[rng.integers(0, 6, 32)])
    for _ in range(args.reps):
        step.launch()
    torch.cuda.synchronize()
    step.close()


def _profile_ppo(args):
    """One PPO rollout update (8 x 128 frames, 4 epochs x 4 minibatches of
    256) replayed `reps` times from its CUDA graph."""
    import torch
    learner, _ = build_ppo(torch.device("cuda", 0), 0)
    learner.capture()
    for _ in range(args.reps):
        learner.replay()
    torch.cuda.synchronize()
    learner.close()


def _profile_rppo(args):
    """One recurrent PPO rollout update (16 x 128 frames, T=32, GRU 256,
    4 epochs x 4 minibatches of 16 sequences) replayed `reps` times."""
    import torch
    from ttrl_b200.algos.ppo import PPOConfig
    from ttrl_b200.algos.recurrent_ppo import RecurrentPPOLearner
    from ttrl_b200.nets import build_recurrent_actor_critic
    np.random.seed(0)
    net = build_recurrent_actor_critic((4, 84, 84), 6, "cuda", batch=512, hidden_size=256)
    learner = RecurrentPPOLearner(net, 128, 16, (4, 84, 84), "cuda",
                                  cfg=PPOConfig(minibatch_size=512), seq_len=32)
    rng = np.random.default_rng(0)
    shape = (128, 16)
    learner.load_rollout(rng.integers(0, 256, shape + (4, 84, 84), dtype=np.uint8),
                         rng.integers(0, 6, shape), np.full(shape, np.log(1 / 6), np.float32),
                         rng.standard_normal(shape), rng.standard_normal(shape),
                         rng.standard_normal(shape),
                         starts=(rng.random(shape) < 0.01).astype(np.float32),
                         hidden=np.zeros((4, 16, 256), np.float32))
    learner.draw_permutations()
    learner.capture()
    for _ in range(args.reps):
        learner.replay()
    torch.cuda.synchronize()
    learner.close()


def _profile_sac(args):
    import torch
    from ttrl_b200.algos.sac import SACLearner
    from ttrl_b200.nets import build_sac_nets
    B, OBS, ACT = 256, 11, 3
    np.random.seed(9)
    nets = build_sac_nets(OBS, ACT, "cuda", batch=B)
    learner = SACLearner(nets, -np.ones(ACT), np.ones(ACT), B, OBS, "cuda")
    rng = np.random.default_rng(4)
    learner.load_batch(obs=rng.standard_normal((B, OBS)), next_obs=rng.standard_normal((B, OBS)),
                       actions=np.tanh(rng.standard_normal((B, ACT))),
                       rewards=rng.standard_normal((B, 1)),
                       dones=(rng.random((B, 1)) < 0.001) * 1.0,
                       discounts=np.full((B, 1), 0.99), noise=rng.standard_normal((B, ACT)),
                       next_noise=rng.standard_normal((B, ACT)))
    for _ in range(args.reps):
        learner.replay()
    torch.cuda.synchronize()
    learner.close()


PROFILE_CASES = {f"{layer}_{kind}": _profile_conv(layer, kind)
                 for layer in PROFILE_CONV for kind in ("fprop", "dgrad", "wgrad")}
PROFILE_CASES.update({
    "fc1_fwd": _profile_fc1("fwd"), "fc1_dgrad": _profile_fc1("dgrad"),
    "fc1_wgrad": _profile_fc1("wgrad"), "adam_dqn": _profile_adam(1), "adam_dqn_x4": _profile_adam(4),
    "sqnorm_dqn": _profile_sqnorm(1), "sqnorm_dqn_x4": _profile_sqnorm(4),
    "u8_s2d": _profile_u8_s2d, "dqn_update": _profile_dqn, "ppo_update": _profile_ppo,
    "rppo_update": _profile_rppo, "sac_update": _profile_sac,
})


def main():
    args = _args()
    if args.profile_case is not None:
        PROFILE_CASES[args.profile_case](args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    run_ours(args)


if __name__ == "__main__":
    main()
