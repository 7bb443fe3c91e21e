"""PPO's learning half on the B200 kernels (ttrl/algos/ppo/{loss,learn}.py).

`objective` has the reference's signature and semantics (clipped surrogate,
PPO2 value clipping with the 0.5, entropy bonus; mean or masked-mean
reduction) and runs as one fused kernel that also produces d loss / d
(logits, value).

`PPOLearner` is the graph-replayed learner: the rollout lives in HBM (uint8
frames plus the per-sample fields), each minibatch is gathered on the device
by index, and one CUDA graph holds every gradient step of a rollout update
-- `epochs x minibatches` of forward, loss, backward, device-side grad-norm
clip and fused Adam. The minibatch permutations are drawn on the host from
the learner's numpy generator exactly as ttrl/buffers/rollout.py:241-283
draws them, and uploaded (a few KB) before each replay.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from ttrl_b200.algos.grads import clip_grad_norm_device
from ttrl_b200.device import PREP_LANE, context
from ttrl_b200.engine.nn import parameter_arena
from ttrl_b200.engine.autograd import Tensor, as_device, no_grad
from ttrl_b200.engine.conv import input_fold
from ttrl_b200.engine.ops import ppo_objective
from ttrl_b200.engine.optim import Adam
from ttrl_b200.engine.trace import capture

__all__ = ["PPOConfig", "PPOLearner", "ReplayedUpdate", "objective", "normalize_advantages"]


@dataclass(frozen=True)
class PPOConfig:
    """The learner fields of ttrl/algos/ppo/config.py:22-211 this path reads."""
    clip_eps: float = 0.1
    value_clip_eps: float = 0.1
    value_coef: float = 0.5
    entropy_coef: float = 0.01
    lr: float = 2.5e-4
    eps: float = 1e-8
    max_grad_norm: float = 0.5
    epochs: int = 4
    minibatch_size: int = 256
    normalize_adv: bool = True
    gamma: float = 0.99
    lam: float = 0.95


def normalize_advantages(adv: np.ndarray) -> np.ndarray:
    """(adv - mean) / (std + 1e-8) over the whole rollout
    (ttrl/buffers/rollout.py:269-270)."""
    adv = np.asarray(adv)
    return (adv - adv.mean()) / (adv.std() + 1e-8)


def objective(logits: Tensor, value: Tensor, batch: dict, cfg: PPOConfig, *, valid=None):
    """-> (loss, parts, new_logp) for one minibatch; `batch` holds device
    tensors actions (int32), old_logp, advantages, returns, values."""
    return ppo_objective(
        logits, value, batch["actions"], batch["old_logp"], batch["advantages"],
        batch["returns"], batch["values"], clip_eps=cfg.clip_eps,
        value_clip_eps=cfg.value_clip_eps, value_coef=cfg.value_coef,
        entropy_coef=cfg.entropy_coef, valid=valid)


class ReplayedUpdate:
    """What a graph-replayed on-policy learner shares: the whole update
    (`steps_per_update` calls of `_minibatch_step`) run op by op or captured
    once and replayed, and the per-step metric rows read back once."""

    METRICS = ("loss", "policy_loss", "value_loss", "entropy", "grad_sq")

    def _update_body(self) -> None:
        for k in range(self.steps_per_update):
            self._minibatch_step(k)

    def update_eager(self) -> None:
        """One rollout update, op by op (no graph)."""
        self._update_body()
        self.optimizer.captured_indices = None

    def capture(self) -> None:
        """Warm up (kernel loading, workspace and gradient buffers), then
        capture one whole rollout update into a CUDA graph."""
        # Warm-up on scratch copies of the parameters would change nothing
        # observable except the first update; run one real minibatch step
        # and roll the optimizer state back so replays start from step 0.
        saved = [p.data.clone() for p in self.params]
        m_saved = [m.clone() for m in self.optimizer.m]
        v_saved = [v.clone() for v in self.optimizer.v]
        steps_saved = self.optimizer._dev_steps.clone()
        host_steps = (self.optimizer.t, list(self.optimizer.steps))
        self._minibatch_step(0)
        torch.cuda.synchronize(self.device)
        for p, s in zip(self.params, saved):
            p.data.copy_(s)
        for m, s in zip(self.optimizer.m, m_saved):
            m.copy_(s)
        for v, s in zip(self.optimizer.v, v_saved):
            v.copy_(s)
        self.optimizer._dev_steps.copy_(steps_saved)
        self.optimizer.t, self.optimizer.steps = host_steps[0], host_steps[1]
        from ttrl_b200._lib import lib
        before = lib().ttrl_launch_count()
        # The side lanes carry only weight gradients and the next step's
        # inputs: the main chain runs at the higher stream priority.
        self._graph, _ = capture(self.device, self._update_body, critical_main=True)
        self.launches_per_replay = int(lib().ttrl_launch_count() - before)

    def replay(self) -> None:
        """One rollout update (epochs x minibatches gradient steps)."""
        if self._graph is None:
            self.capture()
        self._graph.replay()
        opt = self.optimizer
        for _ in range(self.steps_per_update):
            opt.advance(range(len(self.params)))

    def read_metrics(self) -> dict:
        """Mean over the rollout update's steps, like ttrl/algos/ppo/learn.py:69-73."""
        return self._metrics_of(self.metric_buf.detach().to("cpu").numpy())

    def fetch_metrics(self):
        """Start copying this update's metric rows to pinned host memory on the
        current stream and return a handle; `metrics_of(handle)` waits for that
        copy only, so the next update can be enqueued before the host blocks."""
        host = torch.empty(self.metric_buf.shape, dtype=self.metric_buf.dtype, pin_memory=True)
        host.copy_(self.metric_buf, non_blocking=True)
        done = torch.cuda.Event()
        done.record(torch.cuda.current_stream(self.device))
        return host, done

    def metrics_of(self, handle) -> dict:
        host, done = handle
        done.synchronize()
        return self._metrics_of(host.numpy())

    def _metrics_of(self, rows) -> dict:
        host = np.asarray(rows, np.float64)
        out = {k: float(host[:, j].mean()) for j, k in enumerate(self.METRICS)}
        out["grad_norm"] = float(np.sqrt(host[:, 4]).mean())
        out["minibatches"] = float(self.steps_per_update)
        return out

    def close(self) -> None:
        if self._graph is not None:
            self._graph.close()
            self._graph = None

    def _record_metrics(self, k: int, loss, parts, norm) -> None:
        """Step k's metric row: loss, the three parts and the squared grad norm."""
        row = self.metric_buf[k]
        sources = [loss.data.reshape(1)] + [parts[key].data.reshape(1) for key in
                                            ("policy_loss", "value_loss", "entropy")] + [norm[0:1]]
        self.ctx.blend([(row[j:j + 1], src) for j, src in enumerate(sources)])  # one copy launch


class PPOLearner(ReplayedUpdate):
    """Graph-replayed PPO learner over a device-resident rollout."""

    def __init__(self, net, rollout_size: int, obs_shape, device=None, *,
                 cfg: PPOConfig = PPOConfig(), seed: int = 0, minibatches: int | None = None):
        """`minibatches` per epoch fixes the captured graph; it defaults to
        rollout_size // minibatch_size, the count of a rollout without
        autoreset padding (a padded rollout yields valid_slots // size)."""
        self.net = net
        self.cfg = cfg
        self.device = as_device(device)
        self.ctx = context(self.device)
        self.rollout_size = int(rollout_size)
        self.obs_shape = tuple(int(v) for v in obs_shape)
        mb = cfg.minibatch_size
        self.minibatches = self.rollout_size // mb if minibatches is None else int(minibatches)
        if self.minibatches == 0 or self.minibatches * mb > self.rollout_size:
            raise ValueError(f"rollout of {rollout_size} holds no minibatch of {mb}")
        self.steps_per_update = cfg.epochs * self.minibatches
        # One flat arena for the parameters: a replica average is one
        # in-place collective over it (ttrl_b200.engine.mesh.ParamSync).
        self.param_arena = parameter_arena([net])
        self.params = list(net.parameters())
        self.optimizer = Adam(self.params, lr=cfg.lr, eps=cfg.eps)
        self.rng = np.random.default_rng(seed)
        dev = self.device
        c, h, w = self.obs_shape
        R = self.rollout_size
        # Device-resident rollout (address-stable: written in place).
        self.obs = torch.zeros((R, c, h, w), dtype=torch.uint8, device=dev)
        self.actions = torch.zeros(R, dtype=torch.int32, device=dev)
        self.old_logp = torch.zeros(R, dtype=torch.float32, device=dev)
        self.values = torch.zeros(R, dtype=torch.float32, device=dev)
        self.returns = torch.zeros(R, dtype=torch.float32, device=dev)
        self.advantages = torch.zeros(R, dtype=torch.float32, device=dev)
        self.perm = torch.zeros((self.steps_per_update, mb), dtype=torch.int32, device=dev)
        # Three pinned buffers for the host's permutations, so the host may
        # draw the next update's while the last two uploads are in flight.
        self._perm_ring = [torch.zeros((self.steps_per_update, mb), dtype=torch.int32,
                                       pin_memory=True) for _ in range(3)]
        self._perm_events = [None] * len(self._perm_ring)
        self._perm_slot = 0
        # Minibatch staging (gathered per step on the device).
        # Frame rows in the order the first convolution reads (space-to-depth
        # when it folds), gathered and converted from the uint8 rollout.
        self.fold = input_fold(net)
        f2 = self.fold * self.fold
        # Two sets: step k's inputs are gathered on the preparation lane
        # while step k - 1 runs (see _minibatch_step).
        self._mb_sets = [
            (torch.empty((1, 1, mb * h * w // f2, c * f2), dtype=torch.float32, device=dev),
             torch.empty(mb, dtype=torch.int32, device=dev),
             {k: torch.empty(mb, dtype=torch.float32, device=dev)
              for k in ("old_logp", "values", "returns", "advantages")})
            for _ in range(2)]
        self._prepared = None  # the step whose inputs are already being gathered
        self.metric_buf = torch.zeros((self.steps_per_update, len(self.METRICS)),
                                      dtype=torch.float32, device=dev)
        self.keep = None  # valid slot indices when the rollout has padding slots
        self._graph = None
        self.launches_per_replay = 0

    # -- rollout -----------------------------------------------------------

    def load_rollout(self, obs_u8, actions, old_logp, values, returns, advantages) -> None:
        """Upload one rollout (host arrays). Advantages are normalised over
        the rollout here when cfg.normalize_adv, as the reference does."""
        adv = normalize_advantages(advantages) if self.cfg.normalize_adv else advantages
        self.keep = None
        self.obs.copy_(torch.from_numpy(np.ascontiguousarray(obs_u8, np.uint8)))
        self.actions.copy_(torch.from_numpy(np.asarray(actions, np.int32)))
        self.old_logp.copy_(torch.from_numpy(np.asarray(old_logp, np.float32)))
        self.values.copy_(torch.from_numpy(np.asarray(values, np.float32)))
        self.returns.copy_(torch.from_numpy(np.asarray(returns, np.float32)))
        self.advantages.copy_(torch.from_numpy(np.asarray(adv, np.float32)))

    # -- overlapped upload -------------------------------------------------

    _STAGED = ("obs", "actions", "old_logp", "values", "returns", "advantages")

    def stage_rollout(self, obs_u8, actions, old_logp, values, returns,
                      advantages) -> torch.cuda.Event:
        """Start uploading the NEXT rollout (pinned host tensors, already
        normalised advantages) into device staging buffers on a copy stream,
        beside whatever update is running; `commit_staged()` makes it the
        rollout the next replay reads.

        The copies read the host tensors asynchronously. The returned event
        completes once they have; until then the host tensors must not be
        changed (wait on it with `event.synchronize()` before refilling a
        pinned buffer for the next rollout)."""
        if getattr(self, "_staging", None) is None:
            self._staging = {k: torch.empty_like(getattr(self, k)) for k in self._STAGED}
            self._copy_stream = self._upload_stream()
            self._staged = None
            self._committed = None
        src = dict(zip(self._STAGED, (obs_u8, actions, old_logp, values, returns, advantages)))
        with torch.cuda.stream(self._copy_stream):
            if self._committed is not None:
                # The previous commit has read the staging buffers.
                self._copy_stream.wait_event(self._committed)
            for k, t in src.items():
                self._staging[k].copy_(t.reshape(self._staging[k].shape), non_blocking=True)
            self._staged = torch.cuda.Event()
            self._staged.record(self._copy_stream)
        return self._staged

    def _upload_stream(self) -> torch.cuda.Stream:
        """The stream host-to-device uploads run on, beside the updates."""
        if getattr(self, "_uploads", None) is None:
            self._uploads = torch.cuda.Stream(self.device)
        return self._uploads

    def commit_staged(self) -> None:
        """Order the current stream after the staged upload and copy it into
        the buffers the captured update reads (device to device)."""
        if getattr(self, "_staged", None) is None:
            raise RuntimeError("commit_staged: no rollout was staged")
        main = torch.cuda.current_stream(self.device)
        main.wait_event(self._staged)
        # One copy kernel over every staged array (moved as 4-byte words, bit
        # for bit): a device-to-device memcpy runs on a copy engine at a
        # fraction of the SMs' bandwidth (0.3 ms for the 28.9 MB of frames).
        self.ctx.blend([(getattr(self, k).reshape(-1).view(torch.float32),
                         self._staging[k].reshape(-1).view(torch.float32))
                        for k in self._STAGED])
        self.keep = None
        self._committed = torch.cuda.Event()
        self._committed.record(main)
        self._staged = None

    def load_rollout_raw(self, obs_u8, actions, old_logp, values, rewards, dones, last_values,
                         valid=None) -> None:
        """Upload one collected rollout ([n_steps, n_envs] arrays, slot
        t * n_envs + lane; obs [n_steps, n_envs, C, H, W]) and derive the
        advantages and returns on the device: GAE-lambda with cfg.gamma and
        cfg.lam (ttrl/buffers/rollout.py:195-227), then, when
        cfg.normalize_adv, normalisation over the valid slots (:269-270).
        Minibatches then draw only valid slots, as the reference's do."""
        values = np.asarray(values, np.float32)
        steps, envs = values.shape
        if steps * envs != self.rollout_size:
            raise ValueError(f"load_rollout_raw: {steps} x {envs} slots, the learner holds "
                             f"{self.rollout_size}")
        dev = self.device
        up = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)
        self.obs.copy_(torch.from_numpy(np.ascontiguousarray(obs_u8, np.uint8)).reshape(
            self.obs.shape))
        self.actions.copy_(torch.from_numpy(np.asarray(actions, np.int32).reshape(-1)))
        self.old_logp.copy_(up(old_logp).reshape(-1))
        self.values.copy_(up(values).reshape(-1))
        valid_d = None if valid is None else up(valid)
        ctx = self.ctx
        ctx.gae(up(rewards), self.values.reshape(steps, envs), up(dones), valid_d,
                up(last_values).reshape(envs), self.advantages.reshape(steps, envs),
                self.returns.reshape(steps, envs), self.cfg.gamma, self.cfg.lam)
        if self.cfg.normalize_adv:
            ctx.normalize_advantages(self.advantages, None if valid_d is None else
                                     valid_d.reshape(-1), self.advantages)
        self.keep = (None if valid is None else
                     np.flatnonzero(np.asarray(valid, np.float32).reshape(-1) > 0.0))
        total = self.rollout_size if self.keep is None else len(self.keep)
        if total // self.cfg.minibatch_size != self.minibatches:
            raise ValueError(
                f"load_rollout_raw: {total} valid transitions make "
                f"{total // self.cfg.minibatch_size} minibatches of {self.cfg.minibatch_size}, "
                f"and this learner's captured graph holds {self.minibatches} per epoch")

    @property
    def perm_host(self) -> torch.Tensor:
        """The pinned host copy of the last drawn permutations."""
        return self._perm_ring[self._perm_slot]

    def draw_permutations(self) -> None:
        """One permutation of the (valid) rollout slots per epoch, cut into
        minibatches (ttrl/buffers/rollout.py:241-283)."""
        mb = self.cfg.minibatch_size
        slot = (self._perm_slot + 1) % len(self._perm_ring)
        if self._perm_events[slot] is not None:
            # The upload out of this buffer, three draws ago, has read it.
            self._perm_events[slot].synchronize()
        buf = self._perm_ring[slot]
        keep = self.keep
        total = self.rollout_size if keep is None else len(keep)
        rows = []
        for _ in range(self.cfg.epochs):
            perm = self.rng.permutation(total)
            for start in range(0, self.minibatches * mb, mb):
                idx = perm[start:start + mb]
                rows.append(idx if keep is None else keep[idx])
        buf.numpy()[:] = np.stack(rows).astype(np.int32)
        # The host-to-device copy runs on the copy stream into a device
        # staging buffer, queued ahead of any rollout upload issued later; the
        # current stream then moves it into place with one copy kernel. A
        # host-to-device copy on the current stream would wait on the copy
        # engine behind a rollout upload in flight (0.3-1.2 ms per update).
        main = torch.cuda.current_stream(self.device)
        cs = self._upload_stream()
        if getattr(self, "_perm_stage", None) is None:
            self._perm_stage = torch.empty_like(self.perm)
            self._perm_consumed = None
        with torch.cuda.stream(cs):
            if self._perm_consumed is not None:
                cs.wait_event(self._perm_consumed)  # the last move has read the stage
            self._perm_stage.copy_(buf, non_blocking=True)
            done = torch.cuda.Event()
            done.record(cs)
        main.wait_event(done)
        self.ctx.blend([(self.perm.view(-1).view(torch.float32),
                         self._perm_stage.view(-1).view(torch.float32))])
        self._perm_consumed = torch.cuda.Event()
        self._perm_consumed.record(main)
        self._perm_events[slot] = done
        self._perm_slot = slot

    # -- one gradient step ---------------------------------------------------

    def _prepare_inputs(self, k: int) -> None:
        """Gather step k's minibatch into input set k % 2 (on the current
        stream): its frames converted to the first layer's rows, and its
        actions and per-sample fields."""
        mb_rows, mb_actions, mb_fields = self._mb_sets[k % 2]
        idx = self.perm[k]
        c = self.obs_shape[0]
        f2 = self.fold * self.fold
        self.ctx.u8_to_f32(self.obs, idx, mb_rows.reshape(-1, c * f2), 1.0, fold=self.fold)
        self.ctx.gather_rows_multi(
            [(self.actions, mb_actions)]
            + [(src, mb_fields[name]) for name, src in (
                ("old_logp", self.old_logp), ("values", self.values),
                ("returns", self.returns), ("advantages", self.advantages))], idx)

    def _update_body(self) -> None:
        self._prepared = None
        super()._update_body()

    def _minibatch_step(self, k: int) -> None:
        cfg = self.cfg
        ctx = self.ctx
        if self._prepared != k:
            self._prepare_inputs(k)
        # The next step's inputs are gathered on the preparation lane beside
        # this step's forward and backward; the backward's closing join
        # orders this step's optimizer step, and so the next step, after it.
        # The set it fills was last read by step k - 1, which has finished
        # on every lane by now.
        if k + 1 < self.steps_per_update:
            with ctx.side(PREP_LANE):
                self._prepare_inputs(k + 1)
            self._prepared = k + 1
        else:
            self._prepared = None
        mb_rows, mb_actions, mb_fields = self._mb_sets[k % 2]
        self.optimizer.zero_grad()
        rows = Tensor(mb_rows)
        rows._exact = True  # raw 0..255 frame values
        rows._fold = self.fold
        logits, value = self.net(rows)
        loss, parts, _ = ppo_objective(
            logits, value, mb_actions, mb_fields["old_logp"],
            mb_fields["advantages"], mb_fields["returns"], mb_fields["values"],
            clip_eps=cfg.clip_eps, value_clip_eps=cfg.value_clip_eps,
            value_coef=cfg.value_coef, entropy_coef=cfg.entropy_coef)
        loss.backward()
        norm = clip_grad_norm_device(self.params, cfg.max_grad_norm, self.optimizer)
        self.optimizer.step()
        self._record_metrics(k, loss, parts, norm)


def initial_old_logp(net, obs_u8: np.ndarray, actions: np.ndarray, device, chunk: int = 256):
    """log pi_0(a|s) and V_0(s) of the initial policy over a rollout, by the
    device forward (setup only; not part of a timed update)."""
    dev = as_device(device)
    ctx = context(dev)
    n, c, h, w = obs_u8.shape
    logp = np.zeros(n, np.float32)
    vals = np.zeros(n, np.float32)
    frames = torch.from_numpy(np.ascontiguousarray(obs_u8)).to(dev)
    fold = input_fold(net)
    f2 = fold * fold
    rows = torch.empty((1, 1, chunk * h * w // f2, c * f2), dtype=torch.float32, device=dev)
    with no_grad():
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            if e - s != chunk:
                raise ValueError("rollout size must be a multiple of the chunk")
            ctx.u8_to_f32(frames[s:e], None, rows.reshape(-1, c * f2), 1.0, fold=fold)
            x = Tensor(rows)
            x._exact = True
            x._fold = fold
            logits, value = net(x)
            lg = logits.numpy().astype(np.float64)
            mx = lg.max(axis=1, keepdims=True)
            lsm = lg - mx - np.log(np.exp(lg - mx).sum(axis=1, keepdims=True))
            logp[s:e] = lsm[np.arange(e - s), actions[s:e]]
            vals[s:e] = value.numpy().reshape(-1)
    return logp, vals
