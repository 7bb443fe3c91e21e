"""Recurrent PPO's learning half on the B200 kernels
(ttrl/algos/ppo/recurrent.py:179-227 over ttrl/buffers/seqbatch.py and
ttrl/buffers/sequences.py).

The rollout stays in HBM in the reference's [n_steps][n_envs] slot order
(slot t * n_envs + lane): observations, actions, the per-slot fields, the
`valid` and `starts` flags, and the state entering each sequence's first step
(`hidden`, [n_chunks * n_envs][H], indexed by the sequence id
chunk * n_envs + lane). A minibatch is a set of whole sequences: the host draws
the sequence permutation exactly as ttrl/buffers/seqbatch.py:69-84 does,
turns each minibatch into its time-major row -> slot index (row
t * n_seq + s holds slot (chunk_s * seq_len + t) * n_envs + lane_s) and
uploads those few KB before each replay; every gather then runs on the
device. One CUDA graph holds all `epochs x minibatches` gradient steps:
gathers, trunk, the fused GRU unroll, heads, the masked-mean PPO objective,
backward (BPTT), device-side grad-norm clip and fused Adam.

Invalid (autoreset padding) slots have their advantages, returns and old
log-probs zeroed when the rollout is loaded; the reference zeroes the same
per-slot fields per minibatch (ttrl/algos/ppo/recurrent.py:211-218), which is
the same per-slot operation. Advantages are normalised over valid slots only
(ttrl/buffers/seqbatch.py:86-101).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from ttrl_b200.algos.grads import clip_grad_norm_device
from ttrl_b200.algos.ppo import PPOConfig, ReplayedUpdate
from ttrl_b200.device import context
from ttrl_b200.engine.nn import parameter_arena
from ttrl_b200.engine.autograd import Tensor, as_device
from ttrl_b200.engine.conv import input_fold
from ttrl_b200.engine.ops import ppo_objective
from ttrl_b200.engine.optim import Adam
from ttrl_b200.nets.recurrent import ACTOR

__all__ = ["RecurrentConfig", "RecurrentPPOLearner", "chunk_count", "chunks_per_minibatch",
           "shift_to_starts", "normalize_valid_advantages", "sequence_rows"]


@dataclass(frozen=True)
class RecurrentConfig:
    """ttrl/algos/ppo/config.py RecurrentConfig: the GRU width and the BPTT
    length of one sequence."""
    hidden_size: int = 256
    seq_len: int = 32


def chunk_count(n_steps: int, seq_len: int) -> int:
    """Sequences per lane (ttrl/buffers/sequences.py:54-72)."""
    if seq_len < 1:
        raise ValueError(f"seq_len must be >= 1, got {seq_len}")
    if n_steps % seq_len:
        raise ValueError(
            f"seq_len={seq_len} does not divide n_steps={n_steps}, which would leave a final "
            f"sequence of {n_steps % seq_len} steps. The unroll is built for one fixed T, so a "
            f"short tail is a second graph shape rather than a smaller batch. Choose a seq_len "
            f"dividing {n_steps}.")
    return n_steps // seq_len


def chunks_per_minibatch(minibatch_size: int, seq_len: int) -> int:
    """Whole sequences per minibatch (ttrl/buffers/sequences.py:75-90)."""
    if minibatch_size % seq_len:
        raise ValueError(
            f"minibatch_size={minibatch_size} is not a multiple of seq_len={seq_len}. A "
            f"recurrent minibatch is a whole number of sequences of seq_len steps, so its row "
            f"count is n_sequences * seq_len.")
    return minibatch_size // seq_len


def shift_to_starts(boundary, carried) -> np.ndarray:
    """starts[t] = boundary[t - 1], starts[0] = the flag carried over from the
    previous rollout (ttrl/buffers/sequences.py:93-126)."""
    boundary = np.asarray(boundary, dtype=np.float32)
    if boundary.ndim != 2:
        raise ValueError(f"shift_to_starts: boundary must be [T, n_envs], got shape "
                         f"{boundary.shape}")
    carried = np.asarray(carried, dtype=np.float32).reshape(1, -1)
    if carried.shape[1] != boundary.shape[1]:
        raise ValueError(f"shift_to_starts: carried covers {carried.shape[1]} lanes and "
                         f"boundary covers {boundary.shape[1]}")
    return np.concatenate([carried, boundary[:-1]], axis=0)


def normalize_valid_advantages(adv: np.ndarray, valid: np.ndarray) -> np.ndarray:
    """(adv - mean) / (std + 1e-8) with the statistics over valid slots only,
    applied to every slot (ttrl/buffers/seqbatch.py:86-101)."""
    adv = np.asarray(adv, np.float32)
    live = np.asarray(valid) > 0.0
    if not live.any():
        raise ValueError(
            "RolloutBuffer.sequence_minibatches: the rollout holds no valid transitions, so "
            "the advantage statistics have nothing to normalize against")
    values = adv[live]
    return (adv - values.mean()) / (values.std() + 1e-8)


def sequence_rows(ids: np.ndarray, n_envs: int, seq_len: int) -> np.ndarray:
    """Sequence ids -> the time-major slot index of every row: row
    t * n_seq + s is slot (chunk_s * seq_len + t) * n_envs + lane_s, with
    chunk = id // n_envs and lane = id % n_envs (ttrl/buffers/seqbatch.py:80-84,
    ttrl/buffers/sequences.py:129-161)."""
    ids = np.asarray(ids, np.int64)
    chunks, lanes = ids // n_envs, ids % n_envs
    steps = chunks[None, :] * seq_len + np.arange(seq_len, dtype=np.int64)[:, None]
    return (steps * n_envs + lanes[None, :]).reshape(-1)


class RecurrentPPOLearner(ReplayedUpdate):
    """Graph-replayed recurrent PPO over a device-resident sequence rollout.

    `obs_shape` is (C, H, W) for uint8 frames (the Nature-CNN trunk) or (D,)
    for float vectors (the MLP trunk).
    """

    def __init__(self, net, n_steps: int, n_envs: int, obs_shape, device=None, *,
                 cfg: PPOConfig = PPOConfig(minibatch_size=512), seq_len: int = 32,
                 seed: int = 0):
        self.net = net
        self.cfg = cfg
        self.device = as_device(device)
        self.ctx = context(self.device)
        self.n_steps, self.n_envs = int(n_steps), int(n_envs)
        self.seq_len = int(seq_len)
        self.obs_shape = tuple(int(v) for v in obs_shape)
        self.image = len(self.obs_shape) == 3
        self.n_chunks = chunk_count(self.n_steps, self.seq_len)
        self.n_seq = chunks_per_minibatch(cfg.minibatch_size, self.seq_len)
        self.total_sequences = self.n_chunks * self.n_envs
        self.minibatches = self.total_sequences // self.n_seq
        if self.minibatches == 0:
            raise ValueError(
                f"RolloutBuffer.sequence_minibatches: the rollout holds {self.total_sequences} "
                f"sequences of {self.seq_len} steps (n_steps={self.n_steps}, "
                f"n_envs={self.n_envs}) and a minibatch of {cfg.minibatch_size} rows wants "
                f"{self.n_seq} of them, which would yield zero minibatches.")
        self.steps_per_update = cfg.epochs * self.minibatches
        self.rows = self.n_seq * self.seq_len
        hidden = dict(net.hidden_sizes)
        if set(hidden) != {ACTOR}:
            raise ValueError("RecurrentPPOLearner: one shared memory is supported (a single-leaf "
                             f"observation), got memories {sorted(hidden)}")
        self.hidden_size = int(hidden[ACTOR])
        # One flat arena for the parameters: a replica average is one
        # in-place collective over it (ttrl_b200.engine.mesh.ParamSync).
        self.param_arena = parameter_arena([net])
        self.params = list(net.parameters())
        self.optimizer = Adam(self.params, lr=cfg.lr, eps=cfg.eps)
        self.rng = np.random.default_rng(seed)
        dev = self.device
        slots = self.n_steps * self.n_envs
        f32 = dict(dtype=torch.float32, device=dev)
        self.fold = input_fold(net) if self.image else 1
        if self.image:
            self.obs = torch.zeros((slots,) + self.obs_shape, dtype=torch.uint8, device=dev)
            c, h, w = self.obs_shape
            f2 = self.fold * self.fold
            self.mb_rows = torch.empty((1, 1, self.rows * h * w // f2, c * f2), **f32)
        else:
            self.obs = torch.zeros((slots,) + self.obs_shape, **f32)
            self.mb_rows = torch.empty((self.rows,) + self.obs_shape, **f32)
        self.actions = torch.zeros(slots, dtype=torch.int32, device=dev)
        self.fields = {k: torch.zeros(slots, **f32)
                       for k in ("old_logp", "values", "returns", "advantages", "valid", "starts")}
        self.hidden = torch.zeros((self.total_sequences, self.hidden_size), **f32)
        self.valid_host = np.ones(slots, np.float32)
        steps, rows, n_seq = self.steps_per_update, self.rows, self.n_seq
        # Per minibatch: the slot of every row, then the sequence ids.
        self.idx_dev = torch.zeros((steps, rows + n_seq), dtype=torch.int32, device=dev)
        self.row_idx = self.idx_dev[:, :rows]
        self.seq_idx = self.idx_dev[:, rows:]
        self.idx_host = torch.zeros((steps, rows + n_seq), dtype=torch.int32, pin_memory=True)
        self._upload_done = None
        self.mb_actions = torch.empty(rows, dtype=torch.int32, device=dev)
        self.mb_fields = {k: torch.empty(rows, **f32) for k in self.fields}
        self.mb_h0 = torch.empty((n_seq, self.hidden_size), **f32)
        self.metric_buf = torch.zeros((steps, len(self.METRICS)), **f32)
        self._graph = None
        self.launches_per_replay = 0

    # -- rollout -----------------------------------------------------------

    def load_rollout(self, obs, actions, old_logp, values, returns, advantages, *, starts,
                     hidden, valid=None) -> None:
        """Upload one rollout. Per-slot arrays are [n_steps, n_envs] (obs
        [n_steps, n_envs, *obs_shape]); `starts` is the shifted episode-start
        flag of every slot (`shift_to_starts`); `hidden` is
        [n_chunks, n_envs, H], the unmasked state entering each sequence."""
        shape = (self.n_steps, self.n_envs)
        valid = np.ones(shape, np.float32) if valid is None else np.asarray(valid, np.float32)
        for name, arr in (("actions", actions), ("old_logp", old_logp), ("values", values),
                          ("returns", returns), ("advantages", advantages), ("starts", starts),
                          ("valid", valid)):
            if np.shape(arr) != shape:
                raise ValueError(f"load_rollout: {name} must be {shape}, got {np.shape(arr)}")
        adv = np.asarray(advantages, np.float32)
        if self.cfg.normalize_adv:
            adv = normalize_valid_advantages(adv, valid)
        keep = valid.astype(np.float32)
        host = {
            "old_logp": (np.asarray(old_logp, np.float32) * keep).astype(np.float32),
            "values": np.asarray(values, np.float32),
            "returns": (np.asarray(returns, np.float32) * keep).astype(np.float32),
            "advantages": (adv * keep).astype(np.float32),
            "valid": keep,
            "starts": np.asarray(starts, np.float32),
        }
        obs = np.ascontiguousarray(obs, np.uint8 if self.image else np.float32)
        self.obs.copy_(torch.from_numpy(obs.reshape(self.obs.shape)))
        self.actions.copy_(torch.from_numpy(np.asarray(actions, np.int32).reshape(-1)))
        for name, arr in host.items():
            self.fields[name].copy_(torch.from_numpy(np.ascontiguousarray(arr).reshape(-1)))
        hidden = np.asarray(hidden, np.float32)
        if hidden.shape != (self.n_chunks, self.n_envs, self.hidden_size):
            raise ValueError(f"load_rollout: hidden must be "
                             f"{(self.n_chunks, self.n_envs, self.hidden_size)}, got "
                             f"{hidden.shape}")
        self.hidden.copy_(torch.from_numpy(np.ascontiguousarray(hidden).reshape(
            self.total_sequences, self.hidden_size)))
        self.valid_host = keep.reshape(-1).copy()

    def draw_permutations(self) -> None:
        """One permutation of the sequence ids per epoch, cut into minibatches
        of n_seq whole sequences (ttrl/buffers/seqbatch.py:76-84)."""
        if self._upload_done is not None:
            self._upload_done.synchronize()  # the previous upload has read idx_host
        out = self.idx_host.numpy()
        k = 0
        for _ in range(self.cfg.epochs):
            perm = self.rng.permutation(self.total_sequences)
            for start in range(0, self.minibatches * self.n_seq, self.n_seq):
                ids = perm[start:start + self.n_seq]
                slots = sequence_rows(ids, self.n_envs, self.seq_len)
                if float(self.valid_host[slots].sum()) <= 0.0:
                    raise ValueError(
                        "PPO: a sequence minibatch holds no valid transitions, so every loss "
                        "term would reduce over nothing. Every slot in it is autoreset padding, "
                        "which means the rollout is almost entirely padding; raise n_steps or "
                        "check the env's autoreset contract.")
                out[k, :self.rows] = slots
                out[k, self.rows:] = ids
                k += 1
        self.idx_dev.copy_(self.idx_host, non_blocking=True)
        self._upload_done = torch.cuda.Event()
        self._upload_done.record()

    def minibatch_slots(self, k: int):
        """(slot index per row, sequence ids) of minibatch k, host copies."""
        host = self.idx_host.numpy()
        return host[k, :self.rows].copy(), host[k, self.rows:].copy()

    # -- one gradient step ---------------------------------------------------

    def _minibatch_step(self, k: int) -> None:
        cfg = self.cfg
        ctx = self.ctx
        idx = self.row_idx[k]
        if self.image:
            c = self.obs_shape[0]
            f2 = self.fold * self.fold
            ctx.u8_to_f32(self.obs, idx, self.mb_rows.reshape(-1, c * f2), 1.0, fold=self.fold)
        pairs = [] if self.image else [(self.obs, self.mb_rows)]
        pairs += [(self.actions, self.mb_actions)]
        pairs += [(src, self.mb_fields[name]) for name, src in self.fields.items()]
        ctx.gather_rows_multi(pairs, idx)
        ctx.gather_rows(self.hidden, self.seq_idx[k], self.mb_h0)
        self.optimizer.zero_grad()
        rows = Tensor(self.mb_rows)
        rows._exact = self.image  # raw 0..255 frame values
        rows._fold = self.fold
        f = self.mb_fields
        starts = Tensor(f["starts"].reshape(self.seq_len, self.n_seq, 1))
        logits, value = self.net(rows, {ACTOR: Tensor(self.mb_h0)}, starts, seq_len=self.seq_len)
        loss, parts, _ = ppo_objective(
            logits, value, self.mb_actions, f["old_logp"], f["advantages"], f["returns"],
            f["values"], clip_eps=cfg.clip_eps, value_clip_eps=cfg.value_clip_eps,
            value_coef=cfg.value_coef, entropy_coef=cfg.entropy_coef, valid=f["valid"])
        loss.backward()
        norm = clip_grad_norm_device(self.params, cfg.max_grad_norm, self.optimizer)
        self.optimizer.step()
        self._record_metrics(k, loss, parts, norm)
