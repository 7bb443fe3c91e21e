"""Prioritized replay with its priority table on the device
(ttrl/buffers/sampling.py:59-240, ttrl/algos/offpolicy.py:123-145).

`DevicePrioritySampler` keeps the reference's `PrioritySampler` interface
(`on_write`, `draw`, `update`, `state`, `load`) and arithmetic: one
(p + epsilon)^alpha per ring column in float64, fresh columns at the largest
priority seen, a lane quota drawn multinomially from the lanes' priority sums,
a searchsorted draw inside each lane's run, and importance-sampling weights
(N * P)^-beta normalised by the batch maximum. The table, its running maximum
and the per-lane cumulative sums live in HBM; `update` takes the |TD| errors
as the device tensor the DQN loss kernel wrote, so the write-back needs no
host read. The host keeps the generator: the multinomial quota and the
uniforms are drawn there in the reference's order (reading back only one
float64 sum per lane), and the device performs the searchsorted draw on them.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import NamedTuple

import numpy as np
import torch

from ttrl_b200._lib import check, lib
from ttrl_b200.device import context

__all__ = ["PriorityConfig", "beta_at", "Draw", "Window", "DevicePrioritySampler"]


@dataclass(frozen=True)
class PriorityConfig:
    """ttrl/buffers/sampling.py:59-102."""
    alpha: float = 0.6
    beta_start: float = 0.4
    beta_end: float = 1.0
    beta_anneal_updates: int = 1_000_000
    epsilon: float = 1e-6

    def __post_init__(self) -> None:
        if not 0.0 <= self.alpha <= 1.0:
            raise ValueError(f"PriorityConfig: alpha must be in [0, 1], got {self.alpha}")
        for name in ("beta_start", "beta_end"):
            if not 0.0 <= getattr(self, name) <= 1.0:
                raise ValueError(f"PriorityConfig: {name} must be in [0, 1], got "
                                 f"{getattr(self, name)}")
        if self.beta_anneal_updates < 1:
            raise ValueError("PriorityConfig: beta_anneal_updates must be >= 1 gradient steps")
        if self.epsilon <= 0.0:
            raise ValueError(f"PriorityConfig: epsilon must be > 0, got {self.epsilon}")


def beta_at(cfg: PriorityConfig, update: int) -> float:
    """The annealed beta at a gradient-step count (sampling.py:105-108)."""
    frac = min(1.0, max(0, int(update)) / cfg.beta_anneal_updates)
    return cfg.beta_start + frac * (cfg.beta_end - cfg.beta_start)


class Draw(NamedTuple):
    """lanes[i], offsets[i]: lane and run position of sample i; weights: its
    importance-sampling correction (ttrl/buffers/window.py:29-41)."""
    lanes: np.ndarray
    offsets: np.ndarray
    weights: np.ndarray


@dataclass(frozen=True)
class Window:
    """The sampleable runs, one per lane, oldest first (window.py:44-84)."""
    counts: np.ndarray
    start: np.ndarray
    capacity: int

    @property
    def n_lanes(self) -> int:
        return int(self.counts.shape[0])

    @property
    def total(self) -> int:
        return int(self.counts.sum())

    def columns(self, lane: int) -> np.ndarray:
        n = int(self.counts[lane])
        return (int(self.start[lane]) + np.arange(n, dtype=np.int64)) % self.capacity


class DevicePrioritySampler:
    def __init__(self, cfg: PriorityConfig, *, lanes: int, columns: int, device=None):
        self.cfg = cfg
        self.ctx = context(device)
        dev = self.ctx.device
        self.lanes, self.columns = int(lanes), int(columns)
        self.table = torch.zeros((self.lanes, self.columns), dtype=torch.float64, device=dev)
        self.cdf = torch.zeros_like(self.table)
        self.totals = torch.zeros(self.lanes, dtype=torch.float64, device=dev)
        self.max_priority = torch.ones(1, dtype=torch.float64, device=dev)

    def _update(self, lanes, cols, td, from_max: bool) -> None:
        n = int(lanes.numel())
        check(lib().ttrl_per_update(self.table.data_ptr(), self.columns, lanes.data_ptr(),
                                    cols.data_ptr(), None if td is None else td.data_ptr(), n,
                                    float(self.cfg.alpha), float(self.cfg.epsilon),
                                    self.max_priority.data_ptr(), int(from_max),
                                    self.ctx.status_ptr(), self.ctx.stream), "ttrl_per_update")

    def _dev_idx(self, a):
        if isinstance(a, torch.Tensor):
            return a.to(self.ctx.device, torch.int32).reshape(-1)
        return torch.from_numpy(np.asarray(a, np.int32).reshape(-1)).to(self.ctx.device)

    def on_write(self, lanes, cols) -> None:
        """Columns just written take the largest priority seen so far."""
        self._update(self._dev_idx(lanes), self._dev_idx(cols), None, True)

    def update(self, lanes, cols, td_abs) -> None:
        """Fresh priorities for the columns a batch was drawn from; `td_abs`
        may be the loss kernel's device output (no host read)."""
        td = td_abs if isinstance(td_abs, torch.Tensor) else torch.from_numpy(
            np.asarray(td_abs, np.float32))
        td = td.to(self.ctx.device, torch.float32).reshape(-1).contiguous()
        self._update(self._dev_idx(lanes), self._dev_idx(cols), td, False)

    def draw(self, rng: np.random.Generator, window: Window, *, batch_size: int,
             beta: float | None) -> Draw:
        if beta is None:
            raise ValueError("ReplayBuffer.sample: this buffer samples by priority, so the "
                             "batch's importance-sampling weights need a beta.")
        dev = self.ctx.device
        counts = torch.from_numpy(np.asarray(window.counts, np.int32)).to(dev)
        start = torch.from_numpy(np.asarray(window.start, np.int32)).to(dev)
        check(lib().ttrl_per_cdf(self.table.data_ptr(), self.lanes, self.columns,
                                 counts.data_ptr(), start.data_ptr(), self.cdf.data_ptr(),
                                 self.totals.data_ptr(), self.ctx.stream), "ttrl_per_cdf")
        sums = self.totals.cpu().numpy()
        if sums.sum() <= 0.0:
            raise RuntimeError("replay: every priority in the sampleable runs is zero")
        quota = rng.multinomial(batch_size, sums / sums.sum())
        lane_of, uniforms = [], []
        for lane, k in enumerate(int(v) for v in quota):
            if k == 0:
                continue
            lane_of.append(np.full(k, lane, np.int32))
            uniforms.append(rng.random(k))
        lane_of = np.concatenate(lane_of)
        uniforms = np.concatenate(uniforms)
        n = len(lane_of)
        pos = torch.empty(n, dtype=torch.int32, device=dev)
        cols = torch.empty(n, dtype=torch.int32, device=dev)
        picked = torch.empty(n, dtype=torch.float64, device=dev)
        lane_d = torch.from_numpy(lane_of).to(dev)
        u_d = torch.from_numpy(uniforms).to(dev)
        check(lib().ttrl_per_draw(self.cdf.data_ptr(), self.table.data_ptr(), self.columns,
                                  counts.data_ptr(), start.data_ptr(), lane_d.data_ptr(),
                                  u_d.data_ptr(), n, pos.data_ptr(), cols.data_ptr(),
                                  picked.data_ptr(), self.ctx.stream), "ttrl_per_draw")
        probs = picked.cpu().numpy() / sums.sum()
        weights = (window.total * probs) ** (-float(beta))
        return Draw(lane_of.astype(np.int64), pos.cpu().numpy().astype(np.int64),
                    (weights / weights.max()).astype(np.float32))

    def state(self) -> dict:
        return {"weight": self.table.cpu().numpy().copy(),
                "max_priority": float(self.max_priority.cpu().item())}

    def load(self, state: dict) -> None:
        stored = np.asarray(state["weight"], np.float64)
        if stored.shape != tuple(self.table.shape):
            raise ValueError(f"replay priorities in the checkpoint are shaped {stored.shape} "
                             f"and this buffer's table is {tuple(self.table.shape)}")
        self.table.copy_(torch.from_numpy(stored))
        self.max_priority.fill_(float(state["max_priority"]))
