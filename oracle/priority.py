"""Prioritized replay restated in numpy. TEST INFRASTRUCTURE ONLY (see
oracle/__init__.py).

Follows ttrl/buffers/sampling.py:111-240: a float64 table of
(p + epsilon)^alpha per ring column, fresh columns at the largest priority
seen, write-backs where a column drawn twice takes its last value, and the
draw: a multinomial lane quota from the lanes' priority sums, a searchsorted
draw inside each lane's run (oldest first), and importance-sampling weights
(N * P)^-beta normalised by the batch maximum.
"""

from __future__ import annotations

import numpy as np

__all__ = ["PriorityTable"]


class PriorityTable:
    def __init__(self, lanes: int, columns: int, alpha: float, epsilon: float):
        self.weight = np.zeros((lanes, columns), np.float64)
        self.max_priority = 1.0
        self.alpha, self.epsilon = alpha, epsilon

    def _scaled(self, p):
        return (p + self.epsilon) ** self.alpha

    def on_write(self, lane, col):
        self.weight[lane, col] = self._scaled(np.float64(self.max_priority))

    def update(self, lanes, cols, td):
        p = np.abs(np.asarray(td, np.float64).reshape(-1))
        self.weight[lanes, cols] = self._scaled(p)
        self.max_priority = max(self.max_priority, float(p.max()))

    def draw(self, rng, counts, start, capacity, batch_size, beta):
        runs = [self.weight[l, (int(start[l]) + np.arange(int(counts[l]))) % capacity]
                for l in range(len(counts))]
        sums = np.array([w.sum() for w in runs], np.float64)
        quota = rng.multinomial(batch_size, sums / sums.sum())
        lanes, offsets, probs = [], [], []
        for lane, k in enumerate(int(v) for v in quota):
            if k == 0:
                continue
            cdf = np.cumsum(runs[lane])
            picked = np.minimum(np.searchsorted(cdf, rng.random(k) * cdf[-1], side="right"),
                                runs[lane].shape[0] - 1)
            lanes.append(np.full(k, lane, np.int64))
            offsets.append(picked)
            probs.append(runs[lane][picked] / sums.sum())
        w = (int(np.sum(counts)) * np.concatenate(probs)) ** (-beta)
        return np.concatenate(lanes), np.concatenate(offsets), (w / w.max()).astype(np.float32)
