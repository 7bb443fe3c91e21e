"""`ActingCarry`: recurrent state carried from one graph-replayed acting step
to the next (ttrl/engine/carry.py:45-165 is the interface).

An acting step both reads and produces the recurrent state, so a captured
graph cannot read and write one buffer: the second replay would read what the
first already overwrote. The carry keeps two sides. `prev` is the fixed
buffer the captured step reads (it never moves); the step's output is
whatever tensor it produced (fixed under a graph, fresh per call when run
eagerly), recorded by `bind`. `commit`, outside the graph, copies the output
into `prev` on the device with one copy kernel and reads nothing back.

The episode reset is not applied here: `start` is a bound `(lanes, 1)` input
the step masks `prev` with (`apply_done_mask`), the same op the training
unroll uses at the same place.
"""

from __future__ import annotations

import numpy as np
import torch

from ttrl_b200.device import context
from ttrl_b200.engine.autograd import Tensor, as_device
from ttrl_b200.engine.step.inputs import InputBinder
from ttrl_b200.engine.tensor import to_host

__all__ = ["ActingCarry"]


class ActingCarry:
    """The state buffer `prev` `(lanes, size)` and the episode-start flags
    `start` `(lanes, 1)` of one recurrent acting loop."""

    def __init__(self, size: int, device, *, lanes: int, name: str = "h"):
        if int(size) < 1 or int(lanes) < 1:
            raise ValueError(f"ActingCarry({name}): size ({size}) and lanes ({lanes}) must "
                             "both be at least 1")
        self.size, self.lanes, self.name = int(size), int(lanes), str(name)
        self.device = as_device(device)
        self.prev = Tensor(torch.zeros((self.lanes, self.size), device=self.device))
        self.start = Tensor(torch.zeros((self.lanes, 1), device=self.device))
        self._binder = InputBinder(self.device, {"start": self.start})
        self._next = None
        self._prev_ptr = self.prev.data.data_ptr()

    def load_start(self, flags) -> None:
        """The episode-start flags of the step about to run, one per lane:
        1.0 where the lane's previous step ended an episode."""
        arr = np.asarray(flags, np.float32).reshape(-1)
        if arr.size != self.lanes:
            raise ValueError(f"ActingCarry({self.name}).load_start: {arr.size} flags for "
                             f"{self.lanes} lanes")
        self._binder.load("start", arr.reshape(self.lanes, 1))

    @property
    def bound(self) -> bool:
        return self._next is not None

    def bind(self, h_next: Tensor) -> None:
        """Record the state the step produced; `commit` moves it into `prev`."""
        if tuple(int(d) for d in h_next.shape) != (self.lanes, self.size):
            raise ValueError(f"ActingCarry({self.name}).bind: state of shape "
                             f"{tuple(h_next.shape)}, the carry holds ({self.lanes}, "
                             f"{self.size})")
        self._next = h_next

    def commit(self) -> None:
        """prev <- the bound output, on the device, in place."""
        if self._next is None:
            raise RuntimeError(f"ActingCarry({self.name}).commit: no output is bound; the "
                               "step has to bind() the state it produced")
        if self.prev.data.data_ptr() != self._prev_ptr:
            raise RuntimeError(f"ActingCarry({self.name}): prev no longer lives at the "
                               "address the step was captured against; write it in place")
        src = self._next.data if isinstance(self._next, Tensor) else self._next
        context(self.device).copy_strided(self.prev.data, src.reshape(self.prev.data.shape))

    def numpy(self) -> np.ndarray:
        """`prev` on the host (a device read: between steps only)."""
        return to_host(self.prev.data)[: self.lanes, : self.size]

    def zero(self) -> None:
        """Clear the state (between rollouts)."""
        context(self.device).ew("fill", None, None, self.prev.data, 0.0)

    def close(self) -> None:
        self._binder.close()
