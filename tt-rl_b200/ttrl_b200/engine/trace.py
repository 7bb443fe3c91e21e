"""CUDA-graph capture and replay with the reference's trace interface
(ttrl/engine/trace.py): `capture(device, record) -> (CapturedTrace, result)`.

Capture is a callback, as in the reference, so no caller can leave a stream
in capture mode: every exit path out of `record()` ends the capture inside
this module. A host read inside the recorded region (an `.item()`, a
`.numpy()`) is refused by CUDA during capture and surfaces as
`TraceCaptureError`, as the reference's ttnn error does.
"""

from __future__ import annotations

from typing import Callable, TypeVar

import torch

from ttrl_b200.device import context
from ttrl_b200.engine.autograd import as_device
from ttrl_b200.engine.config import DEFAULT, EngineConfig

__all__ = ["CapturedTrace", "TraceCaptureError", "capture", "HOST_READ_DURING_CAPTURE"]

HOST_READ_DURING_CAPTURE = "operation not permitted when stream is capturing"

R = TypeVar("R")


class TraceCaptureError(RuntimeError):
    """Graph capture failed. There is no eager fallback."""


class CapturedTrace:
    """One captured CUDA graph, replayable until closed."""

    __slots__ = ("device", "_graph")

    def __init__(self, device, graph):
        self.device = device
        self._graph = graph

    @property
    def live(self) -> bool:
        return self._graph is not None

    def replay(self, *, cfg: EngineConfig = DEFAULT, blocking: bool | None = None) -> None:
        """Launch the graph on the device's current stream (non-blocking by
        default: a later host read on the same stream is the barrier)."""
        if self._graph is None:
            raise RuntimeError("replay() on a closed CapturedTrace")
        self._graph.replay()
        wait = cfg.trace_blocking if blocking is None else blocking
        if wait:
            torch.cuda.current_stream(self.device).synchronize()

    def close(self) -> None:
        if self._graph is None:
            return
        graph, self._graph = self._graph, None
        graph.reset()

    def __enter__(self) -> "CapturedTrace":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


_CAPTURE_STREAMS: dict = {}


def _capture_stream(dev) -> torch.cuda.Stream:
    """A capture stream at the device's highest priority, above the launch
    lanes' default: where the graph's branches compete for SMs the block
    scheduler serves the capture stream's chain first. That suits an update
    whose side lanes carry only weight gradients, off the critical path (PPO:
    +3%); where the side lanes carry work the critical path waits for (DQN's
    two no-grad forwards), it starves them (DQN -3%), so it is asked for per
    capture."""
    s = _CAPTURE_STREAMS.get(dev)
    if s is None:
        _, highest = torch.cuda.Stream.priority_range()
        s = _CAPTURE_STREAMS[dev] = torch.cuda.Stream(dev, priority=highest)
    return s


def capture(device, record: Callable[[], R], *, pool=None,
            critical_main: bool = False) -> tuple[CapturedTrace, R]:
    """Record `record()`'s device work into a CUDA graph. With
    `critical_main` the capture stream, and so the graph's main chain, runs
    at the highest stream priority (see `_capture_stream`).

    `record` must launch device work only. Run the same work once eagerly
    beforehand (kernel loading, workspace sizing). Nothing has executed when
    this returns; replay once before reading outputs.
    """
    dev = as_device(device)
    graph = torch.cuda.CUDAGraph()
    result = None
    try:
        with torch.cuda.device(dev):
            # Side lanes still pending from eager work are joined here, before
            # the capture: a join inside it would wait on a lane the capture
            # never forked (uncaptured work).
            context(dev).join()
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(graph, pool=pool,
                                  stream=_capture_stream(dev) if critical_main else None,
                                  capture_error_mode="thread_local"):
                result = record()
                # Every side lane rejoins the capture stream before it ends.
                context(dev).join()
    except BaseException as e:
        try:
            graph.reset()
        except Exception:
            pass
        if isinstance(e, (KeyboardInterrupt, SystemExit)):
            raise
        if HOST_READ_DURING_CAPTURE in str(e) or "capturing" in str(e):
            raise TraceCaptureError(
                "graph capture failed because the captured work reads a tensor back "
                "to host (.numpy(), .item(), .cpu()) or allocates with the CUDA "
                "runtime, which CUDA does not allow during capture. Move every host "
                "read after the replay, or run this step eagerly. Error: " + str(e)
            ) from e
        raise TraceCaptureError(f"graph capture failed: {e}") from e
    return CapturedTrace(dev, graph), result
