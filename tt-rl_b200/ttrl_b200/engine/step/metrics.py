"""`MetricPack` and `read_metrics` (ttrl/engine/step/metrics.py): a step's
scalar metrics packed into one device buffer, read back in one transfer."""

from __future__ import annotations

import contextlib

import torch

from ttrl_b200.device import context
from ttrl_b200.engine.autograd import Tensor

__all__ = ["MetricPack", "read_metrics"]


def _numel(t) -> int:
    n = 1
    for d in t.shape:
        n *= int(d)
    return n


class MetricPack:
    """Packs the scalar metrics of one step into one device buffer with one
    copy launch, so reading them back is a single device-to-host transfer."""

    def __init__(self, metrics: dict):
        self.scalar_keys = []
        self.vector_keys = []
        self.passthrough = {}
        self.sources = {}
        for k, v in metrics.items():
            if isinstance(v, Tensor):
                if _numel(v) == 1:
                    self.scalar_keys.append(k)
                else:
                    self.vector_keys.append(k)
                self.sources[k] = v
            else:
                self.passthrough[k] = v
        self.buffer = None
        if self.scalar_keys:
            dev = self.sources[self.scalar_keys[0]].data.device
            ctx = context(dev)
            # On side lane 2 (when lanes are on), beside the optimizer step
            # that follows on the current stream; the caller joins.
            lane = ctx.side(2) if ctx.concurrent else contextlib.nullcontext()
            with lane:
                self.buffer = torch.empty(len(self.scalar_keys), dtype=torch.float32,
                                          device=dev)
                pairs = []
                for i, k in enumerate(self.scalar_keys):
                    src = self.sources[k].data.reshape(1)
                    if src.dtype != torch.float32:
                        src = src.float()
                    pairs.append((self.buffer[i:i + 1], src.contiguous()))
                ctx.blend(pairs)  # every scalar in one copy launch

    def read(self) -> dict:
        out = dict(self.passthrough)
        if self.buffer is not None:
            context(self.buffer.device).join()
            host = self.buffer.detach().to("cpu").numpy()
            for i, k in enumerate(self.scalar_keys):
                out[k] = host[i:i + 1].reshape(self.sources[k].shape)
        for k in self.vector_keys:
            out[k] = self.sources[k].numpy()
        return out

    def fetch(self):
        """Start copying every metric to pinned host memory on the current
        stream; `result(handle)` waits for those copies only."""
        copies = {}
        dev = None
        if self.buffer is not None:
            dev = self.buffer.device
            context(dev).join()
            copies[None] = torch.empty(self.buffer.shape, dtype=self.buffer.dtype,
                                       pin_memory=True)
            copies[None].copy_(self.buffer, non_blocking=True)
        for k in self.vector_keys:
            src = self.sources[k].data
            dev = src.device
            copies[k] = torch.empty(src.shape, dtype=src.dtype, pin_memory=True)
            copies[k].copy_(src, non_blocking=True)
        done = None
        if dev is not None:
            done = torch.cuda.Event()
            done.record(torch.cuda.current_stream(dev))
        return copies, done

    def result(self, handle) -> dict:
        copies, done = handle
        if done is not None:
            done.synchronize()
        out = dict(self.passthrough)
        if None in copies:
            host = copies[None].numpy()
            for i, k in enumerate(self.scalar_keys):
                out[k] = host[i:i + 1].reshape(self.sources[k].shape)
        for k in self.vector_keys:
            out[k] = copies[k].numpy().reshape(self.sources[k].shape)
        return out


def read_metrics(metrics: dict | None) -> dict:
    """Download every tensor-valued metric; scalars in one transfer."""
    if not metrics:
        return {}
    return MetricPack(metrics).read()
