"""`ParamSync`: periodic exact parameter averaging across N replicas
(ttrl/engine/mesh/sync.py:102-249).

Two backends behind the reference's interface:

* **One process per GPU (the B200 design).** Construct with the local
  module(s) and a `torch.distributed` process group (NCCL over NVLink /
  NVSwitch). `average()` packs the online parameters into one flat fp32
  buffer with copy kernels, runs ONE all-reduce with `ReduceOp.AVG` (NCCL's
  average: the sum and the 1/N scale in one collective), and unpacks in
  place. Adam moments stay local, as in the reference.
* **In-process replicas (the reference's shape).** With no group, the N
  modules are averaged by `reduce_fn` (default `host_all_reduce_sum`, the
  reference's exact fp32 host sum in replica order) then divided by N and
  written back in place.

Both keep the reference's contract: online parameters only, validated
schemas (names and shapes), targets refreshed from the averaged weights
when given, and a partial-failure message that says what was averaged.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Sequence

import numpy as np
import torch

from ttrl_b200.device import context
from ttrl_b200.engine.tensor import restore_in_place

__all__ = ["ParamSync", "ParamSyncError", "host_all_reduce_sum", "param_schema",
           "replica_schema"]


class ParamSyncError(RuntimeError):
    """A parameter average could not complete (ttrl/engine/mesh/topology.py)."""


def host_all_reduce_sum(arrays: list) -> list:
    """Exact fp32 elementwise sum in replica order, identical on every entry
    (ttrl/engine/mesh/sync.py:60-70)."""
    summed = np.asarray(arrays[0], dtype=np.float32).copy()
    for a in arrays[1:]:
        summed = summed + np.asarray(a, dtype=np.float32)
    return [summed for _ in arrays]


def param_schema(module) -> tuple:
    params = list(module.parameters())
    names = [n for n, _ in module.named_parameters()]
    if len(names) != len(params):
        raise ParamSyncError(
            f"{type(module).__name__}: {len(names)} parameter names for "
            f"{len(params)} parameters; named_parameters() and parameters() disagree."
        )
    return tuple((str(n), tuple(p.shape)) for n, p in zip(names, params))


def replica_schema(modules: Sequence) -> tuple:
    schemas = [param_schema(m) for m in modules]
    if len(set(schemas)) != 1:
        raise ParamSyncError(
            "replica parameter schemas differ by name or shape, so a positional "
            f"average would mix unrelated tensors: {schemas}. Every replica must build "
            "the identical model in the identical order."
        )
    return schemas[0]


@dataclass
class ParamSync:
    modules: list
    sync_every: int = 1
    reduce_fn: Callable = field(default=host_all_reduce_sum, repr=False)
    group: object = field(default=None, repr=False)
    _updates_since_sync: int = field(default=0, init=False, repr=False)

    def __post_init__(self) -> None:
        if self.sync_every < 1:
            raise ValueError(f"sync_every must be >= 1, got {self.sync_every}")
        self.n = len(self.modules)
        if self.n < 1:
            raise ValueError("ParamSync needs at least one replica, got none")
        self._schema = replica_schema(self.modules)
        self._nparams = len(self._schema)
        self._flat = None
        self._world = 1
        self._nccl = False
        if self.group is not None:
            import torch.distributed as dist
            self._world = dist.get_world_size(self.group)
            self._nccl = str(dist.get_backend(self.group)).lower() == "nccl"

    # -- schedule --------------------------------------------------------

    def maybe_average(self, targets: Sequence | None = None) -> bool:
        self._updates_since_sync += 1
        if self._updates_since_sync >= self.sync_every:
            self._updates_since_sync = 0
            self.average(targets=targets)
            return True
        return False

    def average(self, targets: Sequence | None = None) -> None:
        if targets is not None and len(targets) != self.n:
            raise ValueError(f"expected {self.n} target modules, got {len(targets)}")
        self._require_schema("average")
        if self.group is not None:
            self._average_distributed()
        else:
            self._average_in_process()
        self._refresh_targets(targets)

    # -- NCCL path -------------------------------------------------------

    def _flat_buffer(self, params):
        total = sum(p.data.numel() for p in params)
        if self._flat is None or self._flat.numel() != total:
            self._flat = torch.empty(total, dtype=torch.float32, device=params[0].data.device)
        return self._flat

    def _average_distributed(self) -> None:
        import torch.distributed as dist
        for module in self.modules:
            params = list(module.parameters())
            flat = self._flat_buffer(params)
            # On a GPU the packing runs as this library's copy kernels; host
            # replicas (gloo process groups) pack with plain tensor copies.
            if flat.is_cuda:
                copy = context(flat.device).copy_strided
            else:
                def copy(dst, src):
                    dst.copy_(src)
            off = 0
            for p in params:
                n = p.data.numel()
                copy(flat[off:off + n], p.data.reshape(-1))
                off += n
            try:
                if self._nccl:
                    # NCCL's average: the sum and the 1/N in one collective.
                    dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=self.group)
                else:
                    # gloo has no AVG: sum, then the 1/N (host replicas only).
                    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group)
                    flat.div_(self._world)
            except Exception as e:
                raise ParamSyncError(
                    f"ParamSync.average(): the all-reduce failed: {e}. No parameter was "
                    "written back, so this replica holds its own pre-call values; the "
                    "other ranks may not. Re-sync (broadcast) before resuming."
                ) from e
            off = 0
            for p in params:
                n = p.data.numel()
                copy(p.data.reshape(-1), flat[off:off + n])
                off += n

    # -- in-process path (reference semantics) ---------------------------

    def _average_in_process(self) -> None:
        per_replica = [list(m.parameters()) for m in self.modules]
        for j in range(self._nparams):
            shards = [per_replica[i][j] for i in range(self.n)]
            try:
                self._all_reduce_param(shards)
            except Exception as e:
                raise ParamSyncError(
                    f"ParamSync.average(): the reduction failed on parameter "
                    f"{j}/{self._nparams}: {e}. Parameters 0..{j - 1} may already be "
                    f"fully averaged across replicas; parameter {j} may be PARTIALLY "
                    f"propagated; parameters {j + 1}..{self._nparams - 1} are untouched. "
                    "Re-sync (for example broadcast() from a known-good replica) before "
                    "resuming or checkpointing."
                ) from e

    def _all_reduce_param(self, shards) -> None:
        if self.n == 1:
            return
        arrays = [np.asarray(s.numpy(), dtype=np.float32) for s in shards]
        shape = arrays[0].shape
        for a in arrays[1:]:
            if a.shape != shape:
                raise ParamSyncError(
                    f"parameter shape mismatch across replicas: {shape} vs {a.shape}"
                )
        summed = self.reduce_fn(arrays)
        if len(summed) != len(shards):
            raise ParamSyncError(
                f"reduce_fn returned {len(summed)} results for {len(shards)} replica "
                "shards; a short result would silently leave some replicas unaveraged."
            )
        n = np.float32(self.n)
        for shard, total in zip(shards, summed):
            restore_in_place(shard.data, np.asarray(total, dtype=np.float32) / n)

    # -- broadcast / targets --------------------------------------------

    def broadcast(self, src: int = 0, targets: Sequence | None = None) -> None:
        if targets is not None and len(targets) != self.n:
            raise ValueError(f"expected {self.n} target modules, got {len(targets)}")
        self._require_schema("broadcast")
        if self.group is not None:
            import torch.distributed as dist
            for p in self.modules[0].parameters():
                dist.broadcast(p.data, src=src, group=self.group)
        else:
            if not 0 <= src < self.n:
                raise ValueError(f"src replica {src} out of range for {self.n} replicas")
            per_replica = [list(m.parameters()) for m in self.modules]
            for j in range(self._nparams):
                source = np.asarray(per_replica[src][j].numpy(), dtype=np.float32)
                for i in range(self.n):
                    if i != src:
                        restore_in_place(per_replica[i][j].data, source)
        self._refresh_targets(targets)

    def _require_schema(self, what: str) -> None:
        current = replica_schema(self.modules)
        if current != self._schema:
            raise ParamSyncError(
                "the replica parameter schema changed since ParamSync was built: "
                f"{self._schema} -> {current}. Refusing to {what}."
            )

    def _refresh_targets(self, targets) -> None:
        if targets is None:
            return
        for online, target in zip(self.modules, targets):
            target.copy_from(online)
