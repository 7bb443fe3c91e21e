"""`ParamSync`: exact parameter averaging across N replicas every
`sync_every` updates (ttrl/engine/mesh/sync.py:102-249).

The contract kept from the reference: only the online parameters move (each
replica's Adam moments stay its own), replicas must share one parameter
schema (names and shapes, checked at construction and again before every
average), targets given to `average` are refreshed from the averaged weights
only when the average succeeded, and a failure raises `ParamSyncError`
saying which parameters were written.

Two backends:

* **One process per GPU (the B200 design).** Built with the local module(s)
  and a `torch.distributed` process group. The parameters live in one flat
  fp32 arena (`parameter_arena`), so an average is ONE in-place all-reduce
  of that buffer -- NCCL's `ReduceOp.AVG` over NVLink / NVSwitch, the sum and
  the 1/N in one collective -- with no packing copies around it. A gloo group
  (host replicas, CPU tests) sums and then divides, since gloo has no AVG.
* **In-process replicas (the reference's shape).** With no group, the N
  modules are read to the host, each replica's parameters as one flat
  vector, and `reduce_fn` (default `host_all_reduce_sum`: the exact fp32 sum
  in replica order) combines them in ONE call; the result divided by N is
  written back in place. A reduction that raises or comes back short
  leaves every replica as it was.
"""

from __future__ import annotations

import datetime
from typing import Callable, Sequence

import numpy as np

from ttrl_b200.engine.nn import parameter_arena
from ttrl_b200.engine.tensor import restore_in_place

__all__ = ["ParamSync", "ParamSyncError", "host_all_reduce_sum", "param_schema",
           "replica_schema"]


class ParamSyncError(RuntimeError):
    """A parameter average could not complete (ttrl/engine/mesh/topology.py)."""


def host_all_reduce_sum(arrays: list) -> list:
    """The elementwise fp32 sum of `arrays`, added in replica order, handed
    back once per replica (ttrl/engine/mesh/sync.py:60-70). The caller
    divides by the replica count."""
    total = np.array(arrays[0], dtype=np.float32, copy=True)
    for a in arrays[1:]:
        np.add(total, np.asarray(a, dtype=np.float32), out=total)
    return [total] * len(arrays)


def param_schema(module) -> tuple:
    """((name, shape), ...) of a replica's parameters in order: what every
    replica must agree on before averaging by position makes sense."""
    named = list(module.named_parameters())
    count = sum(1 for _ in module.parameters())
    if count != len(named):
        raise ParamSyncError(
            f"{type(module).__name__} has {count} parameters but names {len(named)}; "
            "a schema cannot be formed from inconsistent listings.")
    return tuple((str(name), tuple(int(d) for d in p.shape)) for name, p in named)


def replica_schema(modules: Sequence) -> tuple:
    """The schema all `modules` share; raises ParamSyncError if any differs."""
    first = param_schema(modules[0])
    for index, module in enumerate(modules[1:], start=1):
        other = param_schema(module)
        if other != first:
            raise ParamSyncError(
                f"replica parameter schemas differ: replica 0 has {first} and replica "
                f"{index} has {other}. Averaging by position would combine unrelated "
                "tensors; build the same model, in the same order, on every replica.")
    return first


class ParamSync:
    """Average the online parameters of N replicas every `sync_every` calls
    of `maybe_average()`.

    `modules`: one module per replica in replica order (in-process), or this
    process's own module(s) when `group` is a process group. With a group,
    the parameters are placed in one flat arena at construction -- build
    the ParamSync before capturing any graph that reads them. `timeout_s`
    bounds the wait for a gloo all-reduce; an NCCL group is bounded by the
    timeout it was created with (its watchdog aborts a stuck collective and
    the next call raises), and either failure surfaces as ParamSyncError."""

    def __init__(self, modules, sync_every: int = 1,
                 reduce_fn: Callable = host_all_reduce_sum, group=None,
                 timeout_s: float | None = None):
        if sync_every < 1:
            raise ValueError(f"ParamSync: sync_every must be at least 1, got {sync_every}")
        self.modules = list(modules)
        if not self.modules:
            raise ValueError("ParamSync: no replica modules were given")
        self.n = len(self.modules)
        self.sync_every = int(sync_every)
        self.reduce_fn = reduce_fn
        self.group = group
        self.timeout_s = timeout_s
        self._since = 0
        self._schema = replica_schema(self.modules)
        self._world = 1
        self._nccl = False
        self._arena = None
        if group is not None:
            import torch.distributed as dist
            self._world = dist.get_world_size(group)
            self._nccl = str(dist.get_backend(group)).lower() == "nccl"
            self._arena = parameter_arena(self.modules)

    # -- schedule --------------------------------------------------------

    def maybe_average(self, targets: Sequence | None = None) -> bool:
        """Count one learner update; average on every `sync_every`-th call.
        Returns whether this call averaged."""
        self._since += 1
        if self._since < self.sync_every:
            return False
        self._since = 0
        self.average(targets=targets)
        return True

    def average(self, targets: Sequence | None = None) -> None:
        """Replace every replica's online parameters by their mean over
        replicas, in place; then, if `targets` are given (one per local
        module), hard-copy each from its averaged online module."""
        self._check_targets(targets)
        self._check_schema("average")
        if self.group is not None:
            self._collective_average()
        else:
            self._host_average()
        self._refresh_targets(targets)

    @property
    def arena(self):
        """The flat buffer the collective reduces (process-group mode)."""
        return self._arena

    # -- process group ----------------------------------------------------

    def _wait(self, work) -> None:
        if self.timeout_s is not None and not self._nccl:
            work.wait(datetime.timedelta(seconds=float(self.timeout_s)))
        else:
            work.wait()

    def _collective_average(self) -> None:
        import torch.distributed as dist
        flat = self._arena
        try:
            if self._nccl:
                self._wait(dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=self.group,
                                           async_op=True))
            else:
                self._wait(dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group,
                                           async_op=True))
                flat.div_(self._world)
        except Exception as exc:
            raise ParamSyncError(
                f"ParamSync.average(): the all-reduce over {self._world} ranks did not "
                f"complete ({exc}). This rank's parameters were not replaced by an "
                "average; other ranks may differ. Broadcast from one rank before "
                "training on.") from exc

    # -- in-process replicas ----------------------------------------------

    def _host_average(self) -> None:
        if self.n == 1:
            return
        per_replica = [list(m.parameters()) for m in self.modules]
        shapes = [tuple(p.shape) for p in per_replica[0]]
        sizes = [int(np.prod(s, dtype=np.int64)) for s in shapes]
        vectors = [np.concatenate([np.asarray(p.numpy(), np.float32).reshape(-1)
                                   for p in params]) for params in per_replica]
        count = len(shapes)
        try:
            summed = self.reduce_fn(vectors)
        except Exception as exc:
            raise ParamSyncError(
                f"ParamSync.average(): the reduction failed on parameter 0 of {count} "
                f"(all {count} parameters reduce together as one vector): {exc}. Nothing "
                "was written; every replica keeps its pre-call parameters.") from exc
        if len(summed) != self.n:
            raise ParamSyncError(
                f"ParamSync.average(): reduce_fn returned {len(summed)} results for "
                f"{self.n} replica vectors; writing them would leave replicas "
                "unaveraged, so nothing was written.")
        for total in summed:
            if np.shape(total) != vectors[0].shape:
                raise ParamSyncError(
                    f"ParamSync.average(): reduce_fn returned a vector of shape "
                    f"{np.shape(total)} for replica vectors of {vectors[0].shape}; nothing "
                    "was written.")
        scale = np.float32(self.n)
        for params, total in zip(per_replica, summed):
            mean = np.asarray(total, np.float32) / scale
            offset = 0
            for p, shape, size in zip(params, shapes, sizes):
                restore_in_place(p.data, mean[offset:offset + size].reshape(shape))
                offset += size

    # -- broadcast / targets ------------------------------------------------

    def broadcast(self, src: int = 0, targets: Sequence | None = None) -> None:
        """Give every replica replica `src`'s online parameters (the start of
        a run: N replicas of one model, not the mean of N initialisations)."""
        self._check_targets(targets)
        self._check_schema("broadcast")
        if self.group is not None:
            import torch.distributed as dist
            try:
                self._wait(dist.broadcast(self._arena, src=src, group=self.group,
                                          async_op=True))
            except Exception as exc:
                raise ParamSyncError(f"ParamSync.broadcast(): the broadcast from rank {src} "
                                     f"did not complete ({exc}).") from exc
        else:
            if not 0 <= src < self.n:
                raise ValueError(f"ParamSync.broadcast: src {src} is not one of the "
                                 f"{self.n} replicas")
            source = [np.asarray(p.numpy(), np.float32)
                      for p in self.modules[src].parameters()]
            for i, module in enumerate(self.modules):
                if i != src:
                    for p, value in zip(module.parameters(), source):
                        restore_in_place(p.data, value)
        self._refresh_targets(targets)

    def _check_targets(self, targets) -> None:
        if targets is not None and len(targets) != self.n:
            raise ValueError(f"ParamSync: {len(targets)} target modules for {self.n} "
                             "replicas")

    def _check_schema(self, what: str) -> None:
        now = replica_schema(self.modules)
        if now != self._schema:
            raise ParamSyncError(
                f"the parameter schema changed since ParamSync was built (was "
                f"{self._schema}, now {now}); will not {what}.")

    def _refresh_targets(self, targets) -> None:
        if targets is not None:
            for online, target in zip(self.modules, targets):
                target.copy_from(online)
