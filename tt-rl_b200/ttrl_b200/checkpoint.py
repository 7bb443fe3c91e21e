"""Reading and writing the reference's checkpoint file
(ttrl/train/checkpoint/file.py:112-218, tree.py:64-160, atomic.py:21-37).

A checkpoint is one `.npz`: every array once, as a plain member, plus a
`__meta__` member holding UTF-8 JSON as uint8. The JSON is a tagged tree:
`{"__array__": name}` and `{"__bytes__": name}` stand for members,
`{"__list__": [...]}` for a list or tuple, `{"__dataclass__": "module:Class",
"fields": {...}}` for a configuration object, and everything else is plain
JSON. The agent's state sits under `agent_state`, its arrays named
`state.<dotted path>`. No pickle anywhere.

This module keeps that layout byte for byte, so a B200 learner resumes from a
file the reference wrote and writes one the reference (and its `ttrl.deploy`
exporter) reads: `Checkpoint.read` -> `load_learner` fills the B200 nets and
optimizers in place; `Checkpoint.update` puts their state back under the same
names, each array in the shape the file held it in (a convolution's Adam
moments in the reference's prepared matrix, ttrl_b200.engine.packing), and
`write` replaces the file atomically. A configuration object is carried as a
`Tagged` node, unchanged: the learner never needs to construct one.

Only numpy and the standard library are imported at module scope, so the
file layer runs on a host with no GPU.
"""

from __future__ import annotations

import io
import json
import os
import uuid
from dataclasses import dataclass
from typing import Any

import numpy as np

from ttrl_b200.engine.packing import solve_cp

__all__ = ["FORMAT", "META_KEY", "Tagged", "Checkpoint", "join", "split", "learner_state",
           "load_learner", "atomic_write_bytes"]

#: The reference's format marker (file.py:103); a file with another is refused.
FORMAT = "ttrl-checkpoint-9c42ad"
META_KEY = "__meta__"
LEVELS = ("L0", "L1")
AGENT_PREFIX = "state"


@dataclass(frozen=True)
class Tagged:
    """A `{"__dataclass__": path, "fields": {...}}` node, fields joined."""
    path: str
    fields: dict


def join(node: Any, arrays: dict, *, file: str = "<checkpoint>") -> Any:
    """The tree a `__meta__` node stands for, members put in place."""
    if isinstance(node, dict):
        if "__array__" in node or "__bytes__" in node:
            raw = "__bytes__" in node
            key = node["__bytes__"] if raw else node["__array__"]
            if key not in arrays:
                raise ValueError(f"checkpoint {file!r} references array {key!r}, which it does "
                                 "not contain")
            return arrays[key].tobytes() if raw else arrays[key]
        if "__list__" in node:
            return [join(v, arrays, file=file) for v in node["__list__"]]
        if "__dataclass__" in node:
            return Tagged(node["__dataclass__"],
                          {k: join(v, arrays, file=file) for k, v in node["fields"].items()})
        return {k: join(v, arrays, file=file) for k, v in node.items()}
    return node


def split(state: Any, prefix: str, arrays: dict) -> Any:
    """Inverse of `join`: arrays into `arrays` under dotted names, the rest
    as tagged JSON."""
    if isinstance(state, np.ndarray):
        arrays[prefix] = state
        return {"__array__": prefix}
    if isinstance(state, (bytes, bytearray)):
        arrays[prefix] = np.frombuffer(bytes(state), dtype=np.uint8)
        return {"__bytes__": prefix}
    if isinstance(state, np.generic):
        return state.item()
    if isinstance(state, Tagged):
        return {"__dataclass__": state.path,
                "fields": {k: split(v, f"{prefix}.{k}", arrays)
                           for k, v in state.fields.items()}}
    if isinstance(state, dict):
        bad = [k for k in state if not isinstance(k, str)]
        if bad:
            raise TypeError(f"checkpoint state at {prefix!r} has non-string keys {bad}")
        return {k: split(v, f"{prefix}.{k}", arrays) for k, v in state.items()}
    if isinstance(state, (list, tuple)):
        return {"__list__": [split(v, f"{prefix}.{i}", arrays) for i, v in enumerate(state)]}
    if isinstance(state, (str, int, float, bool)) or state is None:
        return state
    raise TypeError(f"checkpoint state at {prefix!r} holds {type(state).__name__}, which has "
                    "no JSON or array form")


def _json_default(obj):
    if isinstance(obj, np.ndarray):
        return obj.tolist()
    if isinstance(obj, np.generic):
        return obj.item()
    raise TypeError(f"object of type {type(obj)!r} is not JSON serializable")


def atomic_write_bytes(path: str, data: bytes) -> None:
    """Write beside `path`, fsync, then rename over it: a reader sees the old
    file or the whole new one."""
    directory = os.path.dirname(os.path.abspath(path)) or "."
    os.makedirs(directory, exist_ok=True)
    tmp = os.path.join(directory, f".{os.path.basename(path)}.tmp-{uuid.uuid4().hex}")
    fd = os.open(tmp, os.O_WRONLY | os.O_CREAT | os.O_EXCL, 0o644)
    try:
        with os.fdopen(fd, "wb") as fh:
            fh.write(data)
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, path)
    except BaseException:
        try:
            os.remove(tmp)
        except OSError:
            pass
        raise


class Checkpoint:
    """A checkpoint file's `__meta__` tree and its arrays."""

    def __init__(self, meta: dict, arrays: dict, source: str | None = None):
        self.meta = meta
        self.arrays = arrays
        self.source = source

    @classmethod
    def read(cls, path: str) -> "Checkpoint":
        with np.load(path, allow_pickle=False) as npz:
            if META_KEY not in npz.files:
                raise ValueError(f"{path!r} has no {META_KEY!r} member, so it is not a ttrl "
                                 "checkpoint")
            meta = json.loads(npz[META_KEY].tobytes().decode("utf-8"))
            arrays = {k: npz[k] for k in npz.files if k != META_KEY}
        if meta.get("format") != FORMAT:
            raise ValueError(f"{path!r} has checkpoint format {meta.get('format')!r}; this "
                             f"reader takes {FORMAT!r} only (the format has no migrations)")
        if meta.get("level") not in LEVELS:
            raise ValueError(f"{path!r} has level {meta.get('level')!r}, not one of {LEVELS}")
        return cls(meta, arrays, path)

    @classmethod
    def new(cls, *, agent_state: dict, obs_spec: dict, action_spec: dict, level: str = "L0",
            frame: int = 0, config=None, env_policy_state=None) -> "Checkpoint":
        """A fresh file's tree. `obs_spec` / `action_spec` are the JSON forms
        the reference writes (`dataclasses.asdict` of its ObsGroup and
        ActionSpec); `config` is a `Tagged` run configuration (L1 only)."""
        if level not in LEVELS:
            raise ValueError(f"level must be one of {LEVELS}, got {level!r}")
        if level == "L1" and config is None:
            raise ValueError("an L1 checkpoint carries the run config; pass config=")
        arrays: dict = {}
        meta = {"format": FORMAT, "level": level, "obs_spec": obs_spec,
                "action_spec": action_spec,
                "agent_state": split(agent_state, AGENT_PREFIX, arrays),
                "env_policy_state": (None if env_policy_state is None
                                     else split(env_policy_state, "env_policy_state", arrays)),
                "extra": {}}
        if level == "L1":
            meta["frame"] = int(frame)
            meta["config"] = split(config, "config", arrays)
            meta["env_reward_state"] = None
            meta["replay_state"] = None
            meta["cadence_state"] = None
        return cls(meta, arrays)

    @property
    def level(self) -> str:
        return self.meta["level"]

    def agent_state(self) -> dict:
        return join(self.meta["agent_state"], self.arrays, file=self.source or "<checkpoint>")

    def with_agent_state(self, state: dict) -> "Checkpoint":
        """This checkpoint with its agent state replaced (other members kept)."""
        prefix = AGENT_PREFIX + "."
        arrays = {k: v for k, v in self.arrays.items()
                  if k != AGENT_PREFIX and not k.startswith(prefix)}
        fresh: dict = {}
        meta = dict(self.meta)
        meta["agent_state"] = split(state, AGENT_PREFIX, fresh)
        clash = set(fresh) & set(arrays)
        if clash:
            raise ValueError(f"agent state arrays {sorted(clash)} collide with other members")
        arrays.update(fresh)
        return Checkpoint(meta, arrays, self.source)

    def update(self, *, frame: int | None = None, **parts) -> "Checkpoint":
        """The agent state with the B200 learner's parts written back under
        their keys (`online=`, `target=`, `net=`, `nets=`, `optimizer=`,
        `actor_opt=`, `log_alpha=` ...), each array in its stored form."""
        state = self.agent_state()
        state.update(learner_state(like=state, **parts))
        out = self.with_agent_state(state)
        if frame is not None:
            if out.level != "L1":
                raise ValueError("only an L1 checkpoint carries a frame count")
            out.meta["frame"] = int(frame)
        return out

    def to_bytes(self) -> bytes:
        buf = io.BytesIO()
        payload = dict(self.arrays)
        blob = json.dumps(self.meta, default=_json_default).encode("utf-8")
        payload[META_KEY] = np.frombuffer(blob, dtype=np.uint8)
        np.savez(buf, **payload)
        return buf.getvalue()

    def write(self, path: str) -> None:
        atomic_write_bytes(path, self.to_bytes())


# -- the B200 learner's side ---------------------------------------------------

def _is_optimizer(obj) -> bool:
    return hasattr(obj, "state_dict") and hasattr(obj, "params") and hasattr(obj, "m")


def _optimizer_state(opt, like) -> dict:
    """`opt.state_dict()` with each convolution moment in the form the file
    holds it (`like`: that optimizer's stored state, or None for OIHW)."""
    state = opt.state_dict()
    if like is None:
        return state
    for key in ("m", "v"):
        if len(like[key]) != len(state[key]):
            raise ValueError(f"the checkpoint's optimizer holds {len(like[key])} {key} buffers "
                             f"and this one {len(state[key])}")
    for i, p in enumerate(opt.params):
        layout = getattr(p, "_layout", None)
        stored_m = np.asarray(like["m"][i])
        if layout is None or stored_m.shape == tuple(layout.oihw):
            continue
        prepared = getattr(layout, "stored_layout", None)
        if prepared is None or prepared.shape != stored_m.shape:
            # Not loaded from this file: recover the channel stride from the
            # file's own second moment, refusing to guess when it cannot tell.
            prepared = solve_cp(stored_m.shape, layout.oihw, v=np.asarray(like["v"][i]),
                                strict=True)
        state["m"][i] = prepared.pack(state["m"][i])
        state["v"][i] = prepared.pack(state["v"][i])
    return state


def _state_of(obj, like) -> Any:
    if _is_optimizer(obj):
        return _optimizer_state(obj, like)
    if hasattr(obj, "state_dict"):
        return obj.state_dict()
    if hasattr(obj, "numpy"):
        return np.asarray(obj.numpy(), np.float32)
    return np.asarray(obj)


def learner_state(*, like: dict | None = None, **parts) -> dict:
    """{key: state} for the learner's parts, in the reference's agent-state
    names (ttrl/algos/dqn/agent.py:225-238, ppo/state.py:30-43,
    sac/agent.py:249-264)."""
    out = {}
    for key, obj in parts.items():
        stored = None if like is None else like.get(key)
        out[key] = _state_of(obj, stored)
    return out


def load_learner(agent_state: dict, **parts) -> None:
    """Restore the learner's parts, in place, from an agent state tree."""
    missing = [k for k in parts if k not in agent_state]
    if missing:
        raise KeyError(f"the checkpoint's agent state has no {missing} "
                       f"(it holds {sorted(agent_state)})")
    for key, obj in parts.items():
        state = agent_state[key]
        if _is_optimizer(obj) or hasattr(obj, "load_state_dict"):
            obj.load_state_dict(state)
        elif hasattr(obj, "data"):
            from ttrl_b200.engine.tensor import restore_in_place
            restore_in_place(obj.data, np.asarray(state, np.float32))
        else:
            raise TypeError(f"load_learner: cannot restore {key!r} into {type(obj).__name__}")
