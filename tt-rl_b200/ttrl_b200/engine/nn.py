"""`Module`, `ModuleList`, `ModuleDict`: parameter discovery by attribute
walk, portable state_dict / in-place load_state_dict, and the hard target
copy. Same contract as ttrl/engine/nn/{module,containers,discovery}.py.
"""

from __future__ import annotations

from typing import Iterator

import numpy as np

from ttrl_b200.engine.autograd import Tensor
from ttrl_b200.engine.tensor import copy_tensor_in_place, restore_in_place

__all__ = ["Module", "ModuleList", "ModuleDict"]


def _is_container(value) -> bool:
    return callable(getattr(value, "named_parameters", None))


def _named_from(prefix: str, value, seen: set) -> Iterator[tuple[str, Tensor]]:
    if isinstance(value, Tensor):
        if value.requires_grad and id(value) not in seen:
            seen.add(id(value))
            yield prefix, value
        return
    if _is_container(value):
        for sub, param in value.named_parameters():
            if id(param) not in seen:
                seen.add(id(param))
                yield f"{prefix}.{sub}", param
        return
    if isinstance(value, (list, tuple)):
        for index, item in enumerate(value):
            yield from _named_from(f"{prefix}.{index}", item, seen)
        return
    if isinstance(value, dict):
        for key, item in value.items():
            yield from _named_from(f"{prefix}.{key}", item, seen)


def _serialises_own_state(value) -> bool:
    if not isinstance(value, Module):
        return False
    cls = type(value)
    saves = cls.state_dict is not Module.state_dict
    loads = cls.load_state_dict is not Module.load_state_dict
    if saves != loads:
        raise TypeError(
            f"{cls.__name__} overrides one of state_dict/load_state_dict but not "
            "the other; a module that serialises itself must do both."
        )
    return saves


def _slots_from(prefix: str, value, seen: set):
    if _serialises_own_state(value):
        if id(value) not in seen:
            seen.add(id(value))
            yield prefix, value
        return
    if isinstance(value, Tensor):
        if value.requires_grad and id(value) not in seen:
            seen.add(id(value))
            yield prefix, value
        return
    if isinstance(value, Module):
        for sub, target in value._state_slots(seen):
            yield f"{prefix}.{sub}", target
        return
    if _is_container(value):
        for sub, param in value.named_parameters():
            if id(param) not in seen:
                seen.add(id(param))
                yield f"{prefix}.{sub}", param
        return
    if isinstance(value, (list, tuple)):
        for index, item in enumerate(value):
            yield from _slots_from(f"{prefix}.{index}", item, seen)
        return
    if isinstance(value, dict):
        for key, item in value.items():
            yield from _slots_from(f"{prefix}.{key}", item, seen)


class Module:
    """Base class. Subclasses register Tensors and submodules as attributes."""

    def _slot_sources(self):
        return vars(self).items()

    def _walk(self):
        seen: set[int] = set()
        for name, value in self._slot_sources():
            yield from _named_from(name, value, seen)

    def named_parameters(self) -> Iterator[tuple[str, Tensor]]:
        yield from self._walk()

    def parameters(self) -> Iterator[Tensor]:
        for _, param in self._walk():
            yield param

    def zero_grad(self) -> None:
        for param in self.parameters():
            param.zero_grad()

    def __call__(self, *args, **kwargs):
        return self.forward(*args, **kwargs)

    def forward(self, *args, **kwargs):
        raise NotImplementedError

    def _state_slots(self, seen: set | None = None):
        seen = set() if seen is None else seen
        slots = []
        for name, value in self._slot_sources():
            slots.extend(_slots_from(name, value, seen))
        return slots

    def state_dict(self) -> dict:
        out: dict[str, np.ndarray] = {}
        for name, target in self._state_slots():
            if isinstance(target, Tensor):
                out[name] = target.numpy()
                continue
            for key, array in target.state_dict().items():
                out[f"{name}.{key}"] = array
        return out

    def load_state_dict(self, state: dict, device=None) -> None:
        """Restore parameters in place, after validating every key and shape."""
        slots = self._state_slots()
        reference = self.state_dict()
        got, expected = set(state.keys()), set(reference)
        if got != expected:
            raise ValueError(
                "load_state_dict: checkpoint keys do not match module "
                f"parameters (missing={sorted(expected - got)}, "
                f"extra={sorted(got - expected)})"
            )
        for name, want in reference.items():
            shape = tuple(int(d) for d in np.asarray(state[name]).shape)
            if shape != want.shape:
                raise ValueError(
                    f"load_state_dict: shape mismatch for {name!r}: "
                    f"checkpoint has {shape}, parameter expects {want.shape}"
                )
        for name, target in slots:
            if isinstance(target, Tensor):
                restore_in_place(target.data, state[name])
                continue
            prefix = f"{name}."
            target.load_state_dict(
                {k[len(prefix):]: v for k, v in state.items() if k.startswith(prefix)}
            )

    def copy_from(self, other: "Module") -> None:
        """Hard-copy another module's parameters, in place (target-network sync)."""
        dst_named = list(self.named_parameters())
        src_named = list(other.named_parameters())
        if len(dst_named) != len(src_named):
            raise ValueError(
                f"copy_from: parameter count mismatch ({len(dst_named)} vs "
                f"{len(src_named)}); target and source modules do not match"
            )
        for (dst_name, dst), (src_name, src) in zip(dst_named, src_named, strict=True):
            if dst_name != src_name:
                raise ValueError(
                    f"copy_from: parameter name mismatch ({dst_name!r} vs "
                    f"{src_name!r}); the two modules have different structure"
                )
            if tuple(dst.shape) != tuple(src.shape):
                raise ValueError(
                    f"copy_from: shape mismatch for {dst_name!r}: target "
                    f"{tuple(dst.shape)}, source {tuple(src.shape)}"
                )
            copy_tensor_in_place(dst, src)


class ModuleList(Module):
    """An ordered list of submodules named by index."""

    def __init__(self, modules=()):
        self._items = list(modules)

    def _slot_sources(self):
        return ((str(i), m) for i, m in enumerate(self._items))

    def append(self, module) -> "ModuleList":
        self._items.append(module)
        return self

    def __len__(self) -> int:
        return len(self._items)

    def __iter__(self):
        return iter(self._items)

    def __getitem__(self, index):
        return self._items[index]


class ModuleDict(Module):
    """Submodules keyed by name."""

    def __init__(self, modules=None):
        self._items: dict = {}
        for key, module in (modules or {}).items():
            self[key] = module

    def _slot_sources(self):
        return self._items.items()

    def __setitem__(self, key: str, module) -> None:
        if not isinstance(key, str) or not key or "." in key:
            raise ValueError(f"ModuleDict keys must be non-empty strings without '.', got {key!r}")
        self._items[key] = module

    def __getitem__(self, key: str):
        return self._items[key]

    def __contains__(self, key: str) -> bool:
        return key in self._items

    def __len__(self) -> int:
        return len(self._items)

    def __iter__(self):
        return iter(self._items)

    def keys(self):
        return self._items.keys()

    def items(self):
        return self._items.items()
