"""`Module`, `ModuleList`, `ModuleDict`: parameter discovery by attribute
walk, portable state_dict / in-place load_state_dict, and the hard target
copy. Same contract as ttrl/engine/nn/{module,containers,discovery}.py.
"""

from __future__ import annotations

from typing import Iterator

import numpy as np
import torch

from ttrl_b200.engine.autograd import Tensor
from ttrl_b200.engine.tensor import restore_in_place

__all__ = ["Module", "ModuleList", "ModuleDict", "check_state_layout", "parameter_arena"]


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
        """Write `state` into this module's existing buffers.

        The whole state is checked against the names and shapes this module's
        own `state_dict()` produces before anything is written, so a state
        that does not fit changes nothing. Writes go into the buffers that
        exist (captured graphs keep reading the live weights). `device` is
        accepted for the reference's signature; the buffers carry their own."""
        slots = self._state_slots()
        layout = {}
        for name, target in slots:
            if isinstance(target, Tensor):
                layout[name] = tuple(target.data.shape)
            else:
                for key, array in target.state_dict().items():
                    layout[f"{name}.{key}"] = tuple(np.shape(array))
        check_state_layout(state, layout, type(self).__name__)
        for name, target in slots:
            if isinstance(target, Tensor):
                restore_in_place(target.data, state[name])
            else:
                cut = len(name) + 1
                target.load_state_dict({key[cut:]: value for key, value in state.items()
                                        if key.startswith(name + ".")})

    def copy_from(self, other: "Module") -> None:
        """Make every parameter of this module equal to `other`'s, in place and
        bit for bit, in one launch (the hard target-network sync). The two
        modules must list the same parameter names with the same shapes."""
        mine = dict(self.named_parameters())
        theirs = dict(other.named_parameters())
        if list(mine) != list(theirs):
            raise ValueError(
                f"copy_from: the modules are not the same network; parameters only here: "
                f"{sorted(set(mine) - set(theirs))}, only in the source: "
                f"{sorted(set(theirs) - set(mine))}, or the same names in another order")
        for name, dst in mine.items():
            if tuple(dst.shape) != tuple(theirs[name].shape):
                raise ValueError(f"copy_from: {name!r} is {tuple(dst.shape)} here and "
                                 f"{tuple(theirs[name].shape)} in the source")
        pairs = [(dst.data, theirs[name].data) for name, dst in mine.items()
                 if dst.data.data_ptr() != theirs[name].data.data_ptr()]
        if not pairs:
            return
        if not pairs[0][0].is_cuda:
            # Host replicas (gloo process groups on the CPU) hold host tensors.
            for dst, src in pairs:
                dst.copy_(src)
            return
        from ttrl_b200.device import context
        context(pairs[0][0].device).blend(pairs)


def check_state_layout(state: dict, layout: dict, owner: str) -> None:
    """Raise ValueError unless `state` has exactly the keys of `layout`
    (name -> shape) with those shapes."""
    missing = sorted(set(layout) - set(state))
    unknown = sorted(set(state) - set(layout))
    if missing or unknown:
        raise ValueError(f"{owner}.load_state_dict: the state does not fit this module: "
                         f"missing {missing}, not parameters of it {unknown}")
    for name, shape in layout.items():
        got = tuple(int(d) for d in np.shape(state[name]))
        if got != tuple(shape):
            raise ValueError(f"{owner}.load_state_dict: {name!r} is {got} in the state but "
                             f"{tuple(shape)} in the module")


def parameter_arena(modules, *, align: int = 64) -> torch.Tensor:
    """Place the parameters of `modules` (in order) in one flat fp32 buffer,
    each starting on an `align`-float (256-byte) boundary, and rebind every
    parameter's `.data` to its view of it; returns the buffer. Parameters
    already laid out that way are left where they are.

    Graphs captured before this call keep the old addresses, so call it
    before capturing anything that reads the parameters."""
    params = []
    seen = set()
    for module in modules:
        for p in module.parameters():
            if id(p) not in seen:
                seen.add(id(p))
                params.append(p)
    if not params:
        raise ValueError("parameter_arena: no parameters")
    offsets, total = [], 0
    for p in params:
        offsets.append(total)
        total += (p.data.numel() + align - 1) // align * align
    first = params[0].data
    storage = first.untyped_storage()
    start = first.storage_offset()
    placed = (first.dtype == torch.float32 and storage.nbytes() >= 4 * (start + total)
              and all(p.data.is_contiguous() and p.data.dtype == torch.float32
                      and p.data.untyped_storage().data_ptr() == storage.data_ptr()
                      and p.data.storage_offset() == start + off
                      for p, off in zip(params, offsets)))
    if placed:
        flat = torch.empty(0, dtype=torch.float32, device=first.device)
        return flat.set_(storage, start, (total,), (1,))
    flat = torch.zeros(total, dtype=torch.float32, device=first.device)
    for p, off in zip(params, offsets):
        n = p.data.numel()
        view = flat[off:off + n].view(p.data.shape)
        view.copy_(p.data)
        p.data = view
    return flat


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
