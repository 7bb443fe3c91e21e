"""One tower per observation leaf (ttrl/nets/multi.py:53-145).

The reference hangs every encoder's towers off a `towers` ModuleDict keyed by
leaf name, so a single-leaf observation's first conv is named
`encoder.towers.obs.layers.0.weight`. `MultiEncoder` keeps that tree so the
state_dicts and checkpoints are interchangeable; `forward` takes the leaf
mapping, or for a one-leaf encoder the leaf tensor itself (this backend's
hot path hands the encoder device rows, not a mapping).
"""

from __future__ import annotations

from ttrl_b200.engine.nn import Module, ModuleDict
from ttrl_b200.engine.ops import concat

__all__ = ["MultiEncoder", "DEFAULT_LEAF"]

#: The leaf name of a single-observation spec (ttrl/spaces: ObsGroup.single).
DEFAULT_LEAF = "obs"


class MultiEncoder(Module):
    #: The attribute the towers hang off, and so the name segment a leaf adds.
    SLOT = "towers"

    def __init__(self, towers: dict, names=None):
        self._names = tuple(towers) if names is None else tuple(names)
        if set(self._names) != set(towers) or not self._names:
            raise ValueError(f"MultiEncoder: towers {sorted(towers)} do not match the leaf "
                             f"names {list(self._names)}")
        setattr(self, self.SLOT, ModuleDict({n: towers[n] for n in self._names}))
        self.out_features = sum(int(towers[n].out_features) for n in self._names)

    @property
    def names(self) -> tuple[str, ...]:
        return self._names

    @property
    def towers_by_name(self) -> ModuleDict:
        return getattr(self, self.SLOT)

    def __getitem__(self, leaf: str):
        return self.towers_by_name[leaf]

    def __len__(self) -> int:
        return len(self._names)

    @property
    def has_parameters(self) -> bool:
        return any(len(self.towers_by_name[n]) for n in self._names)

    def forward(self, obs):
        towers = self.towers_by_name
        if not isinstance(obs, dict):
            if len(self._names) != 1:
                raise ValueError(f"MultiEncoder over leaves {list(self._names)} needs the leaf "
                                 "mapping, not one tensor")
            tower = towers[self._names[0]]
            return tower(obs) if len(tower) else obs
        missing = [n for n in self._names if n not in obs]
        if missing:
            raise KeyError(f"MultiEncoder was given leaves {sorted(obs)} and needs "
                           f"{list(self._names)} (missing {missing})")
        feats = [towers[n](obs[n]) if len(towers[n]) else obs[n] for n in self._names]
        return feats[0] if len(feats) == 1 else concat(feats, dim=-1)


def single_leaf(tower) -> MultiEncoder:
    """A one-leaf encoder over `tower`, named like the reference's."""
    return MultiEncoder({DEFAULT_LEAF: tower}, (DEFAULT_LEAF,))
