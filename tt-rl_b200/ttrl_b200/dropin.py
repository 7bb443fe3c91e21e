"""Run tt-rl's own `ttrl.nets` and `ttrl.algos` on this backend.

`install()` makes the reference's `ttrl.engine` package (and the one module
above it that calls ttnn directly, `ttrl.algos.grads`) resolve to this
package's modules of the same names, before anything under `ttrl` is
imported. The reference's nets and algorithms then build their layers,
tapes, optimizers and training steps on the B200 kernels, unchanged.

    from ttrl_b200 import dropin
    dropin.install("/path/to/tt-rl")      # or a directory holding the ttrl package
    from ttrl.nets.build import build_q_net
    from ttrl.algos.dqn.losses import update_loss
"""

from __future__ import annotations

import importlib
import os
import sys

__all__ = ["ENGINE_MODULES", "install", "installed"]

#: `ttrl.engine` submodules the reference's nets, algorithms and buffers
#: import (ttrl/nets/*.py, ttrl/algos/**/*.py), each mapped onto the module
#: of the same role here.
ENGINE_MODULES = {
    "ttrl.engine": "ttrl_b200.engine",
    "ttrl.engine.autograd": "ttrl_b200.engine.autograd",
    "ttrl.engine.ops": "ttrl_b200.engine.ops",
    "ttrl.engine.nn": "ttrl_b200.engine.nn",
    "ttrl.engine.tensor": "ttrl_b200.engine.tensor",
    "ttrl.engine.layers": "ttrl_b200.engine.layers",
    "ttrl.engine.conv": "ttrl_b200.engine.conv",
    "ttrl.engine.recurrent": "ttrl_b200.engine.recurrent",
    "ttrl.engine.optim": "ttrl_b200.engine.optim",
    "ttrl.engine.step": "ttrl_b200.engine.step",
    "ttrl.engine.step.core": "ttrl_b200.engine.step.core",
    "ttrl.engine.step.inputs": "ttrl_b200.engine.step.inputs",
    "ttrl.engine.step.metrics": "ttrl_b200.engine.step.metrics",
    "ttrl.engine.trace": "ttrl_b200.engine.trace",
    "ttrl.engine.mesh": "ttrl_b200.engine.mesh",
    "ttrl.engine.config": "ttrl_b200.engine.config",
    "ttrl.engine.carry": "ttrl_b200.engine.carry",
    # The gradient-norm helpers call ttnn themselves (ttrl/algos/grads.py:6).
    "ttrl.algos.grads": "ttrl_b200.algos.grads",
}


def installed() -> bool:
    return all(sys.modules.get(k) is importlib.import_module(v)
               for k, v in ENGINE_MODULES.items())


def install(reference: str | None = None) -> None:
    """Alias the engine modules; with `reference`, also put that checkout (a
    directory containing the `ttrl` package) first on sys.path. Raises if
    `ttrl.engine` was already imported from the reference itself."""
    for name in ENGINE_MODULES:
        mod = sys.modules.get(name)
        if mod is not None and not mod.__name__.startswith("ttrl_b200"):
            raise RuntimeError(f"{name} was imported before dropin.install(); call install() "
                               "before importing anything under ttrl")
    if reference is not None:
        path = os.path.abspath(reference)
        if not os.path.isdir(os.path.join(path, "ttrl")):
            raise FileNotFoundError(f"no ttrl package under {path}")
        if path not in sys.path:
            sys.path.insert(0, path)
    for name, target in ENGINE_MODULES.items():
        sys.modules[name] = importlib.import_module(target)
