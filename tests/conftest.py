"""Shared pytest set-up: import paths and the `gpu` marker.

`-m "not gpu"` runs everything that needs no GPU (the oracle against the
golden vectors, host logic, the C-ABI library's exported symbols, gloo
multi-process tests). `-m gpu` runs the parity tests proper on a B200.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for path in (ROOT, os.path.join(ROOT, "tt-rl_b200")):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
