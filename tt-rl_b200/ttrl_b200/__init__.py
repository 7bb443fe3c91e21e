"""ttrl_b200: a B200 (sm_100a) backend for scaleresearch/tt-rl's learner update.

Mirrors the reference's ``ttrl.engine`` interface (Tensor tape, ops, Linear,
Conv2d, GRU, Adam, TrainStep, capture, ParamSync) over hand-written CUDA
kernels reached through the C ABI in ``include/ttrl_b200.h``.
"""

__version__ = "0.1.0"
