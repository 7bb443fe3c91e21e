"""Observation encoders (ttrl/nets/encoders.py): the conv tower with
flatten -> Linear(hidden) -> ReLU, and the MLP tower. The observation
scale (1/255 for pixels) folds into the first layer as the reference does
(conv input_scale; ScaledLinear's weight scale)."""

from __future__ import annotations

from ttrl_b200.engine.conv import Conv2d
from ttrl_b200.engine.layers import Flatten, Linear, ReLU, Sequential
from ttrl_b200.engine.ops import linear, mul
from ttrl_b200.nets.towers import NATURE_CNN

__all__ = ["Encoder", "ScaledLinear", "image_encoder", "vector_encoder"]


class ScaledLinear(Linear):
    """y = (scale * x) @ W + b with the scale folded into the weight."""

    def __init__(self, in_features: int, out_features: int, device=None, *, scale: float = 1.0,
                 bias: bool = True):
        super().__init__(in_features, out_features, device, bias=bias)
        if not scale > 0.0:
            raise ValueError(f"ScaledLinear: scale must be positive, got {scale}")
        self.scale = float(scale)

    def _w(self):
        return self.weight if self.scale == 1.0 else mul(self.weight, self.scale)

    def forward(self, x):
        return linear(x, self._w(), self.bias, relu=False)

    def forward_relu(self, x):
        return linear(x, self._w(), self.bias, relu=True)


class Encoder(Sequential):
    def __init__(self, layers, out_features: int):
        super().__init__(*layers)
        self.out_features = int(out_features)


def image_encoder(in_shape, device=None, *, batch: int, hidden: int = 512, tower=NATURE_CNN,
                  scale: float = 1.0 / 255.0, input_needs_grad: bool = False) -> Encoder:
    """Conv tower -> flatten -> Linear(hidden) -> ReLU over a (C, H, W) image."""
    layers = []
    shape = tuple(int(v) for v in in_shape)
    for index, stage in enumerate(tower):
        first = index == 0
        conv = Conv2d(shape, stage.out_channels, stage.kernel, device, batch=batch,
                      stride=stage.stride, padding=stage.padding, fold=stage.fold,
                      input_scale=scale if first else 1.0,
                      needs_input_grad=input_needs_grad if first else True)
        layers += [conv, ReLU()]
        shape = conv.out_shape
    channels, height, width = shape
    flatten = Flatten(height, width, channels)
    layers += [flatten, Linear(flatten.out_features, hidden, device), ReLU()]
    return Encoder(layers, hidden)


def vector_encoder(in_features: int, device=None, *, hidden=(256, 256),
                   scale: float = 1.0) -> Encoder:
    widths = tuple(int(w) for w in hidden)
    if not widths or min(widths) < 1:
        raise ValueError(f"mlp encoder: hidden must be positive widths, got {hidden}")
    layers = []
    prev = int(in_features)
    for index, width in enumerate(widths):
        layers += [ScaledLinear(prev, width, device, scale=scale if index == 0 else 1.0),
                   ReLU()]
        prev = width
    return Encoder(layers, widths[-1])
