"""`Conv2d` over flattened-NHWC activations (ttrl/engine/conv/module.py).

The weight is held on the device as [Cout][KH][KW][Cin] ("KRSC"), the order
the implicit GEMM walks one output row in; `weight_numpy`,
`weight_grad_numpy`, `load_weight_numpy` and the state_dict use the logical
OIHW form, as the reference's do, so checkpoints are interchangeable.

Geometry rules follow ttrl/engine/conv/geometry.py: output sizes, and a
refusal of ragged strides (the input gradient is only the exact adjoint for
exactly divisible strides). A space-to-depth `fold` is accepted and checked
like the reference's.

Space-to-depth on the device: a layer that needs no input gradient (the
first layer over frames) and whose stride s divides its kernel and input
runs as the stride-1 convolution with kernel k/s over s*s*C channels, on
rows in space-to-depth order (channel (dy*s + dx)*C + c, the reference's
fold order, ttrl/engine/conv/packing.py:152-160). The products are the same;
the operand gathers then read contiguous runs of s*s*C channels instead of C.
Its weight is stored in that folded KRSC order. Input rows arrive folded
straight from the frame conversion (`Tensor._fold`), or are folded here.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from ttrl_b200.device import context, conv_geom
from ttrl_b200.engine.autograd import Tensor, as_device
from ttrl_b200.engine.nn import Module, check_state_layout
from ttrl_b200.engine.ops import conv2d_nhwc
from ttrl_b200.engine.packing import default_layout, solve_cp
from ttrl_b200.engine.tensor import restore_in_place

__all__ = ["Conv2d", "ConvGeometry", "ConvDoesNotFit", "conv_out_size", "input_fold"]


class ConvDoesNotFit(ValueError):
    """Kept for interface compatibility (ttrl/engine/conv/geometry.py:127-133).
    A B200 has no per-core L1 ceiling on these layers, so nothing raises it."""


def conv_out_size(size: int, kernel: int, stride: int, padding: int, *, axis: str = "h") -> int:
    """(size + 2*padding - kernel) // stride + 1, with the geometry checked
    (ttrl/engine/conv/geometry.py:94-124)."""
    if kernel <= 0 or stride <= 0 or padding < 0:
        raise ValueError(
            f"conv2d: kernel and stride must be > 0 and padding >= 0, got "
            f"kernel={kernel}, stride={stride}, padding={padding}"
        )
    span = size + 2 * padding - kernel
    if span < 0:
        raise ValueError(
            f"conv2d: input {axis}={size} with padding={padding} is smaller than "
            f"kernel={kernel}; output would be empty"
        )
    if span % stride != 0:
        raise ValueError(
            f"conv2d: ragged geometry on {axis}: (size + 2*padding - kernel) = "
            f"{span} is not a multiple of stride={stride} (size={size}, "
            f"kernel={kernel}, padding={padding}). The input gradient is only "
            f"the true adjoint for exactly divisible strides."
        )
    return span // stride + 1


@dataclass(frozen=True)
class ConvGeometry:
    batch: int
    in_channels: int
    in_h: int
    in_w: int
    out_channels: int
    kernel: int
    stride: int = 1
    padding: int = 0
    fold: int = 1

    def __post_init__(self) -> None:
        if min(self.batch, self.in_channels, self.in_h, self.in_w, self.out_channels) <= 0:
            raise ValueError(f"conv2d: batch, channels and input extent must be > 0, got {self}")
        if self.fold < 1:
            raise ValueError(f"conv2d: fold must be >= 1, got {self.fold}")
        if self.fold > 1:
            if self.stride != self.fold or self.padding != 0:
                raise ValueError(
                    f"conv2d: space-to-depth needs stride == fold and padding == 0, got "
                    f"stride={self.stride} fold={self.fold} padding={self.padding}"
                )
            for name, size in (("kernel", self.kernel), ("in_h", self.in_h), ("in_w", self.in_w)):
                if size % self.fold:
                    raise ValueError(f"conv2d: fold={self.fold} must divide {name}={size}")
        _ = (self.out_h, self.out_w)

    @property
    def out_h(self) -> int:
        return conv_out_size(self.in_h, self.kernel, self.stride, self.padding, axis="h")

    @property
    def out_w(self) -> int:
        return conv_out_size(self.in_w, self.kernel, self.stride, self.padding, axis="w")

    @property
    def out_shape(self) -> tuple[int, int, int]:
        return (self.out_channels, self.out_h, self.out_w)

    @property
    def in_numel(self) -> int:
        return self.batch * self.in_channels * self.in_h * self.in_w

    def kernel_geom(self):
        return conv_geom(self.batch, self.in_h, self.in_w, self.in_channels, self.out_channels,
                         self.kernel, self.kernel, self.stride, self.padding)


class Conv2d(Module):
    """A convolution holding its own weight (KRSC on device) and bias."""

    def __init__(self, in_shape, out_channels: int, kernel: int, device=None, *, batch: int,
                 stride: int = 1, padding: int = 0, bias: bool = True, fold: int = 1,
                 input_scale: float = 1.0, weight=None, needs_input_grad: bool = True,
                 profile=None):
        if len(tuple(in_shape)) != 3:
            raise ValueError(
                f"Conv2d: in_shape must be (channels, height, width), got {tuple(in_shape)}"
            )
        in_channels, in_h, in_w = (int(v) for v in in_shape)
        self.geom = ConvGeometry(
            batch=int(batch), in_channels=in_channels, in_h=in_h, in_w=in_w,
            out_channels=int(out_channels), kernel=int(kernel), stride=int(stride),
            padding=int(padding), fold=int(fold),
        )
        self.device = as_device(device)
        self.input_scale = float(input_scale)
        self.needs_input_grad = bool(needs_input_grad)
        if weight is None:
            bound = 1.0 / math.sqrt(in_channels * kernel * kernel)
            weight = np.random.uniform(
                -bound, bound, (out_channels, in_channels, kernel, kernel)
            ).astype(np.float32)
        else:
            weight = np.asarray(weight, np.float32)
            want = (out_channels, in_channels, kernel, kernel)
            if weight.shape != want:
                raise ValueError(f"Conv2d: weight must have shape {want}, got {weight.shape}")
        self._oihw_shape = weight.shape
        self.s2d = self._space_to_depth_factor()
        self.weight = Tensor.from_numpy(self._to_device_layout(weight), self.device,
                                        requires_grad=True)
        self.weight._layout = ConvWeightLayout(self)
        if bias:
            bound = 1.0 / math.sqrt(in_channels * kernel * kernel)
            b = np.random.uniform(-bound, bound, (1, 1, 1, out_channels)).astype(np.float32)
            self.bias = Tensor.from_numpy(b, self.device, requires_grad=True)
        else:
            self.bias = None
        self._kgeom = self._kernel_geom()

    # -- space-to-depth --------------------------------------------------

    def _space_to_depth_factor(self) -> int:
        g = self.geom
        f = g.stride
        if (not self.needs_input_grad and f > 1 and g.padding == 0 and g.kernel % f == 0
                and g.in_h % f == 0 and g.in_w % f == 0):
            return f
        return 1

    def _to_device_layout(self, w_oihw: np.ndarray) -> np.ndarray:
        """OIHW -> KRSC over the (folded) kernel: [O][k/f][k/f][(dy*f+dx)*C + c]."""
        o, c, k, _ = w_oihw.shape
        f, kb = self.s2d, k // self.s2d
        return np.ascontiguousarray(
            w_oihw.reshape(o, c, kb, f, kb, f).transpose(0, 2, 4, 3, 5, 1)
            .reshape(o, kb, kb, f * f * c))

    def _from_device_layout(self, w_dev: np.ndarray) -> np.ndarray:
        o, c, k, _ = self._oihw_shape
        f, kb = self.s2d, k // self.s2d
        return np.ascontiguousarray(
            w_dev.reshape(o, kb, kb, f, f, c).transpose(0, 5, 1, 3, 2, 4).reshape(o, c, k, k))

    def _kernel_geom(self):
        g, f = self.geom, self.s2d
        if f == 1:
            return g.kernel_geom()
        return conv_geom(g.batch, g.in_h // f, g.in_w // f, g.in_channels * f * f, g.out_channels,
                         g.kernel // f, g.kernel // f, 1, 0)

    def input_fold(self) -> int:
        """The space-to-depth factor this layer reads its input rows in."""
        return self.s2d

    def _fold_input(self, x: Tensor) -> Tensor:
        """Plain NHWC rows -> space-to-depth rows (one strided copy)."""
        g, f = self.geom, self.s2d
        a = g.batch * (g.in_h // f)
        src = x.data.reshape(a, f, g.in_w // f, f * g.in_channels)  # (a, dy, X, dx*C + c)
        out = torch.empty((1, 1, a * (g.in_w // f), f * f * g.in_channels),
                          dtype=torch.float32, device=x.data.device)
        dst = out.reshape(a, g.in_w // f, f, f * g.in_channels).permute(0, 2, 1, 3)
        context(x.data.device).copy_strided(dst, src)
        folded = Tensor(out, requires_grad=False)
        folded._exact = x._exact
        folded._fold = f
        return folded

    @property
    def out_shape(self) -> tuple[int, int, int]:
        return self.geom.out_shape

    @property
    def out_numel(self) -> int:
        return self.geom.batch * int(np.prod(self.geom.out_shape))

    def __repr__(self) -> str:
        g = self.geom
        return (f"Conv2d({g.in_channels}x{g.in_h}x{g.in_w} -> {self.out_shape}, k{g.kernel}, "
                f"s{g.stride}, p{g.padding}, fold={g.fold})")

    # -- parameters ------------------------------------------------------

    def weight_numpy(self) -> np.ndarray:
        return self._from_device_layout(self.weight.numpy())

    def weight_grad_numpy(self) -> np.ndarray:
        if self.weight.grad is None:
            raise ValueError("Conv2d.weight_grad_numpy: no gradient has been accumulated")
        context(self.weight.data.device).join()
        return self._from_device_layout(self.weight.grad.detach().to("cpu").numpy())

    def load_weight_numpy(self, w_oihw) -> None:
        w = np.asarray(w_oihw, np.float32)
        if w.shape != self._oihw_shape:
            raise ValueError(
                f"Conv2d.load_weight_numpy: expected shape {self._oihw_shape}, got {w.shape}"
            )
        restore_in_place(self.weight.data, self._to_device_layout(w))

    def state_dict(self) -> dict:
        state = {"weight": self.weight_numpy()}
        if self.bias is not None:
            state["bias"] = self.bias.numpy()
        return state

    def load_state_dict(self, state: dict, device=None) -> None:
        """OIHW weight (and (1,1,1,C) bias) into the device buffers, in place."""
        layout = {"weight": self._oihw_shape}
        if self.bias is not None:
            layout["bias"] = tuple(self.bias.data.shape)
        check_state_layout(state, layout, "Conv2d")
        self.load_weight_numpy(state["weight"])
        if self.bias is not None:
            restore_in_place(self.bias.data, state["bias"])

    def at_batch(self, batch: int) -> "Conv2d":
        """This layer at another activation batch, sharing weight and bias."""
        view = object.__new__(Conv2d)
        view.__dict__.update(self.__dict__)
        g = self.geom
        view.geom = ConvGeometry(batch=int(batch), in_channels=g.in_channels, in_h=g.in_h,
                                 in_w=g.in_w, out_channels=g.out_channels, kernel=g.kernel,
                                 stride=g.stride, padding=g.padding, fold=g.fold)
        view._kgeom = view._kernel_geom()
        view.needs_input_grad = False
        return view

    # -- call ------------------------------------------------------------

    def _check_input(self, x: Tensor) -> None:
        numel = 1
        for d in x.shape:
            numel *= int(d)
        if numel != self.geom.in_numel:
            raise ValueError(
                f"conv2d: activation has {numel} elements but this layer's geometry "
                f"{self.geom} requires {self.geom.in_numel}; the layer was built for a "
                "different input."
            )

    def _prepare(self, x: Tensor) -> Tensor:
        self._check_input(x)
        if x._fold == self.s2d:
            return x
        if x._fold != 1:
            raise ValueError(f"conv2d: input rows are folded by {x._fold}, this layer reads "
                             f"fold {self.s2d}")
        return self._fold_input(x)

    def forward(self, x: Tensor) -> Tensor:
        return conv2d_nhwc(self._prepare(x), self.weight, self.bias, self._kgeom,
                           input_scale=self.input_scale, relu=False,
                           needs_input_grad=self.needs_input_grad)

    def forward_relu(self, x: Tensor) -> Tensor:
        return conv2d_nhwc(self._prepare(x), self.weight, self.bias, self._kgeom,
                           input_scale=self.input_scale, relu=True,
                           needs_input_grad=self.needs_input_grad)


class ConvWeightLayout:
    """Optimizer state of a convolution weight between this layer's device
    layout (KRSC over the possibly folded kernel) and the portable forms:
    logical OIHW, which `Adam.state_dict` writes, and the reference's
    prepared `[1, 1, rows, cols]` matrix (ttrl_b200.engine.packing), which
    its checkpoints hold the moments in."""

    def __init__(self, conv: "Conv2d"):
        self.oihw = tuple(int(d) for d in conv._oihw_shape)
        self._to_device = conv._to_device_layout
        self._from_device = conv._from_device_layout
        # The prepared layout a checkpoint's moments were read in, if any.
        self.stored_layout = None

    def to_portable(self, device_array) -> np.ndarray:
        return self._from_device(np.asarray(device_array, np.float32))

    def from_stored(self, array, *, v=None) -> np.ndarray:
        """A stored moment (OIHW or prepared) -> this layer's device layout.
        `v`: the stored second moment beside it, which fixes a prepared
        matrix's channel stride."""
        a = np.asarray(array, np.float32)
        if a.shape == self.oihw:
            return self._to_device(a)
        layout = solve_cp(a.shape, self.oihw, v=v)
        # Kept so that writing the moments back packs them into the rows
        # they were read from, even after training has made v ambiguous or
        # for a v that was zero at load.
        self.stored_layout = layout
        return self._to_device(layout.unpack(a))

    def to_stored(self, device_array, like=None, *, v_like=None) -> np.ndarray:
        """The device moment in the form of `like` (a stored array of the
        same moment): prepared when `like` is, OIHW otherwise."""
        w = self.to_portable(device_array)
        if like is None or np.shape(like) == self.oihw:
            return w
        layout = self.stored_layout
        if layout is None or layout.shape != tuple(np.shape(like)):
            layout = solve_cp(np.shape(like), self.oihw, v=v_like, strict=True)
        return layout.pack(w)

    def prepared(self, device_array) -> np.ndarray:
        """The moment in the reference device library's default prepared layout."""
        return default_layout(*self.oihw).pack(self.to_portable(device_array))


def _first_conv(value):
    if isinstance(value, Conv2d):
        return value
    if isinstance(value, Module):
        items = [v for _, v in value._slot_sources()]
    elif isinstance(value, dict):
        items = list(value.values())
    elif isinstance(value, (list, tuple)):
        items = list(value)
    else:
        return None
    for item in items:
        found = _first_conv(item)
        if found is not None:
            return found
    return None


def input_fold(net) -> int:
    """The space-to-depth factor `net`'s first convolution reads its input
    rows in (1 when it has none): frame conversions for this net produce
    rows in that order directly (`DeviceContext.u8_to_f32(..., fold=)`)."""
    conv = _first_conv(net)
    return 1 if conv is None else conv.input_fold()
