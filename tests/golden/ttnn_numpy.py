"""A numpy stand-in for the subset of `ttnn` 0.80 that tt-rl's learner path
calls. TEST INFRASTRUCTURE ONLY: `make_golden.py` installs it as
``sys.modules["ttnn"]`` so the reference's own autograd tape, ops, Adam and
loss modules run unchanged on the host and produce golden vectors.

Every op computes in float32 with float32 scalars, one numpy call per ttnn
call. What this pins is the reference's *composition*: which ops run, in
what order, with which constants. It does not pin ttnn's own rounding.
"""

from __future__ import annotations

import numpy as np

float32 = "float32"
bfloat16 = "bfloat16"
bfloat8_b = "bfloat8_b"
uint32 = "uint32"
int32 = "int32"
TILE_LAYOUT = "TILE"
ROW_MAJOR_LAYOUT = "ROW_MAJOR"
TILE_SIZE = 32


class MathFidelity:
    LoFi, HiFi2, HiFi3, HiFi4 = range(4)


class TensorMemoryLayout:
    """Placement names only: imported by modules this shim never runs."""
    INTERLEAVED, HEIGHT_SHARDED, WIDTH_SHARDED, BLOCK_SHARDED = (
        "INTERLEAVED", "HEIGHT_SHARDED", "WIDTH_SHARDED", "BLOCK_SHARDED")


class _Device:
    def arch(self):
        return "numpy"


DEVICE = _Device()


class Tensor:
    """A host array posing as a device tensor."""

    def __init__(self, array, dtype=float32, *, _dev=None):
        arr = np.asarray(array)
        if dtype == float32:
            arr = arr.astype(np.float32, copy=False)
        self.array = np.ascontiguousarray(arr)
        self.dtype = dtype
        self._dev = _dev

    @property
    def shape(self):
        return tuple(self.array.shape)

    def device(self):
        return self._dev

    def to(self, target):
        if isinstance(target, _Device):
            return Tensor(self.array, self.dtype, _dev=target)
        return self  # a layout

    def cpu(self):
        return Tensor(self.array, self.dtype)

    def to_numpy(self):
        return self.array.copy()

    def get_layout(self):
        return getattr(self, "_layout", ROW_MAJOR_LAYOUT)

    def __repr__(self):
        return f"ttnn_numpy.Tensor(shape={self.shape}, dtype={self.dtype})"


def _arr(x):
    return x.array if isinstance(x, Tensor) else np.float32(x)


def _dev_of(*xs):
    for x in xs:
        if isinstance(x, Tensor) and x._dev is not None:
            return x._dev
    return DEVICE


def _out(result, *inputs, output_tensor=None, dtype=float32):
    res = np.asarray(result)
    if dtype == float32:
        res = res.astype(np.float32, copy=False)
    if output_tensor is not None:
        output_tensor.array[...] = res
        return output_tensor
    return Tensor(res.copy(), dtype, _dev=_dev_of(*inputs))


def _binary(fn):
    def op(a, b, *, output_tensor=None, **_):
        return _out(fn(_arr(a), _arr(b)), a, b, output_tensor=output_tensor)
    return op


add = _binary(lambda a, b: a + b)
sub = _binary(lambda a, b: a - b)
subtract = sub
mul = _binary(lambda a, b: a * b)
multiply = mul
div = _binary(lambda a, b: a / b)
rsub = _binary(lambda a, b: b - a)  # rsub(x, s) = s - x
minimum = _binary(np.minimum)
maximum = _binary(np.maximum)


def addalpha(a, b, alpha, *, output_tensor=None, **_):
    """a + alpha * b."""
    return _out(_arr(a) + np.float32(alpha) * _arr(b), a, b, output_tensor=output_tensor)


def _unary(fn):
    def op(a, *, output_tensor=None, **_):
        return _out(fn(_arr(a)), a, output_tensor=output_tensor)
    return op


neg = _unary(np.negative)
relu = _unary(lambda a: np.maximum(a, np.float32(0.0)))
abs = _unary(np.abs)  # noqa: A001 - ttnn's own name
sign = _unary(np.sign)
exp = _unary(np.exp)
log = _unary(np.log)
tanh = _unary(np.tanh)
sigmoid = _unary(lambda a: np.float32(1.0) / (np.float32(1.0) + np.exp(-a)))
sqrt = _unary(np.sqrt)
square = _unary(np.square)
eqz = _unary(lambda a: (a == 0).astype(np.float32))


def relu_bw(grad, x, **_):
    """[grad * (x > 0)]."""
    return [_out(_arr(grad) * (_arr(x) > 0).astype(np.float32), grad)]


def isfinite(a, **_):
    return _out(np.isfinite(_arr(a)).astype(np.float32), a)


def logical_not(a, **_):
    return _out((_arr(a) == 0).astype(np.float32), a)


def typecast(a, dtype, **_):
    if dtype == float32:
        return _out(_arr(a).astype(np.float32), a)
    return Tensor(_arr(a), dtype, _dev=_dev_of(a))


def full_like(a, value, **_):
    return _out(np.full(a.shape, value, dtype=np.float32), a)


def zeros_like(a, **_):
    return _out(np.zeros(a.shape, dtype=np.float32), a)


def zeros(shape, dtype=float32, layout=None, device=None, **_):
    return Tensor(np.zeros(tuple(shape), np.float32), dtype, _dev=device)


def clone(a, **_):
    return _out(_arr(a).copy(), a)


def _dims(dim, rank):
    if dim is None:
        return None
    if isinstance(dim, (list, tuple)):
        return tuple(d % rank for d in dim)
    return dim % rank


def sum(a, dim=None, keepdim=False, **_):  # noqa: A001 - ttnn's own name
    arr = _arr(a)
    if dim is None:
        # ttnn reduces a whole tensor to one element of the same rank.
        return _out(np.sum(arr, dtype=np.float32).reshape((1,) * max_rank(arr)), a)
    return _out(np.sum(arr, axis=_dims(dim, arr.ndim), keepdims=keepdim, dtype=np.float32), a)


def max(a, dim=None, keepdim=False, **_):  # noqa: A001 - ttnn's own name
    arr = _arr(a)
    if dim is None:
        return _out(np.max(arr).reshape((1,) * max_rank(arr)), a)
    return _out(np.max(arr, axis=_dims(dim, arr.ndim), keepdims=keepdim), a)


def max_rank(arr):
    return arr.ndim if arr.ndim else 1


def argmax(a, dim=None, keepdim=False, **_):
    arr = _arr(a)
    idx = np.argmax(arr, axis=_dims(dim, arr.ndim), keepdims=keepdim)
    return Tensor(idx.astype(np.uint32), uint32, _dev=_dev_of(a))


def reshape(a, shape, **_):
    return _out(_arr(a).reshape(tuple(shape)), a)


def squeeze(a, dim, **_):
    return _out(np.squeeze(_arr(a), axis=dim), a)


def repeat(a, reps, **_):
    return _out(np.tile(_arr(a), tuple(reps)), a)


def concat(tensors, dim=0, **_):
    return _out(np.concatenate([_arr(t) for t in tensors], axis=dim), *tensors)


def slice(a, begins, ends, steps=None, **_):  # noqa: A001 - ttnn's own name
    steps = steps or [1] * len(begins)
    idx = tuple(np.s_[b:e:s] for b, e, s in zip(begins, ends, steps))
    return _out(_arr(a)[idx], a)


def pad(a, padding, value=0.0, **_):
    return _out(np.pad(_arr(a), padding, constant_values=value), a)


def matmul(a, b, *, transpose_a=False, transpose_b=False, **_):
    x = _arr(a)
    y = _arr(b)
    if transpose_a:
        x = np.swapaxes(x, -1, -2)
    if transpose_b:
        y = np.swapaxes(y, -1, -2)
    return _out(np.matmul(x, y), a, b)


def clip(a, lo, hi, **_):
    return _out(np.clip(_arr(a), np.float32(lo), np.float32(hi)), a)


clamp = clip


def init_device_compute_kernel_config(arch, **kwargs):
    return dict(kwargs, arch=arch)


def is_tensor_storage_on_device(t):
    return isinstance(t, Tensor)


def is_device_tensor(t):
    return isinstance(t, Tensor)


def copy_host_to_device_tensor(host, dst, **_):
    dst.array[...] = _arr(host)
    return dst


def to_layout(a, layout, **_):
    """Layouts only tag the tensor here: the values are the same numbers."""
    out = Tensor(_arr(a), getattr(a, "dtype", float32), _dev=_dev_of(a))
    out._layout = layout
    return out


def permute(a, dims, **_):
    return _out(np.transpose(_arr(a), tuple(dims)), a)


def conv_transpose2d(*, input_tensor, weight_tensor, in_channels, out_channels, batch_size,
                     input_height, input_width, kernel_size, stride, padding,
                     output_padding=(0, 0), dilation=(1, 1), groups=1, mirror_kernel=True, **_):
    """Transposed convolution, as documented: the adjoint of a convolution
    with the same kernel, stride and padding (PyTorch's conv_transpose2d
    arithmetic), over row-major NHWC rows [1, 1, N*H*W, Cin]; with
    mirror_kernel the op first mirrors the kernel in both spatial axes.

    The weight is a prepared matrix [1, 1, rows, cols] indexed
    M[r * row_block + q * cp + c, k] = W[r, q, c, k] (c: input channel, k:
    output channel), with the default padding rule of this stand-in's device
    library: cp = in_channels rounded up to 8, row_block = rows / kernel."""
    if tuple(dilation) != (1, 1) or groups != 1 or tuple(output_padding) != (0, 0):
        raise NotImplementedError("conv_transpose2d stand-in: dilation, groups and "
                                  "output_padding are not modelled")
    kh, kw = kernel_size
    sh, sw = stride
    ph, pw = padding
    n, h, w, ci, co = batch_size, input_height, input_width, in_channels, out_channels
    x = _arr(input_tensor).astype(np.float64).reshape(n, h, w, ci)
    m = _arr(weight_tensor).astype(np.float64)
    rows, cols = m.shape[-2], m.shape[-1]
    cp = (ci + 7) // 8 * 8
    row_block = rows // kh
    if rows % kh or row_block < kw * cp or cols < co:
        raise ValueError(f"conv_transpose2d stand-in: weight {m.shape} is not a prepared "
                         f"{kh}x{kw} kernel for {ci} -> {co} channels")
    wk = m.reshape(kh, row_block, cols)[:, :kw * cp].reshape(kh, kw, cp, cols)[:, :, :ci, :co]
    if mirror_kernel:
        wk = wk[::-1, ::-1]
    oh = (h - 1) * sh - 2 * ph + kh
    ow = (w - 1) * sw - 2 * pw + kw
    full = np.zeros((n, (h - 1) * sh + kh, (w - 1) * sw + kw, co))
    for r in range(kh):
        for q in range(kw):
            full[:, r:r + (h - 1) * sh + 1:sh, q:q + (w - 1) * sw + 1:sw, :] += \
                x @ wk[r, q]
    out = full[:, ph:ph + oh, pw:pw + ow, :]
    return _out(out.reshape(1, 1, n * oh * ow, co).astype(np.float32), input_tensor)
