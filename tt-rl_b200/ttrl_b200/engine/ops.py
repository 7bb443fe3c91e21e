"""Autograd ops with the reference's names and semantics, each one launch of
the CUDA kernels in libttrl_b200.so.

Mirrors ttrl/engine/ops/{elementwise,unary,select,reduce,functional,
matmul,shape,broadcast}.py: same forward values, same backward rules
(including the relu-identity spellings of minimum/maximum/clamp whose
gradient is 0 at the bound, ops/select.py:39-63), same shape conventions
(keepdim reductions, (1,)*rank for sum_all).

The fused layer ops (`linear`, `conv2d_nhwc`) and the fused loss heads live
here too; they are what the nets and algos in this package use on the hot
path.
"""

from __future__ import annotations

import numpy as np
import torch

from ttrl_b200 import _lib
from ttrl_b200.device import PREP_LANE, context
from ttrl_b200.engine.autograd import Tensor, _detached, _is_scalar, _needs, backward_root

__all__ = [
    "add", "div", "mul", "sub",
    "abs_", "exp", "log", "neg", "relu", "sigmoid", "sqrt", "square", "tanh",
    "clamp", "maximum", "minimum",
    "matmul",
    "argmax_dim_detached", "max_dim_detached", "mean_all", "mean_dim",
    "sum_all", "sum_dim",
    "concat", "reshape", "split",
    "apply_done_mask", "entropy", "gather_onehot", "huber", "log_softmax",
    "masks", "non_finite_check", "one_hot_device", "one_hot_gather",
    "one_hot_host", "purge_lane_caches", "purge_matmul_caches",
    "linear", "conv2d_nhwc", "dqn_td_huber", "ppo_objective",
    "sac_sample", "sac_critic_loss", "sac_actor_loss",
]


def _ctx(t):
    return context(t.device)


def _new(shape, like):
    return torch.empty(shape, dtype=torch.float32, device=like.device)


def _weight_grad(ctx, receivers, tensors, launch) -> None:
    """Run a weight-gradient launch on a side lane, beside the data-gradient
    chain, when every gradient it writes belongs to a leaf parameter (read
    only after backward() joins the lanes); otherwise on the current stream.
    Each parameter keeps one lane, so its gradient accumulates in order.
    `tensors` are the buffers it touches, kept from reuse until it is done."""
    if ctx.concurrent and all(t._op == "" for t in receivers):
        with ctx.side(ctx.weight_lane(receivers[0].data)) as s:
            for t in tensors:
                if t is not None:
                    t.record_stream(s)
            launch()
    else:
        launch()


def _ew(op, a, b=None, scalar=0.0, shape=None):
    """Run one elementwise kernel; a/b are torch tensors (broadcastable)."""
    if shape is None:
        shape = a.shape if b is None else torch.broadcast_shapes(a.shape, b.shape)
    out = _new(shape, a)
    _ctx(a).ew(op, a, b, out, scalar)
    return out


# --------------------------------------------------------------------------
# broadcast helpers (ttrl/engine/ops/broadcast.py:11-58)
# --------------------------------------------------------------------------

def _sum_dim_raw(x, dim: int):
    """Sum one axis of a contiguous torch tensor, keepdim, on the device."""
    x = x.contiguous()
    shape = tuple(x.shape)
    dim = dim % len(shape)
    outer = int(np.prod(shape[:dim])) if dim else 1
    n = shape[dim]
    inner = int(np.prod(shape[dim + 1:])) if dim + 1 < len(shape) else 1
    out_shape = shape[:dim] + (1,) + shape[dim + 1:]
    out = _new(out_shape, x)
    _ctx(x).reduce(_lib.RED_SUM, x, out, outer, n, inner)
    return out


def _reduce_broadcast_grad(grad, target_shape):
    grad_shape = tuple(grad.shape)
    target_shape = tuple(target_shape)
    pad = len(grad_shape) - len(target_shape)
    assert pad >= 0, "grad rank must be >= operand rank"
    padded = (1,) * pad + target_shape
    for dim, (g, t) in enumerate(zip(grad_shape, padded)):
        if t == 1 and g != 1:
            grad = _sum_dim_raw(grad, dim)
    return grad.reshape(target_shape)


def _broadcast_to(grad, shape):
    """Materialise a broadcast of grad to `shape` (one copy kernel)."""
    shape = tuple(shape)
    if tuple(grad.shape) == shape:
        return grad
    out = _new(shape, grad)
    _ctx(grad).ew("copy", grad.reshape((1,) * (len(shape) - grad.dim()) + tuple(grad.shape)),
                  None, out)
    return out


# --------------------------------------------------------------------------
# binary elementwise (ttrl/engine/ops/elementwise.py)
# --------------------------------------------------------------------------

def _as_tensor(x, like: Tensor) -> Tensor:
    if isinstance(x, Tensor):
        return x
    out = _new(like.shape, like.data)
    _ctx(like.data).ew("fill", None, None, out, float(x))
    return Tensor(out, requires_grad=False)


def add(a: Tensor, b) -> Tensor:
    if _is_scalar(b):
        y = _ew("add_s", a.data, scalar=float(b))
        if not _needs(a):
            return _detached(y)
        out = Tensor(y, True, (a,), "add")

        def _backward_scalar(grad):
            if a.requires_grad:
                a._accumulate(grad)

        out._backward = _backward_scalar
        return out
    b = _as_tensor(b, a)
    y = _ew("add", a.data, b.data)
    if not _needs(a, b):
        return _detached(y)
    out = Tensor(y, True, (a, b), "add")

    def _backward(grad):
        if a.requires_grad:
            a._accumulate(_reduce_broadcast_grad(grad, a.shape))
        if b.requires_grad:
            b._accumulate(_reduce_broadcast_grad(grad, b.shape))

    out._backward = _backward
    return out


def sub(a, b) -> Tensor:
    if isinstance(a, Tensor) and _is_scalar(b):
        y = _ew("sub_s", a.data, scalar=float(b))
        if not _needs(a):
            return _detached(y)
        out = Tensor(y, True, (a,), "sub")

        def _backward_scalar(grad):
            if a.requires_grad:
                a._accumulate(grad)

        out._backward = _backward_scalar
        return out
    if isinstance(b, Tensor) and _is_scalar(a):
        y = _ew("rsub_s", b.data, scalar=float(a))
        if not _needs(b):
            return _detached(y)
        out = Tensor(y, True, (b,), "sub")

        def _backward_rscalar(grad):
            if b.requires_grad:
                b._accumulate(_ew("neg", grad))

        out._backward = _backward_rscalar
        return out
    if not isinstance(a, Tensor) or not isinstance(b, Tensor):
        raise TypeError(f"sub expects Tensor operands or one scalar, got {type(a)} and {type(b)}")
    y = _ew("sub", a.data, b.data)
    if not _needs(a, b):
        return _detached(y)
    out = Tensor(y, True, (a, b), "sub")

    def _backward(grad):
        if a.requires_grad:
            a._accumulate(_reduce_broadcast_grad(grad, a.shape))
        if b.requires_grad:
            b._accumulate(_reduce_broadcast_grad(_ew("neg", grad), b.shape))

    out._backward = _backward
    return out


def mul(a: Tensor, b) -> Tensor:
    if _is_scalar(b):
        s = float(b)
        y = _ew("mul_s", a.data, scalar=s)
        if not _needs(a):
            return _detached(y)
        out = Tensor(y, True, (a,), "mul")

        def _backward_scalar(grad):
            if a.requires_grad:
                a._accumulate(_ew("mul_s", grad, scalar=s))

        out._backward = _backward_scalar
        return out
    b = _as_tensor(b, a)
    y = _ew("mul", a.data, b.data)
    if not _needs(a, b):
        return _detached(y)
    out = Tensor(y, True, (a, b), "mul")
    ad, bd = a.data, b.data

    def _backward(grad):
        if a.requires_grad:
            a._accumulate(_reduce_broadcast_grad(_ew("mul", grad, bd), a.shape))
        if b.requires_grad:
            b._accumulate(_reduce_broadcast_grad(_ew("mul", grad, ad), b.shape))

    out._backward = _backward
    return out


def div(a: Tensor, b) -> Tensor:
    if _is_scalar(b):
        s = float(b)
        y = _ew("div_s", a.data, scalar=s)
        if not _needs(a):
            return _detached(y)
        out = Tensor(y, True, (a,), "div")

        def _backward_scalar(grad):
            if a.requires_grad:
                a._accumulate(_ew("div_s", grad, scalar=s))

        out._backward = _backward_scalar
        return out
    b = _as_tensor(b, a)
    y = _ew("div", a.data, b.data)
    if not _needs(a, b):
        return _detached(y)
    out = Tensor(y, True, (a, b), "div")
    ad, bd = a.data, b.data

    def _backward(grad):
        if a.requires_grad:
            a._accumulate(_reduce_broadcast_grad(_ew("div", grad, bd), a.shape))
        if b.requires_grad:
            # d/db (a/b) = -a/b^2, in the op order of elementwise.py:140-143
            neg_ratio = _ew("neg", _ew("div", ad, _ew("mul", bd, bd)))
            b._accumulate(_reduce_broadcast_grad(_ew("mul", grad, neg_ratio), b.shape))

    out._backward = _backward
    return out


# --------------------------------------------------------------------------
# unary (ttrl/engine/ops/unary.py)
# --------------------------------------------------------------------------

def neg(a: Tensor) -> Tensor:
    return mul(a, -1.0)


def _unary(name, a: Tensor, fwd: str, bwd) -> Tensor:
    y = _ew(fwd, a.data)
    if not _needs(a):
        return _detached(y)
    out = Tensor(y, True, (a,), name)
    ad = a.data

    def _backward(grad):
        if a.requires_grad:
            a._accumulate(bwd(grad, ad, y))

    out._backward = _backward
    return out


def relu(a: Tensor) -> Tensor:
    return _unary("relu", a, "relu", lambda g, x, y: _ew("relu_bw", g, x))


def abs_(a: Tensor) -> Tensor:
    return _unary("abs", a, "abs", lambda g, x, y: _ew("mul", g, _ew("sign", x)))


def square(a: Tensor) -> Tensor:
    return _unary("square", a, "square",
                  lambda g, x, y: _ew("mul", g, _ew("mul_s", x, scalar=2.0)))


def exp(a: Tensor) -> Tensor:
    return _unary("exp", a, "exp", lambda g, x, y: _ew("mul", g, y))


def log(a: Tensor) -> Tensor:
    return _unary("log", a, "log", lambda g, x, y: _ew("div", g, x))


def tanh(a: Tensor) -> Tensor:
    return _unary("tanh", a, "tanh",
                  lambda g, x, y: _ew("mul", g, _ew("rsub_s", _ew("mul", y, y), scalar=1.0)))


def sigmoid(a: Tensor) -> Tensor:
    return _unary("sigmoid", a, "sigmoid",
                  lambda g, x, y: _ew("mul", g, _ew("mul", y, _ew("rsub_s", y, scalar=1.0))))


def sqrt(a: Tensor) -> Tensor:
    return _unary("sqrt", a, "sqrt", lambda g, x, y: _ew("div", g, _ew("mul_s", y, scalar=2.0)))


# --------------------------------------------------------------------------
# select (ttrl/engine/ops/select.py): relu identities, grad 0 at the bound
# --------------------------------------------------------------------------

def minimum(a: Tensor, b) -> Tensor:
    """min(a, b) = a - relu(a - b)."""
    return sub(a, relu(sub(a, b)))


def maximum(a: Tensor, b) -> Tensor:
    """max(a, b) = a + relu(b - a)."""
    return add(a, relu(sub(b, a)))


def clamp(x: Tensor, lo: float, hi: float) -> Tensor:
    lifted_max = add(relu(sub(x, lo)), lo)
    return sub(hi, relu(sub(hi, lifted_max)))


# --------------------------------------------------------------------------
# reductions (ttrl/engine/ops/reduce.py)
# --------------------------------------------------------------------------

def sum_all(a: Tensor) -> Tensor:
    rank = len(a.shape)
    flat = a.data.contiguous()
    out = _new((1,) * max(rank, 1), flat)
    _ctx(flat).reduce(_lib.RED_SUM, flat, out, 1, flat.numel(), 1)
    if not _needs(a):
        return _detached(out)
    node = Tensor(out, True, (a,), "sum_all")
    shape = a.shape

    def _backward(grad):
        if a.requires_grad:
            a._accumulate(_broadcast_to(grad.reshape((1,) * len(shape)), shape))

    node._backward = _backward
    return node


def mean_all(a: Tensor) -> Tensor:
    n = 1
    for d in a.shape:
        n *= int(d)
    return mul(sum_all(a), 1.0 / n)


def sum_dim(a: Tensor, dim: int, keepdim: bool = True) -> Tensor:
    d = dim if dim >= 0 else dim + len(a.shape)
    y = _sum_dim_raw(a.data, d)
    if not keepdim:
        y = y.reshape(tuple(a.shape[:d]) + tuple(a.shape[d + 1:]))
    if not _needs(a):
        return _detached(y)
    out = Tensor(y, True, (a,), "sum_dim")
    shape = a.shape

    def _backward(grad):
        if a.requires_grad:
            g = grad.reshape(tuple(shape[:d]) + (1,) + tuple(shape[d + 1:]))
            a._accumulate(_broadcast_to(g, shape))

    out._backward = _backward
    return out


def mean_dim(a: Tensor, dim: int, keepdim: bool = True) -> Tensor:
    d = dim if dim >= 0 else dim + len(a.shape)
    return mul(sum_dim(a, dim=dim, keepdim=keepdim), 1.0 / int(a.shape[d]))


def _reduce_axis(a: Tensor, op: int, dim: int, keepdim: bool):
    x = a.data.contiguous()
    shape = tuple(x.shape)
    d = dim % len(shape)
    outer = int(np.prod(shape[:d])) if d else 1
    inner = int(np.prod(shape[d + 1:])) if d + 1 < len(shape) else 1
    out = _new(shape[:d] + (1,) + shape[d + 1:], x)
    _ctx(x).reduce(op, x, out, outer, shape[d], inner)
    if not keepdim:
        out = out.reshape(shape[:d] + shape[d + 1:])
    return out


def max_dim_detached(a: Tensor, dim: int, keepdim: bool = True) -> Tensor:
    return Tensor(_reduce_axis(a, _lib.RED_MAX, dim, keepdim), requires_grad=False)


def argmax_dim_detached(a: Tensor, dim: int = -1, keepdim: bool = True) -> Tensor:
    """Index of the (first) maximum as an fp32 device tensor."""
    return Tensor(_reduce_axis(a, _lib.RED_ARGMAX, dim, keepdim), requires_grad=False)


# --------------------------------------------------------------------------
# matmul (ttrl/engine/ops/matmul.py:55-86)
# --------------------------------------------------------------------------

def matmul(a: Tensor, b: Tensor) -> Tensor:
    if len(a.shape) < 2 or len(b.shape) < 2:
        raise ValueError(
            f"matmul expects rank>=2 operands, got {a.shape} @ {b.shape}; "
            "reshape vectors to an explicit (1, K) / (K, 1) matrix first."
        )
    if len(a.shape) != 2 or len(b.shape) != 2:
        raise ValueError(f"matmul on this backend takes rank-2 operands, got {a.shape} @ {b.shape}")
    return linear(a, b, None, relu=False, _op="matmul")


def purge_matmul_caches(device) -> None:
    """No per-device matmul state is kept on this backend."""


# --------------------------------------------------------------------------
# fused layers
# --------------------------------------------------------------------------

def linear(x: Tensor, w: Tensor, b: Tensor | None, *, relu: bool = False,
           _op: str | None = None) -> Tensor:
    """y = x @ W (+ b) (then ReLU): one tcgen05 GEMM with a fused epilogue.

    Backward: dX = g @ W^T with the ReLU mask of x's producer fused in (when
    x carries one), dW = x^T @ g with db = colsum(g) in the same GEMM.
    """
    xd = x.data if x.data.is_contiguous() else x.data.contiguous()
    m, k = xd.shape
    n = w.shape[1]
    y = _new((m, n), xd)
    ctx = _ctx(xd)
    ctx.linear_fwd(xd, w.data, None if b is None else b.data, y, relu)
    parents = (x, w) if b is None else (x, w, b)
    if not _needs(*parents):
        out = _detached(y)
        return out
    op = _op or ("linear_relu" if relu else "linear")
    out = Tensor(y, True, parents, op)
    out._premask = bool(relu)

    def _backward(grad):
        g = grad if grad.is_contiguous() else grad.contiguous()
        # The weight gradient is issued first so that, on a side lane, it
        # starts while the data gradient runs.
        wb = w.requires_grad
        bb = b is not None and b.requires_grad
        if wb or bb:
            if wb:
                dw, accw = w._grad_slot()
            else:
                dw, accw = torch.empty_like(w.data), False
            if bb:
                db, accb = b._grad_slot()
            else:
                db, accb = None, False
            receivers = [t for t, want in ((w, wb), (b, bb)) if want]
            _weight_grad(ctx, receivers, (xd, g, dw, db),
                         lambda: ctx.linear_wgrad(xd, g, dw, db, accw, accb))
            if wb:
                w._set_grad(dw)
            if bb:
                b._set_grad(db)
        if x.requires_grad:
            buf, acc = x._grad_slot()
            ctx.linear_dgrad(g, w.data, xd if x._premask else None, buf, acc)
            x._set_grad(buf)

    out._backward = _backward
    return out


def conv2d_nhwc(x: Tensor, w: Tensor, b: Tensor | None, geom, *, input_scale: float = 1.0,
                relu: bool = False, needs_input_grad: bool = True) -> Tensor:
    """Convolution of flattened-NHWC rows `[1,1,N*H*W,C]` with a KRSC weight,
    bias and optional ReLU fused (implicit-GEMM fprop on tcgen05).

    Backward: dX by a tcgen05 GEMM into kernel-tap columns plus a col2im
    gather with the producer's ReLU mask fused; dW (times input_scale) and db
    by one split-K implicit GEMM with a row of ones for the bias.
    """
    xd = x.data.reshape(-1, geom.c)
    if not xd.is_contiguous():
        xd = xd.contiguous()
    if x._exact:
        geom = geom.with_exact_input(True)
    rows = geom.n * geom.oh * geom.ow
    y = _new((1, 1, rows, geom.cout), xd)
    ctx = _ctx(xd)
    ctx.conv_fprop(xd, w.data, None if b is None else b.data, y.reshape(rows, geom.cout), geom,
                   input_scale, relu)
    parents = (x, w) if b is None else (x, w, b)
    if not _needs(*parents):
        return _detached(y)
    out = Tensor(y, True, parents, "conv2d_relu" if relu else "conv2d")
    out._premask = bool(relu)
    # The data gradient's stacked sub-kernels depend on the weights alone:
    # prepared now on a side lane, beside the rest of the forward, instead of
    # on the backward's critical path.
    wt, wt_ready = None, None
    wt_bytes = ctx.conv_dgrad_weights_bytes(geom) if x.requires_grad and ctx.concurrent else 0
    if wt_bytes:
        wt = torch.empty(wt_bytes // 4, dtype=torch.float32, device=xd.device)
        with ctx.side(PREP_LANE) as s:
            w.data.record_stream(s)
            wt.record_stream(s)
            ctx.conv_dgrad_weights(w.data, wt, geom)
            wt_ready = torch.cuda.Event()
            wt_ready.record(s)

    def _backward(grad):
        g = grad.reshape(rows, geom.cout)
        if not g.is_contiguous():
            g = g.contiguous()
        wb = w.requires_grad
        bb = b is not None and b.requires_grad
        if wb or bb:
            if wb:
                dw, accw = w._grad_slot()
            else:
                dw, accw = torch.empty_like(w.data), False
            if bb:
                db, accb = b._grad_slot()
            else:
                db, accb = None, False
            receivers = [t for t, want in ((w, wb), (b, bb)) if want]
            _weight_grad(ctx, receivers, (xd, g, dw, db),
                         lambda: ctx.conv_wgrad(xd, g, dw, None if db is None else db.reshape(-1),
                                                geom, input_scale, accw, accb))
            if wb:
                w._set_grad(dw)
            if bb:
                b._set_grad(db)
        if x.requires_grad:
            if not needs_input_grad:
                raise RuntimeError(
                    "conv2d: this layer was built with needs_input_grad=False, "
                    "so it has no dX path, but its input requires a gradient. "
                    "Rebuild the layer with needs_input_grad=True, or detach "
                    "the activation it is given."
                )
            buf, acc = x._grad_slot()
            mask = xd if x._premask else None
            if wt is not None:
                torch.cuda.current_stream(xd.device).wait_event(wt_ready)
                ctx.conv_dgrad_prepared(g, wt, mask, buf.reshape(-1, geom.c), geom, acc)
            else:
                ctx.conv_dgrad(g, w.data, mask, buf.reshape(-1, geom.c), geom, acc)
            x._set_grad(buf)

    out._backward = _backward
    return out


# --------------------------------------------------------------------------
# shape (ttrl/engine/ops/shape.py)
# --------------------------------------------------------------------------

def reshape(a: Tensor, shape) -> Tensor:
    shape = tuple(int(d) for d in shape)
    in_shape = tuple(int(d) for d in a.shape)
    src = a.data if a.data.is_contiguous() else a.data.contiguous()
    y = src.reshape(shape)
    if not _needs(a):
        out = _detached(y)
        out._premask = a._premask
        return out
    out = Tensor(y, True, (a,), "reshape")
    out._premask = a._premask

    def _backward(grad):
        if a.requires_grad:
            a._accumulate(grad.reshape(in_shape), premasked=out._premask)

    out._backward = _backward
    return out


def concat(tensors, dim: int = -1) -> Tensor:
    tensors = tuple(tensors)
    if not tensors:
        raise ValueError("concat needs at least one tensor")
    rank = len(tensors[0].shape)
    axis = dim if dim >= 0 else dim + rank
    for t in tensors:
        if len(t.shape) != rank:
            raise ValueError(
                f"concat operands must share a rank, got {[t.shape for t in tensors]}"
            )
    shape = list(tensors[0].shape)
    shape[axis] = sum(int(t.shape[axis]) for t in tensors)
    y = _new(tuple(shape), tensors[0].data)
    ctx = _ctx(y)
    offset = 0
    extents = []
    for t in tensors:
        e = int(t.shape[axis])
        ctx.copy_strided(y.narrow(axis, offset, e), t.data)
        extents.append(e)
        offset += e
    if not _needs(*tensors):
        return _detached(y)
    out = Tensor(y, True, tensors, "concat")

    def _backward(grad):
        off = 0
        for operand, extent in zip(tensors, extents):
            if operand.requires_grad:
                piece = _new(operand.shape, grad)
                ctx.copy_strided(piece, grad.narrow(axis, off, extent))
                operand._accumulate(piece)
            off += extent

    out._backward = _backward
    return out


def split(a: Tensor, sizes, dim: int = -1) -> tuple:
    sizes = tuple(int(s) for s in sizes)
    rank = len(a.shape)
    axis = dim if dim >= 0 else dim + rank
    if not 0 <= axis < rank:
        raise ValueError(
            f"split got dim={dim} for a rank-{rank} tensor of shape "
            f"{tuple(a.shape)}; dim must index an existing axis."
        )
    extent = int(a.shape[axis])
    if any(s <= 0 for s in sizes) or sum(sizes) != extent:
        raise ValueError(
            f"split sizes {sizes} must be positive and sum to {extent}, the "
            f"extent of axis {axis} in shape {tuple(a.shape)}; got sum "
            f"{sum(sizes)}."
        )
    ctx = _ctx(a.data)
    pieces = []
    offset = 0
    for size in sizes:
        shape = list(a.shape)
        shape[axis] = size
        y = _new(tuple(shape), a.data)
        ctx.copy_strided(y, a.data.narrow(axis, offset, size))
        if not _needs(a):
            pieces.append(_detached(y))
        else:
            out = Tensor(y, True, (a,), "split")
            out._backward = _split_backward(a, axis, offset, size)
            pieces.append(out)
        offset += size
    return tuple(pieces)


def _split_backward(a: Tensor, axis: int, offset: int, size: int):
    def _backward(grad):
        if not a.requires_grad:
            return
        full = _new(a.shape, grad)
        ctx = _ctx(grad)
        ctx.ew("fill", None, None, full, 0.0)
        ctx.copy_strided(full.narrow(axis, offset, size), grad)
        a._accumulate(full)

    return _backward


# --------------------------------------------------------------------------
# functional (ttrl/engine/ops/functional.py)
# --------------------------------------------------------------------------

_LANE_CACHE: dict = {}


def apply_done_mask(value: Tensor, done: Tensor) -> Tensor:
    """value * (1 - done)."""
    return mul(value, sub(1.0, done))


masks = apply_done_mask


def huber(pred: Tensor, target: Tensor, delta: float = 1.0) -> Tensor:
    absdiff = abs_(sub(pred, target))
    quad = minimum(absdiff, delta)
    lin = sub(absdiff, quad)
    return add(mul(mul(quad, quad), 0.5), mul(lin, delta))


def _lane_numbers(batch: int, num_classes: int, device) -> Tensor:
    key = (str(device), int(batch), int(num_classes))
    lanes = _LANE_CACHE.get(key)
    if lanes is None:
        rows = np.tile(np.arange(num_classes, dtype=np.float32), (batch, 1))
        lanes = Tensor.from_numpy(rows, device)
        _LANE_CACHE[key] = lanes
    return lanes


def purge_lane_caches(device) -> None:
    dev = str(device)
    for key in [k for k in _LANE_CACHE if k[0] == dev]:
        del _LANE_CACHE[key]


def one_hot_host(indices, num_classes: int, device, dtype=None) -> Tensor:
    idx = np.asarray(indices).reshape(-1).astype(np.int64)
    batch = idx.shape[0]
    onehot = np.zeros((batch, num_classes), dtype=np.float32)
    onehot[np.arange(batch), idx] = 1.0
    return Tensor.from_numpy(onehot, device)


def one_hot_device(indices: Tensor, num_classes: int) -> Tensor:
    """(B,1) integer-valued fp32 ids -> (B, num_classes), on device."""
    lanes = _lane_numbers(int(indices.shape[0]), num_classes, indices.device)
    return Tensor(_ew("eq", lanes.data, indices.data), requires_grad=False)


def gather_onehot(values: Tensor, onehot: Tensor) -> Tensor:
    return sum_dim(mul(values, onehot), dim=-1, keepdim=True)


def one_hot_gather(values: Tensor, indices, num_classes: int) -> Tensor:
    if isinstance(indices, Tensor):
        batch = int(indices.shape[0])
        onehot = one_hot_device(indices, num_classes)
    else:
        idx = np.asarray(indices).reshape(-1)
        batch = int(idx.shape[0])
        onehot = one_hot_host(idx, num_classes, values.device)
    if int(values.shape[0]) != batch:
        raise ValueError(
            f"one_hot_gather: values has batch {values.shape[0]}, indices has {batch}"
        )
    return gather_onehot(values, onehot)


def log_softmax(x: Tensor, dim: int = -1) -> Tensor:
    shifted = sub(x, max_dim_detached(x, dim=dim, keepdim=True))
    sum_exp = sum_dim(exp(shifted), dim=dim, keepdim=True)
    return sub(shifted, log(sum_exp))


def entropy(logits: Tensor, dim: int = -1) -> Tensor:
    logp = log_softmax(logits, dim=dim)
    return mul(sum_dim(mul(exp(logp), logp), dim=dim, keepdim=True), -1.0)


def non_finite_check(tensor) -> bool:
    raw = tensor.data if isinstance(tensor, Tensor) else tensor
    x = raw.contiguous()
    bad = _new(x.shape, x)
    # x - x is 0 for finite values and NaN otherwise; eqz turns that into 1/0.
    _ctx(x).ew("sub", x, x, bad)
    finite = _new(x.shape, x)
    _ctx(x).ew("eqz", bad, None, finite)
    total = _new((1,), x)
    _ctx(x).reduce(_lib.RED_SUM, finite, total, 1, x.numel(), 1)
    return bool(float(total.item()) < x.numel())


# --------------------------------------------------------------------------
# fused loss heads
# --------------------------------------------------------------------------

def _flat(t):
    if t is None:
        return None
    d = t.data if isinstance(t, Tensor) else t
    return d.reshape(-1) if d.is_contiguous() else d.contiguous().reshape(-1)


def _scaled_into_grad(node, grad, pre, target: Tensor):
    """Accumulate `pre` (d node / d target, computed in the forward kernel)
    into target's gradient, scaled by the upstream gradient unless this node
    is the root of the running backward() (whose seed is exactly 1)."""
    if node is not backward_root():
        scaled = _new(pre.shape, pre)
        _ctx(pre).ew("mul", pre, grad.reshape((1,) * pre.dim()), scaled)
        pre = scaled
    target._accumulate(pre)


def dqn_td_huber(q: Tensor, q_sel: Tensor, q_tgt: Tensor, onehot: Tensor, rewards: Tensor,
                 dones: Tensor, discounts: Tensor, *, delta: float = 1.0, next_mask=None,
                 is_weights=None, want_td_abs: bool = False):
    """The DQN loss head of ttrl/algos/dqn/losses.py:95-128 as one kernel.

    -> (loss (1,1), mean_q (1,1), td_abs (B,1) or None). `loss` is
    differentiable in `q` only; the bootstrap target comes from `q_sel`
    (argmax) and `q_tgt` (value), which carry no gradient, as in the
    reference's no_grad block.
    """
    b, a = q.shape
    dev = q.data
    loss = _new((1, 1), dev)
    mean_q = _new((1, 1), dev)
    td_abs = _new((b, 1), dev) if want_td_abs else None
    dq = _new((b, a), dev)
    _ctx(dev).dqn_loss(q.data, q_sel.data, q_tgt.data, onehot.data, _flat(rewards),
                       _flat(dones), _flat(discounts),
                       None if next_mask is None else next_mask.data,
                       _flat(is_weights), loss, mean_q, td_abs, dq, delta)
    mean_q_t = Tensor(mean_q, requires_grad=False)
    td_t = Tensor(td_abs, requires_grad=False) if td_abs is not None else None
    if not _needs(q):
        return _detached(loss), mean_q_t, td_t
    out = Tensor(loss, True, (q,), "dqn_td_huber")

    def _backward(grad):
        if q.requires_grad:
            _scaled_into_grad(out, grad, dq, q)

    out._backward = _backward
    return out, mean_q_t, td_t


def ppo_objective(logits: Tensor, value: Tensor, actions, old_logp, advantages, returns,
                  old_values, *, clip_eps: float, value_clip_eps: float, value_coef: float,
                  entropy_coef: float, valid=None):
    """PPO's objective (ttrl/algos/ppo/loss.py:42-83) as one kernel.

    `actions` is an int32 device tensor [B]; the per-sample fields are
    device tensors [B] (or [B,1]). -> (loss, parts, new_logp) with parts =
    {policy_loss, value_loss, entropy}, all device tensors.
    """
    b, a = logits.shape
    dev = logits.data
    metrics = _new((4,), dev)
    new_logp = _new((b, 1), dev)
    dlogits = _new((b, a), dev)
    dvalue = _new(tuple(value.shape), dev)
    acts = actions.data if isinstance(actions, Tensor) else actions
    _ctx(dev).ppo_loss(logits.data, _flat(value), acts.reshape(-1), _flat(old_logp),
                       _flat(advantages), _flat(returns), _flat(old_values), _flat(valid),
                       metrics, new_logp, dlogits, dvalue.reshape(-1), clip_eps,
                       value_clip_eps, value_coef, entropy_coef)
    parts = {
        "policy_loss": Tensor(metrics[1:2].reshape(1, 1), requires_grad=False),
        "value_loss": Tensor(metrics[2:3].reshape(1, 1), requires_grad=False),
        "entropy": Tensor(metrics[3:4].reshape(1, 1), requires_grad=False),
    }
    loss_data = metrics[0:1].reshape(1, 1)
    nl = Tensor(new_logp, requires_grad=False)
    if not _needs(logits, value):
        return _detached(loss_data), parts, nl
    out = Tensor(loss_data, True, (logits, value), "ppo_objective")

    def _backward(grad):
        if logits.requires_grad:
            _scaled_into_grad(out, grad, dlogits, logits)
        if value.requires_grad:
            _scaled_into_grad(out, grad, dvalue, value)

    out._backward = _backward
    return out, parts, nl


# --------------------------------------------------------------------------
# SAC heads
# --------------------------------------------------------------------------

def _raw_data(t):
    if t is None:
        return None
    d = t.data if isinstance(t, Tensor) else t
    return d if d.is_contiguous() else d.contiguous()


def sac_sample(mean: Tensor, log_std_raw: Tensor, noise, scale, centre, log_det: float, *,
               log_std_min: float, log_std_max: float, obs=None, pack=None):
    """The squashed-Gaussian sample of ttrl/algos/sac/policy.py:30-40 as one
    kernel, from the policy's raw outputs: the log-std clamp of the Gaussian
    head, u = mean + exp(log_std) * noise, the log-density of
    ttrl/algos/gaussian.py:55-90 and the env action tanh(u) * scale + centre.

    The action is written after `obs`'s columns, as the critic input
    concat(obs, action); `pack` = (obs', action') also writes concat(obs',
    action') in the same launch. -> (joint (B, obs + D), logp (B, 1), packed
    joint or None). joint and logp are differentiable in mean and
    log_std_raw; their backward is one kernel, run once both gradients are
    in."""
    b, d = int(mean.shape[0]), int(mean.shape[1])
    o = 0 if obs is None else int(obs.shape[1])
    dev = mean.data
    ctx = _ctx(dev)
    joint = _new((b, o + d), dev)
    logp = _new((b, 1), dev)
    packed = _new((b, o + d), dev) if pack is not None else None
    md, rd, nd = _raw_data(mean), _raw_data(log_std_raw), _raw_data(noise)
    lo, hi = float(log_std_min), float(log_std_max)
    ctx.sac_sample(md, rd, nd, scale, centre, _raw_data(obs), joint, logp, lo, hi, log_det,
                   pack=None if pack is None else (_raw_data(pack[0]), _raw_data(pack[1]), packed))
    packed_t = None if packed is None else Tensor(packed, requires_grad=False)
    if not _needs(mean, log_std_raw):
        return _detached(joint), _detached(logp), packed_t
    out = Tensor(joint, True, (mean, log_std_raw), "sac_sample")
    # logp is a consumer of the joint node, so the joint node's backward runs
    # after logp's: by then both gradients are known.
    lp = Tensor(logp, True, (out,), "sac_logp")
    pending = {}

    def _logp_backward(grad):
        pending["logp"] = grad if grad.is_contiguous() else grad.contiguous()
        if out.grad is None:
            # No action gradient has arrived yet: start the action's gradient
            # at zero for any later consumer to accumulate into, so that the
            # joint node still runs.
            zero = _new(joint.shape, joint)
            ctx.ew("fill", None, None, zero, 0.0)
            out._set_grad(zero)

    def _backward(grad):
        if grad.stride(-1) != 1:
            grad = grad.contiguous()
        if mean.requires_grad:
            mbuf, macc = mean._grad_slot()
        else:
            mbuf, macc = _new(mean.shape, dev), False
        if log_std_raw.requires_grad:
            rbuf, racc = log_std_raw._grad_slot()
        else:
            rbuf, racc = _new(log_std_raw.shape, dev), False
        ctx.sac_sample_backward(md, rd, nd, scale, grad.narrow(1, o, d), grad.stride(0),
                                pending.get("logp"), mbuf, rbuf, macc, racc, lo, hi)
        if mean.requires_grad:
            mean._set_grad(mbuf)
        if log_std_raw.requires_grad:
            log_std_raw._set_grad(rbuf)

    lp._backward = _logp_backward
    out._backward = _backward
    return out, lp, packed_t


def sac_critic_loss(qs, q_targets, next_logp, log_alpha, rewards, dones, discounts, *,
                    weights=None, want_td_abs: bool = False):
    """The twin-critic loss of ttrl/algos/sac/losses.py:46-76 as one kernel,
    from the online critics' Q(s, a) and the targets' Q(s', a') with the
    next log-density (the no_grad target side). alpha = exp(log_alpha) is
    read on the device. -> (loss (1,1), alpha (1,1), target (B,1), |TD| mean
    over critics (B,1) or None); loss is differentiable in every q."""
    qs, q_targets = list(qs), list(q_targets)
    if len(qs) != len(q_targets):
        raise ValueError(f"sac_critic_loss: {len(qs)} critics but {len(q_targets)} targets")
    b = int(qs[0].shape[0])
    dev = qs[0].data
    loss, alpha = _new((1, 1), dev), _new((1, 1), dev)
    target = _new((b, 1), dev)
    td_abs = _new((b, 1), dev) if want_td_abs else None
    dqs = [_new((b, 1), dev) for _ in qs]
    _ctx(dev).sac_critic_loss([_flat(q) for q in qs], [_flat(t) for t in q_targets],
                              _flat(next_logp), _flat(log_alpha), _flat(rewards), _flat(dones),
                              _flat(discounts), _flat(weights), loss, alpha, target, dqs, td_abs)
    alpha_t = Tensor(alpha, requires_grad=False)
    target_t = Tensor(target, requires_grad=False)
    td_t = None if td_abs is None else Tensor(td_abs, requires_grad=False)
    if not _needs(*qs):
        return _detached(loss), alpha_t, target_t, td_t
    out = Tensor(loss, True, tuple(qs), "sac_critic_loss")

    def _backward(grad):
        for q, dq in zip(qs, dqs):
            if q.requires_grad:
                _scaled_into_grad(out, grad, dq.reshape(q.shape), q)

    out._backward = _backward
    return out, alpha_t, target_t, td_t


def sac_actor_loss(qs, logp: Tensor, log_alpha: Tensor, target_entropy: float, *,
                   learn_alpha: bool = True):
    """The actor loss mean(alpha * logp - min_i Q_i(s, a~pi)) of
    ttrl/algos/sac/losses.py:79-84 and the temperature loss of :87-95, one
    kernel. -> (actor loss (1,1) differentiable in every q and in logp,
    temperature loss (1,1) differentiable in log_alpha, or None)."""
    qs = list(qs)
    b = int(qs[0].shape[0])
    dev = qs[0].data
    loss = _new((1, 1), dev)
    dqs = [_new((b, 1), dev) for _ in qs]
    d_logp = _new((b, 1), dev)
    dual = _new((1, 1), dev) if learn_alpha else None
    d_log_alpha = _new(tuple(log_alpha.shape), dev) if learn_alpha else None
    _ctx(dev).sac_actor_loss([_flat(q) for q in qs], _flat(logp), _flat(log_alpha),
                             float(target_entropy), loss, dqs, d_logp, dual, d_log_alpha)
    dual_t = None
    if learn_alpha:
        if _needs(log_alpha):
            dual_t = Tensor(dual, True, (log_alpha,), "sac_alpha_loss")

            def _dual_backward(grad):
                _scaled_into_grad(dual_t, grad, d_log_alpha, log_alpha)

            dual_t._backward = _dual_backward
        else:
            dual_t = _detached(dual)
    parents = (*qs, logp)
    if not _needs(*parents):
        return _detached(loss), dual_t
    out = Tensor(loss, True, parents, "sac_actor_loss")

    def _backward(grad):
        for q, dq in zip(qs, dqs):
            if q.requires_grad:
                _scaled_into_grad(out, grad, dq.reshape(q.shape), q)
        if logp.requires_grad:
            _scaled_into_grad(out, grad, d_logp, logp)

    out._backward = _backward
    return out, dual_t
