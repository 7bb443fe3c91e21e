"""Conv2d / Linear / Adam arithmetic of the reference, restated in numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). Functions work in the
dtype of their inputs, so the same code serves as the fp32 CPU baseline and
as the float64 gradient reference.
"""

from __future__ import annotations

import math

import numpy as np

__all__ = [
    "conv_out", "conv2d_nhwc", "conv2d_dgrad", "conv2d_wgrad", "oihw_to_krsc", "krsc_to_oihw",
    "linear", "linear_backward", "adam_fused_scalars", "adam_step_sv", "relu",
]


def conv_out(size: int, kernel: int, stride: int, padding: int) -> int:
    """`(size + 2*padding - kernel) // stride + 1`, refusing ragged strides.

    ttrl/engine/conv/geometry.py:94-124 (conv_out_size).
    """
    span = size + 2 * padding - kernel
    if span < 0 or span % stride:
        raise ValueError(f"ragged or empty conv geometry: size={size} k={kernel} "
                         f"s={stride} p={padding}")
    return span // stride + 1


def oihw_to_krsc(w):
    """Logical OIHW -> the [Cout][KH][KW][Cin] order the GEMM walks."""
    return np.ascontiguousarray(np.asarray(w).transpose(0, 2, 3, 1))


def krsc_to_oihw(w):
    return np.ascontiguousarray(np.asarray(w).transpose(0, 3, 1, 2))


def relu(x):
    return np.maximum(x, np.asarray(0, dtype=np.asarray(x).dtype))


def _windows(x, kernel: int, stride: int, padding: int):
    """Strided kernel windows of an NHWC batch: [N, OH, OW, C, KH, KW].

    ttrl/deploy/conv.py:31-50 builds the same view with
    sliding_window_view over the (H, W) axes.
    """
    if padding:
        x = np.pad(x, ((0, 0), (padding, padding), (padding, padding), (0, 0)))
    win = np.lib.stride_tricks.sliding_window_view(x, (kernel, kernel), axis=(1, 2))
    return win[:, ::stride, ::stride]


def conv2d_nhwc(x, w_oihw, bias=None, *, stride=1, padding=0, input_scale=1.0,
                apply_relu=False):
    """y = conv(input_scale * x, W) + b on an NHWC batch [N, H, W, C].

    Forward of ttrl/engine/conv/forward.py:185-205 with the input-scale fold
    of :160-182 (the reference multiplies W by the scale; conv is linear in
    its input so this equals scaling the product). Computed as one matmul
    over strided windows, as ttrl/deploy/conv.py:31-50 does.
    Returns [N, OH, OW, Cout].
    """
    x = np.asarray(x)
    w = np.asarray(w_oihw)
    cout, _, k, _ = w.shape
    win = _windows(x, k, stride, padding)
    n, oh, ow = win.shape[:3]
    cols = win.reshape(n * oh * ow, -1)
    scaled = w if input_scale == 1.0 else w * np.asarray(input_scale, w.dtype)
    out = cols @ scaled.reshape(cout, -1).T
    if bias is not None:
        out = out + np.asarray(bias).reshape(1, cout)
    if apply_relu:
        out = relu(out)
    return out.reshape(n, oh, ow, cout)


def conv2d_wgrad(x, dy, kernel: int, *, stride=1, padding=0, input_scale=1.0):
    """dW[k,c,p,q] = input_scale * sum_{n,i,j} dY[n,i,j,k] X[n, i*s+p, j*s+q, c].

    ttrl/engine/conv/backward.py:45-78 (one matmul over k*k strided
    slices), with the input-scale factor of :29-31 and :78. Returns OIHW.
    """
    x = np.asarray(x)
    dy = np.asarray(dy)
    win = _windows(x, kernel, stride, padding)  # [N, OH, OW, C, KH, KW]
    n, oh, ow, c = win.shape[:4]
    cout = dy.shape[-1]
    cols = win.reshape(n * oh * ow, c * kernel * kernel)
    dw = dy.reshape(n * oh * ow, cout).T @ cols
    if input_scale != 1.0:
        dw = dw * np.asarray(input_scale, dw.dtype)
    return dw.reshape(cout, c, kernel, kernel)


def conv2d_dgrad(dy, w_oihw, in_shape, *, stride=1, padding=0, input_scale=1.0):
    """dX of the convolution (its adjoint, conv_transpose2d with the mirrored
    kernel), ttrl/engine/conv/backward.py:33-42. `in_shape` = (N, H, W, C).
    """
    dy = np.asarray(dy)
    w = np.asarray(w_oihw)
    if input_scale != 1.0:
        w = w * np.asarray(input_scale, w.dtype)
    n, h, wd, c = in_shape
    cout, _, k, _ = w.shape
    oh, ow = dy.shape[1], dy.shape[2]
    hp, wp = h + 2 * padding, wd + 2 * padding
    dxp = np.zeros((n, hp, wp, c), dtype=dy.dtype)
    # cols[m, (c, p, q)] = sum_k dY[m, k] W[k, c, p, q]; scatter-add back.
    cols = dy.reshape(n * oh * ow, cout) @ w.reshape(cout, -1)
    cols = cols.reshape(n, oh, ow, c, k, k)
    for p in range(k):
        for q in range(k):
            dxp[:, p:p + stride * (oh - 1) + 1:stride, q:q + stride * (ow - 1) + 1:stride, :] += \
                cols[:, :, :, :, p, q]
    return dxp[:, padding:padding + h, padding:padding + wd, :]


def linear(x, w, b=None):
    """y = x @ W + b with W stored (in, out). ttrl/engine/layers.py:57-61."""
    y = np.asarray(x) @ np.asarray(w)
    if b is not None:
        y = y + np.asarray(b).reshape(1, -1)
    return y


def linear_backward(x, w, dy):
    """(dx, dW, db) of y = x @ W + b: dx = dy W^T, dW = x^T dy, db = sum
    over rows (ttrl/engine/ops/matmul.py:72-84, broadcast.py:11-30)."""
    x = np.asarray(x)
    dy = np.asarray(dy)
    return dy @ np.asarray(w).T, x.T @ dy, dy.sum(axis=0, keepdims=True)


def adam_fused_scalars(lr, b1, b2, eps, t):
    """(alpha_t, eps_t) of ttrl/engine/optim/scalars.py:13-27."""
    if t < 1:
        raise ValueError(f"t must be >= 1, got {t}")
    bc1 = 1 - b1 ** t
    bc2 = 1 - b2 ** t
    c = math.sqrt((1 - b2) / bc2)
    return lr * (1 - b1) / bc1 / c, eps / c


def adam_step_sv(p, g, S, V, t, *, lr, b1=0.9, b2=0.999, eps=1e-8, weight_decay=0.0,
                 grad_scale=None):
    """One Adam update in the reference's stored-S/V form, in the op order of
    ttrl/engine/optim/adam.py:93-134. Returns new (p, S, V); inputs untouched.
    fp32 arrays give fp32 arithmetic (the reference's device precision).
    """
    dt = np.asarray(p).dtype
    g = np.asarray(g, dt)
    if grad_scale is not None:
        g = (g * np.asarray(grad_scale, dt)).astype(dt)
    if weight_decay:
        g = (g + np.asarray(weight_decay, dt) * p).astype(dt)
    alpha_t, eps_t = adam_fused_scalars(lr, b1, b2, eps, t)
    s = g * g
    V = (s + np.asarray(b2, dt) * V).astype(dt)
    S = (g + np.asarray(b1, dt) * S).astype(dt)
    s = np.sqrt(V)
    s = s + np.asarray(eps_t, dt)
    s = S / s
    s = s * np.asarray(alpha_t, dt)
    return (p - s).astype(dt), S, V
