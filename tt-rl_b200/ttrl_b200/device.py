"""Per-device runtime state and typed wrappers over the C ABI.

PyTorch supplies device memory and the current CUDA stream; every
computation is a call into ``libttrl_b200.so``. A ``DeviceContext`` owns the
pieces the kernels share on one GPU: the split-K / col2im workspace, the
device status word bounded waits report into, and the one-time
``ttrl_init``.

Address stability: a workspace, once handed to a kernel, is never freed,
because a captured CUDA graph keeps using the pointer it recorded. Growing
the workspace allocates a larger buffer and retires the old one to a list
that lives as long as the context.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from ttrl_b200 import _lib
from ttrl_b200._lib import check, lib

__all__ = ["DeviceContext", "context", "conv_geom", "PRECISION"]

#: Precision of every tensor-core contraction. Split-TF32 reproduces fp32
#: products to ~1e-6 relative, which is what lets gradients match the
#: fp32 reference well inside the 1e-3 budget.
PRECISION = _lib.PREC_TF32X3

_CONTEXTS: dict[int, "DeviceContext"] = {}


def _ptr(t) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("ttrl_b200 kernels take CUDA tensors; got a CPU tensor")
    return t.data_ptr()


def _f32(t, name: str):
    if t is not None and (t.dtype != torch.float32 or not t.is_contiguous()):
        raise ValueError(f"{name} must be a contiguous float32 CUDA tensor, got "
                         f"{t.dtype} contiguous={t.is_contiguous()}")
    return t


@dataclass(frozen=True)
class Geom:
    n: int
    h: int
    w: int
    c: int
    cout: int
    kh: int
    kw: int
    stride: int
    pad: int

    @property
    def oh(self) -> int:
        return (self.h + 2 * self.pad - self.kh) // self.stride + 1

    @property
    def ow(self) -> int:
        return (self.w + 2 * self.pad - self.kw) // self.stride + 1

    def c_struct(self) -> _lib.ConvGeom:
        return _lib.ConvGeom(self.n, self.h, self.w, self.c, self.cout, self.kh, self.kw,
                             self.stride, self.pad, self.oh, self.ow)


def conv_geom(n, h, w, c, cout, kh, kw=None, stride=1, pad=0) -> Geom:
    return Geom(int(n), int(h), int(w), int(c), int(cout), int(kh), int(kw or kh),
                int(stride), int(pad))


class DeviceContext:
    """Workspace, status word and stream access for one CUDA device."""

    def __init__(self, index: int):
        self.index = int(index)
        self.device = torch.device("cuda", self.index)
        with torch.cuda.device(self.device):
            check(lib().ttrl_init(self.index), "ttrl_init")
            self.status = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._ws = None
        self._ws_bytes = 0
        self._retired: list = []
        self.reserve(64 << 20)

    # -- workspace -------------------------------------------------------

    def reserve(self, nbytes: int) -> None:
        """Make the shared workspace at least `nbytes` long. Never shrinks,
        never frees a buffer a graph may have recorded."""
        if nbytes <= self._ws_bytes:
            return
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(
                f"ttrl_b200: a kernel needs {nbytes} bytes of workspace but only "
                f"{self._ws_bytes} are reserved, and the stream is being captured, "
                "where allocating would invalidate the graph. Run the step once "
                "eagerly before capture so the workspace is sized first."
            )
        size = max(nbytes, 2 * self._ws_bytes)
        size = (size + (1 << 20) - 1) & ~((1 << 20) - 1)
        buf = torch.empty(size, dtype=torch.uint8, device=self.device)
        if self._ws is not None:
            self._retired.append(self._ws)
        self._ws = buf
        self._ws_bytes = size

    def workspace(self, nbytes: int = 0):
        self.reserve(nbytes)
        return self._ws.data_ptr(), self._ws_bytes

    @property
    def stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def status_ptr(self) -> int:
        return self.status.data_ptr()

    def check_status(self) -> None:
        """Raise if a kernel recorded a device-side error (host sync)."""
        code = int(self.status[0].item())
        if code:
            self.status.zero_()
            raise RuntimeError(f"ttrl_b200: a kernel on cuda:{self.index} reported "
                               f"device status {code} (a bounded wait gave up)")

    # -- linear ----------------------------------------------------------

    def linear_fwd(self, x, w, b, y, relu: bool, precision: int = PRECISION) -> None:
        m, k = x.shape[-2], x.shape[-1]
        n = w.shape[1]
        ws, wsb = self.workspace()
        check(lib().ttrl_linear_fwd(_ptr(_f32(x, "x")), _ptr(_f32(w, "w")),
                                    _ptr(_f32(b, "b")), _ptr(_f32(y, "y")), m, k, n,
                                    int(relu), precision, ws, wsb, self.status_ptr(),
                                    self.stream), "ttrl_linear_fwd")

    def linear_dgrad(self, g, w, mask, dx, accumulate: bool,
                     precision: int = PRECISION) -> None:
        m, n = g.shape[-2], g.shape[-1]
        k = w.shape[0]
        ws, wsb = self.workspace()
        check(lib().ttrl_linear_dgrad(_ptr(_f32(g, "g")), _ptr(_f32(w, "w")),
                                      _ptr(_f32(mask, "mask")), _ptr(_f32(dx, "dx")), m, k, n,
                                      int(accumulate), precision, ws, wsb, self.status_ptr(),
                                      self.stream), "ttrl_linear_dgrad")

    def linear_wgrad(self, x, g, dw, db, accumulate: bool, accumulate_db: bool,
                     precision: int = PRECISION) -> None:
        m, k = x.shape[-2], x.shape[-1]
        n = g.shape[-1]
        desc = _lib.GemmDesc()
        desc.m, desc.n, desc.k, desc.precision = k + (1 if db is not None else 0), n, m, precision
        need = lib().ttrl_gemm_workspace_bytes(ctypes.byref(desc))
        ws, wsb = self.workspace(need)
        check(lib().ttrl_linear_wgrad(_ptr(_f32(x, "x")), _ptr(_f32(g, "g")),
                                      _ptr(_f32(dw, "dw")), _ptr(_f32(db, "db")), m, k, n,
                                      int(accumulate), int(accumulate_db), precision, ws, wsb,
                                      self.status_ptr(), self.stream), "ttrl_linear_wgrad")

    # -- conv ------------------------------------------------------------

    def conv_fprop(self, x, w, b, y, geom: Geom, alpha: float, relu: bool,
                   precision: int = PRECISION) -> None:
        g = geom.c_struct()
        ws, wsb = self.workspace()
        check(lib().ttrl_conv_fprop(_ptr(_f32(x, "x")), _ptr(_f32(w, "w")), _ptr(_f32(b, "b")),
                                    _ptr(_f32(y, "y")), ctypes.byref(g), float(alpha),
                                    int(relu), precision, ws, wsb, self.status_ptr(),
                                    self.stream), "ttrl_conv_fprop")

    def conv_dgrad(self, dy, w, mask, dx, geom: Geom, accumulate: bool,
                   precision: int = PRECISION) -> None:
        g = geom.c_struct()
        need = lib().ttrl_conv_dgrad_workspace_bytes(ctypes.byref(g))
        ws, wsb = self.workspace(need)
        check(lib().ttrl_conv_dgrad(_ptr(_f32(dy, "dy")), _ptr(_f32(w, "w")),
                                    _ptr(_f32(mask, "mask")), _ptr(_f32(dx, "dx")),
                                    ctypes.byref(g), int(accumulate), precision, ws, wsb,
                                    self.status_ptr(), self.stream), "ttrl_conv_dgrad")

    def conv_wgrad(self, x, dy, dw, db, geom: Geom, alpha: float, accumulate: bool,
                   accumulate_db: bool, precision: int = PRECISION) -> None:
        g = geom.c_struct()
        need = lib().ttrl_conv_wgrad_workspace_bytes(ctypes.byref(g))
        ws, wsb = self.workspace(need)
        check(lib().ttrl_conv_wgrad(_ptr(_f32(x, "x")), _ptr(_f32(dy, "dy")),
                                    _ptr(_f32(dw, "dw")), _ptr(_f32(db, "db")), ctypes.byref(g),
                                    float(alpha), int(accumulate), int(accumulate_db),
                                    precision, ws, wsb, self.status_ptr(), self.stream),
              "ttrl_conv_wgrad")

    def u8_to_f32(self, frames, index, out, scale: float = 1.0) -> None:
        if frames.dtype != torch.uint8 or frames.dim() != 4:
            raise ValueError("frames must be a uint8 [N, C, H, W] CUDA tensor")
        n = frames.shape[0]
        if index is not None:
            if index.dtype != torch.int32:
                raise ValueError("index must be int32")
            n = index.shape[0]
        c, h, w = frames.shape[1], frames.shape[2], frames.shape[3]
        check(lib().ttrl_u8_nchw_to_f32_nhwc(_ptr(frames), _ptr(index), _ptr(_f32(out, "out")),
                                             n, c, h, w, float(scale), self.stream),
              "ttrl_u8_nchw_to_f32_nhwc")

    # -- optimizer -------------------------------------------------------

    def adam_step(self, tensors, steps, ticket, grad_scale, lr, b1, b2, eps, wd) -> None:
        """`tensors`: list of (param, grad, S, V, step_index)."""
        for start in range(0, len(tensors), 64):
            chunk = tensors[start:start + 64]
            arr = (_lib.AdamTensor * len(chunk))()
            for i, (p, g, s, v, idx) in enumerate(chunk):
                arr[i] = _lib.AdamTensor(_ptr(_f32(p, "param")), _ptr(_f32(g, "grad")),
                                         _ptr(_f32(s, "S")), _ptr(_f32(v, "V")), p.numel(),
                                         int(idx), 0)
            check(lib().ttrl_adam_step(arr, len(chunk), _ptr(steps), _ptr(ticket),
                                       _ptr(grad_scale), float(lr), float(b1), float(b2),
                                       float(eps), float(wd), self.stream), "ttrl_adam_step")

    def grad_sqnorm(self, grads, out, max_norm: float, workspace) -> None:
        if len(grads) > 64:
            raise ValueError("grad_sqnorm: more than 64 tensors per call")
        ptrs = (ctypes.c_void_p * len(grads))(*[_ptr(_f32(g, "grad")) for g in grads])
        numels = (ctypes.c_int64 * len(grads))(*[g.numel() for g in grads])
        need = lib().ttrl_grad_sqnorm_workspace_bytes(numels, len(grads))
        if workspace.numel() < need:
            raise ValueError(f"grad_sqnorm workspace needs {need} bytes")
        check(lib().ttrl_grad_sqnorm(ptrs, numels, len(grads), _ptr(out), float(max_norm),
                                     workspace.data_ptr(), workspace.numel(), self.stream),
              "ttrl_grad_sqnorm")

    @staticmethod
    def sqnorm_workspace_bytes(numels) -> int:
        arr = (ctypes.c_int64 * len(numels))(*numels)
        return int(lib().ttrl_grad_sqnorm_workspace_bytes(arr, len(numels)))


def context(device=None) -> DeviceContext:
    """The (lazily created) context of a CUDA device."""
    if device is None:
        index = torch.cuda.current_device()
    elif isinstance(device, DeviceContext):
        return device
    elif isinstance(device, int):
        index = device
    else:
        d = torch.device(device)
        if d.type != "cuda":
            raise ValueError(f"ttrl_b200 runs on CUDA devices only, got {device!r}")
        index = d.index if d.index is not None else torch.cuda.current_device()
    ctx = _CONTEXTS.get(index)
    if ctx is None:
        ctx = DeviceContext(index)
        _CONTEXTS[index] = ctx
    return ctx
