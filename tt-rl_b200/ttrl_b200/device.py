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

import contextlib
import ctypes
import os
from dataclasses import dataclass

import numpy as np
import torch

from ttrl_b200 import _lib
from ttrl_b200._lib import check, lib

__all__ = ["DeviceContext", "context", "conv_geom", "PRECISION", "SIDE_LANES", "WEIGHT_LANES",
           "PREP_LANE", "FORWARD_LANES"]

#: Side streams a context keeps (lanes 1..SIDE_LANES). Weight gradients are
#: dealt over lanes 1..WEIGHT_LANES; the last lane (PREP_LANE) carries the
#: short weight-only preparations a forward issues for its backward.
SIDE_LANES = 5
WEIGHT_LANES = 2
PREP_LANE = 3
#: Lanes for independent forward branches whose results the main chain waits
#: for (DQN's two no-grad forwards): created at the device's highest stream
#: priority, like a `critical_main` capture stream, so the weight-gradient
#: lanes (default priority) yield SMs to them.
FORWARD_LANES = (4, 5)

#: Precision of every tensor-core contraction. Split-TF32 (the default)
#: reproduces fp32 products to ~1e-6 relative, well inside the 1e-3 budget
#: for TF32 GEMM paths; TTRL_PRECISION=tf32 selects one TF32 pass (about
#: 1e-3 relative per product, half the tensor-core work).
PRECISION = (_lib.PREC_TF32 if os.environ.get("TTRL_PRECISION", "").lower() == "tf32"
             else _lib.PREC_TF32X3)

_CONTEXTS: dict[int, "DeviceContext"] = {}


class _NoProfile:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NO_PROFILE = _NoProfile()


class _Profile:
    """CUDA events around one library call on the launching stream."""

    def __init__(self, ctx, name, flops, call=None):
        self.ctx, self.name, self.flops, self.call = ctx, name, flops, call

    def __enter__(self):
        self.start = torch.cuda.Event(enable_timing=True)
        self.end = torch.cuda.Event(enable_timing=True)
        self.start.record(torch.cuda.current_stream(self.ctx.device))
        return self

    def __exit__(self, *exc):
        self.end.record(torch.cuda.current_stream(self.ctx.device))
        self.ctx.profile.append((self.name, self.flops, self.start, self.end, self.call))
        return False


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
    input_exact: bool = False  # input values exactly representable in tf32

    @property
    def oh(self) -> int:
        return (self.h + 2 * self.pad - self.kh) // self.stride + 1

    @property
    def ow(self) -> int:
        return (self.w + 2 * self.pad - self.kw) // self.stride + 1

    def c_struct(self) -> _lib.ConvGeom:
        return _lib.ConvGeom(self.n, self.h, self.w, self.c, self.cout, self.kh, self.kw,
                             self.stride, self.pad, self.oh, self.ow,
                             _lib.CONV_INPUT_EXACT if self.input_exact else 0)

    def with_exact_input(self, exact: bool) -> "Geom":
        from dataclasses import replace
        return replace(self, input_exact=bool(exact))


def _conv_flops(g: "Geom") -> int:
    return 2 * g.n * g.oh * g.ow * g.cout * g.kh * g.kw * g.c


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
        # Launch lanes: lane 0 is the caller's current stream, lanes 1.. are
        # side streams that run independent work concurrently (inside a
        # captured graph they become parallel branches). Each lane has its own
        # workspace, so concurrent GEMMs never share split-K scratch.
        self._lane = 0
        self._ws: dict = {}
        self._ws_bytes: dict = {}
        self._retired: list = []
        self._streams: dict = {}
        self._joins: set = set()
        self._weight_lanes: dict = {}
        # Weight-gradient GEMMs of leaf parameters run on the side lanes
        # during backward, beside the data-gradient chain.
        self.concurrent = True
        # Contraction precision of every GEMM this context launches (a call
        # may override it); set_precision changes it.
        self.precision = PRECISION
        # When a list, every GEMM-family call appends (name, flops, start, end,
        # call), `call` a closure that issues the same launch again.
        self.profile = None
        for lane in list(range(WEIGHT_LANES + 1)) + list(FORWARD_LANES):
            self.reserve(64 << 20, lane=lane)  # the preparation lane needs none up front

    def _timed(self, name: str, flops: int = 0, call=None):
        if self.profile is None or torch.cuda.is_current_stream_capturing():
            return _NO_PROFILE
        return _Profile(self, name, flops, call)

    def _call(self, name: str, flops: int, call) -> None:
        """Run one library call; when profiling, bracket it with events and
        keep `call` so that it can be issued again for a device timing."""
        with self._timed(name, flops, call):
            call()

    # -- workspace -------------------------------------------------------

    def reserve(self, nbytes: int, lane: int | None = None) -> None:
        """Make a lane's workspace at least `nbytes` long. Never shrinks, never
        frees a buffer a graph may have recorded."""
        lane = self._lane if lane is None else lane
        have = self._ws_bytes.get(lane, 0)
        if nbytes <= have:
            return
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(
                f"ttrl_b200: a kernel needs {nbytes} bytes of workspace but only "
                f"{have} are reserved, and the stream is being captured, "
                "where allocating would invalidate the graph. Run the step once "
                "eagerly before capture so the workspace is sized first."
            )
        size = max(nbytes, 2 * have)
        size = (size + (1 << 20) - 1) & ~((1 << 20) - 1)
        # zeroed: its first 64 KB hold split-K tile counters the kernels
        # expect at zero (and always leave at zero)
        buf = torch.zeros(size, dtype=torch.uint8, device=self.device)
        if lane in self._ws:
            self._retired.append(self._ws[lane])
        self._ws[lane] = buf
        self._ws_bytes[lane] = size

    def workspace(self, nbytes: int = 0):
        self.reserve(max(int(nbytes), 64 << 10))  # at least the split-K counters
        return self._ws[self._lane].data_ptr(), self._ws_bytes[self._lane]

    # -- lanes -----------------------------------------------------------

    def _side_stream(self, lane: int):
        if not 1 <= lane <= SIDE_LANES:
            raise ValueError(f"side lane must be in [1, {SIDE_LANES}], got {lane}")
        s = self._streams.get(lane)
        if s is None:
            if lane in FORWARD_LANES:
                _, highest = torch.cuda.Stream.priority_range()
                s = torch.cuda.Stream(self.device, priority=highest)
            else:
                s = torch.cuda.Stream(self.device)
            self._streams[lane] = s
        return s

    @contextlib.contextmanager
    def side(self, lane: int = 1):
        """Issue the enclosed launches on side lane `lane`: a stream ordered
        after everything issued so far on the current stream, with its own
        workspace. `join()` orders the current stream after it again. Tensors
        the side work reads or writes that may be freed before `join()` must
        be `record_stream`-ed to the yielded stream by the caller."""
        main = torch.cuda.current_stream(self.device)
        s = self._side_stream(lane)
        fork = torch.cuda.Event()
        fork.record(main)
        s.wait_event(fork)
        prev = self._lane
        self._lane = lane
        try:
            with torch.cuda.stream(s):
                yield s
        finally:
            self._lane = prev
            self._joins.add(lane)

    def weight_lane(self, param) -> int:
        """The side lane a parameter's weight gradients run on: lanes are
        dealt round-robin in the order parameters are first seen, and a
        parameter keeps its lane, so its gradient accumulates in order."""
        key = param.data_ptr()
        lane = self._weight_lanes.get(key)
        if lane is None:
            lane = self._weight_lanes[key] = 1 + len(self._weight_lanes) % WEIGHT_LANES
        return lane

    def join(self) -> None:
        """Order the current stream after all side-lane work issued so far."""
        if not self._joins:
            return
        main = torch.cuda.current_stream(self.device)
        for lane in sorted(self._joins):
            done = torch.cuda.Event()
            done.record(self._streams[lane])
            main.wait_event(done)
        self._joins.clear()

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

    def _prec(self, precision: int | None) -> int:
        return self.precision if precision is None else int(precision)

    def set_precision(self, name: str) -> None:
        """'tf32x3' (split-TF32, ~1e-6 relative) or 'tf32' (one pass, ~1e-3
        relative: the accuracy class of the reference's HiFi4 matmuls,
        ttrl/engine/ops/matmul.py:14-20). Affects launches recorded after it."""
        table = {"tf32x3": _lib.PREC_TF32X3, "tf32": _lib.PREC_TF32}
        if name not in table:
            raise ValueError(f"precision must be one of {sorted(table)}, got {name!r}")
        self.precision = table[name]

    def linear_fwd(self, x, w, b, y, relu: bool, precision: int | None = None) -> None:
        prec = self._prec(precision)
        m, k = x.shape[-2], x.shape[-1]
        n = w.shape[1]
        ws, wsb = self.workspace()
        self._call(f"linear_fwd[{m}x{k}x{n}]", 2 * m * k * n,
                   lambda: check(lib().ttrl_linear_fwd(_ptr(_f32(x, "x")), _ptr(_f32(w, "w")),
                                            _ptr(_f32(b, "b")), _ptr(_f32(y, "y")), m, k, n,
                                            int(relu), prec, ws, wsb, self.status_ptr(),
                                            self.stream), "ttrl_linear_fwd"))

    def linear_dgrad(self, g, w, mask, dx, accumulate: bool,
                     precision: int | None = None) -> None:
        prec = self._prec(precision)
        m, n = g.shape[-2], g.shape[-1]
        k = w.shape[0]
        ws, wsb = self.workspace()
        self._call(f"linear_dgrad[{m}x{k}x{n}]", 2 * m * k * n,
                   lambda: check(lib().ttrl_linear_dgrad(_ptr(_f32(g, "g")), _ptr(_f32(w, "w")),
                                              _ptr(_f32(mask, "mask")), _ptr(_f32(dx, "dx")), m, k, n,
                                              int(accumulate), prec, ws, wsb, self.status_ptr(),
                                              self.stream), "ttrl_linear_dgrad"))

    def linear_wgrad(self, x, g, dw, db, accumulate: bool, accumulate_db: bool,
                     precision: int | None = None) -> None:
        prec = self._prec(precision)
        m, k = x.shape[-2], x.shape[-1]
        n = g.shape[-1]
        need = lib().ttrl_linear_wgrad_workspace_bytes(m, k, n)
        ws, wsb = self.workspace(need)
        self._call(f"linear_wgrad[{m}x{k}x{n}]", 2 * m * k * n,
                   lambda: check(lib().ttrl_linear_wgrad(_ptr(_f32(x, "x")), _ptr(_f32(g, "g")),
                                              _ptr(_f32(dw, "dw")), _ptr(_f32(db, "db")), m, k, n,
                                              int(accumulate), int(accumulate_db), prec, ws, wsb,
                                              self.status_ptr(), self.stream), "ttrl_linear_wgrad"))

    # -- conv ------------------------------------------------------------

    def conv_fprop(self, x, w, b, y, geom: Geom, alpha: float, relu: bool,
                   precision: int | None = None) -> None:
        prec = self._prec(precision)
        g = geom.c_struct()
        ws, wsb = self.workspace()
        self._call(f"conv_fprop[{geom.kh}x{geom.kw}/{geom.stride} {geom.c}->{geom.cout}]",
                         _conv_flops(geom),
                   lambda: check(lib().ttrl_conv_fprop(_ptr(_f32(x, "x")), _ptr(_f32(w, "w")), _ptr(_f32(b, "b")),
                                            _ptr(_f32(y, "y")), ctypes.byref(g), float(alpha),
                                            int(relu), prec, ws, wsb, self.status_ptr(),
                                            self.stream), "ttrl_conv_fprop"))

    def conv_dgrad(self, dy, w, mask, dx, geom: Geom, accumulate: bool,
                   precision: int | None = None) -> None:
        prec = self._prec(precision)
        g = geom.c_struct()
        need = lib().ttrl_conv_dgrad_workspace_bytes(ctypes.byref(g))
        ws, wsb = self.workspace(need)
        self._call(f"conv_dgrad[{geom.kh}x{geom.kw}/{geom.stride} {geom.c}->{geom.cout}]",
                         _conv_flops(geom),
                   lambda: check(lib().ttrl_conv_dgrad(_ptr(_f32(dy, "dy")), _ptr(_f32(w, "w")),
                                            _ptr(_f32(mask, "mask")), _ptr(_f32(dx, "dx")),
                                            ctypes.byref(g), int(accumulate), prec, ws, wsb,
                                            self.status_ptr(), self.stream), "ttrl_conv_dgrad"))

    def conv_dgrad_weights_bytes(self, geom: Geom) -> int:
        """Bytes of the stacked sub-kernels of the two-step data gradient, or
        0 when the geometry takes the column path (ttrl_conv_dgrad)."""
        g = geom.c_struct()
        return int(lib().ttrl_conv_dgrad_weights_bytes(ctypes.byref(g)))

    def conv_dgrad_weights(self, w, out, geom: Geom) -> None:
        g = geom.c_struct()
        check(lib().ttrl_conv_dgrad_weights(_ptr(_f32(w, "w")), _ptr(_f32(out, "out")),
                                            ctypes.byref(g), self.stream),
              "ttrl_conv_dgrad_weights")

    def conv_dgrad_prepared(self, dy, wt, mask, dx, geom: Geom, accumulate: bool,
                            precision: int | None = None) -> None:
        prec = self._prec(precision)
        g = geom.c_struct()
        need = lib().ttrl_conv_dgrad_prepared_workspace_bytes(ctypes.byref(g))
        ws, wsb = self.workspace(need)
        self._call(f"conv_dgrad[{geom.kh}x{geom.kw}/{geom.stride} {geom.c}->{geom.cout}]",
                         _conv_flops(geom),
                   lambda: check(lib().ttrl_conv_dgrad_prepared(_ptr(_f32(dy, "dy")), _ptr(_f32(wt, "wt")),
                                                     _ptr(_f32(mask, "mask")), _ptr(_f32(dx, "dx")),
                                                     ctypes.byref(g), int(accumulate), prec, ws, wsb,
                                                     self.status_ptr(), self.stream),
                      "ttrl_conv_dgrad_prepared"))

    def conv_wgrad(self, x, dy, dw, db, geom: Geom, alpha: float, accumulate: bool,
                   accumulate_db: bool, precision: int | None = None) -> None:
        prec = self._prec(precision)
        g = geom.c_struct()
        need = lib().ttrl_conv_wgrad_workspace_bytes(ctypes.byref(g))
        ws, wsb = self.workspace(need)
        self._call(f"conv_wgrad[{geom.kh}x{geom.kw}/{geom.stride} {geom.c}->{geom.cout}]",
                         _conv_flops(geom),
                   lambda: check(lib().ttrl_conv_wgrad(_ptr(_f32(x, "x")), _ptr(_f32(dy, "dy")),
                                            _ptr(_f32(dw, "dw")), _ptr(_f32(db, "db")), ctypes.byref(g),
                                            float(alpha), int(accumulate), int(accumulate_db),
                                            prec, ws, wsb, self.status_ptr(), self.stream),
                      "ttrl_conv_wgrad"))

    def u8_to_f32(self, frames, index, out, scale: float = 1.0, fold: int = 1) -> None:
        """uint8 NCHW frames (optionally gathered by `index`) to fp32 NHWC rows,
        or, with fold > 1, to space-to-depth rows [n*(h/fold)*(w/fold)][fold²c]."""
        if frames.dtype != torch.uint8 or frames.dim() != 4:
            raise ValueError("frames must be a uint8 [N, C, H, W] CUDA tensor")
        n = frames.shape[0]
        if index is not None:
            if index.dtype != torch.int32:
                raise ValueError("index must be int32")
            n = index.shape[0]
        c, h, w = frames.shape[1], frames.shape[2], frames.shape[3]
        if fold > 1:
            check(lib().ttrl_u8_nchw_to_f32_s2d(_ptr(frames), _ptr(index), _ptr(_f32(out, "out")),
                                                n, c, h, w, int(fold), float(scale), self.stream),
                  "ttrl_u8_nchw_to_f32_s2d")
            return
        check(lib().ttrl_u8_nchw_to_f32_nhwc(_ptr(frames), _ptr(index), _ptr(_f32(out, "out")),
                                             n, c, h, w, float(scale), self.stream),
              "ttrl_u8_nchw_to_f32_nhwc")

    # -- optimizer -------------------------------------------------------

    def adam_step(self, tensors, steps, ticket, grad_scale, lr, b1, b2, eps, wd,
                  lr_device=None, bias=None) -> None:
        """`tensors`: list of (param, grad, S, V, step_index[, lr_index])."""
        for start in range(0, len(tensors), 64):
            chunk = tensors[start:start + 64]
            arr = (_lib.AdamTensor * len(chunk))()
            for i, (p, g, s, v, idx, *rest) in enumerate(chunk):
                arr[i] = _lib.AdamTensor(_ptr(_f32(p, "param")), _ptr(_f32(g, "grad")),
                                         _ptr(_f32(s, "S")), _ptr(_f32(v, "V")), p.numel(),
                                         int(idx), int(rest[0]) if rest else 0)
            check(lib().ttrl_adam_step(arr, len(chunk), _ptr(steps), _ptr(ticket),
                                       _ptr(grad_scale), _ptr(lr_device), float(lr), float(b1),
                                       float(b2), float(eps), float(wd), _ptr(bias),
                                       0 if bias is None else bias.shape[0], self.stream),
                  "ttrl_adam_step")

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

    # -- tape primitives ---------------------------------------------------

    def ew(self, op: str, a, b, out, scalar: float = 0.0) -> None:
        """out = op(a, b, scalar); a/b broadcast to out's shape (rank <= 4)."""
        shape = tuple(out.shape) or (1,)
        nd = len(shape)
        if nd > 4:
            raise ValueError(f"elementwise ops support rank <= 4, got {shape}")

        def strides(t):
            if t is None:
                return None, None
            if t.dtype != torch.float32:
                raise ValueError(f"elementwise operand must be float32, got {t.dtype}")
            ex = t.expand(shape) if t.dim() else t.reshape((1,) * nd).expand(shape)
            return t.data_ptr(), (ctypes.c_int64 * nd)(*ex.stride())

        ap, ast = strides(a)
        bp, bst = strides(b)
        if not out.is_contiguous():
            raise ValueError("elementwise output must be contiguous")
        sh = (ctypes.c_int64 * nd)(*shape)
        check(lib().ttrl_ew(_lib.EW[op], ap, ast, bp, bst, out.data_ptr(), sh, nd,
                            float(scalar), self.stream), f"ttrl_ew({op})")

    def reduce(self, op: int, inp, out, outer: int, n: int, inner: int) -> None:
        check(lib().ttrl_reduce(op, _ptr(_f32(inp, "in")), _ptr(_f32(out, "out")), int(outer),
                                int(n), int(inner), self.stream), "ttrl_reduce")

    def copy_strided(self, dst, src, accumulate: bool = False) -> None:
        """dst (=|+=) src elementwise for two same-shape (possibly strided) views."""
        shape = tuple(dst.shape) or (1,)
        nd = len(shape)
        if tuple(src.shape) != tuple(dst.shape):
            raise ValueError(f"copy shape mismatch {tuple(src.shape)} vs {tuple(dst.shape)}")
        sh = (ctypes.c_int64 * nd)(*shape)
        ds = (ctypes.c_int64 * nd)(*(dst.stride() if dst.dim() else (1,)))
        ss = (ctypes.c_int64 * nd)(*(src.stride() if src.dim() else (1,)))
        check(lib().ttrl_copy_strided(dst.data_ptr(), ds, src.data_ptr(), ss, sh, nd,
                                      int(accumulate), self.stream), "ttrl_copy_strided")

    def blend(self, pairs, tau: float | None = None) -> None:
        """One launch over `pairs` of same-size (dst, src) fp32 tensors:
        dst = src bit for bit (tau None: the hard target copy), else the
        Polyak blend dst = (1 - tau) * dst + tau * src."""
        arr = (_lib.BlendPair * max(len(pairs), 1))()
        for i, (d, s_) in enumerate(pairs):
            if d.numel() != s_.numel():
                raise ValueError(f"blend: pair {i} has {d.numel()} and {s_.numel()} elements")
            if not d.is_contiguous() or not s_.is_contiguous():
                raise ValueError(f"blend: pair {i} is not contiguous")
            arr[i] = _lib.BlendPair(_ptr(_f32(d, "dst")), _ptr(_f32(s_, "src")), d.numel())
        mode = _lib.BLEND_COPY if tau is None else _lib.BLEND_POLYAK
        check(lib().ttrl_blend_multi(arr, len(pairs), mode, float(tau or 0.0), self.stream),
              "ttrl_blend_multi")

    def polyak(self, dst, src, tau: float) -> None:
        check(lib().ttrl_polyak(_ptr(_f32(dst, "dst")), _ptr(_f32(src, "src")), dst.numel(),
                                float(tau), self.stream), "ttrl_polyak")

    def gather_rows(self, src, idx, dst) -> None:
        """dst[i] = src[idx[i]] over the leading axis (4-byte elements)."""
        if src.element_size() != 4 or dst.element_size() != 4 or idx.dtype != torch.int32:
            raise ValueError("gather_rows moves 4-byte rows by int32 index")
        row = 1
        for d in src.shape[1:]:
            row *= int(d)
        check(lib().ttrl_gather_rows(src.data_ptr(), idx.data_ptr(), dst.data_ptr(),
                                     int(idx.numel()), row, self.stream), "ttrl_gather_rows")

    def gather_rows_multi(self, pairs, idx) -> None:
        """dst[i] = src[idx[i]] for every (src, dst) of `pairs` (4-byte
        elements, at most 8 pairs), in one launch."""
        if idx.dtype != torch.int32:
            raise ValueError("gather_rows_multi: int32 index")
        jobs = (_lib.GatherJob * len(pairs))()
        for i, (src, dst) in enumerate(pairs):
            if src.element_size() != 4 or dst.element_size() != 4:
                raise ValueError("gather_rows_multi moves 4-byte rows")
            row = 1
            for d in src.shape[1:]:
                row *= int(d)
            jobs[i] = _lib.GatherJob(src.data_ptr(), dst.data_ptr(), row, 0)
        check(lib().ttrl_gather_rows_multi(jobs, len(pairs), idx.data_ptr(), int(idx.numel()),
                                           self.stream), "ttrl_gather_rows_multi")

    def gru_gates_fwd(self, gi, gh, hm, start_next, out, gates, hm_next) -> None:
        """One GRU step's gates after its recurrent GEMM (rows [B][3H])."""
        b, hidden = hm.shape[0], hm.shape[1]
        check(lib().ttrl_gru_gates_fwd(_ptr(gi), _ptr(gh), _ptr(hm), _ptr(start_next), _ptr(out),
                                       _ptr(gates), _ptr(hm_next), b, hidden, self.stream),
              "ttrl_gru_gates_fwd")

    def gru_gates_bwd(self, dout, dhm, start_next, carry: bool, gates, gh, hm, dgi,
                      dgh) -> None:
        """One GRU step's backward; leaves dh * z in `dhm`."""
        b, hidden = hm.shape[0], hm.shape[1]
        check(lib().ttrl_gru_gates_bwd(_ptr(dout), _ptr(dhm), _ptr(start_next), int(carry),
                                       _ptr(gates), _ptr(gh), _ptr(hm), _ptr(dgi), _ptr(dgh), b,
                                       hidden, self.stream), "ttrl_gru_gates_bwd")

    def epsilon_greedy(self, q, mask, draws, alt, eps, actions) -> None:
        """actions = draws < eps ? alt : first argmax of q over legal columns."""
        b, a = q.shape
        check(lib().ttrl_epsilon_greedy(_ptr(q), _ptr(mask), _ptr(draws), _ptr(alt), _ptr(eps),
                                        _ptr(actions), b, a, self.stream), "ttrl_epsilon_greedy")

    def categorical_sample(self, logits, uniforms, actions, logp) -> None:
        """Inverse-CDF draw (uniforms None: argmax) from the log-softmax."""
        b, a = logits.shape
        check(lib().ttrl_categorical_sample(_ptr(logits), _ptr(uniforms), _ptr(actions),
                                            _ptr(logp), b, a, self.stream),
              "ttrl_categorical_sample")

    def gae(self, rewards, values, dones, valid, last_values, advantages, returns,
            gamma: float, lam: float) -> None:
        """GAE-lambda over [n_steps, n_envs] device arrays (bit-exact with the
        reference's float32 recursion)."""
        steps, envs = values.shape
        gamma_lam = float(np.float32(float(gamma) * float(lam)))
        check(lib().ttrl_gae(_ptr(rewards), _ptr(values), _ptr(dones), _ptr(valid),
                             _ptr(last_values), _ptr(advantages), _ptr(returns), steps, envs,
                             float(np.float32(gamma)), gamma_lam, self.stream), "ttrl_gae")

    def normalize_advantages(self, advantages, valid, out) -> None:
        check(lib().ttrl_normalize_advantages(_ptr(advantages), _ptr(valid), _ptr(out),
                                              int(advantages.numel()), self.status_ptr(),
                                              self.stream), "ttrl_normalize_advantages")

    def gru_sequence_supported(self, batch: int, hidden: int) -> bool:
        """Whether the one-launch sequence kernels take this shape here."""
        torch.cuda.set_device(self.index)
        return bool(lib().ttrl_gru_sequence_supported(int(batch), int(hidden)))

    def gru_sequence_fwd(self, gi, h0, starts, w_hh, b_hh, gh, gates, hm, out) -> None:
        """The whole recurrent unroll after the input GEMM, one launch."""
        steps, b, hidden = hm.shape
        check(lib().ttrl_gru_sequence_fwd(_ptr(gi), _ptr(h0), _ptr(starts), _ptr(w_hh),
                                          _ptr(b_hh), _ptr(gh), _ptr(gates), _ptr(hm), _ptr(out),
                                          steps, b, hidden, self.stream), "ttrl_gru_sequence_fwd")

    def gru_sequence_bwd(self, dout, starts, w_hh, gates, gh, hm, dgi, dgh, dh0) -> None:
        """Its backward through time, one launch."""
        steps, b, hidden = hm.shape
        check(lib().ttrl_gru_sequence_bwd(_ptr(dout), _ptr(starts), _ptr(w_hh), _ptr(gates),
                                          _ptr(gh), _ptr(hm), _ptr(dgi), _ptr(dgh), _ptr(dh0),
                                          steps, b, hidden, self.stream), "ttrl_gru_sequence_bwd")

    def gru_mask(self, h, start, out) -> None:
        """out = h * (1 - start) per row (start None: a copy)."""
        b, hidden = h.shape[0], h.shape[1]
        check(lib().ttrl_gru_mask(_ptr(h), _ptr(start), _ptr(out), b, hidden, self.stream),
              "ttrl_gru_mask")

    def dqn_loss(self, q, q_sel, q_tgt, onehot, rewards, dones, discounts, next_mask,
                 is_weights, loss, mean_q, td_abs, dq, delta: float,
                 accumulate: bool = False) -> None:
        b, a = q.shape[0], q.shape[1]
        check(lib().ttrl_dqn_loss(_ptr(q), _ptr(q_sel), _ptr(q_tgt), _ptr(onehot),
                                  _ptr(rewards), _ptr(dones), _ptr(discounts), _ptr(next_mask),
                                  _ptr(is_weights), _ptr(loss), _ptr(mean_q), _ptr(td_abs),
                                  _ptr(dq), b, a, float(delta), int(accumulate), self.stream),
              "ttrl_dqn_loss")

    def ppo_loss(self, logits, value, actions, old_logp, adv, returns, old_values, valid,
                 metrics, new_logp, dlogits, dvalue, clip, vclip, vcoef, entcoef) -> None:
        b, a = logits.shape[0], logits.shape[1]
        if actions.dtype != torch.int32:
            raise ValueError("ppo_loss: actions must be int32")
        check(lib().ttrl_ppo_loss(_ptr(logits), _ptr(value), _ptr(actions), _ptr(old_logp),
                                  _ptr(adv), _ptr(returns), _ptr(old_values), _ptr(valid),
                                  _ptr(metrics), _ptr(new_logp), _ptr(dlogits), _ptr(dvalue), b,
                                  a, float(clip), float(vclip), float(vcoef), float(entcoef),
                                  self.stream), "ttrl_ppo_loss")

    # -- SAC heads ---------------------------------------------------------

    def sac_sample(self, mean, raw, noise, scale, centre, obs, joint, logp, lo: float,
                   hi: float, log_det: float, pack=None) -> None:
        b, d = mean.shape[0], mean.shape[1]
        o = 0 if obs is None else obs.shape[1]
        po, pa, pj = (None, None, None) if pack is None else pack
        check(lib().ttrl_sac_sample(_ptr(mean), _ptr(raw), _ptr(noise), _ptr(scale),
                                    _ptr(centre), _ptr(obs), _ptr(joint), _ptr(logp), b, d, o,
                                    float(lo), float(hi), float(log_det), _ptr(po), _ptr(pa),
                                    _ptr(pj), self.stream), "ttrl_sac_sample")

    def sac_sample_backward(self, mean, raw, noise, scale, d_action, ld: int, d_logp, d_mean,
                            d_raw, acc_mean: bool, acc_raw: bool, lo: float, hi: float) -> None:
        b, d = mean.shape[0], mean.shape[1]
        check(lib().ttrl_sac_sample_backward(_ptr(mean), _ptr(raw), _ptr(noise), _ptr(scale),
                                             _ptr(d_action), int(ld), _ptr(d_logp),
                                             _ptr(d_mean), _ptr(d_raw), int(acc_mean),
                                             int(acc_raw), b, d, float(lo), float(hi),
                                             self.stream), "ttrl_sac_sample_backward")

    def sac_critic_loss(self, qs, q_targets, next_logp, log_alpha, rewards, dones, discounts,
                        is_weights, loss, alpha, target, dqs, td_abs) -> None:
        n = len(qs)
        arr = lambda ts: (ctypes.c_void_p * n)(*[_ptr(t) for t in ts])
        check(lib().ttrl_sac_critic_loss(arr(qs), arr(q_targets), n, _ptr(next_logp),
                                         _ptr(log_alpha), _ptr(rewards), _ptr(dones),
                                         _ptr(discounts), _ptr(is_weights), _ptr(loss),
                                         _ptr(alpha), _ptr(target), arr(dqs), _ptr(td_abs),
                                         int(qs[0].shape[0]), self.stream),
              "ttrl_sac_critic_loss")

    def sac_actor_loss(self, qs, logp, log_alpha, target_entropy: float, loss, dqs, d_logp,
                       alpha_loss, d_log_alpha) -> None:
        n = len(qs)
        arr = lambda ts: (ctypes.c_void_p * n)(*[_ptr(t) for t in ts])
        check(lib().ttrl_sac_actor_loss(arr(qs), n, _ptr(logp), _ptr(log_alpha),
                                        float(target_entropy), _ptr(loss), arr(dqs),
                                        _ptr(d_logp), _ptr(alpha_loss), _ptr(d_log_alpha),
                                        int(qs[0].shape[0]), self.stream), "ttrl_sac_actor_loss")


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
