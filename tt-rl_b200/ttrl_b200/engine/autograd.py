"""Reverse-mode autograd tape over CUDA tensors.

Same contract as the reference tape (ttrl/engine/autograd.py:56-235):
`Tensor(data, requires_grad, _parents, _op)`, fp32 gradient accumulation,
every node's backward run after all of its consumers', a scalar seed of 1.0,
no retain_graph (the tape is released whether backward finishes or raises),
and `no_grad`. The traversal here counts, for every node reachable from the
root, how many of its consumers are still pending, and runs a node once that
count reaches zero (a ready stack, first parent first).

Two additions serve the fused kernels:

* A tensor produced by a fused Linear/Conv2d + ReLU node carries
  `_premask = True`: every gradient it holds is already multiplied by its
  ReLU mask (y > 0). Fused consumers write their input gradient with the
  mask applied in the GEMM epilogue and pass `premasked=True`; any other
  contribution is masked on the way in by `_accumulate`. The fused node's
  backward therefore reads `out.grad` as the gradient of the pre-activation.
* A parameter owns one persistent gradient buffer (`_grad_buf`). Fused
  weight-gradient kernels write into it (or accumulate into it), so a
  captured CUDA graph always finds the gradient at the same address.
"""

from __future__ import annotations

import numpy as np
import torch

from ttrl_b200.device import context

__all__ = ["Tensor", "backward", "no_grad", "is_grad_enabled", "DEFAULT_DTYPE"]

DEFAULT_DTYPE = torch.float32
GRAD_ACCUM_DTYPE = torch.float32

#: Open `no_grad` blocks; recording is on only at depth zero.
_NO_GRAD_DEPTH = 0

#: The tensor whose backward() is running. A fused loss node that is the root
#: receives the unit seed and can skip scaling its precomputed gradient.
_BACKWARD_ROOT = None


def backward_root():
    return _BACKWARD_ROOT


def is_grad_enabled() -> bool:
    return _NO_GRAD_DEPTH == 0


class no_grad:
    """Inside this block no op records a tape node (the forward-only target
    and acting passes), as ttrl/engine/autograd.py:30-44 specifies. Blocks
    nest; leaving the outermost one turns recording back on."""

    def __enter__(self):
        global _NO_GRAD_DEPTH
        _NO_GRAD_DEPTH += 1
        return self

    def __exit__(self, *exc):
        global _NO_GRAD_DEPTH
        _NO_GRAD_DEPTH -= 1
        return False


def _no_backward(grad):
    return None


_UNIT_SEEDS: dict = {}


def _unit_seed(like):
    """d(loss)/d(loss) = 1, shaped like the scalar root: one constant per
    device and shape, made outside any capture (no fill launch per
    backward); inside a first capture, filled by a kernel instead.

    The constant is shared by every backward on the device and is bound as
    the root's `.grad` afterwards, so the root's gradient is read-only: an
    in-place change to it would change the seed of every later backward.
    Its fill is waited for once, on the host, before first use, so a
    backward issued on any stream reads the finished constant."""
    key = (like.device, tuple(like.shape))
    seed = _UNIT_SEEDS.get(key)
    if seed is None:
        if torch.cuda.is_current_stream_capturing():
            seed = torch.empty_like(like, dtype=GRAD_ACCUM_DTYPE)
            context(like.device).ew("fill", None, None, seed, 1.0)
            return seed
        seed = torch.ones(like.shape, dtype=GRAD_ACCUM_DTYPE, device=like.device)
        torch.cuda.current_stream(like.device).synchronize()
        _UNIT_SEEDS[key] = seed
    return seed


def _default_device():
    if not torch.cuda.is_available():
        raise RuntimeError("ttrl_b200 needs a CUDA device; there is no CPU fallback")
    return torch.device("cuda", torch.cuda.current_device())


def as_device(device) -> torch.device:
    """Normalise the reference's `device` argument to a torch CUDA device."""
    if device is None:
        return _default_device()
    if hasattr(device, "torch_device"):
        return device.torch_device
    d = torch.device(device) if not isinstance(device, torch.device) else device
    if d.type != "cuda":
        raise ValueError(f"ttrl_b200 runs on CUDA devices only, got {device!r}")
    if d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return d


class Tensor:
    """A node in the autograd graph, backed by a CUDA tensor."""

    __slots__ = ("data", "requires_grad", "grad", "_backward", "_parents", "_op",
                 "_backward_done", "_premask", "_grad_buf", "_grad_owned", "_exact",
                 "_fold", "_layout", "__weakref__")

    def __init__(self, data, requires_grad: bool = False, _parents=(), _op: str = ""):
        self.data = data
        self.requires_grad = requires_grad
        self.grad = None
        self._backward = _no_backward
        self._parents = tuple(_parents)
        self._op = _op
        self._backward_done = False
        self._premask = False
        self._grad_buf = None
        self._grad_owned = False
        # Every value is exactly representable in tf32 (raw 0..255 pixels):
        # a convolution reading it skips the split-TF32 low part.
        self._exact = False
        # Rows already in space-to-depth order for this fold factor (a first
        # convolution reads them directly); 1: plain NHWC rows.
        self._fold = 1
        # A parameter stored in a device layout other than its portable one
        # (a convolution's KRSC weight): converts optimizer state to and from
        # the portable layout. None: the device layout is the portable one.
        self._layout = None

    # -- construction ------------------------------------------------------

    @staticmethod
    def from_numpy(array, device=None, *, requires_grad=False, dtype=DEFAULT_DTYPE,
                   layout=None) -> "Tensor":
        dev = as_device(device)
        arr = np.ascontiguousarray(np.asarray(array))
        if dtype in (torch.float32, None, np.float32):
            arr = arr.astype(np.float32, copy=False)
            t = torch.from_numpy(arr).to(dev)
        else:
            t = torch.from_numpy(arr).to(dev, dtype=dtype)
        return Tensor(t, requires_grad)

    def numpy(self) -> np.ndarray:
        if self.data.is_cuda:
            context(self.data.device).join()  # written on a side lane, perhaps
        out = self.data.detach().to("cpu").numpy()
        return out.astype(np.float32) if out.dtype != np.float32 and out.dtype.kind == "f" else out

    # -- introspection -----------------------------------------------------

    @property
    def shape(self):
        return tuple(self.data.shape)

    @property
    def device(self):
        return self.data.device

    @property
    def dtype(self):
        return self.data.dtype

    def __repr__(self):
        return f"Tensor(shape={self.shape}, op={self._op or 'leaf'}, grad={self.requires_grad})"

    # -- gradient plumbing -------------------------------------------------

    def _accumulate(self, grad, premasked: bool = False):
        """Add one gradient contribution (a torch tensor shaped like data)."""
        if grad.dtype != GRAD_ACCUM_DTYPE:
            grad = grad.to(GRAD_ACCUM_DTYPE)
        if tuple(grad.shape) != tuple(self.data.shape):
            grad = grad.reshape(self.data.shape)
        ctx = context(self.data.device)
        if self._op == "" and self.grad is not None:
            ctx.join()  # a parameter's gradient may still be written on a side lane
        if self._premask and not premasked:
            masked = torch.empty_like(grad)
            ctx.ew("relu_bw", grad, self.data, masked)
            grad = masked
        if self.grad is None:
            self.grad = grad
            self._grad_owned = False
        elif self._grad_owned:
            ctx.ew("add", self.grad, grad, self.grad)
        else:
            total = torch.empty_like(self.grad)
            ctx.ew("add", self.grad, grad, total)
            self.grad = total
            self._grad_owned = True

    def _grad_slot(self):
        """(buffer, accumulate) for a fused kernel about to write this tensor's
        gradient. Parameters write into their persistent `_grad_buf`."""
        if self.grad is None:
            if self._op == "" and self.requires_grad:
                if self._grad_buf is None or self._grad_buf.shape != self.data.shape:
                    self._grad_buf = torch.empty_like(self.data)
                return self._grad_buf, False
            return torch.empty_like(self.data), False
        if self._grad_owned and self.grad.is_contiguous():
            return self.grad, True
        # A gradient we do not own (bound from another op): copy it into a
        # buffer of our own, then accumulate into that.
        if self._op == "" and self.requires_grad:
            if self._grad_buf is None or self._grad_buf.shape != self.data.shape:
                self._grad_buf = torch.empty_like(self.data)
            buf = self._grad_buf
        else:
            buf = torch.empty_like(self.data)
        if buf.data_ptr() != self.grad.data_ptr():
            context(self.data.device).copy_strided(buf, self.grad.reshape(buf.shape))
        return buf, True

    def _set_grad(self, buf):
        """Record that a fused kernel wrote (or accumulated) `buf`."""
        self.grad = buf
        self._grad_owned = True

    def zero_grad(self):
        self.grad = None
        self._grad_owned = False

    def detach(self) -> "Tensor":
        return Tensor(self.data, requires_grad=False)

    def backward(self):
        """Run the tape from this scalar back to the leaves, once.

        Afterwards `.grad` of this tensor is the shared unit seed: read it,
        never write it in place."""
        if not self.requires_grad:
            raise RuntimeError(
                "backward(): this tensor has requires_grad=False -- it was never "
                "recorded (a leaf without gradient, a detach(), or a result built "
                "under no_grad()), so there is no tape to run and no parameter "
                "would receive a gradient.")
        if self._backward_done:
            raise RuntimeError(
                "backward(): this graph's tape has already been run and released; "
                "saved activations are not kept for a second pass. Run the "
                "forward again to build a new graph.")
        size = 1
        for extent in self.shape:
            size *= extent
        if size != 1:
            raise RuntimeError(
                f"backward(): the root must hold one value, got shape {self.shape} "
                f"({size} values). Reduce it to a scalar (mean or sum) first; a "
                "non-scalar seed is not supported.")

        # Every node reachable from the root, and for each the number of
        # its consumers in this graph that have yet to run.
        pending: dict[int, int] = {id(self): 0}
        nodes: list[Tensor] = [self]
        frontier = [self]
        while frontier:
            node = frontier.pop()
            for parent in node._parents:
                key = id(parent)
                if key in pending:
                    pending[key] += 1
                else:
                    pending[key] = 1
                    nodes.append(parent)
                    frontier.append(parent)

        self.grad = _unit_seed(self.data)
        # Not owned: an op that accumulates into the root's gradient copies
        # it first, so the shared constant is never written.
        self._grad_owned = False
        global _BACKWARD_ROOT
        outer_root, _BACKWARD_ROOT = _BACKWARD_ROOT, self
        try:
            ready = [self]
            while ready:
                node = ready.pop()
                if node.grad is not None:
                    if node._backward_done and node is not self:
                        raise RuntimeError(
                            "backward(): part of this graph was already consumed by an "
                            "earlier backward() (a subgraph shared by two losses); its "
                            "saved activations are gone. Build each loss from its own "
                            "forward pass.")
                    node._backward(node.grad)
                # Parents whose last consumer this was become ready; pushed
                # last-to-first so the first parent is taken next.
                for parent in reversed(node._parents):
                    key = id(parent)
                    pending[key] -= 1
                    if pending[key] == 0:
                        ready.append(parent)
        finally:
            _BACKWARD_ROOT = outer_root
            # Weight gradients issued on side lanes are complete before
            # anything after backward() runs on the current stream.
            context(self.data.device).join()
            # Release the tape. Leaves stay usable by the next step's graph,
            # so only recorded nodes are marked as consumed.
            for node in nodes:
                node._backward_done = node._backward_done or bool(node._op)
                node._backward = _no_backward
                node._parents = ()

    # -- operators ---------------------------------------------------------

    def __add__(self, other):
        from ttrl_b200.engine.ops import add
        return add(self, other)

    __radd__ = __add__

    def __mul__(self, other):
        from ttrl_b200.engine.ops import mul
        return mul(self, other)

    __rmul__ = __mul__

    def __sub__(self, other):
        from ttrl_b200.engine.ops import sub
        return sub(self, other)

    def __rsub__(self, other):
        from ttrl_b200.engine.ops import sub
        return sub(other, self)

    def __neg__(self):
        from ttrl_b200.engine.ops import mul
        return mul(self, -1.0)

    def __truediv__(self, other):
        from ttrl_b200.engine.ops import div
        return div(self, other)


def backward(tensor: Tensor) -> None:
    tensor.backward()


# --------------------------------------------------------------------------
# shared op-building helpers (ttrl/engine/autograd.py:205-235)
# --------------------------------------------------------------------------

def _is_scalar(x) -> bool:
    return not isinstance(x, Tensor) and not hasattr(x, "shape")


def _needs(*tensors) -> bool:
    return _NO_GRAD_DEPTH == 0 and any(t.requires_grad for t in tensors)


def _detached(data) -> Tensor:
    return Tensor(data, requires_grad=False)
