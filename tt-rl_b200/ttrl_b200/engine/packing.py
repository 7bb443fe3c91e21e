"""The reference's prepared convolution-weight matrix, as index arithmetic
(ttrl/engine/conv/packing.py:24-187).

The reference keeps a convolution's master weight, and so the Adam moments
of that weight, as a `[1, 1, rows, cols]` matrix with

    M[r * row_block + s * cp + c, k] = W[k, c, r, s]

and zeros everywhere else: `cp` >= C is the padded channel stride inside one
kernel row, `row_block` >= S * cp the padded extent of one kernel row and
`cols` >= K the padded output-channel count. Its checkpoints store the
network weights in logical OIHW (engine/conv/module.py:182-219) but the
optimizer moments in this matrix (engine/optim/checkpoint.py:30-42), so
reading or writing a reference file's optimizer state goes through here.

`rows` and `cols` are visible in a stored matrix's shape; `cp` is not.
`solve_cp` recovers it from where the stored second moment is non-zero (v > 0
for every weight that ever had a gradient, exactly 0 on padding), and
`default_layout` gives the layout the reference's device library produces
for the shapes its tests pin (cp = C rounded up to a multiple of 8,
row_block = S * cp rounded up to 32, cols = K rounded up to 32: 4-channel
8x8 conv with 32 outputs -> (1, 1, 512, 32)).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

__all__ = ["AmbiguousLayout", "PreparedLayout", "default_layout", "candidate_layouts",
           "solve_cp"]


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass(frozen=True)
class PreparedLayout:
    rows: int
    cols: int
    cp: int
    out_channels: int
    in_channels: int
    kernel_h: int
    kernel_w: int

    def __post_init__(self) -> None:
        if self.rows % self.kernel_h:
            raise ValueError(f"prepared rows={self.rows} is not a multiple of kernel height "
                             f"{self.kernel_h}")
        if self.cp < self.in_channels or self.row_block < self.kernel_w * self.cp:
            raise ValueError(f"prepared layout {self.rows}x{self.cols} with cp={self.cp} cannot "
                             f"hold {self.in_channels} channels of a {self.kernel_h}x"
                             f"{self.kernel_w} kernel")
        if self.cols < self.out_channels:
            raise ValueError(f"prepared cols={self.cols} < {self.out_channels} outputs")

    @property
    def row_block(self) -> int:
        return self.rows // self.kernel_h

    @property
    def shape(self) -> tuple[int, int, int, int]:
        return (1, 1, self.rows, self.cols)

    def _index(self):
        """(flat row index, output column) of every OIHW element, in OIHW order."""
        k, c, r, s = np.meshgrid(np.arange(self.out_channels), np.arange(self.in_channels),
                                 np.arange(self.kernel_h), np.arange(self.kernel_w),
                                 indexing="ij")
        return (r * self.row_block + s * self.cp + c).reshape(-1), k.reshape(-1)

    def pack(self, w_oihw) -> np.ndarray:
        w = np.asarray(w_oihw, np.float32)
        want = (self.out_channels, self.in_channels, self.kernel_h, self.kernel_w)
        if w.shape != want:
            raise ValueError(f"PreparedLayout.pack: weight {w.shape}, layout holds {want}")
        out = np.zeros((self.rows, self.cols), np.float32)
        row, col = self._index()
        out[row, col] = w.reshape(-1)
        return out.reshape(self.shape)

    def unpack(self, m) -> np.ndarray:
        a = np.asarray(m, np.float32).reshape(self.rows, self.cols)
        row, col = self._index()
        return np.ascontiguousarray(a[row, col].reshape(
            self.out_channels, self.in_channels, self.kernel_h, self.kernel_w))

    def padding_is_zero(self, m) -> bool:
        a = np.asarray(m).reshape(self.rows, self.cols)
        live = np.zeros(a.shape, bool)
        row, col = self._index()
        live[row, col] = True
        return not np.any(a[~live])


def default_layout(out_channels: int, in_channels: int, kernel_h: int,
                   kernel_w: int) -> PreparedLayout:
    cp = _round_up(max(in_channels, 1), 8)
    return PreparedLayout(rows=kernel_h * _round_up(kernel_w * cp, 32),
                          cols=_round_up(out_channels, 32), cp=cp, out_channels=out_channels,
                          in_channels=in_channels, kernel_h=kernel_h, kernel_w=kernel_w)


def candidate_layouts(rows: int, cols: int, out_channels: int, in_channels: int, kernel_h: int,
                      kernel_w: int) -> list[PreparedLayout]:
    """Every layout a `(rows, cols)` matrix can be for an (O, C, KH, KW) weight."""
    if rows % kernel_h:
        return []
    out = []
    for cp in range(in_channels, rows // kernel_h // kernel_w + 1):
        try:
            out.append(PreparedLayout(rows, cols, cp, out_channels, in_channels, kernel_h,
                                      kernel_w))
        except ValueError:
            continue
    return out


class AmbiguousLayout(ValueError):
    """The stored moments fit several prepared layouts and cannot tell them
    apart (a second moment that is zero everywhere, for a weight that never
    had a gradient, in a matrix whose shape is not the default layout's)."""


def solve_cp(shape, oihw, *, v=None, strict: bool = False) -> PreparedLayout:
    """The layout of a stored `[1, 1, rows, cols]` moment for an OIHW weight:
    among the candidates, the ones whose padding holds zeros in `v`; of those
    the default layout if it is one, else the one whose live region `v`
    fills most (v > 0 on every trained weight). With `strict` there is no
    preference for the default: several candidates that `v` fills equally
    (an all-zero `v`) raise `AmbiguousLayout` instead of picking one."""
    if len(shape) != 4 or shape[0] != 1 or shape[1] != 1:
        raise ValueError(f"a prepared conv moment is [1, 1, rows, cols], got {tuple(shape)}")
    o, c, kh, kw = (int(d) for d in oihw)
    cands = candidate_layouts(int(shape[2]), int(shape[3]), o, c, kh, kw)
    if not cands:
        raise ValueError(f"no prepared layout of shape {tuple(shape)} holds an {oihw} weight")
    if v is not None:
        cands = [lay for lay in cands if lay.padding_is_zero(v)] or cands
    default = default_layout(o, c, kh, kw)
    if len(cands) == 1 or (default in cands and not strict):
        return default if default in cands else cands[0]
    if v is None:
        if strict and len(cands) > 1:
            raise AmbiguousLayout(f"{len(cands)} prepared layouts of shape {tuple(shape)} hold an "
                                  f"{tuple(oihw)} weight and no second moment tells them apart")
        return cands[0]
    filled = [int(np.count_nonzero(lay.unpack(v))) for lay in cands]
    best = max(filled)
    if strict and filled.count(best) > 1:
        raise AmbiguousLayout(
            f"{filled.count(best)} prepared layouts of shape {tuple(shape)} hold an "
            f"{tuple(oihw)} weight equally well (the stored second moment has "
            f"{best} non-zero live entries), so the channel stride cannot be recovered")
    return cands[filled.index(best)]
