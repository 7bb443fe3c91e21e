"""ctypes binding of ``libttrl_b200.so``, the C ABI declared in
``include/ttrl_b200.h``.

This is the binding a maintainer of the reference would add: the reference
is pure Python over ``ttnn``, so its natural FFI for a native backend is
ctypes over plain pointers. Loading fails loudly when the library is missing;
there is no CPU fallback anywhere in this package.
"""

from __future__ import annotations

import ctypes
import os

__all__ = [
    "LIB_PATH", "TtrlError", "lib", "Operand", "Epilogue", "GemmDesc", "ConvGeom",
    "AdamTensor", "BlendPair", "GatherJob", "BLEND_COPY", "BLEND_POLYAK", "PREC_TF32X3", "PREC_TF32", "OPND_DENSE", "OPND_CONV_FPROP",
    "OPND_CONV_WGRAD", "BIAS_NONE", "BIAS_ROW", "BIAS_COL", "EXPORTED_SYMBOLS",
]

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libttrl_b200.so")

PREC_TF32X3 = 0
PREC_TF32 = 1
OPND_DENSE = 0
OPND_CONV_FPROP = 1
OPND_CONV_WGRAD = 2
BIAS_NONE = 0
BIAS_ROW = 1
BIAS_COL = 2

_c_int = ctypes.c_int
_c_float = ctypes.c_float
_c_double = ctypes.c_double
_c_size = ctypes.c_size_t
_vp = ctypes.c_void_p


class TtrlError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, what: str, message: str):
        super().__init__(f"{what} failed with code {code}: {message}")
        self.code = code


class Operand(ctypes.Structure):
    _fields_ = [
        ("ptr", _vp), ("kind", ctypes.c_int32), ("rows", ctypes.c_int32),
        ("kdim", ctypes.c_int32), ("flags", ctypes.c_int32),
        ("rs", ctypes.c_int64), ("ks", ctypes.c_int64),
        ("n", ctypes.c_int32), ("h", ctypes.c_int32), ("w", ctypes.c_int32),
        ("c", ctypes.c_int32), ("kh", ctypes.c_int32), ("kw", ctypes.c_int32),
        ("stride", ctypes.c_int32), ("pad", ctypes.c_int32),
        ("oh", ctypes.c_int32), ("ow", ctypes.c_int32),
    ]


class Epilogue(ctypes.Structure):
    _fields_ = [
        ("out", _vp), ("ors", ctypes.c_int64), ("ocs", ctypes.c_int64),
        ("alpha", _c_float), ("bias_mode", ctypes.c_int32), ("bias", _vp),
        ("mask", _vp), ("mrs", ctypes.c_int64), ("mcs", ctypes.c_int64),
        ("relu", ctypes.c_int32), ("accumulate", ctypes.c_int32),
    ]


class GemmDesc(ctypes.Structure):
    _fields_ = [
        ("m", ctypes.c_int32), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
        ("precision", ctypes.c_int32), ("splits", ctypes.c_int32), ("pad0", ctypes.c_int32),
        ("a", Operand), ("b", Operand), ("ep", Epilogue),
    ]


class ConvGeom(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in
                ("n", "h", "w", "c", "cout", "kh", "kw", "stride", "pad", "oh", "ow", "flags")]


CONV_INPUT_EXACT = 1


class AdamTensor(ctypes.Structure):
    _fields_ = [
        ("param", _vp), ("grad", _vp), ("s", _vp), ("v", _vp),
        ("numel", ctypes.c_int64), ("step_index", ctypes.c_int32), ("lr_index", ctypes.c_int32),
    ]


class GatherJob(ctypes.Structure):
    _fields_ = [("src", ctypes.c_void_p), ("dst", ctypes.c_void_p), ("row", ctypes.c_int32),
                ("pad0", ctypes.c_int32)]


class BlendPair(ctypes.Structure):
    _fields_ = [("dst", _vp), ("src", _vp), ("n", ctypes.c_int64)]


BLEND_COPY = 0
BLEND_POLYAK = 1


# name -> (restype, argtypes). Every symbol include/ttrl_b200.h declares.
_SIGNATURES = {
    "ttrl_last_error": (ctypes.c_char_p, []),
    "ttrl_version": (_c_int, []),
    "ttrl_launch_count": (ctypes.c_ulonglong, []),
    "ttrl_init": (_c_int, [_c_int]),
    "ttrl_gemm_workspace_bytes": (_c_size, [ctypes.POINTER(GemmDesc)]),
    "ttrl_gemm": (_c_int, [ctypes.POINTER(GemmDesc), _vp, _c_size, _vp, _vp]),
    "ttrl_linear_fwd": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                 _vp, _c_size, _vp, _vp]),
    "ttrl_linear_fwd_noalloc": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                         _c_int, _vp, _vp]),
    "ttrl_linear_wgrad_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int]),
    "ttrl_linear_dgrad": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                   _vp, _c_size, _vp, _vp]),
    "ttrl_linear_wgrad": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                   _c_int, _vp, _c_size, _vp, _vp]),
    "ttrl_conv_fprop": (_c_int, [_vp, _vp, _vp, _vp, ctypes.POINTER(ConvGeom), _c_float, _c_int,
                                 _c_int, _vp, _c_size, _vp, _vp]),
    "ttrl_conv_dgrad": (_c_int, [_vp, _vp, _vp, _vp, ctypes.POINTER(ConvGeom), _c_int, _c_int,
                                 _vp, _c_size, _vp, _vp]),
    "ttrl_conv_dgrad_workspace_bytes": (_c_size, [ctypes.POINTER(ConvGeom)]),
    "ttrl_conv_dgrad_weights_bytes": (_c_size, [ctypes.POINTER(ConvGeom)]),
    "ttrl_conv_dgrad_weights": (_c_int, [_vp, _vp, ctypes.POINTER(ConvGeom), _vp]),
    "ttrl_conv_dgrad_prepared": (_c_int, [_vp, _vp, _vp, _vp, ctypes.POINTER(ConvGeom), _c_int,
                                          _c_int, _vp, _c_size, _vp, _vp]),
    "ttrl_conv_dgrad_prepared_workspace_bytes": (_c_size, [ctypes.POINTER(ConvGeom)]),
    "ttrl_conv_wgrad": (_c_int, [_vp, _vp, _vp, _vp, ctypes.POINTER(ConvGeom), _c_float, _c_int,
                                 _c_int, _c_int, _vp, _c_size, _vp, _vp]),
    "ttrl_conv_wgrad_workspace_bytes": (_c_size, [ctypes.POINTER(ConvGeom)]),
    "ttrl_u8_nchw_to_f32_nhwc": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                          _c_float, _vp]),
    "ttrl_u8_nchw_to_f32_s2d": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                         _c_float, _vp]),
    "ttrl_adam_step": (_c_int, [ctypes.POINTER(AdamTensor), _c_int, _vp, _vp, _vp, _vp,
                                _c_double, _c_double, _c_double, _c_double, _c_double, _vp,
                                ctypes.c_int64, _vp]),
    "ttrl_grad_sqnorm": (_c_int, [ctypes.POINTER(_vp), ctypes.POINTER(ctypes.c_int64), _c_int,
                                  _vp, _c_float, _vp, _c_size, _vp]),
    "ttrl_grad_sqnorm_workspace_bytes": (_c_size, [ctypes.POINTER(ctypes.c_int64), _c_int]),
    "ttrl_ew": (_c_int, [_c_int, _vp, ctypes.POINTER(ctypes.c_int64), _vp,
                         ctypes.POINTER(ctypes.c_int64), _vp, ctypes.POINTER(ctypes.c_int64),
                         _c_int, _c_float, _vp]),
    "ttrl_reduce": (_c_int, [_c_int, _vp, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                             _vp]),
    "ttrl_wait_probe": (_c_int, [_vp, _vp]),
    "ttrl_copy_strided": (_c_int, [_vp, ctypes.POINTER(ctypes.c_int64), _vp,
                                   ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64),
                                   _c_int, _c_int, _vp]),
    "ttrl_polyak": (_c_int, [_vp, _vp, ctypes.c_int64, _c_float, _vp]),
    "ttrl_blend_multi": (_c_int, [ctypes.POINTER(BlendPair), _c_int, _c_int, _c_float, _vp]),
    "ttrl_gather_rows": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _vp]),
    "ttrl_gather_rows_multi": (_c_int, [ctypes.POINTER(GatherJob), _c_int, _vp, _c_int, _vp]),
    "ttrl_dqn_loss": (_c_int, [_vp] * 13 + [_c_int, _c_int, _c_float, _c_int, _vp]),
    "ttrl_ppo_loss": (_c_int, [_vp] * 12 + [_c_int, _c_int, _c_float, _c_float, _c_float,
                                             _c_float, _vp]),
    "ttrl_sac_sample": (_c_int, [_vp] * 8 + [_c_int, _c_int, _c_int, _c_float, _c_float,
                                             _c_float, _vp, _vp, _vp, _vp]),
    "ttrl_sac_sample_backward": (_c_int, [_vp] * 5 + [ctypes.c_int64] + [_vp] * 3
                                 + [_c_int] * 4 + [_c_float, _c_float, _vp]),
    "ttrl_sac_critic_loss": (_c_int, [ctypes.POINTER(_vp), ctypes.POINTER(_vp), _c_int]
                             + [_vp] * 9 + [ctypes.POINTER(_vp), _vp, _c_int, _vp]),
    "ttrl_sac_actor_loss": (_c_int, [ctypes.POINTER(_vp), _c_int, _vp, _vp, _c_float, _vp,
                                     ctypes.POINTER(_vp), _vp, _vp, _vp, _c_int, _vp]),
    "ttrl_gru_gates_fwd": (_c_int, [_vp] * 7 + [_c_int, _c_int, _vp]),
    "ttrl_gru_gates_bwd": (_c_int, [_vp, _vp, _vp, _c_int] + [_vp] * 5 + [_c_int, _c_int, _vp]),
    "ttrl_gru_mask": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _vp]),
    "ttrl_epsilon_greedy": (_c_int, [_vp] * 6 + [_c_int, _c_int, _vp]),
    "ttrl_categorical_sample": (_c_int, [_vp] * 4 + [_c_int, _c_int, _vp]),
    "ttrl_per_update": (_c_int, [_vp, _c_int, _vp, _vp, _vp, _c_int, ctypes.c_double,
                                 ctypes.c_double, _vp, _c_int, _vp, _vp]),
    "ttrl_per_cdf": (_c_int, [_vp, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp]),
    "ttrl_per_draw": (_c_int, [_vp, _vp, _c_int, _vp, _vp, _vp, _vp, _c_int, _vp, _vp, _vp,
                               _vp]),
    "ttrl_gae": (_c_int, [_vp] * 7 + [_c_int, _c_int, _c_float, _c_float, _vp]),
    "ttrl_normalize_advantages": (_c_int, [_vp, _vp, _vp, ctypes.c_longlong, _vp, _vp]),
    "ttrl_gru_sequence_supported": (_c_int, [_c_int, _c_int]),
    "ttrl_gru_sequence_fwd": (_c_int, [_vp] * 9 + [_c_int, _c_int, _c_int, _vp]),
    "ttrl_gru_sequence_bwd": (_c_int, [_vp] * 9 + [_c_int, _c_int, _c_int, _vp]),
}

# Elementwise / reduction op codes (include/ttrl_b200.h).
EW = {name: i for i, name in enumerate((
    "add", "sub", "mul", "div", "add_s", "sub_s", "rsub_s", "mul_s", "div_s", "relu", "relu_bw",
    "abs", "sign", "neg", "exp", "log", "tanh", "sigmoid", "sqrt", "square", "eqz", "fill",
    "copy", "gt_s", "eq"))}
RED_SUM, RED_MAX, RED_ARGMAX = 0, 1, 2

EXPORTED_SYMBOLS = tuple(sorted(_SIGNATURES))

_LIB = None


def lib() -> ctypes.CDLL:
    """The loaded library, with every signature bound. Raises if absent."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: the sm_100a kernels have not been built. "
                "Run `make -C tt-rl_b200/csrc` (or __graft_entry__.build()). There is "
                "no CPU fallback."
            )
        handle = ctypes.CDLL(LIB_PATH)
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _LIB = handle
    return _LIB


def check(code: int, what: str) -> None:
    """Raise TtrlError for a non-zero return code."""
    if code != 0:
        msg = lib().ttrl_last_error().decode(errors="replace")
        raise TtrlError(code, what, msg)
