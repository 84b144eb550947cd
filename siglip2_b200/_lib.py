"""ctypes binding of ``libsiglip2_b200.so`` (the C ABI in
``include/siglip2_b200.h``).  No torch types cross the boundary: callers pass
device pointers, sizes and a ``cudaStream_t`` as integers.

The library is required: importing the package on a machine where the
shared object is missing raises (there is no CPU fallback).
"""
from __future__ import annotations

import ctypes
import os

from .build import LIB_PATH

_c_int, _c_float, _vp = ctypes.c_int, ctypes.c_float, ctypes.c_void_p

# name -> (restype, argtypes); every function in include/siglip2_b200.h
SIGNATURES = {
    "siglip2_version": (_c_int, []),
    "siglip2_last_error": (ctypes.c_char_p, []),
    "siglip2_check_device": (_c_int, [_c_int]),
    "siglip2_launch_count": (ctypes.c_ulonglong, []),
    "siglip2_set_gemm_variant": (_c_int, [_c_int]),
    "siglip2_selftest_wait_timeout": (_c_int, [ctypes.c_longlong, _vp]),
    "siglip2_get_gemm_variant": (_c_int, []),
    "siglip2_set_fmha_variant": (_c_int, [_c_int]),
    "siglip2_get_fmha_variant": (_c_int, []),
    "siglip2_gemm": (_c_int, [_c_int, _c_int, _vp, _c_int, _vp, _c_int, _vp, _c_int, _c_int, _c_int, _c_int,
                              _vp, _vp, _c_int, _vp, _vp, _c_float, _vp]),
    "siglip2_gemm_rowsums": (_c_int, [_c_int, _c_int, _vp, _c_int, _vp, _c_int, _vp, _c_int, _c_int, _c_int, _c_int,
                                      _vp, _vp, _c_int, _vp, _vp, _c_float, _vp, _vp, _vp]),
    "siglip2_gemm_t": (_c_int, [_c_int, _c_int, _c_int, _c_int, _vp, _c_int, _vp, _c_int, _vp, _c_int, _c_int,
                                _c_int, _c_int, _vp, _vp, _c_int, _vp]),
    "siglip2_rowsum_slots": (_c_int, [_c_int, _c_int]),
    "siglip2_rowsum_block": (_c_int, [_c_int, _c_int]),
    "siglip2_rowsums": (_c_int, [_c_int, _vp, _c_int, _c_int, _c_int, _vp, _vp]),
    "siglip2_patch_embed": (_c_int, [_c_int, _vp, _c_int, _vp, _vp, _vp, _c_int, _vp, _vp, _vp, _c_int, _c_int, _vp,
                                     _vp, _vp]),
    "siglip2_layernorm": (_c_int, [_c_int, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_float, _vp, _c_int, _vp]),
    "siglip2_layernorm_backward": (_c_int, [_c_int, _vp, _vp, _vp, _c_int, _c_int, _c_float, _vp, _vp, _vp, _vp,
                                            _c_int, _vp]),
    "siglip2_token_image": (_c_int, [_vp, _c_int, _c_int, _vp, _vp]),
    "siglip2_image_grid": (_c_int, [_c_int, _c_int, _c_int, _c_int, _vp, _vp]),
    "siglip2_l2_normalize": (_c_int, [_c_int, _vp, _c_int, _c_int, _c_int, _c_float, _vp, _c_int, _vp]),
    "siglip2_patchify": (_c_int, [_c_int, _vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp,
                                  _c_int, _vp, _vp, _vp]),
    "siglip2_posemb": (_c_int, [_c_int, _vp, _c_int, _c_int, _vp, _vp, _vp, _c_int, _vp, _vp]),
    "siglip2_fmha_varlen": (_c_int, [_c_int, _vp, _c_int, _vp, _vp, _c_int, _c_int, _c_int, _vp, _c_int, _vp]),
    "siglip2_fmha_varlen_dropout": (_c_int, [_c_int, _vp, _c_int, _vp, _vp, _c_int, _c_int, _c_int, _vp, _c_int,
                                             _c_float, ctypes.c_ulonglong, ctypes.c_ulonglong, _vp]),
    "siglip2_dropout": (_c_int, [_c_int, _vp, _c_int, _c_int, _c_int, _c_float, ctypes.c_ulonglong,
                                 ctypes.c_ulonglong, _vp, _c_int, _vp]),
    "siglip2_fmha_varlen_train": (_c_int, [_c_int, _vp, _c_int, _vp, _vp, _c_int, _c_int, _c_int, _vp, _c_int, _vp,
                                           _c_float, ctypes.c_ulonglong, ctypes.c_ulonglong, _vp]),
    "siglip2_fmha_bwd_dsum": (_c_int, [_c_int, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp]),
    "siglip2_fmha_varlen_backward": (_c_int, [_c_int, _vp, _vp, _c_int, _c_int, _vp, _vp, _c_int, _c_int, _c_int,
                                              _vp, _vp, _vp, _vp]),
    "siglip2_colsum_partial": (_c_int, [_c_int, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp]),
    "siglip2_gemm_t_workspace_size": (ctypes.c_size_t, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int]),
    "siglip2_gemm_t_ws": (_c_int, [_c_int, _c_int, _c_int, _c_int, _vp, _c_int, _vp, _c_int, _vp, _c_int, _c_int,
                                   _c_int, _c_int, _vp, _vp, ctypes.c_size_t, _vp]),
    "siglip2_quantize_e4m3": (_c_int, [_c_int, _vp, _c_int, _c_int, _c_int, _vp, _c_int, _vp, _vp]),
    "siglip2_gemm_e4m3": (_c_int, [_c_int, _c_int, _vp, _c_int, _vp, _vp, _c_int, _vp, _vp, _c_int, _c_int, _c_int,
                                   _c_int, _vp, _vp, _c_int, _vp]),
    "siglip2_padded_head_dim": (_c_int, [_c_int]),
    "siglip2_head_pool": (_c_int, [_c_int, _vp, _c_int, _c_int, _vp, _c_int, _c_int, _vp, _vp, _vp, _vp]),
    "siglip2_head_pool_noalloc": (_c_int, [_c_int, _vp, _c_int, _c_int, _vp, _c_int, _c_int, _c_int, _vp, _vp,
                                           _vp]),
    "siglip2_metadata_size": (_c_int, [_vp, _c_int, _vp, _vp]),
    "siglip2_metadata": (_c_int, [_vp, _c_int, _vp, ctypes.c_size_t]),
    "siglip2_workspace_size": (ctypes.c_size_t, [_vp, _c_int, _c_int]),
    "siglip2_forward": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
}


class Config(ctypes.Structure):
    """``siglip2_config``"""
    _fields_ = [("hidden", _c_int), ("intermediate", _c_int), ("layers", _c_int), ("heads", _c_int),
                ("head_dim", _c_int), ("patch_dim", _c_int), ("pos_grid", _c_int), ("eps", _c_float),
                ("dtype", _c_int), ("has_head", _c_int)]


class LayerWeights(ctypes.Structure):
    """``siglip2_layer_weights``"""
    _fields_ = [(n, _vp) for n in ("qkv_w", "qkv_c1", "qkv_c2", "out_w", "out_b", "fc1_w", "fc1_c1", "fc1_c2",
                                   "fc2_w", "fc2_b")]


class Weights(ctypes.Structure):
    """``siglip2_weights``"""
    _fields_ = [("patch_w", _vp), ("patch_b", _vp), ("pos_table", _vp), ("layers", ctypes.POINTER(LayerWeights)),
                ("post_ln_w", _vp), ("post_ln_b", _vp), ("head_u", _vp), ("head_v_w", _vp), ("head_v_b", _vp),
                ("head_o_w", _vp), ("head_o_b", _vp), ("head_fc1_w", _vp), ("head_fc1_c1", _vp),
                ("head_fc1_c2", _vp), ("head_fc2_w", _vp), ("head_fc2_b", _vp)]

STATUS = {0: "OK", -1: "ERR_ARG", -2: "ERR_ALIGN", -3: "ERR_SHAPE", -4: "ERR_CUDA", -5: "ERR_TIMEOUT",
          -6: "ERR_UNSUPPORTED"}

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
EPI_BIAS, EPI_BIAS_RES, EPI_LN, EPI_LN_GELU, EPI_BIAS_GELU = 0, 1, 2, 3, 4
EPI_LN_ROWSUMS, EPI_LN_ROWSUMS_GELU, EPI_BIAS_RES_ROWSUMS = 5, 6, 7
EPI_BIAS_GELU_GRAD = 9

_lib = None


class Siglip2Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"siglip2 {STATUS.get(code, code)}: {msg}")
        self.code = code


def load(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and type the shared library.  Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or os.environ.get("SIGLIP2_B200_LIB", LIB_PATH)
    if not os.path.exists(path):
        raise ImportError(f"{path} not found: build it with `python -m siglip2_b200.build` "
                          f"(the CUDA library is required; there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(code: int) -> None:
    if code != 0:
        raise Siglip2Error(code, load().siglip2_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))


def check_value(value: int) -> int:
    """For entry points that return a count or a negative status code."""
    if value < 0:
        check(value)
    return value
