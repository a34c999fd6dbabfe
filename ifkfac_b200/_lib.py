"""ctypes binding of libifk.so (the C ABI declared in include/ifk.h).

The library is loaded from this package directory; it is built in-tree by
``python -m ifkfac_b200.build``.  There is no fallback: when the library is
missing or the device is not an sm_100 part, every call raises.
"""
from __future__ import annotations

import ctypes
import os
import re
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libifk.so")
HEADER = os.path.join(os.path.dirname(PKG_DIR), "include", "ifk.h")

OK, ERR_RANK, ERR_NONFINITE, ERR_SHAPE, ERR_TIMEOUT, ERR_CUDA, ERR_WORKSPACE, ERR_DTYPE, \
    ERR_ARG, ERR_DEVICE, ERR_LIMIT = range(11)
NOALLOC_MAX_N = 4096
F32, BF16 = 0, 1
PREC_AUTO, PREC_FP32, PREC_BF16 = 0, 1, 2
FOLD_TRAPEZOIDAL_CHUNK = 1
FOLD_DEBUG_WITHHOLD = 256  # tests of the failure path only

_i64, _sz, _vp, _int, _dbl = ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int, ctypes.c_double

# name -> (restype, argtypes); mirrors include/ifk.h
SIGNATURES = {
    "ifk_version": (ctypes.c_char_p, []),
    "ifk_status_string": (ctypes.c_char_p, [_int]),
    "ifk_device_check": (_int, []),
    "ifk_tsqr_fold_workspace": (_sz, [_i64, _i64]),
    "ifk_tsqr_fold": (_int, [_vp, _i64, _i64, _vp, _i64, _i64, _i64, _int, _int, _int, _vp, _vp, _sz,
                             _vp]),
    "ifk_tsqr_fold_batched_workspace": (_sz, [_int, _vp, _vp]),
    "ifk_tsqr_fold_batched": (_int, [_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _int, _vp,
                                     _vp, _sz, _vp]),
    "ifk_tsqr_fold_segments_workspace": (_sz, [_int, _vp, _vp, _vp, _vp]),
    "ifk_tsqr_fold_segments_fp32_workspace": (_sz, [_int, _vp, _vp, _vp, _vp]),
    "ifk_tsqr_fold_segments": (_int, [_int, _vp, _vp, _vp, _vp, _vp, _vp, _int, _vp, _int, _vp, _vp, _sz, _vp]),
    "ifk_rtree_merge_workspace": (_sz, [_int, _i64]),
    "ifk_rtree_merge": (_int, [_int, _vp, _vp, _vp, _i64, _int, _vp, _vp, _vp, _sz, _vp]),
    "ifk_finalize_workspace": (_sz, [_i64]),
    "ifk_finalize_batched_workspace": (_sz, [_int, _vp]),
    "ifk_finalize_batched": (_int, [_int, _vp, _vp, _vp, _vp, _vp, _dbl, _vp, _vp, _int, _int, _vp,
                                    _vp, _sz, _vp]),
    "ifk_finalize_many": (_int, [_int, _vp, _vp, _vp, _vp, _vp, _dbl, _vp, _vp, _int, _int, _vp, _vp, _sz, _vp]),
    "ifk_finalize": (_int, [_vp, _i64, _i64, _i64, _dbl, _dbl, _vp, _i64, _int, _int, _vp, _vp, _sz,
                            _vp]),
    "ifk_natgrad_workspace": (_sz, [_i64, _i64]),
    "ifk_natgrad": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _int, _vp, _i64, _i64, _i64, _int, _vp,
                           _vp, _sz, _vp]),
    "ifk_natgrad_update_workspace": (_sz, [_i64, _i64]),
    "ifk_natgrad_update": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _int, _vp, _vp, _i64, _i64, _dbl, _dbl, _dbl,
                                  _int, _int, _vp, _vp, _sz, _vp]),
    "ifk_posterior_sample_workspace": (_sz, [_i64, _i64]),
    "ifk_posterior_sample": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _int, _vp, _i64, _i64, _i64, _int, _vp,
                                    _vp, _sz, _vp]),
    "ifk_natgrad_noalloc": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _int, _vp, _i64, _i64, _i64, _int,
                                   _vp, _vp]),
    "ifk_natgrad_batched_workspace": (_sz, [_int, _vp, _vp]),
    "ifk_natgrad_batched": (_int, [_int, _vp, _vp, _vp, _vp, _vp, _vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _int,
                                   _vp, _vp, _sz, _vp]),
    "ifk_natgrad_bias": (_int, [_vp, _vp, _i64, _int, _vp, _i64, _int, _vp, _sz, _vp]),
    "ifk_update_workspace": (_sz, [_i64]),
    "ifk_update": (_int, [_vp, _vp, _vp, _i64, _dbl, _dbl, _dbl, _dbl, _int, _vp, _sz, _vp]),
    "ifk_update_bias": (_int, [_vp, _vp, _i64, _dbl, _dbl, _vp]),
}


PER_SEGMENT_DTYPE = -1  # chunk_dtype of ifk_tsqr_fold_segments: each segment's own


class Conv2d(ctypes.Structure):
    """``ifk_conv2d`` of include/ifk.h: im2col geometry of an NCHW image segment."""
    _fields_ = [("batch", ctypes.c_int64), ("channels", ctypes.c_int64), ("height", ctypes.c_int64),
                ("width", ctypes.c_int64), ("kernel_h", ctypes.c_int32), ("kernel_w", ctypes.c_int32),
                ("stride_h", ctypes.c_int32), ("stride_w", ctypes.c_int32), ("pad_h", ctypes.c_int32),
                ("pad_w", ctypes.c_int32), ("dilation_h", ctypes.c_int32), ("dilation_w", ctypes.c_int32)]


class Segment(ctypes.Structure):
    """``ifk_segment`` of include/ifk.h: rows of a chunk for ifk_tsqr_fold_segments."""
    _fields_ = [("chunk", ctypes.c_void_p), ("ld", ctypes.c_int64), ("rows", ctypes.c_int64),
                ("row_index", ctypes.c_void_p), ("src_rows", ctypes.c_int64), ("cols", ctypes.c_int64),
                ("dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("conv", ctypes.POINTER(Conv2d))]


class IFKError(RuntimeError):
    """A libifk call returned a non-zero status."""

    def __init__(self, status: int, where: str):
        self.status = status
        msg = status_string(status) if _LIB is not None else str(status)
        super().__init__(f"{where}: {msg} (status {status})")


_LIB = None
_LOCK = threading.Lock()


def header_symbols() -> list:
    """Names of the entry points declared in include/ifk.h."""
    with open(HEADER) as f:
        return re.findall(r"IFK_API\s+[\w\s\*]+?\b(ifk_\w+)\s*\(", f.read())


def lib() -> ctypes.CDLL:
    """Load libifk.so once and attach the C signatures."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is not built (python -m ifkfac_b200.build)")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _LIB = L
    return _LIB


def status_string(status: int) -> str:
    return lib().ifk_status_string(int(status)).decode()


def check(status: int, where: str) -> None:
    if status != OK:
        raise IFKError(status, where)
