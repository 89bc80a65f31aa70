"""ctypes binding of ``libsmat_b200.so`` (the C ABI in ``include/smat_b200.h``).

This is the only way the package reaches its kernels.  If the library is
missing the import of the op fails loudly; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsmat_b200.so")

DTYPE_F32 = 0
DTYPE_BF16 = 1

# work items of the *_tiles entry points: tile index in bits 0..23, bit 24 =
# "also the next tile" (forward only)
WORK_PAIR_BIT = 1 << 24
TILE_ROWS = 128

# tile kinds and M^(d) families (include/smat_b200.h)
TILE_FULL, TILE_CAUSAL, TILE_PATTERN = 0, 1, 2
FAMILY_GEOMETRIC, FAMILY_ENDPOINT = 0, 1


class Pattern(ctypes.Structure):
    """``smat_pattern_t``: the M^(d) mask of a layout's PATTERN tiles."""

    _fields_ = [("family", ctypes.c_int), ("n", ctypes.c_int), ("n_P", ctypes.c_int),
                ("B", ctypes.c_int), ("N0", ctypes.c_int), ("row_words", ctypes.c_int),
                ("col_words", ctypes.c_int), ("row_bits", ctypes.c_void_p),
                ("col_bits", ctypes.c_void_p)]


_c_int, _c_i64, _c_f = ctypes.c_int, ctypes.c_int64, ctypes.c_float
_vp = ctypes.c_void_p
_i64p = ctypes.POINTER(ctypes.c_int64)

# symbol -> (restype, argtypes); mirrors include/smat_b200.h
SIGNATURES = {
    "smat_abi_version": (_c_int, []),
    "smat_status_string": (ctypes.c_char_p, [_c_int]),
    "smat_device_supported": (_c_int, [_c_int]),
    "smat_layout_build_block": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int,
                                         _vp, _vp, _vp, _c_i64, _i64p]),
    "smat_layout_transpose": (_c_int, [_c_int, _vp, _vp, _vp, _vp, _vp, _vp]),
    "smat_layout_validate": (_c_int, [_c_int, _c_i64, _vp, _vp, _vp, _c_int,
                                      ctypes.POINTER(ctypes.c_int32)]),
    "smat_fwd": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp,
                          _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                          _c_int, _c_i64, _c_int, _c_int, _c_f, _vp, _vp]),
    # smat_fwd plus (work, n_work) before err_word
    "smat_fwd_tiles": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp,
                                _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                                _c_int, _c_i64, _c_int, _c_int, _c_f, _vp, _c_int, _vp, _vp]),
    "smat_rows_pack": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _c_int, _c_int, _c_int,
                                _c_int, _vp, _c_i64, _vp, _vp, _vp]),
    "smat_rows_unpack": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _c_int, _c_int, _c_int,
                                  _c_int, _vp, _c_i64, _vp, _vp, _vp]),
    "smat_rows_accumulate": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _c_int, _c_int, _c_int,
                                      _c_int, _vp, _c_i64, _vp, _vp, _c_i64, _vp, _vp, _vp]),
    "smat_bwd_preprocess": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp,
                                     _c_int, _c_int, _c_int, _c_int, _vp]),
    "smat_bwd_preprocess_rows": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp,
                                          _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp]),
    "smat_bwd_dkdv": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                               _vp, _vp, _vp, _i64p, _vp, _i64p,
                               _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                               _c_int, _c_i64, _c_int, _c_int, _c_f, _vp, _vp]),
    "smat_bwd_dkdv_tiles": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                                     _vp, _vp, _vp, _i64p, _vp, _i64p,
                                     _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                                     _c_int, _c_i64, _c_int, _c_int, _c_f, _vp, _c_int,
                                     _vp, _vp]),
    "smat_bwd_dq": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                             _vp, _vp, _vp, _i64p,
                             _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                             _c_int, _c_i64, _c_int, _c_int, _c_f, _vp, _vp]),
    "smat_bwd_dq_tiles": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                                   _vp, _vp, _vp, _i64p,
                                   _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                                   _c_int, _c_i64, _c_int, _c_int, _c_f, _vp, _c_int, _vp, _vp]),
    "smat_bwd": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                          _vp, _vp, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                          _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _vp,
                          _c_int, _c_i64, _c_int, _c_int, _c_int, _c_f, _vp, _vp]),
    # fused backward: dK/dV plus the fp32 dQ accumulator, the dQ finish, and
    # smat_bwd with the pattern and the accumulator before scale
    "smat_bwd_dkdv_dq": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                                  _vp, _vp, _vp, _c_i64, _vp, _i64p, _vp, _i64p,
                                  _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                                  _c_int, _c_i64, _c_int, _c_int, _c_f, _vp, _vp]),
    "smat_bwd_dq_finish": (_c_int, [_c_int, _vp, _c_i64, _vp, _i64p,
                                    _c_int, _c_int, _c_int, _c_int, _c_f, _vp]),
    "smat_bwd_acc": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp,
                              _i64p, _vp, _vp, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                              _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _vp,
                              _c_int, _c_i64, _c_int, _c_int, _c_int,
                              ctypes.POINTER(Pattern), _vp, _c_i64, _c_f, _vp, _vp]),
    "smat_pattern_tables": (_c_int, [_c_int, _c_int, _vp, _vp, _vp, _c_int, _vp, _c_int]),
    "smat_layout_build_pattern": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                           _vp, _vp, _vp, _c_i64, _i64p]),
    "smat_layout_validate_pattern": (_c_int, [_c_int, _c_i64, _vp, _vp, _vp, _c_int,
                                              ctypes.POINTER(ctypes.c_int32)]),
    "smat_pattern_mask_rows": (_c_int, [ctypes.POINTER(Pattern), _c_int, _c_int, _c_int, _vp]),
    "smat_pattern_mask_cols": (_c_int, [ctypes.POINTER(Pattern), _c_int, _c_int, _c_int, _vp]),
    # smat_fwd / smat_bwd plus the pattern before scale
    "smat_fwd_pattern": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp,
                                  _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                                  _c_int, _c_i64, _c_int, _c_int, ctypes.POINTER(Pattern),
                                  _c_f, _vp, _vp]),
    "smat_bwd_pattern": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp,
                                  _i64p, _vp, _vp, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                                  _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _vp,
                                  _c_int, _c_i64, _c_int, _c_int, _c_int,
                                  ctypes.POINTER(Pattern), _c_f, _vp, _vp]),
    "smat_decode_workspace": (_c_int, [_c_int, _c_int, _c_int, _c_int, _i64p]),
    "smat_decode": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _vp,
                             _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp,
                             _c_int, _c_i64, _c_int, _c_int, ctypes.POINTER(Pattern),
                             _c_f, _vp, _c_i64, _vp, _vp]),
    "smat_selftest_wait_timeout": (_c_int, [_c_i64, _vp, _vp, _vp]),
    # smat_bwd without the delta workspace (fixed in-library scratch)
    "smat_bwd_noalloc": (_c_int, [_c_int, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp,
                                  _i64p, _vp, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                                  _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _vp,
                                  _c_int, _c_i64, _c_int, _c_int, _c_int, _c_f, _vp, _vp]),
}

_lock = threading.Lock()
_lib = None


class SmatError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, fn: str, status: int, text: str):
        super().__init__(f"{fn} failed: {text} (status {status})")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load the library once and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with "
                    f"`python -m smat_attention_b200.build` (needs nvcc)")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                f = getattr(L, name)
                f.restype, f.argtypes = res, args
            _lib = L
    return _lib


def check(fn: str, status: int) -> None:
    if status != 0:
        text = lib().smat_status_string(status).decode()
        raise SmatError(fn, status, text)


def strides3(t) -> ctypes.Array:
    """Host int64[3] with the (b, h, t) element strides of a [B, H, T, D] tensor."""
    s = t.stride()
    return (ctypes.c_int64 * 3)(s[0], s[1], s[2])
