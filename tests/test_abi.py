"""The C ABI without a GPU: the library loads, exports exactly what
include/smat_b200.h declares, and rejects bad arguments on the host with the
documented status codes before touching the device."""

import ctypes
import os
import re

import numpy as np
import pytest

from smat_attention_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "smat_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"SMAT_API\s+(?:const\s+)?\w+\**\s+\**(smat_\w+)\s*\(", text)))


def test_header_symbols_exported():
    syms = declared_symbols()
    assert len(syms) == 32
    L = _lib.lib()
    for s in syms:
        assert hasattr(L, s), s
    assert set(syms) == set(_lib.SIGNATURES)


def test_version_and_status_strings():
    L = _lib.lib()
    assert L.smat_abi_version() == 6
    assert L.smat_status_string(0) == b"ok"
    assert b"CSR" in L.smat_status_string(7)
    assert L.smat_status_string(999) == b"unknown status"
    assert b"pattern" in L.smat_status_string(15)
    assert b"capture" in L.smat_status_string(16)


def _fwd(**over):
    L = _lib.lib()
    st = (ctypes.c_int64 * 3)(4 * 1024 * 64, 1024 * 64, 64)
    a = dict(dtype=1, q=16, k=16, v=16, o=16, lse=16, B=1, H=4, T=1024, D=64,
             indptr=16, indices=16, kind=16, nblocks=16, nnzb=81, block=64, max_row=6,
             scale=0.125)
    a.update(over)
    return L.smat_fwd(a["dtype"], a["q"], st, a["k"], st, a["v"], st, a["o"], st, a["lse"],
                      a["B"], a["H"], a["T"], a["D"], a["indptr"], a["indices"], a["kind"],
                      a["nblocks"], a["nnzb"], a["block"], a["max_row"], a["scale"], None, None)


@pytest.mark.parametrize("over,code", [
    (dict(B=0), 1), (dict(T=0), 1), (dict(nblocks=15), 1),
    (dict(D=96), 2), (dict(dtype=0, D=48), 2),
    (dict(block=32, nblocks=32), 3), (dict(dtype=7), 4),
    (dict(q=8), 6), (dict(q=None), 8), (dict(lse=None), 8), (dict(indptr=None), 8),
    (dict(nnzb=-1), 7), (dict(scale=float("nan")), 1),
])
def test_fwd_rejects_on_host(over, code):
    assert _fwd(**over) == code


def test_bwd_rejects_on_host():
    L = _lib.lib()
    st = (ctypes.c_int64 * 3)(0, 0, 64)
    bad = (ctypes.c_int64 * 3)(0, 0, 60)   # bf16 rows must be 16-byte aligned
    args = [1, 16, st, 16, st, 16, st, 16, st, 16, 16, 16, st, 1, 1, 128, 64,
            16, 16, 16, 2, 3, 64, 2, 0.125, None, None]
    args_bad = list(args)
    args_bad[12] = bad
    assert L.smat_bwd_dq(*args_bad) == 6
    assert L.smat_bwd_preprocess(1, 16, st, 16, st, None, 1, 1, 128, 64, None) == 8


def test_fused_dq_entry_points_reject_on_host():
    """smat_bwd_dkdv_dq / smat_bwd_dq_finish: bf16 at D = 128 only (finish: D
    64 or 128), the accumulator non-null, 16-byte aligned and B*H*T*D floats
    long; every check runs before the device is touched."""
    L = _lib.lib()
    st = (ctypes.c_int64 * 3)(0, 0, 128)
    n = 128 * 128

    def dkdv_dq(dtype=1, D=128, acc=16, n_acc=n):
        return L.smat_bwd_dkdv_dq(dtype, 16, st, 16, st, 16, st, 16, st, 16, 16, acc, n_acc,
                                  16, st, 16, st, 1, 1, 128, D, 16, 16, 16, 2, 3, 64, 2,
                                  0.125, None, None)

    assert dkdv_dq(acc=None) == 8                   # SMAT_ERR_NULL_POINTER
    assert dkdv_dq(acc=24) == 6                     # SMAT_ERR_BAD_ALIGNMENT
    assert dkdv_dq(n_acc=n - 1) == 1                # SMAT_ERR_BAD_SHAPE
    assert dkdv_dq(dtype=0) == 4                    # fp32: SMAT_ERR_UNSUPPORTED_DTYPE
    st64 = (ctypes.c_int64 * 3)(0, 0, 64)
    assert L.smat_bwd_dkdv_dq(1, 16, st64, 16, st64, 16, st64, 16, st64, 16, 16, 16, n, 16,
                              st64, 16, st64, 1, 1, 128, 64, 16, 16, 16, 2, 3, 64, 2, 0.125,
                              None, None) == 2      # D = 64: SMAT_ERR_UNSUPPORTED_D
    fin = lambda dtype=1, D=128, acc=16, stride=st: L.smat_bwd_dq_finish(
        dtype, acc, n, 16, stride, 1, 1, 128, D, 0.125, None)
    assert fin(dtype=0) == 4
    assert fin(D=96) == 2
    assert fin(acc=None) == 8
    assert fin(stride=None) == 8


def test_work_list_entry_points_reject_on_host():
    L = _lib.lib()
    st = (ctypes.c_int64 * 3)(4 * 1024 * 64, 1024 * 64, 64)
    head = [1, 16, st, 16, st, 16, st, 16, st, 16, 1, 4, 1024, 64, 16, 16, 16, 16, 81, 64, 6,
            0.125]
    # an empty list is a no-op; a missing list or a negative count is an error
    assert L.smat_fwd_tiles(*head, None, 0, None, None) == 0
    assert L.smat_fwd_tiles(*head, None, 3, None, None) == 8
    assert L.smat_fwd_tiles(*head, 16, -1, None, None) == 1
    assert L.smat_fwd_tiles(*(head[:13] + [96] + head[14:]), 16, 1, None, None) == 2
    bwd = [1, 16, st, 16, st, 16, st, 16, st, 16, 16, 16, st]
    tail = [1, 4, 1024, 64, 16, 16, 16, 16, 81, 64, 6, 0.125]
    assert L.smat_bwd_dq_tiles(*bwd, *tail, 16, -2, None, None) == 1
    assert L.smat_bwd_dq_tiles(*bwd, *tail, None, 0, None, None) == 0
    assert L.smat_bwd_dkdv_tiles(*bwd, 16, st, *tail, None, 4, None, None) == 8
    # preprocess rows must lie inside [0, T]
    assert L.smat_bwd_preprocess_rows(1, 16, st, 16, st, 16, 1, 4, 1024, 64, 0, 1025,
                                      None) == 1
    assert L.smat_bwd_preprocess_rows(1, 16, st, 16, st, 16, 1, 4, 1024, 64, 512, 256,
                                      None) == 1
    assert L.smat_bwd_preprocess_rows(1, 16, st, 16, st, 16, 1, 4, 1024, 64, 256, 256,
                                      None) == 0


def test_bwd_checks_every_pass_before_launching():
    """A bad dQ stride is reported before the preprocess would launch (on this
    GPU-less host a launch would fail with SMAT_ERR_LAUNCH instead)."""
    L = _lib.lib()
    st = (ctypes.c_int64 * 3)(0, 0, 64)
    bad = (ctypes.c_int64 * 3)(0, 0, 60)
    args = [1, 16, st, 16, st, 16, st, 16, st, 16, st, 16, 16,
            16, bad, 16, st, 16, st, 1, 1, 128, 64, 16, 16, 16, 16, 16, 16,
            2, 3, 64, 2, 2, 0.125, None, None]
    assert L.smat_bwd(*args) == 6


def test_row_exchange_rejects_on_host():
    L = _lib.lib()
    st = (ctypes.c_int64 * 3)(4 * 1024 * 64, 1024 * 64, 64)
    odd = (ctypes.c_int64 * 3)(4 * 1024 * 64, 1024 * 64, 60)
    # an empty row list is a no-op
    assert L.smat_rows_pack(1, 16, st, 16, st, 1, 4, 1024, 64, None, 0, None, None, None) == 0
    assert L.smat_rows_pack(1, 16, st, 16, st, 1, 4, 1024, 64, 16, 5, None, None, None) == 8
    assert L.smat_rows_pack(1, 16, odd, 16, st, 1, 4, 1024, 64, 16, 5, 16, None, None) == 6
    assert L.smat_rows_pack(1, 16, st, 16, st, 1, 4, 1024, 60, 16, 5, 16, None, None) == 2
    assert L.smat_rows_pack(3, 16, st, 16, st, 1, 4, 1024, 64, 16, 5, 16, None, None) == 4
    assert L.smat_rows_unpack(1, 16, st, 16, st, 0, 4, 1024, 64, 16, 5, 16, None, None) == 1
    assert L.smat_rows_accumulate(1, 16, st, 16, st, 1, 4, 1024, 64, 16, 5, None, 16, 3, 16,
                                  None, None) == 8
    assert L.smat_rows_accumulate(1, 16, st, 16, st, 1, 4, 1024, 64, 16, 5, 16, 16, -1, 16,
                                  None, None) == 1


LM_HEADER = os.path.join(os.path.dirname(HEADER), "smat_lm.h")


def test_lm_header_symbols_exported():
    from smat_attention_b200 import lm_ops
    text = open(LM_HEADER).read()
    syms = sorted(set(re.findall(r"SMAT_API\s+\w+\**\s+\**(smat_\w+)\s*\(", text)))
    assert len(syms) == 7 and set(syms) == set(lm_ops.SIGNATURES)
    L = lm_ops._L()
    for s in syms:
        assert hasattr(L, s), s


def test_lm_ops_reject_on_host():
    from smat_attention_b200 import lm_ops
    L = lm_ops._L()
    assert L.smat_lm_rmsnorm_fwd(None, None, 16, None, 16, 16, 4, 768, 1e-5, None) == 8
    assert L.smat_lm_rmsnorm_fwd(16, 16, 16, None, 16, 16, 4, 768, 1e-5, None) == 8
    assert L.smat_lm_rmsnorm_fwd(16, None, 16, None, 16, 16, 4, 700, 1e-5, None) == 1
    assert L.smat_lm_rmsnorm_fwd(16, None, 16, None, 16, 16, 4, 1280, 1e-5, None) == 1
    assert L.smat_lm_rmsnorm_fwd(8, None, 16, None, 16, 16, 4, 768, 1e-5, None) == 6
    assert L.smat_lm_rmsnorm_bwd(16, 16, 16, 16, None, 16, 16, 0, 4, 768, None) == 1
    assert L.smat_lm_rmsnorm_bwd(16, 16, 16, 16, 24, 16, 16, 4, 4, 768, None) == 6
    assert L.smat_lm_rope_split_fwd(16, 16, 16, 16, 16, 16, 1, 8, 2, 12, None) == 1
    assert L.smat_lm_rope_split_bwd(16, 16, None, 16, 16, 16, 1, 8, 2, 64, None) == 8
    assert L.smat_lm_swiglu_fwd(16, 16, 4, 12, None) == 1
    assert L.smat_lm_swiglu_bwd(16, 16, 8, 4, 16, None) == 6
    assert L.smat_lm_cross_entropy(16, 16, 16, 4, 1001, 1.0, None, None) == 1
    assert L.smat_lm_cross_entropy(16, None, 16, 4, 1000, 1.0, None, None) == 8


def test_kattn_header_symbols_exported():
    from smat_attention_b200 import kernel_attention as KA
    text = open(os.path.join(os.path.dirname(HEADER), "smat_kattn.h")).read()
    syms = sorted(set(re.findall(r"SMAT_API\s+\w+\**\s+\**(smat_\w+)\s*\(", text)))
    assert len(syms) == 12 and set(syms) == set(KA.SIGNATURES)
    L = KA._L()
    assert L.smat_kattn_chunk_local_fwd(16, 16, 16, 16, 16, 1, 64, 64, 65, None, None) == 1
    assert L.smat_kattn_chunk_local_fwd(16, 16, 16, 16, 16, 1, 128, 48, 65, None, None) == 1
    assert L.smat_kattn_chunk_local_fwd(16, 16, 16, 16, 16, 1, 128, 128, 128, None, None) == 1
    assert L.smat_kattn_chunk_local_fwd(8, 16, 16, 16, 16, 1, 128, 64, 65, None, None) == 6
    assert L.smat_kattn_chunk_local_fwd(None, 16, 16, 16, 16, 1, 128, 64, 65, None, None) == 8
    assert L.smat_kattn_pool_fwd(16, 16, 16, 1, 100, 64, 65, 0, 200, 7, None) == 1
    assert L.smat_kattn_pool_fwd(16, 16, 16, 1, 100, 256, 200, 0, 50, 7, None) == 1
    assert L.smat_kattn_incidence(16, 16, 16, 16, 0, 4, 4, 8, None, None) == 1
    assert L.smat_kattn_decode_step(16, 16, 16, 16, 16, 16, 4, 64, 1, 8, 0, None) == 1
    assert L.smat_kattn_decode_step(16, 16, 16, 16, 16, 16, 4, 64, 65, 8, 8, None) == 1
    assert L.smat_kattn_decode_step(16, 16, None, 16, 16, 16, 4, 64, 65, 8, 0, None) == 8
    assert L.smat_kattn_normalise_fwd(16, 16, 10, 1, None) == 1
    assert L.smat_kattn_normalise_bwd(16, None, 16, 10, 65, None) == 8
