"""The block layout: vectorised builder vs the naive oracle restatement,
hand-written known answers, the C builder / transposer / validator in
libsmat_b200.so, and the counts every effective-FLOP figure rests on."""

import ctypes

import numpy as np
import pytest

from oracle import layout as OL
from smat_attention_b200 import _lib
from smat_attention_b200.mask import (KIND_CAUSAL, KIND_FULL, block_layout_stats,
                                      build_block_mask, materialise)

CONFIGS = {  # BASELINE configs c1..c5: (T, bs, W, S, sinks)
    "c1": (1024, 64, 4, 0, 1), "c2": (4096, 64, 8, 16, 1), "c3": (16384, 128, 4, 8, 2),
    "c4": (8192, 64, 8, 16, 1), "c5": (131072, 128, 8, 32, 4),
}
EDGE = [(1, 64, 0, 0, 0), (63, 64, 2, 0, 0), (200, 32, 1, 2, 1), (1000, 64, 3, 5, 2),
        (640, 64, 0, 1, 0), (640, 64, 0, 0, 100), (512, 16, 100, 0, 0), (129, 128, 1, 1, 1),
        (4096, 128, 0, 3, 0), (300, 7, 2, 4, 3)]


@pytest.mark.parametrize("args", list(CONFIGS.values())[:4] + EDGE)
def test_csr_matches_oracle(args):
    s = build_block_mask(*args)
    ip, ix, kd = OL.block_csr(*args)
    assert np.array_equal(s.indptr, ip) and s.indptr.dtype == np.int32
    assert np.array_equal(s.indices, ix) and s.indices.dtype == np.int32
    assert np.array_equal(s.tile_kind, kd) and s.tile_kind.dtype == np.uint8
    tip, tix, tkd = OL.transposed_csr(*args)
    assert np.array_equal(s.t_indptr, tip)
    assert np.array_equal(s.t_indices, tix)
    assert np.array_equal(s.t_kind, tkd)


@pytest.mark.parametrize("args", EDGE + [CONFIGS["c1"]])
def test_dense_matches_oracle(args):
    assert np.array_equal(materialise(build_block_mask(*args)), OL.dense_mask(*args))


def test_known_answers():
    s = build_block_mask(*CONFIGS["c1"])
    assert list(s.indices[s.indptr[10]:s.indptr[11]]) == [0, 6, 7, 8, 9, 10]
    assert list(s.indices[s.indptr[0]:s.indptr[1]]) == [0]
    assert list(s.tile_kind[s.indptr[10]:s.indptr[11]]) == [KIND_FULL] * 5 + [KIND_CAUSAL]
    s = build_block_mask(*CONFIGS["c2"])   # W=8, S=16, 1 sink
    assert list(s.indices[s.indptr[40]:s.indptr[41]]) == [0, 15, 31] + list(range(32, 41))
    s = build_block_mask(*CONFIGS["c3"])   # W=4, S=8, 2 sinks
    assert list(s.indices[s.indptr[20]:s.indptr[21]]) == [0, 1, 7, 15] + list(range(16, 21))
    # key block 0 (a sink) is read by every query block
    assert list(s.t_indices[s.t_indptr[0]:s.t_indptr[1]]) == list(range(128))


# counts from the survey of the BASELINE configs (active tiles, longest row,
# unmasked pairs per head)
@pytest.mark.parametrize("name,tiles,max_row,pairs", [
    ("c1", 81, 6, 299_520), ("c2", 667, 13, 2_603_008), ("c3", 1775, 22, 28_041_216),
    ("c4", 1627, 17, 6_406_144), ("c5", 28_858, 44, 464_486_400)])
def test_counts(name, tiles, max_row, pairs):
    st = block_layout_stats(build_block_mask(*CONFIGS[name]))
    assert (st["tiles"], st["max_row"], st["pairs"]) == (tiles, max_row, pairs)
    if name != "c5":
        assert st["pairs"] == OL.unmasked_pairs(*CONFIGS[name])


@pytest.mark.parametrize("args", list(CONFIGS.values()) + EDGE)
def test_c_builder_transposer_validator(args):
    L = _lib.lib()
    T, bs, W, S, ns = args
    s = build_block_mask(*args)
    nb = s.nqb
    n = ctypes.c_int64(0)
    _lib.check("count", L.smat_layout_build_block(T, bs, W, S, ns, None, None, None, 0,
                                                   ctypes.byref(n)))
    assert n.value == s.nnzb
    ip = np.zeros(nb + 1, np.int32)
    ix = np.zeros(n.value, np.int32)
    kd = np.zeros(n.value, np.uint8)
    _lib.check("build", L.smat_layout_build_block(T, bs, W, S, ns, ip.ctypes.data, ix.ctypes.data,
                                                   kd.ctypes.data, n.value, ctypes.byref(n)))
    assert np.array_equal(ip, s.indptr) and np.array_equal(ix, s.indices)
    assert np.array_equal(kd, s.tile_kind)
    tip = np.zeros(nb + 1, np.int32)
    tix = np.zeros(n.value, np.int32)
    tkd = np.zeros(n.value, np.uint8)
    _lib.check("transpose", L.smat_layout_transpose(nb, ip.ctypes.data, ix.ctypes.data,
                                                     kd.ctypes.data, tip.ctypes.data,
                                                     tix.ctypes.data, tkd.ctypes.data))
    assert np.array_equal(tip, s.t_indptr) and np.array_equal(tix, s.t_indices)
    assert np.array_equal(tkd, s.t_kind)
    mr = ctypes.c_int32(-1)
    _lib.check("validate", L.smat_layout_validate(nb, n.value, ip.ctypes.data, ix.ctypes.data,
                                                   kd.ctypes.data, 0, ctypes.byref(mr)))
    assert mr.value == s.max_row
    _lib.check("validate_t", L.smat_layout_validate(nb, n.value, tip.ctypes.data,
                                                     tix.ctypes.data, tkd.ctypes.data, 1, None))


def _validate(ip, ix, kd, transposed=0):
    L = _lib.lib()
    ip, ix, kd = (np.ascontiguousarray(a) for a in (ip, ix, kd))
    return L.smat_layout_validate(len(ip) - 1, ix.size, ip.ctypes.data, ix.ctypes.data,
                                  kd.ctypes.data, transposed, None)


def test_validator_rejects_corruption():
    s = build_block_mask(1000, 64, 3, 5, 2)
    good = (s.indptr.copy(), s.indices.copy(), s.tile_kind.copy())
    assert _validate(*good) == 0
    bad_ix = good[1].copy(); bad_ix[5] = 99            # out of range
    bad_ord = good[1].copy(); bad_ord[[1, 2]] = bad_ord[[2, 1]]   # not ascending
    bad_kind = good[2].copy(); bad_kind[0] ^= 1        # wrong kind on the diagonal
    bad_ptr = good[0].copy(); bad_ptr[3] = bad_ptr[4] + 1   # decreasing
    future = good[1].copy(); future[s.indptr[2]] = 3   # key block after the query block
    for ip, ix, kd in [(good[0], bad_ix, good[2]), (good[0], bad_ord, good[2]),
                       (good[0], good[1], bad_kind), (bad_ptr, good[1], good[2]),
                       (good[0], future, good[2])]:
        assert _validate(ip, ix, kd) == 7    # SMAT_ERR_CSR_INVALID
    assert _validate(s.t_indptr, s.t_indices, s.t_kind, 1) == 0
    assert _validate(s.t_indptr, s.t_indices, s.t_kind, 0) == 7


def test_bad_arguments():
    for args in [(0, 64, 1, 0, 0), (64, 0, 1, 0, 0), (64, 64, -1, 0, 0), (64, 64, 0, -1, 0)]:
        with pytest.raises(ValueError):
            build_block_mask(*args)
