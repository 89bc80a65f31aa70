"""M^(d) masks as pattern layouts, without a GPU.

The reference's own mask family runs through the softmax kernels as a tiled
layout whose PATTERN tiles the kernels mask element by element from bit
tables of the incidence C (smat_attention_b200/csrc/pattern.cuh).  Pinned here
against the reference's materialise (src/smat/mask.py:557-577) through the
fixtures of tests/golden/mask_md.npz (dense-mask SHA-256 digests written by
tests/golden/make_golden.py from the reference itself):

* the numpy layout builder tiles exactly the dense mask (every tile left out is
  all zeros, every FULL / CAUSAL tile is what its kind says);
* the C builder (smat_layout_build_pattern) and table builder
  (smat_pattern_tables) agree with the numpy ones entry for entry;
* the kernels' word rule, compiled for the host (smat_pattern_mask_rows for
  the row words of the forward and dQ kernels, smat_pattern_mask_cols for the
  column words of dK/dV), reproduces the reference's dense mask bit for bit.
"""

import ctypes
import hashlib
import os

import numpy as np
import pytest

from smat_attention_b200 import _lib
from smat_attention_b200.mask import (KIND_CAUSAL, KIND_FULL, KIND_PATTERN, block_layout_stats,
                                      build_mask, materialise, pattern_layout)

GOLD = os.path.join(os.path.dirname(__file__), "golden", "mask_md.npz")
FIX = np.load(GOLD)
N_CASES = int(FIX["n_cases"])


def _spec(i):
    T, d, chunk, nP = (int(x) for x in FIX[f"c{i}_args"])
    return build_mask(T, d, chunk=chunk, n_P=nP)


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _pattern(s, lay):
    rb, cb = lay.row_bits, lay.col_bits
    fam = _lib.FAMILY_ENDPOINT if s.kind == "endpoint" else _lib.FAMILY_GEOMETRIC
    return _lib.Pattern(fam, s.n, s.n_P, s.B, s.N0, rb.shape[1], cb.shape[1],
                        rb.ctypes.data, cb.ctypes.data)


def _rule_rows(s, lay, lo, hi, cols=False):
    L = _lib.lib()
    out = np.zeros((hi - lo, s.T), np.uint8)
    pt = _pattern(s, lay)
    fn = L.smat_pattern_mask_cols if cols else L.smat_pattern_mask_rows
    _lib.check("mask", fn(ctypes.byref(pt), s.T, lo, hi, out.ctypes.data))
    return out


SMALL = [i for i in range(N_CASES) if int(FIX[f"c{i}_args"][0]) <= 4096]


@pytest.mark.parametrize("i", SMALL)
@pytest.mark.parametrize("bs", [64, 128, 48])
def test_layout_tiles_dense_mask(i, bs):
    s = _spec(i)
    dense = materialise(s, np.uint8)
    assert _sha(dense) == str(FIX[f"c{i}_dense_sha256"])
    lay = pattern_layout(s, bs)
    assert lay.kind == "pattern" and lay.block == bs
    assert np.array_equal(materialise(lay, np.uint8), dense)
    assert block_layout_stats(lay)["pairs"] == int(dense.sum())
    # per row: ascending, causal, diagonal present and last
    for qb in range(lay.nqb):
        row = lay.indices[lay.indptr[qb]:lay.indptr[qb + 1]]
        assert row.size and row[-1] == qb and np.all(np.diff(row) > 0)
    # kinds: CAUSAL only on the diagonal, FULL only off it; a FULL tile is all ones
    row_of = np.repeat(np.arange(lay.nqb), np.diff(lay.indptr))
    diag = lay.indices == row_of
    assert not np.any((lay.tile_kind == KIND_CAUSAL) & ~diag)
    assert not np.any((lay.tile_kind == KIND_FULL) & diag)
    assert set(np.unique(lay.tile_kind)) <= {KIND_FULL, KIND_CAUSAL, KIND_PATTERN}
    # a cached layout per block size
    assert pattern_layout(s, bs) is lay


@pytest.mark.parametrize("i", SMALL)
@pytest.mark.parametrize("bs", [64, 128, 48])
def test_c_builder_matches(i, bs):
    s = _spec(i)
    lay = pattern_layout(s, bs)
    L = _lib.lib()
    fam = _lib.FAMILY_ENDPOINT if s.kind == "endpoint" else _lib.FAMILY_GEOMETRIC
    c_all = int(s.dense_C().all())
    nnz = ctypes.c_int64(0)
    _lib.check("count", L.smat_layout_build_pattern(s.T, bs, fam, s.n, s.n_P, c_all, None, None,
                                                    None, 0, ctypes.byref(nnz)))
    assert nnz.value == lay.nnzb
    ip = np.zeros(lay.nqb + 1, np.int32)
    ix = np.zeros(lay.nnzb, np.int32)
    kd = np.zeros(lay.nnzb, np.uint8)
    _lib.check("build", L.smat_layout_build_pattern(s.T, bs, fam, s.n, s.n_P, c_all,
                                                    ip.ctypes.data, ix.ctypes.data,
                                                    kd.ctypes.data, lay.nnzb, ctypes.byref(nnz)))
    assert np.array_equal(ip, lay.indptr) and np.array_equal(ix, lay.indices)
    assert np.array_equal(kd, lay.tile_kind)
    # capacity too small
    assert L.smat_layout_build_pattern(s.T, bs, fam, s.n, s.n_P, c_all, ip.ctypes.data,
                                       ix.ctypes.data, kd.ctypes.data, lay.nnzb - 1,
                                       ctypes.byref(nnz)) == 13
    # both CSRs pass the pattern validator and fail the block one
    mr = ctypes.c_int32(0)
    for ptr, idx, knd, tr in ((lay.indptr, lay.indices, lay.tile_kind, 0),
                              (lay.t_indptr, lay.t_indices, lay.t_kind, 1)):
        assert L.smat_layout_validate_pattern(lay.nqb, idx.size, ptr.ctypes.data,
                                              idx.ctypes.data, knd.ctypes.data, tr,
                                              ctypes.byref(mr)) == 0
        if (knd == KIND_PATTERN).any():
            assert L.smat_layout_validate(lay.nqb, idx.size, ptr.ctypes.data, idx.ctypes.data,
                                          knd.ctypes.data, tr, None) == 7
    assert mr.value == lay.max_row or tr == 1


@pytest.mark.parametrize("i", range(N_CASES))
def test_tables_match(i):
    s = _spec(i)
    lay = pattern_layout(s, 128)
    L = _lib.lib()
    rw, cw = lay.row_bits.shape[1], lay.col_bits.shape[1]
    assert rw == (s.N0 + 63) // 32 and cw == (s.B + 63) // 32
    rb = np.zeros((s.B, rw), np.uint32)
    cb = np.zeros((s.N0, cw), np.uint32)
    _lib.check("tables", L.smat_pattern_tables(s.B, s.N0, s.C_indptr.ctypes.data,
                                               s.C_indices.ctypes.data, rb.ctypes.data, rw,
                                               cb.ctypes.data, cw))
    assert np.array_equal(rb, lay.row_bits) and np.array_equal(cb, lay.col_bits)
    # wrap-around: bit t of row r is C[r, t mod N0]
    C = s.dense_C()
    t = np.arange(32 * rw)
    bits = (rb[:, t >> 5] >> (t & 31).astype(np.uint32)) & 1
    assert np.array_equal(bits, C[:, t % s.N0])


@pytest.mark.parametrize("i", SMALL)
def test_kernel_rule_matches_reference(i):
    s = _spec(i)
    lay = pattern_layout(s, 128)
    want = str(FIX[f"c{i}_dense_sha256"])
    assert _sha(_rule_rows(s, lay, 0, s.T)) == want
    assert _sha(np.ascontiguousarray(_rule_rows(s, lay, 0, s.T, cols=True).T)) == want


def test_kernel_rule_c3_size():
    """T = 16384, d = 3, chunk 128 (the c3 sequence length): rows of the
    kernels' rule against the reference's dense mask, evaluated in bands."""
    i = next(j for j in range(N_CASES) if int(FIX[f"c{j}_args"][0]) == 16384)
    s = _spec(i)
    lay = pattern_layout(s, 128)
    assert lay.nnzb == 128 * 129 // 2                   # every causal tile
    kinds = np.bincount(lay.tile_kind, minlength=3)
    assert kinds[KIND_PATTERN] == 64 * 64               # recent rows x long-range columns
    dense = materialise(s, np.uint8)
    for lo in (0, s.n - 64, s.n, s.T - 256):
        hi = lo + 256
        assert np.array_equal(_rule_rows(s, lay, lo, hi), dense[lo:hi])
        assert np.array_equal(_rule_rows(s, lay, lo, hi, cols=True), dense[:, lo:hi].T)
    assert block_layout_stats(lay)["pairs"] == int(dense.sum(dtype=np.int64))


def test_rejects():
    s = _spec(3)
    lay = pattern_layout(s, 64)
    L = _lib.lib()
    out = np.zeros((1, s.T), np.uint8)

    def rows(**over):
        f = dict(family=0, n=s.n, n_P=s.n_P, B=s.B, N0=s.N0, row_words=lay.row_bits.shape[1],
                 col_words=lay.col_bits.shape[1], row_bits=lay.row_bits.ctypes.data,
                 col_bits=lay.col_bits.ctypes.data)
        f.update(over)
        pt = _lib.Pattern(*f.values())
        return L.smat_pattern_mask_rows(ctypes.byref(pt), s.T, 0, 1, out.ctypes.data)

    assert rows() == 0
    assert rows(family=2) == 15
    assert rows(n=s.T + 1) == 15
    assert rows(n_P=s.n + 1) == 15
    assert rows(B=0) == 15
    assert rows(row_words=lay.row_bits.shape[1] - 1) == 15
    assert rows(col_words=1) == 15
    assert rows(family=1) == 15                 # endpoint needs N0 >= n - n_P
    assert rows(row_bits=None) == 8
    assert L.smat_pattern_mask_rows(None, s.T, 0, 1, out.ctypes.data) == 8
    # C with an index outside [0, N0)
    bad = s.C_indices.copy()
    bad[0] = s.N0
    rb = np.zeros_like(lay.row_bits)
    cb = np.zeros_like(lay.col_bits)
    assert L.smat_pattern_tables(s.B, s.N0, s.C_indptr.ctypes.data, bad.ctypes.data,
                                 rb.ctypes.data, rb.shape[1], cb.ctypes.data,
                                 cb.shape[1]) == 15
    with pytest.raises(ValueError):
        pattern_layout(lay)
