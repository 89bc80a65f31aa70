"""M^(d) masks: the restated builder against fixtures made by the reference's
own build_mask / materialise (tests/golden/make_golden.py), plus the
structural checks of the reference's test_smat.py:43-136."""

import hashlib
import os

import numpy as np
import pytest

from smat_attention_b200.mask import (build_mask, d_max_geometric, incidence_audit,
                                      materialise, planted_hyperplane_normals)

GOLD = os.path.join(os.path.dirname(__file__), "golden", "mask_md.npz")


def _cases():
    f = np.load(GOLD)
    return f, int(f["n_cases"])


@pytest.mark.parametrize("i", range(14))
def test_matches_reference_fixture(i):
    f, n = _cases()
    assert i < n
    p = f"c{i}_"
    T, d, chunk, nP = (int(x) for x in f[p + "args"])
    s = build_mask(T, d, chunk=chunk, n_P=nP)
    fields = [s.n, s.T_R, s.q, s.dim, s.N0, s.n_dirs, s.B, s.n_planted, s.k, s.n_P,
              s.uniform_deg]
    assert fields == [int(x) for x in f[p + "fields"]]
    assert s.kind == str(f[p + "kind"])
    for name in ("C_indptr", "C_indices", "planted_cols"):
        want = f[p + name]
        got = getattr(s, name)
        assert got.dtype == want.dtype and np.array_equal(got, want), name
    if p + "dense_sha256" in f:
        dense = materialise(s, np.uint8)
        assert hashlib.sha256(np.ascontiguousarray(dense).tobytes()).hexdigest() == \
            str(f[p + "dense_sha256"])
        assert int(dense.sum(dtype=np.int64)) == int(f[p + "nnz"])
        if p + "dense_packed" in f:
            assert np.array_equal(np.packbits(dense, axis=1), f[p + "dense_packed"])


@pytest.mark.parametrize("T,d", [(256, 1), (512, 2), (1024, 2), (1024, 3), (2048, 3), (2048, 4)])
def test_structure(T, d):
    M = materialise(build_mask(T, d, chunk=64))
    L = np.tril(np.ones((T, T)))
    assert np.all(np.triu(M, 1) == 0)
    assert np.all(np.diag(M) == 1)
    assert np.all((M == 0) | (M == 1))
    assert np.all(M <= L)


def test_degenerate_and_ranges():
    for T in (256, 512, 1000):
        assert np.array_equal(materialise(build_mask(T, 1, chunk=64)), np.tril(np.ones((T, T))))
    with pytest.raises(ValueError):
        build_mask(1024, 11, chunk=64)
    with pytest.raises(ValueError):
        build_mask(4, 1)
    assert build_mask(1024, 10, chunk=64).kind == "endpoint"
    with pytest.raises(MemoryError):
        build_mask(16384, 3, chunk=128, max_I_prof=10)
    for T in (4096, 65536):
        assert d_max_geometric(T, chunk=128) < T.bit_length() - 1


@pytest.mark.parametrize("T,d", [(1024, 2), (2048, 3), (4096, 4), (16384, 5)])
def test_planted_identity_and_audit(T, d):
    a = incidence_audit(build_mask(T, d, chunk=64))
    assert a["planted_identity"] and a["exact"]
    hs = planted_hyperplane_normals(d)
    assert all(np.any(x != 0) for x, _ in hs)
    assert len({(tuple(x), b) for x, b in hs}) == len(hs)


@pytest.mark.parametrize("d", [2, 3, 4])
def test_counting_identity(d):
    for T in (2 ** 14, 2 ** 16):
        s = build_mask(T, d, chunk=128)
        assert s.I_prof == s.B * s.q ** (d - 2)
        assert s.I_prof == s.q ** (d - 1) * (s.q ** (d - 1) - 1) // (s.q - 1)
