"""The kernelised-attention oracle (oracle/kernel_attention.py) against the
reference's own torch path (tests/golden/kattn_*.npz, written by
tests/golden/make_golden.py from src/smat/attention.py:391-455 in fp64):
output, gradients (torch autograd through the oracle), and the pooled
intermediates F and U."""

import glob
import os

import numpy as np
import pytest
import torch

from oracle import kernel_attention as OK
from smat_attention_b200.mask import build_mask

CASES = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "kattn_*.npz")))


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(c)[6:-4] for c in CASES])
def test_oracle_matches_reference(path):
    f = np.load(path)
    T, d, chunk, n_P = (int(x) for x in f["args"])
    spec = build_mask(T, d, chunk=chunk, n_P=n_P)
    phi, psi, v = (torch.from_numpy(f[k]).double().requires_grad_(True)
                   for k in ("phi", "psi", "v"))
    Vb = torch.cat([v, torch.ones(*v.shape[:-1], 1, dtype=torch.float64)], dim=-1)
    out = OK.smat_attention(phi, psi, Vb, spec, chunk=chunk)
    assert np.abs(out.detach().numpy() - f["out"]).max() < 1e-11
    (out * torch.from_numpy(f["dout"]).double()).sum().backward()
    for g, k in ((phi.grad, "dphi"), (psi.grad, "dpsi"), (v.grad, "dv")):
        ref = f[k]
        assert np.abs(g.numpy() - ref).max() <= 1e-10 * (1 + np.abs(ref).max()), k
    with torch.no_grad():
        Vb0 = torch.cat([v.detach(), torch.ones(*v.shape[:-1], 1, dtype=torch.float64)], -1)
        F = OK.pool_profiles(psi.detach(), Vb0, spec)
        U = OK.apply_incidence(F, spec)
    assert np.abs(F.numpy() - f["F"]).max() <= 1e-5 * (1 + np.abs(f["F"]).max())
    assert np.abs(U.numpy() - f["U"]).max() <= 1e-5 * (1 + np.abs(f["U"]).max())


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(c)[6:-4] for c in CASES])
def test_oracle_decoder_matches_reference(path):
    """The oracle's streaming decoder against the reference's ``SmatDecoder``
    outputs (rows n .. T-1) and cache size; for the geometric family it also
    reproduces the prefill rows, as the reference's test_smat.py:327-342 checks."""
    f = np.load(path)
    T, d, chunk, n_P = (int(x) for x in f["args"])
    spec = build_mask(T, d, chunk=chunk, n_P=n_P)
    phi, psi, v = (torch.from_numpy(f[k]).double() for k in ("phi", "psi", "v"))
    Vb = torch.cat([v, torch.ones(*v.shape[:-1], 1, dtype=torch.float64)], dim=-1)
    n = spec.n
    dec = OK.SmatDecoder(psi[:, :n], Vb[:, :n], spec)
    got = torch.stack([dec.step(phi[:, i], psi[:, i], Vb[:, i]) for i in range(n, T)], dim=1)
    assert np.abs(got.numpy() - f["dec"]).max() < 1e-11
    assert dec.cache_words() == int(f["dec_words"][0])
    if spec.kind == "geometric":
        assert np.abs(f["dec"] - f["out"][:, n:]).max() < 1e-11


def test_chunk_local_definition():
    g = torch.Generator().manual_seed(0)
    Phi, Psi = (torch.rand(1, 2, 8, 3, generator=g, dtype=torch.float64) for _ in range(2))
    Vb = torch.rand(1, 2, 8, 4, generator=g, dtype=torch.float64)
    Sin = torch.rand(1, 2, 3, 4, generator=g, dtype=torch.float64)
    out = OK.chunk_local(Phi, Psi, Vb, Sin)
    i, c = 5, 1
    want = Phi[0, c, i] @ Sin[0, c] + sum((Phi[0, c, i] @ Psi[0, c, j]) * Vb[0, c, j]
                                          for j in range(i + 1))
    assert torch.allclose(out[0, c, i], want)


def test_torch_parts_match_oracle():
    """The product module's torch-side parts (Walsh incidence for the endpoint
    family, the zeta butterfly, the incidence's transposed CSR) against the
    oracle, on CPU."""
    from smat_attention_b200 import kernel_attention as KA
    g = torch.Generator().manual_seed(3)
    spec = build_mask(1024, 10, chunk=64)                  # endpoint, B = N0 = 512
    F = torch.randn(2, spec.N0, 3, 4, generator=g, dtype=torch.float64)
    assert torch.allclose(KA.walsh_incidence(F), OK.apply_incidence(F, spec), atol=1e-10)
    Fz = torch.randn(1, 64, 2, 3, generator=g, dtype=torch.float64)
    assert torch.allclose(KA.zeta_transform(Fz), OK.zeta_transform(Fz), atol=1e-12)
    spec3 = build_mask(1000, 3, chunk=8)
    # the transposed CSR used by the incidence backward
    ptr = torch.from_numpy(spec3.C_indptr)
    idx = torch.from_numpy(spec3.C_indices)
    t_ptr, t_idx = KA._transpose_csr(ptr, idx, spec3.N0)
    Cd = spec3.dense_C()
    for x in range(0, spec3.N0, 7):
        rows = t_idx[t_ptr[x]:t_ptr[x + 1]].tolist()
        assert rows == np.flatnonzero(Cd[:, x]).tolist()


def test_make_phi_matches_reference_fixture():
    """make_phi draws the reference's projection for the same seed: outputs
    equal the reference's make_phi bit for bit (tests/golden/smat_module.npz)."""
    import os
    from smat_attention_b200 import kernel_attention as KA
    f = np.load(os.path.join(os.path.dirname(__file__), "golden", "smat_module.npz"))
    x = torch.from_numpy(f["xp"])
    assert np.array_equal(KA.make_phi(16, 8, seed=3)(x).numpy(), f["phi_elu"])
    assert np.array_equal(KA.make_phi(16, 8, kind="relu", seed=3)(x).numpy(), f["phi_relu"])
    Phi, Psi, Vb = KA.featurise(x, x, x[:, :4], KA.make_phi(16, 8, seed=3),
                                h=torch.full((5,), 0.5))
    assert torch.equal(Psi, Phi * 0.5) and Vb.shape == (5, 5) and torch.all(Vb[:, -1] == 1)


def test_op_and_module_reject_on_the_host():
    """Argument errors of the op and of the module's smat arm are raised before
    anything reaches a kernel."""
    import pytest
    from smat_attention_b200 import kernel_attention as KA
    from smat_attention_b200.model import Attention
    spec = build_mask(512, 3, chunk=128)
    x = torch.zeros(1, 512, 32)
    vb = torch.zeros(1, 512, 33)
    with pytest.raises(ValueError):
        KA.smat_attention(x, x, vb, spec, acc_dtype=torch.float64)
    with pytest.raises(ValueError):
        KA.smat_attention(x, x, vb, spec, scan_backend="cuda")
    with pytest.raises(ValueError):
        KA.smat_attention(x, x, vb, spec, long_range="dense")
    with pytest.raises(ValueError):
        Attention(32, 2, "smat", spec=spec, decay=True)
    with pytest.raises(ValueError):
        Attention(32, 2, "smat", spec=None)
    with pytest.raises(TypeError):
        Attention(32, 2, "smat", spec=spec, not_an_option=1)
    m = Attention(32, 2, "smat", spec=spec, r=32, phi_kind="taylor", taylor_dim=4)
    assert m.phi(torch.zeros(3, 16)).shape == (3, 1 + 4 + 16)
