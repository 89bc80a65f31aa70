"""GPU parity of the kernelised-attention kernels (include/smat_kattn.h)
against the oracle (oracle/kernel_attention.py, itself pinned to the
reference's torch path by tests/test_kattn_oracle.py).

Tolerances: the chunk-local pass (forward and backward) runs TF32 tensor
cores, as the reference's Triton kernels do (allow_tf32), and is held to 2e-3
of each tensor's largest entry -- the reference's own fp32 kernel-vs-torch
bound (tests/test_smat.py:390); pool and incidence are fp32 arithmetic, held
to 1e-5 relative."""

import glob
import os

import numpy as np
import pytest
import torch

from oracle import kernel_attention as OK
from smat_attention_b200 import kernel_attention as KA
from smat_attention_b200.attention import check_device_errors
from smat_attention_b200.mask import build_mask

pytestmark = pytest.mark.gpu


def _close(got, ref, rel, name):
    scale = ref.abs().max().item() + 1e-30
    err = (got.double().cpu() - ref.double().cpu()).abs().max().item()
    print(f"{name}: max err {err:.3e} (scale {scale:.3e})")
    assert err <= rel * scale, (name, err, scale)


def _feat(*shape, g):
    return torch.nn.functional.elu(torch.randn(*shape, generator=g, dtype=torch.float64)) + 1


@pytest.mark.parametrize("R,P", [(32, 9), (64, 65), (64, 17), (128, 96), (32, 128), (64, 60),
                                 (32, 70), (128, 20)])
def test_chunk_local(cuda_device, R, P):
    g = torch.Generator().manual_seed(R + P)
    nb, nc, C = 2, 3, 128
    Phi, Psi = _feat(nb, nc, C, R, g=g), _feat(nb, nc, C, R, g=g)
    Vb = torch.randn(nb, nc, C, P, generator=g, dtype=torch.float64)
    Sin = torch.rand(nb, nc, R, P, generator=g, dtype=torch.float64) * 10
    dout = torch.randn(nb, nc, C, P, generator=g, dtype=torch.float64)
    ins = [x.float().to(cuda_device).requires_grad_(True) for x in (Phi, Psi, Vb, Sin)]
    out = KA.chunk_local(*ins)
    (out * dout.float().to(cuda_device)).sum().backward()
    torch.cuda.synchronize()
    assert check_device_errors() == 0
    ref_in = [x.float().double().requires_grad_(True) for x in (Phi, Psi, Vb, Sin)]
    ref = OK.chunk_local(*ref_in)
    (ref * dout.float().double()).sum().backward()
    _close(out, ref.detach(), 2e-3, "out")
    for a, b, n in zip(ins, ref_in, ("dphi", "dpsi", "dvb", "dsin")):
        _close(a.grad, b.grad, 2e-3 if n != "dsin" else 1e-4, n)


@pytest.mark.parametrize("T,d,n_P,R,P", [(1024, 3, 0, 64, 65), (2048, 3, 16, 32, 17),
                                          (512, 2, 0, 16, 9), (1000, 3, 0, 64, 65),
                                          (1024, 3, 0, 128, 129), (512, 2, 8, 20, 33)])
def test_pool_and_incidence(cuda_device, T, d, n_P, R, P):
    spec = build_mask(T, d, chunk=8, n_P=n_P)
    g = torch.Generator().manual_seed(T + d)
    nb = 2
    Psi = _feat(nb, T, R, g=g).float().double()
    Vb = torch.randn(nb, T, P, generator=g, dtype=torch.float32).double()
    dF = torch.randn(nb, spec.N0, R, P, generator=g, dtype=torch.float32).double()
    dU = torch.randn(nb, spec.B, R, P, generator=g, dtype=torch.float32).double()
    k = Psi.float().to(cuda_device).requires_grad_(True)
    v = Vb.float().to(cuda_device).requires_grad_(True)
    F = KA.pool_profiles(k, v, spec)
    (F * dF.float().to(cuda_device)).sum().backward()
    rk, rv = Psi.clone().requires_grad_(True), Vb.clone().requires_grad_(True)
    rF = OK.pool_profiles(rk, rv, spec)
    (rF * dF).sum().backward()
    _close(F, rF.detach(), 1e-5, "F")
    _close(k.grad, rk.grad, 1e-5, "dpsi")
    _close(v.grad, rv.grad, 1e-5, "dvb")
    Fg = rF.detach().float().to(cuda_device).requires_grad_(True)
    U = KA.apply_incidence(Fg, spec)
    (U * dU.float().to(cuda_device)).sum().backward()
    rFg = rF.detach().float().double().requires_grad_(True)
    rU = OK.apply_incidence(rFg, spec)
    (rU * dU).sum().backward()
    _close(U, rU.detach(), 1e-5, "U")
    _close(Fg.grad, rFg.grad, 1e-5, "dF")
    torch.cuda.synchronize()
    assert check_device_errors() == 0


def _run_op(spec, Phi, Psi, v, dout, device, chunk=128):
    ins = [x.float().to(device).requires_grad_(True) for x in (Phi, Psi, v)]
    Vb = torch.cat([ins[2], torch.ones(*v.shape[:-1], 1, device=device)], dim=-1)
    out = KA.smat_attention(ins[0], ins[1], Vb, spec, chunk=chunk)
    (out * dout.float().to(device)).sum().backward()
    torch.cuda.synchronize()
    assert check_device_errors() == 0
    return out, [x.grad for x in ins]


def test_op_matches_reference_fixture(cuda_device):
    """The whole op against the reference's own fp64 outputs and gradients
    (tests/golden/kattn_geo3_t1024_c128_np16.npz: M^(3), chunk 128, n_P 16)."""
    path = os.path.join(os.path.dirname(__file__), "golden", "kattn_geo3_t1024_c128_np16.npz")
    f = np.load(path)
    T, d, chunk, n_P = (int(x) for x in f["args"])
    spec = build_mask(T, d, chunk=chunk, n_P=n_P)
    out, grads = _run_op(spec, *(torch.from_numpy(f[k]) for k in ("phi", "psi", "v", "dout")),
                         cuda_device, chunk)
    _close(out, torch.from_numpy(f["out"]), 2e-3, "out")
    for gr, k in zip(grads, ("dphi", "dpsi", "dv")):
        _close(gr, torch.from_numpy(f[k]), 2e-3, k)


@pytest.mark.parametrize("T,d,r,dv", [(4096, 3, 64, 64), (1024, 10, 64, 64), (2048, 2, 32, 32)])
def test_op_matches_oracle(cuda_device, T, d, r, dv):
    spec = build_mask(T, d, chunk=128)
    g = torch.Generator().manual_seed(T + d)
    nb = 2
    Phi, Psi = _feat(nb, T, r, g=g).float().double(), _feat(nb, T, r, g=g).float().double()
    v = torch.randn(nb, T, dv, generator=g, dtype=torch.float32).double()
    dout = torch.randn(nb, T, dv, generator=g, dtype=torch.float32).double()
    out, grads = _run_op(spec, Phi, Psi, v, dout, cuda_device)
    ref_in = [x.clone().requires_grad_(True) for x in (Phi, Psi, v)]
    Vb = torch.cat([ref_in[2], torch.ones(nb, T, 1, dtype=torch.float64)], dim=-1)
    ref = OK.smat_attention(ref_in[0], ref_in[1], Vb, spec, chunk=128)
    (ref * dout).sum().backward()
    _close(out, ref.detach(), 2e-3, "out")
    for gr, rr, k in zip(grads, ref_in, ("dphi", "dpsi", "dv")):
        _close(gr, rr.grad, 2e-3, k)


def test_rejects(cuda_device):
    x = torch.zeros(1, 1, 64, 32, device=cuda_device)
    with pytest.raises(Exception):
        KA.chunk_local(x, x, torch.zeros(1, 1, 64, 9, device=cuda_device),
                       torch.zeros(1, 1, 32, 9, device=cuda_device))     # C = 64
    with pytest.raises(ValueError):
        KA.chunk_local(*(t.cpu() for t in (x, x, x, x)))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(os.path.dirname(__file__),
                                                                 "golden", "kattn_*.npz"))),
                         ids=lambda p: os.path.basename(p)[6:-4])
def test_decoder_matches_reference_fixture(cuda_device, path):
    """``SmatDecoder`` on the decode kernel against the reference's own
    ``SmatDecoder`` outputs (fp64) for rows n .. T-1, stepping one token per
    launch; fp32 state and arithmetic, held to 1e-4 of the largest output."""
    f = np.load(path)
    T, d, chunk, n_P = (int(x) for x in f["args"])
    spec = build_mask(T, d, chunk=chunk, n_P=n_P)
    phi, psi, v = (torch.from_numpy(f[k]).to(cuda_device) for k in ("phi", "psi", "v"))
    Vb = torch.cat([v, torch.ones(*v.shape[:-1], 1, device=cuda_device)], dim=-1)
    n = spec.n
    dec = KA.SmatDecoder(psi[:, :n], Vb[:, :n], spec)
    got = torch.stack([dec.step(phi[:, i], psi[:, i], Vb[:, i]) for i in range(n, T)], dim=1)
    torch.cuda.synchronize()
    assert check_device_errors() == 0
    _close(got, torch.from_numpy(f["dec"]), 1e-4, "dec")
    assert dec.cache_words() == int(f["dec_words"][0])


def test_decoder_matches_oracle_wide(cuda_device):
    """A wider state (r = 128, p = 129) than the fixtures, against the oracle."""
    T, d, r, dv = 2048, 3, 128, 128
    spec = build_mask(T, d, chunk=64)
    g = torch.Generator().manual_seed(17)
    nb = 3
    Phi, Psi = _feat(nb, T, r, g=g).float(), _feat(nb, T, r, g=g).float()
    Vb = torch.cat([torch.randn(nb, T, dv, generator=g), torch.ones(nb, T, 1)], dim=-1)
    n = spec.n
    ref = OK.SmatDecoder(Psi[:, :n].double(), Vb[:, :n].double(), spec)
    dec = KA.SmatDecoder(Psi[:, :n].to(cuda_device), Vb[:, :n].to(cuda_device), spec)
    for i in range(n, min(T, n + 300)):
        got = dec.step(*(x[:, i].to(cuda_device) for x in (Phi, Psi, Vb)))
        want = ref.step(Phi[:, i].double(), Psi[:, i].double(), Vb[:, i].double())
        _close(got, want, 1e-4, f"row {i}")
    with pytest.raises(ValueError):
        dec.step(Phi[:, 0].to(cuda_device), Psi[:, 0].to(cuda_device),
                 Vb[:, 0, :5].to(cuda_device))


@pytest.mark.parametrize("P", [2, 9, 65, 129])
def test_normalise(cuda_device, P):
    """The fused final division and its backward against torch autograd of
    ``H[..., :-1] / H[..., -1:]`` (fp64), within 1e-5 of scale."""
    g = torch.Generator().manual_seed(P)
    H = torch.randn(3, 257, P, generator=g, dtype=torch.float64)
    H[..., -1] = H[..., -1].abs() + 0.5
    dout = torch.randn(3, 257, P - 1, generator=g, dtype=torch.float64)
    x = H.float().to(cuda_device).requires_grad_(True)
    out = KA.normalise(x)
    out.backward(dout.float().to(cuda_device))
    torch.cuda.synchronize()
    r = H.float().double().requires_grad_(True)
    ref = r[..., :-1] / r[..., -1:]
    ref.backward(dout.float().double())
    _close(out, ref.detach(), 1e-5, "out")
    _close(x.grad, r.grad, 1e-5, "dH")


# ---------------------------------------------------------------- glue kernels
def _chunk_prefix_ref(a, b, C, nc0, reverse):
    """fp64 loops: the shifted, segmented prefix of the chunk products."""
    nb, T, R = a.shape
    P = b.shape[-1]
    nc = -(-T // C)
    pad = nc * C - T
    a = torch.nn.functional.pad(a, (0, 0, 0, pad))
    b = torch.nn.functional.pad(b, (0, 0, 0, pad))
    D = a.reshape(nb, nc, C, R).transpose(-1, -2) @ b.reshape(nb, nc, C, P)
    out = torch.zeros_like(D)
    order = range(nc - 1, -1, -1) if reverse else range(nc)
    run = torch.zeros_like(D[:, 0])
    for c in order:
        if (not reverse and c == nc0) or (reverse and c == nc0 - 1):
            run = torch.zeros_like(run)
        out[:, c] = run
        run = run + D[:, c]
    return out


@pytest.mark.parametrize("T,R,P,nc0", [(1024, 64, 65, 4), (1000, 32, 17, 3), (512, 128, 129, 0),
                                       (700, 20, 9, 6)])
def test_chunk_prefix(cuda_device, T, R, P, nc0):
    g = torch.Generator().manual_seed(T + R)
    nb, C = 2, 128
    a = _feat(nb, T, R, g=g).float()
    b = torch.randn(nb, T, P, generator=g)
    L = KA._L()
    nc = -(-T // C)
    for reverse in (0, 1):
        out = torch.empty(nb, nc, R, P, device=cuda_device)
        ad, bd = a.to(cuda_device), b.to(cuda_device)
        assert L.smat_kattn_chunk_prefix(ad.data_ptr(), bd.data_ptr(), out.data_ptr(), nb, T, C,
                                         R, P, nc0, reverse, None) == 0
        torch.cuda.synchronize()
        _close(out, _chunk_prefix_ref(a.double(), b.double(), C, nc0, reverse), 1e-5,
               f"prefix reverse={reverse}")
    # the segments never mix: the recent segment's prefixes are bitwise
    # independent of the landmark chunks (and the other way round, reversed)
    if 0 < nc0 < nc:
        a2, b2 = a.clone(), b.clone()
        a2[:, :nc0 * C] *= 3.0
        b2[:, :nc0 * C] += 1.0
        for x, y in ((a, b), (a2, b2)):
            o = torch.empty(nb, nc, R, P, device=cuda_device)
            xd, yd = x.to(cuda_device), y.to(cuda_device)
            L.smat_kattn_chunk_prefix(xd.data_ptr(), yd.data_ptr(), o.data_ptr(), nb, T, C, R,
                                      P, nc0, 0, None)
            torch.cuda.synchronize()
            if x is a:
                first = o[:, nc0:].clone()
            else:
                assert torch.equal(first, o[:, nc0:])


def test_chunk_expand(cuda_device):
    g = torch.Generator().manual_seed(11)
    nb, T, C, R, P = 2, 900, 128, 64, 65
    nc = -(-T // C)
    a, b = torch.randn(nb, T, R, generator=g), torch.randn(nb, T, P, generator=g)
    dD = torch.randn(nb, nc, R, P, generator=g)
    da0, db0 = torch.randn(nb, T, R, generator=g), torch.randn(nb, T, P, generator=g)
    ad, bd, dDd = (x.to(cuda_device) for x in (a, b, dD))
    da, db = da0.clone().to(cuda_device), db0.clone().to(cuda_device)
    assert KA._L().smat_kattn_chunk_expand(ad.data_ptr(), bd.data_ptr(), dDd.data_ptr(),
                                           da.data_ptr(), db.data_ptr(), nb, T, C, R, P,
                                           None) == 0
    torch.cuda.synchronize()
    pad = nc * C - T
    ap = torch.nn.functional.pad(a.double(), (0, 0, 0, pad)).reshape(nb, nc, C, R)
    bp = torch.nn.functional.pad(b.double(), (0, 0, 0, pad)).reshape(nb, nc, C, P)
    want_da = da0.double() + (bp @ dD.double().transpose(-1, -2)).reshape(nb, -1, R)[:, :T]
    want_db = db0.double() + (ap @ dD.double()).reshape(nb, -1, P)[:, :T]
    _close(da, want_da, 1e-5, "da")
    _close(db, want_db, 1e-5, "db")


@pytest.mark.parametrize("T,d,r,p", [(1024, 3, 64, 65), (2048, 3, 32, 33), (1000, 2, 20, 9)])
def test_query_by_type(cuda_device, T, d, r, p):
    spec = build_mask(T, d, chunk=8)
    g = torch.Generator().manual_seed(T + r)
    nb = 2
    Phi_rec = torch.randn(nb, spec.T_R, r, generator=g, dtype=torch.float32).double()
    U = torch.randn(nb, spec.B, r, p, generator=g, dtype=torch.float32).double()
    dY = torch.randn(nb, spec.T_R, p, generator=g, dtype=torch.float32).double()
    x, u = (t.float().to(cuda_device).requires_grad_(True) for t in (Phi_rec, U))
    Y = KA.query_by_type(x, u, spec)
    (Y * dY.float().to(cuda_device)).sum().backward()
    torch.cuda.synchronize()
    rx, ru = Phi_rec.clone().requires_grad_(True), U.clone().requires_grad_(True)
    rY = OK.query_by_type(rx, ru, spec)
    (rY * dY).sum().backward()
    _close(Y, rY.detach(), 1e-5, "Y")
    _close(x.grad, rx.grad, 1e-5, "dphi")
    _close(u.grad, ru.grad, 1e-5, "dU")


# ---------------------------------------------------------------- the op's arguments
def test_op_arguments(cuda_device):
    """return_parts, the phase timer, and the direct / subtractive long-range
    forms against the pooled schedule and the oracle."""
    T, d, r, dv = 2048, 3, 64, 64
    spec = build_mask(T, d, chunk=128)
    g = torch.Generator().manual_seed(5)
    nb = 2
    Phi, Psi = _feat(nb, T, r, g=g).float(), _feat(nb, T, r, g=g).float()
    v = torch.randn(nb, T, dv, generator=g)
    dev = lambda t: t.to(cuda_device)
    Vb = torch.cat([dev(v), torch.ones(nb, T, 1, device=cuda_device)], -1)
    tm = KA.PhaseTimer(cuda_device)
    out, parts = KA.smat_attention(dev(Phi), dev(Psi), Vb, spec, timer=tm, return_parts=True,
                                   acc_dtype=torch.float32, scan_backend="torch",
                                   incidence_backend="triton")
    phases = tm.results()
    assert set(phases) >= {"lr_pool", "lr_incidence", "lr_query", "scan", "normalise"}
    assert set(parts) == {"U", "Y_lr", "H"}
    ref = OK.smat_attention(Phi.double(), Psi.double(),
                            torch.cat([v.double(), torch.ones(nb, T, 1, dtype=torch.float64)],
                                      -1), spec, chunk=128)
    _close(out, ref, 2e-3, "pooled")
    plain = KA.smat_attention(dev(Phi), dev(Psi), Vb, spec)
    assert torch.equal(plain, out)      # the fused in-place query equals the split one
    from smat_attention_b200.mask import to_device
    to_device(spec, cuda_device, want_direct=True)
    direct = KA.smat_attention(dev(Phi), dev(Psi), Vb, spec, long_range="direct")
    _close(direct, ref, 2e-3, "direct")
    sub, sparts = KA.smat_attention(dev(Phi), dev(Psi), Vb, spec, long_range="subtractive",
                                    return_parts=True)
    _close(sub, ref, 2e-3, "subtractive")
    assert set(sparts) == {"H", "Y_ex"}
    torch.cuda.synchronize()
    assert check_device_errors() == 0


def test_op_landmark_rows_do_not_see_recent_rows(cuda_device):
    """Bitwise non-influence (the reference's property, tests/test_smat.py:292-324):
    the landmark rows' outputs do not change when the recent rows' keys and
    values do, since the scan's segments never mix and the long-range query
    writes only recent rows."""
    T, d, r, dv = 4096, 3, 64, 64
    spec = build_mask(T, d, chunk=128)
    n = spec.n
    g = torch.Generator().manual_seed(9)
    nb = 2
    Phi, Psi = (_feat(nb, T, r, g=g).float().to(cuda_device) for _ in range(2))
    v = torch.randn(nb, T, dv, generator=g).to(cuda_device)
    outs = []
    for bump in (0.0, 5.0):
        Psi2, v2 = Psi.clone(), v.clone()
        Psi2[:, n:] += bump
        v2[:, n:] -= bump
        Vb = torch.cat([v2, torch.ones(nb, T, 1, device=cuda_device)], -1)
        outs.append(KA.smat_attention(Phi, Psi2, Vb, spec))
    torch.cuda.synchronize()
    assert torch.equal(outs[0][:, :n], outs[1][:, :n])
    assert not torch.equal(outs[0][:, n:], outs[1][:, n:])


def test_module_smat_arm_matches_reference_fixture(cuda_device):
    """Attention(arm="smat") (featurise with make_phi of the same seed, then the
    op on the B200 kernels) against the reference module's own output and input
    gradient (tests/golden/smat_module.npz), within the op's 2e-3 TF32 bound."""
    from smat_attention_b200.model import Attention
    f = np.load(os.path.join(os.path.dirname(__file__), "golden", "smat_module.npz"))
    T, d_model, heads, r, seed = (int(x) for x in f["args"])
    spec = build_mask(T, 3, chunk=128)
    m = Attention(d_model, heads, "smat", spec=spec, r=r, chunk=128, seed=seed,
                  device=cuda_device)
    with torch.no_grad():
        m.qkv.weight.copy_(torch.from_numpy(f["qkv"]))
        m.out.weight.copy_(torch.from_numpy(f["out_w"]))
    x = torch.from_numpy(f["x"]).to(cuda_device).requires_grad_(True)
    y = m(x)
    (y * torch.from_numpy(f["dy"]).to(cuda_device)).sum().backward()
    torch.cuda.synchronize()
    assert check_device_errors() == 0
    _close(y, torch.from_numpy(f["y"]), 2e-3, "y")
    _close(x.grad, torch.from_numpy(f["dx"]), 2e-3, "dx")
