"""Generate the golden fixtures in this directory from the reference itself.

Run in a container where the reference source tree is available::

    python tests/golden/make_golden.py /path/to/smat_attention

It imports the reference's ``smat`` package (``src/smat``) and records

``mask_md.npz``
    For a grid of ``(T, d, chunk, n_P)``: the reference ``build_mask`` spec
    fields and incidence CSR, and a SHA-256 of its ``materialise`` dense mask
    (the full packed mask too for ``T <= 512``).

``softmax_<case>.npz``
    Softmax attention outputs computed by the reference's own dense-masked path
    ``dense_masked_kernel_attention(Phi, Psi, Vb, M)``
    (``src/smat/attention.py:485-489``).  That function computes
    ``((Phi Psi^T) * M) [V, 1]`` and divides by the last column; called with
    ``Phi = exp(scale Q K^T - m)`` (``m`` the detached masked row max, one
    ``T``-wide feature per key), ``Psi = I`` it is exactly masked softmax
    attention.  Gradients come from torch autograd through that call.  Inputs
    are fp32-representable values; outputs are fp64.

``kattn_<case>.npz``
    The reference's kernelised op ``smat_attention`` on its torch path (fp64)
    for ``M^(d)`` masks: inputs, output, autograd gradients and the pooled
    intermediates ``F`` (profiles) and ``U`` (per row type), the latter two as fp32,
    and the outputs of its streaming decoder ``SmatDecoder``
    (``src/smat/attention.py:496-535``) prefilled with the first ``n`` columns
    and stepped through rows ``n .. T-1`` (fp64; ``dec``).

``smat_module.npz``
    The reference's ``Attention`` module in its plain ``"smat"`` arm
    (``src/smat/model.py:112-343``; ``make_phi`` feature map, ``featurise``,
    ``smat_attention`` on its torch path) for an ``M^(3)`` mask at chunk 128:
    its weights, an input, the output and the input's gradient for a given
    output gradient; and ``make_phi`` (``src/smat/attention.py:82-97``) applied
    to a fixed input for both kinds.

Nothing at test time imports the reference: the tests read only these files.
"""

from __future__ import annotations

import hashlib
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

MD_GRID = [(256, 1, 64, 0), (512, 2, 64, 0), (1024, 2, 64, 0), (1024, 3, 64, 0),
           (2048, 3, 64, 0), (2048, 4, 64, 0), (2048, 3, 64, 16), (1024, 10, 64, 0),
           (1000, 3, 32, 0), (4096, 3, 128, 0), (16384, 3, 128, 0), (300, 8, 8, 0),
           (256, 7, 16, 0), (512, 3, 1, 0)]

# (name, T, BH, D, mask) -- mask is ("block", bs, W, S, sinks) or ("md", d, chunk)
SOFTMAX_CASES = [
    ("block_t256", 256, 2, 16, ("block", 32, 2, 3, 1)),
    ("block_ragged_t200", 200, 2, 16, ("block", 32, 1, 2, 1)),
    ("md3_t256", 256, 1, 16, ("md", 3, 16)),
]
# one head of config 1 at full size (T = 1024, D = 64, bs 64, W 4, one sink):
# inputs are regenerated from the seed by the test (a digest guards against a
# change of the generator), outputs stored as fp32
C1_CASE = ("c1_t1024", 1024, 1, 64, ("block", 64, 4, 0, 1))


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_mask_md(R):
    out = {}
    for i, (T, d, chunk, nP) in enumerate(MD_GRID):
        s = R.build_mask(T, d, chunk=chunk, n_P=nP)
        p = f"c{i}_"
        out[p + "args"] = np.array([T, d, chunk, nP], dtype=np.int64)
        out[p + "fields"] = np.array([s.n, s.T_R, s.q, s.dim, s.N0, s.n_dirs, s.B,
                                      s.n_planted, s.k, s.n_P, s.uniform_deg],
                                     dtype=np.int64)
        out[p + "kind"] = np.array(s.kind)
        out[p + "C_indptr"] = s.C_indptr
        out[p + "C_indices"] = s.C_indices
        out[p + "planted_cols"] = s.planted_cols
        if T <= 4096:
            dense = R.materialise(s, np.uint8)
            out[p + "dense_sha256"] = np.array(_sha(dense))
            out[p + "nnz"] = np.array(int(dense.sum(dtype=np.int64)))
            if T <= 512:
                out[p + "dense_packed"] = np.packbits(dense, axis=1)
    out["n_cases"] = np.array(len(MD_GRID))
    np.savez_compressed(os.path.join(HERE, "mask_md.npz"), **out)


def _dense_mask(R, T, mask):
    if mask[0] == "block":
        _, bs, W, S, ns = mask
        i = np.arange(T)[:, None]
        j = np.arange(T)[None, :]
        qb, kb = i // bs, j // bs
        act = (kb <= qb) & ((qb - W <= kb) | (kb < ns) |
                            ((S > 0) & (kb % max(S, 1) == max(S, 1) - 1)))
        return (act & (j <= i)).astype(np.float64)
    _, d, chunk = mask
    return R.materialise(R.build_mask(T, d, chunk=chunk))


def c1_inputs(seed):
    """Config 1's inputs for the fixture: N(0, 1) fp32 from a CPU generator."""
    g = torch.Generator().manual_seed(seed)
    T, BH, D = C1_CASE[1], C1_CASE[2], C1_CASE[3]
    return [torch.randn(BH, T, D, generator=g, dtype=torch.float32) for _ in range(4)]


def make_softmax_c1(A, R, seed=0):
    """The reference's dense-masked path on one head of config 1 (fp64), outputs
    and gradients stored as fp32, inputs as a seed plus their SHA-256."""
    name, T, BH, D, mask = C1_CASE
    q, k, v, do = (x.double() for x in c1_inputs(seed))
    M = torch.from_numpy(_dense_mask(R, T, mask))
    scale = 1.0 / math.sqrt(D)
    qg, kg, vg = (x.clone().requires_grad_(True) for x in (q, k, v))
    s = torch.einsum("nta,nsa->nts", qg, kg) * scale
    m = s.masked_fill(M == 0, float("-inf")).amax(-1, keepdim=True).detach()
    Phi = torch.exp(s - m)
    Psi = torch.eye(T, dtype=torch.float64).expand(BH, T, T)
    Vb = torch.cat([vg, torch.ones(BH, T, 1, dtype=torch.float64)], dim=-1)
    o = A.dense_masked_kernel_attention(Phi, Psi, Vb, M)
    (o * do).sum().backward()
    digest = _sha(np.concatenate([x.float().numpy().ravel() for x in (q, k, v, do)]))
    np.savez_compressed(
        os.path.join(HERE, f"softmax_{name}.npz"), seed=np.array(seed),
        inputs_sha256=np.array(digest), mask_sha256=np.array(_sha(M.numpy().astype(np.uint8))),
        mask_args=np.array([str(x) for x in mask]), scale=np.array(scale),
        o=o.detach().float().numpy(), dq=qg.grad.float().numpy(), dk=kg.grad.float().numpy(),
        dv=vg.grad.float().numpy())


def make_softmax(A, R, name, T, BH, D, mask, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v, do = (torch.randn(BH, T, D, generator=g, dtype=torch.float32).double()
                   for _ in range(4))
    M = torch.from_numpy(_dense_mask(R, T, mask))
    scale = 1.0 / math.sqrt(D)
    qg, kg, vg = (x.clone().requires_grad_(True) for x in (q, k, v))
    s = torch.einsum("nta,nsa->nts", qg, kg) * scale
    m = s.masked_fill(M == 0, float("-inf")).amax(-1, keepdim=True).detach()
    Phi = torch.exp(s - m)                                   # (BH, T, T)
    Psi = torch.eye(T, dtype=torch.float64).expand(BH, T, T)
    Vb = torch.cat([vg, torch.ones(BH, T, 1, dtype=torch.float64)], dim=-1)
    o = A.dense_masked_kernel_attention(Phi, Psi, Vb, M)
    (o * do).sum().backward()
    np.savez_compressed(
        os.path.join(HERE, f"softmax_{name}.npz"),
        q=q.float().numpy(), k=k.float().numpy(), v=v.float().numpy(),
        do=do.float().numpy(), mask_sha256=np.array(_sha(M.numpy().astype(np.uint8))),
        mask_args=np.array([str(x) for x in mask]), scale=np.array(scale),
        o=o.detach().numpy(), dq=qg.grad.numpy(), dk=kg.grad.numpy(),
        dv=vg.grad.numpy())


# (name, T, d, chunk, n_P, nb, r, d_v)
KATTN_CASES = [
    ("geo3_t512_c64", 512, 3, 64, 0, 2, 16, 8),
    ("geo3_t1024_c128_np16", 1024, 3, 128, 16, 2, 32, 16),
    ("geo2_t512_c64", 512, 2, 64, 0, 1, 16, 8),
    ("endpoint_t1024_c64", 1024, 10, 64, 0, 1, 16, 8),
]


def make_kattn(A, R, name, T, d, chunk, n_P, nb, r, dv, seed):
    """The reference's kernelised op ``smat_attention`` (``src/smat/attention.py:391-455``)
    on its torch path in fp64, with autograd gradients, plus its pooled
    intermediates ``F = pool_profiles`` and ``U = apply_incidence``.  Features
    are ``elu(x) + 1`` of fp32 normals (strictly positive, as the op assumes)."""
    g = torch.Generator().manual_seed(seed)
    xq, xk = (torch.randn(nb, T, r, generator=g, dtype=torch.float32) for _ in range(2))
    v = torch.randn(nb, T, dv, generator=g, dtype=torch.float32)
    dout = torch.randn(nb, T, dv, generator=g, dtype=torch.float32)
    Phi = (torch.nn.functional.elu(xq.double()) + 1).float().double()
    Psi = (torch.nn.functional.elu(xk.double()) + 1).float().double()
    spec = R.build_mask(T, d, chunk=chunk, n_P=n_P)
    A.to_device(spec, "cpu")
    Pg, Sg, Vg = (x.clone().requires_grad_(True) for x in (Phi, Psi, v.double()))
    Vb = torch.cat([Vg, torch.ones(nb, T, 1, dtype=torch.float64)], dim=-1)
    out = A.smat_attention(Pg, Sg, Vb, spec, chunk=chunk, scan_backend="torch",
                           incidence_backend="torch")
    (out * dout.double()).sum().backward()
    with torch.no_grad():
        Vb0 = torch.cat([v.double(), torch.ones(nb, T, 1, dtype=torch.float64)], dim=-1)
        F = A.pool_profiles(Psi, Vb0, spec, backend="torch")
        U = A.apply_incidence(F, spec, backend="torch")
        n = spec.n
        dec = A.SmatDecoder(Psi[:, :n], Vb0[:, :n], spec, incidence_backend="torch")
        dec_out = torch.stack([dec.step(Phi[:, i], Psi[:, i], Vb0[:, i]) for i in range(n, T)],
                              dim=1)
    np.savez_compressed(
        os.path.join(HERE, f"kattn_{name}.npz"),
        args=np.array([T, d, chunk, n_P]), phi=Phi.float().numpy(), psi=Psi.float().numpy(),
        v=v.numpy(), dout=dout.numpy(), out=out.detach().numpy(), dphi=Pg.grad.numpy(),
        dpsi=Sg.grad.numpy(), dv=Vg.grad.numpy(), F=F.float().numpy(), U=U.float().numpy(),
        dec=dec_out.numpy(), dec_words=np.array([dec.cache_words()]))


def make_module(A, R, M, seed=300):
    """The reference's ``Attention(arm="smat")`` forward and input gradient
    (fp32, torch path on the CPU), plus ``make_phi`` outputs."""
    torch.manual_seed(seed)
    T, d_model, heads, nb = 512, 32, 2, 2
    spec = R.build_mask(T, 3, chunk=128)
    A.to_device(spec, "cpu")
    mod = M.Attention(d_model, heads, "smat", spec=spec, r=32, chunk=128, seed=7)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(nb, T, d_model, generator=g)
    dy = torch.randn(nb, T, d_model, generator=g)
    xg = x.clone().requires_grad_(True)
    y = mod(xg)
    (y * dy).sum().backward()
    xp = torch.randn(5, 16, generator=g)
    phi_elu = A.make_phi(16, 8, seed=3)(xp)
    phi_relu = A.make_phi(16, 8, kind="relu", seed=3)(xp)
    np.savez_compressed(
        os.path.join(HERE, "smat_module.npz"), args=np.array([T, d_model, heads, 32, 7]),
        qkv=mod.qkv.weight.detach().numpy(), out_w=mod.out.weight.detach().numpy(),
        x=x.numpy(), dy=dy.numpy(), y=y.detach().numpy(), dx=xg.grad.numpy(), xp=xp.numpy(),
        phi_elu=phi_elu.numpy(), phi_relu=phi_relu.numpy())


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SMAT_REFERENCE")
    if not ref:
        raise SystemExit("usage: make_golden.py <reference checkout>")
    sys.path.insert(0, os.path.join(ref, "src"))
    from smat import attention as A
    from smat import mask as R
    make_mask_md(R)
    for i, (name, T, BH, D, mask) in enumerate(SOFTMAX_CASES):
        make_softmax(A, R, name, T, BH, D, mask, seed=100 + i)
    make_softmax_c1(A, R)
    for i, case in enumerate(KATTN_CASES):
        make_kattn(A, R, *case, seed=200 + i)
    from smat import model as M
    make_module(A, R, M)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
