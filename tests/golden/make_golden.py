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
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
