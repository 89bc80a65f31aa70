"""The reference's kernelised attention schedule on the CPU -- TEST
INFRASTRUCTURE ONLY.

A restatement, in torch and in the caller's dtype (fp64 in the tests), of the
pooled schedule of ``smat.attention.smat_attention``
(``src/smat/attention.py:391-455``) for ``M^(d)`` masks:

* causal part: one chunked scan with a reset at ``n``
  (``segmented_causal_scan``, ``attention.py:134-192``): per chunk
  ``Phi_b S_b + tril(Phi_b Psi_b^T) Vb_b`` with ``S_b`` the exclusive prefix
  sum of the chunk summaries ``Psi_c^T Vb_c`` inside each segment;
* long-range part: ``F_x = sum_{prof(j) = x} Psi_j Vb_j^T``
  (``pool_profiles``, ``:199-236``), ``U_h = sum_{x in H_h} F_x``
  (``apply_incidence``, ``:239-285``; the CSR rows of ``C``), plus the rank-one
  global term ``Psi_{<n_P}^T Vb_{<n_P}`` (``:425-429``), then
  ``Ybar_i = Phi_i U_{(i - n) mod B}`` for recent rows (``query_by_type``,
  ``:310-330``);
* the endpoint family's landmark block by the subset-sum (zeta) transform
  (``:364-381``, ``:432-441``);
* one division by the last column;
* the streaming decoder (``SmatDecoder``, ``attention.py:496-535``): the type
  table ``U`` from the prefix, then per token ``S += Psi_t Vb_t^T`` and
  ``Phi_t^T (S + U_{i mod B})``, divided by its last column.

Only the tests import this module; the product path is
``smat_attention_b200.kernel_attention``.
"""

from __future__ import annotations

import torch

__all__ = ["chunk_local", "segmented_causal_scan", "pool_profiles", "apply_incidence",
           "query_by_type", "zeta_transform", "smat_attention", "SmatDecoder"]


def chunk_local(Phi_c, Psi_c, Vb_c, Sin):
    """``Phi_b Sin_b + tril(Phi_b Psi_b^T) Vb_b`` per chunk; ``(nb, nc, C, .)``."""
    C = Phi_c.shape[-2]
    tri = torch.ones(C, C, dtype=Phi_c.dtype).tril()
    return Phi_c @ Sin + ((Phi_c @ Psi_c.transpose(-1, -2)) * tri) @ Vb_c


def segmented_causal_scan(Phi, Psi, Vb, n: int, chunk: int):
    nb, T, r = Phi.shape
    p = Vb.shape[-1]
    C = min(chunk, T)
    pad = (-T) % C
    if pad:
        Phi, Psi, Vb = (torch.nn.functional.pad(x, (0, 0, 0, pad)) for x in (Phi, Psi, Vb))
    nc = (T + pad) // C
    Phi_c = Phi.reshape(nb, nc, C, r)
    Psi_c = Psi.reshape(nb, nc, C, r)
    Vb_c = Vb.reshape(nb, nc, C, p)
    Dsum = Psi_c.transpose(-1, -2) @ Vb_c                           # (nb, nc, r, p)
    Sin = torch.zeros_like(Dsum)
    nc0 = n // C
    for lo, hi in ([(0, nc0), (nc0, nc)] if 0 < nc0 < nc else [(0, nc)]):
        run = torch.zeros_like(Dsum[:, 0])
        for c in range(lo, hi):                                      # exclusive prefix
            Sin[:, c] = run
            run = run + Dsum[:, c]
    out = chunk_local(Phi_c, Psi_c, Vb_c, Sin)
    return out.reshape(nb, T + pad, p)[:, :T]


def pool_profiles(Psi, Vb, spec):
    nb, _, r = Psi.shape
    p = Vb.shape[-1]
    n_P, n, N0 = spec.n_P, spec.n, spec.N0
    F = torch.zeros(nb, N0, r, p, dtype=Psi.dtype)
    for j in range(n_P, n):
        x = (j - n_P) % N0
        F[:, x] += Psi[:, j, :, None] * Vb[:, j, None, :]
    return F


def apply_incidence(F, spec):
    nb, _, r, p = F.shape
    U = torch.zeros(nb, spec.B, r, p, dtype=F.dtype)
    for h in range(spec.B):
        idx = torch.from_numpy(spec.C_indices[spec.C_indptr[h]:spec.C_indptr[h + 1]]).long()
        U[:, h] = F[:, idx].sum(1)
    return U


def query_by_type(Phi_rec, U, spec):
    T_R = Phi_rec.shape[1]
    rho = torch.arange(T_R) % spec.B
    return (Phi_rec.unsqueeze(-2) @ U[:, rho]).squeeze(-2)          # (nb, T_R, p)


def zeta_transform(F):
    """``(Z F)_a = sum_{x subset of a} F_x`` over the leading index (a power of two)."""
    N = F.shape[1]
    out = F.clone()
    b = 1
    while b < N:
        for a in range(N):
            if a & b:
                out[:, a] = out[:, a] + out[:, a ^ b]
        b <<= 1
    return out


def smat_attention(Phi, Psi, Vb, spec, chunk: int = 128):
    n = spec.n
    F = pool_profiles(Psi, Vb, spec)
    U = apply_incidence(F, spec)
    if spec.n_P:
        U = U + (Psi[:, :spec.n_P].transpose(-1, -2) @ Vb[:, :spec.n_P]).unsqueeze(1)
    Y_lr = query_by_type(Phi[:, n:], U, spec)
    if spec.kind == "endpoint":
        Fz = Psi[:, :n].unsqueeze(-1) * Vb[:, :n].unsqueeze(-2)
        top = (Phi[:, :n].unsqueeze(-2) @ zeta_transform(Fz)).squeeze(-2)
        loc = segmented_causal_scan(Phi[:, n:], Psi[:, n:], Vb[:, n:], 0, chunk)
        H = torch.cat([top, loc + Y_lr], dim=1)
    else:
        H = segmented_causal_scan(Phi, Psi, Vb, n, chunk)
        H = torch.cat([H[:, :n], H[:, n:] + Y_lr], dim=1)
    return H[..., :-1] / H[..., -1:]


class SmatDecoder:
    """Streaming decode over a pooled prefix (``attention.py:496-535``), in the
    dtype of its inputs."""

    def __init__(self, Psi_prefix, Vb_prefix, spec):
        self.spec = spec
        U = apply_incidence(pool_profiles(Psi_prefix, Vb_prefix, spec), spec)
        if spec.n_P:
            U = U + (Psi_prefix[:, :spec.n_P].transpose(-1, -2)
                     @ Vb_prefix[:, :spec.n_P]).unsqueeze(1)
        self.U = U
        nb, _, r = Psi_prefix.shape
        self.S = torch.zeros(nb, r, Vb_prefix.shape[-1], dtype=Psi_prefix.dtype)
        self.i = 0

    def step(self, Phi_t, Psi_t, Vb_t):
        self.S = self.S + Psi_t.unsqueeze(-1) * Vb_t.unsqueeze(-2)
        o = (Phi_t.unsqueeze(-2) @ (self.S + self.U[:, self.i % self.spec.B])).squeeze(-2)
        self.i += 1
        return o[..., :-1] / o[..., -1:]

    def cache_words(self) -> int:
        return int(self.S.numel() + self.U.numel())
