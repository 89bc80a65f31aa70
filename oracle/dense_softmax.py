"""Dense-masked softmax attention on the CPU -- TEST INFRASTRUCTURE ONLY.

The reference's dense-masked path is ``dense_masked_kernel_attention``
(``src/smat/attention.py:485-489``)::

    A = (Phi Psi^T) * M ;  H = A [V, 1] ;  out = H[:, :-1] / H[:, -1:]

Softmax attention is that same computation with ``Phi Psi^T`` replaced by the
shifted exponential ``exp(scale * Q K^T - m)``, ``m`` the masked row maximum.
:func:`dense_masked_softmax_attention` keeps that three-line form and also
returns the natural-log normaliser ``lse = m + log(H[:, -1])``.
:func:`dense_masked_softmax_backward` states the gradients explicitly (the
same formulas the GPU backward implements), so the tests can check them
against torch autograd as well as against the reference fixtures.

Inputs are torch CPU tensors of shape ``(..., T, D)`` in fp64 or fp32; the
computation runs in the input dtype.  ``M`` is a ``(T, T)`` 0/1 tensor.
"""

from __future__ import annotations

import math

import torch

__all__ = ["dense_masked_softmax_attention", "dense_masked_softmax_backward",
           "dense_masked_softmax_fwd_bwd"]


def _scores(q, k, M, scale):
    s = torch.einsum("...ta,...sa->...ts", q, k) * scale
    keep = M.to(torch.bool)
    return s.masked_fill(~keep, float("-inf")), keep


def dense_masked_softmax_attention(q, k, v, M, scale=None):
    """Return ``(o, lse)``: ``o = softmax_M(scale q k^T) v`` and the row
    log-sum-exp over the unmasked entries (``-inf`` for an empty row, whose
    output is 0)."""
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    s, keep = _scores(q, k, M, scale)
    m = s.amax(dim=-1, keepdim=True)
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    A = torch.exp(s - m) * keep.to(q.dtype)                      # masked exponentials
    ones = torch.ones(*v.shape[:-1], 1, dtype=v.dtype)
    H = torch.einsum("...ts,...sv->...tv", A, torch.cat([v, ones], dim=-1))
    denom = H[..., -1:]
    o = torch.where(denom > 0, H[..., :-1] / denom.clamp_min(torch.finfo(q.dtype).tiny),
                    torch.zeros_like(H[..., :-1]))
    lse = (m + torch.log(denom)).squeeze(-1)
    return o, lse


def dense_masked_softmax_backward(q, k, v, o, lse, do, M, scale=None):
    """Explicit gradients ``(dq, dk, dv)`` of ``<o, do>``.

    ``P = exp(scale q k^T - lse) * M``, ``dV = P^T dO``, ``dP = dO V^T``,
    ``delta = rowsum(dO * O)``, ``dS = P * (dP - delta)``,
    ``dQ = scale dS K``, ``dK = scale dS^T Q``.
    """
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    s, keep = _scores(q, k, M, scale)
    lse_f = torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))
    P = torch.exp(s - lse_f.unsqueeze(-1)) * keep.to(q.dtype)
    dv = torch.einsum("...ts,...td->...sd", P, do)
    dP = torch.einsum("...td,...sd->...ts", do, v)
    delta = (do * o).sum(-1, keepdim=True)
    dS = P * (dP - delta)
    dq = torch.einsum("...ts,...sd->...td", dS, k) * scale
    dk = torch.einsum("...ts,...td->...sd", dS, q) * scale
    return dq, dk, dv


def dense_masked_softmax_fwd_bwd(q, k, v, do, M, scale=None):
    """Forward then backward; returns ``(o, lse, dq, dk, dv)``."""
    o, lse = dense_masked_softmax_attention(q, k, v, M, scale)
    dq, dk, dv = dense_masked_softmax_backward(q, k, v, o, lse, do, M, scale)
    return o, lse, dq, dk, dv


def rowchunked_masked_softmax(q, k, v, do, mask_rows, scale=None, rows=1024,
                              backward=True):
    """The same dense-masked computation, evaluated ``rows`` query rows at a
    time so that long sequences fit in memory (it still visits every
    ``(i, j)`` pair: no block skipping).

    ``q, k, v, do``: ``(N, T, D)`` float tensors (fp64 or fp32, any device);
    ``mask_rows(r0, r1)`` returns the ``(r1 - r0, T)`` 0/1 mask rows.
    Returns ``(o, lse, dq, dk, dv)`` (the gradients are ``None`` when
    ``backward`` is False).
    """
    N, T, D = q.shape
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    o = torch.empty_like(q)
    lse = torch.empty(N, T, dtype=q.dtype, device=q.device)
    for r0 in range(0, T, rows):
        r1 = min(T, r0 + rows)
        keep = mask_rows(r0, r1).to(device=q.device, dtype=torch.bool)
        s = torch.einsum("nta,nsa->nts", q[:, r0:r1], k) * scale
        s = s.masked_fill(~keep, float("-inf"))
        m = s.amax(-1, keepdim=True)
        m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
        e = torch.exp(s - m)
        l = e.sum(-1, keepdim=True)
        o[:, r0:r1] = torch.where(l > 0, (e @ v) / l.clamp_min(torch.finfo(q.dtype).tiny),
                                  torch.zeros_like(o[:, r0:r1]))
        lse[:, r0:r1] = (m + torch.log(l)).squeeze(-1)
        del s, e
    if not backward:
        return o, lse, None, None, None
    delta = (do * o).sum(-1)
    dq = torch.empty_like(q)
    dk = torch.zeros_like(k)
    dv = torch.zeros_like(v)
    for r0 in range(0, T, rows):
        r1 = min(T, r0 + rows)
        keep = mask_rows(r0, r1).to(device=q.device, dtype=torch.bool)
        s = torch.einsum("nta,nsa->nts", q[:, r0:r1], k) * scale
        lf = lse[:, r0:r1]
        lf = torch.where(torch.isfinite(lf), lf, torch.zeros_like(lf))
        P = torch.exp(s - lf.unsqueeze(-1)) * keep.to(q.dtype)
        del s
        dv += torch.einsum("nts,ntd->nsd", P, do[:, r0:r1])
        dP = torch.einsum("ntd,nsd->nts", do[:, r0:r1], v)
        dS = P * (dP - delta[:, r0:r1].unsqueeze(-1))
        del P, dP
        dq[:, r0:r1] = torch.einsum("nts,nsd->ntd", dS, k) * scale
        dk += torch.einsum("nts,ntd->nsd", dS, q[:, r0:r1]) * scale
    return o, lse, dq, dk, dv
