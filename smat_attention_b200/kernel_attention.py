"""The reference's kernelised SMat attention on B200 kernels.

``smat_attention(Phi, Psi, Vb, spec)`` computes what the reference's op
``smat.attention.smat_attention`` (``src/smat/attention.py:391-455``)
computes -- the pooled schedule of its Algorithm 1 for an ``M^(d)`` mask --
with the three passes its Triton module fuses replaced by kernels of
``libsmat_b200.so`` (``include/smat_kattn.h``):

``chunk_local(Phi_c, Psi_c, Vb_c, Sin)``
    ``Phi_b Sin_b + tril(Phi_b Psi_b^T) Vb_b`` per 128-row chunk on tcgen05
    tensor cores (TF32 inputs, fp32 accumulation: the reference's
    ``allow_tf32`` dots, ``kernels/triton_fwd.py:49-152``).  Backward: the
    contractions of the reference's two backward kernels
    (``kernels/triton_bwd.py:50-196``) as three more modes of the same tile
    kernel (dPhi, dVb, dPsi); ``dSin = Phi^T dOut`` is a batched GEMM.
``pool(Psi, Vb, n_P, n, N0)``
    ``F_x = sum_{prof(j) = x} Psi_j Vb_j^T`` (``triton_fwd.py:225-311``) and its
    backward (``triton_bwd.py:203-278``), fp32 on CUDA cores.
``incidence(F, plane_pts, B)``
    ``U_h = sum_{x in H_h} F_x`` (``triton_fwd.py:161-222``) with the transposed
    table as its backward (``triton_bwd.py:281-316``), fp32 on CUDA cores.
``SmatDecoder``
    the streaming decoder (``attention.py:496-535``): the prefill builds the
    type table ``U`` with ``pool`` and ``incidence``; each token is one launch
    that updates the running sum ``S``, queries ``S + U_h`` and normalises.

The scan summaries, the segmented prefix sums, the per-type query
(``query_by_type``) and the endpoint's butterflies are batched library GEMMs
and torch reductions, as in the reference.  All arithmetic is fp32 (inputs of
lower precision are promoted); there is no CPU path.
"""

from __future__ import annotations

import contextlib
import ctypes

import numpy as np
import torch

from . import _lib
from .mask import MaskSpec

__all__ = ["chunk_local", "pool", "incidence", "segmented_causal_scan", "pool_profiles",
           "apply_incidence", "query_by_type", "walsh_incidence", "zeta_transform",
           "direct_long_range", "smat_attention", "SmatDecoder", "normalise", "make_phi",
           "featurise", "PhaseTimer"]

_vp, _ci, _cl = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
SIGNATURES = {
    "smat_kattn_chunk_local_fwd": (_ci, [_vp, _vp, _vp, _vp, _vp, _cl, _ci, _ci, _ci, _vp, _vp]),
    "smat_kattn_chunk_local_bwd": (_ci, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _cl, _ci, _ci,
                                         _ci, _vp, _vp]),
    "smat_kattn_pool_fwd": (_ci, [_vp, _vp, _vp, _ci, _ci, _ci, _ci, _ci, _ci, _ci, _vp]),
    "smat_kattn_pool_bwd": (_ci, [_vp, _vp, _vp, _vp, _vp, _ci, _ci, _ci, _ci, _ci, _ci, _ci,
                                  _vp]),
    "smat_kattn_incidence": (_ci, [_vp, _vp, _vp, _vp, _ci, _ci, _ci, _ci, _vp, _vp]),
    "smat_kattn_decode_step": (_ci, [_vp, _vp, _vp, _vp, _vp, _vp, _ci, _ci, _ci, _ci, _ci,
                                     _vp]),
    "smat_kattn_normalise_fwd": (_ci, [_vp, _vp, _cl, _ci, _vp]),
    "smat_kattn_normalise_bwd": (_ci, [_vp, _vp, _vp, _cl, _ci, _vp]),
    "smat_kattn_chunk_prefix": (_ci, [_vp, _vp, _vp, _ci, _ci, _ci, _ci, _ci, _ci, _ci, _vp]),
    "smat_kattn_chunk_expand": (_ci, [_vp, _vp, _vp, _vp, _vp, _ci, _ci, _ci, _ci, _ci, _vp]),
    "smat_kattn_query_by_type": (_ci, [_vp, _cl, _vp, _vp, _cl, _ci, _ci, _ci, _ci, _ci, _ci,
                                       _vp]),
    "smat_kattn_query_by_type_bwd": (_ci, [_vp, _cl, _vp, _vp, _cl, _vp, _cl, _vp, _ci, _ci,
                                           _ci, _ci, _ci, _vp]),
}
CHUNK = 128
_bound = None


def _L():
    global _bound
    if _bound is None:
        L = _lib.lib()
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        _bound = L
    return _bound


def _f32(x):
    if not x.is_cuda:
        raise ValueError("the kernelised-attention kernels take CUDA tensors (no CPU path)")
    return x.float().contiguous()


def _stream(x):
    return torch.cuda.current_stream(x.device).cuda_stream


def _err(device):
    from .attention import _err_word
    return _err_word(device).data_ptr()


# ---------------------------------------------------------------- chunk_local
class _ChunkLocal(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Phi_c, Psi_c, Vb_c, Sin):
        nb, nc, C, R = Phi_c.shape
        P = Vb_c.shape[-1]
        q, k, v, s = (_f32(x) for x in (Phi_c, Psi_c, Vb_c, Sin))
        out = torch.empty(nb, nc, C, P, dtype=torch.float32, device=q.device)
        _lib.check("smat_kattn_chunk_local_fwd", _L().smat_kattn_chunk_local_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), s.data_ptr(), out.data_ptr(), nb * nc, C,
            R, P, _err(q.device), _stream(q)))
        ctx.save_for_backward(q, k, v, s)
        ctx.dtypes = tuple(x.dtype for x in (Phi_c, Psi_c, Vb_c, Sin))
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, s = ctx.saved_tensors
        nb, nc, C, R = q.shape
        P = v.shape[-1]
        do = dout.float().contiguous()
        dq, dk = torch.empty_like(q), torch.empty_like(k)
        dv = torch.empty_like(v)
        _lib.check("smat_kattn_chunk_local_bwd", _L().smat_kattn_chunk_local_bwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), s.data_ptr(), do.data_ptr(),
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), nb * nc, C, R, P, _err(q.device),
            _stream(q)))
        ds = q.transpose(-1, -2) @ do          # (nb, nc, r, p), a plain batched GEMM
        return tuple(g.to(t) for g, t in zip((dq, dk, dv, ds), ctx.dtypes))


def chunk_local(Phi_c, Psi_c, Vb_c, Sin):
    """``Phi_b Sin_b + tril(Phi_b Psi_b^T) Vb_b`` for every chunk ``b``.

    ``(nb, nc, C, r), (nb, nc, C, r), (nb, nc, C, p), (nb, nc, r, p) -> (nb, nc, C, p)``
    fp32; ``C = 128``, ``r`` in {32, 64, 128}, ``p <= 128`` (``<= 96`` at ``r = 128``).
    """
    return _ChunkLocal.apply(Phi_c, Psi_c, Vb_c, Sin)


# ---------------------------------------------------------------- pool
class _Pool(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Psi, Vb, n_P, n, N0):
        nb, T, R = Psi.shape
        P = Vb.shape[-1]
        k, v = _f32(Psi), _f32(Vb)
        F = torch.empty(nb, N0, R, P, dtype=torch.float32, device=k.device)
        _lib.check("smat_kattn_pool_fwd", _L().smat_kattn_pool_fwd(
            k.data_ptr(), v.data_ptr(), F.data_ptr(), nb, T, R, P, n_P, n, N0, _stream(k)))
        ctx.save_for_backward(k, v)
        ctx.dims = (n_P, n, N0)
        ctx.dtypes = (Psi.dtype, Vb.dtype)
        return F

    @staticmethod
    def backward(ctx, dF):
        k, v = ctx.saved_tensors
        n_P, n, N0 = ctx.dims
        nb, T, R = k.shape
        P = v.shape[-1]
        dk, dv = torch.zeros_like(k), torch.zeros_like(v)
        dF = dF.float().contiguous()
        _lib.check("smat_kattn_pool_bwd", _L().smat_kattn_pool_bwd(
            k.data_ptr(), v.data_ptr(), dF.data_ptr(), dk.data_ptr(), dv.data_ptr(), nb, T, R,
            P, n_P, n, N0, _stream(k)))
        return dk.to(ctx.dtypes[0]), dv.to(ctx.dtypes[1]), None, None, None


def pool(Psi, Vb, n_P: int, n: int, N0: int):
    """``F_x = sum_{prof(j) = x} Psi_j Vb_j^T``: ``(nb, T, r), (nb, T, p) -> (nb, N0, r, p)``."""
    return _Pool.apply(Psi, Vb, int(n_P), int(n), int(N0))


# ---------------------------------------------------------------- incidence
def _csr_of_table(plane_pts):
    B, deg = plane_pts.shape
    ptr = torch.arange(B + 1, dtype=torch.int64, device=plane_pts.device) * deg
    return ptr, plane_pts.reshape(-1).to(torch.int32).contiguous()


def _transpose_csr(ptr, idx, n_cols):
    """(ptr, idx) of the rows listing each column, rows ascending per column."""
    rows = torch.repeat_interleave(torch.arange(ptr.numel() - 1, device=idx.device),
                                   ptr[1:] - ptr[:-1])
    order = torch.argsort(idx.long() * (ptr.numel()) + rows, stable=True)
    t_idx = rows[order].to(torch.int32).contiguous()
    counts = torch.bincount(idx.long(), minlength=n_cols)
    t_ptr = torch.zeros(n_cols + 1, dtype=torch.int64, device=idx.device)
    t_ptr[1:] = torch.cumsum(counts, 0)
    return t_ptr, t_idx


def _gather_sum(F, ptr, idx, n_out):
    nb, n_in = F.shape[:2]
    RP = int(np.prod(F.shape[2:]))
    Ff = _f32(F)
    U = torch.empty(nb, n_out, *F.shape[2:], dtype=torch.float32, device=F.device)
    _lib.check("smat_kattn_incidence", _L().smat_kattn_incidence(
        Ff.data_ptr(), ptr.data_ptr(), idx.data_ptr(), U.data_ptr(), nb, n_in, n_out, RP,
        _err(F.device), _stream(Ff)))
    return U


class _Incidence(torch.autograd.Function):
    """``U = C F`` as a CSR gather-sum; the backward is the same kernel over
    the transposed table (given, or built on the device when needed)."""

    @staticmethod
    def forward(ctx, F, ptr, idx, n_out, t_ptr=None, t_idx=None):
        if t_ptr is None:
            ctx.save_for_backward(ptr, idx)
        else:
            ctx.save_for_backward(t_ptr, t_idx)
        ctx.transposed = t_ptr is not None
        ctx.n_in = F.shape[1]
        ctx.dtype = F.dtype
        return _gather_sum(F, ptr, idx, n_out)

    @staticmethod
    def backward(ctx, dU):
        a, b = ctx.saved_tensors
        t_ptr, t_idx = (a, b) if ctx.transposed else _transpose_csr(a, b, ctx.n_in)
        return (_gather_sum(dU, t_ptr, t_idx, ctx.n_in).to(ctx.dtype),
                None, None, None, None, None)


def incidence(F, plane_pts, B: int):
    """``U_h = sum_{x in H_h} F_x`` with ``plane_pts (B, deg)`` the points of
    each hyperplane: ``(nb, N0, r, p) -> (nb, B, r, p)``."""
    ptr, idx = _csr_of_table(plane_pts)
    return _Incidence.apply(F, ptr, idx, int(B))


def _transpose_csr_host(ptr, idx, n_cols):
    """``_transpose_csr`` on the host (numpy): rows ascending per column."""
    ptr = np.asarray(ptr, np.int64)
    idx = np.asarray(idx, np.int64)
    rows = np.repeat(np.arange(len(ptr) - 1, dtype=np.int64), np.diff(ptr))
    order = np.argsort(idx * len(ptr) + rows, kind="stable")
    t_ptr = np.zeros(n_cols + 1, np.int64)
    t_ptr[1:] = np.cumsum(np.bincount(idx, minlength=n_cols))
    return t_ptr, rows[order].astype(np.int32)


def _incidence_csr(F, spec: MaskSpec):
    """The op's incidence with the spec's table and its transpose staged on
    the device once (the backward then reads the cached transpose)."""
    key = ("kattn_csr", str(F.device))
    if key not in spec.dev:
        as_t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a, dt)).to(F.device)
        t_ptr, t_idx = _transpose_csr_host(spec.C_indptr, spec.C_indices, F.shape[1])
        spec.dev[key] = (as_t(spec.C_indptr, np.int64), as_t(spec.C_indices, np.int32),
                         as_t(t_ptr, np.int64), as_t(t_idx, np.int32))
    ptr, idx, t_ptr, t_idx = spec.dev[key]
    return _Incidence.apply(F, ptr, idx, int(spec.B), t_ptr, t_idx)


# ---------------------------------------------------------------- normalisation
class _Normalise(torch.autograd.Function):
    """``H[..., :-1] / H[..., -1:]`` (reference ``attention.py:450-451``) and its
    backward, one kernel each."""

    @staticmethod
    def forward(ctx, H):
        h = _f32(H)
        p = h.shape[-1]
        out = torch.empty(*h.shape[:-1], p - 1, dtype=torch.float32, device=h.device)
        _lib.check("smat_kattn_normalise_fwd", _L().smat_kattn_normalise_fwd(
            h.data_ptr(), out.data_ptr(), h.numel() // p, p, _stream(h)))
        ctx.save_for_backward(h)
        return out

    @staticmethod
    def backward(ctx, dout):
        (h,) = ctx.saved_tensors
        p = h.shape[-1]
        g = dout.float().contiguous()
        dH = torch.empty_like(h)
        _lib.check("smat_kattn_normalise_bwd", _L().smat_kattn_normalise_bwd(
            h.data_ptr(), g.data_ptr(), dH.data_ptr(), h.numel() // p, p, _stream(h)))
        return dH


def normalise(H):
    """``H[..., :-1] / H[..., -1:]`` for fp32 CUDA ``H`` (the op's last step)."""
    return _Normalise.apply(H)


# ---------------------------------------------------------------- the schedule
_BACKENDS = ("auto", "triton", "torch", "walsh")


def _check_acc(acc_dtype):
    if acc_dtype not in (None, torch.float32):
        raise ValueError("the B200 kernels accumulate in fp32 (acc_dtype None or torch.float32); "
                         "fp64 belongs to the oracle")


def _check_backend(name, value):
    if value not in _BACKENDS:
        raise ValueError(f"{name}={value!r}: expected one of {_BACKENDS}")


class _CausalScan(torch.autograd.Function):
    """``[[L_n, 0], [0, L_{T_R}]] Phi Psi^T Vb`` on whole chunks: the chunk
    prefix kernel (summaries ``Psi_c^T Vb_c`` and their shifted, segmented scan,
    ``Sin``), then the tcgen05 chunk pass.  Backward: the chunk pass's three
    gradients, ``dD`` = the reverse segmented scan of ``Phi_c^T dOut_c`` (the
    same prefix kernel), and its expansion into ``dPsi`` and ``dVb``."""

    @staticmethod
    def forward(ctx, Phi, Psi, Vb, nc0):
        nb, T, r = Phi.shape
        p = Vb.shape[-1]
        nc = T // CHUNK
        q, k, v = _f32(Phi), _f32(Psi), _f32(Vb)
        L = _L()
        Sin = torch.empty(nb, nc, r, p, dtype=torch.float32, device=q.device)
        _lib.check("smat_kattn_chunk_prefix", L.smat_kattn_chunk_prefix(
            k.data_ptr(), v.data_ptr(), Sin.data_ptr(), nb, T, CHUNK, r, p, nc0, 0, _stream(k)))
        out = torch.empty(nb, T, p, dtype=torch.float32, device=q.device)
        _lib.check("smat_kattn_chunk_local_fwd", L.smat_kattn_chunk_local_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), Sin.data_ptr(), out.data_ptr(), nb * nc,
            CHUNK, r, p, _err(q.device), _stream(q)))
        ctx.save_for_backward(q, k, v, Sin)
        ctx.nc0 = nc0
        ctx.dtypes = (Phi.dtype, Psi.dtype, Vb.dtype)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, Sin = ctx.saved_tensors
        nb, T, r = q.shape
        p = v.shape[-1]
        nc = T // CHUNK
        do = dout.float().contiguous()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        L = _L()
        s = _stream(q)
        _lib.check("smat_kattn_chunk_local_bwd", L.smat_kattn_chunk_local_bwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), Sin.data_ptr(), do.data_ptr(),
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), nb * nc, CHUNK, r, p, _err(q.device), s))
        dD = torch.empty_like(Sin)
        _lib.check("smat_kattn_chunk_prefix", L.smat_kattn_chunk_prefix(
            q.data_ptr(), do.data_ptr(), dD.data_ptr(), nb, T, CHUNK, r, p, ctx.nc0, 1, s))
        _lib.check("smat_kattn_chunk_expand", L.smat_kattn_chunk_expand(
            k.data_ptr(), v.data_ptr(), dD.data_ptr(), dk.data_ptr(), dv.data_ptr(), nb, T, CHUNK,
            r, p, s))
        return tuple(g.to(t) for g, t in zip((dq, dk, dv), ctx.dtypes)) + (None,)


def segmented_causal_scan(Phi, Psi, Vb, n: int, chunk: int = CHUNK, acc_dtype=None,
                          backend: str = "auto"):
    """``[[L_n, 0], [0, L_{T_R}]] Phi Psi^T Vb`` by chunks with one reset at ``n``
    (reference ``attention.py:134-192``): chunk summaries ``Psi_c^T Vb_c``, a
    shifted prefix sum inside each segment (a chunk's own summary never enters
    its prefix, and the landmark segment never reaches the recent one), then
    the chunk pass; all in ``libsmat_b200.so`` kernels, fp32.  ``backend`` takes
    the reference's names; every one runs these kernels."""
    _check_acc(acc_dtype)
    _check_backend("backend", backend)
    if chunk != CHUNK:
        raise ValueError(f"the chunk-local kernel runs chunks of {CHUNK} rows")
    nb, T, r = Phi.shape
    C = CHUNK
    if n % C:
        raise ValueError(f"segment boundary n={n} is not a multiple of chunk={C}")
    pad = (-T) % C
    if pad:                                   # the tail lives in the recent segment
        Phi, Psi, Vb = (torch.nn.functional.pad(x.float(), (0, 0, 0, pad))
                        for x in (Phi, Psi, Vb))
    out = _CausalScan.apply(Phi, Psi, Vb, n // C)
    return out[:, :T] if pad else out


def pool_profiles(Psi, Vb, spec: MaskSpec, acc_dtype=None, backend: str = "auto"):
    """``F`` over the landmark columns ``[n_P, n)`` (reference ``attention.py:199-236``)."""
    _check_acc(acc_dtype)
    _check_backend("backend", backend)
    return pool(Psi, Vb, spec.n_P, spec.n, spec.N0)


def walsh_incidence(F):
    """``C = (J + H) / 2`` applied by a Walsh butterfly (the endpoint family;
    reference ``attention.py:288-307``)."""
    nb, N, r, p = F.shape
    k = N.bit_length() - 1
    tot = F.sum(1, keepdim=True)
    H = F.reshape(nb, N, r * p)
    for j in range(k):
        H = H.reshape(nb, N >> (j + 1), 2, 1 << j, r * p)
        a, b = H[:, :, 0], H[:, :, 1]
        H = torch.stack([a + b, a - b], dim=2).reshape(nb, N, r * p)
    return 0.5 * (tot + H.reshape(nb, N, r, p))


def apply_incidence(F, spec: MaskSpec, *, backend: str = "auto", gather_chunk: int = 0):
    """``U_h = sum_{x in H_h} F_x`` (reference ``attention.py:239-285``): the Walsh
    butterfly for the endpoint family under ``"auto"`` / ``"walsh"`` (as in the
    reference), else the CSR gather-sum kernel (any row degree).
    ``gather_chunk`` is the reference's torch-path knob and has no effect."""
    _check_backend("backend", backend)
    if spec.kind == "endpoint" and backend in ("auto", "walsh"):
        return walsh_incidence(F)
    return _incidence_csr(F, spec)


class _Query(torch.autograd.Function):
    """``Y_i = Phi_i U_{i mod B}`` for the rows of ``Phi_rec`` (``query_by_type``
    kernel; backward: ``query_by_type_bwd``)."""

    @staticmethod
    def forward(ctx, Phi_rec, U):
        nb, T_R, r = Phi_rec.shape
        B, p = U.shape[1], U.shape[-1]
        ph, u = _f32(Phi_rec), _f32(U)
        Y = torch.empty(nb, T_R, p, dtype=torch.float32, device=ph.device)
        _lib.check("smat_kattn_query_by_type", _L().smat_kattn_query_by_type(
            ph.data_ptr(), T_R * r, u.data_ptr(), Y.data_ptr(), T_R * p, nb, T_R, r, p, B, 0,
            _stream(ph)))
        ctx.save_for_backward(ph, u)
        ctx.dtypes = (Phi_rec.dtype, U.dtype)
        return Y

    @staticmethod
    def backward(ctx, dY):
        ph, u = ctx.saved_tensors
        nb, T_R, r = ph.shape
        B, p = u.shape[1], u.shape[-1]
        d = dY.float().contiguous()
        dph, du = torch.empty_like(ph), torch.empty_like(u)
        _lib.check("smat_kattn_query_by_type_bwd", _L().smat_kattn_query_by_type_bwd(
            ph.data_ptr(), T_R * r, u.data_ptr(), d.data_ptr(), T_R * p, dph.data_ptr(), T_R * r,
            du.data_ptr(), nb, T_R, r, p, B, _stream(ph)))
        return dph.to(ctx.dtypes[0]), du.to(ctx.dtypes[1])


class _QueryAdd(torch.autograd.Function):
    """``H[:, n:] += query_by_type(Phi[:, n:], U)`` in place on ``H`` (no
    ``(nb, T_R, p)`` intermediate); ``Phi`` is the whole ``(nb, T, r)``."""

    @staticmethod
    def forward(ctx, H, Phi, U, n):
        nb, T, p = H.shape
        r, B = Phi.shape[-1], U.shape[1]
        ph, u = _f32(Phi), _f32(U)
        if H.dtype != torch.float32 or not H.is_contiguous():
            raise ValueError("H must be a contiguous fp32 tensor")
        T_R = T - n
        _lib.check("smat_kattn_query_by_type", _L().smat_kattn_query_by_type(
            ph.data_ptr() + 4 * n * r, T * r, u.data_ptr(), H.data_ptr() + 4 * n * p, T * p, nb,
            T_R, r, p, B, 1, _stream(ph)))
        ctx.mark_dirty(H)
        ctx.save_for_backward(ph, u)
        ctx.n = n
        ctx.dtypes = (Phi.dtype, U.dtype)
        return H

    @staticmethod
    def backward(ctx, dH):
        ph, u = ctx.saved_tensors
        n = ctx.n
        nb, T, r = ph.shape
        B, p = u.shape[1], u.shape[-1]
        d = dH.float().contiguous()
        dph = torch.empty_like(ph)
        if n:
            dph[:, :n].zero_()
        du = torch.empty_like(u)
        _lib.check("smat_kattn_query_by_type_bwd", _L().smat_kattn_query_by_type_bwd(
            ph.data_ptr() + 4 * n * r, T * r, u.data_ptr(), d.data_ptr() + 4 * n * p, T * p,
            dph.data_ptr() + 4 * n * r, T * r, du.data_ptr(), nb, T - n, r, p, B, _stream(ph)))
        return dH, dph.to(ctx.dtypes[0]), du.to(ctx.dtypes[1]), None


def query_by_type(Phi_rec, U, spec: MaskSpec):
    """``Ybar_i = Phi_i U_{(i - n) mod B}`` for the recent rows (reference
    ``attention.py:310-330``): the ``query_by_type`` kernel, one CTA per row
    type and sequence."""
    if U.shape[1] != spec.B:
        raise ValueError(f"U has {U.shape[1]} types, the spec {spec.B}")
    return _Query.apply(Phi_rec, U)


def zeta_transform(F):
    """``(Z F)_a = sum_{x subset of a} F_x`` by a butterfly (reference
    ``attention.py:364-381``)."""
    nb, N, r, p = F.shape
    k = N.bit_length() - 1
    H = F.reshape(nb, N, r * p)
    for j in range(k):
        H = H.reshape(nb, N >> (j + 1), 2, 1 << j, r * p)
        a, b = H[:, :, 0], H[:, :, 1]
        H = torch.stack([a, a + b], dim=2).reshape(nb, N, r * p)
    return H.reshape(nb, N, r, p)


def direct_long_range(Psi, Vb, spec: MaskSpec, acc_dtype=None, type_chunk: int = 64):
    """The unpooled comparison backend (reference ``attention.py:333-362``):
    every landmark column scattered to its row types, ``U_h = sum over the
    columns of type h of Psi_j Vb_j^T`` -- a factor ``~T^{1/d}`` more work than
    the pooled route; batched library GEMMs over the reference's padded column
    table ``spec.type_cols_t`` (``to_device(spec, device, want_direct=True)``)."""
    _check_acc(acc_dtype)
    cols = spec.type_cols_t
    if cols is None:
        raise ValueError("the direct backend needs to_device(..., want_direct=True)")
    nb, _, r = Psi.shape
    p = Vb.shape[-1]
    B, kap = cols.shape
    Ps = torch.cat([Psi[:, spec.n_P:spec.n].float(), Psi.new_zeros(nb, 1, r, dtype=torch.float32)],
                   dim=1)
    Vs = torch.cat([Vb[:, spec.n_P:spec.n].float(), Vb.new_zeros(nb, 1, p, dtype=torch.float32)],
                   dim=1)
    U = torch.empty(nb, B, r, p, device=Psi.device, dtype=torch.float32)
    for lo in range(0, B, type_chunk):
        hi = min(lo + type_chunk, B)
        c = cols[lo:hi].reshape(-1).long()
        U[:, lo:hi] = (Ps[:, c].reshape(nb, hi - lo, kap, r).transpose(-1, -2)
                       @ Vs[:, c].reshape(nb, hi - lo, kap, p))
    return U


def _nullcontext_timer(name):
    return contextlib.nullcontext()


def smat_attention(Phi, Psi, Vb, spec: MaskSpec, *, chunk: int = CHUNK, g=None, acc_dtype=None,
                   timer=None, long_range: str = "pooled", scan_backend: str = "auto",
                   incidence_backend: str = "auto", return_parts: bool = False):
    """The reference's op ``smat_attention`` (``attention.py:391-455``) on these
    kernels: the long-range pass (pool, incidence, the rank-one ``n_P`` term,
    the per-type query) and the segmented causal scan, summed before one
    division.  Returns ``(nb, T, p - 1)`` fp32, or ``(out, parts)`` with
    ``return_parts`` (``U``, ``Y_lr``, ``H``; ``zeta`` for the endpoint family;
    ``H``, ``Y_ex`` for ``"subtractive"``).

    * ``long_range``: ``"pooled"`` (the schedule), ``"direct"`` (the unpooled
      comparison, needs ``to_device(spec, dev, want_direct=True)``), or
      ``"subtractive"`` (one unbroken scan minus the excluded mass, the form
      the reference computes only to measure its cancellation);
    * ``timer``: a callable ``timer(name)`` returning a context manager around
      each phase (``lr_pool``, ``lr_incidence``, ``lr_query``, ``zeta``,
      ``scan``, ``normalise``), e.g. :class:`PhaseTimer`;
    * ``acc_dtype``: ``None`` or ``torch.float32`` (the kernels accumulate in
      fp32; the fp64 path is the oracle's);
    * ``scan_backend`` / ``incidence_backend``: the reference's names, all
      running these kernels (``"walsh"`` / ``"auto"`` pick the Walsh butterfly
      for the endpoint family, as there)."""
    _check_acc(acc_dtype)
    _check_backend("scan_backend", scan_backend)
    _check_backend("incidence_backend", incidence_backend)
    if spec.kind not in ("geometric", "endpoint"):
        raise ValueError("smat_attention needs an M^(d) spec from build_mask")
    if long_range not in ("pooled", "direct", "subtractive"):
        raise ValueError(f"unknown long_range {long_range!r}")
    tm = timer or _nullcontext_timer
    n = spec.n
    parts = {}
    if long_range == "subtractive":
        if spec.kind != "geometric":
            raise ValueError("the subtractive form is defined for the geometric family")
        with tm("lr_pool"):
            F = pool_profiles(Psi, Vb, spec)
        with tm("lr_incidence"):
            U = apply_incidence(F, spec, backend=incidence_backend)
            Ubar = F.sum(1, keepdim=True) - U
        with tm("lr_query"):
            Y_ex = query_by_type(Phi[:, n:], Ubar, spec)
        with tm("scan"):
            H = segmented_causal_scan(Phi, Psi, Vb, 0, chunk)
        H = torch.cat([H[:, :n], H[:, n:] - Y_ex], dim=1)
        with tm("normalise"):
            out = normalise(H)
            if g is not None:
                out = out * g.unsqueeze(-1).to(out.dtype)
        return (out, {"H": H, "Y_ex": Y_ex}) if return_parts else out

    with tm("lr_pool"):
        F = pool_profiles(Psi, Vb, spec)
    with tm("lr_incidence"):
        if long_range == "direct":
            U = direct_long_range(Psi, Vb, spec)
        else:
            U = apply_incidence(F, spec, backend=incidence_backend)
        if spec.n_P:                                   # the rank-one global term
            b = Psi[:, :spec.n_P].float().transpose(-1, -2) @ Vb[:, :spec.n_P].float()
            U = U + b.unsqueeze(1)
    Y_lr = None
    if spec.kind == "endpoint" or return_parts:
        with tm("lr_query"):
            Y_lr = query_by_type(Phi[:, n:], U, spec)
    if spec.kind == "endpoint":
        with tm("zeta"):
            Fz = Psi[:, :n].float().unsqueeze(-1) * Vb[:, :n].float().unsqueeze(-2)
            top = (Phi[:, :n].float().unsqueeze(-2) @ zeta_transform(Fz)).squeeze(-2)
        with tm("scan"):
            loc = segmented_causal_scan(Phi[:, n:], Psi[:, n:], Vb[:, n:], 0, chunk)
        H = torch.cat([top, loc + Y_lr], dim=1)
        parts["zeta"] = top
    else:
        with tm("scan"):
            H = segmented_causal_scan(Phi, Psi, Vb, n, chunk)
        if Y_lr is None and not H.is_contiguous():   # a padded tail leaves a strided view
            with tm("lr_query"):
                Y_lr = query_by_type(Phi[:, n:], U, spec)
        if Y_lr is not None:
            H = torch.cat([H[:, :n], H[:, n:] + Y_lr], dim=1)
        else:
            with tm("lr_query"):   # added into the recent rows in place
                H = _QueryAdd.apply(H, Phi, U, n)
    parts.update(U=U, Y_lr=Y_lr, H=H)
    with tm("normalise"):
        out = normalise(H)
        if g is not None:
            out = out * g.unsqueeze(-1).to(out.dtype)
    return (out, parts) if return_parts else out


class PhaseTimer:
    """``with timer("name"):`` attribution with CUDA events, accumulated per
    name (the reference's ``PhaseTimer``, ``analysis/bench_prefill.py:51-75``);
    pass it as ``smat_attention(..., timer=PhaseTimer(device))``."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.spans = []

    @contextlib.contextmanager
    def __call__(self, name):
        a, b = (torch.cuda.Event(enable_timing=True) for _ in range(2))
        a.record(torch.cuda.current_stream(self.device))
        yield
        b.record(torch.cuda.current_stream(self.device))
        self.spans.append((name, a, b))

    def results(self):
        torch.cuda.synchronize(self.device)
        out = {}
        for name, a, b in self.spans:
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out


# ---------------------------------------------------------------- feature maps
def make_phi(d_qk: int, r: int, *, kind: str = "elu1", device="cpu", dtype=torch.float32,
             seed: int = 0):
    """A strictly positive feature map ``R^{d_qk} -> R^r`` (reference
    ``attention.py:82-97``): the same random projection for the same seed
    (``N(0, 1) / sqrt(d_qk)`` drawn in fp64 from a CPU generator), then
    ``elu + 1`` or ``relu + 1e-3``."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    W = (torch.randn(r, d_qk, generator=gen, dtype=torch.float64)
         / np.sqrt(d_qk)).to(device=device, dtype=dtype)
    if kind == "elu1":
        return lambda x: torch.nn.functional.elu(x @ W.T) + 1.0
    if kind == "relu":
        return lambda x: torch.nn.functional.relu(x @ W.T) + 1e-3
    raise ValueError(f"unknown feature map {kind!r}")


def featurise(Q, K, V, phi, *, g=None, h=None):
    """``(Q, K, V) -> (Phi, Psi, Vb)`` with the key gate ``h`` folded into
    ``Psi`` and ``Vb = [V, 1]`` (reference ``attention.py:100-106``)."""
    Phi = phi(Q)
    Psi = phi(K)
    if h is not None:
        Psi = Psi * h.unsqueeze(-1)
    ones = torch.ones(*V.shape[:-1], 1, device=V.device, dtype=V.dtype)
    return Phi, Psi, torch.cat([V, ones], dim=-1)


# ---------------------------------------------------------------- streaming decode
class SmatDecoder:
    """Exact autoregressive decoding at ``O(r p)`` per token (reference
    ``SmatDecoder``, ``attention.py:496-535``).

    Every landmark key precedes every recent query, so the type table
    ``U_h`` is fixed once the prefix is pooled; token ``n + i`` is
    ``Phi^T (U_{i mod B} + sum_{n < u <= n + i} Psi_u Vb_u^T)``.  The prefill
    runs the ``pool`` and ``incidence`` kernels (plus the rank-one global term
    for ``n_P > 0``); each :meth:`step` is one ``smat_kattn_decode_step``
    launch over all ``nb`` sequences.  State and arithmetic are fp32;
    ``acc_dtype`` other than fp32 is rejected (there is no CPU path).
    ``incidence_backend`` is accepted for the reference's signature; the
    incidence always runs the CSR kernel (the Walsh butterfly for the
    endpoint family)."""

    def __init__(self, Psi_prefix, Vb_prefix, spec: MaskSpec, *, acc_dtype=None,
                 incidence_backend: str = "auto"):
        if acc_dtype not in (None, torch.float32):
            raise ValueError("the decode kernel accumulates in fp32")
        if spec.kind not in ("geometric", "endpoint"):
            raise ValueError("SmatDecoder needs an M^(d) spec from build_mask")
        self.spec = spec
        self.acc = torch.float32
        nb, _, r = Psi_prefix.shape
        p = Vb_prefix.shape[-1]
        self.nb, self.r, self.p = nb, r, p
        F = pool_profiles(Psi_prefix, Vb_prefix, spec)
        U = apply_incidence(F, spec)
        if spec.n_P:
            b = (Psi_prefix[:, :spec.n_P].float().transpose(-1, -2)
                 @ Vb_prefix[:, :spec.n_P].float())
            U = U + b.unsqueeze(1)
        self.U = U.float().contiguous()
        self.S = torch.zeros(nb, r, p, device=Psi_prefix.device, dtype=torch.float32)
        self.i = 0
        self._fn = None
        self._S_ptr, self._U_ptr, self._nU = self.S.data_ptr(), self.U.data_ptr(), self.U.shape[1]

    def step(self, Phi_t, Psi_t, Vb_t):
        """One token: ``Phi_t, Psi_t (nb, r)``, ``Vb_t (nb, p)`` -> ``(nb, p - 1)`` fp32."""
        dev = self.S.device
        ins = []
        for x in (Phi_t, Psi_t, Vb_t):
            # tokens usually arrive fp32 and contiguous on the device: no copies
            if not (x.dtype is torch.float32 and x.device == dev and x.is_contiguous()):
                if x.device.type != "cuda":
                    raise ValueError("SmatDecoder.step takes CUDA tensors (there is no CPU path)")
                x = x.to(dev, torch.float32).contiguous()
            ins.append(x)
        phi, psi, vb = ins
        if phi.shape != (self.nb, self.r) or psi.shape != (self.nb, self.r) \
                or vb.shape != (self.nb, self.p):
            raise ValueError("step expects Phi_t, Psi_t (nb, r) and Vb_t (nb, p)")
        out = torch.empty(self.nb, self.p - 1, dtype=torch.float32, device=dev)
        if self._fn is None:
            self._fn = _L().smat_kattn_decode_step
        args = (phi.data_ptr(), psi.data_ptr(), vb.data_ptr(), self._S_ptr, self._U_ptr,
                out.data_ptr(), self.nb, self.r, self.p, self._nU, self.i % self.spec.B,
                torch.cuda.current_stream(dev).cuda_stream)
        if torch.cuda.current_device() == dev.index:
            rc = self._fn(*args)
        else:   # the launch goes to dev's stream, so dev must be current
            with torch.cuda.device(dev):
                rc = self._fn(*args)
        if rc:
            _lib.check("smat_kattn_decode_step", rc)
        self.i += 1
        return out

    def cache_words(self) -> int:
        return int(self.S.numel() + self.U.numel())

    @staticmethod
    def kv_cache_words(nb: int, T: int, d_v: int) -> int:
        return int(nb * 2 * T * d_v)
