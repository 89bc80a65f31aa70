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

import ctypes

import numpy as np
import torch

from . import _lib
from .mask import MaskSpec

__all__ = ["chunk_local", "pool", "incidence", "segmented_causal_scan", "pool_profiles",
           "apply_incidence", "query_by_type", "walsh_incidence", "zeta_transform",
           "smat_attention", "SmatDecoder", "normalise"]

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
    @staticmethod
    def forward(ctx, F, ptr, idx, n_out):
        ctx.save_for_backward(ptr, idx)
        ctx.n_in = F.shape[1]
        ctx.dtype = F.dtype
        return _gather_sum(F, ptr, idx, n_out)

    @staticmethod
    def backward(ctx, dU):
        ptr, idx = ctx.saved_tensors
        t_ptr, t_idx = _transpose_csr(ptr, idx, ctx.n_in)
        return _gather_sum(dU, t_ptr, t_idx, ctx.n_in).to(ctx.dtype), None, None, None


def incidence(F, plane_pts, B: int):
    """``U_h = sum_{x in H_h} F_x`` with ``plane_pts (B, deg)`` the points of
    each hyperplane: ``(nb, N0, r, p) -> (nb, B, r, p)``."""
    ptr, idx = _csr_of_table(plane_pts)
    return _Incidence.apply(F, ptr, idx, int(B))


def _incidence_csr(F, spec: MaskSpec):
    key = ("kattn_csr", str(F.device))
    if key not in spec.dev:
        spec.dev[key] = (torch.from_numpy(np.ascontiguousarray(spec.C_indptr, np.int64)).to(F.device),
                         torch.from_numpy(np.ascontiguousarray(spec.C_indices, np.int32)).to(F.device))
    ptr, idx = spec.dev[key]
    return _Incidence.apply(F, ptr, idx, int(spec.B))


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
def segmented_causal_scan(Phi, Psi, Vb, n: int, chunk: int = CHUNK):
    """``[[L_n, 0], [0, L_{T_R}]] Phi Psi^T Vb`` by chunks with one reset at ``n``
    (reference ``attention.py:134-192``): chunk summaries ``Psi_c^T Vb_c``, an
    exclusive prefix sum inside each segment, then :func:`chunk_local`."""
    if chunk != CHUNK:
        raise ValueError(f"the chunk-local kernel runs chunks of {CHUNK} rows")
    nb, T, r = Phi.shape
    p = Vb.shape[-1]
    C = CHUNK
    if n % C:
        raise ValueError(f"segment boundary n={n} is not a multiple of chunk={C}")
    pad = (-T) % C
    Phi, Psi, Vb = (x.float() for x in (Phi, Psi, Vb))
    if pad:
        Phi, Psi, Vb = (torch.nn.functional.pad(x, (0, 0, 0, pad)) for x in (Phi, Psi, Vb))
    nc = (T + pad) // C
    nc0 = n // C
    Phi_c, Psi_c = Phi.reshape(nb, nc, C, r), Psi.reshape(nb, nc, C, r)
    Vb_c = Vb.reshape(nb, nc, C, p)
    D = Psi_c.transpose(-1, -2) @ Vb_c                                  # (nb, nc, r, p)
    # exclusive prefix sums inside each segment: inclusive cumsum minus D
    if 0 < nc0 < nc:
        Sin = torch.cat([torch.cumsum(D[:, :nc0], dim=1), torch.cumsum(D[:, nc0:], dim=1)],
                        dim=1) - D
    else:
        Sin = torch.cumsum(D, dim=1) - D
    out = chunk_local(Phi_c, Psi_c, Vb_c, Sin)
    return out.reshape(nb, T + pad, p)[:, :T]


def pool_profiles(Psi, Vb, spec: MaskSpec):
    """``F`` over the landmark columns ``[n_P, n)`` (reference ``attention.py:199-236``)."""
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


def apply_incidence(F, spec: MaskSpec):
    """``U_h = sum_{x in H_h} F_x`` (reference ``attention.py:239-285``): the CSR
    gather-sum kernel, or the Walsh butterfly for the endpoint family."""
    if spec.kind == "endpoint":
        return walsh_incidence(F)
    return _incidence_csr(F, spec)


def query_by_type(Phi_rec, U, spec: MaskSpec):
    """``Ybar_i = Phi_i U_{(i - n) mod B}`` for the recent rows (reference
    ``attention.py:310-330``): one batched GEMM over the stride-B slices."""
    nb, T_R, r = Phi_rec.shape
    B, p = spec.B, U.shape[-1]
    U = U.float()
    c, rem = divmod(T_R, B)
    pieces = []
    if c:
        head = Phi_rec[:, :c * B].float().reshape(nb, c, B, r).transpose(1, 2)   # (nb,B,c,r)
        pieces.append((head @ U).transpose(1, 2).reshape(nb, c * B, p))
    if rem:
        tail = Phi_rec[:, c * B:].float().unsqueeze(-2)
        pieces.append((tail @ U[:, :rem]).squeeze(-2))
    return torch.cat(pieces, dim=1)


def _add_query_by_type(H_rec, Phi_rec, U, spec: MaskSpec):
    """``H_rec += query_by_type(Phi_rec, U, spec)`` in place, with no
    intermediate copy of the ``(nb, T_R, p)`` result."""
    nb, T_R, r = Phi_rec.shape
    B, p = spec.B, U.shape[-1]
    U = U.float()
    c, rem = divmod(T_R, B)
    if c:
        head = Phi_rec[:, :c * B].float().reshape(nb, c, B, r).transpose(1, 2)   # (nb,B,c,r)
        H_rec[:, :c * B].view(nb, c, B, p).add_((head @ U).transpose(1, 2))
    if rem:
        tail = Phi_rec[:, c * B:].float().unsqueeze(-2)
        H_rec[:, c * B:].add_((tail @ U[:, :rem]).squeeze(-2))


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


def smat_attention(Phi, Psi, Vb, spec: MaskSpec, *, chunk: int = CHUNK, g=None):
    """The pooled schedule of the reference's ``smat_attention``
    (``attention.py:391-455``) on these kernels; returns ``(nb, T, p - 1)``
    fp32 (the last column of ``Vb`` is the normaliser's)."""
    if spec.kind not in ("geometric", "endpoint"):
        raise ValueError("smat_attention needs an M^(d) spec from build_mask")
    n = spec.n
    F = pool_profiles(Psi, Vb, spec)
    U = apply_incidence(F, spec)
    if spec.n_P:
        b = Psi[:, :spec.n_P].float().transpose(-1, -2) @ Vb[:, :spec.n_P].float()
        U = U + b.unsqueeze(1)
    if spec.kind == "endpoint":
        Y_lr = query_by_type(Phi[:, n:], U, spec)
        Fz = Psi[:, :n].float().unsqueeze(-1) * Vb[:, :n].float().unsqueeze(-2)
        top = (Phi[:, :n].float().unsqueeze(-2) @ zeta_transform(Fz)).squeeze(-2)
        loc = segmented_causal_scan(Phi[:, n:], Psi[:, n:], Vb[:, n:], 0, chunk)
        H = torch.cat([top, loc + Y_lr], dim=1)
    else:
        H = segmented_causal_scan(Phi, Psi, Vb, n, chunk)
        _add_query_by_type(H[:, n:], Phi[:, n:], U, spec)
    out = normalise(H)
    if g is not None:
        out = out * g.unsqueeze(-1).to(out.dtype)
    return out


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
