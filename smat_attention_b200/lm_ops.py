"""Autograd wrappers of the fused LM kernels (``include/smat_lm.h``).

Each op takes and returns CUDA bf16 tensors and has no CPU path; the plain
torch forms of the same formulas live in :mod:`smat_attention_b200.lm`
(``fused=False``) and are what the tests compare these against.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

__all__ = ["rms_norm", "add_rms_norm", "rope_split", "swiglu", "linear_cross_entropy"]

_vp, _ci, _cl, _cf = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
_fp = ctypes.c_void_p

SIGNATURES = {
    "smat_lm_rmsnorm_fwd": (_ci, [_vp, _vp, _vp, _vp, _vp, _fp, _cl, _ci, _cf, _vp]),
    "smat_lm_rmsnorm_bwd": (_ci, [_vp, _vp, _fp, _vp, _vp, _vp, _fp, _ci, _cl, _ci, _vp]),
    "smat_lm_rope_split_fwd": (_ci, [_vp, _fp, _fp, _vp, _vp, _vp, _ci, _ci, _ci, _ci, _vp]),
    "smat_lm_rope_split_bwd": (_ci, [_vp, _vp, _vp, _fp, _fp, _vp, _ci, _ci, _ci, _ci, _vp]),
    "smat_lm_swiglu_fwd": (_ci, [_vp, _vp, _cl, _ci, _vp]),
    "smat_lm_swiglu_bwd": (_ci, [_vp, _vp, _vp, _cl, _ci, _vp]),
    "smat_lm_cross_entropy": (_ci, [_vp, _vp, _fp, _cl, _ci, _cf, _vp, _vp]),
}

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


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_bf16(*ts):
    for t in ts:
        if not t.is_cuda or t.dtype != torch.bfloat16:
            raise TypeError("the LM kernels take CUDA bf16 tensors (there is no CPU path)")


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        _check_bf16(x, w)
        d = x.shape[-1]
        x2 = x.contiguous().view(-1, d)
        w = w.contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        _lib.check("smat_lm_rmsnorm_fwd", _L().smat_lm_rmsnorm_fwd(
            x2.data_ptr(), None, w.data_ptr(), None, y.data_ptr(), rstd.data_ptr(),
            x2.shape[0], d, float(eps), _stream(x)))
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        dx, dw = _rms_bwd(x2, w, rstd, dy, None)
        return dx.view(ctx.shape), dw, None


def _rms_bwd(h2, w, rstd, dy, dh):
    d = h2.shape[1]
    dy = dy.contiguous().view(-1, d)
    dh = None if dh is None else dh.contiguous().view(-1, d)
    dx = torch.empty_like(h2)
    n_part = max(1, min(148 * 8, (h2.shape[0] + 7) // 8))   # one full wave of 8-warp CTAs
    part = torch.empty(n_part, d, dtype=torch.float32, device=h2.device)
    _lib.check("smat_lm_rmsnorm_bwd", _L().smat_lm_rmsnorm_bwd(
        h2.data_ptr(), w.data_ptr(), rstd.data_ptr(), dy.data_ptr(),
        None if dh is None else dh.data_ptr(), dx.data_ptr(), part.data_ptr(), n_part,
        h2.shape[0], d, _stream(h2)))
    return dx, part.sum(0).to(w.dtype)


def rms_norm(x, w, eps=1e-5):
    """``x / sqrt(mean(x^2) + eps) * w`` over the last dimension."""
    return _RMSNorm.apply(x, w, eps)


class _AddRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, r, w, eps):
        _check_bf16(x, r, w)
        d = x.shape[-1]
        x2, r2 = x.contiguous().view(-1, d), r.contiguous().view(-1, d)
        w = w.contiguous()
        h = torch.empty_like(x2)
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        _lib.check("smat_lm_rmsnorm_fwd", _L().smat_lm_rmsnorm_fwd(
            x2.data_ptr(), r2.data_ptr(), w.data_ptr(), h.data_ptr(), y.data_ptr(),
            rstd.data_ptr(), x2.shape[0], d, float(eps), _stream(x)))
        ctx.save_for_backward(h, w, rstd)
        ctx.shape = x.shape
        return h.view(x.shape), y.view(x.shape)

    @staticmethod
    def backward(ctx, dh, dy):
        h, w, rstd = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(h)
        dx, dw = _rms_bwd(h, w, rstd, dy, dh)
        dx = dx.view(ctx.shape)
        return dx, dx, dw, None


def add_rms_norm(x, r, w, eps=1e-5):
    """``h = x + r`` and ``rms_norm(h, w)`` in one pass; returns ``(h, y)``."""
    return _AddRMSNorm.apply(x, r, w, eps)


class _RopeSplit(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, cos, sin):
        _check_bf16(qkv)
        B, T, three, H, D = qkv.shape
        assert three == 3
        qkv = qkv.contiguous()
        cos, sin = cos.float().contiguous(), sin.float().contiguous()
        q, k, v = (torch.empty(B, H, T, D, dtype=qkv.dtype, device=qkv.device) for _ in range(3))
        _lib.check("smat_lm_rope_split_fwd", _L().smat_lm_rope_split_fwd(
            qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), q.data_ptr(), k.data_ptr(),
            v.data_ptr(), B, T, H, D, _stream(qkv)))
        ctx.save_for_backward(cos, sin)
        ctx.dims = (B, T, H, D)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        cos, sin = ctx.saved_tensors
        B, T, H, D = ctx.dims
        grads = []
        for g in (dq, dk, dv):
            grads.append(torch.zeros(B, H, T, D, dtype=torch.bfloat16, device=cos.device)
                         if g is None else g.contiguous())
        dqkv = torch.empty(B, T, 3, H, D, dtype=torch.bfloat16, device=cos.device)
        _lib.check("smat_lm_rope_split_bwd", _L().smat_lm_rope_split_bwd(
            grads[0].data_ptr(), grads[1].data_ptr(), grads[2].data_ptr(), cos.data_ptr(),
            sin.data_ptr(), dqkv.data_ptr(), B, T, H, D, _stream(dqkv)))
        return dqkv, None, None


def rope_split(qkv, cos, sin):
    """``qkv [B, T, 3, H, D]`` -> ``q, k, v [B, H, T, D]`` with interleaved RoPE
    on q and k (tables ``[T, D/2]``)."""
    return _RopeSplit.apply(qkv, cos, sin)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a):
        _check_bf16(a)
        h2 = a.shape[-1]
        a2 = a.contiguous().view(-1, h2)
        g = torch.empty(a2.shape[0], h2 // 2, dtype=a.dtype, device=a.device)
        _lib.check("smat_lm_swiglu_fwd", _L().smat_lm_swiglu_fwd(
            a2.data_ptr(), g.data_ptr(), a2.shape[0], h2 // 2, _stream(a)))
        ctx.save_for_backward(a2)
        ctx.shape = a.shape
        return g.view(*a.shape[:-1], h2 // 2)

    @staticmethod
    def backward(ctx, dg):
        (a2,) = ctx.saved_tensors
        dg = dg.contiguous().view(a2.shape[0], -1)
        da = torch.empty_like(a2)
        _lib.check("smat_lm_swiglu_bwd", _L().smat_lm_swiglu_bwd(
            a2.data_ptr(), dg.data_ptr(), da.data_ptr(), a2.shape[0], a2.shape[1] // 2,
            _stream(a2)))
        return da.view(ctx.shape)


def swiglu(a):
    """``a = (a1 | a3)`` on the last dimension -> ``silu(a1) * a3``."""
    return _SwiGLU.apply(a)


class _LinearCrossEntropy(torch.autograd.Function):
    """Mean cross-entropy of ``h W^T`` against ``tgt``.  The logits exist only
    as one bf16 buffer: the kernel turns them into their gradient in place,
    and both gradient GEMMs run in the forward (the loss is the graph's end),
    so the backward only scales them."""

    @staticmethod
    def forward(ctx, h, W, tgt):
        _check_bf16(h, W)
        N, V = h.shape[0], W.shape[0]
        z = h @ W.t()                                   # [N, V] bf16 logits
        loss_rows = torch.empty(N, dtype=torch.float32, device=h.device)
        from .attention import _err_word
        _lib.check("smat_lm_cross_entropy", _L().smat_lm_cross_entropy(
            z.data_ptr(), tgt.contiguous().data_ptr(), loss_rows.data_ptr(), N, V, 1.0 / N,
            _err_word(h.device).data_ptr(), _stream(h)))
        need_h, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dh = z @ W if need_h else None
        dW = z.t() @ h if need_w else None
        del z
        ctx.save_for_backward(*(t for t in (dh, dW) if t is not None))
        ctx.has = (need_h, need_w)
        return loss_rows.mean()

    @staticmethod
    def backward(ctx, g):
        saved = list(ctx.saved_tensors)
        dh = saved.pop(0) * g.to(torch.bfloat16) if ctx.has[0] else None
        dW = saved.pop(0) * g.to(torch.bfloat16) if ctx.has[1] else None
        return dh, dW, None


def linear_cross_entropy(h, W, tgt):
    """``mean_n CE(h[n] W^T, tgt[n])`` with ``h [N, d]``, ``W [V, d]`` (bf16)."""
    return _LinearCrossEntropy.apply(h, W, tgt)
