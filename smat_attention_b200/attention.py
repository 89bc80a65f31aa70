"""Block-sparse causal softmax attention under an SMat block layout or an
``M^(d)`` mask.

``smat_softmax_attention(q, k, v, spec, scale=None) -> (o, lse)`` is the op.
It runs the sm_100a kernels of ``libsmat_b200.so`` through the C ABI and is
differentiable through :class:`SmatSoftmaxFn`:

* forward: ``o = softmax(scale q k^T + mask) v`` and the fp32 natural-log
  normaliser ``lse`` (non-differentiable output);
* backward: the ``delta = rowsum(dO * o)`` preprocess, then dK/dV over the
  layout's transposed CSR and dQ over its forward CSR (bitwise
  reproducible).  Optionally, for bf16 at D = 128, the dK/dV kernel also
  accumulates dQ (fp32 reductions into a workspace, then one conversion
  pass), which skips the second pass's recomputation of S and dP; that dQ
  can differ in its last bits between runs.  ``FUSED_DQ = True`` (or the
  environment variable ``SMAT_FUSED_DQ=1``) selects it; on B200 at config 3
  it is not faster than the two passes.

Tensors are ``[B, H, T, D]`` on a CUDA device, bf16 (tensor-core kernels,
D in {64, 128}, block in {64, 128}) or fp32 (full-fp32 CUDA-core kernels,
D in {32, 64, 128}).  There is no CPU path: a CPU tensor, an unsupported
shape or a missing library raises.

The mask is a ``kind="block"`` layout, or one of the reference's own ``M^(d)``
masks (``build_mask``, reference ``src/smat/mask.py:244-425``), which runs as
its pattern layout: the same kernels with PATTERN tiles whose mask they
evaluate from bit tables of the incidence (``smat_fwd_pattern`` /
``smat_bwd_pattern``), equal element for element to ``materialise``.

This is the softmax counterpart of the reference's op entry
``smat.attention.smat_attention`` (``src/smat/attention.py:391-455``), which
computes kernelised attention; its fused-kernel plugin table
(``attention.py:37-40``, ``kernels/triton_bwd.py:331-346``) has no analogue
here because there is exactly one implementation per dtype.
"""

from __future__ import annotations

import ctypes
import math
import os
from typing import Dict, Tuple

import numpy as np
import torch

from . import _lib
from .mask import MaskSpec, pattern_layout, to_device

__all__ = ["smat_softmax_attention", "SmatSoftmaxFn", "layout_device_args",
           "kernel_layout", "check_device_errors", "fwd", "bwd"]

_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}

# False: the backward's dQ comes from its own pass over the forward CSR
# (bitwise reproducible); True: bf16 at D = 128 accumulates dQ inside the
# dK/dV kernel (fewer MMAs, last bits vary between runs)
FUSED_DQ = os.environ.get("SMAT_FUSED_DQ", "0") == "1"


def fused_dq_applies(dtype, D: int) -> bool:
    """Whether :func:`bwd` accumulates dQ inside the dK/dV kernel."""
    return dtype == torch.bfloat16 and D == 128
_ERR: Dict[str, torch.Tensor] = {}


def _err_word(device) -> torch.Tensor:
    key = str(device)
    t = _ERR.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _ERR[key] = t
    return t


def check_device_errors(device=None, reset: bool = True) -> int:
    """Synchronise and return the device error bits the kernels recorded on
    ``device`` (0 = none; bit 1 wait timeout, 2 malformed CSR, 4 schedule
    overflow)."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    t = _err_word(device)
    val = int(t.item())
    if reset and val:
        t.zero_()
    return val


def kernel_layout(spec: MaskSpec) -> MaskSpec:
    """The tiled layout the kernels run: ``spec`` itself for a block or
    pattern layout, :func:`~smat_attention_b200.mask.pattern_layout` (128-row
    tiles) for an ``M^(d)`` spec from ``build_mask``."""
    if spec.kind in ("block", "pattern"):
        return spec
    if spec.kind in ("geometric", "endpoint"):
        return pattern_layout(spec, 128)
    raise ValueError(f"unsupported mask kind {spec.kind!r}")


def _validate(spec: MaskSpec) -> Tuple[int, int]:
    """Check both CSRs once on the host (C validator); cache the longest rows."""
    cached = getattr(spec, "_validated", None)
    if cached is not None:
        return cached
    if spec.kind not in ("block", "pattern"):
        raise ValueError(f"the softmax kernels need a block or pattern layout, "
                         f"got kind={spec.kind!r}")
    L = _lib.lib()
    validate = (L.smat_layout_validate_pattern if spec.kind == "pattern"
                else L.smat_layout_validate)
    rows = []
    for ptr, idx, knd, tr in ((spec.indptr, spec.indices, spec.tile_kind, 0),
                              (spec.t_indptr, spec.t_indices, spec.t_kind, 1)):
        ptr = np.ascontiguousarray(ptr, dtype=np.int32)
        idx = np.ascontiguousarray(idx, dtype=np.int32)
        knd = np.ascontiguousarray(knd, dtype=np.uint8)
        mr = ctypes.c_int32(0)
        _lib.check("smat_layout_validate", validate(
            spec.nqb, idx.size, ptr.ctypes.data, idx.ctypes.data, knd.ctypes.data, tr,
            ctypes.byref(mr)))
        rows.append(int(mr.value))
    spec._validated = (rows[0], rows[1])
    return spec._validated


def layout_device_args(spec: MaskSpec, device) -> Dict[str, object]:
    """Device CSR tensors of ``spec`` (staged once per device) plus sizes; for
    a pattern layout also ``pattern``, the ``smat_pattern_t`` pointing at the
    staged bit tables."""
    spec = kernel_layout(spec)
    max_row, t_max_row = _validate(spec)
    to_device(spec, device)
    d = spec.dev[str(torch.device(device))]
    out = dict(d, nblocks=spec.nqb, nnzb=spec.nnzb, block=spec.block,
               max_row=max_row, t_max_row=t_max_row, pattern=None)
    if spec.kind == "pattern":
        pt = d.get("pattern")
        if pt is None:
            pt = _lib.Pattern(
                _lib.FAMILY_ENDPOINT if spec.source == "endpoint" else _lib.FAMILY_GEOMETRIC,
                spec.n, spec.n_P, spec.B, spec.N0, spec.row_bits.shape[1],
                spec.col_bits.shape[1], d["row_bits"].data_ptr(), d["col_bits"].data_ptr())
            d["pattern"] = pt
        out["pattern"] = ctypes.byref(pt)
    return out


def _prep(x: torch.Tensor, name: str) -> torch.Tensor:
    if not x.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path)")
    if x.dim() != 4:
        raise ValueError(f"{name} must be [B, H, T, D], got shape {tuple(x.shape)}")
    if x.dtype not in _DTYPES:
        raise TypeError(f"{name} must be bf16 or fp32, got {x.dtype}")
    if x.stride(-1) != 1 or any(s % 8 for s in x.stride()[:3]) or x.data_ptr() % 16:
        x = x.contiguous()
    return x


def fwd(q, k, v, spec: MaskSpec, scale: float, o=None):
    """Launch the forward kernel; returns ``(o, lse)``.  ``o`` may be given
    as any ``[B, H, T, D]``-shaped view (strides are passed through)."""
    q, k, v = _prep(q, "q"), _prep(k, "k"), _prep(v, "v")
    B, H, T, D = q.shape
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k and v must have the same shape")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k and v must have the same dtype")
    if spec.T != T:
        raise ValueError(f"layout was built for T={spec.T}, inputs have T={T}")
    lay = layout_device_args(spec, q.device)
    if o is None:
        o = torch.empty_like(q)
    lse = torch.empty(B, H, T, dtype=torch.float32, device=q.device)
    L = _lib.lib()
    args = [_DTYPES[q.dtype],
            q.data_ptr(), _lib.strides3(q), k.data_ptr(), _lib.strides3(k),
            v.data_ptr(), _lib.strides3(v), o.data_ptr(), _lib.strides3(o),
            lse.data_ptr(), B, H, T, D,
            lay["indptr"].data_ptr(), lay["indices"].data_ptr(), lay["kind"].data_ptr(),
            lay["nblocks"], lay["nnzb"], lay["block"], lay["max_row"]]
    tail = [float(scale), _err_word(q.device).data_ptr(),
            torch.cuda.current_stream(q.device).cuda_stream]
    if lay["pattern"] is None:
        _lib.check("smat_fwd", L.smat_fwd(*args, *tail))
    else:
        _lib.check("smat_fwd_pattern", L.smat_fwd_pattern(*args, lay["pattern"], *tail))
    return o, lse


def bwd(q, k, v, o, lse, do, spec: MaskSpec, scale: float, fused_dq=None):
    """Launch preprocess + dK/dV + dQ; returns ``(dq, dk, dv)``.

    ``fused_dq`` (default: the module's ``FUSED_DQ``) accumulates dQ inside
    the dK/dV kernel where that applies (bf16, D = 128).
    """
    q, k, v, o, do = (_prep(x, n) for x, n in ((q, "q"), (k, "k"), (v, "v"), (o, "o"), (do, "do")))
    if do.dtype != q.dtype:
        do = do.to(q.dtype)
    B, H, T, D = q.shape
    lay = layout_device_args(spec, q.device)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    delta = torch.empty(B, H, T, dtype=torch.float32, device=q.device)
    L = _lib.lib()
    args = [_DTYPES[q.dtype],
            q.data_ptr(), _lib.strides3(q), k.data_ptr(), _lib.strides3(k),
            v.data_ptr(), _lib.strides3(v), o.data_ptr(), _lib.strides3(o),
            do.data_ptr(), _lib.strides3(do), lse.data_ptr(), delta.data_ptr(),
            dq.data_ptr(), _lib.strides3(dq), dk.data_ptr(), _lib.strides3(dk),
            dv.data_ptr(), _lib.strides3(dv), B, H, T, D,
            lay["indptr"].data_ptr(), lay["indices"].data_ptr(), lay["kind"].data_ptr(),
            lay["t_indptr"].data_ptr(), lay["t_indices"].data_ptr(),
            lay["t_kind"].data_ptr(), lay["nblocks"], lay["nnzb"], lay["block"],
            lay["max_row"], lay["t_max_row"]]
    tail = [float(scale), _err_word(q.device).data_ptr(),
            torch.cuda.current_stream(q.device).cuda_stream]
    if fused_dq is None:
        fused_dq = FUSED_DQ
    if fused_dq and fused_dq_applies(q.dtype, D):
        acc = torch.empty(B * H * T * D, dtype=torch.float32, device=q.device)
        _lib.check("smat_bwd_acc", L.smat_bwd_acc(*args, lay["pattern"], acc.data_ptr(),
                                                  acc.numel(), *tail))
    elif lay["pattern"] is None:
        _lib.check("smat_bwd", L.smat_bwd(*args, *tail))
    else:
        _lib.check("smat_bwd_pattern", L.smat_bwd_pattern(*args, lay["pattern"], *tail))
    return dq, dk, dv


class SmatSoftmaxFn(torch.autograd.Function):
    """Differentiable block-sparse softmax attention (``o`` differentiable,
    ``lse`` not)."""

    @staticmethod
    def forward(ctx, q, k, v, spec, scale, tokens_major=False):
        o = None
        if tokens_major:
            # O in [B, T, H, D] memory, handed out as its [B, H, T, D] view
            B, H, T, D = q.shape
            o = torch.empty(B, T, H, D, dtype=q.dtype, device=q.device).transpose(1, 2)
        o, lse = fwd(q, k, v, spec, scale, o=o)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.spec, ctx.scale = spec, scale
        ctx.mark_non_differentiable(lse)
        return o, lse

    @staticmethod
    def backward(ctx, do, _dlse):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = bwd(q, k, v, o, lse, do, ctx.spec, ctx.scale)
        return dq, dk, dv, None, None, None


def smat_softmax_attention(q, k, v, spec: MaskSpec, scale=None, tokens_major=False):
    """``(o, lse)`` of block-sparse causal softmax attention under ``spec``.

    ``q, k, v``: ``[B, H, T, D]`` CUDA tensors, bf16 or fp32, same shape.
    ``spec``: a ``kind="block"`` layout from
    :func:`smat_attention_b200.mask.build_block_mask`, or an ``M^(d)`` spec
    from :func:`smat_attention_b200.mask.build_mask` (run through its pattern
    layout, :func:`smat_attention_b200.mask.pattern_layout`), with
    ``spec.T == T``.  ``scale`` defaults to ``1 / sqrt(D)``.
    ``tokens_major=True`` stores ``o`` in ``[B, T, H, D]`` memory (returned as
    its ``[B, H, T, D]`` view), so ``o.transpose(1, 2).reshape(B, T, H * D)``
    is free for the output projection.
    """
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    return SmatSoftmaxFn.apply(q, k, v, spec, float(scale), bool(tokens_major))
