"""Autoregressive decoding with a KV cache under a block layout or an ``M^(d)``
mask: the softmax counterpart of the reference's streaming decoder
``SmatDecoder`` (``src/smat/attention.py:496-535``).

The reference decodes its kernelised arm in ``O(r p)`` per token from pooled
state; softmax attention has no such summary, so each step reads the keys and
values the new query sees -- its CSR row of the layout, at most ``max_row``
blocks -- from a cache of the whole sequence.  :func:`decode_attention` is
the op (``smat_decode`` of the C ABI: one launch, each row's splits one
thread-block cluster that combines them); :class:`SmatSoftmaxDecoder` keeps
the cache and the positions and mirrors ``SmatDecoder``'s ``step`` /
``cache_words`` / ``kv_cache_words``.
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _lib
from .attention import _err_word, kernel_layout, layout_device_args
from .mask import MaskSpec

__all__ = ["decode_attention", "SmatSoftmaxDecoder"]

_WS = {}


def _workspace(device, floats: int) -> torch.Tensor:
    key = str(device)
    t = _WS.get(key)
    if t is None or t.numel() < floats:
        t = torch.empty(floats, dtype=torch.float32, device=device)
        _WS[key] = t
    return t


def decode_attention(q, k_cache, v_cache, pos, spec: MaskSpec, scale: Optional[float] = None,
                     o: Optional[torch.Tensor] = None):
    """``(o, lse)`` of one query per (batch, head) at positions ``pos``.

    ``q``: ``[B, H, D]`` bf16; ``k_cache, v_cache``: ``[B, H, T, D]`` bf16 (rows
    ``<= pos[b]`` filled); ``pos``: int32 CUDA tensor ``[B]``; ``spec``: the
    layout (or ``M^(d)`` spec) the sequence is masked by, with ``spec.T == T``.
    """
    if not (q.is_cuda and k_cache.is_cuda and v_cache.is_cuda and pos.is_cuda):
        raise ValueError("decode_attention takes CUDA tensors (there is no CPU path)")
    if q.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or \
            v_cache.dtype != torch.bfloat16:
        raise TypeError("decode_attention runs bf16 caches")
    B, H, T, D = k_cache.shape
    if q.shape != (B, H, D) or v_cache.shape != k_cache.shape:
        raise ValueError("q must be [B, H, D] and the caches [B, H, T, D]")
    if pos.dtype != torch.int32 or pos.shape != (B,):
        raise ValueError("pos must be an int32 tensor of shape [B]")
    lay = kernel_layout(spec)
    if lay.T != T:
        raise ValueError(f"layout was built for T={lay.T}, the cache holds T={T}")
    args = layout_device_args(lay, q.device)
    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    if q.stride(-1) != 1 or q.stride(0) % 8 or q.stride(1) % 8 or q.data_ptr() % 16:
        q = q.contiguous()
    if o is None:
        o = torch.empty(B, H, D, dtype=torch.bfloat16, device=q.device)
    lse = torch.empty(B, H, dtype=torch.float32, device=q.device)
    L = _lib.lib()
    floats = ctypes.c_int64(0)
    _lib.check("smat_decode_workspace",
               L.smat_decode_workspace(B, H, D, args["max_row"], ctypes.byref(floats)))
    ws = _workspace(q.device, floats.value)
    s2 = lambda t: (ctypes.c_int64 * 3)(t.stride(0), t.stride(1), 0)
    _lib.check("smat_decode", L.smat_decode(
        _lib.DTYPE_BF16, q.data_ptr(), s2(q), k_cache.data_ptr(), _lib.strides3(k_cache),
        v_cache.data_ptr(), _lib.strides3(v_cache), o.data_ptr(), s2(o), lse.data_ptr(),
        pos.data_ptr(), B, H, T, D, args["indptr"].data_ptr(), args["indices"].data_ptr(),
        args["kind"].data_ptr(), args["nblocks"], args["nnzb"], args["block"], args["max_row"],
        args["pattern"], scale, ws.data_ptr(), ws.numel(), _err_word(q.device).data_ptr(),
        torch.cuda.current_stream(q.device).cuda_stream))
    return o, lse


class SmatSoftmaxDecoder:
    """Token-by-token softmax attention over a preallocated KV cache.

    ``prefill(k, v)`` stores the first ``t0`` keys and values; each
    ``step(q_t, k_t, v_t)`` appends one key / value per (batch, head) at the
    current position and returns the attention output of ``q_t`` there
    (``[B, H, D]``), under the same mask the full-sequence op applies.
    """

    def __init__(self, spec: MaskSpec, B: int, H: int, D: int, *, device,
                 scale: Optional[float] = None):
        self.spec = spec
        T = spec.T
        self.k = torch.zeros(B, H, T, D, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros_like(self.k)
        self.B, self.H, self.D, self.T = B, H, D, T
        self.scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
        self.t = 0
        self.pos = torch.zeros(B, dtype=torch.int32, device=device)

    def prefill(self, k, v):
        t0 = k.shape[2]
        if t0 > self.T:
            raise ValueError("prefix longer than the layout")
        self.k[:, :, :t0] = k
        self.v[:, :, :t0] = v
        self.t = t0

    def step(self, q_t, k_t, v_t):
        if self.t >= self.T:
            raise ValueError(f"the cache holds {self.T} positions")
        self.k[:, :, self.t] = k_t
        self.v[:, :, self.t] = v_t
        self.pos.fill_(self.t)
        o, _ = decode_attention(q_t, self.k, self.v, self.pos, self.spec, self.scale)
        self.t += 1
        return o

    def cache_words(self) -> int:
        return int(self.k.numel() + self.v.numel())

    @staticmethod
    def kv_cache_words(nb: int, T: int, d_v: int) -> int:
        return int(nb * 2 * T * d_v)
