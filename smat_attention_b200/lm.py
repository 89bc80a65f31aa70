"""Decoder-only language model with the block-sparse softmax arm in every
layer, and its training step.

The model follows the reference's LM template (``tasks/lm.py:45-126``):
token embedding with a tied output head, ``n_layers`` pre-norm blocks
``x + attn(norm(x))``, ``x + mlp(norm2(x))``, a final RMSNorm, init
``N(0, 0.02)``.  RMSNorm is ``tasks/lm.py:45-48`` (fp32 statistics, learned
scale, eps 1e-5); RoPE is the interleaved form of ``tasks/lm.py:57-60``
(pairs ``(x[2i], x[2i+1])`` rotated by ``t / 10000^(2i / D)``).  The MLP is
SwiGLU, ``w2(silu(w1 x) * w3 x)``, and attention runs on the sm_100a kernels
under a block layout (or an ``M^(d)`` mask) instead of SDPA
(``tasks/lm.py:61-65``).

Training keeps bf16 weights and activations for compute and fp32 master
weights in the optimizer (:class:`MasterAdamW`): AdamW with betas (0.9, 0.95),
weight decay on matrices only and gradient clipping at 1.0, as
``tasks/lm.py:172-175, 206-207``.

The elementwise parts (RMSNorm, RoPE with the [B, T, 3, H, D] -> [B, H, T, D]
relayout, SwiGLU, the cross-entropy over the tied head's logits) run as fused
CUDA kernels of ``libsmat_b200.so`` (``csrc/lm_ops.cu``) when ``fused=True``,
else as plain torch expressions of the same formulas (the reference form the
tests compare against).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import smat_softmax_attention
from .mask import MaskSpec, build_block_mask

__all__ = ["LMConfig", "RMSNorm", "Rotary", "SwiGLU", "Block", "LM", "MasterAdamW",
           "allreduce_grads", "train_step", "C4"]


@dataclass
class LMConfig:
    vocab: int = 32000
    d_model: int = 768
    n_layers: int = 12
    n_heads: int = 12
    mlp_hidden: int = 2048
    seq_len: int = 8192
    block: int = 64
    window: int = 8
    stride: int = 16
    n_sink: int = 1
    rope_base: float = 10000.0
    eps: float = 1e-5
    init_std: float = 0.02

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    def mask(self) -> MaskSpec:
        return build_block_mask(self.seq_len, self.block, self.window, self.stride, self.n_sink)

    def n_params(self) -> int:
        d, h = self.d_model, self.mlp_hidden
        per_layer = 4 * d * d + 3 * d * h + 2 * d
        return self.vocab * d + self.n_layers * per_layer + d


# 12 layers, d_model 768, 12 heads x 64, SwiGLU 2048,
# vocab 32000, batch 8 x 8192, block 64, window 8, stride 16, 1 sink
C4 = LMConfig()


def _lm_ops():
    from . import lm_ops
    return lm_ops


class RMSNorm(nn.Module):
    """``x / sqrt(mean(x^2) + eps) * w`` with fp32 statistics (``tasks/lm.py:45-48``)."""

    def __init__(self, d: int, eps: float = 1e-5, fused: bool = True, device=None, dtype=None):
        super().__init__()
        self.w = nn.Parameter(torch.ones(d, device=device, dtype=dtype))
        self.eps = eps
        self.fused = fused

    def forward(self, x):
        if self.fused:
            return _lm_ops().rms_norm(x, self.w, self.eps)
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype) * self.w

    def add(self, x, r):
        """The residual add before a pre-norm: ``h = x + r`` and ``(h, norm(h))``
        (one fused pass when ``fused``)."""
        if self.fused:
            return _lm_ops().add_rms_norm(x, r, self.w, self.eps)
        h = x + r
        return h, self.forward(h)


class Rotary(nn.Module):
    """Interleaved RoPE tables (``tasks/lm.py:55-60``): angle ``t * inv[i]`` for
    the pair ``(2 i, 2 i + 1)``."""

    def __init__(self, head_dim: int, base: float = 10000.0):
        super().__init__()
        inv = 1.0 / (base ** (torch.arange(0, head_dim, 2).float() / head_dim))
        self.register_buffer("inv", inv, persistent=False)
        self._cache = {}

    def tables(self, T: int, device):
        key = (T, str(device))
        if key not in self._cache:
            t = torch.arange(T, device=device).float()
            f = torch.outer(t, self.inv.to(device))
            self._cache[key] = (f.cos().contiguous(), f.sin().contiguous())
        return self._cache[key]

    @staticmethod
    def rotate(x, cos, sin):
        """Plain form: ``x [..., T, D]`` rotated pairwise (the reference's expression)."""
        x1, x2 = x[..., ::2].float(), x[..., 1::2].float()
        return torch.stack([x1 * cos - x2 * sin, x1 * sin + x2 * cos], -1).flatten(-2).to(x.dtype)


class Attention(nn.Module):
    """qkv projection, RoPE on q and k, softmax attention under ``spec`` on the
    sm_100a kernels, output projection."""

    def __init__(self, cfg: LMConfig, spec: MaskSpec, rotary: Rotary, fused: bool = True,
                 device=None, dtype=None):
        super().__init__()
        self.h, self.dh = cfg.n_heads, cfg.head_dim
        self.spec, self.rotary, self.fused = spec, rotary, fused
        self.qkv = nn.Linear(cfg.d_model, 3 * cfg.d_model, bias=False, device=device, dtype=dtype)
        self.out = nn.Linear(cfg.d_model, cfg.d_model, bias=False, device=device, dtype=dtype)

    def forward(self, x):
        b, T, C = x.shape
        cos, sin = self.rotary.tables(T, x.device)
        qkv = self.qkv(x)
        if self.fused:
            q, k, v = _lm_ops().rope_split(qkv.view(b, T, 3, self.h, self.dh), cos, sin)
        else:
            q, k, v = qkv.view(b, T, 3, self.h, self.dh).permute(2, 0, 3, 1, 4)
            q, k = Rotary.rotate(q, cos, sin), Rotary.rotate(k, cos, sin)
        o, _ = smat_softmax_attention(q, k, v, self.spec, tokens_major=True)
        return self.out(o.transpose(1, 2).reshape(b, T, C))


class SwiGLU(nn.Module):
    """``w2(silu(w1 x) * w3 x)``."""

    def __init__(self, d: int, hidden: int, fused: bool = True, device=None, dtype=None):
        super().__init__()
        self.w13 = nn.Linear(d, 2 * hidden, bias=False, device=device, dtype=dtype)
        self.w2 = nn.Linear(hidden, d, bias=False, device=device, dtype=dtype)
        self.fused = fused

    def forward(self, x):
        a = self.w13(x)
        if self.fused:
            g = _lm_ops().swiglu(a)
        else:
            a1, a3 = a.chunk(2, dim=-1)
            g = F.silu(a1.float()).to(a.dtype) * a3
        return self.w2(g)


class Block(nn.Module):
    def __init__(self, cfg: LMConfig, spec: MaskSpec, rotary: Rotary, fused: bool = True,
                 device=None, dtype=None):
        super().__init__()
        self.norm = RMSNorm(cfg.d_model, cfg.eps, fused, device, dtype)
        self.attn = Attention(cfg, spec, rotary, fused, device, dtype)
        self.norm2 = RMSNorm(cfg.d_model, cfg.eps, fused, device, dtype)
        self.mlp = SwiGLU(cfg.d_model, cfg.mlp_hidden, fused, device, dtype)

    def forward(self, x, pending=None):
        """``x + attn(norm(x))``, then ``+ mlp(norm2(.))``; the MLP output is
        returned unadded (``pending``) so that the next norm adds it in its own
        pass.  Returns ``(residual stream, pending)``."""
        if pending is None:
            y = self.norm(x)
        else:
            x, y = self.norm.add(x, pending)
        x, y = self.norm2.add(x, self.attn(y))
        return x, self.mlp(y)


class LM(nn.Module):
    """Token embedding (tied head) -> blocks -> RMSNorm -> logits
    (``tasks/lm.py:115-126``)."""

    def __init__(self, cfg: LMConfig, spec: Optional[MaskSpec] = None, fused: bool = True,
                 device=None, dtype=torch.bfloat16, seed: int = 0):
        super().__init__()
        self.cfg, self.fused = cfg, fused
        self.spec = spec if spec is not None else cfg.mask()
        self.rotary = Rotary(cfg.head_dim, cfg.rope_base)
        self.emb = nn.Embedding(cfg.vocab, cfg.d_model, device=device, dtype=dtype)
        self.blocks = nn.ModuleList([Block(cfg, self.spec, self.rotary, fused, device, dtype)
                                     for _ in range(cfg.n_layers)])
        self.norm = RMSNorm(cfg.d_model, cfg.eps, fused, device, dtype)
        g = torch.Generator(device="cpu").manual_seed(seed)
        with torch.no_grad():
            for m in self.modules():
                if isinstance(m, (nn.Linear, nn.Embedding)):
                    m.weight.copy_(torch.randn(m.weight.shape, generator=g) * cfg.init_std)

    def hidden(self, idx):
        x, pending = self.emb(idx), None
        for b in self.blocks:
            x, pending = b(x, pending)
        return self.norm(x) if pending is None else self.norm.add(x, pending)[1]

    def forward(self, idx):
        return F.linear(self.hidden(idx), self.emb.weight)

    def loss(self, idx, tgt):
        """Mean next-token cross-entropy; the fused path never materialises
        fp32 logits."""
        h = self.hidden(idx)
        if self.fused:
            return _lm_ops().linear_cross_entropy(h.reshape(-1, h.shape[-1]), self.emb.weight,
                                                  tgt.reshape(-1))
        logits = F.linear(h, self.emb.weight)
        return F.cross_entropy(logits.float().view(-1, logits.shape[-1]), tgt.reshape(-1))


class MasterAdamW:
    """AdamW over fp32 master copies of a bf16 model's parameters.

    Each step casts the bf16 gradients into fp32 master gradients, clips their
    global norm, runs AdamW (torch's fused multi-tensor kernel) on the masters
    and writes the masters back into the bf16 parameters.  Matrices and
    embeddings get weight decay, vectors (norm scales) do not
    (``tasks/lm.py:172-175``)."""

    def __init__(self, params, lr: float = 6e-4, betas=(0.9, 0.95), eps: float = 1e-8,
                 weight_decay: float = 0.1, clip: Optional[float] = 1.0):
        self.params: List[torch.Tensor] = [p for p in params if p.requires_grad]
        self.master = [p.detach().float().clone() for p in self.params]
        for m in self.master:
            m.grad = torch.zeros_like(m)
        decay = [m for m, p in zip(self.master, self.params) if p.ndim >= 2]
        no_decay = [m for m, p in zip(self.master, self.params) if p.ndim < 2]
        fused = all(m.is_cuda for m in self.master)
        self.opt = torch.optim.AdamW([{"params": decay, "weight_decay": weight_decay},
                                      {"params": no_decay, "weight_decay": 0.0}],
                                     lr=lr, betas=betas, eps=eps, fused=fused)
        self.clip = clip

    def step(self) -> torch.Tensor:
        """One optimizer step; returns the pre-clip gradient norm (a device tensor)."""
        grads = [p.grad if p.grad is not None else torch.zeros_like(p) for p in self.params]
        torch._foreach_copy_([m.grad for m in self.master], grads)
        if self.clip is not None:
            norm = torch.nn.utils.clip_grad_norm_(self.master, self.clip, foreach=True)
        else:
            norm = torch.linalg.vector_norm(torch.stack(
                [torch.linalg.vector_norm(m.grad) for m in self.master]))
        self.opt.step()
        with torch.no_grad():
            torch._foreach_copy_(self.params, self.master)
        for p in self.params:
            p.grad = None
        return norm


def allreduce_grads(model: nn.Module, dist, group=None) -> None:
    """Average the bf16 gradients over the ranks of a data-parallel group:
    one NCCL all-reduce over a flat buffer (the only exchange of the step)."""
    grads = [p.grad for p in model.parameters() if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, group=group)
    flat.div_(dist.get_world_size(group))
    parts = flat.split([g.numel() for g in grads])
    torch._foreach_copy_(grads, [c.view_as(g) for c, g in zip(parts, grads)])


def train_step(model: LM, opt: MasterAdamW, tokens: torch.Tensor,
               before_step=None) -> torch.Tensor:
    """Forward, backward and optimizer step on ``tokens`` ``[B, T + 1]``
    (inputs ``tokens[:, :-1]``, targets ``tokens[:, 1:]``); returns the loss
    as a device tensor (no host synchronisation).  ``before_step`` runs
    between the backward and the optimizer (the data-parallel all-reduce)."""
    inp, tgt = tokens[:, :-1], tokens[:, 1:]
    loss = model.loss(inp, tgt)
    loss.backward()
    if before_step is not None:
        before_step()
    opt.step()
    return loss.detach()
