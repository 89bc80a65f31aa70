"""The attention module of the reference's model layer, with the block-sparse
softmax arm.

``Attention(d_model, n_heads, arm, spec=...)`` keeps the constructor and
forward signature of the reference's ``smat.model.Attention``
(``src/smat/model.py:112-343``): a bias-free ``qkv`` projection, optional
QK-norm, the attention op, and a bias-free ``out`` projection.  Arms:

``"softmax"``       dense causal softmax through torch SDPA, exactly the
                    reference's baseline arm (``model.py:217-220``);
``"smat_softmax"``  causal softmax under ``spec`` on the sm_100a kernels:
                    a ``kind="block"`` layout, or an ``M^(d)`` mask from
                    ``build_mask`` (run through its pattern layout).

The reference's kernelised ``"smat"`` arm and its variants (decay, gates,
content hashing, Mamba mixers) are not part of this package.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import smat_softmax_attention
from .mask import MaskSpec

__all__ = ["Attention", "ARMS"]

ARMS = ("softmax", "smat_softmax")

# options of the reference's kernelised arm; accepted at their defaults so a
# constructor call written for the reference still works for the softmax arms
_KERNEL_ARM_DEFAULTS = dict(r=64, learn_phi=False, chunk=128, triton_bwd=False, no_lr=False,
                            gate=False, phi_kind="elu1", taylor_dim=16, decay=False,
                            dir_head="linear", dir_soft=False, dir_window=4,
                            dt_init=(1e-3, 1e-1), A_init=(1.0, 16.0), type_offsets=None,
                            scan_kernel="phi", assign="positional", read_mode="point",
                            pos_read="plane", hash_src="hidden", hash_freeze=False,
                            hash_shift=0, vocab=None, hash_conv=0)


class Attention(nn.Module):
    def __init__(self, d_model: int, n_heads: int, arm: str, *, spec: MaskSpec = None,
                 device=None, seed: int = 0, qk_norm: bool = False, **kernel_arm_options):
        super().__init__()
        if arm not in ARMS:
            raise ValueError(f"arm {arm!r} is not provided here; choose one of {ARMS} "
                             f"(the kernelised 'smat' arm belongs to the reference)")
        for name, val in kernel_arm_options.items():
            if name not in _KERNEL_ARM_DEFAULTS:
                raise TypeError(f"unexpected option {name!r}")
            if val != _KERNEL_ARM_DEFAULTS[name]:
                raise ValueError(f"option {name}={val!r} belongs to the kernelised arm")
        if d_model % n_heads:
            raise ValueError("d_model must be a multiple of n_heads")
        if arm == "smat_softmax":
            if spec is None or spec.kind not in ("block", "pattern", "geometric", "endpoint"):
                raise ValueError("arm 'smat_softmax' needs spec=build_block_mask(...) or "
                                 "spec=build_mask(...)")
        self.h, self.dh = n_heads, d_model // n_heads
        self.arm, self.spec = arm, spec
        self.qn = nn.LayerNorm(self.dh) if qk_norm else nn.Identity()
        self.kn = nn.LayerNorm(self.dh) if qk_norm else nn.Identity()
        self.qkv = nn.Linear(d_model, 3 * d_model, bias=False, device=device)
        self.out = nn.Linear(d_model, d_model, bias=False, device=device)

    def forward(self, x, emb=None, ids=None):
        nb, T, C = x.shape
        q, k, v = self.qkv(x).view(nb, T, 3, self.h, self.dh).unbind(2)
        q, k = self.qn(q), self.kn(k)
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)   # (nb, h, T, dh)
        if self.arm == "softmax":
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        else:
            if self.spec.T != T:
                raise ValueError(f"spec was built for T={self.spec.T}, input has T={T}")
            o, _ = smat_softmax_attention(q, k, v, self.spec)
        return self.out(o.transpose(1, 2).reshape(nb, T, C))
