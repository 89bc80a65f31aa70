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
                    ``build_mask`` (run through its pattern layout);
``"smat"``          the reference's plain kernelised arm (``model.py:224-320``,
                    its last branch): heads folded into the batch in fp32,
                    ``featurise`` with the feature map (``make_phi`` of the
                    same seed, a learned ``elu + 1`` map, or the Taylor map),
                    then ``kernel_attention.smat_attention`` on the B200
                    kernels.

The kernelised arm's variants (decay, key gates, content-addressed types,
mask banks, the landmark-free control) are not part of this package; their
options are accepted only at their defaults.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import smat_softmax_attention
from .kernel_attention import featurise, make_phi, smat_attention
from .mask import MaskSpec

__all__ = ["Attention", "ARMS"]

ARMS = ("softmax", "smat_softmax", "smat")

# options of the reference's kernelised arm (model.py:113-119)
_KERNEL_ARM_DEFAULTS = dict(r=64, learn_phi=False, chunk=128, triton_bwd=False, no_lr=False,
                            gate=False, phi_kind="elu1", taylor_dim=16, decay=False,
                            dir_head="linear", dir_soft=False, dir_window=4,
                            dt_init=(1e-3, 1e-1), A_init=(1.0, 16.0), type_offsets=None,
                            scan_kernel="phi", assign="positional", read_mode="point",
                            pos_read="plane", hash_src="hidden", hash_freeze=False,
                            hash_shift=0, vocab=None, hash_conv=0)
# the ones the plain "smat" arm uses (any value); the rest select variants
_SMAT_ARM_OPTIONS = ("r", "learn_phi", "chunk", "triton_bwd", "phi_kind", "taylor_dim")


class Attention(nn.Module):
    def __init__(self, d_model: int, n_heads: int, arm: str, *, spec: MaskSpec = None,
                 device=None, seed: int = 0, qk_norm: bool = False, **kernel_arm_options):
        super().__init__()
        if arm not in ARMS:
            raise ValueError(f"arm {arm!r} is not provided here; choose one of {ARMS}")
        opts = dict(_KERNEL_ARM_DEFAULTS)
        for name, val in kernel_arm_options.items():
            if name not in _KERNEL_ARM_DEFAULTS:
                raise TypeError(f"unexpected option {name!r}")
            if val != _KERNEL_ARM_DEFAULTS[name] and (arm != "smat"
                                                      or name not in _SMAT_ARM_OPTIONS):
                raise ValueError(f"option {name}={val!r} selects a variant of the kernelised "
                                 f"arm that this package does not provide")
            opts[name] = val
        if d_model % n_heads:
            raise ValueError("d_model must be a multiple of n_heads")
        if arm == "smat_softmax":
            if spec is None or spec.kind not in ("block", "pattern", "geometric", "endpoint"):
                raise ValueError("arm 'smat_softmax' needs spec=build_block_mask(...) or "
                                 "spec=build_mask(...)")
        if arm == "smat":
            if spec is None or spec.kind not in ("geometric", "endpoint"):
                raise ValueError("arm 'smat' needs spec=build_mask(...)")
            if opts["phi_kind"] not in ("elu1", "relu", "taylor"):
                raise ValueError(f"unknown feature map {opts['phi_kind']!r}")
        self.h, self.dh = n_heads, d_model // n_heads
        self.arm, self.spec, self.chunk = arm, spec, opts["chunk"]
        self.phi_kind = opts["phi_kind"]
        self.key_keep = None        # optional (nb, T) 0/1 gate on keys (the reference's h)
        self.probe = False          # keep (Phi, Psi) of the last forward
        self._last = None
        self.qn = nn.LayerNorm(self.dh) if qk_norm else nn.Identity()
        self.kn = nn.LayerNorm(self.dh) if qk_norm else nn.Identity()
        self.qkv = nn.Linear(d_model, 3 * d_model, bias=False, device=device)
        self.out = nn.Linear(d_model, d_model, bias=False, device=device)
        if arm == "smat":
            if opts["phi_kind"] == "taylor":
                # phi(x) = [1, z, z (x) z / sqrt 2] on a learned projection z:
                # phi(q).phi(k) = 1 + s + s^2 / 2, s = z_q . z_k
                self.P_phi = nn.Linear(self.dh, opts["taylor_dim"], bias=False, device=device)
                self.phi = self._taylor
            elif opts["learn_phi"]:
                self.W_phi = nn.Linear(self.dh, opts["r"], bias=False, device=device)
                self.phi = lambda t: F.elu(self.W_phi(t)) + 1.0
            else:
                self.phi = make_phi(self.dh, opts["r"], kind=opts["phi_kind"], device=device,
                                    dtype=torch.float32, seed=seed)

    def _taylor(self, x):
        z = self.P_phi(x)
        outer = (z.unsqueeze(-1) * z.unsqueeze(-2)).flatten(-2) / math.sqrt(2.0)
        return torch.cat([torch.ones_like(z[..., :1]), z, outer], dim=-1)

    def forward(self, x, emb=None, ids=None):
        nb, T, C = x.shape
        q, k, v = self.qkv(x).view(nb, T, 3, self.h, self.dh).unbind(2)
        q, k = self.qn(q), self.kn(k)
        if self.spec is not None and self.arm != "softmax" and self.spec.T != T:
            raise ValueError(f"spec was built for T={self.spec.T}, input has T={T}")
        if self.arm == "smat":
            # heads folded into the batch, the op in fp32 outside autocast (it
            # divides by a learned-feature normaliser), as the reference does
            with torch.autocast(device_type=x.device.type, enabled=False):
                fold = lambda t: t.transpose(1, 2).reshape(nb * self.h, T, self.dh).float()
                keep = None
                if self.key_keep is not None:
                    keep = (self.key_keep.float().unsqueeze(1).expand(nb, self.h, T)
                            .reshape(nb * self.h, T))
                Phi, Psi, Vb = featurise(fold(q), fold(k), fold(v), self.phi, h=keep)
                if self.probe:
                    self._last = (Phi.detach(), Psi.detach())
                o = smat_attention(Phi, Psi, Vb, self.spec, chunk=self.chunk,
                                   acc_dtype=torch.float32)
                o = o.view(nb, self.h, T, self.dh).transpose(1, 2).to(x.dtype)
            return self.out(o.reshape(nb, T, C))
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)   # (nb, h, T, dh)
        if self.arm == "softmax":
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        else:
            o, _ = smat_softmax_attention(q, k, v, self.spec)
        return self.out(o.transpose(1, 2).reshape(nb, T, C))
