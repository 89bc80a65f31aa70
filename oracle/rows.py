"""CPU restatement of the row exchange kernels (test infrastructure).

Same contract as ``smat_attention_b200.sharding.CudaRowOps`` (the kernels of
``csrc/rows.cu``): wire row ``r`` of a flat buffer holds ``[2][B][H][D]``
elements, ``a[:, :, rows[r]]`` then ``b[:, :, rows[r]]``.  Used by the gloo
tests of the sharded exchanges in place of the kernels, and on the GPU as
the checker of those kernels.  The layout has no reference counterpart (the
reference has no multi-GPU path).
"""

from __future__ import annotations


class TorchRowOps:
    """pack / unpack / accumulate with torch indexing on any device."""

    @staticmethod
    def _wire(wire, n, a):
        B, H, _, D = a.shape
        return wire[:n * 2 * B * H * D].view(n, 2, B, H, D)

    def pack(self, a, b, rows, wire):
        w = self._wire(wire, rows.numel(), a)
        r = rows.to(a.device)
        w[:, 0] = a.index_select(2, r).permute(2, 0, 1, 3)
        w[:, 1] = b.index_select(2, r).permute(2, 0, 1, 3)

    def unpack(self, a, b, rows, wire):
        w = self._wire(wire, rows.numel(), a)
        r = rows.to(a.device)
        a.index_copy_(2, r, w[:, 0].permute(1, 2, 0, 3))
        b.index_copy_(2, r, w[:, 1].permute(1, 2, 0, 3))

    def accumulate(self, a, b, rows, contrib_ptr, contrib_wire, wire, n_wire):
        w = self._wire(wire, n_wire, a)
        ptr = contrib_ptr.tolist()
        cw = contrib_wire.tolist()
        for e, row in enumerate(rows.tolist()):
            acc_a = a[:, :, row].float()
            acc_b = b[:, :, row].float()
            for c in range(ptr[e], ptr[e + 1]):
                acc_a = acc_a + w[cw[c], 0].float()
                acc_b = acc_b + w[cw[c], 1].float()
            a[:, :, row] = acc_a.to(a.dtype)
            b[:, :, row] = acc_b.to(b.dtype)
