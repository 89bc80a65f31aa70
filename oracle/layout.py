"""Independent restatement of the block layout -- TEST INFRASTRUCTURE ONLY.

The block layout has no counterpart in the reference.  Its definition (query
block ``qb``, key block ``kb``, block size ``bs``): ``(qb, kb)`` is active iff
``kb <= qb`` and (``qb - W <= kb`` or ``kb < n_sink`` or ``S > 0 and
kb % S == S - 1``); the diagonal tile is element-wise causal, the others full.

This module evaluates that predicate pair by pair in plain Python loops (no
shared code with ``smat_attention_b200.mask``), and element by element for the
dense mask, so that the product's vectorised builder is checked against a
second, naive statement of the same rule.
"""

from __future__ import annotations

import numpy as np

FULL, CAUSAL = 0, 1


def tile_active(qb: int, kb: int, W: int, S: int, n_sink: int) -> bool:
    if kb > qb:
        return False
    return (qb - W <= kb) or (kb < n_sink) or (S > 0 and kb % S == S - 1)


def block_csr(T: int, bs: int, W: int, S: int, n_sink: int):
    """``(indptr, indices, kinds)`` by a double loop over tiles."""
    nqb = (T + bs - 1) // bs
    indptr, indices, kinds = [0], [], []
    for qb in range(nqb):
        for kb in range(nqb):
            if tile_active(qb, kb, W, S, n_sink):
                indices.append(kb)
                kinds.append(CAUSAL if kb == qb else FULL)
        indptr.append(len(indices))
    return (np.array(indptr, dtype=np.int32), np.array(indices, dtype=np.int32),
            np.array(kinds, dtype=np.uint8))


def transposed_csr(T: int, bs: int, W: int, S: int, n_sink: int):
    """Per key block, the query blocks that read it, ascending."""
    nqb = (T + bs - 1) // bs
    indptr, indices, kinds = [0], [], []
    for kb in range(nqb):
        for qb in range(nqb):
            if tile_active(qb, kb, W, S, n_sink):
                indices.append(qb)
                kinds.append(CAUSAL if kb == qb else FULL)
        indptr.append(len(indices))
    return (np.array(indptr, dtype=np.int32), np.array(indices, dtype=np.int32),
            np.array(kinds, dtype=np.uint8))


def dense_mask(T: int, bs: int, W: int, S: int, n_sink: int) -> np.ndarray:
    """``M[i, j] = 1`` iff ``j <= i`` and tile ``(i // bs, j // bs)`` is active."""
    i = np.arange(T)[:, None]
    j = np.arange(T)[None, :]
    qb, kb = i // bs, j // bs
    act = (kb <= qb) & ((qb - W <= kb) | (kb < n_sink) |
                        ((S > 0) & (kb % max(S, 1) == max(S, 1) - 1)))
    return (act & (j <= i)).astype(np.float64)


def unmasked_pairs(T: int, bs: int, W: int, S: int, n_sink: int) -> int:
    """Count of unmasked ``(i, j)`` pairs, summed row block by row block."""
    total = 0
    nqb = (T + bs - 1) // bs
    for qb in range(nqb):
        r = min(bs, T - qb * bs)
        for kb in range(qb + 1):
            if tile_active(qb, kb, W, S, n_sink):
                c = min(bs, T - kb * bs)
                total += r * (r + 1) // 2 if kb == qb else r * c
    return total


def block_mask_rows(T: int, bs: int, W: int, S: int, n_sink: int, device=None):
    """``mask_rows(r0, r1)`` callable for the row-chunked oracle: rows
    ``[r0, r1)`` of :func:`dense_mask`, built on ``device`` with torch."""
    import torch

    def rows(r0: int, r1: int):
        i = torch.arange(r0, r1, device=device)[:, None]
        j = torch.arange(T, device=device)[None, :]
        qb, kb = i // bs, j // bs
        s = max(S, 1)
        act = (kb <= qb) & ((qb - W <= kb) | (kb < n_sink) |
                            ((S > 0) & (kb % s == s - 1)))
        return act & (j <= i)

    return rows
