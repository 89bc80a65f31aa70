"""Query-block sharding of one long sequence across the GPUs of a node.

For the longest sequences (B * H too small to spread over the GPUs by
(batch, head)), each rank owns a set of 128-row query tiles and computes O,
LSE and dQ for those rows, and dK / dV for the key rows of the same tiles.
The layout is known on every rank, so every rank derives every other rank's
plan on the host without communication:

* ownership is zig-zag: the tiles are cut into ``2 * world`` runs of whole
  tile pairs and rank ``r`` owns runs ``r`` and ``2 world - 1 - r``; a row's
  cost grows with its position (one more summary block every ``stride``
  blocks), so pairing an early run with a late one balances the ranks;
* a rank's rows read the K/V blocks of their CSR rows: its own, the window
  halo before each owned run, every sink and every summary block before its
  last row.  One ``all_to_all_single`` with exact split sizes moves, for
  every pair of ranks, the K and V rows of exactly the blocks one owns and
  the other reads (nothing else crosses NVLink) into the reader's full-length
  K and V buffers (:func:`gather_kv`);
* backward: dK / dV of a key block is a sum over the query blocks reading it.
  Each rank runs the dK/dV kernel over the transposed CSR filtered to its own
  query blocks, for every key tile that filter leaves non-empty, and so holds
  partial sums for the blocks it imported.  The reverse all-to-all returns
  those partials to the owners, which add them to their own in fp32
  (:func:`reduce_dkdv`).  dQ needs no exchange.

Both exchanges are a pack kernel, one NCCL ``all_to_all_single`` and an
unpack (or fp32 accumulate) kernel (csrc/rows.cu), run on a side stream:
the K/V exchange can go head group by head group so that the forward of
one group overlaps the exchange of the next, and the dK/dV return overlaps
the dQ pass, which does not touch dK / dV.

Tensors stay full length (``[B, H, T, D]``) on every rank; only the owned
rows of q, k, v and dO need to be valid on input, and only the owned rows of
o, lse, dq, dk and dv are defined on output.  This module has no counterpart
in the reference, which has no multi-GPU path.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Tuple

import numpy as np
import torch

from . import _lib
from .mask import MaskSpec

__all__ = ["ShardPlan", "make_plan", "make_plans", "zigzag_tile_owner", "gather_kv",
           "reduce_dkdv", "sharded_fwd", "sharded_bwd", "owned_rows", "CudaRowOps"]

TILE = _lib.TILE_ROWS


def zigzag_tile_owner(n_tiles: int, world: int) -> np.ndarray:
    """Owner rank of every 128-row tile: ``2 * world`` runs of whole tile
    pairs, rank ``r`` owning runs ``r`` and ``2 world - 1 - r``."""
    if world < 1:
        raise ValueError("world must be >= 1")
    n_pairs = (n_tiles + 1) // 2
    n_runs = 2 * world
    owner = np.empty(n_tiles, dtype=np.int32)
    for c in range(n_runs):
        p_lo, p_hi = c * n_pairs // n_runs, (c + 1) * n_pairs // n_runs
        r = c if c < world else n_runs - 1 - c
        owner[2 * p_lo:min(2 * p_hi, n_tiles)] = r
    return owner


def _runs(mask: np.ndarray) -> List[Tuple[int, int]]:
    """Maximal runs [lo, hi) of True in a boolean array."""
    runs, lo = [], None
    for i, m in enumerate(mask.tolist() + [False]):
        if m and lo is None:
            lo = i
        elif not m and lo is not None:
            runs.append((lo, i))
            lo = None
    return runs


@dataclass
class ShardPlan:
    """Everything one rank needs to run its shard (host arrays; device copies
    are staged on first use)."""

    world: int
    rank: int
    T: int
    block: int
    nqb: int
    n_tiles: int
    tile_owner: np.ndarray           # (n_tiles,) int32
    block_owner: np.ndarray          # (nqb,) int32
    runs: List[Tuple[int, int]]      # owned tile runs [lo, hi)
    imports: np.ndarray              # key blocks this rank reads and does not own
    send_rows: List[np.ndarray]      # per peer: token rows of own blocks the peer reads
    recv_rows: List[np.ndarray]      # per peer: token rows of the peer's blocks read here
    fwd_work: np.ndarray             # forward work items (tile | pair bit), heaviest first
    dq_work: np.ndarray              # owned query tiles, heaviest first
    dkdv_work: np.ndarray            # key tiles with a non-empty filtered column
    t_indptr: np.ndarray             # transposed CSR filtered to the owned query blocks
    t_indices: np.ndarray
    t_kind: np.ndarray
    t_max_row: int
    max_row: int
    dev: Dict[str, Dict[str, torch.Tensor]] = field(default_factory=dict)

    def owned_row_mask(self) -> np.ndarray:
        m = np.zeros(self.T, dtype=bool)
        for lo, hi in self.runs:
            m[lo * TILE:min(hi * TILE, self.T)] = True
        return m

    def device(self, device) -> Dict[str, torch.Tensor]:
        """Device copies of the work lists, the filtered CSR and the gather /
        scatter row indices, staged once per device."""
        key = str(torch.device(device))
        d = self.dev.get(key)
        if d is not None:
            return d
        as_t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a, dtype=dt)).to(device)
        d = {
            "fwd_work": as_t(self.fwd_work, np.int32),
            "dq_work": as_t(self.dq_work, np.int32),
            "dkdv_work": as_t(self.dkdv_work, np.int32),
            "t_indptr": as_t(self.t_indptr, np.int32),
            "t_indices": as_t(self.t_indices, np.int32),
            "t_kind": as_t(self.t_kind, np.uint8),
        }
        # exchange lists: rows packed for the peers (peer order), rows the
        # peers' data lands on, and for the return the union of sent rows
        # with, per row, the received wire rows that hold its partials
        cat = lambda xs: np.concatenate(list(xs) + [np.zeros(0, np.int64)]).astype(np.int64)
        send_cat, recv_cat = cat(self.send_rows), cat(self.recv_rows)
        exp = np.unique(send_cat)
        slot = np.searchsorted(exp, send_cat)
        order = np.argsort(slot, kind="stable")
        ptr = np.zeros(exp.size + 1, dtype=np.int64)
        np.cumsum(np.bincount(slot, minlength=exp.size), out=ptr[1:])
        d["send_cat"] = as_t(send_cat, np.int64)
        d["recv_cat"] = as_t(recv_cat, np.int64)
        d["exp_rows"] = as_t(exp, np.int64)
        d["contrib_ptr"] = as_t(ptr, np.int32)
        d["contrib_wire"] = as_t(order, np.int64)
        self.dev[key] = d
        return d


def _needed_blocks(spec: MaskSpec, qblocks: np.ndarray) -> np.ndarray:
    """Sorted union of the CSR rows of the given query blocks."""
    if qblocks.size == 0:
        return np.zeros(0, dtype=np.int64)
    parts = [spec.indices[spec.indptr[q]:spec.indptr[q + 1]] for q in qblocks.tolist()]
    return np.unique(np.concatenate(parts).astype(np.int64))


def make_plans(spec: MaskSpec, world: int) -> List[ShardPlan]:
    """The plans of all ``world`` ranks for the block layout ``spec``."""
    if spec.kind != "block":
        raise ValueError("query sharding needs a block layout (kind='block')")
    if TILE % spec.block:
        raise ValueError(f"block must divide {TILE}, got {spec.block}")
    T, bs, nqb = spec.T, spec.block, spec.nqb
    sub = TILE // bs
    n_tiles = -(-T // TILE)
    tile_owner = zigzag_tile_owner(n_tiles, world)
    block_owner = tile_owner[np.arange(nqb) // sub].astype(np.int32)
    row_len = np.diff(spec.indptr).astype(np.int64)
    tile_cost = np.zeros(n_tiles, dtype=np.int64)
    np.add.at(tile_cost, np.arange(nqb) // sub, row_len)

    owned_q = [np.flatnonzero(block_owner == r) for r in range(world)]
    needed = [_needed_blocks(spec, owned_q[r]) for r in range(world)]
    imports = [n[block_owner[n] != r] for r, n in enumerate(needed)]
    def rows_of(blocks):
        if len(blocks) == 0:
            return np.zeros(0, dtype=np.int64)
        r = (np.asarray(blocks, np.int64)[:, None] * bs
             + np.arange(bs, dtype=np.int64)[None, :]).reshape(-1)
        return r[r < T]

    # send[r][o]: rows of the blocks r owns and o reads
    send = [[rows_of(imports[o][block_owner[imports[o]] == r]) if o != r
             else np.zeros(0, np.int64) for o in range(world)] for r in range(world)]

    # transposed CSR: per key block the query blocks reading it, ascending
    t_row = np.repeat(np.arange(nqb), np.diff(spec.t_indptr))
    plans = []
    for r in range(world):
        runs = _runs(tile_owner == r)
        items = []
        for lo, hi in runs:
            for t in range(lo, hi, 2):
                if t + 1 < hi:
                    items.append((tile_cost[t] + tile_cost[t + 1], t | _lib.WORK_PAIR_BIT))
                else:
                    items.append((tile_cost[t], t))
        items.sort(key=lambda x: -x[0])
        fwd_work = np.array([w for _, w in items], dtype=np.int32)
        own_tiles = np.flatnonzero(tile_owner == r)
        dq_work = own_tiles[np.argsort(-tile_cost[own_tiles], kind="stable")].astype(np.int32)

        keep = block_owner[spec.t_indices] == r
        t_len = np.bincount(t_row[keep], minlength=nqb).astype(np.int64)
        t_indptr = np.zeros(nqb + 1, dtype=np.int64)
        np.cumsum(t_len, out=t_indptr[1:])
        t_indices = spec.t_indices[keep].astype(np.int32)
        t_kind = spec.t_kind[keep].astype(np.uint8)
        kt_cost = np.zeros(n_tiles, dtype=np.int64)
        np.add.at(kt_cost, np.arange(nqb) // sub, t_len)
        kt = np.flatnonzero(kt_cost > 0)
        dkdv_work = kt[np.argsort(-kt_cost[kt], kind="stable")].astype(np.int32)

        plans.append(ShardPlan(
            world=world, rank=r, T=T, block=bs, nqb=nqb, n_tiles=n_tiles,
            tile_owner=tile_owner, block_owner=block_owner, runs=runs,
            imports=imports[r], send_rows=send[r], recv_rows=[send[o][r] for o in range(world)],
            fwd_work=fwd_work, dq_work=dq_work, dkdv_work=dkdv_work,
            t_indptr=t_indptr.astype(np.int32), t_indices=t_indices, t_kind=t_kind,
            t_max_row=int(t_len.max()) if nqb else 0,
            max_row=int(row_len.max()) if nqb else 0))
    return plans


def make_plan(spec: MaskSpec, world: int, rank: int) -> ShardPlan:
    """This rank's plan (computed from the layout alone, identical on every rank)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    return make_plans(spec, world)[rank]


def owned_rows(plan: ShardPlan) -> np.ndarray:
    """Token rows this rank owns (ascending)."""
    return np.flatnonzero(plan.owned_row_mask())


# --------------------------------------------------------------------------- collectives

class CudaRowOps:
    """The row exchange kernels of libsmat_b200 (csrc/rows.cu): pack listed
    rows of two [B, H, T, D] tensors into a flat wire buffer, unpack, and
    add wire rows into rows in fp32."""

    @staticmethod
    def _args(a, b, rows):
        from .attention import _DTYPES
        if not (a.is_cuda and b.is_cuda and rows.is_cuda):
            raise ValueError("the row exchange runs on CUDA tensors only (no CPU path)")
        B, H, T, D = a.shape
        return (_DTYPES[a.dtype], a.data_ptr(), _lib.strides3(a), b.data_ptr(),
                _lib.strides3(b), B, H, T, D, rows.data_ptr(), rows.numel())

    @staticmethod
    def _tail(a):
        from .attention import _err_word
        return _err_word(a.device).data_ptr(), torch.cuda.current_stream(a.device).cuda_stream

    def pack(self, a, b, rows, wire):
        _lib.check("smat_rows_pack", _lib.lib().smat_rows_pack(
            *self._args(a, b, rows), wire.data_ptr(), *self._tail(a)))

    def unpack(self, a, b, rows, wire):
        _lib.check("smat_rows_unpack", _lib.lib().smat_rows_unpack(
            *self._args(a, b, rows), wire.data_ptr(), *self._tail(a)))

    def accumulate(self, a, b, rows, contrib_ptr, contrib_wire, wire, n_wire):
        _lib.check("smat_rows_accumulate", _lib.lib().smat_rows_accumulate(
            *self._args(a, b, rows), contrib_ptr.data_ptr(), contrib_wire.data_ptr(), n_wire,
            wire.data_ptr(), *self._tail(a)))


def _a2a(recv, send, recv_counts, send_counts, per_row, group):
    torch.distributed.all_to_all_single(recv, send,
                                        output_split_sizes=[c * per_row for c in recv_counts],
                                        input_split_sizes=[c * per_row for c in send_counts],
                                        group=group)


def gather_kv(plan: ShardPlan, k: torch.Tensor, v: torch.Tensor, group=None, ops=None) -> None:
    """Fill the rows of ``k`` and ``v`` (``[B, H, T, D]``, full length; a
    head or batch sub-view is fine) that this rank reads but does not own,
    from their owners: pack, one all-to-all that carries exactly the blocks
    each reader needs, unpack.  Every rank of ``group`` must call it with the
    same shapes, on its current stream."""
    ops = ops or CudaRowOps()
    if isinstance(ops, CudaRowOps) and not (k.is_cuda and v.is_cuda):
        raise ValueError("the row exchange runs on CUDA tensors only (no CPU path)")
    B, H, T, D = k.shape
    d = plan.device(k.device)
    per_row = 2 * B * H * D
    sc = [r.size for r in plan.send_rows]
    rc = [r.size for r in plan.recv_rows]
    send = torch.empty(sum(sc) * per_row, dtype=k.dtype, device=k.device)
    recv = torch.empty(sum(rc) * per_row, dtype=k.dtype, device=k.device)
    if send.numel():
        ops.pack(k, v, d["send_cat"], send)
    _a2a(recv, send, rc, sc, per_row, group)
    if recv.numel():
        ops.unpack(k, v, d["recv_cat"], recv)


def reduce_dkdv(plan: ShardPlan, dk: torch.Tensor, dv: torch.Tensor, group=None,
                ops=None) -> None:
    """Return the partial dK / dV this rank holds for the blocks it imported
    to their owners, and add the partials it receives for its own blocks:
    the reverse all-to-all of :func:`gather_kv`.  Partials travel in the
    tensors' dtype (the kernels' bf16 partials are exact there) and are
    summed in fp32 at the owner, own partial first, then the peers' in rank
    order, and rounded once."""
    ops = ops or CudaRowOps()
    if isinstance(ops, CudaRowOps) and not (dk.is_cuda and dv.is_cuda):
        raise ValueError("the row exchange runs on CUDA tensors only (no CPU path)")
    B, H, T, D = dk.shape
    d = plan.device(dk.device)
    per_row = 2 * B * H * D
    sc = [r.size for r in plan.recv_rows]      # partials go back to the owners
    rc = [r.size for r in plan.send_rows]
    send = torch.empty(sum(sc) * per_row, dtype=dk.dtype, device=dk.device)
    recv = torch.empty(sum(rc) * per_row, dtype=dk.dtype, device=dk.device)
    if send.numel():
        ops.pack(dk, dv, d["recv_cat"], send)
    _a2a(recv, send, rc, sc, per_row, group)
    if d["exp_rows"].numel():
        ops.accumulate(dk, dv, d["exp_rows"], d["contrib_ptr"], d["contrib_wire"], recv,
                       sum(rc))


# --------------------------------------------------------------------------- compute

def _layout(spec: MaskSpec, device):
    from .attention import layout_device_args
    return layout_device_args(spec, device)


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


_SIDE: Dict[str, "torch.cuda.Stream"] = {}


def _side_stream(device) -> "torch.cuda.Stream":
    key = str(torch.device(device))
    s = _SIDE.get(key)
    if s is None:
        s = torch.cuda.Stream(device=device)
        _SIDE[key] = s
    return s


def _groups(B: int, H: int, n: int) -> List[Tuple[slice, slice]]:
    """(batch, head) slices for ``n`` exchange groups: heads when B == 1, else
    batches (an [B, H, T] lse / delta slice must stay one contiguous range)."""
    if B == 1:
        n = max(1, min(n, H))
        cut = [H * i // n for i in range(n + 1)]
        return [(slice(0, 1), slice(cut[i], cut[i + 1])) for i in range(n)]
    n = max(1, min(n, B))
    cut = [B * i // n for i in range(n + 1)]
    return [(slice(cut[i], cut[i + 1]), slice(0, H)) for i in range(n)]


def _fwd_launch(plan, lay, d, q, k, v, o, lse, scale):
    from .attention import _DTYPES, _err_word
    B, H, T, D = q.shape
    w = d["fwd_work"]
    _lib.check("smat_fwd_tiles", _lib.lib().smat_fwd_tiles(
        _DTYPES[q.dtype], q.data_ptr(), _lib.strides3(q), k.data_ptr(), _lib.strides3(k),
        v.data_ptr(), _lib.strides3(v), o.data_ptr(), _lib.strides3(o), lse.data_ptr(),
        B, H, T, D, lay["indptr"].data_ptr(), lay["indices"].data_ptr(), lay["kind"].data_ptr(),
        lay["nblocks"], lay["nnzb"], lay["block"], lay["max_row"], float(scale),
        w.data_ptr(), w.numel(), _err_word(q.device).data_ptr(), _stream(q)))


def sharded_fwd(plan: ShardPlan, spec: MaskSpec, q, k, v, scale: float, *, o=None, lse=None,
                group=None, gather: bool = True, groups: int = 1, ops=None):
    """This rank's forward: bring in the imported K/V rows (unless
    ``gather`` is False), then O and LSE of the owned query tiles.  With
    ``groups`` > 1 the exchange runs group by group (heads, or batches when
    B > 1) on a side stream and the forward of a group starts as soon as its
    rows have landed (on B200 at c5 / 2 GPUs one group measured faster: the
    split forward launches lose more to wave tails than the overlap saves).
    Returns ``(o, lse)`` (full length; owned rows defined).  ``k`` and ``v``
    are filled in place."""
    from .attention import _prep
    q = _prep(q, "q")
    kp, vp = _prep(k, "k"), _prep(v, "v")
    if kp is not k or vp is not v:
        raise ValueError("k and v are filled in place: they must be [B, H, T, D] CUDA tensors "
                         "with D contiguous, 16-byte aligned rows and strides of 8 elements")
    B, H, T, D = q.shape
    if k.shape != q.shape or v.shape != q.shape or T != plan.T:
        raise ValueError("q, k, v must have the same [B, H, T, D] shape with T = plan.T")
    lay = _layout(spec, q.device)
    d = plan.device(q.device)
    if o is None:
        o = torch.empty_like(q)
    if lse is None:
        lse = torch.empty(B, H, T, dtype=torch.float32, device=q.device)
    if not gather or plan.world == 1:
        _fwd_launch(plan, lay, d, q, k, v, o, lse, scale)
        return o, lse
    main = torch.cuda.current_stream(q.device)
    side = _side_stream(q.device)
    side.wait_stream(main)                       # K / V (owned rows) are ready
    ready = []
    with torch.cuda.stream(side):
        for bs, hs in _groups(B, H, groups):
            gather_kv(plan, k[bs, hs], v[bs, hs], group, ops)
            ev = torch.cuda.Event()
            ev.record(side)
            ready.append((bs, hs, ev))
    for bs, hs, ev in ready:
        main.wait_event(ev)
        _fwd_launch(plan, lay, d, q[bs, hs], k[bs, hs], v[bs, hs], o[bs, hs], lse[bs, hs], scale)
    return o, lse


def sharded_bwd(plan: ShardPlan, spec: MaskSpec, q, k, v, o, lse, do, scale: float, *,
                group=None, reduce: bool = True, overlap: bool = True, ops=None):
    """This rank's backward: delta of the owned rows, dK/dV partials over the
    filtered transposed CSR, dQ of the owned tiles, and (unless ``reduce`` is
    False) the dK/dV return, which with ``overlap`` runs on a side stream
    while the dQ pass runs.  ``k`` and ``v`` must already hold the imported
    rows (as left by :func:`sharded_fwd`).  Returns ``(dq, dk, dv)`` (full
    length; owned rows defined)."""
    from .attention import _DTYPES, _err_word, _prep
    q, k, v, o, do = (_prep(x, n) for x, n in ((q, "q"), (k, "k"), (v, "v"), (o, "o"),
                                               (do, "do")))
    B, H, T, D = q.shape
    lay = _layout(spec, q.device)
    d = plan.device(q.device)
    dt = _DTYPES[q.dtype]
    L = _lib.lib()
    s = _stream(q)
    err = _err_word(q.device).data_ptr()
    delta = torch.empty(B, H, T, dtype=torch.float32, device=q.device)
    for lo, hi in plan.runs:
        _lib.check("smat_bwd_preprocess_rows", L.smat_bwd_preprocess_rows(
            dt, o.data_ptr(), _lib.strides3(o), do.data_ptr(), _lib.strides3(do),
            delta.data_ptr(), B, H, T, D, lo * TILE, min(hi * TILE, T), s))
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    wk = d["dkdv_work"]
    _lib.check("smat_bwd_dkdv_tiles", L.smat_bwd_dkdv_tiles(
        dt, q.data_ptr(), _lib.strides3(q), k.data_ptr(), _lib.strides3(k),
        v.data_ptr(), _lib.strides3(v), do.data_ptr(), _lib.strides3(do),
        lse.data_ptr(), delta.data_ptr(), dk.data_ptr(), _lib.strides3(dk),
        dv.data_ptr(), _lib.strides3(dv), B, H, T, D,
        d["t_indptr"].data_ptr(), d["t_indices"].data_ptr(), d["t_kind"].data_ptr(),
        lay["nblocks"], int(d["t_indices"].numel()), lay["block"], plan.t_max_row,
        float(scale), wk.data_ptr(), wk.numel(), err, s))
    exchange = reduce and plan.world > 1
    main = torch.cuda.current_stream(q.device)
    side = _side_stream(q.device) if exchange and overlap else None
    if side is not None:
        side.wait_stream(main)                   # the partials are written
        with torch.cuda.stream(side):
            reduce_dkdv(plan, dk, dv, group, ops)
    wq = d["dq_work"]
    _lib.check("smat_bwd_dq_tiles", L.smat_bwd_dq_tiles(
        dt, q.data_ptr(), _lib.strides3(q), k.data_ptr(), _lib.strides3(k),
        v.data_ptr(), _lib.strides3(v), do.data_ptr(), _lib.strides3(do),
        lse.data_ptr(), delta.data_ptr(), dq.data_ptr(), _lib.strides3(dq), B, H, T, D,
        lay["indptr"].data_ptr(), lay["indices"].data_ptr(), lay["kind"].data_ptr(),
        lay["nblocks"], lay["nnzb"], lay["block"], lay["max_row"], float(scale),
        wq.data_ptr(), wq.numel(), err, s))
    if side is not None:
        main.wait_stream(side)
    elif exchange:
        reduce_dkdv(plan, dk, dv, group, ops)
    return dq, dk, dv
