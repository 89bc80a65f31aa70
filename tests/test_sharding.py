"""Query-block sharding without a GPU: the plan every rank derives from the
layout, and the two exchanges (K/V gather, dK/dV return) run as gloo ranks
on CPU with the oracle standing in for the kernels.

The plan is checked against naive loops over tiles (oracle.layout); the
exchanges against the oracle's full-sequence gradients: a rank's dK/dV
partial is the oracle backward with dO zeroed on the query rows it does not
own (those rows then contribute nothing), and after the exchange every owned
key row must hold the full sum.
"""

import datetime
import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import layout as OL
from oracle.dense_softmax import rowchunked_masked_softmax
from oracle.rows import TorchRowOps
from smat_attention_b200 import _lib
from smat_attention_b200.mask import build_block_mask
from smat_attention_b200.sharding import (gather_kv, make_plan, make_plans, reduce_dkdv,
                                          zigzag_tile_owner)

LAYOUTS = [
    (4096, 128, 4, 8, 2),     # c3-shaped layout, short
    (2048, 64, 8, 16, 1),     # c2-shaped (two blocks per tile)
    (1000, 64, 2, 4, 1),      # ragged last block and tile
]


def _decode(work):
    tiles = []
    for w in work.tolist():
        t = w & 0xFFFFFF
        tiles.append(t)
        if w & _lib.WORK_PAIR_BIT:
            tiles.append(t + 1)
    return tiles


@pytest.mark.parametrize("n_tiles,world", [(8, 1), (8, 2), (9, 2), (16, 3), (1024, 8), (5, 4)])
def test_zigzag_owner(n_tiles, world):
    own = zigzag_tile_owner(n_tiles, world)
    assert own.shape == (n_tiles,) and own.min() >= 0 and own.max() < world
    for r in range(world):
        tiles = np.flatnonzero(own == r)
        runs = np.split(tiles, np.flatnonzero(np.diff(tiles) != 1) + 1) if tiles.size else []
        assert len(runs) <= 2
        for run in runs:
            assert run[0] % 2 == 0          # runs start on a tile pair
    # zig-zag: rank r holds an early and a late run
    if n_tiles >= 4 * world:
        for r in range(world):
            tiles = np.flatnonzero(own == r)
            assert tiles.min() < n_tiles // 2 <= tiles.max() or world == 1


@pytest.mark.parametrize("lay", LAYOUTS)
@pytest.mark.parametrize("world", [1, 2, 3, 4])
def test_plan_matches_naive_loops(lay, world):
    T, bs, W, S, n_sink = lay
    spec = build_block_mask(T, bs, W, S, n_sink)
    plans = make_plans(spec, world)
    nqb = spec.nqb
    sub = 128 // bs
    seen_tiles = []
    all_pairs = []
    for p in plans:
        own_tiles = np.flatnonzero(p.tile_owner == p.rank)
        # forward work covers the owned tiles once, pairs never leave a run
        fwd_tiles = _decode(p.fwd_work)
        assert sorted(fwd_tiles) == own_tiles.tolist()
        for w in p.fwd_work.tolist():
            if w & _lib.WORK_PAIR_BIT:
                t = w & 0xFFFFFF
                assert p.tile_owner[t] == p.tile_owner[t + 1] == p.rank
        assert sorted(p.dq_work.tolist()) == own_tiles.tolist()
        seen_tiles += own_tiles.tolist()
        # imports: key blocks of owned rows not owned here
        own_q = [qb for qb in range(nqb) if p.tile_owner[qb // sub] == p.rank]
        need = {kb for qb in own_q for kb in range(qb + 1) if OL.tile_active(qb, kb, W, S, n_sink)}
        imports = sorted(kb for kb in need if p.tile_owner[kb // sub] != p.rank)
        assert p.imports.tolist() == imports
        # filtered transposed CSR: the columns restricted to owned query blocks
        for kb in range(nqb):
            col = p.t_indices[p.t_indptr[kb]:p.t_indptr[kb + 1]].tolist()
            want = [qb for qb in own_q if qb >= kb and OL.tile_active(qb, kb, W, S, n_sink)]
            assert col == want
            all_pairs += [(kb, qb) for qb in col]
        kt = {kb // sub for kb in range(nqb) if p.t_indptr[kb + 1] > p.t_indptr[kb]}
        assert sorted(p.dkdv_work.tolist()) == sorted(kt)
        # every exchange row pair is symmetric and names only imported blocks
        for o in range(world):
            assert np.array_equal(p.recv_rows[o], plans[o].send_rows[p.rank])
            blocks = set((p.recv_rows[o] // bs).tolist())
            assert blocks <= set(imports)
            assert all(p.tile_owner[b // sub] == o for b in blocks)
        got = set()
        for o in range(world):
            got |= set((p.recv_rows[o] // bs).tolist())
        assert got == set(imports)
    assert sorted(seen_tiles) == list(range(-(-T // 128)))
    # the filtered columns partition the full transposed CSR
    full = [(kb, qb) for kb in range(nqb) for qb in
            spec.t_indices[spec.t_indptr[kb]:spec.t_indptr[kb + 1]].tolist()]
    assert sorted(all_pairs) == sorted(full)


def test_c5_balance():
    """At the c5 layout the zig-zag ranks' CSR work differs by < 3 %."""
    spec = build_block_mask(131072, 128, 8, 32, 4)
    rl = np.diff(spec.indptr)
    for world in (2, 4, 8):
        plans = make_plans(spec, world)
        cost = [int(rl[np.repeat(p.tile_owner == p.rank, 1)].sum()) for p in plans]
        assert max(cost) / (sum(cost) / world) < 1.03, cost
        # the exchange moves far less than the sequence
        recv = max(sum(r.size for r in p.recv_rows) for p in plans)
        assert recv < 131072 // 16


def test_make_plan_rejects():
    spec = build_block_mask(1024, 64, 2, 4, 1)
    with pytest.raises(ValueError):
        make_plan(spec, 2, 2)
    with pytest.raises(ValueError):
        make_plans(build_block_mask(1024, 256, 2, 4, 1), 2)


# --------------------------------------------------------------------------- gloo ranks

def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _exchange_worker(rank, world, port, lay):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        T, bs, W, S, n_sink = lay
        B, H, D = 1, 2, 16
        spec = build_block_mask(T, bs, W, S, n_sink)
        plan = make_plan(spec, world, rank)
        g = torch.Generator().manual_seed(7)
        q, k, v, do = (torch.randn(B, H, T, D, generator=g, dtype=torch.float64)
                       for _ in range(4))
        own = torch.from_numpy(plan.owned_row_mask())
        mask_rows = OL.block_mask_rows(T, bs, W, S, n_sink)
        f = lambda x: x.reshape(B * H, T, D)
        scale = 1.0 / math.sqrt(D)
        _, _, _, dk_ref, dv_ref = rowchunked_masked_softmax(f(q), f(k), f(v), f(do), mask_rows,
                                                            scale, rows=256)

        # K/V gather: only owned rows are valid on entry
        kk, vv = k.clone(), v.clone()
        kk[:, :, ~own] = float("nan")
        vv[:, :, ~own] = float("nan")
        gather_kv(plan, kk, vv, ops=TorchRowOps())
        imp_rows = np.concatenate([r for r in plan.recv_rows] + [np.zeros(0, np.int64)])
        readable = own.clone()
        readable[torch.from_numpy(imp_rows)] = True
        assert torch.equal(kk[:, :, readable], k[:, :, readable])
        assert torch.equal(vv[:, :, readable], v[:, :, readable])
        assert torch.isnan(kk[:, :, ~readable]).all()      # nothing else written

        # dK/dV return: this rank's partial = oracle with dO zeroed off-shard
        do_own = do * own.view(1, 1, T, 1).to(do.dtype)
        _, _, _, pdk, pdv = rowchunked_masked_softmax(f(q), f(k), f(v), f(do_own), mask_rows,
                                                      scale, rows=256)
        dk = torch.full_like(k, float("nan"))
        dv = torch.full_like(v, float("nan"))
        dk[:, :, readable] = pdk.reshape(B, H, T, D)[:, :, readable]
        dv[:, :, readable] = pdv.reshape(B, H, T, D)[:, :, readable]
        reduce_dkdv(plan, dk, dv, ops=TorchRowOps())
        err_k = (dk[:, :, own] - dk_ref.reshape(B, H, T, D)[:, :, own]).abs().max().item()
        err_v = (dv[:, :, own] - dv_ref.reshape(B, H, T, D)[:, :, own]).abs().max().item()
        assert err_k < 1e-5 and err_v < 1e-5, (err_k, err_v)
        # the product's row kernels take CUDA tensors only (no CPU path)
        with pytest.raises(ValueError):
            gather_kv(plan, kk, vv)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,lay", [(2, (2048, 128, 2, 4, 1)), (3, (2048, 64, 4, 8, 2)),
                                       (2, (1000, 64, 2, 4, 1))])
def test_exchange_gloo(world, lay):
    mp.spawn(_exchange_worker, args=(world, _free_port(), lay), nprocs=world, join=True)
