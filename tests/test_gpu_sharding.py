"""GPU parity of the query-sharded path.

1. Emulated ranks on one GPU: for every rank of a plan, the work-list entry
   points (smat_fwd_tiles, smat_bwd_preprocess_rows, smat_bwd_dkdv_tiles,
   smat_bwd_dq_tiles) run on the full inputs.  O, LSE and dQ of the owned
   rows must equal the whole-sequence kernels bit for bit (same CTAs, same
   arithmetic); the ranks' dK/dV partials, summed in fp32, must match the
   oracle within the bf16 tolerance (2e-2 max-abs; fp32 path 1e-4).
2. Two ranks over NCCL (skipped with fewer than two GPUs): sharded_fwd and
   sharded_bwd with only the owned rows valid on entry, against the oracle.
"""

import datetime
import math
import os
import socket

import numpy as np
import pytest
import torch

from oracle import layout as OL
from oracle.dense_softmax import rowchunked_masked_softmax
from oracle.rows import TorchRowOps
from smat_attention_b200 import _lib
from smat_attention_b200.attention import (_DTYPES, _err_word, bwd, check_device_errors, fwd,
                                           layout_device_args)
from smat_attention_b200.mask import build_block_mask
from smat_attention_b200.sharding import (CudaRowOps, make_plan, make_plans, sharded_bwd,
                                          sharded_fwd)

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: 2e-2, torch.float32: 1e-4}


def _inputs(B, H, T, D, dtype, seed, device):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, T, D, generator=g).to(device=device, dtype=dtype)
            for _ in range(4)]


def _oracle(q, k, v, do, lay):
    B, H, T, D = q.shape
    f = lambda x: x.float().reshape(B * H, T, D)
    out = rowchunked_masked_softmax(f(q), f(k), f(v), f(do),
                                    OL.block_mask_rows(T, *lay, device=q.device),
                                    1.0 / math.sqrt(D), rows=512)
    return [x.reshape(B, H, T, -1).squeeze(-1) for x in out]


def _rank_kernels(plan, spec, q, k, v, o, lse, do, scale):
    """One emulated rank: the work-list launches sharded_bwd would make,
    without the exchange (the inputs here are valid on every row)."""
    B, H, T, D = q.shape
    L = _lib.lib()
    lay = layout_device_args(spec, q.device)
    d = plan.device(q.device)
    dt = _DTYPES[q.dtype]
    s = torch.cuda.current_stream().cuda_stream
    err = _err_word(q.device).data_ptr()
    o_r, lse_r = sharded_fwd(plan, spec, q, k, v, scale, gather=False)
    delta = torch.full((B, H, T), float("nan"), device=q.device)
    for lo, hi in plan.runs:
        _lib.check("pre", L.smat_bwd_preprocess_rows(
            dt, o.data_ptr(), _lib.strides3(o), do.data_ptr(), _lib.strides3(do),
            delta.data_ptr(), B, H, T, D, lo * 128, min(hi * 128, T), s))
    dq, dk, dv = (torch.full_like(q, float("nan")) for _ in range(3))
    wk, wq = d["dkdv_work"], d["dq_work"]
    _lib.check("dkdv", L.smat_bwd_dkdv_tiles(
        dt, q.data_ptr(), _lib.strides3(q), k.data_ptr(), _lib.strides3(k),
        v.data_ptr(), _lib.strides3(v), do.data_ptr(), _lib.strides3(do),
        lse.data_ptr(), delta.data_ptr(), dk.data_ptr(), _lib.strides3(dk),
        dv.data_ptr(), _lib.strides3(dv), B, H, T, D,
        d["t_indptr"].data_ptr(), d["t_indices"].data_ptr(), d["t_kind"].data_ptr(),
        lay["nblocks"], int(d["t_indices"].numel()), lay["block"], plan.t_max_row,
        scale, wk.data_ptr(), wk.numel(), err, s))
    _lib.check("dq", L.smat_bwd_dq_tiles(
        dt, q.data_ptr(), _lib.strides3(q), k.data_ptr(), _lib.strides3(k),
        v.data_ptr(), _lib.strides3(v), do.data_ptr(), _lib.strides3(do),
        lse.data_ptr(), delta.data_ptr(), dq.data_ptr(), _lib.strides3(dq), B, H, T, D,
        lay["indptr"].data_ptr(), lay["indices"].data_ptr(), lay["kind"].data_ptr(),
        lay["nblocks"], lay["nnzb"], lay["block"], lay["max_row"], scale,
        wq.data_ptr(), wq.numel(), err, s))
    return o_r, lse_r, dq, dk, dv, delta


@pytest.mark.parametrize("B,H,T,D,lay,dtype,world", [
    (1, 4, 4096, 128, (128, 4, 8, 2), torch.bfloat16, 2),
    (1, 4, 4096, 128, (128, 4, 8, 2), torch.bfloat16, 3),
    (2, 2, 3000, 64, (64, 8, 16, 1), torch.bfloat16, 4),
    (1, 2, 1000, 64, (64, 2, 4, 1), torch.float32, 2),
    (1, 2, 1152, 32, (32, 2, 4, 1), torch.float32, 3),
])
def test_emulated_ranks(B, H, T, D, lay, dtype, world):
    spec = build_block_mask(T, *lay)
    q, k, v, do = _inputs(B, H, T, D, dtype, 11, "cuda")
    scale = 1.0 / math.sqrt(D)
    o, lse = fwd(q, k, v, spec, scale)
    dq_full, _, _ = bwd(q, k, v, o, lse, do, spec, scale)
    delta_full = (o.float() * do.float()).sum(-1)
    ro, rlse, rdq, rdk, rdv = _oracle(q, k, v, do, lay)
    dk_sum = torch.zeros(B, H, T, D, device="cuda")
    dv_sum = torch.zeros(B, H, T, D, device="cuda")
    covered = torch.zeros(T, dtype=torch.bool, device="cuda")
    for plan in make_plans(spec, world):
        own = torch.from_numpy(plan.owned_row_mask()).cuda()
        o_r, lse_r, dq_r, dk_r, dv_r, delta_r = _rank_kernels(plan, spec, q, k, v, o, lse, do,
                                                              scale)
        torch.cuda.synchronize()
        assert check_device_errors() == 0
        assert torch.equal(o_r[:, :, own], o[:, :, own])
        assert torch.equal(lse_r[:, :, own], lse[:, :, own])
        assert torch.equal(dq_r[:, :, own], dq_full[:, :, own])
        assert (delta_r[:, :, own] - delta_full[:, :, own]).abs().max().item() < 1e-3
        # rows outside the rank's tiles are never written
        assert torch.isnan(dq_r[:, :, ~own]).all()
        kt = np.zeros(T, dtype=bool)
        for t in plan.dkdv_work.tolist():
            kt[t * 128:(t + 1) * 128] = True
        kt = torch.from_numpy(kt).cuda()
        assert torch.isnan(dk_r[:, :, ~kt]).all()
        dk_sum[:, :, kt] += dk_r[:, :, kt].float()
        dv_sum[:, :, kt] += dv_r[:, :, kt].float()
        covered |= own
    assert covered.all()
    tol = TOL[dtype]
    assert (dk_sum - rdk).abs().max().item() < tol
    assert (dv_sum - rdv).abs().max().item() < tol
    assert (dq_full.float() - rdq).abs().max().item() < tol


def test_bad_work_item_sets_error_bit():
    """A tile past the end is rejected by the CTA that reads it: error bit 8,
    nothing written, the context stays usable."""
    T, D = 1024, 64
    spec = build_block_mask(T, 64, 2, 4, 1)
    q, k, v, _ = _inputs(1, 2, T, D, torch.bfloat16, 3, "cuda")
    lay = layout_device_args(spec, "cuda")
    o = torch.full_like(q, float("nan"))
    lse = torch.empty(1, 2, T, device="cuda")
    work = torch.tensor([8, 3 | _lib.WORK_PAIR_BIT * 4], dtype=torch.int32, device="cuda")
    check_device_errors()
    L = _lib.lib()
    _lib.check("fwd_tiles", L.smat_fwd_tiles(
        1, q.data_ptr(), _lib.strides3(q), k.data_ptr(), _lib.strides3(k), v.data_ptr(),
        _lib.strides3(v), o.data_ptr(), _lib.strides3(o), lse.data_ptr(), 1, 2, T, D,
        lay["indptr"].data_ptr(), lay["indices"].data_ptr(), lay["kind"].data_ptr(),
        lay["nblocks"], lay["nnzb"], lay["block"], lay["max_row"], 0.125,
        work.data_ptr(), 2, _err_word(q.device).data_ptr(),
        torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert check_device_errors() == 8
    assert torch.isnan(o).all()
    # the next launch on the same context works
    o2, _ = fwd(q, k, v, spec, 0.125)
    torch.cuda.synchronize()
    assert torch.isfinite(o2.float()).all()


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float32, 64)])
def test_row_kernels_match_oracle(dtype, D):
    """pack / unpack / accumulate of csrc/rows.cu equal the oracle's
    restatement bit for bit, on whole tensors and on head-slice views."""
    B, H, T = 2, 4, 700
    g = torch.Generator().manual_seed(9)
    a, b = (torch.randn(B, H, T, D, generator=g).to("cuda", dtype) for _ in range(2))
    cu, ref = CudaRowOps(), TorchRowOps()
    rows = torch.tensor([5, 699, 0, 128, 129, 5], dtype=torch.int64, device="cuda")
    for x, y in ((a, b), (a[:, 1:3], b[:, 1:3])):
        Bx, Hx = x.shape[:2]
        w1 = torch.full((rows.numel() * 2 * Bx * Hx * D,), float("nan"), dtype=dtype,
                        device="cuda")
        w2 = w1.clone()
        cu.pack(x, y, rows, w1)
        ref.pack(x, y, rows, w2)
        torch.cuda.synchronize()
        assert torch.equal(w1, w2)
        # unpack of distinct rows into copies
        urows = rows[:5]
        wire = torch.randn(urows.numel() * 2 * Bx * Hx * D, generator=g).to("cuda", dtype)
        x1, y1, x2, y2 = x.clone(), y.clone(), x.clone(), y.clone()
        cu.unpack(x1, y1, urows, wire)
        ref.unpack(x2, y2, urows, wire)
        torch.cuda.synchronize()
        assert torch.equal(x1, x2) and torch.equal(y1, y2)
        # accumulate: row 3 gets wire rows 1, 0; row 10 none; row 600 gets 3, 4, 2
        exp = torch.tensor([3, 10, 600], dtype=torch.int64, device="cuda")
        ptr = torch.tensor([0, 2, 2, 5], dtype=torch.int32, device="cuda")
        cw = torch.tensor([1, 0, 3, 4, 2], dtype=torch.int64, device="cuda")
        x1, y1, x2, y2 = x.clone(), y.clone(), x.clone(), y.clone()
        cu.accumulate(x1, y1, exp, ptr, cw, wire, 5)
        ref.accumulate(x2, y2, exp, ptr, cw, wire, 5)
        torch.cuda.synchronize()
        assert torch.equal(x1, x2) and torch.equal(y1, y2)
    assert check_device_errors() == 0


def test_row_kernels_flag_bad_rows():
    """A row index outside [0, T) is skipped and reported (error bit 8)."""
    a, b = (torch.zeros(1, 2, 256, 64, dtype=torch.bfloat16, device="cuda") for _ in range(2))
    wire = torch.ones(2 * 2 * 2 * 64, dtype=torch.bfloat16, device="cuda")
    rows = torch.tensor([3, 256], dtype=torch.int64, device="cuda")
    check_device_errors()
    CudaRowOps().unpack(a, b, rows, wire)
    torch.cuda.synchronize()
    assert check_device_errors() == 8
    assert a[:, :, 3].float().sum().item() == 2 * 64 and a.float().sum().item() == 2 * 64


# --------------------------------------------------------------------------- NCCL ranks

def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _nccl_worker(rank, world, port, case, overlap):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        B, H, T, D, lay = case
        dev = torch.device("cuda", rank)
        spec = build_block_mask(T, *lay)
        plan = make_plan(spec, world, rank)
        q, k, v, do = _inputs(B, H, T, D, torch.bfloat16, 5, dev)
        scale = 1.0 / math.sqrt(D)
        own = torch.from_numpy(plan.owned_row_mask()).to(dev)
        # only the owned rows are valid on entry
        qs, ks, vs, dos = (x.clone() for x in (q, k, v, do))
        for x in (qs, ks, vs, dos):
            x[:, :, ~own] = float("nan")
        o, lse = sharded_fwd(plan, spec, qs, ks, vs, scale, groups=4 if overlap else 1)
        dq, dk, dv = sharded_bwd(plan, spec, qs, ks, vs, o, lse, dos, scale, overlap=overlap)
        torch.cuda.synchronize()
        assert check_device_errors(dev) == 0
        ro, rlse, rdq, rdk, rdv = _oracle(q, k, v, do, lay)
        for name, got, ref in (("o", o, ro), ("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
            err = (got[:, :, own].float() - ref[:, :, own]).abs().max().item()
            assert err < 2e-2, (rank, name, err)
        assert (lse[:, :, own] - rlse[:, :, own]).abs().max().item() < 1e-3
        # forward rows equal the single-GPU kernels bit for bit
        o1, lse1 = fwd(q, k, v, spec, scale)
        assert torch.equal(o[:, :, own], o1[:, :, own])
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("case,overlap", [((1, 4, 8192, 128, (128, 4, 8, 2)), True),
                                          ((1, 4, 8192, 128, (128, 4, 8, 2)), False),
                                          ((2, 2, 4096, 64, (64, 8, 16, 1)), True)])
def test_two_ranks_nccl(case, overlap):
    import torch.multiprocessing as mp
    ctx = mp.start_processes(_nccl_worker, args=(2, _free_port(), case, overlap), nprocs=2,
                             join=False, start_method="spawn")
    import time
    deadline = time.time() + 240
    while not ctx.join(timeout=5):
        if time.time() > deadline:
            for p in ctx.processes:
                if p.is_alive():
                    p.kill()
            pytest.fail("NCCL ranks did not finish in 240 s")
