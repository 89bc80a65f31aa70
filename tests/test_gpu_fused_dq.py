"""The fused backward: dQ accumulated inside the dK/dV kernel (bf16, D = 128).

``bwd(..., fused_dq=True)`` takes this path for bf16 at D = 128
(``smat_bwd_acc``: preprocess, ``smat_bwd_dkdv_dq``, ``smat_bwd_dq_finish``).
Here it is held to the two-pass backward on the same inputs (dV bit for bit,
dK and dQ to a few bf16 ulps, since only the order of fp32 additions
differs), to the oracle on ragged and 64-row-block layouts, and the C entry
points' argument checks are exercised.
"""

import ctypes
import math

import pytest
import torch

from oracle import layout as OL
from oracle.dense_softmax import rowchunked_masked_softmax
from smat_attention_b200 import _lib
from smat_attention_b200.attention import (bwd, check_device_errors, fwd, layout_device_args,
                                           _err_word)
from smat_attention_b200.mask import build_block_mask, build_mask, pattern_layout

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2


def _inputs(B, H, T, D, seed, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, T, D, generator=g).to(device=device, dtype=torch.bfloat16)
            for _ in range(4)]


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1.0)).item()


CASES = [  # (B, H, T, (bs, W, S, sinks))
    (2, 2, 1000, (128, 2, 3, 2)),
    (2, 2, 1000, (64, 3, 5, 2)),
    (1, 4, 4096, (128, 4, 8, 2)),
    (1, 2, 2048, (64, 8, 16, 1)),
    (2, 1, 200, (64, 1, 2, 1)),
    (1, 2, 384, (64, 100, 0, 0)),
]


@pytest.mark.parametrize("B,H,T,lay", CASES)
def test_fused_matches_two_pass_and_oracle(cuda_device, B, H, T, lay):
    D = 128
    spec = build_block_mask(T, *lay)
    q, k, v, do = _inputs(B, H, T, D, seed=T + lay[0])
    scale = 1.0 / math.sqrt(D)
    o, lse = fwd(q, k, v, spec, scale)
    dq_f, dk_f, dv_f = bwd(q, k, v, o, lse, do, spec, scale, fused_dq=True)
    dq_d, dk_d, dv_d = bwd(q, k, v, o, lse, do, spec, scale, fused_dq=False)
    torch.cuda.synchronize()
    assert check_device_errors() == 0
    assert torch.equal(dv_f, dv_d)
    # same bf16 dS^T operand, read from shared memory instead of TMEM
    assert _rel(dk_f, dk_d) < 8e-3, _rel(dk_f, dk_d)
    # per-pair fp32 partials added in L2 against one TMEM accumulator
    assert _rel(dq_f, dq_d) < 8e-3, _rel(dq_f, dq_d)
    f = lambda x: x.float().reshape(B * H, T, D)
    _, _, rdq, rdk, rdv = rowchunked_masked_softmax(
        f(q), f(k), f(v), f(do), OL.block_mask_rows(T, *lay, device=q.device), scale, rows=512)
    # 2e-2 plus the bf16 rounding of the output itself (half an ulp, at most
    # 2^-8 |ref|): rows with |value| >= 4 round by more than 1e-2 on their own
    for name, got, ref in (("dq", dq_f, rdq), ("dk", dk_f, rdk), ("dv", dv_f, rdv)):
        ref = ref.reshape(B, H, T, D)
        excess = ((got.float() - ref).abs() - (TOL_BF16 + ref.abs() * 2.0 ** -8)).max().item()
        assert excess <= 0, (name, excess)


def test_fused_repeatable_except_dq_order(cuda_device):
    """dK and dV are bitwise reproducible; dQ stays within rounding of itself."""
    B, H, T, D, lay = 1, 4, 4096, 128, (128, 4, 8, 2)
    spec = build_block_mask(T, *lay)
    q, k, v, do = _inputs(B, H, T, D, seed=3)
    o, lse = fwd(q, k, v, spec, 1 / math.sqrt(D))
    runs = [bwd(q, k, v, o, lse, do, spec, 1 / math.sqrt(D), fused_dq=True)
            for _ in range(3)]
    torch.cuda.synchronize()
    for dq, dk, dv in runs[1:]:
        assert torch.equal(dk, runs[0][1]) and torch.equal(dv, runs[0][2])
        assert _rel(dq, runs[0][0]) < 8e-3


def test_fused_pattern_layout(cuda_device):
    """An M^(3) mask's pattern layout through the fused path equals the two-pass one."""
    spec = build_mask(1024, 3, chunk=64)
    layout = pattern_layout(spec)
    B, H, D = 1, 2, 128
    q, k, v, do = _inputs(B, H, 1024, D, seed=5)
    scale = 1.0 / math.sqrt(D)
    o, lse = fwd(q, k, v, layout, scale)
    dq_f, dk_f, dv_f = bwd(q, k, v, o, lse, do, layout, scale, fused_dq=True)
    dq_d, dk_d, dv_d = bwd(q, k, v, o, lse, do, layout, scale, fused_dq=False)
    torch.cuda.synchronize()
    assert check_device_errors() == 0
    assert torch.equal(dv_f, dv_d)
    assert _rel(dk_f, dk_d) < 8e-3 and _rel(dq_f, dq_d) < 8e-3


def test_fused_entry_checks(cuda_device):
    L = _lib.lib()
    B, H, T, D, lay = 1, 2, 256, 128, (128, 1, 0, 1)
    spec = build_block_mask(T, *lay)
    q, k, v, do = _inputs(B, H, T, D, seed=1)
    o, lse = fwd(q, k, v, spec, 1 / math.sqrt(D))
    d = layout_device_args(spec, q.device)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    delta = torch.empty(B, H, T, dtype=torch.float32, device=q.device)
    acc = torch.empty(B * H * T * D + 4, dtype=torch.float32, device=q.device)
    err = _err_word(q.device).data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    s3 = _lib.strides3

    def call(acc_ptr, acc_n):
        return L.smat_bwd_acc(
            _lib.DTYPE_BF16, q.data_ptr(), s3(q), k.data_ptr(), s3(k), v.data_ptr(), s3(v),
            o.data_ptr(), s3(o), do.data_ptr(), s3(do), lse.data_ptr(), delta.data_ptr(),
            dq.data_ptr(), s3(dq), dk.data_ptr(), s3(dk), dv.data_ptr(), s3(dv), B, H, T, D,
            d["indptr"].data_ptr(), d["indices"].data_ptr(), d["kind"].data_ptr(),
            d["t_indptr"].data_ptr(), d["t_indices"].data_ptr(), d["t_kind"].data_ptr(),
            d["nblocks"], d["nnzb"], d["block"], d["max_row"], d["t_max_row"], None,
            acc_ptr, acc_n, 1 / math.sqrt(D), err, stream)

    n = B * H * T * D
    assert call(None, n) == 8                          # SMAT_ERR_NULL_POINTER
    assert call(acc.data_ptr(), n - 1) == 1            # SMAT_ERR_BAD_SHAPE
    assert call(acc.data_ptr() + 4, n) == 6            # SMAT_ERR_BAD_ALIGNMENT
    assert call(acc.data_ptr(), n) == 0
    # the finish pass is bf16 only
    assert L.smat_bwd_dq_finish(_lib.DTYPE_F32, acc.data_ptr(), n, dq.data_ptr(), s3(dq),
                                B, H, T, D, 0.1, stream) == 4
    torch.cuda.synchronize()
    assert check_device_errors() == 0
    dq_d, dk_d, dv_d = bwd(q, k, v, o, lse, do, spec, 1 / math.sqrt(D), fused_dq=False)
    assert torch.equal(dv, dv_d) and _rel(dq, dq_d) < 8e-3
    assert ctypes.sizeof(ctypes.c_void_p) == 8
