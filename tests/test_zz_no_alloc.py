"""smat_bwd_noalloc: the backward for callers that cannot allocate device memory.

Some callers of this library own no device allocator of their own: their
memory belongs to a framework's pool, or cudaMalloc's implicit synchronisation
is not allowed on their path, or their budget is fixed at start-up.
smat_bwd_noalloc serves them by keeping the backward's only scratch buffer
(the fp32 row sums delta) in a fixed array inside the library.  These tests
call it through the C ABI and hold it to the allocating smat_bwd on the same
inputs, for the bf16 tensor-core backward and the fp32 CUDA-core one, twice in
a row: first a larger problem, then a smaller one, so the second call runs over
the first call's leftover rows in the shared array.  Both entry points run the
same deterministic kernels (no atomics), so the gradients must be equal bit for
bit.  A problem larger than the array must be refused before anything runs.

This file is named to be collected last, so a stop-at-first-failure run has
already run every other test when it gets here.
"""

import ctypes
import math

import pytest
import torch

from smat_attention_b200 import _lib
from smat_attention_b200.attention import check_device_errors, fwd, layout_device_args
from smat_attention_b200.mask import build_block_mask

pytestmark = pytest.mark.gpu

MAX_ROWS = 1 << 22


def _backward(noalloc, q, k, v, o, lse, do, spec, scale):
    L = _lib.lib()
    lay = layout_device_args(spec, q.device)
    B, H, T, D = q.shape
    dtype = _lib.DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.DTYPE_F32
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    err = torch.zeros(1, dtype=torch.int32, device=q.device)
    sp = _lib.strides3
    common_head = [dtype, q.data_ptr(), sp(q), k.data_ptr(), sp(k), v.data_ptr(), sp(v),
                   o.data_ptr(), sp(o), do.data_ptr(), sp(do), lse.data_ptr()]
    common_tail = [dq.data_ptr(), sp(dq), dk.data_ptr(), sp(dk), dv.data_ptr(), sp(dv),
                   B, H, T, D, lay["indptr"].data_ptr(), lay["indices"].data_ptr(),
                   lay["kind"].data_ptr(), lay["t_indptr"].data_ptr(),
                   lay["t_indices"].data_ptr(), lay["t_kind"].data_ptr(), lay["nblocks"],
                   lay["nnzb"], lay["block"], lay["max_row"], lay["t_max_row"], scale,
                   err.data_ptr(), torch.cuda.current_stream().cuda_stream]
    if noalloc:
        st = L.smat_bwd_noalloc(*common_head, *common_tail)
    else:
        delta = torch.empty(B, H, T, dtype=torch.float32, device=q.device)
        st = L.smat_bwd(*common_head, delta.data_ptr(), *common_tail)
    _lib.check("smat_bwd_noalloc" if noalloc else "smat_bwd", st)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return dq, dk, dv


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.bfloat16, 64),
                                     (torch.float32, 64)])
def test_noalloc_matches_allocating_backward(cuda_device, dtype, D):
    T, lay = 1024, (128, 2, 3, 1)
    spec = build_block_mask(T, *lay)
    scale = 1.0 / math.sqrt(D)
    # a larger problem first, then a smaller one over its leftovers
    for call, (B, H, seed) in enumerate(((4, 4, 31), (2, 2, 32))):
        g = torch.Generator().manual_seed(seed)
        q, k, v, do = (torch.randn(B, H, T, D, generator=g).to(cuda_device, dtype)
                       for _ in range(4))
        o, lse = fwd(q, k, v, spec, scale)
        want = _backward(False, q, k, v, o, lse, do, spec, scale)
        got = _backward(True, q, k, v, o, lse, do, spec, scale)
        for name, a, b in zip(("dq", "dk", "dv"), got, want):
            assert torch.isfinite(a).all(), (call, name)
            assert torch.equal(a, b), (call, name, (a.float() - b.float()).abs().max().item())
    assert check_device_errors(cuda_device) == 0


def test_noalloc_refuses_problems_beyond_its_scratch(cuda_device):
    L = _lib.lib()
    st = (ctypes.c_int64 * 3)(0, 0, 128)
    T = MAX_ROWS // 4 + 128          # B * H * T just above the limit with B = 1, H = 4
    nb = (T + 127) // 128
    rc = L.smat_bwd_noalloc(1, 16, st, 16, st, 16, st, 16, st, 16, st, 16, 16, st, 16, st, 16,
                            st, 1, 4, T, 128, 16, 16, 16, 16, 16, 16, nb, 1, 128, 1, 1, 0.1,
                            None, None)
    assert rc == 14   # SMAT_ERR_SCRATCH_LIMIT, returned before anything is launched
    assert b"scratch" in L.smat_status_string(rc)
