"""The bounded-wait failure path on the device.

Every mbarrier wait in the pipelined kernels gives up after a cycle limit,
ORs SMAT_DEVERR_WAIT_TIMEOUT (bit 1) into the caller's error word, raises the
CTA's abort flag (the other warp roles leave through it), drains its own copies
in flight with a bounded wait, frees TMEM and returns.  The self-test entry
point runs that code with a short limit on a barrier nothing ever arrives on,
so the path is exercised without a fault, a trap or an unbounded wait.  The
test then checks that the context is still usable: the next forward and
backward on the same stream pass parity against the oracle.
"""

import ctypes

import pytest
import torch

from smat_attention_b200 import _lib
from smat_attention_b200.attention import check_device_errors
from test_gpu_kernels import _run_case

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT = 1   # SMAT_DEVERR_WAIT_TIMEOUT


def _selftest(limit, device):
    L = _lib.lib()
    err = torch.zeros(1, dtype=torch.int32, device=device)
    report = torch.full((4,), -1, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)
    _lib.check("smat_selftest_wait_timeout",
               L.smat_selftest_wait_timeout(limit, err.data_ptr(), report.data_ptr(),
                                            stream.cuda_stream))
    torch.cuda.synchronize(device)
    return int(err.item()), report.cpu().tolist()


def test_wait_timeout_reports_and_context_survives(cuda_device):
    assert check_device_errors(cuda_device) == 0
    for limit in (1_000_000, 4_000_000):   # ~0.5 ms and ~2 ms of SM clock
        err, report = _selftest(limit, cuda_device)
        assert err & WAIT_TIMEOUT, (limit, err)
        # first wait gave up, second left through the abort flag before its own
        # limit, both drain waits gave up (each 1 when the path behaved)
        assert report == [1, 1, 1, 1], (limit, report)
    # the context is intact: a normal forward + backward on the same stream
    # still matches the oracle
    _run_case(2, 2, 1000, 128, (128, 2, 3, 2), torch.bfloat16, seed=7)
    _run_case(1, 2, 256, 64, (64, 1, 2, 1), torch.float32, seed=8)


def test_selftest_rejects_bad_arguments(cuda_device):
    L = _lib.lib()
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    report = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    assert L.smat_selftest_wait_timeout(10, err.data_ptr(), report.data_ptr(), None) == 1
    assert L.smat_selftest_wait_timeout(1 << 40, err.data_ptr(), report.data_ptr(), None) == 1
    assert L.smat_selftest_wait_timeout(1_000_000, None, report.data_ptr(), None) == 8
    torch.cuda.synchronize(cuda_device)
    assert int(err.item()) == 0 and ctypes.sizeof(ctypes.c_int64) == 8
