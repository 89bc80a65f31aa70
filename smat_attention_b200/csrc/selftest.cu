// smat_selftest_wait_timeout: drives the kernels' bounded-wait failure path on
// the device with a wait that can never complete, so that the path that turns
// a stuck pipeline into an error bit (instead of a hung GPU) is exercised by a
// test rather than only by reading.
//
// One CTA of two warps follows the protocol every pipelined kernel here
// follows when a wait runs out:
//   * warp 1 allocates TMEM, as the MMA warps do;
//   * lane 0 of warp 0 waits (mbar_wait_for, the same code as the kernels'
//     mbar_wait) on an mbarrier nothing arrives on, with the caller's short
//     limit: it gives up, raises the CTA abort flag and ORs
//     SMAT_DEVERR_WAIT_TIMEOUT into the error word;
//   * lane 0 of warp 1 waits on a second such barrier with a limit 64x longer:
//     it must leave through the abort flag raised by warp 0, not through its
//     own limit, as the other roles of a kernel do;
//   * both then run the drain wait (mbar_wait_drain_for) on their barrier with
//     the short limit, which also gives up;
//   * warp 1 frees its TMEM and the CTA returns.
// report[0..3]: warp 0's wait returned false (1), warp 1's wait returned false
// (1), warp 1 left before its own limit (1), both drains gave up (1).
// The reference counterpart is the fallback that retires a failing kernel
// with a warning instead of failing the job (src/smat/attention.py:58-75).
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/smat_b200.h"
#include "common.cuh"

namespace smat {
namespace {

__global__ void __launch_bounds__(64, 1)
    selftest_wait_kernel(long long limit, int32_t* err, int32_t* report) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_ptr;
  __shared__ int abort_word;
  volatile int* abort_flag = &abort_word;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars[0]), 1);
    mbar_init(smem_u32(&bars[1]), 1);
    fence_barrier_init();
    abort_word = 0;
    report[0] = report[1] = report[2] = 0;
    report[3] = 1;
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_ptr), 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_ptr;
  if (lane == 0) {
    const uint32_t bar = smem_u32(&bars[warp]);
    const long long my_limit = warp == 0 ? limit : 64 * limit;
    const long long t0 = clock64();
    const bool ok = mbar_wait_for(bar, 0, abort_flag, err, my_limit);
    const long long waited = clock64() - t0;
    report[warp] = ok ? 0 : 1;
    if (warp == 1) report[2] = (!ok && waited < my_limit) ? 1 : 0;
    const bool drained = mbar_wait_drain_for(bar, 0, limit);
    atomicAnd(&report[3], drained ? 0 : 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tbase, 32);
  }
}

}  // namespace
}  // namespace smat

extern "C" int smat_selftest_wait_timeout(int64_t limit_cycles, int32_t* err_word,
                                          int32_t* report, void* stream) {
  if (limit_cycles < 1000 || limit_cycles > SMAT_SELFTEST_MAX_LIMIT) return SMAT_ERR_BAD_SHAPE;
  if (!err_word || !report) return SMAT_ERR_NULL_POINTER;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  smat::selftest_wait_kernel<<<1, 64, 0, s>>>(static_cast<long long>(limit_cycles), err_word,
                                              report);
  return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH;
}
