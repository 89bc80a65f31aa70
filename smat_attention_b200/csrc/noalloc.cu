// smat_bwd_noalloc: the whole backward without any device allocation.
//
// The backward needs one scratch buffer beyond its inputs and outputs: the
// fp32 row sums delta = rowsum(dO * O), B*H*T floats.  smat_bwd takes it from
// the caller.  Some callers cannot provide it: code whose device memory is
// owned by another allocator (a framework's caching pool that a stray
// cudaMalloc would bypass), code on a latency-critical path where cudaMalloc's
// implicit device synchronisation is not acceptable, and code that runs under
// a memory budget fixed at start-up.  For them this entry point keeps delta in
// a fixed array compiled into the library.
//
// Limits and rules:
//   * B*H*T <= SMAT_NOALLOC_MAX_ROWS (4,194,304 rows = 16 MiB of fp32, e.g. 32
//     heads at T = 131072); larger problems get SMAT_ERR_SCRATCH_LIMIT before
//     anything is launched.
//   * The array exists once per GPU that loads the library and is held until
//     the process exits.
//   * Every call shares the one array.  The preprocess kernel overwrites every
//     element the later kernels read, so nothing needs clearing between calls,
//     but two calls whose kernels overlap on the GPU (different streams, no
//     ordering between them) race on it.
//   * The first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it; make
//     that first call before any stream capture.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/smat_b200.h"

namespace {

// The array's name is only a host-side stand-in in host code; the kernels
// receive the device address looked up below.
__device__ __align__(256) float g_delta_scratch[SMAT_NOALLOC_MAX_ROWS];

constexpr int kMaxDevices = 128;
float* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of this device's copy of the array, looked up once.
int scratch_for_current_device(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return SMAT_ERR_NO_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_delta_scratch) != cudaSuccess || !p) {
      cudaGetLastError();
      return SMAT_ERR_NO_DEVICE;
    }
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[dev];
  return SMAT_OK;
}

}  // namespace

extern "C" int smat_bwd_noalloc(
    int dtype, const void* q, const int64_t* q_stride, const void* k, const int64_t* k_stride,
    const void* v, const int64_t* v_stride, const void* o, const int64_t* o_stride,
    const void* dout, const int64_t* do_stride, const float* lse, void* dq,
    const int64_t* dq_stride, void* dk, const int64_t* dk_stride, void* dv,
    const int64_t* dv_stride, int B, int H, int T, int D, const int32_t* indptr,
    const int32_t* indices, const uint8_t* kind, const int32_t* t_indptr,
    const int32_t* t_indices, const uint8_t* t_kind, int nblocks, int64_t nnzb, int block,
    int max_row, int t_max_row, float scale, int32_t* err_word, void* stream) {
  if (B < 1 || H < 1 || T < 1) return SMAT_ERR_BAD_SHAPE;
  if (static_cast<int64_t>(B) * H * T > SMAT_NOALLOC_MAX_ROWS) return SMAT_ERR_SCRATCH_LIMIT;
  float* delta = nullptr;
  const int rc = scratch_for_current_device(&delta);
  if (rc != SMAT_OK) return rc;
  return smat_bwd(dtype, q, q_stride, k, k_stride, v, v_stride, o, o_stride, dout, do_stride, lse,
                  delta, dq, dq_stride, dk, dk_stride, dv, dv_stride, B, H, T, D, indptr, indices,
                  kind, t_indptr, t_indices, t_kind, nblocks, nnzb, block, max_row, t_max_row,
                  scale, err_word, stream);
}
