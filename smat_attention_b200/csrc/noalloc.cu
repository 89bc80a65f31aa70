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
//     (cudaGetSymbolAddress, with that device current) and caches it together
//     with the identity of the device's current context; make that first call
//     before any stream capture (during a capture the lookup is refused with
//     SMAT_ERR_CAPTURE).  A later call made under another context (after
//     cudaDeviceReset, which reloads the module) looks the address up again.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/smat_b200.h"

namespace {

// The array's name is only a host-side stand-in in host code; the kernels
// receive the device address looked up below.
__device__ __align__(256) float g_delta_scratch[SMAT_NOALLOC_MAX_ROWS];

constexpr int kMaxDevices = 128;
struct ScratchSlot {
  float* addr = nullptr;
  unsigned long long ctx_id = 0;   // context the address belongs to (0: none yet)
};
ScratchSlot g_slots[kMaxDevices];
std::mutex g_scratch_mu;

using PFN_ctx_get_current = CUresult (*)(CUcontext*);
using PFN_ctx_get_id = CUresult (*)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current context (cuCtxGetId, CUDA >= 12.0),
// reached through the runtime's driver entry points; 0 when unavailable.
unsigned long long current_ctx_id() {
  static PFN_ctx_get_current get_current = nullptr;
  static PFN_ctx_get_id get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_ctx_get_current>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_ctx_get_id>(p);
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// The cause of a failed lookup, as a status the caller can act on.
int lookup_status(cudaError_t e) {
  switch (e) {
    case cudaErrorStreamCaptureUnsupported:
    case cudaErrorStreamCaptureInvalidated:
    case cudaErrorStreamCaptureImplicit:
    case cudaErrorStreamCaptureWrongThread:
      return SMAT_ERR_CAPTURE;
    case cudaErrorNoDevice:
    case cudaErrorInvalidDevice:
    case cudaErrorNoKernelImageForDevice:
    case cudaErrorInsufficientDriver:
      return SMAT_ERR_NO_DEVICE;
    default:
      return SMAT_ERR_LAUNCH;
  }
}

// Device address of this device's copy of the array, looked up once per
// device and context.
int scratch_for_current_device(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return e == cudaSuccess ? SMAT_ERR_NO_DEVICE : lookup_status(e);
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot& slot = g_slots[dev];
  const unsigned long long ctx = slot.addr ? current_ctx_id() : 0;
  if (!slot.addr || ctx == 0 || ctx != slot.ctx_id) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_delta_scratch);
    if (e != cudaSuccess || !p) {
      cudaGetLastError();
      slot.addr = nullptr;
      return e == cudaSuccess ? SMAT_ERR_LAUNCH : lookup_status(e);
    }
    slot.addr = static_cast<float*>(p);
    slot.ctx_id = current_ctx_id();   // the lookup made the device's context current
  }
  *out = slot.addr;
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
