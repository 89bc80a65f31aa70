// C ABI of libsmat_b200.so (declared in include/smat_b200.h): argument checks,
// TMA descriptor construction and kernel launches.  Nothing here allocates
// device memory and nothing synchronises; every check that can fail runs on
// the host before the first launch.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/smat_b200.h"
#include "bwd_tc.cuh"
#include "fwd_tc.cuh"
#include "simt_fp32.cuh"

namespace {

using namespace smat;

struct TArg {
  const void* p;
  int64_t sb, sh, st;
};

TArg targ(const void* p, const int64_t* s) { return TArg{p, s[0], s[1], s[2]}; }

// Optional list of tiles to compute (device array); items == nullptr means
// every tile of the sequence.
struct Work {
  const int32_t* items;
  int n;
};
constexpr Work kAllTiles{nullptr, 0};
constexpr MdPattern kNoPattern{nullptr, nullptr, 0, 0, 0, 1, 1, 0, 0};

int check_work(const Work& w) {
  if (w.n < 0) return SMAT_ERR_BAD_SHAPE;
  if (w.n > 0 && !w.items) return SMAT_ERR_NULL_POINTER;
  return SMAT_OK;
}

// ---------------------------------------------------------------- checks
int check_common(int dtype, int B, int H, int T, int D, int nblocks, int block) {
  if (B < 1 || H < 1 || T < 1) return SMAT_ERR_BAD_SHAPE;
  if (block < 1) return SMAT_ERR_UNSUPPORTED_BLOCK;
  if (nblocks != (T + block - 1) / block) return SMAT_ERR_BAD_SHAPE;
  if (dtype == SMAT_DTYPE_BF16) {
    if (D != 64 && D != 128) return SMAT_ERR_UNSUPPORTED_D;
    if (block != 64 && block != 128) return SMAT_ERR_UNSUPPORTED_BLOCK;
  } else if (dtype == SMAT_DTYPE_F32) {
    if (D != 32 && D != 64 && D != 128) return SMAT_ERR_UNSUPPORTED_D;
  } else {
    return SMAT_ERR_UNSUPPORTED_DTYPE;
  }
  if (static_cast<int64_t>(B) * H > (1LL << 30) / std::max(1, (T + 127) / 128))
    return SMAT_ERR_BAD_SHAPE;  // linear grid index must fit an int
  return SMAT_OK;
}

// Tensor argument: non-null, strides non-negative; for bf16 the TMA / vector
// store rules (16-byte aligned base, strides a multiple of 8 elements).
int check_tensor(const TArg& t, int dtype) {
  if (!t.p) return SMAT_ERR_NULL_POINTER;
  if (t.sb < 0 || t.sh < 0 || t.st < 0) return SMAT_ERR_BAD_STRIDE;
  if (dtype == SMAT_DTYPE_BF16) {
    if (reinterpret_cast<uintptr_t>(t.p) % 16) return SMAT_ERR_BAD_ALIGNMENT;
    if (t.sb % 8 || t.sh % 8 || t.st % 8) return SMAT_ERR_BAD_ALIGNMENT;
  } else {
    if (reinterpret_cast<uintptr_t>(t.p) % 4) return SMAT_ERR_BAD_ALIGNMENT;
  }
  return SMAT_OK;
}

int check_layout_args(const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                      int64_t nnzb, int max_row, int block) {
  if (!indptr || !kind || (!indices && nnzb > 0)) return SMAT_ERR_NULL_POINTER;
  if (nnzb < 0 || nnzb > (1LL << 31) - 1 || max_row < 0) return SMAT_ERR_CSR_INVALID;
  return SMAT_OK;
}

// M^(d) pattern of a layout's PATTERN tiles: field ranges (the device rule
// indexes the tables only within them) and, for launches, the tables.
int check_pattern(const smat_pattern_t* pt, int T, bool need_tables, MdPattern* out) {
  if (!pt) return SMAT_ERR_NULL_POINTER;
  if (pt->family != SMAT_FAMILY_GEOMETRIC && pt->family != SMAT_FAMILY_ENDPOINT)
    return SMAT_ERR_BAD_PATTERN;
  if (pt->n_P < 0 || pt->n < pt->n_P || pt->n > T || pt->B < 1 || pt->N0 < 1)
    return SMAT_ERR_BAD_PATTERN;
  if (static_cast<int64_t>(pt->row_words) < (static_cast<int64_t>(pt->N0) + 63) / 32 ||
      static_cast<int64_t>(pt->col_words) < (static_cast<int64_t>(pt->B) + 63) / 32)
    return SMAT_ERR_BAD_PATTERN;
  if (pt->family == SMAT_FAMILY_ENDPOINT && pt->N0 < pt->n - pt->n_P) return SMAT_ERR_BAD_PATTERN;
  if (need_tables && (!pt->row_bits || !pt->col_bits)) return SMAT_ERR_NULL_POINTER;
  *out = MdPattern{pt->row_bits, pt->col_bits, pt->family, pt->n,        pt->n_P,
                   pt->B,        pt->N0,       pt->row_words, pt->col_words};
  return SMAT_OK;
}

// Layout checks shared by smat_layout_validate (FULL / CAUSAL kinds) and
// smat_layout_validate_pattern (PATTERN allowed anywhere).
int validate_layout(int nblocks, int64_t nnzb, const int32_t* indptr, const int32_t* indices,
                    const uint8_t* kind, int transposed, bool allow_pattern, int32_t* max_row_out) {
  if (nblocks < 0 || nnzb < 0) return SMAT_ERR_CSR_INVALID;
  if (!indptr || (nnzb > 0 && (!indices || !kind))) return SMAT_ERR_NULL_POINTER;
  if (indptr[0] != 0 || indptr[nblocks] != nnzb) return SMAT_ERR_CSR_INVALID;
  int32_t longest = 0;
  for (int r = 0; r < nblocks; ++r) {
    const int64_t a = indptr[r], b = indptr[r + 1];
    if (b < a || b > nnzb) return SMAT_ERR_CSR_INVALID;
    longest = std::max<int32_t>(longest, static_cast<int32_t>(b - a));
    int32_t prev = -1;
    for (int64_t e = a; e < b; ++e) {
      const int32_t c = indices[e];
      if (c < 0 || c >= nblocks || c <= prev) return SMAT_ERR_CSR_INVALID;
      if (transposed ? (c < r) : (c > r)) return SMAT_ERR_CSR_INVALID;
      const uint8_t want = (c == r) ? SMAT_TILE_CAUSAL : SMAT_TILE_FULL;
      if (kind[e] != want && !(allow_pattern && kind[e] == SMAT_TILE_PATTERN))
        return SMAT_ERR_CSR_INVALID;
      prev = c;
    }
  }
  if (max_row_out) *max_row_out = longest;
  return SMAT_OK;
}

// ---------------------------------------------------------------- TMA
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 4-D map over a [B, H, T, D] bf16 tensor, box {64, rows, 1, 1}, 128 B swizzle.
int make_map(CUtensorMap* m, const TArg& t, int B, int H, int T, int D, int rows) {
  auto enc = get_encode();
  if (!enc) return SMAT_ERR_NO_DEVICE;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(T),
                        static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(t.st) * 2, static_cast<cuuint64_t>(t.sh) * 2,
                           static_cast<cuuint64_t>(t.sb) * 2};
  // a size-1 dimension may carry any stride; give it a legal one
  if (H == 1) strides[1] = std::max<cuuint64_t>(strides[1], 16);
  if (B == 1) strides[2] = std::max<cuuint64_t>(strides[2], 16);
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(t.p), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SMAT_OK : SMAT_ERR_TMA_DESCRIPTOR;
}

template <typename K>
int set_smem(K kernel, int bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) ==
                 cudaSuccess
             ? SMAT_OK
             : SMAT_ERR_LAUNCH;
}

int launch_status() {
  return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH;
}

// ---------------------------------------------------------------- forward
template <int D, int NT, int BN = 128>
int fwd_tc(const TArg& q, const TArg& k, const TArg& v, const TArg& o, float* lse, int B, int H,
           int T, const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
           int nblocks, int64_t nnzb, int block, float scale, const Work& work,
           const MdPattern& md, int32_t* err, cudaStream_t s) {
  using C = FwdCfg<D, NT, BN>;
  CUtensorMap mq, mk, mv, mo;
  int rc;
  if ((rc = make_map(&mq, q, B, H, T, D, C::BM))) return rc;
  if ((rc = make_map(&mo, o, B, H, T, D, C::BM))) return rc;   // O is stored by TMA
  if ((rc = make_map(&mk, k, B, H, T, D, C::BOX))) return rc;
  if ((rc = make_map(&mv, v, B, H, T, D, C::BOX))) return rc;
  FwdParams p{};
  p.indptr = indptr;
  p.indices = indices;
  p.kind = kind;
  p.o = static_cast<__nv_bfloat16*>(const_cast<void*>(o.p));
  p.lse = lse;
  p.o_sb = o.sb;
  p.o_sh = o.sh;
  p.o_st = o.st;
  p.B = B;
  p.H = H;
  p.T = T;
  p.nblocks = nblocks;
  p.nnzb = static_cast<int>(nnzb);
  p.bs = block;
  p.n_tiles = (T + C::BM - 1) / C::BM;
  p.n_pairs = (p.n_tiles + 1) / 2;
  p.work = work.items;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = err;
  p.md = md;
  auto kern = smat_fwd_tc_kernel<D, NT, BN>;
  if ((rc = set_smem(kern, C::SMEM_BYTES))) return rc;
  const int64_t grid =
      static_cast<int64_t>(work.items ? work.n * (3 - NT) : (p.n_tiles + NT - 1) / NT) * B * H;
  if (grid == 0) return SMAT_OK;
  kern<<<static_cast<unsigned>(grid), C::THREADS, C::SMEM_BYTES, s>>>(mq, mk, mv, mo, p);
  return launch_status();
}

SimtParams simt_params(int B, int H, int T, int block, float scale, const int32_t* indptr,
                       const int32_t* indices, const uint8_t* kind, int nblocks, int64_t nnzb,
                       int32_t* err, const Work& work, int span_tiles, const MdPattern& md) {
  SimtParams p{};
  p.md = md;
  p.work = work.items;
  p.span_tiles = span_tiles;
  p.B = B;
  p.H = H;
  p.T = T;
  p.bs = block;
  p.scale = scale;
  p.indptr = indptr;
  p.indices = indices;
  p.kind = kind;
  p.nblocks = nblocks;
  p.nnzb = static_cast<int>(nnzb);
  p.err = err;
  return p;
}

void set3(int64_t* dst, const TArg& t) {
  dst[0] = t.sb;
  dst[1] = t.sh;
  dst[2] = t.st;
}

template <template <int> class Launch>
int dispatch_simt_d(int D, SimtParams& p, int T, int n_work, int BH, cudaStream_t s) {
  switch (D) {
    case 32: return Launch<32>::run(p, T, n_work, BH, s);
    case 64: return Launch<64>::run(p, T, n_work, BH, s);
    case 128: return Launch<128>::run(p, T, n_work, BH, s);
  }
  return SMAT_ERR_UNSUPPORTED_D;
}

template <int D>
struct FwdSimt {
  static int run(SimtParams& p, int T, int n_work, int BH, cudaStream_t s) {
    constexpr int RPC = SIMT_THREADS / (D / 32);
    const int64_t gx = p.work ? static_cast<int64_t>(n_work) * p.span_tiles * SIMT_TILE / RPC
                              : (T + RPC - 1) / RPC;
    if (gx == 0) return SMAT_OK;
    dim3 grid(static_cast<unsigned>(gx), BH);
    smat_fwd_simt_kernel<D><<<grid, SIMT_THREADS, 0, s>>>(p);
    return launch_status();
  }
};
template <int D>
struct DqSimt {
  static int run(SimtParams& p, int T, int n_work, int BH, cudaStream_t s) {
    constexpr int RPC = SIMT_THREADS / (D / 32);
    const int64_t gx = p.work ? static_cast<int64_t>(n_work) * p.span_tiles * SIMT_TILE / RPC
                              : (T + RPC - 1) / RPC;
    if (gx == 0) return SMAT_OK;
    dim3 grid(static_cast<unsigned>(gx), BH);
    smat_dq_simt_kernel<D><<<grid, SIMT_THREADS, 0, s>>>(p);
    return launch_status();
  }
};
template <int D>
struct DkdvSimt {
  static int run(SimtParams& p, int T, int n_work, int BH, cudaStream_t s) {
    constexpr int RPC = SIMT_THREADS / (D / 32);
    const int64_t gx = p.work ? static_cast<int64_t>(n_work) * p.span_tiles * SIMT_TILE / RPC
                              : (T + RPC - 1) / RPC;
    if (gx == 0) return SMAT_OK;
    dim3 grid(static_cast<unsigned>(gx), BH);
    smat_dkdv_simt_kernel<D><<<grid, SIMT_THREADS, 0, s>>>(p);
    return launch_status();
  }
};

// ---------------------------------------------------------------- backward
template <bool DKDV, int D, int CN, bool FQ = false>
int bwd_tc_cn(const TArg& r0, const TArg& r1, const TArg& c0, const TArg& c1, const float* lse,
              const float* delta, const TArg& out0, const TArg* out1, int B, int H, int T,
              const int32_t* indptr, const int32_t* indices, const uint8_t* kind, int nblocks,
              int64_t nnzb, int block, float scale, const Work& work, const MdPattern& md,
              int32_t* err, cudaStream_t s, float* dq_acc = nullptr) {
  using C = BwdCfg<DKDV, D, CN, FQ>;
  CUtensorMap m0, m1, mc0, mc1, mo0, mo1;
  int rc;
  if ((rc = make_map(&m0, r0, B, H, T, D, C::BM))) return rc;
  if ((rc = make_map(&m1, r1, B, H, T, D, C::BM))) return rc;
  if ((rc = make_map(&mc0, c0, B, H, T, D, C::BOX))) return rc;
  if ((rc = make_map(&mc1, c1, B, H, T, D, C::BOX))) return rc;
  // the outputs are stored by TMA from the SW128 tile layout
  if ((rc = make_map(&mo0, out0, B, H, T, D, C::BM))) return rc;
  if ((rc = make_map(&mo1, out1 ? *out1 : out0, B, H, T, D, C::BM))) return rc;
  BwdParams p{};
  p.indptr = indptr;
  p.indices = indices;
  p.kind = kind;
  p.lse = lse;
  p.delta = delta;
  p.out0 = static_cast<__nv_bfloat16*>(const_cast<void*>(out0.p));
  p.o0_sb = out0.sb;
  p.o0_sh = out0.sh;
  p.o0_st = out0.st;
  if (out1) {
    p.out1 = static_cast<__nv_bfloat16*>(const_cast<void*>(out1->p));
    p.o1_sb = out1->sb;
    p.o1_sh = out1->sh;
    p.o1_st = out1->st;
  }
  p.B = B;
  p.H = H;
  p.T = T;
  p.nblocks = nblocks;
  p.nnzb = static_cast<int>(nnzb);
  p.bs = block;
  p.n_tiles = (T + C::BM - 1) / C::BM;
  p.work = work.items;
  // dK/dV: key tiles interleaved over groups of 16 (b, h), so the long sink
  // and summary tiles of one head overlap the other heads' short ones (at 16
  // (b, h) per GPU head by head left them alone at the end: 0.665 ms against
  // 0.489); dQ: head by head (its tiles cost about the same)
  p.head_group = DKDV ? 16 : 1;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.dq_acc = dq_acc;
  p.err = err;
  p.md = md;
  auto kern = smat_bwd_tc_kernel<DKDV, D, CN, FQ>;
  if ((rc = set_smem(kern, C::SMEM_BYTES))) return rc;
  const int64_t grid = static_cast<int64_t>(work.items ? work.n : p.n_tiles) * B * H;
  if (grid == 0) return SMAT_OK;
  kern<<<static_cast<unsigned>(grid), C::THREADS, C::SMEM_BYTES, s>>>(m0, m1, mc0, mc1, mo0, mo1,
                                                                       p);
  return launch_status();
}
// dq = bf16(scale * acc), acc fp32 [B*H, T, D] contiguous; one thread per 8
// elements (two 16-byte loads, one 16-byte store)
template <int D>
__global__ void __launch_bounds__(256) smat_dq_finish_kernel(const float* __restrict__ acc,
                                                             __nv_bfloat16* __restrict__ dq,
                                                             int64_t sb, int64_t sh, int64_t st,
                                                             int H, int T, int64_t n8,
                                                             float scale) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const int64_t row = i / (D / 8);
  const int c = static_cast<int>(i % (D / 8)) * 8;
  const int64_t bh = row / T;
  const int t = static_cast<int>(row % T);
  const float4* a = reinterpret_cast<const float4*>(acc + row * D + c);
  const float4 x = __ldcs(a), y = __ldcs(a + 1);
  *reinterpret_cast<uint4*>(dq + (bh / H) * sb + (bh % H) * sh + t * st + c) =
      make_uint4(pack_bf16(x.x * scale, x.y * scale), pack_bf16(x.z * scale, x.w * scale),
                 pack_bf16(y.x * scale, y.y * scale), pack_bf16(y.z * scale, y.w * scale));
}

// D = 64 with 64-row blocks: 64-row chunks, two CTAs per SM; otherwise
// 128-row chunks.  The choice depends on (D, block) only, so launches with
// and without a work list chunk alike.
template <bool DKDV, int D>
int bwd_tc(const TArg& r0, const TArg& r1, const TArg& c0, const TArg& c1, const float* lse,
           const float* delta, const TArg& out0, const TArg* out1, int B, int H, int T,
           const int32_t* indptr, const int32_t* indices, const uint8_t* kind, int nblocks,
           int64_t nnzb, int block, float scale, const Work& work, const MdPattern& md,
           int32_t* err, cudaStream_t s) {
  if constexpr (D == 64) {
    if (block == 64)
      return bwd_tc_cn<DKDV, 64, 64>(r0, r1, c0, c1, lse, delta, out0, out1, B, H, T, indptr,
                                     indices, kind, nblocks, nnzb, block, scale, work, md, err, s);
  }
  return bwd_tc_cn<DKDV, D, 128>(r0, r1, c0, c1, lse, delta, out0, out1, B, H, T, indptr, indices,
                                 kind, nblocks, nnzb, block, scale, work, md, err, s);
}

}  // namespace

// ====================================================================== C ABI
extern "C" {

int smat_abi_version(void) { return 6; }

const char* smat_status_string(int status) {
  switch (status) {
    case SMAT_OK: return "ok";
    case SMAT_ERR_BAD_SHAPE: return "bad shape";
    case SMAT_ERR_UNSUPPORTED_D: return "unsupported head dimension D";
    case SMAT_ERR_UNSUPPORTED_BLOCK: return "unsupported block size";
    case SMAT_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case SMAT_ERR_BAD_STRIDE: return "bad stride";
    case SMAT_ERR_BAD_ALIGNMENT: return "bad alignment (bf16 needs 16-byte aligned rows)";
    case SMAT_ERR_CSR_INVALID: return "invalid block CSR";
    case SMAT_ERR_NULL_POINTER: return "null pointer";
    case SMAT_ERR_LAUNCH: return "kernel launch failed";
    case SMAT_ERR_NO_DEVICE: return "no supported device (sm_100 required)";
    case SMAT_ERR_TMA_DESCRIPTOR: return "TMA descriptor rejected";
    case SMAT_ERR_ROW_TOO_LONG: return "layout row longer than the kernels support";
    case SMAT_ERR_CAPACITY: return "output capacity too small";
    case SMAT_ERR_SCRATCH_LIMIT:
      return "B*H*T exceeds the fixed scratch of smat_bwd_noalloc (SMAT_NOALLOC_MAX_ROWS)";
    case SMAT_ERR_BAD_PATTERN: return "invalid M^(d) pattern (fields, table sizes or C)";
    case SMAT_ERR_CAPTURE:
      return "one-time set-up refused during stream capture (make the first call outside it)";
  }
  return "unknown status";
}

int smat_device_supported(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) {
    cudaGetLastError();
    return SMAT_ERR_NO_DEVICE;
  }
  return (major == 10 && minor == 0) ? SMAT_OK : SMAT_ERR_NO_DEVICE;
}

// ---------------------------------------------------------------- layouts
int smat_layout_build_block(int T, int block, int window, int stride, int n_sink, int32_t* indptr,
                            int32_t* indices, uint8_t* kind, int64_t capacity, int64_t* nnzb_out) {
  if (T < 1 || block < 1 || window < 0 || stride < 0 || n_sink < 0) return SMAT_ERR_BAD_SHAPE;
  if (!nnzb_out) return SMAT_ERR_NULL_POINTER;
  const int nb = (T + block - 1) / block;
  int64_t n = 0;
  if (indptr) indptr[0] = 0;
  for (int qb = 0; qb < nb; ++qb) {
    const int lo = std::max(0, qb - window);
    for (int kb = 0; kb <= qb; ++kb) {
      const bool far = kb < n_sink || (stride > 0 && kb % stride == stride - 1);
      if (kb < lo && !far) continue;
      if (indices) {
        if (n >= capacity || !kind) return SMAT_ERR_CAPACITY;
        indices[n] = kb;
        kind[n] = kb == qb ? SMAT_TILE_CAUSAL : SMAT_TILE_FULL;
      }
      ++n;
    }
    if (indptr) indptr[qb + 1] = static_cast<int32_t>(n);
    if (n > (1LL << 31) - 1) return SMAT_ERR_CAPACITY;
  }
  *nnzb_out = n;
  return SMAT_OK;
}

int smat_layout_transpose(int nblocks, const int32_t* indptr, const int32_t* indices,
                          const uint8_t* kind, int32_t* t_indptr, int32_t* t_indices,
                          uint8_t* t_kind) {
  if (nblocks < 0) return SMAT_ERR_BAD_SHAPE;
  if (!indptr || !t_indptr) return SMAT_ERR_NULL_POINTER;
  const int64_t nnz = indptr[nblocks];
  if (nnz > 0 && (!indices || !kind || !t_indices || !t_kind)) return SMAT_ERR_NULL_POINTER;
  std::vector<int64_t> count(static_cast<size_t>(nblocks) + 1, 0);
  for (int64_t e = 0; e < nnz; ++e) {
    const int32_t c = indices[e];
    if (c < 0 || c >= nblocks) return SMAT_ERR_CSR_INVALID;
    ++count[c + 1];
  }
  for (int i = 0; i < nblocks; ++i) count[i + 1] += count[i];
  for (int i = 0; i <= nblocks; ++i) t_indptr[i] = static_cast<int32_t>(count[i]);
  // rows are visited in ascending order, so each column list comes out ascending
  for (int r = 0; r < nblocks; ++r) {
    if (indptr[r + 1] < indptr[r]) return SMAT_ERR_CSR_INVALID;
    for (int64_t e = indptr[r]; e < indptr[r + 1]; ++e) {
      const int64_t dst = count[indices[e]]++;
      t_indices[dst] = r;
      t_kind[dst] = kind[e];
    }
  }
  return SMAT_OK;
}

int smat_layout_validate(int nblocks, int64_t nnzb, const int32_t* indptr, const int32_t* indices,
                         const uint8_t* kind, int transposed, int32_t* max_row_out) {
  return validate_layout(nblocks, nnzb, indptr, indices, kind, transposed, false, max_row_out);
}

int smat_layout_validate_pattern(int nblocks, int64_t nnzb, const int32_t* indptr,
                                 const int32_t* indices, const uint8_t* kind, int transposed,
                                 int32_t* max_row_out) {
  return validate_layout(nblocks, nnzb, indptr, indices, kind, transposed, true, max_row_out);
}

// ---------------------------------------------------------------- M^(d) masks
int smat_pattern_tables(int B, int N0, const int64_t* C_indptr, const int32_t* C_indices,
                        uint32_t* row_bits, int row_words, uint32_t* col_bits, int col_words) {
  if (B < 1 || N0 < 1) return SMAT_ERR_BAD_PATTERN;
  if (static_cast<int64_t>(row_words) < (static_cast<int64_t>(N0) + 63) / 32 ||
      static_cast<int64_t>(col_words) < (static_cast<int64_t>(B) + 63) / 32)
    return SMAT_ERR_BAD_PATTERN;
  if (!C_indptr || !row_bits || !col_bits) return SMAT_ERR_NULL_POINTER;
  if (C_indptr[0] != 0) return SMAT_ERR_BAD_PATTERN;
  for (int r = 0; r < B; ++r)
    if (C_indptr[r + 1] < C_indptr[r]) return SMAT_ERR_BAD_PATTERN;
  if (C_indptr[B] > 0 && !C_indices) return SMAT_ERR_NULL_POINTER;
  const int64_t rbits = 32LL * row_words, cbits = 32LL * col_words;
  std::memset(row_bits, 0, sizeof(uint32_t) * static_cast<size_t>(B) * row_words);
  std::memset(col_bits, 0, sizeof(uint32_t) * static_cast<size_t>(N0) * col_words);
  for (int r = 0; r < B; ++r) {
    for (int64_t e = C_indptr[r]; e < C_indptr[r + 1]; ++e) {
      const int32_t c = C_indices[e];
      if (c < 0 || c >= N0) return SMAT_ERR_BAD_PATTERN;
      uint32_t* rw = row_bits + static_cast<int64_t>(r) * row_words;
      for (int64_t t = c; t < rbits; t += N0) rw[t >> 5] |= 1u << (t & 31);
      uint32_t* cw = col_bits + static_cast<int64_t>(c) * col_words;
      for (int64_t t = r; t < cbits; t += B) cw[t >> 5] |= 1u << (t & 31);
    }
  }
  return SMAT_OK;
}

int smat_layout_build_pattern(int T, int block, int family, int n, int n_P, int c_all_ones,
                              int32_t* indptr, int32_t* indices, uint8_t* kind, int64_t capacity,
                              int64_t* nnzb_out) {
  if (T < 1 || block < 1) return SMAT_ERR_BAD_SHAPE;
  if ((family != SMAT_FAMILY_GEOMETRIC && family != SMAT_FAMILY_ENDPOINT) || n_P < 0 || n < n_P ||
      n > T)
    return SMAT_ERR_BAD_PATTERN;
  if (!nnzb_out) return SMAT_ERR_NULL_POINTER;
  const int nb = (T + block - 1) / block;
  const bool pow2 = (block & (block - 1)) == 0;
  int64_t cnt = 0;
  if (indptr) indptr[0] = 0;
  for (int qb = 0; qb < nb; ++qb) {
    const int r0 = qb * block, r1 = std::min(T, r0 + block);
    for (int kb = 0; kb <= qb; ++kb) {
      const int c0 = kb * block, c1 = std::min(T, c0 + block);
      uint8_t k;
      if (r1 <= n) {          // landmark rows: the lower triangle or the subset relation
        if (family == SMAT_FAMILY_GEOMETRIC) {
          k = kb == qb ? SMAT_TILE_CAUSAL : SMAT_TILE_FULL;
        } else {
          // i = qb block + a, j = kb block + b: j within i iff kb within qb and b within a
          if (pow2 && (kb & ~qb) != 0) continue;
          k = SMAT_TILE_PATTERN;
        }
      } else if (r0 >= n) {   // recent rows: global, long-range and recent columns
        if (kb == qb) {
          k = SMAT_TILE_CAUSAL;
        } else {
          const int g0 = std::max(c0, n_P), g1 = std::min(c1, n);
          k = (g0 >= g1 || c_all_ones) ? SMAT_TILE_FULL : SMAT_TILE_PATTERN;
        }
      } else {                // rows straddle n
        k = SMAT_TILE_PATTERN;
      }
      if (indices) {
        if (cnt >= capacity || !kind) return SMAT_ERR_CAPACITY;
        indices[cnt] = kb;
        kind[cnt] = k;
      }
      ++cnt;
    }
    if (cnt > (1LL << 31) - 1) return SMAT_ERR_CAPACITY;
    if (indptr) indptr[qb + 1] = static_cast<int32_t>(cnt);
  }
  *nnzb_out = cnt;
  return SMAT_OK;
}

int smat_pattern_mask_rows(const smat_pattern_t* pattern, int T, int row_lo, int row_hi,
                           uint8_t* out) {
  MdPattern md;
  int rc;
  if (T < 1) return SMAT_ERR_BAD_SHAPE;
  if ((rc = check_pattern(pattern, T, true, &md))) return rc;
  if (row_lo < 0 || row_hi < row_lo || row_hi > T) return SMAT_ERR_BAD_SHAPE;
  if (!out && row_hi > row_lo) return SMAT_ERR_NULL_POINTER;
  for (int i = row_lo; i < row_hi; ++i) {
    uint8_t* o = out + static_cast<int64_t>(i - row_lo) * T;
    for (int j0 = 0; j0 < T; j0 += 32) {
      const uint32_t w = md_row_word(md, T, i, j0);
      for (int c = 0; c < 32 && j0 + c < T; ++c) o[j0 + c] = (w >> c) & 1u;
    }
  }
  return SMAT_OK;
}

int smat_pattern_mask_cols(const smat_pattern_t* pattern, int T, int col_lo, int col_hi,
                           uint8_t* out) {
  MdPattern md;
  int rc;
  if (T < 1) return SMAT_ERR_BAD_SHAPE;
  if ((rc = check_pattern(pattern, T, true, &md))) return rc;
  if (col_lo < 0 || col_hi < col_lo || col_hi > T) return SMAT_ERR_BAD_SHAPE;
  if (!out && col_hi > col_lo) return SMAT_ERR_NULL_POINTER;
  for (int j = col_lo; j < col_hi; ++j) {
    uint8_t* o = out + static_cast<int64_t>(j - col_lo) * T;
    for (int i0 = 0; i0 < T; i0 += 32) {
      const uint32_t w = md_col_word(md, T, j, i0);
      for (int c = 0; c < 32 && i0 + c < T; ++c) o[i0 + c] = (w >> c) & 1u;
    }
  }
  return SMAT_OK;
}

// ---------------------------------------------------------------- forward
}  // extern "C"

namespace {

int fwd_impl(int dtype, const void* q, const int64_t* q_stride, const void* k,
             const int64_t* k_stride, const void* v, const int64_t* v_stride, void* o,
             const int64_t* o_stride, float* lse, int B, int H, int T, int D,
             const int32_t* indptr, const int32_t* indices, const uint8_t* kind, int nblocks,
             int64_t nnzb, int block, int max_row, float scale, const Work& work,
             const MdPattern& md, int32_t* err_word, void* stream) {
  int rc;
  if (!q_stride || !k_stride || !v_stride || !o_stride) return SMAT_ERR_NULL_POINTER;
  if ((rc = check_common(dtype, B, H, T, D, nblocks, block))) return rc;
  if ((rc = check_work(work))) return rc;
  const TArg tq = targ(q, q_stride), tk = targ(k, k_stride), tv = targ(v, v_stride),
             to = targ(o, o_stride);
  for (const TArg* t : {&tq, &tk, &tv, &to})
    if ((rc = check_tensor(*t, dtype))) return rc;
  if (!lse) return SMAT_ERR_NULL_POINTER;
  if ((rc = check_layout_args(indptr, indices, kind, nnzb, max_row, block))) return rc;
  if (!std::isfinite(scale) || scale <= 0.f) return SMAT_ERR_BAD_SHAPE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == SMAT_DTYPE_BF16) {
    // D = 64: one tile per CTA; 64-key chunks and four CTAs per SM with
    // 64-row blocks, else 128-key chunks and two (with or without a work
    // list, so that both launches group a tile's keys into the same chunks)
    if (D == 64 && block == 64)
      return fwd_tc<64, 1, 64>(tq, tk, tv, to, lse, B, H, T, indptr, indices, kind, nblocks,
                               nnzb, block, scale, work, md, err_word, s);
    if (D == 64)
      return fwd_tc<64, 1>(tq, tk, tv, to, lse, B, H, T, indptr, indices, kind, nblocks, nnzb,
                           block, scale, work, md, err_word, s);
    return fwd_tc<128, 2>(tq, tk, tv, to, lse, B, H, T, indptr, indices, kind, nblocks, nnzb,
                          block, scale, work, md, err_word, s);
  }
  SimtParams p = simt_params(B, H, T, block, scale, indptr, indices, kind, nblocks, nnzb, err_word,
                             work, 2, md);
  p.q = static_cast<const float*>(q);
  p.k = static_cast<const float*>(k);
  p.v = static_cast<const float*>(v);
  p.out0 = static_cast<float*>(o);
  p.out1 = lse;
  set3(p.q_s, tq);
  set3(p.k_s, tk);
  set3(p.v_s, tv);
  set3(p.out0_s, to);
  return dispatch_simt_d<FwdSimt>(D, p, T, work.n, B * H, s);
}

// ---------------------------------------------------------------- backward
int pre_impl(int dtype, const void* o, const int64_t* o_stride, const void* dout,
             const int64_t* do_stride, float* delta, int B, int H, int T, int D, int row_lo,
             int row_hi, void* stream) {
  int rc;
  if (!o_stride || !do_stride) return SMAT_ERR_NULL_POINTER;
  if ((rc = check_common(dtype, B, H, T, D, (T + 63) / 64, 64))) return rc;
  if (row_lo < 0 || row_hi < row_lo || row_hi > T) return SMAT_ERR_BAD_SHAPE;
  const TArg to = targ(o, o_stride), td = targ(dout, do_stride);
  for (const TArg* t : {&to, &td})
    if ((rc = check_tensor(*t, dtype))) return rc;
  if (!delta) return SMAT_ERR_NULL_POINTER;
  if (dtype == SMAT_DTYPE_F32 && (to.sb % 4 || to.sh % 4 || to.st % 4 || td.sb % 4 || td.sh % 4 ||
                                  td.st % 4 || reinterpret_cast<uintptr_t>(o) % 16 ||
                                  reinterpret_cast<uintptr_t>(dout) % 16))
    return SMAT_ERR_BAD_ALIGNMENT;
  const int n_rows = row_hi - row_lo;
  if (n_rows == 0) return SMAT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t rows = static_cast<int64_t>(B) * H * n_rows;
  const int elem = dtype == SMAT_DTYPE_BF16 ? 2 : 4;
  const int lpr = D * elem / 16;
  const int64_t threads = rows * lpr;
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
#define SMAT_PRE(TY, DD)                                                                        \
  do {                                                                                          \
    if (threads < (int64_t{1} << 31))                                                           \
      smat_bwd_pre_kernel<TY, DD, uint32_t><<<grid, 256, 0, s>>>(                               \
          static_cast<const TY*>(o), static_cast<const TY*>(dout), delta, to.sb, to.sh, to.st,  \
          td.sb, td.sh, td.st, H, T, row_lo, n_rows, rows);                                     \
    else                                                                                        \
      smat_bwd_pre_kernel<TY, DD, int64_t><<<grid, 256, 0, s>>>(                                \
          static_cast<const TY*>(o), static_cast<const TY*>(dout), delta, to.sb, to.sh, to.st,  \
          td.sb, td.sh, td.st, H, T, row_lo, n_rows, rows);                                     \
  } while (0)
  if (dtype == SMAT_DTYPE_BF16) {
    if (D == 64) SMAT_PRE(__nv_bfloat16, 64);
    else SMAT_PRE(__nv_bfloat16, 128);
  } else {
    if (D == 32) SMAT_PRE(float, 32);
    else if (D == 64) SMAT_PRE(float, 64);
    else SMAT_PRE(float, 128);
  }
#undef SMAT_PRE
  return launch_status();
}

// launch == false runs the host-side checks only (smat_bwd checks all three
// passes before it launches the first)
int dkdv_impl(int dtype, const void* q, const int64_t* q_stride, const void* k,
              const int64_t* k_stride, const void* v, const int64_t* v_stride, const void* dout,
              const int64_t* do_stride, const float* lse, const float* delta, void* dk,
              const int64_t* dk_stride, void* dv, const int64_t* dv_stride, int B, int H, int T,
              int D, const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind,
              int nblocks, int64_t nnzb, int block, int t_max_row, float scale, const Work& work,
              const MdPattern& md, int32_t* err_word, void* stream, bool launch) {
  int rc;
  if (!q_stride || !k_stride || !v_stride || !do_stride || !dk_stride || !dv_stride)
    return SMAT_ERR_NULL_POINTER;
  if ((rc = check_common(dtype, B, H, T, D, nblocks, block))) return rc;
  if ((rc = check_work(work))) return rc;
  const TArg tq = targ(q, q_stride), tk = targ(k, k_stride), tv = targ(v, v_stride),
             td = targ(dout, do_stride), tdk = targ(dk, dk_stride), tdv = targ(dv, dv_stride);
  for (const TArg* t : {&tq, &tk, &tv, &td, &tdk, &tdv})
    if ((rc = check_tensor(*t, dtype))) return rc;
  if (!lse || !delta) return SMAT_ERR_NULL_POINTER;
  if ((rc = check_layout_args(t_indptr, t_indices, t_kind, nnzb, t_max_row, block))) return rc;
  if (!std::isfinite(scale) || scale <= 0.f) return SMAT_ERR_BAD_SHAPE;
  if (!launch) return SMAT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == SMAT_DTYPE_BF16) {
    if (D == 64)
      return bwd_tc<true, 64>(tk, tv, tq, td, lse, delta, tdk, &tdv, B, H, T, t_indptr, t_indices,
                              t_kind, nblocks, nnzb, block, scale, work, md, err_word, s);
    return bwd_tc<true, 128>(tk, tv, tq, td, lse, delta, tdk, &tdv, B, H, T, t_indptr, t_indices,
                             t_kind, nblocks, nnzb, block, scale, work, md, err_word, s);
  }
  SimtParams p = simt_params(B, H, T, block, scale, t_indptr, t_indices, t_kind, nblocks, nnzb,
                             err_word, work, 1, md);
  p.q = static_cast<const float*>(q);
  p.k = static_cast<const float*>(k);
  p.v = static_cast<const float*>(v);
  p.dout = static_cast<const float*>(dout);
  p.lse = lse;
  p.delta = delta;
  p.out0 = static_cast<float*>(dk);
  p.out1 = static_cast<float*>(dv);
  set3(p.q_s, tq);
  set3(p.k_s, tk);
  set3(p.v_s, tv);
  set3(p.do_s, td);
  set3(p.out0_s, tdk);
  set3(p.out1_s, tdv);
  return dispatch_simt_d<DkdvSimt>(D, p, T, work.n, B * H, s);
}

int dq_impl(int dtype, const void* q, const int64_t* q_stride, const void* k,
            const int64_t* k_stride, const void* v, const int64_t* v_stride, const void* dout,
            const int64_t* do_stride, const float* lse, const float* delta, void* dq,
            const int64_t* dq_stride, int B, int H, int T, int D, const int32_t* indptr,
            const int32_t* indices, const uint8_t* kind, int nblocks, int64_t nnzb, int block,
            int max_row, float scale, const Work& work, const MdPattern& md, int32_t* err_word,
            void* stream, bool launch) {
  int rc;
  if (!q_stride || !k_stride || !v_stride || !do_stride || !dq_stride) return SMAT_ERR_NULL_POINTER;
  if ((rc = check_common(dtype, B, H, T, D, nblocks, block))) return rc;
  if ((rc = check_work(work))) return rc;
  const TArg tq = targ(q, q_stride), tk = targ(k, k_stride), tv = targ(v, v_stride),
             td = targ(dout, do_stride), tdq = targ(dq, dq_stride);
  for (const TArg* t : {&tq, &tk, &tv, &td, &tdq})
    if ((rc = check_tensor(*t, dtype))) return rc;
  if (!lse || !delta) return SMAT_ERR_NULL_POINTER;
  if ((rc = check_layout_args(indptr, indices, kind, nnzb, max_row, block))) return rc;
  if (!std::isfinite(scale) || scale <= 0.f) return SMAT_ERR_BAD_SHAPE;
  if (!launch) return SMAT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == SMAT_DTYPE_BF16) {
    if (D == 64)
      return bwd_tc<false, 64>(tq, td, tk, tv, lse, delta, tdq, nullptr, B, H, T, indptr, indices,
                               kind, nblocks, nnzb, block, scale, work, md, err_word, s);
    return bwd_tc<false, 128>(tq, td, tk, tv, lse, delta, tdq, nullptr, B, H, T, indptr, indices,
                              kind, nblocks, nnzb, block, scale, work, md, err_word, s);
  }
  SimtParams p = simt_params(B, H, T, block, scale, indptr, indices, kind, nblocks, nnzb, err_word,
                             work, 1, md);
  p.q = static_cast<const float*>(q);
  p.k = static_cast<const float*>(k);
  p.v = static_cast<const float*>(v);
  p.dout = static_cast<const float*>(dout);
  p.lse = lse;
  p.delta = delta;
  p.out0 = static_cast<float*>(dq);
  set3(p.q_s, tq);
  set3(p.k_s, tk);
  set3(p.v_s, tv);
  set3(p.do_s, td);
  set3(p.out0_s, tdq);
  return dispatch_simt_d<DqSimt>(D, p, T, work.n, B * H, s);
}

// preprocess, dK/dV and dQ; every pass is checked before the first launches
int bwd_all(int dtype, const void* q, const int64_t* q_stride, const void* k,
            const int64_t* k_stride, const void* v, const int64_t* v_stride, const void* o,
            const int64_t* o_stride, const void* dout, const int64_t* do_stride, const float* lse,
            float* delta, void* dq, const int64_t* dq_stride, void* dk, const int64_t* dk_stride,
            void* dv, const int64_t* dv_stride, int B, int H, int T, int D,
            const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
            const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind, int nblocks,
            int64_t nnzb, int block, int max_row, int t_max_row, float scale,
            const MdPattern& md, int32_t* err_word, void* stream) {
  int rc;
  for (int pass = 0; pass < 2; ++pass) {
    const bool launch = pass == 1;
    if (launch && (rc = pre_impl(dtype, o, o_stride, dout, do_stride, delta, B, H, T, D, 0, T,
                                 stream)))
      return rc;
    if ((rc = dkdv_impl(dtype, q, q_stride, k, k_stride, v, v_stride, dout, do_stride, lse, delta,
                        dk, dk_stride, dv, dv_stride, B, H, T, D, t_indptr, t_indices, t_kind,
                        nblocks, nnzb, block, t_max_row, scale, kAllTiles, md, err_word, stream,
                        launch)))
      return rc;
    if ((rc = dq_impl(dtype, q, q_stride, k, k_stride, v, v_stride, dout, do_stride, lse, delta,
                      dq, dq_stride, B, H, T, D, indptr, indices, kind, nblocks, nnzb, block,
                      max_row, scale, kAllTiles, md, err_word, stream, launch)))
      return rc;
  }
  return SMAT_OK;
}

// The fused backward (bf16, D = 128): dK, dV and an fp32 dQ accumulator from
// one kernel over the transposed CSR, then dQ = bf16(scale * acc).
bool fused_dq_applies(int dtype, int D) { return dtype == SMAT_DTYPE_BF16 && D == 128; }

int check_dq_acc(const float* dq_acc, int64_t dq_acc_floats, int B, int H, int T, int D) {
  if (!dq_acc) return SMAT_ERR_NULL_POINTER;
  if (reinterpret_cast<uintptr_t>(dq_acc) % 16) return SMAT_ERR_BAD_ALIGNMENT;
  if (dq_acc_floats < static_cast<int64_t>(B) * H * T * D) return SMAT_ERR_BAD_SHAPE;
  return SMAT_OK;
}

int dkdv_dq_impl(int dtype, const void* q, const int64_t* q_stride, const void* k,
                 const int64_t* k_stride, const void* v, const int64_t* v_stride,
                 const void* dout, const int64_t* do_stride, const float* lse, const float* delta,
                 float* dq_acc, int64_t dq_acc_floats, void* dk, const int64_t* dk_stride,
                 void* dv, const int64_t* dv_stride, int B, int H, int T, int D,
                 const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind,
                 int nblocks, int64_t nnzb, int block, int t_max_row, float scale,
                 const MdPattern& md, int32_t* err_word, void* stream, bool launch) {
  int rc;
  // the dK/dV checks cover every argument but the accumulator
  if ((rc = dkdv_impl(dtype, q, q_stride, k, k_stride, v, v_stride, dout, do_stride, lse, delta,
                      dk, dk_stride, dv, dv_stride, B, H, T, D, t_indptr, t_indices, t_kind,
                      nblocks, nnzb, block, t_max_row, scale, kAllTiles, md, err_word, stream,
                      false)))
    return rc;
  if (dtype != SMAT_DTYPE_BF16) return SMAT_ERR_UNSUPPORTED_DTYPE;
  if (D != 128) return SMAT_ERR_UNSUPPORTED_D;
  if ((rc = check_dq_acc(dq_acc, dq_acc_floats, B, H, T, D))) return rc;
  if (!launch) return SMAT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(dq_acc, 0, sizeof(float) * static_cast<size_t>(B) * H * T * D, s) !=
      cudaSuccess)
    return SMAT_ERR_LAUNCH;
  const TArg tq = targ(q, q_stride), tk = targ(k, k_stride), tv = targ(v, v_stride),
             td = targ(dout, do_stride), tdk = targ(dk, dk_stride), tdv = targ(dv, dv_stride);
  return bwd_tc_cn<true, 128, 128, true>(tk, tv, tq, td, lse, delta, tdk, &tdv, B, H, T,
                                         t_indptr, t_indices, t_kind, nblocks, nnzb, block, scale,
                                         kAllTiles, md, err_word, s, dq_acc);
}

int dq_finish_impl(int dtype, const float* dq_acc, int64_t dq_acc_floats, void* dq,
                   const int64_t* dq_stride, int B, int H, int T, int D, float scale,
                   void* stream, bool launch) {
  int rc;
  if (!dq_stride) return SMAT_ERR_NULL_POINTER;
  if ((rc = check_common(dtype, B, H, T, D, (T + 63) / 64, 64))) return rc;
  if (dtype != SMAT_DTYPE_BF16) return SMAT_ERR_UNSUPPORTED_DTYPE;
  if (D != 128 && D != 64) return SMAT_ERR_UNSUPPORTED_D;
  const TArg tdq = targ(dq, dq_stride);
  if ((rc = check_tensor(tdq, dtype))) return rc;
  if ((rc = check_dq_acc(dq_acc, dq_acc_floats, B, H, T, D))) return rc;
  if (!std::isfinite(scale) || scale <= 0.f) return SMAT_ERR_BAD_SHAPE;
  if (!launch) return SMAT_OK;
  const int64_t n8 = static_cast<int64_t>(B) * H * T * (D / 8);
  if (n8 == 0) return SMAT_OK;
  const unsigned grid = static_cast<unsigned>((n8 + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* out = static_cast<__nv_bfloat16*>(dq);
  if (D == 128)
    smat_dq_finish_kernel<128><<<grid, 256, 0, s>>>(dq_acc, out, tdq.sb, tdq.sh, tdq.st, H, T, n8,
                                                    scale);
  else
    smat_dq_finish_kernel<64><<<grid, 256, 0, s>>>(dq_acc, out, tdq.sb, tdq.sh, tdq.st, H, T, n8,
                                                   scale);
  return launch_status();
}

// preprocess, fused dK/dV/dQ-accumulate, dQ finish; every pass is checked
// before the first launches.  Layouts the fused kernel does not cover run the
// two-kernel backward (dq_acc unused).
int bwd_acc_all(int dtype, const void* q, const int64_t* q_stride, const void* k,
                const int64_t* k_stride, const void* v, const int64_t* v_stride, const void* o,
                const int64_t* o_stride, const void* dout, const int64_t* do_stride,
                const float* lse, float* delta, void* dq, const int64_t* dq_stride, void* dk,
                const int64_t* dk_stride, void* dv, const int64_t* dv_stride, int B, int H, int T,
                int D, const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind,
                int nblocks, int64_t nnzb, int block, int max_row, int t_max_row,
                const MdPattern& md, float* dq_acc, int64_t dq_acc_floats, float scale,
                int32_t* err_word, void* stream) {
  if (!fused_dq_applies(dtype, D))
    return bwd_all(dtype, q, q_stride, k, k_stride, v, v_stride, o, o_stride, dout, do_stride, lse,
                   delta, dq, dq_stride, dk, dk_stride, dv, dv_stride, B, H, T, D, indptr,
                   indices, kind, t_indptr, t_indices, t_kind, nblocks, nnzb, block, max_row,
                   t_max_row, scale, md, err_word, stream);
  int rc;
  for (int pass = 0; pass < 2; ++pass) {
    const bool launch = pass == 1;
    // the forward CSR is not read, but it is the caller's layout: check it too
    if (!launch && (rc = dq_impl(dtype, q, q_stride, k, k_stride, v, v_stride, dout, do_stride,
                                 lse, delta, dq, dq_stride, B, H, T, D, indptr, indices, kind,
                                 nblocks, nnzb, block, max_row, scale, kAllTiles, md, err_word,
                                 stream, false)))
      return rc;
    if (launch && (rc = pre_impl(dtype, o, o_stride, dout, do_stride, delta, B, H, T, D, 0, T,
                                 stream)))
      return rc;
    if ((rc = dkdv_dq_impl(dtype, q, q_stride, k, k_stride, v, v_stride, dout, do_stride, lse,
                           delta, dq_acc, dq_acc_floats, dk, dk_stride, dv, dv_stride, B, H, T, D,
                           t_indptr, t_indices, t_kind, nblocks, nnzb, block, t_max_row, scale,
                           md, err_word, stream, launch)))
      return rc;
    if ((rc = dq_finish_impl(dtype, dq_acc, dq_acc_floats, dq, dq_stride, B, H, T, D, scale,
                             stream, launch)))
      return rc;
  }
  return SMAT_OK;
}

}  // namespace

extern "C" {

int smat_fwd(int dtype, const void* q, const int64_t* q_stride, const void* k,
             const int64_t* k_stride, const void* v, const int64_t* v_stride, void* o,
             const int64_t* o_stride, float* lse, int B, int H, int T, int D,
             const int32_t* indptr, const int32_t* indices, const uint8_t* kind, int nblocks,
             int64_t nnzb, int block, int max_row, float scale, int32_t* err_word,
             void* stream) {
  return fwd_impl(dtype, q, q_stride, k, k_stride, v, v_stride, o, o_stride, lse, B, H, T, D,
                  indptr, indices, kind, nblocks, nnzb, block, max_row, scale, kAllTiles, kNoPattern,
                  err_word, stream);
}

int smat_fwd_tiles(int dtype, const void* q, const int64_t* q_stride, const void* k,
                   const int64_t* k_stride, const void* v, const int64_t* v_stride, void* o,
                   const int64_t* o_stride, float* lse, int B, int H, int T, int D,
                   const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                   int nblocks, int64_t nnzb, int block, int max_row, float scale,
                   const int32_t* work, int n_work, int32_t* err_word, void* stream) {
  if (!work && n_work == 0) return SMAT_OK;
  if (!work) return SMAT_ERR_NULL_POINTER;
  return fwd_impl(dtype, q, q_stride, k, k_stride, v, v_stride, o, o_stride, lse, B, H, T, D,
                  indptr, indices, kind, nblocks, nnzb, block, max_row, scale, Work{work, n_work}, kNoPattern,
                  err_word, stream);
}

int smat_bwd_preprocess(int dtype, const void* o, const int64_t* o_stride, const void* dout,
                        const int64_t* do_stride, float* delta, int B, int H, int T, int D,
                        void* stream) {
  return pre_impl(dtype, o, o_stride, dout, do_stride, delta, B, H, T, D, 0, T, stream);
}

int smat_bwd_preprocess_rows(int dtype, const void* o, const int64_t* o_stride, const void* dout,
                             const int64_t* do_stride, float* delta, int B, int H, int T, int D,
                             int row_lo, int row_hi, void* stream) {
  return pre_impl(dtype, o, o_stride, dout, do_stride, delta, B, H, T, D, row_lo, row_hi, stream);
}

int smat_bwd_dkdv(int dtype, const void* q, const int64_t* q_stride, const void* k,
                  const int64_t* k_stride, const void* v, const int64_t* v_stride,
                  const void* dout, const int64_t* do_stride, const float* lse,
                  const float* delta, void* dk, const int64_t* dk_stride, void* dv,
                  const int64_t* dv_stride, int B, int H, int T, int D, const int32_t* t_indptr,
                  const int32_t* t_indices, const uint8_t* t_kind, int nblocks, int64_t nnzb,
                  int block, int t_max_row, float scale, int32_t* err_word, void* stream) {
  return dkdv_impl(dtype, q, q_stride, k, k_stride, v, v_stride, dout, do_stride, lse, delta, dk,
                   dk_stride, dv, dv_stride, B, H, T, D, t_indptr, t_indices, t_kind, nblocks,
                   nnzb, block, t_max_row, scale, kAllTiles, kNoPattern, err_word, stream, true);
}

int smat_bwd_dkdv_tiles(int dtype, const void* q, const int64_t* q_stride, const void* k,
                        const int64_t* k_stride, const void* v, const int64_t* v_stride,
                        const void* dout, const int64_t* do_stride, const float* lse,
                        const float* delta, void* dk, const int64_t* dk_stride, void* dv,
                        const int64_t* dv_stride, int B, int H, int T, int D,
                        const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind,
                        int nblocks, int64_t nnzb, int block, int t_max_row, float scale,
                        const int32_t* work, int n_work, int32_t* err_word, void* stream) {
  if (!work && n_work == 0) return SMAT_OK;
  if (!work) return SMAT_ERR_NULL_POINTER;
  return dkdv_impl(dtype, q, q_stride, k, k_stride, v, v_stride, dout, do_stride, lse, delta, dk,
                   dk_stride, dv, dv_stride, B, H, T, D, t_indptr, t_indices, t_kind, nblocks,
                   nnzb, block, t_max_row, scale, Work{work, n_work}, kNoPattern, err_word, stream, true);
}

int smat_bwd_dq(int dtype, const void* q, const int64_t* q_stride, const void* k,
                const int64_t* k_stride, const void* v, const int64_t* v_stride, const void* dout,
                const int64_t* do_stride, const float* lse, const float* delta, void* dq,
                const int64_t* dq_stride, int B, int H, int T, int D, const int32_t* indptr,
                const int32_t* indices, const uint8_t* kind, int nblocks, int64_t nnzb,
                int block, int max_row, float scale, int32_t* err_word, void* stream) {
  return dq_impl(dtype, q, q_stride, k, k_stride, v, v_stride, dout, do_stride, lse, delta, dq,
                 dq_stride, B, H, T, D, indptr, indices, kind, nblocks, nnzb, block, max_row,
                 scale, kAllTiles, kNoPattern, err_word, stream, true);
}

int smat_bwd_dq_tiles(int dtype, const void* q, const int64_t* q_stride, const void* k,
                      const int64_t* k_stride, const void* v, const int64_t* v_stride,
                      const void* dout, const int64_t* do_stride, const float* lse,
                      const float* delta, void* dq, const int64_t* dq_stride, int B, int H, int T,
                      int D, const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                      int nblocks, int64_t nnzb, int block, int max_row, float scale,
                      const int32_t* work, int n_work, int32_t* err_word, void* stream) {
  if (!work && n_work == 0) return SMAT_OK;
  if (!work) return SMAT_ERR_NULL_POINTER;
  return dq_impl(dtype, q, q_stride, k, k_stride, v, v_stride, dout, do_stride, lse, delta, dq,
                 dq_stride, B, H, T, D, indptr, indices, kind, nblocks, nnzb, block, max_row,
                 scale, Work{work, n_work}, kNoPattern, err_word, stream, true);
}

int smat_bwd(int dtype, const void* q, const int64_t* q_stride, const void* k,
             const int64_t* k_stride, const void* v, const int64_t* v_stride, const void* o,
             const int64_t* o_stride, const void* dout, const int64_t* do_stride, const float* lse,
             float* delta, void* dq, const int64_t* dq_stride, void* dk, const int64_t* dk_stride,
             void* dv, const int64_t* dv_stride, int B, int H, int T, int D,
             const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
             const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind,
             int nblocks, int64_t nnzb, int block, int max_row, int t_max_row, float scale,
             int32_t* err_word, void* stream) {
  return bwd_all(dtype, q, q_stride, k, k_stride, v, v_stride, o, o_stride, dout, do_stride, lse,
                 delta, dq, dq_stride, dk, dk_stride, dv, dv_stride, B, H, T, D, indptr, indices,
                 kind, t_indptr, t_indices, t_kind, nblocks, nnzb, block, max_row, t_max_row,
                 scale, kNoPattern, err_word, stream);
}

int smat_bwd_dkdv_dq(int dtype, const void* q, const int64_t* q_stride, const void* k,
                     const int64_t* k_stride, const void* v, const int64_t* v_stride,
                     const void* dout, const int64_t* do_stride, const float* lse,
                     const float* delta, float* dq_acc, int64_t dq_acc_floats, void* dk,
                     const int64_t* dk_stride, void* dv, const int64_t* dv_stride, int B, int H,
                     int T, int D, const int32_t* t_indptr, const int32_t* t_indices,
                     const uint8_t* t_kind, int nblocks, int64_t nnzb, int block, int t_max_row,
                     float scale, int32_t* err_word, void* stream) {
  return dkdv_dq_impl(dtype, q, q_stride, k, k_stride, v, v_stride, dout, do_stride, lse, delta,
                      dq_acc, dq_acc_floats, dk, dk_stride, dv, dv_stride, B, H, T, D, t_indptr,
                      t_indices, t_kind, nblocks, nnzb, block, t_max_row, scale, kNoPattern,
                      err_word, stream, true);
}

int smat_bwd_dq_finish(int dtype, const float* dq_acc, int64_t dq_acc_floats, void* dq,
                       const int64_t* dq_stride, int B, int H, int T, int D, float scale,
                       void* stream) {
  return dq_finish_impl(dtype, dq_acc, dq_acc_floats, dq, dq_stride, B, H, T, D, scale, stream,
                        true);
}

int smat_bwd_acc(int dtype, const void* q, const int64_t* q_stride, const void* k,
                 const int64_t* k_stride, const void* v, const int64_t* v_stride, const void* o,
                 const int64_t* o_stride, const void* dout, const int64_t* do_stride,
                 const float* lse, float* delta, void* dq, const int64_t* dq_stride, void* dk,
                 const int64_t* dk_stride, void* dv, const int64_t* dv_stride, int B, int H,
                 int T, int D, const int32_t* indptr, const int32_t* indices,
                 const uint8_t* kind, const int32_t* t_indptr, const int32_t* t_indices,
                 const uint8_t* t_kind, int nblocks, int64_t nnzb, int block, int max_row,
                 int t_max_row, const smat_pattern_t* pattern, float* dq_acc,
                 int64_t dq_acc_floats, float scale, int32_t* err_word, void* stream) {
  MdPattern md = kNoPattern;
  if (pattern) {
    const int rc = check_pattern(pattern, T, true, &md);
    if (rc) return rc;
  }
  return bwd_acc_all(dtype, q, q_stride, k, k_stride, v, v_stride, o, o_stride, dout, do_stride,
                     lse, delta, dq, dq_stride, dk, dk_stride, dv, dv_stride, B, H, T, D, indptr,
                     indices, kind, t_indptr, t_indices, t_kind, nblocks, nnzb, block, max_row,
                     t_max_row, md, dq_acc, dq_acc_floats, scale, err_word, stream);
}

int smat_fwd_pattern(int dtype, const void* q, const int64_t* q_stride, const void* k,
                     const int64_t* k_stride, const void* v, const int64_t* v_stride, void* o,
                     const int64_t* o_stride, float* lse, int B, int H, int T, int D,
                     const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                     int nblocks, int64_t nnzb, int block, int max_row,
                     const smat_pattern_t* pattern, float scale, int32_t* err_word,
                     void* stream) {
  MdPattern md;
  const int rc = check_pattern(pattern, T, true, &md);
  if (rc) return rc;
  return fwd_impl(dtype, q, q_stride, k, k_stride, v, v_stride, o, o_stride, lse, B, H, T, D,
                  indptr, indices, kind, nblocks, nnzb, block, max_row, scale, kAllTiles, md,
                  err_word, stream);
}

int smat_bwd_pattern(int dtype, const void* q, const int64_t* q_stride, const void* k,
                     const int64_t* k_stride, const void* v, const int64_t* v_stride,
                     const void* o, const int64_t* o_stride, const void* dout,
                     const int64_t* do_stride, const float* lse, float* delta, void* dq,
                     const int64_t* dq_stride, void* dk, const int64_t* dk_stride, void* dv,
                     const int64_t* dv_stride, int B, int H, int T, int D,
                     const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                     const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind,
                     int nblocks, int64_t nnzb, int block, int max_row, int t_max_row,
                     const smat_pattern_t* pattern, float scale, int32_t* err_word,
                     void* stream) {
  MdPattern md;
  const int rc = check_pattern(pattern, T, true, &md);
  if (rc) return rc;
  return bwd_all(dtype, q, q_stride, k, k_stride, v, v_stride, o, o_stride, dout, do_stride, lse,
                 delta, dq, dq_stride, dk, dk_stride, dv, dv_stride, B, H, T, D, indptr, indices,
                 kind, t_indptr, t_indices, t_kind, nblocks, nnzb, block, max_row, t_max_row,
                 scale, md, err_word, stream);
}

}  // extern "C"
