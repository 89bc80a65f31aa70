// Row exchange kernels of the query-sharded path: gather listed token rows of
// two [B, H, T, D] tensors (K and V, or dK and dV) into a contiguous wire
// buffer, scatter a wire buffer back into rows, and add wire rows (partial
// sums from other GPUs) into rows in fp32.
//
// Wire format: wire row r holds [2][B][H][D] elements (tensor, batch, head,
// feature), so the rows sent to one peer are one contiguous range and an
// all-to-all can split the buffer by row counts.  Every thread moves one
// 16-byte vector; reads and writes are coalesced along D on both sides.
// All three are HBM-bound copies: 2 x B x H x D x elem bytes per row each way.
#include <cstdint>

#include "../../include/smat_b200.h"
#include "common.cuh"

namespace {

using namespace smat;

struct RowArgs {
  const uint8_t* a;  // tensor 0 (K / dK)
  const uint8_t* b;  // tensor 1 (V / dV)
  int64_t a_sb, a_sh, a_st, b_sb, b_sh, b_st;  // element strides
  int B, H, T, D, elem;
  const int64_t* rows;
  int64_t n_rows;
  int32_t* err;
};

// (wire row r, tensor t, b, h, 16-byte vector v) of global thread g
struct Unit {
  int64_t r;
  int t, b, h, v;
};

__device__ __forceinline__ bool unit_of(const RowArgs& p, int64_t g, Unit& u) {
  const int vpr = p.D * p.elem / 16;
  const int bh2 = 2 * p.B * p.H;
  const int64_t unit = g / vpr;
  if (unit >= p.n_rows * bh2) return false;
  u.v = static_cast<int>(g % vpr);
  u.r = unit / bh2;
  const int rem = static_cast<int>(unit % bh2);
  u.t = rem / (p.B * p.H);
  const int bh = rem % (p.B * p.H);
  u.b = bh / p.H;
  u.h = bh % p.H;
  return true;
}

__device__ __forceinline__ int64_t row_off(const RowArgs& p, const Unit& u, int64_t row) {
  const int64_t e = u.t ? u.b * p.b_sb + u.h * p.b_sh + row * p.b_st
                        : u.b * p.a_sb + u.h * p.a_sh + row * p.a_st;
  return e * p.elem + u.v * 16;
}

__device__ __forceinline__ int64_t wire_off(const RowArgs& p, int64_t r, const Unit& u) {
  const int64_t unit = (r * 2 + u.t) * p.B * p.H + static_cast<int64_t>(u.b) * p.H + u.h;
  return unit * p.D * p.elem + u.v * 16;
}

__device__ __forceinline__ bool row_ok(const RowArgs& p, int64_t row) {
  if (row >= 0 && row < p.T) return true;
  if (p.err) atomicOr(p.err, DEV_ERR_BAD_WORK);
  return false;
}

__global__ void __launch_bounds__(256) rows_pack_kernel(const RowArgs p, uint8_t* wire) {
  const int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  Unit u;
  if (!unit_of(p, g, u)) return;
  const int64_t row = __ldg(p.rows + u.r);
  if (!row_ok(p, row)) return;
  const uint8_t* src = (u.t ? p.b : p.a) + row_off(p, u, row);
  *reinterpret_cast<uint4*>(wire + wire_off(p, u.r, u)) = *reinterpret_cast<const uint4*>(src);
}

__global__ void __launch_bounds__(256) rows_unpack_kernel(const RowArgs p, const uint8_t* wire) {
  const int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  Unit u;
  if (!unit_of(p, g, u)) return;
  const int64_t row = __ldg(p.rows + u.r);
  if (!row_ok(p, row)) return;
  uint8_t* dst = const_cast<uint8_t*>(u.t ? p.b : p.a) + row_off(p, u, row);
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(wire + wire_off(p, u.r, u));
}

template <typename TY>
__device__ __forceinline__ void add_vec(float* acc, const uint4& w) {
  if constexpr (sizeof(TY) == 2) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  } else {
    const float* f = reinterpret_cast<const float*>(&w);
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] += f[i];
  }
}

// rows[e] += sum of wire rows contrib_wire[contrib_ptr[e] .. contrib_ptr[e+1]),
// accumulated in fp32 in list order and rounded once
template <typename TY>
__global__ void __launch_bounds__(256) rows_accumulate_kernel(const RowArgs p,
                                                              const int32_t* contrib_ptr,
                                                              const int64_t* contrib_wire,
                                                              int64_t n_wire,
                                                              const uint8_t* wire) {
  constexpr int N = 16 / sizeof(TY);
  const int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  Unit u;
  if (!unit_of(p, g, u)) return;
  const int64_t row = __ldg(p.rows + u.r);
  if (!row_ok(p, row)) return;
  uint8_t* dst = const_cast<uint8_t*>(u.t ? p.b : p.a) + row_off(p, u, row);
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  add_vec<TY>(acc, *reinterpret_cast<const uint4*>(dst));
  const int c0 = __ldg(contrib_ptr + u.r), c1 = __ldg(contrib_ptr + u.r + 1);
  for (int c = c0; c < c1; ++c) {
    const int64_t w = __ldg(contrib_wire + c);
    if (w < 0 || w >= n_wire) {
      if (p.err) atomicOr(p.err, DEV_ERR_BAD_WORK);
      return;
    }
    add_vec<TY>(acc, *reinterpret_cast<const uint4*>(wire + wire_off(p, w, u)));
  }
  uint4 out;
  if constexpr (sizeof(TY) == 2) {
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
  } else {
    float* f = reinterpret_cast<float*>(&out);
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] = acc[i];
  }
  *reinterpret_cast<uint4*>(dst) = out;
}

int make_args(RowArgs& p, int dtype, const void* a, const int64_t* as, const void* b,
              const int64_t* bs, int B, int H, int T, int D, const int64_t* rows, int64_t n_rows,
              int32_t* err) {
  if (dtype != SMAT_DTYPE_BF16 && dtype != SMAT_DTYPE_F32) return SMAT_ERR_UNSUPPORTED_DTYPE;
  if (B < 1 || H < 1 || T < 1 || n_rows < 0) return SMAT_ERR_BAD_SHAPE;
  if (!as || !bs) return SMAT_ERR_NULL_POINTER;
  const int elem = dtype == SMAT_DTYPE_BF16 ? 2 : 4;
  if (D < 1 || (D * elem) % 16) return SMAT_ERR_UNSUPPORTED_D;
  if (n_rows > 0 && (!a || !b || !rows)) return SMAT_ERR_NULL_POINTER;
  const int64_t v = 16 / elem;
  for (const int64_t* s : {as, bs})
    for (int i = 0; i < 3; ++i) {
      if (s[i] < 0) return SMAT_ERR_BAD_STRIDE;
      if (s[i] % v) return SMAT_ERR_BAD_ALIGNMENT;
    }
  if (reinterpret_cast<uintptr_t>(a) % 16 || reinterpret_cast<uintptr_t>(b) % 16)
    return SMAT_ERR_BAD_ALIGNMENT;
  p.a = static_cast<const uint8_t*>(a);
  p.b = static_cast<const uint8_t*>(b);
  p.a_sb = as[0];
  p.a_sh = as[1];
  p.a_st = as[2];
  p.b_sb = bs[0];
  p.b_sh = bs[1];
  p.b_st = bs[2];
  p.B = B;
  p.H = H;
  p.T = T;
  p.D = D;
  p.elem = elem;
  p.rows = rows;
  p.n_rows = n_rows;
  p.err = err;
  return SMAT_OK;
}

int64_t n_threads(const RowArgs& p) {
  return p.n_rows * 2 * p.B * p.H * (p.D * p.elem / 16);
}

int launched() { return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH; }

}  // namespace

extern "C" {

int smat_rows_pack(int dtype, const void* a, const int64_t* a_stride, const void* b,
                   const int64_t* b_stride, int B, int H, int T, int D, const int64_t* rows,
                   int64_t n_rows, void* wire, int32_t* err_word, void* stream) {
  RowArgs p;
  int rc = make_args(p, dtype, a, a_stride, b, b_stride, B, H, T, D, rows, n_rows, err_word);
  if (rc) return rc;
  if (n_rows == 0) return SMAT_OK;
  if (!wire) return SMAT_ERR_NULL_POINTER;
  if (reinterpret_cast<uintptr_t>(wire) % 16) return SMAT_ERR_BAD_ALIGNMENT;
  const int64_t n = n_threads(p);
  rows_pack_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                     static_cast<cudaStream_t>(stream)>>>(p, static_cast<uint8_t*>(wire));
  return launched();
}

int smat_rows_unpack(int dtype, void* a, const int64_t* a_stride, void* b,
                     const int64_t* b_stride, int B, int H, int T, int D, const int64_t* rows,
                     int64_t n_rows, const void* wire, int32_t* err_word, void* stream) {
  RowArgs p;
  int rc = make_args(p, dtype, a, a_stride, b, b_stride, B, H, T, D, rows, n_rows, err_word);
  if (rc) return rc;
  if (n_rows == 0) return SMAT_OK;
  if (!wire) return SMAT_ERR_NULL_POINTER;
  if (reinterpret_cast<uintptr_t>(wire) % 16) return SMAT_ERR_BAD_ALIGNMENT;
  const int64_t n = n_threads(p);
  rows_unpack_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0,
                       static_cast<cudaStream_t>(stream)>>>(p, static_cast<const uint8_t*>(wire));
  return launched();
}

int smat_rows_accumulate(int dtype, void* a, const int64_t* a_stride, void* b,
                         const int64_t* b_stride, int B, int H, int T, int D,
                         const int64_t* rows, int64_t n_rows, const int32_t* contrib_ptr,
                         const int64_t* contrib_wire, int64_t n_wire, const void* wire,
                         int32_t* err_word, void* stream) {
  RowArgs p;
  int rc = make_args(p, dtype, a, a_stride, b, b_stride, B, H, T, D, rows, n_rows, err_word);
  if (rc) return rc;
  if (n_rows == 0) return SMAT_OK;
  if (!contrib_ptr) return SMAT_ERR_NULL_POINTER;
  if (n_wire < 0) return SMAT_ERR_BAD_SHAPE;
  if (n_wire > 0 && (!wire || !contrib_wire)) return SMAT_ERR_NULL_POINTER;
  if (reinterpret_cast<uintptr_t>(wire) % 16) return SMAT_ERR_BAD_ALIGNMENT;
  const int64_t n = n_threads(p);
  const unsigned grid = static_cast<unsigned>((n + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == SMAT_DTYPE_BF16)
    rows_accumulate_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        p, contrib_ptr, contrib_wire, n_wire, static_cast<const uint8_t*>(wire));
  else
    rows_accumulate_kernel<float><<<grid, 256, 0, s>>>(p, contrib_ptr, contrib_wire, n_wire,
                                                       static_cast<const uint8_t*>(wire));
  return launched();
}

}  // extern "C"
