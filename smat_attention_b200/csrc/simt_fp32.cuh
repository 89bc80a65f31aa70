// fp32 path: block-sparse causal softmax attention on CUDA cores.
//
// The fp32 contract is 1e-4 max-abs against an fp32 reference, which a
// tensor-core tf32 product cannot meet, so fp32 inputs run here in full fp32
// (fmaf, expf, logf).  These kernels serve the small fp32 configurations; the
// bf16 path uses the tcgen05 kernels.
//
// Each query (or key) row is owned by TPR = D / 32 adjacent lanes holding 32
// of its D components; dot products are reduced across those lanes with
// shuffles.  The walk over the layout is the same CSR walk the tensor-core
// kernels do, one key (or query) at a time, causal inside diagonal tiles and
// masked by the pattern.cuh rule inside M^(d) PATTERN tiles.
#pragma once

#include "common.cuh"
#include "pattern.cuh"

namespace smat {

struct SimtParams {
  const float* q;
  const float* k;
  const float* v;
  const float* o;
  const float* dout;
  const float* lse;
  const float* delta;
  float* out0;  // o (fwd) / dq / dk
  float* out1;  // lse (fwd) / dv
  int64_t q_s[3], k_s[3], v_s[3], o_s[3], do_s[3], out0_s[3], out1_s[3];
  const int32_t* indptr;
  const int32_t* indices;
  const uint8_t* kind;
  int B, H, T, nblocks, nnzb, bs;
  const int32_t* work;  // optional work list of 128-row tiles; null = all rows
  int span_tiles;       // tiles one work item may span: 2 (forward) or 1
  float scale;
  int32_t* err;
  MdPattern md;         // tables of PATTERN tiles (null row_bits: the layout has none)
};

constexpr int SIMT_TILE = 128;
constexpr int SIMT_THREADS = 64;   // threads per CTA (64: c1 1.18 ms, 128: 1.33, 32: 1.20)

// Row of group g in this CTA.  Without a work list CTA x covers rows
// [x RPC, x RPC + RPC); with one, each item owns span_tiles * 128 / RPC CTAs
// and rows outside the item's tiles are inactive.  False for an invalid item
// (the CTA then returns without touching memory).
template <int RPC>
__device__ __forceinline__ bool simt_row(const SimtParams& p, int g, int& row, bool& active) {
  if (!p.work) {
    row = blockIdx.x * RPC + g;
    active = row < p.T;
    return true;
  }
  const int per = p.span_tiles * SIMT_TILE / RPC;
  const int w = __ldg(p.work + blockIdx.x / per);
  const int tile = w & WORK_TILE_MASK;
  const int n = (w & WORK_PAIR_BIT) ? 2 : 1;
  const int n_tiles = (p.T + SIMT_TILE - 1) / SIMT_TILE;
  if ((w >> 25) != 0 || n > p.span_tiles || tile + n > n_tiles) {
    if (threadIdx.x == 0 && p.err) atomicOr(p.err, DEV_ERR_BAD_WORK);
    return false;
  }
  const int off = (blockIdx.x % per) * RPC + g;
  row = tile * SIMT_TILE + off;
  active = off < n * SIMT_TILE && row < p.T;
  return true;
}

// Sum over the TPR lanes that own one row.  Only those lanes take part (the
// mask names them), so rows of one warp may walk different key counts.
template <int TPR>
__device__ __forceinline__ float group_sum(float x) {
  if (TPR == 1) return x;
  const unsigned lane = threadIdx.x & 31u;
  const unsigned mask = ((1u << TPR) - 1u) << (lane & ~static_cast<unsigned>(TPR - 1));
#pragma unroll
  for (int o = 1; o < TPR; o <<= 1) x += __shfl_xor_sync(mask, x, o);
  return x;
}

// Is (query i, key j) visible in a tile of kind `kd` (0 full, 1 causal diagonal,
// 2 M^(d) pattern)?  For pattern tiles `w` caches the mask word of the 32-aligned
// group holding the varying index (j for a row walk, i for a column walk);
// `fresh` asks for it to be reloaded.
__device__ __forceinline__ bool simt_visible(const SimtParams& p, uint8_t kd, int i, int j,
                                             bool col_walk, bool fresh, uint32_t& w) {
  if (kd == 1) return j <= i;
  if (kd != 2) return true;
  if (!p.md.row_bits) {
    if (p.err) atomicOr(p.err, DEV_ERR_BAD_CSR);
    return false;
  }
  const int v = col_walk ? i : j;
  if (fresh || (v & 31) == 0)
    w = col_walk ? md_col_word(p.md, p.T, j, v & ~31) : md_row_word(p.md, p.T, i, v & ~31);
  return (w >> (v & 31)) & 1u;
}

__device__ __forceinline__ const float* row_ptr(const float* base, const int64_t* s, int b, int h,
                                                int t) {
  return base + b * s[0] + h * s[1] + static_cast<int64_t>(t) * s[2];
}

// Rows of keys staged in shared memory for all rows of a CTA: SIMT_KB rows of
// D floats at a stride of D + 4 (the TPR lanes of a row read different
// 32-float parts of a key without bank conflicts).  Every thread of the CTA
// takes part; consecutive threads read consecutive floats.
constexpr int SIMT_KB = 32;
template <int D>
__device__ __forceinline__ void simt_stage(float* dst, const float* base, const int64_t* s, int b,
                                           int h, int j0, int n) {
  for (int idx = threadIdx.x; idx < n * D; idx += SIMT_THREADS) {
    const int r = idx / D, c = idx % D;
    dst[r * (D + 4) + c] = row_ptr(base, s, b, h, j0 + r)[c];
  }
}

// grid: (ceil(T / rows_per_cta) or n_work * span_tiles * 128 / rows_per_cta, B * H);
// block SIMT_THREADS threads.
template <int D>
__global__ void __launch_bounds__(SIMT_THREADS) smat_fwd_simt_kernel(const SimtParams p) {
  constexpr int TPR = D / 32;
  constexpr int RPC = SIMT_THREADS / TPR;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int g = threadIdx.x / TPR, part = threadIdx.x % TPR;
  int i;
  bool active;
  if (!simt_row<RPC>(p, g, i, active)) return;
  const int ii = active ? i : p.T - 1;
  float q[32], acc[32];
  const float* qr = row_ptr(p.q, p.q_s, b, h, ii) + part * 32;
#pragma unroll
  for (int d = 0; d < 32; ++d) {
    q[d] = qr[d] * p.scale;
    acc[d] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  // one key of the walk: score, visibility, online softmax update
  auto step = [&](int j, int j0, uint8_t kd, uint32_t& w, const float* kr, const float* vr) {
    float s = 0.f;
#pragma unroll
    for (int d = 0; d < 32; ++d) s = fmaf(q[d], kr[d], s);
    s = group_sum<TPR>(s);
    if (!simt_visible(p, kd, ii, j, false, j == j0, w)) return;
    if (s > m) {
      const float alpha = (m == -INFINITY) ? 0.f : expf(m - s);
      l *= alpha;
#pragma unroll
      for (int d = 0; d < 32; ++d) acc[d] *= alpha;
      m = s;
    }
    const float pr = expf(s - m);
    l += pr;
#pragma unroll
    for (int d = 0; d < 32; ++d) acc[d] = fmaf(pr, vr[d], acc[d]);
  };
  // When every row of the CTA lies in one query block, the rows share a CSR
  // row: its keys and values are staged in shared memory once for all of
  // them, SIMT_KB at a time.  Otherwise each row walks its own CSR row
  // reading K and V from global memory.
  int first;
  bool first_active;
  simt_row<RPC>(p, 0, first, first_active);
  const int last = min(first + RPC - 1, p.T - 1);
  const bool shared = first < p.T && first / p.bs == last / p.bs;
  if (shared) {
    __shared__ float ks[SIMT_KB * (D + 4)], vs[SIMT_KB * (D + 4)];
    const int qb = first / p.bs;
    const int e0 = p.indptr[qb], e1 = p.indptr[qb + 1];
    for (int e = e0; e < e1; ++e) {
      const int kb = p.indices[e];
      const uint8_t kd = p.kind[e];
      const int j0 = kb * p.bs, j1 = min(p.T, j0 + p.bs);
      uint32_t w = 0u;
      for (int jb = j0; jb < j1; jb += SIMT_KB) {
        const int n = min(SIMT_KB, j1 - jb);
        __syncthreads();   // the previous keys are consumed
        simt_stage<D>(ks, p.k, p.k_s, b, h, jb, n);
        simt_stage<D>(vs, p.v, p.v_s, b, h, jb, n);
        __syncthreads();
        for (int jj = 0; jj < n; ++jj)
          step(jb + jj, j0, kd, w, ks + jj * (D + 4) + part * 32, vs + jj * (D + 4) + part * 32);
      }
    }
  } else {
    const int qb = ii / p.bs;
    const int e0 = p.indptr[qb], e1 = p.indptr[qb + 1];
    for (int e = e0; e < e1; ++e) {
      const int kb = p.indices[e];
      const uint8_t kd = p.kind[e];
      const int j0 = kb * p.bs, j1 = min(p.T, j0 + p.bs);
      uint32_t w = 0u;
      for (int j = j0; j < j1; ++j)
        step(j, j0, kd, w, row_ptr(p.k, p.k_s, b, h, j) + part * 32,
             row_ptr(p.v, p.v_s, b, h, j) + part * 32);
    }
  }
  if (!active) return;
  const float inv = l > 0.f ? 1.f / l : 0.f;
  float* orow = p.out0 + b * p.out0_s[0] + h * p.out0_s[1] + static_cast<int64_t>(i) * p.out0_s[2] +
                part * 32;
#pragma unroll
  for (int d = 0; d < 32; ++d) orow[d] = acc[d] * inv;
  if (part == 0) p.out1[static_cast<int64_t>(bh) * p.T + i] = l > 0.f ? m + logf(l) : -INFINITY;
}

// dQ: per query row, walk the forward CSR.
template <int D>
__global__ void __launch_bounds__(SIMT_THREADS) smat_dq_simt_kernel(const SimtParams p) {
  constexpr int TPR = D / 32;
  constexpr int RPC = SIMT_THREADS / TPR;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int g = threadIdx.x / TPR, part = threadIdx.x % TPR;
  int i;
  bool active;
  if (!simt_row<RPC>(p, g, i, active)) return;
  const int ii = active ? i : p.T - 1;
  float q[32], dor[32], dq[32];
  const float* qr = row_ptr(p.q, p.q_s, b, h, ii) + part * 32;
  const float* dr = row_ptr(p.dout, p.do_s, b, h, ii) + part * 32;
#pragma unroll
  for (int d = 0; d < 32; ++d) {
    q[d] = qr[d] * p.scale;
    dor[d] = dr[d];
    dq[d] = 0.f;
  }
  const float lse = p.lse[static_cast<int64_t>(bh) * p.T + ii];
  const float dl = p.delta[static_cast<int64_t>(bh) * p.T + ii];
  auto step = [&](int j, int j0, uint8_t kd, uint32_t& w, const float* kr, const float* vr) {
    float s = 0.f, dp = 0.f;
#pragma unroll
    for (int d = 0; d < 32; ++d) {
      s = fmaf(q[d], kr[d], s);
      dp = fmaf(dor[d], vr[d], dp);
    }
    s = group_sum<TPR>(s);
    dp = group_sum<TPR>(dp);
    if (!simt_visible(p, kd, ii, j, false, j == j0, w)) return;
    const float pr = expf(s - lse);
    const float ds = pr * (dp - dl);
#pragma unroll
    for (int d = 0; d < 32; ++d) dq[d] = fmaf(ds, kr[d], dq[d]);
  };
  // rows of one query block share their CSR row: K and V staged once (as in
  // the forward)
  int first;
  bool first_active;
  simt_row<RPC>(p, 0, first, first_active);
  const int last = min(first + RPC - 1, p.T - 1);
  if (first < p.T && first / p.bs == last / p.bs) {
    __shared__ float ks[SIMT_KB * (D + 4)], vs[SIMT_KB * (D + 4)];
    const int qb = first / p.bs;
    for (int e = p.indptr[qb]; e < p.indptr[qb + 1]; ++e) {
      const int kb = p.indices[e];
      const uint8_t kd = p.kind[e];
      const int j0 = kb * p.bs, j1 = min(p.T, j0 + p.bs);
      uint32_t w = 0u;
      for (int jb = j0; jb < j1; jb += SIMT_KB) {
        const int n = min(SIMT_KB, j1 - jb);
        __syncthreads();
        simt_stage<D>(ks, p.k, p.k_s, b, h, jb, n);
        simt_stage<D>(vs, p.v, p.v_s, b, h, jb, n);
        __syncthreads();
        for (int jj = 0; jj < n; ++jj)
          step(jb + jj, j0, kd, w, ks + jj * (D + 4) + part * 32, vs + jj * (D + 4) + part * 32);
      }
    }
  } else {
    const int qb = ii / p.bs;
    for (int e = p.indptr[qb]; e < p.indptr[qb + 1]; ++e) {
      const int kb = p.indices[e];
      const uint8_t kd = p.kind[e];
      const int j0 = kb * p.bs, j1 = min(p.T, j0 + p.bs);
      uint32_t w = 0u;
      for (int j = j0; j < j1; ++j)
        step(j, j0, kd, w, row_ptr(p.k, p.k_s, b, h, j) + part * 32,
             row_ptr(p.v, p.v_s, b, h, j) + part * 32);
    }
  }
  if (!active) return;
  float* out = p.out0 + b * p.out0_s[0] + h * p.out0_s[1] + static_cast<int64_t>(i) * p.out0_s[2] +
               part * 32;
#pragma unroll
  for (int d = 0; d < 32; ++d) out[d] = dq[d] * p.scale;
}

// dK, dV: per key row, walk the transposed CSR.
template <int D>
__global__ void __launch_bounds__(SIMT_THREADS) smat_dkdv_simt_kernel(const SimtParams p) {
  constexpr int TPR = D / 32;
  constexpr int RPC = SIMT_THREADS / TPR;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int g = threadIdx.x / TPR, part = threadIdx.x % TPR;
  int j;
  bool active;
  if (!simt_row<RPC>(p, g, j, active)) return;
  const int jj = active ? j : p.T - 1;
  float kr[32], vr[32], dk[32], dv[32];
  const float* kp = row_ptr(p.k, p.k_s, b, h, jj) + part * 32;
  const float* vp = row_ptr(p.v, p.v_s, b, h, jj) + part * 32;
#pragma unroll
  for (int d = 0; d < 32; ++d) {
    kr[d] = kp[d] * p.scale;
    vr[d] = vp[d];
    dk[d] = 0.f;
    dv[d] = 0.f;
  }
  auto step = [&](int i, int i0, uint8_t kd, uint32_t& w, const float* qp, const float* dp_,
                  float lse, float dl) {
    float s = 0.f, dp = 0.f;
#pragma unroll
    for (int d = 0; d < 32; ++d) {
      s = fmaf(qp[d], kr[d], s);
      dp = fmaf(dp_[d], vr[d], dp);
    }
    s = group_sum<TPR>(s);
    dp = group_sum<TPR>(dp);
    if (!simt_visible(p, kd, i, jj, true, i == i0, w)) return;
    const float pr = expf(s - lse);
    const float ds = pr * (dp - dl);
#pragma unroll
    for (int d = 0; d < 32; ++d) {
      dv[d] = fmaf(pr, dp_[d], dv[d]);
      dk[d] = fmaf(ds, qp[d], dk[d]);
    }
  };
  const float* lse_bh = p.lse + static_cast<int64_t>(bh) * p.T;
  const float* dl_bh = p.delta + static_cast<int64_t>(bh) * p.T;
  // rows (keys) of one key block share their transposed CSR row: Q, dO and
  // the queries' lse / delta staged once for all of them
  int first;
  bool first_active;
  simt_row<RPC>(p, 0, first, first_active);
  const int last = min(first + RPC - 1, p.T - 1);
  if (first < p.T && first / p.bs == last / p.bs) {
    __shared__ float qs[SIMT_KB * (D + 4)], ds_[SIMT_KB * (D + 4)], ls[SIMT_KB], dls[SIMT_KB];
    const int kb = first / p.bs;
    for (int e = p.indptr[kb]; e < p.indptr[kb + 1]; ++e) {
      const int qb = p.indices[e];
      const uint8_t kd = p.kind[e];
      const int i0 = qb * p.bs, i1 = min(p.T, i0 + p.bs);
      uint32_t w = 0u;
      for (int ib = i0; ib < i1; ib += SIMT_KB) {
        const int n = min(SIMT_KB, i1 - ib);
        __syncthreads();
        simt_stage<D>(qs, p.q, p.q_s, b, h, ib, n);
        simt_stage<D>(ds_, p.dout, p.do_s, b, h, ib, n);
        for (int r = threadIdx.x; r < n; r += SIMT_THREADS) {
          ls[r] = lse_bh[ib + r];
          dls[r] = dl_bh[ib + r];
        }
        __syncthreads();
        for (int r = 0; r < n; ++r)
          step(ib + r, i0, kd, w, qs + r * (D + 4) + part * 32, ds_ + r * (D + 4) + part * 32,
               ls[r], dls[r]);
      }
    }
  } else {
    const int kb = jj / p.bs;
    for (int e = p.indptr[kb]; e < p.indptr[kb + 1]; ++e) {
      const int qb = p.indices[e];
      const uint8_t kd = p.kind[e];
      const int i0 = qb * p.bs, i1 = min(p.T, i0 + p.bs);
      uint32_t w = 0u;
      for (int i = i0; i < i1; ++i)
        step(i, i0, kd, w, row_ptr(p.q, p.q_s, b, h, i) + part * 32,
             row_ptr(p.dout, p.do_s, b, h, i) + part * 32, lse_bh[i], dl_bh[i]);
    }
  }
  if (!active) return;
  float* ko = p.out0 + b * p.out0_s[0] + h * p.out0_s[1] + static_cast<int64_t>(j) * p.out0_s[2] +
              part * 32;
  float* vo = p.out1 + b * p.out1_s[0] + h * p.out1_s[1] + static_cast<int64_t>(j) * p.out1_s[2] +
              part * 32;
#pragma unroll
  for (int d = 0; d < 32; ++d) {
    ko[d] = dk[d] * p.scale;
    vo[d] = dv[d];
  }
}

// delta[row] = sum_d O[row, d] dO[row, d] over rows (b, h, row_lo + t),
// t < n_rows; LPR lanes per row, one 16-byte vector of O and dO each.  IDX is
// the index type: 32-bit when rows * LPR fits (the divisions that locate a
// row are then 32-bit), else 64-bit.
template <typename T, int D, typename IDX>
__global__ void __launch_bounds__(256) smat_bwd_pre_kernel(const T* __restrict__ o,
                                                           const T* __restrict__ dout,
                                                           float* __restrict__ delta,
                                                           int64_t o_sb, int64_t o_sh,
                                                           int64_t o_st, int64_t d_sb,
                                                           int64_t d_sh, int64_t d_st, int H,
                                                           int T_, int row_lo, int n_rows,
                                                           int64_t rows) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int LPR = D / VEC;  // lanes per row
  static_assert(LPR <= 32 && 32 % LPR == 0, "unsupported D");
  const IDX gt = static_cast<IDX>(blockIdx.x) * blockDim.x + threadIdx.x;
  const IDX row = gt / LPR;
  const int part = static_cast<int>(gt % LPR);
  const IDX nr = static_cast<IDX>(n_rows);
  const int t = row_lo + static_cast<int>(row % nr);
  const IDX bh = row / nr;
  const bool in = static_cast<int64_t>(row) < rows;
  float acc = 0.f;
  if (in) {
    const int b = static_cast<int>(bh / static_cast<IDX>(H)), h = static_cast<int>(bh % static_cast<IDX>(H));
    const T* op = o + b * o_sb + h * o_sh + t * o_st + part * VEC;
    const T* dp = dout + b * d_sb + h * d_sh + t * d_st + part * VEC;
    const uint4 ov = *reinterpret_cast<const uint4*>(op);
    const uint4 dv = *reinterpret_cast<const uint4*>(dp);
    const T* oe = reinterpret_cast<const T*>(&ov);
    const T* de = reinterpret_cast<const T*>(&dv);
#pragma unroll
    for (int i = 0; i < VEC; ++i) acc = fmaf(static_cast<float>(oe[i]), static_cast<float>(de[i]), acc);
  }
#pragma unroll
  for (int off = 1; off < LPR; off <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (in && part == 0) delta[static_cast<int64_t>(bh) * T_ + t] = acc;
}

}  // namespace smat
