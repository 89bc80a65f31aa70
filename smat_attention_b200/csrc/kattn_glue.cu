// The kernelised op's glue between its fused passes (include/smat_kattn.h):
// the chunk summaries and their segmented prefix sums of the causal scan, the
// backward's expansion of the summary gradient, and the per-type long-range
// query, with its backward.  All fp32 FMA on CUDA cores (the reference runs
// them as fp32 torch GEMMs and cumsums, src/smat/attention.py:134-192 and
// :310-330); each moves more bytes than it computes per element.
//
// chunk prefix (forward Sin, backward dD):
//   D_c      = a_c^T b_c                      one CTA per (chunk, sequence), 8 x 4
//                                             register tiles over shared memory
//   out_c    = sum of D_c' over the chunks c' before c (or after c, reverse)
//              in c's segment [0, nc0) or [nc0, nc)   one thread per element,
//                                             sequential over the chunks (a
//                                             shifted scan: D_c never enters
//                                             out_c, and the segments never mix)
// chunk expand:  db_c += a_c dD_c and da_c += b_c dD_c^T (8 x 4 register tiles)
// query by type: out_i (+)= phi_i U_{i mod nU}; its backward dphi_i =
//                dout_i U^T, dU_h = sum over the rows of type h of phi_i^T dout_i
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "../../include/smat_b200.h"
#include "../../include/smat_kattn.h"
#include "common.cuh"

namespace {

using namespace smat;

constexpr int GLUE_SMEM_MAX = 200 * 1024;
constexpr int QT_ROWS = 16;   // rows of one type handled per pass of the query kernels

__host__ __device__ inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

// rows [row0, row0 + nrows) of a row-major [T, W] matrix into shared [nrows][WS]
// (zero-filled past T and past W), by asynchronous 4-byte copies
__device__ __forceinline__ void stage_rows(float* dst, const float* src, int row0, int nrows,
                                           int T, int W, int WS) {
  for (int e = threadIdx.x; e < nrows * WS; e += blockDim.x) {
    const int i = e / WS, c = e % WS;
    const bool in = c < W && row0 + i < T;
    cp_async4(smem_u32(dst + e), in ? src + static_cast<int64_t>(row0 + i) * W + c : src,
              in ? 4u : 0u);
  }
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ bool al16d(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}


// ---------------------------------------------------------------- chunk sums
// D[s, c] = a_c^T b_c over the C rows of chunk c (rows past T count as zero).
// Shared: a rows [C][RA], b rows [C][PB]; a thread owns an 8 (r) x 4 (p) tile
// and walks the chunk's rows in order.
__global__ void __launch_bounds__(256) kattn_chunk_sum_kernel(const float* __restrict__ a,
                                                              const float* __restrict__ b,
                                                              float* __restrict__ D, int T,
                                                              int C, int R, int P) {
  extern __shared__ float4 sm4[];
  float* sm = reinterpret_cast<float*>(sm4);
  const int c = blockIdx.x, s = blockIdx.y, nc = gridDim.x;
  const int RA = round_up(R, 8), PB = round_up(P, 4);
  float* sa = sm;
  float* sb = sm + C * RA;
  float* flat = sb + C * PB;    // [C * P] staging of the b chunk as one run
  const float* as = a + static_cast<int64_t>(s) * T * R;
  const float* bs = b + static_cast<int64_t>(s) * T * P;
  const int rows = min(C, T - c * C);
  if ((R & 7) == 0 && al16d(as)) {
    // whole rows of 16-byte units; rows past T zero
    const int u = R / 4;
    for (int e = threadIdx.x; e < C * u; e += blockDim.x) {
      const int i = e / u, k = (e % u) * 4;
      if (i < rows)
        cp_async16(smem_u32(sa + i * RA + k), as + static_cast<int64_t>(c * C + i) * R + k);
      else
        *reinterpret_cast<float4*>(sa + i * RA + k) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  } else {
    stage_rows(sa, as, c * C, C, T, R, RA);
  }
  const float* bc = bs + static_cast<int64_t>(c) * C * P;
  const int nflat = rows * P;
  const bool flat16 = al16d(bc) && (nflat & 3) == 0;
  if (flat16) {
    for (int e = threadIdx.x * 4; e < nflat; e += blockDim.x * 4)
      cp_async16(smem_u32(flat + e), bc + e);
  } else {
    stage_rows(sb, bs, c * C, C, T, P, PB);
  }
  cp_async_wait_all();
  __syncthreads();
  if (flat16) {   // [rows * P] -> [C][PB], zero padding
    for (int e = threadIdx.x; e < C * PB; e += blockDim.x) {
      const int i = e / PB, p = e % PB;
      sb[e] = (i < rows && p < P) ? flat[i * P + p] : 0.f;
    }
    __syncthreads();
  }
  const int PG = PB / 4, tiles = (RA / 8) * PG;
  float* out = D + (static_cast<int64_t>(s) * nc + c) * R * P;
  for (int t = threadIdx.x; t < tiles; t += blockDim.x) {
    const int r0 = (t / PG) * 8, p0 = (t % PG) * 4;
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 4
    for (int k = 0; k < C; ++k) {
      const float4 x0 = *reinterpret_cast<const float4*>(sa + k * RA + r0);
      const float4 x1 = *reinterpret_cast<const float4*>(sa + k * RA + r0 + 4);
      const float4 y = *reinterpret_cast<const float4*>(sb + k * PB + p0);
      const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
      const float yv[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xv[i], yv[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (r0 + i < R && p0 + j < P) out[(r0 + i) * P + p0 + j] = acc[i][j];
  }
}

// In place over D [nb, nc, RP]: element e of chunk c becomes the sum of the
// elements of the chunks before c (reverse: after c) in c's segment.  The
// chunk values are loaded eight at a time ahead of the dependent adds.
__global__ void __launch_bounds__(256) kattn_seg_scan_kernel(float* __restrict__ D, int nc,
                                                             int64_t RP, int nc0, int reverse) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= RP) return;
  float* base = D + static_cast<int64_t>(blockIdx.y) * nc * RP + e;
  float run = 0.f;
  for (int i0 = 0; i0 < nc; i0 += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = i0 + j;
      const int c = reverse ? nc - 1 - i : i;
      v[j] = i < nc ? base[static_cast<int64_t>(c) * RP] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = i0 + j;
      if (i >= nc) break;
      const int c = reverse ? nc - 1 - i : i;
      // a segment starts here: nothing before it (after it, reverse) reaches it
      if ((!reverse && c == nc0) || (reverse && c == nc0 - 1)) run = 0.f;
      base[static_cast<int64_t>(c) * RP] = run;
      run += v[j];
    }
  }
}

// ---------------------------------------------------------------- chunk expand
// Chunk c of sequence s: db[rows] += a_c dD_c, da[rows] += b_c dD_c^T (the
// backward of D = a_c^T b_c).  Shared, row-major: a rows [CS][RA] (16-byte
// copies when R is a multiple of 4), b rows [CS][PB], dD [RA][PB] and dD^T
// [PB][RA] (4-byte copies -- P is odd in the reference); all copies are
// issued before one wait and read global memory in consecutive addresses.  A
// thread owns an 8-row x 4-column tile of db or da and reads its 8 rows four
// k at a time.
__global__ void __launch_bounds__(256) kattn_chunk_expand_kernel(
    const float* __restrict__ a, const float* __restrict__ b, const float* __restrict__ dD,
    float* __restrict__ da, float* __restrict__ db, int T, int C, int R, int P) {
  extern __shared__ float4 sm4[];
  float* sm = reinterpret_cast<float*>(sm4);
  const int c = blockIdx.x, s = blockIdx.y, nc = gridDim.x;
  const int RA = round_up(R, 8), PB = round_up(P, 8), CS = round_up(C, 8);
  float* sa = sm;                  // [CS][RA]
  float* sb = sa + CS * RA;        // [CS][PB]
  float* sd = sb + CS * PB;        // [RA][PB]  dD
  float* sdT = sd + RA * PB;       // [PB][RA]  dD^T
  const int64_t row0 = static_cast<int64_t>(c) * C;
  const int rows = static_cast<int>(T - row0 < C ? T - row0 : C);
  const float* as = a + static_cast<int64_t>(s) * T * R;
  const float* bs = b + static_cast<int64_t>(s) * T * P;
  if ((R & 3) == 0 && al16d(as)) {
    for (int e = threadIdx.x; e < CS * (RA / 4); e += blockDim.x) {
      const int i = e / (RA / 4), k = (e % (RA / 4)) * 4;
      if (i < rows && k < R)
        cp_async16(smem_u32(sa + i * RA + k), as + (row0 + i) * R + k);
      else
        *reinterpret_cast<float4*>(sa + i * RA + k) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  } else {
    stage_rows(sa, as, static_cast<int>(row0), CS, T, R, RA);
  }
  stage_rows(sb, bs, static_cast<int>(row0), CS, T, P, PB);
  const float* dd = dD + (static_cast<int64_t>(s) * nc + c) * R * P;
  for (int e = threadIdx.x; e < RA * PB; e += blockDim.x) {
    const int r = e / PB, p = e % PB;
    const bool in = r < R && p < P;
    const float* src = in ? dd + r * P + p : dd;
    cp_async4(smem_u32(sd + e), src, in ? 4u : 0u);
    cp_async4(smem_u32(sdT + p * RA + r), src, in ? 4u : 0u);
  }
  cp_async_wait_all();
  __syncthreads();
  // db tiles: 8 rows x 4 p, K = R (X = a rows, Y = dD); then da tiles: 8 rows
  // x 4 r, K = P (X = b rows, Y = dD^T)
  const int tb = (CS / 8) * (PB / 4), ta = (CS / 8) * (RA / 4);
  for (int t = threadIdx.x; t < tb + ta; t += blockDim.x) {
    const bool is_b = t < tb;
    const int u = is_b ? t : t - tb;
    const int W = is_b ? PB : RA;          // output width (padded)
    const int K = is_b ? RA : PB;          // contraction length (padded, multiple of 8)
    const float* X = is_b ? sa : sb;       // [CS][K]
    const float* Y = is_b ? sd : sdT;      // [K][W]
    const int i0 = (u / (W / 4)) * 8, j0 = (u % (W / 4)) * 4;
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 2
    for (int k = 0; k < K; k += 4) {
      float xv[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 x = *reinterpret_cast<const float4*>(X + (i0 + i) * K + k);
        xv[i][0] = x.x;
        xv[i][1] = x.y;
        xv[i][2] = x.z;
        xv[i][3] = x.w;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float4 y = *reinterpret_cast<const float4*>(Y + (k + kk) * W + j0);
        const float yv[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xv[i][kk], yv[j], acc[i][j]);
      }
    }
    const int Wo = is_b ? P : R;
    float* dst = (is_b ? db + static_cast<int64_t>(s) * T * P : da + static_cast<int64_t>(s) * T * R) +
                 row0 * Wo;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (i0 + i < rows && j0 + j < Wo) dst[(i0 + i) * Wo + j0 + j] += acc[i][j];
  }
}

// ---------------------------------------------------------------- query by type
// out[s, i] (+)= phi[s, i] U[s, i mod nU] for i < T_R.  One CTA per (type h,
// sequence): U_h (R x P, contiguous) and the rows of type h (h, h + nU, ...,
// QT_ROWS per pass) are staged in shared memory by asynchronous copies issued
// all at once (16 bytes each where the layout allows), then thread = output
// column p sums over r from shared memory (U_h rows conflict-free, phi
// broadcast).

__global__ void __launch_bounds__(128) kattn_query_kernel(
    const float* __restrict__ phi, int64_t phi_sb, const float* __restrict__ U,
    float* __restrict__ out, int64_t out_sb, int T_R, int R, int P, int nU, int accumulate) {
  extern __shared__ float4 sm4[];
  const int RA = round_up(R, 4);
  float* su = reinterpret_cast<float*>(sm4);    // [R][P] = U_h
  float* sph = su + round_up(R * P, 4);         // [QT_ROWS][RA]
  const int h = blockIdx.x, s = blockIdx.y;
  const float* Uh = U + (static_cast<int64_t>(s) * nU + h) * R * P;
  const float* ph = phi + s * phi_sb;
  float* os = out + s * out_sb;
  const int RP = R * P;
  if ((RP & 3) == 0 && al16d(Uh)) {
    for (int e = threadIdx.x * 4; e < RP; e += blockDim.x * 4) cp_async16(smem_u32(su + e), Uh + e);
  } else {
    for (int e = threadIdx.x; e < RP; e += blockDim.x) cp_async4(smem_u32(su + e), Uh + e, 4u);
  }
  const bool vec_phi = (R & 3) == 0 && al16d(ph) && ((nU * static_cast<int64_t>(R)) & 3) == 0;
  const int n_rows = h < T_R ? (T_R - h + nU - 1) / nU : 0;
  for (int g0 = 0; g0 < n_rows; g0 += QT_ROWS) {
    const int ng = min(QT_ROWS, n_rows - g0);
    if (g0 > 0) __syncthreads();   // the previous pass has finished reading sph
    if (vec_phi) {
      for (int e = threadIdx.x * 4; e < QT_ROWS * RA; e += blockDim.x * 4) {
        const int i = e / RA, r = e % RA;
        if (i < ng) {
          cp_async16(smem_u32(sph + e),
                     ph + static_cast<int64_t>(h + (g0 + i) * static_cast<int64_t>(nU)) * R + r);
        } else {
          *reinterpret_cast<float4*>(sph + e) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    } else {
      for (int e = threadIdx.x; e < QT_ROWS * RA; e += blockDim.x) {
        const int i = e / RA, r = e % RA;
        const bool in = i < ng && r < R;
        cp_async4(smem_u32(sph + e),
                  in ? ph + static_cast<int64_t>(h + (g0 + i) * static_cast<int64_t>(nU)) * R + r
                     : ph,
                  in ? 4u : 0u);
      }
    }
    cp_async_wait_all();
    __syncthreads();
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
      float acc[QT_ROWS];
#pragma unroll
      for (int i = 0; i < QT_ROWS; ++i) acc[i] = 0.f;
      for (int r0 = 0; r0 < RA; r0 += 4) {
        float u[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) u[j] = (r0 + j < R) ? su[(r0 + j) * P + p] : 0.f;
#pragma unroll
        for (int i = 0; i < QT_ROWS; ++i) {
          const float4 x = *reinterpret_cast<const float4*>(sph + i * RA + r0);
          acc[i] = fmaf(x.x, u[0], acc[i]);
          acc[i] = fmaf(x.y, u[1], acc[i]);
          acc[i] = fmaf(x.z, u[2], acc[i]);
          acc[i] = fmaf(x.w, u[3], acc[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < QT_ROWS; ++i) {
        if (i < ng) {
          float* o = os + static_cast<int64_t>(h + (g0 + i) * static_cast<int64_t>(nU)) * P + p;
          *o = accumulate ? *o + acc[i] : acc[i];
        }
      }
    }
  }
  cp_async_wait_all();   // a type without rows still drains its U copy
}

// dphi[s, i] = dout[s, i] U_h^T and dU[s, h] = sum over rows i of type h of
// phi[s, i]^T dout[s, i].  One CTA of 128 threads per (h, sequence), at most
// 64 registers a thread so that eight CTAs share an SM: a CTA loads U_h,
// computes and stores in turn, and more resident CTAs keep more of those
// loads in flight.  U_h goes to shared memory [RA][PU] once (PU = P rounded
// up to 4, plus 4 when that makes an even count of 16-byte units, so rows 1
// apart sit in different bank groups); the rows of type h follow QT_ROWS at
// a time (phi [QT_ROWS][RA], dout [QT_ROWS][PU]), all by asynchronous copies
// issued before one wait.  Per pass, dphi: a thread owns 2 rows x 4 r
// (r = r0 + 16 k), each 16-byte step along p loading two dout and four U_h
// vectors for 32 FMAs; dU: 4 x 4 blocks (4 r, 4 p), one at a time per
// thread, each row adding one 16-byte phi load and one 16-byte dout load per
// 16 FMAs, the block then stored to dU (added on later passes: a block
// belongs to one thread).

__host__ __device__ inline int query_pu(int P) {
  const int pu = round_up(P, 4);
  return ((pu / 4) % 2 == 0) ? pu + 4 : pu;
}

__global__ void __launch_bounds__(128, 8) kattn_query_bwd_kernel(
    const float* __restrict__ phi, int64_t phi_sb, const float* __restrict__ U,
    const float* __restrict__ dout, int64_t dout_sb, float* __restrict__ dphi, int64_t dphi_sb,
    float* __restrict__ dU, int T_R, int R, int P, int nU) {
  extern __shared__ float4 sm4[];
  const int RA = round_up(R, 4), PU = query_pu(P);
  float* su = reinterpret_cast<float*>(sm4);    // [RA][PU] = U_h (zero-padded)
  float* sph = su + RA * PU;                    // [QT_ROWS][RA]
  float* sdo = sph + QT_ROWS * RA;              // [QT_ROWS][PU]
  const int h = blockIdx.x, s = blockIdx.y, tid = threadIdx.x;
  const float* Uh = U + (static_cast<int64_t>(s) * nU + h) * R * P;
  float* dUh = dU + (static_cast<int64_t>(s) * nU + h) * R * P;
  const float* ph = phi + s * phi_sb;
  const float* dos = dout + s * dout_sb;
  const int n_rows = h < T_R ? (T_R - h + nU - 1) / nU : 0;
  if (n_rows == 0) {   // a type without rows: dU_h = 0
    for (int e = tid; e < R * P; e += blockDim.x) dUh[e] = 0.f;
    return;
  }
  for (int e = tid; e < RA * PU; e += blockDim.x) {
    const int r = e / PU, c = e % PU;
    const bool in = r < R && c < P;
    cp_async4(smem_u32(su + e), in ? Uh + r * P + c : Uh, in ? 4u : 0u);
  }
  const int nbp = PU / 4, nblk = (RA / 4) * nbp;
  const bool vec_phi = (R & 3) == 0 && al16d(ph) && ((nU * static_cast<int64_t>(R)) & 3) == 0;
  for (int g0 = 0; g0 < n_rows; g0 += QT_ROWS) {
    const int ng = min(QT_ROWS, n_rows - g0);
    if (g0 > 0) __syncthreads();   // the previous pass has finished with sph / sdo
    if (vec_phi) {
      for (int e = tid * 4; e < QT_ROWS * RA; e += blockDim.x * 4) {
        const int i = e / RA;
        if (i < ng)
          cp_async16(smem_u32(sph + e),
                     ph + static_cast<int64_t>(h + (g0 + i) * static_cast<int64_t>(nU)) * R +
                         e % RA);
        else
          *reinterpret_cast<float4*>(sph + e) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    } else {
      for (int e = tid; e < QT_ROWS * RA; e += blockDim.x) {
        const int i = e / RA, r = e % RA;
        const bool in = i < ng && r < R;
        cp_async4(smem_u32(sph + e),
                  in ? ph + static_cast<int64_t>(h + (g0 + i) * static_cast<int64_t>(nU)) * R + r
                     : ph,
                  in ? 4u : 0u);
      }
    }
    for (int e = tid; e < QT_ROWS * PU; e += blockDim.x) {
      const int i = e / PU, c = e % PU;
      const bool in = i < ng && c < P;
      cp_async4(smem_u32(sdo + e),
                in ? dos + static_cast<int64_t>(h + (g0 + i) * static_cast<int64_t>(nU)) * P + c
                   : dos,
                in ? 4u : 0u);
    }
    cp_async_wait_all();
    __syncthreads();
    // dphi: rows 2 ib, 2 ib + 1 of this pass, r = rb + rl + 16 kk
    const int rl = tid & 15;
    for (int ib = tid >> 4; 2 * ib < ng; ib += blockDim.x >> 4) {
      for (int rb = 0; rb < RA; rb += 64) {
        float o[2][4] = {};
        for (int q = 0; q < PU; q += 4) {
          const float4 d0 = *reinterpret_cast<const float4*>(sdo + (2 * ib) * PU + q);
          const float4 d1 = *reinterpret_cast<const float4*>(sdo + (2 * ib + 1) * PU + q);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const int r = rb + rl + 16 * kk;
            if (r < RA) {
              const float4 u = *reinterpret_cast<const float4*>(su + r * PU + q);
              o[0][kk] += d0.x * u.x + d0.y * u.y + d0.z * u.z + d0.w * u.w;
              o[1][kk] += d1.x * u.x + d1.y * u.y + d1.z * u.z + d1.w * u.w;
            }
          }
        }
#pragma unroll
        for (int a = 0; a < 2; ++a) {
          const int i = 2 * ib + a;
          if (i < ng) {
            float* drow = dphi + s * dphi_sb +
                          static_cast<int64_t>(h + (g0 + i) * static_cast<int64_t>(nU)) * R;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const int r = rb + rl + 16 * kk;
              if (r < R) drow[r] = o[a][kk];
            }
          }
        }
      }
    }
    // dU blocks of this pass
    for (int bk = tid; bk < nblk; bk += blockDim.x) {
      const int r0 = (bk / nbp) * 4, p0 = (bk % nbp) * 4;
      float acc[4][4] = {};
      for (int i = 0; i < ng; ++i) {
        const float4 a = *reinterpret_cast<const float4*>(sph + i * RA + r0);
        const float4 v = *reinterpret_cast<const float4*>(sdo + i * PU + p0);
        const float av[4] = {a.x, a.y, a.z, a.w}, vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int aa = 0; aa < 4; ++aa)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[aa][c] = fmaf(av[aa], vv[c], acc[aa][c]);
      }
#pragma unroll
      for (int aa = 0; aa < 4; ++aa) {
        if (r0 + aa < R) {
          float* drow = dUh + (r0 + aa) * P;
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (p0 + c < P) drow[p0 + c] = g0 == 0 ? acc[aa][c] : drow[p0 + c] + acc[aa][c];
        }
      }
    }
  }
}

cudaStream_t st(void* s) { return static_cast<cudaStream_t>(s); }

int launch_ok() { return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH; }

template <typename K>
int allow_smem(K kernel, int bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) ==
                 cudaSuccess
             ? SMAT_OK
             : SMAT_ERR_LAUNCH;
}

int sum_smem(int C, int R, int P) { return C * (round_up(R, 8) + round_up(P, 4) + P) * 4; }
int expand_smem(int C, int R, int P) {
  const int RA = round_up(R, 8), PB = round_up(P, 8), CS = round_up(C, 8);
  return (RA * CS + PB * CS + 2 * RA * PB) * 4;
}

}  // namespace

extern "C" {

int smat_kattn_chunk_prefix(const float* a, const float* b, float* out, int nb, int T, int C,
                            int R, int P, int nc0, int reverse, void* stream) {
  if (!a || !b || !out) return SMAT_ERR_NULL_POINTER;
  if (nb < 1 || nb > 65535 || T < 1 || C < 1 || R < 1 || P < 1) return SMAT_ERR_BAD_SHAPE;
  const int nc = (T + C - 1) / C;
  if (nc0 < 0 || nc0 > nc || sum_smem(C, R, P) > GLUE_SMEM_MAX) return SMAT_ERR_BAD_SHAPE;
  const int smem = sum_smem(C, R, P);
  int rc = allow_smem(kattn_chunk_sum_kernel, smem);
  if (rc) return rc;
  const int tiles = (round_up(R, 8) / 8) * (round_up(P, 4) / 4);
  const int threads = std::min(256, round_up(tiles, 32));
  kattn_chunk_sum_kernel<<<dim3(nc, nb), threads, smem, st(stream)>>>(a, b, out, T, C, R, P);
  if ((rc = launch_ok())) return rc;
  const int64_t RP = static_cast<int64_t>(R) * P;
  kattn_seg_scan_kernel<<<dim3(static_cast<unsigned>((RP + 255) / 256), nb), 256, 0,
                          st(stream)>>>(out, nc, RP, nc0, reverse ? 1 : 0);
  return launch_ok();
}

int smat_kattn_chunk_expand(const float* a, const float* b, const float* dD, float* da,
                            float* db, int nb, int T, int C, int R, int P, void* stream) {
  if (!a || !b || !dD || !da || !db) return SMAT_ERR_NULL_POINTER;
  if (nb < 1 || nb > 65535 || T < 1 || C < 1 || R < 1 || P < 1) return SMAT_ERR_BAD_SHAPE;
  const int smem = expand_smem(C, R, P);
  if (smem > GLUE_SMEM_MAX) return SMAT_ERR_BAD_SHAPE;
  int rc = allow_smem(kattn_chunk_expand_kernel, smem);
  if (rc) return rc;
  const int nc = (T + C - 1) / C;
  kattn_chunk_expand_kernel<<<dim3(nc, nb), 256, smem, st(stream)>>>(a, b, dD, da, db, T, C, R,
                                                                    P);
  return launch_ok();
}

int smat_kattn_query_by_type(const float* phi, int64_t phi_seq_stride, const float* U,
                             float* out, int64_t out_seq_stride, int nb, int T_R, int R, int P,
                             int nU, int accumulate, void* stream) {
  if (!phi || !U || !out) return SMAT_ERR_NULL_POINTER;
  if (nb < 1 || nb > 65535 || T_R < 0 || R < 1 || P < 1 || nU < 1 || phi_seq_stride < 0 ||
      out_seq_stride < 0)
    return SMAT_ERR_BAD_SHAPE;
  if (T_R == 0) return SMAT_OK;
  const int smem = (round_up(R * P, 4) + QT_ROWS * round_up(R, 4)) * 4;
  if (smem > GLUE_SMEM_MAX) return SMAT_ERR_BAD_SHAPE;
  int rc = allow_smem(kattn_query_kernel, smem);
  if (rc) return rc;
  const int threads = std::min(128, round_up(P, 32));
  kattn_query_kernel<<<dim3(std::min(nU, T_R), nb), threads, smem, st(stream)>>>(
      phi, phi_seq_stride, U, out, out_seq_stride, T_R, R, P, nU, accumulate ? 1 : 0);
  return launch_ok();
}

int smat_kattn_query_by_type_bwd(const float* phi, int64_t phi_seq_stride, const float* U,
                                 const float* dout, int64_t dout_seq_stride, float* dphi,
                                 int64_t dphi_seq_stride, float* dU, int nb, int T_R, int R,
                                 int P, int nU, void* stream) {
  if (!phi || !U || !dout || !dphi || !dU) return SMAT_ERR_NULL_POINTER;
  if (nb < 1 || nb > 65535 || T_R < 0 || R < 1 || P < 1 || nU < 1 || phi_seq_stride < 0 ||
      dout_seq_stride < 0 || dphi_seq_stride < 0)
    return SMAT_ERR_BAD_SHAPE;
  const int RA = round_up(R, 4), PU = query_pu(P);
  const int smem = (RA * PU + QT_ROWS * (RA + PU)) * 4;
  if (smem > GLUE_SMEM_MAX) return SMAT_ERR_BAD_SHAPE;
  int rc = allow_smem(kattn_query_bwd_kernel, smem);
  if (rc) return rc;
  // every type gets a CTA: types without rows write dU_h = 0
  kattn_query_bwd_kernel<<<dim3(nU, nb), 128, smem, st(stream)>>>(
      phi, phi_seq_stride, U, dout, dout_seq_stride, dphi, dphi_seq_stride, dU, T_R, R, P, nU);
  return launch_ok();
}

}  // extern "C"
