// The reference's kernelised-attention schedule (include/smat_kattn.h): the
// fused chunk-local pass on tcgen05 tensor cores (kind::tf32, the precision of
// the reference's TF32 Triton dots) and the long-range pooling / incidence
// passes on CUDA cores (they move far more bytes than they compute).
//
// chunk_local, one CTA per 128-row chunk b:
//   S    = Phi_b Psi_b^T            tcgen05.mma 128 x 128, K = R, both K-major (TMA)
//   S   := tril(S)                  4 warps, thread = row = TMEM lane
//   O    = S Vb_b + Phi_b Sin_b     A = S from TMEM (TS) / Phi from smem (SS),
//                                   B = Vb_b / Sin_b MN-major, N = P rounded to 32
// Vb and Sin rows are P floats (P = d_v + 1 is odd in the reference), which
// TMA cannot describe, so the compute warps copy them with 4-byte cp.async
// (zero-filling the padding) into the MN-major layout tcgen05 takes for tf32:
// the 128-byte swizzle with 32-byte atomicity.
//
// pool:      F[b, x] = sum over j = n_P + x + s N0 < n of Psi[b, j] Vb[b, j]^T
// incidence: U[b, h] = sum over e in [ptr[h], ptr[h+1]) of F[b, idx[e]]
//            (with the transposed table it is its own backward)
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "../../include/smat_b200.h"
#include "../../include/smat_kattn.h"
#include "common.cuh"

namespace {

using namespace smat;

constexpr int KC = 128;   // chunk rows on the tensor-core path

__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4)                                  // D format: f32
         | (2u << 7)                                // A format: tf32
         | (2u << 10)                               // B format: tf32
         | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_tf32_ts(uint32_t d, uint32_t a_tmem, uint64_t b,
                                            uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Shared-memory descriptor of an MN-major 32-bit operand: the 128-byte
// swizzle with 32-byte atomicity (layout type 1), the only MN-major layout
// tcgen05 accepts for tf32.  Rows (K) are 128 bytes apart, a swizzle atom is
// 4 rows (sbo = 512 bytes between atoms along K), `lbo` is the stride between
// 32-column panels along MN.
__device__ __forceinline__ uint64_t sdesc_mn32(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((512u >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(1) << 61;
  return d;
}
// Byte offset of fp32 column c (0..31) of row r in such a panel: 32-byte units
// XOR-ed with the row index mod 4.
__device__ __forceinline__ uint32_t mn32_offset(uint32_t r, uint32_t c) {
  return r * 128u + ((((c >> 3) ^ (r & 3u)) & 3u) << 5) + (c & 7u) * 4u;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

struct ChunkParams {
  const float* vb;     // [n_chunks, KC, P]
  const float* sin;    // [n_chunks, R, P]
  float* out;          // [n_chunks, KC, P]
  int P;
  int32_t* err;
};

// R: feature width (K of S and of Phi Sin); PN: P rounded up to 32.
template <int R, int PN>
struct ChunkCfg {
  static constexpr int PANEL = KC * 128;                 // 32 fp32 columns x 128 rows
  static constexpr int KR = R / 32;                      // K-major panels of Phi / Psi
  static constexpr int OFF_PHI = 0;
  static constexpr int OFF_PSI = OFF_PHI + KR * PANEL;
  static constexpr int VB_PANEL = KC * 128;              // Vb: 128 K-rows x 32 columns
  static constexpr int SIN_PANEL = R * 128;              // Sin: R K-rows x 32 columns
  static constexpr int OFF_VB = OFF_PSI + KR * PANEL;
  static constexpr int OFF_SIN = OFF_VB + (PN / 32) * VB_PANEL;
  static constexpr int OFF_BAR = OFF_SIN + (PN / 32) * SIN_PANEL;
  // barriers: phi/psi full, vb/sin full (128 arrivals), s full, s masked (4), o full
  static constexpr int BAR_QK = 0, BAR_VS = 1, BAR_SF = 2, BAR_SM = 3, BAR_OF = 4, NBAR = 5;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static constexpr int COL_S = 0, COL_O = 128;
  static constexpr int TMEM_COLS = 256;
  static_assert(COL_O + PN <= TMEM_COLS, "TMEM budget");
  static constexpr uint32_t IDESC_S = idesc_tf32(128, 128, false, false);
  static constexpr uint32_t IDESC_O = idesc_tf32(128, PN, false, true);
};

// 192 threads: warps 0-3 copy Vb / Sin, mask S and store O (thread = row);
// warp 4 issues the TMA loads; warp 5 allocates TMEM and issues the MMAs.
template <int R, int PN>
__global__ void __launch_bounds__(192, 1)
    kattn_chunk_fwd_kernel(const __grid_constant__ CUtensorMap tm_phi,
                           const __grid_constant__ CUtensorMap tm_psi, const ChunkParams p) {
  using C = ChunkCfg<R, PN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto bar = [&](int i) { return bar0 + 8u * i; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t chunk = blockIdx.x;

  if (tid == 0) {
    mbar_init(bar(C::BAR_QK), 1);
    mbar_init(bar(C::BAR_VS), 128);
    mbar_init(bar(C::BAR_SF), 1);
    mbar_init(bar(C::BAR_SM), 4);
    mbar_init(bar(C::BAR_OF), 1);
    fence_barrier_init();
    misc[1] = 0;
  }
  if (warp == 5) {
    tmem_alloc(sbase + C::OFF_MISC, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = misc[0];

  if (warp == 4) {
    if (lane == 0) {
      mbar_expect_tx(bar(C::BAR_QK), 2 * C::KR * C::PANEL);
      const int row0 = static_cast<int>(chunk * KC);
#pragma unroll
      for (int k = 0; k < C::KR; ++k) {
        tma_load_2d(sbase + C::OFF_PHI + k * C::PANEL, &tm_phi, bar(C::BAR_QK), 32 * k, row0);
        tma_load_2d(sbase + C::OFF_PSI + k * C::PANEL, &tm_psi, bar(C::BAR_QK), 32 * k, row0);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      bool ok = mbar_wait(bar(C::BAR_QK), 0, abort_flag, p.err);
      if (ok) {
        tc_fence_after();
        // S = Phi Psi^T: K = R in steps of 8 (32 bytes of a 128-byte row)
#pragma unroll
        for (int kk = 0; kk < R / 8; ++kk) {
          const uint32_t off = (kk >> 2) * C::PANEL + (kk & 3) * 32;
          mma_tf32(tbase + C::COL_S, sdesc_sw128(sbase + C::OFF_PHI + off, 16, 1024),
                   sdesc_sw128(sbase + C::OFF_PSI + off, 16, 1024), C::IDESC_S, kk > 0);
        }
        tc_commit(bar(C::BAR_SF));
        ok = mbar_wait(bar(C::BAR_VS), 0, abort_flag, p.err);
      }
      if (ok) {
        tc_fence_after();
        // O = Phi Sin (SS): B = Sin, MN-major, 8 K-rows (one 1024-byte atom) per step
#pragma unroll
        for (int kk = 0; kk < R / 8; ++kk) {
          const uint32_t off = (kk >> 2) * C::PANEL + (kk & 3) * 32;
          mma_tf32(tbase + C::COL_O, sdesc_sw128(sbase + C::OFF_PHI + off, 16, 1024),
                   sdesc_mn32(sbase + C::OFF_SIN + kk * 1024, C::SIN_PANEL), C::IDESC_O,
                   kk > 0);
        }
        ok = mbar_wait(bar(C::BAR_SM), 0, abort_flag, p.err);
      }
      if (ok) {
        tc_fence_after();
        // O += tril(S) Vb (TS): A = S from TMEM, 8 columns per step
#pragma unroll 4
        for (int kk = 0; kk < KC / 8; ++kk)
          mma_tf32_ts(tbase + C::COL_O, tbase + C::COL_S + 8 * kk,
                      sdesc_mn32(sbase + C::OFF_VB + kk * 1024, C::VB_PANEL), C::IDESC_O, 1u);
        tc_commit(bar(C::BAR_OF));
      }
      if (*abort_flag) {   // let issued MMAs finish before TMEM is freed
        tc_commit(bar(C::BAR_OF));
        mbar_wait_drain(bar(C::BAR_OF), 0);
      }
    }
  } else {
    // ---------------------------------------------------------------- warps 0-3
    const int r = warp * 32 + lane;      // chunk row = TMEM lane
    // Vb [KC x P] and Sin [R x P] into MN-major SW128 panels of 32 columns
    const float* vb = p.vb + chunk * KC * p.P;
    const float* sn = p.sin + chunk * R * p.P;
    for (int c = 0; c < PN; ++c) {
      const uint32_t dst = sbase + C::OFF_VB + (c >> 5) * C::VB_PANEL + mn32_offset(r, c & 31);
      cp_async4(dst, vb + static_cast<int64_t>(r) * p.P + (c < p.P ? c : 0), c < p.P ? 4u : 0u);
    }
    for (int kr = r; kr < R; kr += 128)
      for (int c = 0; c < PN; ++c) {
        const uint32_t dst = sbase + C::OFF_SIN + (c >> 5) * C::SIN_PANEL + mn32_offset(kr, c & 31);
        cp_async4(dst, sn + static_cast<int64_t>(kr) * p.P + (c < p.P ? c : 0),
                  c < p.P ? 4u : 0u);
      }
    asm volatile("cp.async.wait_all;" ::: "memory");
    fence_proxy_async_smem();
    mbar_arrive(bar(C::BAR_VS));
    const uint32_t lane_base = tbase + (static_cast<uint32_t>(warp * 32) << 16);
    bool alive = __all_sync(0xffffffffu, mbar_wait(bar(C::BAR_SF), 0, abort_flag, p.err));
    if (alive) {
      tc_fence_after();
      // keep S[r, j] for j <= r: 32-column blocks past the diagonal become 0
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
        if (32 * q > warp * 32 + 31) {
          float z[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) z[i] = 0.f;
          tmem_st32(lane_base + C::COL_S + 32 * q, z);
        } else if (q == warp) {
          float s[32];
          tmem_ld32(lane_base + C::COL_S + 32 * q, s);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (32 * q + i > r) s[i] = 0.f;
          tmem_st32(lane_base + C::COL_S + 32 * q, s);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C::BAR_SM));
      alive = __all_sync(0xffffffffu, mbar_wait(bar(C::BAR_OF), 0, abort_flag, p.err));
    }
    if (alive) {
      tc_fence_after();
      float* orow = p.out + (chunk * KC + r) * p.P;
#pragma unroll 1
      for (int c0 = 0; c0 < PN; c0 += 32) {
        float o[32];
        tmem_ld32(lane_base + C::COL_O + c0, o);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c0 + i < p.P) orow[c0 + i] = o[i];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- pool
// One CTA per (profile x, b); 256 threads, each accumulating R P / 256 outputs
// (16 for R = 64, P = 65) over the profile's columns, staged 32 at a time.
__global__ void __launch_bounds__(256) kattn_pool_kernel(const float* __restrict__ psi,
                                                         const float* __restrict__ vb,
                                                         float* __restrict__ F, int T, int R,
                                                         int P, int n_P, int n, int N0) {
  extern __shared__ float stage[];   // [32][R] psi rows, then [32][P] vb rows
  const int x = blockIdx.x, b = blockIdx.y;
  float* sp = stage;
  float* sv = stage + 32 * R;
  const int RP = R * P;
  constexpr int MAXO = 64;            // outputs per thread (R P <= 16384)
  float acc[MAXO];
#pragma unroll
  for (int i = 0; i < MAXO; ++i) acc[i] = 0.f;
  const int n_X = n - n_P;
  const int g = (n_X - x + N0 - 1) / N0;   // columns of this profile
  const float* pb = psi + static_cast<int64_t>(b) * T * R;
  const float* vbb = vb + static_cast<int64_t>(b) * T * P;
  for (int s0 = 0; s0 < g; s0 += 32) {
    const int ns = min(32, g - s0);
    __syncthreads();
    for (int e = threadIdx.x; e < ns * R; e += blockDim.x) {
      const int s = e / R, c = e % R;
      sp[s * R + c] = pb[static_cast<int64_t>(n_P + x + (s0 + s) * N0) * R + c];
    }
    for (int e = threadIdx.x; e < ns * P; e += blockDim.x) {
      const int s = e / P, c = e % P;
      sv[s * P + c] = vbb[static_cast<int64_t>(n_P + x + (s0 + s) * N0) * P + c];
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < MAXO; ++i) {
      const int o = threadIdx.x + i * 256;
      if (o < RP) {
        const int rr = o / P, pp = o % P;
        float a = acc[i];
        for (int s = 0; s < ns; ++s) a = fmaf(sp[s * R + rr], sv[s * P + pp], a);
        acc[i] = a;
      }
    }
  }
  float* fo = F + (static_cast<int64_t>(b) * N0 + x) * RP;
#pragma unroll
  for (int i = 0; i < MAXO; ++i) {
    const int o = threadIdx.x + i * 256;
    if (o < RP) fo[o] = acc[i];
  }
}

// For every column j of profile x: dpsi_j = dF_x vb_j, dvb_j = dF_x^T psi_j.
// One CTA per (x, b), dF_x staged in shared memory.
__global__ void __launch_bounds__(256) kattn_pool_bwd_kernel(
    const float* __restrict__ psi, const float* __restrict__ vb, const float* __restrict__ dF,
    float* __restrict__ dpsi, float* __restrict__ dvb, int T, int R, int P, int n_P, int n,
    int N0) {
  extern __shared__ float sdf[];   // [R][P]
  const int x = blockIdx.x, b = blockIdx.y;
  const int RP = R * P;
  const float* df = dF + (static_cast<int64_t>(b) * N0 + x) * RP;
  for (int e = threadIdx.x; e < RP; e += blockDim.x) sdf[e] = df[e];
  __syncthreads();
  const int n_X = n - n_P;
  const int g = (n_X - x + N0 - 1) / N0;
  for (int s = 0; s < g; ++s) {
    const int64_t j = static_cast<int64_t>(b) * T + n_P + x + s * N0;
    const float* pr = psi + j * R;
    const float* vr = vb + j * P;
    for (int rr = threadIdx.x; rr < R; rr += blockDim.x) {
      float a = 0.f;
      for (int pp = 0; pp < P; ++pp) a = fmaf(sdf[rr * P + pp], vr[pp], a);
      dpsi[j * R + rr] = a;
    }
    for (int pp = threadIdx.x; pp < P; pp += blockDim.x) {
      float a = 0.f;
      for (int rr = 0; rr < R; ++rr) a = fmaf(sdf[rr * P + pp], pr[rr], a);
      dvb[j * P + pp] = a;
    }
  }
}

// ---------------------------------------------------------------- incidence
// U[b, h, :] = sum over the CSR row h of F[b, idx, :].  Grid (H rows, nb,
// RP / 1024): the RP tile is the slowest axis, so CTAs resident together read
// one slice of F, which L2 then serves for all its uses.
__global__ void __launch_bounds__(256) kattn_incidence_kernel(
    const float* __restrict__ F, const int64_t* __restrict__ ptr, const int32_t* __restrict__ idx,
    float* __restrict__ U, int N_in, int N_out, int RP, int32_t* err) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int o0 = blockIdx.z * 1024 + threadIdx.x * 4;
  const int64_t e0 = ptr[h], e1 = ptr[h + 1];
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const bool vec = (RP & 3) == 0;
  float sacc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t e = e0; e < e1; ++e) {
    const int x = idx[e];
    if (x < 0 || x >= N_in) {
      if (threadIdx.x == 0 && err) atomicOr(err, SMAT_DEVERR_BAD_CSR);
      continue;
    }
    const float* src = F + (static_cast<int64_t>(b) * N_in + x) * RP;
    if (vec) {
      if (o0 + 3 < RP) {
        const float4 v = *reinterpret_cast<const float4*>(src + o0);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (o0 + i < RP) sacc[i] += src[o0 + i];
    }
  }
  float* dst = U + (static_cast<int64_t>(b) * N_out + h) * RP;
  if (vec) {
    if (o0 + 3 < RP) *reinterpret_cast<float4*>(dst + o0) = acc;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (o0 + i < RP) dst[o0 + i] = sacc[i];
  }
}

// ---------------------------------------------------------------- host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 2-D fp32 map over [rows, R], box {32, 128}, 128-byte swizzle
int map_rows(CUtensorMap* m, const float* base, int64_t rows, int R) {
  auto enc = encode_fn();
  if (!enc) return SMAT_ERR_NO_DEVICE;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(R), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(R) * 4};
  cuuint32_t box[2] = {32, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SMAT_OK : SMAT_ERR_TMA_DESCRIPTOR;
}

template <int R, int PN>
int chunk_fwd_launch(const CUtensorMap& mphi, const CUtensorMap& mpsi, const ChunkParams& p,
                     int64_t n_chunks, cudaStream_t s) {
  using C = ChunkCfg<R, PN>;
  auto kern = kattn_chunk_fwd_kernel<R, PN>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) !=
      cudaSuccess)
    return SMAT_ERR_LAUNCH;
  kern<<<static_cast<unsigned>(n_chunks), 192, C::SMEM_BYTES, s>>>(mphi, mpsi, p);
  return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH;
}

template <int R>
int chunk_fwd_p(const CUtensorMap& a, const CUtensorMap& b, const ChunkParams& p, int64_t nc,
                cudaStream_t s) {
  const int pn = (p.P + 31) / 32 * 32;
  switch (pn) {
    case 32: return chunk_fwd_launch<R, 32>(a, b, p, nc, s);
    case 64: return chunk_fwd_launch<R, 64>(a, b, p, nc, s);
    case 96: return chunk_fwd_launch<R, 96>(a, b, p, nc, s);
    case 128:
      // R = 128 with P > 96 exceeds the shared memory (four 64 KB operands)
      if constexpr (R < 128) return chunk_fwd_launch<R, 128>(a, b, p, nc, s);
      break;
  }
  return SMAT_ERR_BAD_SHAPE;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int smat_kattn_chunk_local_fwd(const float* phi, const float* psi, const float* vb,
                               const float* sin_, float* out, int64_t n_chunks, int C, int R,
                               int P, int32_t* err_word, void* stream) {
  if (!phi || !psi || !vb || !sin_ || !out) return SMAT_ERR_NULL_POINTER;
  if (C != KC || (R != 32 && R != 64 && R != 128) || P < 1 || P > (R == 128 ? 96 : 128) ||
      n_chunks < 0 || n_chunks > 0x7FFFFFFF / KC)
    return SMAT_ERR_BAD_SHAPE;
  if (!al16(phi) || !al16(psi)) return SMAT_ERR_BAD_ALIGNMENT;
  if (n_chunks == 0) return SMAT_OK;
  CUtensorMap mphi, mpsi;
  int rc;
  if ((rc = map_rows(&mphi, phi, n_chunks * KC, R))) return rc;
  if ((rc = map_rows(&mpsi, psi, n_chunks * KC, R))) return rc;
  ChunkParams p{vb, sin_, out, P, err_word};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (R) {
    case 32: return chunk_fwd_p<32>(mphi, mpsi, p, n_chunks, s);
    case 64: return chunk_fwd_p<64>(mphi, mpsi, p, n_chunks, s);
    default: return chunk_fwd_p<128>(mphi, mpsi, p, n_chunks, s);
  }
}

int smat_kattn_pool_fwd(const float* psi, const float* vb, float* F, int nb, int T, int R, int P,
                        int n_P, int n, int N0, void* stream) {
  if (!psi || !vb || !F) return SMAT_ERR_NULL_POINTER;
  if (nb < 1 || T < 1 || R < 1 || P < 1 || R * P > 64 * 256 || N0 < 1 || n_P < 0 ||
      n < n_P || n > T)
    return SMAT_ERR_BAD_SHAPE;
  const int bytes = 32 * (R + P) * 4;
  if (bytes > 96 * 1024) return SMAT_ERR_BAD_SHAPE;
  if (cudaFuncSetAttribute(kattn_pool_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           96 * 1024) != cudaSuccess)
    return SMAT_ERR_LAUNCH;
  kattn_pool_kernel<<<dim3(N0, nb), 256, bytes, static_cast<cudaStream_t>(stream)>>>(
      psi, vb, F, T, R, P, n_P, n, N0);
  return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH;
}

int smat_kattn_pool_bwd(const float* psi, const float* vb, const float* dF, float* dpsi,
                        float* dvb, int nb, int T, int R, int P, int n_P, int n, int N0,
                        void* stream) {
  if (!psi || !vb || !dF || !dpsi || !dvb) return SMAT_ERR_NULL_POINTER;
  if (nb < 1 || T < 1 || R < 1 || P < 1 || N0 < 1 || n_P < 0 || n < n_P || n > T)
    return SMAT_ERR_BAD_SHAPE;
  const int bytes = R * P * 4;
  if (bytes > 96 * 1024) return SMAT_ERR_BAD_SHAPE;
  if (cudaFuncSetAttribute(kattn_pool_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           96 * 1024) != cudaSuccess)
    return SMAT_ERR_LAUNCH;
  kattn_pool_bwd_kernel<<<dim3(N0, nb), 256, bytes, static_cast<cudaStream_t>(stream)>>>(
      psi, vb, dF, dpsi, dvb, T, R, P, n_P, n, N0);
  return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH;
}

int smat_kattn_incidence(const float* F, const int64_t* ptr, const int32_t* idx, float* U,
                         int nb, int N_in, int N_out, int RP, int32_t* err_word, void* stream) {
  if (!F || !ptr || !U) return SMAT_ERR_NULL_POINTER;
  if (nb < 1 || N_in < 1 || N_out < 1 || RP < 1 || nb > 65535) return SMAT_ERR_BAD_SHAPE;
  if ((RP & 3) == 0 && (!al16(F) || !al16(U))) return SMAT_ERR_BAD_ALIGNMENT;
  const dim3 grid(N_out, nb, (RP + 1023) / 1024);
  kattn_incidence_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      F, ptr, idx, U, N_in, N_out, RP, err_word);
  return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH;
}

}  // extern "C"
