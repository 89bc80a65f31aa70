// The reference's kernelised-attention schedule (include/smat_kattn.h): the
// fused chunk-local pass on tcgen05 tensor cores (kind::tf32, the precision of
// the reference's TF32 Triton dots) and the long-range pooling / incidence
// passes on CUDA cores (they move far more bytes than they compute).
//
// chunk_local, one CTA per 128-row chunk b (kattn_tile_kernel, mode FWD):
//   S    = Phi_b Psi_b^T            tcgen05.mma 128 x 128, K = R, both K-major (TMA)
//   S   := tril(S)                  4 warps, thread = row = TMEM lane
//   O    = S Vb_b + Phi_b Sin_b     A = S from TMEM (TS) / Phi from smem (SS),
//                                   B = Vb_b / Sin_b MN-major, N = P rounded to 32
// and its backward in three more modes of the same kernel (dPhi, dVb, dPsi).
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

// One 128-row chunk tile, four modes sharing one pipeline:
//   G   = A1 B1^T                     128 x 128, K = K1, both K-major
//   G  := mask(G)                     lower (j <= i) or upper (j >= i) triangle
//   OUT = [A1 EX] + G B2              B2 MN-major (32-byte atoms), N = NO
//
//   mode  A1        B1        mask   EX (SS term)      B2    OUT
//   FWD   Phi (T)   Psi (T)   lower  Phi Sin (MN)      Vb    out  = Phi Sin + tril(Phi Psi^T) Vb
//   DPHI  dO (c)    Vb (c)    lower  dO Sin^T (K)      Psi   dPhi = dO Sin^T + tril(dO Vb^T) Psi
//   DV    Psi (T)   Phi (T)   upper  -                 dO    dVb  = tril(Phi Psi^T)^T dO
//   DPSI  Vb (c)    dO (c)    upper  -                 Phi   dPsi = tril(dO Vb^T)^T Phi
// (T: TMA from [rows, R]; c: 4-byte cp.async from rows of P floats, zero-padded
// to PN.)  Phi / Psi as B2 come by TMA in the 32-byte-atom swizzle.
enum : int { TM_FWD = 0, TM_DPHI = 1, TM_DV = 2, TM_DPSI = 3 };

struct TileParams {
  const float* vb;     // [n_chunks, KC, P]
  const float* sin;    // [n_chunks, R, P]
  const float* dout;   // [n_chunks, KC, P]
  float* out;          // [n_chunks, KC, n_store]
  int P, n_store;
  int32_t* err;
};

template <int MODE, int R, int PN>
struct TileCfg {
  static constexpr bool KR_G1 = MODE == TM_FWD || MODE == TM_DV;     // G contracts over R
  static constexpr int K1 = KR_G1 ? R : PN;
  static constexpr int NO = KR_G1 ? PN : R;                           // OUT columns (padded)
  static constexpr bool EXTRA = MODE == TM_FWD || MODE == TM_DPHI;
  static constexpr bool LOWER = MODE == TM_FWD || MODE == TM_DPHI;
  static constexpr int PANEL = KC * 128;                 // 128 rows x 32 fp32
  static constexpr int EX_PANEL = R * 128;               // R rows x 32 fp32
  static constexpr int SZ_A1 = (K1 / 32) * PANEL, SZ_B1 = SZ_A1, SZ_B2 = (NO / 32) * PANEL;
  static constexpr int SZ_EX = EXTRA ? (PN / 32) * EX_PANEL : 0;
  // barriers: TMA full, copies full (128 arrivals), G full, G masked (4), OUT
  // full, B2 full (the late B2 of the aliased layout)
  static constexpr int BAR_TMA = 0, BAR_CP = 1, BAR_SF = 2, BAR_SM = 3, BAR_OF = 4, BAR_B2 = 5,
                       NBAR = 6;
  static constexpr int TAIL = NBAR * 8 + 16 + 1024;   // barriers, misc, alignment slack
  // Two CTAs per SM need <= 113 KB each.  B2 is read only by the last MMA
  // group, B1 only by the first: where that brings the layout under the
  // limit, B2 is loaded over B1 once G has been computed (the other CTA on
  // the SM covers the load).
  static constexpr int CAP2 = 113 * 1024;
  static constexpr int PLAIN = SZ_A1 + SZ_B1 + SZ_B2 + SZ_EX + TAIL;
  static constexpr int SZ_B12 = SZ_B1 > SZ_B2 ? SZ_B1 : SZ_B2;
  static constexpr bool ALIAS = PLAIN > CAP2 && SZ_A1 + SZ_B12 + SZ_EX + TAIL <= CAP2;
  static constexpr int OFF_A1 = 0;
  static constexpr int OFF_B1 = OFF_A1 + SZ_A1;
  static constexpr int OFF_B2 = ALIAS ? OFF_B1 : OFF_B1 + SZ_B1;
  static constexpr int OFF_EX = OFF_B1 + (ALIAS ? SZ_B12 : SZ_B1 + SZ_B2);
  static constexpr int OFF_BAR = OFF_EX + SZ_EX;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static constexpr int MIN_BLOCKS = SMEM_BYTES <= CAP2 ? 2 : 1;
  // OUT is staged in the operand tiles: KC rows at a stride of NO + 1 words
  static constexpr int STAGE_LD = NO + 1;
  static_assert(KC * STAGE_LD * 4 <= OFF_BAR, "OUT staging");
  static constexpr int COL_G = 0, COL_O = 128, TMEM_COLS = 256;
  static_assert(COL_O + NO <= TMEM_COLS, "TMEM budget");
  // bytes the producer's TMA loads bring
  static constexpr int TMA_BYTES = KR_G1 ? 2 * (K1 / 32) * PANEL : (NO / 32) * PANEL;
  static constexpr uint32_t IDESC_G = idesc_tf32(128, 128, false, false);
  static constexpr uint32_t IDESC_O = idesc_tf32(128, NO, false, true);
  static constexpr uint32_t IDESC_EX = idesc_tf32(128, NO, false, MODE == TM_FWD);
};

// rows [0, nrows) x PN fp32 columns of `src` (row stride P, the rows
// contiguous) into a K-major SWIZZLE_128B tile (panels of nrows x 32).  Thread
// t of nt copies elements t, t + nt, ... of the run, so a warp's 32 copies
// read 32 consecutive floats (columns past P are zero-filled).
template <int PN>
__device__ __forceinline__ void cp_kmajor(uint32_t dst, const float* src, int t, int nt,
                                          int nrows, int P) {
  for (int e = t; e < nrows * PN; e += nt) {
    const int row = e / PN, k = e % PN;
    cp_async4(dst + (k >> 5) * (nrows * 128) + sw128_offset(row, (k & 31) >> 2) + (k & 3) * 4,
              src + static_cast<int64_t>(row) * P + (k < P ? k : 0), k < P ? 4u : 0u);
  }
}
// the same rows into an MN-major tile with 32-byte swizzle atoms (rows = K)
template <int PN>
__device__ __forceinline__ void cp_mn32(uint32_t dst, const float* src, int t, int nt, int nrows,
                                        int P) {
  for (int e = t; e < nrows * PN; e += nt) {
    const int row = e / PN, c = e % PN;
    cp_async4(dst + (c >> 5) * (nrows * 128) + mn32_offset(row, c & 31),
              src + static_cast<int64_t>(row) * P + (c < P ? c : 0), c < P ? 4u : 0u);
  }
}

// 192 threads: warps 0-3 copy the cp.async operands, mask G and store OUT
// (thread = row = TMEM lane); warp 4 issues the TMA loads; warp 5 allocates
// TMEM and issues the MMAs.
template <int MODE, int R, int PN>
__global__ void __launch_bounds__(192, (TileCfg<MODE, R, PN>::MIN_BLOCKS))
    kattn_tile_kernel(const __grid_constant__ CUtensorMap tm0,
                      const __grid_constant__ CUtensorMap tm1, const TileParams p) {
  using C = TileCfg<MODE, R, PN>;
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
    mbar_init(bar(C::BAR_TMA), 1);
    mbar_init(bar(C::BAR_CP), 128);
    mbar_init(bar(C::BAR_SF), 1);
    mbar_init(bar(C::BAR_SM), 4);
    mbar_init(bar(C::BAR_OF), 1);
    mbar_init(bar(C::BAR_B2), C::KR_G1 ? 128 : 1);   // compute warps' copies, or TMA
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
      mbar_expect_tx(bar(C::BAR_TMA), C::TMA_BYTES);
      const int row0 = static_cast<int>(chunk * KC);
      if (C::KR_G1) {          // A1, B1 from the two K-major maps
#pragma unroll
        for (int k = 0; k < C::K1 / 32; ++k) {
          tma_load_2d(sbase + C::OFF_A1 + k * C::PANEL, &tm0, bar(C::BAR_TMA), 32 * k, row0);
          tma_load_2d(sbase + C::OFF_B1 + k * C::PANEL, &tm1, bar(C::BAR_TMA), 32 * k, row0);
        }
      } else if (!C::ALIAS) {  // B2 from the 32-byte-atom map
#pragma unroll
        for (int k = 0; k < C::NO / 32; ++k)
          tma_load_2d(sbase + C::OFF_B2 + k * C::PANEL, &tm0, bar(C::BAR_TMA), 32 * k, row0);
      } else if (mbar_wait(bar(C::BAR_SF), 0, abort_flag, p.err)) {
        // aliased: B2 over B1 once G (the only reader of B1) has completed
        tc_fence_after();
        mbar_expect_tx(bar(C::BAR_B2), C::SZ_B2);
#pragma unroll
        for (int k = 0; k < C::NO / 32; ++k)
          tma_load_2d(sbase + C::OFF_B2 + k * C::PANEL, &tm0, bar(C::BAR_B2), 32 * k, row0);
        mbar_wait_drain(bar(C::BAR_B2), 0);   // never exit with the load in flight
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // (the aliased layouts without TMA operands before G load nothing there)
      bool ok = ((!C::KR_G1 && C::ALIAS) || mbar_wait(bar(C::BAR_TMA), 0, abort_flag, p.err)) &&
                mbar_wait(bar(C::BAR_CP), 0, abort_flag, p.err);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C::K1 / 8; ++kk) {
          const uint32_t off = (kk >> 2) * C::PANEL + (kk & 3) * 32;
          mma_tf32(tbase + C::COL_G, sdesc_sw128(sbase + C::OFF_A1 + off, 16, 1024),
                   sdesc_sw128(sbase + C::OFF_B1 + off, 16, 1024), C::IDESC_G, kk > 0);
        }
        tc_commit(bar(C::BAR_SF));
        if (C::EXTRA) {
          // FWD: Phi (A1, K = R) x Sin (MN-major); DPHI: dO (A1, K = PN) x Sin^T (K-major)
#pragma unroll
          for (int kk = 0; kk < C::K1 / 8; ++kk) {
            const uint32_t off = (kk >> 2) * C::PANEL + (kk & 3) * 32;
            const uint64_t bd =
                MODE == TM_FWD
                    ? sdesc_mn32(sbase + C::OFF_EX + kk * 1024, C::EX_PANEL)
                    : sdesc_sw128(sbase + C::OFF_EX + (kk >> 2) * C::EX_PANEL + (kk & 3) * 32, 16,
                                  1024);
            mma_tf32(tbase + C::COL_O, sdesc_sw128(sbase + C::OFF_A1 + off, 16, 1024), bd,
                     C::IDESC_EX, kk > 0);
          }
        }
        ok = mbar_wait(bar(C::BAR_SM), 0, abort_flag, p.err) &&
             (!C::ALIAS || mbar_wait(bar(C::BAR_B2), 0, abort_flag, p.err));
      }
      if (ok) {
        tc_fence_after();
        // OUT += mask(G) B2 (TS): A = G from TMEM, 8 columns per step
#pragma unroll 4
        for (int kk = 0; kk < KC / 8; ++kk)
          mma_tf32_ts(tbase + C::COL_O, tbase + C::COL_G + 8 * kk,
                      sdesc_mn32(sbase + C::OFF_B2 + kk * 1024, C::PANEL), C::IDESC_O,
                      (C::EXTRA || kk > 0) ? 1u : 0u);
        tc_commit(bar(C::BAR_OF));
      }
      if (*abort_flag) {   // let issued MMAs finish before TMEM is freed
        tc_commit(bar(C::BAR_OF));
        mbar_wait_drain(bar(C::BAR_OF), 0);
      }
    }
  } else {
    // ---------------------------------------------------------------- warps 0-3
    const int r = warp * 32 + lane;      // tile row = TMEM lane
    const int64_t rows_off = chunk * KC * p.P;
    const float* vb = p.vb + rows_off;
    const float* dO = p.dout + rows_off;
    const float* sn = p.sin + chunk * R * p.P;
    if (MODE == TM_FWD) {
      if (!C::ALIAS) cp_mn32<PN>(sbase + C::OFF_B2, vb, r, 128, KC, p.P);
      cp_mn32<PN>(sbase + C::OFF_EX, sn, r, 128, R, p.P);
    } else if (MODE == TM_DPHI) {
      cp_kmajor<PN>(sbase + C::OFF_A1, dO, r, 128, KC, p.P);
      cp_kmajor<PN>(sbase + C::OFF_B1, vb, r, 128, KC, p.P);
      cp_kmajor<PN>(sbase + C::OFF_EX, sn, r, 128, R, p.P);
    } else if (MODE == TM_DV) {
      if (!C::ALIAS) cp_mn32<PN>(sbase + C::OFF_B2, dO, r, 128, KC, p.P);
    } else {
      cp_kmajor<PN>(sbase + C::OFF_A1, vb, r, 128, KC, p.P);
      cp_kmajor<PN>(sbase + C::OFF_B1, dO, r, 128, KC, p.P);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    fence_proxy_async_smem();
    mbar_arrive(bar(C::BAR_CP));
    const uint32_t lane_base = tbase + (static_cast<uint32_t>(warp * 32) << 16);
    bool alive = __all_sync(0xffffffffu, mbar_wait(bar(C::BAR_SF), 0, abort_flag, p.err));
    if (alive) {
      tc_fence_after();
      // aliased FWD / DV: B2 over B1, which G has read; the copies overlap
      // the masking below
      if (C::ALIAS && C::KR_G1) cp_mn32<PN>(sbase + C::OFF_B2, MODE == TM_FWD ? vb : dO, r, 128,
                                            KC, p.P);
      // lower: keep G[r, j] for j <= r; upper: keep j >= r
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
        const bool all_out = C::LOWER ? q > warp : q < warp;
        if (all_out) {
          float z[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) z[i] = 0.f;
          tmem_st32(lane_base + C::COL_G + 32 * q, z);
        } else if (q == warp) {
          float g[32];
          tmem_ld32(lane_base + C::COL_G + 32 * q, g);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (C::LOWER ? (32 * q + i > r) : (32 * q + i < r)) g[i] = 0.f;
          tmem_st32(lane_base + C::COL_G + 32 * q, g);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C::BAR_SM));
      if (C::ALIAS && C::KR_G1) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        fence_proxy_async_smem();
        mbar_arrive(bar(C::BAR_B2));
      }
      alive = __all_sync(0xffffffffu, mbar_wait(bar(C::BAR_OF), 0, abort_flag, p.err));
    }
    // OUT leaves through shared memory (every operand tile is free once the
    // last MMA has completed): each thread writes its row at a stride of
    // NO + 1 words (no bank conflicts), then the four warps copy the chunk's
    // contiguous [KC, n_store] block to global memory in coalesced stores.
    float* stg = reinterpret_cast<float*>(smem + C::OFF_A1);
    if (alive) {
      tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < C::NO; c0 += 32) {
        float o[32];
        tmem_ld32(lane_base + C::COL_O + c0, o);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c0 + i < p.n_store) stg[r * C::STAGE_LD + c0 + i] = o[i];
      }
    }
    named_barrier_sync(1, 128);
    if (alive) {
      float* dst = p.out + chunk * KC * p.n_store;
      int row = r / p.n_store, col = r % p.n_store;
      const int step_rows = 128 / p.n_store, step_cols = 128 % p.n_store;
      for (int e = r; e < KC * p.n_store; e += 128) {
        dst[e] = stg[row * C::STAGE_LD + col];
        row += step_rows;
        col += step_cols;
        if (col >= p.n_store) {
          col -= p.n_store;
          ++row;
        }
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
// One CTA per (profile x, b).  The profile's columns (about n_X / N0, 16 at
// c3 sizes) are staged in shared memory -- psi rows [mg][RR] and vb rows
// [mg][SP], mg = that count rounded up to 4 (at most POOL_MAXG), zero-padded
// to multiples of 4 -- and each thread
// accumulates 4 x 4 tiles of the R x P outer-product sum in registers (two
// 16-byte shared loads per 16 FMAs, columns in order, so the sum is the same
// sequence of fmaf as a scalar loop).  The tile goes back to global memory
// through shared memory as one contiguous run of R P floats.
constexpr int POOL_MAXG = 64;   // columns staged per round at most
constexpr int POOL_SMEM_MAX = 200 * 1024;

// columns staged per round: a profile's column count, rounded up to 4, up to
// POOL_MAXG (shared memory sized to it, so more CTAs share an SM)
inline int pool_round(int n_P, int n, int N0) {
  const int gmax = std::max(1, std::min(POOL_MAXG, (n - n_P + N0 - 1) / N0));
  return (gmax + 3) & ~3;
}

// Row stride of a zero-padded shared row of P floats: a multiple of 4 whose
// count of 16-byte units is odd, so 8 consecutive rows hit 8 distinct bank
// groups.
__host__ __device__ inline int pool_stride(int P) {
  int sp = (P + 3) & ~3;
  if (((sp >> 2) & 1) == 0) sp += 4;
  return sp;
}

__global__ void __launch_bounds__(256) kattn_pool_kernel(const float* __restrict__ psi,
                                                         const float* __restrict__ vb,
                                                         float* __restrict__ F, int T, int R,
                                                         int P, int n_P, int n, int N0, int mg) {
  extern __shared__ float4 stage4[];   // psi [MAXG][RR] | vb [MAXG][SP] | F_x [RR][SP]
  float* stage = reinterpret_cast<float*>(stage4);
  const int x = blockIdx.x, b = blockIdx.y;
  const int RR = (R + 3) & ~3, SP = pool_stride(P);
  float* sp = stage;
  float* sv = sp + mg * RR;
  float* so = sv + mg * SP;
  const int RP = R * P;
  const int n_X = n - n_P;
  const int g = x < n_X ? (n_X - x + N0 - 1) / N0 : 0;   // columns of this profile
  const float* pb = psi + static_cast<int64_t>(b) * T * R;
  const float* vbb = vb + static_cast<int64_t>(b) * T * P;
  float* fo = F + (static_cast<int64_t>(b) * N0 + x) * RP;
  const int cg = SP >> 2;                 // 4-column groups per row
  const int ntile = (RR >> 2) * cg;
  for (int e = threadIdx.x; e < RR * SP; e += blockDim.x) so[e] = 0.f;
  // rounds of up to mg staged columns (one round unless a profile has more
  // than POOL_MAXG columns)
  for (int s0 = 0; s0 < g; s0 += mg) {
    const int ns = min(mg, g - s0);
    __syncthreads();
    // asynchronous 4-byte copies (zero-filled padding), all in flight at once
    for (int e = threadIdx.x; e < ns * RR; e += blockDim.x) {
      const int si = e / RR, c = e % RR;
      const bool in = c < R;
      cp_async4(smem_u32(sp + e),
                in ? pb + static_cast<int64_t>(n_P + x + (s0 + si) * N0) * R + c : pb, in ? 4u : 0u);
    }
    for (int e = threadIdx.x; e < ns * SP; e += blockDim.x) {
      const int si = e / SP, c = e % SP;
      const bool in = c < P;
      cp_async4(smem_u32(sv + e),
                in ? vbb + static_cast<int64_t>(n_P + x + (s0 + si) * N0) * P + c : vbb,
                in ? 4u : 0u);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    for (int t = threadIdx.x; t < ntile; t += blockDim.x) {
      const int r0 = (t / cg) * 4, c0 = (t % cg) * 4;
      float acc[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 o = *reinterpret_cast<const float4*>(so + (r0 + i) * SP + c0);
        acc[i][0] = o.x;
        acc[i][1] = o.y;
        acc[i][2] = o.z;
        acc[i][3] = o.w;
      }
      for (int si = 0; si < ns; ++si) {
        const float4 a = *reinterpret_cast<const float4*>(sp + si * RR + r0);
        const float4 v = *reinterpret_cast<const float4*>(sv + si * SP + c0);
        const float av[4] = {a.x, a.y, a.z, a.w}, vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], vv[j], acc[i][j]);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<float4*>(so + (r0 + i) * SP + c0) =
            make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    }
  }
  __syncthreads();
  for (int o = threadIdx.x; o < RP; o += blockDim.x) fo[o] = so[(o / P) * SP + o % P];
}

// For every column j of profile x: dpsi_j = dF_x vb_j, dvb_j = dF_x^T psi_j.
// One CTA per (x, b); dF_x [R][SP] and the profile's columns are staged in
// shared memory (zero-padded as in the forward).  dpsi: a thread owns one row
// rr of dF_x and four columns j, 16-byte loads along p; dvb: a thread owns four
// p of one column j, one 16-byte dF load and one broadcast psi load per four
// FMAs.  Staging is by asynchronous 4-byte copies.
__global__ void __launch_bounds__(256) kattn_pool_bwd_kernel(
    const float* __restrict__ psi, const float* __restrict__ vb, const float* __restrict__ dF,
    float* __restrict__ dpsi, float* __restrict__ dvb, int T, int R, int P, int n_P, int n,
    int N0, int mg) {
  extern __shared__ float4 sm4[];   // dF [R][SP] | psi [MAXG][R] | vb [MAXG][SP]
  float* sm = reinterpret_cast<float*>(sm4);
  const int x = blockIdx.x, b = blockIdx.y;
  const int RP = R * P, SP = pool_stride(P), cg = SP >> 2;
  float* sdf = sm;
  float* sp = sm + R * SP;
  float* sv = sp + mg * R;
  const float* df = dF + (static_cast<int64_t>(b) * N0 + x) * RP;
  const int n_X = n - n_P;
  const int g = x < n_X ? (n_X - x + N0 - 1) / N0 : 0;
  if (g == 0) return;   // a profile without columns has nothing to write
  for (int e = threadIdx.x; e < R * SP; e += blockDim.x) {
    const int rr = e / SP, c = e % SP;
    const bool in = c < P;
    cp_async4(smem_u32(sdf + e), in ? df + rr * P + c : df, in ? 4u : 0u);
  }
  const int64_t row0 = static_cast<int64_t>(b) * T + n_P + x;
  for (int s0 = 0; s0 < g; s0 += mg) {
    const int ns = min(mg, g - s0);
    const int nsb = (ns + 3) >> 2;   // blocks of four columns
    __syncthreads();
    for (int e = threadIdx.x; e < nsb * 4 * R; e += blockDim.x) {
      const int si = e / R, c = e % R;
      const bool in = si < ns;
      cp_async4(smem_u32(sp + e),
                in ? psi + (row0 + static_cast<int64_t>(s0 + si) * N0) * R + c : psi,
                in ? 4u : 0u);
    }
    for (int e = threadIdx.x; e < nsb * 4 * SP; e += blockDim.x) {
      const int si = e / SP, c = e % SP;
      const bool in = si < ns && c < P;
      cp_async4(smem_u32(sv + e),
                in ? vb + (row0 + static_cast<int64_t>(s0 + si) * N0) * P + c : vb,
                in ? 4u : 0u);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    for (int e = threadIdx.x; e < nsb * R; e += blockDim.x) {   // dpsi[j, rr]
      const int rr = e % R, sb = e / R;
      float a[4] = {0.f, 0.f, 0.f, 0.f};
      for (int q = 0; q < cg; ++q) {
        const float4 d = *reinterpret_cast<const float4*>(sdf + rr * SP + 4 * q);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 v = *reinterpret_cast<const float4*>(sv + (4 * sb + i) * SP + 4 * q);
          a[i] = fmaf(d.x, v.x, a[i]);
          a[i] = fmaf(d.y, v.y, a[i]);
          a[i] = fmaf(d.z, v.z, a[i]);
          a[i] = fmaf(d.w, v.w, a[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (4 * sb + i < ns)
          dpsi[(row0 + static_cast<int64_t>(s0 + 4 * sb + i) * N0) * R + rr] = a[i];
    }
    for (int e = threadIdx.x; e < ns * cg; e += blockDim.x) {   // dvb[j, pp]
      const int q = e % cg, si = e / cg;
      float a[2][4] = {};   // even / odd rows: two independent chains
      const float* pr = sp + si * R;
      int rr = 0;
      for (; rr + 2 <= R; rr += 2) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const float4 d = *reinterpret_cast<const float4*>(sdf + (rr + k) * SP + 4 * q);
          const float pv = pr[rr + k];
          a[k][0] = fmaf(pv, d.x, a[k][0]);
          a[k][1] = fmaf(pv, d.y, a[k][1]);
          a[k][2] = fmaf(pv, d.z, a[k][2]);
          a[k][3] = fmaf(pv, d.w, a[k][3]);
        }
      }
      if (rr < R) {
        const float4 d = *reinterpret_cast<const float4*>(sdf + rr * SP + 4 * q);
        const float pv = pr[rr];
        a[0][0] = fmaf(pv, d.x, a[0][0]);
        a[0][1] = fmaf(pv, d.y, a[0][1]);
        a[0][2] = fmaf(pv, d.z, a[0][2]);
        a[0][3] = fmaf(pv, d.w, a[0][3]);
      }
      float* dst = dvb + (row0 + static_cast<int64_t>(s0 + si) * N0) * P;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (4 * q + c < P) dst[4 * q + c] = a[0][c] + a[1][c];
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

// ---------------------------------------------------------------- normalisation
// The op's last step (attention.py:450-451): out[row, c] = H[row, c] / H[row, P-1]
// for c < P - 1, and its backward dH[row, c] = dout[row, c] / den for c < P - 1,
// dH[row, P - 1] = -sum_c dout[row, c] out[row, c] / den.  One warp per row.
__global__ void __launch_bounds__(256) kattn_norm_fwd_kernel(const float* __restrict__ H,
                                                             float* __restrict__ out,
                                                             int64_t rows, int P) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* h = H + row * P;
  float* o = out + row * (P - 1);
  const float inv = 1.f / h[P - 1];
  for (int c = lane; c < P - 1; c += 32) o[c] = h[c] * inv;
}

__global__ void __launch_bounds__(256) kattn_norm_bwd_kernel(const float* __restrict__ H,
                                                             const float* __restrict__ dout,
                                                             float* __restrict__ dH,
                                                             int64_t rows, int P) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;   // whole warps: rows are warp-uniform
  const float* h = H + row * P;
  const float* g = dout + row * (P - 1);
  float* d = dH + row * P;
  const float inv = 1.f / h[P - 1];
  float acc = 0.f;
  for (int c = lane; c < P - 1; c += 32) {
    const float gc = g[c] * inv;
    d[c] = gc;
    acc = fmaf(gc, h[c], acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) d[P - 1] = -acc * inv;
}

// ---------------------------------------------------------------- streaming decode
// One token for every sequence b (SmatDecoder.step, attention.py:521-527):
// S_b += psi_b vb_b^T, o_b = phi_b^T (S_b + U_b[h]), out_b = o_b[:P-1] / o_b[P-1].
// One CTA per b; thread (rg, c) walks rows rg, rg + 4, ... of column c, so
// every S / U access is a coalesced 256-byte row segment read once.
constexpr int DEC_THREADS = 256, DEC_MAX_RP = 1024;
__global__ void __launch_bounds__(DEC_THREADS)
    kattn_decode_kernel(const float* __restrict__ phi, const float* __restrict__ psi,
                        const float* __restrict__ vb, float* __restrict__ S,
                        const float* __restrict__ U, float* __restrict__ out, int R, int P,
                        int nU, int h) {
  extern __shared__ float dsm[];  // phi[R] | psi[R] | part[4][P]
  float* sphi = dsm;
  float* spsi = dsm + R;
  float* part = dsm + 2 * R;
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x;
  for (int a = tid; a < R; a += DEC_THREADS) {
    sphi[a] = phi[b * R + a];
    spsi[a] = psi[b * R + a];
  }
  __syncthreads();
  const int rg = tid >> 6, cl = tid & 63;
  float* Sb = S + b * R * P;
  const float* Ub = U + (b * nU + h) * R * P;
  for (int c = cl; c < P; c += 64) {
    const float v = vb[b * P + c];
    float acc = 0.f;
    for (int a = rg; a < R; a += 4) {
      const int64_t o = static_cast<int64_t>(a) * P + c;
      const float sv = Sb[o] + spsi[a] * v;
      Sb[o] = sv;
      acc = fmaf(sphi[a], sv + Ub[o], acc);
    }
    part[rg * P + c] = acc;
  }
  __syncthreads();
  for (int c = tid; c < P; c += DEC_THREADS)
    part[c] = (part[c] + part[P + c]) + (part[2 * P + c] + part[3 * P + c]);
  __syncthreads();
  const float den = part[P - 1];
  for (int c = tid; c < P - 1; c += DEC_THREADS) out[b * (P - 1) + c] = part[c] / den;
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

bool al16(const void* p);

// 2-D fp32 map over [rows, R], box {32, 128}: 128-byte swizzle (K-major
// operand tiles) or its 32-byte-atom form (MN-major operand tiles)
int map_rows(CUtensorMap* m, const float* base, int64_t rows, int R, bool atom32 = false) {
  auto enc = encode_fn();
  if (!enc) return SMAT_ERR_NO_DEVICE;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(R), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(R) * 4};
  cuuint32_t box[2] = {32, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SMAT_OK : SMAT_ERR_TMA_DESCRIPTOR;
}

template <int MODE, int R, int PN>
int tile_launch(const CUtensorMap& m0, const CUtensorMap& m1, const TileParams& p,
                int64_t n_chunks, cudaStream_t s) {
  using C = TileCfg<MODE, R, PN>;
  auto kern = kattn_tile_kernel<MODE, R, PN>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES) !=
      cudaSuccess)
    return SMAT_ERR_LAUNCH;
  kern<<<static_cast<unsigned>(n_chunks), 192, C::SMEM_BYTES, s>>>(m0, m1, p);
  return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH;
}

template <int MODE, int R>
int tile_p(const CUtensorMap& a, const CUtensorMap& b, const TileParams& p, int64_t nc,
           cudaStream_t s) {
  switch ((p.P + 31) / 32 * 32) {
    case 32: return tile_launch<MODE, R, 32>(a, b, p, nc, s);
    case 64: return tile_launch<MODE, R, 64>(a, b, p, nc, s);
    case 96: return tile_launch<MODE, R, 96>(a, b, p, nc, s);
    case 128:
      // R = 128 with P > 96 exceeds the shared memory (four 64 KB operands)
      if constexpr (R < 128) return tile_launch<MODE, R, 128>(a, b, p, nc, s);
      break;
  }
  return SMAT_ERR_BAD_SHAPE;
}

template <int MODE>
int tile_r(const CUtensorMap& a, const CUtensorMap& b, const TileParams& p, int R, int64_t nc,
           cudaStream_t s) {
  switch (R) {
    case 32: return tile_p<MODE, 32>(a, b, p, nc, s);
    case 64: return tile_p<MODE, 64>(a, b, p, nc, s);
    case 128: return tile_p<MODE, 128>(a, b, p, nc, s);
  }
  return SMAT_ERR_BAD_SHAPE;
}

int check_chunk(const float* phi, const float* psi, int64_t n_chunks, int C, int R, int P) {
  if (!phi || !psi) return SMAT_ERR_NULL_POINTER;
  if (C != KC || (R != 32 && R != 64 && R != 128) || P < 1 || P > (R == 128 ? 96 : 128) ||
      n_chunks < 0 || n_chunks > 0x7FFFFFFF / KC)
    return SMAT_ERR_BAD_SHAPE;
  if (!al16(phi) || !al16(psi)) return SMAT_ERR_BAD_ALIGNMENT;
  return SMAT_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int smat_kattn_chunk_local_fwd(const float* phi, const float* psi, const float* vb,
                               const float* sin_, float* out, int64_t n_chunks, int C, int R,
                               int P, int32_t* err_word, void* stream) {
  int rc = check_chunk(phi, psi, n_chunks, C, R, P);
  if (rc) return rc;
  if (!vb || !sin_ || !out) return SMAT_ERR_NULL_POINTER;
  if (n_chunks == 0) return SMAT_OK;
  CUtensorMap mphi, mpsi;
  if ((rc = map_rows(&mphi, phi, n_chunks * KC, R))) return rc;
  if ((rc = map_rows(&mpsi, psi, n_chunks * KC, R))) return rc;
  TileParams p{vb, sin_, nullptr, out, P, P, err_word};
  return tile_r<TM_FWD>(mphi, mpsi, p, R, n_chunks, static_cast<cudaStream_t>(stream));
}

int smat_kattn_chunk_local_bwd(const float* phi, const float* psi, const float* vb,
                               const float* sin_, const float* dout, float* dphi, float* dpsi,
                               float* dvb, int64_t n_chunks, int C, int R, int P,
                               int32_t* err_word, void* stream) {
  int rc = check_chunk(phi, psi, n_chunks, C, R, P);
  if (rc) return rc;
  if (!vb || !sin_ || !dout || !dphi || !dpsi || !dvb) return SMAT_ERR_NULL_POINTER;
  if (n_chunks == 0) return SMAT_OK;
  CUtensorMap kphi, kpsi, mphi, mpsi;
  if ((rc = map_rows(&kphi, phi, n_chunks * KC, R))) return rc;
  if ((rc = map_rows(&kpsi, psi, n_chunks * KC, R))) return rc;
  if ((rc = map_rows(&mphi, phi, n_chunks * KC, R, true))) return rc;
  if ((rc = map_rows(&mpsi, psi, n_chunks * KC, R, true))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  TileParams p{vb, sin_, dout, dphi, P, R, err_word};
  if ((rc = tile_r<TM_DPHI>(mpsi, mpsi, p, R, n_chunks, s))) return rc;
  p.out = dvb;
  p.n_store = P;
  if ((rc = tile_r<TM_DV>(kpsi, kphi, p, R, n_chunks, s))) return rc;
  p.out = dpsi;
  p.n_store = R;
  return tile_r<TM_DPSI>(mphi, mphi, p, R, n_chunks, s);
}

int smat_kattn_pool_fwd(const float* psi, const float* vb, float* F, int nb, int T, int R, int P,
                        int n_P, int n, int N0, void* stream) {
  if (!psi || !vb || !F) return SMAT_ERR_NULL_POINTER;
  if (nb < 1 || T < 1 || R < 1 || P < 1 || N0 < 1 || n_P < 0 || n < n_P || n > T)
    return SMAT_ERR_BAD_SHAPE;
  const int RR = (R + 3) & ~3, SP = pool_stride(P);
  const int mg = pool_round(n_P, n, N0);
  const int64_t bytes = (static_cast<int64_t>(mg) * (RR + SP) + RR * SP) * 4;
  if (bytes > POOL_SMEM_MAX) return SMAT_ERR_BAD_SHAPE;
  if (cudaFuncSetAttribute(kattn_pool_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           POOL_SMEM_MAX) != cudaSuccess)
    return SMAT_ERR_LAUNCH;
  kattn_pool_kernel<<<dim3(N0, nb), 256, bytes, static_cast<cudaStream_t>(stream)>>>(
      psi, vb, F, T, R, P, n_P, n, N0, mg);
  return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH;
}

int smat_kattn_pool_bwd(const float* psi, const float* vb, const float* dF, float* dpsi,
                        float* dvb, int nb, int T, int R, int P, int n_P, int n, int N0,
                        void* stream) {
  if (!psi || !vb || !dF || !dpsi || !dvb) return SMAT_ERR_NULL_POINTER;
  if (nb < 1 || T < 1 || R < 1 || P < 1 || N0 < 1 || n_P < 0 || n < n_P || n > T)
    return SMAT_ERR_BAD_SHAPE;
  const int SP = pool_stride(P);
  const int mg = pool_round(n_P, n, N0);
  const int64_t bytes = (static_cast<int64_t>(R) * SP + static_cast<int64_t>(mg) * (R + SP)) * 4;
  if (bytes > POOL_SMEM_MAX) return SMAT_ERR_BAD_SHAPE;
  if (cudaFuncSetAttribute(kattn_pool_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           POOL_SMEM_MAX) != cudaSuccess)
    return SMAT_ERR_LAUNCH;
  kattn_pool_bwd_kernel<<<dim3(N0, nb), 256, bytes, static_cast<cudaStream_t>(stream)>>>(
      psi, vb, dF, dpsi, dvb, T, R, P, n_P, n, N0, mg);
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

int smat_kattn_decode_step(const float* phi, const float* psi, const float* vb, float* S,
                           const float* U, float* out, int nb, int R, int P, int nU, int h,
                           void* stream) {
  if (!phi || !psi || !vb || !S || !U || !out) return SMAT_ERR_NULL_POINTER;
  if (nb < 1 || R < 1 || R > DEC_MAX_RP || P < 2 || P > DEC_MAX_RP || nU < 1 || h < 0 ||
      h >= nU)
    return SMAT_ERR_BAD_SHAPE;
  const size_t smem = (2 * static_cast<size_t>(R) + 4 * static_cast<size_t>(P)) * sizeof(float);
  kattn_decode_kernel<<<nb, DEC_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(
      phi, psi, vb, S, U, out, R, P, nU, h);
  return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH;
}

int smat_kattn_normalise_fwd(const float* H, float* out, int64_t rows, int P, void* stream) {
  if (!H || !out) return SMAT_ERR_NULL_POINTER;
  if (rows < 0 || P < 2 || rows > 8 * static_cast<int64_t>(0x7FFFFFFF)) return SMAT_ERR_BAD_SHAPE;
  if (rows == 0) return SMAT_OK;
  const int64_t blocks = (rows + 7) / 8;
  kattn_norm_fwd_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                          static_cast<cudaStream_t>(stream)>>>(H, out, rows, P);
  return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH;
}

int smat_kattn_normalise_bwd(const float* H, const float* dout, float* dH, int64_t rows, int P,
                             void* stream) {
  if (!H || !dout || !dH) return SMAT_ERR_NULL_POINTER;
  if (rows < 0 || P < 2 || rows > 8 * static_cast<int64_t>(0x7FFFFFFF)) return SMAT_ERR_BAD_SHAPE;
  if (rows == 0) return SMAT_OK;
  const int64_t blocks = (rows + 7) / 8;
  kattn_norm_bwd_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                          static_cast<cudaStream_t>(stream)>>>(H, dout, dH, rows, P);
  return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH;
}

}  // extern "C"
