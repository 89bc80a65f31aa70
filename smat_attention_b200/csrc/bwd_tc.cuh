// Block-sparse causal softmax attention, backward, bf16 on sm_100a tensor cores.
//
// Two kernels, no atomics (results are deterministic):
//
// dK/dV  one CTA per 128-row key tile of one (batch, head); it walks the
//        union of the tile's transposed-CSR rows (the query blocks that read
//        it) in 64-query chunks:
//          S^T  = K Q_c^T          dP^T = V dO_c^T        (TMEM, double-buffered)
//          P^T  = exp2(S^T c - lse_c log2 e)   dS^T = P^T (dP^T - delta_c)
//          dV  += P^T dO_c         dK  += dS^T Q_c        (TMEM accumulators)
// dQ     one CTA per 128-row query tile; it walks the forward CSR in 64-key
//        chunks:
//          S = Q K_c^T   dP = dO V_c^T   dS = P (dP - delta)   dQ += dS K_c
//
// Warp roles (320 threads): warps 0-7 compute -- warp w reads TMEM lanes
// 32 (w % 4) .. +31 (its 32 tile rows) and chunk columns 32 (w / 4) .. +31;
// warp 8 is the TMA producer; warp 9 allocates TMEM and issues the MMAs.
// P^T / dS^T / dS (bf16) are written back into the TMEM columns of the S / dP
// they came from (each warp over columns it has already read) and feed the
// tensor core as the A operand straight from TMEM; the S/dP double buffer
// lets the compute warps work on the next chunk meanwhile.
#pragma once

#include "common.cuh"
#include "fwd_tc.cuh"
#include "schedule.cuh"

namespace smat {

struct BwdParams {
  const int32_t* indptr;   // forward CSR (dQ) or transposed CSR (dK/dV)
  const int32_t* indices;
  const uint8_t* kind;
  const float* lse;        // [B*H, T]
  const float* delta;      // [B*H, T]
  __nv_bfloat16* out0;     // dK or dQ
  __nv_bfloat16* out1;     // dV (dK/dV kernel only)
  int64_t o0_sb, o0_sh, o0_st, o1_sb, o1_sh, o1_st;
  int B, H, T, nblocks, nnzb, bs, n_tiles;
  const int32_t* work;     // optional work list (one tile per CTA and (b, h)); null = all tiles
  float scale;             // softmax scale
  float scale_log2;        // softmax scale * log2(e)
  int32_t* err;
};

template <bool DKDV, int D>
struct BwdCfg {
  static constexpr int BM = 128;     // tile rows
  static constexpr int CN = 64;      // chunk width (queries for dK/dV, keys for dQ)
  static constexpr int ROW_BYTES = BM * D * 2;   // one resident operand
  static constexpr int CH_BYTES = CN * D * 2;    // one streamed operand chunk
  static constexpr int LD_BYTES = DKDV ? 2 * CN * 4 : 0;   // lse + delta per stage
  // as many stages as the shared memory holds (at most 8)
  static constexpr int FIXED = 2 * ROW_BYTES + 1536;  // + barriers, alignment
  static constexpr int STAGES_FIT = (227 * 1024 - FIXED) / (2 * CH_BYTES + LD_BYTES);
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int OFF_R0 = 0;                              // K (dK/dV) or Q (dQ)
  static constexpr int OFF_R1 = OFF_R0 + ROW_BYTES;             // V (dK/dV) or dO (dQ)
  static constexpr int OFF_C0 = OFF_R1 + ROW_BYTES;             // Q_c (dK/dV) or K_c (dQ)
  static constexpr int OFF_C1 = OFF_C0 + STAGES * CH_BYTES;     // dO_c (dK/dV) or V_c (dQ)
  static constexpr int OFF_LD = OFF_C1 + STAGES * CH_BYTES;     // per stage: lse [CN], delta [CN]
  static constexpr int OFF_BAR = OFF_LD + STAGES * LD_BYTES;
  // barriers: r_full, c_full[S], c_empty[S], s_full[2], a_full[2], a_done[2], drain
  static constexpr int BAR_R = 0, BAR_CF = 1, BAR_CE = 1 + STAGES, BAR_SF = 1 + 2 * STAGES,
                       BAR_AF = BAR_SF + 2, BAR_AD = BAR_AF + 2, BAR_DRAIN = BAR_AD + 2,
                       BAR_RT = BAR_DRAIN + 1, NBAR = BAR_RT + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static_assert(STAGES >= 2, "at least two stages");
  // TMEM: [S 64 | dP 64] x 2 buffers, then the accumulators
  static constexpr int COL_S = 0, COL_DP = CN, BUF_COLS = 2 * CN, COL_ACC0 = 2 * BUF_COLS,
                       COL_ACC1 = COL_ACC0 + D;
  // dQ: the resident Q and dO also go to TMEM (bf16 pairs per column), so S
  // and dP read only the streamed chunk from shared memory
  static constexpr bool RES_TMEM = !DKDV;
  static constexpr int COL_RT0 = COL_ACC0 + D, COL_RT1 = COL_RT0 + D / 2;
  static_assert(!RES_TMEM || COL_RT1 + D / 2 <= 512, "TMEM budget");
  static constexpr int TMEM_COLS = 512;
  // compute warps: NCW / 4 groups of 4; group g owns chunk columns
  // [g CW, (g + 1) CW) of all 128 tile rows
  static constexpr int NCW = 16, CW = CN * 4 / NCW;
  static constexpr int PRODUCER_WARP = NCW, MMA_WARP = NCW + 1, THREADS = (NCW + 2) * 32;
  static constexpr uint32_t IDESC_SC = idesc_bf16(BM, CN, false, false);  // S, dP
  static constexpr uint32_t IDESC_ACC = idesc_bf16(BM, D, false, true);   // dV, dK, dQ
};

template <bool DKDV, int D>
__global__ void __launch_bounds__((BwdCfg<DKDV, D>::NCW + 2) * 32, 1)
    smat_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_r0,
                       const __grid_constant__ CUtensorMap tm_r1,
                       const __grid_constant__ CUtensorMap tm_c0,
                       const __grid_constant__ CUtensorMap tm_c1, const BwdParams p) {
  using C = BwdCfg<DKDV, D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto bar = [&](int i) { return bar0 + 8u * i; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int BH = p.B * p.H;
  const int lin = blockIdx.x;
  const int bh = lin % BH;
  // dQ: latest query tiles are the heaviest; dK/dV: earliest key tiles are
  // (sinks and summaries are read by every later query)
  int tile;
  if (p.work) {
    // caller-chosen tiles (a shard of the rows), in the caller's order
    const int w = __ldg(p.work + lin / BH);
    tile = w & WORK_TILE_MASK;
    if ((w >> 24) != 0 || tile >= p.n_tiles) {
      if (threadIdx.x == 0 && p.err) atomicOr(p.err, DEV_ERR_BAD_WORK);
      return;
    }
  } else {
    tile = DKDV ? lin / BH : p.n_tiles - 1 - lin / BH;
  }
  const int b = bh / p.H, h = bh % p.H;
  const int sub = C::BM / p.bs;   // CSR rows per tile: 1 or 2
  const int cpb = p.bs / C::CN;   // chunks per block: 2 or 1
  const int row0 = tile * sub;

  if (tid == 0) {
    mbar_init(bar(C::BAR_R), 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar(C::BAR_CF + s), 1);
      mbar_init(bar(C::BAR_CE + s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(C::BAR_SF + i), 1);
      mbar_init(bar(C::BAR_AF + i), C::NCW);
      mbar_init(bar(C::BAR_AD + i), 1);
    }
    mbar_init(bar(C::BAR_DRAIN), 1);
    mbar_init(bar(C::BAR_RT), C::NCW);
    fence_barrier_init();
    misc[1] = 0;
  }
  if (warp == C::MMA_WARP) {
    tmem_alloc(sbase + C::OFF_MISC, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == C::PRODUCER_WARP && lane == 0) {
    prefetch_tmap(&tm_r0);
    prefetch_tmap(&tm_r1);
    prefetch_tmap(&tm_c0);
    prefetch_tmap(&tm_c1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = misc[0];

  if (warp == C::PRODUCER_WARP) {
    // ------------------------------------------------------------ producer
    // Lane 0 issues the TMA loads; for dK/dV all 32 lanes also copy the
    // chunk's lse and delta next to it with cp.async, tracked by the same
    // stage barrier, so nobody waits on a global load.
    ChunkIter<2> it;
    it.init(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, row0, sub, cpb, p.err);
    if (lane == 0) {
      mbar_expect_tx(bar(C::BAR_R), 2 * C::ROW_BYTES);
#pragma unroll
      for (int pn = 0; pn < D / 64; ++pn) {
        tma_load_4d(sbase + C::OFF_R0 + pn * (C::BM * 128), &tm_r0, bar(C::BAR_R), pn * 64,
                    tile * C::BM, h, b);
        tma_load_4d(sbase + C::OFF_R1 + pn * (C::BM * 128), &tm_r1, bar(C::BAR_R), pn * 64,
                    tile * C::BM, h, b);
      }
    }
    int issued = 0;
    uint32_t e;
    int c;
    for (int j = 0; it.next(e, c, p.err); ++j) {
      const int s = j % C::STAGES;
      bool ok = true;
      if (lane == 0 && j >= C::STAGES)
        ok = mbar_wait(bar(C::BAR_CE + s), ((j / C::STAGES) - 1) & 1, abort_flag, p.err);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      __syncwarp();
      const int row = static_cast<int>(sched_block(e)) * p.bs + c * C::CN;
      if (DKDV) {
        const uint32_t lds = sbase + C::OFF_LD + s * C::LD_BYTES;
#pragma unroll
        for (int u = 0; u < C::CN / 32; ++u) {
          const int qi = row + u * 32 + lane;
          const bool in = qi < p.T;
          const int64_t gi = in ? static_cast<int64_t>(bh) * p.T + qi : 0;
          cp_async4(lds + (u * 32 + lane) * 4, p.lse + gi, in ? 4u : 0u);
          cp_async4(lds + (C::CN + u * 32 + lane) * 4, p.delta + gi, in ? 4u : 0u);
        }
        cp_async_arrive(bar(C::BAR_CF + s));
        __syncwarp();
      }
      if (lane == 0) {
        mbar_expect_tx(bar(C::BAR_CF + s), 2 * C::CH_BYTES);
#pragma unroll
        for (int pn = 0; pn < D / 64; ++pn) {
          tma_load_4d(sbase + C::OFF_C0 + s * C::CH_BYTES + pn * (C::CN * 128), &tm_c0,
                      bar(C::BAR_CF + s), pn * 64, row, h, b);
          tma_load_4d(sbase + C::OFF_C1 + s * C::CH_BYTES + pn * (C::CN * 128), &tm_c1,
                      bar(C::BAR_CF + s), pn * 64, row, h, b);
        }
      }
      issued = j + 1;
    }
    if (lane == 0) {
      mbar_wait_drain(bar(C::BAR_R), 0);
      if (*abort_flag) {
        for (int j = max(0, issued - C::STAGES); j < issued; ++j)
          mbar_wait_drain(bar(C::BAR_CF + j % C::STAGES), (j / C::STAGES) & 1);
      }
    }
  } else if (warp == C::MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      ChunkIter<2> it;
      it.init(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, row0, sub, cpb, p.err);
      // S-like products of chunk j into TMEM buffer j & 1:
      //   buffer.S  = R0 . C0_j^T,   buffer.dP = R1 . C1_j^T
      auto issue_sc = [&](int j) {
        const int s = j % C::STAGES;
        const uint32_t tb = tbase + (j & 1) * C::BUF_COLS;
        const uint32_t r0 = sbase + C::OFF_R0, r1 = sbase + C::OFF_R1;
        const uint32_t c0 = sbase + C::OFF_C0 + s * C::CH_BYTES;
        const uint32_t c1 = sbase + C::OFF_C1 + s * C::CH_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (C::BM * 128) + (kk & 3) * 32;
          const uint32_t offc = (kk >> 2) * (C::CN * 128) + (kk & 3) * 32;
          if (C::RES_TMEM)   // A = 16 d-elements = 8 packed columns per k-step
            tc_mma_ts(tb + C::COL_S, tbase + C::COL_RT0 + kk * 8,
                      sdesc_sw128(c0 + offc, 16, 1024), C::IDESC_SC, kk > 0 ? 1u : 0u);
          else
            tc_mma(tb + C::COL_S, sdesc_sw128(r0 + off, 16, 1024),
                   sdesc_sw128(c0 + offc, 16, 1024), C::IDESC_SC, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (C::BM * 128) + (kk & 3) * 32;
          const uint32_t offc = (kk >> 2) * (C::CN * 128) + (kk & 3) * 32;
          if (C::RES_TMEM)
            tc_mma_ts(tb + C::COL_DP, tbase + C::COL_RT1 + kk * 8,
                      sdesc_sw128(c1 + offc, 16, 1024), C::IDESC_SC, kk > 0 ? 1u : 0u);
          else
            tc_mma(tb + C::COL_DP, sdesc_sw128(r1 + off, 16, 1024),
                   sdesc_sw128(c1 + offc, 16, 1024), C::IDESC_SC, kk > 0 ? 1u : 0u);
        }
        tc_commit(bar(C::BAR_SF + (j & 1)));
      };
      bool ok = mbar_wait(bar(C::BAR_R), 0, abort_flag, p.err);
      if (C::RES_TMEM && ok) ok = mbar_wait(bar(C::BAR_RT), 0, abort_flag, p.err);
      uint32_t e;
      int c;
      bool has = ok && it.next(e, c, p.err);
      if (has) {
        ok = mbar_wait(bar(C::BAR_CF + 0), 0, abort_flag, p.err);
        if (ok) {
          tc_fence_after();
          issue_sc(0);
        }
      }
      for (int j = 0; ok && has; ++j) {
        has = it.next(e, c, p.err);
        // S/dP of the next chunk go first if its operands already landed;
        // otherwise this chunk's accumulator MMAs are not held up behind it
        bool early = false;
        if (has && mbar_try_wait(bar(C::BAR_CF + (j + 1) % C::STAGES), ((j + 1) / C::STAGES) & 1)) {
          tc_fence_after();
          issue_sc(j + 1);
          early = true;
        }
        if (!mbar_wait(bar(C::BAR_AF + (j & 1)), (j >> 1) & 1, abort_flag, p.err)) break;
        tc_fence_after();
        const int s = j % C::STAGES;
        const uint32_t c0 = sbase + C::OFF_C0 + s * C::CH_BYTES;
        const uint32_t c1 = sbase + C::OFF_C1 + s * C::CH_BYTES;
        const uint32_t tb = tbase + (j & 1) * C::BUF_COLS;
        const uint32_t acc = (j > 0) ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < C::CN / 16; ++kk) {
          // A in TMEM: the 16 chunk columns of k-step kk are 8 packed columns
          // at the start of the column group of the warps that wrote them
          const uint32_t aoff = (16 * kk / C::CW) * C::CW + (16 * kk % C::CW) / 2;
          if (DKDV) {
            // dV += P^T dO_c ; dK += dS^T Q_c   (B operands MN-major)
            tc_mma_ts(tbase + C::COL_ACC1, tb + C::COL_S + aoff,
                      sdesc_sw128(c1 + kk * 2048, C::CN * 128, 1024), C::IDESC_ACC,
                      (acc || kk > 0) ? 1u : 0u);
            tc_mma_ts(tbase + C::COL_ACC0, tb + C::COL_DP + aoff,
                      sdesc_sw128(c0 + kk * 2048, C::CN * 128, 1024), C::IDESC_ACC,
                      (acc || kk > 0) ? 1u : 0u);
          } else {
            // dQ += dS K_c
            tc_mma_ts(tbase + C::COL_ACC0, tb + C::COL_DP + aoff,
                      sdesc_sw128(c0 + kk * 2048, C::CN * 128, 1024), C::IDESC_ACC,
                      (acc || kk > 0) ? 1u : 0u);
          }
        }
        tc_commit(bar(C::BAR_AD + (j & 1)));
        tc_commit(bar(C::BAR_CE + s));
        if (has && !early) {
          const int s1 = (j + 1) % C::STAGES;
          if (!mbar_wait(bar(C::BAR_CF + s1), ((j + 1) / C::STAGES) & 1, abort_flag, p.err)) break;
          tc_fence_after();
          issue_sc(j + 1);
        }
      }
      if (*abort_flag) {  // let the MMAs in flight finish before TMEM is freed
        tc_commit(bar(C::BAR_DRAIN));
        mbar_wait_drain(bar(C::BAR_DRAIN), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ compute
    constexpr int CW = C::CW;
    const int quad = warp & 3, grp = warp >> 2;
    const int r = quad * 32 + lane;                 // tile row = TMEM lane
    const int pos = tile * C::BM + r;               // key (dK/dV) or query (dQ) position
    const int srow = (sub == 2) ? (r >> 6) : 0;     // CSR row of this tile row
    const int col0 = grp * CW;                      // this warp's chunk columns
    const uint32_t lane_base = tbase + (static_cast<uint32_t>(quad * 32) << 16);
    const float LOG2E = 1.4426950408889634f;
    const float* ld = reinterpret_cast<const float*>(smem + C::OFF_LD);  // [STAGES][lse | delta]
    float row_lse2 = 0.f, row_delta = 0.f;
    if (!DKDV) {
      const bool in = pos < p.T;
      row_lse2 = in ? p.lse[static_cast<int64_t>(bh) * p.T + pos] * LOG2E : INFINITY;
      row_delta = in ? p.delta[static_cast<int64_t>(bh) * p.T + pos] : 0.f;
    }
    bool alive = true;
    if (C::RES_TMEM) {
      // copy this warp's share of the resident rows (Q, dO) into TMEM: row r,
      // 16-byte chunk q of the row = packed columns [4 q, 4 q + 4)
      alive = __all_sync(0xffffffffu, mbar_wait(bar(C::BAR_R), 0, abort_flag, p.err));
      if (alive) {
        constexpr int QPG = D / 8 / (C::NCW / 4);   // 16-byte chunks per warp group
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const uint8_t* src = smem + (t == 0 ? C::OFF_R0 : C::OFF_R1);
          uint32_t w[QPG * 4];
#pragma unroll
          for (int u = 0; u < QPG; ++u) {
            const int q = grp * QPG + u;
            const uint4 v = *reinterpret_cast<const uint4*>(
                src + (q >> 3) * (C::BM * 128) + sw128_offset(r, q & 7));
            w[4 * u] = v.x;
            w[4 * u + 1] = v.y;
            w[4 * u + 2] = v.z;
            w[4 * u + 3] = v.w;
          }
          const uint32_t dst = lane_base + (t == 0 ? C::COL_RT0 : C::COL_RT1) + grp * QPG * 4;
          if (QPG * 4 == 16) tmem_st16u(dst, w);
          else tmem_st8u(dst, w);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(C::BAR_RT));
      }
    }
    int n = 0;
    ChunkIter<2> it;
    it.init(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, row0, sub, cpb, p.err);
    uint32_t e;
    int c;
    for (int j = 0; alive && it.next(e, c, p.err); ++j) {
      n = j + 1;
      const int c0pos = static_cast<int>(sched_block(e)) * p.bs + c * C::CN;
      const uint32_t st = sched_state(e, srow);
      const float* ldj = ld + (j % C::STAGES) * (C::LD_BYTES / 4);
      // dK/dV reads the lse/delta the producer staged with this chunk
      if (DKDV && !__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_CF + j % C::STAGES),
                                                     (j / C::STAGES) & 1, abort_flag, p.err))) {
        alive = false;
        break;
      }
      if (!__all_sync(0xffffffffu,
                      mbar_wait(bar(C::BAR_SF + (j & 1)), (j >> 1) & 1, abort_flag, p.err))) {
        alive = false;
        break;
      }
      tc_fence_after();
      const uint32_t tb = lane_base + (j & 1) * C::BUF_COLS;
      float sv[CW], dp[CW];
      if (CW == 32) {
        tmem_ld32x2(tb + C::COL_S + col0, tb + C::COL_DP + col0, sv, dp);
      } else {
        tmem_ld16x2(tb + C::COL_S + col0, tb + C::COL_DP + col0, sv, dp);
      }
      // warp-uniform: no element of this warp's 32 x CW block is masked
      const bool all_valid = (st == ST_FULL) && (!DKDV || c0pos + C::CN <= p.T);
      // per-column terms: -lse log2(e) and delta of the chunk's queries (dK/dV),
      // or the row's own (dQ)
      float nl2[CW], dl[CW];
      if (DKDV) {
        const float4* l4 = reinterpret_cast<const float4*>(ldj + col0);
        const float4* d4 = reinterpret_cast<const float4*>(ldj + C::CN + col0);
#pragma unroll
        for (int q = 0; q < CW / 4; ++q) {
          const float4 a = l4[q], dd = d4[q];
          nl2[4 * q] = a.x * -LOG2E;
          nl2[4 * q + 1] = a.y * -LOG2E;
          nl2[4 * q + 2] = a.z * -LOG2E;
          nl2[4 * q + 3] = a.w * -LOG2E;
          dl[4 * q] = dd.x;
          dl[4 * q + 1] = dd.y;
          dl[4 * q + 2] = dd.z;
          dl[4 * q + 3] = dd.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < CW; ++i) {
          nl2[i] = -row_lse2;
          dl[i] = row_delta;
        }
      }
      float pv[CW];
      if (all_valid) {
#pragma unroll
        for (int i = 0; i < CW; ++i) pv[i] = ex2_approx(fmaf(sv[i], p.scale_log2, nl2[i]));
      } else {
#pragma unroll
        for (int i = 0; i < CW; ++i) {
          const int cpos = c0pos + col0 + i;
          // dK/dV: row = key `pos`, column = query `cpos`; dQ: the reverse
          const bool valid =
              DKDV ? ((st == ST_FULL || (st == ST_CAUSAL && cpos >= pos)) && cpos < p.T)
                   : (st == ST_CAUSAL && cpos <= pos);
          pv[i] = valid ? ex2_approx(fmaf(sv[i], p.scale_log2, nl2[i])) : 0.f;
        }
      }
      uint32_t wp[CW / 2], wd[CW / 2];
#pragma unroll
      for (int i = 0; i < CW / 2; ++i) {
        wp[i] = pack_bf16(pv[2 * i], pv[2 * i + 1]);
        wd[i] = pack_bf16(pv[2 * i] * (dp[2 * i] - dl[2 * i]),
                          pv[2 * i + 1] * (dp[2 * i + 1] - dl[2 * i + 1]));
      }
      // P^T / dS^T / dS over the S / dP columns this warp has already read
      if (CW == 32) {
        if (DKDV) tmem_st16u(tb + C::COL_S + col0, wp);
        tmem_st16u(tb + C::COL_DP + col0, wd);
      } else {
        if (DKDV) tmem_st8u(tb + C::COL_S + col0, wp);
        tmem_st8u(tb + C::COL_DP + col0, wd);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C::BAR_AF + (j & 1)));
    }
    // ------------------------------------------------------------ epilogue
    if (alive && n > 0 &&
        !__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_AD + ((n - 1) & 1)), ((n - 1) >> 1) & 1,
                                           abort_flag, p.err)))
      alive = false;
    if (alive) {
      tc_fence_after();
      const bool store = pos < p.T;
      __nv_bfloat16* o0 = p.out0 + static_cast<int64_t>(b) * p.o0_sb +
                          static_cast<int64_t>(h) * p.o0_sh + static_cast<int64_t>(pos) * p.o0_st;
      __nv_bfloat16* o1 = DKDV ? p.out1 + static_cast<int64_t>(b) * p.o1_sb +
                                     static_cast<int64_t>(h) * p.o1_sh +
                                     static_cast<int64_t>(pos) * p.o1_st
                               : nullptr;
      constexpr int EW = D / (C::NCW / 4);   // accumulator columns per warp group
#pragma unroll
      for (int acc = 0; acc < (DKDV ? 2 : 1); ++acc) {
        __nv_bfloat16* dst = acc == 0 ? o0 : o1;
        const float mul = acc == 0 ? p.scale : 1.f;  // dK and dQ carry the softmax scale
#pragma unroll
        for (int cc = grp * EW; cc < (grp + 1) * EW; cc += 16) {
          float v[16];
          if (n > 0) {
            tmem_ld16(lane_base + C::COL_ACC0 + acc * D + cc, v);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
          }
          if (store) {
#pragma unroll
            for (int i = 0; i < 16; i += 8) {
              uint4 w = make_uint4(pack_bf16(v[i] * mul, v[i + 1] * mul),
                                   pack_bf16(v[i + 2] * mul, v[i + 3] * mul),
                                   pack_bf16(v[i + 4] * mul, v[i + 5] * mul),
                                   pack_bf16(v[i + 6] * mul, v[i + 7] * mul));
              *reinterpret_cast<uint4*>(dst + cc + i) = w;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == C::MMA_WARP) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

}  // namespace smat
