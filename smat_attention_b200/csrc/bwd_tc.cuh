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
// Warp roles as in the forward kernel: warps 0-3 compute (thread r owns tile
// row r = TMEM lane r), warp 4 TMA producer, warp 5 TMEM allocator + MMA
// issuer.  P^T / dS^T / dS are written to shared memory in the SWIZZLE_128B
// K-major layout and fed back to the tensor core as the A operand.
#pragma once

#include "common.cuh"
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
  float scale;             // softmax scale
  float scale_log2;        // softmax scale * log2(e)
  int32_t* err;
};

template <int D>
struct BwdCfg {
  static constexpr int BM = 128;     // tile rows
  static constexpr int CN = 64;      // chunk width (queries for dK/dV, keys for dQ)
  static constexpr int STAGES = 2;
  static constexpr int ROW_BYTES = BM * D * 2;   // one resident operand
  static constexpr int CH_BYTES = CN * D * 2;    // one streamed operand chunk
  static constexpr int AB_BYTES = BM * CN * 2;   // P^T / dS^T / dS tile
  static constexpr int OFF_R0 = 0;                              // K (dK/dV) or Q (dQ)
  static constexpr int OFF_R1 = OFF_R0 + ROW_BYTES;             // V (dK/dV) or dO (dQ)
  static constexpr int OFF_C0 = OFF_R1 + ROW_BYTES;             // Q_c (dK/dV) or K_c (dQ)
  static constexpr int OFF_C1 = OFF_C0 + STAGES * CH_BYTES;     // dO_c (dK/dV) or V_c (dQ)
  static constexpr int OFF_A0 = OFF_C1 + STAGES * CH_BYTES;     // P^T (dK/dV) or dS (dQ)
  static constexpr int OFF_A1 = OFF_A0 + AB_BYTES;              // dS^T (dK/dV)
  static constexpr int OFF_LD = OFF_A1 + AB_BYTES;              // lse/delta chunk staging [2][2][CN]
  static constexpr int OFF_BAR = OFF_LD + 2 * 2 * CN * 4;
  // barriers: r_full, c_full[S], c_empty[S], s_full[2], a_full, a_done
  static constexpr int BAR_R = 0, BAR_CF = 1, BAR_CE = 1 + STAGES, BAR_SF = 1 + 2 * STAGES,
                       BAR_AF = 3 + 2 * STAGES, BAR_AD = 4 + 2 * STAGES,
                       BAR_LD = 5 + 2 * STAGES,  // [2]: lse/delta staging, 128 arrivals
                       BAR_DRAIN = 7 + 2 * STAGES, NBAR = 8 + 2 * STAGES;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int OFF_SCHED = OFF_MISC + 16;
  static constexpr int MAX_CHUNKS = 512;
  static constexpr int SMEM_USED = OFF_SCHED + MAX_CHUNKS * 4 + 1024;
  // every CTA takes all 512 TMEM columns: take more than half the shared
  // memory too, so a second CTA is never resident and waiting in tcgen05.alloc
  static constexpr int SMEM_BYTES = SMEM_USED < 120 * 1024 ? 120 * 1024 : SMEM_USED;
  // TMEM: [S 64 | dP 64] x 2 buffers, then accumulators
  static constexpr int COL_S = 0, COL_DP = CN, BUF_COLS = 2 * CN, COL_ACC0 = 2 * BUF_COLS,
                       COL_ACC1 = COL_ACC0 + D;
  static constexpr int TMEM_COLS = 512;
  static constexpr uint32_t IDESC_SC = idesc_bf16(BM, CN, false, false);  // S, dP
  static constexpr uint32_t IDESC_ACC = idesc_bf16(BM, D, false, true);   // dV, dK, dQ
};

// Chunk c of a schedule whose blocks are `bs` wide covers block
// sched[c / CPB], sub-chunk c % CPB, CPB = bs / 64.
template <bool DKDV, int D>
__global__ void __launch_bounds__(192, 1)
    smat_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_r0,
                       const __grid_constant__ CUtensorMap tm_r1,
                       const __grid_constant__ CUtensorMap tm_c0,
                       const __grid_constant__ CUtensorMap tm_c1, const BwdParams p) {
  using C = BwdCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto bar = [&](int i) { return bar0 + 8u * i; };
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  uint32_t* sched = reinterpret_cast<uint32_t*>(smem + C::OFF_SCHED);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int BH = p.B * p.H;
  const int lin = blockIdx.x;
  const int bh = lin % BH;
  // dQ: latest query tiles are the heaviest; dK/dV: earliest key tiles are
  // (sinks and summaries are read by every later query)
  const int tile = DKDV ? lin / BH : p.n_tiles - 1 - lin / BH;
  const int b = bh / p.H, h = bh % p.H;
  const int sub_blocks = C::BM / p.bs;  // 1 or 2
  const int cpb = p.bs / C::CN;         // chunks per block: 1 or 2

  if (tid == 0) {
    mbar_init(bar(C::BAR_R), 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar(C::BAR_CF + s), 1);
      mbar_init(bar(C::BAR_CE + s), 1);
    }
    mbar_init(bar(C::BAR_SF + 0), 1);
    mbar_init(bar(C::BAR_SF + 1), 1);
    mbar_init(bar(C::BAR_AF), 4);
    mbar_init(bar(C::BAR_AD), 1);
    mbar_init(bar(C::BAR_LD + 0), 128);
    mbar_init(bar(C::BAR_LD + 1), 128);
    mbar_init(bar(C::BAR_DRAIN), 1);
    fence_barrier_init();
    misc[1] = 0;
    misc[2] = build_schedule(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, tile * sub_blocks,
                             sub_blocks, sched, C::MAX_CHUNKS, p.err);
  }
  if (warp == 5) {
    tmem_alloc(sbase + C::OFF_MISC, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&tm_r0);
    prefetch_tmap(&tm_r1);
    prefetch_tmap(&tm_c0);
    prefetch_tmap(&tm_c1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = misc[0];
  const int n = static_cast<int>(misc[2]) * cpb;  // chunks

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n > 0) {
      mbar_expect_tx(bar(C::BAR_R), 2 * C::ROW_BYTES);
#pragma unroll
      for (int pn = 0; pn < D / 64; ++pn) {
        tma_load_4d(sbase + C::OFF_R0 + pn * (C::BM * 128), &tm_r0, bar(C::BAR_R), pn * 64,
                    tile * C::BM, h, b);
        tma_load_4d(sbase + C::OFF_R1 + pn * (C::BM * 128), &tm_r1, bar(C::BAR_R), pn * 64,
                    tile * C::BM, h, b);
      }
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int s = j % C::STAGES;
        if (j >= C::STAGES &&
            !mbar_wait(bar(C::BAR_CE + s), ((j / C::STAGES) - 1) & 1, abort_flag, p.err))
          break;
        const int blk = static_cast<int>(sched_block(sched[j / cpb]));
        const int row = blk * p.bs + (j % cpb) * C::CN;
        mbar_expect_tx(bar(C::BAR_CF + s), 2 * C::CH_BYTES);
#pragma unroll
        for (int pn = 0; pn < D / 64; ++pn) {
          tma_load_4d(sbase + C::OFF_C0 + s * C::CH_BYTES + pn * (C::CN * 128), &tm_c0,
                      bar(C::BAR_CF + s), pn * 64, row, h, b);
          tma_load_4d(sbase + C::OFF_C1 + s * C::CH_BYTES + pn * (C::CN * 128), &tm_c1,
                      bar(C::BAR_CF + s), pn * 64, row, h, b);
        }
        issued = j + 1;
      }
      if (*abort_flag) {
        for (int j = max(0, issued - C::STAGES); j < issued; ++j)
          mbar_wait_drain(bar(C::BAR_CF + j % C::STAGES), (j / C::STAGES) & 1);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n > 0) {
      bool ok = mbar_wait(bar(C::BAR_R), 0, abort_flag, p.err);
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
          tc_mma(tb + C::COL_S, sdesc_sw128(r0 + off, 16, 1024), sdesc_sw128(c0 + offc, 16, 1024),
                 C::IDESC_SC, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (C::BM * 128) + (kk & 3) * 32;
          const uint32_t offc = (kk >> 2) * (C::CN * 128) + (kk & 3) * 32;
          tc_mma(tb + C::COL_DP, sdesc_sw128(r1 + off, 16, 1024), sdesc_sw128(c1 + offc, 16, 1024),
                 C::IDESC_SC, kk > 0 ? 1u : 0u);
        }
        tc_commit(bar(C::BAR_SF + (j & 1)));
      };
      if (ok) ok = mbar_wait(bar(C::BAR_CF + 0), 0, abort_flag, p.err);
      if (ok) {
        tc_fence_after();
        issue_sc(0);
      }
      for (int j = 0; ok && j < n; ++j) {
        if (j + 1 < n) {
          const int s1 = (j + 1) % C::STAGES;
          if (!mbar_wait(bar(C::BAR_CF + s1), ((j + 1) / C::STAGES) & 1, abort_flag, p.err)) break;
          tc_fence_after();
          issue_sc(j + 1);
        }
        if (!mbar_wait(bar(C::BAR_AF), j & 1, abort_flag, p.err)) break;
        tc_fence_after();
        const int s = j % C::STAGES;
        const uint32_t c0 = sbase + C::OFF_C0 + s * C::CH_BYTES;
        const uint32_t c1 = sbase + C::OFF_C1 + s * C::CH_BYTES;
        const uint32_t a0 = sbase + C::OFF_A0, a1 = sbase + C::OFF_A1;
        const uint32_t acc = (j > 0) ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < C::CN / 16; ++kk) {
          const uint64_t ad0 = sdesc_sw128(a0 + (kk & 3) * 32, 16, 1024);
          if (DKDV) {
            // dV += P^T dO_c ; dK += dS^T Q_c   (B operands MN-major)
            const uint64_t ad1 = sdesc_sw128(a1 + (kk & 3) * 32, 16, 1024);
            tc_mma(tbase + C::COL_ACC1, ad0, sdesc_sw128(c1 + kk * 2048, C::CN * 128, 1024),
                   C::IDESC_ACC, (acc || kk > 0) ? 1u : 0u);
            tc_mma(tbase + C::COL_ACC0, ad1, sdesc_sw128(c0 + kk * 2048, C::CN * 128, 1024),
                   C::IDESC_ACC, (acc || kk > 0) ? 1u : 0u);
          } else {
            // dQ += dS K_c
            tc_mma(tbase + C::COL_ACC0, ad0, sdesc_sw128(c0 + kk * 2048, C::CN * 128, 1024),
                   C::IDESC_ACC, (acc || kk > 0) ? 1u : 0u);
          }
        }
        tc_commit(bar(C::BAR_AD));
        tc_commit(bar(C::BAR_CE + s));
      }
      if (*abort_flag) {  // let the MMAs in flight finish before TMEM is freed
        tc_commit(bar(C::BAR_DRAIN));
        mbar_wait_drain(bar(C::BAR_DRAIN), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ compute
    const int r = tid;
    const int pos = tile * C::BM + r;               // key (dK/dV) or query (dQ) position
    const int sub = (p.bs == 64) ? (r >> 6) : 0;
    const uint32_t lane_base = tbase + (static_cast<uint32_t>(warp * 32) << 16);
    const float LOG2E = 1.4426950408889634f;
    float* ld = reinterpret_cast<float*>(smem + C::OFF_LD);  // [2][lse CN | delta CN]
    float row_lse2 = 0.f, row_delta = 0.f;
    if (!DKDV) {
      const bool in = pos < p.T;
      row_lse2 = in ? p.lse[static_cast<int64_t>(bh) * p.T + pos] * LOG2E : INFINITY;
      row_delta = in ? p.delta[static_cast<int64_t>(bh) * p.T + pos] : 0.f;
    }
    bool alive = true;
    for (int j = 0; j < n && alive; ++j) {
      const uint32_t e = sched[j / cpb];
      const int c0pos = static_cast<int>(sched_block(e)) * p.bs + (j % cpb) * C::CN;
      const uint32_t st = sched_state(e, sub);
      float* ldj = ld + (j & 1) * 2 * C::CN;
      if (DKDV) {
        // stage this chunk's per-query lse (log2 units) and delta
        const int qi = c0pos + (r & (C::CN - 1));
        const bool in = qi < p.T;
        if (r < C::CN)
          ldj[r] = in ? p.lse[static_cast<int64_t>(bh) * p.T + qi] * LOG2E : INFINITY;
        else
          ldj[r] = in ? p.delta[static_cast<int64_t>(bh) * p.T + qi] : 0.f;
        mbar_arrive(bar(C::BAR_LD + (j & 1)));
        if (!__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_LD + (j & 1)), (j >> 1) & 1,
                                               abort_flag, p.err))) {
          alive = false;
          break;
        }
      }
      if (!__all_sync(0xffffffffu,
                      mbar_wait(bar(C::BAR_SF + (j & 1)), (j >> 1) & 1, abort_flag, p.err))) {
        alive = false;
        break;
      }
      tc_fence_after();
      const uint32_t tb = lane_base + (j & 1) * C::BUF_COLS;
      float sv[C::CN], dp[C::CN];
      tmem_ld32(tb + C::COL_S, sv);
      tmem_ld32(tb + C::COL_S + 32, sv + 32);
      tmem_ld32(tb + C::COL_DP, dp);
      tmem_ld32(tb + C::COL_DP + 32, dp + 32);
      // the A-operand buffers are free once the previous chunk's MMAs completed
      if (j > 0 && !__all_sync(0xffffffffu,
                               mbar_wait(bar(C::BAR_AD), (j - 1) & 1, abort_flag, p.err))) {
        alive = false;
        break;
      }
      uint8_t* a0 = smem + C::OFF_A0;
      uint8_t* a1 = smem + C::OFF_A1;
#pragma unroll
      for (int c16 = 0; c16 < C::CN / 8; ++c16) {
        uint32_t wp[4], wd[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float pv[2], dsv[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int c = c16 * 8 + 2 * i + u;
            const int cpos = c0pos + c;
            bool valid;
            float lse2, dl;
            if (DKDV) {
              // row = key `pos`, column = query `cpos`
              valid = (st == ST_FULL || (st == ST_CAUSAL && cpos >= pos)) && cpos < p.T;
              lse2 = ldj[c];
              dl = ldj[C::CN + c];
            } else {
              valid = (st == ST_FULL) || (st == ST_CAUSAL && cpos <= pos);
              lse2 = row_lse2;
              dl = row_delta;
            }
            const float pr = valid ? ex2_approx(fmaf(sv[c], p.scale_log2, -lse2)) : 0.f;
            pv[u] = pr;
            dsv[u] = pr * (dp[c] - dl);
          }
          wp[i] = pack_bf16(pv[0], pv[1]);
          wd[i] = pack_bf16(dsv[0], dsv[1]);
        }
        const uint32_t off = sw128_offset(r, c16);
        if (DKDV) {
          *reinterpret_cast<uint4*>(a0 + off) = make_uint4(wp[0], wp[1], wp[2], wp[3]);
          *reinterpret_cast<uint4*>(a1 + off) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        } else {
          *reinterpret_cast<uint4*>(a0 + off) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C::BAR_AF));
    }
    // ------------------------------------------------------------ epilogue
    if (alive && n > 0 &&
        !__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_AD), (n - 1) & 1, abort_flag, p.err)))
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
#pragma unroll
      for (int acc = 0; acc < (DKDV ? 2 : 1); ++acc) {
        __nv_bfloat16* dst = acc == 0 ? o0 : o1;
        const float mul = acc == 0 ? p.scale : 1.f;  // dK and dQ carry the softmax scale
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          float v[32];
          if (n > 0) {
            tmem_ld32(lane_base + C::COL_ACC0 + acc * D + c, v);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = 0.f;
          }
          if (store) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 w = make_uint4(pack_bf16(v[i] * mul, v[i + 1] * mul),
                                   pack_bf16(v[i + 2] * mul, v[i + 3] * mul),
                                   pack_bf16(v[i + 4] * mul, v[i + 5] * mul),
                                   pack_bf16(v[i + 6] * mul, v[i + 7] * mul));
              *reinterpret_cast<uint4*>(dst + c + i) = w;
            }
          }
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

}  // namespace smat
