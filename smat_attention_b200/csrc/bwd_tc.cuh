// Block-sparse causal softmax attention, backward, bf16 on sm_100a tensor cores.
//
// Two kernels, no atomics (results are deterministic), and an opt-in fused
// variant of the first (FQ below) that also accumulates dQ:
//
// dK/dV  one CTA per 128-row key tile of one (batch, head); it walks the
//        union of the tile's transposed-CSR rows (the query blocks that read
//        it) in chunks of 128 queries:
//          S^T  = K Q_c^T          dP^T = V dO_c^T        (TMEM, 128 x 128 each)
//          P^T  = exp2(S^T c - lse_c log2 e)   dS^T = P^T (dP^T - delta_c)
//          dV  += P^T dO_c         dK  += dS^T Q_c        (TMEM accumulators)
// dQ     one CTA per 128-row query tile; it walks the forward CSR in chunks
//        of 128 keys:
//          S = Q K_c^T   dP = dO V_c^T   dS = P (dP - delta)   dQ += dS K_c
//        Q and dO are copied into TMEM once per tile (S and dP take their A
//        operand from there), after which their shared-memory tiles serve
//        as one more slot of the K_c / V_c ring.
//
// Every tcgen05.mma is 128 x 128 (or 128 x D): on B200 an N = 64 MMA costs
// nearly as many cycles as an N = 128 one, so the chunk is 128 wide.  TMEM
// (512 columns) then holds one S, one dP and the accumulators, so S and dP
// are single-buffered and the hand-offs are split to keep the tensor core
// fed: as soon as P^T is in TMEM (dK/dV), or S has been read (dQ, which
// keeps P in registers), the MMA warp issues dV and the next S; as soon as
// dS is ready it issues dK (or dQ) and the next dP.  The compute warps turn
// dP into dS while the tensor core runs dV and the next S.
// With bs = 64 a chunk is two 64-row blocks of the merged list (TMA loads
// each half separately; a missing second half is loaded from row T, i.e.
// zero-filled, and masked).  A warp's 32 x 32 block is masked by one 32-bit
// word per row: the causal span on the diagonal, and for M^(d) PATTERN tiles
// the row word (dQ) or column word (dK/dV) of pattern.cuh.
//
// Warp roles (576 threads; 320 with 64-row chunks): warps 0 .. NCW-1 compute
// -- warp w reads TMEM lanes 32 (w % 4) .. +31 (its 32 tile rows) and chunk
// columns 32 (w / 4) .. +31; warp NCW is the TMA producer; warp NCW + 1
// allocates TMEM and issues the MMAs.
// P^T / dS^T / dS (bf16) are written back into the TMEM columns of the S / dP
// they came from (each warp over columns it has already read) and feed the
// tensor core as the A operand straight from TMEM.
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
  const int32_t* work;     // optional work list (one tile per CTA and (b, h)); null = all tiles
  int head_group;          // without a work list: (b, h) per tile-interleaved group (>= 1)
  float scale;             // softmax scale
  float scale_log2;        // softmax scale * log2(e)
  float* dq_acc;           // fused dQ (dK/dV kernel with FQ): fp32 [B*H, T, D], pre-zeroed
  int32_t* err;
  MdPattern md;            // tables of PATTERN tiles (null row_bits: the layout has none)
};

// CN_ chunk rows: 128, or 64 at D = 64 with 64-row blocks -- TMEM then needs
// 256 columns and shared memory <= 113 KB, so two CTAs share an SM and one's
// set-up, hand-off waits and epilogue overlap the other's chunks.
// FQ_ (dK/dV only, D = 128): the same kernel also forms dQ_c = dS_c K for each
// chunk and adds it into an fp32 dQ accumulator in global memory, so no
// second kernel recomputes S and dP for dQ (5 MMAs per chunk instead of 4 + 3).
// dS^T then goes to shared memory, over the chunk's dO once dV has read it,
// where it is the A operand of dK (K-major) and the B operand of dQ_c^T =
// K^T dS_c^T (MN-major); dQ_c^T lands in the TMEM columns of dP, which the
// compute warps have already read.  Transposed, a TMEM lane holds one column
// of D for the chunk's queries, so a warp's reduction instruction adds 32
// consecutive floats of one dQ row (one 128-byte line) instead of 16 bytes
// of 32 rows; the warps drain it before the next dP is issued.
template <bool DKDV, int D, int CN_ = 128, bool FQ_ = false>
struct BwdCfg {
  static constexpr int BM = 128;     // tile rows
  static constexpr int CN = CN_;     // chunk rows (queries for dK/dV, keys for dQ)
  static constexpr bool FQ = FQ_;
  static_assert(CN == 128 || (CN == 64 && D == 64), "chunk rows");
  // dS^T (CN x BM bf16) takes the place of a dO chunk (CN x D bf16)
  static_assert(!FQ || (DKDV && D == BM && CN == 128), "fused dQ shape");
  static constexpr int MIN_BLOCKS = CN == 64 ? 2 : 1;   // CTAs per SM
  static constexpr int SMEM_CAP = (CN == 64 ? 113 : 227) * 1024;
  static constexpr int BOX = 64;     // TMA box rows of a chunk load
  static constexpr int ROW_BYTES = BM * D * 2;   // one resident operand
  static constexpr int CH_BYTES = CN * D * 2;    // one streamed operand chunk
  static constexpr int PANEL_R = BM * 128;       // one 64-column SWIZZLE_128B panel
  static constexpr int PANEL_C = CN * 128;
  static constexpr int LD_BYTES = DKDV ? 2 * CN * 4 : 0;   // lse + delta per stage
  // as many stages as the shared memory holds (at most 8)
  static constexpr int FIXED = 2 * ROW_BYTES + 2048;  // + barriers, alignment
  static constexpr int STAGES_FIT = (SMEM_CAP - FIXED) / (2 * CH_BYTES + LD_BYTES);
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int OFF_R0 = 0;                              // K (dK/dV) or Q (dQ)
  static constexpr int OFF_R1 = OFF_R0 + ROW_BYTES;             // V (dK/dV) or dO (dQ)
  static constexpr int OFF_C0 = OFF_R1 + ROW_BYTES;             // Q_c (dK/dV) or K_c (dQ)
  static constexpr int OFF_C1 = OFF_C0 + STAGES * CH_BYTES;     // dO_c (dK/dV) or V_c (dQ)
  static constexpr int OFF_LD = OFF_C1 + STAGES * CH_BYTES;     // per stage: lse [CN], delta [CN]
  // dQ: once Q and dO sit in TMEM (below) their shared-memory tiles hold one
  // more slot of the chunk ring (C0 over R0, C1 over R1)
  static constexpr bool TA = !DKDV;
  static constexpr int RING = TA ? STAGES + 1 : STAGES;
  static_assert(!TA || CH_BYTES <= ROW_BYTES, "ring slot over the resident tiles");
  __host__ __device__ static constexpr uint32_t c_off(int s, int which) {
    return s < STAGES ? static_cast<uint32_t>((which ? OFF_C1 : OFF_C0) + s * CH_BYTES)
                      : static_cast<uint32_t>(which ? OFF_R1 : OFF_R0);
  }
  static constexpr int OFF_BAR = OFF_LD + STAGES * LD_BYTES;
  // barriers: r_full, c_full[S], c_empty[S], s_full, dp_full, p_ready, ds_ready,
  // acc_done, drain
  // (+ with FQ: dv_done, dq_full, dq_empty)
  // (+ with FQ: dv_done, dq_full, dq_empty; the dQ kernel: resident tiles in TMEM)
  static constexpr int BAR_R = 0, BAR_CF = 1, BAR_CE = 1 + RING, BAR_SF = 1 + 2 * RING,
                       BAR_DPF = BAR_SF + 1, BAR_PR = BAR_DPF + 1, BAR_DSR = BAR_PR + 1,
                       BAR_AD = BAR_DSR + 1, BAR_DRAIN = BAR_AD + 1, BAR_DVD = BAR_DRAIN + 1,
                       BAR_DQF = BAR_DVD + 1, BAR_DQE = BAR_DQF + 1, BAR_RT = BAR_DQE + 1,
                       NBAR = BAR_RT + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static_assert(SMEM_BYTES <= SMEM_CAP, "shared memory budget");
  static_assert(STAGES >= 2, "at least two stages");
  // the epilogue stages the output tile(s) in the chunk buffers of C0
  static_assert((DKDV ? 2 : 1) * ROW_BYTES <= STAGES * CH_BYTES, "epilogue staging");
  // TMEM: S | dP | accumulators (| Q | dO for dQ).  A 128 x 128 x 16 MMA
  // step with both operands in shared memory reads 8 KB in the 64 cycles it
  // computes, the whole 128 B/cycle of the SM's shared-memory path, which
  // TMA writes and the epilogue share; an operand read from TMEM halves it.
  // The dQ kernel has the columns for its resident Q and dO tiles (bf16
  // pairs, D / 2 columns each): its S and dP take A from TMEM.  The dK/dV
  // kernel's accumulators leave no room, so its S^T and dP^T read K and V
  // from shared memory.
  static constexpr int COL_S = 0, COL_DP = CN, COL_ACC0 = 2 * CN, COL_ACC1 = COL_ACC0 + D;
  static constexpr int COL_RA = COL_ACC0 + (DKDV ? 2 : 1) * D;   // TA: Q | dO
  static constexpr int TMEM_USED = COL_RA + (TA ? D : 0);
  // TA: warp (quad, grp) with grp < RA_GROUPS copies one 64-column panel of
  // Q or dO for its 32 rows into TMEM
  static constexpr int RA_GROUPS = 2 * D / 64;
  static_assert(!TA || RA_GROUPS <= CN / 32, "resident-tile copy warps");
  static constexpr int TMEM_COLS = TMEM_USED <= 256 ? 256 : 512;
  static_assert(TMEM_USED <= TMEM_COLS && TMEM_COLS * MIN_BLOCKS <= 512, "TMEM budget");
  // compute warps: CN / 32 groups of 4; group g owns chunk columns [32 g, 32 g + 32)
  static constexpr int CW = 32, NCW = 4 * (CN / CW);
  static constexpr int PRODUCER_WARP = NCW, MMA_WARP = NCW + 1, THREADS = (NCW + 2) * 32;
  static constexpr uint32_t IDESC_SC = idesc_bf16(BM, CN, false, false);  // S, dP
  static constexpr uint32_t IDESC_ACC = idesc_bf16(BM, D, false, true);   // dV, dK, dQ
  // fused dQ_c^T = K^T dS_c^T: A = K^T (D x keys) read MN-major from the K
  // tile, B = dS^T (keys x queries) MN-major
  static constexpr uint32_t IDESC_DQ = idesc_bf16(D, CN, true, true);
};

// TMEM column (packed bf16 pairs) of the A operand's k-step kk (16 chunk
// columns): group kk / 2 wrote chunk columns [32 (kk / 2), +32) packed into
// its first 16 columns
__device__ __forceinline__ uint32_t a_col(int kk) { return 32u * (kk >> 1) + 8u * (kk & 1); }

template <bool DKDV, int D, int CN, bool FQ = false>
__global__ void __launch_bounds__(BwdCfg<DKDV, D, CN, FQ>::THREADS,
                                  BwdCfg<DKDV, D, CN, FQ>::MIN_BLOCKS)
    smat_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_r0,
                       const __grid_constant__ CUtensorMap tm_r1,
                       const __grid_constant__ CUtensorMap tm_c0,
                       const __grid_constant__ CUtensorMap tm_c1,
                       const __grid_constant__ CUtensorMap tm_o0,
                       const __grid_constant__ CUtensorMap tm_o1, const BwdParams p) {
  using C = BwdCfg<DKDV, D, CN, FQ>;
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
  int bh = lin % BH;
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
    // (b, h) in groups of head_group: within a group the tiles run one tile
    // index across the group's heads at a time (heaviest first: dQ the latest
    // query tiles, dK/dV the earliest key tiles, since sinks and summaries are
    // read by every later query), so a long tile of one head overlaps the
    // tiles of the others; groups run one after another, so the resident
    // CTAs share a few heads' streamed chunks in L2
    const int G = p.head_group;
    const int grp = lin / (G * p.n_tiles);
    const int g0 = grp * G, gs = min(G, BH - g0);
    const int r = lin - grp * G * p.n_tiles;
    const int t = r / gs;
    bh = g0 + r % gs;
    tile = DKDV ? t : p.n_tiles - 1 - t;
  }
  const int b = bh / p.H, h = bh % p.H;
  const int sub = C::BM / p.bs;   // CSR rows per tile: 1 or 2
  const int row0 = tile * sub;

  if (tid == 0) {
    mbar_init(bar(C::BAR_R), 1);
    for (int s = 0; s < C::RING; ++s) {
      mbar_init(bar(C::BAR_CF + s), 1);
      mbar_init(bar(C::BAR_CE + s), 1);
    }
    mbar_init(bar(C::BAR_SF), 1);
    mbar_init(bar(C::BAR_DPF), 1);
    mbar_init(bar(C::BAR_PR), C::NCW);
    mbar_init(bar(C::BAR_DSR), C::NCW);
    mbar_init(bar(C::BAR_AD), 1);
    mbar_init(bar(C::BAR_DRAIN), 1);
    if constexpr (FQ) {
      mbar_init(bar(C::BAR_DVD), 1);
      mbar_init(bar(C::BAR_DQF), 1);
      mbar_init(bar(C::BAR_DQE), C::NCW);
    }
    if constexpr (C::TA) mbar_init(bar(C::BAR_RT), 4 * C::RA_GROUPS);
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
    // the resident tiles first: they do not depend on the schedule reads
    if (lane == 0) {
      mbar_expect_tx(bar(C::BAR_R), 2 * C::ROW_BYTES);
#pragma unroll
      for (int pn = 0; pn < D / 64; ++pn) {
        tma_load_4d(sbase + C::OFF_R0 + pn * C::PANEL_R, &tm_r0, bar(C::BAR_R), pn * 64,
                    tile * C::BM, h, b);
        tma_load_4d(sbase + C::OFF_R1 + pn * C::PANEL_R, &tm_r1, bar(C::BAR_R), pn * 64,
                    tile * C::BM, h, b);
      }
    }
    ChunkPair<2> it;
    it.init(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, row0, sub, p.bs, p.err, C::CN);
    int issued = 0;
    uint32_t e[2];
    for (int j = 0; it.next(e, p.err); ++j) {
      const int s = j % C::RING;
      bool ok = true;
      if (lane == 0 && j >= C::RING)
        ok = mbar_wait(bar(C::BAR_CE + s), ((j / C::RING) - 1) & 1, abort_flag, p.err);
      // the ring slot over the resident tiles is free once they are in TMEM
      if (C::TA && lane == 0 && j == C::STAGES && ok)
        ok = mbar_wait(bar(C::BAR_RT), 0, abort_flag, p.err);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      __syncwarp();
      // first row of each 64-row half of the chunk; a missing half reads row
      // T onwards, which TMA fills with zeros
      int prow[2] = {p.T, p.T};
#pragma unroll
      for (int q = 0; q < C::CN / 64; ++q) {
        const uint32_t eq = (p.bs == 64) ? e[q] : e[0];
        prow[q] = entry_present(eq) ? static_cast<int>(sched_block(eq)) * p.bs + (q * 64) % p.bs
                                    : p.T;
      }
      if (DKDV) {
        const uint32_t lds = sbase + C::OFF_LD + s * C::LD_BYTES;
#pragma unroll
        for (int u = 0; u < C::CN / 32; ++u) {
          const int col = u * 32 + lane;
          const int qi = prow[col >> 6] + (col & 63);
          const bool in = qi < p.T;
          const int64_t gi = in ? static_cast<int64_t>(bh) * p.T + qi : 0;
          cp_async4(lds + col * 4, p.lse + gi, in ? 4u : 0u);
          cp_async4(lds + (C::CN + col) * 4, p.delta + gi, in ? 4u : 0u);
        }
        cp_async_arrive(bar(C::BAR_CF + s));
        __syncwarp();
      }
      if (lane == 0) {
        mbar_expect_tx(bar(C::BAR_CF + s), 2 * C::CH_BYTES);
#pragma unroll
        for (int pn = 0; pn < D / 64; ++pn)
#pragma unroll
          for (int q = 0; q < C::CN / 64; ++q) {
            const uint32_t off = pn * C::PANEL_C + q * (C::BOX * 128);
            tma_load_4d(sbase + C::c_off(s, 0) + off, &tm_c0, bar(C::BAR_CF + s), pn * 64,
                        prow[q], h, b);
            tma_load_4d(sbase + C::c_off(s, 1) + off, &tm_c1, bar(C::BAR_CF + s), pn * 64,
                        prow[q], h, b);
          }
      }
      issued = j + 1;
    }
    if (lane == 0) {
      mbar_wait_drain(bar(C::BAR_R), 0);
      if (*abort_flag) {
        for (int j = max(0, issued - C::RING); j < issued; ++j)
          mbar_wait_drain(bar(C::BAR_CF + j % C::RING), (j / C::RING) & 1);
      }
    }
  } else if (warp == C::MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      ChunkPair<2> it;
      it.init(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, row0, sub, p.bs, p.err, C::CN);
      // S (S^T) of chunk j:  R0 . C0_j^T;  dP (dP^T):  R1 . C1_j^T
      auto issue_sd = [&](int j, bool dp) {
        const int s = j % C::RING;
        const uint32_t r = sbase + (dp ? C::OFF_R1 : C::OFF_R0);
        const uint32_t c = sbase + C::c_off(s, dp ? 1 : 0);
        const uint32_t d = tbase + (dp ? C::COL_DP : C::COL_S);
        const uint64_t rd = sdesc_sw128(r, 16, 1024), cd = sdesc_sw128(c, 16, 1024);
        // TA: A (Q or dO) from TMEM, k-step kk in columns 8 kk .. 8 kk + 7
        const uint32_t ra = tbase + C::COL_RA + (dp ? D / 2 : 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::PANEL_R + (kk & 3) * 32;
          const uint32_t offc = (kk >> 2) * C::PANEL_C + (kk & 3) * 32;
          if constexpr (C::TA)
            tc_mma_ts(d, ra + 8 * kk, sdesc_add(cd, offc), C::IDESC_SC, kk > 0 ? 1u : 0u);
          else
            tc_mma(d, sdesc_add(rd, off), sdesc_add(cd, offc), C::IDESC_SC, kk > 0 ? 1u : 0u);
        }
        tc_commit(bar(dp ? C::BAR_DPF : C::BAR_SF));
      };
      // acc (+)= A_j . C_j with A = P^T / dS^T / dS in TMEM at column `acol`,
      // C_j the chunk operand (MN-major): 16 chunk rows per k-step
      auto issue_acc = [&](uint32_t dcol, uint32_t acol, uint32_t cbase, bool first) {
        const uint64_t cd = sdesc_sw128(cbase, C::PANEL_C, 1024);
        const uint32_t dt = tbase + dcol, at = tbase + acol;
#pragma unroll
        for (int kk = 0; kk < C::CN / 16; ++kk)
          tc_mma_ts(dt, at + a_col(kk), sdesc_add(cd, kk * 2048), C::IDESC_ACC,
                    (!first || kk > 0) ? 1u : 0u);
      };
      // FQ: dQ_c^T = K^T dS_c^T into the dP columns (both operands MN-major,
      // 16 keys per k-step), and dK += dS^T Q_c with the dS^T tile K-major
      constexpr uint32_t PDS = C::BM * 128;   // one 64-query panel of the dS^T tile
      auto issue_dq = [&](uint32_t dsb) {
        const uint64_t kd = sdesc_sw128(sbase + C::OFF_R0, C::PANEL_R, 1024);
        const uint64_t bd = sdesc_sw128(dsb, PDS, 1024);
#pragma unroll
        for (int kk = 0; kk < C::BM / 16; ++kk)
          tc_mma(tbase + C::COL_DP, sdesc_add(kd, kk * 2048), sdesc_add(bd, kk * 2048),
                 C::IDESC_DQ, kk > 0 ? 1u : 0u);
      };
      auto issue_dk = [&](uint32_t dsb, uint32_t cbase, bool first) {
        const uint64_t ad = sdesc_sw128(dsb, 16, 1024);
        const uint64_t cd = sdesc_sw128(cbase, C::PANEL_C, 1024);
#pragma unroll
        for (int kk = 0; kk < C::CN / 16; ++kk)
          tc_mma(tbase + C::COL_ACC0, sdesc_add(ad, (kk >> 2) * PDS + (kk & 3) * 32),
                 sdesc_add(cd, kk * 2048), C::IDESC_ACC, (!first || kk > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(bar(C::BAR_R), 0, abort_flag, p.err);
      // TA: the compute warps have put Q and dO into TMEM
      if (C::TA && ok) ok = mbar_wait(bar(C::BAR_RT), 0, abort_flag, p.err);
      uint32_t e[2];
      bool has = ok && it.next(e, p.err);
      if (has) {
        ok = mbar_wait(bar(C::BAR_CF + 0), 0, abort_flag, p.err);
        if (ok) {
          tc_fence_after();
          issue_sd(0, false);
          issue_sd(0, true);
        }
      }
      for (int j = 0; ok && has; ++j) {
        const bool nxt = it.next(e, p.err);
        const int s = j % C::RING;
        const uint32_t c0 = sbase + C::c_off(s, 0);
        const uint32_t c1 = sbase + C::c_off(s, 1);
        // P^T written (dK/dV) or S read (dQ)
        if (!mbar_wait(bar(C::BAR_PR), j & 1, abort_flag, p.err)) break;
        tc_fence_after();
        if (DKDV) issue_acc(C::COL_ACC1, C::COL_S, c1, j == 0);      // dV += P^T dO_c
        if constexpr (FQ) tc_commit(bar(C::BAR_DVD));   // dO_c may take dS^T once dV is done
        // the next S goes in behind it if its operands already landed
        bool s_next = false;
        if (nxt && mbar_try_wait(bar(C::BAR_CF + (j + 1) % C::RING), ((j + 1) / C::RING) & 1)) {
          tc_fence_after();
          issue_sd(j + 1, false);
          s_next = true;
        }
        if (!mbar_wait(bar(C::BAR_DSR), j & 1, abort_flag, p.err)) break;
        tc_fence_after();
        if constexpr (FQ) {
          issue_dq(c1);                     // dQ_c^T = K^T dS_c^T
          tc_commit(bar(C::BAR_DQF));
          issue_dk(c1, c0, j == 0);         // dK += dS^T Q_c
        } else {
          issue_acc(C::COL_ACC0, C::COL_DP, c0, j == 0);   // dK += dS^T Q_c  or  dQ += dS K_c
        }
        tc_commit(bar(C::BAR_CE + s));                    // chunk j's operands are consumed
        if (nxt) {
          if (!s_next) {
            if (!mbar_wait(bar(C::BAR_CF + (j + 1) % C::RING), ((j + 1) / C::RING) & 1,
                           abort_flag, p.err))
              break;
            tc_fence_after();
            issue_sd(j + 1, false);
          }
          // FQ: the next dP overwrites dQ_c once the compute warps have read it
          if (FQ && !mbar_wait(bar(C::BAR_DQE), j & 1, abort_flag, p.err)) break;
          tc_fence_after();
          issue_sd(j + 1, true);
        }
        has = nxt;
      }
      tc_commit(bar(C::BAR_AD));
      if (*abort_flag) {  // let the MMAs in flight finish before TMEM is freed
        tc_commit(bar(C::BAR_DRAIN));
        mbar_wait_drain(bar(C::BAR_DRAIN), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ compute
    const int quad = warp & 3, grp = warp >> 2;
    const int r = quad * 32 + lane;                 // tile row = TMEM lane
    const int pos = tile * C::BM + r;               // key (dK/dV) or query (dQ) position
    const int srow = (sub == 2) ? (r >> 6) : 0;     // CSR row of this tile row
    const int col0 = grp * C::CW;                   // this warp's chunk columns
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
    if constexpr (C::TA) {
      // Q (grp < D / 64) or dO: one SW128 panel (64 columns of D) of this
      // warp's 32 rows, unswizzled into 32 TMEM columns of bf16 pairs
      if (grp < C::RA_GROUPS) {
        if (!__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_R), 0, abort_flag, p.err))) {
          alive = false;
        } else {
          const int ten = grp / (D / 64), pn = grp % (D / 64);
          const uint32_t src =
              sbase + (ten ? C::OFF_R1 : C::OFF_R0) + pn * C::PANEL_R + r * 128;
          uint32_t w[32];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint4 x = ld_shared_v4(src + ((u ^ (r & 7)) << 4));
            w[4 * u] = x.x;
            w[4 * u + 1] = x.y;
            w[4 * u + 2] = x.z;
            w[4 * u + 3] = x.w;
          }
          tmem_st32u(lane_base + C::COL_RA + ten * (D / 2) + pn * 32, w);
          tmem_st_wait();
          fence_proxy_async_smem();   // the tile's bytes are read before TMA refills them
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(C::BAR_RT));
        }
      }
    }
    int n = 0;
    ChunkPair<2> it;
    it.init(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, row0, sub, p.bs, p.err, C::CN);
    uint32_t e[2];
    for (int j = 0; alive && it.next(e, p.err); ++j) {
      n = j + 1;
      // this warp's 32 columns lie in one 64-row half of the chunk
      const uint32_t ew = (p.bs == 64 && col0 >= 64) ? e[1] : e[0];
      const int cbase = entry_present(ew) ? static_cast<int>(sched_block(ew)) * p.bs + col0 % p.bs
                                          : p.T;
      const uint32_t st = entry_present(ew) ? sched_state(ew, srow) : ST_ABSENT;
      // visibility of this row's 32 columns (bit c: column cbase + c); for
      // PATTERN tiles the table loads overlap the waits below
      uint32_t vw = 0u;
      if (st == ST_FULL) {
        vw = DKDV ? span_word(cbase, 0, p.T) : 0xffffffffu;
      } else if (st == ST_CAUSAL) {
        vw = DKDV ? span_word(cbase, pos, p.T) : span_word(cbase, 0, pos + 1);
      } else if (st == ST_PATTERN) {
        if (p.md.row_bits)
          vw = DKDV ? md_col_word(p.md, p.T, pos, cbase) : md_row_word(p.md, p.T, pos, cbase);
        else if (p.err)
          atomicOr(p.err, DEV_ERR_BAD_CSR);
      }
      const float* ldj = ld + (j % C::RING) * (C::LD_BYTES / 4);
      // dK/dV reads the lse/delta the producer staged with this chunk
      if (DKDV && !__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_CF + j % C::RING),
                                                     (j / C::RING) & 1, abort_flag, p.err))) {
        alive = false;
        break;
      }
      if (!__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_SF), j & 1, abort_flag, p.err))) {
        alive = false;
        break;
      }
      tc_fence_after();
      // ---- P (P^T): 32 columns of S
      float pv[C::CW];
      tmem_ld32(lane_base + C::COL_S + col0, pv);
      if (!DKDV) {
        // dQ keeps P in registers: S's columns are free for the next S now
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(C::BAR_PR));
      }
      // warp-uniform: no element of this warp's 32 x 32 block is masked
      const bool all_valid = (st == ST_FULL) && (!DKDV || cbase + C::CW <= p.T);
      const float4* l4 = reinterpret_cast<const float4*>(ldj + col0);
      const uint64_t c2 = f2_bits(p.scale_log2, p.scale_log2);
      const uint64_t nlog2e2 = f2_bits(-LOG2E, -LOG2E);
#pragma unroll
      for (int q = 0; q < C::CW / 4; ++q) {
        // exponent arguments s c - lse log2 e, two columns per f32x2 op
        uint64_t nl01, nl23;
        if (DKDV) {
          const float4 a4 = l4[q];
          nl01 = fmul2(f2_bits(a4.x, a4.y), nlog2e2);
          nl23 = fmul2(f2_bits(a4.z, a4.w), nlog2e2);
        } else {
          nl01 = nl23 = f2_bits(-row_lse2, -row_lse2);
        }
        float x[4];
        f2_split(ffma2(f2_bits(pv[4 * q], pv[4 * q + 1]), c2, nl01), x[0], x[1]);
        f2_split(ffma2(f2_bits(pv[4 * q + 2], pv[4 * q + 3]), c2, nl23), x[2], x[3]);
        if (all_valid) {
#pragma unroll
          for (int i = 0; i < 4; ++i) pv[4 * q + i] = ex2_approx(x[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            pv[4 * q + i] = ((vw >> (4 * q + i)) & 1u) ? ex2_approx(x[i]) : 0.f;
        }
      }
      if (DKDV) {
        // P^T over the S columns this warp has read; it feeds dV
        uint32_t wp[C::CW / 2];
#pragma unroll
        for (int i = 0; i < C::CW / 2; ++i) wp[i] = pack_bf16(pv[2 * i], pv[2 * i + 1]);
        tmem_st16u(lane_base + C::COL_S + col0, wp);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(C::BAR_PR));
      }
      // ---- dS (dS^T) = P (dP - delta)
      if (!__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_DPF), j & 1, abort_flag, p.err))) {
        alive = false;
        break;
      }
      tc_fence_after();
      const float4* d4 = reinterpret_cast<const float4*>(ldj + C::CN + col0);
      uint32_t wd[C::CW / 2];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float dp[16];
        tmem_ld16(lane_base + C::COL_DP + col0 + 16 * hf, dp);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float dl[4];
          if (DKDV) {
            const float4 dd = d4[4 * hf + q];
            dl[0] = dd.x;
            dl[1] = dd.y;
            dl[2] = dd.z;
            dl[3] = dd.w;
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) dl[i] = row_delta;
          }
          const int k = 16 * hf + 4 * q;
          // dS = P (dP - delta), two columns per f32x2 op
          float d[4];
          f2_split(fmul2(f2_bits(pv[k], pv[k + 1]),
                         fsub2(f2_bits(dp[4 * q], dp[4 * q + 1]), f2_bits(dl[0], dl[1]))),
                   d[0], d[1]);
          f2_split(fmul2(f2_bits(pv[k + 2], pv[k + 3]),
                         fsub2(f2_bits(dp[4 * q + 2], dp[4 * q + 3]), f2_bits(dl[2], dl[3]))),
                   d[2], d[3]);
          wd[k / 2] = pack_bf16(d[0], d[1]);
          wd[k / 2 + 1] = pack_bf16(d[2], d[3]);
        }
      }
      if constexpr (FQ) {
        // dS^T into this chunk's dO buffer (SW128, panels of 64 queries) once
        // dV has read it: row r, chunk columns col0 .. col0 + 31
        if (!__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_DVD), j & 1, abort_flag, p.err))) {
          alive = false;
          break;
        }
        const uint32_t dsr = sbase + C::c_off(j % C::RING, 1) +
                             (col0 >> 6) * (C::BM * 128) + r * 128;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t unit = static_cast<uint32_t>((col0 & 63) >> 3) + u;
          st_shared_v4(dsr + ((unit ^ (r & 7u)) << 4),
                       make_uint4(wd[4 * u], wd[4 * u + 1], wd[4 * u + 2], wd[4 * u + 3]));
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(C::BAR_DSR));
        // dQ_c^T: this lane's column quad * 32 + lane of D for the warp's
        // chunk columns col0 .. col0 + 31 (queries cbase ..), read out of the
        // dP columns, released, then added into dq_acc: each instruction adds
        // 32 consecutive floats of one query's row
        if (!__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_DQF), j & 1, abort_flag, p.err))) {
          alive = false;
          break;
        }
        tc_fence_after();
        float dq[32];
        tmem_ld32(lane_base + C::COL_DP + col0, dq);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(C::BAR_DQE));
        const int nq = min(C::CW, p.T - cbase);   // cbase = T for an absent half
        if (nq > 0) {
          float* dst =
              p.dq_acc + (static_cast<int64_t>(bh) * p.T + cbase) * D + quad * 32 + lane;
          if (nq == C::CW) {
#pragma unroll
            for (int i = 0; i < C::CW; ++i) red_add_f32(dst + i * D, dq[i]);
          } else {
#pragma unroll
            for (int i = 0; i < C::CW; ++i)
              if (i < nq) red_add_f32(dst + i * D, dq[i]);
          }
        }
      } else {
        tmem_st16u(lane_base + C::COL_DP + col0, wd);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(C::BAR_DSR));
      }
    }
    // ------------------------------------------------------------ epilogue
    // The accumulators leave through shared memory: each thread writes its
    // row's bf16 values into the SW128 layout of the output tensor maps (the
    // chunk stages are free once the last MMA has completed), then one thread
    // stores the tiles with TMA.  Stored row by row from registers, every warp
    // instruction would touch 32 rows, i.e. 32 cache lines.
    if (alive && n > 0 &&
        !__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_AD), 0, abort_flag, p.err)))
      alive = false;
    if (alive) {
      tc_fence_after();
      constexpr int EW = D / (C::NCW / 4);   // accumulator columns per warp group
#pragma unroll
      for (int acc = 0; acc < (DKDV ? 2 : 1); ++acc) {
        const float mul = acc == 0 ? p.scale : 1.f;  // dK and dQ carry the softmax scale
        const uint32_t stage = sbase + C::OFF_C0 + acc * C::ROW_BYTES;
#pragma unroll
        for (int cc = grp * EW; cc < (grp + 1) * EW; cc += 16) {
          float v[16];
          if (n > 0) {
            tmem_ld16(lane_base + C::COL_ACC0 + acc * D + cc, v);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
          }
#pragma unroll
          for (int i = 0; i < 16; i += 8) {
            const int col = cc + i;   // 8 columns = one 16-byte unit of the 128-byte row
            const uint32_t addr = stage + (col >> 6) * C::PANEL_R + r * 128 +
                                  ((((col & 63) >> 3) ^ (r & 7)) << 4);
            st_shared_v4(addr, make_uint4(pack_bf16(v[i] * mul, v[i + 1] * mul),
                                          pack_bf16(v[i + 2] * mul, v[i + 3] * mul),
                                          pack_bf16(v[i + 4] * mul, v[i + 5] * mul),
                                          pack_bf16(v[i + 6] * mul, v[i + 7] * mul)));
          }
        }
      }
      fence_proxy_async_smem();
    }
    named_barrier_sync(1, C::NCW * 32);
    if (tid == 0 && !*abort_flag) {
#pragma unroll
      for (int acc = 0; acc < (DKDV ? 2 : 1); ++acc)
#pragma unroll
        for (int pn = 0; pn < D / 64; ++pn)
          tma_store_4d(acc == 0 ? &tm_o0 : &tm_o1,
                       sbase + C::OFF_C0 + acc * C::ROW_BYTES + pn * C::PANEL_R, pn * 64,
                       tile * C::BM, h, b);
      bulk_commit_group();
      bulk_wait_read_all();   // the source must stay valid until it has been read
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
