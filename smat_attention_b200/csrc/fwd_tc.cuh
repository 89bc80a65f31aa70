// Block-sparse causal softmax attention, forward, bf16 on sm_100a tensor cores.
//
// One CTA computes TWO adjacent 128-row query tiles of one (batch, head).
// Their CSR rows overlap almost entirely (same sinks and summary blocks,
// windows shifted by one block), so the CTA walks the union of the rows in
// chunks of 128 keys, loads each K/V chunk once, and runs it against
// whichever of the two tiles it is active for:
//
//   S_x  = Q_x K^T          tcgen05.mma 128 x 128, A = Q_x (smem), B = K (smem)
//   P_x  = exp2(S_x c - m)  softmax warpgroup x, online max, lazy rescale;
//                           P (bf16) is written back over S_x in TMEM
//   O_x += P_x V            tcgen05.mma 128 x D, A = P_x (TMEM), B = V (smem, MN-major)
//
// Every MMA has N = 128 (or D): on B200 an N = 64 MMA costs nearly as many
// cycles as an N = 128 one.  Each tile has one S buffer (TMEM: S_x 128
// columns + O_x D columns per tile); the MMA warp alternates the tiles --
// PV_0(j), S_0(j+1), PV_1(j), S_1(j+1) -- so while warpgroup 0 turns S_0 into
// P_0 the tensor core works on tile 1, and the other way round.  With
// bs = 64 a chunk is two 64-key blocks of the merged list; a missing second
// half is loaded from row T (zero-filled) and masked.
//
// Warp roles (384 threads; 256 with one tile per CTA, see FwdCfg):
//   warps 0-3 / 4-7  softmax + epilogue of tile 0 / tile 1; thread r of a
//                    warpgroup owns row r of its tile = TMEM lane r
//   warp 8           TMA producer (lane 0: both Q tiles, then the K ring;
//                    lane 1: the V ring)
//   warp 9           TMEM allocator and MMA issuer (one lane)
//   warps 10-11      idle (they complete the last warpgroup)
// The softmax warpgroups take registers from warpgroup 2 (setmaxnreg) so a
// thread holds its whole 128-score row: S is read from TMEM once per chunk.
// P of key half h (keys 64 h .. 64 h + 63) is packed into the first 32 of
// that half's own S columns.
// Masked scores become -inf before the row max, so a key outside the mask
// never enters the max or the sum.  Each quarter's mask is one 32-bit word per
// row: all ones for a full block, a span for the causal diagonal, and for an
// M^(d) PATTERN tile the word pattern.cuh evaluates from the C bit tables.  A
// row may see no visible key in a tile (its max stays -inf, its P is 0).
#pragma once

#include "common.cuh"
#include "schedule.cuh"

namespace smat {

struct FwdParams {
  const int32_t* indptr;
  const int32_t* indices;
  const uint8_t* kind;
  __nv_bfloat16* o;
  float* lse;
  int64_t o_sb, o_sh, o_st;  // element strides of O over (b, h, t); d stride is 1
  int B, H, T, nblocks, nnzb, bs, n_tiles, n_pairs;
  const int32_t* work;       // optional work list (one item per CTA and (b, h)); null = all tiles
  float scale_log2;          // softmax scale * log2(e)
  int32_t* err;
  MdPattern md;              // tables of PATTERN tiles (null row_bits: the layout has none)
};

// NT_ query tiles per CTA: 2 (one CTA per SM; its two softmax warpgroups
// alternate on the tensor core) or 1 (D = 64 only: several CTAs per SM
// alternate, and one CTA's set-up and epilogue overlap the others' chunks).
// BN_ keys per chunk: 128, or 64 (D = 64 with 64-row blocks, one tile per
// CTA): a tile then needs 128 TMEM columns and four CTAs share an SM (64
// registers each at launch: the softmax warpgroup takes 96, the others 32,
// with a small spill; c2 0.209 ms against 0.223 with three CTAs at 112 / 48).
template <int D, int NT_, int BN_ = 128>
struct FwdCfg {
  static constexpr int BM = 128, NT = NT_, BN = BN_, BOX = 64;
  static_assert(NT == 2 || (NT == 1 && D == 64), "tiles per CTA");
  static_assert(BN == 128 || (BN == 64 && D == 64 && NT == 1), "keys per chunk");
  static constexpr int NH = BN / 64, NQ = BN / 32;   // 64-key halves, 32-key quarters
  static constexpr int MIN_BLOCKS = BN == 64 ? 4 : 3 - NT;   // CTAs per SM
  // per-CTA shared memory: the SM's 228 KB shared by MIN_BLOCKS CTAs (1 KB
  // reserved each)
  static constexpr int SMEM_CAP =
      (MIN_BLOCKS == 1 ? 227 : (MIN_BLOCKS == 2 ? 113 : (MIN_BLOCKS == 3 ? 75 : 56))) * 1024;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int PANEL_Q = BM * 128, PANEL_KV = BN * 128;  // 64-column SW128 panels
  // K and V have separate rings: K_j is read by S(j) only and frees its slot
  // early, V_j by PV(j) only; the shared memory left over after Q holds
  // KS + VS chunk slots, K taking the larger share (at most 8 each)
  static constexpr int FIXED = NT * Q_BYTES + 2048;  // + barriers, alignment
  static constexpr int SLOTS = (SMEM_CAP - FIXED) / KV_BYTES;
  static constexpr int VS = (SLOTS / 2) > 8 ? 8 : SLOTS / 2;
  static constexpr int KS = (SLOTS - VS) > 8 ? 8 : SLOTS - VS;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + NT * Q_BYTES;
  static constexpr int OFF_V = OFF_K + KS * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + VS * KV_BYTES;
  // barriers: q_full, k_full[KS], k_empty[KS], v_full[VS], v_empty[VS],
  // s_full[NT], p_full[NT], pv_done[NT], drain
  static constexpr int BAR_Q = 0, BAR_KF = 1, BAR_KE = 1 + KS, BAR_VF = 1 + 2 * KS,
                       BAR_VE = BAR_VF + VS, BAR_SF = BAR_VE + VS, BAR_PF = BAR_SF + NT,
                       BAR_PV = BAR_PF + NT, BAR_DRAIN = BAR_PV + NT, NBAR = BAR_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;  // tmem ptr, abort flag
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
  static_assert(SMEM_BYTES <= SMEM_CAP, "shared memory budget");
  static_assert(KS >= 2 && VS >= 2, "at least two slots per ring");
  static constexpr int TILE_COLS = BN + D <= 128 ? 128 : 256, COL_O = BN;
  static constexpr int TMEM_COLS = NT * TILE_COLS;
  static_assert(COL_O + D <= TILE_COLS && TMEM_COLS * MIN_BLOCKS <= 512, "TMEM budget");
  // warpgroups 0 (and 1) softmax, the last warpgroup the producer and MMA
  // warps (and two idle ones, so that every warpgroup is whole for the
  // register split)
  static constexpr int PRODUCER_WARP = 4 * NT, MMA_WARP = 4 * NT + 1;
  static constexpr int THREADS = 128 * (NT + 1);
  static constexpr int REGS_LAUNCH = (65536 / (THREADS * MIN_BLOCKS)) & ~7;   // 168 / 128
  static constexpr int REGS_SOFTMAX = NT == 2 ? 192 : (MIN_BLOCKS == 2 ? 176 : 96);
  static constexpr int REGS_OTHER = NT == 2 ? 112 : (MIN_BLOCKS == 2 ? 80 : 32);
  static_assert(128 * (NT * REGS_SOFTMAX + REGS_OTHER) <= THREADS * REGS_LAUNCH,
                "register split exceeds the launch allocation");
  static constexpr uint32_t IDESC_S = idesc_bf16(BM, BN, false, false);
  static constexpr uint32_t IDESC_O = idesc_bf16(BM, D, false, true);
};

// TMEM column of P's k-step kk (16 keys): key half kk / 4 packed at the start
// of that half's S columns
__device__ __forceinline__ uint32_t p_col(int kk) { return 64u * (kk >> 2) + 8u * (kk & 3); }

template <int D, int NT, int BN>
__global__ void __launch_bounds__(FwdCfg<D, NT, BN>::THREADS, FwdCfg<D, NT, BN>::MIN_BLOCKS)
    smat_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_o, const FwdParams p) {
  using C = FwdCfg<D, NT, BN>;
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
  int bh_sel = lin % BH;
  int tile0, ntile;
  if (p.work) {
    // caller-chosen tiles (a shard of the queries), in the caller's order.
    // With one tile per CTA an item takes two CTAs (the second returns at
    // once for a single-tile item), so every tile walks its own chunk list
    // exactly as in the launch without a work list -- the per-row results
    // are bitwise the same.
    constexpr int PER = 3 - NT;   // CTAs per item
    const int w = __ldg(p.work + lin / (BH * PER));
    const int half = (lin / BH) % PER;
    tile0 = (w & WORK_TILE_MASK) + half;
    ntile = (w & WORK_PAIR_BIT) ? 2 : 1;
    if ((w >> 25) != 0 || (w & WORK_TILE_MASK) + ntile > p.n_tiles) {
      if (threadIdx.x == 0 && p.err) atomicOr(p.err, DEV_ERR_BAD_WORK);
      return;
    }
    if (NT == 1) {
      if (half >= ntile) return;
      ntile = 1;
    }
  } else {
    // heaviest (latest) tiles first, one tile index across a group of 16
    // (b, h) at a time (across all of them: c3 forward 2.32-2.35 ms against
    // 2.28 -- the resident CTAs then span more heads' K / V than L2 holds)
    const int np = (p.n_tiles + NT - 1) / NT;
    constexpr int G = 16;
    const int grp = lin / (G * np);
    const int g0 = grp * G, gs = min(G, BH - g0);
    const int rr = lin - grp * G * np;
    bh_sel = g0 + rr % gs;
    tile0 = NT * (np - 1 - rr / gs);
    ntile = min(NT, p.n_tiles - tile0);
  }
  const int bh = bh_sel;
  const int b = bh / p.H, h = bh % p.H;
  const int sub = C::BM / p.bs;   // CSR rows per tile: 1 (bs 128) or 2 (bs 64)
  const int row0 = tile0 * sub;
  // is entry pair e active for tile x (any of its CSR rows)?
  auto active = [&](const uint32_t* e, int x) {
    return (sched_states(e[0], x * sub, sub) | sched_states(e[1], x * sub, sub)) != 0u;
  };

  if (tid == 0) {
    mbar_init(bar(C::BAR_Q), 1);
    for (int s = 0; s < C::KS; ++s) {
      mbar_init(bar(C::BAR_KF + s), 1);
      mbar_init(bar(C::BAR_KE + s), 1);
    }
    for (int s = 0; s < C::VS; ++s) {
      mbar_init(bar(C::BAR_VF + s), 1);
      mbar_init(bar(C::BAR_VE + s), 1);
    }
    for (int x = 0; x < C::NT; ++x) {
      mbar_init(bar(C::BAR_SF + x), 1);
      mbar_init(bar(C::BAR_PF + x), 4);
      mbar_init(bar(C::BAR_PV + x), 1);
    }
    mbar_init(bar(C::BAR_DRAIN), 1);
    fence_barrier_init();
    misc[1] = 0;
  }
  if (warp == C::MMA_WARP) {
    tmem_alloc(sbase + C::OFF_MISC, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == C::PRODUCER_WARP && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = misc[0];

  // Each warpgroup changes its register count at the top of its own branch, so
  // that no code path joins between the change and the role's code.
  if (warp >= C::PRODUCER_WARP) {
    regs_dec<C::REGS_OTHER>();
    if (warp == C::PRODUCER_WARP) {
      // ------------------------------------------------------------ producer
      // lane 0: both Q tiles, then the K ring; lane 1: the V ring.  Each lane
      // walks the schedule on its own, so a V slot that frees late never holds
      // up the next K load.
      if (lane < 2) {
        const bool kl = lane == 0;
        const int NS = kl ? C::KS : C::VS;
        const int full = kl ? C::BAR_KF : C::BAR_VF, empty = kl ? C::BAR_KE : C::BAR_VE;
        const uint32_t ring = sbase + (kl ? C::OFF_K : C::OFF_V);
        const CUtensorMap* tm = kl ? &tm_k : &tm_v;
        // the Q tiles first: they do not depend on the schedule reads
        if (kl) {
          mbar_expect_tx(bar(C::BAR_Q), C::NT * C::Q_BYTES);
  #pragma unroll
          for (int x = 0; x < C::NT; ++x)
  #pragma unroll
            for (int pn = 0; pn < D / 64; ++pn)
              tma_load_4d(sbase + C::OFF_Q + x * C::Q_BYTES + pn * C::PANEL_Q, &tm_q,
                          bar(C::BAR_Q), pn * 64, (tile0 + x) * C::BM, h, b);
        }
        ChunkPair<2 * NT> it;
        it.init(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, row0, ntile * sub, p.bs, p.err,
                C::BN);
        int issued = 0;
        uint32_t e[2];
        for (int j = 0; it.next(e, p.err); ++j) {
          const int s = j % NS;
          if (j >= NS && !mbar_wait(bar(empty + s), ((j / NS) - 1) & 1, abort_flag, p.err)) break;
          // first key of each 64-key half; a missing half reads row T onwards,
          // which TMA fills with zeros
          int krow[2] = {p.T, p.T};
  #pragma unroll
          for (int q = 0; q < C::NH; ++q) {
            const uint32_t eq = (p.bs == 64) ? e[q] : e[0];
            krow[q] = entry_present(eq) ? static_cast<int>(sched_block(eq)) * p.bs + (q * 64) % p.bs
                                        : p.T;
          }
          mbar_expect_tx(bar(full + s), C::KV_BYTES);
  #pragma unroll
          for (int pn = 0; pn < D / 64; ++pn)
  #pragma unroll
            for (int q = 0; q < C::NH; ++q)
              tma_load_4d(ring + s * C::KV_BYTES + pn * C::PANEL_KV + q * (C::BOX * 128), tm,
                          bar(full + s), pn * 64, krow[q], h, b);
          issued = j + 1;
        }
        if (kl) mbar_wait_drain(bar(C::BAR_Q), 0);  // never exit with Q in flight
        if (*abort_flag) {
          for (int j = max(0, issued - NS); j < issued; ++j)
            mbar_wait_drain(bar(full + j % NS), (j / NS) & 1);
        }
      }
    } else if (warp == C::MMA_WARP) {
      // ------------------------------------------------------------ MMA issuer
      if (lane == 0) {
        ChunkPair<2 * NT> it;
        it.init(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, row0, ntile * sub, p.bs, p.err,
                C::BN);
        int cp[C::NT] = {};   // PVs issued per tile
        // S_x of chunk j (K slot j % KS)
        auto issue_s = [&](int j, int x) {
          const uint32_t ka = sbase + C::OFF_K + (j % C::KS) * C::KV_BYTES;
          const uint32_t qa = sbase + C::OFF_Q + x * C::Q_BYTES;
          const uint32_t dst = tbase + x * C::TILE_COLS;
          const uint64_t qd = sdesc_sw128(qa, 16, 1024), kd = sdesc_sw128(ka, 16, 1024);
  #pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk & 3) * 32u;
            tc_mma(dst, sdesc_add(qd, (kk >> 2) * C::PANEL_Q + off),
                   sdesc_add(kd, (kk >> 2) * C::PANEL_KV + off), C::IDESC_S, kk > 0 ? 1u : 0u);
          }
          tc_commit(bar(C::BAR_SF + x));
        };
        bool ok = mbar_wait(bar(C::BAR_Q), 0, abort_flag, p.err);
        uint32_t e[2], en[2];
        bool has = ok && it.next(e, p.err);
        if (has) {
          ok = mbar_wait(bar(C::BAR_KF + 0), 0, abort_flag, p.err);
          if (ok) {
            tc_fence_after();
  #pragma unroll
            for (int x = 0; x < C::NT; ++x)
              if (active(e, x)) issue_s(0, x);
            tc_commit(bar(C::BAR_KE + 0));   // every S of chunk 0 is issued
          }
        }
        for (int j = 0; ok && has; ++j) {
          const bool nxt = it.next(en, p.err);
          const int sv = j % C::VS;
          const int k1 = (j + 1) % C::KS;
          const int k1par = ((j + 1) / C::KS) & 1;
          const uint32_t va = sbase + C::OFF_V + sv * C::KV_BYTES;
          if (!mbar_wait(bar(C::BAR_VF + sv), (j / C::VS) & 1, abort_flag, p.err)) break;
          bool loaded = false;     // K of chunk j + 1 has landed
          bool pending[C::NT] = {};
  #pragma unroll
          for (int x = 0; x < C::NT; ++x) {
            if (active(e, x)) {
              if (!mbar_wait(bar(C::BAR_PF + x), cp[x] & 1, abort_flag, p.err)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t pa = tbase + x * C::TILE_COLS;   // P in TMEM
              const uint32_t dst = pa + C::COL_O;
              // V is MN-major: 64-column panels BN*128 bytes apart (LBO),
              // 8-row groups 1024 bytes apart (SBO); 16 rows per k-step
              const uint64_t vd = sdesc_sw128(va, C::PANEL_KV, 1024);
  #pragma unroll
              for (int kk = 0; kk < C::BN / 16; ++kk)
                tc_mma_ts(dst, pa + p_col(kk), sdesc_add(vd, kk * 2048), C::IDESC_O,
                          (cp[x] > 0 || kk > 0) ? 1u : 0u);
              tc_commit(bar(C::BAR_PV + x));
              ++cp[x];
            }
            // the tile's next S goes in behind its PV if the K chunk has landed
            if (nxt && active(en, x)) {
              if (!loaded) loaded = mbar_try_wait(bar(C::BAR_KF + k1), k1par);
              if (loaded) {
                tc_fence_after();
                issue_s(j + 1, x);
              } else {
                pending[x] = true;
              }
            }
          }
          if (!ok) break;
          tc_commit(bar(C::BAR_VE + sv));   // V_j is read by both PVs
          bool any_pending = false;
  #pragma unroll
          for (int x = 0; x < C::NT; ++x) any_pending |= pending[x];
          if (any_pending) {
            if (!mbar_wait(bar(C::BAR_KF + k1), k1par, abort_flag, p.err)) break;
            tc_fence_after();
  #pragma unroll
            for (int x = 0; x < C::NT; ++x)
              if (pending[x]) issue_s(j + 1, x);
          }
          if (nxt) tc_commit(bar(C::BAR_KE + k1));   // every S of chunk j + 1 is issued
          e[0] = en[0];
          e[1] = en[1];
          has = nxt;
        }
        if (*abort_flag) {  // let the MMAs in flight finish before TMEM is freed
          tc_commit(bar(C::BAR_DRAIN));
          mbar_wait_drain(bar(C::BAR_DRAIN), 0);
        }
      }
    }
  } else {
    regs_inc<C::REGS_SOFTMAX>();
    // ------------------------------------------------------------ softmax
    const int x = warp >> 2;                   // tile of this warpgroup
    const int r = (warp & 3) * 32 + lane;      // row within the tile = TMEM lane
    const int q_pos = (tile0 + x) * C::BM + r;
    const bool store = x < ntile && q_pos < p.T;   // rows this CTA writes
    const int srow = x * sub + ((sub == 2) ? (r >> 6) : 0);   // CSR row of this query
    const uint32_t lane_base =
        tbase + (static_cast<uint32_t>((warp & 3) * 32) << 16) + x * C::TILE_COLS;
    float m = -INFINITY, l = 0.f;
    int cnt = 0;
    bool alive = true;
    ChunkPair<2 * NT> it;
    it.init(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, row0, ntile * sub, p.bs, p.err,
                C::BN);
    uint32_t e[2];
    while (alive && it.next(e, p.err)) {
      if (!active(e, x)) continue;
      // per 64-key half: state of this row (warp-uniform) and first key
      uint32_t st[2] = {ST_ABSENT, ST_ABSENT};
      int k0[2] = {0, 0};
#pragma unroll
      for (int hf = 0; hf < C::NH; ++hf) {
        const uint32_t eh = (p.bs == 64) ? e[hf] : e[0];
        st[hf] = entry_present(eh) ? sched_state(eh, srow) : ST_ABSENT;
        k0[hf] = static_cast<int>(sched_block(eh)) * p.bs + (hf * 64) % p.bs;
      }
      // visibility words of the four quarters (bit i: key 32 qq + i of the
      // chunk); computed before the wait so pattern-table loads overlap it
      auto qword = [&](int qq) -> uint32_t {
        const uint32_t sq = (qq >> 1) ? st[1] : st[0];
        const int kq = ((qq >> 1) ? k0[1] : k0[0]) + 32 * (qq & 1);
        if (sq == ST_FULL) return 0xffffffffu;
        if (sq == ST_CAUSAL) return span_word(kq, 0, q_pos + 1);
        if (sq == ST_PATTERN && p.md.row_bits) return md_row_word(p.md, p.T, q_pos, kq);
        if (sq == ST_PATTERN && p.err) atomicOr(p.err, DEV_ERR_BAD_CSR);
        return 0u;
      };
      uint32_t mw[C::NQ];
#pragma unroll
      for (int qq = 0; qq < C::NQ; ++qq) mw[qq] = qword(qq);
      if (!__all_sync(0xffffffffu,
                      mbar_wait(bar(C::BAR_SF + x), cnt & 1, abort_flag, p.err))) {
        alive = false;
        break;
      }
      tc_fence_after();
      // the whole row of scores in one TMEM read
      float s[C::BN];
      if constexpr (C::BN == 128)
        tmem_ld128(lane_base, s);
      else
        tmem_ld32x2(lane_base, lane_base + 32, s, s + 32);
      // quarter qq (32 keys, TMEM columns 32 qq ..): mask of this row
#pragma unroll
      for (int qq = 0; qq < C::NQ; ++qq) {
        const uint32_t sq = (qq >> 1) ? st[1] : st[0];
        if (sq != ST_FULL) {   // uniform per warp: its 32 rows share one CSR row
          const uint32_t w = mw[qq];
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (!((w >> i) & 1u)) s[32 * qq + i] = -INFINITY;
        }
      }
      float mx[8];   // three-input max: BN / 2 instructions per BN scores
#pragma unroll
      for (int a = 0; a < 8; ++a) mx[a] = s[a];
#pragma unroll
      for (int i = 8; i < C::BN; i += 2) mx[(i >> 1) & 7] = fmax3(mx[(i >> 1) & 7], s[i], s[i + 1]);
      const float m_new = fmaxf(
          m, fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7])) *
                 p.scale_log2);
      const bool need = m_new > m + 8.0f;
      const bool rescale = __any_sync(0xffffffffu, need);
      const float alpha = need ? ex2_approx(m - m_new) : 1.f;
      if (need) {
        l *= alpha;
        m = m_new;
      }
      const float neg_m = (m == -INFINITY) ? 0.f : -m;
      const uint64_t c2 = f2_bits(p.scale_log2, p.scale_log2), nm2 = f2_bits(neg_m, neg_m);
      uint64_t rs2[4];   // row-sum partials, two lanes each (f32x2)
#pragma unroll
      for (int a = 0; a < 4; ++a) rs2[a] = 0ull;
      // P of quarter qq packed into 16 columns at the start of its half's S
      // columns (64 h + 16 (qq % 2))
#pragma unroll
      for (int qq = 0; qq < C::NQ; ++qq) {
        uint32_t pw[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float xa, xb;
          f2_split(ffma2(f2_bits(s[32 * qq + 2 * i], s[32 * qq + 2 * i + 1]), c2, nm2), xa, xb);
          const float a = ex2_approx(xa), bb = ex2_approx(xb);
          rs2[i & 3] = fadd2(rs2[i & 3], f2_bits(a, bb));
          pw[i] = pack_bf16(a, bb);
        }
        tmem_st16u(lane_base + 64 * (qq >> 1) + 16 * (qq & 1), pw);
      }
      rs2[0] = fadd2(fadd2(rs2[0], rs2[1]), fadd2(rs2[2], rs2[3]));
      float rlo, rhi;
      f2_split(rs2[0], rlo, rhi);
      l += rlo + rhi;
      // O may be rescaled only once this tile's previous PV has completed
      if (rescale && cnt > 0) {
        if (!__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_PV + x), (cnt - 1) & 1, abort_flag,
                                               p.err))) {
          alive = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < D; cc += 32) {
          float ov[32];
          tmem_ld32(lane_base + C::COL_O + cc, ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= alpha;
          tmem_st32(lane_base + C::COL_O + cc, ov);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C::BAR_PF + x));
      ++cnt;
    }
    // ------------------------------------------------------------ epilogue
    if (alive && cnt > 0 &&
        !__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_PV + x), (cnt - 1) & 1, abort_flag, p.err)))
      alive = false;
    // O leaves through shared memory: each thread writes its row in the SW128
    // layout of the output tensor map into its tile's Q buffer (free once the
    // tile's last MMA has completed; a tile without chunks first lets its Q
    // load land), then one thread per warpgroup stores the tile with TMA.
    if (alive && cnt == 0 &&
        !__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_Q), 0, abort_flag, p.err)))
      alive = false;
    const uint32_t stage = sbase + C::OFF_Q + x * C::Q_BYTES;
    if (alive) {
      tc_fence_after();
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
#pragma unroll
      for (int cc = 0; cc < D; cc += 32) {
        float ov[32];
        if (cnt > 0) {
          tmem_ld32(lane_base + C::COL_O + cc, ov);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          const int col = cc + i;   // 8 columns = one 16-byte unit of the 128-byte row
          const uint32_t addr = stage + (col >> 6) * C::PANEL_Q + r * 128 +
                                ((((col & 63) >> 3) ^ (r & 7)) << 4);
          st_shared_v4(addr, make_uint4(pack_bf16(ov[i] * inv, ov[i + 1] * inv),
                                        pack_bf16(ov[i + 2] * inv, ov[i + 3] * inv),
                                        pack_bf16(ov[i + 4] * inv, ov[i + 5] * inv),
                                        pack_bf16(ov[i + 6] * inv, ov[i + 7] * inv)));
        }
      }
      fence_proxy_async_smem();
      if (store)
        p.lse[static_cast<int64_t>(bh) * p.T + q_pos] =
            (l > 0.f) ? (m + __log2f(l)) * 0.69314718055994531f : -INFINITY;
    }
    named_barrier_sync(1 + x, 128);
    if ((warp & 3) == 0 && lane == 0 && x < ntile && !*abort_flag) {
#pragma unroll
      for (int pn = 0; pn < D / 64; ++pn)
        tma_store_4d(&tm_o, stage + pn * C::PANEL_Q, pn * 64, (tile0 + x) * C::BM, h, b);
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
