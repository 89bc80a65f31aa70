// Block-sparse causal softmax attention, forward, bf16 on sm_100a tensor cores.
//
// One CTA computes TWO adjacent 128-row query tiles of one (batch, head).
// Their CSR rows overlap almost entirely (same sinks and summary blocks,
// windows shifted by one block), so the CTA walks the union of the rows in
// 64-key chunks, loads each K/V chunk once, and runs it against whichever of
// the two tiles it is active for:
//
//   S_x  = Q_x K^T          tcgen05.mma, A = Q_x (smem), B = K (smem), D in TMEM
//   P_x  = exp2(S_x c - m)  softmax warpgroup x, online max, lazy rescale;
//                           P (bf16) is written back over S_x in TMEM
//   O_x += P_x V            tcgen05.mma, A = P_x (TMEM), B = V (smem, MN-major)
//
// While warpgroup 0 turns S_0 into P_0, the tensor core works on tile 1 and
// the other way round.  Warp roles (320 threads):
//   warps 0-3 / 4-7  softmax + epilogue of tile 0 / tile 1; thread r of a
//                    warpgroup owns row r of its tile = TMEM lane r
//   warp 8           TMA producer (both Q tiles once, then the K/V ring)
//   warp 9           TMEM allocator and MMA issuer (one lane)
// TMEM (512 columns): tile x owns [256 x, 256 x + 256): S / P double buffer
// at +0 / +64 (P packs two bf16 per column into the first 32), O at +128.
// Shared memory (SWIZZLE_128B panels of 64 bf16 columns, 128-byte rows):
// Q [2][128 x D], K ring and V ring [STAGES][64 x D].
// Masked scores become -inf before the row max, so a key outside the mask
// never enters the max or the sum.
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
};

template <int D>
struct FwdCfg {
  static constexpr int BM = 128, NT = 2, BN = 64;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  // as many K/V stages as the shared memory holds (at most 8): the ring hides
  // the L2 -> shared latency of the loads
  static constexpr int FIXED = NT * Q_BYTES + 1536;  // + barriers, alignment
  static constexpr int STAGES_FIT = (227 * 1024 - FIXED) / (2 * KV_BYTES);
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + NT * Q_BYTES;
  static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + STAGES * KV_BYTES;
  // barriers: q_full, kv_full[S], kv_empty[S], s_full[NT][2], p_full[NT][2], pv_done[NT], drain
  static constexpr int BAR_Q = 0, BAR_KVF = 1, BAR_KVE = 1 + STAGES, BAR_SF = 1 + 2 * STAGES,
                       BAR_PF = BAR_SF + 2 * NT, BAR_PV = BAR_PF + 2 * NT, BAR_DRAIN = BAR_PV + NT,
                       NBAR = BAR_DRAIN + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;  // tmem ptr, abort flag
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + alignment slack
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static_assert(STAGES >= 2, "at least two stages");
  static constexpr int TMEM_COLS = 512, TILE_COLS = 256, COL_O = 128;
  static constexpr int THREADS = 320;
  static constexpr uint32_t IDESC_S = idesc_bf16(BM, BN, false, false);
  static constexpr uint32_t IDESC_O = idesc_bf16(BM, D, false, true);
};

// Walks a merged CSR schedule in 64-row chunks (blocks of 128 rows give two
// chunks each).
template <int MAXROWS>
struct ChunkIter {
  MergeIter<MAXROWS> it;
  uint32_t e;
  int sub, cpb;
  __device__ __forceinline__ void init(const int32_t* indptr, const int32_t* indices,
                                       const uint8_t* kind, int nblocks, int nnzb, int row0,
                                       int nrows, int cpb_, int32_t* err) {
    it.init(indptr, indices, kind, nblocks, nnzb, row0, nrows, err);
    cpb = cpb_;
    sub = cpb_;
    e = 0;
  }
  __device__ __forceinline__ bool next(uint32_t& entry, int& c, int32_t* err) {
    if (sub >= cpb) {
      if (!it.next(e, err)) return false;
      sub = 0;
    }
    entry = e;
    c = sub++;
    return true;
  }
};

template <int D>
__global__ void __launch_bounds__(320, 1)
    smat_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  using C = FwdCfg<D>;
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
  int tile0, ntile;
  if (p.work) {
    // caller-chosen tiles (a shard of the queries), in the caller's order
    const int w = __ldg(p.work + lin / BH);
    tile0 = w & WORK_TILE_MASK;
    ntile = (w & WORK_PAIR_BIT) ? 2 : 1;
    if ((w >> 25) != 0 || tile0 + ntile > p.n_tiles) {
      if (threadIdx.x == 0 && p.err) atomicOr(p.err, DEV_ERR_BAD_WORK);
      return;
    }
  } else {
    tile0 = 2 * (p.n_pairs - 1 - lin / BH);  // heaviest (latest) tiles first
    ntile = min(2, p.n_tiles - tile0);
  }
  const int b = bh / p.H, h = bh % p.H;
  const int sub = C::BM / p.bs;   // CSR rows per tile: 1 (bs 128) or 2 (bs 64)
  const int cpb = p.bs / C::BN;   // chunks per block: 2 (bs 128) or 1 (bs 64)
  const int row0 = tile0 * sub;

  if (tid == 0) {
    mbar_init(bar(C::BAR_Q), 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar(C::BAR_KVF + s), 1);
      mbar_init(bar(C::BAR_KVE + s), 1);
    }
    for (int i = 0; i < 2 * C::NT; ++i) {
      mbar_init(bar(C::BAR_SF + i), 1);
      mbar_init(bar(C::BAR_PF + i), 4);
    }
    for (int x = 0; x < C::NT; ++x) mbar_init(bar(C::BAR_PV + x), 1);
    mbar_init(bar(C::BAR_DRAIN), 1);
    fence_barrier_init();
    misc[1] = 0;
  }
  if (warp == 9) {
    tmem_alloc(sbase + C::OFF_MISC, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = misc[0];

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      ChunkIter<4> it;
      it.init(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, row0, ntile * sub, cpb, p.err);
      mbar_expect_tx(bar(C::BAR_Q), C::NT * C::Q_BYTES);
#pragma unroll
      for (int x = 0; x < C::NT; ++x)
#pragma unroll
        for (int pn = 0; pn < D / 64; ++pn)
          tma_load_4d(sbase + C::OFF_Q + x * C::Q_BYTES + pn * (C::BM * 128), &tm_q,
                      bar(C::BAR_Q), pn * 64, (tile0 + x) * C::BM, h, b);
      int issued = 0;
      uint32_t e;
      int c;
      for (int j = 0; it.next(e, c, p.err); ++j) {
        const int s = j % C::STAGES;
        if (j >= C::STAGES &&
            !mbar_wait(bar(C::BAR_KVE + s), ((j / C::STAGES) - 1) & 1, abort_flag, p.err))
          break;
        const int row = static_cast<int>(sched_block(e)) * p.bs + c * C::BN;
        mbar_expect_tx(bar(C::BAR_KVF + s), 2 * C::KV_BYTES);
#pragma unroll
        for (int pn = 0; pn < D / 64; ++pn) {
          tma_load_4d(sbase + C::OFF_K + s * C::KV_BYTES + pn * (C::BN * 128), &tm_k,
                      bar(C::BAR_KVF + s), pn * 64, row, h, b);
          tma_load_4d(sbase + C::OFF_V + s * C::KV_BYTES + pn * (C::BN * 128), &tm_v,
                      bar(C::BAR_KVF + s), pn * 64, row, h, b);
        }
        issued = j + 1;
      }
      mbar_wait_drain(bar(C::BAR_Q), 0);  // Q is always loaded; never exit with it in flight
      if (*abort_flag) {
        for (int j = max(0, issued - C::STAGES); j < issued; ++j)
          mbar_wait_drain(bar(C::BAR_KVF + j % C::STAGES), (j / C::STAGES) & 1);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      ChunkIter<4> it;
      it.init(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, row0, ntile * sub, cpb, p.err);
      int cs[C::NT] = {0, 0}, cp[C::NT] = {0, 0};
      auto active = [&](uint32_t e, int x) { return sched_states(e, x * sub, sub) != 0; };
      auto issue_s = [&](int j, uint32_t e) {
        const int s = j % C::STAGES;
        const uint32_t ka = sbase + C::OFF_K + s * C::KV_BYTES;
#pragma unroll
        for (int x = 0; x < C::NT; ++x) {
          if (!active(e, x)) continue;
          const uint32_t qa = sbase + C::OFF_Q + x * C::Q_BYTES;
          const uint32_t dst = tbase + x * C::TILE_COLS + (cs[x] & 1) * C::BN;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk & 3) * 32u;
            tc_mma(dst, sdesc_sw128(qa + (kk >> 2) * (C::BM * 128) + off, 16, 1024),
                   sdesc_sw128(ka + (kk >> 2) * (C::BN * 128) + off, 16, 1024), C::IDESC_S,
                   kk > 0 ? 1u : 0u);
          }
          tc_commit(bar(C::BAR_SF + 2 * x + (cs[x] & 1)));
          ++cs[x];
        }
      };
      bool ok = mbar_wait(bar(C::BAR_Q), 0, abort_flag, p.err);
      uint32_t e_next = 0;
      int c_next = 0;
      bool has = ok && it.next(e_next, c_next, p.err);
      if (has) {
        ok = mbar_wait(bar(C::BAR_KVF + 0), 0, abort_flag, p.err);
        if (ok) {
          tc_fence_after();
          issue_s(0, e_next);
        }
      }
      for (int j = 0; ok && has; ++j) {
        const uint32_t e = e_next;
        has = it.next(e_next, c_next, p.err);
        // S of the next chunk goes first if its K/V already landed; otherwise
        // the PVs of this chunk are not held up behind that load
        bool early = false;
        if (has && mbar_try_wait(bar(C::BAR_KVF + (j + 1) % C::STAGES), ((j + 1) / C::STAGES) & 1)) {
          tc_fence_after();
          issue_s(j + 1, e_next);
          early = true;
        }
        const int s = j % C::STAGES;
        const uint32_t va = sbase + C::OFF_V + s * C::KV_BYTES;
#pragma unroll
        for (int x = 0; x < C::NT; ++x) {
          if (!active(e, x)) continue;
          if (!mbar_wait(bar(C::BAR_PF + 2 * x + (cp[x] & 1)), (cp[x] >> 1) & 1, abort_flag,
                         p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t pa = tbase + x * C::TILE_COLS + (cp[x] & 1) * C::BN;   // P in TMEM
          const uint32_t dst = tbase + x * C::TILE_COLS + C::COL_O;
#pragma unroll
          for (int kk = 0; kk < C::BN / 16; ++kk) {
            // A: 16 keys = 8 packed columns per k-step.  V is MN-major:
            // 64-column panels BN*128 bytes apart (LBO), 8-row groups 1024
            // bytes apart (SBO); 16 rows per k-step = 2048 bytes.
            tc_mma_ts(dst, pa + kk * 8, sdesc_sw128(va + kk * 2048, C::BN * 128, 1024),
                      C::IDESC_O, (cp[x] > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(bar(C::BAR_PV + x));
          ++cp[x];
        }
        if (!ok) break;
        tc_commit(bar(C::BAR_KVE + s));
        if (has && !early) {
          const int s1 = (j + 1) % C::STAGES;
          if (!mbar_wait(bar(C::BAR_KVF + s1), ((j + 1) / C::STAGES) & 1, abort_flag, p.err)) break;
          tc_fence_after();
          issue_s(j + 1, e_next);
        }
      }
      if (*abort_flag) {  // let the MMAs in flight finish before TMEM is freed
        tc_commit(bar(C::BAR_DRAIN));
        mbar_wait_drain(bar(C::BAR_DRAIN), 0);
      }
    }
  } else {
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
    ChunkIter<4> it;
    it.init(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, row0, ntile * sub, cpb, p.err);
    uint32_t e;
    int c;
    while (alive && it.next(e, c, p.err)) {
      if (sched_states(e, x * sub, sub) == 0) continue;
      const uint32_t st = sched_state(e, srow);
      const int k0 = static_cast<int>(sched_block(e)) * p.bs + c * C::BN;
      if (!__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_SF + 2 * x + (cnt & 1)), (cnt >> 1) & 1,
                                             abort_flag, p.err))) {
        alive = false;
        break;
      }
      tc_fence_after();
      float s[C::BN];
      tmem_ld64(lane_base + (cnt & 1) * C::BN, s);
      if (st != ST_FULL) {   // uniform per warp: its 32 rows share one CSR row
#pragma unroll
        for (int i = 0; i < C::BN; ++i)
          if (!(st == ST_CAUSAL && k0 + i <= q_pos)) s[i] = -INFINITY;
      }
      // row max of the raw scores (scale > 0), eight independent chains
      float mx8[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) mx8[a] = s[a];
#pragma unroll
      for (int i = 8; i < C::BN; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], s[i]);
#pragma unroll
      for (int w = 4; w > 0; w >>= 1)
#pragma unroll
        for (int a = 0; a < w; ++a) mx8[a] = fmaxf(mx8[a], mx8[a + w]);
      const float m_new = fmaxf(m, mx8[0] * p.scale_log2);
      const bool need = m_new > m + 8.0f;
      const bool rescale = __any_sync(0xffffffffu, need);
      const float alpha = need ? ex2_approx(m - m_new) : 1.f;
      if (need) {
        l *= alpha;
        m = m_new;
      }
      // exponentials first: they do not depend on the previous PV
      const float neg_m = (m == -INFINITY) ? 0.f : -m;
      float rs8[8];
      uint32_t pw[C::BN / 2];
#pragma unroll
      for (int i = 0; i < C::BN / 2; ++i) {
        const float a = ex2_approx(fmaf(s[2 * i], p.scale_log2, neg_m));
        const float bb = ex2_approx(fmaf(s[2 * i + 1], p.scale_log2, neg_m));
        if (i < 8) {
          rs8[i] = a + bb;
        } else {
          rs8[i & 7] += a + bb;
        }
        pw[i] = pack_bf16(a, bb);
      }
#pragma unroll
      for (int w = 4; w > 0; w >>= 1)
#pragma unroll
        for (int a = 0; a < w; ++a) rs8[a] += rs8[a + w];
      l += rs8[0];
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
        tmem_st_wait();
      }
      // P over the S columns this thread has already read
      tmem_st32u(lane_base + (cnt & 1) * C::BN, pw);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C::BAR_PF + 2 * x + (cnt & 1)));
      ++cnt;
    }
    // ------------------------------------------------------------ epilogue
    if (alive && cnt > 0 &&
        !__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_PV + x), (cnt - 1) & 1, abort_flag, p.err)))
      alive = false;
    if (alive) {
      tc_fence_after();
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.o + static_cast<int64_t>(b) * p.o_sb +
                            static_cast<int64_t>(h) * p.o_sh + static_cast<int64_t>(q_pos) * p.o_st;
#pragma unroll
      for (int cc = 0; cc < D; cc += 32) {
        float ov[32];
        if (cnt > 0) {
          tmem_ld32(lane_base + C::COL_O + cc, ov);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = 0.f;
        }
        if (store) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w = make_uint4(pack_bf16(ov[i] * inv, ov[i + 1] * inv),
                                 pack_bf16(ov[i + 2] * inv, ov[i + 3] * inv),
                                 pack_bf16(ov[i + 4] * inv, ov[i + 5] * inv),
                                 pack_bf16(ov[i + 6] * inv, ov[i + 7] * inv));
            *reinterpret_cast<uint4*>(orow + cc + i) = w;
          }
        }
      }
      if (store)
        p.lse[static_cast<int64_t>(bh) * p.T + q_pos] =
            (l > 0.f) ? (m + __log2f(l)) * 0.69314718055994531f : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

}  // namespace smat
