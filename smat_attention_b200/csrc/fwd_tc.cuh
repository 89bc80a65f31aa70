// Block-sparse causal softmax attention, forward, bf16 on sm_100a tensor cores.
//
// One CTA computes one 128-row query tile of one (batch, head).  It walks the
// tile's chunk list (the union of its CSR rows, see schedule.cuh) and for each
// active key block of BN rows:
//
//   S   = Q K^T            tcgen05.mma, A = Q (smem), B = K (smem), D in TMEM
//   P   = exp2(S*c - m)    softmax warps, online max with lazy rescale
//   O  += P V              tcgen05.mma, A = P (smem), B = V (smem, MN-major)
//
// Warp roles (192 threads):
//   warps 0-3  softmax + epilogue; thread r owns query row r = TMEM lane r
//   warp 4     TMA producer (Q once, then K/V per chunk into a 2-stage ring)
//   warp 5     TMEM allocator and MMA issuer (one elected lane)
//
// TMEM columns: S double buffer [0, 2 BN), O [2 BN, 2 BN + D).
// Shared memory (all SWIZZLE_128B panels of 64 bf16 columns, 128 B rows):
//   Q [128 x D], K/V ring [STAGES][BN x D] each, P [128 x BN].
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
  int B, H, T, nblocks, nnzb, bs, n_tiles;
  float scale_log2;          // softmax scale * log2(e)
  int32_t* err;
};

template <int D, int BN>
struct FwdCfg {
  static constexpr int BM = 128;
  static constexpr int STAGES = 2;
  static constexpr int SUB = BM / BN;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr int OFF_P = OFF_V + STAGES * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + P_BYTES;
  // barriers: q_full, kv_full[S], kv_empty[S], s_full[2], p_full, pv_done
  static constexpr int BAR_Q = 0, BAR_KVF = 1, BAR_KVE = 1 + STAGES, BAR_SF = 1 + 2 * STAGES,
                       BAR_PF = 3 + 2 * STAGES, BAR_PV = 4 + 2 * STAGES,
                       BAR_DRAIN = 5 + 2 * STAGES, NBAR = 6 + 2 * STAGES;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;  // tmem ptr, abort flag, n_chunks
  static constexpr int OFF_SCHED = OFF_MISC + 16;
  static constexpr int MAX_CHUNKS = 512;
  static constexpr int COL_S = 0, COL_O = 2 * BN;
  static constexpr int TMEM_COLS = (2 * BN + D) <= 256 ? 256 : 512;
  // + alignment slack; a CTA that takes all 512 TMEM columns also takes more
  // than half the shared memory, so a second CTA never waits in tcgen05.alloc
  static constexpr int SMEM_USED = OFF_SCHED + MAX_CHUNKS * 4 + 1024;
  static constexpr int SMEM_BYTES =
      (TMEM_COLS == 512 && SMEM_USED < 120 * 1024) ? 120 * 1024 : SMEM_USED;
  static constexpr int THREADS = 192;
  static constexpr uint32_t IDESC_S = idesc_bf16(BM, BN, false, false);
  static constexpr uint32_t IDESC_O = idesc_bf16(BM, D, false, true);
};

template <int D, int BN>
__global__ void __launch_bounds__(192, 1)
    smat_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  using C = FwdCfg<D, BN>;
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
  const int tile = p.n_tiles - 1 - lin / BH;  // heaviest (latest) tiles first
  const int b = bh / p.H, h = bh % p.H;

  if (tid == 0) {
    mbar_init(bar(C::BAR_Q), 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar(C::BAR_KVF + s), 1);
      mbar_init(bar(C::BAR_KVE + s), 1);
    }
    mbar_init(bar(C::BAR_SF + 0), 1);
    mbar_init(bar(C::BAR_SF + 1), 1);
    mbar_init(bar(C::BAR_PF), 4);
    mbar_init(bar(C::BAR_PV), 1);
    mbar_init(bar(C::BAR_DRAIN), 1);
    fence_barrier_init();
    misc[1] = 0;
    misc[2] = build_schedule(p.indptr, p.indices, p.kind, p.nblocks, p.nnzb, tile * C::SUB,
                             C::SUB, sched, C::MAX_CHUNKS, p.err);
  }
  if (warp == 5) {
    tmem_alloc(sbase + C::OFF_MISC, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = misc[0];
  const int n = static_cast<int>(misc[2]);

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n > 0) {
      mbar_expect_tx(bar(C::BAR_Q), C::Q_BYTES);
#pragma unroll
      for (int pn = 0; pn < D / 64; ++pn)
        tma_load_4d(sbase + C::OFF_Q + pn * (C::BM * 128), &tm_q, bar(C::BAR_Q), pn * 64,
                    tile * C::BM, h, b);
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int s = j % C::STAGES;
        if (j >= C::STAGES &&
            !mbar_wait(bar(C::BAR_KVE + s), ((j / C::STAGES) - 1) & 1, abort_flag, p.err))
          break;
        const int kb = static_cast<int>(sched_block(sched[j]));
        mbar_expect_tx(bar(C::BAR_KVF + s), 2 * C::KV_BYTES);
#pragma unroll
        for (int pn = 0; pn < D / 64; ++pn) {
          tma_load_4d(sbase + C::OFF_K + s * C::KV_BYTES + pn * (BN * 128), &tm_k,
                      bar(C::BAR_KVF + s), pn * 64, kb * p.bs, h, b);
          tma_load_4d(sbase + C::OFF_V + s * C::KV_BYTES + pn * (BN * 128), &tm_v,
                      bar(C::BAR_KVF + s), pn * 64, kb * p.bs, h, b);
        }
        issued = j + 1;
      }
      // On abort, drain the loads still in flight before the CTA exits.
      if (*abort_flag) {
        for (int j = max(0, issued - C::STAGES); j < issued; ++j)
          mbar_wait_drain(bar(C::BAR_KVF + j % C::STAGES), (j / C::STAGES) & 1);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n > 0) {
      const uint32_t tS = tbase + C::COL_S, tO = tbase + C::COL_O;
      bool ok = mbar_wait(bar(C::BAR_Q), 0, abort_flag, p.err);
      auto issue_s = [&](int j) {
        const int s = j % C::STAGES;
        const uint32_t qa = sbase + C::OFF_Q, ka = sbase + C::OFF_K + s * C::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk & 3) * 32u;
          const uint64_t ad = sdesc_sw128(qa + (kk >> 2) * (C::BM * 128) + off, 16, 1024);
          const uint64_t bd = sdesc_sw128(ka + (kk >> 2) * (BN * 128) + off, 16, 1024);
          tc_mma(tS + (j & 1) * BN, ad, bd, C::IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(bar(C::BAR_SF + (j & 1)));
      };
      if (ok) ok = mbar_wait(bar(C::BAR_KVF + 0), 0, abort_flag, p.err);
      if (ok) {
        tc_fence_after();
        issue_s(0);
      }
      for (int j = 0; ok && j < n; ++j) {
        if (j + 1 < n) {
          const int s1 = (j + 1) % C::STAGES;
          if (!mbar_wait(bar(C::BAR_KVF + s1), ((j + 1) / C::STAGES) & 1, abort_flag, p.err)) break;
          tc_fence_after();
          issue_s(j + 1);
        }
        if (!mbar_wait(bar(C::BAR_PF), j & 1, abort_flag, p.err)) break;
        tc_fence_after();
        const int s = j % C::STAGES;
        const uint32_t pa = sbase + C::OFF_P, va = sbase + C::OFF_V + s * C::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(pa + (kk >> 2) * (C::BM * 128) + (kk & 3) * 32, 16, 1024);
          // V is MN-major: 64-column panels BN*128 bytes apart (LBO), 8-row
          // groups 1024 bytes apart (SBO); 16 rows per k-step = 2048 bytes.
          const uint64_t bd = sdesc_sw128(va + kk * 2048, BN * 128, 1024);
          tc_mma(tO, ad, bd, C::IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(bar(C::BAR_PV));
        tc_commit(bar(C::BAR_KVE + s));
      }
      if (*abort_flag) {  // let the MMAs in flight finish before TMEM is freed
        tc_commit(bar(C::BAR_DRAIN));
        mbar_wait_drain(bar(C::BAR_DRAIN), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int r = tid;                      // query row within the tile = TMEM lane
    const int q_pos = tile * C::BM + r;
    const int sub = (C::SUB == 2) ? (r >> 6) : 0;
    const uint32_t lane_base = tbase + (static_cast<uint32_t>(warp * 32) << 16);
    float m = -INFINITY, l = 0.f;
    uint8_t* pbuf = smem + C::OFF_P;
    bool alive = true;
    for (int j = 0; j < n && alive; ++j) {
      const uint32_t e = sched[j];
      const int k0 = static_cast<int>(sched_block(e)) * p.bs;
      const uint32_t st = sched_state(e, sub);
      if (!__all_sync(0xffffffffu,
                      mbar_wait(bar(C::BAR_SF + (j & 1)), (j >> 1) & 1, abort_flag, p.err))) {
        alive = false;
        break;
      }
      tc_fence_after();
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 32) tmem_ld32(lane_base + C::COL_S + (j & 1) * BN + c, s + c);
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        const bool valid = (st == ST_FULL) || (st == ST_CAUSAL && k0 + c <= q_pos);
        s[c] = valid ? s[c] * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, s[c]);
      }
      const float m_new = fmaxf(m, mx);
      const bool need = m_new > m + 8.0f;
      // the P buffer and O are free once the previous chunk's PV has completed
      if (j > 0 && !__all_sync(0xffffffffu,
                               mbar_wait(bar(C::BAR_PV), (j - 1) & 1, abort_flag, p.err))) {
        alive = false;
        break;
      }
      if (__any_sync(0xffffffffu, need)) {
        const float alpha = need ? ex2_approx(m - m_new) : 1.f;
        if (need) {
          l *= alpha;
          m = m_new;
        }
        if (j > 0) {
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D; c += 32) {
            float ov[32];
            tmem_ld32(lane_base + C::COL_O + c, ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= alpha;
            tmem_st32(lane_base + C::COL_O + c, ov);
          }
          tmem_st_wait();
        }
      }
      const float m_use = (m == -INFINITY) ? 0.f : m;
      float rs = 0.f;
#pragma unroll
      for (int c16 = 0; c16 < BN / 8; ++c16) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float a = ex2_approx(s[c16 * 8 + 2 * i] - m_use);
          const float bb = ex2_approx(s[c16 * 8 + 2 * i + 1] - m_use);
          rs += a + bb;
          w[i] = pack_bf16(a, bb);
        }
        const int pn = c16 >> 3;
        uint4* dst = reinterpret_cast<uint4*>(pbuf + pn * (C::BM * 128) + sw128_offset(r, c16 & 7));
        *dst = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l += rs;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C::BAR_PF));
    }
    // ------------------------------------------------------------ epilogue
    if (alive && n > 0 &&
        !__all_sync(0xffffffffu, mbar_wait(bar(C::BAR_PV), (n - 1) & 1, abort_flag, p.err)))
      alive = false;
    if (alive) {
      tc_fence_after();
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.o + static_cast<int64_t>(b) * p.o_sb +
                            static_cast<int64_t>(h) * p.o_sh + static_cast<int64_t>(q_pos) * p.o_st;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        float ov[32];
        if (n > 0) {
          tmem_ld32(lane_base + C::COL_O + c, ov);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = 0.f;
        }
        if (q_pos < p.T) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w = make_uint4(pack_bf16(ov[i] * inv, ov[i + 1] * inv),
                                 pack_bf16(ov[i + 2] * inv, ov[i + 3] * inv),
                                 pack_bf16(ov[i + 4] * inv, ov[i + 5] * inv),
                                 pack_bf16(ov[i + 6] * inv, ov[i + 7] * inv));
            *reinterpret_cast<uint4*>(orow + c + i) = w;
          }
        }
      }
      if (q_pos < p.T)
        p.lse[static_cast<int64_t>(bh) * p.T + q_pos] =
            (l > 0.f) ? (m + __log2f(l)) * 0.69314718055994531f : -INFINITY;
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
