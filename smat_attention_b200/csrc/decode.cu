// Decode: one new query per (batch, head) attending over its KV cache under a
// block layout or an M^(d) pattern layout (smat_decode in include/smat_b200.h).
//
// One query row reads every visible key and value once, so decode is
// HBM-bound (2 D bytes per key and value at bf16) and runs on CUDA cores:
//
//   grid (B H, n_split), 288 threads, two CTAs per SM.  The query's CSR row
//   is a sequence of steps (64 keys of one entry each); split s walks steps
//   [s sps, (s + 1) sps), the split count chosen for the most even work per
//   SM.  A producer warp copies each step's K and V rows into a shared-memory
//   ring with bulk copies; eight compute warps score them: a key is owned by
//   a group of D / 8 lanes (16-byte vectors), the dot product is reduced
//   inside the group and each group keeps an online softmax (max, sum,
//   8 outputs per lane).  Groups and warps are merged into one partial
//   (m, l, o[D]) per split, in base-2 exponent units.  The splits of a row
//   form one thread-block cluster: CTA rank 0 reads the others' partials from
//   their shared memory, rescales them to the common max and writes o (bf16)
//   and the natural-log LSE.
//
// Visibility of key j for query position t: FULL entries all keys, CAUSAL
// entries j <= t, PATTERN entries the row word of pattern.cuh.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "../../include/smat_b200.h"
#include "common.cuh"
#include "pattern.cuh"

namespace {

using namespace smat;

struct DecodeParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* o;
  float* lse;
  const int32_t* pos;
  const int32_t* indptr;
  const int32_t* indices;
  const uint8_t* kind;
  int64_t q_sb, q_sh, k_sb, k_sh, k_st, v_sb, v_sh, v_st, o_sb, o_sh;
  int B, H, T, nblocks, nnzb, bs, n_split, sps;
  float scale_log2;
  int32_t* err;
  MdPattern md;
};

struct alignas(16) V8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void unpack8(const V8& v, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// merge (m2, l2, o2) into (m, l, o): all in base-2 exponent units
template <int N>
__device__ __forceinline__ void merge_state(float& m, float& l, float* o, float m2, float l2,
                                            const float* o2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;
  const float a = exp2f(m - mm), b = exp2f(m2 - mm);
  l = l * a + l2 * b;
#pragma unroll
  for (int i = 0; i < N; ++i) o[i] = o[i] * a + o2[i] * b;
  m = mm;
}

template <int D>
struct DecCfg {
  static constexpr int G = D / 8;                // lanes per key
  static constexpr int KPW = 32 / G;             // keys per warp and unrolled step
  static constexpr int NW = 8;                   // compute warps
  static constexpr int U = D == 64 ? 2 : 4;      // unrolled keys per lane group
  static constexpr int STEP = NW * KPW * U;      // keys per step: 64
  static constexpr int ROW = D * 2;              // bytes of one key row
  static constexpr int STAGE = 2 * STEP * ROW;   // K rows, then V rows
  static constexpr int NS = (96 * 1024) / STAGE; // ring stages (96 KB)
  static constexpr int OFF_BAR = NS * STAGE;     // full[NS], empty[NS]
  static constexpr int OFF_MISC = OFF_BAR + 2 * NS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16;
  static constexpr int THREADS = 32 * (NW + 1);  // compute warps + the producer warp
  static constexpr int KPL = STEP / 32;          // keys per producer lane
  static_assert(STEP == 64 && NS >= 2, "ring layout");
  static_assert(SMEM_BYTES + 1024 + NW * (D + 2) * 4 <= 113 * 1024, "two CTAs per SM");
};

template <int D>
__global__ void __launch_bounds__(DecCfg<D>::THREADS, 2)
    decode_partial_kernel(const DecodeParams p) {
  using C = DecCfg<D>;
  constexpr int G = C::G, KPW = C::KPW, U = C::U, STEP = C::STEP, NW = C::NW;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red_m[NW], red_l[NW];
  __shared__ float red_o[NW][D];
  __shared__ float fin[D + 2];   // this split's partial: m, l, o[D] (base-2 units)
  const uint32_t sbase = smem_u32(smem);
  auto full = [&](int i) { return sbase + C::OFF_BAR + 8u * i; };
  auto empty = [&](int i) { return sbase + C::OFF_BAR + 8u * (C::NS + i); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC);
  const int bh = blockIdx.x, split = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slot = lane / G, part = lane % G;

  // The row's keys as one sequence of steps: step g covers entry e0 + g / spb,
  // keys (g % spb) STEP .. + STEP - 1 of it.  The producer warp copies each
  // step's K and V rows into a ring stage with bulk copies up to NS - 1
  // steps ahead; compute warp w scores keys w KPW U + u KPW + slot of it.
  const int spb = (p.bs + STEP - 1) / STEP;     // steps per block
  const int t = __ldg(p.pos + b);
  int e0 = 0, s0 = 0, nsteps = 0;
  if (t < 0 || t >= p.T) {
    if (threadIdx.x == 0 && p.err) atomicOr(p.err, DEV_ERR_BAD_WORK);
  } else {
    const int qb = t / p.bs;
    const int a = __ldg(p.indptr + qb), z = __ldg(p.indptr + qb + 1);
    if (a < 0 || z < a || z > p.nnzb) {
      if (threadIdx.x == 0 && p.err) atomicOr(p.err, DEV_ERR_BAD_CSR);
    } else {
      e0 = a;
      s0 = split * p.sps;
      nsteps = max(0, min((z - a) * spb - s0, p.sps));
    }
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(full(i), 1);
      mbar_init(empty(i), NW);
    }
    fence_barrier_init();
    *abort_flag = 0;
  }
  __syncthreads();

  // entry of step g: its first key, the keys in range, its kind (a bad entry
  // is reported and read as empty)
  auto entry = [&](int g, int& j0, int& jn, uint8_t& kd) {
    const int e = e0 + g / spb;
    const int kb = __ldg(p.indices + e);
    kd = __ldg(p.kind + e);
    const bool ok = kb >= 0 && kb < p.nblocks && kb * p.bs <= t;
    if (!ok && lane == 0 && p.err) atomicOr(p.err, DEV_ERR_BAD_CSR);
    j0 = ok ? kb * p.bs : 0;
    jn = ok ? min(p.bs, p.T - j0) : 0;
  };
  float m = -INFINITY, l = 0.f, o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.f;

  if (warp == NW) {
    // ------------------------------------------------------------ producer
    const __nv_bfloat16* kb0 = p.k + b * p.k_sb + h * p.k_sh;
    const __nv_bfloat16* vb0 = p.v + b * p.v_sb + h * p.v_sh;
    const bool dense = p.k_st == D && p.v_st == D;   // a step's rows are one run
    int issued = 0;
    for (int k = 0; k < nsteps; ++k) {
      const int st = k % C::NS;
      bool ok = true;
      if (lane == 0 && k >= C::NS)
        ok = mbar_wait(empty(st), ((k / C::NS) - 1) & 1, abort_flag, p.err);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      const int g = s0 + k;
      int j0, jn;
      uint8_t kd;
      entry(g, j0, jn, kd);
      const int base = (g % spb) * STEP;
      const int nv = max(0, min(jn - base, STEP));   // keys of the step in range
      const uint32_t sk = sbase + st * C::STAGE, sv = sk + STEP * C::ROW;
      if (lane == 0) mbar_expect_tx(full(st), 2u * nv * C::ROW);
      __syncwarp();
      if (nv > 0) {
        const int64_t j = j0 + base;
        if (dense) {
          if (lane == 0) {
            bulk_load(sk, kb0 + j * D, nv * C::ROW, full(st));
            bulk_load(sv, vb0 + j * D, nv * C::ROW, full(st));
          }
        } else {
#pragma unroll
          for (int q = 0; q < C::KPL; ++q) {
            const int kk = lane * C::KPL + q;
            if (kk < nv) {
              bulk_load(sk + kk * C::ROW, kb0 + (j + kk) * p.k_st, C::ROW, full(st));
              bulk_load(sv + kk * C::ROW, vb0 + (j + kk) * p.v_st, C::ROW, full(st));
            }
          }
        }
      }
      issued = k + 1;
    }
    // never exit with copies in flight
    if (lane == 0 && *abort_flag)
      for (int k = max(0, issued - C::NS); k < issued; ++k)
        mbar_wait_drain(full(k % C::NS), (k / C::NS) & 1);
  } else {
    // ------------------------------------------------------------ compute
    float qv[8];
    {
      const V8 raw = *reinterpret_cast<const V8*>(p.q + b * p.q_sb + h * p.q_sh + part * 8);
      unpack8(raw, qv);
#pragma unroll
      for (int i = 0; i < 8; ++i) qv[i] *= p.scale_log2;
    }
    for (int k = 0; k < nsteps; ++k) {
      const int st = k % C::NS;
      const int g = s0 + k;
      int j0, jn;
      uint8_t kd;
      entry(g, j0, jn, kd);
      // visibility of this lane group's keys, before the wait
      bool vis[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int jj = (g % spb) * STEP + warp * KPW * U + u * KPW + slot;
        const int j = j0 + jj;
        bool vs = jj < jn;
        if (kd == 1) {
          vs = vs && j <= t;
        } else if (kd == 2) {
          if (p.md.row_bits) {
            vs = vs && ((md_row_word(p.md, p.T, t, j & ~31) >> (j & 31)) & 1u);
          } else {
            vs = false;
            if (part == 0 && p.err) atomicOr(p.err, DEV_ERR_BAD_CSR);
          }
        }
        vis[u] = vs;
      }
      if (!__all_sync(0xffffffffu, mbar_wait(full(st), (k / C::NS) & 1, abort_flag, p.err)))
        break;
      const uint8_t* sk = smem + st * C::STAGE;
      const uint8_t* sv = sk + STEP * C::ROW;
      // the U keys are independent until the softmax update: dot products
      // and group reductions interleave, then one max, at most one rescale,
      // and the U accumulations (rows out of range were not copied: their
      // scores are never used)
      float sc[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int kk = warp * KPW * U + u * KPW + slot;
        const V8 raw = *reinterpret_cast<const V8*>(sk + kk * C::ROW + part * 16);
        float kv[8];
        unpack8(raw, kv);
        float a0 = qv[0] * kv[0], a1 = qv[1] * kv[1];
#pragma unroll
        for (int i = 2; i < 8; i += 2) {
          a0 = fmaf(qv[i], kv[i], a0);
          a1 = fmaf(qv[i + 1], kv[i + 1], a1);
        }
        sc[u] = a0 + a1;
      }
#pragma unroll
      for (int off = G / 2; off > 0; off >>= 1)
#pragma unroll
        for (int u = 0; u < U; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], off);
      float mx = m;
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (vis[u]) mx = fmaxf(mx, sc[u]);
      if (mx > m) {
        const float a = exp2f(m - mx);   // 0 when m is still -inf
        l *= a;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] *= a;
        m = mx;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (!vis[u]) continue;
        const int kk = warp * KPW * U + u * KPW + slot;
        const V8 raw = *reinterpret_cast<const V8*>(sv + kk * C::ROW + part * 16);
        float vv[8];
        unpack8(raw, vv);
        const float pr = exp2f(sc[u] - m);
        l += pr;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = fmaf(pr, vv[i], o[i]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty(st));
    }
    // merge the KPW groups of the warp: lanes with the same part, xor over slot bits
#pragma unroll
    for (int off = G; off < 32; off <<= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
      const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
      float o2[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o2[i] = __shfl_xor_sync(0xffffffffu, o[i], off);
      merge_state<8>(m, l, o, m2, l2, o2);
    }
    if (slot == 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) red_o[warp][part * 8 + i] = o[i];
      if (part == 0) {
        red_m[warp] = m;
        red_l[warp] = l;
      }
    }
  }
  __syncthreads();
  // merge the compute warps
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float M = red_m[0], L = red_l[0], O = red_o[0][d];
#pragma unroll
    for (int w = 1; w < NW; ++w) merge_state<1>(M, L, &O, red_m[w], red_l[w], &red_o[w][d]);
    fin[2 + d] = O;
    if (d == 0) {
      fin[0] = M;
      fin[1] = L;
    }
  }
  // combine the row's splits: rank 0 reads every CTA's partial in place
  cluster_sync();
  if (cluster_ctarank() == 0) {
    const uint32_t nr = gridDim.y;   // the cluster is the row's splits
    const uint32_t fa = smem_u32(fin);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float M = -INFINITY;
      for (uint32_t r = 0; r < nr; ++r) M = fmaxf(M, ld_cluster_f32(fa, r));
      float L = 0.f, O = 0.f;
      if (M != -INFINITY) {
        for (uint32_t r = 0; r < nr; ++r) {
          const float w = exp2f(ld_cluster_f32(fa, r) - M);   // 0 for an empty split
          L = fmaf(ld_cluster_f32(fa + 4, r), w, L);
          O = fmaf(ld_cluster_f32(fa + 4 * (2 + d), r), w, O);
        }
      }
      const float res = L > 0.f ? O / L : 0.f;
      p.o[b * p.o_sb + h * p.o_sh + d] = __float2bfloat16_rn(res);
      if (d == 0 && p.lse)
        p.lse[bh] = L > 0.f ? (M + log2f(L)) * 0.69314718055994531f : -INFINITY;
    }
  }
  cluster_sync();   // the partials stay in place until rank 0 has read them
}

int status() { return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH; }

int sm_count() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    sms = 148;
  return sms;
}
constexpr int DEC_STEP = 64;       // keys per step (DecCfg<D>::STEP)
constexpr int DEC_RESIDENT = 2;    // CTAs per SM (a 96 KB ring each)
constexpr int DEC_MAX_SPLITS = 8;   // a row's splits are one (portable-size) cluster
// Splits per row: the count whose busiest SM finishes first, with an SM's
// time taken as the steps of the CTAs it runs plus a set-up of two steps per
// round of resident CTAs.  (B H rows rarely divide evenly over the SMs.)
int n_splits(int B, int H, int bs, int max_row) {
  const int64_t bh = static_cast<int64_t>(B) * H, sms = sm_count();
  const int64_t row_steps =
      std::max<int64_t>(1, static_cast<int64_t>(max_row) * ((bs + DEC_STEP - 1) / DEC_STEP));
  int best = 1;
  int64_t best_cost = -1;
  for (int64_t ns = 1; ns <= std::min<int64_t>(row_steps, DEC_MAX_SPLITS); ++ns) {
    const int64_t sps = (row_steps + ns - 1) / ns;
    const int64_t per_sm = (bh * ns + sms - 1) / sms;
    const int64_t cost = per_sm * sps + 2 * ((per_sm + DEC_RESIDENT - 1) / DEC_RESIDENT);
    if (best_cost < 0 || cost <= best_cost) {   // ties: more splits, more copies in flight
      best_cost = cost;
      best = static_cast<int>(ns);
    }
  }
  return best;
}
int steps_per_split(int B, int H, int bs, int max_row) {
  const int64_t row_steps =
      std::max<int64_t>(1, static_cast<int64_t>(max_row) * ((bs + DEC_STEP - 1) / DEC_STEP));
  const int ns = n_splits(B, H, bs, max_row);
  return static_cast<int>((row_steps + ns - 1) / ns);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int smat_decode_workspace(int B, int H, int D, int max_row, int64_t* floats_out) {
  if (B < 1 || H < 1 || max_row < 0 || (D != 64 && D != 128)) return SMAT_ERR_BAD_SHAPE;
  if (!floats_out) return SMAT_ERR_NULL_POINTER;
  *floats_out = 0;   // the splits are combined in the kernel (kept for the ABI)
  return SMAT_OK;
}

int smat_decode(int dtype, const void* q, const int64_t* q_stride, const void* k_cache,
                const int64_t* k_stride, const void* v_cache, const int64_t* v_stride, void* o,
                const int64_t* o_stride, float* lse, const int32_t* pos, int B, int H, int T,
                int D, const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                int nblocks, int64_t nnzb, int block, int max_row, const smat_pattern_t* pattern,
                float scale, float* workspace, int64_t workspace_floats, int32_t* err_word,
                void* stream) {
  if (dtype != SMAT_DTYPE_BF16) return SMAT_ERR_UNSUPPORTED_DTYPE;
  if (D != 64 && D != 128) return SMAT_ERR_UNSUPPORTED_D;
  if (B < 1 || H < 1 || T < 1 || block < 1 || nblocks != (T + block - 1) / block)
    return SMAT_ERR_BAD_SHAPE;
  (void)workspace;   // unused: the splits are combined in the kernel
  (void)workspace_floats;
  if (!q || !k_cache || !v_cache || !o || !pos || !indptr || !kind ||
      !q_stride || !k_stride || !v_stride || !o_stride || (!indices && nnzb > 0))
    return SMAT_ERR_NULL_POINTER;
  if (nnzb < 0 || nnzb > 0x7FFFFFFF || max_row < 1) return SMAT_ERR_CSR_INVALID;
  if (!std::isfinite(scale) || scale <= 0.f) return SMAT_ERR_BAD_SHAPE;
  const int64_t* strides[4] = {q_stride, k_stride, v_stride, o_stride};
  const void* ptrs[4] = {q, k_cache, v_cache, o};
  for (int i = 0; i < 4; ++i) {
    const int ns = (i == 0 || i == 3) ? 2 : 3;
    for (int j = 0; j < ns; ++j)
      if (strides[i][j] < 0) return SMAT_ERR_BAD_STRIDE;
    if (i != 3) {
      for (int j = 0; j < ns; ++j)
        if (strides[i][j] % 8) return SMAT_ERR_BAD_ALIGNMENT;
      if (!aligned16(ptrs[i])) return SMAT_ERR_BAD_ALIGNMENT;
    }
  }
  DecodeParams p{};
  if (pattern) {
    const smat_pattern_t* pt = pattern;
    if (pt->family != SMAT_FAMILY_GEOMETRIC && pt->family != SMAT_FAMILY_ENDPOINT)
      return SMAT_ERR_BAD_PATTERN;
    if (pt->n_P < 0 || pt->n < pt->n_P || pt->n > T || pt->B < 1 || pt->N0 < 1 ||
        static_cast<int64_t>(pt->row_words) < (static_cast<int64_t>(pt->N0) + 63) / 32 ||
        static_cast<int64_t>(pt->col_words) < (static_cast<int64_t>(pt->B) + 63) / 32 ||
        (pt->family == SMAT_FAMILY_ENDPOINT && pt->N0 < pt->n - pt->n_P))
      return SMAT_ERR_BAD_PATTERN;
    if (!pt->row_bits || !pt->col_bits) return SMAT_ERR_NULL_POINTER;
    p.md = MdPattern{pt->row_bits, pt->col_bits, pt->family, pt->n,        pt->n_P,
                     pt->B,        pt->N0,       pt->row_words, pt->col_words};
  }
  const int ns = n_splits(B, H, block, max_row);
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k_cache);
  p.v = static_cast<const __nv_bfloat16*>(v_cache);
  p.o = static_cast<__nv_bfloat16*>(o);
  p.lse = lse;
  p.pos = pos;
  p.indptr = indptr;
  p.indices = indices;
  p.kind = kind;
  p.q_sb = q_stride[0];
  p.q_sh = q_stride[1];
  p.k_sb = k_stride[0];
  p.k_sh = k_stride[1];
  p.k_st = k_stride[2];
  p.v_sb = v_stride[0];
  p.v_sh = v_stride[1];
  p.v_st = v_stride[2];
  p.o_sb = o_stride[0];
  p.o_sh = o_stride[1];
  p.B = B;
  p.H = H;
  p.T = T;
  p.nblocks = nblocks;
  p.nnzb = static_cast<int>(nnzb);
  p.bs = block;
  p.n_split = ns;
  p.sps = steps_per_split(B, H, block, max_row);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = err_word;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // one cluster per row: its ns splits (ns <= 8, the portable cluster size)
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(B * H), static_cast<unsigned>(ns));
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(ns);
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (D == 64) {
    if (cudaFuncSetAttribute(decode_partial_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DecCfg<64>::SMEM_BYTES) != cudaSuccess)
      return SMAT_ERR_LAUNCH;
    cfg.blockDim = dim3(DecCfg<64>::THREADS);
    cfg.dynamicSmemBytes = DecCfg<64>::SMEM_BYTES;
    if (cudaLaunchKernelEx(&cfg, decode_partial_kernel<64>, p) != cudaSuccess)
      return SMAT_ERR_LAUNCH;
  } else {
    if (cudaFuncSetAttribute(decode_partial_kernel<128>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DecCfg<128>::SMEM_BYTES) != cudaSuccess)
      return SMAT_ERR_LAUNCH;
    cfg.blockDim = dim3(DecCfg<128>::THREADS);
    cfg.dynamicSmemBytes = DecCfg<128>::SMEM_BYTES;
    if (cudaLaunchKernelEx(&cfg, decode_partial_kernel<128>, p) != cudaSuccess)
      return SMAT_ERR_LAUNCH;
  }
  return status();
}

}  // extern "C"
