// Decode: one new query per (batch, head) attending over its KV cache under a
// block layout or an M^(d) pattern layout (smat_decode in include/smat_b200.h).
//
// One query row reads every visible key and value once, so decode is
// HBM-bound (2 D bytes per key and value at bf16) and runs on CUDA cores:
//
//   partial  grid (B H, n_split), 128 threads.  The query's CSR row is a
//            sequence of steps (STEP keys of one entry each); split s walks
//            steps [s sps, (s + 1) sps), sps chosen so that the grid fills
//            whole waves of resident CTAs.  A key is owned by
//            a group of D / 8 lanes (16-byte vectors, a 256-byte row read by
//            16 lanes at D = 128), each warp handling 4 x 32 / (D / 8) keys
//            per step with all their loads issued first (values only for
//            visible keys); the dot product is reduced inside the group and each
//            group keeps an online softmax (max, sum, D / 8 x 8 outputs).
//            Groups and warps are merged at the end into one partial
//            (m, l, o[D]) per split, in base-2 exponent units.
//   combine  grid B H, D threads: rescales the partials to their common max
//            and writes o (bf16) and the natural-log LSE.
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
  float* part;               // [B H][n_split][D + 2]: m, l, o[D]
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
__global__ void __launch_bounds__(128) decode_partial_kernel(const DecodeParams p) {
  constexpr int G = D / 8;        // lanes per key
  constexpr int KPW = 32 / G;     // keys per warp and unrolled step
  constexpr int U = 4;            // unrolled steps
  __shared__ float red_m[4][KPW], red_l[4][KPW];
  __shared__ float red_o[4][D];
  const int bh = blockIdx.x, split = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slot = lane / G, part = lane % G;
  float* out = p.part + (static_cast<int64_t>(bh) * p.n_split + split) * (D + 2);

  // The row's keys as one sequence of steps: step g covers entry e0 + g / spb,
  // keys (g % spb) STEP + warp KPW U + u KPW + slot of it.  The loads of step
  // k + 1 are issued before the arithmetic of step k (two register buffers),
  // so every warp keeps loads in flight while it computes.
  constexpr int STEP = 4 * KPW * U;             // keys per CTA step
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

  float qv[8];
  {
    const V8 raw = *reinterpret_cast<const V8*>(p.q + b * p.q_sb + h * p.q_sh + part * 8);
    unpack8(raw, qv);
#pragma unroll
    for (int i = 0; i < 8; ++i) qv[i] *= p.scale_log2;
  }
  float m = -INFINITY, l = 0.f, o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.f;
  const __nv_bfloat16* kbase = p.k + b * p.k_sb + h * p.k_sh + part * 8;
  const __nv_bfloat16* vbase = p.v + b * p.v_sb + h * p.v_sh + part * 8;

  V8 kr[2][U], vr[2][U];
  bool vis[2][U];
  auto issue = [&](int k, int buf) {
    const int g = s0 + k;
    const int e = e0 + g / spb;
    const int kb = __ldg(p.indices + e);
    const uint8_t kd = __ldg(p.kind + e);
    const bool ok = kb >= 0 && kb < p.nblocks && kb * p.bs <= t;
    if (!ok && threadIdx.x == 0 && p.err) atomicOr(p.err, DEV_ERR_BAD_CSR);
    const int j0 = ok ? kb * p.bs : 0;
    const int jn = ok ? min(p.bs, p.T - j0) : 0;
    const int base = (g % spb) * STEP + warp * KPW * U;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int jj = base + u * KPW + slot;
      const bool in = jj < jn;
      const int j = j0 + (in ? jj : 0);
      bool vs = in;
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
      vis[buf][u] = vs;
      kr[buf][u] = *reinterpret_cast<const V8*>(kbase + static_cast<int64_t>(j) * p.k_st);
      if (vs) vr[buf][u] = *reinterpret_cast<const V8*>(vbase + static_cast<int64_t>(j) * p.v_st);
    }
  };
  // A step's U keys are independent until the softmax update: their dot
  // products and group reductions interleave, then one max, at most one
  // rescale, and the U accumulations.
  auto consume = [&](int buf) {
    float sc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float kv[8];
      unpack8(kr[buf][u], kv);
      float s0 = qv[0] * kv[0], s1 = qv[1] * kv[1];
#pragma unroll
      for (int i = 2; i < 8; i += 2) {
        s0 = fmaf(qv[i], kv[i], s0);
        s1 = fmaf(qv[i + 1], kv[i + 1], s1);
      }
      sc[u] = s0 + s1;
    }
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1)
#pragma unroll
      for (int u = 0; u < U; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], off);
    float mx = m;
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (vis[buf][u]) mx = fmaxf(mx, sc[u]);
    if (mx > m) {
      const float a = exp2f(m - mx);   // 0 when m is still -inf
      l *= a;
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] *= a;
      m = mx;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (!vis[buf][u]) continue;
      float vv[8];
      unpack8(vr[buf][u], vv);
      const float pr = exp2f(sc[u] - m);
      l += pr;
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = fmaf(pr, vv[i], o[i]);
    }
  };
  // buffers are named by constants (a runtime index would move them to the stack)
  if (nsteps > 0) issue(0, 0);
  for (int k = 0; k < nsteps; k += 2) {
    if (k + 1 < nsteps) issue(k + 1, 1);
    consume(0);
    if (k + 1 < nsteps) {
      if (k + 2 < nsteps) issue(k + 2, 0);
      consume(1);
    }
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
  // merge the four warps
  if (slot == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) red_o[warp][part * 8 + i] = o[i];
    if (part == 0) {
      red_m[warp][0] = m;
      red_l[warp][0] = l;
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float M = red_m[0][0], L = red_l[0][0], O = red_o[0][d];
#pragma unroll
    for (int w = 1; w < 4; ++w) merge_state<1>(M, L, &O, red_m[w][0], red_l[w][0], &red_o[w][d]);
    out[2 + d] = O;
    if (d == 0) {
      out[0] = M;
      out[1] = L;
    }
  }
}

template <int D>
__global__ void __launch_bounds__(D) decode_combine_kernel(const DecodeParams p) {
  const int bh = blockIdx.x, d = threadIdx.x;
  const int b = bh / p.H, h = bh % p.H;
  const float* in = p.part + static_cast<int64_t>(bh) * p.n_split * (D + 2);
  // two passes with independent loads (the maxima, then the rescaled sums), so
  // the loads of all splits are in flight together
  float M = -INFINITY;
#pragma unroll 8
  for (int s = 0; s < p.n_split; ++s) M = fmaxf(M, in[s * (D + 2)]);
  float L = 0.f, O = 0.f;
  if (M != -INFINITY) {
#pragma unroll 8
    for (int s = 0; s < p.n_split; ++s) {
      const float* ps = in + s * (D + 2);
      const float w = exp2f(ps[0] - M);   // 0 for an empty split (m = -inf)
      L = fmaf(ps[1], w, L);
      O = fmaf(ps[2 + d], w, O);
    }
  }
  const float r = L > 0.f ? O / L : 0.f;
  p.o[b * p.o_sb + h * p.o_sh + d] = __float2bfloat16_rn(r);
  if (d == 0 && p.lse)
    p.lse[bh] = L > 0.f ? (M + log2f(L)) * 0.69314718055994531f : -INFINITY;
}

int status() { return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH; }

// CTAs resident at once: four per SM (128 threads at 128 registers)
int64_t resident_ctas() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    sms = 148;
  return 4LL * sms;
}
// Steps per split (a step is 32 keys at D = 128, 64 at D = 64): the grid is
// sized to the most whole waves of resident CTAs (up to four) whose splits
// keep at least 8 steps, so a split's set-up is amortised and the last wave
// is not left mostly empty; then the split count is trimmed so that no split
// is empty.
int steps_per_split(int B, int H, int D, int bs, int max_row) {
  const int64_t bh = static_cast<int64_t>(B) * H, slots = resident_ctas();
  const int step = D == 64 ? 64 : 32;
  const int64_t row_steps = std::max<int64_t>(1, static_cast<int64_t>(max_row) * ((bs + step - 1) / step));
  int64_t best = row_steps;
  for (int w = 1; w <= 4; ++w) {
    const int64_t ns = std::max<int64_t>(1, w * slots / bh);
    const int64_t sps = (row_steps + ns - 1) / ns;
    if (w == 1 || sps >= 8) best = sps;
  }
  return static_cast<int>(best);
}
int n_splits(int B, int H, int D, int bs, int max_row) {
  const int64_t step = D == 64 ? 64 : 32;
  const int64_t row_steps = std::max<int64_t>(1, static_cast<int64_t>(max_row) * ((bs + step - 1) / step));
  const int sps = steps_per_split(B, H, D, bs, max_row);
  return static_cast<int>((row_steps + sps - 1) / sps);
}
// an upper bound of n_splits over block sizes (the workspace query has none):
// the grid never exceeds four waves, and a row has at least one split
int max_splits(int B, int H) {
  const int64_t bh = static_cast<int64_t>(B) * H;
  return static_cast<int>(std::max<int64_t>(1, 4 * resident_ctas() / bh));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int smat_decode_workspace(int B, int H, int D, int max_row, int64_t* floats_out) {
  if (B < 1 || H < 1 || max_row < 0 || (D != 64 && D != 128)) return SMAT_ERR_BAD_SHAPE;
  if (!floats_out) return SMAT_ERR_NULL_POINTER;
  *floats_out = static_cast<int64_t>(B) * H * max_splits(B, H) * (D + 2);
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
  if (!q || !k_cache || !v_cache || !o || !pos || !indptr || !kind || !workspace ||
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
  const int ns = n_splits(B, H, D, block, max_row);
  if (workspace_floats < static_cast<int64_t>(B) * H * ns * (D + 2)) return SMAT_ERR_CAPACITY;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k_cache);
  p.v = static_cast<const __nv_bfloat16*>(v_cache);
  p.o = static_cast<__nv_bfloat16*>(o);
  p.lse = lse;
  p.pos = pos;
  p.indptr = indptr;
  p.indices = indices;
  p.kind = kind;
  p.part = workspace;
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
  p.sps = steps_per_split(B, H, D, block, max_row);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = err_word;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(B * H), static_cast<unsigned>(ns));
  if (D == 64) {
    decode_partial_kernel<64><<<grid, 128, 0, s>>>(p);
    decode_combine_kernel<64><<<B * H, 64, 0, s>>>(p);
  } else {
    decode_partial_kernel<128><<<grid, 128, 0, s>>>(p);
    decode_combine_kernel<128><<<B * H, 128, 0, s>>>(p);
  }
  return status();
}

}  // extern "C"
