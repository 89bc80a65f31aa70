// Fused elementwise kernels of the language-model training step
// (include/smat_lm.h): RMSNorm, RoPE with the head relayout, SwiGLU and the
// softmax cross-entropy over the tied head's logits.  All are HBM-bound: each
// reads its inputs once and writes its outputs once with 16-byte vectors,
// computes in fp32 and rounds to bf16 once.  The formulas are the reference
// LM template's (tasks/lm.py:45-60: RMSNorm, interleaved RoPE) plus SwiGLU
// and cross-entropy.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/smat_b200.h"
#include "../../include/smat_lm.h"

namespace {

using bf16 = __nv_bfloat16;

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

__device__ __forceinline__ V8 pack8(const float* f) {
  V8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

int status() { return cudaGetLastError() == cudaSuccess ? SMAT_OK : SMAT_ERR_LAUNCH; }

unsigned blocks_for(int64_t threads, int per) {
  return static_cast<unsigned>((threads + per - 1) / per);
}

// ------------------------------------------------------------------ RMSNorm
// One warp per row; lane l holds the 16-byte vectors l, l + 32, ... (VPL of
// them, d = 256 VPL).  With a residual r: h = bf16(x + r) is written and
// normalised (the pre-norm block's residual add fused into its norm).
template <int VPL>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const bf16* __restrict__ x,
                                                          const bf16* __restrict__ res,
                                                          const bf16* __restrict__ w,
                                                          bf16* __restrict__ h,
                                                          bf16* __restrict__ y,
                                                          float* __restrict__ rstd,
                                                          int64_t rows, float eps) {
  constexpr int D = 256 * VPL;
  const int lane = threadIdx.x & 31;
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  const V8* xr = reinterpret_cast<const V8*>(x + row * D);
  float v[VPL][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < VPL; ++c) {
    unpack8(xr[lane + 32 * c], v[c]);
    if (res) {
      float rv[8];
      unpack8(reinterpret_cast<const V8*>(res + row * D)[lane + 32 * c], rv);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] += rv[i];
      const V8 hv = pack8(v[c]);
      reinterpret_cast<V8*>(h + row * D)[lane + 32 * c] = hv;
      unpack8(hv, v[c]);   // normalise the stored (rounded) sum
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[c][i], v[c][i], ss);
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / D + eps);
  if (lane == 0) rstd[row] = r;
  const V8* wr = reinterpret_cast<const V8*>(w);
  V8* yr = reinterpret_cast<V8*>(y + row * D);
#pragma unroll
  for (int c = 0; c < VPL; ++c) {
    float wf[8], o[8];
    unpack8(wr[lane + 32 * c], wf);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = v[c][i] * r * wf[i];
    yr[lane + 32 * c] = pack8(o);
  }
}

// dx = dh + r (g - xh mean(xh g)), g = dy w, xh = x r (dh: the gradient that
// reaches the normalised input through the residual stream, may be null);
// dw partial per CTA over the rows its warps visit (grid-stride), reduced
// through shared memory into dw_part[blockIdx.x][:] (the caller sums them).
template <int VPL>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(
    const bf16* __restrict__ x, const bf16* __restrict__ w, const float* __restrict__ rstd,
    const bf16* __restrict__ dy, const bf16* __restrict__ dh, bf16* __restrict__ dx,
    float* __restrict__ dw_part, int64_t rows) {
  constexpr int D = 256 * VPL;
  __shared__ float red[8][D];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const V8* wr = reinterpret_cast<const V8*>(w);
  float wf[VPL][8], acc[VPL][8];
#pragma unroll
  for (int c = 0; c < VPL; ++c) {
    unpack8(wr[lane + 32 * c], wf[c]);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[c][i] = 0.f;
  }
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * 8;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp; row < rows; row += nwarps) {
    const V8* xr = reinterpret_cast<const V8*>(x + row * D);
    const V8* gr = reinterpret_cast<const V8*>(dy + row * D);
    const float r = rstd[row];
    float xh[VPL][8], g[VPL][8];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < VPL; ++c) {
      float dyv[8];
      unpack8(xr[lane + 32 * c], xh[c]);
      unpack8(gr[lane + 32 * c], dyv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        xh[c][i] *= r;
        g[c][i] = dyv[i] * wf[c][i];
        acc[c][i] = fmaf(dyv[i], xh[c][i], acc[c][i]);
        dot = fmaf(xh[c][i], g[c][i], dot);
      }
    }
    const float m = warp_sum(dot) / D;
    V8* dr = reinterpret_cast<V8*>(dx + row * D);
#pragma unroll
    for (int c = 0; c < VPL; ++c) {
      float o[8], hv[8];
      if (dh) {
        unpack8(reinterpret_cast<const V8*>(dh + row * D)[lane + 32 * c], hv);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) hv[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = hv[i] + r * (g[c][i] - xh[c][i] * m);
      dr[lane + 32 * c] = pack8(o);
    }
  }
#pragma unroll
  for (int c = 0; c < VPL; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) red[warp][(lane + 32 * c) * 8 + i] = acc[c][i];
  __syncthreads();
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) sum += red[k][j];
    dw_part[static_cast<int64_t>(blockIdx.x) * D + j] = sum;
  }
}

// ------------------------------------------------------------------ RoPE
// qkv [B, T, 3, H, D] -> q, k, v [B, H, T, D]; q and k rotated pairwise:
// (x1, x2) -> (x1 c - x2 s, x1 s + x2 c) with c, s = cos, sin of t inv[i]
// (tables [T, D/2]).  One thread per 8 elements.  The backward applies the
// transposed rotation and writes dqkv in the [B, T, 3, H, D] layout.
template <bool BWD>
__global__ void __launch_bounds__(256) rope_kernel(bf16* __restrict__ packed,
                                                   bf16* __restrict__ q, bf16* __restrict__ k,
                                                   bf16* __restrict__ v,
                                                   const float* __restrict__ cosv,
                                                   const float* __restrict__ sinv, int B, int T,
                                                   int H, int D) {
  // 32-bit index arithmetic (the host keeps B T 3 H D / 8 below 2^31)
  const unsigned vd = D / 8;
  const unsigned total = static_cast<unsigned>(B) * T * 3 * H * vd;
  const unsigned id = blockIdx.x * blockDim.x + threadIdx.x;
  if (id >= total) return;
  const int c8 = static_cast<int>(id % vd);
  unsigned r = id / vd;
  const int h = static_cast<int>(r % H);
  r /= H;
  const int s = static_cast<int>(r % 3);
  r /= 3;
  const int t = static_cast<int>(r % T);
  const int b = static_cast<int>(r / T);
  V8* pk = reinterpret_cast<V8*>(packed) + id;   // [b][t][s][h][c8] in vectors
  bf16* dst = s == 0 ? q : (s == 1 ? k : v);
  V8* hv = reinterpret_cast<V8*>(dst + ((static_cast<int64_t>(b) * H + h) * T + t) * D) + c8;
  float in[8], out[8];
  unpack8(BWD ? *hv : *pk, in);
  if (s < 2) {
    const float* cr = cosv + static_cast<int64_t>(t) * (D / 2) + c8 * 4;
    const float* sr = sinv + static_cast<int64_t>(t) * (D / 2) + c8 * 4;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float c = cr[p], sn = BWD ? -sr[p] : sr[p];
      const float x1 = in[2 * p], x2 = in[2 * p + 1];
      out[2 * p] = x1 * c - x2 * sn;
      out[2 * p + 1] = x1 * sn + x2 * c;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = in[i];
  }
  if (BWD)
    *pk = pack8(out);
  else
    *hv = pack8(out);
}

// ------------------------------------------------------------------ SwiGLU
// a [rows, 2 h] = (a1 | a3); g = silu(a1) a3.  Backward:
// da1 = dg a3 s (1 + a1 (1 - s)), da3 = dg a1 s, s = sigmoid(a1).
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

template <bool BWD>
__global__ void __launch_bounds__(256) swiglu_kernel(const bf16* __restrict__ a,
                                                     const bf16* __restrict__ dg,
                                                     bf16* __restrict__ out, int64_t rows,
                                                     int hidden) {
  const int vh = hidden / 8;
  const int64_t id = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (id >= rows * vh) return;
  const int64_t row = id / vh;
  const int c8 = static_cast<int>(id % vh);
  const V8* ar = reinterpret_cast<const V8*>(a + row * 2 * hidden);
  float a1[8], a3[8];
  unpack8(ar[c8], a1);
  unpack8(ar[vh + c8], a3);
  if (!BWD) {
    float g[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) g[i] = a1[i] * sigmoid_f(a1[i]) * a3[i];
    reinterpret_cast<V8*>(out + row * hidden)[c8] = pack8(g);
  } else {
    float d[8], d1[8], d3[8];
    unpack8(reinterpret_cast<const V8*>(dg + row * hidden)[c8], d);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float sg = sigmoid_f(a1[i]);
      d1[i] = d[i] * a3[i] * sg * (1.f + a1[i] * (1.f - sg));
      d3[i] = d[i] * a1[i] * sg;
    }
    V8* o = reinterpret_cast<V8*>(out + row * 2 * hidden);
    o[c8] = pack8(d1);
    o[vh + c8] = pack8(d3);
  }
}

// ------------------------------------------------------------------ cross-entropy
// One CTA per row of logits z [rows, V] (bf16): lse = log sum exp z,
// loss[row] = lse - z[tgt]; then z is overwritten by the gradient of
// scale * loss[row]: scale (exp(z - lse) - 1{j = tgt}).  With STAGE the row
// is read from HBM once into shared memory (V * 2 bytes) and both passes run
// from there; otherwise the second pass re-reads it (from L2, mostly).
template <bool STAGE>
__global__ void __launch_bounds__(256) xent_kernel(bf16* __restrict__ z,
                                                   const int64_t* __restrict__ tgt,
                                                   float* __restrict__ loss, int V, float scale,
                                                   int32_t* __restrict__ err) {
  extern __shared__ uint4 xent_smem[];
  __shared__ float sm[8], ss[8];
  const int64_t row = blockIdx.x;
  bf16* zr = z + row * V;
  const int vv = V / 8;
  V8* zv = reinterpret_cast<V8*>(zr);
  V8* src = STAGE ? reinterpret_cast<V8*>(xent_smem) : zv;
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x; c < vv; c += blockDim.x) {
    const V8 raw = zv[c];
    if (STAGE) src[c] = raw;
    float f[8];
    unpack8(raw, f);
    float mx = f[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, f[i]);
    if (mx > m) {
      s *= expf(m - mx);
      m = mx;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) s += expf(f[i] - m);
  }
  // combine (m, s) pairs: warp, then block
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * expf(m2 - mm));
    m = mm;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  float M = sm[0];
  for (int w = 1; w < 8; ++w) M = fmaxf(M, sm[w]);
  float S = 0.f;
  for (int w = 0; w < 8; ++w) S += ss[w] * expf(sm[w] - M);
  const float lse = M + logf(S);
  const int64_t t = tgt[row];
  const bool ok = t >= 0 && t < V;
  if (threadIdx.x == 0) {
    loss[row] = ok ? lse - __bfloat162float(zr[t]) : 0.f;
    if (!ok && err) atomicOr(err, SMAT_DEVERR_BAD_WORK);
  }
  __syncthreads();   // the target logit is read before any thread overwrites it
  for (int c = threadIdx.x; c < vv; c += blockDim.x) {
    float f[8];
    unpack8(src[c], f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int j = c * 8 + i;
      f[i] = scale * (expf(f[i] - lse) - (j == t ? 1.f : 0.f));
    }
    zv[c] = pack8(f);
  }
}

// 16-byte aligned (or null: optional arguments are checked for presence separately)
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// row widths of the RMSNorm kernels: d = 256 VPL with VPL in {1, 2, 3, 4, 6}
// (the backward's shared-memory reduction holds 8 warps x d floats, 48 KB at 1536)
bool rms_width_ok(int d) {
  const int v = d / 256;
  return d % 256 == 0 && (v == 1 || v == 2 || v == 3 || v == 4 || v == 6);
}

}  // namespace

extern "C" {

int smat_lm_rmsnorm_fwd(const void* x, const void* residual, const void* w, void* h, void* y,
                        float* rstd, int64_t rows, int d, float eps, void* stream) {
  if (!x || !w || !y || !rstd || (residual && !h)) return SMAT_ERR_NULL_POINTER;
  if (rows < 0 || !rms_width_ok(d)) return SMAT_ERR_BAD_SHAPE;
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) || !aligned16(residual) || !aligned16(h))
    return SMAT_ERR_BAD_ALIGNMENT;
  if (rows == 0) return SMAT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned grid = blocks_for(rows * 32, 256);
  const bf16 *xb = static_cast<const bf16*>(x), *rb = static_cast<const bf16*>(residual),
             *wb = static_cast<const bf16*>(w);
  bf16 *hb = static_cast<bf16*>(h), *yb = static_cast<bf16*>(y);
#define SMAT_RMS_FWD(V) rmsnorm_fwd_kernel<V><<<grid, 256, 0, s>>>(xb, rb, wb, hb, yb, rstd, rows, eps)
  switch (d / 256) {
    case 1: SMAT_RMS_FWD(1); break;
    case 2: SMAT_RMS_FWD(2); break;
    case 3: SMAT_RMS_FWD(3); break;
    case 4: SMAT_RMS_FWD(4); break;
    case 6: SMAT_RMS_FWD(6); break;
  }
#undef SMAT_RMS_FWD
  return status();
}

int smat_lm_rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy,
                        const void* dh, void* dx, float* dw_part, int n_part, int64_t rows, int d,
                        void* stream) {
  if (!x || !w || !rstd || !dy || !dx || !dw_part) return SMAT_ERR_NULL_POINTER;
  if (rows < 0 || n_part < 1 || !rms_width_ok(d)) return SMAT_ERR_BAD_SHAPE;
  if (!aligned16(x) || !aligned16(w) || !aligned16(dy) || !aligned16(dx) || !aligned16(dh))
    return SMAT_ERR_BAD_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bf16 *xb = static_cast<const bf16*>(x), *wb = static_cast<const bf16*>(w),
             *gb = static_cast<const bf16*>(dy), *hb = static_cast<const bf16*>(dh);
  bf16* db = static_cast<bf16*>(dx);
#define SMAT_RMS_BWD(V) \
  rmsnorm_bwd_kernel<V><<<n_part, 256, 0, s>>>(xb, wb, rstd, gb, hb, db, dw_part, rows)
  switch (d / 256) {
    case 1: SMAT_RMS_BWD(1); break;
    case 2: SMAT_RMS_BWD(2); break;
    case 3: SMAT_RMS_BWD(3); break;
    case 4: SMAT_RMS_BWD(4); break;
    case 6: SMAT_RMS_BWD(6); break;
  }
#undef SMAT_RMS_BWD
  return status();
}

static int rope_check(const void* a, const void* q, const void* k, const void* v, const float* c,
                      const float* s, int B, int T, int H, int D) {
  if (!a || !q || !k || !v || !c || !s) return SMAT_ERR_NULL_POINTER;
  if (B < 1 || T < 1 || H < 1 || D < 8 || D % 8) return SMAT_ERR_BAD_SHAPE;
  if (static_cast<int64_t>(B) * T * 3 * H * (D / 8) > 0x7FFFFFFF) return SMAT_ERR_BAD_SHAPE;
  if (!aligned16(a) || !aligned16(q) || !aligned16(k) || !aligned16(v)) return SMAT_ERR_BAD_ALIGNMENT;
  return SMAT_OK;
}

int smat_lm_rope_split_fwd(const void* qkv, const float* cos_t, const float* sin_t, void* q,
                           void* k, void* v, int B, int T, int H, int D, void* stream) {
  int rc = rope_check(qkv, q, k, v, cos_t, sin_t, B, T, H, D);
  if (rc) return rc;
  const int64_t total = static_cast<int64_t>(B) * T * 3 * H * (D / 8);
  rope_kernel<false><<<blocks_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      const_cast<bf16*>(static_cast<const bf16*>(qkv)), static_cast<bf16*>(q),
      static_cast<bf16*>(k), static_cast<bf16*>(v), cos_t, sin_t, B, T, H, D);
  return status();
}

int smat_lm_rope_split_bwd(const void* dq, const void* dk, const void* dv, const float* cos_t,
                           const float* sin_t, void* dqkv, int B, int T, int H, int D,
                           void* stream) {
  int rc = rope_check(dqkv, dq, dk, dv, cos_t, sin_t, B, T, H, D);
  if (rc) return rc;
  const int64_t total = static_cast<int64_t>(B) * T * 3 * H * (D / 8);
  rope_kernel<true><<<blocks_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<bf16*>(dqkv), const_cast<bf16*>(static_cast<const bf16*>(dq)),
      const_cast<bf16*>(static_cast<const bf16*>(dk)),
      const_cast<bf16*>(static_cast<const bf16*>(dv)), cos_t, sin_t, B, T, H, D);
  return status();
}

int smat_lm_swiglu_fwd(const void* a, void* g, int64_t rows, int hidden, void* stream) {
  if (!a || !g) return SMAT_ERR_NULL_POINTER;
  if (rows < 0 || hidden < 8 || hidden % 8) return SMAT_ERR_BAD_SHAPE;
  if (!aligned16(a) || !aligned16(g)) return SMAT_ERR_BAD_ALIGNMENT;
  if (rows == 0) return SMAT_OK;
  swiglu_kernel<false><<<blocks_for(rows * (hidden / 8), 256), 256, 0,
                         static_cast<cudaStream_t>(stream)>>>(
      static_cast<const bf16*>(a), nullptr, static_cast<bf16*>(g), rows, hidden);
  return status();
}

int smat_lm_swiglu_bwd(const void* a, const void* dg, void* da, int64_t rows, int hidden,
                       void* stream) {
  if (!a || !dg || !da) return SMAT_ERR_NULL_POINTER;
  if (rows < 0 || hidden < 8 || hidden % 8) return SMAT_ERR_BAD_SHAPE;
  if (!aligned16(a) || !aligned16(dg) || !aligned16(da)) return SMAT_ERR_BAD_ALIGNMENT;
  if (rows == 0) return SMAT_OK;
  swiglu_kernel<true><<<blocks_for(rows * (hidden / 8), 256), 256, 0,
                        static_cast<cudaStream_t>(stream)>>>(
      static_cast<const bf16*>(a), static_cast<const bf16*>(dg), static_cast<bf16*>(da), rows,
      hidden);
  return status();
}

int smat_lm_cross_entropy(void* logits, const int64_t* targets, float* loss, int64_t rows, int V,
                          float grad_scale, int32_t* err_word, void* stream) {
  if (!logits || !targets || !loss) return SMAT_ERR_NULL_POINTER;
  if (rows < 0 || rows > 0x7FFFFFFF || V < 8 || V % 8) return SMAT_ERR_BAD_SHAPE;
  if (!aligned16(logits)) return SMAT_ERR_BAD_ALIGNMENT;
  if (rows == 0) return SMAT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int bytes = V * 2;
  bf16* zb = static_cast<bf16*>(logits);
  // The two-pass form (second read mostly from L2) at full occupancy measured
  // faster than staging the row in shared memory (64 KB at V = 32000, three
  // CTAs per SM): 2.3 ms against 3.1 ms for 65,536 rows.
  (void)bytes;
  xent_kernel<false><<<static_cast<unsigned>(rows), 256, 0, s>>>(zb, targets, loss, V, grad_scale,
                                                                 err_word);
  return status();
}

}  // extern "C"
