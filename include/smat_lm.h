/*
 * smat_lm.h -- fused elementwise kernels of the language-model training step
 * (libsmat_b200.so, next to the attention ABI of smat_b200.h).
 *
 * The model is the reference's LM template (tasks/lm.py:45-126: RMSNorm,
 * interleaved RoPE, tied head) with a SwiGLU MLP; these kernels replace its
 * eager elementwise torch expressions.  Tensors are bf16 device arrays,
 * row-major and contiguous, 16-byte aligned; statistics and arithmetic are
 * fp32, each output is rounded to bf16 once.  Status codes are those of
 * smat_b200.h.  Kernels are enqueued on `stream` and do not synchronise.
 * No counterpart exists on the reference's softmax path (tasks/lm.py runs
 * these steps as torch expressions).
 */
#ifndef SMAT_LM_H_
#define SMAT_LM_H_

#include <stdint.h>

#include "smat_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* y = h / sqrt(mean(h^2) + eps) * w over rows of d (tasks/lm.py:45-48) with
 * h = x, or, given a residual r (may be NULL), h = bf16(x + r) written to
 * h_out (the pre-norm block's residual add fused into its norm);
 * rstd[row] = 1 / sqrt(mean(h^2) + eps) (fp32) for the backward.
 * d in {256, 512, 768, 1024, 1536}. */
SMAT_API int smat_lm_rmsnorm_fwd(const void* x, const void* residual, const void* w, void* h_out,
                        void* y, float* rstd, int64_t rows, int d, float eps, void* stream);

/* dx = dh + (gradient of the RMSNorm above at h through dy), dh (may be
 * NULL) being the gradient h receives along the residual stream;
 * dw_part[n_part][d] (fp32) receives per-CTA partial sums of dy * h * rstd,
 * which the caller adds up (deterministic). */
SMAT_API int smat_lm_rmsnorm_bwd(const void* h, const void* w, const float* rstd, const void* dy,
                        const void* dh, void* dx, float* dw_part, int n_part, int64_t rows,
                        int d, void* stream);

/* qkv [B, T, 3, H, D] -> q, k, v [B, H, T, D] with q and k rotated pairwise,
 * (x[2i], x[2i+1]) -> (x1 c - x2 s, x1 s + x2 c), c / s = cos / sin tables
 * [T, D/2] fp32 of t / base^(2i/D) (tasks/lm.py:57-60).  D % 8 == 0. */
SMAT_API int smat_lm_rope_split_fwd(const void* qkv, const float* cos_t, const float* sin_t,
                           void* q, void* k, void* v, int B, int T, int H, int D,
                           void* stream);

/* The backward: dq, dk (rotated back), dv [B, H, T, D] -> dqkv [B, T, 3, H, D]. */
SMAT_API int smat_lm_rope_split_bwd(const void* dq, const void* dk, const void* dv,
                           const float* cos_t, const float* sin_t, void* dqkv,
                           int B, int T, int H, int D, void* stream);

/* a [rows, 2 hidden] = (a1 | a3) -> g [rows, hidden] = silu(a1) * a3. */
SMAT_API int smat_lm_swiglu_fwd(const void* a, void* g, int64_t rows, int hidden, void* stream);

/* da [rows, 2 hidden] from a and dg [rows, hidden]. */
SMAT_API int smat_lm_swiglu_bwd(const void* a, const void* dg, void* da, int64_t rows, int hidden,
                       void* stream);

/* Softmax cross-entropy over logits [rows, V] (bf16, overwritten):
 * loss[row] = logsumexp(z_row) - z_row[target[row]] (fp32), then
 * z_row := grad_scale * (softmax(z_row) - onehot(target[row])) in bf16.
 * A target outside [0, V) sets SMAT_DEVERR_BAD_WORK in *err_word (may be
 * NULL) and that row's loss is 0.  V % 8 == 0. */
SMAT_API int smat_lm_cross_entropy(void* logits, const int64_t* targets, float* loss, int64_t rows,
                          int V, float grad_scale, int32_t* err_word, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SMAT_LM_H_ */
