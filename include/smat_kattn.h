/*
 * smat_kattn.h -- the reference's kernelised-attention schedule on B200
 * (libsmat_b200.so, beside the softmax ABI of smat_b200.h).
 *
 * The reference computes smat_attention(Phi, Psi, Vb, spec) (src/smat/
 * attention.py:391-455) from three fused passes that its Triton module exports
 * (src/smat/kernels/triton_fwd.py:49-311, triton_bwd.py:50-312); these entry
 * points are their counterparts.  All tensors are fp32, contiguous, device
 * memory; statuses are those of smat_b200.h; kernels are enqueued on
 * `stream`.
 */
#ifndef SMAT_KATTN_H_
#define SMAT_KATTN_H_

#include <stdint.h>

#include "smat_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* out[b] = phi[b] sin[b] + tril(phi[b] psi[b]^T) vb[b] for every chunk b
 * (chunk_local, triton_fwd.py:49-152): phi, psi [n_chunks, C, R], vb, out
 * [n_chunks, C, P], sin [n_chunks, R, P].  tcgen05 kind::tf32 (TF32 inputs,
 * fp32 accumulation, the reference's allow_tf32 dots).  C = 128, R in {32, 64,
 * 128}, 1 <= P <= 128 (<= 96 when R = 128); phi and psi 16-byte aligned. */
SMAT_API int smat_kattn_chunk_local_fwd(const float* phi, const float* psi, const float* vb,
                               const float* sin_, float* out, int64_t n_chunks, int C,
                               int R, int P, int32_t* err_word, void* stream);

/* The backward of chunk_local (triton_bwd.py:50-196) except dsin (= phi^T dout
 * per chunk, a plain GEMM left to the caller): dphi = dout sin^T +
 * tril(dout vb^T) psi, dpsi = tril(dout vb^T)^T phi, dvb = tril(phi psi^T)^T
 * dout, written to dphi, dpsi [n_chunks, C, R] and dvb [n_chunks, C, P].
 * Three launches of the same tcgen05 kind::tf32 tile kernel; shapes as for
 * smat_kattn_chunk_local_fwd. */
SMAT_API int smat_kattn_chunk_local_bwd(const float* phi, const float* psi, const float* vb,
                               const float* sin_, const float* dout, float* dphi,
                               float* dpsi, float* dvb, int64_t n_chunks, int C, int R, int P,
                               int32_t* err_word, void* stream);

/* F[b, x] = sum_{j in [n_P, n), (j - n_P) mod N0 = x} psi[b, j] vb[b, j]^T
 * (pool, triton_fwd.py:225-311): psi [nb, T, R], vb [nb, T, P], F [nb, N0, R, P];
 * shared staging of 64 (R4 + S) + R4 S floats <= 200 KB (R4 = R rounded up to
 * 4, S = P rounded up to 4 with an odd count of 4-float units).  fp32 FMAs,
 * columns in order. */
SMAT_API int smat_kattn_pool_fwd(const float* psi, const float* vb, float* F, int nb, int T,
                        int R, int P, int n_P, int n, int N0, void* stream);

/* Its backward (triton_bwd.py:203-278): for every column j of profile x,
 * dpsi[b, j] = dF[b, x] vb[b, j], dvb[b, j] = dF[b, x]^T psi[b, j]; rows outside
 * [n_P, n) are not written (the caller zeroes them).  (R S + 64 (R + S)) floats
 * of staging <= 200 KB, S as above. */
SMAT_API int smat_kattn_pool_bwd(const float* psi, const float* vb, const float* dF,
                        float* dpsi, float* dvb, int nb, int T, int R, int P, int n_P,
                        int n, int N0, void* stream);

/* U[b, h] = sum_{e in [ptr[h], ptr[h+1])} F[b, idx[e]] over rows of RP floats
 * (incidence, triton_fwd.py:161-222): F [nb, N_in, RP], U [nb, N_out, RP],
 * ptr (int64, N_out + 1) and idx (int32) a CSR in device memory.  With the
 * transposed CSR it is its own backward (triton_bwd.py:281-316).  An index
 * outside [0, N_in) sets SMAT_DEVERR_BAD_CSR and is skipped. */
SMAT_API int smat_kattn_incidence(const float* F, const int64_t* ptr, const int32_t* idx,
                         float* U, int nb, int N_in, int N_out, int RP,
                         int32_t* err_word, void* stream);

/* The op's final division (attention.py:450-451) over rows of P floats:
 * out[r, c] = H[r, c] / H[r, P - 1], c < P - 1 (H [rows, P], out [rows, P - 1],
 * both contiguous fp32). */
SMAT_API int smat_kattn_normalise_fwd(const float* H, float* out, int64_t rows, int P,
                             void* stream);

/* Its backward: dH[r, c] = dout[r, c] / H[r, P - 1] for c < P - 1 and
 * dH[r, P - 1] = -sum_c dout[r, c] H[r, c] / H[r, P - 1]^2 (dout [rows, P - 1],
 * dH [rows, P]). */
SMAT_API int smat_kattn_normalise_bwd(const float* H, const float* dout, float* dH,
                             int64_t rows, int P, void* stream);

/* One streaming-decode token of the kernelised op for nb sequences
 * (SmatDecoder.step, attention.py:521-527): S[b] += psi[b] vb[b]^T, then
 * o = phi[b]^T (S[b] + U[b, h]) and out[b, c] = o[c] / o[P - 1] for c < P - 1.
 * phi, psi [nb, R]; vb [nb, P]; S [nb, R, P] (updated in place);
 * U [nb, nU, R, P] (the prefill's type table); out [nb, P - 1]; h the
 * token's type (its step index mod nU).  R, P <= 1024. */
SMAT_API int smat_kattn_decode_step(const float* phi, const float* psi, const float* vb,
                           float* S, const float* U, float* out, int nb, int R, int P,
                           int nU, int h, void* stream);

/* The causal scan's chunk prefix (segmented_causal_scan, attention.py:134-192):
 * for every sequence s and chunk c of C rows (nc = ceil(T / C), rows past T
 * count as zero),
 *   out[s, c] = sum over chunks c' of c's segment with c' < c of a_c'^T b_c'
 * (reverse != 0: c' > c), where a_c' = rows [c' C, c' C + C) of a[s] ([T, R]) and
 * b_c' likewise of b[s] ([T, P]); the segments are chunks [0, nc0) and
 * [nc0, nc).  A shifted scan: a chunk's own product never enters its output,
 * and nothing crosses the segment boundary.  Forward: (psi, vb) -> Sin; backward:
 * (phi, dout), reverse -> the summaries' gradient.  a [nb, T, R], b [nb, T, P],
 * out [nb, nc, R, P], all contiguous fp32.  C (RA + PB) * 4 <= 200 KB (RA = R
 * rounded up to 8, PB = P rounded up to 4). */
SMAT_API int smat_kattn_chunk_prefix(const float* a, const float* b, float* out, int nb, int T,
                                     int C, int R, int P, int nc0, int reverse, void* stream);

/* The summaries' backward: for every chunk c, da_c += b_c dD_c^T and
 * db_c += a_c dD_c (the gradient of D_c = a_c^T b_c; rows past T untouched).
 * a, da [nb, T, R]; b, db [nb, T, P]; dD [nb, nc, R, P]. */
SMAT_API int smat_kattn_chunk_expand(const float* a, const float* b, const float* dD, float* da,
                                     float* db, int nb, int T, int C, int R, int P,
                                     void* stream);

/* query_by_type (attention.py:310-330): out[s, i] (+)= phi[s, i] U[s, i mod nU] for
 * the T_R recent rows i (accumulate != 0 adds into out).  phi rows of R floats,
 * out rows of P floats, both contiguous within a sequence, sequence strides
 * given in floats (so phi may be Phi[:, n:] and out H[:, n:] of the whole
 * tensors); U [nb, nU, R, P] contiguous. */
SMAT_API int smat_kattn_query_by_type(const float* phi, int64_t phi_seq_stride, const float* U,
                                      float* out, int64_t out_seq_stride, int nb, int T_R, int R,
                                      int P, int nU, int accumulate, void* stream);

/* Its backward: dphi[s, i] = dout[s, i] U[s, i mod nU]^T (written) and
 * dU[s, h] = sum over the rows i of type h of phi[s, i]^T dout[s, i] (written,
 * zero for a type without rows); strides as above. */
SMAT_API int smat_kattn_query_by_type_bwd(const float* phi, int64_t phi_seq_stride,
                                          const float* U, const float* dout,
                                          int64_t dout_seq_stride, float* dphi,
                                          int64_t dphi_seq_stride, float* dU, int nb, int T_R,
                                          int R, int P, int nU, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SMAT_KATTN_H_ */
