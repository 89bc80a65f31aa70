/*
 * smat_b200.h -- C ABI of the B200 (sm_100a) SMat block-sparse causal softmax
 * attention library (libsmat_b200.so).
 *
 * Conventions
 *   - Tensors q, k, v, o, dO, dq, dk, dv are [B, H, T, D] with the D dimension
 *     contiguous; each is passed as a device pointer plus a host array of three
 *     int64 element strides {stride_b, stride_h, stride_t}.
 *   - lse and delta are contiguous fp32 [B * H * T] device arrays.  lse is the
 *     natural-log normaliser log(sum_j exp(scale * q_i . k_j)) over the
 *     unmasked keys of row i (-inf for an empty row).
 *   - The layout is an int32 CSR over blocks of `block` positions:
 *     indptr[nblocks + 1], indices[nnzb] (key blocks per query block,
 *     ascending) and one kind byte per entry (SMAT_TILE_FULL or
 *     SMAT_TILE_CAUSAL).  The backward dK/dV pass takes the transposed CSR
 *     (query blocks per key block).  All of them live in device memory.
 *   - Every buffer is caller-allocated; no entry point allocates device
 *     memory.  Kernels are enqueued on `stream` (a cudaStream_t, NULL for the
 *     legacy default stream) and the calls return without synchronising.
 *   - Return value: SMAT_OK or an smat_status code; argument errors are
 *     detected on the host before anything is launched.  Device-side faults
 *     of the pipeline (a bounded wait that timed out, a malformed CSR seen by
 *     a kernel) are OR-ed into *err_word (device int32, may be NULL), which the
 *     caller reads after synchronising.
 *   - dtype SMAT_DTYPE_BF16 runs the tcgen05 tensor-core kernels (D in {64,
 *     128}, block in {64, 128}); SMAT_DTYPE_F32 runs full-fp32 CUDA-core
 *     kernels (D in {32, 64, 128}, any block size).
 *
 * These entry points replace, for the softmax arm, the reference's attention
 * call sites: the dense causal SDPA of the softmax arm
 * (src/smat/model.py:217-220) and the fused-kernel table the SMat arm looks up
 * as module attributes (src/smat/attention.py:37-40, 183-185) with its
 * differentiable wrappers (src/smat/kernels/triton_bwd.py:154-196, 331-346).
 */
#ifndef SMAT_B200_H
#define SMAT_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define SMAT_API __attribute__((visibility("default")))
#else
#define SMAT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum smat_status {
  SMAT_OK = 0,
  SMAT_ERR_BAD_SHAPE = 1,
  SMAT_ERR_UNSUPPORTED_D = 2,
  SMAT_ERR_UNSUPPORTED_BLOCK = 3,
  SMAT_ERR_UNSUPPORTED_DTYPE = 4,
  SMAT_ERR_BAD_STRIDE = 5,
  SMAT_ERR_BAD_ALIGNMENT = 6,
  SMAT_ERR_CSR_INVALID = 7,
  SMAT_ERR_NULL_POINTER = 8,
  SMAT_ERR_LAUNCH = 9,
  SMAT_ERR_NO_DEVICE = 10,
  SMAT_ERR_TMA_DESCRIPTOR = 11,
  SMAT_ERR_ROW_TOO_LONG = 12,
  SMAT_ERR_CAPACITY = 13,
  SMAT_ERR_SCRATCH_LIMIT = 14,
  SMAT_ERR_BAD_PATTERN = 15,
  SMAT_ERR_CAPTURE = 16
} smat_status;

enum { SMAT_DTYPE_F32 = 0, SMAT_DTYPE_BF16 = 1 };
enum { SMAT_TILE_FULL = 0, SMAT_TILE_CAUSAL = 1, SMAT_TILE_PATTERN = 2 };

/* Bits of *err_word. */
enum {
  SMAT_DEVERR_WAIT_TIMEOUT = 1,
  SMAT_DEVERR_BAD_CSR = 2,
  SMAT_DEVERR_SCHED_OVERFLOW = 4,
  SMAT_DEVERR_BAD_WORK = 8
};

/* ABI version of this header (incremented when an entry point changes or is added): 5. */
SMAT_API int smat_abi_version(void);

/* Human-readable name of a status code (static string). */
SMAT_API const char* smat_status_string(int status);

/* SMAT_OK if `device` is an sm_100 GPU this library was built for. */
SMAT_API int smat_device_supported(int device);

/* ---------------------------------------------------------------- layouts
 * Host-side builders and checks on host arrays (no GPU needed).
 *
 * smat_layout_build_block: the block layout of the module's mask builder
 * (smat_attention_b200.mask.build_block_mask).  Tile (qb, kb) is active iff
 * kb <= qb and (qb - window <= kb or kb < n_sink or (stride > 0 and
 * kb % stride == stride - 1)); the diagonal tile is SMAT_TILE_CAUSAL.  With
 * indices == NULL only *nnzb_out is computed.  indptr has nblocks + 1 =
 * ceil(T / block) + 1 entries; indices/kind need `capacity` >= nnzb entries.
 * Replaces, for the block kind, the reference's mask constructor
 * (src/smat/mask.py:244-389, build_mask).
 */
SMAT_API int smat_layout_build_block(int T, int block, int window, int stride, int n_sink,
                            int32_t* indptr, int32_t* indices, uint8_t* kind,
                            int64_t capacity, int64_t* nnzb_out);

/* Transposed CSR (per key block, ascending query blocks, kinds carried). */
SMAT_API int smat_layout_transpose(int nblocks, const int32_t* indptr, const int32_t* indices,
                          const uint8_t* kind, int32_t* t_indptr, int32_t* t_indices,
                          uint8_t* t_kind);

/* Checks a (forward or transposed) layout: indptr starts at 0, never
 * decreases and ends at nnzb; indices are in [0, nblocks) and strictly
 * ascending per row; every entry is causal (key block <= query block, i.e.
 * index <= row for the forward CSR and index >= row for the transposed one);
 * the kind is SMAT_TILE_CAUSAL exactly on the diagonal and SMAT_TILE_FULL
 * elsewhere.  Writes the longest row to *max_row_out (may be NULL). */
SMAT_API int smat_layout_validate(int nblocks, int64_t nnzb, const int32_t* indptr,
                         const int32_t* indices, const uint8_t* kind, int transposed,
                         int32_t* max_row_out);

/* ---------------------------------------------------------------- M^(d) masks
 * The reference's own mask family (src/smat/mask.py:244-425, build_mask) run
 * through the softmax kernels.  Its dense mask (mask.py:557-577, materialise)
 * over T positions, n landmark positions and n_P global columns is
 *
 *   rows i <  n:  M[i,j] = (j <= i)                 family SMAT_FAMILY_GEOMETRIC
 *                 M[i,j] = ((i & j) == j)           family SMAT_FAMILY_ENDPOINT
 *   rows i >= n:  M[i,j] = 1 (j < n_P),  C[(i-n) mod B, (j-n_P) mod N0] (n_P <= j < n),
 *                 (j <= i) (j >= n)
 *
 * with C the B x N0 0/1 incidence (CSR C_indptr / C_indices of the spec).  A
 * layout for it has every causal tile that holds a 1; tiles that are all ones
 * are SMAT_TILE_FULL, the diagonal tiles of the two triangles
 * SMAT_TILE_CAUSAL, the rest SMAT_TILE_PATTERN, whose mask the kernels
 * evaluate element-exactly from two bit tables of C with wrap-around:
 *
 *   row_bits[r * row_words + (t >> 5)] bit (t & 31) = C[r][t mod N0],  row_words >= (N0 + 63) / 32
 *   col_bits[c * col_words + (t >> 5)] bit (t & 31) = C[t mod B][c],   col_words >= (B + 63) / 32
 *
 * The endpoint family needs N0 >= n - n_P (its profiles are the identity).
 * Tables passed to the kernels live in device memory; the smat_pattern_mask_*
 * checks read host copies. */
enum { SMAT_FAMILY_GEOMETRIC = 0, SMAT_FAMILY_ENDPOINT = 1 };

typedef struct smat_pattern {
  int family;               /* SMAT_FAMILY_GEOMETRIC or SMAT_FAMILY_ENDPOINT */
  int n;                    /* landmark positions [0, n), 0 <= n_P <= n <= T */
  int n_P;                  /* global columns [0, n_P) */
  int B;                    /* rows of C (row types), >= 1 */
  int N0;                   /* columns of C (profiles), >= 1 */
  int row_words;            /* words per row of row_bits */
  int col_words;            /* words per row of col_bits */
  const uint32_t* row_bits; /* [B][row_words] */
  const uint32_t* col_bits; /* [N0][col_words] */
} smat_pattern_t;

/* Fills both bit tables from C's CSR (host arrays; C_indptr[B + 1], indices
 * in [0, N0)). */
SMAT_API int smat_pattern_tables(int B, int N0, const int64_t* C_indptr, const int32_t* C_indices,
                        uint32_t* row_bits, int row_words, uint32_t* col_bits, int col_words);

/* Tile layout of an M^(d) mask over T positions with square tiles of `block`
 * rows (same CSR conventions as smat_layout_build_block).  c_all_ones != 0
 * says every entry of C is 1 (the d = 1 mask), which makes the long-range
 * tiles full.  Endpoint tiles of the landmark triangle are left out when
 * they hold no 1 (block a power of two dividing n: key block kb meets query
 * block qb iff kb & ~qb == 0). */
SMAT_API int smat_layout_build_pattern(int T, int block, int family, int n, int n_P, int c_all_ones,
                              int32_t* indptr, int32_t* indices, uint8_t* kind, int64_t capacity,
                              int64_t* nnzb_out);

/* smat_layout_validate for M^(d) layouts: SMAT_TILE_PATTERN may appear on
 * any causal entry, SMAT_TILE_CAUSAL only on the diagonal, SMAT_TILE_FULL
 * only off it. */
SMAT_API int smat_layout_validate_pattern(int nblocks, int64_t nnzb, const int32_t* indptr,
                                 const int32_t* indices, const uint8_t* kind, int transposed,
                                 int32_t* max_row_out);

/* Host evaluation of the kernels' mask rule (host tables): rows
 * [row_lo, row_hi) of the dense T x T mask as 0/1 bytes, out[(i - row_lo) * T
 * + j], through the row words the forward and dQ kernels use; the _cols form
 * writes columns [row_lo, row_hi) as rows (out[(j - row_lo) * T + i] =
 * M[i, j]) through the column words of the dK/dV kernel.  The native
 * counterpart of the reference's materialise (mask.py:557-577). */
SMAT_API int smat_pattern_mask_rows(const smat_pattern_t* pattern, int T, int row_lo, int row_hi,
                           uint8_t* out);
SMAT_API int smat_pattern_mask_cols(const smat_pattern_t* pattern, int T, int col_lo, int col_hi,
                           uint8_t* out);

/* ---------------------------------------------------------------- forward
 * o = softmax_M(scale q k^T) v and lse, for the layout (indptr, indices,
 * kind).  max_row is the longest CSR row (from smat_layout_validate).
 * Replaces the softmax arm's F.scaled_dot_product_attention call
 * (src/smat/model.py:217-220) and, as the fused forward of the attention op,
 * the reference's chunk_local launcher (src/smat/kernels/triton_fwd.py:118-152).
 */
SMAT_API int smat_fwd(int dtype,
             const void* q, const int64_t* q_stride,
             const void* k, const int64_t* k_stride,
             const void* v, const int64_t* v_stride,
             void* o, const int64_t* o_stride,
             float* lse,
             int B, int H, int T, int D,
             const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
             int nblocks, int64_t nnzb, int block, int max_row,
             float scale, int32_t* err_word, void* stream);

/* ---------------------------------------------------------------- work lists
 * The *_tiles / *_rows entry points compute a subset of the rows: a shard of
 * the queries (forward, dQ) or of the keys (dK/dV) when one sequence is split
 * across GPUs by query blocks.  `work` is a DEVICE array of n_work int32
 * items, one per CTA and (b, h), run in the given order (put the heaviest
 * first).  Item bits 0..23: a 128-row tile index t (rows [128 t, 128 t + 128)
 * of T); bit 24, forward only: the CTA also computes tile t + 1 (two adjacent
 * query tiles share their K/V loads).  Rows outside the listed tiles are not
 * written.  An item naming a tile past the end, or bit 24 where it is not
 * allowed, sets SMAT_DEVERR_BAD_WORK in *err_word and its CTA does nothing.
 * The layout arguments are the whole layout (or a filtered copy of it, see
 * smat_attention_b200.sharding); outputs of the listed tiles are complete
 * sums over their CSR rows / columns.  No counterpart in the reference, which
 * has no multi-GPU path. */
SMAT_API int smat_fwd_tiles(int dtype,
                   const void* q, const int64_t* q_stride,
                   const void* k, const int64_t* k_stride,
                   const void* v, const int64_t* v_stride,
                   void* o, const int64_t* o_stride,
                   float* lse,
                   int B, int H, int T, int D,
                   const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                   int nblocks, int64_t nnzb, int block, int max_row,
                   float scale, const int32_t* work, int n_work,
                   int32_t* err_word, void* stream);

/* ---------------------------------------------------------------- row exchange
 * Copies of listed token rows between two [B, H, T, D] tensors (a: K or dK,
 * b: V or dV, element strides as elsewhere) and a contiguous wire buffer, for
 * the GPU-to-GPU exchanges of the query-sharded path.  Wire row r holds
 * [2][B][H][D] elements: a[.., rows[r], :] then b[.., rows[r], :].  `rows`
 * (int64, n_rows entries) and the contribution lists are DEVICE arrays; a row
 * outside [0, T) or a contribution outside [0, n_wire) sets
 * SMAT_DEVERR_BAD_WORK and is skipped.  D * element size must be a multiple
 * of 16 bytes and bases / strides 16-byte aligned.  No reference counterpart
 * (the reference has no multi-GPU path).
 *
 * smat_rows_pack:       wire[r] = (a, b)[rows[r]]
 * smat_rows_unpack:     (a, b)[rows[r]] = wire[r]
 * smat_rows_accumulate: (a, b)[rows[e]] += sum over c in
 *                       [contrib_ptr[e], contrib_ptr[e+1]) of wire[contrib_wire[c]],
 *                       in fp32, in list order, rounded once. */
SMAT_API int smat_rows_pack(int dtype, const void* a, const int64_t* a_stride,
                   const void* b, const int64_t* b_stride, int B, int H, int T, int D,
                   const int64_t* rows, int64_t n_rows, void* wire,
                   int32_t* err_word, void* stream);
SMAT_API int smat_rows_unpack(int dtype, void* a, const int64_t* a_stride,
                     void* b, const int64_t* b_stride, int B, int H, int T, int D,
                     const int64_t* rows, int64_t n_rows, const void* wire,
                     int32_t* err_word, void* stream);
SMAT_API int smat_rows_accumulate(int dtype, void* a, const int64_t* a_stride,
                         void* b, const int64_t* b_stride, int B, int H, int T, int D,
                         const int64_t* rows, int64_t n_rows,
                         const int32_t* contrib_ptr, const int64_t* contrib_wire,
                         int64_t n_wire, const void* wire,
                         int32_t* err_word, void* stream);

/* ---------------------------------------------------------------- backward
 * delta[b, h, t] = sum_d dO[b,h,t,d] * o[b,h,t,d]
 * (the row-sum preprocess of the reference's backward,
 * src/smat/kernels/triton_bwd.py:154-196, restated for softmax). */
SMAT_API int smat_bwd_preprocess(int dtype,
                        const void* o, const int64_t* o_stride,
                        const void* dout, const int64_t* do_stride,
                        float* delta, int B, int H, int T, int D, void* stream);

/* smat_bwd_preprocess for rows [row_lo, row_hi) of every (b, h) only; delta
 * keeps its [B*H, T] layout. */
SMAT_API int smat_bwd_preprocess_rows(int dtype,
                             const void* o, const int64_t* o_stride,
                             const void* dout, const int64_t* do_stride,
                             float* delta, int B, int H, int T, int D,
                             int row_lo, int row_hi, void* stream);

/* dk, dv over the transposed CSR (t_indptr, t_indices, t_kind); t_max_row is
 * its longest row.  Replaces the reference's column-parallel backward kernel
 * (src/smat/kernels/triton_bwd.py:98-147). */
SMAT_API int smat_bwd_dkdv(int dtype,
                  const void* q, const int64_t* q_stride,
                  const void* k, const int64_t* k_stride,
                  const void* v, const int64_t* v_stride,
                  const void* dout, const int64_t* do_stride,
                  const float* lse, const float* delta,
                  void* dk, const int64_t* dk_stride,
                  void* dv, const int64_t* dv_stride,
                  int B, int H, int T, int D,
                  const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind,
                  int nblocks, int64_t nnzb, int block, int t_max_row,
                  float scale, int32_t* err_word, void* stream);

/* smat_bwd_dkdv for the key tiles of a work list (items without bit 24). */
SMAT_API int smat_bwd_dkdv_tiles(int dtype,
                        const void* q, const int64_t* q_stride,
                        const void* k, const int64_t* k_stride,
                        const void* v, const int64_t* v_stride,
                        const void* dout, const int64_t* do_stride,
                        const float* lse, const float* delta,
                        void* dk, const int64_t* dk_stride,
                        void* dv, const int64_t* dv_stride,
                        int B, int H, int T, int D,
                        const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind,
                        int nblocks, int64_t nnzb, int block, int t_max_row,
                        float scale, const int32_t* work, int n_work,
                        int32_t* err_word, void* stream);

/* dq over the forward CSR.  Replaces the reference's row-parallel backward
 * kernel (src/smat/kernels/triton_bwd.py:50-94). */
SMAT_API int smat_bwd_dq(int dtype,
                const void* q, const int64_t* q_stride,
                const void* k, const int64_t* k_stride,
                const void* v, const int64_t* v_stride,
                const void* dout, const int64_t* do_stride,
                const float* lse, const float* delta,
                void* dq, const int64_t* dq_stride,
                int B, int H, int T, int D,
                const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                int nblocks, int64_t nnzb, int block, int max_row,
                float scale, int32_t* err_word, void* stream);

/* smat_bwd_dq for the query tiles of a work list (items without bit 24). */
SMAT_API int smat_bwd_dq_tiles(int dtype,
                      const void* q, const int64_t* q_stride,
                      const void* k, const int64_t* k_stride,
                      const void* v, const int64_t* v_stride,
                      const void* dout, const int64_t* do_stride,
                      const float* lse, const float* delta,
                      void* dq, const int64_t* dq_stride,
                      int B, int H, int T, int D,
                      const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                      int nblocks, int64_t nnzb, int block, int max_row,
                      float scale, const int32_t* work, int n_work,
                      int32_t* err_word, void* stream);

/* The whole backward: preprocess into the caller's delta workspace
 * (fp32 [B*H*T]), then dK/dV and dQ.  Replaces the autograd backward of the
 * reference's fused path (src/smat/kernels/triton_bwd.py:162-196).  All
 * three passes are checked before the first launches. */
SMAT_API int smat_bwd(int dtype,
             const void* q, const int64_t* q_stride,
             const void* k, const int64_t* k_stride,
             const void* v, const int64_t* v_stride,
             const void* o, const int64_t* o_stride,
             const void* dout, const int64_t* do_stride,
             const float* lse, float* delta,
             void* dq, const int64_t* dq_stride,
             void* dk, const int64_t* dk_stride,
             void* dv, const int64_t* dv_stride,
             int B, int H, int T, int D,
             const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
             const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind,
             int nblocks, int64_t nnzb, int block, int max_row, int t_max_row,
             float scale, int32_t* err_word, void* stream);

/* The fused backward (bf16, D = 128).  smat_bwd_dkdv_dq zeroes the caller's
 * fp32 accumulator dq_acc ([B*H, T, D] contiguous, 16-byte aligned, at least
 * B*H*T*D floats) and runs one kernel over the transposed CSR that writes dK
 * and dV as smat_bwd_dkdv does and adds dS K (unscaled) for every block pair
 * into dq_acc; smat_bwd_dq_finish then writes dq = bf16(scale * dq_acc) (D in
 * {64, 128}).  dQ needs no second pass over the forward CSR, which would
 * recompute S and dP: 5 block-pair MMAs per pair instead of 7.  The additions
 * into dq_acc are fp32 reductions in L2 whose order varies between runs, so
 * dQ may differ in its last bits from run to run (dK, dV are deterministic);
 * smat_bwd stays the bitwise-deterministic backward.
 * smat_bwd_acc: smat_bwd (pattern may be NULL) through these two passes where
 * they apply (bf16, D = 128), else exactly smat_bwd (dq_acc unused, may be
 * NULL).  The reference's autograd backward (src/smat/kernels/triton_bwd.py:
 * 162-196) accumulates dQ per query block instead. */
SMAT_API int smat_bwd_dkdv_dq(int dtype,
                     const void* q, const int64_t* q_stride,
                     const void* k, const int64_t* k_stride,
                     const void* v, const int64_t* v_stride,
                     const void* dout, const int64_t* do_stride,
                     const float* lse, const float* delta,
                     float* dq_acc, int64_t dq_acc_floats,
                     void* dk, const int64_t* dk_stride,
                     void* dv, const int64_t* dv_stride,
                     int B, int H, int T, int D,
                     const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind,
                     int nblocks, int64_t nnzb, int block, int t_max_row,
                     float scale, int32_t* err_word, void* stream);
SMAT_API int smat_bwd_dq_finish(int dtype, const float* dq_acc, int64_t dq_acc_floats,
                       void* dq, const int64_t* dq_stride,
                       int B, int H, int T, int D, float scale, void* stream);
SMAT_API int smat_bwd_acc(int dtype,
                 const void* q, const int64_t* q_stride,
                 const void* k, const int64_t* k_stride,
                 const void* v, const int64_t* v_stride,
                 const void* o, const int64_t* o_stride,
                 const void* dout, const int64_t* do_stride,
                 const float* lse, float* delta,
                 void* dq, const int64_t* dq_stride,
                 void* dk, const int64_t* dk_stride,
                 void* dv, const int64_t* dv_stride,
                 int B, int H, int T, int D,
                 const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                 const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind,
                 int nblocks, int64_t nnzb, int block, int max_row, int t_max_row,
                 const smat_pattern_t* pattern, float* dq_acc, int64_t dq_acc_floats,
                 float scale, int32_t* err_word, void* stream);

/* smat_fwd and smat_bwd for a layout with SMAT_TILE_PATTERN tiles (from
 * smat_layout_build_pattern) and the device bit tables of its M^(d) mask:
 * the reference's M^(d) masks (src/smat/mask.py:244-425) under softmax
 * attention.  The layout arguments and outputs are those of smat_fwd /
 * smat_bwd; `pattern` is a host struct pointing at device tables, checked
 * (SMAT_ERR_BAD_PATTERN) before any launch.  A PATTERN tile given to the
 * entry points without a pattern sets SMAT_DEVERR_BAD_CSR and counts as
 * masked. */
SMAT_API int smat_fwd_pattern(int dtype,
                     const void* q, const int64_t* q_stride,
                     const void* k, const int64_t* k_stride,
                     const void* v, const int64_t* v_stride,
                     void* o, const int64_t* o_stride,
                     float* lse,
                     int B, int H, int T, int D,
                     const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                     int nblocks, int64_t nnzb, int block, int max_row,
                     const smat_pattern_t* pattern,
                     float scale, int32_t* err_word, void* stream);
SMAT_API int smat_bwd_pattern(int dtype,
                     const void* q, const int64_t* q_stride,
                     const void* k, const int64_t* k_stride,
                     const void* v, const int64_t* v_stride,
                     const void* o, const int64_t* o_stride,
                     const void* dout, const int64_t* do_stride,
                     const float* lse, float* delta,
                     void* dq, const int64_t* dq_stride,
                     void* dk, const int64_t* dk_stride,
                     void* dv, const int64_t* dv_stride,
                     int B, int H, int T, int D,
                     const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                     const int32_t* t_indptr, const int32_t* t_indices, const uint8_t* t_kind,
                     int nblocks, int64_t nnzb, int block, int max_row, int t_max_row,
                     const smat_pattern_t* pattern,
                     float scale, int32_t* err_word, void* stream);

/* ---------------------------------------------------------------- decode
 * One new query per (batch, head) against its KV cache: for b, h,
 *   o[b,h] = softmax_j(scale q[b,h] . k[b,h,j]) v[b,h,j] over the keys j the
 *   layout shows to query position t = pos[b] (its CSR row t / block; FULL
 *   entries all keys, CAUSAL entries j <= t, PATTERN entries the M^(d) rule
 *   of `pattern`, which may be NULL for layouts without PATTERN tiles),
 * and lse[b*H + h] (natural log, may be NULL).  q, o: [B, H, D] with (b, h)
 * element strides q_stride[2] / o_stride[2]; k_cache, v_cache: [B, H, T, D]
 * with (b, h, t) strides; pos: DEVICE int32 [B], each in [0, T) (else
 * SMAT_DEVERR_BAD_WORK and that row's output is 0).  bf16 only, D in {64,
 * 128}.  The splits of a row are combined inside the kernel (one thread-block
 * cluster per row), so `workspace` is not used: it may be NULL, and
 * smat_decode_workspace reports 0 floats (both kept for ABI compatibility).
 * The softmax counterpart of the reference's streaming decoder
 * (src/smat/attention.py:496-535, SmatDecoder.step). */
SMAT_API int smat_decode_workspace(int B, int H, int D, int max_row, int64_t* floats_out);
SMAT_API int smat_decode(int dtype,
                const void* q, const int64_t* q_stride,
                const void* k_cache, const int64_t* k_stride,
                const void* v_cache, const int64_t* v_stride,
                void* o, const int64_t* o_stride,
                float* lse, const int32_t* pos,
                int B, int H, int T, int D,
                const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                int nblocks, int64_t nnzb, int block, int max_row,
                const smat_pattern_t* pattern,
                float scale, float* workspace, int64_t workspace_floats,
                int32_t* err_word, void* stream);

/* smat_bwd_noalloc: smat_bwd for callers that cannot allocate device memory
 * (their memory belongs to another allocator, or cudaMalloc's implicit
 * synchronisation is not allowed on their path, or their budget is fixed at
 * start-up).  Same arguments as smat_bwd minus the delta workspace: delta is
 * kept in a fixed array compiled into the library, 16 MiB per GPU that loads
 * it, held until the process exits.  B*H*T must be <= SMAT_NOALLOC_MAX_ROWS,
 * else SMAT_ERR_SCRATCH_LIMIT before any launch.  All calls share the array:
 * calls whose kernels overlap on the GPU race.  The first call on a device
 * looks up the array's address with that device current and caches it with
 * the identity of the device's context (a call under a new context, e.g.
 * after cudaDeviceReset, looks it up again); make that first call before any
 * stream capture (during a capture the lookup returns SMAT_ERR_CAPTURE).  It
 * has no counterpart in the reference. */
#define SMAT_NOALLOC_MAX_ROWS (1 << 22)
SMAT_API int smat_bwd_noalloc(int dtype,
                              const void* q, const int64_t* q_stride,
                              const void* k, const int64_t* k_stride,
                              const void* v, const int64_t* v_stride,
                              const void* o, const int64_t* o_stride,
                              const void* dout, const int64_t* do_stride,
                              const float* lse,
                              void* dq, const int64_t* dq_stride,
                              void* dk, const int64_t* dk_stride,
                              void* dv, const int64_t* dv_stride,
                              int B, int H, int T, int D,
                              const int32_t* indptr, const int32_t* indices, const uint8_t* kind,
                              const int32_t* t_indptr, const int32_t* t_indices,
                              const uint8_t* t_kind,
                              int nblocks, int64_t nnzb, int block, int max_row, int t_max_row,
                              float scale, int32_t* err_word, void* stream);

/* ---------------------------------------------------------------- self-test
 * smat_selftest_wait_timeout: runs the kernels' bounded-wait failure path on
 * the device.  One CTA waits on an mbarrier nothing arrives on with the same
 * wait code the kernels use, but with a limit of `limit_cycles` SM cycles
 * (1000 .. SMAT_SELFTEST_MAX_LIMIT, about 0.5 ms at 1e6): the wait gives up,
 * ORs SMAT_DEVERR_WAIT_TIMEOUT into *err_word and raises the CTA's abort flag;
 * a second warp waiting elsewhere leaves through that flag; both run the
 * bounded drain wait; the CTA frees its TMEM and returns, leaving the context
 * usable.  report: device int32[4], written by the kernel: {first wait gave up,
 * second wait gave up, second wait left through the abort flag, both drains
 * gave up}, each 1 when the path behaved.  Counterpart of the reference's
 * per-kernel retire-with-warning fallback (src/smat/attention.py:58-75). */
#define SMAT_SELFTEST_MAX_LIMIT (100000000LL)
SMAT_API int smat_selftest_wait_timeout(int64_t limit_cycles, int32_t* err_word, int32_t* report,
                                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SMAT_B200_H */
