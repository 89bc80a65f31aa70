// Per-tile chunk schedule.  The tensor-core kernels work on 128-row tiles; a
// tile covers SUB = 128 / bs consecutive blocks of the layout (SUB is 1 for
// bs = 128 and 2 for bs = 64).  The tile's chunk list is the sorted union of
// those SUB CSR rows, each entry carrying, per sub-block, whether the chunk is
// absent, fully visible or causal for that sub-block's rows.
#pragma once

#include "common.cuh"

namespace smat {

enum : uint32_t { ST_ABSENT = 0, ST_FULL = 1, ST_CAUSAL = 2 };

__device__ __forceinline__ uint32_t sched_block(uint32_t e) { return e & 0xFFFFFFu; }
__device__ __forceinline__ uint32_t sched_state(uint32_t e, int sub) {
  return (e >> (24 + 2 * sub)) & 3u;
}

// Merge CSR rows [row0, row0 + sub) into `out` (capacity `cap`).  Invalid CSR
// content (indptr out of range or decreasing, block index >= nblocks, rows not
// ascending) sets DEV_ERR_BAD_CSR and yields an empty or truncated list.
// Returns the number of entries.  Run by one thread.
__device__ __forceinline__ int build_schedule(const int32_t* __restrict__ indptr,
                                              const int32_t* __restrict__ indices,
                                              const uint8_t* __restrict__ kind, int nblocks,
                                              int nnzb, int row0, int sub, uint32_t* out, int cap,
                                              int32_t* err) {
  int lo[2] = {0, 0}, hi[2] = {0, 0};
  int nrows = 0;
  for (int s = 0; s < sub; ++s) {
    const int r = row0 + s;
    if (r >= nblocks) break;
    const int a = indptr[r], b = indptr[r + 1];
    if (a < 0 || b < a || b > nnzb) {
      if (err) atomicOr(err, DEV_ERR_BAD_CSR);
      return 0;
    }
    lo[s] = a;
    hi[s] = b;
    nrows = s + 1;
  }
  int n = 0;
  int last = -1;
  while (true) {
    // smallest head among the rows
    int best = 0x7FFFFFFF;
    for (int s = 0; s < nrows; ++s)
      if (lo[s] < hi[s]) best = min(best, indices[lo[s]]);
    if (best == 0x7FFFFFFF) break;
    if (best <= last || best < 0 || best >= nblocks) {
      if (err) atomicOr(err, DEV_ERR_BAD_CSR);
      break;
    }
    uint32_t e = static_cast<uint32_t>(best);
    for (int s = 0; s < nrows; ++s) {
      if (lo[s] < hi[s] && indices[lo[s]] == best) {
        const uint32_t st = kind[lo[s]] == 1 ? ST_CAUSAL : ST_FULL;
        e |= st << (24 + 2 * s);
        ++lo[s];
      }
    }
    if (n >= cap) {
      if (err) atomicOr(err, DEV_ERR_SCHED_OVERFLOW);
      break;
    }
    out[n++] = e;
    last = best;
  }
  return n;
}

}  // namespace smat
