// Chunk schedules of the tensor-core kernels.
//
// A CTA owns NROWS consecutive rows of a block CSR (query blocks for the
// forward / dQ kernels, key blocks for dK/dV over the transposed CSR).  Its
// chunk list is the sorted union of those rows; each entry carries, for every
// owned row, whether the block is absent, fully visible, causal (diagonal) or
// patterned (an M^(d) tile, masked by the rule in pattern.cuh) for that row.
// MergeIter produces the list one entry at a time straight
// from the CSR in global memory, so rows of any length are supported; every
// warp role runs its own iterator and all see the same sequence.
#pragma once

#include "common.cuh"
#include "pattern.cuh"

namespace smat {

enum : uint32_t { ST_ABSENT = 0, ST_FULL = 1, ST_CAUSAL = 2, ST_PATTERN = 3 };

// row state of a CSR kind byte: 1 causal, 2 pattern, anything else full
__device__ __forceinline__ uint32_t kind_state(uint8_t k) {
  return k == 1 ? ST_CAUSAL : (k == 2 ? ST_PATTERN : ST_FULL);
}

// entry: bits 0..23 block index, bits 24 + 2 r .. 25 + 2 r the state of row r
__device__ __forceinline__ uint32_t sched_block(uint32_t e) { return e & 0xFFFFFFu; }
__device__ __forceinline__ uint32_t sched_state(uint32_t e, int r) {
  return (e >> (24 + 2 * r)) & 3u;
}
// states of rows [r0, r0 + n) as one bit field (non-zero = any row active)
__device__ __forceinline__ uint32_t sched_states(uint32_t e, int r0, int n) {
  return (e >> (24 + 2 * r0)) & ((1u << (2 * n)) - 1u);
}

template <int MAXROWS>
struct MergeIter {
  const int32_t* idx;
  const uint8_t* kind;
  int lo[MAXROWS], hi[MAXROWS];
  int head[MAXROWS];     // block index at lo (prefetched), INT_MAX once a row is done
  uint8_t hk[MAXROWS];   // its kind byte
  int last;
  int nb;
  bool bad;

  __device__ __forceinline__ void fetch(int s) {
    if (lo[s] < hi[s]) {
      head[s] = __ldg(idx + lo[s]);
      hk[s] = __ldg(kind + lo[s]);
    } else {
      head[s] = 0x7FFFFFFF;
      hk[s] = 0;
    }
  }

  // Rows [row0, row0 + nrows) of the CSR; rows >= nblocks are empty.  Invalid
  // CSR content sets DEV_ERR_BAD_CSR in *err and ends the sequence.
  __device__ __forceinline__ void init(const int32_t* __restrict__ indptr,
                                       const int32_t* __restrict__ indices,
                                       const uint8_t* __restrict__ kinds, int nblocks, int nnzb,
                                       int row0, int nrows, int32_t* err) {
    idx = indices;
    kind = kinds;
    nb = nblocks;
    last = -1;
    bad = false;
#pragma unroll
    for (int s = 0; s < MAXROWS; ++s) {
      lo[s] = hi[s] = 0;
      const int r = row0 + s;
      if (s < nrows && r < nblocks) {
        const int a = indptr[r], b = indptr[r + 1];
        if (a < 0 || b < a || b > nnzb) {
          bad = true;
        } else {
          lo[s] = a;
          hi[s] = b;
        }
      }
      fetch(s);
    }
    if (bad && err) atomicOr(err, DEV_ERR_BAD_CSR);
  }

  // Next entry of the union; false at the end (or on invalid content).  The
  // heads consumed here were loaded by the previous call, and the loads for
  // the following call are issued before returning, so their latency hides
  // behind the caller's work on this entry.
  __device__ __forceinline__ bool next(uint32_t& e, int32_t* err) {
    if (bad) return false;
    int best = 0x7FFFFFFF;
#pragma unroll
    for (int s = 0; s < MAXROWS; ++s) best = min(best, head[s]);
    if (best == 0x7FFFFFFF) return false;
    if (best <= last || best < 0 || best >= nb || best > 0xFFFFFF) {
      bad = true;
      if (err) atomicOr(err, DEV_ERR_BAD_CSR);
      return false;
    }
    uint32_t out = static_cast<uint32_t>(best);
#pragma unroll
    for (int s = 0; s < MAXROWS; ++s) {
      if (head[s] == best) {
        out |= kind_state(hk[s]) << (24 + 2 * s);
        ++lo[s];
        fetch(s);
      }
    }
    last = best;
    e = out;
    return true;
  }
};

// Chunks of `cn` streamed rows (128, or 64 with bs = 64): cn / bs consecutive
// entries of the merged list (one entry for bs = cn, two for bs = 64 and
// cn = 128).  A missing second entry is 0 (no row states).
template <int MAXROWS>
struct ChunkPair {
  MergeIter<MAXROWS> it;
  int epc;
  __device__ __forceinline__ void init(const int32_t* indptr, const int32_t* indices,
                                       const uint8_t* kinds, int nblocks, int nnzb, int row0,
                                       int nrows, int bs, int32_t* err, int cn = 128) {
    it.init(indptr, indices, kinds, nblocks, nnzb, row0, nrows, err);
    epc = cn / bs;
  }
  __device__ __forceinline__ bool next(uint32_t* e, int32_t* err) {
    if (!it.next(e[0], err)) return false;
    e[1] = 0u;
    if (epc == 2) {
      uint32_t t;
      if (it.next(t, err)) e[1] = t;
    }
    return true;
  }
};
__device__ __forceinline__ bool entry_present(uint32_t e) { return (e >> 24) != 0u; }

}  // namespace smat
