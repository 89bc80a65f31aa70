// M^(d) masks inside the softmax kernels: the in-tile mask of PATTERN tiles.
//
// The dense mask of an M^(d) spec (reference src/smat/mask.py:557-577,
// materialise) over T positions, n landmark positions and n_P global columns:
//
//   rows i <  n:  M[i, j] = (j <= i)                  geometric family (L_n)
//                 M[i, j] = ((i & j) == j)            endpoint family (zeta)
//                 (columns j >= n are 0)
//   rows i >= n:  M[i, j] = 1                          j <  n_P
//                 M[i, j] = C[(i - n) mod B, prof(j)]  n_P <= j < n
//                 M[i, j] = (j <= i)                   j >= n
//
// with prof(j) = (j - n_P) mod N0 (geometric; reference mask.py prof_of_column)
// or j - n_P (endpoint, where N0 >= n - n_P so the same expression holds) and
// C the B x N0 incidence.  The kernels read M in 32-bit words: bit c of a row
// word is M[i, j0 + c] (one query row, 32 keys; forward and dQ), bit c of a
// column word is M[i0 + c, j] (one key, 32 queries; dK/dV).  C enters through
// two bit tables with wrap-around, so that any 32 consecutive profiles (or row
// types) are one funnel shift of two adjacent words:
//
//   row_bits[r][t] = C[r][t mod N0]   for t < 32 row_words, row_words >= (N0 + 63) / 32
//   col_bits[c][t] = C[t mod B][c]    for t < 32 col_words, col_words >= (B + 63) / 32
//
// The functions are host + device so the host library can evaluate the very
// same rule when it checks a layout against a dense mask.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define SMAT_HD __host__ __device__ __forceinline__
#else
#define SMAT_HD inline
#endif

namespace smat {

enum : int { MD_GEOMETRIC = 0, MD_ENDPOINT = 1 };

struct MdPattern {
  const uint32_t* row_bits;  // [B][row_words]
  const uint32_t* col_bits;  // [N0][col_words]
  int family;                // MD_GEOMETRIC or MD_ENDPOINT
  int n, n_P, B, N0;
  int row_words, col_words;
};

SMAT_HD uint32_t md_load(const uint32_t* p) {
#if defined(__CUDA_ARCH__)
  return __ldg(p);
#else
  return *p;
#endif
}

// bits c of [0, 32) with a <= j0 + c < b
SMAT_HD uint32_t span_word(int j0, int a, int b) {
  const int lo = a - j0 > 0 ? a - j0 : 0;
  const int hi = b - j0 < 32 ? b - j0 : 32;
  if (hi <= lo) return 0u;
  const uint32_t upper = hi >= 32 ? 0xffffffffu : ((1u << hi) - 1u);
  return upper & ~((1u << lo) - 1u);
}

// 32 bits of a bit row starting at bit t (the row has a word past t >> 5)
SMAT_HD uint32_t bits32(const uint32_t* row, int t) {
  const uint32_t lo = md_load(row + (t >> 5)), hi = md_load(row + (t >> 5) + 1);
  const int sh = t & 31;
  return sh ? ((lo >> sh) | (hi << (32 - sh))) : lo;
}

// bits c of [0, 32) with c a subset of s (c & ~s == 0), s < 32
SMAT_HD uint32_t subset_word(int s) {
  uint32_t w = 1u;
  for (int b = 0; b < 5; ++b)
    if ((s >> b) & 1) w |= w << (1 << b);
  return w;
}

// bits c of [0, 32) with c a superset of s (c & s == s), s < 32
SMAT_HD uint32_t superset_word(int s) {
  uint32_t w = 1u << s;
  for (int b = 0; b < 5; ++b)
    if (!((s >> b) & 1)) w |= w << (1 << b);
  return w;
}

// Row word: bit c = M[i, j0 + c] for query i (any i >= 0) and j0 % 32 == 0;
// keys at or past T are 0.
SMAT_HD uint32_t md_row_word(const MdPattern& m, int T, int i, int j0) {
  uint32_t w;
  if (i < m.n) {
    // endpoint: j = j0 + c with c < 32 is a subset of i iff the bits of j0
    // lie in i and c is a subset of i's low five bits
    w = m.family == MD_ENDPOINT ? (((j0 & ~i) == 0) ? subset_word(i & 31) : 0u) : 0xffffffffu;
    w &= span_word(j0, 0, m.n);
  } else {
    w = span_word(j0, 0, m.n_P);
    const int g0 = j0 > m.n_P ? j0 : m.n_P;
    const int g1 = j0 + 32 < m.n ? j0 + 32 : m.n;
    if (g0 < g1) {
      const int rho = (i - m.n) % m.B;
      const uint32_t b = bits32(m.row_bits + static_cast<int64_t>(rho) * m.row_words,
                                (g0 - m.n_P) % m.N0);
      w |= (b << (g0 - j0)) & span_word(j0, g0, g1);
    }
    w |= span_word(j0, m.n, i + 1);
  }
  return w & span_word(j0, 0, i + 1 < T ? i + 1 : T);
}

// Column word: bit c = M[i0 + c, j] for key j (any j >= 0) and i0 % 32 == 0;
// queries at or past T are 0.
SMAT_HD uint32_t md_col_word(const MdPattern& m, int T, int j, int i0) {
  uint32_t w = 0u;
  if (j < m.n) {   // landmark rows [j, n)
    w = span_word(i0, j, m.n);
    if (m.family == MD_ENDPOINT)
      w &= ((j & ~31 & ~i0) == 0) ? superset_word(j & 31) : 0u;
  }
  if (j < m.n_P) {
    w |= span_word(i0, m.n, T);
  } else if (j < m.n) {
    const int r0 = i0 > m.n ? i0 : m.n;
    const int r1 = i0 + 32 < T ? i0 + 32 : T;
    if (r0 < r1) {
      const int pj = (j - m.n_P) % m.N0;
      const uint32_t b = bits32(m.col_bits + static_cast<int64_t>(pj) * m.col_words,
                                (r0 - m.n) % m.B);
      w |= (b << (r0 - i0)) & span_word(i0, r0, r1);
    }
  } else {
    w |= span_word(i0, j, T);
  }
  return w & span_word(i0, 0, T);
}

}  // namespace smat
