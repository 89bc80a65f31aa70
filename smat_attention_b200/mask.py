"""Mask constructors for SMat attention.

Two mask families share one container, :class:`MaskSpec`:

``kind="geometric"`` / ``kind="endpoint"``
    The ``M^(d)`` point-hyperplane incidence masks of the reference
    (``src/smat/mask.py:244-425``), restated here so that a user of
    ``smat.mask.build_mask`` / ``materialise`` / ``incidence_audit`` gets the
    same spec, the same incidence CSR and the same dense mask, bit for bit.

``kind="block"``
    The block-sparse causal layout consumed by the B200 softmax kernels.  With
    block size ``bs``, query block ``qb`` and key block ``kb``, the tile
    ``(qb, kb)`` is active iff ``kb <= qb`` and at least one of

    * ``qb - window <= kb``                 (local window plus the diagonal),
    * ``kb < n_sink``                       (sink blocks),
    * ``stride > 0 and kb % stride == stride - 1``  (strided summary blocks)

    holds.  The diagonal tile ``kb == qb`` is element-wise causal (``j <= i``);
    every other active tile is fully unmasked.  The layout is emitted as an
    int32 CSR of active key blocks per query block (ascending, the diagonal
    last), a per-entry tile kind byte (``KIND_FULL`` / ``KIND_CAUSAL``), and the
    transposed CSR (per key block, the query blocks that read it), which the
    backward dK/dV pass walks.  The reference has no block layout; this
    definition is the one the parity tests hold the kernels to.

``kind="pattern"``
    An ``M^(d)`` mask tiled for the same kernels (:func:`pattern_layout`).
    Every causal tile that holds a 1 is active; tiles that are all ones are
    ``KIND_FULL``, the diagonal tiles of the landmark and recent triangles
    ``KIND_CAUSAL``, and the rest ``KIND_PATTERN``: the kernels evaluate their
    mask element by element from two bit tables of the incidence ``C`` (its
    rows and its columns, each extended by wrap-around so that any 32
    consecutive profiles or row types are one shift of two words).

Everything here is host-side numpy; :func:`to_device` stages the int32 arrays
as torch tensors for the CUDA kernels.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import numpy as np

__all__ = [
    "MaskSpec",
    "build_mask",
    "build_block_mask",
    "incidence_audit",
    "materialise",
    "estimate_cost",
    "next_prime",
    "d_max_geometric",
    "planted_hyperplane_normals",
    "block_layout_stats",
    "to_device",
    "KIND_FULL",
    "KIND_CAUSAL",
    "KIND_PATTERN",
    "pattern_layout",
]

KIND_FULL = 0      # tile fully unmasked
KIND_CAUSAL = 1    # diagonal tile: key position <= query position
KIND_PATTERN = 2   # M^(d) tile: mask evaluated from the bit tables of C


# ---------------------------------------------------------------------------
# number theory over F_q
# ---------------------------------------------------------------------------

def _is_prime(x: int) -> bool:
    if x < 2:
        return False
    if x in (2, 3):
        return True
    if x % 2 == 0:
        return False
    f = 3
    while f * f <= x:
        if x % f == 0:
            return False
        f += 2
    return True


def next_prime(x: int) -> int:
    """Smallest prime ``>= max(2, x)`` (reference ``src/smat/mask.py:82-87``)."""
    p = max(2, int(x))
    while not _is_prime(p):
        p += 1
    return p


def _lex_points(q: int, dim: int) -> np.ndarray:
    """All ``q**dim`` points of ``F_q^dim`` as base-``q`` digit rows.

    Point ``idx`` has coordinates ``x_k = (idx // q^(dim-1-k)) mod q`` (most
    significant digit first), so the basis vector ``e_l`` is point
    ``q^(dim-l)``.  This numbering is part of the spec's format: the incidence
    CSR stores point indices (reference ``src/smat/mask.py:90-100``).
    """
    if dim == 0:
        return np.zeros((1, 0), dtype=np.int64)
    idx = np.arange(q ** dim, dtype=np.int64)
    digits = np.empty((idx.size, dim), dtype=np.int64)
    rest = idx.copy()
    for k in range(dim - 1, -1, -1):
        digits[:, k] = rest % q
        rest //= q
    return digits


def planted_hyperplane_normals(d: int) -> List[Tuple[np.ndarray, int]]:
    """The ``2^(d-1)`` planted hyperplanes ``(a_R, b_R)``, ``R`` a bitmask.

    For a proper subset ``R``: ``a_R`` has a 0 at coordinate ``k`` iff bit ``k``
    of ``R`` is set, else 1, and ``b_R = 0``.  For the full set: ``a_R`` all
    ones, ``b_R = 1``.  Then ``e_i in H_R  <=>  i in R`` (reference
    ``src/smat/mask.py:103-126``).
    """
    dim = d - 1
    full = (1 << dim) - 1
    out: List[Tuple[np.ndarray, int]] = []
    for R in range(1 << dim):
        bits = np.array([(R >> k) & 1 for k in range(dim)], dtype=np.int64)
        if R == full:
            out.append((np.ones(dim, dtype=np.int64), 1))
        else:
            out.append((1 - bits, 0))
    return out


def d_max_geometric(T: int, *, chunk: int = 1, n_P: int = 0) -> int:
    """Largest ``d`` with a geometric ``M^(d)`` at this ``T``
    (reference ``src/smat/mask.py:129-143``)."""
    d = 1
    while True:
        try:
            build_mask(T, d + 1, chunk=chunk, n_P=n_P, _probe=True)
        except (ValueError, NotImplementedError):
            return d
        d += 1


# ---------------------------------------------------------------------------
# the spec
# ---------------------------------------------------------------------------

@dataclass
class MaskSpec:
    """A precompiled mask.  Arrays are numpy; :func:`to_device` stages them.

    Field names and meanings for the ``M^(d)`` kinds follow the reference's
    ``MaskSpec`` (``src/smat/mask.py:150-237``).  The ``block`` kind adds the
    layout parameters and the two CSRs described in the module docstring.
    """

    T: int
    d: int
    kind: str                 # "geometric" | "endpoint" | "block"
    n: int                    # landmark positions [0, n)   (0 for "block")
    T_R: int                  # recent positions [n, T)
    chunk_align: int = 1

    # --- geometric --------------------------------------------------------
    q: int = 0
    dim: int = 0
    N0: int = 1
    n_dirs: int = 0
    B: int = 1
    n_planted: int = 0
    planted_cols: Optional[np.ndarray] = None

    # --- endpoint ---------------------------------------------------------
    k: int = 0

    # --- optional global channel ------------------------------------------
    n_P: int = 0

    # --- the incidence C, CSR by row --------------------------------------
    C_indptr: Optional[np.ndarray] = None       # (B+1,) int64
    C_indices: Optional[np.ndarray] = None      # (nnz,) int32
    uniform_deg: int = 0

    build_times: Dict[str, float] = field(default_factory=dict)
    warnings: List[str] = field(default_factory=list)

    # torch views, filled by to_device
    C_indptr_t: object = None
    C_indices_t: object = None
    plane_pts_t: object = None
    type_cols_t: object = None

    # --- block layout -----------------------------------------------------
    block: int = 0
    window: int = 0
    stride: int = 0
    n_sink: int = 0
    nqb: int = 0
    indptr: Optional[np.ndarray] = None         # (nqb+1,) int32
    indices: Optional[np.ndarray] = None        # (nnzb,) int32, ascending per row
    tile_kind: Optional[np.ndarray] = None      # (nnzb,) uint8
    t_indptr: Optional[np.ndarray] = None       # (nqb+1,) int32, per key block
    t_indices: Optional[np.ndarray] = None      # (nnzb,) int32, query blocks
    t_kind: Optional[np.ndarray] = None         # (nnzb,) uint8
    dev: Dict[str, object] = field(default_factory=dict)   # device -> staged tensors

    # --- pattern layout (kind="pattern") ----------------------------------
    source: str = ""                            # "geometric" | "endpoint"
    row_bits: Optional[np.ndarray] = None       # (B, row_words) uint32, C rows wrapped
    col_bits: Optional[np.ndarray] = None       # (N0, col_words) uint32, C columns wrapped
    layouts: Dict[int, object] = field(default_factory=dict)   # block -> pattern layout

    # -- derived -----------------------------------------------------------
    @property
    def n_X(self) -> int:
        return self.n - self.n_P

    @property
    def I_prof(self) -> int:
        return int(self.C_indices.size)

    @property
    def profile_degree(self) -> np.ndarray:
        return np.bincount(self.C_indices, minlength=self.N0).astype(np.int64)

    @property
    def I_tok(self) -> int:
        return int(self.profile_degree[self.prof_of_column()].sum())

    @property
    def nnzb(self) -> int:
        """Active tiles of a block layout."""
        return 0 if self.indices is None else int(self.indices.size)

    @property
    def max_row(self) -> int:
        """Longest CSR row (active key blocks of one query block)."""
        if self.indptr is None or self.nqb == 0:
            return 0
        return int(np.diff(self.indptr).max())

    @property
    def family(self) -> str:
        """The M^(d) family of the mask: "geometric" or "endpoint"."""
        return self.source if self.kind == "pattern" else self.kind

    def prof_of_column(self) -> np.ndarray:
        if self.family == "endpoint":
            return np.arange(self.n_X, dtype=np.int64)
        return np.arange(self.n_X, dtype=np.int64) % self.N0

    def row_type(self, i):
        return i % self.B

    def dense_C(self) -> np.ndarray:
        C = np.zeros((self.B, self.N0), dtype=np.int8)
        rows = np.repeat(np.arange(self.B), np.diff(self.C_indptr))
        C[rows, self.C_indices] = 1
        return C

    def summary(self) -> str:
        if self.kind == "pattern":
            kinds = np.bincount(self.tile_kind, minlength=3)
            return (f"M^({self.d}) {self.source} T={self.T} tiled by {self.block}: "
                    f"{self.nnzb} tiles ({kinds[KIND_FULL]} full, {kinds[KIND_CAUSAL]} "
                    f"causal, {kinds[KIND_PATTERN]} pattern), C {self.B}x{self.N0}")
        if self.kind == "block":
            return (f"block layout T={self.T} bs={self.block} W={self.window} "
                    f"S={self.stride} sinks={self.n_sink}: {self.nqb} query "
                    f"blocks, {self.nnzb} active tiles, max row {self.max_row}")
        if self.kind == "endpoint":
            return (f"M^({self.d}) endpoint T={self.T}: k={self.k} n={self.n} "
                    f"B={self.B} nnz(C)={self.I_prof:,}")
        return (f"M^({self.d}) T={self.T}: q={self.q} N0={self.N0} B={self.B} "
                f"deg={self.uniform_deg} n={self.n} T_R={self.T_R} "
                f"I_prof={self.I_prof:,} I_tok={self.I_tok:,}")


# ---------------------------------------------------------------------------
# M^(d) construction
# ---------------------------------------------------------------------------

def build_mask(T: int, d: int, *, chunk: int = 1, n_P: int = 0,
               B_frac: float = 1.0, max_I_prof: Optional[int] = None,
               _probe: bool = False) -> MaskSpec:
    """Build ``M^(d)`` for context length ``T`` (reference ``mask.py:244-389``).

    ``n = chunk * floor(T / 2 chunk)`` landmark positions, ``T_R = T - n``
    recent ones.  For ``2 <= d < floor(log2 T)`` the long-range block is
    ``G_ij = 1{prof(j) in H_(i mod B)}`` over affine hyperplanes of
    ``F_q^(d-1)`` with ``q = nextprime(ceil(n^(1/d)))``; ``d = 1`` is the plain
    causal mask and ``d = floor(log2 T)`` is the Boolean zeta / Walsh endpoint.
    Raises ``ValueError`` for out-of-range arguments and ``MemoryError`` when
    ``nnz(C)`` would exceed ``max_I_prof`` (checked before anything large is
    built).
    """
    if T < 8:
        raise ValueError(f"build_mask: context length T={T} is below the minimum of 8")
    d_ceiling = int(T).bit_length() - 1
    if not (1 <= d <= d_ceiling):
        raise ValueError(f"build_mask: d={d} is outside the admissible range [1, {d_ceiling}] "
                         f"(the top is floor(log2 T))")
    c = max(1, int(chunk))
    n = c * (T // (2 * c))
    if n <= 0:
        raise ValueError(f"build_mask: chunk={c} leaves no landmark positions at T={T}")
    T_R = T - n
    t0 = time.perf_counter()

    if d == d_ceiling and d >= 2:
        return _endpoint_spec(T, d, c, t0, _probe=_probe)

    if d == 1:
        spec = MaskSpec(T=T, d=1, kind="geometric", n=n, T_R=T_R, chunk_align=c,
                        q=0, dim=0, N0=1, n_dirs=0, B=1, n_planted=0,
                        planted_cols=np.zeros(0, dtype=np.int64), n_P=0,
                        C_indptr=np.array([0, 1], dtype=np.int64),
                        C_indices=np.zeros(1, dtype=np.int32), uniform_deg=1)
        spec.build_times["total"] = time.perf_counter() - t0
        return spec

    times: Dict[str, float] = {}
    warns: List[str] = []
    dim = d - 1
    # the same floating-point expression as the reference, so q agrees exactly
    q = next_prime(int(np.ceil(n ** (1.0 / d))))
    N0 = q ** dim
    if n_P < 0 or n_P >= n:
        raise ValueError(f"build_mask: n_P={n_P} global columns do not fit in [0, n={n})")
    if N0 > n - n_P:
        raise ValueError(f"build_mask: {N0} points of F_{q}^{dim} need more than the "
                         f"{n - n_P} profiled landmark columns of T={T}, d={d}")

    t = time.perf_counter()
    pts = _lex_points(q, dim)
    # a point is a normalised direction iff it is nonzero and its first
    # nonzero coordinate equals 1
    first_nz = np.full(N0, -1, dtype=np.int64)
    for k in range(dim - 1, -1, -1):
        first_nz = np.where(pts[:, k] != 0, k, first_nz)
    lead_val = np.where(first_nz >= 0,
                        pts[np.arange(N0), np.maximum(first_nz, 0)], 0)
    is_dir = (first_nz >= 0) & (lead_val == 1)
    dir_pts = np.flatnonzero(is_dir)                       # point index per direction
    n_dirs = int(dir_pts.size)
    if n_dirs != (q ** dim - 1) // (q - 1):
        raise AssertionError("normalised directions: count differs from (q^dim - 1) / (q - 1)")
    dir_of_point = np.full(N0, -1, dtype=np.int64)
    dir_of_point[dir_pts] = np.arange(n_dirs)
    n_planes_all = n_dirs * q
    times["dir_table"] = time.perf_counter() - t

    n_planted = 1 << dim
    B = max(n_planted, min(int(round(B_frac * n_planes_all)), n_planes_all))
    if T_R < 2 * B:
        msg = (f"build_mask T={T}, d={d}: only {T_R} recent rows for {B} row types, "
               f"fewer than two full passes over the types")
        if _probe:
            raise ValueError(msg)
        warns.append(msg)

    per_plane = q ** (dim - 1)
    if max_I_prof is not None and B * per_plane > max_I_prof:
        raise MemoryError(f"build_mask T={T}, d={d}: the incidence would hold "
                          f"{B * per_plane:,} entries, above max_I_prof={max_I_prof:,}")
    if _probe:
        return MaskSpec(T=T, d=d, kind="geometric", n=n, T_R=T_R, chunk_align=c,
                        q=q, dim=dim, N0=N0, n_dirs=n_dirs, B=B,
                        n_planted=n_planted, n_P=n_P, uniform_deg=per_plane)

    # hyperplane h = e*q + b is {x : <a_e, x> = b (mod q)}; its points are
    # listed in increasing point index.  A counting sort of the inner products
    # per direction yields every (e, b) list at once.
    t = time.perf_counter()
    A = pts[dir_pts]                                        # (n_dirs, dim)
    inner = (pts @ A.T) % q                                 # (N0, n_dirs)
    key = inner.T * N0 + np.arange(N0)[None, :]             # (n_dirs, N0)
    order = np.argsort(key, axis=1) % N0                    # sort by (b, point)
    planes = order.reshape(n_dirs * q, per_plane)                 # row e*q+b
    times["plane_lists"] = time.perf_counter() - t

    t = time.perf_counter()
    weights = q ** np.arange(dim - 1, -1, -1, dtype=np.int64)
    planted = []
    for a, b in planted_hyperplane_normals(d):
        e = int(dir_of_point[int((a * weights).sum())])
        if e < 0:
            raise AssertionError("a planted hyperplane normal is not among the normalised directions")
        planted.append(e * q + b)
    if len(set(planted)) != n_planted:
        raise AssertionError("two planted hyperplanes coincide")
    taken = np.zeros(n_planes_all, dtype=bool)
    taken[planted] = True
    row_order = np.concatenate([np.asarray(planted, dtype=np.int64),
                              np.flatnonzero(~taken)])[:B]
    plane_lists = planes[row_order].astype(np.int32)
    times["planted_first"] = time.perf_counter() - t

    planted_cols = np.array([n_P + q ** (dim - l) for l in range(1, dim + 1)],
                            dtype=np.int64)
    times["total"] = time.perf_counter() - t0
    return MaskSpec(T=T, d=d, kind="geometric", n=n, T_R=T_R, chunk_align=c,
                    q=q, dim=dim, N0=N0, n_dirs=n_dirs, B=B, n_planted=n_planted,
                    planted_cols=planted_cols, n_P=n_P,
                    C_indptr=np.arange(B + 1, dtype=np.int64) * per_plane,
                    C_indices=plane_lists.reshape(-1), uniform_deg=per_plane,
                    build_times=times, warnings=warns)


def _endpoint_spec(T: int, d: int, c: int, t0: float, *,
                   _probe: bool = False) -> MaskSpec:
    """``d = floor(log2 T)``: zeta landmarks, ``C[h, a] = 1{<h, a> = 0 over F_2}``
    (reference ``src/smat/mask.py:392-425``)."""
    k = d - 1
    n = 1 << k
    T_R = T - n
    B = 1 << k
    warns: List[str] = []
    if T_R < B:
        warns.append(f"build_mask T={T}: only {T_R} recent rows for {B} row types, "
                     f"less than one pass over the Walsh types")
    if _probe:
        raise NotImplementedError("build_mask: the endpoint mask has no geometric probe")
    a = np.arange(B, dtype=np.int64)
    parity = np.bitwise_count(a[:, None] & a[None, :]) & 1      # (B, B)
    keep = parity == 0
    indptr = np.concatenate([[0], np.cumsum(keep.sum(1))]).astype(np.int64)
    indices = np.nonzero(keep)[1].astype(np.int32)               # row-major order
    spec = MaskSpec(T=T, d=d, kind="endpoint", n=n, T_R=T_R, chunk_align=c,
                    q=2, dim=k, N0=n, n_dirs=B, B=B, n_planted=0,
                    planted_cols=np.array([1 << j for j in range(k)], dtype=np.int64),
                    k=k, n_P=0, C_indptr=indptr, C_indices=indices,
                    uniform_deg=0, warnings=warns)
    spec.build_times["total"] = time.perf_counter() - t0
    return spec


# ---------------------------------------------------------------------------
# block layout construction
# ---------------------------------------------------------------------------

def build_block_mask(T: int, block: int, window: int, stride: int = 0,
                     n_sink: int = 0) -> MaskSpec:
    """The block-sparse causal layout (``kind="block"``), see module docstring.

    ``T`` need not be a multiple of ``block``: the last block is ragged and
    the kernels clip it.  Raises ``ValueError`` for non-positive ``T`` or
    ``block`` and negative ``window`` / ``stride`` / ``n_sink``.
    """
    T, block = int(T), int(block)
    window, stride, n_sink = int(window), int(stride), int(n_sink)
    if T < 1:
        raise ValueError(f"T must be >= 1, got {T}")
    if block < 1:
        raise ValueError(f"block must be >= 1, got {block}")
    if window < 0 or stride < 0 or n_sink < 0:
        raise ValueError("window, stride and n_sink must be >= 0")
    t0 = time.perf_counter()
    nqb = -(-T // block)
    kb_all = np.arange(nqb, dtype=np.int64)
    summary = (kb_all % stride == stride - 1) if stride > 0 else np.zeros(nqb, bool)
    far = summary | (kb_all < n_sink)                 # active for every later qb
    far_idx = np.flatnonzero(far)

    rows = []
    for qb in range(nqb):
        lo = max(0, qb - window)
        head = far_idx[:np.searchsorted(far_idx, lo)]          # far blocks < lo
        rows.append(np.concatenate([head, np.arange(lo, qb + 1, dtype=np.int64)]))
    lens = np.fromiter((r.size for r in rows), dtype=np.int64, count=nqb)
    indptr = np.zeros(nqb + 1, dtype=np.int64)
    np.cumsum(lens, out=indptr[1:])
    indices = np.concatenate(rows) if nqb else np.zeros(0, np.int64)
    row_of = np.repeat(np.arange(nqb, dtype=np.int64), lens)
    kind = np.where(indices == row_of, KIND_CAUSAL, KIND_FULL).astype(np.uint8)

    # transposed CSR: per key block, the query blocks reading it, ascending
    order = np.lexsort((row_of, indices))
    t_indices = row_of[order]
    t_kind = kind[order]
    t_lens = np.bincount(indices, minlength=nqb)
    t_indptr = np.zeros(nqb + 1, dtype=np.int64)
    np.cumsum(t_lens, out=t_indptr[1:])

    spec = MaskSpec(T=T, d=0, kind="block", n=0, T_R=T, chunk_align=block,
                    block=block, window=window, stride=stride, n_sink=n_sink,
                    nqb=nqb,
                    indptr=indptr.astype(np.int32), indices=indices.astype(np.int32),
                    tile_kind=kind,
                    t_indptr=t_indptr.astype(np.int32),
                    t_indices=t_indices.astype(np.int32), t_kind=t_kind)
    spec.build_times["total"] = time.perf_counter() - t0
    return spec


def _csr_transpose(nqb: int, indptr: np.ndarray, indices: np.ndarray, kind: np.ndarray):
    """Per key block, the query blocks reading it (ascending) and their kinds."""
    lens = np.diff(indptr)
    row_of = np.repeat(np.arange(nqb, dtype=np.int64), lens)
    order = np.lexsort((row_of, indices))
    t_lens = np.bincount(indices, minlength=nqb)
    t_indptr = np.zeros(nqb + 1, dtype=np.int64)
    np.cumsum(t_lens, out=t_indptr[1:])
    return t_indptr.astype(np.int32), row_of[order].astype(np.int32), kind[order]


def _wrapped_bits(rows: np.ndarray, period: int, words: int) -> np.ndarray:
    """Bit table: bit t of row r is ``rows[r, t mod period]`` for ``t < 32 words``."""
    ext = rows[:, np.arange(32 * words, dtype=np.int64) % period].astype(np.uint8)
    packed = np.packbits(ext, axis=1, bitorder="little")          # (R, 4 words) bytes
    return np.ascontiguousarray(packed).view("<u4").astype(np.uint32)


def pattern_layout(spec: MaskSpec, block: int = 128) -> MaskSpec:
    """Tile layout (``kind="pattern"``) of an ``M^(d)`` spec for the softmax kernels.

    The dense mask it stands for is :func:`materialise` of ``spec`` (reference
    ``mask.py:557-577``), tile by tile: with query tile rows ``[r0, r1)``, key
    tile columns ``[c0, c1)`` and ``kb <= qb``,

    * landmark rows (``r1 <= n``): geometric tiles are full below the diagonal
      and causal on it; endpoint tiles follow ``(i & j) == j`` and are PATTERN
      (left out when empty, which for a power-of-two block is ``kb & ~qb != 0``);
    * recent rows (``r0 >= n``): the diagonal tile is causal; an off-diagonal
      tile is full unless it meets the long-range columns ``[n_P, n)`` and
      ``C`` has a 0, in which case it is PATTERN;
    * tiles whose rows straddle ``n`` are PATTERN.

    The result is cached on ``spec`` per block size.  ``spec`` keeps its own
    meaning; the layout carries copies of the fields the kernels need plus the
    two bit tables of ``C`` (``row_bits``, ``col_bits``).
    """
    if spec.kind not in ("geometric", "endpoint"):
        raise ValueError(f"pattern_layout needs an M^(d) spec, got kind={spec.kind!r}")
    block = int(block)
    if block < 1:
        raise ValueError(f"block must be >= 1, got {block}")
    cached = spec.layouts.get(block)
    if cached is not None:
        return cached
    t0 = time.perf_counter()
    T, n, n_P = spec.T, spec.n, spec.n_P
    endpoint = spec.kind == "endpoint"
    C = spec.dense_C()
    c_all = bool(C.all())
    pow2 = (block & (block - 1)) == 0
    nqb = -(-T // block)
    rows, kinds = [], []
    for qb in range(nqb):
        r0, r1 = qb * block, min(T, (qb + 1) * block)
        kb = np.arange(qb + 1, dtype=np.int64)
        if r1 <= n:
            if endpoint:
                if pow2:
                    kb = kb[(kb & ~qb) == 0]
                k = np.full(kb.size, KIND_PATTERN, np.uint8)
            else:
                k = np.where(kb == qb, KIND_CAUSAL, KIND_FULL).astype(np.uint8)
        elif r0 >= n:
            c0 = kb * block
            c1 = np.minimum(T, c0 + block)
            plain = (np.maximum(c0, n_P) >= np.minimum(c1, n)) | c_all
            k = np.where(kb == qb, KIND_CAUSAL,
                         np.where(plain, KIND_FULL, KIND_PATTERN)).astype(np.uint8)
        else:
            k = np.full(kb.size, KIND_PATTERN, np.uint8)
        rows.append(kb)
        kinds.append(k)
    lens = np.fromiter((r.size for r in rows), dtype=np.int64, count=nqb)
    indptr = np.zeros(nqb + 1, dtype=np.int64)
    np.cumsum(lens, out=indptr[1:])
    indices = np.concatenate(rows)
    kind = np.concatenate(kinds)
    t_indptr, t_indices, t_kind = _csr_transpose(nqb, indptr, indices, kind)
    row_words, col_words = (spec.N0 + 63) // 32, (spec.B + 63) // 32
    lay = MaskSpec(T=T, d=spec.d, kind="pattern", n=n, T_R=spec.T_R,
                   chunk_align=spec.chunk_align, q=spec.q, dim=spec.dim, N0=spec.N0,
                   n_dirs=spec.n_dirs, B=spec.B, n_planted=spec.n_planted,
                   planted_cols=spec.planted_cols, k=spec.k, n_P=n_P,
                   C_indptr=spec.C_indptr, C_indices=spec.C_indices,
                   uniform_deg=spec.uniform_deg,
                   block=block, nqb=nqb, indptr=indptr.astype(np.int32),
                   indices=indices.astype(np.int32), tile_kind=kind,
                   t_indptr=t_indptr, t_indices=t_indices, t_kind=t_kind,
                   source=spec.kind,
                   row_bits=_wrapped_bits(C, spec.N0, row_words),
                   col_bits=_wrapped_bits(np.ascontiguousarray(C.T), spec.B, col_words))
    lay.build_times["total"] = time.perf_counter() - t0
    spec.layouts[block] = lay
    return lay


def _md_pairs(spec: MaskSpec) -> int:
    """Ones of the dense ``M^(d)`` mask, counted without building it."""
    n, T_R, n_P = spec.n, spec.T_R, spec.n_P
    if spec.family == "endpoint":
        top = int((np.int64(1) << np.bitwise_count(np.arange(n, dtype=np.int64)).astype(np.int64)).sum())
    else:
        top = n * (n + 1) // 2
    mult = np.bincount(np.arange(T_R, dtype=np.int64) % spec.B, minlength=spec.B)
    pmult = np.bincount(spec.prof_of_column(), minlength=spec.N0)
    long_range = int(mult @ spec.dense_C().astype(np.int64) @ pmult)
    return top + T_R * (T_R + 1) // 2 + T_R * n_P + long_range


def block_layout_stats(spec: MaskSpec) -> Dict[str, int]:
    """Unmasked ``(i, j)`` pairs per head and tile counts of a block layout
    (for an ``M^(d)`` spec or its pattern layout: the ones of the dense mask
    and the tiles of :func:`pattern_layout`).

    A full tile contributes ``rows * cols`` (both clipped to ``T``); a causal
    diagonal tile of ``r`` rows contributes ``r (r + 1) / 2``.  The effective
    FLOP count of one head is ``4 D * pairs`` forward and ``3.5x`` that for
    forward plus backward.
    """
    if spec.kind in ("geometric", "endpoint", "pattern"):
        lay = pattern_layout(spec) if spec.kind != "pattern" else spec
        return {"pairs": _md_pairs(lay), "tiles": lay.nnzb, "nqb": lay.nqb,
                "max_row": lay.max_row, "causal_pairs": lay.T * (lay.T + 1) // 2,
                "pattern_tiles": int((lay.tile_kind == KIND_PATTERN).sum())}
    if spec.kind != "block":
        raise ValueError("block_layout_stats needs a block layout")
    bs, T = spec.block, spec.T
    size = np.minimum(bs, T - np.arange(spec.nqb, dtype=np.int64) * bs)
    row_of = np.repeat(np.arange(spec.nqb), np.diff(spec.indptr))
    rq = size[row_of]
    ck = size[spec.indices]
    full = spec.tile_kind == KIND_FULL
    pairs = int((rq * ck)[full].sum() + (rq * (rq + 1) // 2)[~full].sum())
    return {"pairs": pairs, "tiles": spec.nnzb, "nqb": spec.nqb,
            "max_row": spec.max_row, "causal_pairs": T * (T + 1) // 2}


# ---------------------------------------------------------------------------
# audit (M^(d))
# ---------------------------------------------------------------------------

def incidence_audit(spec: MaskSpec) -> Dict[str, object]:
    """Counting identities of the incidence ``C`` (reference ``mask.py:432-482``).

    ``nnz(C) = sum_x nu(x)``; rows list distinct profiles; for the geometric
    family every row has ``q^(d-2)`` points, every point lies on ``n_dirs``
    hyperplanes when the full family is used, and the planted hyperplanes
    satisfy ``e_i in H_R <=> i in R``.
    """
    if spec.kind == "block":
        raise ValueError("incidence_audit applies to M^(d) masks, not block layouts")
    nu = spec.profile_degree
    row_deg = np.diff(spec.C_indptr)
    step = max(1, spec.B // 32)
    distinct = all(
        np.unique(spec.C_indices[spec.C_indptr[h]:spec.C_indptr[h + 1]]).size == row_deg[h]
        for h in range(0, spec.B, step))
    out: Dict[str, object] = {
        "kind": spec.kind, "d": spec.d, "T": spec.T,
        "q": spec.q, "N0": spec.N0, "B": spec.B,
        "I_prof": spec.I_prof, "I_tok": spec.I_tok,
        "pool_gain": spec.I_tok / max(1, spec.I_prof),
        "row_deg_min": int(row_deg.min()), "row_deg_max": int(row_deg.max()),
        "col_deg_min": int(nu.min()), "col_deg_max": int(nu.max()),
        "nnz_eq_sum_nu": bool(spec.I_prof == int(nu.sum())),
        "rows_distinct_cols": bool(distinct),
    }
    if spec.kind == "geometric" and spec.d >= 2:
        q, dim = spec.q, spec.dim
        out["deg_is_q_pow_d_minus_2"] = bool(row_deg.min() == row_deg.max() == q ** (dim - 1))
        full = spec.B == spec.n_dirs * q
        out["full_hyperplane_family"] = bool(full)
        if full:
            out["nu_is_D"] = bool(nu.min() == nu.max() == spec.n_dirs)
        C = spec.dense_C()
        pcols = spec.planted_cols - spec.n_P
        ok = all(bool(C[R, pcols[l]]) == bool((R >> l) & 1)
                 for R in range(spec.n_planted) for l in range(dim))
        out["planted_identity"] = bool(ok)
        out["B_ge_2_pow_d_minus_1"] = bool(spec.B >= (1 << dim))
        out["T_R_ge_2B"] = bool(spec.T_R >= 2 * spec.B)
    if spec.kind == "endpoint":
        out["T_R_ge_B"] = bool(spec.T_R >= spec.B)
    out["exact"] = bool(out["nnz_eq_sum_nu"] and out["rows_distinct_cols"]
                        and out.get("planted_identity", True)
                        and out.get("deg_is_q_pow_d_minus_2", True))
    return out


# ---------------------------------------------------------------------------
# dense materialisation (verification only, O(T^2))
# ---------------------------------------------------------------------------

def materialise(spec: MaskSpec, dtype=np.float64) -> np.ndarray:
    """The dense ``T x T`` 0/1 mask (reference ``mask.py:557-577`` for ``M^(d)``)."""
    T = spec.T
    M = np.zeros((T, T), dtype=dtype)
    if spec.kind == "block":
        bs = spec.block
        for qb in range(spec.nqb):
            r0, r1 = qb * bs, min(T, (qb + 1) * bs)
            for e in range(spec.indptr[qb], spec.indptr[qb + 1]):
                kb = int(spec.indices[e])
                c0, c1 = kb * bs, min(T, (kb + 1) * bs)
                if spec.tile_kind[e] == KIND_CAUSAL:
                    ii = np.arange(r0, r1)[:, None]
                    jj = np.arange(c0, c1)[None, :]
                    M[r0:r1, c0:c1] = (jj <= ii).astype(dtype)
                else:
                    M[r0:r1, c0:c1] = 1
        return M

    if spec.kind == "pattern":
        # the tiles of the layout only: full / causal by kind, pattern tiles
        # copied from the source mask; everything outside them stays 0
        src = _materialise_md(spec, dtype)
        bs = spec.block
        for qb in range(spec.nqb):
            r0, r1 = qb * bs, min(T, (qb + 1) * bs)
            for e in range(spec.indptr[qb], spec.indptr[qb + 1]):
                kb = int(spec.indices[e])
                c0, c1 = kb * bs, min(T, (kb + 1) * bs)
                if spec.tile_kind[e] == KIND_FULL:
                    M[r0:r1, c0:c1] = 1
                elif spec.tile_kind[e] == KIND_CAUSAL:
                    ii = np.arange(r0, r1)[:, None]
                    jj = np.arange(c0, c1)[None, :]
                    M[r0:r1, c0:c1] = (jj <= ii).astype(dtype)
                else:
                    M[r0:r1, c0:c1] = src[r0:r1, c0:c1]
        return M
    return _materialise_md(spec, dtype)


def _materialise_md(spec: MaskSpec, dtype) -> np.ndarray:
    T = spec.T
    M = np.zeros((T, T), dtype=dtype)
    n, T_R = spec.n, spec.T_R
    if spec.family == "endpoint":
        a = np.arange(n, dtype=np.int64)
        M[:n, :n] = ((a[:, None] & a[None, :]) == a[None, :]).astype(dtype)
    else:
        M[:n, :n] = np.tril(np.ones((n, n), dtype=dtype))
    M[n:, n:] = np.tril(np.ones((T_R, T_R), dtype=dtype))
    if spec.n_P:
        M[n:, :spec.n_P] = 1
    C = spec.dense_C()
    rho = np.arange(T_R, dtype=np.int64) % spec.B
    M[n:, spec.n_P:n] = C[np.ix_(rho, spec.prof_of_column())].astype(dtype)
    return M


def estimate_cost(T: int, d: int, r: int, d_v: int, *, chunk: int = 128,
                  n_P: int = 0) -> Dict[str, float]:
    """MACs and bytes of the reference's kernel-attention schedule for
    ``M^(d)``, predicted without building the incidence
    (reference ``mask.py:584-614``)."""
    try:
        s = build_mask(T, d, chunk=chunk, n_P=n_P, _probe=True)
    except NotImplementedError:
        s = None
    except ValueError as e:
        return {"feasible": False, "reason": str(e)}
    p = d_v + 1
    if s is None:
        k = d - 1
        B = N0 = 1 << k
        I_prof = B * (1 << max(0, k - 1))
        q = 2
    else:
        B, N0, q = s.B, s.N0, s.q
        I_prof = B * (s.uniform_deg if d >= 2 else 1)
    macs = 2 * T * r * d_v + T * chunk * (r + p) + 3 * T * r * p + I_prof * r * p
    return {"feasible": True, "q": q, "B": B, "N0": N0, "I_prof": I_prof,
            "macs": float(macs), "table_bytes_fp32": 4.0 * (B + N0) * r * p,
            "dense_mask_bytes_fp32": 4.0 * T * T,
            "flash_macs": float(T) * T * (r + d_v)}


# ---------------------------------------------------------------------------
# device staging
# ---------------------------------------------------------------------------

def to_device(spec: MaskSpec, device, *, want_direct: bool = False) -> MaskSpec:
    """Stage the spec's index arrays on ``device`` as torch tensors.

    ``M^(d)`` kinds get the reference's views (``attention.py:542-555``):
    ``C_indptr_t`` / ``C_indices_t`` (int64) and ``plane_pts_t``.  A block or
    pattern layout gets its int32 CSR, kinds and transposed CSR (and, for a
    pattern layout, the two bit tables of ``C``) in ``spec.dev[device]`` (the
    arrays the CUDA kernels read), cached per device.
    """
    import torch

    if spec.kind in ("block", "pattern"):
        key = str(torch.device(device))
        if key not in spec.dev:
            as_t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
            d = {
                "indptr": as_t(spec.indptr), "indices": as_t(spec.indices),
                "kind": as_t(spec.tile_kind), "t_indptr": as_t(spec.t_indptr),
                "t_indices": as_t(spec.t_indices), "t_kind": as_t(spec.t_kind),
            }
            if spec.kind == "pattern":
                d["row_bits"] = as_t(spec.row_bits.view(np.int32))
                d["col_bits"] = as_t(spec.col_bits.view(np.int32))
            spec.dev[key] = d
        return spec

    spec.C_indptr_t = torch.from_numpy(spec.C_indptr).to(device)
    spec.C_indices_t = torch.from_numpy(spec.C_indices.astype(np.int64)).to(device)
    spec.plane_pts_t = (spec.C_indices_t.view(spec.B, spec.uniform_deg)
                        if spec.uniform_deg else None)
    if want_direct:
        if not spec.uniform_deg:
            raise ValueError("the direct table needs a uniform row degree")
        n_X, N0 = spec.n_X, spec.N0
        g = -(-n_X // N0)
        pts = spec.C_indices.reshape(spec.B, -1).astype(np.int64)
        base = pts[:, :, None] + np.arange(g, dtype=np.int64)[None, None, :] * N0
        cols = np.where(base < n_X, base, n_X).reshape(spec.B, -1).astype(np.int32)
        spec.type_cols_t = torch.from_numpy(cols).to(device)
    return spec
