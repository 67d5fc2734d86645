// Row-balanced ("merge-path") schedule for segmented sum and max.
//
// The work of a call is the merge of two sorted lists: the N rows and the B
// segment ends (segment k ends after row offsets[k+1]-1).  Walking the merge
// consumes a row (fold it into the current segment) or an end (finalise the
// current segment).  The path has N + B items; it is cut into equal pieces,
// one per "unit", so every unit does the same amount of work whatever the
// length distribution -- one 50M-row segment or millions of empty ones.
// (Merge-path partitioning: Odeh, Green, Mwassi, Shmueli, Birk, "Merge
// Path - Parallel Merging Made Simple", IPDPSW 2012; applied to CSR rows by
// Merrill and Garland, "Merge-based parallel sparse matrix-vector
// multiplication", SC 2016.)
//
// A unit is a group of G lanes that together cover one row tile (G * VEC
// features); a warp holds 32 / G units, a CTA NW warps.  Each unit streams
// its own contiguous rows (one 16-byte vector per lane per row), so every
// segment that starts and ends inside a unit is reduced entirely in that
// unit's registers and stored directly -- no shuffles or shared memory on
// the common path.  A segment cut by a unit boundary leaves f32 pieces in
// shared memory: the unit where it starts a TAIL piece, units it covers
// completely THROUGH pieces and the unit that consumes its end a HEAD
// piece.  At the end the CTA merges its units' pieces in row order,
// finishing every segment cut only inside the CTA, and leaves at most one
// HEAD and one TAIL/THROUGH piece per CTA in global memory.  The fix-up
// kernel merges each segment cut by CTA boundaries in row order and writes
// its output once (one rounding to the output dtype), so results are
// deterministic.
#pragma once

#include "common.cuh"

namespace rgb {

constexpr int kRowbalThreads = 256;
constexpr int kRowbalSmem = 0;  // dynamic shared memory per CTA

// Streaming knobs, chosen by measurement on B200 (c1, c5):
// U rows per register batch, DB = keep a second batch in flight while
// folding, MINB = minimum resident CTAs per SM requested from ptxas.
struct RowbalTuning {
  static constexpr int kUnroll = 4;
  static constexpr bool kDoubleBuffer = false;
  static constexpr int kMinBlocks = 3;
};
constexpr int kSumBlock = 8;  // rows summed plainly before a compensated add

// Piece slot kinds in the unit metadata.
enum : int32_t { PIECE_NONE = 0, PIECE_TAIL = 1, PIECE_THROUGH = 2 };

struct UnitMeta {
  int64_t head_seg;  // segment whose end this unit consumed but that started earlier; -1 if none
  int64_t tail_seg;  // segment open at this unit's end; -1 if none
  int32_t tail_kind; // PIECE_TAIL (started in this unit) or PIECE_THROUGH
  int32_t pad;
};

// Accumulator of one lane for the row-balanced sum: blocks of kSumBlock
// rows are summed plainly, each block total is added with compensation.
template <int OP, int VEC>
struct RowAcc;

template <int VEC>
struct RowAcc<OP_SUM, VEC> {
  static constexpr int kWidth = 2;  // floats per feature in a piece (s, c)
  float s[VEC], c[VEC], p[VEC];
  int count;
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int v = 0; v < VEC; ++v) { s[v] = 0.0f; c[v] = 0.0f; p[v] = 0.0f; }
    count = 0;
  }
  __device__ __forceinline__ void fold(const float (&x)[VEC]) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) p[v] = __fadd_rn(p[v], x[v]);
    if (++count == kSumBlock) {
#pragma unroll
      for (int v = 0; v < VEC; ++v) { kahan_add(s[v], c[v], p[v]); p[v] = 0.0f; }
      count = 0;
    }
  }
  __device__ __forceinline__ void settle() {
#pragma unroll
    for (int v = 0; v < VEC; ++v) { kahan_add(s[v], c[v], p[v]); p[v] = 0.0f; }
    count = 0;
  }
  // Runs of rows: fold_raw adds a row to the plain block without counting
  // it; account(rows) counts the run and closes the block once it holds
  // kSumBlock rows or more.
  __device__ __forceinline__ void fold_raw(const float (&x)[VEC]) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) p[v] = __fadd_rn(p[v], x[v]);
  }
  __device__ __forceinline__ void account(int rows) {
    count += rows;
    if (count >= kSumBlock) settle();
  }
  __device__ __forceinline__ void value(float (&y)[VEC]) {
    settle();
#pragma unroll
    for (int v = 0; v < VEC; ++v) y[v] = kahan_value(s[v], c[v]);
  }
  // Piece storage: s then c, each VEC floats, at piece + 0 and piece + stride.
  __device__ __forceinline__ void store_piece(float *piece, int64_t stride) {
    settle();
#pragma unroll
    for (int v = 0; v < VEC; ++v) { piece[v] = s[v]; piece[stride + v] = c[v]; }
  }
  __device__ __forceinline__ void load_piece(const float *piece, int64_t stride) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) { s[v] = piece[v]; c[v] = piece[stride + v]; p[v] = 0.0f; }
    count = 0;
  }
  __device__ __forceinline__ void merge_piece(const float *piece, int64_t stride) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) kahan_merge(s[v], c[v], piece[v], piece[stride + v]);
  }
  // Warp scans over settled accumulators: the value of lane - delta, and
  // this = this (earlier rows) + later.
  __device__ __forceinline__ RowAcc shfl_up(int delta) const {
    RowAcc r;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      r.s[v] = __shfl_up_sync(0xffffffffu, s[v], delta);
      r.c[v] = __shfl_up_sync(0xffffffffu, c[v], delta);
      r.p[v] = 0.0f;
    }
    r.count = 0;
    return r;
  }
  __device__ __forceinline__ void merge(const RowAcc &later) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) kahan_merge(s[v], c[v], later.s[v], later.c[v]);
  }
};

template <int VEC>
struct RowAcc<OP_MAX, VEC> {
  static constexpr int kWidth = 1;
  float m[VEC];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int v = 0; v < VEC; ++v) m[v] = -kInf;
  }
  __device__ __forceinline__ void fold(const float (&x)[VEC]) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) m[v] = max_nan(m[v], x[v]);
  }
  __device__ __forceinline__ void fold_raw(const float (&x)[VEC]) { fold(x); }
  __device__ __forceinline__ void account(int) {}
  __device__ __forceinline__ void value(float (&y)[VEC]) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) y[v] = m[v];
  }
  __device__ __forceinline__ void store_piece(float *piece, int64_t) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) piece[v] = m[v];
  }
  __device__ __forceinline__ void load_piece(const float *piece, int64_t) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) m[v] = piece[v];
  }
  __device__ __forceinline__ void merge_piece(const float *piece, int64_t) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) m[v] = max_nan(m[v], piece[v]);
  }
  __device__ __forceinline__ RowAcc shfl_up(int delta) const {
    RowAcc r;
#pragma unroll
    for (int v = 0; v < VEC; ++v) r.m[v] = __shfl_up_sync(0xffffffffu, m[v], delta);
    return r;
  }
  __device__ __forceinline__ void merge(const RowAcc &later) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) m[v] = max_nan(m[v], later.m[v]);
  }
};

// Softmax statistics pass: per feature the online statistics of
// common.cuh (lagging reference, compensated mass).  A piece is (reference,
// total mass); a finished segment's statistics go to the f32 statistics
// buffer (emit), which the normalise pass reads.
template <int VEC>
struct RowAcc<OP_SOFTMAX, VEC> {
  static constexpr int kWidth = 2;
  Stats st[VEC];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int v = 0; v < VEC; ++v) st[v] = stats_empty();
  }
  __device__ __forceinline__ void fold(const float (&x)[VEC]) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const float one[1] = {x[v]};
      stats_fold<1>(st[v], one);
    }
  }
  template <int U>
  __device__ __forceinline__ void fold_batch(const float (&x)[U][VEC]) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      float col[U];
#pragma unroll
      for (int u = 0; u < U; ++u) col[u] = x[u][v];
      stats_fold<U>(st[v], col);
    }
  }
  __device__ __forceinline__ void store_piece(float *piece, int64_t stride) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      piece[v] = st[v].r;
      piece[stride + v] = kahan_value(st[v].s, st[v].c);
    }
  }
  __device__ __forceinline__ void load_piece(const float *piece, int64_t stride) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) st[v] = Stats{piece[v], piece[stride + v], 0.0f};
  }
  __device__ __forceinline__ void merge_piece(const float *piece, int64_t stride) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) stats_merge(st[v], Stats{piece[v], piece[stride + v], 0.0f});
  }
};

// A finished segment: sum and max round once to the output dtype; softmax
// statistics go to the f32 statistics buffer [B][2][D] passed as `out`.
template <typename T, int OP, int VEC>
__device__ __forceinline__ void emit(RowAcc<OP, VEC> &acc, T *out, int64_t seg, int64_t d, int64_t col) {
  if constexpr (OP == OP_SOFTMAX) {
    acc.store_piece(reinterpret_cast<float *>(out) + seg * 2 * d + col, d);
  } else {
    float y[VEC];
    acc.value(y);
    VecIO<T, VEC>::store(out + seg * d + col, y);
  }
}

template <typename OffT>
__device__ __forceinline__ int64_t load_offset(const OffT *offsets, int64_t i) {
  return static_cast<int64_t>(__ldg(offsets + i));
}

// Merge-path coordinate: the number of segment ends consumed before
// diagonal `diag`, i.e. the first k in [0, B] with offsets[k+1] + k >= diag.
// All G lanes of a group search together (G-ary search, G probes per step);
// every lane of the group returns the same answer.
template <typename OffT>
__device__ int64_t path_search(const OffT *offsets, int64_t b, int64_t diag, int g, int gl,
                               unsigned group_mask, int group_base) {
  int64_t lo = 0, hi = b;  // answer in [lo, hi]; k = b means "all ends"
  while (hi - lo > 0) {
    const int64_t span = hi - lo;
    const int64_t step = (span + g) / (g + 1) > 0 ? (span + g) / (g + 1) : 1;
    // probe k = lo + (gl + 1) * step - 1, clamped below hi
    int64_t k = lo + static_cast<int64_t>(gl + 1) * step - 1;
    const bool valid = k < hi;
    bool pred = false;
    if (valid) pred = load_offset(offsets, k + 1) + k >= diag;
    const unsigned ballot = __ballot_sync(group_mask, valid && pred) >> group_base;
    const unsigned valid_bits = __ballot_sync(group_mask, valid) >> group_base;
    if (ballot) {
      const int first = __ffs(ballot) - 1;
      hi = lo + static_cast<int64_t>(first + 1) * step - 1;
      lo = lo + static_cast<int64_t>(first) * step;
    } else {
      const int last = 31 - __clz(valid_bits);
      lo = lo + static_cast<int64_t>(last + 1) * step;
    }
    if (lo > hi) lo = hi;
  }
  return lo;
}

// Whether segment `seg` has a slot in [seg0, seg1) (seg1 == 0: every one).
__device__ __forceinline__ bool has_slot(int64_t seg, int64_t seg0, int64_t seg1) {
  return seg1 == 0 || (seg >= seg0 && seg < seg1);
}

// Combine `count` consecutive units' pieces in row order, for one column
// lane.  piece(k, slot) points at unit k's slot (0 = HEAD, 1 = TAIL or
// THROUGH) for this lane, `pstride` floats between its s and c halves.  A
// segment whose pieces all lie among these units is finished and stored to
// out (when `active`); the remaining HEAD and TAIL / THROUGH pieces go to
// head_dst / tail_dst (`dstride` between halves) and, if `m` is not null,
// their segments and kind to *m.
template <typename T, int OP, int VEC, typename PieceFn>
__device__ __forceinline__ void combine_pieces(int count, PieceFn piece, int pstride, const int64_t *heads,
                                               const int64_t *tails, const int32_t *kinds, bool active, T *out,
                                               int64_t d, int64_t col, float *head_dst, float *tail_dst,
                                               int64_t dstride, UnitMeta *m, int64_t seg0, int64_t seg1) {
  using Acc = RowAcc<OP, VEC>;
  Acc carry;
  carry.init();
  bool have = false, here = false;
  int64_t carry_seg = -1, head_seg = -1;
  for (int k = 0; k < count; ++k) {
    const int64_t h = heads[k];
    if (h >= 0) {
      if (have && carry_seg == h) {
        carry.merge_piece(piece(k, 0), pstride);
      } else {
        carry.load_piece(piece(k, 0), pstride);
        here = false;
      }
      if (here) {
        if (active && has_slot(h, seg0, seg1)) emit<T, OP, VEC>(carry, out, h - seg0, d, col);
      } else {
        if (active) carry.store_piece(head_dst, dstride);
        head_seg = h;
      }
      have = false;
    }
    const int kind = kinds[k];
    if (kind == PIECE_TAIL) {
      carry.load_piece(piece(k, 1), pstride);
      have = true;
      here = true;
      carry_seg = tails[k];
    } else if (kind == PIECE_THROUGH) {
      if (have && carry_seg == tails[k]) {
        carry.merge_piece(piece(k, 1), pstride);
      } else {
        carry.load_piece(piece(k, 1), pstride);
        have = true;
        here = false;
        carry_seg = tails[k];
      }
    }
  }
  if (have && active) carry.store_piece(tail_dst, dstride);
  if (m) {
    m->head_seg = head_seg;
    m->tail_seg = have ? carry_seg : -1;
    m->tail_kind = have ? (here ? PIECE_TAIL : PIECE_THROUGH) : PIECE_NONE;
  }
}

// Rows of the whole array that one launch covers.  A single-GPU call covers
// [0, N); a rank of a sharded call covers its own rows [row0, row1), with
// values[0] holding row row0 (see shard.cu).
struct RowWindow {
  int64_t row0, row1;
  int first;     // the first window: it also consumes the segment ends at row 0
  int64_t seg0;  // softmax statistics: segment seg is written at slot seg - seg0 (0: all segments)
  int64_t seg1;  // ... for seg0 <= seg < seg1 only (0: no bound)
};

// Segment ends at or before row `row`: the first k in [0, B] with
// offsets[k+1] > row (G-ary search by the G lanes of a group; every lane
// returns the same answer).
template <typename OffT>
__device__ int64_t ends_upto(const OffT *offsets, int64_t b, int64_t row, int g, int gl, unsigned group_mask,
                             int group_base) {
  int64_t lo = 0, hi = b;
  while (hi - lo > 0) {
    const int64_t span = hi - lo;
    const int64_t step = (span + g) / (g + 1) > 0 ? (span + g) / (g + 1) : 1;
    const int64_t k = lo + static_cast<int64_t>(gl + 1) * step - 1;
    const bool valid = k < hi;
    const bool pred = valid && load_offset(offsets, k + 1) > row;
    const unsigned ballot = __ballot_sync(group_mask, pred) >> group_base;
    const unsigned valid_bits = __ballot_sync(group_mask, valid) >> group_base;
    if (ballot) {
      const int first = __ffs(ballot) - 1;
      hi = lo + static_cast<int64_t>(first + 1) * step - 1;
      lo = lo + static_cast<int64_t>(first) * step;
    } else {
      const int last = 31 - __clz(valid_bits);
      lo = lo + static_cast<int64_t>(last + 1) * step;
    }
    if (lo > hi) lo = hi;
  }
  return lo;
}

// Merge-path diagonal after row `row` - 1 and every segment end at or
// before `row`: where a window starting or ending at `row` is cut.  The
// first window starts at diagonal 0 instead (it also consumes the ends at
// row 0: empty segments at the start, or every segment when N = 0).
template <typename OffT>
__device__ __forceinline__ int64_t window_diag(const OffT *offsets, int64_t n, int64_t b, int64_t row, int g,
                                               int gl, unsigned group_mask, int group_base) {
  if (row >= n) return n + b;
  return row + ends_upto(offsets, b, row, g, gl, group_mask, group_base);
}

// XF (softmax statistics, one GPU): the input transform `xf` (scale,
// additive mask) applied to every row as it is loaded.
template <typename T, typename OffT, int OP, int VEC, int U = RowbalTuning::kUnroll,
          bool DB = RowbalTuning::kDoubleBuffer, int MINB = RowbalTuning::kMinBlocks, bool XF = false>
__global__ void __launch_bounds__(kRowbalThreads, MINB)
rowbal_kernel(const T *__restrict__ values, const OffT *__restrict__ offsets, T *__restrict__ out,
              int64_t n, int64_t b, int64_t d, int g_shift, int vec_cols, int64_t units,
              float *__restrict__ pieces, UnitMeta *__restrict__ meta, RowWindow window,
              unsigned long long *__restrict__ work, Xform xf = Xform{}) {
  using Acc = RowAcc<OP, VEC>;
  const int lane = threadIdx.x & 31;
  const int G = 1 << g_shift;
  const int q = lane >> g_shift;          // unit within the warp
  const int gl = lane & (G - 1);          // lane within the unit
  const int group_base = q << g_shift;
  const unsigned group_mask = (G == 32) ? 0xffffffffu : (((1u << G) - 1u) << group_base);
  const int units_per_cta = (kRowbalThreads / 32) << (5 - g_shift);
  const int unit_in_cta = (threadIdx.x >> 5) * (32 >> g_shift) + q;
  const int64_t vctas = units / units_per_cta;  // virtual CTAs of the launch
  const int tiles = gridDim.y;
  const int64_t d_lo = window.first ? 0 : window_diag(offsets, n, b, window.row0, G, gl, group_mask, group_base);
  const int64_t d_hi = window_diag(offsets, n, b, window.row1, G, gl, group_mask, group_base);
  const int64_t path = d_hi - d_lo;
  __shared__ int64_t s_claim;

  // Virtual CTAs: with `work`, the resident CTAs take them from a counter
  // (several per CTA, so CTAs that run slower -- the far die, a busier
  // memory channel -- take fewer and the kernel does not wait on the
  // slowest of one static wave); without it, virtual CTA = blockIdx.x.
  for (int64_t claim = blockIdx.x * tiles + blockIdx.y;;) {
    if (work) {
      if (threadIdx.x == 0) s_claim = static_cast<int64_t>(atomicAdd(work, 1ull));
      __syncthreads();
      claim = s_claim;
      __syncthreads();
    }
    if (claim >= vctas * tiles) break;
    const int64_t vcta = claim / tiles;
    const int tile = static_cast<int>(claim % tiles);
  const int64_t unit = vcta * units_per_cta + unit_in_cta;  // < units by construction
  const int cv = tile * 32 + gl;
  const bool active = cv < vec_cols;
  const int64_t col = static_cast<int64_t>(cv) * VEC;

  // This unit's slice of the merge path.
  const int64_t d0 = d_lo + path / units * unit + min(unit, path % units);
  const int64_t d1 = d0 + path / units + (unit < path % units ? 1 : 0);
  const int64_t i0 = path_search(offsets, b, d0, G, gl, group_mask, group_base);
  const int64_t i1 = path_search(offsets, b, d1, G, gl, group_mask, group_base);
  const int64_t j0 = d0 - i0, j1 = d1 - i1;  // rows [j0, j1)

  // Window of G segment ends: lane gl holds offsets[wbase + gl].
  int64_t seg = i0;
  int64_t wbase = seg + 1;
  int64_t win = (wbase + gl <= b) ? load_offset(offsets, wbase + gl) : INT64_MAX;
  auto end_of = [&](int64_t s) -> int64_t {  // offsets[s + 1], s < b
    if (s + 1 - wbase >= G) {
      wbase = s + 1;
      win = (wbase + gl <= b) ? load_offset(offsets, wbase + gl) : INT64_MAX;
    }
    return __shfl_sync(group_mask, win, static_cast<int>(s + 1 - wbase), G);
  };
  int64_t next_b = seg < b ? end_of(seg) : INT64_MAX;
  bool first = true;
  const bool first_started_here = seg < b ? load_offset(offsets, seg) >= j0 : true;

  // Unit pieces stay in shared memory: slot 0 = HEAD, slot 1 = TAIL or
  // THROUGH, VEC * kWidth floats per lane; the unit's metadata beside them.
  constexpr int W = Acc::kWidth;
  __shared__ float s_piece[2][kRowbalThreads * VEC * W];
  __shared__ int64_t s_head[kRowbalThreads], s_tail[kRowbalThreads];
  __shared__ int32_t s_kind[kRowbalThreads];
  float *const my_head = &s_piece[0][threadIdx.x * VEC * W];
  float *const my_tail = &s_piece[1][threadIdx.x * VEC * W];
  Acc acc;
  acc.init();

  // Finalise `seg` (its end is consumed by this unit).
  auto finish = [&]() {
    if (first && !first_started_here) {
      acc.store_piece(my_head, VEC);
      if (gl == 0) s_head[unit_in_cta] = seg;
    } else if (active && has_slot(seg, window.seg0, window.seg1)) {
      emit<T, OP, VEC>(acc, out, seg - window.seg0, d, col);
    }
    first = false;
    acc.init();
    ++seg;
    next_b = seg < b ? end_of(seg) : INT64_MAX;
  };

  if (gl == 0) {
    s_head[unit_in_cta] = -1;
    s_tail[unit_in_cta] = -1;
    s_kind[unit_in_cta] = PIECE_NONE;
  }

  // Register batches of U rows.  With DB a second batch is in flight while
  // one is folded, so a warp always has loads pending.  A batch without a
  // segment boundary takes the fast path (no per-row boundary test).
  using Raw = typename VecIO<T, VEC>::Raw;
  const T *ptr = values + (j0 - window.row0) * d + col;
  MaskVec<VEC> mk[U];  // XF: the mask vectors of the batch's rows
  auto load_batch = [&](Raw (&raw)[U], int64_t rel) {  // rows j0 + rel .. + U
#pragma unroll
    for (int t = 0; t < U; ++t)
      if (active && j0 + rel + t < j1) {
        raw[t] = VecIO<T, VEC>::load_raw(ptr + (rel + t) * d);
        if constexpr (XF) {
          if (xf.mask) mk[t] = load_mask<VEC>(xf, j0 + rel + t, col);
        }
      }
  };
  auto unpack_row = [&](const Raw &raw, int t, float (&x)[VEC]) {
    VecIO<T, VEC>::unpack(raw, x);
    if constexpr (XF) apply_xform<VEC>(x, xf, mk[t]);
  };
  auto fold_batch = [&](const Raw (&raw)[U], int64_t r) {
    if (r + U <= j1 && next_b >= r + U) {
      if constexpr (OP == OP_SOFTMAX) {
        float x[U][VEC];
#pragma unroll
        for (int t = 0; t < U; ++t) unpack_row(raw[t], t, x[t]);
        acc.template fold_batch<U>(x);  // one recentring test per batch and feature
      } else {
#pragma unroll
        for (int t = 0; t < U; ++t) {
          float x[VEC];
          VecIO<T, VEC>::unpack(raw[t], x);
          acc.fold(x);
        }
      }
    } else if constexpr (OP == OP_SOFTMAX) {
      // A segment boundary inside the batch: fold each segment's rows as a
      // whole batch with the other rows at -inf (they add no mass and do
      // not move the reference), so the online statistics take one
      // recentring test per piece instead of one per row.
      float x[U][VEC];
#pragma unroll
      for (int t = 0; t < U; ++t) unpack_row(raw[t], t, x[t]);
      int t0 = 0;
      const int tn = j1 - r < U ? static_cast<int>(j1 - r) : U;
      while (t0 < tn) {
        while (next_b <= r + t0) finish();  // segments ending before this row (incl. empty ones)
        const int64_t stop = next_b - r;
        const int t1 = stop < tn ? static_cast<int>(stop) : tn;
        float xm[U][VEC];
#pragma unroll
        for (int t = 0; t < U; ++t)
#pragma unroll
          for (int v = 0; v < VEC; ++v) xm[t][v] = (t >= t0 && t < t1) ? x[t][v] : -kInf;
        acc.template fold_batch<U>(xm);
        t0 = t1;
      }
    } else {
#pragma unroll
      for (int t = 0; t < U; ++t) {
        if (r + t < j1) {
          while (next_b <= r + t) finish();  // segments ending before this row (incl. empty ones)
          float x[VEC];
          VecIO<T, VEC>::unpack(raw[t], x);
          acc.fold(x);
        }
      }
    }
  };
  static_assert(!(XF && DB), "the fused transform keeps one batch of mask vectors");
  if constexpr (DB) {
    Raw ra[U], rb[U];
    load_batch(ra, 0);
    load_batch(rb, U);
    for (int64_t rel = 0; j0 + rel < j1; rel += 2 * U) {
      fold_batch(ra, j0 + rel);
      load_batch(ra, rel + 2 * U);
      if (j0 + rel + U >= j1) break;
      fold_batch(rb, j0 + rel + U);
      load_batch(rb, rel + 3 * U);
    }
  } else {
    for (int64_t rel = 0; j0 + rel < j1; rel += U) {
      Raw ra[U];
      load_batch(ra, rel);
      fold_batch(ra, j0 + rel);
    }
  }
  while (seg < i1) finish();  // ends consumed after the last row
  // Segment open at the end of this unit, if the unit holds rows of it:
  // a THROUGH piece when it also started before the unit, else a TAIL.
  if (seg < b) {
    const int64_t start = load_offset(offsets, seg);
    if ((start > j0 ? start : j0) < j1) {
      acc.store_piece(my_tail, VEC);
      if (gl == 0) {
        s_tail[unit_in_cta] = seg;
        s_kind[unit_in_cta] = start < j0 ? PIECE_THROUGH : PIECE_TAIL;
      }
    }
  }
  __syncthreads();

  // Combine the CTA's unit pieces in row order (one thread per column lane):
  // a segment whose TAIL, THROUGH and HEAD pieces all lie in this CTA is
  // finished here; what remains is at most one CTA-level HEAD (a segment
  // open at the CTA's start that ends in it) and one TAIL / THROUGH (open
  // at its end), written to global memory for the fix-up.  With several
  // units per warp (rows narrower than 32 vectors) the merge is two-level:
  // each warp merges its own units (their pieces are its lanes' registers
  // stored in shared memory, so a __syncwarp orders them), leaving its
  // HEAD and TAIL / THROUGH in its first unit's slots, then the warps'
  // pieces merge across the CTA -- 32 / G + 8 dependent merges per column
  // instead of 256 / G.
  constexpr int NW = kRowbalThreads / 32;
  __shared__ int64_t w_head[NW], w_tail[NW];
  __shared__ int32_t w_kind[NW];
  const int upw = 32 >> g_shift;  // units per warp
  const int c_cv_base = tile * 32;
  if (upw == 1) {
    if (threadIdx.x < G) {
      const int c_lane = threadIdx.x;
      const int c_cv = c_cv_base + c_lane;
      float *const cta_pieces = pieces + vcta * 2 * W * d;
      const int64_t c_col = static_cast<int64_t>(c_cv) * VEC;
      auto piece = [&](int k, int slot) { return &s_piece[slot][((k << g_shift) + c_lane) * VEC * W]; };
      combine_pieces<T, OP, VEC>(units_per_cta, piece, VEC, s_head, s_tail, s_kind, c_cv < vec_cols, out, d, c_col,
                                 cta_pieces + c_col, cta_pieces + W * d + c_col, d,
                                 tile == 0 && c_lane == 0 ? &meta[vcta] : nullptr, window.seg0, window.seg1);
    }
  } else {
    const int warp = threadIdx.x >> 5;
    if (q == 0) {  // level 1: lanes gl of the warp's first unit
      const int c_cv = c_cv_base + gl;
      const int64_t c_col = static_cast<int64_t>(c_cv) * VEC;
      const int first_unit = warp * upw;
      auto piece = [&](int k, int slot) {
        return &s_piece[slot][(((first_unit + k) << g_shift) + gl) * VEC * W];
      };
      UnitMeta m;
      combine_pieces<T, OP, VEC>(upw, piece, VEC, s_head + first_unit, s_tail + first_unit, s_kind + first_unit,
                                 c_cv < vec_cols, out, d, c_col, piece(0, 0), piece(0, 1), VEC,
                                 gl == 0 ? &m : nullptr, window.seg0, window.seg1);
      if (gl == 0) {
        w_head[warp] = m.head_seg;
        w_tail[warp] = m.tail_seg;
        w_kind[warp] = m.tail_kind;
      }
    }
    __syncthreads();
    if (threadIdx.x < G) {  // level 2: the warps' pieces, in warp order
      const int c_lane = threadIdx.x;
      const int c_cv = c_cv_base + c_lane;
      float *const cta_pieces = pieces + vcta * 2 * W * d;
      const int64_t c_col = static_cast<int64_t>(c_cv) * VEC;
      auto piece = [&](int k, int slot) { return &s_piece[slot][(((k * upw) << g_shift) + c_lane) * VEC * W]; };
      combine_pieces<T, OP, VEC>(NW, piece, VEC, w_head, w_tail, w_kind, c_cv < vec_cols, out, d, c_col,
                                 cta_pieces + c_col, cta_pieces + W * d + c_col, d,
                                 tile == 0 && c_lane == 0 ? &meta[vcta] : nullptr, window.seg0, window.seg1);
    }
  }
    if (!work) break;
    __syncthreads();  // the combine is done with the shared pieces before the next virtual CTA
  }
}

// Narrow rows (D * sizeof(T) in {2, 4, 8, 16} bytes): every lane is a unit and
// folds 16-byte packets of R = 16 / (D * sizeof(T)) whole rows, a packet at
// once when no segment boundary falls inside it.  A warp finds its slice of
// the merge path with a 32-ary search; each lane then finds its own slice by
// binary search inside the warp's segment range.  The next four segment
// ends sit in a register window that is refilled one entry per finished
// segment, so short segments do not wait on offsets loads.
//
// A lane's rows are contiguous but far from its neighbours', so a warp load
// of one packet per lane would touch 32 lines.  Instead the warp stages its
// lanes' next kPackedRun packets (128 bytes each) into shared memory with
// cp.async, each instruction copying the runs of 32 / kPackedRun lanes
// (whole 128-byte runs, 4 lines per instruction), two rounds in flight
// while the lanes fold the previous one from shared memory.  A lane's run
// occupies kPackedRun + 1 slots, so the eight lanes of a 16-byte shared
// load phase read eight different bank groups.
//
// Pieces are combined per warp (lane 0 over 32 units) and then per CTA
// (thread 0 over the 8 warps), leaving one HEAD and one TAIL / THROUGH per
// CTA for the fix-up kernel.
constexpr int kPackedRun = 8;     // packets per lane per staged round
constexpr int kPackedStages = 2;  // rounds in flight per warp
constexpr int kPackedStageBytes =
    (kRowbalThreads / 32) * kPackedStages * 32 * (kPackedRun + 1) * 16;  // dynamic shared memory per CTA
static_assert(32 % kPackedRun == 0, "a staging instruction copies whole runs of 32 / kPackedRun lanes");

// First k in [lo, hi] with offsets[k+1] + k >= diag, for one thread.
template <typename OffT>
__device__ __forceinline__ int64_t path_search_range(const OffT *offsets, int64_t lo, int64_t hi, int64_t diag) {
  while (lo < hi) {
    const int64_t mid = lo + (hi - lo) / 2;
    if (load_offset(offsets, mid + 1) + mid >= diag) hi = mid; else lo = mid + 1;
  }
  return lo;
}

template <typename T, typename OffT, int OP, int DS, int U = 4, int MINB = 2>
__global__ void __launch_bounds__(kRowbalThreads, MINB)
rowbal_packed_kernel(const T *__restrict__ values, const OffT *__restrict__ offsets, T *__restrict__ out,
                     int64_t n, int64_t b, int64_t units, float *__restrict__ pieces, UnitMeta *__restrict__ meta) {
  using Acc = RowAcc<OP, DS>;
  constexpr int W = Acc::kWidth;
  constexpr int R = 16 / (DS * static_cast<int>(sizeof(T)));  // rows per 16-byte packet
  constexpr int NW = kRowbalThreads / 32;
  constexpr int E = 16 / static_cast<int>(sizeof(T));         // elements per packet
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t path = n + b;
  auto diag_of = [&](int64_t u) { return path / units * u + (u < path % units ? u : path % units); };
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * kRowbalThreads + threadIdx.x;
  const int64_t warp_unit = unit - lane;
  const int64_t wi0 = path_search(offsets, b, diag_of(warp_unit), 32, lane, 0xffffffffu, 0);
  const int64_t wi1 = path_search(offsets, b, diag_of(warp_unit + 32), 32, lane, 0xffffffffu, 0);
  const int64_t d0 = diag_of(unit), d1 = diag_of(unit + 1);
  const int64_t i0 = path_search_range(offsets, wi0, wi1, d0);
  const int64_t i1 = path_search_range(offsets, i0, wi1, d1);
  const int64_t j0 = d0 - i0, j1 = d1 - i1;

  __shared__ float s_piece[2][kRowbalThreads * DS * W];
  __shared__ int64_t s_head[kRowbalThreads], s_tail[kRowbalThreads];
  __shared__ int32_t s_kind[kRowbalThreads];
  __shared__ float w_piece[2][NW * DS * W];
  __shared__ int64_t w_head[NW], w_tail[NW];
  __shared__ int32_t w_kind[NW];
  float *const my_head = &s_piece[0][threadIdx.x * DS * W];
  float *const my_tail = &s_piece[1][threadIdx.x * DS * W];
  s_head[threadIdx.x] = -1;
  s_tail[threadIdx.x] = -1;
  s_kind[threadIdx.x] = PIECE_NONE;

  int64_t seg = i0;
  auto end_at = [&](int64_t s1) -> int64_t { return s1 <= b ? load_offset(offsets, s1) : INT64_MAX; };
  int64_t w0 = end_at(seg + 1), w1 = end_at(seg + 2), w2 = end_at(seg + 3), w3 = end_at(seg + 4);
  bool first = true;
  const bool first_started_here = seg < b ? load_offset(offsets, seg) >= j0 : true;
  Acc acc;
  acc.init();
  auto finish = [&]() {
    if (first && !first_started_here) {
      acc.store_piece(my_head, DS);
      s_head[threadIdx.x] = seg;
    } else {
      float y[DS];
      acc.value(y);
      VecIO<T, DS>::store(out + seg * DS, y);
    }
    first = false;
    acc.init();
    ++seg;
    w0 = w1;
    w1 = w2;
    w2 = w3;
    w3 = end_at(seg + 4);
  };
  // Staged rows are read from shared memory; rows outside this lane's
  // slice read as the operation's identity (0 for sum, -inf for max).
  // A pass folds its rows into two independent chains (even and odd rows
  // of the run), merged into the accumulator at the end of the pass.
  constexpr float kIdentity = OP == OP_MAX ? -kInf : 0.0f;
  auto chain_fold = [&](float (&q)[DS], const float (&x)[E], int k, bool in) {
#pragma unroll
    for (int f = 0; f < DS; ++f) {
      const float v = in ? x[k * DS + f] : kIdentity;
      q[f] = OP == OP_MAX ? max_nan(q[f], v) : __fadd_rn(q[f], v);
    }
  };

  const uint4 *packets = reinterpret_cast<const uint4 *>(values);
  const int64_t p_begin = j0 / R, p_end = (j1 + R - 1) / R;
  const int my_packets = static_cast<int>(p_end - p_begin);
  __shared__ int64_t s_pbegin[kRowbalThreads];
  __shared__ int32_t s_pcount[kRowbalThreads];
  s_pbegin[threadIdx.x] = p_begin;
  s_pcount[threadIdx.x] = my_packets;
  const int rounds = (__reduce_max_sync(0xffffffffu, my_packets) + kPackedRun - 1) / kPackedRun;
  __syncwarp();
  extern __shared__ uint4 s_stage[];  // [NW][kPackedStages][32][kPackedRun + 1]
  constexpr int kLaneSlots = kPackedRun + 1, kStageSlots = 32 * kLaneSlots;
  constexpr int kRunsPerCopy = 32 / kPackedRun;
  uint4 *const w_stage = s_stage + warp * kPackedStages * kStageSlots;
  // This lane's copies: copy m moves packet k_copy of the run of lane
  // m * kRunsPerCopy + lane / kPackedRun, in every round.
  const int k_copy = lane % kPackedRun;
  const uint4 *copy_src[kPackedRun];
  int copy_left[kPackedRun];  // round r copies while r * kPackedRun < copy_left
#pragma unroll
  for (int m = 0; m < kPackedRun; ++m) {
    const int src = warp * 32 + m * kRunsPerCopy + lane / kPackedRun;
    copy_src[m] = packets + s_pbegin[src] + k_copy;
    copy_left[m] = s_pcount[src] - k_copy;
  }
  const uint32_t copy_dst = smem_u32(w_stage) + ((lane / kPackedRun) * kLaneSlots + k_copy) * 16;
  auto issue = [&](int r) {
    const uint32_t dst = copy_dst + (r % kPackedStages) * kStageSlots * 16;
    const int idx = r * kPackedRun;
#pragma unroll
    for (int m = 0; m < kPackedRun; ++m)
      if (idx < copy_left[m]) cp_async<16>(dst + m * kRunsPerCopy * kLaneSlots * 16, copy_src[m] + idx);
    cp_async_commit();
  };
#pragma unroll
  for (int r = 0; r < kPackedStages; ++r) issue(r);
  constexpr int kRunRows = kPackedRun * R;
  for (int r = 0; r < rounds; ++r) {
    cp_async_wait<kPackedStages - 1>();
    __syncwarp();
    const uint4 *const mine = w_stage + (r % kPackedStages) * kStageSlots + lane * kLaneSlots;
    const int64_t run_row = (p_begin + static_cast<int64_t>(r) * kPackedRun) * R;  // first staged row
    const int64_t lo = j0 > run_row ? j0 : run_row;
    const int64_t hi = j1 < run_row + kRunRows ? j1 : run_row + kRunRows;
    if (lo < hi) {
      while (w0 <= lo) finish();
      const int a = static_cast<int>(lo - run_row), e = static_cast<int>(hi - run_row);
      // Fold staged rows [from, to) in one pass (predicated unless the pass
      // covers the whole run).
      auto pass = [&](int from, int to) {
        float q[2][DS];
#pragma unroll
        for (int f = 0; f < DS; ++f) q[0][f] = q[1][f] = kIdentity;
        if (from == 0 && to == kRunRows) {
#pragma unroll
          for (int k = 0; k < kPackedRun; ++k) {
            float x[E];
            VecIO<T, E>::unpack(*reinterpret_cast<const typename VecIO<T, E>::Raw *>(&mine[k]), x);
#pragma unroll
            for (int kk = 0; kk < R; ++kk) chain_fold(q[(k * R + kk) & 1], x, kk, true);
          }
        } else {
#pragma unroll
          for (int k = 0; k < kPackedRun; ++k) {
            float x[E];
            VecIO<T, E>::unpack(*reinterpret_cast<const typename VecIO<T, E>::Raw *>(&mine[k]), x);
#pragma unroll
            for (int kk = 0; kk < R; ++kk)
              chain_fold(q[(k * R + kk) & 1], x, kk, k * R + kk >= from && k * R + kk < to);
          }
        }
        float merged[DS];
#pragma unroll
        for (int f = 0; f < DS; ++f) merged[f] = OP == OP_MAX ? max_nan(q[0][f], q[1][f]) : __fadd_rn(q[0][f], q[1][f]);
        acc.fold_raw(merged);
        acc.account(to - from);
      };
      if (w2 >= hi) {
        // At most two segment ends inside [lo, hi): one pass per piece
        // between them (a run of empty segments ending at the same row is
        // finished between two passes).
        for (int cur = a;;) {
          const int stop = w0 < hi ? static_cast<int>(w0 - run_row) : e;
          pass(cur, stop);
          if (stop == e) break;
          do finish(); while (w0 <= run_row + stop);
          cur = stop;
        }
      } else {
        // Three or more ends inside: each piece between them row by row
        // (plain adds into the block, counted once per piece).
        const T *const rows = reinterpret_cast<const T *>(mine);
        for (int cur = a;;) {
          const int stop = w0 < hi ? static_cast<int>(w0 - run_row) : e;
          for (int i = cur; i < stop; ++i) {
            float x[DS];
            VecIO<T, DS>::unpack(*reinterpret_cast<const typename VecIO<T, DS>::Raw *>(rows + i * DS), x);
            acc.fold_raw(x);
          }
          acc.account(stop - cur);
          if (stop == e) break;
          do finish(); while (w0 <= run_row + stop);
          cur = stop;
        }
      }
    }
    __syncwarp();  // every lane is done with this stage before it is refilled
    issue(r + kPackedStages);
  }
  cp_async_wait<0>();  // the groups issued past the last round are empty
  while (seg < i1) finish();
  if (seg < b) {
    const int64_t start = load_offset(offsets, seg);
    if ((start > j0 ? start : j0) < j1) {
      acc.store_piece(my_tail, DS);
      s_tail[threadIdx.x] = seg;
      s_kind[threadIdx.x] = start < j0 ? PIECE_THROUGH : PIECE_TAIL;
    }
  }
  __syncwarp();
  // Level 1: the warp's 32 units by a segmented scan of their TAIL /
  // THROUGH pieces across lanes (a TAIL -- a segment starting in the lane --
  // restarts the scan; a lane without a piece passes it on).  A lane with a
  // HEAD adds the scan of the lanes before it: the segment is finished if a
  // TAIL precedes it in the warp (its start), else the sum is the warp's
  // HEAD piece.  The last lane with path items holds the warp's open piece.
  {
    const unsigned full = 0xffffffffu;
    const int kind = s_kind[threadIdx.x];
    Acc run;
    if (kind != PIECE_NONE) run.load_piece(my_tail, DS); else run.init();
    bool restart = kind == PIECE_TAIL;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      Acc up = run.shfl_up(off);
      const bool up_restart = __shfl_up_sync(full, restart, off);
      if (lane >= off && !restart) {
        up.merge(run);
        run = up;
        restart = up_restart;
      }
    }
    Acc before = run.shfl_up(1);  // the scan up to the previous lane
    const bool before_tail = __shfl_up_sync(full, restart, 1) && lane > 0;
    const int64_t h = s_head[threadIdx.x];
    const bool warp_head = h >= 0 && !before_tail;
    if (h >= 0) {
      if (lane == 0) before.init();
      Acc head;
      head.load_piece(my_head, DS);
      before.merge(head);
      if (before_tail) {
        float y[DS];
        before.value(y);
        VecIO<T, DS>::store(out + h * DS, y);
      } else {
        before.store_piece(&w_piece[0][warp * DS * W], DS);
      }
    }
    const unsigned head_lanes = __ballot_sync(full, warp_head);  // at most one lane
    if (lane == (head_lanes ? __ffs(head_lanes) - 1 : 0)) w_head[warp] = warp_head ? h : -1;
    const unsigned busy = __ballot_sync(full, d1 > d0);
    const int last = busy ? 31 - __clz(busy) : 0;
    if (lane == last) {
      const bool open = busy && kind != PIECE_NONE;
      if (open) run.store_piece(&w_piece[1][warp * DS * W], DS);
      w_tail[warp] = open ? s_tail[threadIdx.x] : -1;
      w_kind[warp] = open ? (restart ? PIECE_TAIL : PIECE_THROUGH) : PIECE_NONE;
    }
  }
  __syncthreads();
  // Level 2: thread 0 combines the warps into the CTA's pieces.
  if (threadIdx.x == 0) {
    auto piece = [&](int k, int slot) { return &w_piece[slot][k * DS * W]; };
    float *const cta_pieces = pieces + static_cast<int64_t>(blockIdx.x) * 2 * W * DS;
    combine_pieces<T, OP, DS>(NW, piece, DS, w_head, w_tail, w_kind, true, out, DS, 0, cta_pieces,
                              cta_pieces + W * DS, DS, &meta[blockIdx.x], 0, 0);
  }
}

// Merge the pieces of every segment cut by CTA boundaries.  One CTA of
// kFixupThreads per (owner, column tile): the owner is the main kernel's
// CTA where the segment starts (its TAIL piece).  The fix-up CTA first
// finds the chain's end -- the CTA holding the HEAD piece -- scanning
// kFixupThreads metadata entries per step, then its warps merge contiguous
// runs of the pieces in between in parallel, and warp 0 merges the runs'
// partials in order and the HEAD.  The merge tree depends only on the
// chain, so results are deterministic.
//
// Sharded calls (edges != nullptr) have open chains at the window's edges:
// the segment open at the window's start (started on an earlier rank: THROUGH
// pieces up to its HEAD, or through the whole window) and the one open at
// its end (TAIL and THROUGH pieces, no HEAD).  Their merged f32 pieces go
// to the window's edge record instead of out; one extra CTA (blockIdx.x ==
// units) handles the start and writes the record's header.
constexpr int kFixupThreads = 512;

// Edge record of one window (floats): a header of kEdgeHeader floats
// holding int64 {head_seg, head_ends, tail_seg, 0}, then the head piece and
// the tail piece, W * d floats each (W = 2 for sum: s then c; 1 for max),
// padded to a multiple of 16 bytes.
constexpr int kEdgeHeader = 8;

// Floats between consecutive ranks' records: the record rounded up to 16
// bytes, so that every gathered record starts 16-byte aligned.
__host__ __device__ __forceinline__ int64_t edge_record_floats(int64_t width_times_d) {
  return (kEdgeHeader + 2 * width_times_d + 3) / 4 * 4;
}

template <int OP, int VEC>
__device__ __forceinline__ void chain_merge(RowAcc<OP, VEC> &total, const float *__restrict__ pieces,
                                            const UnitMeta *__restrict__ meta, int64_t d, int64_t col, bool active,
                                            int64_t lo, int64_t hi, bool head_at_hi, float (*s_part)[2][32 * VEC]) {
  // Slot-1 pieces (TAIL / THROUGH) of CTAs [lo, hi), then the HEAD (slot 0)
  // of CTA hi when head_at_hi.  Result in `total` of warp 0's lanes.
  using Acc = RowAcc<OP, VEC>;
  constexpr int NW = kFixupThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t span = 2 * Acc::kWidth * d;
  const int64_t count = hi > lo ? hi - lo : 0;
  const int64_t per = (count + NW - 1) / NW;
  const int64_t a = lo + warp * per, e = a + per < hi ? a + per : hi;
  // Every CTA of a chain holds a slot-1 piece, so no metadata is read: four
  // pieces' loads are issued together, then merged in order.
  Acc acc;
  acc.init();
  if (active) {
    int64_t v = a;
    for (; v + 4 <= e; v += 4) {
      float buf[4][Acc::kWidth][VEC];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float *src = pieces + (v + i) * span + Acc::kWidth * d + col;
#pragma unroll
        for (int k = 0; k < Acc::kWidth; ++k)
#pragma unroll
          for (int x = 0; x < VEC; ++x) buf[i][k][x] = __ldcg(src + k * d + x);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) acc.merge_piece(&buf[i][0][0], VEC);
    }
    for (; v < e; ++v) acc.merge_piece(pieces + v * span + Acc::kWidth * d + col, d);
  }
  if (active) acc.store_piece(&s_part[warp][0][lane * VEC], 32 * VEC);
  __syncthreads();
  if (warp == 0 && active) {
    total.init();
#pragma unroll
    for (int w = 0; w < NW; ++w) total.merge_piece(&s_part[w][0][lane * VEC], 32 * VEC);
    if (head_at_hi) total.merge_piece(pieces + hi * span + col, d);
  }
}

// First CTA v in [from, units) whose HEAD piece belongs to `seg`
// (INT64_MAX if none), scanning kFixupThreads entries per step.
__device__ __forceinline__ int64_t find_head(const UnitMeta *__restrict__ meta, int64_t from, int64_t units,
                                             int64_t seg, int64_t *s_end) {
  if (threadIdx.x == 0) *s_end = INT64_MAX;
  __syncthreads();
  for (int64_t base = from; base < units; base += kFixupThreads) {
    const int64_t v = base + threadIdx.x;
    if (v < units && meta[v].head_seg == seg)
      atomicMin(reinterpret_cast<unsigned long long *>(s_end), static_cast<unsigned long long>(v));
    __syncthreads();
    if (*s_end != INT64_MAX) break;  // uniform: read after the barrier
    __syncthreads();
  }
  return *s_end;
}

template <typename T, int OP, int VEC>
__global__ void __launch_bounds__(kFixupThreads)
rowbal_fixup_kernel(T *__restrict__ out, int64_t d, int vec_cols, int64_t units,
                    const float *__restrict__ pieces, const UnitMeta *__restrict__ meta, float *__restrict__ edges,
                    int64_t seg0 = 0, int64_t seg1 = 0) {
  using Acc = RowAcc<OP, VEC>;
  constexpr int NW = kFixupThreads / 32;
  __shared__ int64_t s_end;
  __shared__ float s_part[NW][2][32 * VEC];  // per-warp partials: (s, c) or (m)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cv = blockIdx.y * 32 + lane;
  const bool active = cv < vec_cols;
  const int64_t col = static_cast<int64_t>(cv) * VEC;
  const int64_t wd = Acc::kWidth * d;
  const int64_t u = blockIdx.x;
  Acc total;
  if (u == units) {
    // ---- window start (sharded calls only): the segment open at row0
    const int64_t head0 = meta[0].head_seg;
    const int64_t seg0 = head0 >= 0 ? head0 : (meta[0].tail_kind == PIECE_THROUGH ? meta[0].tail_seg : -1);
    int64_t end = INT64_MAX;
    if (seg0 >= 0) {
      end = head0 >= 0 ? 0 : find_head(meta, 1, units, seg0, &s_end);
      const bool ends = end < units;
      chain_merge<OP, VEC>(total, pieces, meta, d, col, active, 0, ends ? end : units, ends, s_part);
      if (warp == 0 && active) total.store_piece(edges + kEdgeHeader + col, d);
    }
    if (threadIdx.x == 0 && blockIdx.y == 0) {
      int64_t *hdr = reinterpret_cast<int64_t *>(edges);
      const bool through = seg0 >= 0 && end >= units;
      const UnitMeta &last = meta[units - 1];
      hdr[0] = seg0;
      hdr[1] = seg0 >= 0 && !through;
      hdr[2] = (!through && last.tail_kind != PIECE_NONE) ? last.tail_seg : -1;
      hdr[3] = 0;
    }
    return;
  }
  if (meta[u].tail_kind != PIECE_TAIL) return;  // uniform across the CTA
  const int64_t seg = meta[u].tail_seg;
  const int64_t end = find_head(meta, u + 1, units, seg, &s_end);
  if (end >= units) {
    // ---- window end (sharded calls): TAIL and THROUGH pieces, no HEAD
    if (edges == nullptr) return;  // unreachable for a whole-array call with valid offsets
    chain_merge<OP, VEC>(total, pieces, meta, d, col, active, u, units, false, s_part);
    if (warp == 0 && active) total.store_piece(edges + kEdgeHeader + wd + col, d);
    return;
  }
  chain_merge<OP, VEC>(total, pieces, meta, d, col, active, u, end, true, s_part);
  if (warp == 0 && active && has_slot(seg, seg0, seg1)) emit<T, OP, VEC>(total, out, seg - seg0, d, col);
}

// Softmax of a sharded call: the final statistics of the segments cut at
// this rank's edges (the one open at its first row, the one open at its
// last), merged in rank order from every rank's edge record -- a starting
// rank's TAIL piece, then HEAD pieces of the ranks the segment passes
// through or ends in -- into this rank's slots (segment s at s - seg0).
// Every rank holding rows of a cut segment computes the same statistics.
template <int VEC>
__global__ void __launch_bounds__(32)
shard_softmax_combine_kernel(float *__restrict__ stats, int64_t d, int vec_cols, int world, int rank,
                             const float *__restrict__ gathered, int64_t seg0, int64_t seg1) {
  using Acc = RowAcc<OP_SOFTMAX, VEC>;
  const int64_t wd = Acc::kWidth * d;
  const int64_t rec = edge_record_floats(wd);
  const int cv = blockIdx.y * 32 + threadIdx.x;
  if (cv >= vec_cols) return;
  const int64_t col = static_cast<int64_t>(cv) * VEC;
  const int64_t *mine = reinterpret_cast<const int64_t *>(gathered + rank * rec);
  for (int which = 0; which < 2; ++which) {
    const int64_t s = mine[which == 0 ? 0 : 2];
    if (s < 0 || !has_slot(s, seg0, seg1)) continue;
    Acc total;
    total.init();
    for (int k = 0; k < world; ++k) {
      const int64_t *h = reinterpret_cast<const int64_t *>(gathered + k * rec);
      if (h[2] == s) total.merge_piece(gathered + k * rec + kEdgeHeader + wd + col, d);  // started in rank k
      else if (h[0] == s) total.merge_piece(gathered + k * rec + kEdgeHeader + col, d);   // open at k's start
    }
    total.store_piece(stats + (s - seg0) * 2 * d + col, d);
  }
}

// Finish the segments cut by shard boundaries on the rank that consumed
// their end: gathered[k] is rank k's edge record (kEdgeHeader + 2 W d
// floats).  Rank `rank` owns the segment of its head piece if it consumed
// that segment's end; the pieces merge in rank order: the starting rank's
// tail piece, the head pieces of ranks the segment passes through, then
// this rank's head piece.  A rank whose window holds no rows (a split with
// repeated boundaries) records no piece: header (-1, 0, -1).  Such a record
// can only sit inside the segment's chain, because a rank with rows inside
// an open segment always records it, so the walk back steps over it and its
// (unwritten) pieces are never read.  One CTA per column tile.
template <typename T, int OP, int VEC>
__global__ void __launch_bounds__(32)
shard_combine_kernel(T *__restrict__ out, int64_t d, int vec_cols, int world, int rank,
                     const float *__restrict__ gathered) {
  using Acc = RowAcc<OP, VEC>;
  const int64_t wd = Acc::kWidth * d;
  const int64_t rec = edge_record_floats(wd);
  const int64_t *hdr = reinterpret_cast<const int64_t *>(gathered + rank * rec);
  const int64_t seg = hdr[0];
  if (seg < 0 || hdr[1] == 0) return;
  const int cv = blockIdx.y * 32 + threadIdx.x;
  if (cv >= vec_cols) return;
  const int64_t col = static_cast<int64_t>(cv) * VEC;
  auto header = [&](int k) { return reinterpret_cast<const int64_t *>(gathered + k * rec); };
  auto empty = [&](const int64_t *h) { return h[0] < 0 && h[2] < 0; };
  int k = rank - 1;  // walk back over ranks the segment passes through (or that hold no rows)
  while (k >= 0) {
    const int64_t *h = header(k);
    if ((h[0] == seg && h[1] == 0) || empty(h)) --k;
    else break;
  }
  Acc total;
  total.init();
  if (k >= 0) {
    const int64_t *h = header(k);
    if (h[2] == seg) total.merge_piece(gathered + k * rec + kEdgeHeader + wd + col, d);  // the starting rank's tail
  }
  for (int j = k + 1; j < rank; ++j)  // ranks the segment passes through (their head pieces)
    if (header(j)[0] == seg) total.merge_piece(gathered + j * rec + kEdgeHeader + col, d);
  total.merge_piece(gathered + rank * rec + kEdgeHeader + col, d);  // this rank's head
  float y[VEC];
  total.value(y);
  VecIO<T, VEC>::store(out + seg * d + col, y);
}

// Segment of row x, given that segment `seg` starts after x: the first k in
// [0, seg) with offsets[k + 1] > x.  Galloping backwards from seg - 1, then
// a binary search: O(log gap) dependent loads however many empty segments
// lie between (a walk of one load per segment took 35 ms per unit on runs of
// empty segments).
template <typename OffT>
__device__ __forceinline__ int64_t segment_before(const OffT *offsets, int64_t seg, int64_t x) {
  int64_t hi = seg - 1;  // offsets[hi + 1] = offsets[seg] > x: the answer is <= hi
  int64_t step = 1;
  int64_t lo = hi;       // invariant: offsets[lo + 1] > x
  while (lo - step >= 0 && load_offset(offsets, lo - step + 1) > x) {
    lo -= step;
    step *= 2;
  }
  // The answer lies in [max(0, lo - step + 1), lo]: offsets[k + 1] <= x for k = lo - step (if >= 0).
  int64_t a = lo - step + 1 > 0 ? lo - step + 1 : 0, b = lo;
  while (a < b) {
    const int64_t mid = a + (b - a) / 2;
    if (load_offset(offsets, mid + 1) > x) b = mid; else a = mid + 1;
  }
  return a;
}

// Softmax normalise pass of the row-balanced schedule: out = e^(x - ref) /
// total with the statistics the statistics pass left per segment.  Rows are
// split evenly over the units (every row costs the same); each unit walks
// its rows from the last to the first, so the rows the statistics pass read
// last -- the ends of its units' slices -- are re-read while still in L2.
template <typename T, typename OffT, int VEC, int U = 8, bool XF = false>
__global__ void __launch_bounds__(kRowbalThreads, 3)
rowbal_normalize_kernel(const T *__restrict__ values, const OffT *__restrict__ offsets, T *__restrict__ out,
                        const float *__restrict__ stats, int64_t n, int64_t b, int64_t d, int g_shift, int vec_cols,
                        int64_t units, int64_t row_base = 0, int64_t seg0 = 0, int64_t seg1 = 0,
                        Xform xf = Xform{}) {
  // values[i] and out[i] hold row row_base + i of the whole array (a rank's
  // window of a sharded call; 0 otherwise); the statistics of segment s sit
  // at slot s - seg0 (seg1: end of the slots, 0 = unbounded).
  const int lane = threadIdx.x & 31;
  const int G = 1 << g_shift;
  const int q = lane >> g_shift, gl = lane & (G - 1);
  const int group_base = q << g_shift;
  const unsigned group_mask = (G == 32) ? 0xffffffffu : (((1u << G) - 1u) << group_base);
  const int units_per_cta = (kRowbalThreads / 32) << (5 - g_shift);
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * units_per_cta + (threadIdx.x >> 5) * (32 >> g_shift) + q;
  const int cv = blockIdx.y * 32 + gl;
  const bool active = cv < vec_cols;
  const int64_t col = static_cast<int64_t>(cv) * VEC;
  const int64_t r0 = row_base + n / units * unit + min(unit, n % units);  // whole-array rows
  const int64_t r1 = r0 + n / units + (unit < n % units ? 1 : 0);
  if (r1 <= r0) return;  // uniform per unit; no barriers below
  // Segment of the last row: the first k with offsets[k + 1] > r1 - 1.
  int64_t seg = ends_upto(offsets, b, r1 - 1, G, gl, group_mask, group_base);
  int64_t start = load_offset(offsets, seg);
  float ref[VEC], inv[VEC];
  auto load_stats = [&]() {
    const bool slot = seg1 == 0 || (seg >= seg0 && seg < seg1);  // a wrong caller range: NaN, never out of bounds
    const float *st = stats + (slot ? seg - seg0 : 0) * 2 * d + col;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      ref[v] = slot ? __ldcg(st + v) : __int_as_float(0x7fffffff);
      inv[v] = slot ? stats_inverse(__ldcg(st + d + v)) : __int_as_float(0x7fffffff);
    }
  };
  if (active) load_stats();
  using Raw = typename VecIO<T, VEC>::Raw;
  const T *const src = values + col;  // row r sits at (r - row_base) * d
  T *const dst = out + col;
  auto normalize_row = [&](const Raw &raw, const MaskVec<VEC> &mk, int64_t r) {
    float x[VEC], y[VEC];
    VecIO<T, VEC>::unpack(raw, x);
    if constexpr (XF) apply_xform<VEC>(x, xf, mk);
#pragma unroll
    for (int v = 0; v < VEC; ++v) y[v] = stats_normalize(x[v], ref[v], inv[v]);
    VecIO<T, VEC>::store(dst + (r - row_base) * d, y);
  };
  int64_t r = r1 - 1;
  for (; r - (U - 1) >= r0; r -= U) {
    Raw raw[U];
    MaskVec<VEC> mk[U];
#pragma unroll
    for (int t = 0; t < U; ++t)
      if (active) {
        raw[t] = VecIO<T, VEC>::load_raw(src + (r - t - row_base) * d);
        if constexpr (XF) {
          if (xf.mask) mk[t] = load_mask<VEC>(xf, r - t, col);
        }
      }
#pragma unroll
    for (int t = 0; t < U; ++t) {
      if (r - t < start) {  // an earlier segment (skipping empty ones)
        seg = segment_before(offsets, seg, r - t);
        start = load_offset(offsets, seg);
        if (active) load_stats();
      }
      if (active) normalize_row(raw[t], mk[t], r - t);
    }
  }
  for (; r >= r0; --r) {
    if (r < start) {
      seg = segment_before(offsets, seg, r);
      start = load_offset(offsets, seg);
      if (active) load_stats();
    }
    if (active) {
      MaskVec<VEC> mk;
      if constexpr (XF) {
        if (xf.mask) mk = load_mask<VEC>(xf, r, col);
      }
      normalize_row(VecIO<T, VEC>::load_raw(src + (r - row_base) * d), mk, r);
    }
  }
}

}  // namespace rgb
