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
// the common path.  A segment cut by a unit boundary leaves f32 pieces: the
// unit where it starts writes a TAIL piece, units it covers completely write
// THROUGH pieces and the unit that consumes its end writes a HEAD piece.
// The fix-up kernel merges each cut segment's pieces in row order and
// writes its output once (one rounding to the output dtype), so results are
// deterministic.
#pragma once

#include "common.cuh"

namespace rgb {

constexpr int kRowbalThreads = 256;
constexpr int kRowbalUnroll = 8;
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
};

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

template <typename T, typename OffT, int OP, int VEC>
__global__ void __launch_bounds__(kRowbalThreads)
rowbal_kernel(const T *__restrict__ values, const OffT *__restrict__ offsets, T *__restrict__ out,
              int64_t n, int64_t b, int64_t d, int g_shift, int vec_cols, int64_t units,
              float *__restrict__ pieces, UnitMeta *__restrict__ meta) {
  using Acc = RowAcc<OP, VEC>;
  constexpr int U = kRowbalUnroll;
  const int lane = threadIdx.x & 31;
  const int G = 1 << g_shift;
  const int q = lane >> g_shift;          // unit within the warp
  const int gl = lane & (G - 1);          // lane within the unit
  const int group_base = q << g_shift;
  const unsigned group_mask = (G == 32) ? 0xffffffffu : (((1u << G) - 1u) << group_base);
  const int units_per_cta = (kRowbalThreads / 32) << (5 - g_shift);
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * units_per_cta + (threadIdx.x >> 5) * (32 >> g_shift) + q;
  if (unit >= units) return;  // whole groups exit together
  const int cv = blockIdx.y * 32 + gl;
  const bool active = cv < vec_cols;
  const int64_t col = static_cast<int64_t>(cv) * VEC;

  // This unit's slice of the merge path.
  const int64_t path = n + b;
  const int64_t d0 = path / units * unit + min(unit, path % units);
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

  float *const unit_pieces = pieces + unit * 2 * Acc::kWidth * d;  // [2][kWidth][d]
  const int64_t stride = d;                                          // between s and c
  Acc acc;
  acc.init();

  // Finalise `seg` (its end is consumed by this unit).
  auto finish = [&]() {
    if (first && !first_started_here) {
      if (active) acc.store_piece(unit_pieces + col, stride);
      if (blockIdx.y == 0 && gl == 0) meta[unit].head_seg = seg;
    } else if (active) {
      float y[VEC];
      acc.value(y);
      VecIO<T, VEC>::store(out + seg * d + col, y);
    }
    first = false;
    acc.init();
    ++seg;
    next_b = seg < b ? end_of(seg) : INT64_MAX;
  };

  if (blockIdx.y == 0 && gl == 0) {
    meta[unit].head_seg = -1;
    meta[unit].tail_seg = -1;
    meta[unit].tail_kind = PIECE_NONE;
  }

  for (int64_t r = j0; r < j1; r += U) {
    // Issue U row loads of this unit's stream, then fold them in order.
    typename VecIO<T, VEC>::Raw raw[U];
    const T *row_ptr = values + r * d + col;
#pragma unroll
    for (int t = 0; t < U; ++t) {
      if (active && r + t < j1) raw[t] = VecIO<T, VEC>::load_raw(row_ptr + t * d);
    }
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
  while (seg < i1) finish();  // ends consumed after the last row
  // Segment open at the end of this unit, if the unit holds rows of it:
  // a THROUGH piece when it also started before the unit, else a TAIL.
  if (seg < b) {
    const int64_t start = load_offset(offsets, seg);
    if ((start > j0 ? start : j0) < j1) {
      if (active) acc.store_piece(unit_pieces + Acc::kWidth * d + col, stride);
      if (blockIdx.y == 0 && gl == 0) {
        meta[unit].tail_seg = seg;
        meta[unit].tail_kind = start < j0 ? PIECE_THROUGH : PIECE_TAIL;
      }
    }
  }
}

// Merge the pieces of every segment cut by unit boundaries.  One warp per
// (owner unit, column tile): the owner is the unit where the segment
// starts; it walks the following units' THROUGH pieces and ends at the
// HEAD piece of the unit that consumed the segment's end.
template <typename T, int OP, int VEC>
__global__ void __launch_bounds__(32)
rowbal_fixup_kernel(T *__restrict__ out, int64_t d, int vec_cols, int64_t units,
                    const float *__restrict__ pieces, const UnitMeta *__restrict__ meta) {
  using Acc = RowAcc<OP, VEC>;
  const int64_t u = blockIdx.x;
  if (meta[u].tail_kind != PIECE_TAIL) return;
  const int64_t seg = meta[u].tail_seg;
  const int cv = blockIdx.y * 32 + threadIdx.x;
  if (cv >= vec_cols) return;
  const int64_t col = static_cast<int64_t>(cv) * VEC;
  const int64_t stride = d;
  const int64_t piece_span = 2 * Acc::kWidth * d;
  Acc acc;
  acc.load_piece(pieces + u * piece_span + Acc::kWidth * d + col, stride);
  for (int64_t v = u + 1; v < units; ++v) {
    const UnitMeta m = meta[v];
    if (m.head_seg < 0 && m.tail_seg < 0) continue;  // a unit with an empty slice of the path
    if (m.head_seg == seg) {
      acc.merge_piece(pieces + v * piece_span + col, stride);
      break;
    }
    if (m.tail_seg == seg && m.tail_kind == PIECE_THROUGH) {
      acc.merge_piece(pieces + v * piece_span + Acc::kWidth * d + col, stride);
      continue;
    }
    break;
  }
  float y[VEC];
  acc.value(y);
  VecIO<T, VEC>::store(out + seg * d + col, y);
}

}  // namespace rgb
