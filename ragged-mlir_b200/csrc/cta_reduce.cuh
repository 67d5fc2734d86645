// CTA- and warp-level segment reduction of the classified schedule.
//
// Geometry: G = 2^g_shift lanes cover one row tile (VEC features each), a
// warp covers 32 / G rows per load, NW warps cover NW * 32 / G rows per
// step.  Rows are strided across the "row lanes"; each thread folds its
// rows into an Acc, row groups merge with xor shuffles and warps through
// shared memory in a fixed order, so results are deterministic.
//
// Rows come from a "source": global memory (read-only path) or a block of
// consecutive rows staged in shared memory by a bulk copy.  Both hand out
// the raw vector of row r for this thread's column.
#pragma once

#include "common.cuh"

namespace rgb {

constexpr int kFoldUnroll = 4;

// A thread's rows are begin + row_lane + k * step for k = 0, 1, ...: a
// source hands out a cursor at the first one, and the cursor the raw vector
// of the k-th (one pointer and one stride per loop, no per-row index math).
template <typename T, int VEC>
struct GlobalRows {
  using Raw = typename VecIO<T, VEC>::Raw;
  const T *values;
  int64_t d, col;
  struct Cursor {
    const T *p;
    int64_t stride;
    __device__ __forceinline__ Raw raw(int k) const { return VecIO<T, VEC>::load_raw(p + k * stride); }
  };
  __device__ __forceinline__ Cursor at(int64_t r, int64_t step) const { return Cursor{values + r * d + col, step * d}; }
  __device__ __forceinline__ Raw raw(int64_t r) const { return VecIO<T, VEC>::load_raw(values + r * d + col); }
};

// Rows [row0, ...) staged contiguously at `base` (shared memory), row_bytes
// apart; this thread's vector sits col_bytes into each row.
template <typename T, int VEC>
struct SharedRows {
  using Raw = typename VecIO<T, VEC>::Raw;
  char *base;
  int64_t row0;
  int row_bytes, col_bytes;
  struct Cursor {
    char *p;
    int stride;
    __device__ __forceinline__ Raw raw(int k) const { return *reinterpret_cast<const Raw *>(p + k * stride); }
    // Overwrite the k-th vector (the softmax mass pass keeps its terms there).
    __device__ __forceinline__ void put(int k, const Raw &v) const { *reinterpret_cast<Raw *>(p + k * stride) = v; }
  };
  __device__ __forceinline__ Cursor at(int64_t r, int64_t step) const {
    return Cursor{base + static_cast<int>(r - row0) * row_bytes + col_bytes, static_cast<int>(step) * row_bytes};
  }
  __device__ __forceinline__ Raw raw(int64_t r) const {
    return *reinterpret_cast<const Raw *>(base + static_cast<int>(r - row0) * row_bytes + col_bytes);
  }
};

// Rows of this thread in [begin, end): begin + row_lane + k * step.  Every
// step here is a power of two (lanes per row and warps per team or CTA
// are), so the count is a shift.
__device__ __forceinline__ int lane_rows(int64_t begin, int64_t end, int64_t row_lane, int64_t step) {
  const int64_t first = begin + row_lane;
  return first < end ? static_cast<int>((end - first + step - 1) >> (__ffsll(step) - 1)) : 0;
}

// Fold rows [begin, end) with stride `step` starting at begin + row_lane:
// batches of kFoldUnroll rows (loads issued together, one recentring test
// per softmax batch), then the remainder row by row.
template <typename T, int OP, int VEC, typename Src>
__device__ __forceinline__ void fold_rows(Acc<OP, VEC> &acc, const Src &src, int64_t begin, int64_t end,
                                          int64_t row_lane, int64_t step) {
  constexpr int U = kFoldUnroll;
  using Raw = typename VecIO<T, VEC>::Raw;
  const int count = lane_rows(begin, end, row_lane, step);
  const auto cur = src.at(begin + row_lane, step);
  int k = 0;
  for (; k + U <= count; k += U) {
    Raw raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) raw[u] = cur.raw(k + u);
    float x[U][VEC];
#pragma unroll
    for (int u = 0; u < U; ++u) VecIO<T, VEC>::unpack(raw[u], x[u]);
    acc.template fold_batch<U>(x);
  }
  for (; k < count; ++k) {
    float x[VEC];
    VecIO<T, VEC>::unpack(cur.raw(k), x);
    acc.fold(x);
  }
}

// Per-thread maximum of rows [begin, end) (stride `step` from begin +
// row_lane), NaN-propagating, -inf when the thread has no rows.  bf16 rows
// are compared as packed pairs (exact: the maximum of bf16 values is one of
// them).
template <typename T, int VEC, typename Src>
__device__ __forceinline__ void rows_max(float (&m)[VEC], const Src &src, int64_t begin, int64_t end,
                                         int64_t row_lane, int64_t step) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value && VEC == 8) {
    const __nv_bfloat162 lowest = __floats2bfloat162_rn(-kInf, -kInf);
    __nv_bfloat162 acc[4] = {lowest, lowest, lowest, lowest};
    const int count = lane_rows(begin, end, row_lane, step);
    const auto cur = src.at(begin + row_lane, step);
#pragma unroll 4
    for (int k = 0; k < count; ++k) {
      const uint4 raw = cur.raw(k);
      acc[0] = __hmax2_nan(acc[0], *reinterpret_cast<const __nv_bfloat162 *>(&raw.x));
      acc[1] = __hmax2_nan(acc[1], *reinterpret_cast<const __nv_bfloat162 *>(&raw.y));
      acc[2] = __hmax2_nan(acc[2], *reinterpret_cast<const __nv_bfloat162 *>(&raw.z));
      acc[3] = __hmax2_nan(acc[3], *reinterpret_cast<const __nv_bfloat162 *>(&raw.w));
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t u = *reinterpret_cast<const uint32_t *>(&acc[k]);
      m[2 * k] = bf16_lo(u);
      m[2 * k + 1] = bf16_hi(u);
    }
  } else {
#pragma unroll
    for (int v = 0; v < VEC; ++v) m[v] = -kInf;
    const int count = lane_rows(begin, end, row_lane, step);
    const auto cur = src.at(begin + row_lane, step);
#pragma unroll 4
    for (int k = 0; k < count; ++k) {
      float x[VEC];
      VecIO<T, VEC>::unpack(cur.raw(k), x);
#pragma unroll
      for (int v = 0; v < VEC; ++v) m[v] = max_nan(m[v], x[v]);
    }
  }
}

// Softmax statistics of a thread's rows held in shared memory (read three
// times in all, HBM once): the exact maximum m, then the mass sum e^(x-m)
// (terms at most 1, summed plainly).  A thread whose values are all -inf
// (or that has no rows) contributes no mass; +inf or NaN make the mass NaN
// through the arithmetic.  The result is an online-statistics accumulator
// that merges like any other (stats_merge).
template <typename T, int VEC, typename Src>
__device__ __forceinline__ void staged_stats(Acc<OP_SOFTMAX, VEC> &acc, const Src &src, int64_t begin, int64_t end,
                                             int64_t row_lane, int64_t step) {
  constexpr int U = kFoldUnroll;
  using Raw = typename VecIO<T, VEC>::Raw;
  float m[VEC], base[VEC], s[VEC];
  rows_max<T, VEC>(m, src, begin, end, row_lane, step);
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
    base[v] = m[v] == -kInf ? 0.0f : m[v];  // all -inf: every term is e^-inf = 0
    s[v] = 0.0f;
  }
  if constexpr (VEC % 2 == 0) {
    constexpr int P = VEC / 2;
    unsigned long long b2[P], s2[P];
#pragma unroll
    for (int k = 0; k < P; ++k) {
      b2[k] = pack2(base[2 * k], base[2 * k + 1]);
      s2[k] = pack2(0.0f, 0.0f);
    }
    auto add_row = [&](const Raw &raw) {
      float x[VEC];
      VecIO<T, VEC>::unpack(raw, x);
#pragma unroll
      for (int k = 0; k < P; ++k) s2[k] = add2_rn(s2[k], exp_diff2(pack2(x[2 * k], x[2 * k + 1]), b2[k]));
    };
    const int count = lane_rows(begin, end, row_lane, step);
    const auto cur = src.at(begin + row_lane, step);
    int k = 0;
    for (; k + U <= count; k += U) {
      Raw raw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) raw[u] = cur.raw(k + u);
#pragma unroll
      for (int u = 0; u < U; ++u) add_row(raw[u]);
    }
    for (; k < count; ++k) add_row(cur.raw(k));
#pragma unroll
    for (int k = 0; k < P; ++k) unpack2(s2[k], s[2 * k], s[2 * k + 1]);
  } else {
    const int count = lane_rows(begin, end, row_lane, step);
    const auto cur = src.at(begin + row_lane, step);
#pragma unroll 4
    for (int k = 0; k < count; ++k) {
      float x[VEC];
      VecIO<T, VEC>::unpack(cur.raw(k), x);
#pragma unroll
      for (int v = 0; v < VEC; ++v) s[v] = __fadd_rn(s[v], exp_diff(x[v], base[v]));
    }
  }
#pragma unroll
  for (int v = 0; v < VEC; ++v) acc.st[v] = Stats{m[v], s[v], 0.0f};
}

// VEC f32 values in the raw form of T (bf16: round to nearest even).
template <typename T, int VEC>
__device__ __forceinline__ typename VecIO<T, VEC>::Raw pack_raw(const float (&y)[VEC]) {
  using Raw = typename VecIO<T, VEC>::Raw;
  Raw raw;
  if constexpr (std::is_same<T, float>::value) {
    static_assert(sizeof(Raw) == VEC * 4, "f32 raw form");
    memcpy(&raw, y, sizeof raw);
  } else if constexpr (VEC == 8) {
    raw = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                     pack_bf16x2(y[6], y[7]));
  } else if constexpr (VEC == 4) {
    raw = make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
  } else if constexpr (VEC == 2) {
    raw = pack_bf16x2(y[0], y[1]);
  } else {
    const __nv_bfloat16 h = __float2bfloat16_rn(y[0]);
    raw = *reinterpret_cast<const unsigned short *>(&h);
  }
  return raw;
}

// Softmax statistics of a thread's staged rows, like staged_stats, that
// also keep every term e = e^(x - b) in the stage in place of x (in T: a
// bf16 term is rounded once more), so the normalisation multiplies instead
// of recomputing the exponential: out = e * e^(b - M) / total, with b the
// thread's own maximum (0 when every value it saw is -inf) returned in
// `base`.  Keeping the terms halves the SFU work of a staged softmax; for
// bf16 output the extra rounding keeps the result within one ulp of the
// rounded exact value (a half-ulp error on e, then the final rounding).
template <typename T, int VEC, bool XF = false>
__device__ __forceinline__ void staged_stats_keep(Acc<OP_SOFTMAX, VEC> &acc, const SharedRows<T, VEC> &src,
                                                  int64_t begin, int64_t end, int64_t row_lane, int64_t step,
                                                  float (&base)[VEC], const Xform &xf = Xform{}, int64_t col = 0) {
  constexpr int U = kFoldUnroll;
  using Raw = typename VecIO<T, VEC>::Raw;
  static_assert(VEC % 2 == 0, "packed pairs");
  constexpr int P = VEC / 2;
  float m[VEC], s[VEC];
  const int count = lane_rows(begin, end, row_lane, step);
  const auto cur = src.at(begin + row_lane, step);
  const int64_t row = begin + row_lane;  // whole-array row of this thread's k = 0 (the mask's row)
  if (XF && !xf.mask && xf.scaled && xf.scale > 0.0f) {
    // A positive scale keeps the order and rounding is monotone, so the
    // maximum of the scaled values is the scaled maximum (NaN and infinities
    // included): the packed maximum of the stored values, scaled once.
    rows_max<T, VEC>(m, src, begin, end, row_lane, step);
#pragma unroll
    for (int v = 0; v < VEC; ++v) m[v] = __fmul_rn(m[v], xf.scale);
  } else if constexpr (XF) {
    // Transformed maximum: f32 arithmetic (a mask or scale leaves the bf16 grid).
#pragma unroll
    for (int v = 0; v < VEC; ++v) m[v] = -kInf;
    int k = 0;
    for (; k + U <= count; k += U) {
      Raw raw[U];
      MaskVec<VEC> mk[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        raw[u] = cur.raw(k + u);
        if (xf.mask) mk[u] = load_mask<VEC>(xf, row + (k + u) * step, col);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float x[VEC];
        VecIO<T, VEC>::unpack(raw[u], x);
        apply_xform<VEC>(x, xf, mk[u]);
#pragma unroll
        for (int v = 0; v < VEC; ++v) m[v] = max_nan(m[v], x[v]);
      }
    }
    for (; k < count; ++k) {
      float x[VEC];
      MaskVec<VEC> mk;
      if (xf.mask) mk = load_mask<VEC>(xf, row + k * step, col);
      VecIO<T, VEC>::unpack(cur.raw(k), x);
      apply_xform<VEC>(x, xf, mk);
#pragma unroll
      for (int v = 0; v < VEC; ++v) m[v] = max_nan(m[v], x[v]);
    }
  } else {
    rows_max<T, VEC>(m, src, begin, end, row_lane, step);
  }
#pragma unroll
  for (int v = 0; v < VEC; ++v) base[v] = m[v] == -kInf ? 0.0f : m[v];  // all -inf: every term is e^-inf = 0
  unsigned long long b2[P], s2[P];
#pragma unroll
  for (int k = 0; k < P; ++k) {
    b2[k] = pack2(base[2 * k], base[2 * k + 1]);
    s2[k] = pack2(0.0f, 0.0f);
  }
  auto keep_row = [&](const Raw &raw, const MaskVec<VEC> &mk, int k) {
    float x[VEC], e[VEC];
    VecIO<T, VEC>::unpack(raw, x);
    if constexpr (XF) apply_xform<VEC>(x, xf, mk);
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const unsigned long long t = exp_diff2(pack2(x[2 * j], x[2 * j + 1]), b2[j]);
      s2[j] = add2_rn(s2[j], t);
      unpack2(t, e[2 * j], e[2 * j + 1]);
    }
    cur.put(k, pack_raw<T, VEC>(e));
  };
  int k = 0;
  for (; k + U <= count; k += U) {
    Raw raw[U];
    MaskVec<VEC> mk[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      raw[u] = cur.raw(k + u);
      if constexpr (XF) {
        if (xf.mask) mk[u] = load_mask<VEC>(xf, row + (k + u) * step, col);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) keep_row(raw[u], mk[u], k + u);
  }
  for (; k < count; ++k) {
    MaskVec<VEC> mk;
    if constexpr (XF) {
      if (xf.mask) mk = load_mask<VEC>(xf, row + k * step, col);
    }
    keep_row(cur.raw(k), mk, k);
  }
#pragma unroll
  for (int j = 0; j < P; ++j) unpack2(s2[j], s[2 * j], s[2 * j + 1]);
#pragma unroll
  for (int v = 0; v < VEC; ++v) acc.st[v] = Stats{m[v], s[v], 0.0f};
}

// Factor of the kept terms of a thread: e^(base - ref) / total per
// feature.  A thread whose values were all -inf kept zeros: its factor is
// 0 * inv, which stays NaN for a column that is -inf throughout (total 0).
template <int VEC>
__device__ __forceinline__ void kept_factor(const float (&base)[VEC], const float (&m)[VEC], const float (&ref)[VEC],
                                            const float (&inv)[VEC], float (&f)[VEC]) {
#pragma unroll
  for (int v = 0; v < VEC; ++v)
    f[v] = m[v] == -kInf ? __fmul_rn(0.0f, inv[v]) : __fmul_rn(exp_diff(base[v], ref[v]), inv[v]);
}

// Normalise kept rows [begin, end): out = term * f per feature.
template <typename T, int VEC>
__device__ __forceinline__ void normalize_kept(const SharedRows<T, VEC> &src, T *__restrict__ out, int64_t d,
                                               int64_t col, int64_t begin, int64_t end, int64_t row_lane,
                                               int64_t step, const float (&f)[VEC]) {
  constexpr int U = kFoldUnroll;
  using Raw = typename VecIO<T, VEC>::Raw;
  constexpr int P = VEC / 2;
  unsigned long long f2[P];
#pragma unroll
  for (int j = 0; j < P; ++j) f2[j] = pack2(f[2 * j], f[2 * j + 1]);
  const int count = lane_rows(begin, end, row_lane, step);
  const auto cur = src.at(begin + row_lane, step);
  T *const o = out + (begin + row_lane) * d + col;
  const int64_t ostride = step * d;
  auto scale_row = [&](const Raw &raw, int k) {
    float x[VEC], y[VEC];
    VecIO<T, VEC>::unpack(raw, x);
#pragma unroll
    for (int j = 0; j < P; ++j) unpack2(mul2_rn(pack2(x[2 * j], x[2 * j + 1]), f2[j]), y[2 * j], y[2 * j + 1]);
    VecIO<T, VEC>::store(o + k * ostride, y);
  };
  int k = 0;
  for (; k + U <= count; k += U) {
    Raw raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) raw[u] = cur.raw(k + u);
#pragma unroll
    for (int u = 0; u < U; ++u) scale_row(raw[u], k + u);
  }
  for (; k < count; ++k) scale_row(cur.raw(k), k);
}

// Merge the row groups of each warp, then the NW warps, leaving the result
// for column lane cl in part[0][cl] (visible to every thread on return).
template <int OP, int VEC, int NW>
__device__ __forceinline__ void cta_merge(Acc<OP, VEC> &acc, Acc<OP, VEC> (*part)[32], int warp, int q, int cl,
                                          int G) {
  for (int m = 16; m >= G; m >>= 1) acc.shfl_xor_merge(m);
  __syncthreads();  // part[] of a previous use has been consumed
  if (q == 0) part[warp][cl] = acc;
  __syncthreads();
  if (warp == 0 && q == 0) {
    Acc<OP, VEC> total = part[0][cl];
#pragma unroll
    for (int w = 1; w < NW; ++w) total.merge(part[w][cl]);
    part[0][cl] = total;
  }
  __syncthreads();
}

// Merge the row groups of one warp; every lane of column cl gets the total.
template <int OP, int VEC>
__device__ __forceinline__ void warp_merge(Acc<OP, VEC> &acc, int G) {
  for (int m = 16; m >= G; m >>= 1) acc.shfl_xor_merge(m);
}

// Softmax statistics of a merged accumulator: reference and reciprocal of
// the total mass per feature.
template <int VEC>
__device__ __forceinline__ void stats_of(const Acc<OP_SOFTMAX, VEC> &acc, float (&ref)[VEC], float (&inv)[VEC]) {
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
    ref[v] = acc.st[v].r;
    inv[v] = stats_inverse(kahan_value(acc.st[v].s, acc.st[v].c));
  }
}

// Normalise one row's VEC features: e^(x - ref) * inv, packed in pairs.
template <int VEC>
__device__ __forceinline__ void normalize_vec(const float (&x)[VEC], float (&y)[VEC], const float (&ref)[VEC],
                                              const float (&inv)[VEC]) {
  if constexpr (VEC % 2 == 0) {
#pragma unroll
    for (int k = 0; k < VEC / 2; ++k) {
      const unsigned long long e =
          exp_diff2(pack2(x[2 * k], x[2 * k + 1]), pack2(ref[2 * k], ref[2 * k + 1]));
      unpack2(mul2_rn(e, pack2(inv[2 * k], inv[2 * k + 1])), y[2 * k], y[2 * k + 1]);
    }
  } else {
#pragma unroll
    for (int v = 0; v < VEC; ++v) y[v] = stats_normalize(x[v], ref[v], inv[v]);
  }
}

// Normalise rows [begin, end) (stride `step` from begin + row_lane) with
// the per-feature reference and reciprocal total; results to out (global).
template <typename T, int VEC, typename Src>
__device__ __forceinline__ void normalize_rows(const Src &src, T *__restrict__ out, int64_t d, int64_t col,
                                               int64_t begin, int64_t end, int64_t row_lane, int64_t step,
                                               const float (&ref)[VEC], const float (&inv)[VEC]) {
  constexpr int U = kFoldUnroll;
  using Raw = typename VecIO<T, VEC>::Raw;
  const int count = lane_rows(begin, end, row_lane, step);
  const auto cur = src.at(begin + row_lane, step);
  T *const o = out + (begin + row_lane) * d + col;
  const int64_t ostride = step * d;
  int k = 0;
  for (; k + U <= count; k += U) {
    Raw raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) raw[u] = cur.raw(k + u);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float x[VEC], y[VEC];
      VecIO<T, VEC>::unpack(raw[u], x);
      normalize_vec<VEC>(x, y, ref, inv);
      VecIO<T, VEC>::store(o + (k + u) * ostride, y);
    }
  }
  for (; k < count; ++k) {
    float x[VEC], y[VEC];
    VecIO<T, VEC>::unpack(cur.raw(k), x);
    normalize_vec<VEC>(x, y, ref, inv);
    VecIO<T, VEC>::store(o + k * ostride, y);
  }
}

}  // namespace rgb
