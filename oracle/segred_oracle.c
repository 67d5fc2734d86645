/*
 * segred_oracle.c -- TEST INFRASTRUCTURE ONLY (the CPU checker and the timed
 * CPU baseline; never linked into or called by the product library).
 *
 * A C, float64 restatement of the reference's NumPy oracle
 * (simon-jd/ragged-mlir, oracle/reference.py):
 *   sum      oracle/reference.py:78-79   (np.sum in float64; +0 for an empty segment)
 *   max      oracle/reference.py:80-82   (np.max, NaN propagates, -inf identity)
 *   softmax  oracle/reference.py:94-106  (exp(x - max) / sum, float64)
 *   abs-sum  sum of |x| per segment: the scale of the sum tolerance in
 *            oracle/reference.py:109-174 (np.abs(values) summed per segment)
 * Inputs are f32 or bf16 (raw uint16 bits) values[N, D] and i32/i64
 * offsets[B+1]; outputs are float64, exactly as the reference returns them.
 *
 * Work is split across OpenMP threads by equal ROW ranges, so one giant
 * segment does not serialise the run: every thread reduces the pieces of the
 * segments that intersect its rows, writes the segments that start and end
 * inside its range, and the pieces of segments that cross thread boundaries
 * are merged afterwards in thread order.  float64 accumulation makes the
 * merge order irrelevant at the f32/bf16 tolerances the oracle checks.
 *
 * Offsets are assumed valid (validate them with the Python port first).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { SO_SUM = 0, SO_MAX = 1, SO_SOFTMAX = 2, SO_ABSSUM = 3 };
enum { SO_F32 = 0, SO_BF16 = 1 };
enum { SO_I32 = 0, SO_I64 = 1 };

static inline double load_value(const void *values, int dtype, int64_t index) {
  if (dtype == SO_F32) return (double)((const float *)values)[index];
  uint32_t bits = (uint32_t)((const uint16_t *)values)[index] << 16;
  float f;
  memcpy(&f, &bits, sizeof f);
  return (double)f;
}

static inline int64_t load_offset(const void *offsets, int index_dtype, int64_t i) {
  return index_dtype == SO_I32 ? (int64_t)((const int32_t *)offsets)[i]
                               : ((const int64_t *)offsets)[i];
}

/* NaN-propagating maximum (np.maximum semantics). */
static inline double max_nan(double a, double b) {
  if (isnan(a) || isnan(b)) return NAN;
  return a > b ? a : b;
}

/* First segment s with offsets[s] >= row (lower bound over offsets[0..B]). */
static int64_t lower_bound(const void *offsets, int index_dtype, int64_t b, int64_t row) {
  int64_t lo = 0, hi = b + 1;
  while (lo < hi) {
    int64_t mid = lo + (hi - lo) / 2;
    if (load_offset(offsets, index_dtype, mid) < row) lo = mid + 1; else hi = mid;
  }
  return lo;
}

/* Reduction of rows [r0, r1) of every feature into acc[D].  kind SUM/MAX; for
 * the softmax denominator (kind == SO_SOFTMAX) acc += exp(x - shift[d]). */
static void fold_rows(const void *values, int dtype, int64_t d, int kind, int64_t r0, int64_t r1,
                      const double *shift, double *acc) {
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t base = r * d;
    if (kind == SO_SUM) {
      for (int64_t j = 0; j < d; ++j) acc[j] += load_value(values, dtype, base + j);
    } else if (kind == SO_MAX) {
      for (int64_t j = 0; j < d; ++j) acc[j] = max_nan(acc[j], load_value(values, dtype, base + j));
    } else if (kind == SO_ABSSUM) {
      for (int64_t j = 0; j < d; ++j) acc[j] += fabs(load_value(values, dtype, base + j));
    } else {
      for (int64_t j = 0; j < d; ++j) acc[j] += exp(load_value(values, dtype, base + j) - shift[j]);
    }
  }
}

static void combine(int kind, double *into, const double *piece, int64_t d) {
  for (int64_t j = 0; j < d; ++j)
    into[j] = kind == SO_MAX ? max_nan(into[j], piece[j]) : into[j] + piece[j];
}

/* Row-balanced segmented reduction (see file comment).  out is [B, D].
 * For kind == SO_SOFTMAX, ``shift`` is the [B, D] per-segment maximum. */
static int reduce_rows(int kind, int dtype, int index_dtype, int64_t n, int64_t d, int64_t b,
                       const void *values, const void *offsets, const double *shift, double *out,
                       int threads) {
  const double identity = kind == SO_MAX ? -INFINITY : 0.0;
  for (int64_t i = 0; i < b * d; ++i) out[i] = identity;
  if (n == 0 || b == 0) return 0;
  if (threads < 1) threads = 1;
  if ((int64_t)threads > n) threads = (int)n;
  /* Per thread: the piece of the segment that was open at the range start
   * (head) and of the segment still open at its end (tail). */
  double *head = (double *)calloc((size_t)threads * (size_t)d, sizeof(double));
  double *tail = (double *)calloc((size_t)threads * (size_t)d, sizeof(double));
  int64_t *head_seg = (int64_t *)malloc(sizeof(int64_t) * (size_t)threads);
  int64_t *tail_seg = (int64_t *)malloc(sizeof(int64_t) * (size_t)threads);
  if (!head || !tail || !head_seg || !tail_seg) {
    free(head); free(tail); free(head_seg); free(tail_seg);
    return 1;
  }
#pragma omp parallel num_threads(threads)
  {
    int t = 0;
#ifdef _OPENMP
    t = omp_get_thread_num();
#endif
    const int64_t r0 = n * t / threads, r1 = n * (t + 1) / threads;
    double *acc = (double *)malloc(sizeof(double) * (size_t)d);
    head_seg[t] = -1;
    tail_seg[t] = -1;
    /* The segment containing r0 (if it started before r0) is a head piece. */
    /* First segment starting at or after r0 (empty ones at r0 belong to this
     * thread); if none starts exactly at r0, the one before contains r0. */
    int64_t s = lower_bound(offsets, index_dtype, b, r0);
    if (load_offset(offsets, index_dtype, s) > r0) s -= 1;
    for (; s < b; ++s) {
      const int64_t begin = load_offset(offsets, index_dtype, s);
      const int64_t end = load_offset(offsets, index_dtype, s + 1);
      if (begin >= r1) break;
      const int64_t lo = begin > r0 ? begin : r0;
      const int64_t hi = end < r1 ? end : r1;
      for (int64_t j = 0; j < d; ++j) acc[j] = identity;
      fold_rows(values, dtype, d, kind, lo, hi, shift ? shift + s * d : NULL, acc);
      const int starts_before = begin < r0, ends_after = end > r1;
      if (!starts_before && !ends_after) {
        memcpy(out + s * d, acc, sizeof(double) * (size_t)d);
      } else if (starts_before) {
        head_seg[t] = s;
        memcpy(head + (int64_t)t * d, acc, sizeof(double) * (size_t)d);
        if (ends_after) tail_seg[t] = s;  /* spans the whole range */
      } else {
        tail_seg[t] = s;
        memcpy(tail + (int64_t)t * d, acc, sizeof(double) * (size_t)d);
      }
    }
    free(acc);
  }
  /* Merge crossing pieces in row order: a segment's pieces are the tail of
   * the thread where it starts and the heads of the following threads. */
  for (int t = 0; t < threads; ++t) {
    if (tail_seg[t] >= 0 && head_seg[t] != tail_seg[t])
      memcpy(out + tail_seg[t] * d, tail + (int64_t)t * d, sizeof(double) * (size_t)d);
  }
  for (int t = 0; t < threads; ++t) {
    if (head_seg[t] >= 0) combine(kind, out + head_seg[t] * d, head + (int64_t)t * d, d);
  }
  free(head); free(tail); free(head_seg); free(tail_seg);
  return 0;
}

/* Segmented sum, max or sum of |x|: out[B, D] float64.  Returns 0 on success. */
int so_segment_reduce(int op, int dtype, int index_dtype, int64_t n, int64_t d, int64_t b,
                      const void *values, const void *offsets, double *out, int threads) {
  if (op != SO_SUM && op != SO_MAX && op != SO_ABSSUM) return 2;
  return reduce_rows(op, dtype, index_dtype, n, d, b, values, offsets, NULL, out, threads);
}

/* Segmented softmax: out[N, D] float64 = exp(x - max) / sum(exp(x - max)). */
int so_segment_softmax(int dtype, int index_dtype, int64_t n, int64_t d, int64_t b,
                       const void *values, const void *offsets, double *out, int threads) {
  if (n == 0 || b == 0) return 0;
  double *maxima = (double *)malloc(sizeof(double) * (size_t)(b * d));
  double *totals = (double *)malloc(sizeof(double) * (size_t)(b * d));
  if (!maxima || !totals) { free(maxima); free(totals); return 1; }
  int status = reduce_rows(SO_MAX, dtype, index_dtype, n, d, b, values, offsets, NULL, maxima, threads);
  if (!status)
    status = reduce_rows(SO_SOFTMAX, dtype, index_dtype, n, d, b, values, offsets, maxima, totals, threads);
  if (!status) {
    if (threads < 1) threads = 1;
#pragma omp parallel num_threads(threads)
    {
      int t = 0;
#ifdef _OPENMP
      t = omp_get_thread_num();
#endif
      const int64_t r0 = n * t / threads, r1 = n * (t + 1) / threads;
      int64_t s = lower_bound(offsets, index_dtype, b, r0);
      if (load_offset(offsets, index_dtype, s) > r0) s -= 1;
      for (int64_t r = r0; r < r1; ++r) {
        while (load_offset(offsets, index_dtype, s + 1) <= r) ++s;
        for (int64_t j = 0; j < d; ++j) {
          const double x = load_value(values, dtype, r * d + j);
          out[r * d + j] = exp(x - maxima[s * d + j]) / totals[s * d + j];
        }
      }
    }
  }
  free(maxima);
  free(totals);
  return status;
}

int so_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
