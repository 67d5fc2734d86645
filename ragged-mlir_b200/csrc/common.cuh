// Shared device numerics and vector I/O for the sm_100a segmented kernels.
//
// Semantics follow the reference's specification (simon-jd/ragged-mlir,
// docs/semantics.md:49-67): f32 accumulation, sum identity +0, max identity
// -inf with NaN propagation, softmax columns that see NaN, +inf or only -inf
// become NaN.  The per-lane compensated sum restates the reference's
// `compensatedAdd` (lib/Conversion/ToGPU.cpp:377-387); the online softmax
// statistics restate its lagging-reference update and merge
// (ToGPU.cpp:486-557) in batched form.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

namespace rgb {

enum Op : int { OP_SUM = 0, OP_MAX = 1, OP_SOFTMAX = 2 };

constexpr float kInf = __builtin_huge_valf();

// ---------------------------------------------------------------- scalars --

// NaN-propagating maximum (IEEE 754-2019 maximum; PTX max.NaN).
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ bool is_finite(float x) { return fabsf(x) < kInf; }

// Compensated (Kahan) accumulation: the true running total is s - c.  The
// correction is cleared whenever the total stops being finite, so that
// +inf + finite stays +inf while +inf + -inf and NaN still poison s.
// Rounded intrinsics keep nvcc from contracting or reordering the steps.
__device__ __forceinline__ void kahan_add(float &s, float &c, float x) {
  const float y = __fsub_rn(x, c);
  const float t = __fadd_rn(s, y);
  const float z = __fsub_rn(__fsub_rn(t, s), y);
  c = is_finite(t) ? z : 0.0f;
  s = t;
}

// Same, for a batch whose total is known to stay finite (no check).
__device__ __forceinline__ void kahan_add_finite(float &s, float &c, float x) {
  const float y = __fsub_rn(x, c);
  const float t = __fadd_rn(s, y);
  c = __fsub_rn(__fsub_rn(t, s), y);
  s = t;
}

// Merge two compensated totals (s1 - c1) + (s2 - c2) with an error-free
// TwoSum of s1 + s2 (Knuth), keeping the merged correction.
__device__ __forceinline__ void kahan_merge(float &s1, float &c1, float s2, float c2) {
  const float t = __fadd_rn(s1, s2);
  const float bp = __fsub_rn(t, s1);
  const float ap = __fsub_rn(t, bp);
  const float e = __fadd_rn(__fsub_rn(s1, ap), __fsub_rn(s2, bp));  // t + e == s1 + s2
  const float c = __fsub_rn(__fadd_rn(c1, c2), e);
  c1 = is_finite(t) ? c : 0.0f;
  s1 = t;
}

__device__ __forceinline__ float kahan_value(float s, float c) {
  return is_finite(s) ? __fsub_rn(s, c) : s;
}

// exp for the softmax statistics and output.  CUDA's expf (accurate to a
// couple of ulp over the whole range) is called, never restated.
__device__ __forceinline__ float exp_f(float x) { return expf(x); }

// --------------------------------------------------- online softmax stats --
//
// State per feature: reference r, compensated mass (s, c) relative to r.
// A batch of values with batch maximum bm is folded as in the reference:
// the reference recentres only when it is empty (-inf), unordered (NaN) or
// when the maximum exceeds it by more than one, so every mass stays below
// e and earlier rounding errors are damped by each rescale.  A +inf anchor
// makes the column NaN; a -inf anchor means every value so far was -inf and
// adds no mass.

struct Stats {
  float r, s, c;
};

__device__ __forceinline__ Stats stats_empty() { return Stats{-kInf, 0.0f, 0.0f}; }

// Fold `count` values x[0..count) (count is a compile-time bound; entries
// beyond the valid ones must be -inf) into st.
template <int COUNT>
__device__ __forceinline__ void stats_fold(Stats &st, const float (&x)[COUNT]) {
  float bm = x[0];
#pragma unroll
  for (int i = 1; i < COUNT; ++i) bm = max_nan(bm, x[i]);
  const float m = max_nan(st.r, bm);
  const bool empty = st.r == -kInf;
  const bool unordered = (st.r != st.r) || (bm != bm);
  const bool advance = __fsub_rn(m, st.r) > 1.0f;
  const float anchor = (empty || unordered || advance) ? m : st.r;
  if (anchor != st.r) {
    if (empty) {
      st.s = 0.0f;
      st.c = 0.0f;
    } else {
      const float scale = exp_f(__fsub_rn(st.r, anchor));
      st.s = __fmul_rn(st.s, scale);
      st.c = __fmul_rn(st.c, scale);
    }
    st.r = anchor;
  }
  if (anchor == kInf || anchor != anchor) {
    st.s = __int_as_float(0x7fffffff);
    st.c = 0.0f;
    return;
  }
  if (anchor == -kInf) return;  // every value so far is -inf: no mass
#pragma unroll
  for (int i = 0; i < COUNT; ++i) kahan_add_finite(st.s, st.c, exp_f(__fsub_rn(x[i], anchor)));
}

// Merge statistics b into a (ToGPU.cpp:486-508 `mergeStatistics`, with the
// compensations folded in): the larger reference wins, the other mass is
// rescaled; -inf references carry no mass; a +inf reference gives NaN.
__device__ __forceinline__ void stats_merge(Stats &a, const Stats &b) {
  const float m = max_nan(a.r, b.r);
  float sa = kahan_value(a.s, a.c), sb = kahan_value(b.s, b.c);
  float total;
  if (a.r == -kInf) {
    total = sb;
  } else if (b.r == -kInf) {
    total = sa;
  } else {
    total = __fadd_rn(__fmul_rn(sa, exp_f(__fsub_rn(a.r, m))),
                      __fmul_rn(sb, exp_f(__fsub_rn(b.r, m))));
  }
  if (m == kInf) total = __int_as_float(0x7fffffff);
  a.r = m;
  a.s = total;
  a.c = 0.0f;
}

// Final normalisation of one value with the merged statistics.
__device__ __forceinline__ float stats_normalize(float x, float r, float total) {
  return __fdiv_rn(exp_f(__fsub_rn(x, r)), total);
}

// ------------------------------------------------------------- vector I/O --

template <typename T>
struct Elem;
template <>
struct Elem<float> {
  static constexpr int kBytes = 4;
};
template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kBytes = 2;
};

__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // RNE, NaN stays NaN
  return *reinterpret_cast<uint32_t *>(&v);
}

// Global loads of VEC elements, read-only path.  `Raw` is the loaded
// register form (kept while loads are in flight), `unpack` converts it to
// f32; `load` does both.
template <typename T, int VEC>
struct VecIO;

template <int VEC>
struct VecIO<float, VEC> {
  using Raw = typename std::conditional<VEC == 4, float4, typename std::conditional<VEC == 2, float2, float>::type>::type;
  static __device__ __forceinline__ Raw load_raw(const float *p) { return __ldg(reinterpret_cast<const Raw *>(p)); }
  static __device__ __forceinline__ void unpack(const Raw &v, float (&x)[VEC]) {
    if constexpr (VEC == 4) {
      x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
    } else if constexpr (VEC == 2) {
      x[0] = v.x; x[1] = v.y;
    } else {
      x[0] = v;
    }
  }
  static __device__ __forceinline__ void load(const float *p, float (&x)[VEC]) { unpack(load_raw(p), x); }
  static __device__ __forceinline__ void store(float *p, const float (&x)[VEC]) {
    if constexpr (VEC == 4) {
      *reinterpret_cast<float4 *>(p) = make_float4(x[0], x[1], x[2], x[3]);
    } else if constexpr (VEC == 2) {
      *reinterpret_cast<float2 *>(p) = make_float2(x[0], x[1]);
    } else {
      *p = x[0];
    }
  }
};

template <int VEC>
struct VecIO<__nv_bfloat16, VEC> {
  using Raw = typename std::conditional<
      VEC == 8, uint4,
      typename std::conditional<VEC == 4, uint2,
                                typename std::conditional<VEC == 2, unsigned int, unsigned short>::type>::type>::type;
  static __device__ __forceinline__ Raw load_raw(const __nv_bfloat16 *p) {
    return __ldg(reinterpret_cast<const Raw *>(p));
  }
  static __device__ __forceinline__ void unpack(const Raw &v, float (&x)[VEC]) {
    if constexpr (VEC == 8) {
      x[0] = bf16_lo(v.x); x[1] = bf16_hi(v.x); x[2] = bf16_lo(v.y); x[3] = bf16_hi(v.y);
      x[4] = bf16_lo(v.z); x[5] = bf16_hi(v.z); x[6] = bf16_lo(v.w); x[7] = bf16_hi(v.w);
    } else if constexpr (VEC == 4) {
      x[0] = bf16_lo(v.x); x[1] = bf16_hi(v.x); x[2] = bf16_lo(v.y); x[3] = bf16_hi(v.y);
    } else if constexpr (VEC == 2) {
      x[0] = bf16_lo(v); x[1] = bf16_hi(v);
    } else {
      x[0] = __uint_as_float(static_cast<uint32_t>(v) << 16);
    }
  }
  static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float (&x)[VEC]) { unpack(load_raw(p), x); }
  static __device__ __forceinline__ void store(__nv_bfloat16 *p, const float (&x)[VEC]) {
    if constexpr (VEC == 8) {
      *reinterpret_cast<uint4 *>(p) = make_uint4(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]),
                                                 pack_bf16x2(x[4], x[5]), pack_bf16x2(x[6], x[7]));
    } else if constexpr (VEC == 4) {
      *reinterpret_cast<uint2 *>(p) = make_uint2(pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]));
    } else if constexpr (VEC == 2) {
      *reinterpret_cast<uint32_t *>(p) = pack_bf16x2(x[0], x[1]);
    } else {
      *p = __float2bfloat16_rn(x[0]);
    }
  }
};

// --------------------------------------------------------------- cp.async --
//
// Asynchronous global -> shared copies of 4, 8 or 16 bytes (L1 bypassed for
// 16); completion is per thread (commit / wait_group).

template <int BYTES>
__device__ __forceinline__ void cp_async(uint32_t smem_addr, const void *gmem) {
  static_assert(BYTES == 4 || BYTES == 8 || BYTES == 16 || BYTES == 2, "cp.async size");
  if constexpr (BYTES == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr), "l"(gmem) : "memory");
  } else if constexpr (BYTES == 8) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(smem_addr), "l"(gmem) : "memory");
  } else if constexpr (BYTES == 4) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_addr), "l"(gmem) : "memory");
  } else {
    // 2-byte elements (bf16, one per thread): a plain load and shared store.
    *reinterpret_cast<unsigned short *>(__cvta_shared_to_generic(smem_addr)) =
        __ldg(reinterpret_cast<const unsigned short *>(gmem));
  }
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// ------------------------------------------------------------ accumulators --
//
// One accumulator per thread covers VEC adjacent features of one column.

template <int OP, int VEC>
struct Acc;

template <int VEC>
struct Acc<OP_SUM, VEC> {
  float s[VEC], c[VEC];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int v = 0; v < VEC; ++v) { s[v] = 0.0f; c[v] = 0.0f; }
  }
  __device__ __forceinline__ void fold(const float (&x)[VEC]) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) kahan_add(s[v], c[v], x[v]);
  }
  __device__ __forceinline__ void merge(const Acc &o) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) kahan_merge(s[v], c[v], o.s[v], o.c[v]);
  }
  __device__ __forceinline__ void shfl_xor_merge(int lane_mask) {
    Acc o;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      o.s[v] = __shfl_xor_sync(0xffffffffu, s[v], lane_mask);
      o.c[v] = __shfl_xor_sync(0xffffffffu, c[v], lane_mask);
    }
    merge(o);
  }
  __device__ __forceinline__ void result(float (&y)[VEC]) const {
#pragma unroll
    for (int v = 0; v < VEC; ++v) y[v] = kahan_value(s[v], c[v]);
  }
};

template <int VEC>
struct Acc<OP_MAX, VEC> {
  float m[VEC];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int v = 0; v < VEC; ++v) m[v] = -kInf;
  }
  __device__ __forceinline__ void fold(const float (&x)[VEC]) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) m[v] = max_nan(m[v], x[v]);
  }
  __device__ __forceinline__ void merge(const Acc &o) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) m[v] = max_nan(m[v], o.m[v]);
  }
  __device__ __forceinline__ void shfl_xor_merge(int lane_mask) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) m[v] = max_nan(m[v], __shfl_xor_sync(0xffffffffu, m[v], lane_mask));
  }
  __device__ __forceinline__ void result(float (&y)[VEC]) const {
#pragma unroll
    for (int v = 0; v < VEC; ++v) y[v] = m[v];
  }
};

template <int VEC>
struct Acc<OP_SOFTMAX, VEC> {
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
  __device__ __forceinline__ void merge(const Acc &o) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) stats_merge(st[v], o.st[v]);
  }
  __device__ __forceinline__ void shfl_xor_merge(int lane_mask) {
    Acc o;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      o.st[v].r = __shfl_xor_sync(0xffffffffu, st[v].r, lane_mask);
      o.st[v].s = __shfl_xor_sync(0xffffffffu, st[v].s, lane_mask);
      o.st[v].c = __shfl_xor_sync(0xffffffffu, st[v].c, lane_mask);
    }
    merge(o);
  }
};

}  // namespace rgb
