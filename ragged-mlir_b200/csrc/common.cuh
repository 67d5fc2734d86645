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

// e^t for the softmax statistics and output, as 2^(t * log2 e) on the SFU
// (PTX ex2.approx.ftz.f32: about 2 ulp; results below 2^-126 flush to +0).
// t = x - r is rounded once and the product once, so a term e^t carries a
// relative error of about |t| * 2^-23: under 1e-5 for every term the f32
// softmax tolerance (|a - ref| <= 1e-5 |ref| + FLT_MIN) does not already
// absorb.  One SFU instruction and two FMA-pipe instructions per term keep
// the D=128 bf16 softmax below the HBM time on B200.
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float exp2_sfu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float exp_diff(float x, float r) { return exp2_sfu(__fmul_rn(__fsub_rn(x, r), kLog2e)); }

// Packed pairs on sm_100's two-wide FP32 pipe (add/sub/mul.rn.f32x2): one
// instruction per two lanes' worth of work, each half rounded exactly as
// the scalar __fadd_rn / __fsub_rn / __fmul_rn.
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(unsigned long long v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long add2_rn(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long sub2_rn(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long mul2_rn(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// e^(x - r) for two features at once: the packed subtraction and scaling,
// then one SFU exponential per half (same rounding as exp_diff).
__device__ __forceinline__ unsigned long long exp_diff2(unsigned long long x, unsigned long long r) {
  const unsigned long long t = mul2_rn(sub2_rn(x, r), pack2(kLog2e, kLog2e));
  float lo, hi;
  unpack2(t, lo, hi);
  return pack2(exp2_sfu(lo), exp2_sfu(hi));
}

// --------------------------------------------------- online softmax stats --
//
// State per feature: reference r, compensated mass (s, c) relative to r.
// A batch of values with batch maximum bm is folded as in the reference:
// the reference recentres only when it is empty (-inf), unordered (NaN) or
// when the maximum exceeds it by more than one, so every term stays below
// e and earlier rounding errors are damped by each rescale.  A +inf anchor
// makes the column NaN; a -inf anchor means every value so far was -inf and
// adds no mass.  The batch's terms are summed plainly (each is at most e)
// and the batch total is added with compensation.

struct Stats {
  float r, s, c;
};

__device__ __forceinline__ Stats stats_empty() { return Stats{-kInf, 0.0f, 0.0f}; }

// Move the reference for a batch whose maximum is bm (the first step of
// stats_fold).  Afterwards the batch's terms are e^(x - st.r), unless st.r
// is -inf (no mass: every value so far is -inf) or not finite (the column
// is NaN already).
__device__ __forceinline__ void stats_recenter(Stats &st, float bm) {
  const float m = max_nan(st.r, bm);
  const bool empty = st.r == -kInf;
  const bool unordered = (st.r != st.r) || (bm != bm);
  const bool advance = __fsub_rn(m, st.r) > 1.0f;
  if (empty || unordered || advance) {
    if (empty) {
      st.s = 0.0f;
      st.c = 0.0f;
    } else {
      const float scale = exp_diff(st.r, m);
      st.s = __fmul_rn(st.s, scale);
      st.c = __fmul_rn(st.c, scale);
    }
    st.r = m;
    if (m == kInf || m != m) {
      st.s = __int_as_float(0x7fffffff);
      st.c = 0.0f;
    }
  }
}

__device__ __forceinline__ bool stats_has_mass(const Stats &st) { return st.r != -kInf && is_finite(st.r); }

// Fold `count` values x[0..count) (count is a compile-time bound; entries
// beyond the valid ones must be -inf) into st.
template <int COUNT>
__device__ __forceinline__ void stats_fold(Stats &st, const float (&x)[COUNT]) {
  float bm = x[0];
#pragma unroll
  for (int i = 1; i < COUNT; ++i) bm = max_nan(bm, x[i]);
  stats_recenter(st, bm);
  if (!stats_has_mass(st)) return;  // no mass yet, or the column is already NaN
  float p = exp_diff(x[0], st.r);
#pragma unroll
  for (int i = 1; i < COUNT; ++i) p = __fadd_rn(p, exp_diff(x[i], st.r));
  kahan_add_finite(st.s, st.c, p);
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
    total = __fadd_rn(__fmul_rn(sa, exp_diff(a.r, m)), __fmul_rn(sb, exp_diff(b.r, m)));
  }
  if (m == kInf) total = __int_as_float(0x7fffffff);
  a.r = m;
  a.s = total;
  a.c = 0.0f;
}

// Reciprocal of a column's total mass (once per column; IEEE rounded).
__device__ __forceinline__ float stats_inverse(float total) { return __frcp_rn(total); }

// Final normalisation of one value with the merged reference r and the
// reciprocal of the total mass: e^(x - r) / total within 2 ulp + the term's
// error.  NaN, +inf and all -inf columns come out NaN through the
// arithmetic (NaN terms, NaN total, or 0 * inf).
__device__ __forceinline__ float stats_normalize(float x, float r, float inv_total) {
  return __fmul_rn(exp_diff(x, r), inv_total);
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

// ------------------------------------------------ bulk copies (TMA, 1-D) --
//
// cp.async.bulk moves a contiguous, 16-byte aligned block of global memory
// (a multiple of 16 bytes) into this CTA's shared memory and signals an
// mbarrier with the byte count: one instruction keeps tens of KB in flight.
// No cluster multicast form is used anywhere in this library.

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make barrier initialisation and earlier generic-proxy shared-memory
// accesses visible to the asynchronous (bulk copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// Arrive (count 1) and expect `bytes` of transactions on this phase.
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_copy_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(smem_dst)),
               "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Acquire load of a counter other CTAs increment (a spin-wait's poll).
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait for phase `parity` of `bar` (each try_wait itself suspends
// for a while); false after the limit, so a lost transaction cannot hang
// the GPU.
constexpr int kMbarWaitLimit = 1 << 22;
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  for (int i = 0; i < kMbarWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
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
  // U rows summed plainly, then added with compensation.
  template <int U>
  __device__ __forceinline__ void fold_batch(const float (&x)[U][VEC]) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      float p = x[0][v];
#pragma unroll
      for (int u = 1; u < U; ++u) p = __fadd_rn(p, x[u][v]);
      kahan_add(s[v], c[v], p);
    }
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
  template <int U>
  __device__ __forceinline__ void fold_batch(const float (&x)[U][VEC]) {
#pragma unroll
    for (int u = 0; u < U; ++u) fold(x[u]);
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

// ------------------------------------------------------ input transform --

// The reference's input transform (ProgramSpec scale and additive softmax
// mask; its lib/Conversion/ToGPU.cpp:604-618 loadInput) applied as rows
// are loaded: x = f32(v), then x * scale when scaled, then + mask, each
// rounded to f32 with no fused multiply-add, so the results equal those of
// a schedule run on materialised f32 logits.  `mask` (f32 [N][D], 16-byte
// aligned rows) is null when there is none.
struct Xform {
  const float *mask;
  int64_t d;
  float scale;
  int scaled;
};

// This thread's mask vector of row r (VEC floats from column col), loaded
// in pieces of up to 16 bytes (the mask rows are aligned to VEC floats).
template <int VEC>
struct MaskVec {
  using Piece = typename std::conditional<VEC % 4 == 0, float4,
                                          typename std::conditional<VEC % 2 == 0, float2, float>::type>::type;
  static constexpr int kPer = sizeof(Piece) / 4;
  Piece part[VEC / kPer];
  __device__ __forceinline__ float get(int v) const {
    const Piece &p = part[v / kPer];
    if constexpr (kPer == 4) {
      switch (v % 4) {
        case 0: return p.x;
        case 1: return p.y;
        case 2: return p.z;
        default: return p.w;
      }
    } else if constexpr (kPer == 2) {
      return v % 2 == 0 ? p.x : p.y;
    } else {
      return p;
    }
  }
};

template <int VEC>
__device__ __forceinline__ MaskVec<VEC> load_mask(const Xform &xf, int64_t r, int64_t col) {
  using M = MaskVec<VEC>;
  M m;
  const typename M::Piece *p = reinterpret_cast<const typename M::Piece *>(xf.mask + r * xf.d + col);
#pragma unroll
  for (int i = 0; i < VEC / M::kPer; ++i) m.part[i] = __ldg(p + i);
  return m;
}

template <int VEC>
__device__ __forceinline__ void apply_xform(float (&x)[VEC], const Xform &xf, const MaskVec<VEC> &m) {
  if (xf.scaled) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) x[v] = __fmul_rn(x[v], xf.scale);
  }
  if (xf.mask) {
#pragma unroll
    for (int v = 0; v < VEC; ++v) x[v] = __fadd_rn(x[v], m.get(v));
  }
}

}  // namespace rgb
