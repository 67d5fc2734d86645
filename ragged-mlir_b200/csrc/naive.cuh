// Block-per-segment schedule ("naive" strategy of the reference,
// lib/Conversion/ToGPU.cpp:1283-1349): one CTA per segment and column tile,
// no scratch, one launch.  It is the fallback the cost model can choose.
//
// Thread geometry (shared by every schedule, see geometry.h): a row of D
// features is C = D / VEC vector columns of VEC adjacent features (16-byte
// vectors when D allows); G = min(32, pow2ceil(C)) lanes cover one row, so a
// warp covers 32 / G rows per load and the CTA covers NW * 32 / G rows per
// step.  Column tiles of 32 vector columns are the grid's y dimension.
#pragma once

#include "common.cuh"

namespace rgb {

constexpr int kNaiveThreads = 256;
constexpr int kNaiveUnroll = 4;

template <typename T, typename OffT, int OP, int VEC>
__global__ void __launch_bounds__(kNaiveThreads)
naive_kernel(const T *__restrict__ values, const OffT *__restrict__ offsets, T *__restrict__ out,
             int64_t num_segments, int64_t d, int g_shift, int vec_cols) {
  constexpr int NW = kNaiveThreads / 32;
  constexpr int U = kNaiveUnroll;
  __shared__ Acc<OP, VEC> part[NW][32];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = 1 << g_shift;
  const int q = lane >> g_shift, cl = lane & (G - 1);
  const int64_t step = static_cast<int64_t>(NW) << (5 - g_shift);
  const int64_t row_lane = static_cast<int64_t>(warp) * (32 >> g_shift) + q;
  const int cv = blockIdx.y * 32 + cl;
  const bool active = cv < vec_cols;
  const int64_t col = static_cast<int64_t>(cv) * VEC;

  for (int64_t s = blockIdx.x; s < num_segments; s += gridDim.x) {
    const int64_t begin = static_cast<int64_t>(offsets[s]);
    const int64_t end = static_cast<int64_t>(offsets[s + 1]);
    Acc<OP, VEC> acc;
    acc.init();
    if (active) {
      int64_t r = begin + row_lane;
      for (; r + (U - 1) * step < end; r += U * step) {
        float x[U][VEC];
#pragma unroll
        for (int u = 0; u < U; ++u) VecIO<T, VEC>::load(values + (r + u * step) * d + col, x[u]);
        if constexpr (OP == OP_SOFTMAX) {
          acc.template fold_batch<U>(x);
        } else {
#pragma unroll
          for (int u = 0; u < U; ++u) acc.fold(x[u]);
        }
      }
      for (; r < end; r += step) {
        float x[VEC];
        VecIO<T, VEC>::load(values + r * d + col, x);
        acc.fold(x);
      }
    }
    // Row groups of the warp, then warps in a fixed order: deterministic.
    for (int m = 16; m >= G; m >>= 1) acc.shfl_xor_merge(m);
    __syncthreads();  // part[] of the previous segment has been consumed
    if (q == 0) part[warp][cl] = acc;
    __syncthreads();
    if (warp == 0) {
      acc = part[0][cl];
#pragma unroll
      for (int w = 1; w < NW; ++w) acc.merge(part[w][cl]);
      if constexpr (OP != OP_SOFTMAX) {
        if (q == 0 && active) {
          float y[VEC];
          acc.result(y);
          VecIO<T, VEC>::store(out + s * d + col, y);
        }
      } else {
        if (q == 0) part[0][cl] = acc;
      }
    }
    if constexpr (OP == OP_SOFTMAX) {
      __syncthreads();
      if (active && end > begin) {
        const Acc<OP, VEC> fin = part[0][cl];
        float ref[VEC], total[VEC];
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
          ref[v] = fin.st[v].r;
          total[v] = stats_inverse(kahan_value(fin.st[v].s, fin.st[v].c));
        }
        int64_t r = begin + row_lane;
        for (; r + (U - 1) * step < end; r += U * step) {
          float x[U][VEC];
#pragma unroll
          for (int u = 0; u < U; ++u) VecIO<T, VEC>::load(values + (r + u * step) * d + col, x[u]);
#pragma unroll
          for (int u = 0; u < U; ++u) {
            float y[VEC];
#pragma unroll
            for (int v = 0; v < VEC; ++v) y[v] = stats_normalize(x[u][v], ref[v], total[v]);
            VecIO<T, VEC>::store(out + (r + u * step) * d + col, y);
          }
        }
        for (; r < end; r += step) {
          float x[VEC], y[VEC];
          VecIO<T, VEC>::load(values + r * d + col, x);
#pragma unroll
          for (int v = 0; v < VEC; ++v) y[v] = stats_normalize(x[v], ref[v], total[v]);
          VecIO<T, VEC>::store(out + r * d + col, y);
        }
      }
    }
  }
}

}  // namespace rgb
