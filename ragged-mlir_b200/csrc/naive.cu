// Instantiation and launch of the block-per-segment schedule.
#include "internal.h"
#include "naive.cuh"

namespace rgb {

namespace {

template <typename T, typename OffT, int OP, int VEC>
int launch_typed(const Problem &p, const Geometry &g, cudaStream_t stream, rg_report *report) {
  const int64_t max_grid_x = 2147483647LL;
  dim3 grid(static_cast<unsigned>(p.b < max_grid_x ? p.b : max_grid_x), g.col_tiles, 1);
  naive_kernel<T, OffT, OP, VEC><<<grid, kNaiveThreads, 0, stream>>>(
      static_cast<const T *>(p.values), static_cast<const OffT *>(p.offsets), static_cast<T *>(p.out),
      p.b, p.d, g.g_shift, g.vec_cols);
  record_launch(report, K_NAIVE, grid, kNaiveThreads, 0);
  return check_cuda(cudaGetLastError(), "naive_kernel launch");
}

template <typename T, typename OffT, int OP>
int launch_vec(const Problem &p, const Geometry &g, cudaStream_t stream, rg_report *report) {
  switch (g.vec) {
    case 1: return launch_typed<T, OffT, OP, 1>(p, g, stream, report);
    case 2: return launch_typed<T, OffT, OP, 2>(p, g, stream, report);
    case 4: return launch_typed<T, OffT, OP, 4>(p, g, stream, report);
    case 8:
      if constexpr (sizeof(T) == 2) return launch_typed<T, OffT, OP, 8>(p, g, stream, report);
      break;
  }
  return fail(RG_ERR_INVALID_ARGUMENT, "unsupported vector width");
}

template <typename T, typename OffT>
int launch_op(const Problem &p, const Geometry &g, cudaStream_t stream, rg_report *report) {
  switch (p.op) {
    case RG_OP_SUM: return launch_vec<T, OffT, OP_SUM>(p, g, stream, report);
    case RG_OP_MAX: return launch_vec<T, OffT, OP_MAX>(p, g, stream, report);
    case RG_OP_SOFTMAX: return launch_vec<T, OffT, OP_SOFTMAX>(p, g, stream, report);
  }
  return fail(RG_ERR_INVALID_ARGUMENT, "unknown op");
}

template <typename T>
int launch_index(const Problem &p, const Geometry &g, cudaStream_t stream, rg_report *report) {
  return p.index_dtype == RG_INDEX_I32 ? launch_op<T, int32_t>(p, g, stream, report)
                                       : launch_op<T, int64_t>(p, g, stream, report);
}

}  // namespace

int launch_naive(const Problem &p, const Geometry &g, cudaStream_t stream, rg_report *report) {
  if (p.b == 0) return RG_OK;
  return p.dtype == RG_DTYPE_F32 ? launch_index<float>(p, g, stream, report)
                                 : launch_index<__nv_bfloat16>(p, g, stream, report);
}

}  // namespace rgb
