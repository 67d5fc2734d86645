// Planning, workspace layout and launch of the row-balanced schedule.
#include <map>
#include <mutex>
#include <utility>

#include "internal.h"
#include "rowbal.cuh"

namespace rgb {

namespace {
std::mutex g_occupancy_mutex;
std::map<std::pair<const void *, int>, int> g_occupancy;  // (kernel, device) -> blocks per SM
}  // namespace

// Resident CTAs per SM of a row-balanced kernel (`smem` bytes of dynamic
// shared memory), queried once per (kernel, device) and cached.
int rowbal_occupancy(const void *kernel, int device, int threads, int *blocks, int smem) {
  const auto key = std::make_pair(kernel, device);
  std::lock_guard<std::mutex> lock(g_occupancy_mutex);
  auto it = g_occupancy.find(key);
  if (it != g_occupancy.end()) {
    *blocks = it->second;
    return RG_OK;
  }
  int n = 0;
  int status = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem),
                      "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  if (status) return status;
  g_occupancy[key] = n < 1 ? 1 : n;
  *blocks = g_occupancy[key];
  return RG_OK;
}

namespace {

// Resident CTAs per SM requested from ptxas: 3 for sum and max; the softmax
// statistics (3 floats per feature) get the registers of 2.
constexpr int minb_of(int op) { return op == OP_SOFTMAX ? 2 : RowbalTuning::kMinBlocks; }

template <typename T, typename OffT, int OP, int VEC, bool XF = false>
const void *kernel_ptr() {
  return reinterpret_cast<const void *>(
      &rowbal_kernel<T, OffT, OP, VEC, RowbalTuning::kUnroll, RowbalTuning::kDoubleBuffer, minb_of(OP), XF>);
}

// Narrow rows that pack whole rows into 16-byte packets (2, 4, 8 or 16 bytes
// a row) take the packed kernel; VEC equals D for them.
bool packs(const Problem &p, const Geometry &g) {
  const int64_t row_bytes = p.d * elem_bytes(p.dtype);
  return !(p.flags & RG_FLAG_NO_VECTORIZE) && row_bytes <= 16 && 16 % row_bytes == 0 && g.vec == p.d;
}

// The packed kernel, its staging area (above the 48 KB default of dynamic
// shared memory) allowed on the current device; null where it does not apply.
template <typename T, typename OffT, int OP, int VEC>
const void *packed_ptr(int *status) {
  *status = RG_OK;
  if constexpr (VEC * sizeof(T) <= 16 && OP != OP_SOFTMAX) {
    const void *kernel = reinterpret_cast<const void *>(&rowbal_packed_kernel<T, OffT, OP, VEC>);
    *status = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPackedStageBytes),
                         "cudaFuncSetAttribute(rowbal_packed_kernel)");
    return kernel;
  }
  return nullptr;
}

constexpr int64_t kAlign = 256;
int64_t align_up(int64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Virtual CTAs per resident CTA of the row-balanced kernel: the kernel's
// CTAs take virtual CTAs from a counter, so a slower SM takes fewer.  Up
// to 8, one per 16K path items of a CTA's share: a small call keeps one
// static wave (a virtual CTA's start, its merge-path searches, is not free).
int64_t virtual_per_cta(int64_t path, int64_t resident) {
  const int64_t k = path / (resident * 16384);
  return k < 1 ? 1 : (k > 8 ? 8 : k);
}

struct Plan {
  int64_t packed_ctas;  // packed narrow-row kernel: one static wave
  int64_t vctas;        // row-balanced kernel: virtual CTAs ...
  int64_t grid;         // ... taken by this many resident CTAs (per column tile)
  int64_t pieces_bytes, meta_bytes, counter;  // workspace: pieces, metadata, claim counter
  int64_t stats, stats_bytes;                  // softmax statistics
};

// Units of 8 to 64 path items (rowbal_wanted_ctas); the packed kernel runs one
// resident wave, the row-balanced kernel kVirtualPerCta virtual CTAs per
// resident CTA.
int make_plan(const Problem &p, const Geometry &g, const void *kernel, const void *packed, Plan *plan) {
  DeviceProps dev;
  int status = device_props(&dev);
  if (status) return status;
  int per_sm = 0;
  status = rowbal_occupancy(kernel, dev.device, kRowbalThreads, &per_sm);
  if (status) return status;
  const int units_per_cta = (kRowbalThreads / 32) << (5 - g.g_shift);
  const int64_t path = p.n + p.b;
  int64_t resident = static_cast<int64_t>(per_sm) * dev.sm_count / g.col_tiles;
  if (resident < 1) resident = 1;
  const int64_t wanted = rowbal_wanted_ctas(path, resident, units_per_cta);
  int64_t vctas = resident * virtual_per_cta(path, resident);
  if (vctas > wanted) vctas = wanted;
  plan->vctas = vctas;
  plan->grid = resident < vctas ? resident : vctas;
  plan->packed_ctas = 0;
  if (packed) {
    int packed_per_sm = 0;
    status = rowbal_occupancy(packed, dev.device, kRowbalThreads, &packed_per_sm, kPackedStageBytes);
    if (status) return status;
    int64_t ctas = static_cast<int64_t>(packed_per_sm) * dev.sm_count;
    const int64_t packed_wanted = rowbal_wanted_ctas(path, ctas, kRowbalThreads);
    if (ctas > packed_wanted) ctas = packed_wanted;
    plan->packed_ctas = ctas < 1 ? 1 : ctas;
  }
  const int64_t slots = plan->vctas > plan->packed_ctas ? plan->vctas : plan->packed_ctas;
  const int width = p.op == RG_OP_MAX ? 1 : 2;
  plan->pieces_bytes = align_up(slots * 2 * width * p.d * static_cast<int64_t>(sizeof(float)));
  plan->meta_bytes = align_up(slots * static_cast<int64_t>(sizeof(UnitMeta)));
  plan->counter = plan->pieces_bytes + plan->meta_bytes;
  // Softmax: the statistics pass leaves (reference, total) per segment and
  // feature in [B][2][D] f32 for the normalise pass.
  plan->stats = plan->counter + kAlign;
  plan->stats_bytes = p.op == RG_OP_SOFTMAX ? align_up(p.b * 2 * p.d * static_cast<int64_t>(sizeof(float))) : 0;
  return RG_OK;
}

// XF (softmax only): the input transform `xf` fused into the statistics and
// normalise passes' loads.
template <typename T, typename OffT, int OP, int VEC, bool XF = false>
int run_typed(const Problem &p, const Geometry &g, void *workspace, int64_t *bytes, cudaStream_t stream,
              rg_report *report, const Xform &xf = Xform{}) {
  static_assert(!XF || OP == OP_SOFTMAX, "the fused transform is a softmax route");
  Plan plan;
  int status = RG_OK;
  const void *packed = XF ? nullptr : (packs(p, g) ? packed_ptr<T, OffT, OP, VEC>(&status) : nullptr);
  if (status) return status;
  status = make_plan(p, g, kernel_ptr<T, OffT, OP, VEC, XF>(), packed, &plan);
  if (status) return status;
  if (bytes) {
    *bytes = plan.stats + plan.stats_bytes;
    return RG_OK;
  }
  float *pieces = static_cast<float *>(workspace);
  UnitMeta *meta = reinterpret_cast<UnitMeta *>(static_cast<char *>(workspace) + plan.pieces_bytes);
  if constexpr (VEC * sizeof(T) <= 16 && OP != OP_SOFTMAX) {
    if (packed && reinterpret_cast<uintptr_t>(p.values) % 16 == 0) {
      const int64_t ctas = plan.packed_ctas;
      dim3 grid(static_cast<unsigned>(ctas), 1, 1);
      rowbal_packed_kernel<T, OffT, OP, VEC><<<grid, kRowbalThreads, kPackedStageBytes, stream>>>(
          static_cast<const T *>(p.values), static_cast<const OffT *>(p.offsets), static_cast<T *>(p.out), p.n, p.b,
          ctas * kRowbalThreads, pieces, meta);
      record_launch(report, K_ROWBAL_PACKED, grid, kRowbalThreads, kPackedStageBytes);
      status = check_cuda(cudaGetLastError(), "rowbal_packed_kernel launch");
      if (status || ctas < 2) return status;
      dim3 fix_grid(static_cast<unsigned>(ctas), 1, 1);
      rowbal_fixup_kernel<T, OP, VEC><<<fix_grid, kFixupThreads, 0, stream>>>(static_cast<T *>(p.out), p.d,
                                                                              g.vec_cols, ctas, pieces, meta, nullptr);
      record_launch(report, K_ROWBAL_FIXUP, fix_grid, kFixupThreads, 0);
      return check_cuda(cudaGetLastError(), "rowbal_fixup_kernel launch");
    }
  }
  // Claims only when there are more virtual CTAs than resident ones; one
  // static wave needs no counter (and no memset).
  unsigned long long *counter = nullptr;
  if (plan.vctas > plan.grid) {
    counter = reinterpret_cast<unsigned long long *>(static_cast<char *>(workspace) + plan.counter);
    status = check_cuda(cudaMemsetAsync(counter, 0, sizeof *counter, stream), "cudaMemsetAsync");
    if (status) return status;
    if (report) report->memsets += 1;
  }
  const int64_t units = plan.vctas * ((kRowbalThreads / 32) << (5 - g.g_shift));
  // Sum and max write out; the softmax statistics pass writes the statistics buffer.
  T *const target = OP == OP_SOFTMAX ? reinterpret_cast<T *>(static_cast<char *>(workspace) + plan.stats)
                                     : static_cast<T *>(p.out);
  dim3 grid(static_cast<unsigned>(plan.grid), g.col_tiles, 1);
  rowbal_kernel<T, OffT, OP, VEC, RowbalTuning::kUnroll, RowbalTuning::kDoubleBuffer, minb_of(OP), XF>
      <<<grid, kRowbalThreads, kRowbalSmem, stream>>>(
      static_cast<const T *>(p.values), static_cast<const OffT *>(p.offsets), target, p.n, p.b,
      p.d, g.g_shift, g.vec_cols, units, pieces, meta, RowWindow{0, p.n, 1}, counter, xf);
  record_launch(report, K_ROWBAL, grid, kRowbalThreads, kRowbalSmem);
  status = check_cuda(cudaGetLastError(), "rowbal_kernel launch");
  if (status) return status;
  if (plan.vctas >= 2) {
    dim3 fix_grid(static_cast<unsigned>(plan.vctas), g.col_tiles, 1);
    rowbal_fixup_kernel<T, OP, VEC><<<fix_grid, kFixupThreads, 0, stream>>>(target, p.d, g.vec_cols, plan.vctas,
                                                                            pieces, meta, nullptr);
    record_launch(report, K_ROWBAL_FIXUP, fix_grid, kFixupThreads, 0);
    status = check_cuda(cudaGetLastError(), "rowbal_fixup_kernel launch");
    if (status) return status;
  }
  if constexpr (OP == OP_SOFTMAX) {
    if (p.n > 0) {
      const int units_per_cta = (kRowbalThreads / 32) << (5 - g.g_shift);
      int64_t ctas = plan.grid;
      const int64_t wanted = (p.n + 16 * units_per_cta - 1) / (16 * units_per_cta);  // >= 16 rows per unit
      if (ctas > wanted) ctas = wanted;
      dim3 ngrid(static_cast<unsigned>(ctas), g.col_tiles, 1);
      rowbal_normalize_kernel<T, OffT, VEC, 8, XF><<<ngrid, kRowbalThreads, 0, stream>>>(
          static_cast<const T *>(p.values), static_cast<const OffT *>(p.offsets), static_cast<T *>(p.out),
          reinterpret_cast<const float *>(target), p.n, p.b, p.d, g.g_shift, g.vec_cols, ctas * units_per_cta,
          0, 0, 0, xf);
      record_launch(report, K_ROWBAL_NORMALIZE, ngrid, kRowbalThreads, 0);
      status = check_cuda(cudaGetLastError(), "rowbal_normalize_kernel launch");
    }
  }
  return status;
}

template <typename T, typename OffT, int OP>
int run_vec(const Problem &p, const Geometry &g, void *ws, int64_t *bytes, cudaStream_t s, rg_report *r) {
  switch (g.vec) {
    case 1: return run_typed<T, OffT, OP, 1>(p, g, ws, bytes, s, r);
    case 2: return run_typed<T, OffT, OP, 2>(p, g, ws, bytes, s, r);
    case 4: return run_typed<T, OffT, OP, 4>(p, g, ws, bytes, s, r);
    case 8:
      if constexpr (sizeof(T) == 2) return run_typed<T, OffT, OP, 8>(p, g, ws, bytes, s, r);
      break;
  }
  return fail(RG_ERR_INVALID_ARGUMENT, "unsupported vector width");
}

template <typename T, typename OffT>
int run_op(const Problem &p, const Geometry &g, void *ws, int64_t *bytes, cudaStream_t s, rg_report *r) {
  switch (p.op) {
    case RG_OP_SUM: return run_vec<T, OffT, OP_SUM>(p, g, ws, bytes, s, r);
    case RG_OP_MAX: return run_vec<T, OffT, OP_MAX>(p, g, ws, bytes, s, r);
    case RG_OP_SOFTMAX: return run_vec<T, OffT, OP_SOFTMAX>(p, g, ws, bytes, s, r);
  }
  return fail(RG_ERR_INVALID_ARGUMENT, "unknown op");
}

template <typename T>
int run_index(const Problem &p, const Geometry &g, void *ws, int64_t *bytes, cudaStream_t s, rg_report *r) {
  return p.index_dtype == RG_INDEX_I32 ? run_op<T, int32_t>(p, g, ws, bytes, s, r)
                                       : run_op<T, int64_t>(p, g, ws, bytes, s, r);
}

int dispatch(const Problem &p, const Geometry &g, void *ws, int64_t *bytes, cudaStream_t s, rg_report *r) {
  return p.dtype == RG_DTYPE_F32 ? run_index<float>(p, g, ws, bytes, s, r)
                                 : run_index<__nv_bfloat16>(p, g, ws, bytes, s, r);
}

template <typename T, typename OffT>
int fused_vec(const Problem &p, const Geometry &g, void *ws, int64_t *bytes, cudaStream_t s, rg_report *r,
              const Xform &xf) {
  switch (g.vec) {
    case 1: return run_typed<T, OffT, OP_SOFTMAX, 1, true>(p, g, ws, bytes, s, r, xf);
    case 2: return run_typed<T, OffT, OP_SOFTMAX, 2, true>(p, g, ws, bytes, s, r, xf);
    case 4: return run_typed<T, OffT, OP_SOFTMAX, 4, true>(p, g, ws, bytes, s, r, xf);
    case 8:
      if constexpr (sizeof(T) == 2) return run_typed<T, OffT, OP_SOFTMAX, 8, true>(p, g, ws, bytes, s, r, xf);
      break;
  }
  return fail(RG_ERR_INVALID_ARGUMENT, "unsupported vector width");
}

}  // namespace

bool rowbal_fuses(const Problem &p, const Geometry &, const float *mask) {
  // The mask is read VEC floats at a time: its rows must be aligned to them.
  const int vec = make_geometry(p).vec;
  return p.op == RG_OP_SOFTMAX && (!mask || aligned(mask, 4 * vec));
}

int launch_rowbal_fused(const Problem &p, const Geometry &g, void *workspace, const float *mask, float scale,
                        cudaStream_t stream, rg_report *report) {
  if (p.b == 0) return RG_OK;
  const Xform xf{mask, p.d, scale, scale != 1.0f ? 1 : 0};
  const bool i32 = p.index_dtype == RG_INDEX_I32;
  if (p.dtype == RG_DTYPE_F32)
    return i32 ? fused_vec<float, int32_t>(p, g, workspace, nullptr, stream, report, xf)
               : fused_vec<float, int64_t>(p, g, workspace, nullptr, stream, report, xf);
  return i32 ? fused_vec<__nv_bfloat16, int32_t>(p, g, workspace, nullptr, stream, report, xf)
             : fused_vec<__nv_bfloat16, int64_t>(p, g, workspace, nullptr, stream, report, xf);
}

int rowbal_workspace(const Problem &p, const Geometry &g, int64_t *bytes) {
  if (p.b == 0) {
    *bytes = 0;
    return RG_OK;
  }
  return dispatch(p, g, nullptr, bytes, nullptr, nullptr);
}

int launch_rowbal(const Problem &p, const Geometry &g, void *workspace, cudaStream_t stream, rg_report *report) {
  if (p.b == 0) return RG_OK;
  return dispatch(p, g, workspace, nullptr, stream, report);
}

}  // namespace rgb
