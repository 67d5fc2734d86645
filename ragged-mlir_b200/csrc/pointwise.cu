// Pointwise input transform (the reference's ProgramSpec `scale` and additive
// softmax `mask`, docs/mask-abi.md; lowering lib/Conversion/ToGPU.cpp:41-60
// transformedInput and :604-618 loadInput) on the reference's materialised
// route (pointwise fusion off): the transformed f32 logits are written once,
// the unchanged f32 schedule reads them, and bf16 results are rounded once
// at the end.
//
//   pointwise_logits   x = f32(values[i]); x = x * scale (when scale != 1);
//                      x = x + mask[i] (softmax with a mask) -- two f32
//                      roundings, no fused multiply-add, as the reference.
//   <schedule>         sum / max / softmax over the f32 logits into f32
//                      results: the caller's `out` for f32 values, else a
//                      scratch buffer (softmax: the logits themselves, in place).
//   pointwise_cast     bf16 values only: the f32 results rounded to nearest
//                      even into `out`.
//
// Every schedule computes in f32 and rounds once when it stores, so results
// are bitwise those of a kernel that applied the transform as it loaded.
// Extra HBM traffic: the logits (written once, read by the schedule) and,
// for bf16, the f32 results (written and read once).
#include <cmath>
#include <cstring>

#include "internal.h"

namespace rgb {

namespace {

constexpr int kPointwiseThreads = 256;

template <typename T>
__device__ __forceinline__ float to_f32(T v) {
  if constexpr (std::is_same<T, float>::value) {
    return v;
  } else {
    return __bfloat162float(v);
  }
}

// Four elements per step when every pointer is 16-byte aligned and the
// count is a multiple of four (V4), else one.
template <typename T, bool V4>
__global__ void __launch_bounds__(kPointwiseThreads)
pointwise_logits_kernel(const T *__restrict__ values, const float *__restrict__ mask, float scale, int scaled,
                        float *__restrict__ logits, int64_t count) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if constexpr (V4) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count / 4; i += stride) {
      float x[4];
      if constexpr (std::is_same<T, float>::value) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(values) + i);
        x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
      } else {
        const uint2 v = __ldg(reinterpret_cast<const uint2 *>(values) + i);
        x[0] = __uint_as_float(v.x << 16); x[1] = __uint_as_float(v.x & 0xffff0000u);
        x[2] = __uint_as_float(v.y << 16); x[3] = __uint_as_float(v.y & 0xffff0000u);
      }
      if (scaled) {
#pragma unroll
        for (int k = 0; k < 4; ++k) x[k] = __fmul_rn(x[k], scale);
      }
      if (mask) {
        const float4 m = __ldg(reinterpret_cast<const float4 *>(mask) + i);
        x[0] = __fadd_rn(x[0], m.x); x[1] = __fadd_rn(x[1], m.y);
        x[2] = __fadd_rn(x[2], m.z); x[3] = __fadd_rn(x[3], m.w);
      }
      reinterpret_cast<float4 *>(logits)[i] = make_float4(x[0], x[1], x[2], x[3]);
    }
  } else {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride) {
      float x = to_f32(values[i]);
      if (scaled) x = __fmul_rn(x, scale);
      if (mask) x = __fadd_rn(x, __ldg(mask + i));
      logits[i] = x;
    }
  }
}

template <bool V4>
__global__ void __launch_bounds__(kPointwiseThreads)
pointwise_cast_kernel(const float *__restrict__ results, __nv_bfloat16 *__restrict__ out, int64_t count) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if constexpr (V4) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count / 4; i += stride) {
      const float4 y = reinterpret_cast<const float4 *>(results)[i];
      __nv_bfloat162 lo = __floats2bfloat162_rn(y.x, y.y), hi = __floats2bfloat162_rn(y.z, y.w);
      reinterpret_cast<uint2 *>(out)[i] =
          make_uint2(*reinterpret_cast<uint32_t *>(&lo), *reinterpret_cast<uint32_t *>(&hi));
    }
  } else {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += stride)
      out[i] = __float2bfloat16_rn(results[i]);
  }
}

constexpr int64_t kAlign = 256;
int64_t align_up(int64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Workspace: the f32 logits [N][D], then (bf16 sum / max) the f32 results
// [B][D], then the inner schedule's scratch.
struct PointwiseLayout {
  int64_t logits_bytes, results_bytes, inner_offset, inner_bytes, total;
};

Problem inner_problem(const Problem &p, const void *logits, void *results) {
  Problem q = p;
  q.dtype = RG_DTYPE_F32;
  q.values = logits;
  q.out = results;
  q.flags = p.flags & RG_FLAG_NO_VECTORIZE;
  if (p.op == RG_OP_SOFTMAX && p.dtype == RG_DTYPE_BF16) q.flags |= RG_FLAG_IN_PLACE;  // results = logits
  return q;
}

int layout_of(const Problem &p, int schedule, PointwiseLayout *l) {
  l->logits_bytes = align_up(p.n * p.d * 4);
  l->results_bytes = (p.dtype == RG_DTYPE_BF16 && p.op != RG_OP_SOFTMAX) ? align_up(p.b * p.d * 4) : 0;
  l->inner_offset = l->logits_bytes + l->results_bytes;
  const Problem q = inner_problem(p, nullptr, nullptr);
  int status = workspace_for(q, make_geometry(q), schedule, &l->inner_bytes);
  if (status) return status;
  l->total = l->inner_offset + align_up(l->inner_bytes);
  return RG_OK;
}

// How a call runs its transform.  Fused routes (softmax only, fusion not
// switched off, not in place over values a mask aliases):
//   row-balanced schedule  the statistics and normalise passes read values
//                          and mask together (mask rows aligned to the
//                          call's vector width);
//   classified schedule    with staged rows and a scale but no mask: the
//                          worker scales rows as it reads them from shared
//                          memory.  (With a mask the worker would wait on
//                          global mask loads between shared-memory passes;
//                          measured on B200 that is slower than the
//                          materialised route, so a mask goes there.)
// Everything else materialises the transformed f32 logits first.
enum Route { MATERIALIZED = 0, FUSED_ROWBAL = 1, FUSED_CLASSIFIED = 2 };

int route_of(const Problem &p, const Geometry &g, int schedule, const float *mask) {
  if (p.op != RG_OP_SOFTMAX || (p.flags & RG_FLAG_NO_POINTWISE_FUSION)) return MATERIALIZED;
  if (mask && (p.flags & RG_FLAG_IN_PLACE)) {
    const uintptr_t mb = reinterpret_cast<uintptr_t>(mask), me = mb + p.n * p.d * 4;
    const uintptr_t vb = reinterpret_cast<uintptr_t>(p.values), ve = vb + p.n * p.d * elem_bytes(p.dtype);
    if (mb < ve && vb < me) return MATERIALIZED;
  }
  if (schedule == RG_SCHEDULE_ROWBALANCED && rowbal_fuses(p, g, mask)) return FUSED_ROWBAL;
  if (schedule == RG_SCHEDULE_CLASSIFIED && !mask && classified_fuses(p, g)) return FUSED_CLASSIFIED;
  return MATERIALIZED;
}

// Scratch of a fused route (the schedule's own workspace for the original problem).
int fused_workspace(const Problem &p, const Geometry &g, int route, int64_t *bytes) {
  *bytes = 0;
  if (route == FUSED_ROWBAL) return rowbal_workspace(p, g, bytes);
  if (route == FUSED_CLASSIFIED) return classified_workspace(p, g, bytes);
  return RG_OK;
}

int grid_for(int64_t items, const DeviceProps &dev) {
  int64_t blocks = (items + kPointwiseThreads - 1) / kPointwiseThreads;
  const int64_t cap = static_cast<int64_t>(dev.sm_count) * 8;
  if (blocks > cap) blocks = cap;
  return blocks < 1 ? 1 : static_cast<int>(blocks);
}

template <typename T>
int launch_logits(const Problem &p, const float *mask, float scale, float *logits, const DeviceProps &dev,
                  cudaStream_t s, rg_report *report) {
  const int64_t count = p.n * p.d;
  if (count == 0) return RG_OK;
  const bool v4 = count % 4 == 0 && aligned(p.values, 4 * static_cast<int>(sizeof(T))) &&
                  (!mask || aligned(mask, 16)) && aligned(logits, 16);
  const int scaled = scale != 1.0f;
  dim3 grid(static_cast<unsigned>(grid_for(v4 ? count / 4 : count, dev)), 1, 1);
  if (v4) {
    pointwise_logits_kernel<T, true><<<grid, kPointwiseThreads, 0, s>>>(static_cast<const T *>(p.values), mask,
                                                                        scale, scaled, logits, count);
  } else {
    pointwise_logits_kernel<T, false><<<grid, kPointwiseThreads, 0, s>>>(static_cast<const T *>(p.values), mask,
                                                                         scale, scaled, logits, count);
  }
  record_launch(report, K_POINTWISE_LOGITS, grid, kPointwiseThreads, 0);
  return check_cuda(cudaGetLastError(), "pointwise_logits_kernel launch");
}

int launch_cast(const float *results, void *out, int64_t count, const DeviceProps &dev, cudaStream_t s,
                rg_report *report) {
  if (count == 0) return RG_OK;
  const bool v4 = count % 4 == 0 && aligned(results, 16) && aligned(out, 8);
  dim3 grid(static_cast<unsigned>(grid_for(v4 ? count / 4 : count, dev)), 1, 1);
  if (v4) {
    pointwise_cast_kernel<true><<<grid, kPointwiseThreads, 0, s>>>(results, static_cast<__nv_bfloat16 *>(out), count);
  } else {
    pointwise_cast_kernel<false><<<grid, kPointwiseThreads, 0, s>>>(results, static_cast<__nv_bfloat16 *>(out),
                                                                    count);
  }
  record_launch(report, K_POINTWISE_CAST, grid, kPointwiseThreads, 0);
  return check_cuda(cudaGetLastError(), "pointwise_cast_kernel launch");
}

bool shape_ok(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b) {
  return op >= RG_OP_SUM && op <= RG_OP_SOFTMAX && (dtype == RG_DTYPE_F32 || dtype == RG_DTYPE_BF16) &&
         (index_dtype == RG_INDEX_I32 || index_dtype == RG_INDEX_I64) && d >= 1 && d <= 1024 && n >= 0 && b >= 0;
}

}  // namespace

}  // namespace rgb

using namespace rgb;

extern "C" {

int rg_pointwise_workspace_bytes(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b,
                                 int schedule, int64_t max_len, uint32_t flags, int64_t *bytes) {
  if (!bytes) return fail(RG_ERR_INVALID_ARGUMENT, "bytes is NULL");
  if (!shape_ok(op, dtype, index_dtype, d, n, b)) return fail(RG_ERR_INVALID_ARGUMENT, "invalid problem description");
  if (n > INT64_MAX / 4 / d || b > INT64_MAX / 4 / d)
    return fail(RG_ERR_INVALID_ARGUMENT, "tensor byte size overflows signed 64-bit");
  *bytes = 0;
  if (b == 0) return RG_OK;
  DeviceProps dev;
  int status = check_device(&dev);
  if (status) return status;
  Problem p{op, dtype, index_dtype, d, n, b, nullptr, nullptr, nullptr, max_len, flags};
  PointwiseLayout l;
  status = layout_of(p, schedule, &l);
  if (status) return status;
  *bytes = l.total;
  // Enough for a fused route too (which route runs depends on the mask pointer).
  const Geometry g = make_geometry(p);
  for (int route : {FUSED_ROWBAL, FUSED_CLASSIFIED}) {
    const bool possible = route == FUSED_ROWBAL ? schedule == RG_SCHEDULE_ROWBALANCED && op == RG_OP_SOFTMAX
                                                : schedule == RG_SCHEDULE_CLASSIFIED && classified_fuses(p, g);
    if (!possible) continue;
    int64_t fused = 0;
    status = fused_workspace(p, g, route, &fused);
    if (status) return status;
    if (fused > *bytes) *bytes = fused;
  }
  return RG_OK;
}

int rg_run_pointwise(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, const void *values,
                     const void *offsets, const float *mask, float scale, void *out, void *workspace,
                     int64_t workspace_bytes, int schedule, int64_t max_len, uint32_t flags, void *stream,
                     rg_report *report) {
  Problem p{op, dtype, index_dtype, d, n, b, values, offsets, out, max_len, flags};
  if (report) {
    std::memset(report, 0, sizeof *report);
    report->status_offset = -1;
    report->schedule = schedule;
    report->streams = 1;
  }
  int status = validate(p);
  if (status) return status;
  if (!std::isfinite(scale))
    return fail(RG_ERR_INVALID_ARGUMENT, "scale must be a finite f32 value");
  if (mask) {
    if (op != RG_OP_SOFTMAX) return fail(RG_ERR_INVALID_ARGUMENT, "an additive mask is only defined for softmax");
    if (!aligned(mask, 4)) return fail(RG_ERR_INVALID_ARGUMENT, "mask must be 4-byte aligned");
    // The mask may alias values (read-only input) but neither out nor offsets.
    const uintptr_t mb = reinterpret_cast<uintptr_t>(mask), me = mb + n * d * 4;
    const uintptr_t ob = reinterpret_cast<uintptr_t>(out), oe = ob + n * d * elem_bytes(dtype);
    const uintptr_t fb = reinterpret_cast<uintptr_t>(offsets),
                    fe = fb + (b + 1) * (index_dtype == RG_INDEX_I32 ? 4 : 8);
    if (n > 0 && mb < oe && ob < me) return fail(RG_ERR_INVALID_ARGUMENT, "mask overlaps out");
    if (n > 0 && b > 0 && mb < fe && fb < me) return fail(RG_ERR_INVALID_ARGUMENT, "mask overlaps offsets");
  }
  if (b == 0) return RG_OK;
  DeviceProps dev;
  status = check_device(&dev);
  if (status) return status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const Geometry g0 = make_geometry(p);
  const int route = route_of(p, g0, schedule, mask);
  if (route != MATERIALIZED) {
    int64_t need = 0;
    status = fused_workspace(p, g0, route, &need);
    if (status) return status;
    if (report) {
      report->workspace_bytes = need;
      report->d_vector = g0.vec;
      report->d_tile = 1 << g0.g_shift;
    }
    if (!workspace || workspace_bytes < need) return fail(RG_ERR_WORKSPACE, "workspace missing or too small");
    if (!aligned(workspace, 256)) return fail(RG_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    return route == FUSED_ROWBAL ? launch_rowbal_fused(p, g0, workspace, mask, scale, s, report)
                                 : launch_classified_fused(p, g0, workspace, mask, scale, s, report);
  }
  PointwiseLayout l;
  status = layout_of(p, schedule, &l);
  if (status) return status;
  if (report) report->workspace_bytes = l.total;
  if (!workspace || workspace_bytes < l.total) return fail(RG_ERR_WORKSPACE, "workspace missing or too small");
  if (!aligned(workspace, 256)) return fail(RG_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  char *ws = static_cast<char *>(workspace);
  float *logits = reinterpret_cast<float *>(ws);
  float *results = dtype == RG_DTYPE_F32 ? static_cast<float *>(out)
                                         : (op == RG_OP_SOFTMAX ? logits : reinterpret_cast<float *>(ws + l.logits_bytes));
  status = dtype == RG_DTYPE_F32 ? launch_logits<float>(p, mask, scale, logits, dev, s, report)
                                 : launch_logits<__nv_bfloat16>(p, mask, scale, logits, dev, s, report);
  if (status) return status;
  const Problem q = inner_problem(p, logits, results);
  const Geometry g = make_geometry(q);
  if (report) {
    report->d_vector = g.vec;
    report->d_tile = 1 << g.g_shift;
  }
  status = run_schedule(q, g, schedule, ws + l.inner_offset, s, report);
  if (report && report->status_offset >= 0) report->status_offset += l.inner_offset;
  if (status || dtype == RG_DTYPE_F32) return status;
  const int64_t rows_out = op == RG_OP_SOFTMAX ? n : b;
  return launch_cast(results, out, rows_out * d, dev, s, report);
}

}  // extern "C"
