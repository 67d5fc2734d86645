// Host-side types shared by the launcher and the per-schedule launch code.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/ragged_b200.h"

namespace rgb {

struct Problem {
  int op, dtype, index_dtype;
  int64_t d, n, b;
  const void *values;
  const void *offsets;
  void *out;
  int64_t max_len;  // -1: unknown
  uint32_t flags;
};

// Thread geometry: VEC adjacent features per thread (16-byte vectors where D
// and the base addresses allow, the reference's d_vector rule of
// python/ragged/optimizations.py:41-56), C = D / VEC vector columns,
// G = 2^g_shift = min(32, pow2ceil(C)) lanes per row (the reference's
// d_tile), and ceil(C / 32) column tiles.
struct Geometry {
  int vec;
  int g_shift;
  int vec_cols;
  int col_tiles;
};

struct DeviceProps {
  int device;
  int sm_count;
  int cc_major, cc_minor;
  int64_t l2_bytes;
  int smem_optin;
  int max_threads_per_sm;
};

// Kernel ids reported through rg_report (names in launcher.cu).
enum KernelId : int {
  K_NAIVE = 1,
  K_CLASSIFY = 2,
  K_WORKER = 3,
  K_SPLIT_NORMALIZE = 4,
  K_ROWBAL = 5,
  K_ROWBAL_FIXUP = 6,
  K_SHARD_COMBINE = 7,
  K_ROWBAL_PACKED = 8,
  K_ROWBAL_NORMALIZE = 9,
  K_OFFSETS_INIT = 10,
  K_OFFSETS_CHECK = 11,
  K_POINTWISE_LOGITS = 12,
  K_POINTWISE_CAST = 13,
};

// Recording helper for rg_report.
void record_launch(rg_report *report, int kernel_id, dim3 grid, int block, int shared_bytes);

// Thread-local error detail.
int fail(int status, const std::string &message);
int check_cuda(cudaError_t err, const char *what);

int elem_bytes(int dtype);
bool aligned(const void *p, int bytes);
Geometry make_geometry(const Problem &p);
int device_props(DeviceProps *props);  // current device
int validate(const Problem &p);           // argument checks of rg_run
int check_device(DeviceProps *props);     // current device must be sm_100

// Per-schedule entry points (launch on stream, record into report).
int launch_naive(const Problem &p, const Geometry &g, cudaStream_t stream, rg_report *report);
int rowbal_workspace(const Problem &p, const Geometry &g, int64_t *bytes);
int launch_rowbal(const Problem &p, const Geometry &g, void *workspace, cudaStream_t stream, rg_report *report);
// Resident CTAs per SM of a row-balanced kernel launched with `smem` bytes
// of dynamic shared memory, cached per (kernel, device).
int rowbal_occupancy(const void *kernel, int device, int threads, int *blocks, int smem = 0);
// Virtual CTAs a row-balanced launch wants for `path` merge-path items:
// 64 items per unit, fewer (down to 8) when that leaves the `resident`
// CTAs idle, so a small call spreads over the GPU instead of a few CTAs
// whose threads each walk 64 items (and one thread each merges their pieces).
inline int64_t rowbal_wanted_ctas(int64_t path, int64_t resident, int units_per_cta) {
  int64_t per_unit = path / (resident * units_per_cta);
  per_unit = per_unit < 8 ? 8 : (per_unit > 64 ? 64 : per_unit);
  const int64_t chunk = per_unit * units_per_cta;
  const int64_t wanted = (path + chunk - 1) / chunk;
  return wanted < 1 ? 1 : wanted;
}
int classified_workspace(const Problem &p, const Geometry &g, int64_t *bytes);
// Softmax on the classified schedule with the input transform (scale,
// additive mask) fused into the loads: for rows the pipelined worker stages.
bool classified_fuses(const Problem &p, const Geometry &g);
int launch_classified_fused(const Problem &p, const Geometry &g, void *workspace, const float *mask, float scale,
                            cudaStream_t stream, rg_report *report);
// Softmax on the row-balanced schedule with the transform fused into both
// passes' loads (the workspace is rowbal_workspace's).
bool rowbal_fuses(const Problem &p, const Geometry &g, const float *mask);
int launch_rowbal_fused(const Problem &p, const Geometry &g, void *workspace, const float *mask, float scale,
                        cudaStream_t stream, rg_report *report);
int launch_classified(const Problem &p, const Geometry &g, void *workspace, cudaStream_t stream, rg_report *report);

// Any schedule: its scratch bytes, and its launch for a validated problem.
int workspace_for(const Problem &p, const Geometry &g, int schedule, int64_t *bytes);
int run_schedule(const Problem &p, const Geometry &g, int schedule, void *workspace, cudaStream_t stream,
                 rg_report *report);

}  // namespace rgb
