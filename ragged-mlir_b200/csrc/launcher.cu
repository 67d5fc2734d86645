// The C ABI (include/ragged_b200.h): argument validation, device queries,
// geometry, workspace sizing and schedule dispatch.  No exception crosses
// the boundary; every entry point returns an rg_status.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "internal.h"

namespace rgb {

namespace {
thread_local std::string g_last_error;

std::mutex g_device_mutex;
std::vector<DeviceProps> g_devices;  // by ordinal; sm_count == 0 means "not queried"
}  // namespace

int fail(int status, const std::string &message) {
  g_last_error = message;
  return status;
}

int check_cuda(cudaError_t err, const char *what) {
  if (err == cudaSuccess) return RG_OK;
  char buffer[512];
  std::snprintf(buffer, sizeof buffer, "%s: %s (%d): %s", what, cudaGetErrorName(err), static_cast<int>(err),
                cudaGetErrorString(err));
  return fail(RG_ERR_CUDA, buffer);
}

void record_launch(rg_report *report, int kernel_id, dim3 grid, int block, int shared_bytes) {
  if (!report || report->num_launches >= RG_MAX_LAUNCHES) return;
  const int i = report->num_launches++;
  report->kernel_ids[i] = kernel_id;
  report->grid[i][0] = static_cast<int32_t>(grid.x);
  report->grid[i][1] = static_cast<int32_t>(grid.y);
  report->grid[i][2] = static_cast<int32_t>(grid.z);
  report->block[i] = block;
  report->shared_bytes[i] = shared_bytes;
}

int elem_bytes(int dtype) { return dtype == RG_DTYPE_F32 ? 4 : 2; }

bool aligned(const void *p, int bytes) {
  return (reinterpret_cast<uintptr_t>(p) % static_cast<uintptr_t>(bytes)) == 0;
}

Geometry make_geometry(const Problem &p) {
  const int esize = elem_bytes(p.dtype);
  int vec = 1;
  if (!(p.flags & RG_FLAG_NO_VECTORIZE)) {
    while (2 * vec * esize <= 16 && p.d % (2 * vec) == 0) vec *= 2;
  }
  Geometry g;
  g.vec = vec;
  g.vec_cols = static_cast<int>(p.d / vec);
  int lanes = 1, shift = 0;
  while (lanes < g.vec_cols && lanes < 32) {
    lanes *= 2;
    ++shift;
  }
  g.g_shift = shift;
  g.col_tiles = (g.vec_cols + 31) / 32;
  return g;
}

int device_props(DeviceProps *props) {
  int device = 0;
  int status = check_cuda(cudaGetDevice(&device), "cudaGetDevice");
  if (status) return status;
  std::lock_guard<std::mutex> lock(g_device_mutex);
  if (device >= static_cast<int>(g_devices.size())) g_devices.resize(device + 1, DeviceProps{});
  DeviceProps &d = g_devices[device];
  if (d.sm_count == 0) {
    cudaDeviceProp prop;
    status = check_cuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (status) return status;
    d.device = device;
    d.sm_count = prop.multiProcessorCount;
    d.cc_major = prop.major;
    d.cc_minor = prop.minor;
    d.l2_bytes = prop.l2CacheSize;
    d.smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
    d.max_threads_per_sm = prop.maxThreadsPerMultiProcessor;
  }
  *props = d;
  return RG_OK;
}

int validate(const Problem &p) {
  if (p.op < RG_OP_SUM || p.op > RG_OP_SOFTMAX) return fail(RG_ERR_INVALID_ARGUMENT, "op must be sum, max or softmax");
  if (p.dtype != RG_DTYPE_F32 && p.dtype != RG_DTYPE_BF16)
    return fail(RG_ERR_INVALID_ARGUMENT, "dtype must be f32 or bf16");
  if (p.index_dtype != RG_INDEX_I32 && p.index_dtype != RG_INDEX_I64)
    return fail(RG_ERR_INVALID_ARGUMENT, "offsets dtype must be i32 or i64");
  if (p.d < 1 || p.d > 1024) return fail(RG_ERR_INVALID_ARGUMENT, "D must lie in [1, 1024]");
  if (p.n < 0 || p.b < 0) return fail(RG_ERR_INVALID_ARGUMENT, "N and B must be nonnegative");
  if (p.b == 0 && p.n != 0) return fail(RG_ERR_INVALID_ARGUMENT, "B=0 requires N=0");
  if (p.index_dtype == RG_INDEX_I32 && p.n > 2147483647LL)
    return fail(RG_ERR_INVALID_ARGUMENT, "N exceeds the i32 offsets range");
  if (p.b >= (int64_t{1} << 40)) return fail(RG_ERR_INVALID_ARGUMENT, "B is beyond this build's segment-id range");
  if (p.max_len < -1) return fail(RG_ERR_INVALID_ARGUMENT, "max_len must be -1 (unknown) or nonnegative");
  // Byte sizes must fit signed 64-bit arithmetic.
  const int64_t esize = elem_bytes(p.dtype);
  const int64_t rows_out = p.op == RG_OP_SOFTMAX ? p.n : p.b;
  if (p.n > INT64_MAX / p.d / esize || rows_out > INT64_MAX / p.d / esize)
    return fail(RG_ERR_INVALID_ARGUMENT, "tensor byte size overflows signed 64-bit");
  if (p.b == 0) return RG_OK;
  if (!p.offsets) return fail(RG_ERR_INVALID_ARGUMENT, "offsets pointer is NULL");
  if (p.n > 0 && !p.values) return fail(RG_ERR_INVALID_ARGUMENT, "values pointer is NULL");
  if (rows_out > 0 && !p.out) return fail(RG_ERR_INVALID_ARGUMENT, "out pointer is NULL");
  // out must be disjoint from values (or, in place, be values) and from offsets.
  const uintptr_t ob = reinterpret_cast<uintptr_t>(p.out), oe = ob + rows_out * p.d * esize;
  const uintptr_t vb = reinterpret_cast<uintptr_t>(p.values), ve = vb + p.n * p.d * esize;
  const uintptr_t fb = reinterpret_cast<uintptr_t>(p.offsets),
                  fe = fb + (p.b + 1) * (p.index_dtype == RG_INDEX_I32 ? 4 : 8);
  if (p.flags & RG_FLAG_IN_PLACE) {
    if (p.op != RG_OP_SOFTMAX) return fail(RG_ERR_INVALID_ARGUMENT, "in-place output is only defined for softmax");
    if (p.n > 0 && p.out != p.values) return fail(RG_ERR_INVALID_ARGUMENT, "in place, out must be values");
  } else if (rows_out > 0 && p.n > 0 && ob < ve && vb < oe) {
    return fail(RG_ERR_INVALID_ARGUMENT, "out overlaps values");
  }
  if (rows_out > 0 && ob < fe && fb < oe) return fail(RG_ERR_INVALID_ARGUMENT, "out overlaps offsets");
  if (!aligned(p.offsets, p.index_dtype == RG_INDEX_I32 ? 4 : 8))
    return fail(RG_ERR_INVALID_ARGUMENT, "offsets must be aligned to their element size");
  const Geometry g = make_geometry(p);
  const int need = g.vec * static_cast<int>(esize);
  if ((p.n > 0 && !aligned(p.values, need)) || (rows_out > 0 && !aligned(p.out, need))) {
    char buffer[200];
    std::snprintf(buffer, sizeof buffer,
                  "values and out must be %d-byte aligned: this call accesses %d features at a time", need, g.vec);
    return fail(RG_ERR_INVALID_ARGUMENT, buffer);
  }
  return RG_OK;
}

int check_device(DeviceProps *props) {
  int status = device_props(props);
  if (status) return status;
  if (props->cc_major != 10 || props->cc_minor != 0) {
    char buffer[160];
    std::snprintf(buffer, sizeof buffer,
                  "libragged_b200 is built for sm_100a only; device %d is sm_%d%d", props->device, props->cc_major,
                  props->cc_minor);
    return fail(RG_ERR_DEVICE, buffer);
  }
  return RG_OK;
}

// Scratch bytes of `schedule` for this problem (status on failure).
int workspace_for(const Problem &p, const Geometry &g, int schedule, int64_t *bytes) {
  *bytes = 0;
  switch (schedule) {
    case RG_SCHEDULE_NAIVE: return RG_OK;
    case RG_SCHEDULE_CLASSIFIED: return classified_workspace(p, g, bytes);
    case RG_SCHEDULE_ROWBALANCED: return rowbal_workspace(p, g, bytes);
  }
  return fail(RG_ERR_UNSUPPORTED, "schedule not available in this build");
}

// Launch `schedule` for a validated problem (workspace sized by workspace_for).
int run_schedule(const Problem &p, const Geometry &g, int schedule, void *workspace, cudaStream_t s,
                 rg_report *report) {
  switch (schedule) {
    case RG_SCHEDULE_NAIVE: return launch_naive(p, g, s, report);
    case RG_SCHEDULE_CLASSIFIED: return launch_classified(p, g, workspace, s, report);
    case RG_SCHEDULE_ROWBALANCED: return launch_rowbal(p, g, workspace, s, report);
  }
  return fail(RG_ERR_UNSUPPORTED, "schedule not available in this build");
}

}  // namespace rgb

using namespace rgb;

extern "C" {

const char *rg_version(void) { return "ragged-b200 0.1.0 (sm_100a)"; }

const char *rg_error_string(int status) {
  switch (status) {
    case RG_OK: return "success";
    case RG_ERR_INVALID_ARGUMENT: return "invalid argument";
    case RG_ERR_UNSUPPORTED: return "unsupported request";
    case RG_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case RG_ERR_CUDA: return "CUDA error";
    case RG_ERR_DEVICE: return "no supported (sm_100) CUDA device";
  }
  return "unknown status";
}

const char *rg_last_error(void) { return g_last_error.c_str(); }

const char *rg_kernel_name(int kernel_id) {
  switch (kernel_id) {
    case K_NAIVE: return "block_per_segment";
    case K_CLASSIFY: return "classify";
    case K_WORKER: return "classified_worker";
    case K_SPLIT_NORMALIZE: return "split_normalize";
    case K_ROWBAL: return "rowbalanced";
    case K_ROWBAL_FIXUP: return "rowbalanced_fixup";
    case K_SHARD_COMBINE: return "shard_combine";
    case K_ROWBAL_PACKED: return "rowbalanced_packed";
    case K_ROWBAL_NORMALIZE: return "rowbalanced_normalize";
    case K_OFFSETS_INIT: return "offsets_init";
    case K_OFFSETS_CHECK: return "offsets_check";
    case K_POINTWISE_LOGITS: return "pointwise_logits";
    case K_POINTWISE_CAST: return "pointwise_cast";
  }
  return "";
}

int rg_get_device_info(int device, rg_device_info *info) {
  if (!info) return fail(RG_ERR_INVALID_ARGUMENT, "info is NULL");
  int previous = 0;
  int status = check_cuda(cudaGetDevice(&previous), "cudaGetDevice");
  if (status) return status;
  if (device != previous) {
    status = check_cuda(cudaSetDevice(device), "cudaSetDevice");
    if (status) return status;
  }
  DeviceProps props;
  status = device_props(&props);
  if (device != previous) cudaSetDevice(previous);
  if (status) return status;
  info->device = props.device;
  info->sm_count = props.sm_count;
  info->cc_major = props.cc_major;
  info->cc_minor = props.cc_minor;
  info->l2_bytes = props.l2_bytes;
  info->smem_per_block_optin = props.smem_optin;
  info->max_threads_per_sm = props.max_threads_per_sm;
  return RG_OK;
}

int rg_workspace_bytes(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, int schedule,
                       int64_t max_len, uint32_t flags, int64_t *bytes) {
  if (!bytes) return fail(RG_ERR_INVALID_ARGUMENT, "bytes is NULL");
  Problem p{op, dtype, index_dtype, d, n, b, nullptr, nullptr, nullptr, max_len, flags};
  // Pointer-free validation: shapes only.
  if (op < RG_OP_SUM || op > RG_OP_SOFTMAX || (dtype != RG_DTYPE_F32 && dtype != RG_DTYPE_BF16) ||
      (index_dtype != RG_INDEX_I32 && index_dtype != RG_INDEX_I64) || d < 1 || d > 1024 || n < 0 || b < 0)
    return fail(RG_ERR_INVALID_ARGUMENT, "invalid problem description");
  DeviceProps dev;
  int status = check_device(&dev);
  if (status) return status;
  return workspace_for(p, make_geometry(p), schedule, bytes);
}

int rg_run(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, const void *values,
           const void *offsets, void *out, void *workspace, int64_t workspace_bytes, int schedule, int64_t max_len,
           uint32_t flags, void *stream, rg_report *report) {
  Problem p{op, dtype, index_dtype, d, n, b, values, offsets, out, max_len, flags};
  if (report) {
    std::memset(report, 0, sizeof *report);
    report->status_offset = -1;
    report->schedule = schedule;
    report->streams = 1;
  }
  int status = validate(p);
  if (status) return status;
  const Geometry g = make_geometry(p);
  if (report) {
    report->d_vector = g.vec;
    report->d_tile = 1 << g.g_shift;
  }
  if (b == 0) return RG_OK;  // no launch (reference runtime.py:461-465)
  DeviceProps dev;
  status = check_device(&dev);
  if (status) return status;
  int64_t need = 0;
  status = workspace_for(p, g, schedule, &need);
  if (status) return status;
  if (report) report->workspace_bytes = need;
  if (need > 0) {
    if (!workspace || workspace_bytes < need) return fail(RG_ERR_WORKSPACE, "workspace missing or too small");
    if (!aligned(workspace, 256)) return fail(RG_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  }
  return run_schedule(p, g, schedule, workspace, static_cast<cudaStream_t>(stream), report);
}


}  // extern "C"
