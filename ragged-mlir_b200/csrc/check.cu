// Checked offsets mode: device validation of the offsets before any main
// kernel or output write (the reference's offsets-check-v1 ABI,
// docs/checked-abi.md; kernels of lib/Conversion/ToGPU.cpp:1067-1189).
//
// offsets_init_kernel writes INT64_MAX to the seven status slots;
// offsets_check_kernel visits every offset index i in [0, B] once and keeps,
// per condition, the earliest offending index with a signed 64-bit atomic
// minimum:
//   0 first_nonzero   offsets[0] != 0                          index 0
//   1 final_mismatch  offsets[B] != N                          index B
//   2 negative        offsets[i] < 0                           offset i
//   3 above_n         offsets[i] > N                           offset i
//   4 nonmonotone     offsets[i+1] < offsets[i]                segment i
//   5 below_min_len   length < min_len (valid segments only)   segment i
//   6 above_max_len   length > max_len (valid segments only)   segment i
// A length is formed only after both endpoints lie in [0, N] and the pair is
// monotone, so extreme i64 offsets cannot overflow the subtraction.
#include <climits>
#include <cstring>

#include "internal.h"

namespace rgb {

namespace {

constexpr int kCheckThreads = 128;

__global__ void __launch_bounds__(kCheckThreads) offsets_init_kernel(long long *__restrict__ status) {
  if (threadIdx.x < 7) status[threadIdx.x] = LLONG_MAX;
}

template <typename OffT>
__global__ void __launch_bounds__(kCheckThreads)
offsets_check_kernel(const OffT *__restrict__ offsets, int64_t n, int64_t b, int64_t min_len, int64_t max_len,
                     long long *__restrict__ status) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i <= b; i += stride) {
    const int64_t o = static_cast<int64_t>(offsets[i]);
    if (i == 0 && o != 0) atomicMin(&status[0], 0ll);
    if (i == b && o != n) atomicMin(&status[1], static_cast<long long>(b));
    if (o < 0) atomicMin(&status[2], static_cast<long long>(i));
    if (o > n) atomicMin(&status[3], static_cast<long long>(i));
    if (i < b) {
      const int64_t e = static_cast<int64_t>(offsets[i + 1]);
      if (e < o) atomicMin(&status[4], static_cast<long long>(i));
      if (o >= 0 && e <= n && o <= e) {
        const int64_t len = e - o;
        if (min_len >= 0 && len < min_len) atomicMin(&status[5], static_cast<long long>(i));
        if (max_len >= 0 && len > max_len) atomicMin(&status[6], static_cast<long long>(i));
      }
    }
  }
}

}  // namespace

}  // namespace rgb

using namespace rgb;

extern "C" int rg_check_offsets(int index_dtype, int64_t n, int64_t b, const void *offsets, int64_t min_len,
                                int64_t max_len, int64_t *status, void *stream, rg_report *report) {
  if (report) {
    std::memset(report, 0, sizeof *report);
    report->status_offset = -1;
    report->streams = 1;
  }
  if (index_dtype != RG_INDEX_I32 && index_dtype != RG_INDEX_I64)
    return fail(RG_ERR_INVALID_ARGUMENT, "offsets dtype must be i32 or i64");
  if (n < 0 || b < 0) return fail(RG_ERR_INVALID_ARGUMENT, "N and B must be nonnegative");
  if (!offsets || !status) return fail(RG_ERR_INVALID_ARGUMENT, "offsets and status must not be NULL");
  if (reinterpret_cast<uintptr_t>(status) % 8) return fail(RG_ERR_INVALID_ARGUMENT, "status must be 8-byte aligned");
  if (min_len < -1 || max_len < -1) return fail(RG_ERR_INVALID_ARGUMENT, "length bounds must be -1 (none) or >= 0");
  DeviceProps dev;
  int st = check_device(&dev);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  long long *slots = reinterpret_cast<long long *>(status);
  offsets_init_kernel<<<1, kCheckThreads, 0, s>>>(slots);
  record_launch(report, K_OFFSETS_INIT, dim3(1, 1, 1), kCheckThreads, 0);
  st = check_cuda(cudaGetLastError(), "offsets_init_kernel launch");
  if (st) return st;
  int64_t blocks = (b + 1 + kCheckThreads - 1) / kCheckThreads;  // b < 2^40: no overflow
  const int64_t cap = static_cast<int64_t>(dev.sm_count) * 16;
  if (blocks > cap) blocks = cap;
  dim3 grid(static_cast<unsigned>(blocks), 1, 1);
  if (index_dtype == RG_INDEX_I32)
    offsets_check_kernel<int32_t><<<grid, kCheckThreads, 0, s>>>(static_cast<const int32_t *>(offsets), n, b,
                                                                 min_len, max_len, slots);
  else
    offsets_check_kernel<int64_t><<<grid, kCheckThreads, 0, s>>>(static_cast<const int64_t *>(offsets), n, b,
                                                                 min_len, max_len, slots);
  record_launch(report, K_OFFSETS_CHECK, grid, kCheckThreads, 0);
  return check_cuda(cudaGetLastError(), "offsets_check_kernel launch");
}
