// rg_run_noalloc: the row-balanced sum / max with its scratch in a static
// device array, for callers that cannot allocate device memory.
//
// Some hosts of this library cannot hand it a workspace or let it allocate
// one: an application that reserves all device memory for its own pool at
// start-up and forbids any other allocation, a plugin interface whose
// execute callback may not allocate, or a latency-critical path that must
// not pay for cudaMalloc's implicit device-wide synchronisation.  This entry
// point serves them.  It calls no cudaMalloc, cudaFree or allocating
// library routine: its scratch (the per-unit pieces and unit metadata of
// the row-balanced schedule) lives in `g_static_scratch`, a fixed 8 MiB
// array that every GPU loading the library holds until the process exits.
//
// * Size limit: the CTA count is reduced until the pieces (two per CTA)
//   fit in 8 MiB, down to one CTA per SM; a problem whose pieces would
//   still not fit is rejected with RG_ERR_WORKSPACE and the byte counts.
//   On a 148-SM B200 every D <= 1024 fits with room to spare (an f32 sum
//   with D = 1024 needs 16 KiB per CTA).
// * Set-up: the first call on each device resolves the array's device
//   address with cudaGetSymbolAddress (with that device current) and caches
//   it; make that first call before any stream capture.
// * Sharing: every call on a device uses the same array and leaves its
//   contents behind.  Nothing in it has to start at zero (the kernel writes
//   each unit's metadata before the fix-up reads it), but two calls that
//   overlap on the GPU -- on different streams, or on the same device from
//   different threads without ordering -- race on it.
#include <cstdio>
#include <mutex>
#include <vector>

#include "internal.h"
#include "rowbal.cuh"

namespace rgb {

namespace {

constexpr int64_t kStaticScratchBytes = int64_t{8} << 20;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
std::vector<void *> g_scratch_address;  // by device ordinal; nullptr = not resolved

// Device address of g_static_scratch on `device` (the current device).
int static_scratch(int device, void **address) {
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (device >= static_cast<int>(g_scratch_address.size())) g_scratch_address.resize(device + 1, nullptr);
  if (!g_scratch_address[device]) {
    void *ptr = nullptr;
    const int status = check_cuda(cudaGetSymbolAddress(&ptr, g_static_scratch), "cudaGetSymbolAddress");
    if (status) return status;
    g_scratch_address[device] = ptr;
  }
  *address = g_scratch_address[device];
  return RG_OK;
}

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

template <typename T, typename OffT, int OP, int VEC>
int run_typed(const Problem &p, const Geometry &g, const DeviceProps &dev, void *scratch, cudaStream_t stream) {
  int per_sm = 0;
  int status = rowbal_occupancy(reinterpret_cast<const void *>(&rowbal_kernel<T, OffT, OP, VEC>), dev.device,
                                kRowbalThreads, &per_sm);
  if (status) return status;
  const int units_per_cta = (kRowbalThreads / 32) << (5 - g.g_shift);
  const int width = OP == OP_SUM ? 2 : 1;
  const int64_t unit_piece_bytes = 2 * width * p.d * static_cast<int64_t>(sizeof(float));
  const int64_t cta_bytes = unit_piece_bytes + static_cast<int64_t>(sizeof(UnitMeta));  // per CTA
  // As the standard plan: one resident wave, no more than one unit per 64 path items ...
  int64_t ctas = static_cast<int64_t>(per_sm) * dev.sm_count / g.col_tiles;
  if (ctas < 1) ctas = 1;
  const int64_t path = p.n + p.b;
  const int64_t wanted = (path + 64 * units_per_cta - 1) / (64 * units_per_cta);
  if (wanted < ctas) ctas = wanted < 1 ? 1 : wanted;
  // ... then as many CTAs as the static scratch holds (alignment slack: 512 B).
  const int64_t fit = (kStaticScratchBytes - 512) / cta_bytes;
  const int64_t floor_ctas = wanted < (dev.sm_count + g.col_tiles - 1) / g.col_tiles
                                 ? (wanted < 1 ? 1 : wanted)
                                 : (dev.sm_count + g.col_tiles - 1) / g.col_tiles;
  if (fit < floor_ctas) {
    char buffer[256];
    std::snprintf(buffer, sizeof buffer,
                  "rg_run_noalloc needs %lld bytes of scratch for %lld CTAs; its static scratch holds %lld bytes",
                  static_cast<long long>(floor_ctas * cta_bytes + 512), static_cast<long long>(floor_ctas),
                  static_cast<long long>(kStaticScratchBytes));
    return fail(RG_ERR_WORKSPACE, buffer);
  }
  if (ctas > fit) ctas = fit;
  const int64_t units = ctas * units_per_cta;
  float *pieces = static_cast<float *>(scratch);
  UnitMeta *meta = reinterpret_cast<UnitMeta *>(static_cast<char *>(scratch) + align256(ctas * unit_piece_bytes));
  dim3 grid(static_cast<unsigned>(ctas), g.col_tiles, 1);
  rowbal_kernel<T, OffT, OP, VEC><<<grid, kRowbalThreads, kRowbalSmem, stream>>>(
      static_cast<const T *>(p.values), static_cast<const OffT *>(p.offsets), static_cast<T *>(p.out), p.n, p.b,
      p.d, g.g_shift, g.vec_cols, units, pieces, meta, RowWindow{0, p.n, 1}, nullptr);
  status = check_cuda(cudaGetLastError(), "rowbal_kernel launch (no-alloc)");
  if (status || ctas < 2) return status;
  dim3 fix_grid(static_cast<unsigned>(ctas), g.col_tiles, 1);
  rowbal_fixup_kernel<T, OP, VEC><<<fix_grid, kFixupThreads, 0, stream>>>(static_cast<T *>(p.out), p.d,
                                                                          g.vec_cols, ctas, pieces, meta, nullptr);
  return check_cuda(cudaGetLastError(), "rowbal_fixup_kernel launch (no-alloc)");
}

template <typename T, typename OffT, int OP>
int run_vec(const Problem &p, const Geometry &g, const DeviceProps &dev, void *scratch, cudaStream_t s) {
  switch (g.vec) {
    case 1: return run_typed<T, OffT, OP, 1>(p, g, dev, scratch, s);
    case 2: return run_typed<T, OffT, OP, 2>(p, g, dev, scratch, s);
    case 4: return run_typed<T, OffT, OP, 4>(p, g, dev, scratch, s);
    case 8:
      if constexpr (sizeof(T) == 2) return run_typed<T, OffT, OP, 8>(p, g, dev, scratch, s);
      break;
  }
  return fail(RG_ERR_INVALID_ARGUMENT, "unsupported vector width");
}

template <typename T, typename OffT>
int run_op(const Problem &p, const Geometry &g, const DeviceProps &dev, void *scratch, cudaStream_t s) {
  if (p.op == RG_OP_SUM) return run_vec<T, OffT, OP_SUM>(p, g, dev, scratch, s);
  return run_vec<T, OffT, OP_MAX>(p, g, dev, scratch, s);
}

template <typename T>
int run_index(const Problem &p, const Geometry &g, const DeviceProps &dev, void *scratch, cudaStream_t s) {
  return p.index_dtype == RG_INDEX_I32 ? run_op<T, int32_t>(p, g, dev, scratch, s)
                                       : run_op<T, int64_t>(p, g, dev, scratch, s);
}

}  // namespace

}  // namespace rgb

using namespace rgb;

extern "C" int rg_run_noalloc(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b,
                              const void *values, const void *offsets, void *out, uint32_t flags, void *stream) {
  Problem p{op, dtype, index_dtype, d, n, b, values, offsets, out, -1, flags};
  int status = validate(p);
  if (status) return status;
  if (op != RG_OP_SUM && op != RG_OP_MAX) return fail(RG_ERR_UNSUPPORTED, "rg_run_noalloc computes sum and max only");
  if (b == 0) return RG_OK;
  DeviceProps dev;
  status = check_device(&dev);
  if (status) return status;
  void *scratch = nullptr;
  status = static_scratch(dev.device, &scratch);
  if (status) return status;
  const Geometry g = make_geometry(p);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return p.dtype == RG_DTYPE_F32 ? run_index<float>(p, g, dev, scratch, s)
                                 : run_index<__nv_bfloat16>(p, g, dev, scratch, s);
}
