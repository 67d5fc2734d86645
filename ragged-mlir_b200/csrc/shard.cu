// Row-sharded sum / max across the GPUs of one node (one process per GPU).
//
// Rank r of `world` owns rows [row0, row1) = [r N / world, (r+1) N / world)
// of the packed values (rg_shard_rows) and holds only those rows; every rank
// holds the whole offsets array.  rg_run_shard runs the row-balanced kernel
// over the rank's window of the merge path (rowbal.cuh, RowWindow): the
// window starts at the diagonal of row0 (rows before it plus the segment
// ends at or before it) and ends at the diagonal of row1, so the windows of
// the ranks tile the path and every segment end is consumed by exactly one
// rank.  A segment that starts and ends inside one window is written there;
// the segment open at a window's start and the one open at its end leave
// f32 pieces in the rank's edge record.  The ranks all-gather their edge
// records (NCCL over NVLink, a few KB per rank: torch.distributed in the
// Python layer), and rg_shard_combine finishes, on the rank that consumed
// each cut segment's end, the merge of its pieces in rank order -- so the
// result does not depend on NCCL's reduction order, max keeps NaN
// propagation, and each output row is rounded once.
//
// No kernel here waits on another rank: the exchange is a collective
// between two launches.
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "internal.h"
#include "rowbal.cuh"

namespace rgb {

namespace {

std::mutex g_shard_mutex;
std::map<std::pair<const void *, int>, int> g_shard_occupancy;

int shard_blocks_per_sm(const void *kernel, int device, int *blocks) {
  std::lock_guard<std::mutex> lock(g_shard_mutex);
  const auto key = std::make_pair(kernel, device);
  auto it = g_shard_occupancy.find(key);
  if (it == g_shard_occupancy.end()) {
    int n = 0;
    const int status = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kRowbalThreads, 0),
                                  "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (status) return status;
    it = g_shard_occupancy.emplace(key, n < 1 ? 1 : n).first;
  }
  *blocks = it->second;
  return RG_OK;
}

struct ShardPlan {
  int64_t vctas, grid;
  int64_t pieces_bytes, meta_bytes, counter;
  int64_t stats, stats_bytes;  // softmax: statistics of the window's segments [seg1 - seg0][2][D]
};

// Row-balanced kernel of a sharded call (the softmax statistics pass gets the
// registers of two CTAs per SM, as on one GPU).
template <typename T, typename OffT, int OP, int VEC>
constexpr auto shard_kernel() {
  return &rowbal_kernel<T, OffT, OP, VEC, RowbalTuning::kUnroll, RowbalTuning::kDoubleBuffer,
                        OP == OP_SOFTMAX ? 2 : RowbalTuning::kMinBlocks>;
}

constexpr int64_t kAlign = 256;
int64_t align_up(int64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Virtual CTAs of the row-balanced kernel (several per resident CTA, taken
// from a counter), units of 8 to 64 items of the window's path
// (bounded by its rows plus all segment ends).
template <typename T, typename OffT, int OP, int VEC>
int shard_plan(const Problem &p, const Geometry &g, int64_t rows, int64_t slots, ShardPlan *plan) {
  DeviceProps dev;
  int status = device_props(&dev);
  if (status) return status;
  int per_sm = 0;
  status = shard_blocks_per_sm(reinterpret_cast<const void *>(shard_kernel<T, OffT, OP, VEC>()), dev.device, &per_sm);
  if (status) return status;
  const int units_per_cta = (kRowbalThreads / 32) << (5 - g.g_shift);
  int64_t resident = static_cast<int64_t>(per_sm) * dev.sm_count / g.col_tiles;
  if (resident < 1) resident = 1;
  const int64_t path = rows + p.b;
  const int64_t wanted = rowbal_wanted_ctas(path, resident, units_per_cta);
  const int64_t per = path / (resident * 16384);  // as the single-GPU plan: up to 8 per CTA
  int64_t vctas = resident * (per < 1 ? 1 : (per > 8 ? 8 : per));
  if (vctas > wanted) vctas = wanted;
  plan->vctas = vctas;
  plan->grid = resident < vctas ? resident : vctas;
  const int width = OP == OP_MAX ? 1 : 2;
  plan->pieces_bytes = align_up(vctas * 2 * width * p.d * static_cast<int64_t>(sizeof(float)));
  plan->meta_bytes = align_up(vctas * static_cast<int64_t>(sizeof(UnitMeta)));
  plan->counter = plan->pieces_bytes + plan->meta_bytes;
  plan->stats = plan->counter + kAlign;
  plan->stats_bytes = OP == OP_SOFTMAX ? align_up(slots * 2 * p.d * static_cast<int64_t>(sizeof(float))) : 0;
  return RG_OK;
}

struct ShardCall {
  int64_t row0, row1;
  int first;
  float *edges;
  int64_t seg0 = 0, seg1 = 0;  // softmax: the window's segments (statistics slots)
};

template <typename T, typename OffT, int OP, int VEC>
int shard_typed(const Problem &p, const Geometry &g, const ShardCall &c, void *workspace, int64_t *bytes,
                cudaStream_t stream, rg_report *report) {
  ShardPlan plan;
  int status = shard_plan<T, OffT, OP, VEC>(p, g, c.row1 - c.row0, c.seg1 - c.seg0, &plan);
  if (status) return status;
  if (bytes) {
    *bytes = plan.stats + plan.stats_bytes;
    return RG_OK;
  }
  float *pieces = static_cast<float *>(workspace);
  UnitMeta *meta = reinterpret_cast<UnitMeta *>(static_cast<char *>(workspace) + plan.pieces_bytes);
  unsigned long long *counter = nullptr;  // claims only with more virtual CTAs than resident ones
  if (plan.vctas > plan.grid) {
    counter = reinterpret_cast<unsigned long long *>(static_cast<char *>(workspace) + plan.counter);
    status = check_cuda(cudaMemsetAsync(counter, 0, sizeof *counter, stream), "cudaMemsetAsync");
    if (status) return status;
    if (report) report->memsets += 1;
  }
  const int64_t units = plan.vctas * ((kRowbalThreads / 32) << (5 - g.g_shift));
  // Sum and max write out (all B rows); the softmax statistics pass writes
  // the window's statistics slots.
  T *const target = OP == OP_SOFTMAX ? reinterpret_cast<T *>(static_cast<char *>(workspace) + plan.stats)
                                     : static_cast<T *>(p.out);
  const int64_t seg0 = OP == OP_SOFTMAX ? c.seg0 : 0, seg1 = OP == OP_SOFTMAX ? c.seg1 : 0;
  dim3 grid(static_cast<unsigned>(plan.grid), g.col_tiles, 1);
  shard_kernel<T, OffT, OP, VEC>()<<<grid, kRowbalThreads, kRowbalSmem, stream>>>(
      static_cast<const T *>(p.values), static_cast<const OffT *>(p.offsets), target, p.n, p.b, p.d,
      g.g_shift, g.vec_cols, units, pieces, meta, RowWindow{c.row0, c.row1, c.first, seg0, seg1}, counter,
      Xform{});
  record_launch(report, K_ROWBAL, grid, kRowbalThreads, kRowbalSmem);
  status = check_cuda(cudaGetLastError(), "rowbal_kernel launch (shard)");
  if (status) return status;
  // Every virtual CTA with a TAIL piece, plus one CTA for the window's start
  // and the edge record's header.
  dim3 fix_grid(static_cast<unsigned>(plan.vctas + 1), g.col_tiles, 1);
  rowbal_fixup_kernel<T, OP, VEC><<<fix_grid, kFixupThreads, 0, stream>>>(target, p.d, g.vec_cols, plan.vctas, pieces,
                                                                          meta, c.edges, seg0, seg1);
  record_launch(report, K_ROWBAL_FIXUP, fix_grid, kFixupThreads, 0);
  return check_cuda(cudaGetLastError(), "rowbal_fixup_kernel launch (shard)");
}

template <typename T, typename OffT, int OP>
int shard_vec(const Problem &p, const Geometry &g, const ShardCall &c, void *ws, int64_t *bytes, cudaStream_t s,
              rg_report *r) {
  switch (g.vec) {
    case 1: return shard_typed<T, OffT, OP, 1>(p, g, c, ws, bytes, s, r);
    case 2: return shard_typed<T, OffT, OP, 2>(p, g, c, ws, bytes, s, r);
    case 4: return shard_typed<T, OffT, OP, 4>(p, g, c, ws, bytes, s, r);
    case 8:
      if constexpr (sizeof(T) == 2) return shard_typed<T, OffT, OP, 8>(p, g, c, ws, bytes, s, r);
      break;
  }
  return fail(RG_ERR_INVALID_ARGUMENT, "unsupported vector width");
}

template <typename T>
int shard_dispatch(const Problem &p, const Geometry &g, const ShardCall &c, void *ws, int64_t *bytes, cudaStream_t s,
                   rg_report *r) {
  const bool i32 = p.index_dtype == RG_INDEX_I32;
  if (p.op == RG_OP_SUM)
    return i32 ? shard_vec<T, int32_t, OP_SUM>(p, g, c, ws, bytes, s, r) : shard_vec<T, int64_t, OP_SUM>(p, g, c, ws, bytes, s, r);
  if (p.op == RG_OP_SOFTMAX)
    return i32 ? shard_vec<T, int32_t, OP_SOFTMAX>(p, g, c, ws, bytes, s, r)
               : shard_vec<T, int64_t, OP_SOFTMAX>(p, g, c, ws, bytes, s, r);
  return i32 ? shard_vec<T, int32_t, OP_MAX>(p, g, c, ws, bytes, s, r) : shard_vec<T, int64_t, OP_MAX>(p, g, c, ws, bytes, s, r);
}

// Softmax, after the exchange: the final statistics of the window's cut
// segments from the gathered edge records, then the window's rows
// normalised (values and out hold the window's rows).
template <typename T, typename OffT, int VEC>
int finish_typed(const Problem &p, const Geometry &g, const ShardCall &c, int world, int rank, const float *gathered,
                 void *workspace, cudaStream_t s, rg_report *report) {
  ShardPlan plan;
  int status = shard_plan<T, OffT, OP_SOFTMAX, VEC>(p, g, c.row1 - c.row0, c.seg1 - c.seg0, &plan);
  if (status) return status;
  float *stats = reinterpret_cast<float *>(static_cast<char *>(workspace) + plan.stats);
  dim3 cgrid(1, g.col_tiles, 1);
  shard_softmax_combine_kernel<VEC><<<cgrid, 32, 0, s>>>(stats, p.d, g.vec_cols, world, rank, gathered, c.seg0,
                                                        c.seg1);
  record_launch(report, K_SHARD_COMBINE, cgrid, 32, 0);
  status = check_cuda(cudaGetLastError(), "shard_softmax_combine_kernel launch");
  if (status) return status;
  const int64_t rows = c.row1 - c.row0;
  if (rows == 0) return RG_OK;
  const int units_per_cta = (kRowbalThreads / 32) << (5 - g.g_shift);
  int64_t ctas = plan.grid;
  const int64_t wanted = (rows + 16 * units_per_cta - 1) / (16 * units_per_cta);  // >= 16 rows per unit
  if (ctas > wanted) ctas = wanted;
  if (ctas < 1) ctas = 1;
  dim3 ngrid(static_cast<unsigned>(ctas), g.col_tiles, 1);
  rowbal_normalize_kernel<T, OffT, VEC><<<ngrid, kRowbalThreads, 0, s>>>(
      static_cast<const T *>(p.values), static_cast<const OffT *>(p.offsets), static_cast<T *>(p.out), stats, rows,
      p.b, p.d, g.g_shift, g.vec_cols, ctas * units_per_cta, c.row0, c.seg0, c.seg1);
  record_launch(report, K_ROWBAL_NORMALIZE, ngrid, kRowbalThreads, 0);
  return check_cuda(cudaGetLastError(), "rowbal_normalize_kernel launch (shard)");
}

template <typename T, typename OffT>
int finish_vec(const Problem &p, const Geometry &g, const ShardCall &c, int world, int rank, const float *gathered,
               void *ws, cudaStream_t s, rg_report *r) {
  switch (g.vec) {
    case 1: return finish_typed<T, OffT, 1>(p, g, c, world, rank, gathered, ws, s, r);
    case 2: return finish_typed<T, OffT, 2>(p, g, c, world, rank, gathered, ws, s, r);
    case 4: return finish_typed<T, OffT, 4>(p, g, c, world, rank, gathered, ws, s, r);
    case 8:
      if constexpr (sizeof(T) == 2) return finish_typed<T, OffT, 8>(p, g, c, world, rank, gathered, ws, s, r);
      break;
  }
  return fail(RG_ERR_INVALID_ARGUMENT, "unsupported vector width");
}

int finish_run(const Problem &p, const Geometry &g, const ShardCall &c, int world, int rank, const float *gathered,
               void *ws, cudaStream_t s, rg_report *r) {
  const bool i32 = p.index_dtype == RG_INDEX_I32;
  if (p.dtype == RG_DTYPE_F32)
    return i32 ? finish_vec<float, int32_t>(p, g, c, world, rank, gathered, ws, s, r)
               : finish_vec<float, int64_t>(p, g, c, world, rank, gathered, ws, s, r);
  return i32 ? finish_vec<__nv_bfloat16, int32_t>(p, g, c, world, rank, gathered, ws, s, r)
             : finish_vec<__nv_bfloat16, int64_t>(p, g, c, world, rank, gathered, ws, s, r);
}

int shard_run(const Problem &p, const Geometry &g, const ShardCall &c, void *ws, int64_t *bytes, cudaStream_t s,
              rg_report *r) {
  return p.dtype == RG_DTYPE_F32 ? shard_dispatch<float>(p, g, c, ws, bytes, s, r)
                                 : shard_dispatch<__nv_bfloat16>(p, g, c, ws, bytes, s, r);
}

template <typename T, int OP>
int combine_typed(const Geometry &g, int64_t d, int world, int rank, const float *gathered, T *out, cudaStream_t s) {
  dim3 grid(1, g.col_tiles, 1);
  switch (g.vec) {
    case 1: shard_combine_kernel<T, OP, 1><<<grid, 32, 0, s>>>(out, d, g.vec_cols, world, rank, gathered); break;
    case 2: shard_combine_kernel<T, OP, 2><<<grid, 32, 0, s>>>(out, d, g.vec_cols, world, rank, gathered); break;
    case 4: shard_combine_kernel<T, OP, 4><<<grid, 32, 0, s>>>(out, d, g.vec_cols, world, rank, gathered); break;
    case 8:
      if constexpr (sizeof(T) == 2) {
        shard_combine_kernel<T, OP, 8><<<grid, 32, 0, s>>>(out, d, g.vec_cols, world, rank, gathered);
        break;
      }
      return fail(RG_ERR_INVALID_ARGUMENT, "unsupported vector width");
    default: return fail(RG_ERR_INVALID_ARGUMENT, "unsupported vector width");
  }
  return check_cuda(cudaGetLastError(), "shard_combine_kernel launch");
}

// Op and split checks shared by the shard entry points; the rank's rows:
// splits[rank], splits[rank + 1] from the caller's split (host memory,
// world + 1 nondecreasing entries from 0 to n), or the even row split.
int shard_window(int op, int64_t n, int world, int rank, const int64_t *splits, int64_t *row0, int64_t *row1) {
  if (op < RG_OP_SUM || op > RG_OP_SOFTMAX) return fail(RG_ERR_INVALID_ARGUMENT, "op must be sum, max or softmax");
  if (n < 0 || world < 1 || rank < 0 || rank >= world)
    return fail(RG_ERR_INVALID_ARGUMENT, "need N >= 0, world >= 1 and 0 <= rank < world");
  if (splits) {
    if (splits[0] != 0 || splits[world] != n)
      return fail(RG_ERR_INVALID_ARGUMENT, "a split must run from row 0 to row N");
    for (int k = 0; k < world; ++k)
      if (splits[k] > splits[k + 1]) return fail(RG_ERR_INVALID_ARGUMENT, "split boundaries must not decrease");
    *row0 = splits[rank];
    *row1 = splits[rank + 1];
    return RG_OK;
  }
  const int64_t q = n / world, rem = n % world;
  *row0 = q * rank + (rank < rem ? rank : rem);
  *row1 = *row0 + q + (rank < rem ? 1 : 0);
  return RG_OK;
}

// Segment ends at or before row r (host offsets).
template <typename OffT>
int64_t ends_at_or_before(const OffT *offsets, int64_t b, int64_t r) {
  int64_t lo = 0, hi = b;  // first k with offsets[k+1] > r
  while (lo < hi) {
    const int64_t mid = lo + (hi - lo) / 2;
    if (static_cast<int64_t>(offsets[mid + 1]) > r) hi = mid; else lo = mid + 1;
  }
  return lo;
}

template <typename OffT>
void balanced_split(const OffT *offsets, int64_t b, int world, double end_weight, int64_t *splits) {
  const int64_t n = b > 0 ? static_cast<int64_t>(offsets[b]) : 0;
  const double total = static_cast<double>(n) + end_weight * static_cast<double>(b);
  splits[0] = 0;
  for (int k = 1; k < world; ++k) {
    const double target = total * k / world;
    int64_t lo = splits[k - 1], hi = n;  // first row r with cost(r) >= target
    while (lo < hi) {
      const int64_t mid = lo + (hi - lo) / 2;
      const double cost = static_cast<double>(mid) + end_weight * static_cast<double>(ends_at_or_before(offsets, b, mid));
      if (cost >= target) hi = mid; else lo = mid + 1;
    }
    splits[k] = lo;
  }
  splits[world] = n;
}

}  // namespace

}  // namespace rgb

using namespace rgb;

extern "C" {

int rg_shard_rows(int64_t n, int world, int rank, int64_t *row0, int64_t *row1) {
  if (!row0 || !row1) return fail(RG_ERR_INVALID_ARGUMENT, "row0 and row1 must not be NULL");
  if (n < 0 || world < 1 || rank < 0 || rank >= world)
    return fail(RG_ERR_INVALID_ARGUMENT, "need N >= 0, world >= 1 and 0 <= rank < world");
  // Row-balanced split; n / world * r + min(r, n % world) avoids overflow.
  return shard_window(RG_OP_SUM, n, world, rank, nullptr, row0, row1);
}

int rg_shard_split(const void *offsets, int index_dtype, int64_t b, int world, double end_weight, int64_t *splits) {
  if (!offsets || !splits) return fail(RG_ERR_INVALID_ARGUMENT, "offsets and splits must not be NULL");
  if (b < 0 || world < 1) return fail(RG_ERR_INVALID_ARGUMENT, "need B >= 0 and world >= 1");
  if (!(end_weight >= 0.0)) return fail(RG_ERR_INVALID_ARGUMENT, "end_weight must be nonnegative");
  if (index_dtype == RG_INDEX_I32) balanced_split(static_cast<const int32_t *>(offsets), b, world, end_weight, splits);
  else if (index_dtype == RG_INDEX_I64) balanced_split(static_cast<const int64_t *>(offsets), b, world, end_weight, splits);
  else return fail(RG_ERR_INVALID_ARGUMENT, "offsets dtype must be i32 or i64");
  return RG_OK;
}

int rg_shard_edge_bytes(int op, int64_t d, int64_t *bytes) {
  if (!bytes) return fail(RG_ERR_INVALID_ARGUMENT, "bytes is NULL");
  if (d < 1 || d > 1024) return fail(RG_ERR_INVALID_ARGUMENT, "D must lie in [1, 1024]");
  if (op < RG_OP_SUM || op > RG_OP_SOFTMAX) return fail(RG_ERR_INVALID_ARGUMENT, "op must be sum, max or softmax");
  const int64_t width = op == RG_OP_MAX ? 1 : 2;
  *bytes = edge_record_floats(width * d) * static_cast<int64_t>(sizeof(float));
  return RG_OK;
}

int rg_shard_workspace_bytes(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, int world,
                             int rank, const int64_t *splits, uint32_t flags, int64_t *bytes) {
  if (!bytes) return fail(RG_ERR_INVALID_ARGUMENT, "bytes is NULL");
  if (op == RG_OP_SOFTMAX) return fail(RG_ERR_INVALID_ARGUMENT, "softmax: rg_shard_softmax_workspace_bytes");
  int64_t row0 = 0, row1 = 0;
  int status = shard_window(op, n, world, rank, splits, &row0, &row1);
  if (status) return status;
  Problem p{op, dtype, index_dtype, d, n, b, nullptr, nullptr, nullptr, -1, flags};
  if ((dtype != RG_DTYPE_F32 && dtype != RG_DTYPE_BF16) || (index_dtype != RG_INDEX_I32 && index_dtype != RG_INDEX_I64) ||
      d < 1 || d > 1024 || b < 0)
    return fail(RG_ERR_INVALID_ARGUMENT, "invalid problem description");
  if (b == 0) {
    *bytes = 0;
    return RG_OK;
  }
  DeviceProps dev;
  status = check_device(&dev);
  if (status) return status;
  return shard_run(p, make_geometry(p), ShardCall{row0, row1, rank == 0, nullptr}, nullptr, bytes, nullptr, nullptr);
}

int rg_run_shard(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, int world, int rank,
                 const int64_t *splits, const void *values, const void *offsets, void *out, void *edges,
                 void *workspace, int64_t workspace_bytes, uint32_t flags, void *stream, rg_report *report) {
  if (report) {
    std::memset(report, 0, sizeof *report);
    report->status_offset = -1;
    report->schedule = RG_SCHEDULE_ROWBALANCED;
    report->streams = 1;
  }
  if (op == RG_OP_SOFTMAX) return fail(RG_ERR_INVALID_ARGUMENT, "softmax: rg_run_shard_softmax");
  int64_t row0 = 0, row1 = 0;
  int status = shard_window(op, n, world, rank, splits, &row0, &row1);
  if (status) return status;
  // The local tensors: values holds the window's rows, out all B rows.
  Problem local{op, dtype, index_dtype, d, row1 - row0, b, values, offsets, out, -1, flags};
  if (index_dtype == RG_INDEX_I32 && n > 2147483647LL) return fail(RG_ERR_INVALID_ARGUMENT, "N exceeds the i32 offsets range");
  if (b == 0 && n != 0) return fail(RG_ERR_INVALID_ARGUMENT, "B=0 requires N=0");
  if (b > 0) {
    status = validate(local);
    if (status) return status;
  }
  if (!edges) return fail(RG_ERR_INVALID_ARGUMENT, "edges must hold rg_shard_edge_bytes() bytes of device memory");
  if (reinterpret_cast<uintptr_t>(edges) % 16) return fail(RG_ERR_INVALID_ARGUMENT, "edges must be 16-byte aligned");
  const Geometry g = make_geometry(local);
  if (report) {
    report->d_vector = g.vec;
    report->d_tile = 1 << g.g_shift;
  }
  DeviceProps dev;
  status = check_device(&dev);
  if (status) return status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Problem p{op, dtype, index_dtype, d, n, b, values, offsets, out, -1, flags};
  if (b == 0) {
    // No segments: an all-ones header (every field -1) says "nothing cut".
    return check_cuda(cudaMemsetAsync(edges, 0xff, kEdgeHeader * sizeof(float), s), "cudaMemsetAsync (edges)");
  }
  int64_t need = 0;
  status = shard_run(p, g, ShardCall{row0, row1, rank == 0, nullptr}, nullptr, &need, nullptr, nullptr);
  if (status) return status;
  if (report) report->workspace_bytes = need;
  if (!workspace || workspace_bytes < need) return fail(RG_ERR_WORKSPACE, "workspace missing or too small");
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return fail(RG_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  return shard_run(p, g, ShardCall{row0, row1, rank == 0, static_cast<float *>(edges)}, workspace, nullptr, s, report);
}

int rg_shard_combine(int op, int dtype, int64_t d, int world, int rank, const void *gathered, void *out,
                     uint32_t flags, void *stream) {
  if (op != RG_OP_SUM && op != RG_OP_MAX) return fail(RG_ERR_INVALID_ARGUMENT, "softmax: rg_shard_softmax_finish");
  if (dtype != RG_DTYPE_F32 && dtype != RG_DTYPE_BF16) return fail(RG_ERR_INVALID_ARGUMENT, "dtype must be f32 or bf16");
  if (d < 1 || d > 1024) return fail(RG_ERR_INVALID_ARGUMENT, "D must lie in [1, 1024]");
  if (world < 1 || rank < 0 || rank >= world) return fail(RG_ERR_INVALID_ARGUMENT, "need 0 <= rank < world");
  if (!gathered || !out) return fail(RG_ERR_INVALID_ARGUMENT, "gathered and out must not be NULL");
  if (rank == 0) return RG_OK;  // rank 0 has no segment open at its start
  DeviceProps dev;
  int status = check_device(&dev);
  if (status) return status;
  Problem p{op, dtype, RG_INDEX_I64, d, 0, 1, nullptr, nullptr, out, -1, flags};
  const Geometry g = make_geometry(p);
  if (reinterpret_cast<uintptr_t>(out) % (g.vec * elem_bytes(dtype)))
    return fail(RG_ERR_INVALID_ARGUMENT, "out is not aligned for this call's vector width");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float *gath = static_cast<const float *>(gathered);
  if (dtype == RG_DTYPE_F32) {
    return op == RG_OP_SUM ? combine_typed<float, OP_SUM>(g, d, world, rank, gath, static_cast<float *>(out), s)
                           : combine_typed<float, OP_MAX>(g, d, world, rank, gath, static_cast<float *>(out), s);
  }
  return op == RG_OP_SUM
             ? combine_typed<__nv_bfloat16, OP_SUM>(g, d, world, rank, gath, static_cast<__nv_bfloat16 *>(out), s)
             : combine_typed<__nv_bfloat16, OP_MAX>(g, d, world, rank, gath, static_cast<__nv_bfloat16 *>(out), s);
}

// ------------------------------------------------------------ sharded softmax

int rg_shard_segments(const void *offsets, int index_dtype, int64_t b, int world, int rank, const int64_t *splits,
                      int64_t *seg0, int64_t *seg1) {
  if (!offsets || !seg0 || !seg1) return fail(RG_ERR_INVALID_ARGUMENT, "offsets, seg0 and seg1 must not be NULL");
  if (b < 0) return fail(RG_ERR_INVALID_ARGUMENT, "B must be nonnegative");
  if (index_dtype != RG_INDEX_I32 && index_dtype != RG_INDEX_I64)
    return fail(RG_ERR_INVALID_ARGUMENT, "offsets dtype must be i32 or i64");
  const bool i32 = index_dtype == RG_INDEX_I32;
  const int64_t n = b == 0 ? 0 : (i32 ? static_cast<const int32_t *>(offsets)[b] : static_cast<const int64_t *>(offsets)[b]);
  int64_t row0 = 0, row1 = 0;
  int status = shard_window(RG_OP_SOFTMAX, n, world, rank, splits, &row0, &row1);
  if (status) return status;
  auto ends = [&](int64_t r) {
    return i32 ? ends_at_or_before(static_cast<const int32_t *>(offsets), b, r)
               : ends_at_or_before(static_cast<const int64_t *>(offsets), b, r);
  };
  // Segments whose end this window consumes, plus the one open at its end.
  *seg0 = rank == 0 ? 0 : ends(row0);
  const int64_t hi = ends(row1) + 1;
  *seg1 = hi < b ? hi : b;
  if (*seg1 < *seg0) *seg1 = *seg0;
  return RG_OK;
}

int rg_shard_softmax_workspace_bytes(int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, int world,
                                     int rank, const int64_t *splits, int64_t seg0, int64_t seg1, uint32_t flags,
                                     int64_t *bytes) {
  if (!bytes) return fail(RG_ERR_INVALID_ARGUMENT, "bytes is NULL");
  int64_t row0 = 0, row1 = 0;
  int status = shard_window(RG_OP_SOFTMAX, n, world, rank, splits, &row0, &row1);
  if (status) return status;
  if ((dtype != RG_DTYPE_F32 && dtype != RG_DTYPE_BF16) || (index_dtype != RG_INDEX_I32 && index_dtype != RG_INDEX_I64) ||
      d < 1 || d > 1024 || b < 0 || seg0 < 0 || seg1 < seg0 || seg1 > b)
    return fail(RG_ERR_INVALID_ARGUMENT, "invalid problem description or segment range");
  if (b == 0) {
    *bytes = 0;
    return RG_OK;
  }
  DeviceProps dev;
  status = check_device(&dev);
  if (status) return status;
  Problem p{RG_OP_SOFTMAX, dtype, index_dtype, d, n, b, nullptr, nullptr, nullptr, -1, flags};
  ShardCall c{row0, row1, rank == 0, nullptr};
  c.seg0 = seg0;
  c.seg1 = seg1;
  return shard_run(p, make_geometry(p), c, nullptr, bytes, nullptr, nullptr);
}

// Checks shared by the two softmax phases; fills the call.
static int softmax_shard_call(int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, int world, int rank,
                              const int64_t *splits, int64_t seg0, int64_t seg1, const void *values,
                              const void *offsets, void *out, void *workspace, int64_t workspace_bytes,
                              uint32_t flags, Problem *p, Geometry *g, ShardCall *c) {
  int64_t row0 = 0, row1 = 0;
  int status = shard_window(RG_OP_SOFTMAX, n, world, rank, splits, &row0, &row1);
  if (status) return status;
  if (index_dtype == RG_INDEX_I32 && n > 2147483647LL) return fail(RG_ERR_INVALID_ARGUMENT, "N exceeds the i32 offsets range");
  if (b == 0 && n != 0) return fail(RG_ERR_INVALID_ARGUMENT, "B=0 requires N=0");
  if (seg0 < 0 || seg1 < seg0 || seg1 > b) return fail(RG_ERR_INVALID_ARGUMENT, "invalid segment range");
  // The local problem: values and out hold the window's rows.  The
  // statistics phase writes no rows (out NULL): its checks see an in-place
  // call.
  const uint32_t kept = flags & (RG_FLAG_NO_VECTORIZE | RG_FLAG_IN_PLACE);
  Problem local{RG_OP_SOFTMAX, dtype, index_dtype, d, row1 - row0, b, values, offsets, out ? out : const_cast<void *>(values),
                -1, out ? kept : (kept | RG_FLAG_IN_PLACE)};
  if (b > 0) {
    status = validate(local);
    if (status) return status;
  }
  *g = make_geometry(local);
  DeviceProps dev;
  status = check_device(&dev);
  if (status) return status;
  *p = Problem{RG_OP_SOFTMAX, dtype, index_dtype, d, n, b, values, offsets, out, -1, flags & RG_FLAG_NO_VECTORIZE};
  *c = ShardCall{row0, row1, rank == 0, nullptr};
  c->seg0 = seg0;
  c->seg1 = seg1;
  if (b == 0) return RG_OK;
  int64_t need = 0;
  status = shard_run(*p, *g, *c, nullptr, &need, nullptr, nullptr);
  if (status) return status;
  if (!workspace || workspace_bytes < need) return fail(RG_ERR_WORKSPACE, "workspace missing or too small");
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return fail(RG_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  return RG_OK;
}

int rg_run_shard_softmax(int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, int world, int rank,
                         const int64_t *splits, int64_t seg0, int64_t seg1, const void *values, const void *offsets,
                         void *edges, void *workspace, int64_t workspace_bytes, uint32_t flags, void *stream,
                         rg_report *report) {
  if (report) {
    std::memset(report, 0, sizeof *report);
    report->status_offset = -1;
    report->schedule = RG_SCHEDULE_ROWBALANCED;
    report->streams = 1;
  }
  if (!edges) return fail(RG_ERR_INVALID_ARGUMENT, "edges must hold rg_shard_edge_bytes() bytes of device memory");
  if (reinterpret_cast<uintptr_t>(edges) % 16) return fail(RG_ERR_INVALID_ARGUMENT, "edges must be 16-byte aligned");
  Problem p{};
  Geometry g{};
  ShardCall c{0, 0, 0, nullptr};
  // out is written only by the finishing phase; pass values as a stand-in.
  int status = softmax_shard_call(dtype, index_dtype, d, n, b, world, rank, splits, seg0, seg1, values, offsets,
                                  nullptr, workspace, workspace_bytes, flags, &p, &g, &c);
  if (status) return status;
  if (report) {
    report->d_vector = g.vec;
    report->d_tile = 1 << g.g_shift;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (b == 0) return check_cuda(cudaMemsetAsync(edges, 0xff, kEdgeHeader * sizeof(float), s), "cudaMemsetAsync (edges)");
  c.edges = static_cast<float *>(edges);
  return shard_run(p, g, c, workspace, nullptr, s, report);
}

int rg_shard_softmax_finish(int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, int world, int rank,
                            const int64_t *splits, int64_t seg0, int64_t seg1, const void *values, const void *offsets,
                            const void *gathered, void *out, void *workspace, int64_t workspace_bytes, uint32_t flags,
                            void *stream, rg_report *report) {
  if (report) {
    std::memset(report, 0, sizeof *report);
    report->status_offset = -1;
    report->schedule = RG_SCHEDULE_ROWBALANCED;
    report->streams = 1;
  }
  if (!gathered) return fail(RG_ERR_INVALID_ARGUMENT, "gathered must hold every rank's edge record");
  Problem p{};
  Geometry g{};
  ShardCall c{0, 0, 0, nullptr};
  int status = softmax_shard_call(dtype, index_dtype, d, n, b, world, rank, splits, seg0, seg1, values, offsets, out,
                                  workspace, workspace_bytes, flags, &p, &g, &c);
  if (status || b == 0) return status;
  if (report) {
    report->d_vector = g.vec;
    report->d_tile = 1 << g.g_shift;
  }
  return finish_run(p, g, c, world, rank, static_cast<const float *>(gathered), workspace,
                    static_cast<cudaStream_t>(stream), report);
}

}  // extern "C"
