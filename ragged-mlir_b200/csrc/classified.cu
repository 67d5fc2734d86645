// Workspace layout and launches of the classified schedule (classified.cuh).
//
// Workspace (each part 256-byte aligned), sized from N and B only -- never
// from the caller's max_len, so a wrong hint cannot under-size it:
//   state      ClsState counters                       } zeroed by one
//   done       [splits][col_tiles] u32 chunk counters  } cudaMemsetAsync
//   late       softmax: [chunks] u32 flags             }
//   ids        [B] i64 warp-class ids (from the front), CTA-class ids (from the back)
//   split_seg  [splits] i64,  split_base [splits] i64 (first chunk number)
//   partials   [chunks][W][D] f32
//   seg_stats  softmax only: [splits][2][D] f32
// with T = item_rows (the CTA-class bound and chunk length), splits =
// min(B, N / (T + 1)) (the reference's B_split rule, docs/classified-abi.md
// "B_split") and chunks = N / T + splits.
#include <cstddef>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "internal.h"
#include "pipeline.cuh"

namespace rgb {

namespace {

constexpr int64_t kAlign = 256;
int64_t align_up(int64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct ClsLayout {
  int64_t splits, chunks;
  int64_t state, done, late, ids, split_seg, split_base, partials, seg_stats, total;
  int64_t memset_bytes;
};

// Rows that bulk copies can stage: one column tile and 16-byte vectors (so
// every row starts on a 16-byte boundary; rg_run checks the base address).
bool staged_of(const Problem &p, const Geometry &g) {
  return g.col_tiles == 1 && g.vec * elem_bytes(p.dtype) == 16 && (p.d * elem_bytes(p.dtype)) % 16 == 0;
}

template <int OP>
int pipe_stage_bytes_vec(int vec) {
  switch (vec) {
    case 1: return PipeLayout<OP, 1>::kStageBytes;
    case 2: return PipeLayout<OP, 2>::kStageBytes;
    case 4: return PipeLayout<OP, 4>::kStageBytes;
    default: return PipeLayout<OP, 8>::kStageBytes;
  }
}

int pipe_stage_bytes(int op, int vec) {
  switch (op) {
    case RG_OP_SUM: return pipe_stage_bytes_vec<OP_SUM>(vec);
    case RG_OP_MAX: return pipe_stage_bytes_vec<OP_MAX>(vec);
    default: return pipe_stage_bytes_vec<OP_SOFTMAX>(vec);
  }
}

// Rows of one CTA item (CTA-class bound, split chunk length): 4096 rows
// (the reference's bound), or fewer: one shared-memory stage of the
// pipelined worker, or 64 KiB of one column tile (at least 64 rows) for the
// unstaged worker.
int64_t item_rows_of(const Problem &p, const Geometry &g) {
  int64_t rows;
  if (staged_of(p, g)) {
    rows = pipe_stage_bytes(p.op, g.vec) / (p.d * elem_bytes(p.dtype));
  } else {
    const int64_t tile_bytes =
        static_cast<int64_t>(g.vec_cols < 32 ? g.vec_cols : 32) * g.vec * elem_bytes(p.dtype);
    rows = kItemBytes / tile_bytes;
    if (rows < 64) rows = 64;
  }
  return rows > kCtaClassMax ? kCtaClassMax : rows;
}

ClsLayout layout_of(const Problem &p, const Geometry &g) {
  ClsLayout l{};
  const int64_t item_rows = item_rows_of(p, g);
  l.splits = p.n / (item_rows + 1);
  if (l.splits > p.b) l.splits = p.b;
  l.chunks = p.n / item_rows + l.splits;
  const int width = p.op == RG_OP_MAX ? 1 : 2;
  int64_t at = 0;
  l.state = at;
  at += align_up(sizeof(ClsState));
  l.done = at;
  at += align_up(l.splits * g.col_tiles * static_cast<int64_t>(sizeof(unsigned)));
  l.late = at;
  if (p.op == RG_OP_SOFTMAX) at += align_up(l.chunks * static_cast<int64_t>(sizeof(unsigned)));
  l.memset_bytes = at;
  l.ids = at;
  at += align_up(p.b * 8);
  l.split_seg = at;
  at += align_up(l.splits * 8);
  l.split_base = at;
  at += align_up(l.splits * 8);
  l.partials = at;
  at += align_up(l.chunks * width * p.d * 4);
  l.seg_stats = at;
  if (p.op == RG_OP_SOFTMAX) at += align_up(l.splits * 2 * p.d * 4);
  l.total = at;
  return l;
}

// Polls before a worker's wait for a split segment gives up: kChunkWaitPolls,
// or RAGGED_B200_CHUNK_WAIT_POLLS (read once; 0 makes every wait give up at
// once, which exercises the late-chunk path of split_normalize_kernel).
int chunk_wait_polls() {
  static const int polls = [] {
    const char *text = std::getenv("RAGGED_B200_CHUNK_WAIT_POLLS");
    if (!text || !*text) return kChunkWaitPolls;
    const long value = std::strtol(text, nullptr, 10);
    return value < 0 ? 0 : (value > kChunkWaitPolls ? kChunkWaitPolls : static_cast<int>(value));
  }();
  return polls;
}

std::mutex g_occ_mutex;
std::map<std::pair<const void *, int>, int> g_occ;

// Resident CTAs per SM of `kernel` with `smem` bytes of dynamic shared
// memory; the first query per device also raises the kernel's dynamic
// shared-memory limit to `smem`.
int blocks_per_sm(const void *kernel, int device, int threads, int smem, int *blocks) {
  std::lock_guard<std::mutex> lock(g_occ_mutex);
  const auto key = std::make_pair(kernel, device);
  auto it = g_occ.find(key);
  if (it == g_occ.end()) {
    int status = RG_OK;
    if (smem > 0) {
      status = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                          "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
      if (status) return status;
    }
    int n = 0;
    status = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem),
                        "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    if (status) return status;
    it = g_occ.emplace(key, n < 1 ? 1 : n).first;
  }
  *blocks = it->second;
  return RG_OK;
}

// XF (softmax, staged rows only): the input transform `xf` fused into the
// worker's and the normalise kernel's loads.
template <typename T, typename OffT, int OP, int VEC, bool STAGED, bool XF = false>
int launch_typed(const Problem &p, const Geometry &g, char *ws, cudaStream_t stream, rg_report *report,
                 const Xform &xf = Xform{}) {
  DeviceProps dev;
  int status = device_props(&dev);
  if (status) return status;
  const ClsLayout l = layout_of(p, g);
  ClsArgs a;
  a.b = p.b;
  a.d = p.d;
  a.item_rows = item_rows_of(p, g);
  a.row_bytes = static_cast<int>(p.d * elem_bytes(p.dtype));
  a.g_shift = g.g_shift;
  a.vec_cols = g.vec_cols;
  a.col_tiles = g.col_tiles;
  a.state = reinterpret_cast<ClsState *>(ws + l.state);
  a.done = reinterpret_cast<unsigned *>(ws + l.done);
  a.ids = reinterpret_cast<const int64_t *>(ws + l.ids);
  a.split_seg = reinterpret_cast<const int64_t *>(ws + l.split_seg);
  a.split_base = reinterpret_cast<const int64_t *>(ws + l.split_base);
  a.partials = reinterpret_cast<float *>(ws + l.partials);
  a.seg_stats = reinterpret_cast<float *>(ws + l.seg_stats);
  a.wait_rows = 0;
  a.late = reinterpret_cast<unsigned *>(ws + l.late);
  a.wait_polls = chunk_wait_polls();
  a.xform = xf;
  a.claim = kPipeClaim;

  // The pipelined worker's grid (one resident wave).  Softmax split segments
  // of at most min(kWaitChunks, ctas / 2) chunks are normalised by the
  // worker itself (classified.cuh, normalized_in_worker: the waiting teams
  // of the one partly claimed segment then hold stages of fewer than half
  // the CTAs, so the others keep claiming its chunks).
  int per_sm = 0;
  int64_t pipe_ctas = 0;
  if constexpr (STAGED) {
    using PL = PipeLayout<OP, VEC>;
    const void *worker = reinterpret_cast<const void *>(&pipe_worker_kernel<T, OffT, OP, VEC, XF>);
    status = blocks_per_sm(worker, dev.device, kPipeThreads, PL::kTotalBytes, &per_sm);
    if (status) return status;
    pipe_ctas = static_cast<int64_t>(per_sm) * dev.sm_count;
    const int64_t max_items = (p.b + kPipeClaim - 1) / kPipeClaim + l.chunks;
    if (pipe_ctas > max_items) pipe_ctas = max_items;
    if (pipe_ctas < 1) pipe_ctas = 1;
    // Many segments per CTA (8 claims of kRunMax each or more): claims of
    // kRunMax segments, so runs of short segments fill more of a stage.
    if (p.b >= pipe_ctas * 8 * kRunMax) a.claim = kRunMax;
    if constexpr (OP == OP_SOFTMAX) {
      const int64_t wait_chunks = pipe_ctas / 2 < kWaitChunks ? pipe_ctas / 2 : kWaitChunks;
      a.wait_rows = wait_chunks * a.item_rows;
    }
  }

  status = check_cuda(cudaMemsetAsync(ws, 0, static_cast<size_t>(l.memset_bytes), stream), "cudaMemsetAsync");
  if (status) return status;
  if (report) report->memsets += 1;

  const OffT *offsets = static_cast<const OffT *>(p.offsets);
  int64_t cls_blocks = (p.b + 255) / 256;
  if (cls_blocks > static_cast<int64_t>(dev.sm_count) * 8) cls_blocks = static_cast<int64_t>(dev.sm_count) * 8;
  dim3 cgrid(static_cast<unsigned>(cls_blocks), 1, 1);
  classify_kernel<OffT><<<cgrid, 256, 0, stream>>>(offsets, p.b, a.item_rows, p.op == RG_OP_SOFTMAX, STAGED ? 1 : 0,
                                                   a.wait_rows, a.state, reinterpret_cast<int64_t *>(ws + l.ids),
                                                   reinterpret_cast<int64_t *>(ws + l.split_seg),
                                                   reinterpret_cast<int64_t *>(ws + l.split_base));
  record_launch(report, K_CLASSIFY, cgrid, 256, 0);
  status = check_cuda(cudaGetLastError(), "classify_kernel launch");
  if (status) return status;

  if constexpr (STAGED) {
    using PL = PipeLayout<OP, VEC>;
    dim3 wgrid(static_cast<unsigned>(pipe_ctas), 1, 1);
    pipe_worker_kernel<T, OffT, OP, VEC, XF><<<wgrid, kPipeThreads, PL::kTotalBytes, stream>>>(
        static_cast<const T *>(p.values), offsets, static_cast<T *>(p.out), a);
    record_launch(report, K_WORKER, wgrid, kPipeThreads, PL::kTotalBytes);
    status = check_cuda(cudaGetLastError(), "pipe_worker_kernel launch");
  } else {
    const void *worker = reinterpret_cast<const void *>(&cls_worker_kernel<T, OffT, OP, VEC>);
    status = blocks_per_sm(worker, dev.device, kClsThreads, 0, &per_sm);
    if (status) return status;
    const int64_t max_items = (l.chunks + p.b + (p.b + kWarpSegsPerItem - 1) / kWarpSegsPerItem) * g.col_tiles;
    int64_t ctas = static_cast<int64_t>(per_sm) * dev.sm_count;
    if (ctas > max_items) ctas = max_items;
    if (ctas < 1) ctas = 1;
    dim3 wgrid(static_cast<unsigned>(ctas), 1, 1);
    cls_worker_kernel<T, OffT, OP, VEC><<<wgrid, kClsThreads, 0, stream>>>(
        static_cast<const T *>(p.values), offsets, static_cast<T *>(p.out), a);
    record_launch(report, K_WORKER, wgrid, kClsThreads, 0);
    status = check_cuda(cudaGetLastError(), "cls_worker_kernel launch");
  }
  if (status) return status;

  if constexpr (OP == OP_SOFTMAX) {
    if (l.splits > 0) {
      const void *norm = reinterpret_cast<const void *>(&split_normalize_kernel<T, OffT, VEC, XF>);
      status = blocks_per_sm(norm, dev.device, kClsThreads, 0, &per_sm);
      if (status) return status;
      int64_t nctas = static_cast<int64_t>(per_sm) * dev.sm_count;
      const int64_t warps_needed = l.chunks * g.col_tiles;  // one warp per chunk and column tile
      if (nctas > (warps_needed + kClsWarps - 1) / kClsWarps) nctas = (warps_needed + kClsWarps - 1) / kClsWarps;
      if (nctas < 1) nctas = 1;
      dim3 ngrid(static_cast<unsigned>(nctas), 1, 1);
      split_normalize_kernel<T, OffT, VEC, XF><<<ngrid, kClsThreads, 0, stream>>>(
          static_cast<const T *>(p.values), offsets, static_cast<T *>(p.out), a);
      record_launch(report, K_SPLIT_NORMALIZE, ngrid, kClsThreads, 0);
      status = check_cuda(cudaGetLastError(), "split_normalize_kernel launch");
    }
  }
  return status;
}

template <typename T, typename OffT, int OP, int VEC>
int launch_staging(const Problem &p, const Geometry &g, char *ws, cudaStream_t s, rg_report *r) {
  if constexpr (VEC * sizeof(T) == 16) {
    if (staged_of(p, g)) return launch_typed<T, OffT, OP, VEC, true>(p, g, ws, s, r);
  }
  return launch_typed<T, OffT, OP, VEC, false>(p, g, ws, s, r);
}

template <typename T, typename OffT, int OP>
int launch_vec(const Problem &p, const Geometry &g, char *ws, cudaStream_t s, rg_report *r) {
  switch (g.vec) {
    case 1: return launch_staging<T, OffT, OP, 1>(p, g, ws, s, r);
    case 2: return launch_staging<T, OffT, OP, 2>(p, g, ws, s, r);
    case 4: return launch_staging<T, OffT, OP, 4>(p, g, ws, s, r);
    case 8:
      if constexpr (sizeof(T) == 2) return launch_staging<T, OffT, OP, 8>(p, g, ws, s, r);
      break;
  }
  return fail(RG_ERR_INVALID_ARGUMENT, "unsupported vector width");
}

template <typename T, typename OffT>
int launch_op(const Problem &p, const Geometry &g, char *ws, cudaStream_t s, rg_report *r) {
  switch (p.op) {
    case RG_OP_SUM: return launch_vec<T, OffT, OP_SUM>(p, g, ws, s, r);
    case RG_OP_MAX: return launch_vec<T, OffT, OP_MAX>(p, g, ws, s, r);
    case RG_OP_SOFTMAX: return launch_vec<T, OffT, OP_SOFTMAX>(p, g, ws, s, r);
  }
  return fail(RG_ERR_INVALID_ARGUMENT, "unknown op");
}

template <typename T>
int launch_index(const Problem &p, const Geometry &g, char *ws, cudaStream_t s, rg_report *r) {
  return p.index_dtype == RG_INDEX_I32 ? launch_op<T, int32_t>(p, g, ws, s, r)
                                       : launch_op<T, int64_t>(p, g, ws, s, r);
}

template <typename T, typename OffT>
int launch_fused_index(const Problem &p, const Geometry &g, char *ws, cudaStream_t s, rg_report *r,
                       const Xform &xf) {
  constexpr int VEC = 16 / static_cast<int>(sizeof(T));
  return launch_typed<T, OffT, OP_SOFTMAX, VEC, true, true>(p, g, ws, s, r, xf);
}

}  // namespace

bool classified_fuses(const Problem &p, const Geometry &g) {
  return p.op == RG_OP_SOFTMAX && !(p.flags & RG_FLAG_NO_VECTORIZE) && staged_of(p, g);
}

int launch_classified_fused(const Problem &p, const Geometry &g, void *workspace, const float *mask, float scale,
                            cudaStream_t stream, rg_report *report) {
  if (!classified_fuses(p, g)) return fail(RG_ERR_UNSUPPORTED, "fused transform needs staged softmax rows");
  if (p.b == 0) return RG_OK;
  if (report) {
    report->thresholds[0] = kWarpClassMax;
    report->thresholds[1] = item_rows_of(p, g);
    report->status_offset = static_cast<int64_t>(offsetof(ClsState, error));
  }
  const Xform xf{mask, p.d, scale, scale != 1.0f ? 1 : 0};
  char *ws = static_cast<char *>(workspace);
  const bool i32 = p.index_dtype == RG_INDEX_I32;
  if (p.dtype == RG_DTYPE_F32)
    return i32 ? launch_fused_index<float, int32_t>(p, g, ws, stream, report, xf)
               : launch_fused_index<float, int64_t>(p, g, ws, stream, report, xf);
  return i32 ? launch_fused_index<__nv_bfloat16, int32_t>(p, g, ws, stream, report, xf)
             : launch_fused_index<__nv_bfloat16, int64_t>(p, g, ws, stream, report, xf);
}

int classified_workspace(const Problem &p, const Geometry &g, int64_t *bytes) {
  *bytes = p.b == 0 ? 0 : layout_of(p, g).total;
  return RG_OK;
}

int launch_classified(const Problem &p, const Geometry &g, void *workspace, cudaStream_t stream,
                      rg_report *report) {
  if (p.b == 0) return RG_OK;
  if (report) {
    report->thresholds[0] = kWarpClassMax;
    report->thresholds[1] = item_rows_of(p, g);
    report->status_offset = static_cast<int64_t>(offsetof(ClsState, error));  // ClsState sits at offset 0
  }
  char *ws = static_cast<char *>(workspace);
  return p.dtype == RG_DTYPE_F32 ? launch_index<float>(p, g, ws, stream, report)
                                 : launch_index<__nv_bfloat16>(p, g, ws, stream, report);
}

}  // namespace rgb
