// Pipelined classified worker: one producer warp keeps the next stages of
// rows in flight with bulk copies while consumer warps reduce the stages
// already in shared memory.
//
// Work is taken in segment order.  The producer claims 32 consecutive
// segments at a time (one atomic), and packs runs of consecutive short
// segments (at most `item_rows` rows each) into stages: consecutive
// segments are contiguous in memory, so a run is ONE bulk copy
// (cp.async.bulk, TMA's 1-D form) of at most `item_rows` rows.  Segments
// longer than `item_rows` are the split class: the classify kernel lists
// them, and after all runs the producer hands out their chunks, each as
// consecutive stages for one team.  So every row is read from HBM once by the worker; for softmax the
// statistics and the normalisation both read shared memory.
//
// Each stage belongs to one team of 2 consumer warps (the producer rotates
// the four teams over the four stages), so four stages are reduced at once
// and a team's barriers never wait on another team.  Every segment of a run goes to ONE warp of
// the team (shuffles only, no barrier): the warps take contiguous groups of
// the run's segments with about equal rows.  (The reference splits its
// non-split segments at 32 rows between warp and CTA workers, lib/
// Conversion/ToGPU.cpp:923-998; here a warp-per-segment run measured 1.3x
// faster on B200 than a 4-warp merge for the segments of 33 to item_rows
// rows.)  A split chunk's stages all go to one team, whose warps split the
// rows and merge through a named barrier; chunks leave f32 partials, and
// the team finishing a segment's last chunk merges them (see classified.cuh).
//
// Stage protocol: full[s] completes when the producer has written the
// stage's record and the copy's bytes have landed (arrive.expect_tx +
// complete_tx); empty[s] completes when every consumer warp is done with the
// stage.  Every wait is bounded; a wait that gives up records an error in
// the call's state and the protocol carries on (no thread leaves early, so
// no named barrier can be left waiting).
#pragma once

#include "classified.cuh"

namespace rgb {

// One producer warp, 8 consumer warps in 4 teams of 2, 4 stages of 56 KB:
// on B200 the c3 softmax call (bf16, D = 128) took 205 us with this shape,
// against 235 us for 12 consumer warps in 3 teams of 4 over 3 stages of
// 63 KB; 5 or 6 stages, 6 teams, or 4-warp teams over 4 stages measured
// 210-255 us (smaller stages put more segments in the split class).
#ifndef RG_PIPE_TEAM_WARPS
#define RG_PIPE_TEAM_WARPS 2
#endif
#ifndef RG_PIPE_STAGES
#define RG_PIPE_STAGES 4
#endif
#ifndef RG_PIPE_CONSUMER_WARPS
#define RG_PIPE_CONSUMER_WARPS 8
#endif

constexpr int kPipeConsumerWarps = RG_PIPE_CONSUMER_WARPS;
constexpr int kPipeTeamWarps = RG_PIPE_TEAM_WARPS;
static_assert(kPipeConsumerWarps % kPipeTeamWarps == 0, "teams must split the consumer warps evenly");
// A team's row step (kPipeTeamWarps << (5 - g_shift)) must be a power of
// two: lane_rows counts a thread's rows with a shift.
static_assert((kPipeTeamWarps & (kPipeTeamWarps - 1)) == 0, "warps per team must be a power of two");
constexpr int kPipeTeams = kPipeConsumerWarps / kPipeTeamWarps;
constexpr int kPipeThreads = 32 * (kPipeConsumerWarps + 1);
constexpr int kPipeProducer = kPipeConsumerWarps;  // warp index of the producer
constexpr int kPipeClaim = 32;                     // segments claimed per atomic (calls with few segments per CTA)
constexpr int kRunMax = 128;                       // segments per run (and per claim of calls with many)
constexpr int kGroupRows = 32;                     // run segments up to this many rows: one lane group each
#ifndef RG_PIPE_SMEM_KB
#define RG_PIPE_SMEM_KB 227
#endif
constexpr int kSmemBudget = RG_PIPE_SMEM_KB * 1024;
constexpr uint32_t kPieceBytes = 4096;  // bytes per bulk-copy request (a multiple of 16)

// The same stage count for every op.
template <int OP>
struct PipeStages {
  static constexpr int value = RG_PIPE_STAGES;
};

enum : int32_t { STAGE_RUN = 0, STAGE_SPLIT = 1, STAGE_DONE = 2 };

struct StageRecord {
  int32_t kind;
  int32_t count;       // RUN: segments in the run
  int32_t team;        // SPLIT: team that reduces the chunk
  int32_t pad;
  int64_t seg;         // RUN: first segment; SPLIT: the split segment
  int64_t r0, r1;      // rows in the stage
  int64_t index, first, chunks;  // SPLIT: split-list index, first chunk number, chunk count
  int64_t chunk;       // SPLIT: chunk number
  int32_t chunk_first, chunk_last;  // SPLIT: this stage starts / ends its chunk
  int32_t wait;        // SPLIT (softmax): the team waits for the segment and normalises the stage
  int32_t pad2;
  int32_t ends[kRunMax];         // RUN: end row of each segment of the run, relative to r0
};

// Shared memory: the stages, their records, the barriers and, for softmax,
// one merge area per team (a team that normalises a split chunk from its
// stage merges its warps' statistics there, leaving the rows intact; the
// other ops merge inside the stage they hold).
template <int OP, int VEC>
struct PipeLayout {
  static constexpr int kStages = PipeStages<OP>::value;
  static constexpr int kRecordBytes = kStages * static_cast<int>(sizeof(StageRecord));
  static constexpr int kBarrierBytes = 2 * kStages * 8 + 64;
  static constexpr int kTeamScratch = kPipeTeamWarps * 32 * static_cast<int>(sizeof(Acc<OP, VEC>));
  static constexpr int kScratchBytes = OP == OP_SOFTMAX ? kPipeTeams * kTeamScratch : 0;
  static constexpr int kStageBytes =
      ((kSmemBudget - kRecordBytes - kBarrierBytes - kScratchBytes - 256) / kStages) / 1024 * 1024;
  static constexpr int kTotalBytes = kStages * kStageBytes + kRecordBytes + kBarrierBytes + kScratchBytes + 128;
  static_assert(kStageBytes >= kTeamScratch, "stage too small");
};

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}

// Merge the row groups of a team (kPipeTeamWarps warps) through `part`,
// the start of the stage the team holds: warp w's partial for column lane
// cl goes to part[w * 32 + cl].  The first barrier also means every warp of
// the team is done reading the stage's rows (and a previous merge's
// partials) before they are overwritten, so the partials need no shared
// memory of their own and the stages get it.  Every thread merges the
// team's warp partials itself (in warp order, so all of them hold the same
// bits): two barriers, no serial merge.  The caller fences the generic
// writes against the bulk copy that next fills the stage.
template <int OP, int VEC>
__device__ __forceinline__ void team_merge(Acc<OP, VEC> &acc, Acc<OP, VEC> *part, int team, int wit, int q, int cl,
                                           int G) {
  for (int m = 16; m >= G; m >>= 1) acc.shfl_xor_merge(m);
  named_sync(1 + team, 32 * kPipeTeamWarps);
  if (q == 0) part[wit * 32 + cl] = acc;
  named_sync(1 + team, 32 * kPipeTeamWarps);
  acc = part[cl];
#pragma unroll
  for (int w = 1; w < kPipeTeamWarps; ++w) acc.merge(part[w * 32 + cl]);
}

// Fold rows held in shared memory: softmax takes its exact-maximum
// statistics (three shared-memory reads), sum and max the plain fold.
template <typename T, int OP, int VEC, typename Src>
__device__ __forceinline__ void fold_staged(Acc<OP, VEC> &acc, const Src &src, int64_t begin, int64_t end,
                                            int64_t row_lane, int64_t step) {
  if constexpr (OP == OP_SOFTMAX) {
    staged_stats<T, VEC>(acc, src, begin, end, row_lane, step);
  } else {
    fold_rows<T, OP, VEC>(acc, src, begin, end, row_lane, step);
  }
}

#ifndef RG_PIPE_MIN_BLOCKS
#define RG_PIPE_MIN_BLOCKS 1
#endif
// XF: softmax with the input transform fused into the loads (a.xform).
template <typename T, typename OffT, int OP, int VEC, bool XF = false>
__global__ void __launch_bounds__(kPipeThreads, RG_PIPE_MIN_BLOCKS)
pipe_worker_kernel(const T *__restrict__ values, const OffT *__restrict__ offsets, T *__restrict__ out, ClsArgs a) {
  using L = PipeLayout<OP, VEC>;
  constexpr int S = L::kStages;
  constexpr int NC = kPipeConsumerWarps;
  constexpr int W = PartialWidth<OP>::value;
  extern __shared__ __align__(128) char smem[];
  char *const stages = smem;
  StageRecord *const rec = reinterpret_cast<StageRecord *>(smem + S * L::kStageBytes);
  uint64_t *const full = reinterpret_cast<uint64_t *>(smem + S * L::kStageBytes + L::kRecordBytes);
  uint64_t *const empty = full + S;
  int *const last_flag = reinterpret_cast<int *>(empty + S);  // [kPipeTeams]
  char *const scratch = smem + S * L::kStageBytes + L::kRecordBytes + L::kBarrierBytes;  // softmax team merges

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t d = a.d;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NC);
    }
    fence_barrier_init();
    fence_proxy_async_shared();
  }
  __syncthreads();

  const unsigned long long packed = __ldcg(&a.state->split_packed);
  const int64_t n_split = static_cast<int64_t>(packed & kSplitCountMask);
  const int64_t n_chunks = static_cast<int64_t>(packed >> kSplitCountBits);

  if (warp == kPipeProducer) {
    // ------------------------------------------------------------ producer
    int64_t it = 0;
    bool ok = true;
    // Next stage: wait until the consumers released it.
    auto acquire = [&](int &s) {
      s = static_cast<int>(it % S);
      if (it >= S) ok &= mbar_wait(&empty[s], static_cast<uint32_t>(((it / S) - 1) & 1));
      ++it;
    };
    // Publish stage s: record written by this warp, then the copy (if any).
    // The copy is cut into kPieceBytes pieces issued by the warp's lanes in
    // parallel (one TMA request each), all completing on full[s].
    auto publish = [&](int s, const void *src, uint32_t bytes) {
      __syncwarp();
      if (lane == 0) {
        if (bytes > 0) {
          fence_proxy_async_shared();
          mbar_expect_tx(&full[s], bytes);
        } else {
          mbar_arrive(&full[s]);
        }
      }
      __syncwarp();
      char *const dst = stages + static_cast<int64_t>(s) * L::kStageBytes;
      for (uint32_t at = static_cast<uint32_t>(lane) * kPieceBytes; at < bytes; at += 32u * kPieceBytes) {
        const uint32_t n = bytes - at < kPieceBytes ? bytes - at : kPieceBytes;
        bulk_copy_g2s(dst + at, static_cast<const char *>(src) + at, n, &full[s]);
      }
    };
    // Runs of consecutive short segments.  A claim is a.claim segments (32,
    // or kRunMax when the call has many segments per CTA), read as
    // sub-batches of 32, one per lane; a run may continue across the
    // sub-batches of its claim up to kRunMax segments and one stage of
    // rows.  Claims are prefetched: while the stages of claim k are
    // published, the atomic of claim k + 2 and the offsets of claim k + 1
    // are in flight.
    constexpr int kSub = kRunMax / 32;
    auto claim_offsets = [&](int64_t base, int64_t (&c0)[kSub], int64_t (&c1)[kSub]) {
#pragma unroll
      for (int q = 0; q < kSub; ++q) {
        const int64_t sg = base + q * 32 + lane;
        const bool v = q * 32 < a.claim && sg < a.b;
        c0[q] = v ? static_cast<int64_t>(offsets[sg]) : 0;
        c1[q] = v ? static_cast<int64_t>(offsets[sg + 1]) : 0;
      }
    };
    int team = 0;  // team of the next stage (runs) or chunk (split)
    unsigned long long pending = 0;
    const unsigned long long claim = static_cast<unsigned long long>(a.claim);
    if (lane == 0) pending = atomicAdd(&a.state->work, claim);
    int64_t base = static_cast<int64_t>(__shfl_sync(0xffffffffu, pending, 0));
    if (lane == 0 && base < a.b) pending = atomicAdd(&a.state->work, claim);
    int64_t c0[kSub], c1[kSub];
    if (base < a.b) claim_offsets(base, c0, c1);
    while (base < a.b) {
      const int64_t next = static_cast<int64_t>(__shfl_sync(0xffffffffu, pending, 0));
      if (lane == 0 && next < a.b) pending = atomicAdd(&a.state->work, claim);
      int64_t n0[kSub], n1[kSub];
      if (next < a.b) claim_offsets(next, n0, n1);
      // The open run: stage so, rows [run_start, run_end), run_count segments from run_seg.
      bool open = false;
      int so = 0, run_count = 0;
      int64_t run_start = 0, run_end = 0, run_seg = 0;
      auto close_run = [&]() {
        if (lane == 0) {
          StageRecord &r = rec[so];
          r.kind = STAGE_RUN;
          r.team = team;
          r.count = run_count;
          r.seg = run_seg;
          r.r0 = run_start;
          r.r1 = run_end;
        }
        team = team + 1 == kPipeTeams ? 0 : team + 1;
        publish(so, values + run_start * d, static_cast<uint32_t>((run_end - run_start) * a.row_bytes));
        open = false;
      };
#pragma unroll
      for (int q = 0; q < kSub; ++q) {
        const int64_t sb = base + q * 32;
        if (q * 32 >= a.claim || sb >= a.b) break;
        const int64_t o0 = c0[q], o1 = c1[q];
        const bool valid = sb + lane < a.b;
        const bool is_long = valid && (o1 - o0) > a.item_rows;
        const unsigned valid_mask = __ballot_sync(0xffffffffu, valid);
        const unsigned long_mask = __ballot_sync(0xffffffffu, is_long);
        int i = 0;
        while (i < 32 && ((valid_mask >> i) & 1u)) {
          if ((long_mask >> i) & 1u) {
            if (open) close_run();
            ++i;
            continue;
          }
          // Extend the open run (or a new one from segment i) while segments
          // are short, the rows fit one stage and the record has room.
          const int64_t start = open ? run_start : __shfl_sync(0xffffffffu, o0, i);
          const int room = kRunMax - (open ? run_count : 0);
          const bool stop = lane >= i && (!valid || is_long || o1 - start > a.item_rows || lane - i >= room);
          const unsigned stop_mask = __ballot_sync(0xffffffffu, stop) & (~0u << i);
          const int j = stop_mask ? __ffs(stop_mask) - 1 : 32;  // first segment not in the run
          if (j == i) {
            // Segment i does not fit the open run (a new run always takes it).
            if (open) close_run(); else ++i;
            continue;
          }
          if (!open) {
            acquire(so);
            open = true;
            run_start = start;
            run_seg = sb + i;
            run_count = 0;
          }
          if (lane >= i && lane < j) rec[so].ends[run_count + lane - i] = static_cast<int32_t>(o1 - run_start);
          run_end = __shfl_sync(0xffffffffu, o1, j - 1);
          run_count += j - i;
          i = j;
        }
      }
      if (open) close_run();
      base = next;
#pragma unroll
      for (int q = 0; q < kSub; ++q) {
        c0[q] = n0[q];
        c1[q] = n1[q];
      }
    }
    // Split chunks in chunk order, one per atomic, claimed only once the
    // stage for it is held (a claimed chunk always reaches its team: the
    // waits of normalized_in_worker rely on it).  Each chunk is published as
    // consecutive stages for one team.  Lane l caches split entry wbase + l
    // (first chunk, segment, rows), so walking consecutive chunks needs no
    // search.
    int64_t wbase = -1, w_first = INT64_MAX, w_seg = 0, w_begin = 0, w_end = 0, w_rows = 1, w_chunks = 0;
    auto load_window = [&](int64_t start) {
      wbase = start;
      const int64_t idx = start + lane;
      const bool v = idx < n_split;
      w_first = v ? __ldcg(a.split_base + idx) : INT64_MAX;
      w_seg = v ? __ldcg(a.split_seg + idx) : 0;
      w_begin = v ? static_cast<int64_t>(offsets[w_seg]) : 0;
      w_end = v ? static_cast<int64_t>(offsets[w_seg + 1]) : 0;
      w_rows = v ? chunk_rows_of(w_end - w_begin, a.item_rows) : 1;
      w_chunks = v ? (w_end - w_begin + w_rows - 1) / w_rows : 0;
    };
    // Lane whose entry holds chunk c, or -1.
    auto find = [&](int64_t c) -> int {
      const unsigned m = __ballot_sync(0xffffffffu, w_first <= c && c < w_first + w_chunks);
      return m ? __ffs(m) - 1 : -1;
    };
    int s;
    for (;;) {
      acquire(s);
      if (lane == 0) pending = atomicAdd(&a.state->split_work, 1ull);
      const int64_t c = static_cast<int64_t>(__shfl_sync(0xffffffffu, pending, 0));
      if (c >= n_chunks) break;  // stage s stays acquired for the DONE record
      int k = find(c);
      if (k < 0) {
        // 32-ary search of the split list for the last i with base[i] <= c.
        int64_t lo = 0, hi = n_split - 1;
        while (lo < hi) {
          const int64_t step = (hi - lo + 31) / 32;
          const int64_t probe = lo + (lane + 1) * step;
          const bool le = probe <= hi && __ldcg(a.split_base + probe) <= c;
          const unsigned m = __ballot_sync(0xffffffffu, le);
          const int n = m ? 32 - __clz(m) : 0;  // probes lo + 1..n*step are <= c
          const int64_t cut = lo + static_cast<int64_t>(n + 1) * step - 1;
          hi = n < 32 && cut < hi ? cut : hi;
          lo = lo + static_cast<int64_t>(n) * step;
        }
        load_window(lo);
        k = find(c);
      }
      const int64_t seg = __shfl_sync(0xffffffffu, w_seg, k);
      const int64_t first = __shfl_sync(0xffffffffu, w_first, k);
      const int64_t begin = __shfl_sync(0xffffffffu, w_begin, k);
      const int64_t end = __shfl_sync(0xffffffffu, w_end, k);
      const int64_t rows_per_chunk = __shfl_sync(0xffffffffu, w_rows, k);
      const int64_t chunks = __shfl_sync(0xffffffffu, w_chunks, k);
      const int64_t r0 = begin + (c - first) * rows_per_chunk;
      const int64_t r1 = r0 + rows_per_chunk < end ? r0 + rows_per_chunk : end;
      const bool wait = OP == OP_SOFTMAX && normalized_in_worker(end - begin, a.item_rows, a.wait_rows);
      for (int64_t a0 = r0; a0 < r1; a0 += a.item_rows) {
        const int64_t a1 = a0 + a.item_rows < r1 ? a0 + a.item_rows : r1;
        if (a0 != r0) acquire(s);  // later stages of a chunk longer than one stage
        if (lane == 0) {
          StageRecord &r = rec[s];
          r.kind = STAGE_SPLIT;
          r.team = team;
          r.seg = seg;
          r.r0 = a0;
          r.r1 = a1;
          r.index = wbase + k;
          r.first = first;
          r.chunks = chunks;
          r.chunk = c;
          r.chunk_first = a0 == r0;
          r.chunk_last = a1 == r1;
          r.wait = wait;
        }
        publish(s, values + a0 * d, static_cast<uint32_t>((a1 - a0) * a.row_bytes));
      }
      team = team + 1 == kPipeTeams ? 0 : team + 1;
    }
    if (lane == 0) rec[s].kind = STAGE_DONE;
    publish(s, nullptr, 0);
    if (!ok && lane == 0) atomicExch(&a.state->error, 1ull);
    return;
  }

  // -------------------------------------------------------------- consumers
  const int G = 1 << a.g_shift;
  const int q = lane >> a.g_shift, cl = lane & (G - 1);
  const bool active = cl < a.vec_cols;
  const int64_t col = static_cast<int64_t>(cl) * VEC;
  const int col_bytes = cl * VEC * static_cast<int>(sizeof(T));
  const int team = warp / kPipeTeamWarps, wit = warp % kPipeTeamWarps;
  const int64_t warp_step = 32 >> a.g_shift;
  const int64_t team_step = static_cast<int64_t>(kPipeTeamWarps) << (5 - a.g_shift);
  const int64_t team_lane = static_cast<int64_t>(wit) * (32 >> a.g_shift) + q;
  bool ok = true;
  Acc<OP, VEC> split_acc;  // this team's chunk in progress (stages of one chunk arrive in order)
  split_acc.init();
  for (int64_t it = 0;; ++it) {
    const int s = static_cast<int>(it % S);
    ok &= mbar_wait(&full[s], static_cast<uint32_t>((it / S) & 1));
    const StageRecord &r = rec[s];
    const int kind = r.kind;
    if (kind == STAGE_DONE) break;
    const SharedRows<T, VEC> rows{stages + static_cast<int64_t>(s) * L::kStageBytes, r.r0, a.row_bytes, col_bytes};
    if (kind == STAGE_RUN && r.team == team) {
      // A whole run belongs to one team, and each of its segments to one
      // warp of the team: no team barrier.  Segment k goes to the warp whose
      // quarter of the run's rows holds the segment's middle row, so the
      // warps get contiguous groups of segments with about equal rows.
      const int64_t r0 = r.r0, span = r.r1 - r.r0;
      const int count = r.count;
      // Segments of at most kGroupRows rows go to single lane groups (group
      // g of the team takes run segments g, g + groups, ...): a group holds
      // whole rows, so it needs no merge with other groups, and the warp
      // works on 32 / G segments at once.
      // (Not with the fused transform: its register budget is spent.)
      constexpr int64_t kGroupMax = XF ? -1 : kGroupRows;
      const int groups = kPipeTeamWarps << (5 - a.g_shift);
      for (int k = XF ? count : static_cast<int>(team_lane); k < count; k += groups) {
        const int64_t begin = k ? r0 + r.ends[k - 1] : r0, end = r0 + r.ends[k];
        if (end - begin > kGroupMax || !active) continue;
        Acc<OP, VEC> acc;
        acc.init();
        if constexpr (OP == OP_SOFTMAX) {
          float base[VEC], mine[VEC], ref[VEC], inv[VEC], f[VEC];
          staged_stats_keep<T, VEC, XF>(acc, rows, begin, end, 0, 1, base, a.xform, col);
#pragma unroll
          for (int v = 0; v < VEC; ++v) mine[v] = acc.st[v].r;
          stats_of<VEC>(acc, ref, inv);
          kept_factor<VEC>(base, mine, ref, inv, f);
          normalize_kept<T, VEC>(rows, out, d, col, begin, end, 0, 1, f);
        } else {
          fold_staged<T, OP, VEC>(acc, rows, begin, end, 0, 1);
          float y[VEC];
          acc.result(y);
          VecIO<T, VEC>::store(out + (r.seg + k) * d + col, y);
        }
      }
      // Longer segments: one warp each (relative rows fit 32 bits: a run is
      // at most one stage).
      int begin_rel = 0;
      const int span32 = static_cast<int>(span);
      for (int k = 0; k < count; ++k) {
        const int end_rel = r.ends[k];
        const int64_t begin = r0 + begin_rel, end = r0 + end_rel;
        const int64_t seg = r.seg + k;
        const bool big = end_rel - begin_rel > kGroupMax;
        const int owner = big && span32 > 0 ? ((begin_rel + end_rel) * kPipeTeamWarps) / (2 * span32) : 0;
        if (big && (owner < kPipeTeamWarps ? owner : kPipeTeamWarps - 1) == wit) {
          Acc<OP, VEC> acc;
          acc.init();
          if constexpr (OP == OP_SOFTMAX) {
            // The mass pass keeps its terms in the stage; the normalisation
            // scales them by e^(base - M) / total.
            float base[VEC], mine[VEC];
            if (active) staged_stats_keep<T, VEC, XF>(acc, rows, begin, end, q, warp_step, base, a.xform, col);
#pragma unroll
            for (int v = 0; v < VEC; ++v) mine[v] = acc.st[v].r;
            warp_merge<OP, VEC>(acc, G);
            if (active) {
              float ref[VEC], inv[VEC], f[VEC];
              stats_of<VEC>(acc, ref, inv);
              kept_factor<VEC>(base, mine, ref, inv, f);
              normalize_kept<T, VEC>(rows, out, d, col, begin, end, q, warp_step, f);
            }
          } else {
            if (active) fold_staged<T, OP, VEC>(acc, rows, begin, end, q, warp_step);
            warp_merge<OP, VEC>(acc, G);
            if (q == 0 && active) {
              float y[VEC];
              acc.result(y);
              VecIO<T, VEC>::store(out + seg * d + col, y);
            }
          }
        }
        begin_rel = end_rel;
      }
    } else if (kind == STAGE_SPLIT && r.team == team) {
      // ---- split chunk: one team folds the chunk's stages, publishes an
      // f32 partial, and the team finishing the segment's last chunk merges
      const int64_t c = r.chunk, index = r.index, first = r.first, chunks = r.chunks, seg = r.seg;
      if (r.chunk_first) split_acc.init();
      float base[VEC], mine[VEC];  // softmax: the thread's kept terms are e^(x - base); mine = its maximum
      if (active) {
        if constexpr (OP == OP_SOFTMAX) {
          Acc<OP, VEC> stage_acc;
          staged_stats_keep<T, VEC, XF>(stage_acc, rows, r.r0, r.r1, team_lane, team_step, base, a.xform, col);
#pragma unroll
          for (int v = 0; v < VEC; ++v) mine[v] = stage_acc.st[v].r;
          split_acc.merge(stage_acc);
        } else {
          fold_rows<T, OP, VEC>(split_acc, rows, r.r0, r.r1, team_lane, team_step);
        }
      }
      if (!r.chunk_last) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        continue;
      }
      // Softmax merges in the team's own area, so a waiting chunk's rows stay
      // in its stage; the other ops merge inside the stage they hold.
      Acc<OP, VEC> *const part = reinterpret_cast<Acc<OP, VEC> *>(
          OP == OP_SOFTMAX ? scratch + team * L::kTeamScratch : stages + static_cast<int64_t>(s) * L::kStageBytes);
      Acc<OP, VEC> acc = split_acc;
      team_merge<OP, VEC>(acc, part, team, wit, q, cl, G);
      if (wit == 0 && q == 0 && active) store_partial<OP, VEC>(acc, a.partials + (c * W) * d + col, d);
      __threadfence();  // release: the partial before the count
      named_sync(1 + team, 32 * kPipeTeamWarps);
      bool wait = OP == OP_SOFTMAX && r.wait;
      if (wit == 0 && lane == 0) {
        const bool last = atomicAdd(a.done + index, 1u) == static_cast<unsigned>(chunks - 1);
        int flag = last ? 1 : 0;
        if (wait && !last) {  // bounded wait until every chunk of the segment has published
          bool complete = ld_acquire_gpu(a.done + index) >= static_cast<unsigned>(chunks);
          for (int i = 0; !complete && i < a.wait_polls; ++i) {
            __nanosleep(256);
            complete = ld_acquire_gpu(a.done + index) >= static_cast<unsigned>(chunks);
          }
          if (!complete) {  // gave up: split_normalize_kernel normalises this chunk
            a.late[c] = 1u;
            atomicAdd(&a.state->late_chunks, 1ull);
            flag |= 2;
          }
        }
        last_flag[team] = flag;
      }
      named_sync(1 + team, 32 * kPipeTeamWarps);
      const int flag = last_flag[team];
      if (flag & 2) wait = false;
      if ((flag & 1) || wait) {
        __threadfence();  // acquire: every chunk's partial is visible
        Acc<OP, VEC> m;
        m.init();
        if (active) {  // one partial at a time: a merge runs once per segment, registers matter more
          for (int64_t j = first + team_lane; j < first + chunks; j += team_step) {
            Acc<OP, VEC> pj;
            load_partial<OP, VEC>(pj, a.partials + (j * W) * d + col, d);
            m.merge(pj);
          }
        }
        team_merge<OP, VEC>(m, part, team, wit, q, cl, G);
        if constexpr (OP == OP_SOFTMAX) {
          // The last chunk also leaves the statistics for the normalise kernel
          // (every chunk of a long segment, a chunk whose wait gave up).
          if ((flag & 1) && wit == 0 && q == 0 && active)
            store_partial<OP, VEC>(m, a.seg_stats + index * 2 * d + col, d);
          if (wait && active) {  // every team of the segment merged the same partials in the same order
            float ref[VEC], inv[VEC], f[VEC];
            stats_of<VEC>(m, ref, inv);
            kept_factor<VEC>(base, mine, ref, inv, f);
            normalize_kept<T, VEC>(rows, out, d, col, r.r0, r.r1, team_lane, team_step, f);
          }
        } else if (wit == 0 && q == 0 && active) {
          float y[VEC];
          m.result(y);
          VecIO<T, VEC>::store(out + seg * d + col, y);
        }
      }
      if constexpr (OP != OP_SOFTMAX) fence_proxy_async_shared();  // partials written into the stage
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (!ok && lane == 0) atomicExch(&a.state->error, 1ull);
}

}  // namespace rgb
