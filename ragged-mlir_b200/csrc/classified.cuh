// Classified schedule: segments are binned by length on the device and
// reduced by workers sized to their class (the reference's "classified"
// strategy, lib/Conversion/ToGPU.cpp:748-1062, docs/classified-abi.md).
//
//   classify   one thread per segment: length <= 32 rows -> WARP class,
//              <= T rows -> CTA class, longer -> SPLIT class, cut into
//              chunks of T rows (more for segments over 1024 T rows, so that
//              no segment has more than 1024 chunks).  The reference fixes T = 4096
//              (lib/Transforms/Passes.cpp:17-18); here T is 4096 or the rows
//              of one shared-memory stage (pipelined worker) or of 64 KiB
//              (unstaged worker), whichever is smaller, so that no CTA owns
//              more than a small slice of an HBM-bound call on 148 SMs.
//              Warp ballots give each thread its rank in its class; one
//              atomic per warp and class reserves the list positions.  One
//              64-bit atomic per warp reserves split-list positions and
//              chunk numbers together, so the split list is ordered by
//              first chunk.
//   worker     one persistent launch, one resident wave.  CTAs take work
//              items from an atomic counter: CTA-class segments, then groups
//              of warp-class segments (one warp per segment, shuffles only),
//              then split chunks.  A split chunk leaves f32 partials; the CTA
//              that completes a segment's last chunk (a counter per segment,
//              release/acquire fences) merges them in a fixed tree and writes
//              the output -- or, for softmax, the segment's statistics.
//   normalize  softmax only: the rows of split segments, normalised with
//              the merged statistics, in reverse chunk order so the chunks
//              the worker read last are re-read from L2.
//
// Rows that bulk copies can stage (one column tile, rows a multiple of 16
// bytes) take the pipelined worker of pipeline.cuh instead of the worker
// below; it walks short segments in order and uses only the split list.
//
// The reference launches one kernel chain per class on three streams; here
// all classes share one persistent launch, so no class waits for a stream
// or leaves SMs idle while another class still has work.  Results do not
// depend on which CTA takes which item: each item's arithmetic order is
// fixed, and split partials merge in a tree that depends only on the
// segment's chunk count.
#pragma once

#include "cta_reduce.cuh"

namespace rgb {

constexpr int kClsThreads = 256;
constexpr int kClsWarps = kClsThreads / 32;
constexpr int64_t kWarpClassMax = 32;    // Passes.cpp:17 kWarpMaxLength
constexpr int64_t kCtaClassMax = 4096;   // Passes.cpp:18 kCtaMaxLength
constexpr int kItemBytes = 64 * 1024;   // bytes of one CTA item per column tile (unstaged worker)
constexpr int kWarpSegsPerWarp = 4;      // warp-class segments per warp per work item
constexpr int kWarpSegsPerItem = kClsWarps * kWarpSegsPerWarp;
constexpr int kSplitCountBits = 28;      // split list position bits of the packed counter
constexpr unsigned long long kSplitCountMask = (1ull << kSplitCountBits) - 1;

// Device counters of one call (zeroed before classify).
struct ClsState {
  unsigned long long warp_count;   // warp-class segments
  unsigned long long cta_count;    // CTA-class segments
  unsigned long long split_packed; // (chunks << 28) | split segments
  unsigned long long work;         // next work item of the worker
  unsigned long long error;        // nonzero: a bounded wait gave up
  unsigned long long split_work;   // next split chunk of the pipelined worker
  unsigned long long late_chunks;  // softmax: chunks left to split_normalize_kernel
};

// Chunk length of a split segment of `len` rows: the item length, or longer
// for very long segments so that no segment has more than kMaxChunks
// chunks (its last chunk merges that many partials).
constexpr int64_t kMaxChunks = 1024;
__host__ __device__ __forceinline__ int64_t chunk_rows_of(int64_t len, int64_t item_rows) {
  const int64_t spread = (len + kMaxChunks - 1) / kMaxChunks;
  return spread > item_rows ? spread : item_rows;
}

// Softmax split segments the pipelined worker normalises itself: every
// chunk is one stage (chunk rows == item rows) and there are at most
// min(kWaitChunks, worker CTAs / 2) of them.  The team holding a chunk
// publishes its statistics, waits (bounded) until every chunk of the
// segment has published, merges them and normalises the chunk's rows
// straight from its stage, so these rows are read from HBM once.  Longer
// segments leave their statistics to split_normalize_kernel, which re-reads
// their rows.
//
// Why the wait ends: the worker claims a chunk only after it holds a stage
// for it, and the team owning that stage reaches it (a team holds one stage
// at a time), so every claimed chunk publishes its statistics.  Chunks are
// claimed in list order, so at any moment only one segment can be partly
// claimed; its waiting teams hold the stages of fewer than half the
// worker's CTAs, so while those CTAs are resident some producer always
// reaches the segment's next chunk.  Nothing relies on that residency for
// correctness: a wait gives up after ClsArgs::wait_polls polls (about a
// millisecond by default, kChunkWaitPolls; a normal wait lasts a few
// microseconds; the environment variable RAGGED_B200_CHUNK_WAIT_POLLS
// overrides the count, so tests can make every wait give up), marks its
// chunk late and leaves its rows to split_normalize_kernel, which
// normalises late chunks with the statistics the segment's last chunk
// writes.
constexpr int64_t kWaitChunks = 64;
constexpr int kChunkWaitPolls = 1 << 12;
__host__ __device__ __forceinline__ bool normalized_in_worker(int64_t len, int64_t item_rows, int64_t wait_rows) {
  return len <= wait_rows && chunk_rows_of(len, item_rows) == item_rows;
}

// Floats per feature in a split partial.
template <int OP>
struct PartialWidth {
  static constexpr int value = OP == OP_MAX ? 1 : 2;
};

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Warp-aggregated append of this lane's id to a class list when `take`:
// one atomic per warp; the position within the warp follows lane order.
__device__ __forceinline__ int64_t warp_append(bool take, unsigned long long *counter) {
  const unsigned mask = __ballot_sync(0xffffffffu, take);
  if (!mask) return -1;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(mask) - 1;
  unsigned long long base = 0;
  if (lane == leader) base = atomicAdd(counter, static_cast<unsigned long long>(__popc(mask)));
  base = __shfl_sync(0xffffffffu, base, leader);
  return take ? static_cast<int64_t>(base) + __popc(mask & lanemask_lt()) : -1;
}

// Segment ids: the warp class fills ids[0, warp_count) upward, the CTA class
// fills ids[b - cta_count, b) downward, so one [B] array holds both.
// wait_rows: softmax split segments up to this length are normalised by the
// worker (normalized_in_worker); the chunks of longer ones are counted in
// state->late_chunks for split_normalize_kernel.
template <typename OffT>
__global__ void __launch_bounds__(256)
classify_kernel(const OffT *__restrict__ offsets, int64_t b, int64_t item_rows, int softmax, int split_only,
                int64_t wait_rows, ClsState *__restrict__ state, int64_t *__restrict__ ids,
                int64_t *__restrict__ split_seg, int64_t *__restrict__ split_base) {
  const int lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x; base < b; base += stride) {
    const int64_t s = base + threadIdx.x;
    int cls = -1;
    int64_t chunks = 0;
    bool late = false;
    if (s < b) {
      const int64_t len = static_cast<int64_t>(offsets[s + 1]) - static_cast<int64_t>(offsets[s]);
      if (len <= kWarpClassMax) {
        cls = (softmax && len == 0) ? -1 : 0;  // an empty softmax segment has no rows to write
      } else if (len <= item_rows) {
        cls = 1;
      } else {
        cls = 2;
        const int64_t cr = chunk_rows_of(len, item_rows);
        chunks = (len + cr - 1) / cr;
        late = softmax && !normalized_in_worker(len, item_rows, wait_rows);
      }
    }
    if (__any_sync(0xffffffffu, late)) {  // chunks left to the normalise kernel: one atomic per warp
      int64_t mine = late ? chunks : 0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
      if (lane == 0) atomicAdd(&state->late_chunks, static_cast<unsigned long long>(mine));
    }
    if (!split_only) {  // the pipelined worker walks short segments in order and needs no lists
      const int64_t wpos = warp_append(cls == 0, &state->warp_count);
      if (cls == 0) ids[wpos] = s;
      const int64_t cpos = warp_append(cls == 1, &state->cta_count);
      if (cls == 1) ids[b - 1 - cpos] = s;
    }
    // Split class: inclusive scan of chunk counts over the warp, then one
    // packed atomic for (positions, chunk numbers).
    const unsigned smask = __ballot_sync(0xffffffffu, cls == 2);
    if (smask) {
      int64_t scan = chunks;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t up = __shfl_up_sync(0xffffffffu, scan, o);
        if (lane >= o) scan += up;
      }
      const int64_t total = __shfl_sync(0xffffffffu, scan, 31);
      unsigned long long old = 0;
      if (lane == 0)
        old = atomicAdd(&state->split_packed,
                        (static_cast<unsigned long long>(total) << kSplitCountBits) | __popc(smask));
      old = __shfl_sync(0xffffffffu, old, 0);
      if (cls == 2) {
        const int64_t pos = static_cast<int64_t>(old & kSplitCountMask) + __popc(smask & lanemask_lt());
        split_seg[pos] = s;
        split_base[pos] = static_cast<int64_t>(old >> kSplitCountBits) + scan - chunks;
      }
    }
  }
}

// Split partial storage: partial j of column col at p + j * W * d + k * d + col.
template <int OP, int VEC>
__device__ __forceinline__ void store_partial(const Acc<OP, VEC> &acc, float *p, int64_t d) {
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
    if constexpr (OP == OP_SUM) {
      p[v] = acc.s[v];
      p[d + v] = acc.c[v];
    } else if constexpr (OP == OP_MAX) {
      p[v] = acc.m[v];
    } else {
      p[v] = acc.st[v].r;
      p[d + v] = kahan_value(acc.st[v].s, acc.st[v].c);
    }
  }
}

// Partials written by other CTAs: read through L2 (never a stale L1 line).
template <int OP, int VEC>
__device__ __forceinline__ void load_partial(Acc<OP, VEC> &acc, const float *p, int64_t d) {
#pragma unroll
  for (int v = 0; v < VEC; ++v) {
    if constexpr (OP == OP_SUM) {
      acc.s[v] = __ldcg(p + v);
      acc.c[v] = __ldcg(p + d + v);
    } else if constexpr (OP == OP_MAX) {
      acc.m[v] = __ldcg(p + v);
    } else {
      acc.st[v].r = __ldcg(p + v);
      acc.st[v].s = __ldcg(p + d + v);
      acc.st[v].c = 0.0f;
    }
  }
}

// Chunk c of the split list: its split index (binary search over the
// ascending first-chunk numbers), segment, rows, first chunk and count.
template <typename OffT>
__device__ __forceinline__ void locate_chunk(int64_t c, int64_t item_rows, const int64_t *split_base,
                                             const int64_t *split_seg, int64_t n_split, const OffT *offsets,
                                             int64_t &index, int64_t &seg, int64_t &r0, int64_t &r1,
                                             int64_t &first, int64_t &count) {
  int64_t lo = 0, hi = n_split - 1;  // last i with split_base[i] <= c
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) / 2;
    if (__ldcg(split_base + mid) <= c) lo = mid; else hi = mid - 1;
  }
  index = lo;
  seg = __ldcg(split_seg + lo);
  first = __ldcg(split_base + lo);
  const int64_t begin = static_cast<int64_t>(offsets[seg]), end = static_cast<int64_t>(offsets[seg + 1]);
  const int64_t cr = chunk_rows_of(end - begin, item_rows);
  r0 = begin + (c - first) * cr;
  r1 = r0 + cr < end ? r0 + cr : end;
  count = (end - begin + cr - 1) / cr;
}

struct ClsArgs {
  int64_t b, d;
  int64_t item_rows;   // CTA-class bound and split chunk rows
  int g_shift, vec_cols, col_tiles;
  int row_bytes;       // D * element size (staged kernels: the whole column tile)
  ClsState *state;
  const int64_t *ids, *split_seg, *split_base;
  float *partials;     // [chunks][W][D]
  float *seg_stats;    // softmax: [splits][2][D] (reference, total)
  unsigned *done;      // [splits][col_tiles] chunks finished
  int64_t wait_rows;   // softmax split segments up to this length are normalised by the worker (0: none)
  unsigned *late;      // softmax: [chunks] nonzero = chunk whose wait gave up (normalised by split_normalize)
  int wait_polls;      // polls before a wait gives up
  int claim;           // pipelined worker: segments per producer claim (kPipeClaim or kRunMax)
  Xform xform;         // softmax input transform fused into the loads (pipelined worker, normalise kernel)
};

// Worker of the classified schedule for rows that cannot be staged by bulk
// copies (several column tiles, or rows not a multiple of 16 bytes): rows
// are read from global memory, kFoldUnroll loads in flight per thread; the
// softmax normalisation re-reads the rows (L1/L2).
template <typename T, typename OffT, int OP, int VEC>
__global__ void __launch_bounds__(kClsThreads, 2)
cls_worker_kernel(const T *__restrict__ values, const OffT *__restrict__ offsets, T *__restrict__ out, ClsArgs a) {
  constexpr int NW = kClsWarps;
  constexpr int W = PartialWidth<OP>::value;
  __shared__ Acc<OP, VEC> part[NW][32];
  __shared__ int64_t item_slot[2];
  __shared__ int last;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = 1 << a.g_shift;
  const int q = lane >> a.g_shift, cl = lane & (G - 1);
  const int64_t cta_step = static_cast<int64_t>(NW) << (5 - a.g_shift);
  const int64_t cta_lane = static_cast<int64_t>(warp) * (32 >> a.g_shift) + q;
  const int64_t warp_step = 32 >> a.g_shift;
  const int64_t d = a.d;

  const unsigned long long packed = __ldcg(&a.state->split_packed);
  const int64_t n_split = static_cast<int64_t>(packed & kSplitCountMask);
  const int64_t n_chunks = static_cast<int64_t>(packed >> kSplitCountBits);
  const int64_t n_cta = static_cast<int64_t>(__ldcg(&a.state->cta_count));
  const int64_t n_warp = static_cast<int64_t>(__ldcg(&a.state->warp_count));
  const int64_t n_groups = (n_warp + kWarpSegsPerItem - 1) / kWarpSegsPerItem;
  const int64_t total = (n_cta + n_groups + n_chunks) * a.col_tiles;

  for (int parity = 0;; parity ^= 1) {
    // Double-buffered item slot: one barrier per item.
    if (threadIdx.x == 0) item_slot[parity] = static_cast<int64_t>(atomicAdd(&a.state->work, 1ull));
    __syncthreads();
    const int64_t w = item_slot[parity];
    if (w >= total) break;
    const int tile = static_cast<int>(w % a.col_tiles);
    const int64_t item = w / a.col_tiles;
    const int cv = tile * 32 + cl;
    const bool active = cv < a.vec_cols;
    const int64_t col = static_cast<int64_t>(cv) * VEC;
    const GlobalRows<T, VEC> rows{values, d, col};

    if (item < n_cta || item >= n_cta + n_groups) {
      // ---- a CTA-class segment or a split chunk: the whole CTA
      const bool split = item >= n_cta;
      int64_t seg, r0, r1, index = 0, first = 0, count = 0;
      const int64_t c = item - n_cta - n_groups;
      if (split) {
        locate_chunk(c, a.item_rows, a.split_base, a.split_seg, n_split, offsets, index, seg, r0, r1, first, count);
      } else {
        seg = __ldcg(a.ids + (a.b - 1 - item));
        r0 = static_cast<int64_t>(offsets[seg]);
        r1 = static_cast<int64_t>(offsets[seg + 1]);
      }
      Acc<OP, VEC> acc;
      acc.init();
      if (active) fold_rows<T, OP, VEC>(acc, rows, r0, r1, cta_lane, cta_step);
      cta_merge<OP, VEC, NW>(acc, part, warp, q, cl, G);
      if (!split) {
        if constexpr (OP == OP_SOFTMAX) {
          if (active) {
            float ref[VEC], inv[VEC];
            stats_of<VEC>(part[0][cl], ref, inv);
            normalize_rows<T, VEC>(rows, out, d, col, r0, r1, cta_lane, cta_step, ref, inv);
          }
        } else if (threadIdx.x < G && active) {
          float y[VEC];
          part[0][threadIdx.x].result(y);
          VecIO<T, VEC>::store(out + seg * d + col, y);
        }
        continue;
      }
      // Split chunk: publish the partial; the CTA finishing the segment's
      // last chunk merges all of them.
      if (threadIdx.x < G && active) store_partial<OP, VEC>(part[0][threadIdx.x], a.partials + (c * W) * d + col, d);
      __threadfence();  // release: this CTA's partial before its count
      __syncthreads();
      unsigned *const done = a.done + index * a.col_tiles + tile;
      if (threadIdx.x == 0) last = atomicAdd(done, 1u) == static_cast<unsigned>(count - 1);
      __syncthreads();
      if (!last) continue;
      __threadfence();  // acquire: every chunk's partial is visible
      Acc<OP, VEC> m;
      m.init();
      if (active) {
        int64_t j = first + cta_lane;
        for (; j + 3 * cta_step < first + count; j += 4 * cta_step) {
          Acc<OP, VEC> p0, p1, p2, p3;  // four loads in flight
          load_partial<OP, VEC>(p0, a.partials + (j * W) * d + col, d);
          load_partial<OP, VEC>(p1, a.partials + ((j + cta_step) * W) * d + col, d);
          load_partial<OP, VEC>(p2, a.partials + ((j + 2 * cta_step) * W) * d + col, d);
          load_partial<OP, VEC>(p3, a.partials + ((j + 3 * cta_step) * W) * d + col, d);
          p0.merge(p1);
          p2.merge(p3);
          p0.merge(p2);
          m.merge(p0);
        }
        for (; j < first + count; j += cta_step) {
          Acc<OP, VEC> pj;
          load_partial<OP, VEC>(pj, a.partials + (j * W) * d + col, d);
          m.merge(pj);
        }
      }
      cta_merge<OP, VEC, NW>(m, part, warp, q, cl, G);
      if (threadIdx.x < G && active) {
        const Acc<OP, VEC> &fin = part[0][threadIdx.x];
        if constexpr (OP == OP_SOFTMAX) {
          store_partial<OP, VEC>(fin, a.seg_stats + index * 2 * d + col, d);
        } else {
          float y[VEC];
          fin.result(y);
          VecIO<T, VEC>::store(out + seg * d + col, y);
        }
      }
    } else {
      // ---- warp-class segments: one warp each
      const int64_t first = (item - n_cta) * kWarpSegsPerItem + warp * kWarpSegsPerWarp;
      for (int k = 0; k < kWarpSegsPerWarp; ++k) {
        if (first + k >= n_warp) break;  // uniform across the warp
        const int64_t seg = __ldcg(a.ids + first + k);
        const int64_t begin = static_cast<int64_t>(offsets[seg]), end = static_cast<int64_t>(offsets[seg + 1]);
        Acc<OP, VEC> acc;
        acc.init();
        if (active) fold_rows<T, OP, VEC>(acc, rows, begin, end, q, warp_step);
        warp_merge<OP, VEC>(acc, G);
        if constexpr (OP == OP_SOFTMAX) {
          if (active) {
            float ref[VEC], inv[VEC];
            stats_of<VEC>(acc, ref, inv);
            normalize_rows<T, VEC>(rows, out, d, col, begin, end, q, warp_step, ref, inv);
          }
        } else if (q == 0 && active) {
          float y[VEC];
          acc.result(y);
          VecIO<T, VEC>::store(out + seg * d + col, y);
        }
      }
    }
  }
}

// Softmax: normalise the rows of split segments with their merged
// statistics.  One warp per item (a chunk and column tile), items spread
// statically over the warps in reverse chunk order, so the chunks the
// worker read last are re-read first, from L2.  A warp finds its chunk's
// split entry with a 32-ary search of split_base (three steps for 32K
// split segments) and keeps 8 rows per lane group in flight.  XF: the
// softmax input transform (a.xform) is applied as rows are loaded.
template <typename T, typename OffT, int VEC, bool XF = false>
__global__ void __launch_bounds__(kClsThreads, 2)
split_normalize_kernel(const T *__restrict__ values, const OffT *__restrict__ offsets, T *__restrict__ out,
                       ClsArgs a) {
  constexpr int U = 8;
  using Raw = typename VecIO<T, VEC>::Raw;
  const int lane = threadIdx.x & 31;
  const int G = 1 << a.g_shift;
  const int q = lane >> a.g_shift, cl = lane & (G - 1);
  const int upw = 32 >> a.g_shift;
  if (__ldcg(&a.state->late_chunks) == 0) return;  // the worker normalised every split segment
  const unsigned long long packed = __ldcg(&a.state->split_packed);
  const int64_t n_split = static_cast<int64_t>(packed & kSplitCountMask);
  const int64_t n_chunks = static_cast<int64_t>(packed >> kSplitCountBits);
  const int64_t items = n_chunks * a.col_tiles;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); w < items;
       w += warps) {
    const int tile = static_cast<int>(w % a.col_tiles);
    const int64_t c = n_chunks - 1 - w / a.col_tiles;
    // Last split entry i with split_base[i] <= c (32-ary search).
    int64_t lo = 0, hi = n_split - 1;
    while (lo < hi) {
      const int64_t step = (hi - lo + 31) / 32;
      const int64_t probe = lo + (lane + 1) * step;
      const bool le = probe <= hi && __ldcg(a.split_base + probe) <= c;
      const unsigned m = __ballot_sync(0xffffffffu, le);
      const int k = m ? 32 - __clz(m) : 0;  // probes lo + 1..k * step are <= c
      const int64_t cut = lo + static_cast<int64_t>(k + 1) * step - 1;
      hi = k < 32 && cut < hi ? cut : hi;
      lo = lo + static_cast<int64_t>(k) * step;
    }
    const int64_t index = lo;
    const int64_t seg = __ldcg(a.split_seg + index), first = __ldcg(a.split_base + index);
    const int64_t begin = static_cast<int64_t>(offsets[seg]), end = static_cast<int64_t>(offsets[seg + 1]);
    if (normalized_in_worker(end - begin, a.item_rows, a.wait_rows) && __ldcg(a.late + c) == 0)
      continue;  // normalised by the worker (uniform per warp)
    const int64_t cr = chunk_rows_of(end - begin, a.item_rows);
    const int64_t r0 = begin + (c - first) * cr;
    const int64_t r1 = r0 + cr < end ? r0 + cr : end;
    const int cv = tile * 32 + cl;
    if (cv >= a.vec_cols) continue;
    const int64_t col = static_cast<int64_t>(cv) * VEC;
    float ref[VEC], inv[VEC];
    const float *st = a.seg_stats + index * 2 * a.d + col;
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      ref[v] = __ldcg(st + v);
      inv[v] = stats_inverse(__ldcg(st + a.d + v));
    }
    const int64_t step = upw;
    int64_t r = r0 + q;
    for (; r + (U - 1) * step < r1; r += U * step) {
      Raw raw[U];
      MaskVec<VEC> mk[U];
#pragma unroll
      for (int t = 0; t < U; ++t) {
        raw[t] = VecIO<T, VEC>::load_raw(values + (r + t * step) * a.d + col);
        if constexpr (XF) {
          if (a.xform.mask) mk[t] = load_mask<VEC>(a.xform, r + t * step, col);
        }
      }
#pragma unroll
      for (int t = 0; t < U; ++t) {
        float x[VEC], y[VEC];
        VecIO<T, VEC>::unpack(raw[t], x);
        if constexpr (XF) apply_xform<VEC>(x, a.xform, mk[t]);
        normalize_vec<VEC>(x, y, ref, inv);
        VecIO<T, VEC>::store(out + (r + t * step) * a.d + col, y);
      }
    }
    for (; r < r1; r += step) {
      float x[VEC], y[VEC];
      VecIO<T, VEC>::unpack(VecIO<T, VEC>::load_raw(values + r * a.d + col), x);
      if constexpr (XF) {
        MaskVec<VEC> mk;
        if (a.xform.mask) mk = load_mask<VEC>(a.xform, r, col);
        apply_xform<VEC>(x, a.xform, mk);
      }
      normalize_vec<VEC>(x, y, ref, inv);
      VecIO<T, VEC>::store(out + r * a.d + col, y);
    }
  }
}

}  // namespace rgb
