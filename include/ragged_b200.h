/*
 * ragged_b200.h -- C ABI of the B200 (sm_100a) segmented sum / max / softmax
 * library, libragged_b200.so.
 *
 * It replaces the reference's native launcher (simon-jd/ragged-mlir):
 * the nanobind module `ragged._native.DriverModule` declared in
 * runtime/Driver.h:21-54 and bound in runtime/bindings.cpp:11-36, which
 * loaded MLIR-generated cubins and ran manifest-described launch plans.
 * Here the kernels are built into the library, so the ABI takes the problem
 * (op, dtypes, D, N, B) and plain device pointers instead of a cubin and
 * memref descriptors.  No C++ exception crosses it: every entry point
 * returns an rg_status (0 = success) and rg_last_error() explains failures.
 *
 * Tensor contract (the reference's docs/abi.md and runtime.py:304-365):
 *   values  [N, D] row-major, f32 or bf16, device memory
 *   offsets [B + 1] i32 or i64, offsets[0] = 0, nondecreasing, offsets[B] = N
 *   out     [B, D] for sum / max, [N, D] for softmax, same dtype as values,
 *           disjoint from values and offsets
 * All launches are asynchronous on the caller's stream; nothing is read back
 * and nothing synchronises (the reference's "validated" mode).
 */
#ifndef RAGGED_B200_H
#define RAGGED_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; everything declared here is
 * exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ------------------------------------------------------------- constants */
enum rg_status {
  RG_OK = 0,
  RG_ERR_INVALID_ARGUMENT = 1, /* shape, dtype, pointer or alignment problem  */
  RG_ERR_UNSUPPORTED = 2,      /* valid request this build does not implement */
  RG_ERR_WORKSPACE = 3,        /* workspace missing, misaligned or too small  */
  RG_ERR_CUDA = 4,             /* a CUDA runtime call or launch failed        */
  RG_ERR_DEVICE = 5            /* no device, or not compute capability 10.0   */
};

enum rg_op { RG_OP_SUM = 0, RG_OP_MAX = 1, RG_OP_SOFTMAX = 2 };
enum rg_dtype { RG_DTYPE_F32 = 0, RG_DTYPE_BF16 = 1 };
enum rg_index { RG_INDEX_I32 = 0, RG_INDEX_I64 = 1 };

/* Schedules.  CLASSIFIED and NAIVE are the reference's two strategies
 * (python/ragged/runtime.py:252-268); ROWBALANCED is this build's
 * row-balanced (merge-path) schedule for sum and max. */
enum rg_schedule {
  RG_SCHEDULE_CLASSIFIED = 0,
  RG_SCHEDULE_NAIVE = 1,
  RG_SCHEDULE_ROWBALANCED = 2
};

/* rg_run flags */
#define RG_FLAG_NO_VECTORIZE 1u /* one feature per thread (reference Optimizations(vectorize=False)) */
/* Softmax only: out IS values (same pointer, N rows), the reference's
 * ProgramSpec(alias="inplace") (python/ragged/model.py:119-122,
 * docs/classified-abi.md:208-214).  Every schedule finishes a segment's
 * statistics reads before it writes any of the segment's rows, and writes
 * each element only after its last read. */
#define RG_FLAG_IN_PLACE 2u
/* rg_run_pointwise: always materialise the transformed f32 logits (the
 * reference's Optimizations(pointwise_fusion=False) route).  Without it, a
 * softmax on the classified schedule whose rows the worker stages applies
 * the transform as it loads. */
#define RG_FLAG_NO_POINTWISE_FUSION 4u

#define RG_MAX_LAUNCHES 8

/* What one call launched (the reference's ExecutionReport grid / kernel
 * fields, python/ragged/model.py:215-252). */
typedef struct rg_report {
  int32_t schedule;                       /* rg_schedule that ran             */
  int32_t num_launches;                   /* kernel launches                  */
  int32_t kernel_ids[RG_MAX_LAUNCHES];    /* see rg_kernel_name()             */
  int32_t grid[RG_MAX_LAUNCHES][3];
  int32_t block[RG_MAX_LAUNCHES];
  int32_t shared_bytes[RG_MAX_LAUNCHES];
  int32_t memsets;                        /* cudaMemsetAsync calls            */
  int32_t d_vector;                       /* adjacent features per thread     */
  int32_t d_tile;                         /* threads spanning one row tile    */
  int32_t streams;                        /* streams used (1: caller's only)  */
  int64_t workspace_bytes;                /* scratch the call required        */
  int64_t thresholds[2];                  /* classified: warp- and CTA-class length bounds (rows) */
  /* Byte offset in the workspace of the call's device status word (int64;
   * nonzero once the stream has run the call means a bounded wait inside
   * a kernel gave up and the call's results are undefined), or -1 when the
   * schedule keeps none.  Checked mode reads it back after the call. */
  int64_t status_offset;
} rg_report;

typedef struct rg_device_info {
  int32_t device;
  int32_t sm_count;
  int32_t cc_major, cc_minor;
  int64_t l2_bytes;
  int32_t smem_per_block_optin;
  int32_t max_threads_per_sm;
} rg_device_info;

/* ----------------------------------------------------------- entry points */

/* Library version string, e.g. "ragged-b200 0.1.0 (sm_100a)". */
const char *rg_version(void);

/* Static description of a status code. */
const char *rg_error_string(int status);

/* Detail of the last failure on the calling thread ("" if none).  Replaces
 * the reference's std::runtime_error text (runtime/Driver.cpp:85-95). */
const char *rg_last_error(void);

/* Properties of CUDA device `device`, queried once and cached.  Replaces
 * the reference's device() / residentBlocks() helpers (Driver.h:34-37) and
 * the L2 query of runtime.py:165-178. */
int rg_get_device_info(int device, rg_device_info *info);

/* Scratch bytes rg_run needs for this problem on the current device (0 for
 * the block-per-segment schedule); `flags` as for rg_run.  Replaces the workspace sizing of the
 * reference's layout.py:186-243 (resolve_layout) and runtime.py:534-542. */
int rg_workspace_bytes(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b,
                       int schedule, int64_t max_len, uint32_t flags, int64_t *bytes);

/* Launch one segmented operation on `stream` (a cudaStream_t; NULL = the
 * legacy default stream).  `workspace` must hold rg_workspace_bytes() bytes
 * (256-byte aligned) and may be NULL when that is 0.  `max_len` is the
 * caller's bound on the longest segment or -1 when unknown.  `report` may be
 * NULL.  Replaces DriverModule.launch / add_plan / run_plan
 * (runtime/Driver.h:31-47, runtime/Driver.cpp:247-353). */
int rg_run(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b,
           const void *values, const void *offsets, void *out, void *workspace,
           int64_t workspace_bytes, int schedule, int64_t max_len, uint32_t flags,
           void *stream, rg_report *report);

/* Pointwise input transform (the reference's ProgramSpec scale / mask,
 * docs/mask-abi.md; python/ragged/runtime.py:346-356 for the mask rules):
 * every value becomes x = f32(values) * scale (scale != 1) + mask (f32
 * [N][D], softmax only; NULL = none), two f32 roundings, and `op` runs on x
 * with `schedule`; results round once to `dtype`.  A softmax on the
 * classified schedule whose rows the worker stages (one column tile of
 * 16-byte vectors; a mask 16-byte aligned and, in place, disjoint from
 * values) applies the transform as it loads, as the reference's
 * loadInput does (lib/Conversion/ToGPU.cpp:604-618); every other call, and
 * any call with RG_FLAG_NO_POINTWISE_FUSION, materialises the transformed
 * values in `workspace` first (the reference's route with pointwise fusion
 * off, ToGPU.cpp:41-60).  rg_report.kernel_ids show which route ran.  The
 * mask may alias values but not out or offsets.  Workspace from
 * rg_pointwise_workspace_bytes (enough for either route); otherwise as
 * rg_run. */
int rg_pointwise_workspace_bytes(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b,
                                 int schedule, int64_t max_len, uint32_t flags, int64_t *bytes);
int rg_run_pointwise(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b,
                     const void *values, const void *offsets, const float *mask, float scale, void *out,
                     void *workspace, int64_t workspace_bytes, int schedule, int64_t max_len, uint32_t flags,
                     void *stream, rg_report *report);

/* Name of a kernel id reported in rg_report.kernel_ids ("" if unknown). */
const char *rg_kernel_name(int kernel_id);

/* Checked mode: validate offsets[0..b] on the device (caller's stream)
 * before any main launch.  status (device memory, 7 x int64) receives, per
 * condition, the earliest offending index or INT64_MAX: 0 offsets[0] != 0,
 * 1 offsets[b] != n, 2 an offset < 0, 3 an offset > n, 4 a decreasing pair
 * (left index), 5 a segment shorter than min_len, 6 longer than max_len
 * (bounds -1 = none; lengths only of in-range monotone pairs).  The caller
 * reads status back after the stream completes.  Replaces the reference's
 * offsets-check-v1 validation kernels (docs/checked-abi.md,
 * lib/Conversion/ToGPU.cpp:1067-1189). */
int rg_check_offsets(int index_dtype, int64_t n, int64_t b, const void *offsets, int64_t min_len, int64_t max_len,
                     int64_t *status, void *stream, rg_report *report);

/* ------------------------------------------------ sharded calls (multi-GPU)
 *
 * One process per GPU.  Rank r of `world` holds rows [row0, row1) of the
 * packed values (rg_shard_rows: a row-balanced split) and the whole offsets
 * array.  rg_run_shard reduces the rank's rows and writes every segment
 * that ends in its rows and started there; the pieces of the segments cut
 * at its edges go to its edge record.  The caller all-gathers the edge
 * records of all ranks in rank order (e.g. NCCL all-gather; a few KB per
 * rank) and calls rg_shard_combine, which writes the cut segments this rank
 * finishes.  Together the ranks write every output row exactly once (each
 * on the rank that holds the segment's end).  Sum and max only.
 * Every `splits` argument below is NULL (the even row split) or HOST memory
 * holding exactly world + 1 nondecreasing row boundaries from 0 to n: the
 * library reads world + 1 entries and cannot check the array's length.
 * The reference is single-GPU; these entry points are this build's
 * multi-GPU extension of its launcher (runtime/Driver.h:21-54). */

/* Rows [*row0, *row1) of rank `rank` in the even row split of n rows. */
int rg_shard_rows(int64_t n, int world, int rank, int64_t *row0, int64_t *row1);

/* A split balanced by work: splits[0..world] (host memory) such that every
 * rank holds about the same rows + end_weight x segment ends (a segment end
 * writes an output row; 1.25 balances bf16 D=256 on B200).  offsets is
 * HOST memory (b + 1 entries).  Pass the split to the calls below; NULL
 * there means the even row split. */
int rg_shard_split(const void *offsets, int index_dtype, int64_t b, int world, double end_weight, int64_t *splits);

/* Bytes of one rank's edge record (header + two f32 pieces of D features). */
int rg_shard_edge_bytes(int op, int64_t d, int64_t *bytes);

/* Scratch bytes rg_run_shard needs (256-byte aligned) on the current device. */
int rg_shard_workspace_bytes(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, int world,
                             int rank, const int64_t *splits, uint32_t flags, int64_t *bytes);

/* Reduce rank `rank`'s rows (splits[rank] to splits[rank + 1], or the even
 * split when splits is NULL) of a call over n rows and b segments: values
 * holds those rows (the first first), offsets all b + 1 entries (device),
 * out all b rows (only the rows this rank finishes are written), edges this
 * rank's edge record (rg_shard_edge_bytes, 16-byte aligned device memory).
 * Segments that end at row 0 belong to rank 0. */
int rg_run_shard(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, int world, int rank,
                 const int64_t *splits, const void *values, const void *offsets, void *out, void *edges,
                 void *workspace, int64_t workspace_bytes, uint32_t flags, void *stream, rg_report *report);

/* Finish the segments cut by shard boundaries that this rank owns, from
 * the gathered edge records of ranks 0..world-1 (device memory, rank
 * order). */
int rg_shard_combine(int op, int dtype, int64_t d, int world, int rank, const void *gathered, void *out,
                     uint32_t flags, void *stream);

/* Sharded softmax (this build's multi-GPU extension; no counterpart in the
 * reference, which runs one device): rank r normalises its own rows
 * [row0, row1) into out (its rows only).  rg_shard_segments gives, from host
 * offsets, the window's segments [seg0, seg1) (those whose end the window
 * consumes, plus the one open at its end), whose statistics the rank keeps
 * (2 D floats each) in its workspace.  rg_run_shard_softmax computes them
 * and the edge record (reference and mass pieces of the segments cut at the
 * window's edges, rg_shard_edge_bytes(RG_OP_SOFTMAX, d) bytes); after the
 * all-gather, rg_shard_softmax_finish merges, in rank order, the cut
 * segments' pieces from every rank's record and normalises the window's
 * rows.  The workspace must persist between the two phases. */
int rg_shard_segments(const void *offsets_host, int index_dtype, int64_t b, int world, int rank,
                      const int64_t *splits, int64_t *seg0, int64_t *seg1);
int rg_shard_softmax_workspace_bytes(int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, int world,
                                     int rank, const int64_t *splits, int64_t seg0, int64_t seg1, uint32_t flags,
                                     int64_t *bytes);
int rg_run_shard_softmax(int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, int world, int rank,
                         const int64_t *splits, int64_t seg0, int64_t seg1, const void *values,
                         const void *offsets, void *edges, void *workspace, int64_t workspace_bytes,
                         uint32_t flags, void *stream, rg_report *report);
int rg_shard_softmax_finish(int dtype, int index_dtype, int64_t d, int64_t n, int64_t b, int world, int rank,
                            const int64_t *splits, int64_t seg0, int64_t seg1, const void *values,
                            const void *offsets, const void *gathered, void *out, void *workspace,
                            int64_t workspace_bytes, uint32_t flags, void *stream, rg_report *report);

/* Row-balanced segmented sum or max that allocates nothing and takes no
 * workspace: for callers that may not allocate device memory (a host that
 * reserves all device memory for its own pool, a plugin callback that may
 * not allocate, a path that cannot afford cudaMalloc's synchronisation).
 * It has no counterpart in the reference.  Its scratch is a static 8 MiB
 * device array per GPU, held until the process exits; the CTA count is
 * reduced to fit it (RG_ERR_WORKSPACE if even one CTA per SM would not).
 * The first call on a device resolves the array's address and should come
 * before any stream capture.  All calls on a device share the array, so
 * calls that overlap on the GPU race; nothing in it needs zeroing.
 * Arguments as for rg_run (sum and max only). */
int rg_run_noalloc(int op, int dtype, int index_dtype, int64_t d, int64_t n, int64_t b,
                   const void *values, const void *offsets, void *out, uint32_t flags, void *stream);

/* ------------------------------------------------------- schedule choice
 * This build's extension (the reference chooses in Python,
 * python/ragged/selection.py:106-126): the scores of the boosted decision
 * trees that ragged/selection.py's TreeChooser stores as flat node arrays.
 * Node i tests x[feature[i]] <= threshold[i] (then left[i], else right[i])
 * unless leaf[i] != 0, where it holds value[i]; scores[c] = baseline[c] plus
 * the leaf values reached in the trees whose tree_class is c.  Host memory
 * only, no device needed.  RG_ERR_INVALID_ARGUMENT for an index out of range
 * or a walk longer than max_depth. */
int rg_tree_scores(int64_t nodes, const int32_t *feature, const double *threshold, const int32_t *left,
                   const int32_t *right, const double *value, const uint8_t *leaf, int64_t trees,
                   const int32_t *roots, const int32_t *tree_class, int classes, const double *baseline,
                   int features, const double *x, int max_depth, double *scores);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* RAGGED_B200_H */
