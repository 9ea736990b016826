/*
 * bfknn -- exact brute-force k-NN for NVIDIA B200 (sm_100a), C ABI.
 *
 * Drop-in boundary for the reference's `bf/` kernels (hantaoyu-theory/gpu_algo).
 * Every entry point takes plain pointers and sizes; device pointers are
 * caller-owned CUDA device memory, `stream` is a cudaStream_t (NULL = the
 * legacy default stream).  Launches go on that stream, and the searches and
 * bfk_merge return without waiting for them (bfk_prepare, bfk_filter_values and
 * bfk_search_stats wait).  A kernel's bounded wait that runs out (a device fault the
 * search cannot report at return) is recorded in the workspace and read back by
 * bfk_search_stats as device_error.  No entry point allocates device memory, calls
 * exit(), or throws.  Results:
 *   out_dists (n, k) float32  squared L2 distances, ascending;
 *   out_ids   (n, k) int32    id_offset + database row, ties by lower index;
 *   missing slots (m < k, or rows whose distance is NaN) are padded with
 *   (3.402823e38f, -1); a distance that overflows to +inf is a value like any
 *   other: such rows come last, as the reference's general kernel keeps them
 *   (heap_push, bf/fp32.py:8-27; its small-k kernel drops them instead).
 * Distances are bit-identical to the reference kernels' direct-difference
 * arithmetic (bf/fp32.py:74-82: dif = q - x; dist = fma(dif, dif, dist),
 * in dimension order).
 */
#ifndef BFKNN_H_
#define BFKNN_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define BFK_API __attribute__((visibility("default")))
#else
#define BFK_API
#endif

#define BFK_VERSION_MAJOR 0
#define BFK_VERSION_MINOR 1

typedef enum {
  BFK_OK = 0,
  BFK_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad shape, k <= 0, misaligned pointer */
  BFK_ERR_UNSUPPORTED = 2,      /* shape/k outside what the library was built for   */
  BFK_ERR_WORKSPACE = 3,        /* workspace too small or not 256-byte aligned       */
  BFK_ERR_CUDA = 4,             /* a CUDA runtime call failed                        */
  BFK_ERR_DEVICE_TIMEOUT = 5,   /* a kernel's bounded wait ran out (device status)   */
  BFK_ERR_NO_DEVICE = 6         /* no sm_100 device is current                       */
} bfk_status_t;

typedef enum {
  BFK_ENGINE_AUTO = 0,   /* pick per shape                                              */
  BFK_ENGINE_DIRECT = 1, /* SIMT direct differences with a fused per-query top-k        */
  BFK_ENGINE_TC_F16 = 2  /* tcgen05 f16 distance filter + exact FP32 re-rank            */
} bfk_engine_t;

#define BFK_FLAG_TIME_MAIN 1 /* time the main kernel of every call with CUDA events      */
#define BFK_FLAG_CTA_PAIR 2  /* TC engine: CTA pairs (tcgen05.mma.cta_group::2, M = 256);
                                without it or BFK_FLAG_SINGLE_CTA, pairs are used for
                                d <= 256, more than 128 queries and at least 4M rows
                                (opts.plan_rows when given, else m)                      */
#define BFK_FLAG_PREPARED 4  /* the search reads its rows' TC form from a prepared buffer
                                (bfk_search_prepared); the workspace then holds no rows */
#define BFK_FLAG_SINGLE_CTA 8 /* TC engine: one CTA per query tile (no CTA pairs)         */

/*
 * Called by the TC engine after each filter level with `bound` (device, `count`
 * floats).  A sharded search replaces every value by its minimum over all
 * shards, enqueued on `stream`, before returning.  Optional.
 *   shards <= 1: count = n, per query an upper bound on (k-th distance - ||q||^2)
 *                plus the query's error margin;
 *   shards > 1:  count = 2n, that bound followed by the negated bound that the
 *                shard's ceil(k / shards)-th smallest value gives (its minimum is
 *                minus the maximum over the shards, which bounds the k-th
 *                distance of the union).
 */
typedef void (*bfk_level_hook_t)(float *bound, int64_t count, void *user, void *stream);

typedef struct {
  int32_t engine;         /* bfk_engine_t                                                */
  int32_t slices;         /* database slices per query block, 0 = auto                   */
  int32_t max_candidates; /* TC engines: per-query candidate pool, 0 = auto              */
  int32_t flags;          /* BFK_FLAG_*                                                  */
  int32_t shards;         /* TC engine: shards whose level_hook reduces over all of them
                             (the process group size), 0 = this search alone          */
  int32_t reserved[3];    /* must be zero                                                */
  bfk_level_hook_t level_hook; /* TC engine: see bfk_level_hook_t, NULL = none           */
  void *hook_user;        /* passed to level_hook                                        */
  int64_t plan_rows;      /* TC engine: rows the sampling levels are planned for, 0 = m.
                             Shards of one search pass the same value, so every shard
                             calls level_hook the same number of times.                */
} bfk_opts_t;

typedef struct {
  int32_t num_regs;
  int32_t shared_size_bytes;   /* static shared memory                                  */
  int32_t dynamic_smem_bytes;  /* dynamic shared memory the launch requests             */
  int32_t local_size_bytes;
  int32_t const_size_bytes;
  int32_t max_threads_per_block;
  int32_t binary_version;
  int32_t ptx_version;
  int32_t block_threads;       /* threads per block used at launch                      */
  int32_t reserved[7];
} bfk_attrs_t;

typedef struct {
  int32_t engine_used;         /* bfk_engine_t actually run                              */
  int32_t fallback_queries;    /* TC engines: queries finished by the exact SIMT engine  */
  int64_t candidates;          /* TC engines: candidates written by the filter           */
  int32_t max_query_candidates;
  int32_t slices;
  int64_t survivors;           /* TC engines: rows re-ranked with exact FP32             */
  int32_t device_error;        /* device status word (0 = none)                          */
  int32_t kernel_launches;     /* kernels the last call launched                         */
  int32_t timed_calls;         /* calls timed since the last read (BFK_FLAG_TIME_MAIN)   */
  float main_kernel_ms;        /* summed main-kernel time of those calls                 */
  int32_t cta_pair;            /* TC engine: the plan uses CTA pairs                     */
  int32_t reserved[1];
} bfk_stats_t;

typedef struct {
  int32_t engine;              /* bfk_engine_t the search would run                      */
  int32_t cta_pair;            /* TC engine: the plan uses CTA pairs                     */
  int32_t levels;              /* TC engine: filter passes; the last one reads every tile */
  int32_t q_tiles;             /* TC engine: 128-query tiles (even with CTA pairs)       */
  int32_t cand_cap;            /* TC engine: candidate entries per query                 */
  int32_t reserved0;
  int64_t level_tiles[6];      /* TC engine: 256-row tiles level l reads                 */
  int32_t level_slices[6];     /* TC engine: database slices of level l                  */
} bfk_plan_info_t;

/* Library version.  No reference counterpart. */
BFK_API bfk_status_t bfk_version(int32_t *major, int32_t *minor);

/* Human-readable status.  No reference counterpart (the reference raises CuPy errors). */
BFK_API const char *bfk_status_string(int32_t status);

/* The last failing CUDA call of the calling thread ("file:line call: error (code)").
 * No reference counterpart. */
BFK_API const char *bfk_last_error(void);

/*
 * Device-memory workspace `bfk_search` needs for this shape (bytes, a multiple
 * of 256).  Replaces the per-call CuPy allocations of the reference runners
 * (bf/fp32.py:261-262, bf/fp32_tiled.py:204-207, bf/fp32_qgroup.py:245-248).
 */
BFK_API bfk_status_t bfk_workspace_size(int64_t n, int64_t m, int32_t d, int32_t k,
                                const bfk_opts_t *opts, uint64_t *bytes);

/*
 * Exact k-NN of Q (n, d) against X (m, d), both row-major float32 device
 * arrays.  Replaces one launch of the reference kernels:
 *   bf_fp32 / bf_fp32_smallk   bf/fp32.py:265-271 (kernel bf/fp32.py:53-92, 115-192)
 *   bf_fp32_heap               bf/fp32_heap.py:160-166
 *   bf_fp32_tiled partial+merge bf/fp32_tiled.py:212-224
 *   bf_fp32_qgroup partial+merge bf/fp32_qgroup.py:253-268
 *   bf_fp32_q2                 bf/fp32_q2.py:160-166
 * with the same (out_ids, out_dists) contract, sorted ascending.
 * `workspace` must be 256-byte aligned and at least bfk_workspace_size bytes.
 */
BFK_API bfk_status_t bfk_search(const float *Q, int64_t n, const float *X, int64_t m, int32_t d,
                        int32_t k, int64_t id_offset, float *out_dists, int32_t *out_ids,
                        void *workspace, uint64_t workspace_bytes, const bfk_opts_t *opts,
                        void *stream);

/*
 * Prepared database.  No reference counterpart (the reference re-reads X in FP32 on every
 * call).  bfk_prepare converts X (m, d) once into the TC engine's row form: f16 rows in
 * 64-row groups scaled by powers of two, ||x||^2 and the group scales, with a header that
 * records m and d.  bfk_search_prepared then skips that pass; it still reads X for the
 * exact FP32 re-rank, so X must be the array the buffer was prepared from.  The buffer's
 * bytes are position-independent: copied to a file and back, they stay valid for the same
 * X and library version.  `prepared` is device memory, 256-byte aligned.
 */
BFK_API bfk_status_t bfk_prepared_size(int64_t m, int32_t d, uint64_t *bytes);
BFK_API bfk_status_t bfk_prepare(const float *X, int64_t m, int32_t d, void *prepared,
                                 uint64_t bytes, void *stream);
/* bfk_search with the rows' TC form from `prepared`; `opts` must carry BFK_FLAG_PREPARED
 * (bfk_workspace_size with that flag sizes the smaller workspace).  A buffer made for other
 * (m, d) is rejected with BFK_ERR_INVALID_ARGUMENT: every such search reads the buffer's
 * description back (a synchronous copy of 256 bytes) before it launches anything.  Shapes that the SIMT engine takes
 * ignore the buffer. */
BFK_API bfk_status_t bfk_search_prepared(const float *Q, int64_t n, const float *X,
                                         const void *prepared, int64_t m, int32_t d, int32_t k,
                                         int64_t id_offset, float *out_dists, int32_t *out_ids,
                                         void *workspace, uint64_t workspace_bytes,
                                         const bfk_opts_t *opts, void *stream);

/*
 * Merge `lists` sorted candidate lists per query, laid out (lists, n, k), into
 * the k best per query by (distance, index); index -1 entries are padding.
 * Replaces bf_fp32_tiled_merge (bf/fp32_tiled.py:118-178) and
 * bf_fp32_qgroup_merge (bf/fp32_qgroup.py:153-213); also merges the per-GPU
 * lists of a sharded search.
 */
BFK_API bfk_status_t bfk_merge(const float *cand_dists, const int32_t *cand_ids, int64_t n,
                       int32_t lists, int32_t k, float *out_dists, int32_t *out_ids,
                       void *stream);

/*
 * bfk_merge with list l's (n, k) block of distances (ids) starting l * list_stride
 * elements after cand_dists (cand_ids); list_stride >= n * k.  No reference
 * counterpart: a sharded search all-gathers each rank's distances and ids as one
 * block per rank ([distances | ids], list_stride = 2 n k) and merges them in place.
 */
BFK_API bfk_status_t bfk_merge_strided(const float *cand_dists, const int32_t *cand_ids,
                                       int64_t n, int32_t lists, int64_t list_stride, int32_t k,
                                       float *out_dists, int32_t *out_ids, void *stream);

/*
 * Attributes of the main kernel an engine launches for (d, k).  Replaces
 * kernel_attrs (bf/fp32.py:238-249, CuPy RawKernel.attributes).
 */
BFK_API bfk_status_t bfk_kernel_attrs(int32_t engine, int32_t d, int32_t k, bfk_attrs_t *out);

/*
 * Attributes of the kernel bfk_merge launches for `lists` sorted lists of k per
 * query (the rank merge for a few lists, the sorting network for many).  Replaces
 * kernel_attrs of bf_fp32_tiled_merge / bf_fp32_qgroup_merge, which the reference
 * runners report (bf/fp32_tiled.py:229-239, bf/fp32_qgroup.py:279-291).
 */
BFK_API bfk_status_t bfk_merge_attrs(int32_t lists, int32_t k, bfk_attrs_t *out);

/*
 * The plan a search of this shape would run under these options, computed on the host
 * (no GPU, no workspace): the engine, and for the tensor-core engine its filter levels,
 * the tiles and slices of each, its CTA-pair choice and candidate pool.  The same checks
 * as bfk_workspace_size.  No reference counterpart.
 */
BFK_API bfk_status_t bfk_plan_info(int64_t n, int64_t m, int32_t d, int32_t k,
                                   const bfk_opts_t *opts, bfk_plan_info_t *out);

/*
 * Statistics of the last bfk_search that used this workspace (synchronises
 * `stream`); also returns and resets the main-kernel times this thread
 * recorded with BFK_FLAG_TIME_MAIN.  No reference counterpart.
 */
BFK_API bfk_status_t bfk_search_stats(const void *workspace, int64_t n, int64_t m, int32_t d, int32_t k,
                              const bfk_opts_t *opts, void *stream, bfk_stats_t *out);

/*
 * Test infrastructure for the tensor-core engine's error margin.  No reference
 * counterpart.  Runs the engine's preparation and one filter pass over every row
 * with no bound, and reports the filter value v of every (query, row) pair:
 *   out_v      (n, m) float32  v = ||x||^2 - 2 q.x as the filter computes it
 *                              (NaN where the filter reported none: v not finite);
 *   out_qinfo  (n, 2) float32  ||q||^2 in FP32 and the query's margin m_q;
 *   exact_only                 nonzero when the inputs fall outside what the margin
 *                              covers (a search would use the exact SIMT engine).
 * The engine's exactness rests on |(||q||^2 + v) - D| <= m_q for every pair, D the
 * reference distance (bf/fp32.py:74-82); tests check it against the oracle.
 * Requires n * m <= 2^28.  Synchronises `stream`.
 */
BFK_API bfk_status_t bfk_filter_values_workspace(int64_t n, int64_t m, int32_t d,
                                                 uint64_t *bytes);
BFK_API bfk_status_t bfk_filter_values(const float *Q, int64_t n, const float *X, int64_t m,
                                       int32_t d, float *out_v, float *out_qinfo,
                                       int32_t *exact_only, void *workspace,
                                       uint64_t workspace_bytes, void *stream);

/*
 * Exact k-NN like bfk_search (exact SIMT engine) for callers that cannot
 * allocate device memory at search time (inside another allocator's callback,
 * on a real-time thread that must not block on cudaMalloc, or with only fixed
 * pre-registered buffers).  No counterpart in the reference.
 *
 * It takes no workspace: its scratch is a 16 MiB array inside the library that
 * every GPU loading the library holds until exit.  Requires
 * 16 * n * k <= 16 MiB (n * k <= 1,048,576); larger shapes return
 * BFK_ERR_UNSUPPORTED.  It allocates nothing.  The first call on each device
 * looks the array's device address up (cudaGetSymbolAddress) and keeps it for
 * the life of the process; make that first call outside any stream capture, and
 * do not call cudaDeviceReset between calls (the kept address would be stale).
 * All calls share the array: calls that overlap on the GPU (other streams or
 * threads) race and must be serialised by the caller.
 */
BFK_API bfk_status_t bfk_search_noalloc(const float *Q, int64_t n, const float *X, int64_t m,
                                        int32_t d, int32_t k, int64_t id_offset,
                                        float *out_dists, int32_t *out_ids, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* BFKNN_H_ */
