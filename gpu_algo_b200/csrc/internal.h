// Host-side launch wrappers shared between the translation units of libbfknn.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace bfk {

// Records the last failing CUDA call of this thread (reported by bfk_last_error).
void note_cuda_error(cudaError_t e, const char *file, int line, const char *what);
#define BFK_NOTE(e, what) ::bfk::note_cuda_error((e), __FILE__, __LINE__, (what))

// direct.cu -- exact SIMT engine
size_t direct_smem_bytes(int tq, int k);
const void *direct_kernel_ptr(int tq);
cudaError_t launch_direct(const float *Q, int64_t n, const float *X, int64_t m, int d, int k,
                          int64_t id_offset, int slices, int tq, float *out_d, int32_t *out_i,
                          cudaStream_t stream);

// the exact search for a query count held on the device (the tensor-core engine's
// fallback): lists of fallback_slices(*count, ...) slices, slice s at out + s * count * k
cudaError_t launch_direct_count(const float *Q, const int *count, const float *X, int64_t m,
                                int d, int k, int64_t id_offset, int64_t part_entries,
                                float *out_d, int32_t *out_i, cudaStream_t stream);

// merge.cu -- sorted-list merge
// streaming scan for n <= 16 queries (scan.cu): `blocks` row ranges, each writing its
// sorted top-k per query to out + b*n*k
bool scan_supported(int64_t n, int d, int k);
int scan_blocks(int64_t m, int k);
cudaError_t launch_scan(const float *Q, int64_t n, const float *X, int64_t m, int d, int k,
                        int64_t id_offset, int blocks, float *out_d, int32_t *out_i,
                        cudaStream_t stream);
cudaError_t launch_merge(const float *cand_d, const int32_t *cand_i, int64_t n, int lists, int k,
                         float *out_d, int32_t *out_i, cudaStream_t stream);
// the same, list l's (n, k) block starting l * stride elements after the first
cudaError_t launch_merge_strided(const float *cand_d, const int32_t *cand_i, int64_t n, int lists,
                                 int k, int64_t stride, float *out_d, int32_t *out_i,
                                 cudaStream_t stream);
int merge_max_k();
// merge of launch_direct_count's lists, query q written to output row list[q]
cudaError_t launch_merge_count(const float *cand_d, const int32_t *cand_i, const int *count,
                               int64_t m, int k, int64_t part_entries, const int *list,
                               float *out_d, int32_t *out_i, cudaStream_t stream);
// the kernel launch_merge runs for `lists` lists of k, and its dynamic shared memory
const void *merge_kernel_for(int lists, int k, size_t *smem);
int merge_threads();
cudaError_t launch_fill_pad(float *out_d, int32_t *out_i, int64_t count, cudaStream_t stream);

// tc.cu -- tcgen05 filter engine
constexpr int kMaxLevels = 6;
struct LevelPlan {
  int64_t tiles;            // 256-row tiles this level reads (evenly spaced)
  int64_t tiles_per_slice;
  int slices;
  int region;               // candidate entries per (query, slice)
};
struct TcPlan {
  int64_t n, m;
  int d, k;
  int d_pad;        // d rounded up to 64 (f16 K chunks of 128 bytes)
  int q_tiles;      // ceil(n / 128), rounded up to even when pair
  bool pair;        // CTA pairs issue tcgen05.mma.cta_group::2 (M = 256)
  int64_t x_tiles;  // ceil(m / 256)
  int levels;       // filter passes; the last one reads every tile
  LevelPlan level[kMaxLevels];
  int slices;       // slices of the last level
  int64_t tiles_per_slice;
  int max_slices;
  int cand_cap;     // candidate entries per query
  // workspace offsets (bytes from the workspace base)
  size_t off_xh, off_xnorm, off_xscale, off_qh, off_qinfo, off_rlev, off_cand, off_ccount,
      off_flags, off_fbq, off_fbpart_d, off_fbpart_i, off_invsq, total;
  int fb_slices;
  bool prepared;    // the rows' f16 form, norms and scales come from a prepared buffer
};

// A prepared database (bfk_prepare): the TC engine's row arrays for one X, made once.
// Layout, every part 256-byte aligned: a 256-byte status block (the rows' norm bound, their
// largest f16 rounding error and the exact-only flag, set for a non-finite row, as the
// workspace header holds them), a 256-byte description
// (PreparedInfo), the f16 rows (m, d_pad), ||x||^2 (x_tiles * 256) and a 32-byte record
// of every 64-row group (x_tiles * 4): the minimum ||x||^2 of each of its 16-row chunks,
// then its scale and the scale's inverse.
struct PreparedInfo {
  char magic[8];     // "BFKPREP3"
  int32_t version;   // 3
  int32_t d;
  int64_t m;
  int32_t d_pad;
  int32_t reserved0;
  int64_t x_tiles;
  uint64_t total;    // bytes of the whole buffer
};
struct PreparedLayout {
  size_t off_status, off_info, off_xh, off_xnorm, off_xmeta, total;
};
PreparedLayout tc_prepared_layout(int64_t m, int d);
// Fills `prep` from X on `stream` and waits for it; 0 ok, 1 CUDA error.
int tc_prepare(const float *X, int64_t m, int d, void *prep, cudaStream_t stream);
// Reads the description of `prep` back and checks it against (m, d); 0 ok, 1 CUDA
// error, 3 mismatch.
int tc_check_prepared(const void *prep, int64_t m, int d);
bool tc_supported(int d, int k);
// pair_mode: 1 CTA pairs, -1 single CTAs, 0 tc_pair_default
bool tc_pair_default(int d, int64_t n, int64_t rows);
// shards > 1: the number of shards that share level bounds
bool tc_make_plan(int64_t n, int64_t m, int d, int k, int slices, int cand_cap, int pair_mode,
                  int64_t plan_rows, int shards, bool prepared, TcPlan *p);
// Returns 0 ok, 1 CUDA error; it does not wait for the stream (a device timeout is
// left in the workspace header for bfk_search_stats).  t0/t1 (may be null) are
// recorded around the main kernel; *launches counts the kernels launched.
// `hook` (may be null) is called after every level with the level's bounds;
// `shards` > 1 shards share them, which doubles the bounds handed to the hook.
typedef void (*LevelHook)(float *bound, int64_t count, void *user, void *stream);
int tc_run(const float *Q, const float *X, int64_t id_offset, float *out_d, int32_t *out_i,
           void *ws, const TcPlan &p, cudaStream_t stream, cudaEvent_t t0, cudaEvent_t t1,
           int *launches, LevelHook hook, void *hook_user, int shards,
           const void *prepared = nullptr);
// The filter value of every (query, row) pair (margin audit, test infrastructure):
// a one-level plan whose regions hold every column, and the run that fills out_v
// (n, m) (NaN where no value was reported) and out_qinfo (n, 2) (||q||^2 in FP32,
// margin).  Returns 0 ok, 1 CUDA error, 2 device timeout.
bool tc_make_values_plan(int64_t n, int64_t m, int d, TcPlan *p);
int tc_filter_values(const float *Q, const float *X, float *out_v, float *out_qinfo,
                     int *exact_only, void *ws, const TcPlan &p, cudaStream_t stream);
const void *tc_kernel_ptr(int d, int k);
size_t tc_smem_bytes(int d, int k);
int tc_threads();

}  // namespace bfk
