// C ABI of libbfknn: argument validation, workspace layout, engine dispatch.
#include <cstdio>
#include <cstring>
#include <utility>
#include <vector>

#include "../../include/bfknn.h"
#include "common.cuh"
#include "internal.h"

using namespace bfk;

namespace {

constexpr int kMaxK = 1024;
constexpr int kMaxD = 4096;
constexpr int64_t kMaxAuditPairs = (int64_t)1 << 28;  // bfk_filter_values: (query, row) pairs

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct DirectPlan {
  int tq, slices;
  bool scan;  // small batch: the streaming scan kernel, `slices` blocks of rows
  size_t off_part_d, off_part_i, total;
};

int sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

DirectPlan direct_plan(int64_t n, int64_t m, int d, int k, int slices_req) {
  DirectPlan p{};
  if (slices_req <= 0 && m >= 8192 && scan_supported(n, d, k)) {
    // a handful of queries: one streaming pass over the rows, many warps in flight
    p.scan = true;
    p.slices = scan_blocks(m, k);
    size_t off = sizeof(WsHeader);
    p.off_part_d = off;
    off = align256(off + (size_t)p.slices * n * k * sizeof(float));
    p.off_part_i = off;
    off = align256(off + (size_t)p.slices * n * k * sizeof(int32_t));
    p.total = align256(off);
    return p;
  }
  p.tq = (n >= 64 && k <= 512) ? 4 : 1;
  const int qb = 8 * p.tq;
  const int64_t qblocks = (n + qb - 1) / qb;
  int slices = slices_req;
  if (slices <= 0) {
    const int64_t target = 3LL * sm_count();
    slices = (int)((target + qblocks - 1) / (qblocks > 0 ? qblocks : 1));
    const int64_t by_rows = (m + 1023) / 1024;
    if (slices > by_rows) slices = (int)by_rows;
    // keep the partial lists under 1 GiB
    const int64_t per_slice = (n > 0 ? n : 1) * (int64_t)k * 8;
    const int64_t by_mem = ((int64_t)1 << 30) / per_slice;
    if (slices > by_mem) slices = (int)by_mem;
    if (slices < 1) slices = 1;
  }
  if (slices > 65535) slices = 65535;
  p.slices = slices;
  size_t off = sizeof(WsHeader);
  if (slices > 1) {
    p.off_part_d = off;
    off = align256(off + (size_t)slices * n * k * sizeof(float));
    p.off_part_i = off;
    off = align256(off + (size_t)slices * n * k * sizeof(int32_t));
  }
  p.total = align256(off);
  (void)d;
  return p;
}

// the TC engine's plan under these options (BFK_FLAG_PREPARED: rows from a prepared buffer)
bool make_plan(int64_t n, int64_t m, int32_t d, int32_t k, const bfk_opts_t *opts, TcPlan *p) {
  const int flags = opts ? opts->flags : 0;
  const int pair_mode = (flags & BFK_FLAG_CTA_PAIR) ? 1 : (flags & BFK_FLAG_SINGLE_CTA) ? -1 : 0;
  return tc_make_plan(n, m, d, k, opts ? opts->slices : 0, opts ? opts->max_candidates : 0,
                      pair_mode, opts ? opts->plan_rows : 0,
                      opts && opts->level_hook ? opts->shards : 0,
                      opts && (opts->flags & BFK_FLAG_PREPARED), p);
}

bool opts_ok(const bfk_opts_t *o) {
  if (!o) return true;
  for (int i = 0; i < 3; i++)
    if (o->reserved[i] != 0) return false;
  return o->engine >= BFK_ENGINE_AUTO && o->engine <= BFK_ENGINE_TC_F16 && o->slices >= 0 &&
         o->max_candidates >= 0 && o->plan_rows >= 0 && o->shards >= 0 &&
         (o->flags & ~(BFK_FLAG_TIME_MAIN | BFK_FLAG_CTA_PAIR | BFK_FLAG_PREPARED |
                       BFK_FLAG_SINGLE_CTA)) == 0 &&
         (o->flags & (BFK_FLAG_CTA_PAIR | BFK_FLAG_SINGLE_CTA)) !=
             (BFK_FLAG_CTA_PAIR | BFK_FLAG_SINGLE_CTA);
}

int choose_engine(int64_t n, int64_t m, int d, int k, const bfk_opts_t *o) {
  const int req = o ? o->engine : BFK_ENGINE_AUTO;
  if (req != BFK_ENGINE_AUTO) return req;
  // Shards of one search (plan_rows set) decide on the largest shard's rows, so that
  // every shard picks the same engine and makes the same level-hook calls.
  const int64_t rows = (o && o->plan_rows > m) ? o->plan_rows : m;
  // the filter engine needs whole 128-query tiles' worth of work to pay off
  if (tc_supported(d, k) && n >= 64 && rows >= 4096) return BFK_ENGINE_TC_F16;
  return BFK_ENGINE_DIRECT;
}

bfk_status_t check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BFK_ERR_NO_DEVICE;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return BFK_ERR_NO_DEVICE;
  return major == 10 ? BFK_OK : BFK_ERR_NO_DEVICE;
}

bfk_status_t validate(int64_t n, int64_t m, int32_t d, int32_t k, int64_t id_offset) {
  if (n < 0 || m < 0 || d <= 0 || k <= 0) return BFK_ERR_INVALID_ARGUMENT;
  if (d > kMaxD || k > kMaxK) return BFK_ERR_UNSUPPORTED;
  if (n > INT32_MAX) return BFK_ERR_UNSUPPORTED;
  if (id_offset < 0 || id_offset + m > (int64_t)INT32_MAX) return BFK_ERR_UNSUPPORTED;
  return BFK_OK;
}

bfk_status_t cuda_status_at(cudaError_t e, const char *file, int line) {
  if (e == cudaSuccess) return BFK_OK;
  bfk::note_cuda_error(e, file, line, "launch");
  return BFK_ERR_CUDA;
}
#define cuda_status(e) cuda_status_at((e), __FILE__, __LINE__)

thread_local char g_last_error[256] = "no error";

// Per-thread record of main-kernel timings (BFK_FLAG_TIME_MAIN) and of the
// number of kernels the last call launched.
struct CallRecord {
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending, spare;
  int launches = 0;
  ~CallRecord() {
    for (auto &p : pending) { cudaEventDestroy(p.first); cudaEventDestroy(p.second); }
    for (auto &p : spare) { cudaEventDestroy(p.first); cudaEventDestroy(p.second); }
  }
  bool take(cudaEvent_t *a, cudaEvent_t *b) {
    if (pending.size() >= 4096) return false;
    if (spare.empty()) {
      cudaEvent_t x, y;
      if (cudaEventCreate(&x) != cudaSuccess) return false;
      if (cudaEventCreate(&y) != cudaSuccess) { cudaEventDestroy(x); return false; }
      spare.emplace_back(x, y);
    }
    *a = spare.back().first;
    *b = spare.back().second;
    pending.push_back(spare.back());
    spare.pop_back();
    return true;
  }
  // The pair of the latest take() was never recorded (the call failed first): reading
  // its elapsed time would fail and leave that error for the next cudaGetLastError().
  void give_back() {
    if (pending.empty()) return;
    spare.push_back(pending.back());
    pending.pop_back();
  }
};
thread_local CallRecord g_calls;

}  // namespace

namespace bfk {
void note_cuda_error(cudaError_t e, const char *file, int line, const char *what) {
  const char *base = std::strrchr(file, '/');
  std::snprintf(g_last_error, sizeof(g_last_error), "%s:%d %s: %s (%d)", base ? base + 1 : file,
                line, what, cudaGetErrorString(e), (int)e);
}
}  // namespace bfk

extern "C" {

const char *bfk_last_error(void) { return g_last_error; }

bfk_status_t bfk_version(int32_t *major, int32_t *minor) {
  if (!major || !minor) return BFK_ERR_INVALID_ARGUMENT;
  *major = BFK_VERSION_MAJOR;
  *minor = BFK_VERSION_MINOR;
  return BFK_OK;
}

const char *bfk_status_string(int32_t s) {
  switch (s) {
    case BFK_OK: return "ok";
    case BFK_ERR_INVALID_ARGUMENT: return "invalid argument";
    case BFK_ERR_UNSUPPORTED: return "unsupported shape or k";
    case BFK_ERR_WORKSPACE: return "workspace too small or misaligned";
    case BFK_ERR_CUDA: return "CUDA runtime error";
    case BFK_ERR_DEVICE_TIMEOUT: return "a kernel's bounded wait ran out";
    case BFK_ERR_NO_DEVICE: return "no sm_100 device is current";
    default: return "unknown status";
  }
}

bfk_status_t bfk_workspace_size(int64_t n, int64_t m, int32_t d, int32_t k,
                                const bfk_opts_t *opts, uint64_t *bytes) {
  if (!bytes || !opts_ok(opts)) return BFK_ERR_INVALID_ARGUMENT;
  bfk_status_t s = validate(n, m, d, k, 0);
  if (s != BFK_OK) return s;
  const int eng = choose_engine(n, m, d, k, opts);
  if (eng == BFK_ENGINE_TC_F16) {
    if (!tc_supported(d, k)) return BFK_ERR_UNSUPPORTED;
    TcPlan p;
    if (!make_plan(n, m, d, k, opts, &p))
      return BFK_ERR_UNSUPPORTED;
    *bytes = p.total;
  } else {
    *bytes = direct_plan(n, m, d, k, opts ? opts->slices : 0).total;
  }
  return BFK_OK;
}

bfk_status_t bfk_plan_info(int64_t n, int64_t m, int32_t d, int32_t k, const bfk_opts_t *opts,
                           bfk_plan_info_t *out) {
  if (!out || !opts_ok(opts)) return BFK_ERR_INVALID_ARGUMENT;
  bfk_status_t s = validate(n, m, d, k, 0);
  if (s != BFK_OK) return s;
  bfk_plan_info_t info{};
  info.engine = choose_engine(n, m, d, k, opts);
  if (info.engine == BFK_ENGINE_TC_F16) {
    TcPlan p;
    if (!tc_supported(d, k) || !make_plan(n, m, d, k, opts, &p)) return BFK_ERR_UNSUPPORTED;
    info.cta_pair = p.pair ? 1 : 0;
    info.levels = p.levels;
    info.q_tiles = p.q_tiles;
    info.cand_cap = p.cand_cap;
    for (int l = 0; l < p.levels && l < 6; l++) {
      info.level_tiles[l] = p.level[l].tiles;
      info.level_slices[l] = p.level[l].slices;
    }
  }
  *out = info;
  return BFK_OK;
}

static bfk_status_t search_body(const float *Q, int64_t n, const float *X, const void *prepared,
                                int64_t m, int32_t d, int32_t k, int64_t id_offset,
                                float *out_dists, int32_t *out_ids, void *workspace,
                                uint64_t workspace_bytes, const bfk_opts_t *opts, void *stream_,
                                bool *timed);

static bfk_status_t search_impl(const float *Q, int64_t n, const float *X, const void *prepared,
                                int64_t m, int32_t d, int32_t k, int64_t id_offset,
                                float *out_dists, int32_t *out_ids, void *workspace,
                                uint64_t workspace_bytes, const bfk_opts_t *opts, void *stream_) {
  g_calls.launches = 0;
  bool timed = false;
  const bfk_status_t s = search_body(Q, n, X, prepared, m, d, k, id_offset, out_dists, out_ids,
                                     workspace, workspace_bytes, opts, stream_, &timed);
  if (timed && s != BFK_OK) g_calls.give_back();
  return s;
}

// *timed: an event pair was taken for BFK_FLAG_TIME_MAIN (it is recorded on success)
static bfk_status_t search_body(const float *Q, int64_t n, const float *X, const void *prepared,
                                int64_t m, int32_t d, int32_t k, int64_t id_offset,
                                float *out_dists, int32_t *out_ids, void *workspace,
                                uint64_t workspace_bytes, const bfk_opts_t *opts, void *stream_,
                                bool *timed) {
  if (!opts_ok(opts)) return BFK_ERR_INVALID_ARGUMENT;
  // a prepared buffer comes with BFK_FLAG_PREPARED (which sizes the workspace without rows)
  if ((prepared != nullptr) != (opts && (opts->flags & BFK_FLAG_PREPARED)))
    return BFK_ERR_INVALID_ARGUMENT;
  bfk_status_t s = validate(n, m, d, k, id_offset);
  if (s != BFK_OK) return s;
  if (n == 0) return BFK_OK;
  if (!Q || !out_dists || !out_ids || (m > 0 && !X) || !workspace) return BFK_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(X) |
       reinterpret_cast<uintptr_t>(out_dists) | reinterpret_cast<uintptr_t>(out_ids)) & 3u)
    return BFK_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return BFK_ERR_WORKSPACE;
  if ((s = check_device()) != BFK_OK) return s;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const int eng = choose_engine(n, m, d, k, opts);
  unsigned char *ws = static_cast<unsigned char *>(workspace);
  cudaEvent_t t0 = nullptr, t1 = nullptr;
  if (opts && (opts->flags & BFK_FLAG_TIME_MAIN) && !g_calls.take(&t0, &t1)) t0 = t1 = nullptr;
  *timed = t0 != nullptr;

  if (eng == BFK_ENGINE_TC_F16) {
    if (!tc_supported(d, k)) return BFK_ERR_UNSUPPORTED;
    TcPlan p;
    if (!make_plan(n, m, d, k, opts, &p))
      return BFK_ERR_UNSUPPORTED;
    if (workspace_bytes < p.total) return BFK_ERR_WORKSPACE;
    if (prepared) {
      const int pc = tc_check_prepared(prepared, m, d);
      if (pc == 1) return BFK_ERR_CUDA;
      if (pc == 3) return BFK_ERR_INVALID_ARGUMENT;  // made for other rows
    }
    int rc = tc_run(Q, X, id_offset, out_dists, out_ids, ws, p, stream, t0, t1, &g_calls.launches,
                    opts ? opts->level_hook : nullptr, opts ? opts->hook_user : nullptr,
                    opts ? opts->shards : 0, prepared);
    if (rc == 1) return BFK_ERR_CUDA;
    if (rc == 2) return BFK_ERR_DEVICE_TIMEOUT;
    return BFK_OK;
  }

  // exact SIMT engine
  DirectPlan p = direct_plan(n, m, d, k, opts ? opts->slices : 0);
  if (workspace_bytes < p.total) return BFK_ERR_WORKSPACE;
  WsHeader *hdr = reinterpret_cast<WsHeader *>(ws);
  cudaError_t e = cudaMemsetAsync(hdr, 0, sizeof(WsHeader), stream);
  if (e != cudaSuccess) return cuda_status(e);
  if (m == 0) {
    // nothing to search: every slot is padding (the fill is the timed kernel)
    g_calls.launches = 1;
    if (t0) cudaEventRecord(t0, stream);
    e = launch_fill_pad(out_dists, out_ids, n * k, stream);
    if (t1) cudaEventRecord(t1, stream);
    return cuda_status(e);
  }
  if (t0) cudaEventRecord(t0, stream);
  if (p.scan) {
    const bool one = p.slices == 1;
    float *pd = one ? out_dists : reinterpret_cast<float *>(ws + p.off_part_d);
    int32_t *pi = one ? out_ids : reinterpret_cast<int32_t *>(ws + p.off_part_i);
    e = launch_scan(Q, n, X, m, d, k, id_offset, p.slices, pd, pi, stream);
    if (t1) cudaEventRecord(t1, stream);
    if (e != cudaSuccess || one) {
      g_calls.launches = 1;
      return cuda_status(e);
    }
    g_calls.launches = 2;
    return cuda_status(launch_merge(pd, pi, n, p.slices, k, out_dists, out_ids, stream));
  }
  if (p.slices == 1) {
    e = launch_direct(Q, n, X, m, d, k, id_offset, 1, p.tq, out_dists, out_ids, stream);
    if (t1) cudaEventRecord(t1, stream);
    g_calls.launches = 1;
    return cuda_status(e);
  }
  float *pd = reinterpret_cast<float *>(ws + p.off_part_d);
  int32_t *pi = reinterpret_cast<int32_t *>(ws + p.off_part_i);
  e = launch_direct(Q, n, X, m, d, k, id_offset, p.slices, p.tq, pd, pi, stream);
  if (t1) cudaEventRecord(t1, stream);
  if (e != cudaSuccess) return cuda_status(e);
  g_calls.launches = 2;
  return cuda_status(launch_merge(pd, pi, n, p.slices, k, out_dists, out_ids, stream));
}

bfk_status_t bfk_search(const float *Q, int64_t n, const float *X, int64_t m, int32_t d,
                        int32_t k, int64_t id_offset, float *out_dists, int32_t *out_ids,
                        void *workspace, uint64_t workspace_bytes, const bfk_opts_t *opts,
                        void *stream) {
  return search_impl(Q, n, X, nullptr, m, d, k, id_offset, out_dists, out_ids, workspace,
                     workspace_bytes, opts, stream);
}

bfk_status_t bfk_search_prepared(const float *Q, int64_t n, const float *X, const void *prepared,
                                 int64_t m, int32_t d, int32_t k, int64_t id_offset,
                                 float *out_dists, int32_t *out_ids, void *workspace,
                                 uint64_t workspace_bytes, const bfk_opts_t *opts, void *stream) {
  if (!prepared || (reinterpret_cast<uintptr_t>(prepared) & 255u)) return BFK_ERR_INVALID_ARGUMENT;
  return search_impl(Q, n, X, prepared, m, d, k, id_offset, out_dists, out_ids, workspace,
                     workspace_bytes, opts, stream);
}

bfk_status_t bfk_prepared_size(int64_t m, int32_t d, uint64_t *bytes) {
  if (!bytes || m < 0 || m > INT32_MAX || d <= 0) return BFK_ERR_INVALID_ARGUMENT;
  if (!tc_supported(d, 1)) return BFK_ERR_UNSUPPORTED;
  *bytes = tc_prepared_layout(m, d).total;
  return BFK_OK;
}

bfk_status_t bfk_prepare(const float *X, int64_t m, int32_t d, void *prepared, uint64_t bytes,
                         void *stream) {
  if (!prepared || (m > 0 && !X) || m < 0 || m > INT32_MAX || d <= 0) return BFK_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(prepared) & 255u) || (reinterpret_cast<uintptr_t>(X) & 3u))
    return BFK_ERR_INVALID_ARGUMENT;
  if (!tc_supported(d, 1)) return BFK_ERR_UNSUPPORTED;
  if (bytes < tc_prepared_layout(m, d).total) return BFK_ERR_WORKSPACE;
  bfk_status_t s = check_device();
  if (s != BFK_OK) return s;
  return tc_prepare(X, m, d, prepared, reinterpret_cast<cudaStream_t>(stream)) == 0 ? BFK_OK
                                                                                    : BFK_ERR_CUDA;
}

bfk_status_t bfk_filter_values_workspace(int64_t n, int64_t m, int32_t d, uint64_t *bytes) {
  if (!bytes || n <= 0 || m <= 0 || d <= 0) return BFK_ERR_INVALID_ARGUMENT;
  if (n > INT32_MAX || m > INT32_MAX || n * m > kMaxAuditPairs || !tc_supported(d, 1))
    return BFK_ERR_UNSUPPORTED;
  TcPlan p;
  if (!tc_make_values_plan(n, m, d, &p)) return BFK_ERR_UNSUPPORTED;
  *bytes = p.total;
  return BFK_OK;
}

bfk_status_t bfk_filter_values(const float *Q, int64_t n, const float *X, int64_t m, int32_t d,
                               float *out_v, float *out_qinfo, int32_t *exact_only,
                               void *workspace, uint64_t workspace_bytes, void *stream) {
  uint64_t need = 0;
  const bfk_status_t s = bfk_filter_values_workspace(n, m, d, &need);
  if (s != BFK_OK) return s;
  if (!Q || !X || !out_v || !out_qinfo || !exact_only || !workspace)
    return BFK_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(X) |
       reinterpret_cast<uintptr_t>(out_v) | reinterpret_cast<uintptr_t>(out_qinfo)) & 3u)
    return BFK_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) || workspace_bytes < need)
    return BFK_ERR_WORKSPACE;
  const bfk_status_t dev = check_device();
  if (dev != BFK_OK) return dev;
  TcPlan p;
  tc_make_values_plan(n, m, d, &p);
  int eo = 0;
  const int rc = tc_filter_values(Q, X, out_v, out_qinfo, &eo, workspace, p,
                                  reinterpret_cast<cudaStream_t>(stream));
  if (rc == 1) return BFK_ERR_CUDA;
  if (rc == 2) return BFK_ERR_DEVICE_TIMEOUT;
  *exact_only = eo;
  return BFK_OK;
}

bfk_status_t bfk_merge(const float *cand_dists, const int32_t *cand_ids, int64_t n,
                       int32_t lists, int32_t k, float *out_dists, int32_t *out_ids,
                       void *stream) {
  if (n < 0 || lists <= 0 || k <= 0) return BFK_ERR_INVALID_ARGUMENT;
  if (k > merge_max_k()) return BFK_ERR_UNSUPPORTED;
  if (n == 0) return BFK_OK;
  if (!cand_dists || !cand_ids || !out_dists || !out_ids) return BFK_ERR_INVALID_ARGUMENT;
  bfk_status_t s = check_device();
  if (s != BFK_OK) return s;
  return cuda_status(launch_merge(cand_dists, cand_ids, n, lists, k, out_dists, out_ids,
                                  reinterpret_cast<cudaStream_t>(stream)));
}

static void fill_attrs(const cudaFuncAttributes &a, size_t dyn, int threads, bfk_attrs_t *out) {
  std::memset(out, 0, sizeof(*out));
  out->num_regs = a.numRegs;
  out->shared_size_bytes = (int32_t)a.sharedSizeBytes;
  out->dynamic_smem_bytes = (int32_t)dyn;
  out->local_size_bytes = (int32_t)a.localSizeBytes;
  out->const_size_bytes = (int32_t)a.constSizeBytes;
  out->max_threads_per_block = a.maxThreadsPerBlock;
  out->binary_version = a.binaryVersion;
  out->ptx_version = a.ptxVersion;
  out->block_threads = threads;
}

bfk_status_t bfk_merge_strided(const float *cand_dists, const int32_t *cand_ids, int64_t n,
                               int32_t lists, int64_t list_stride, int32_t k, float *out_dists,
                               int32_t *out_ids, void *stream) {
  if (n < 0 || lists <= 0 || k <= 0 || list_stride < n * k) return BFK_ERR_INVALID_ARGUMENT;
  if (k > merge_max_k()) return BFK_ERR_UNSUPPORTED;
  if (n == 0) return BFK_OK;
  if (!cand_dists || !cand_ids || !out_dists || !out_ids) return BFK_ERR_INVALID_ARGUMENT;
  bfk_status_t s = check_device();
  if (s != BFK_OK) return s;
  return cuda_status(launch_merge_strided(cand_dists, cand_ids, n, lists, k, list_stride,
                                          out_dists, out_ids,
                                          reinterpret_cast<cudaStream_t>(stream)));
}

bfk_status_t bfk_kernel_attrs(int32_t engine, int32_t d, int32_t k, bfk_attrs_t *out) {
  if (!out || d <= 0 || k <= 0) return BFK_ERR_INVALID_ARGUMENT;
  if (d > kMaxD || k > kMaxK) return BFK_ERR_UNSUPPORTED;
  const void *fn = nullptr;
  int threads = 256;
  size_t dyn = 0;
  if (engine == BFK_ENGINE_TC_F16) {
    if (!tc_supported(d, k)) return BFK_ERR_UNSUPPORTED;
    fn = tc_kernel_ptr(d, k);
    threads = tc_threads();
    dyn = tc_smem_bytes(d, k);
  } else if (engine == BFK_ENGINE_DIRECT || engine == BFK_ENGINE_AUTO) {
    const int tq = k <= 512 ? 4 : 1;
    fn = direct_kernel_ptr(tq);
    dyn = direct_smem_bytes(tq, k);
  } else {
    return BFK_ERR_INVALID_ARGUMENT;
  }
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, fn) != cudaSuccess) return BFK_ERR_CUDA;
  fill_attrs(a, dyn, threads, out);
  return BFK_OK;
}

bfk_status_t bfk_merge_attrs(int32_t lists, int32_t k, bfk_attrs_t *out) {
  if (!out || lists <= 0 || k <= 0) return BFK_ERR_INVALID_ARGUMENT;
  if (k > merge_max_k()) return BFK_ERR_UNSUPPORTED;
  size_t dyn = 0;
  const void *fn = merge_kernel_for(lists, k, &dyn);
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, fn) != cudaSuccess) return BFK_ERR_CUDA;
  fill_attrs(a, dyn, merge_threads(), out);
  return BFK_OK;
}

bfk_status_t bfk_search_stats(const void *workspace, int64_t n, int64_t m, int32_t d, int32_t k,
                              const bfk_opts_t *opts, void *stream, bfk_stats_t *out) {
  if (!workspace || !out || !opts_ok(opts)) return BFK_ERR_INVALID_ARGUMENT;
  bfk_status_t s = validate(n, m, d, k, 0);
  if (s != BFK_OK) return s;
  WsHeader h;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(&h, workspace, sizeof(h), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return BFK_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return BFK_ERR_CUDA;
  std::memset(out, 0, sizeof(*out));
  const int eng = choose_engine(n, m, d, k, opts);
  out->engine_used = eng;
  out->fallback_queries = h.fallback;
  out->candidates = (int64_t)h.candidates;
  out->max_query_candidates = h.max_cand;
  out->survivors = (int64_t)h.survivors;
  out->device_error = h.error;
  out->kernel_launches = g_calls.launches;
  float total = 0.f;
  int timed = 0;
  for (auto &pr : g_calls.pending) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, pr.first, pr.second) == cudaSuccess) {
      total += ms;
      timed++;
    }
    g_calls.spare.push_back(pr);
  }
  g_calls.pending.clear();
  out->timed_calls = timed;
  out->main_kernel_ms = total;
  if (eng == BFK_ENGINE_TC_F16) {
    TcPlan p;
    if (make_plan(n, m, d, k, opts, &p)) {
      out->slices = p.slices;
      out->cta_pair = p.pair ? 1 : 0;
    }
  } else {
    out->slices = direct_plan(n, m, d, k, opts ? opts->slices : 0).slices;
  }
  return BFK_OK;
}

}  // extern "C"
