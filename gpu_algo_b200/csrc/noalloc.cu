// bfk_search_noalloc: the exact SIMT engine with its scratch memory in a
// fixed, library-owned device array instead of a caller-provided workspace.
//
// Some callers of this library cannot allocate device memory at search time:
// code that runs inside another allocator's callback, real-time threads that
// must not block on cudaMalloc's implicit synchronisation, or hosts that hand
// out only fixed, pre-registered buffers for inputs and outputs.  This entry
// point serves them.  It keeps its scratch (the per-slice partial top-k lists)
// in `g_noalloc_scratch`, a file-scope device array of kNoAllocScratchBytes
// that every GPU loading the library holds until the process exits.  It calls
// no cudaMalloc, cudaFree or allocating library routine.
#include <atomic>
#include <cstring>

#include "../../include/bfknn.h"
#include "common.cuh"
#include "internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB per device
constexpr int kMaxDevices = 64;
// one entry of a partial list: a float distance and an int32 id
constexpr size_t kEntryBytes = sizeof(float) + sizeof(int32_t);

// The partial lists of every slice: all distances, then all ids.  Shared by every
// call: calls that overlap on the GPU (different streams or threads) race on it.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device, looked up once per device.
std::atomic<void *> g_scratch_addr[kMaxDevices];

// The symbol's host-side name is only a stand-in: the kernel needs the device
// address, which cudaGetSymbolAddress returns for the current device.
void *scratch_address(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  void *p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (p) return p;
  void *addr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
  if (e != cudaSuccess || !addr) {
    BFK_NOTE(e == cudaSuccess ? cudaErrorInvalidSymbol : e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    return nullptr;
  }
  g_scratch_addr[dev].store(addr, std::memory_order_release);
  return addr;
}

}  // namespace

extern "C" BFK_API bfk_status_t bfk_search_noalloc(const float *Q, int64_t n, const float *X,
                                                   int64_t m, int32_t d, int32_t k,
                                                   int64_t id_offset, float *out_dists,
                                                   int32_t *out_ids, void *stream_) {
  using namespace bfk;
  if (n < 0 || m < 0 || d <= 0 || k <= 0) return BFK_ERR_INVALID_ARGUMENT;
  if (d > 4096 || k > 1024 || n > INT32_MAX || id_offset < 0 ||
      id_offset + m > (int64_t)INT32_MAX)
    return BFK_ERR_UNSUPPORTED;
  // two slices of partial lists must fit in the scratch: 2 * n * k entries; the
  // comparison is a division, so no product here can wrap
  const int64_t max_nk = (int64_t)(kNoAllocScratchBytes / (2 * kEntryBytes));
  if (n > max_nk / k) return BFK_ERR_UNSUPPORTED;
  if (n == 0) return BFK_OK;
  if (!Q || !out_dists || !out_ids || (m > 0 && !X)) return BFK_ERR_INVALID_ARGUMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BFK_ERR_NO_DEVICE;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      major != 10)
    return BFK_ERR_NO_DEVICE;
  unsigned char *scratch = static_cast<unsigned char *>(scratch_address(dev));
  if (!scratch) return BFK_ERR_CUDA;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  cudaError_t e;
  if (m == 0) {
    e = launch_fill_pad(out_dists, out_ids, n * k, stream);
    if (e != cudaSuccess) { BFK_NOTE(e, "fill"); return BFK_ERR_CUDA; }
    return BFK_OK;
  }
  // Every slice's kernel writes all n * k entries of its partial list before the
  // merge reads them, so nothing left in the scratch by an earlier call is read.
  // As many database slices as the scratch holds (and as help to fill the GPU).
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t per_slice = (size_t)n * (size_t)k * kEntryBytes;  // <= 8 MiB by the check above
  const int tq = (n >= 64 && k <= 512) ? 4 : 1;
  const int64_t qblocks = (n + 8 * tq - 1) / (8 * tq);
  int64_t slices = (3LL * sms + qblocks - 1) / qblocks;
  const int64_t fit = (int64_t)(kNoAllocScratchBytes / per_slice);
  if (slices > fit) slices = fit;
  if (slices > (m + 1023) / 1024) slices = (m + 1023) / 1024;
  if (slices < 2) slices = 2;  // the variant always goes through the scratch lists
  float *pd = reinterpret_cast<float *>(scratch);
  int32_t *pi = reinterpret_cast<int32_t *>(scratch + (size_t)slices * n * k * sizeof(float));
  e = launch_direct(Q, n, X, m, d, k, id_offset, (int)slices, tq, pd, pi, stream);
  if (e != cudaSuccess) { BFK_NOTE(e, "direct"); return BFK_ERR_CUDA; }
  e = launch_merge(pd, pi, n, (int)slices, k, out_dists, out_ids, stream);
  if (e != cudaSuccess) { BFK_NOTE(e, "merge"); return BFK_ERR_CUDA; }
  return BFK_OK;
}
