// k-way merge of sorted candidate lists (per query) into the k best by
// (distance, index).  Replaces bf_fp32_tiled_merge (bf/fp32_tiled.py:118-178)
// and bf_fp32_qgroup_merge (bf/fp32_qgroup.py:153-213), which re-insert every
// partial through a per-thread heap and a thread-0 serial merge; here one
// block per query sorts 64-bit (distance, index) keys with a shared-memory
// bitonic network, taking the lists in groups so any number of lists fits.
#include "common.cuh"
#include "internal.h"

namespace bfk {

constexpr int kMergeThreads = 256;
constexpr int kMergeCap = 8192;  // keys sorted at once (64 KB of shared memory)
constexpr int kRankMergeLists = 16;  // more lists: the bitonic path is cheaper

__device__ void block_bitonic_sort(uint64_t *keys, int P) {
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int t = threadIdx.x; t < P / 2; t += blockDim.x) {
        int lo = 2 * stride * (t / stride) + (t % stride);
        int hi = lo + stride;
        bool up = ((lo & size) == 0);
        uint64_t a = keys[lo], b = keys[hi];
        if ((a > b) == up) { keys[lo] = b; keys[hi] = a; }
      }
    }
  }
  __syncthreads();
}

// The k best of query qi's `lists` sorted lists (list l at cand + l * stride + qi * k) into
// (od, oi) (k entries), by one block: the lists are taken in groups so that any number
// fits in kMergeCap keys, each group sorted with the survivors of the previous ones.
__device__ void merge_block(const float *__restrict__ cand_d, const int32_t *__restrict__ cand_i,
                            int64_t qi, int lists, int k, int64_t stride, float *od, int32_t *oi,
                            uint64_t *keys) {
  const int group = (kMergeCap - k) / k;  // lists added per round (>= 1 since k <= kMergeCap/2)
  int have = 0;                           // keys carried from the previous round (sorted)
  for (int l0 = 0; l0 < lists; l0 += group) {
    const int l1 = l0 + group < lists ? l0 + group : lists;
    const int total = have + (l1 - l0) * k;
    int P = 1;
    while (P < total) P <<= 1;
    for (int e = threadIdx.x; e < P - have; e += blockDim.x) {
      uint64_t key = ~0ull;
      if (e < (l1 - l0) * k) {
        const int l = l0 + e / k, j = e % k;
        const int64_t off = (int64_t)l * stride + qi * k + j;
        key = pair_key(cand_d[off], cand_i[off]);
      }
      keys[have + e] = key;
    }
    block_bitonic_sort(keys, P);
    have = k;
  }
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const uint64_t key = keys[j];
    const bool pad = key == ~0ull;
    od[j] = pad ? BFK_PAD_DIST : ord2f((uint32_t)(key >> 32));
    oi[j] = pad ? -1 : (int32_t)(uint32_t)(key & 0xffffffffu);
  }
  __syncthreads();  // the keys are reused by the block's next query
}

// grid (n), block kMergeThreads, dynamic smem kMergeCap * 8.
// cand: list l's (n, k) block starts `stride` elements after list l-1's -> out (n, k)
__global__ void __launch_bounds__(kMergeThreads) knn_merge_kernel(
    const float *__restrict__ cand_d, const int32_t *__restrict__ cand_i, int64_t n, int lists,
    int k, int64_t stride, float *__restrict__ out_d, int32_t *__restrict__ out_i) {
  extern __shared__ __align__(16) uint64_t keys[];
  const int64_t qi = blockIdx.x;
  merge_block(cand_d, cand_i, qi, lists, k, stride, out_d + qi * k, out_i + qi * k, keys);
}

// The exact fallback's merge, for a query count known only on the device (*count):
// the partial lists of fallback_slices(*count, ...) slices, laid out with stride
// count * k, merged per query (grid-stride over the queries) and written to the row of
// the output that list[q] names.
__global__ void __launch_bounds__(kMergeThreads) knn_merge_count_kernel(
    const float *__restrict__ cand_d, const int32_t *__restrict__ cand_i,
    const int *__restrict__ count, int64_t m, int k, int64_t part_entries,
    const int *__restrict__ list, float *__restrict__ out_d, int32_t *__restrict__ out_i) {
  extern __shared__ __align__(16) uint64_t keys[];
  const int64_t n = *count;
  if (n == 0) return;
  const int lists = (int)fallback_slices(n, m, k, part_entries);
  for (int64_t qi = blockIdx.x; qi < n; qi += gridDim.x) {
    const int64_t row = list[qi];
    merge_block(cand_d, cand_i, qi, lists, k, n * k, out_d + row * k, out_i + row * k, keys);
  }
}

// Merge by rank, for up to kRankMergeLists lists and lists * k <= kMergeCap: every key's place in the merged order
// is its index in its own list plus, in every other list, the number of keys
// before it (binary searches; equal keys order by list), so one pass places
// each of the first k keys without a sort.  grid (n), dynamic smem lists*k*8.
__global__ void __launch_bounds__(kMergeThreads) knn_merge_rank_kernel(
    const float *__restrict__ cand_d, const int32_t *__restrict__ cand_i, int64_t n, int lists,
    int k, int64_t stride, float *__restrict__ out_d, int32_t *__restrict__ out_i) {
  extern __shared__ __align__(16) uint64_t keys[];
  const int64_t qi = blockIdx.x;
  const int total = lists * k;
  for (int e = threadIdx.x; e < total; e += blockDim.x) {
    const int l = e / k, j = e - l * k;
    const int64_t off = (int64_t)l * stride + qi * k + j;
    keys[e] = pair_key(cand_d[off], cand_i[off]);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < total; e += blockDim.x) {
    const int l = e / k;
    int rank = e - l * k;
    const uint64_t key = keys[e];
    for (int o = 0; o < lists && rank < k; o++) {
      if (o == l) continue;
      // keys of list o before this one: < key, or <= key for a list that comes first
      const uint64_t *b = keys + o * k;
      int lo = 0, hi = k;
      if (o < l) {
        while (lo < hi) { const int mid = (lo + hi) >> 1; if (b[mid] <= key) lo = mid + 1; else hi = mid; }
      } else {
        while (lo < hi) { const int mid = (lo + hi) >> 1; if (b[mid] < key) lo = mid + 1; else hi = mid; }
      }
      rank += lo;
    }
    if (rank < k) {
      const bool pad = key == ~0ull;
      out_d[qi * k + rank] = pad ? BFK_PAD_DIST : ord2f((uint32_t)(key >> 32));
      out_i[qi * k + rank] = pad ? -1 : (int32_t)(uint32_t)(key & 0xffffffffu);
    }
  }
}

cudaError_t launch_merge(const float *cand_d, const int32_t *cand_i, int64_t n, int lists, int k,
                         float *out_d, int32_t *out_i, cudaStream_t stream) {
  return launch_merge_strided(cand_d, cand_i, n, lists, k, n * k, out_d, out_i, stream);
}

cudaError_t launch_merge_strided(const float *cand_d, const int32_t *cand_i, int64_t n, int lists,
                                 int k, int64_t stride, float *out_d, int32_t *out_i,
                                 cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  // by rank for a few lists (each key binary-searches every other list); sorting for many
  if (lists <= kRankMergeLists && (int64_t)lists * k <= kMergeCap) {
    const size_t rsmem = (size_t)lists * k * sizeof(uint64_t);
    cudaError_t e = cudaFuncSetAttribute((const void *)knn_merge_rank_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)(kMergeCap * sizeof(uint64_t)));
    if (e != cudaSuccess) return e;
    knn_merge_rank_kernel<<<(unsigned)n, kMergeThreads, rsmem, stream>>>(cand_d, cand_i, n, lists,
                                                                          k, stride, out_d, out_i);
    return cudaGetLastError();
  }
  const size_t smem = (size_t)kMergeCap * sizeof(uint64_t);
  cudaError_t e = cudaFuncSetAttribute((const void *)knn_merge_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  knn_merge_kernel<<<(unsigned)n, kMergeThreads, smem, stream>>>(cand_d, cand_i, n, lists, k,
                                                                 stride, out_d, out_i);
  return cudaGetLastError();
}

int merge_max_k() { return kMergeCap / 2; }

cudaError_t launch_merge_count(const float *cand_d, const int32_t *cand_i, const int *count,
                               int64_t m, int k, int64_t part_entries, const int *list,
                               float *out_d, int32_t *out_i, cudaStream_t stream) {
  const size_t smem = (size_t)kMergeCap * sizeof(uint64_t);
  cudaError_t e = cudaFuncSetAttribute((const void *)knn_merge_count_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  knn_merge_count_kernel<<<2 * 148, kMergeThreads, smem, stream>>>(
      cand_d, cand_i, count, m, k, part_entries, list, out_d, out_i);
  return cudaGetLastError();
}

const void *merge_kernel_for(int lists, int k, size_t *smem) {
  if (lists <= kRankMergeLists && (int64_t)lists * k <= kMergeCap) {
    *smem = (size_t)lists * k * sizeof(uint64_t);
    return (const void *)knn_merge_rank_kernel;
  }
  *smem = (size_t)kMergeCap * sizeof(uint64_t);
  return (const void *)knn_merge_kernel;
}

int merge_threads() { return kMergeThreads; }

__global__ void fill_pad_kernel(float *out_d, int32_t *out_i, int64_t count) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < count;
       e += (int64_t)gridDim.x * blockDim.x) {
    out_d[e] = BFK_PAD_DIST;
    out_i[e] = -1;
  }
}

cudaError_t launch_fill_pad(float *out_d, int32_t *out_i, int64_t count, cudaStream_t stream) {
  if (count == 0) return cudaSuccess;
  int64_t blocks = (count + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  fill_pad_kernel<<<(unsigned)blocks, 256, 0, stream>>>(out_d, out_i, count);
  return cudaGetLastError();
}

}  // namespace bfk
