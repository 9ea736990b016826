// Exact SIMT engine: direct-difference distances with a fused per-query top-k.
//
// Reference behaviour followed (bf/fp32.py:53-92, bf/fp32_qgroup.py:37-146):
// every distance is dist = fma(q-x, q-x, dist) over dimensions in order, the k
// smallest per query are kept and emitted ascending.  Differences from the
// reference's structure (not its results): a block holds QB = 8*TQ queries
// (the reference's QPB idea), each database tile of 128 rows x 32 dims is
// staged once in shared memory and reused by every query of the block, each
// thread keeps a TQ x 4 register tile of partial distances, and each warp
// keeps the sorted top-k of its own TQ queries in shared memory, inserting
// survivors warp-cooperatively instead of the reference's thread-0 serial merge
// (bf/fp32.py:85-91).
#include "common.cuh"
#include "internal.h"

namespace bfk {

constexpr int kDirRT = 128;  // database rows per tile
constexpr int kDirDC = 32;   // dimensions per chunk

// One block's work: queries [qb0, qb0 + QB) against rows [rbeg, rend), the sorted top-k of
// each written to (out_d, out_i) (n, k).
template <int TQ>
__device__ __forceinline__ void direct_block(const float *__restrict__ Q, int64_t n,
                                             const float *__restrict__ X, int d, int k,
                                             int64_t qb0, int64_t rbeg, int64_t rend,
                                             int64_t id_offset, float *out_d, int32_t *out_i,
                                             unsigned char *smem_raw) {
  constexpr int QB = 8 * TQ;
  float *xs = reinterpret_cast<float *>(smem_raw);          // [kDirRT][kDirDC + 1]
  float *qs = xs + kDirRT * (kDirDC + 1);                    // [kDirDC][QB]
  float *lists_d = qs + kDirDC * QB;                         // [QB][k]
  int32_t *lists_i = reinterpret_cast<int32_t *>(lists_d + QB * k);  // [QB][k]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  int cnt[TQ];
  float kth_d[TQ];
  int32_t kth_i[TQ];
#pragma unroll
  for (int i = 0; i < TQ; i++) { cnt[i] = 0; kth_d[i] = BFK_PAD_DIST; kth_i[i] = -1; }

  for (int64_t r0 = rbeg; r0 < rend; r0 += kDirRT) {
    float acc[TQ][4];
#pragma unroll
    for (int i = 0; i < TQ; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) acc[i][j] = 0.f;

    for (int c0 = 0; c0 < d; c0 += kDirDC) {
      __syncthreads();
      const bool cv = c0 + lane < d;
#pragma unroll 4
      for (int rr = warp; rr < kDirRT; rr += 8) {
        int64_t row = r0 + rr;
        float v = 0.f;
        if (cv && row < rend) v = __ldg(X + row * d + c0 + lane);
        xs[rr * (kDirDC + 1) + lane] = v;
      }
#pragma unroll
      for (int qq = warp; qq < QB; qq += 8) {
        int64_t qi = qb0 + qq;
        float v = 0.f;
        if (cv && qi < n) v = __ldg(Q + qi * d + c0 + lane);
        qs[lane * QB + qq] = v;
      }
      __syncthreads();
      // padded dimensions hold 0 in both q and x, so they add exactly nothing
#pragma unroll 8
      for (int c = 0; c < kDirDC; c++) {
        float xv[4];
#pragma unroll
        for (int j = 0; j < 4; j++) xv[j] = xs[(lane + 32 * j) * (kDirDC + 1) + c];
        float qv[TQ];
#pragma unroll
        for (int i = 0; i < TQ; i++) qv[i] = qs[c * QB + warp * TQ + i];
#pragma unroll
        for (int i = 0; i < TQ; i++)
#pragma unroll
          for (int j = 0; j < 4; j++) acc[i][j] = dist_step(qv[i], xv[j], acc[i][j]);
      }
    }

    // selection: this warp owns queries warp*TQ + i; lane holds rows r0 + lane + 32j
#pragma unroll
    for (int i = 0; i < TQ; i++) {
      const int ql = warp * TQ + i;
      if (qb0 + ql >= n) continue;
      float *ld = lists_d + ql * k;
      int32_t *li = lists_i + ql * k;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int64_t row = r0 + lane + 32 * j;
        const float dv = acc[i][j];
        const int32_t gid = (int32_t)(id_offset + row);
        const bool valid = row < rend && dv == dv;
        bool pass = valid && (cnt[i] < k || pair_lt(dv, gid, kth_d[i], kth_i[i]));
        unsigned mask = __ballot_sync(0xffffffffu, pass);
        while (mask) {
          const int src = __ffs(mask) - 1;
          const float sd = __shfl_sync(0xffffffffu, dv, src);
          const int32_t sg = __shfl_sync(0xffffffffu, gid, src);
          warp_insert(ld, li, cnt[i], k, sd, sg, lane);
          if (cnt[i] == k) { kth_d[i] = ld[k - 1]; kth_i[i] = li[k - 1]; }
          mask &= mask - 1;
          // the threshold may have dropped: re-test the remaining survivors
          pass = pass && (cnt[i] < k || pair_lt(dv, gid, kth_d[i], kth_i[i]));
          mask &= __ballot_sync(0xffffffffu, pass);
        }
      }
    }
  }

  // emit
  __syncwarp();
#pragma unroll
  for (int i = 0; i < TQ; i++) {
    const int ql = warp * TQ + i;
    const int64_t qi = qb0 + ql;
    if (qi >= n) continue;
    const float *ld = lists_d + ql * k;
    const int32_t *li = lists_i + ql * k;
    float *od = out_d + qi * k;
    int32_t *oi = out_i + qi * k;
    for (int e = lane; e < k; e += 32) {
      const bool have = e < cnt[i];
      od[e] = have ? ld[e] : BFK_PAD_DIST;
      oi[e] = have ? li[e] : -1;
    }
  }
}

// grid (ceil(n / QB), slices); block 256 threads.
// Slice s covers rows [s*slice_len, min((s+1)*slice_len, m)).  With one slice
// the sorted top-k goes to (out_d, out_i) (n, k); with more, slice s writes
// its sorted list to out + s*n*k for a later merge.
template <int TQ>
__global__ void __launch_bounds__(256) knn_direct_kernel(const float *__restrict__ Q, int64_t n,
                                                         const float *__restrict__ X, int64_t m,
                                                         int d, int k, int64_t slice_len,
                                                         int64_t id_offset, float *out_d,
                                                         int32_t *out_i) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int64_t rbeg = (int64_t)blockIdx.y * slice_len;
  const int64_t rend = rbeg + slice_len < m ? rbeg + slice_len : m;
  const int64_t off = gridDim.y > 1 ? (int64_t)blockIdx.y * n * k : 0;
  direct_block<TQ>(Q, n, X, d, k, (int64_t)blockIdx.x * (8 * TQ), rbeg, rend, id_offset,
                   out_d + off, out_i + off, smem_raw);
}

// The same search for a query count known only on the device (*count): the exact
// fallback of the tensor-core engine, launched whether or not any query needs it, so
// the host never waits for the count.  Runs only when lo <= *count < hi (one launch
// per block shape).  The (query block, slice) items are taken grid-stride; the slice
// count is fallback_slices(*count, ...), and slice s writes its sorted lists to
// out + s * count * k.
template <int TQ>
__global__ void __launch_bounds__(256) knn_direct_count_kernel(
    const float *__restrict__ Q, const int *__restrict__ count, int lo, int hi,
    const float *__restrict__ X, int64_t m, int d, int k, int64_t id_offset,
    int64_t part_entries, float *out_d, int32_t *out_i) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int64_t n = *count;
  if (n < lo || n >= hi || n == 0) return;
  constexpr int QB = 8 * TQ;
  const int64_t slices = fallback_slices(n, m, k, part_entries);
  const int64_t slice_len = ((m + slices - 1) / slices + kDirRT - 1) / kDirRT * kDirRT;
  const int64_t qblocks = (n + QB - 1) / QB;
  for (int64_t item = blockIdx.x; item < qblocks * slices; item += gridDim.x) {
    const int64_t qb = item / slices, sl = item - qb * slices;
    const int64_t rbeg = sl * slice_len;
    const int64_t rend = rbeg + slice_len < m ? rbeg + slice_len : m;
    __syncthreads();  // the previous item's lists are no longer read
    direct_block<TQ>(Q, n, X, d, k, qb * QB, rbeg, rend, id_offset, out_d + sl * n * k,
                     out_i + sl * n * k, smem_raw);
  }
}

size_t direct_smem_bytes(int tq, int k) {
  const int qb = 8 * tq;
  return sizeof(float) * ((size_t)kDirRT * (kDirDC + 1) + (size_t)kDirDC * qb) +
         (size_t)qb * k * (sizeof(float) + sizeof(int32_t));
}

const void *direct_kernel_ptr(int tq) {
  return tq >= 4 ? (const void *)knn_direct_kernel<4> : (const void *)knn_direct_kernel<1>;
}

cudaError_t launch_direct_count(const float *Q, const int *count, const float *X, int64_t m,
                                int d, int k, int64_t id_offset, int64_t part_entries,
                                float *out_d, int32_t *out_i, cudaStream_t stream) {
  // few queries: 8 per block; many: 32 per block
  const int grid = 2 * 148;
  for (int tq : {1, 4}) {
    const size_t smem = direct_smem_bytes(tq, k);
    const void *fn = tq == 4 ? (const void *)knn_direct_count_kernel<4>
                             : (const void *)knn_direct_count_kernel<1>;
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (tq == 4)
      knn_direct_count_kernel<4><<<grid, 256, smem, stream>>>(Q, count, 64, 0x7fffffff, X, m, d, k,
                                                              id_offset, part_entries, out_d, out_i);
    else
      knn_direct_count_kernel<1><<<grid, 256, smem, stream>>>(Q, count, 1, 64, X, m, d, k,
                                                              id_offset, part_entries, out_d, out_i);
  }
  return cudaGetLastError();
}

cudaError_t launch_direct(const float *Q, int64_t n, const float *X, int64_t m, int d, int k,
                          int64_t id_offset, int slices, int tq, float *out_d, int32_t *out_i,
                          cudaStream_t stream) {
  const int qb = 8 * tq;
  const int64_t slice_len =
      ((m + slices - 1) / slices + kDirRT - 1) / kDirRT * kDirRT;  // tile-aligned
  const size_t smem = direct_smem_bytes(tq, k);
  const void *fn = direct_kernel_ptr(tq);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((n + qb - 1) / qb), (unsigned)slices);
  if (tq >= 4)
    knn_direct_kernel<4><<<grid, 256, smem, stream>>>(Q, n, X, m, d, k, slice_len, id_offset,
                                                      out_d, out_i);
  else
    knn_direct_kernel<1><<<grid, 256, smem, stream>>>(Q, n, X, m, d, k, slice_len, id_offset,
                                                      out_d, out_i);
  return cudaGetLastError();
}

}  // namespace bfk
