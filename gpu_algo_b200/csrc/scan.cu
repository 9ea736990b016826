// Exact SIMT scan for small query batches (n <= 16): the database is read once,
// at HBM speed, by many independent warps.
//
// Reference behaviour followed (bf/fp32.py:53-92): every distance is
// dist = fma(q-x, q-x, dist) over dimensions in order; the k smallest per
// query are kept and emitted ascending by (distance, index).  With a handful of
// queries the work per row is tiny, so what matters is keeping enough loads in
// flight: each warp streams its own 32-row tiles (one row per lane), stages a
// 32-row x 32-dimension chunk transposed in warp-private shared memory with one
// load per row in flight at once, and keeps its own sorted top-k per query.
// No block-wide barrier is on the streaming path.  At the end the block merges
// its warps' lists by rank (binary searches) and writes one partial list per
// query; bfk_merge reduces the blocks' partials.
#include "common.cuh"
#include "internal.h"

namespace bfk {

constexpr int kScanWarps = 8;

// dist_step for two queries against one row value in packed FP32 instructions:
// (qa, qb) - (x, x) and fma(dif, dif, acc), each element rounded to nearest exactly
// as the scalar __fsub_rn / __fmaf_rn of dist_step.  q2 and acc2 hold the pairs
// packed (low word: the first query), x2 the row value twice.
__device__ __forceinline__ void dist_step2(unsigned long long q2, unsigned long long x2,
                                           unsigned long long &acc2) {
  unsigned long long dif;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(dif) : "l"(q2), "l"(x2));
  asm("fma.rn.f32x2 %0, %1, %1, %0;" : "+l"(acc2) : "l"(dif));
}
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(unsigned long long v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
constexpr int kScanPad = 33;  // transposed chunk row stride (conflict-free)

__host__ __device__ inline size_t scan_smem_bytes(int nq, int d, int k) {
  return sizeof(float) * ((size_t)d * nq +                      // queries, [d][nq]
                          (size_t)kScanWarps * 32 * kScanPad +   // per-warp chunks
                          (size_t)kScanWarps * nq * 32) +        // per-warp distances
         (size_t)kScanWarps * nq * 3 * sizeof(int32_t) +         // per-warp count, k-th
         (size_t)kScanWarps * nq * k * (sizeof(float) + sizeof(int32_t));  // per-warp lists
}

// grid (blocks), block 256.  Block b covers rows [b*slice_len, min((b+1)*slice_len, m))
// and writes its sorted top-k per query to out + b*n*k.
template <int NQ>
__global__ void __launch_bounds__(kScanWarps * 32) knn_scan_kernel(
    const float *__restrict__ Q, int n, const float *__restrict__ X, int64_t m, int d, int k,
    int64_t slice_len, int64_t id_offset, float *__restrict__ out_d, int32_t *__restrict__ out_i) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float *qs = reinterpret_cast<float *>(smem_raw);                 // [d][NQ]
  float *xt_all = qs + (size_t)d * NQ;                              // [warps][32][kScanPad]
  float *dist_all = xt_all + kScanWarps * 32 * kScanPad;            // [warps][NQ][32]
  int32_t *cnt_all = reinterpret_cast<int32_t *>(dist_all + kScanWarps * NQ * 32);  // [warps][NQ]
  float *kthd_all = reinterpret_cast<float *>(cnt_all + kScanWarps * NQ);          // [warps][NQ]
  int32_t *kthi_all = reinterpret_cast<int32_t *>(kthd_all + kScanWarps * NQ);     // [warps][NQ]
  float *lists_d = reinterpret_cast<float *>(kthi_all + kScanWarps * NQ);         // [warps][NQ][k]
  int32_t *lists_i = reinterpret_cast<int32_t *>(lists_d + kScanWarps * NQ * k);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float *xt = xt_all + warp * 32 * kScanPad;
  float *wdist = dist_all + warp * NQ * 32;
  int32_t *wcnt = cnt_all + warp * NQ;
  float *wkth_d = kthd_all + warp * NQ;
  int32_t *wkth_i = kthi_all + warp * NQ;
  float *wl_d = lists_d + warp * NQ * k;
  int32_t *wl_i = lists_i + warp * NQ * k;

  for (int e = threadIdx.x; e < d * NQ; e += blockDim.x) {
    const int c = e / NQ, qq = e % NQ;
    qs[e] = qq < n ? Q[(int64_t)qq * d + c] : 0.f;
  }
  __syncthreads();

  const int64_t rbeg = (int64_t)blockIdx.x * slice_len;
  const int64_t rend = rbeg + slice_len < m ? rbeg + slice_len : m;
  for (int i = lane; i < NQ; i += 32) { wcnt[i] = 0; wkth_d[i] = BFK_PAD_DIST; wkth_i[i] = -1; }
  __syncwarp();

  for (int64_t t = rbeg + (int64_t)warp * 32; t < rend; t += kScanWarps * 32) {
    float acc[NQ];
    unsigned long long acc2[NQ / 2 > 0 ? NQ / 2 : 1];
#pragma unroll
    for (int i = 0; i < NQ; i++) acc[i] = 0.f;
#pragma unroll
    for (int i = 0; i < NQ / 2; i++) acc2[i] = 0ull;  // two +0.0f
    const int64_t my_row = t + lane;
    for (int c0 = 0; c0 < d; c0 += 32) {
      // rows t .. t+31 of dimensions c0 .. c0+31, lane = dimension, all loads in flight
      float v[32];
      const bool cv = c0 + lane < d;
#pragma unroll
      for (int j = 0; j < 32; j++) {
        const int64_t row = t + j;
        v[j] = (cv && row < rend) ? __ldg(X + row * d + c0 + lane) : 0.f;
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 32; j++) xt[lane * kScanPad + j] = v[j];  // [dimension][row]
      __syncwarp();
      const int cw = d - c0 < 32 ? d - c0 : 32;
      for (int c = 0; c < cw; c++) {
        const float xv = xt[c * kScanPad + lane];
        const float *qc = qs + (size_t)(c0 + c) * NQ;
        if (NQ == 1) {
          acc[0] = dist_step(qc[0], xv, acc[0]);
        } else {
          // two queries per packed step (round to nearest per element, as dist_step)
          const unsigned long long x2 = pack2(xv, xv);
          const unsigned long long *qc2 = reinterpret_cast<const unsigned long long *>(qc);
#pragma unroll
          for (int i = 0; i < NQ / 2; i++) dist_step2(qc2[i], x2, acc2[i]);
        }
      }
    }
    if (NQ > 1) {
#pragma unroll
      for (int i = 0; i < NQ / 2; i++) unpack2(acc2[i], acc[2 * i], acc[2 * i + 1]);
    }
    // this lane's row against each query's running k-th (the distances go through
    // shared memory so that the loop over queries is not unrolled)
#pragma unroll
    for (int i = 0; i < NQ; i++) wdist[i * 32 + lane] = acc[i];
    __syncwarp();
    const int32_t gid = (int32_t)(id_offset + my_row);
    const bool row_ok = my_row < rend;
    for (int i = 0; i < n; i++) {
      float *ld = wl_d + i * k;
      int32_t *li = wl_i + i * k;
      const float dv = wdist[i * 32 + lane];
      int cnt = wcnt[i];
      float kd = wkth_d[i];
      int32_t ki = wkth_i[i];
      bool pass = row_ok && dv == dv && (cnt < k || pair_lt(dv, gid, kd, ki));
      unsigned mask = __ballot_sync(0xffffffffu, pass);
      if (!mask) continue;
      while (mask) {
        const int src = __ffs(mask) - 1;
        const float sd = __shfl_sync(0xffffffffu, dv, src);
        const int32_t sg = __shfl_sync(0xffffffffu, gid, src);
        warp_insert(ld, li, cnt, k, sd, sg, lane);
        if (cnt == k) { kd = ld[k - 1]; ki = li[k - 1]; }
        mask &= mask - 1;
        // the threshold may have dropped: re-test the remaining survivors
        pass = pass && (cnt < k || pair_lt(dv, gid, kd, ki));
        mask &= __ballot_sync(0xffffffffu, pass);
      }
      __syncwarp();
      if (lane == 0) { wcnt[i] = cnt; wkth_d[i] = kd; wkth_i[i] = ki; }
      __syncwarp();
    }
  }
  // pad each warp's lists to k
  for (int i = 0; i < NQ; i++) {
    for (int e = wcnt[i] + lane; e < k; e += 32) {
      wl_d[i * k + e] = BFK_PAD_DIST;
      wl_i[i * k + e] = -1;
    }
  }
  __syncthreads();

  // merge the warps' sorted lists per query by rank: an entry's place is its index in
  // its own list plus the entries before it in every other list (equal keys by warp)
  float *od = out_d + (int64_t)blockIdx.x * n * k;
  int32_t *oi = out_i + (int64_t)blockIdx.x * n * k;
  const int per_q = kScanWarps * k;
  for (int e = threadIdx.x; e < n * per_q; e += blockDim.x) {
    const int qq = e / per_q, r = e % per_q, w = r / k, j = r % k;
    const float *base_d = lists_d + qq * k;  // list of warp ww: base + ww * NQ * k
    const int32_t *base_i = lists_i + qq * k;
    const uint64_t key = pair_key(base_d[w * NQ * k + j], base_i[w * NQ * k + j]);
    int rank = j;
    for (int ww = 0; ww < kScanWarps && rank < k; ww++) {
      if (ww == w) continue;
      const float *ld = base_d + ww * NQ * k;
      const int32_t *li = base_i + ww * NQ * k;
      int lo = 0, hi = k;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        const uint64_t km = pair_key(ld[mid], li[mid]);
        if (ww < w ? km <= key : km < key) lo = mid + 1; else hi = mid;
      }
      rank += lo;
    }
    if (rank < k) {
      const bool pad = key == ~0ull;
      od[(int64_t)qq * k + rank] = pad ? BFK_PAD_DIST : base_d[w * NQ * k + j];
      oi[(int64_t)qq * k + rank] = pad ? -1 : base_i[w * NQ * k + j];
    }
  }
}

bool scan_supported(int64_t n, int d, int k) { return n >= 1 && n <= 16 && d <= 1024 && k <= 64; }

int scan_blocks(int64_t m, int k) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t b = 4LL * (sms > 0 ? sms : 148);
  const int64_t by_merge = 8192 / k;            // the merge of the partials stays one pass
  const int64_t by_rows = (m + 4095) / 4096;    // at least 4096 rows a block
  if (b > by_merge) b = by_merge;
  if (b > by_rows) b = by_rows;
  return b < 1 ? 1 : (int)b;
}

cudaError_t launch_scan(const float *Q, int64_t n, const float *X, int64_t m, int d, int k,
                        int64_t id_offset, int blocks, float *out_d, int32_t *out_i,
                        cudaStream_t stream) {
  const int nq = n <= 1 ? 1 : n <= 2 ? 2 : n <= 4 ? 4 : n <= 8 ? 8 : 16;
  const int64_t slice_len = (m + blocks - 1) / blocks;
  const size_t smem = scan_smem_bytes(nq, d, k);
  const void *fn = nq == 1 ? (const void *)knn_scan_kernel<1>
                 : nq == 2 ? (const void *)knn_scan_kernel<2>
                 : nq == 4 ? (const void *)knn_scan_kernel<4>
                 : nq == 8 ? (const void *)knn_scan_kernel<8>
                           : (const void *)knn_scan_kernel<16>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int ni = (int)n;
#define BFK_SCAN(NQ_)                                                                        \
  knn_scan_kernel<NQ_><<<(unsigned)blocks, kScanWarps * 32, smem, stream>>>(                 \
      Q, ni, X, m, d, k, slice_len, id_offset, out_d, out_i)
  switch (nq) {
    case 1: BFK_SCAN(1); break;
    case 2: BFK_SCAN(2); break;
    case 4: BFK_SCAN(4); break;
    case 8: BFK_SCAN(8); break;
    default: BFK_SCAN(16); break;
  }
#undef BFK_SCAN
  return cudaGetLastError();
}

}  // namespace bfk
