// Tensor-core engine: tcgen05 f16 distance filter passes under sampled
// per-query thresholds, then an exact FP32 re-rank of the few survivors.
//
// Pass 0 (prep): queries and database rows are scaled by powers of two and
//   rounded to f16 (rows in 64-row groups sharing one scale), with their FP32
//   squared norms, the largest f16 rounding error of a row and each query's, and
//   a per-query error margin m, a bound on |approximate distance - reference
//   distance| (derived in tc_prep_q_kernel).
// Filter passes (one CTA, or a CTA pair, per (query tile, slice of a tile set)):
//   TMA streams f16 row tiles (256 rows x 64 dims, 128-byte swizzle) into a
//   shared-memory ring; tcgen05.mma (M = 128 queries, or 256 over a CTA pair;
//   N = 256 rows; K = 16) accumulates into a double-buffered FP32 accumulator in
//   tensor memory, issued by two threads on alternate tiles when a tile is at
//   most two K chunks; sixteen epilogue warps (four per TMEM lane quarter, one
//   per 64-column group) read it with tcgen05.ld, one query per thread.  A
//   16-column chunk whose largest accumulator is at most a threshold T (in the
//   accumulator's units) holds no candidate; the others get their exact
//       v = ||x||^2 - 2 q.x     (approximate distance - ||q||^2)
//   and rows with v <= theta_q are appended to the query's candidate region
//   (plain stores into a per-(query, slice, column group) region: no atomics).
// Levels: the tile sets grow geometrically: level 0 is a handful of evenly
//   spaced tiles with theta = +inf; after each level a select pass sets
//   R_q = k-th smallest v among the level's candidates and the next level uses
//   theta_q = R_q + 2m.  R_q is the k-th smallest v over a set of real rows, so
//   ||q||^2 + R_q + m bounds the k-th reference distance from above and no true
//   neighbour is dropped.  The last level is every tile; the sample levels
//   cost about 1/ratio of it.
// Final select: R* = k-th smallest v among the last level's candidates; rows
//   with v <= R* + 2m are re-ranked with the reference arithmetic
//   (dif = q - x; acc = fma(dif, dif, acc), bf/fp32.py:80) and the k best by
//   (distance, index) are written, so output distances are bit-identical to
//   the reference kernels'.  A query whose final candidate region overflowed
//   (degenerate data) is finished by the exact SIMT engine, and so is every
//   query when the inputs hold a non-finite norm or norms too small for the
//   margin or too large for FP32 (qn + Rx outside [2^-48, 2^63), see
//   tc_prep_q_kernel).  The count of such queries stays on the device: the
//   fallback kernels always run and read it, so the host never waits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cfloat>
#include <cstring>
#include <cmath>

#include "common.cuh"
#include "internal.h"

namespace bfk {

constexpr int kBM = 128;            // queries per tile (MMA M, TMEM lanes)
constexpr int kBN = 256;            // rows per tile (MMA N, accumulator columns)
constexpr int kBK = 64;             // f16 elements per K chunk (128 bytes, one swizzle atom row)
constexpr int kAChunkBytes = kBM * kBK * 2;   // 16 KB
constexpr int kBChunkBytes = kBN * kBK * 2;   // 32 KB
constexpr int kEpiWarps = 16;       // four warps per TMEM lane quarter, one per 64-column group
constexpr int kColGroups = 4;       // column groups of a tile (regions per slice)
constexpr int kGroupN = kBN / kColGroups;  // accumulator columns an epilogue warp reads per tile
// warp 0 TMA, warps 1 and kIssuerWarp2 MMA (alternate tiles), warps 2 .. 17 epilogue
constexpr int kIssuerWarp2 = 2 + kEpiWarps;
constexpr int kTcThreads = 32 * (kIssuerWarp2 + 1);
constexpr int kSmemLimit = 232448;  // 227 KB opt-in per block
constexpr int kResidentKch = 4;     // d <= 256: the query tile stays in shared memory
constexpr int kMaxKch = 16;         // d <= 1024: query K chunks stream with the row chunks
constexpr int kTcMaxK = 512;
constexpr int kSelThreads = 256;
constexpr int kSurvCap = 2048;      // exact re-rank capacity per query
constexpr int kRankSortMax = 512;   // survivors ordered by rank counting up to this many
constexpr int kDefaultPool = 16384;  // candidate entries per query (all regions of a level)
constexpr int kLevelTarget = 3072;   // expected candidates per query of a filter level
constexpr int kMinLevelTarget = 256;

struct FilterArgs {
  const float *xnorm;    // (x_tiles*256) ||x||^2, +inf past m
  const float4 *xmeta;   // (x_tiles * 4) groups of 64 rows, two float4 each: the minimum
                         // ||x||^2 of each 16-row chunk, then (1/scale, scale, 0, 0)
  const float2 *qinfo;   // (q_tiles*128) (||q||^2, 2*margin); NaN margin for padding rows
  const float *inv_sq;   // 1/scale of the queries (device scalar)
  const float *r_in;     // (n) bound B of the previous level (B + margin), null = none
  bool two_bounds;       // r_in holds (n) B and (n) -B2 (shards sharing bounds)
  int64_t n;
  int64_t x_tiles;       // tiles of the whole database
  int64_t level_tiles;   // tiles of this level (evenly spaced over the database)
  int q_tiles, slices, tiles_per_slice;
  int region;            // entries per (query, slice, column group) region
  int pool;              // entries per query
  int max_slices;        // count array stride / kColGroups
  uint2 *cand;           // (n, pool) (row, v bits)
  int *ccount;           // (n, kColGroups * max_slices)
  WsHeader *hdr;
};

// ---------------------------------------------------------------------------
// shared-memory layout of the filter kernel
// ---------------------------------------------------------------------------
// per epilogue warp and accumulator buffer: the group's 64 ||x||^2 values and the
// minimum of each group of 8 of them
constexpr int kNxStage = kGroupN + 8;

struct TcLayout {
  int kch, ns;
  bool stream_a;    // the query tile's K chunks travel through the stages with the rows'
  uint32_t bchunk;  // bytes of one row-tile K chunk in this CTA (half of it in a CTA pair)
  uint32_t stage;   // bytes of one stage: [query chunk if stream_a] + row chunk
  size_t a_off, b_off, nx_off, bar_off, total;
};
__host__ __device__ inline TcLayout tc_layout(int kch, bool pair) {
  TcLayout L{};
  L.kch = kch;
  L.stream_a = kch > kResidentKch;
  L.bchunk = pair ? kBChunkBytes / 2 : kBChunkBytes;
  L.stage = L.bchunk + (L.stream_a ? kAChunkBytes : 0);
  L.a_off = 0;
  L.b_off = L.stream_a ? 0 : (size_t)kch * kAChunkBytes;
  const size_t fixed = (size_t)kEpiWarps * 2 * kNxStage * 4 + 256;
  size_t ns = ((size_t)kSmemLimit - 1024 - L.b_off - fixed) / L.stage;
  if (ns > 12) ns = 12;
  L.ns = (int)ns;
  L.nx_off = L.b_off + (size_t)L.ns * L.stage;
  L.bar_off = L.nx_off + (size_t)kEpiWarps * 2 * kNxStage * 4;
  L.total = L.bar_off + 256 + 1024;  // + alignment slack
  return L;
}

__device__ __forceinline__ void set_error(WsHeader *h, int code, volatile int *abort_flag) {
  atomicCAS(&h->error, 0, code);
  *abort_flag = 1;
}


// (a0, a1) * c + (b0, b1) in one packed FP32 instruction (round to nearest)
__device__ __forceinline__ void fma2(float a0, float a1, float c, float b0, float b1, float &d0,
                                     float &d1) {
  unsigned long long pa, pc, pb, pd;
  asm("mov.b64 %0, {%1, %2};" : "=l"(pa) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(pc) : "f"(c));
  asm("mov.b64 %0, {%1, %2};" : "=l"(pb) : "f"(b0), "f"(b1));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(pd) : "l"(pa), "l"(pc), "l"(pb));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(pd));
}
// three-input minimum / maximum (NaN inputs are ignored, as by fminf / fmaxf)
__device__ __forceinline__ float min3f(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// v[i] for a lane-varying i in [0, 16), by selects (no local-memory indexing)
__device__ __forceinline__ float pick16(const float *v, int i) {
  const bool b0 = i & 1, b1 = i & 2, b2 = i & 4, b3 = i & 8;
  float s[8], t[4], u[2];
#pragma unroll
  for (int j = 0; j < 8; j++) s[j] = b0 ? v[2 * j + 1] : v[2 * j];
#pragma unroll
  for (int j = 0; j < 4; j++) t[j] = b1 ? s[2 * j + 1] : s[2 * j];
  u[0] = b2 ? t[1] : t[0];
  u[1] = b2 ? t[3] : t[2];
  return b3 ? u[1] : u[0];
}
// maximum of 16 accumulator values (FP32 bit patterns), three-input max.f32
__device__ __forceinline__ float max16u(const uint32_t *a) {
  const float m0 = max3f(__uint_as_float(a[0]), __uint_as_float(a[1]), __uint_as_float(a[2]));
  const float m1 = max3f(__uint_as_float(a[3]), __uint_as_float(a[4]), __uint_as_float(a[5]));
  const float m2 = max3f(__uint_as_float(a[6]), __uint_as_float(a[7]), __uint_as_float(a[8]));
  const float m3 = max3f(__uint_as_float(a[9]), __uint_as_float(a[10]), __uint_as_float(a[11]));
  const float m4 = max3f(__uint_as_float(a[12]), __uint_as_float(a[13]), __uint_as_float(a[14]));
  return fmaxf(max3f(m0, m1, m2), max3f(m3, m4, __uint_as_float(a[15])));
}
// the filter values of 8 columns: v = fma(c, acc, ||x||^2), one rounding each
__device__ __forceinline__ void exact_v8(const uint32_t *acc, float c, float4 n0, float4 n1,
                                         float *v) {
  fma2(__uint_as_float(acc[0]), __uint_as_float(acc[1]), c, n0.x, n0.y, v[0], v[1]);
  fma2(__uint_as_float(acc[2]), __uint_as_float(acc[3]), c, n0.z, n0.w, v[2], v[3]);
  fma2(__uint_as_float(acc[4]), __uint_as_float(acc[5]), c, n1.x, n1.y, v[4], v[5]);
  fma2(__uint_as_float(acc[6]), __uint_as_float(acc[7]), c, n1.z, n1.w, v[6], v[7]);
}

// the bound a level select wrote for query q (both halves when the shards share them)
__device__ __forceinline__ float read_bound(const float *r, int64_t n, int64_t q, bool two) {
  const float b = r[q];
  return two ? fminf(b, -r[n + q]) : b;
}

// Tile j of a level is floor(j * x_tiles / level_tiles): evenly spaced over the
// database, every tile for the full level.  A walk steps j by one with the
// quotient and remainder of x_tiles / level_tiles (one division per walk).
struct TileWalk {
  uint32_t tile, rem, q, r, div;  // tiles < 2^23 (m <= 2^31 rows)
  __device__ __forceinline__ TileWalk(const FilterArgs &a, int64_t j) {
    div = (uint32_t)a.level_tiles;
    q = (uint32_t)(a.x_tiles / a.level_tiles);
    r = (uint32_t)(a.x_tiles - (int64_t)q * a.level_tiles);
    const int64_t p = j * a.x_tiles;
    const int64_t t = p / a.level_tiles;
    tile = (uint32_t)t;
    rem = (uint32_t)(p - t * a.level_tiles);
  }
  __device__ __forceinline__ void next() {
    tile += q;
    rem += r;
    if (rem >= div) { rem -= div; tile++; }
  }
};

// The stage ring is split in two, one per MMA issuer: the chunks of tile lt pass
// through ring lt & 1 (stages [base, base + count)) in order, so every ring has one
// producer and one consumer, and a waiter is never more than one phase ahead of a
// barrier (the condition for parity waits).
struct StageRings {
  uint32_t count0, count1;  // stages of ring 0 (first) and ring 1
  __device__ __forceinline__ StageRings(int ns, bool split)
      : count0(split ? (uint32_t)(ns + 1) / 2 : (uint32_t)ns), count1(split ? (uint32_t)ns / 2 : 1u) {}
  __device__ __forceinline__ uint32_t count(int r) const { return r ? count1 : count0; }
  __device__ __forceinline__ uint32_t stage(int r, uint32_t pos) const {
    return r ? count0 + pos % count1 : pos % count0;
  }
  __device__ __forceinline__ uint32_t parity(int r, uint32_t pos) const {
    return (pos / count(r)) & 1u;
  }
};

// Two MMA issuers only for tiles of at most two chunks (d <= 128): a longer tile does
// not fit in half of the ring, and its loads would wait for the other issuer's tile.
__host__ __device__ inline bool two_issuers(int kch) { return kch <= 2; }

// 608 threads in one block (19 warps): at most 96 registers a thread.
// PAIR: the kernel runs as clusters of two CTAs on two SMs.  The even CTA issues
// tcgen05.mma.cta_group::2 with M = 256 (its query tile and its peer's) and
// N = 256 rows, each CTA holding its query tile and half of each row tile; the
// accumulator of each CTA's 128 queries lands in its own tensor memory.
template <bool PAIR>
__global__ void __maxnreg__(96)
    knn_tc_filter_kernel(const __grid_constant__ CUtensorMap tmap_q,
                         const __grid_constant__ CUtensorMap tmap_x, const FilterArgs a, int kch) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // align the dynamic smem base to 1024 bytes (swizzle atoms)
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const TcLayout L = tc_layout(kch, PAIR);
  unsigned char *sA = smem + L.a_off;
  unsigned char *sB = smem + L.b_off;
  float *nxs = reinterpret_cast<float *>(smem + L.nx_off);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar_off);
  uint64_t *full = bars;                 // [ns]
  uint64_t *empty = bars + L.ns;         // [ns]
  uint64_t *a_full = bars + 2 * L.ns;    // [1]
  uint64_t *acc_full = a_full + 1;       // [2]
  uint64_t *acc_empty = acc_full + 2;    // [2]
  uint64_t *drain = acc_empty + 2;       // [1]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile int *epi_stop = abort_flag + 1;  // the epilogue's copy of abort_flag, one per tile

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTA pairs: blocks (2p, 2p+1) form a cluster and take query tiles (2qp, 2qp+1)
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int units_per_slice = PAIR ? a.q_tiles / 2 : a.q_tiles;
  const int qt = PAIR ? 2 * (unit % units_per_slice) + (int)rank : unit % units_per_slice;
  const int s = unit / units_per_slice;
  const int64_t j_begin = (int64_t)s * a.tiles_per_slice;
  int64_t j_end = j_begin + a.tiles_per_slice;
  if (j_end > a.level_tiles) j_end = a.level_tiles;
  const int ntiles = j_end > j_begin ? (int)(j_end - j_begin) : 0;
  const int ns = L.ns;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ns; i++) { mbar_init(full + i, 1); mbar_init(empty + i, 1); }
    mbar_init(a_full, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_full + 1, 1);
    // both CTAs' epilogues release the pair's accumulator on the even CTA's barrier
    mbar_init(acc_empty, PAIR ? 2 * kEpiWarps : kEpiWarps);
    mbar_init(acc_empty + 1, PAIR ? 2 * kEpiWarps : kEpiWarps);
    mbar_init(drain, two_issuers(kch) ? 2 : 1);  // every MMA issuer commits
    *abort_flag = 0;
    *epi_stop = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_slot, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // the peer signals this CTA's barriers: both must be initialised first
  if (PAIR) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && ntiles > 0) {
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_x);
      // in a pair, only the even CTA arms the barriers; both CTAs' copies count on them
      if (!L.stream_a) {
        if (rank == 0) mbar_arrive_expect_tx(a_full, (uint32_t)((PAIR ? 2 : 1) * kch * kAChunkBytes));
        for (int c = 0; c < kch; c++) {
          if (PAIR) tma_load_2d_pair(sA + c * kAChunkBytes, &tmap_q, a_full, c * kBK, qt * kBM);
          else tma_load_2d(sA + c * kAChunkBytes, &tmap_q, a_full, c * kBK, qt * kBM);
        }
      }
      uint32_t issued0 = 0, issued1 = 0;  // chunks loaded into each ring
      bool ok = true;
      const uint32_t bchunk = L.bchunk, stage = L.stage;
      const uint32_t boff = L.stream_a ? kAChunkBytes : 0;  // row chunk after the query chunk
      const uint32_t tx = (PAIR ? 2 : 1) * (bchunk + (L.stream_a ? kAChunkBytes : 0));
      const bool split = two_issuers(kch);
      const StageRings R(ns, split);
      TileWalk walk(a, j_begin);
      for (int lt = 0; lt < ntiles && ok; lt++, walk.next()) {
        const int rg = split ? (lt & 1) : 0;
        // a pair's CTAs load rows [0, 128) and [128, 256) of the tile
        const int32_t row0 = (int32_t)(walk.tile * kBN) + (int32_t)(rank * (kBN / 2));
        for (int c = 0; c < kch; c++) {
          const uint32_t pos = rg ? issued1 : issued0;
          const uint32_t st = R.stage(rg, pos), ph = R.parity(rg, pos);
          if (!mbar_wait_bounded(empty + st, ph ^ 1, abort_flag)) {
            set_error(a.hdr, ERR_TIMEOUT_PRODUCER, abort_flag);
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(full + st, tx);
          unsigned char *sst = sB + st * stage;
          if (L.stream_a) {
            if (PAIR) tma_load_2d_pair(sst, &tmap_q, full + st, c * kBK, qt * kBM);
            else tma_load_2d(sst, &tmap_q, full + st, c * kBK, qt * kBM);
          }
          if (PAIR) tma_load_2d_pair(sst + boff, &tmap_x, full + st, c * kBK, row0);
          else tma_load_2d(sst + boff, &tmap_x, full + st, c * kBK, row0);
          if (rg) issued1 = pos + 1; else issued0 = pos + 1;
        }
      }
      // every issued copy must land before the CTA may exit; in a pair the even
      // CTA's barriers count the peer's copies too, and the peer waits for it below
      if (rank == 0) {
        for (int rg = 0; rg < 2; rg++) {
          const uint32_t done = rg ? issued1 : issued0;
          const uint32_t first = done > R.count(rg) ? done - R.count(rg) : 0u;
          for (uint32_t i = first; i < done; i++)
            mbar_wait_bounded(full + R.stage(rg, i), R.parity(rg, i), abort_flag);
        }
        if (!L.stream_a) mbar_wait_bounded(a_full, 0, abort_flag);
      }
    }
  } else if (warp == 1 || warp == kIssuerWarp2) {
    // ---------------- MMA issuers ----------------
    // For tiles of one or two chunks, two threads issue the MMAs, issuer X taking tiles
    // X, X + 2, ... (accumulator buffer X): a thread that waits on a barrier stops
    // issuing for a while, and the tensor pipe keeps little work queued, so with short
    // tiles one issuer issues while the other waits.  Longer tiles use issuer 0 alone.
    const bool split = two_issuers(kch);
    if (lane == 0 && ntiles > 0 && rank == 0 && (split || warp == 1)) {
      const int X = warp == 1 ? 0 : 1;
      const int step = split ? 2 : 1;
      constexpr uint32_t idesc = idesc_f16_f32(PAIR ? 2 * kBM : kBM, kBN);
      const uint32_t stage = L.stage;
      const uint32_t a_addr = smem_u32(sA), b_addr = smem_u32(sB);
      const uint32_t boff = L.stream_a ? kAChunkBytes : 0;
      // shared-memory descriptors, split into the 32-bit word holding the start address
      // (which the loop advances) and the constant upper word
      const uint64_t d0 = umma_desc_k_sw128(0);
      const uint32_t desc_hi = (uint32_t)(d0 >> 32);
      const uint32_t a_lo0 = (uint32_t)umma_desc_k_sw128(a_addr);
      const uint32_t sa_lo0 = (uint32_t)umma_desc_k_sw128(b_addr);          // streamed query chunk
      const uint32_t b_lo0 = (uint32_t)umma_desc_k_sw128(b_addr + boff);
      bool ok = L.stream_a || mbar_wait_bounded(a_full, 0, abort_flag);
      if (!ok) set_error(a.hdr, ERR_TIMEOUT_MMA, abort_flag);
      const StageRings R(ns, split);
      for (int lt = X; lt < ntiles && ok; lt += step) {
        const int b = lt & 1;
        uint32_t pos = (uint32_t)(lt / step) * (uint32_t)kch;  // this tile's first chunk in ring X
        if (!mbar_wait_bounded(acc_empty + b, ((lt >> 1) & 1) ^ 1, abort_flag)) {
          set_error(a.hdr, ERR_TIMEOUT_MMA, abort_flag);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(b * kBN);
        for (int c = 0; c < kch && ok; c++, pos++) {
          const uint32_t st = R.stage(X, pos), ph = R.parity(X, pos);
          if (!mbar_wait_bounded(full + st, ph, abort_flag)) {
            set_error(a.hdr, ERR_TIMEOUT_MMA, abort_flag);
            ok = false;
            break;
          }
          tc_fence_after();
          // descriptors of this chunk: the start-address field moves by 32 bytes per K step
          const uint32_t b_lo = b_lo0 + st * (stage >> 4);
          const uint32_t a_lo = L.stream_a ? sa_lo0 + st * (stage >> 4)
                                           : a_lo0 + (uint32_t)c * (kAChunkBytes >> 4);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; kk++) {
            const uint64_t ad = desc_from(a_lo + 2u * kk, desc_hi);
            const uint64_t bd = desc_from(b_lo + 2u * kk, desc_hi);
            if (PAIR) tc_mma_f16_pair(d_tmem, ad, bd, idesc, (c | kk) != 0);
            else tc_mma_f16(d_tmem, ad, bd, idesc, (c | kk) != 0);
          }
          if (PAIR) tc_commit_pair_mc(empty + st, 0x3);  // frees the stage in both CTAs
          else tc_commit(empty + st);
        }
        if (ok) {
          if (PAIR) tc_commit_pair_mc(acc_full + b, 0x3);  // both epilogues
          else tc_commit(acc_full + b);
        }
      }
      // all issued MMAs must finish before tensor memory is released
      if (PAIR) tc_commit_pair(drain);
      else tc_commit(drain);
      mbar_wait_bounded(drain, 0, abort_flag);
    }
  } else if (warp < 2 + kEpiWarps) {
    // ------------- epilogue: one query per thread, 64 columns of each tile per warp -------------
    const int e = warp - 2;                   // 0..15
    const int quarter = warp & 3;             // TMEM lanes this warp may access (warp % 4)
    const int cg = e >> 2;                    // columns [cg*64, cg*64 + 64) of each tile
    const int r = quarter * 32 + lane;        // query row within the tile
    const int64_t q = (int64_t)qt * kBM + r;
    const bool valid = q < a.n;
    const float margin = a.qinfo[(size_t)qt * kBM + r].y;
    // theta = B + margin, B = (k-th smallest v of the previous level) + margin, rounded up.
    // Rows past m carry ||x||^2 = +inf, so theta stays finite: FLT_MAX when there is no bound.
    const bool all_pass = a.r_in == nullptr;  // the first level: no bound yet
    float theta = -INFINITY;
    if (valid)
      theta = a.r_in ? fminf(__fadd_ru(read_bound(a.r_in, a.n, q, a.two_bounds), margin), FLT_MAX)
                     : FLT_MAX;
    // the next float above theta: a chunk whose bound reaches it holds no v <= theta
    const float theta2 = theta == -INFINITY ? -INFINITY : nextafterf(theta, INFINITY);
    uint2 *region = a.cand + (size_t)(valid ? q : 0) * a.pool +
                    (size_t)(kColGroups * s + cg) * a.region;
    const int last = a.region - 1;            // a full region keeps overwriting its last slot
    int cnt = 0;
    const uint32_t taddr0 = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(cg * kGroupN);
    const float inv_sq = *a.inv_sq;
    const float nhsq = -0.5f * __frcp_rn(inv_sq);  // -s_q / 2 (powers of two, exact)
    float *nxw = nxs + e * 2 * kNxStage;      // this warp's ||x||^2 staging, two buffers
    // prefetch ||x||^2 (2 rows per lane) and the group record of the first tile
    float2 pre_nx = make_float2(0.f, 0.f);
    float4 pre_gmin = make_float4(0.f, 0.f, 0.f, 0.f), pre_sc = pre_gmin;
    TileWalk walk(a, j_begin);
    if (ntiles > 0) {
      const uint32_t t0 = walk.tile;
      pre_nx = *reinterpret_cast<const float2 *>(a.xnorm + (size_t)t0 * kBN + cg * kGroupN + lane * 2);
      pre_gmin = __ldg(a.xmeta + 2 * ((size_t)t0 * kColGroups + cg));
      pre_sc = __ldg(a.xmeta + 2 * ((size_t)t0 * kColGroups + cg) + 1);
    }

    for (int lt = 0; lt < ntiles; lt++) {
      const int b = lt & 1;
      const uint32_t tile = walk.tile;
      walk.next();  // the walk is one tile ahead from here on
      float *nxt = nxw + b * kNxStage;
      *reinterpret_cast<float2 *>(nxt + lane * 2) = pre_nx;
      // v = fma(c, acc, ||x||^2) with c = -2 / (s_q s_x), an exact power of two
      const float cscale = -2.0f * inv_sq * pre_sc.x;
      // Chunk thresholds: every v of 16-column chunk j exceeds theta when the chunk's
      // largest accumulator is <= T_j = (theta2 - min ||x||^2) / c, rounded so that
      // T_j is below the exact quotient (c < 0; 1/c = -s_q s_x / 2, exact when normal).
      float T[4];
      {
        const float inv_c = nhsq * pre_sc.y;
        const bool ok = fabsf(inv_c) >= FLT_MIN && fabsf(inv_c) <= FLT_MAX;
        T[0] = ok ? __fmul_rd(__fsub_ru(theta2, pre_gmin.x), inv_c) : -INFINITY;
        T[1] = ok ? __fmul_rd(__fsub_ru(theta2, pre_gmin.y), inv_c) : -INFINITY;
        T[2] = ok ? __fmul_rd(__fsub_ru(theta2, pre_gmin.z), inv_c) : -INFINITY;
        T[3] = ok ? __fmul_rd(__fsub_ru(theta2, pre_gmin.w), inv_c) : -INFINITY;
      }
      if (lt + 1 < ntiles) {
        const uint32_t tn = walk.tile;
        pre_nx = *reinterpret_cast<const float2 *>(a.xnorm + (size_t)tn * kBN + cg * kGroupN + lane * 2);
        pre_gmin = __ldg(a.xmeta + 2 * ((size_t)tn * kColGroups + cg));
        pre_sc = __ldg(a.xmeta + 2 * ((size_t)tn * kColGroups + cg) + 1);
      }
      // tcgen05.ld is warp-collective: the whole warp proceeds or none of it
      const bool got = __all_sync(0xffffffffu, mbar_wait_bounded(acc_full + b, (lt >> 1) & 1,
                                                                 abort_flag));
      if (!got) {
        set_error(a.hdr, ERR_TIMEOUT_EPILOGUE, abort_flag);
        break;
      }
      tc_fence_after();
      const uint32_t row0 = tile * kBN + (uint32_t)(cg * kGroupN);
      // 16 columns at a time; the load of the next 16 is in flight while these are checked
      uint32_t ra[16], rb[16];
      tmem_ld_32x32b_x16(taddr0 + (uint32_t)(b * kBN), ra);
      tmem_ld_wait(ra);
      __syncwarp();  // the ||x||^2 staging written above is visible to every lane
#pragma unroll
      for (int qq = 0; qq < 4; qq++) {
        uint32_t (&cur)[16] = (qq & 1) ? rb : ra;
        uint32_t (&nxb)[16] = (qq & 1) ? ra : rb;
        if (qq < 3) tmem_ld_32x32b_x16(taddr0 + (uint32_t)(b * kBN + (qq + 1) * 16), nxb);
        if (qq == 2) {
          // the last 16 columns are in registers: release the accumulator buffer to the
          // MMA issuer before checking chunks 2 and 3
          tmem_ld_wait(nxb);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (PAIR) mbar_arrive_cluster(acc_empty + b, 0);
            else mbar_arrive(acc_empty + b);
          }
        }
        const float4 *nx4 = reinterpret_cast<const float4 *>(nxt + qq * 16);
        const uint32_t rg = row0 + (uint32_t)(qq * 16);
        if (all_pass) {
          // no bound yet: every finite v is kept, one predicated store per column
#pragma unroll
          for (int g = 0; g < 2; g++) {
            float v[8];
            exact_v8(cur + 8 * g, cscale, nx4[2 * g], nx4[2 * g + 1], v);
#pragma unroll
            for (int i = 0; i < 8; i++) {
              const bool keep = v[i] <= theta;
              if (keep) region[min(cnt, last)] = make_uint2(rg + 8 * g + i, __float_as_uint(v[i]));
              cnt += keep ? 1 : 0;
            }
          }
        } else {
          // one bound for the chunk: its largest accumulator against T; a lane whose
          // chunk passes computes every exact v of it (packed FMAs) and appends the kept
          // ones.  A plain per-lane branch measured fastest: a warp vote with the detail
          // marked unlikely, or exact values only for the columns whose own accumulator
          // passes, made 1M x d=8 queries twice as slow and 1M x d=128 ones 14 % slower
          // (norms that vary within a chunk loosen T, so chunks pass often there), and
          // did not help the 10M-row unit-vector pass.
          const bool pass = max16u(cur) > T[qq];
          if (pass) {
            float v[16];
            exact_v8(cur, cscale, nx4[0], nx4[1], v);
            exact_v8(cur + 8, cscale, nx4[2], nx4[3], v + 8);
            unsigned keep = 0;
#pragma unroll
            for (int i = 0; i < 16; i++) keep |= (v[i] <= theta ? 1u : 0u) << i;
            while (keep) {
              const int i = __ffs(keep) - 1;
              keep &= keep - 1;
              region[min(cnt, last)] = make_uint2(rg + i, __float_as_uint(pick16(v, i)));
              cnt++;
            }
          }
        }
        if (qq < 2) tmem_ld_wait(nxb);
      }
      __syncwarp();  // the staging buffer of this tile is reused two tiles later
    }
    if (valid) a.ccount[(size_t)q * kColGroups * a.max_slices + kColGroups * s + cg] = cnt;
  }

  tc_fence_before();
  __syncthreads();
  // neither CTA of a pair leaves while the pair's MMAs may still touch its memory
  if (PAIR) cluster_sync_all();
  tc_fence_after();
  if (warp == 1) {
    if (PAIR) tmem_dealloc_pair(tmem_base, 512);
    else tmem_dealloc(tmem_base, 512);
  }
}

// ---------------------------------------------------------------------------
// prep: database rows -> f16 (256-row blocks share a power-of-two scale)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float pow2_scale_for(float maxabs) {
  // scale s = 2^e with maxabs * s in [2^13, 2^14): f16 max is 65504
  if (!(maxabs > 0.f) || !isfinite(maxabs)) return 1.f;
  int e;
  frexpf(maxabs, &e);  // maxabs = f * 2^e, f in [0.5, 1)
  int p = 14 - e;
  if (p > 126) p = 126;
  if (p < -126) p = -126;
  return ldexpf(1.f, p);
}

// Squared rounding error of four values against their f16 forms h (scaled by 1/inv),
// accumulated into acc.  v - h * inv is exact (h * inv is a power-of-two scaling of a
// value within 2^-11 of v, so the difference is exact by Sterbenz' lemma, up to
// underflow below the margin's own FP32 terms).
__device__ __forceinline__ float round_err4(float4 v, __half2 lo, __half2 hi, float inv,
                                            float acc) {
  const float2 a = __half22float2(lo), b = __half22float2(hi);
  float e = v.x - a.x * inv;
  acc = __fmaf_rn(e, e, acc);
  e = v.y - a.y * inv;
  acc = __fmaf_rn(e, e, acc);
  e = v.z - b.x * inv;
  acc = __fmaf_rn(e, e, acc);
  e = v.w - b.y * inv;
  return __fmaf_rn(e, e, acc);
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// A warp's largest row rounding error (sum of squares) into hdr->ex_bits as a norm,
// rounded up (non-negative floats, +inf included, order like their bit patterns).
__device__ __forceinline__ float norm_up(float sum_sq, int d);
__device__ __forceinline__ void note_row_error(float emax2, int d, WsHeader *hdr) {
  if ((threadIdx.x & 31) == 0 && emax2 > 0.f)  // NaN rows are exact-only already
    atomicMax(&hdr->ex_bits, __float_as_uint(norm_up(emax2, d)));
}
// sqrt of an FP32 sum of d squares, rounded so that it bounds the exact norm: each of the
// d + 2 roundings (sum, square root) is at most 2^-24 relative
__device__ __forceinline__ float norm_up(float sum_sq, int d) {
  return __fmul_ru(__fsqrt_ru(sum_sq), 1.f + (float)(d + 3) * 5.9604645e-8f);
}

// Database rows -> f16.  Each group of 64 rows (one epilogue warp's columns of a
// tile) shares a power-of-two scale.  grid (ceil(m / 64)), block 256: eight warps
// of eight rows each.  VEC (d % 4 == 0, d <= 256): each row is read once, as
// float4s held in registers between the norm pass and the conversion.
constexpr int kScaleRows = kBN / kColGroups;  // 64
template <bool VEC, int W4>
__global__ void __launch_bounds__(256) tc_prep_x_kernel(const float *__restrict__ X, int64_t m,
                                                        int d, int d_pad, __half *__restrict__ Xh,
                                                        float *__restrict__ xnorm,
                                                        float4 *__restrict__ xmeta, WsHeader *hdr) {
  __shared__ float s_max[8], s_rn[8], s_min[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t grp = blockIdx.x;
  const int64_t row_base = grp * kScaleRows + warp * 8;
  const int d4 = d >> 2;
  float4 xr[8][W4];  // VEC: rows of up to 128 * W4 floats, W4 float4 per lane
  float ss[8], mx[8];
#pragma unroll
  for (int u = 0; u < 8; u++) {
    ss[u] = 0.f;
    mx[u] = 0.f;
    const int64_t row = row_base + u;
    if (VEC) {
#pragma unroll
      for (int h = 0; h < W4; h++) {
        const int c = lane + 32 * h;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row < m && c < d4) v = __ldg(reinterpret_cast<const float4 *>(X + row * d) + c);
        xr[u][h] = v;
        ss[u] = __fmaf_rn(v.x, v.x, ss[u]);
        ss[u] = __fmaf_rn(v.y, v.y, ss[u]);
        ss[u] = __fmaf_rn(v.z, v.z, ss[u]);
        ss[u] = __fmaf_rn(v.w, v.w, ss[u]);
        mx[u] = fmaxf(mx[u], fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
    } else if (row < m) {
      const float *x = X + row * d;
      for (int c = lane; c < d; c += 32) {
        const float v = __ldg(x + c);
        ss[u] = __fmaf_rn(v, v, ss[u]);
        mx[u] = fmaxf(mx[u], fabsf(v));
      }
    }
  }
  float wmax = 0.f, wrn = 0.f, wmin = INFINITY;
  bool bad = false;
#pragma unroll
  for (int u = 0; u < 8; u++) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ss[u] += __shfl_xor_sync(0xffffffffu, ss[u], o);
      mx[u] = fmaxf(mx[u], __shfl_xor_sync(0xffffffffu, mx[u], o));
    }
    const int64_t row = row_base + u;
    if (row < m) {
      if (!isfinite(ss[u])) bad = true;
      wmax = fmaxf(wmax, mx[u]);
      wrn = fmaxf(wrn, sqrtf(ss[u]));
      wmin = fminf(wmin, ss[u]);
    }
    // rows past m: v = +inf never passes a finite threshold
    if (lane == u) xnorm[row] = row < m ? ss[u] : INFINITY;
  }
  if (lane == 0) { s_max[warp] = wmax; s_rn[warp] = wrn; s_min[warp] = wmin; }
  if (bad && lane == 0) atomicOr(&hdr->exact_only, 1);
  __syncthreads();
  float gmax = 0.f, rn = 0.f;
#pragma unroll
  for (int w = 0; w < 8; w++) { gmax = fmaxf(gmax, s_max[w]); rn = fmaxf(rn, s_rn[w]); }
  const float sc = pow2_scale_for(gmax);
  if (threadIdx.x == 0) {
    // the group's record: min ||x||^2 of each 16-row chunk (warps 2j, 2j+1; +inf for a
    // chunk of padding rows), then the scale and its inverse
    xmeta[2 * grp] = make_float4(fminf(s_min[0], s_min[1]), fminf(s_min[2], s_min[3]),
                                 fminf(s_min[4], s_min[5]), fminf(s_min[6], s_min[7]));
    xmeta[2 * grp + 1] = make_float4(1.f / sc, sc, 0.f, 0.f);
    // sqrt of an FP32 sum of d squares: (1 + 2^-10) covers its rounding for d <= 4096;
    // the bound only grows, and non-negative floats order like their bit patterns
    if (isfinite(rn)) atomicMax(&hdr->rx_bits, __float_as_uint(rn * (1.f + 0.0009765625f)));
  }
  // the conversion, and each row's rounding error ||x - f16 form|| (its largest into hdr)
  const float inv = 1.f / sc;
  float emax = 0.f;
#pragma unroll
  for (int u = 0; u < 8; u++) {
    const int64_t row = row_base + u;
    if (row >= m) break;
    __half *xh = Xh + row * d_pad;
    float e2 = 0.f;
    if (VEC) {
      // four halves (8 bytes) per lane and step; columns past d are zero
#pragma unroll
      for (int h = 0; h < W4; h++) {
        const int c = lane + 32 * h;
        if (c < (d_pad >> 2)) {
          const float4 v = xr[u][h];
          __half2 lo = __floats2half2_rn(v.x * sc, v.y * sc);
          __half2 hi = __floats2half2_rn(v.z * sc, v.w * sc);
          e2 = round_err4(v, lo, hi, inv, e2);
          uint2 pk;
          pk.x = *reinterpret_cast<uint32_t *>(&lo);
          pk.y = *reinterpret_cast<uint32_t *>(&hi);
          reinterpret_cast<uint2 *>(xh)[c] = pk;
        }
      }
    } else {
      const float *x = X + row * d;
      for (int c = lane; c < d_pad; c += 32) {
        const float v = c < d ? x[c] : 0.f;
        const __half hv = __float2half_rn(v * sc);
        const float e = v - __half2float(hv) * inv;
        e2 = __fmaf_rn(e, e, e2);
        xh[c] = hv;
      }
    }
    emax = fmaxf(emax, warp_sum(e2));
  }
  note_row_error(emax, d, hdr);
}

// A prepared database's row status (norm bound, non-finite rows) into this search's header.
__global__ void tc_take_row_status(const WsHeader *src, WsHeader *dst) {
  if (threadIdx.x == 0) {
    dst->rx_bits = src->rx_bits;
    dst->ex_bits = src->ex_bits;
    dst->exact_only = src->exact_only;
  }
}

// Database rows -> f16 for wide rows (d % 4 == 0, d > 256): the same 64-row scale
// groups as tc_prep_x_kernel, in two passes over each row with float4 loads (four in
// flight per lane): norms and the group maximum, then the conversion, whose re-read of
// the group's rows mostly hits L2.  grid (ceil(m / 64)), block 256: eight warps of eight
// rows each.
__global__ void __launch_bounds__(256) tc_prep_x_wide_kernel(const float *__restrict__ X,
                                                             int64_t m, int d, int d_pad,
                                                             __half *__restrict__ Xh,
                                                             float *__restrict__ xnorm,
                                                             float4 *__restrict__ xmeta,
                                                             WsHeader *hdr) {
  __shared__ float s_max[8], s_rn[8], s_min[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t grp = blockIdx.x;
  const int64_t row_base = grp * kScaleRows + warp * 8;
  const int d4 = d >> 2, dp4 = d_pad >> 2;
  float wmax = 0.f, wrn = 0.f, wmin = INFINITY;
  bool bad = false;
  for (int u = 0; u < 8; u++) {
    const int64_t row = row_base + u;
    float ss = 0.f, mx = 0.f;
    if (row < m) {
      const float4 *x4 = reinterpret_cast<const float4 *>(X + row * d);
      for (int c0 = lane; c0 < d4; c0 += 4 * 32) {
        float4 v[4];
#pragma unroll
        for (int h = 0; h < 4; h++) {
          const int c = c0 + 32 * h;
          v[h] = c < d4 ? __ldg(x4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int h = 0; h < 4; h++) {
          ss = __fmaf_rn(v[h].x, v[h].x, ss);
          ss = __fmaf_rn(v[h].y, v[h].y, ss);
          ss = __fmaf_rn(v[h].z, v[h].z, ss);
          ss = __fmaf_rn(v[h].w, v[h].w, ss);
          mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[h].x), fabsf(v[h].y)), fmaxf(fabsf(v[h].z), fabsf(v[h].w))));
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (row < m) {
      if (!isfinite(ss)) bad = true;
      wmax = fmaxf(wmax, mx);
      wrn = fmaxf(wrn, sqrtf(ss));
      wmin = fminf(wmin, ss);
    }
    // rows past m: v = +inf never passes a finite threshold
    if (lane == 0) xnorm[row] = row < m ? ss : INFINITY;
  }
  if (lane == 0) { s_max[warp] = wmax; s_rn[warp] = wrn; s_min[warp] = wmin; }
  if (bad && lane == 0) atomicOr(&hdr->exact_only, 1);
  __syncthreads();
  float gmax = 0.f, rn = 0.f;
#pragma unroll
  for (int w = 0; w < 8; w++) { gmax = fmaxf(gmax, s_max[w]); rn = fmaxf(rn, s_rn[w]); }
  const float sc = pow2_scale_for(gmax);
  if (threadIdx.x == 0) {
    // the group's record: min ||x||^2 of each 16-row chunk (warps 2j, 2j+1; +inf for a
    // chunk of padding rows), then the scale and its inverse
    xmeta[2 * grp] = make_float4(fminf(s_min[0], s_min[1]), fminf(s_min[2], s_min[3]),
                                 fminf(s_min[4], s_min[5]), fminf(s_min[6], s_min[7]));
    xmeta[2 * grp + 1] = make_float4(1.f / sc, sc, 0.f, 0.f);
    // sqrt of an FP32 sum of d squares: (1 + 2^-10) covers its rounding for d <= 4096;
    // the bound only grows, and non-negative floats order like their bit patterns
    if (isfinite(rn)) atomicMax(&hdr->rx_bits, __float_as_uint(rn * (1.f + 0.0009765625f)));
  }
  const float inv = 1.f / sc;
  float emax = 0.f;
  for (int u = 0; u < 8; u++) {
    const int64_t row = row_base + u;
    if (row >= m) break;
    const float4 *x4 = reinterpret_cast<const float4 *>(X + row * d);
    uint2 *xh2 = reinterpret_cast<uint2 *>(Xh + row * d_pad);
    float e2 = 0.f;
    for (int c0 = lane; c0 < dp4; c0 += 4 * 32) {
      float4 v[4];
#pragma unroll
      for (int h = 0; h < 4; h++) {
        const int c = c0 + 32 * h;
        v[h] = c < d4 ? __ldg(x4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int h = 0; h < 4; h++) {
        const int c = c0 + 32 * h;
        if (c < dp4) {
          // four halves (8 bytes) per lane and step; columns past d are zero
          __half2 lo = __floats2half2_rn(v[h].x * sc, v[h].y * sc);
          __half2 hi = __floats2half2_rn(v[h].z * sc, v[h].w * sc);
          e2 = round_err4(v[h], lo, hi, inv, e2);
          uint2 pk;
          pk.x = *reinterpret_cast<uint32_t *>(&lo);
          pk.y = *reinterpret_cast<uint32_t *>(&hi);
          xh2[c] = pk;
        }
      }
    }
    emax = fmaxf(emax, warp_sum(e2));
  }
  note_row_error(emax, d, hdr);
}

// max |Q| -> hdr->qmax_bits
__global__ void tc_qmax_kernel(const float *__restrict__ Q, int64_t count, WsHeader *hdr) {
  float mx = 0.f;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < count;
       e += (int64_t)gridDim.x * blockDim.x)
    mx = fmaxf(mx, fabsf(Q[e]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0 && mx > 0.f) {
    if (isfinite(mx)) atomicMax(&hdr->qmax_bits, __float_as_uint(mx));
    else atomicOr(&hdr->exact_only, 1);
  }
}

// grid (q_rows / 8), block 256: one warp per query row.  Writes the f16 query
// tile rows (zero for padding rows), ||q||^2 and the error margin.
__global__ void __launch_bounds__(256) tc_prep_q_kernel(const float *__restrict__ Q, int64_t n,
                                                        int d, int d_pad, int64_t q_rows,
                                                        __half *__restrict__ Qh,
                                                        float2 *__restrict__ qinfo,
                                                        float *__restrict__ inv_sq_out,
                                                        WsHeader *hdr) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= q_rows) return;
  const float qmax = __uint_as_float(hdr->qmax_bits);
  const float sq = pow2_scale_for(qmax);
  if (row == 0 && lane == 0) *inv_sq_out = 1.f / sq;
  __half *qh = Qh + row * d_pad;
  if (row >= n) {
    for (int c = lane; c < d_pad; c += 32) qh[c] = __float2half_rn(0.f);
    if (lane == 0) qinfo[row] = make_float2(0.f, NAN);
    return;
  }
  const float *qp = Q + row * d;
  const float inv_sq = 1.f / sq;
  float ss = 0.f, e2 = 0.f;  // ||q||^2 and ||q - f16 form of q||^2
  for (int c = lane; c < d_pad; c += 32) {
    const float v = c < d ? qp[c] : 0.f;
    ss = __fmaf_rn(v, v, ss);
    const __half h = __float2half_rn(v * sq);
    const float e = v - __half2float(h) * inv_sq;
    e2 = __fmaf_rn(e, e, e2);
    qh[c] = h;
  }
  ss = warp_sum(ss);
  e2 = warp_sum(e2);
  if (lane == 0) {
    if (!isfinite(ss)) atomicOr(&hdr->exact_only, 1);
    // Error margin.  With qn >= ||q||, Rx >= max ||x|| and the measured f16 rounding
    // errors (q~ the f16 form of q scaled back, x~ likewise, both exact in FP32):
    //   e_q >= ||q - q~||,  e_x >= max over rows ||x - x~||   (at most 2^-11 ||q||,
    //                       2^-11 ||x|| above the f16 subnormal range; measured instead)
    //   dot rounding  <= e_q Rx + qn e_x + e_q e_x      (|q~.x~ - q.x|, Cauchy-Schwarz)
    //   accumulation  <= (d_pad + 16) 2^-22 (qn + e_q)(Rx + e_x)   (tensor-core FP32 sums)
    //   FP32 terms    <= 2 (d + 8) 2^-24 (qn + Rx)^2  (norms, the fused epilogue step,
    //                                                  and the reference's own rounding)
    //   margin = 2 (dot rounding + accumulation) + FP32 terms.
    // Then |(||q||^2 + v) - D| <= margin for every row, v the epilogue value and D
    // the reference kernel's FP32 distance.
    const double qn = sqrt((double)ss) * (1.0 + ldexp(1.0, -10));
    const double rx = (double)__uint_as_float(hdr->rx_bits);
    // the FP32 sum of d squares is within (d + 2) 2^-24 of the exact one, its root half that
    const double eq = sqrt((double)e2) * (1.0 + (double)(d + 3) * ldexp(1.0, -24));
    const double ex = (double)__uint_as_float(hdr->ex_bits);
    const double dotr = eq * rx + qn * ex + eq * ex;
    const double acc = (double)(d_pad + 16) * ldexp(1.0, -22) * (qn + eq) * (rx + ex);
    const double f32 = 2.0 * (double)(d + 8) * ldexp(1.0, -24) * (qn + rx) * (qn + rx);
    const double margin = 2.0 * (dotr + acc) + f32;
    // The filter needs 2^-48 <= qn + Rx < 2^63; outside it the search goes to the exact
    // SIMT engine:
    // * below, the epilogue's factor -2/(s_q s_x) can underflow to zero
    //   (s_q s_x > 2^150) and FP32 rounding stops being relative (subnormals), so
    //   |(||q||^2 + v) - D| can exceed the margin (every norm under about 3.6e-15);
    // * from 2^63 on, (||q|| + ||x||)^2 >= 2^126 and a distance or v can overflow to
    //   +inf.  A row with v = +inf is never a candidate, but an infinite distance is
    //   still returned when fewer than k rows have a finite one.
    // The margin is then +inf, so that the level bounds this search hands to the other
    // shards of a sharded search (whose rows may be in range) bound nothing.
    const bool in_range = qn + rx >= ldexp(1.0, -48) && qn + rx < ldexp(1.0, 63);
    if (!in_range) atomicOr(&hdr->exact_only, 1);
    qinfo[row] = make_float2(ss, in_range ? __double2float_ru(margin * (1.0 + 1e-6)) : INFINITY);
  }
}

// ---------------------------------------------------------------------------
// selection helpers
// ---------------------------------------------------------------------------
__device__ void bitonic_sort_u64(uint64_t *keys, int P) {
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int t = threadIdx.x; t < P / 2; t += blockDim.x) {
        const int lo = 2 * stride * (t / stride) + (t % stride);
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const uint64_t x = keys[lo], y = keys[hi];
        if ((x > y) == up) { keys[lo] = y; keys[hi] = x; }
      }
    }
  }
  __syncthreads();
}

// Candidate regions of one query: counts clamped to the region size, their
// exclusive prefix offsets, and whether a region lost entries.
struct QueryRegions {
  const uint2 *base;   // this query's pool
  int region;          // entries per region
  int nreg;            // regions of the level
  int total;
  bool over;
  int stage_cap;       // candidates the caller's shared memory can stage
};

__device__ QueryRegions load_regions(const uint2 *cand, const int *ccount, int64_t q, int pool,
                                     int region, int nreg, int stride, int *s_cnt, int *s_off,
                                     int *s_misc) {
  for (int i = threadIdx.x; i < nreg; i += blockDim.x) s_cnt[i] = ccount[(size_t)q * stride + i];
  __syncthreads();
  if (threadIdx.x < 32) {
    // warp 0: exclusive scan of the clamped counts, 8 regions per lane (nreg <= 256)
    const int lane = threadIdx.x;
    int loc[8], sum = 0, over = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int i = lane * 8 + j;
      int c = i < nreg ? s_cnt[i] : 0;
      if (c > region) { over = 1; c = region; }
      loc[j] = c;
      sum += c;
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    int run = incl - sum;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int i = lane * 8 + j;
      if (i < nreg) { s_cnt[i] = loc[j]; s_off[i] = run; }
      run += loc[j];
    }
    over = __any_sync(0xffffffffu, over);
    if (lane == 31) { s_misc[0] = incl; s_misc[1] = over; }
  }
  __syncthreads();
  QueryRegions R;
  R.base = cand + (size_t)q * pool;
  R.region = region;
  R.nreg = nreg;
  R.total = s_misc[0];
  R.over = s_misc[1] != 0;
  R.stage_cap = 0;
  return R;
}

constexpr int kSelStage = 6144;  // candidates staged in shared memory (more: read in place)
constexpr int kSelBins = 1024;

// Copy the candidates into shared memory and return the block-wide min and max
// of v (smem staging when total <= kSelStage).  Thread t takes entries t, t + B,
// ... of the regions' concatenation, four loads in flight at a time; the region
// of an entry is the last one whose prefix offset is <= its position.
__device__ void stage_candidates(const QueryRegions &R, const int *s_cnt, const int *s_off,
                                 uint2 *cs, float *s_red, float *vmin, float *vmax) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const bool stage = R.total <= R.stage_cap;
  float lo = INFINITY, hi = -INFINITY;
  for (int e0 = threadIdx.x; e0 < R.total; e0 += 4 * blockDim.x) {
    uint2 ent[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int e = e0 + u * (int)blockDim.x;
      ent[u] = make_uint2(0u, 0x7fc00000u);  // NaN: ignored by the min and max
      if (e < R.total) {
        int a = 0, b = R.nreg - 1;
        while (a < b) {
          const int mid = (a + b + 1) >> 1;
          if (s_off[mid] <= e) a = mid; else b = mid - 1;
        }
        ent[u] = R.base[(size_t)a * R.region + (e - s_off[a])];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int e = e0 + u * (int)blockDim.x;
      if (e < R.total) {
        const float v = __uint_as_float(ent[u].y);
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
        if (stage) cs[e] = ent[u];
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if (lane == 0) { s_red[warp] = lo; s_red[32 + warp] = hi; }
  __syncthreads();
  lo = INFINITY;
  hi = -INFINITY;
  for (int w = 0; w < nw; w++) { lo = fminf(lo, s_red[w]); hi = fmaxf(hi, s_red[32 + w]); }
  *vmin = lo;
  *vmax = hi;
  __syncthreads();
}

// Apply f(entry) to every candidate (shared-memory copy when staged).
template <class F>
__device__ __forceinline__ void for_each_candidate(const QueryRegions &R, const int *s_cnt,
                                                   const uint2 *cs, F f) {
  if (R.total <= R.stage_cap) {
    for (int e = threadIdx.x; e < R.total; e += blockDim.x) f(cs[e]);
  } else {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int rg = warp; rg < R.nreg; rg += nw) {
      const uint2 *src = R.base + (size_t)rg * R.region;
      const int c = s_cnt[rg];
      for (int e = lane; e < c; e += 32) f(src[e]);
    }
  }
}

// Upper bounds R1 >= the k1-th and R2 >= the k2-th smallest v, each itself the
// value of a candidate of rank >= k1 (k2): values are binned linearly over
// [vmin, vmax]; R is the largest v in the bins up to the one where the running
// count reaches k.  Any such R is a valid threshold (at least k candidates have
// v <= R).  The caller guarantees total >= k1 >= k2 >= 1.
__device__ float2 block_kth_bounds(const QueryRegions &R, const int *s_cnt, const uint2 *cs,
                                   int k1, int k2, float vmin, float vmax, int *hist,
                                   float *s_red, int *s_bin) {
  const float span = vmax - vmin;
  const float scale = span > 0.f ? (float)(kSelBins - 1) / span : 0.f;
  for (int b = threadIdx.x; b < kSelBins; b += blockDim.x) hist[b] = 0;
  __syncthreads();
  auto bin_of = [&](float v) {
    int b = (int)((v - vmin) * scale);
    return b < 0 ? 0 : (b > kSelBins - 1 ? kSelBins - 1 : b);
  };
  for_each_candidate(R, s_cnt, cs, [&](uint2 ent) { atomicAdd(&hist[bin_of(__uint_as_float(ent.y))], 1); });
  __syncthreads();
  if (threadIdx.x < 32) {
    // warp 0: first bins where the running count reaches k1 and k2 (32 bins per lane)
    const int lane = threadIdx.x;
    int sum = 0;
    for (int j = 0; j < kSelBins / 32; j++) sum += hist[lane * (kSelBins / 32) + j];
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const int excl = incl - sum;
#pragma unroll
    for (int w = 0; w < 2; w++) {
      const int kk = w == 0 ? k1 : k2;
      if (excl < kk && incl >= kk) {
        int run = excl, b = lane * (kSelBins / 32);
        for (;; b++) {
          run += hist[b];
          if (run >= kk) break;
        }
        s_bin[w] = b;
      }
    }
  }
  __syncthreads();
  const int kb1 = s_bin[0], kb2 = s_bin[1];
  float m1 = -INFINITY, m2 = -INFINITY;
  for_each_candidate(R, s_cnt, cs, [&](uint2 ent) {
    const float v = __uint_as_float(ent.y);
    const int b = bin_of(v);
    if (b <= kb1) m1 = fmaxf(m1, v);
    if (b <= kb2) m2 = fmaxf(m2, v);
  });
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, o));
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { s_red[64 + warp] = m1; s_red[96 + warp] = m2; }
  __syncthreads();
  float r1 = -INFINITY, r2 = -INFINITY;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) {
    r1 = fmaxf(r1, s_red[64 + w]);
    r2 = fmaxf(r2, s_red[96 + w]);
  }
  __syncthreads();
  return make_float2(r1, r2);
}

struct LevelSelArgs {
  const uint2 *cand;
  const int *ccount;
  const float2 *qinfo;
  int64_t n;
  int k, pool, region;
  int nreg, stride;  // regions of the level and the count-array stride
  int k2;            // shards > 1: ceil(k / shards), else 0
  int stage_cap;     // candidates staged in shared memory (dynamic smem stage_cap * 8)
  float *r_out;      // (n) bound B = R + margin for the next level, +inf when fewer than k;
                     // k2 > 0: then (n) -(R2 + margin), R2 >= the k2-th smallest v
};

// one block per query: R_q for the next level; dynamic smem kSelStage * 8
__global__ void __launch_bounds__(kSelThreads) tc_level_select_kernel(const LevelSelArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint2 *cs = reinterpret_cast<uint2 *>(smem_raw);
  __shared__ int hist[kSelBins], s_cnt[256], s_off[256], s_misc[2], s_bin[2];
  __shared__ float s_red[128];
  const int64_t q = blockIdx.x;
  QueryRegions R = load_regions(a.cand, a.ccount, q, a.pool, a.region, a.nreg, a.stride, s_cnt,
                                s_off, s_misc);
  R.stage_cap = a.stage_cap;
  // entries lost to a full region only make R larger than it could be: still a
  // valid bound, since R is taken over real rows that were kept
  const int k2 = a.k2 > 0 ? a.k2 : a.k;
  float2 r = make_float2(INFINITY, INFINITY);
  if (R.total >= k2) {
    float vmin, vmax;
    stage_candidates(R, s_cnt, s_off, cs, s_red, &vmin, &vmax);
    r = block_kth_bounds(R, s_cnt, cs, min(a.k, R.total), k2, vmin, vmax, hist, s_red, s_bin);
    if (R.total < a.k) r.x = INFINITY;
  }
  // B = R + margin bounds the k-th reference distance minus ||q||^2 from above; the
  // minimum of B over the shards of a sharded search stays a bound.  So does the
  // maximum over the shards of R2 + margin: the shards together hold at least
  // shards * k2 >= k rows below it; it is stored negated, for a MIN reduction.
  if (threadIdx.x == 0) {
    const float m = a.qinfo[q].y;
    a.r_out[q] = __fadd_ru(r.x, m);
    if (a.k2 > 0) a.r_out[a.n + q] = -__fadd_ru(r.y, m);
  }
}

// The kk-th smallest (1-based, kk <= count) of `count` ordered keys in shared
// memory, by one warp: four passes of an 8-bit radix select, most significant digit
// first; `hist` is the warp's own 256 counters.
// Keys at positions >= `staged` are not in shared memory: `more(e)` loads them (each
// pass reads them again).
template <class More>
__device__ uint32_t warp_select_key(const uint32_t *keys, int staged, int count, int kk, int *hist,
                                    More more) {
  const int lane = threadIdx.x & 31;
  uint32_t prefix = 0, mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = lane; b < 256; b += 32) hist[b] = 0;
    __syncwarp();
    for (int e = lane; e < count; e += 32) {
      const uint32_t key = e < staged ? keys[e] : more(e);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
    }
    __syncwarp();
    // the digit whose running count reaches kk (8 bins per lane)
    int sum = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) sum += hist[lane * 8 + j];
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const int excl = incl - sum;
    const unsigned hit = __ballot_sync(0xffffffffu, excl < kk && incl >= kk);
    const int src = __ffs(hit) - 1;
    int dgt = 0, run = 0;
    if (lane == src) {
      run = excl;
      dgt = lane * 8;
      for (;; dgt++) {
        if (run + hist[dgt] >= kk) break;
        run += hist[dgt];
      }
    }
    dgt = __shfl_sync(0xffffffffu, dgt, src);
    run = __shfl_sync(0xffffffffu, run, src);
    prefix |= (uint32_t)dgt << shift;
    kk -= run;
    mask |= 255u << shift;
    __syncwarp();
  }
  return prefix;
}

constexpr int kWarpSelCap = 1024;   // candidates a warp-level select stages per query
constexpr int kWarpSelQueries = 8;  // queries (warps) per block

// Level select of shards that share bounds, one warp per query: each shard holds a
// small share of a query's candidates, so a warp stages up to kWarpSelCap of them
// (as ordered keys of v) and selects the exact k-th and k2-th smallest.  The
// candidates of a query with more are read again from global memory by every pass.  dynamic smem: 8 * (kWarpSelCap + 256 + 256) * 4
__global__ void __launch_bounds__(kSelThreads) tc_level_select_warp_kernel(const LevelSelArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t *keys = reinterpret_cast<uint32_t *>(smem_raw) + warp * kWarpSelCap;
  int *hist = reinterpret_cast<int *>(smem_raw) + kWarpSelQueries * kWarpSelCap + warp * 256;
  int *off = reinterpret_cast<int *>(smem_raw) + kWarpSelQueries * (kWarpSelCap + 256) + warp * 256;
  const int64_t q = (int64_t)blockIdx.x * kWarpSelQueries + warp;
  if (q >= a.n) return;
  // regions' kept counts (clamped to the region size) and their prefix offsets
  int loc[8], sum = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int i = lane * 8 + j;
    int c = i < a.nreg ? a.ccount[(size_t)q * a.stride + i] : 0;
    c = min(c, a.region);
    loc[j] = c;
    sum += c;
  }
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  int run = incl - sum;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int i = lane * 8 + j;
    if (i < a.nreg) off[i] = run;
    run += loc[j];
  }
  const int total = __shfl_sync(0xffffffffu, incl, 31);
  const int staged = min(total, kWarpSelCap);
  __syncwarp();
  const uint2 *base = a.cand + (size_t)q * a.pool;
  for (int e0 = lane; e0 < staged; e0 += 4 * 32) {
    uint2 ent[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int e = e0 + u * 32;
      ent[u] = make_uint2(0u, 0x7fc00000u);
      if (e < staged) {
        int lo = 0, hi = a.nreg - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (off[mid] <= e) lo = mid; else hi = mid - 1;
        }
        ent[u] = base[(size_t)lo * a.region + (e - off[lo])];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int e = e0 + u * 32;
      const float v = __uint_as_float(ent[u].y);
      if (e < staged) keys[e] = v == v ? f2ord(v) : 0xffffffffu;
    }
  }
  __syncwarp();
  auto more = [&](int e) {
    int lo = 0, hi = a.nreg - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (off[mid] <= e) lo = mid; else hi = mid - 1;
    }
    const float v = __uint_as_float(base[(size_t)lo * a.region + (e - off[lo])].y);
    return v == v ? f2ord(v) : 0xffffffffu;
  };
  // R (R2): the k-th (k2-th) smallest v of real candidates; +inf when there are fewer
  float r1 = INFINITY, r2 = INFINITY;
  if (total >= a.k) {
    const uint32_t key = warp_select_key(keys, staged, total, a.k, hist, more);
    if (key != 0xffffffffu) r1 = ord2f(key);
  }
  if (a.k2 > 0 && total >= a.k2) {
    const uint32_t key = warp_select_key(keys, staged, total, a.k2, hist, more);
    if (key != 0xffffffffu) r2 = ord2f(key);
  }
  if (lane == 0) {
    const float m = a.qinfo[q].y;
    a.r_out[q] = __fadd_ru(r1, m);
    if (a.k2 > 0) a.r_out[a.n + q] = -__fadd_ru(r2, m);
  }
}

struct SelArgs {
  const float *Q;
  const float *X;
  int64_t n, m;
  int d, k, pool, region, nreg, stride;
  int64_t id_offset;
  const float2 *qinfo;
  const uint2 *cand;
  const int *ccount;
  const float *r_bound;   // bounds B of the last level (minimised over the shards of a
                          // sharded search)
  bool two_bounds;        // r_bound holds (n) B and (n) -B2
  int *fb_list;       // queries left to the SIMT engine
  WsHeader *hdr;
  float *out_d;
  int32_t *out_i;
};

// Apply f(entry) to every candidate of R read from global memory: thread t takes
// entries t, t + B, ... of the regions' concatenation, four loads in flight at a
// time (the region of an entry: the last whose prefix offset is <= its position).
template <class F>
__device__ __forceinline__ void scan_candidates(const QueryRegions &R, const int *s_off, F f) {
  for (int e0 = threadIdx.x; e0 < R.total; e0 += 4 * blockDim.x) {
    uint2 ent[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int e = e0 + u * (int)blockDim.x;
      ent[u] = make_uint2(0u, 0x7fc00000u);  // NaN: never a survivor
      if (e < R.total) {
        int lo = 0, hi = R.nreg - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (s_off[mid] <= e) lo = mid; else hi = mid - 1;
        }
        ent[u] = R.base[(size_t)lo * R.region + (e - s_off[lo])];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) f(ent[u]);
  }
}

constexpr int kRerankDims = 16;  // dimensions of a survivor row staged at a time

// one block per query; dynamic smem: kSurvCap * 8 (survivor keys) +
// warps * 32 * (kRerankDims + 1) * 4 (row chunks) + d * 4 (query)
__global__ void __launch_bounds__(kSelThreads) tc_final_select_kernel(const SelArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint64_t *keys = reinterpret_cast<uint64_t *>(smem_raw);
  float *rows = reinterpret_cast<float *>(keys + kSurvCap);
  float *qs = rows + (kSelThreads / 32) * 32 * (kRerankDims + 1);
  __shared__ int s_cnt[256], s_off[256], s_misc[2], s_nsurv;
  const int64_t q = blockIdx.x;
  const QueryRegions R = load_regions(a.cand, a.ccount, q, a.pool, a.region, a.nreg, a.stride,
                                      s_cnt, s_off, s_misc);
  // a region that lost entries, or inputs the margin does not cover (exact_only)
  if (R.over || a.hdr->exact_only) {
    if (threadIdx.x == 0) {
      const int slot = atomicAdd(&a.hdr->fallback, 1);
      a.fb_list[slot] = (int)q;
    }
    return;
  }
  for (int c = threadIdx.x; c < a.d; c += blockDim.x) qs[c] = a.Q[q * a.d + c];
  if (threadIdx.x == 0) s_nsurv = 0;
  // B (from the level select of the last level, minimised over the shards of a
  // sharded search) bounds the k-th reference distance minus ||q||^2, so the rows of
  // the top k all have v <= B + margin.  B is +inf when there were fewer than k
  // candidates: then every candidate survives.  A shard returns fewer than k rows
  // when the other shards hold the rest.
  const float theta = __fadd_ru(read_bound(a.r_bound, a.n, q, a.two_bounds), a.qinfo[q].y);
  __syncthreads();
  // survivors: the rows with v <= theta, listed in `keys`
  scan_candidates(R, s_off, [&](uint2 ent) {
    if (__uint_as_float(ent.y) <= theta) {
      const int slot = atomicAdd(&s_nsurv, 1);
      if (slot < kSurvCap) keys[slot] = ent.x;
    }
  });
  __syncthreads();
  const int ns = s_nsurv;
  if (ns > kSurvCap) {
    if (threadIdx.x == 0) {
      const int slot = atomicAdd(&a.hdr->fallback, 1);
      a.fb_list[slot] = (int)q;
    }
    return;
  }
  // Exact distances with the reference arithmetic.  A warp takes 32 survivors
  // at a time, one per lane; their rows pass through shared memory in chunks of
  // kRerankDims dimensions: lanes (j, c) load element c of survivor j's chunk with
  // coalesced reads, and each lane then accumulates its own row in dimension order.
  {
    constexpr int W = kRerankDims, P = kRerankDims + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float *tile = rows + warp * (32 * P);
    for (int b0 = warp * 32; b0 < ns; b0 += nw * 32) {
      const int nb = min(32, ns - b0);
      const uint32_t myrow = lane < nb ? (uint32_t)keys[b0 + lane] : 0u;
      float acc = 0.f;
      const int c = lane % W, j0 = lane / W;  // this lane loads column c of survivors j0, j0+2, ...
      for (int c0 = 0; c0 < a.d; c0 += W) {
        const int cw = min(W, a.d - c0);
        float t[32 / (32 / W)];
#pragma unroll
        for (int u = 0; u < 32 / (32 / W); u++) {
          const int j = j0 + u * (32 / W);
          const uint32_t rj = __shfl_sync(0xffffffffu, myrow, j);
          t[u] = (j < nb && c < cw) ? __ldg(a.X + (size_t)rj * a.d + c0 + c) : 0.f;
        }
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 32 / (32 / W); u++) tile[(j0 + u * (32 / W)) * P + c] = t[u];
        __syncwarp();
        if (lane < nb)
          for (int cc = 0; cc < cw; cc++) acc = dist_step(qs[c0 + cc], tile[lane * P + cc], acc);
      }
      if (lane < nb)
        keys[b0 + lane] = acc == acc ? pair_key(acc, (int32_t)(a.id_offset + myrow)) : ~0ull;
    }
  }
  __syncthreads();
  if (ns <= kRankSortMax) {
    // few survivors: each key's place is the number of keys before it (equal keys,
    // the non-finite distances, order by slot), one pass and no block-wide sort
    for (int e = threadIdx.x; e < ns; e += blockDim.x) {
      const uint64_t key = keys[e];
      int rank = 0;
      for (int j = 0; j < ns; j++) {
        const uint64_t kj = keys[j];
        rank += (kj < key || (kj == key && j < e)) ? 1 : 0;
      }
      if (rank < a.k) {
        const bool pad = key == ~0ull;
        a.out_d[q * a.k + rank] = pad ? BFK_PAD_DIST : ord2f((uint32_t)(key >> 32));
        a.out_i[q * a.k + rank] = pad ? -1 : (int32_t)(uint32_t)(key & 0xffffffffu);
      }
    }
    for (int j = ns + threadIdx.x; j < a.k; j += blockDim.x) {
      a.out_d[q * a.k + j] = BFK_PAD_DIST;
      a.out_i[q * a.k + j] = -1;
    }
  } else {
    int P = 2;
    while (P < ns) P <<= 1;
    for (int e = ns + threadIdx.x; e < P; e += blockDim.x) keys[e] = ~0ull;
    bitonic_sort_u64(keys, P);
    for (int j = threadIdx.x; j < a.k; j += blockDim.x) {
      const uint64_t key = j < ns ? keys[j] : ~0ull;
      const bool pad = key == ~0ull;
      a.out_d[q * a.k + j] = pad ? BFK_PAD_DIST : ord2f((uint32_t)(key >> 32));
      a.out_i[q * a.k + j] = pad ? -1 : (int32_t)(uint32_t)(key & 0xffffffffu);
    }
  }
  if (threadIdx.x == 0) {
    atomicAdd(&a.hdr->survivors, (unsigned long long)ns);
    atomicAdd(&a.hdr->candidates, (unsigned long long)R.total);
    atomicMax(&a.hdr->max_cand, R.total);
  }
}

constexpr int kWarpFinalQueries = 4;   // queries (warps) per block of the warp-level final select
constexpr int kWarpSurvCap = 512;      // survivors a warp re-ranks; more: the SIMT engine

// Final select of shards that share bounds, one warp per query: a shard holds few of
// a query's candidates and fewer survivors, so the block-wide phases of
// tc_final_select_kernel would be mostly waiting.  Same steps, per warp: survivors
// below the shared bound, exact re-rank in dimension order, rank-count ordering.
// dynamic smem: 4 * warp_final_smem(d)
__host__ __device__ inline size_t warp_final_smem(int d) {
  // keys, row chunk, region offsets, query; a multiple of 16 bytes keeps every warp's
  // 64-bit keys aligned
  const size_t b = (size_t)kWarpSurvCap * 8 + 32 * (kRerankDims + 1) * 4 + 256 * 4 + (size_t)d * 4;
  return (b + 15) & ~(size_t)15;
}
__global__ void __launch_bounds__(kWarpFinalQueries * 32) tc_final_select_warp_kernel(const SelArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  constexpr int W = kRerankDims, P = kRerankDims + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t per_warp = warp_final_smem(a.d);
  unsigned char *mine = smem_raw + warp * per_warp;
  uint64_t *keys = reinterpret_cast<uint64_t *>(mine);
  float *tile = reinterpret_cast<float *>(keys + kWarpSurvCap);
  int *off = reinterpret_cast<int *>(tile + 32 * P);
  float *qs = reinterpret_cast<float *>(off + 256);
  const int64_t q = (int64_t)blockIdx.x * kWarpFinalQueries + warp;
  if (q >= a.n) return;
  int loc[8], sum = 0, over = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int i = lane * 8 + j;
    int c = i < a.nreg ? a.ccount[(size_t)q * a.stride + i] : 0;
    if (c > a.region) { over = 1; c = a.region; }
    loc[j] = c;
    sum += c;
  }
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  int run = incl - sum;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int i = lane * 8 + j;
    if (i < a.nreg) off[i] = run;
    run += loc[j];
  }
  const int total = __shfl_sync(0xffffffffu, incl, 31);
  // a region that lost entries, or inputs the margin does not cover (exact_only)
  if (__any_sync(0xffffffffu, over) || a.hdr->exact_only) {
    if (lane == 0) {
      const int slot = atomicAdd(&a.hdr->fallback, 1);
      a.fb_list[slot] = (int)q;
    }
    return;
  }
  for (int c = lane; c < a.d; c += 32) qs[c] = a.Q[q * a.d + c];
  const float theta = __fadd_ru(read_bound(a.r_bound, a.n, q, a.two_bounds), a.qinfo[q].y);
  __syncwarp();
  // survivors, appended in warp order with a ballot per round of 32 entries
  const uint2 *base = a.cand + (size_t)q * a.pool;
  int ns = 0;
  for (int e = lane; e - lane < total; e += 32) {
    bool keep = false;
    uint32_t row = 0;
    if (e < total) {
      int lo = 0, hi = a.nreg - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (off[mid] <= e) lo = mid; else hi = mid - 1;
      }
      const uint2 ent = base[(size_t)lo * a.region + (e - off[lo])];
      keep = __uint_as_float(ent.y) <= theta;
      row = ent.x;
    }
    const unsigned m = __ballot_sync(0xffffffffu, keep);
    const int slot = ns + __popc(m & ((1u << lane) - 1u));
    if (keep && slot < kWarpSurvCap) keys[slot] = row;
    ns += __popc(m);
  }
  if (ns > kWarpSurvCap) {
    if (lane == 0) {
      const int slot = atomicAdd(&a.hdr->fallback, 1);
      a.fb_list[slot] = (int)q;
    }
    return;
  }
  __syncwarp();
  // exact distances: 32 survivors at a time, rows staged in chunks of W dimensions
  for (int b0 = 0; b0 < ns; b0 += 32) {
    const int nb = min(32, ns - b0);
    const uint32_t myrow = lane < nb ? (uint32_t)keys[b0 + lane] : 0u;
    float acc = 0.f;
    const int c = lane % W, j0 = lane / W;
    for (int c0 = 0; c0 < a.d; c0 += W) {
      const int cw = min(W, a.d - c0);
      float t[32 / (32 / W)];
#pragma unroll
      for (int u = 0; u < 32 / (32 / W); u++) {
        const int j = j0 + u * (32 / W);
        const uint32_t rj = __shfl_sync(0xffffffffu, myrow, j);
        t[u] = (j < nb && c < cw) ? __ldg(a.X + (size_t)rj * a.d + c0 + c) : 0.f;
      }
      __syncwarp();
#pragma unroll
      for (int u = 0; u < 32 / (32 / W); u++) tile[(j0 + u * (32 / W)) * P + c] = t[u];
      __syncwarp();
      if (lane < nb)
        for (int cc = 0; cc < cw; cc++) acc = dist_step(qs[c0 + cc], tile[lane * P + cc], acc);
    }
    __syncwarp();
    if (lane < nb) keys[b0 + lane] = acc == acc ? pair_key(acc, (int32_t)(a.id_offset + myrow)) : ~0ull;
  }
  __syncwarp();
  // order by rank counting; equal keys (non-finite distances) order by slot
  for (int e = lane; e < ns; e += 32) {
    const uint64_t key = keys[e];
    int rank = 0;
    for (int j = 0; j < ns; j++) {
      const uint64_t kj = keys[j];
      rank += (kj < key || (kj == key && j < e)) ? 1 : 0;
    }
    if (rank < a.k) {
      const bool pad = key == ~0ull;
      a.out_d[q * a.k + rank] = pad ? BFK_PAD_DIST : ord2f((uint32_t)(key >> 32));
      a.out_i[q * a.k + rank] = pad ? -1 : (int32_t)(uint32_t)(key & 0xffffffffu);
    }
  }
  for (int j = ns + lane; j < a.k; j += 32) {
    a.out_d[q * a.k + j] = BFK_PAD_DIST;
    a.out_i[q * a.k + j] = -1;
  }
  if (lane == 0) {
    atomicAdd(&a.hdr->survivors, (unsigned long long)ns);
    atomicAdd(&a.hdr->candidates, (unsigned long long)total);
    atomicMax(&a.hdr->max_cand, total);
  }
}

// fallback helper: the rows of Q that the final select listed (*count of them)
__global__ void tc_gather_rows(const float *__restrict__ Q, int d, const int *__restrict__ list,
                               const int *__restrict__ count, float *__restrict__ out) {
  const int64_t total = (int64_t)*count * d;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x)
    out[e] = Q[(int64_t)list[e / d] * d + e % d];
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

static int kch_for(int d) { return (d + kBK - 1) / kBK; }

bool tc_supported(int d, int k) {
  if (d <= 0 || d > kMaxKch * kBK || k <= 0 || k > kTcMaxK) return false;
  const TcLayout L = tc_layout(kch_for(d), false);
  return L.ns >= 2 && L.total <= (size_t)kSmemLimit;
}

size_t tc_smem_bytes(int d, int) { return tc_layout(kch_for(d), true).total; }

const void *tc_kernel_ptr(int, int) { return (const void *)knn_tc_filter_kernel<true>; }

int tc_threads() { return kTcThreads; }

static int num_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

// slices for a level of `tiles` tiles: the count (at most `max_s`) whose last wave
// of CTAs is fullest, keeping at least 16 tiles per slice where possible
static int choose_slices(int q_tiles, int64_t tiles, int sms, int max_s) {
  int best = 1;
  double best_score = -1.0;
  for (int s = 1; s <= max_s && s <= tiles; s++) {
    const int64_t tps = (tiles + s - 1) / s;
    const int64_t used = (tiles + tps - 1) / tps;  // slices that get tiles
    if (used != s) continue;
    if (s > 1 && tps < 16) break;
    const int64_t ctas = (int64_t)q_tiles * s;
    const int64_t waves = (ctas + sms - 1) / sms;
    // work per wave slot, counting the last slice's shorter share of tiles
    const double eff = (double)tiles * q_tiles / ((double)waves * sms * tps);
    const double score = eff - 0.0005 * s;  // among equals, fewer and longer slices
    if (score > best_score) { best_score = score; best = s; }
  }
  return best;
}

// Workspace offsets of a plan (its sizes set): every array 256-byte aligned.
static void layout_workspace(TcPlan &P) {
  const int64_t n = P.n, m = P.m;
  const int d = P.d, k = P.k, max_s = P.max_slices;
  const bool prepared = P.prepared;
  const int64_t q_rows = (int64_t)P.q_tiles * kBM;
  size_t off = sizeof(WsHeader);
  // the row arrays live in the workspace unless a prepared buffer holds them
  const size_t rows_f = prepared ? 0 : 1;
  P.off_xh = off;       off = al256(off + rows_f * (size_t)m * P.d_pad * 2);
  P.off_xnorm = off;    off = al256(off + rows_f * (size_t)P.x_tiles * kBN * 4);
  P.off_xscale = off;   off = al256(off + rows_f * (size_t)P.x_tiles * kColGroups * 32);
  P.off_invsq = off;    off = al256(off + 16);
  P.off_qh = off;       off = al256(off + (size_t)q_rows * P.d_pad * 2);
  P.off_qinfo = off;    off = al256(off + (size_t)q_rows * 8);
  P.off_rlev = off;     off = al256(off + (size_t)n * 8);  // two bounds per query
  P.off_cand = off;     off = al256(off + (size_t)n * P.cand_cap * 8);
  P.off_ccount = off;   off = al256(off + (size_t)n * kColGroups * max_s * 4);
  P.off_flags = off;    off = al256(off + (size_t)n * 4);
  P.off_fbq = off;      off = al256(off + (size_t)n * d * 4);
  P.off_fbpart_d = off; off = al256(off + (size_t)P.fb_slices * n * k * 4);
  P.off_fbpart_i = off; off = al256(off + (size_t)P.fb_slices * n * k * 4);
  P.total = off;
}

constexpr int64_t kPairMinRows = 4000000;

bool tc_pair_default(int d, int64_t n, int64_t rows) {
  // CTA pairs halve the row bytes each SM streams.  For short tiles (d <= 256, the query
  // tile resident) they measured faster over 10M rows and 1-2 % slower over 1M-3M rows,
  // so they are the default from kPairMinRows on; they need two query tiles
  return kch_for(d) <= kResidentKch && n > kBM && rows >= kPairMinRows;
}

bool tc_make_plan(int64_t n, int64_t m, int d, int k, int slices, int pool, int pair_mode,
                  int64_t plan_rows, int shards, bool prepared, TcPlan *p) {
  if (!tc_supported(d, k) || n <= 0 || m <= 0) return false;
  TcPlan P{};
  P.n = n;
  P.m = m;
  P.d = d;
  P.k = k;
  P.d_pad = kch_for(d) * kBK;
  P.q_tiles = (int)((n + kBM - 1) / kBM);
  // CTA pairs (M = 256): forced (pair_mode > 0), off (< 0) or by tc_pair_default; they need
  // two query tiles, and the tile count is then even
  // (a sharded search decides on the largest shard's rows, so that all shards agree)
  const bool want = pair_mode > 0 ||
                    (pair_mode == 0 && tc_pair_default(d, n, plan_rows > 0 ? plan_rows : m));
  P.pair = want && P.q_tiles >= 2;
  if (P.pair) P.q_tiles += P.q_tiles & 1;
  P.x_tiles = (m + kBN - 1) / kBN;
  P.cand_cap = pool > 0 ? pool : kDefaultPool;
  if (P.cand_cap < 2 * k) P.cand_cap = 2 * k;

  // level sizes: each level's expected candidates ~ target (the pool holds 5x that)
  // a level's expected candidates: 32 k, between kMinLevelTarget and kLevelTarget (each
  // level keeps about target rows per query; the next level is target / k times larger)
  int64_t target = std::min<int64_t>(kLevelTarget, std::max<int64_t>(kMinLevelTarget, 32 * (int64_t)k));
  if (target < 4 * (int64_t)k) target = 4 * (int64_t)k;
  if (target > P.cand_cap / 4) target = P.cand_cap / 4;
  int64_t ratio = target / k;
  if (ratio < 4) ratio = 4;
  // plan on `basis` tiles (this search's own, or those plan_rows gives, so that the
  // shards of one sharded search get the same number of levels), then map the
  // sample sizes onto this search's tiles
  const int64_t basis = plan_rows > 0 ? (plan_rows + kBN - 1) / kBN : P.x_tiles;
  int64_t sizes[kMaxLevels];
  int nl = 0;
  sizes[nl++] = basis;
  while (nl < kMaxLevels && sizes[nl - 1] * kBN > target) {
    int64_t prev = (sizes[nl - 1] + ratio - 1) / ratio;
    if (prev * kBN < 2 * k) prev = (2 * k + kBN - 1) / kBN;  // the base needs >= k rows
    if (prev >= sizes[nl - 1]) break;
    sizes[nl++] = prev;
  }
  sizes[0] = P.x_tiles;
  for (int l = 1; l < nl; l++) {
    int64_t s = (sizes[l] * P.x_tiles + basis - 1) / basis;
    if (s * kBN < 2 * k) s = (2 * k + kBN - 1) / kBN;
    if (s > sizes[l - 1]) s = sizes[l - 1];
    if (s < 1) s = 1;
    sizes[l] = s;
  }
  // Shards that share bounds keep their own full first level.  Pooling it (each shard
  // sampling 1/shards of it, the shards together as many rows as one search alone) was
  // measured slower: the bound it shares is the largest over the shards of each one's
  // ceil(k / shards)-th value among fewer rows, so the next level keeps about five times
  // the candidates (8 shards of 1.25M rows: that level went from about 0.3 to 1.8 ms).
  (void)shards;
  P.levels = nl;
  const int sms = num_sms();
  int max_s = 1;
  for (int l = 0; l < nl; l++) {
    LevelPlan &lv = P.level[l];
    lv.tiles = sizes[nl - 1 - l];
    const bool last = l == nl - 1;
    // slices fill the SMs with CTAs (a pair counts as two)
    int s = (last && slices > 0) ? slices : choose_slices(P.q_tiles, lv.tiles, sms, 64);
    if (s > lv.tiles) s = (int)lv.tiles;
    if (s < 1) s = 1;
    lv.tiles_per_slice = (lv.tiles + s - 1) / s;
    lv.slices = (int)((lv.tiles + lv.tiles_per_slice - 1) / lv.tiles_per_slice);
    lv.region = P.cand_cap / (kColGroups * lv.slices);
    if (lv.slices > max_s) max_s = lv.slices;
  }
  P.max_slices = max_s;
  P.slices = P.level[nl - 1].slices;
  P.tiles_per_slice = P.level[nl - 1].tiles_per_slice;
  // fallback: the SIMT engine over up to n queries in slices
  P.fb_slices = (int)((m + 262143) / 262144);
  if (P.fb_slices > 32) P.fb_slices = 32;
  if (P.fb_slices < 1) P.fb_slices = 1;
  P.prepared = prepared;
  layout_workspace(P);
  *p = P;
  return true;
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2D f16 tensor map: rows x cols (cols contiguous), box box_rows x 64, 128B swizzle
static bool make_tmap(CUtensorMap *map, const void *base, int64_t rows, int cols_pad,
                      int box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols_pad, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols_pad * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// rows -> f16 in 64-row scale groups, ||x||^2, inverse scales; norm bound and
// exact-only flag (set for a non-finite row) into hdr
static void launch_prep_rows(const float *X, int64_t m, int d, int d_pad, int64_t x_tiles,
                             __half *Xh, float *xnorm, float4 *xmeta, WsHeader *hdr,
                             cudaStream_t stream) {
  const unsigned groups = (unsigned)(x_tiles * kColGroups);  // 64-row scale groups
  const bool vec = (d & 3) == 0 && (reinterpret_cast<uintptr_t>(X) & 15) == 0;
  if (vec && d_pad <= 128)
    tc_prep_x_kernel<true, 1><<<groups, 256, 0, stream>>>(X, m, d, d_pad, Xh, xnorm, xmeta, hdr);
  else if (vec && d_pad <= 256)
    tc_prep_x_kernel<true, 2><<<groups, 256, 0, stream>>>(X, m, d, d_pad, Xh, xnorm, xmeta, hdr);
  else if (vec)
    tc_prep_x_wide_kernel<<<groups, 256, 0, stream>>>(X, m, d, d_pad, Xh, xnorm, xmeta, hdr);
  else
    tc_prep_x_kernel<false, 1><<<groups, 256, 0, stream>>>(X, m, d, d_pad, Xh, xnorm, xmeta, hdr);
}

PreparedLayout tc_prepared_layout(int64_t m, int d) {
  PreparedLayout L{};
  const int d_pad = kch_for(d) * kBK;
  const int64_t x_tiles = (m + kBN - 1) / kBN;
  size_t off = 0;
  L.off_status = off; off = al256(off + sizeof(WsHeader));
  L.off_info = off;   off = al256(off + sizeof(PreparedInfo));
  L.off_xh = off;     off = al256(off + (size_t)m * d_pad * 2);
  L.off_xnorm = off;  off = al256(off + (size_t)x_tiles * kBN * 4);
  L.off_xmeta = off;  off = al256(off + (size_t)x_tiles * kColGroups * 32);
  L.total = off;
  return L;
}

static PreparedInfo prepared_info(int64_t m, int d) {
  PreparedInfo I{};
  memcpy(I.magic, "BFKPREP3", 8);
  I.version = 3;
  I.d = d;
  I.m = m;
  I.d_pad = kch_for(d) * kBK;
  I.x_tiles = (m + kBN - 1) / kBN;
  I.total = tc_prepared_layout(m, d).total;
  return I;
}

int tc_prepare(const float *X, int64_t m, int d, void *prep, cudaStream_t stream) {
  const PreparedLayout L = tc_prepared_layout(m, d);
  unsigned char *pb = static_cast<unsigned char *>(prep);
  WsHeader *status = reinterpret_cast<WsHeader *>(pb + L.off_status);
  const PreparedInfo I = prepared_info(m, d);
  cudaError_t e = cudaMemsetAsync(status, 0, sizeof(WsHeader), stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(pb + L.off_info, &I, sizeof(I), cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess) {
    launch_prep_rows(X, m, d, I.d_pad, I.x_tiles, reinterpret_cast<__half *>(pb + L.off_xh),
                     reinterpret_cast<float *>(pb + L.off_xnorm),
                     reinterpret_cast<float4 *>(pb + L.off_xmeta), status, stream);
    e = cudaGetLastError();
  }
  // the description is copied from this stack frame: wait before returning
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) {
    BFK_NOTE(e, "bfk_prepare");
    return 1;
  }
  return 0;
}

int tc_check_prepared(const void *prep, int64_t m, int d) {
  const PreparedLayout L = tc_prepared_layout(m, d);
  PreparedInfo got{};
  const cudaError_t e = cudaMemcpy(&got, static_cast<const unsigned char *>(prep) + L.off_info,
                                   sizeof(got), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    BFK_NOTE(e, "bfk_search_prepared: reading the description");
    return 1;
  }
  const PreparedInfo want = prepared_info(m, d);
  return memcmp(&got, &want, sizeof(got)) == 0 ? 0 : 3;
}

int tc_run(const float *Q, const float *X, int64_t id_offset, float *out_d, int32_t *out_i,
           void *ws_, const TcPlan &p, cudaStream_t stream, cudaEvent_t t0, cudaEvent_t t1,
           int *launches, LevelHook hook, void *hook_user, int shards, const void *prepared) {
  unsigned char *ws = static_cast<unsigned char *>(ws_);
  WsHeader *hdr = reinterpret_cast<WsHeader *>(ws);
  __half *Xh = reinterpret_cast<__half *>(ws + p.off_xh);
  float *xnorm = reinterpret_cast<float *>(ws + p.off_xnorm);
  float4 *xmeta = reinterpret_cast<float4 *>(ws + p.off_xscale);
  float *inv_sq = reinterpret_cast<float *>(ws + p.off_invsq);
  const unsigned char *pb = static_cast<const unsigned char *>(prepared);
  if (prepared) {
    const PreparedLayout PL = tc_prepared_layout(p.m, p.d);
    Xh = reinterpret_cast<__half *>(const_cast<unsigned char *>(pb) + PL.off_xh);
    xnorm = reinterpret_cast<float *>(const_cast<unsigned char *>(pb) + PL.off_xnorm);
    xmeta = reinterpret_cast<float4 *>(const_cast<unsigned char *>(pb) + PL.off_xmeta);
  }
  __half *Qh = reinterpret_cast<__half *>(ws + p.off_qh);
  float2 *qinfo = reinterpret_cast<float2 *>(ws + p.off_qinfo);
  float *rlev = reinterpret_cast<float *>(ws + p.off_rlev);
  uint2 *cand = reinterpret_cast<uint2 *>(ws + p.off_cand);
  int *ccount = reinterpret_cast<int *>(ws + p.off_ccount);
  int *fb_list = reinterpret_cast<int *>(ws + p.off_flags);
  const int64_t q_rows = (int64_t)p.q_tiles * kBM;
  int nl = 0;

#define BFK_TRY(x)                         \
  do {                                     \
    const cudaError_t e_ = (x);            \
    if (e_ != cudaSuccess) {               \
      BFK_NOTE(e_, #x);                    \
      return 1;                            \
    }                                      \
  } while (0)

  BFK_TRY(cudaMemsetAsync(hdr, 0, sizeof(WsHeader), stream));
  // pass 0: prep
  tc_qmax_kernel<<<592, 256, 0, stream>>>(Q, p.n * p.d, hdr);
  if (prepared) {
    // the rows' norm bound and exact-only flag, as their preparation found them
    const PreparedLayout PL = tc_prepared_layout(p.m, p.d);
    tc_take_row_status<<<1, 32, 0, stream>>>(
        reinterpret_cast<const WsHeader *>(pb + PL.off_status), hdr);
  } else {
    launch_prep_rows(X, p.m, p.d, p.d_pad, p.x_tiles, Xh, xnorm, xmeta, hdr, stream);
  }
  tc_prep_q_kernel<<<(unsigned)(q_rows / 8), 256, 0, stream>>>(Q, p.n, p.d, p.d_pad, q_rows, Qh,
                                                                qinfo, inv_sq, hdr);
  nl += 3;
  BFK_TRY(cudaGetLastError());

  CUtensorMap tq, tx;
  // a CTA of a pair loads half of every row tile
  if (!make_tmap(&tq, Qh, q_rows, p.d_pad, kBM) ||
      !make_tmap(&tx, Xh, p.m, p.d_pad, p.pair ? kBN / 2 : kBN)) {
    BFK_NOTE(cudaErrorInvalidValue, "cuTensorMapEncodeTiled");
    return 1;
  }
  const int kch = p.d_pad / kBK;
  const size_t smem = tc_layout(kch, p.pair).total;
  const void *filter = p.pair ? (const void *)knn_tc_filter_kernel<true>
                              : (const void *)knn_tc_filter_kernel<false>;
  BFK_TRY(cudaFuncSetAttribute(filter, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int stage_cap = kSelStage;
  const size_t lsmem = (size_t)stage_cap * 8;
  BFK_TRY(cudaFuncSetAttribute((const void *)tc_level_select_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lsmem));
  const size_t wsmem = (size_t)kWarpSelQueries * (kWarpSelCap + 512) * 4;
  BFK_TRY(cudaFuncSetAttribute((const void *)tc_level_select_warp_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsmem));
  FilterArgs A{};
  A.xnorm = xnorm;
  A.xmeta = xmeta;
  A.qinfo = qinfo;
  A.inv_sq = inv_sq;
  A.n = p.n;
  A.x_tiles = p.x_tiles;
  A.q_tiles = p.q_tiles;
  A.pool = p.cand_cap;
  A.max_slices = p.max_slices;
  A.cand = cand;
  A.ccount = ccount;
  A.hdr = hdr;
  // shards that share bounds also share a second one per query (see tc_level_select_kernel)
  const bool two = hook != nullptr && shards > 1;
  for (int l = 0; l < p.levels; l++) {
    const LevelPlan &lv = p.level[l];
    const bool last = l == p.levels - 1;
    A.r_in = l == 0 ? nullptr : rlev;
    A.two_bounds = two;
    A.level_tiles = lv.tiles;
    A.slices = lv.slices;
    A.tiles_per_slice = (int)lv.tiles_per_slice;
    A.region = lv.region;
    if (last && t0) cudaEventRecord(t0, stream);
    if (p.pair) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(p.q_tiles * lv.slices));
      cfg.blockDim = dim3(kTcThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      BFK_TRY(cudaLaunchKernelEx(&cfg, knn_tc_filter_kernel<true>, tq, tx, A, kch));
    } else {
      knn_tc_filter_kernel<false><<<(unsigned)(p.q_tiles * lv.slices), kTcThreads, smem, stream>>>(
          tq, tx, A, kch);
    }
    if (last && t1) cudaEventRecord(t1, stream);
    nl++;
    BFK_TRY(cudaGetLastError());
    // after the last level too: the final select keeps the rows below its bound (on a
    // sharded search, the bound shared by all shards: rows that can be in the global top-k)
    {
      LevelSelArgs S{};
      S.cand = cand;
      S.ccount = ccount;
      S.qinfo = qinfo;
      S.n = p.n;
      S.k = p.k;
      S.pool = p.cand_cap;
      S.region = lv.region;
      S.nreg = kColGroups * lv.slices;  // regions: column groups of every slice
      S.stride = kColGroups * p.max_slices;
      S.r_out = rlev;
      S.k2 = two ? (p.k + shards - 1) / shards : 0;
      S.stage_cap = stage_cap;
      if (two)
        tc_level_select_warp_kernel<<<(unsigned)((p.n + kWarpSelQueries - 1) / kWarpSelQueries),
                                      kSelThreads, wsmem, stream>>>(S);
      else
        tc_level_select_kernel<<<(unsigned)p.n, kSelThreads, lsmem, stream>>>(S);
      nl++;
      BFK_TRY(cudaGetLastError());
      // a sharded search replaces each query's bound by the minimum over all shards
      if (hook) hook(rlev, two ? 2 * p.n : p.n, hook_user, stream);
    }
  }

  // final select + exact re-rank
  const LevelPlan &lv = p.level[p.levels - 1];
  SelArgs S{};
  S.Q = Q;
  S.X = X;
  S.n = p.n;
  S.m = p.m;
  S.d = p.d;
  S.k = p.k;
  S.pool = p.cand_cap;
  S.region = lv.region;
  S.nreg = kColGroups * lv.slices;  // regions: column groups of every slice
  S.stride = kColGroups * p.max_slices;
  S.id_offset = id_offset;
  S.qinfo = qinfo;
  S.cand = cand;
  S.ccount = ccount;
  S.r_bound = rlev;
  S.two_bounds = two;
  S.fb_list = fb_list;
  S.hdr = hdr;
  S.out_d = out_d;
  S.out_i = out_i;
  const size_t ssmem = (size_t)kSurvCap * 8 +
                       (size_t)(kSelThreads / 32) * 32 * (kRerankDims + 1) * 4 + (size_t)p.d * 4;
  BFK_TRY(cudaFuncSetAttribute((const void *)tc_final_select_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssmem));
  if (two) {
    const size_t wfsmem = (size_t)kWarpFinalQueries * warp_final_smem(p.d);
    BFK_TRY(cudaFuncSetAttribute((const void *)tc_final_select_warp_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wfsmem));
    tc_final_select_warp_kernel<<<(unsigned)((p.n + kWarpFinalQueries - 1) / kWarpFinalQueries),
                                  kWarpFinalQueries * 32, wfsmem, stream>>>(S);
  } else {
    tc_final_select_kernel<<<(unsigned)p.n, kSelThreads, ssmem, stream>>>(S);
  }
  nl++;
  BFK_TRY(cudaGetLastError());

  // Queries the filter could not finish -> exact SIMT engine.  Their count stays on the
  // device: the three kernels below run whether or not there are any (they return at
  // once for none), so the host never waits for the stream here.
  {
    float *Qf = reinterpret_cast<float *>(ws + p.off_fbq);
    float *pd = reinterpret_cast<float *>(ws + p.off_fbpart_d);
    int32_t *pi = reinterpret_cast<int32_t *>(ws + p.off_fbpart_i);
    const int *count = &hdr->fallback;
    const int64_t part_entries = (int64_t)p.fb_slices * p.n * p.k;
    tc_gather_rows<<<256, 256, 0, stream>>>(Q, p.d, fb_list, count, Qf);
    BFK_TRY(cudaGetLastError());
    BFK_TRY(launch_direct_count(Qf, count, X, p.m, p.d, p.k, id_offset, part_entries, pd, pi,
                                stream));
    BFK_TRY(launch_merge_count(pd, pi, count, p.m, p.k, part_entries, fb_list, out_d, out_i,
                               stream));
    nl += 4;
  }
  *launches = nl;
  return 0;
#undef BFK_TRY
}

// ---------------------------------------------------------------------------
// The filter value v of every (query, row) pair, for the margin audit (test
// infrastructure).  One level reads every tile with no bound, so the filter's
// first-level path appends every finite v; regions hold a slice's every column.
// ---------------------------------------------------------------------------
__global__ void tc_scatter_values(const uint2 *__restrict__ cand, const int *__restrict__ ccount,
                                  int64_t m, int pool, int region, int nreg, int stride,
                                  float *__restrict__ out_v) {
  const int64_t q = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int rg = warp; rg < nreg; rg += nw) {
    const int c = min(ccount[(size_t)q * stride + rg], region);
    const uint2 *src = cand + (size_t)q * pool + (size_t)rg * region;
    for (int e = lane; e < c; e += 32) {
      const uint2 ent = src[e];
      if (ent.x < (uint64_t)m) out_v[q * m + ent.x] = __uint_as_float(ent.y);
    }
  }
}

bool tc_make_values_plan(int64_t n, int64_t m, int d, TcPlan *p) {
  if (!tc_supported(d, 1) || n <= 0 || m <= 0) return false;
  TcPlan P{};
  P.n = n;
  P.m = m;
  P.d = d;
  P.k = 1;
  P.d_pad = kch_for(d) * kBK;
  P.q_tiles = (int)((n + kBM - 1) / kBM);
  P.x_tiles = (m + kBN - 1) / kBN;
  P.levels = 1;
  LevelPlan &lv = P.level[0];
  lv.tiles = P.x_tiles;
  int s = choose_slices(P.q_tiles, lv.tiles, num_sms(), 64);
  if (s > lv.tiles) s = (int)lv.tiles;
  lv.tiles_per_slice = (lv.tiles + s - 1) / s;
  lv.slices = (int)((lv.tiles + lv.tiles_per_slice - 1) / lv.tiles_per_slice);
  lv.region = (int)(lv.tiles_per_slice * kGroupN);  // a column group's every column
  P.cand_cap = lv.slices * kColGroups * lv.region;
  P.max_slices = lv.slices;
  P.slices = lv.slices;
  P.tiles_per_slice = lv.tiles_per_slice;
  P.fb_slices = 1;
  P.prepared = false;
  layout_workspace(P);
  *p = P;
  return true;
}

int tc_filter_values(const float *Q, const float *X, float *out_v, float *out_qinfo,
                     int *exact_only, void *ws_, const TcPlan &p, cudaStream_t stream) {
  unsigned char *ws = static_cast<unsigned char *>(ws_);
  WsHeader *hdr = reinterpret_cast<WsHeader *>(ws);
  __half *Xh = reinterpret_cast<__half *>(ws + p.off_xh);
  float *xnorm = reinterpret_cast<float *>(ws + p.off_xnorm);
  float4 *xmeta = reinterpret_cast<float4 *>(ws + p.off_xscale);
  float *inv_sq = reinterpret_cast<float *>(ws + p.off_invsq);
  __half *Qh = reinterpret_cast<__half *>(ws + p.off_qh);
  float2 *qinfo = reinterpret_cast<float2 *>(ws + p.off_qinfo);
  uint2 *cand = reinterpret_cast<uint2 *>(ws + p.off_cand);
  int *ccount = reinterpret_cast<int *>(ws + p.off_ccount);
  const int64_t q_rows = (int64_t)p.q_tiles * kBM;
  const LevelPlan &lv = p.level[0];
#define BFK_TRY(x)                         \
  do {                                     \
    const cudaError_t e_ = (x);            \
    if (e_ != cudaSuccess) {               \
      BFK_NOTE(e_, #x);                    \
      return 1;                            \
    }                                      \
  } while (0)
  BFK_TRY(cudaMemsetAsync(hdr, 0, sizeof(WsHeader), stream));
  // NaN (all bits set) marks a pair the filter did not report
  BFK_TRY(cudaMemsetAsync(out_v, 0xff, (size_t)p.n * p.m * sizeof(float), stream));
  tc_qmax_kernel<<<592, 256, 0, stream>>>(Q, p.n * p.d, hdr);
  launch_prep_rows(X, p.m, p.d, p.d_pad, p.x_tiles, Xh, xnorm, xmeta, hdr, stream);
  tc_prep_q_kernel<<<(unsigned)(q_rows / 8), 256, 0, stream>>>(Q, p.n, p.d, p.d_pad, q_rows, Qh,
                                                                qinfo, inv_sq, hdr);
  BFK_TRY(cudaGetLastError());
  CUtensorMap tq, tx;
  if (!make_tmap(&tq, Qh, q_rows, p.d_pad, kBM) || !make_tmap(&tx, Xh, p.m, p.d_pad, kBN)) {
    BFK_NOTE(cudaErrorInvalidValue, "cuTensorMapEncodeTiled");
    return 1;
  }
  const int kch = p.d_pad / kBK;
  const size_t smem = tc_layout(kch, false).total;
  BFK_TRY(cudaFuncSetAttribute((const void *)knn_tc_filter_kernel<false>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  FilterArgs A{};
  A.xnorm = xnorm;
  A.xmeta = xmeta;
  A.qinfo = qinfo;
  A.inv_sq = inv_sq;
  A.r_in = nullptr;  // no bound: every finite v is appended
  A.two_bounds = false;
  A.n = p.n;
  A.x_tiles = p.x_tiles;
  A.level_tiles = lv.tiles;
  A.q_tiles = p.q_tiles;
  A.slices = lv.slices;
  A.tiles_per_slice = (int)lv.tiles_per_slice;
  A.region = lv.region;
  A.pool = p.cand_cap;
  A.max_slices = p.max_slices;
  A.cand = cand;
  A.ccount = ccount;
  A.hdr = hdr;
  knn_tc_filter_kernel<false><<<(unsigned)(p.q_tiles * lv.slices), kTcThreads, smem, stream>>>(
      tq, tx, A, kch);
  BFK_TRY(cudaGetLastError());
  tc_scatter_values<<<(unsigned)p.n, 256, 0, stream>>>(cand, ccount, p.m, p.cand_cap, lv.region,
                                                       kColGroups * lv.slices,
                                                       kColGroups * p.max_slices, out_v);
  BFK_TRY(cudaGetLastError());
  // (||q||^2, margin) of each query: the first n float2 of qinfo
  BFK_TRY(cudaMemcpyAsync(out_qinfo, qinfo, (size_t)p.n * sizeof(float2),
                          cudaMemcpyDeviceToDevice, stream));
  WsHeader h;
  BFK_TRY(cudaMemcpyAsync(&h, hdr, sizeof(h), cudaMemcpyDeviceToHost, stream));
  BFK_TRY(cudaStreamSynchronize(stream));
  *exact_only = h.exact_only;
  return h.error ? 2 : 0;
#undef BFK_TRY
}

}  // namespace bfk
