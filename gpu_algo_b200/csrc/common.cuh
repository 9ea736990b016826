// Shared device helpers for the bfknn kernels (sm_100a).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#define BFK_PAD_DIST 3.402823e+38f

namespace bfk {

// ---------------------------------------------------------------------------
// Workspace header: the first 256 bytes of every workspace.
// ---------------------------------------------------------------------------
struct WsHeader {
  int32_t error;          // device status word: 0 ok, else an ErrCode below
  uint32_t rx_bits;       // max row norm of X (float bits, positive => ordered as uint)
  uint32_t qmax_bits;     // max |Q| (float bits)
  int32_t exact_only;     // the filter cannot be trusted (a non-finite norm, or norms
                          // outside its range): every query goes to the exact SIMT engine
  int32_t fallback;       // queries routed to the exact SIMT engine
  int32_t max_cand;       // max candidates of one query
  uint32_t ex_bits;       // max over rows of ||x - f16 form of x|| (float bits, rounded up)
  int32_t pad0;
  unsigned long long candidates;  // total candidates appended by the filter
  unsigned long long survivors;   // total rows re-ranked exactly
  int32_t pad[52];
};
static_assert(sizeof(WsHeader) == 256, "header is 256 bytes");

enum ErrCode : int32_t {
  ERR_NONE = 0,
  ERR_TIMEOUT_PRODUCER = 1,
  ERR_TIMEOUT_MMA = 2,
  ERR_TIMEOUT_EPILOGUE = 3,
};

// ---------------------------------------------------------------------------
// Ordering helpers.
// ---------------------------------------------------------------------------
// float -> uint32 whose unsigned order equals the float order (no NaN input)
__device__ __forceinline__ uint32_t f2ord(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord2f(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}
// 64-bit key ordered by (distance, index); padding = all ones
__device__ __forceinline__ uint64_t pair_key(float d, int32_t i) {
  if (i < 0) return ~0ull;
  return ((uint64_t)f2ord(d) << 32) | (uint32_t)i;
}
__device__ __forceinline__ bool pair_lt(float da, int32_t ia, float db, int32_t ib) {
  return da < db || (da == db && ia < ib);
}

// Insert (d, gid) into the sorted list (ld, li) of length cnt <= k; warp-collective.
__device__ __forceinline__ void warp_insert(float *ld, int32_t *li, int &cnt, int k, float d,
                                            int32_t gid, int lane) {
  int p = 0;
  for (int b = 0; b < cnt; b += 32) {
    int e = b + lane;
    bool lt = e < cnt && pair_lt(ld[e], li[e], d, gid);
    p += __popc(__ballot_sync(0xffffffffu, lt));
  }
  const int newcnt = cnt + 1 < k ? cnt + 1 : k;
  for (int top = newcnt - 1; top > p; top -= 32) {
    int e = top - lane;
    bool act = e > p;
    float td = 0.f;
    int32_t ti = 0;
    if (act) { td = ld[e - 1]; ti = li[e - 1]; }
    __syncwarp();
    if (act) { ld[e] = td; li[e] = ti; }
    __syncwarp();
  }
  if (lane == 0) { ld[p] = d; li[p] = gid; }
  __syncwarp();
  cnt = newcnt;
}

// Database slices of the exact fallback for `count` queries: as many as its partial
// lists (part_entries entries) hold, at most 512 and one per 1024 rows, at least one.
__host__ __device__ inline int64_t fallback_slices(int64_t count, int64_t m, int k,
                                                   int64_t part_entries) {
  int64_t s = count > 0 ? part_entries / (count * (int64_t)k) : 1;
  if (s > 512) s = 512;
  if (s > (m + 1023) / 1024) s = (m + 1023) / 1024;
  return s < 1 ? 1 : s;
}

// The reference kernels' distance step (bf/fp32.py:80), spelled out so that
// no other contraction can happen: dif = q - x (rounded), acc = fma(dif, dif, acc).
__device__ __forceinline__ float dist_step(float q, float x, float acc) {
  float dif = __fsub_rn(q, x);
  return __fmaf_rn(dif, dif, acc);
}

// ---------------------------------------------------------------------------
// Bounded waiting: every spin on the device gives up after a wall-clock limit,
// records an error code in the workspace header and lets the kernel return.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s; a healthy wait is microseconds

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait that suspends the thread until the phase completes or `hint_ns` passes,
// so a waiting warp takes no issue slots from the warps that share its scheduler
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
constexpr uint32_t kWaitSliceNs = 20000;  // one suspended try_wait; the limits are checked between
// Returns false when the limit ran out or `abort_flag` was raised by another role.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  volatile int *abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, kWaitSliceNs)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// non-blocking test of a phase
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait of the single-thread roles whose reaction time is on the tensor pipe's critical
// path (the TMA producer and the MMA issuer): tests the phase without suspending the
// thread; the abort flag and the wall-clock limit are checked every 256 tests.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t *bar, uint32_t parity,
                                               volatile int *abort_flag) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    for (int i = 0; i < 256; i++)
      if (mbar_test_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}
// try_wait with relaxed semantics: no acquire ordering of this thread's later memory
// operations after the phase.
__device__ __forceinline__ bool mbar_try_wait_relaxed(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.relaxed.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_relaxed(uint64_t *bar, uint32_t parity,
                                                  volatile int *abort_flag) {
  if (mbar_try_wait_relaxed(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    for (int i = 0; i < 16; i++)
      if (mbar_try_wait_relaxed(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}
// The same with try_wait and no time hint (the hardware's own suspend limit).
__device__ __forceinline__ bool mbar_wait_try(uint64_t *bar, uint32_t parity,
                                              volatile int *abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    for (int i = 0; i < 16; i++)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// ---------------------------------------------------------------------------
// TMA (2D tiled loads, no multicast) and bulk copies
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const void *tmap, uint64_t *bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, accumulators in tensor memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16, cta_group::1
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` once every previously issued tcgen05.mma of this thread has completed
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// 32 lanes x 32 consecutive columns of 32-bit data: thread i gets lane (base+i), columns c..c+31
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// The wait, with the loaded registers as operands: the compiler cannot move a use of
// them above it (the load writes them asynchronously).
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (clusters of two SMs sharing one tcgen05.mma.cta_group::2)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// every thread of both CTAs arrives and waits
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// 2D tiled load into this CTA's shared memory whose completion is counted on the
// barrier at the same offset in the pair's even (MMA-issuing) CTA; no multicast
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const void *tmap, uint64_t *bar,
                                                 int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar) & 0xFEFFFFFFu), "r"(x), "r"(y)
      : "memory");
}
// arrive on the barrier at the same offset in CTA `rank` of the cluster.  The arrive
// releases at CTA scope (the default): the waiting thread needs only the order of the
// arriving thread's tensor-memory reads (fenced by tcgen05.fence::before_thread_sync),
// not its global stores, which a cluster-scope release would first wait for.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t *bar, uint32_t rank) {
  asm volatile(
      "{\n\t.reg .b32 ra;\n\t"
      "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
      "mbarrier.arrive.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_u32(bar)),
      "r"(rank)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D[tmem of both CTAs] (+)= A (M split over the pair) * B (N split over the pair)^T
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive (once per CTA in `mask`) on the barrier at this offset when the pair's
// previously issued MMAs have completed
__device__ __forceinline__ void tc_commit_pair_mc(uint64_t *bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor, K-major operand, 128-byte swizzle: rows of
// 128 bytes, 8-row groups 1024 bytes apart.  `addr` must sit in a
// 1024-byte-aligned swizzle atom (plus a K offset of a multiple of 32 bytes).
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t addr) {
  uint64_t desc = 0;
  desc |= (uint64_t)((addr >> 4) & 0x3FFFu);          // start address  [0,14)
  desc |= (uint64_t)1u << 16;                          // LBO (unused for SW128 K-major) [16,30)
  desc |= (uint64_t)(1024u >> 4) << 32;                // SBO = 1024 B   [32,46)
  desc |= (uint64_t)1u << 46;                          // descriptor version (sm_100) [46,48)
  desc |= (uint64_t)2u << 61;                          // layout: SWIZZLE_128B [61,64)
  return desc;
}

// a descriptor from its two 32-bit words
__device__ __forceinline__ uint64_t desc_from(uint32_t lo, uint32_t hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
  return d;
}

// Instruction descriptor for kind::f16: f16 x f16 -> f32, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4)                        // D format: F32
         | (0u << 7)                      // A format: F16
         | (0u << 10)                     // B format: F16
         | ((uint32_t)(N >> 3) << 17)     // N / 8
         | ((uint32_t)(M >> 4) << 24);    // M / 16
}

}  // namespace bfk
