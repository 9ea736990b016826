/*
 * CPU oracle for exact brute-force k-NN (TEST INFRASTRUCTURE ONLY).
 *
 * This file is the checker: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it.  The product path never calls it.
 *
 * It restates the arithmetic of the reference kernels in plain C:
 *   - distance: bf/fp32.py:74-82 (and the identical loops in
 *     bf/fp32_heap.py:90-101, bf/fp32_tiled.py:66-77, bf/fp32_qgroup.py:85-103,
 *     bf/fp32_q2.py:72-90):
 *         float dist = 0.f;
 *         for (di = 0; di < D; di++) { float dif = q[di] - x[di]; dist += dif*dif; }
 *     NVRTC/nvcc contract `dist += dif*dif` into one fused multiply-add, so the
 *     per-dimension step is acc = fmaf(dif, dif, acc), strictly in order
 *     di = 0 .. d-1.  The oracle reproduces that order exactly (it vectorises
 *     across database rows, never across d).
 *   - selection: the k smallest squared distances per query, output ascending
 *     (bf/fp32.py:39-44 sorts ascending); ties are ordered by the lower row
 *     index; missing slots (m < k) are padded with 3.402823e38f and -1
 *     (bf/fp32.py:71, bf/fp32_heap.py:103-107).
 *   - rows whose distance is NaN are never returned (the reference's strict
 *     `dist < lmax` test rejects them once a list is full; the oracle rejects
 *     them always, which is the defined behaviour of this engine).
 *   - a distance that overflowed to +inf is a value: such rows come last and
 *     are returned when fewer than k rows are finite, as the general kernel's
 *     heap_push (bf/fp32.py:8-27) keeps any distance while its list is not
 *     full (the small-k kernel, bf/fp32.py:100-112, drops them instead).
 *   - merge of sorted per-shard lists: bf/fp32_tiled.py:118-178 (the
 *     reference's merge re-inserts every partial with heap_push; here the
 *     lists are merged under the same (distance, index) order).
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define PAD_DIST 3.402823e+38f
#define ROWS_PER_BLOCK 16

typedef struct {
  float d;
  int32_t i;
} pair_t;

/* (d, i) lexicographic "greater than" */
static inline int pair_gt(pair_t a, pair_t b) {
  return (a.d > b.d) || (a.d == b.d && a.i > b.i);
}

/* bounded max-heap of the k smallest pairs */
static void heap_sift_down(pair_t *h, int n, int p) {
  for (;;) {
    int l = 2 * p + 1, r = l + 1, g = p;
    if (l < n && pair_gt(h[l], h[g])) g = l;
    if (r < n && pair_gt(h[r], h[g])) g = r;
    if (g == p) return;
    pair_t t = h[p]; h[p] = h[g]; h[g] = t;
    p = g;
  }
}

static void heap_sift_up(pair_t *h, int c) {
  while (c > 0) {
    int p = (c - 1) / 2;
    if (!pair_gt(h[c], h[p])) return;
    pair_t t = h[p]; h[p] = h[c]; h[c] = t;
    c = p;
  }
}

static inline void heap_offer(pair_t *h, int *n, int k, float d, int32_t i) {
  if (d != d) return; /* NaN: never returned */
  pair_t p = {d, i};
  if (*n < k) {
    h[*n] = p;
    heap_sift_up(h, *n);
    (*n)++;
  } else if (pair_gt(h[0], p)) {
    h[0] = p;
    heap_sift_down(h, k, 0);
  }
}

static int pair_cmp(const void *a, const void *b) {
  pair_t x = *(const pair_t *)a, y = *(const pair_t *)b;
  if (pair_gt(x, y)) return 1;
  if (pair_gt(y, x)) return -1;
  return 0;
}

static void heap_emit(pair_t *h, int n, int k, float *out_d, int32_t *out_i) {
  qsort(h, (size_t)n, sizeof(pair_t), pair_cmp);
  for (int j = 0; j < k; j++) {
    if (j < n) { out_d[j] = h[j].d; out_i[j] = h[j].i; }
    else { out_d[j] = PAD_DIST; out_i[j] = -1; }
  }
}

/* One distance with the reference's exact operation order. */
float oracle_ref_dist(const float *q, const float *x, int32_t d) {
  float acc = 0.f;
  for (int32_t i = 0; i < d; i++) {
    float dif = q[i] - x[i];
    acc = fmaf(dif, dif, acc);
  }
  return acc;
}

/* All n*m distances (row-major (n, m)); small cases only. */
void oracle_all_dists(const float *Q, int64_t n, const float *X, int64_t m, int32_t d,
                      float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t qi = 0; qi < n; qi++)
    for (int64_t j = 0; j < m; j++)
      out[qi * m + j] = oracle_ref_dist(Q + qi * d, X + j * d, d);
}

/*
 * Exact top-k.  Q (n, d) and X (m, d) row-major float32.  Row indices are
 * reported as id_offset + row.  Returns 0 on success, -1 on bad arguments.
 */
int oracle_knn(const float *Q, int64_t n, const float *X, int64_t m, int32_t d, int32_t k,
               int64_t id_offset, float *out_d, int32_t *out_i, int32_t nthreads) {
  if (n < 0 || m < 0 || d <= 0 || k <= 0) return -1;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
  int bad = 0;
#pragma omp parallel
  {
    pair_t *heap = (pair_t *)malloc(sizeof(pair_t) * (size_t)k);
    float *xt = (float *)malloc(sizeof(float) * (size_t)d * ROWS_PER_BLOCK);
    if (!heap || !xt) {
#pragma omp atomic write
      bad = 1;
    } else {
#pragma omp for schedule(dynamic, 1)
      for (int64_t q0 = 0; q0 < n; q0 += 8) {
        int64_t q1 = q0 + 8 < n ? q0 + 8 : n;
        for (int64_t qi = q0; qi < q1; qi++) {
          const float *q = Q + qi * d;
          int hn = 0;
          for (int64_t r0 = 0; r0 < m; r0 += ROWS_PER_BLOCK) {
            int nr = (int)((m - r0) < ROWS_PER_BLOCK ? (m - r0) : ROWS_PER_BLOCK);
            /* transpose the row block so the inner loop runs across rows */
            for (int r = 0; r < nr; r++)
              for (int32_t c = 0; c < d; c++)
                xt[(size_t)c * ROWS_PER_BLOCK + r] = X[(r0 + r) * d + c];
            for (int r = nr; r < ROWS_PER_BLOCK; r++)
              for (int32_t c = 0; c < d; c++) xt[(size_t)c * ROWS_PER_BLOCK + r] = 0.f;
            float acc[ROWS_PER_BLOCK];
            for (int r = 0; r < ROWS_PER_BLOCK; r++) acc[r] = 0.f;
            for (int32_t c = 0; c < d; c++) {
              const float qc = q[c];
              const float *xc = xt + (size_t)c * ROWS_PER_BLOCK;
              for (int r = 0; r < ROWS_PER_BLOCK; r++) {
                float dif = qc - xc[r];
                acc[r] = fmaf(dif, dif, acc[r]);
              }
            }
            for (int r = 0; r < nr; r++)
              heap_offer(heap, &hn, k, acc[r], (int32_t)(id_offset + r0 + r));
          }
          heap_emit(heap, hn, k, out_d + qi * k, out_i + qi * k);
        }
      }
    }
    free(heap);
    free(xt);
  }
  return bad ? -1 : 0;
}

/*
 * Merge `lists` sorted (distance, index) lists of length k per query
 * (layout (lists, n, k)) into the k smallest per query.  Entries with index
 * -1 are padding and are skipped.
 */
int oracle_merge(const float *cand_d, const int32_t *cand_i, int64_t n, int32_t lists, int32_t k,
                 float *out_d, int32_t *out_i) {
  if (n < 0 || lists <= 0 || k <= 0) return -1;
  int bad = 0;
#pragma omp parallel
  {
    pair_t *heap = (pair_t *)malloc(sizeof(pair_t) * (size_t)k);
    if (!heap) {
#pragma omp atomic write
      bad = 1;
    } else {
#pragma omp for schedule(static)
      for (int64_t qi = 0; qi < n; qi++) {
        int hn = 0;
        for (int32_t l = 0; l < lists; l++) {
          const float *dd = cand_d + ((int64_t)l * n + qi) * k;
          const int32_t *ii = cand_i + ((int64_t)l * n + qi) * k;
          for (int32_t j = 0; j < k; j++)
            if (ii[j] >= 0) heap_offer(heap, &hn, k, dd[j], ii[j]);
        }
        heap_emit(heap, hn, k, out_d + qi * k, out_i + qi * k);
      }
    }
    free(heap);
  }
  return bad ? -1 : 0;
}
