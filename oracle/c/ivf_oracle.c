/* C port of the reference's IVF search (test infrastructure and timed CPU
 * baseline only; never part of the product path).
 *
 *  - coarse step: pairwise_L2sqr (python/metalfaiss/distances.py:140-173) in fp32,
 *    (||q||^2 + ||c||^2) - (q.c + q.c) clamped at 0, then the nprobe smallest in
 *    ascending order, ties to the lower centroid (a stable sort).
 *  - list scan: ivf_list_topk_l2 (python/metalfaiss/faissmlx/kernels/ivf_kernels.py:43-50):
 *    acc = fma(x - q, x - q, acc) over j in order; candidates in probe order,
 *    then row order; top-k by insertion, ties keep the earlier candidate.
 *  - padding: (+inf, -1) past the candidates.
 * Queries run in parallel over OpenMP threads; each query is sequential.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static void insert_topk(float* vd, int64_t* vi, int* n, int k, float d, int64_t id) {
  if (*n == k && !(d < vd[k - 1])) return;
  int p = (*n < k) ? (*n)++ : k - 1;
  while (p > 0 && d < vd[p - 1]) {
    vd[p] = vd[p - 1];
    vi[p] = vi[p - 1];
    --p;
  }
  vd[p] = d;
  vi[p] = id;
}

void mfo_coarse(const float* xq, int64_t nq, const float* cents, int nlist, int d, int nprobe,
                int64_t* probes, int threads) {
  float* cn = (float*)malloc(sizeof(float) * (size_t)nlist);
  for (int c = 0; c < nlist; ++c) {
    float s = 0.f;
    for (int j = 0; j < d; ++j) s += cents[(size_t)c * d + j] * cents[(size_t)c * d + j];
    cn[c] = s;
  }
  int P = nprobe < nlist ? nprobe : nlist;
#pragma omp parallel for num_threads(threads) schedule(dynamic, 1)
  for (int64_t q = 0; q < nq; ++q) {
    const float* x = xq + (size_t)q * d;
    float qn = 0.f;
    for (int j = 0; j < d; ++j) qn += x[j] * x[j];
    float* bd = (float*)malloc(sizeof(float) * (size_t)P);
    int64_t* bi = (int64_t*)malloc(sizeof(int64_t) * (size_t)P);
    int n = 0;
    for (int c = 0; c < nlist; ++c) {
      const float* y = cents + (size_t)c * d;
      float dot = 0.f;
      for (int j = 0; j < d; ++j) dot += x[j] * y[j];
      float dist = (qn + cn[c]) - (dot + dot);
      if (dist < 0.f) dist = 0.f;
      insert_topk(bd, bi, &n, P, dist, c);
    }
    for (int t = 0; t < P; ++t) probes[(size_t)q * P + t] = t < n ? bi[t] : -1;
    free(bd);
    free(bi);
  }
  free(cn);
}

void mfo_ivf_scan(const float* xq, int64_t nq, const int64_t* probes, int nprobe,
                  const int64_t* offsets, const float* vecs, const int64_t* ids, int d, int k,
                  float* D, int64_t* I, int threads) {
#pragma omp parallel for num_threads(threads) schedule(dynamic, 1)
  for (int64_t q = 0; q < nq; ++q) {
    const float* x = xq + (size_t)q * d;
    float* vd = D + (size_t)q * k;
    int64_t* vi = I + (size_t)q * k;
    int n = 0;
    for (int p = 0; p < nprobe; ++p) {
      int64_t l = probes[(size_t)q * nprobe + p];
      if (l < 0) continue;
      for (int64_t r = offsets[l]; r < offsets[l + 1]; ++r) {
        const float* y = vecs + (size_t)r * d;
        float acc = 0.f;
        for (int j = 0; j < d; ++j) {
          float diff = y[j] - x[j];
          acc = fmaf(diff, diff, acc);
        }
        insert_topk(vd, vi, &n, k, acc, ids[r]);
      }
    }
    for (int t = n; t < k; ++t) {
      vd[t] = INFINITY;
      vi[t] = -1;
    }
  }
}
