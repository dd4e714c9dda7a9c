/*
 * LAPACK CPU baseline for the batched SPD solve — TEST / BENCH INFRASTRUCTURE.
 *
 * The reference's own CPU comparator is MLX's CPU stream, which calls LAPACK
 * (benchmarks/bench_linalg.py:92-93 uses mx.linalg.solve(..., stream=mx.cpu);
 * src/mlx_addons/linalg/_det.py:30 uses mx.linalg.lu_factor(stream=mx.cpu)).
 * MLX is not available here, so this harness calls the LAPACK that ships in
 * the image (numpy's OpenBLAS, ILP64 symbols) directly: spotrf + spotrs per
 * matrix, logdet = 2 sum log diag L, with the batch split over host threads
 * and OpenBLAS itself kept single-threaded. Function pointers are resolved by
 * the caller (oracle/__init__.py), so nothing links against OpenBLAS here.
 *
 * Row-major input: the lower triangle of a row-major matrix is the upper
 * triangle of its column-major view, so uplo = 'U' yields the row-major
 * lower factor L.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef void (*potrf_fn)(const char *uplo, const int64_t *n, float *a, const int64_t *lda,
                         int64_t *info, size_t uplo_len);
typedef void (*potrs_fn)(const char *uplo, const int64_t *n, const int64_t *nrhs, const float *a,
                         const int64_t *lda, float *b, const int64_t *ldb, int64_t *info,
                         size_t uplo_len);

typedef struct {
  potrf_fn potrf;
  potrs_fn potrs;
  const float *A, *b;
  float *x, *logdet;
  int64_t lo, hi;
  int n, m;
  int64_t bad;
} lap_job;

static void *lap_run(void *p) {
  lap_job *j = (lap_job *)p;
  const int n = j->n, m = j->m;
  const int64_t nn = (int64_t)n * n;
  float *a = (float *)malloc((size_t)nn * sizeof(float));
  float *rhs = (float *)malloc((size_t)n * (m > 0 ? m : 1) * sizeof(float));
  const char uplo = 'U';
  const int64_t N = n, M = m;
  for (int64_t i = j->lo; i < j->hi; i++) {
    memcpy(a, j->A + i * nn, (size_t)nn * sizeof(float));
    int64_t info = 0;
    j->potrf(&uplo, &N, a, &N, &info, 1);
    if (info != 0) j->bad++;
    if (m > 0) {
      /* row-major (n x m) b -> column-major (n x m) */
      const float *bi = j->b + i * (int64_t)n * m;
      for (int r = 0; r < n; r++)
        for (int c = 0; c < m; c++) rhs[(size_t)c * n + r] = bi[(size_t)r * m + c];
      j->potrs(&uplo, &N, &M, a, &N, rhs, &N, &info, 1);
      float *xi = j->x + i * (int64_t)n * m;
      for (int r = 0; r < n; r++)
        for (int c = 0; c < m; c++) xi[(size_t)r * m + c] = rhs[(size_t)c * n + r];
    }
    if (j->logdet) {
      float s = 0.0f;
      for (int d = 0; d < n; d++) s += logf(a[(size_t)d * n + d]);
      j->logdet[i] = 2.0f * s;
    }
  }
  free(a);
  free(rhs);
  return NULL;
}

/* Returns the number of matrices LAPACK reported as not positive definite. */
int64_t lapack_posv_batch(void *potrf, void *potrs, const float *A, const float *b, float *x,
                          float *logdet, int64_t B, int n, int m, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 512) nthreads = 512;
  if ((int64_t)nthreads > B) nthreads = B > 0 ? (int)B : 1;
  lap_job jobs[512];
  pthread_t th[512];
  for (int t = 0; t < nthreads; t++) {
    lap_job jb = {(potrf_fn)potrf, (potrs_fn)potrs, A, b, x, logdet,
                  B * t / nthreads, B * (t + 1) / nthreads, n, m, 0};
    jobs[t] = jb;
  }
  for (int t = 1; t < nthreads; t++) pthread_create(&th[t], NULL, lap_run, &jobs[t]);
  lap_run(&jobs[0]);
  int64_t bad = jobs[0].bad;
  for (int t = 1; t < nthreads; t++) {
    pthread_join(th[t], NULL);
    bad += jobs[t].bad;
  }
  return bad;
}
