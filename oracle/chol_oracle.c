/*
 * CPU oracle for the batched SPD Cholesky-solve path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product (mlx_addons_b200/) links,
 * loads or calls this file. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py use it, as the checker and
 * as the timed CPU baseline ("port").
 *
 * Plain-C restatement of guillaume-osmo/mlx-addons `mlx_addons.linalg`
 * (paths relative to the reference project root):
 *   - unblocked left-looking Cholesky with the sqrt(max(s, 1e-12)) pivot clamp
 *     and the multiply-by-1/Ljj column scaling:
 *       src/mlx_addons/linalg/_metal_kernels.py:36-50  (tier ST, k <= 32)
 *       src/mlx_addons/linalg/_metal_kernels.py:161-180 (tier TG, 33..80)
 *       src/mlx_addons/linalg/_metal_kernels.py:311    (tier LG = ST source)
 *     The three tiers do the same float operations in the same order, so one
 *     routine restates all of them.
 *   - forward / back substitution by division, and triu_solve meaning L^T x = b:
 *       _metal_kernels.py:52-71, :103-141, :187-205, :248-304
 *   - the 80-wide blocked factorisation (potrf -> TRSM via tril_solve of A_ij^T
 *     -> full-GEMM trailing update) and the blocked substitution:
 *       src/mlx_addons/linalg/_blocked.py:31, :34-137, :140-217
 *   - logdet_spd = 2 * sum(log(diag L)): src/mlx_addons/linalg/_det.py:51-67
 *   - solve_lu (LU with partial pivoting, non-SPD): _metal_kernels.py:701-969
 *   - Householder qr: _metal_kernels.py:319-473, :641-694
 *   - slogdet via LU with partial pivoting (MLX mx.linalg.lu_factor on the CPU
 *     stream, i.e. LAPACK sgetrf): _det.py:17-48. The third-party algorithm
 *     is LAPACK xGETF2 (first max |a_ij| as pivot, swap, scale, rank-1 update);
 *     MLX is an unpinned dependency (pyproject.toml: mlx>=0.20.0).
 *
 * Compile with -ffp-contract=off so every multiply and add rounds separately,
 * exactly as written.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_CLAMP 1e-12f
#define ORC_QR_SHARED_K_MAX 63 /* _metal_kernels.py:383 */
#define ORC_BLOCK 80 /* _blocked.py:31  BLOCK_SIZE = SHARED_K_MAX (= 80) */

/* ------------------------------------------------------------------------ */
/* Unblocked kernels (one matrix, leading dimension ld)                      */
/* ------------------------------------------------------------------------ */

/* Left-looking Cholesky in place on the lower triangle of L; the strict upper
 * triangle is neither read nor written (_metal_kernels.py:36-50). */
static void chol_unblocked(float *L, int k, int ld) {
  for (int j = 0; j < k; j++) {
    float s = L[(size_t)j * ld + j];
    for (int p = 0; p < j; p++) {
      float v = L[(size_t)j * ld + p];
      s -= v * v;
    }
    L[(size_t)j * ld + j] = sqrtf(fmaxf(s, ORC_CLAMP));
    float inv = 1.0f / L[(size_t)j * ld + j];
    for (int i = j + 1; i < k; i++) {
      float t = L[(size_t)i * ld + j];
      for (int p = 0; p < j; p++) t -= L[(size_t)i * ld + p] * L[(size_t)j * ld + p];
      L[(size_t)i * ld + j] = t * inv;
    }
  }
}

/* L y = b for one right-hand-side vector y (in place), _metal_kernels.py:57-62. */
static void fwd_vec(const float *L, int k, int ld, float *y) {
  for (int i = 0; i < k; i++) {
    float t = y[i];
    for (int p = 0; p < i; p++) t -= L[(size_t)i * ld + p] * y[p];
    y[i] = t / L[(size_t)i * ld + i];
  }
}

/* L^T x = y (in place), _metal_kernels.py:63-68 and :132-137. */
static void bwd_vec(const float *L, int k, int ld, float *y) {
  for (int i = k - 1; i >= 0; i--) {
    float t = y[i];
    for (int p = i + 1; p < k; p++) t -= L[(size_t)p * ld + i] * y[p];
    y[i] = t / L[(size_t)i * ld + i];
  }
}

/* Column-by-column triangular solve of a (k x m) row-major RHS block with
 * leading dimension ldb; mode 0 = L x = b, 1 = L^T x = b, 2 = both (fused
 * Cholesky solve). y is scratch of length k. */
static void trsm_cols(const float *L, int k, int ld, const float *b, float *x,
                      int m, int ldb, int mode, float *y) {
  for (int col = 0; col < m; col++) {
    for (int i = 0; i < k; i++) y[i] = b[(size_t)i * ldb + col];
    if (mode == 0 || mode == 2) fwd_vec(L, k, ld, y);
    if (mode == 1 || mode == 2) bwd_vec(L, k, ld, y);
    for (int i = 0; i < k; i++) x[(size_t)i * ldb + col] = y[i];
  }
}

static void zero_upper(float *L, int k, int ld) {
  for (int i = 0; i < k; i++)
    for (int j = i + 1; j < k; j++) L[(size_t)i * ld + j] = 0.0f;
}

/* ------------------------------------------------------------------------ */
/* Blocked factorisation, _blocked.py:34-137                                 */
/* ------------------------------------------------------------------------ */

/* work: n*n scratch (becomes the running trailing matrix); L: n*n output with
 * the upper triangle zeroed; y: scratch of length >= ORC_BLOCK. */
static void chol_blocked(const float *A, float *L, int n, float *work, float *y) {
  memcpy(work, A, (size_t)n * n * sizeof(float));
  memset(L, 0, (size_t)n * n * sizeof(float));
  const int B = ORC_BLOCK;
  int nblocks = (n + B - 1) / B;
  for (int j = 0; j < nblocks; j++) {
    int j0 = j * B, bj = (n - j0 < B) ? n - j0 : B;
    /* 1. small Cholesky of the diagonal block; upper zeroed (_blocked.py:80-84,
     * _metal_kernels.py:98-99 / :242-245). */
    for (int r = 0; r < bj; r++)
      memcpy(&L[(size_t)(j0 + r) * n + j0], &work[(size_t)(j0 + r) * n + j0], bj * sizeof(float));
    chol_unblocked(&L[(size_t)j0 * n + j0], bj, n);
    zero_upper(&L[(size_t)j0 * n + j0], bj, n);
    /* 2. TRSM: L_ij = tril_solve(L_jj, A_ij^T)^T, i.e. every row of A_ij is a
     * right-hand side of a forward substitution (_blocked.py:88-96). */
    for (int i0 = j0 + bj; i0 < n; i0++) {
      for (int p = 0; p < bj; p++) y[p] = work[(size_t)i0 * n + j0 + p];
      fwd_vec(&L[(size_t)j0 * n + j0], bj, n, y);
      for (int p = 0; p < bj; p++) L[(size_t)i0 * n + j0 + p] = y[p];
    }
    /* 3. trailing update work -= L_col L_col^T (_blocked.py:100-121). Only the
     * lower triangle of work is ever read again, so only it is updated. */
    int r0 = j0 + bj;
    for (int r = r0; r < n; r++) {
      const float *lr = &L[(size_t)r * n + j0];
      for (int c = r0; c <= r; c++) {
        const float *lc = &L[(size_t)c * n + j0];
        float u = 0.0f;
        for (int p = 0; p < bj; p++) u += lr[p] * lc[p];
        work[(size_t)r * n + c] = work[(size_t)r * n + c] - u;
      }
    }
  }
}

/* Blocked substitution, _blocked.py:166-213. b, x: n*m row-major; t: n*m
 * scratch for y; y: scratch of length >= ORC_BLOCK. */
static void solve_blocked(const float *L, int n, const float *b, float *x, int m,
                          float *t, float *y) {
  const int B = ORC_BLOCK;
  int nblocks = (n + B - 1) / B;
  /* forward: rhs = b_i - sum_{j<i} L_ij @ y_j ; y_i = tril_solve(L_ii, rhs) */
  for (int i = 0; i < nblocks; i++) {
    int i0 = i * B, bi = (n - i0 < B) ? n - i0 : B;
    for (int r = 0; r < bi; r++)
      for (int c = 0; c < m; c++) t[(size_t)(i0 + r) * m + c] = b[(size_t)(i0 + r) * m + c];
    for (int j = 0; j < i; j++) {
      int j0 = j * B, bj = (n - j0 < B) ? n - j0 : B;
      for (int r = 0; r < bi; r++)
        for (int c = 0; c < m; c++) {
          float u = 0.0f;
          for (int p = 0; p < bj; p++) u += L[(size_t)(i0 + r) * n + j0 + p] * t[(size_t)(j0 + p) * m + c];
          t[(size_t)(i0 + r) * m + c] = t[(size_t)(i0 + r) * m + c] - u;
        }
    }
    trsm_cols(&L[(size_t)i0 * n + i0], bi, n, &t[(size_t)i0 * m], &t[(size_t)i0 * m], m, m, 0, y);
  }
  /* backward: rhs = y_i - sum_{j>i} L_ji^T @ x_j ; x_i = triu_solve(L_ii, rhs) */
  for (int i = nblocks - 1; i >= 0; i--) {
    int i0 = i * B, bi = (n - i0 < B) ? n - i0 : B;
    for (int r = 0; r < bi; r++)
      for (int c = 0; c < m; c++) x[(size_t)(i0 + r) * m + c] = t[(size_t)(i0 + r) * m + c];
    for (int j = i + 1; j < nblocks; j++) {
      int j0 = j * B, bj = (n - j0 < B) ? n - j0 : B;
      for (int r = 0; r < bi; r++)
        for (int c = 0; c < m; c++) {
          float u = 0.0f;
          for (int p = 0; p < bj; p++) u += L[(size_t)(j0 + p) * n + i0 + r] * x[(size_t)(j0 + p) * m + c];
          x[(size_t)(i0 + r) * m + c] = x[(size_t)(i0 + r) * m + c] - u;
        }
    }
    trsm_cols(&L[(size_t)i0 * n + i0], bi, n, &x[(size_t)i0 * m], &x[(size_t)i0 * m], m, m, 1, y);
  }
}

/* 2 * sum(log(diag L)) (_det.py:65-67). */
static float logdet_from_L(const float *L, int n, int ld) {
  float s = 0.0f;
  for (int j = 0; j < n; j++) s += logf(L[(size_t)j * ld + j]);
  return 2.0f * s;
}

/* LU with partial pivoting, LAPACK xGETF2 semantics (first index of max |.|,
 * swap only when the pivot is non-zero, scale by the reciprocal when
 * |pivot| >= FLT_MIN, else divide), then the sign / log|det| of _det.py:30-46:
 * sign = (-1)^{#(piv[j] != j)} * prod sign(U_jj), logabsdet = sum log|U_jj|. */
static void slogdet_one(float *a, int n, float *sign_out, float *lad_out) {
  int swaps = 0;
  for (int j = 0; j < n; j++) {
    int p = j;
    float best = fabsf(a[(size_t)j * n + j]);
    for (int i = j + 1; i < n; i++) {
      float v = fabsf(a[(size_t)i * n + j]);
      if (v > best) { best = v; p = i; }
    }
    if (p != j) swaps++;
    if (a[(size_t)p * n + j] != 0.0f) {
      if (p != j)
        for (int c = 0; c < n; c++) {
          float tmp = a[(size_t)j * n + c];
          a[(size_t)j * n + c] = a[(size_t)p * n + c];
          a[(size_t)p * n + c] = tmp;
        }
      float piv = a[(size_t)j * n + j];
      if (fabsf(piv) >= 1.17549435e-38f) {
        float r = 1.0f / piv;
        for (int i = j + 1; i < n; i++) a[(size_t)i * n + j] *= r;
      } else {
        for (int i = j + 1; i < n; i++) a[(size_t)i * n + j] /= piv;
      }
    }
    for (int i = j + 1; i < n; i++) {
      float lij = a[(size_t)i * n + j];
      for (int c = j + 1; c < n; c++) a[(size_t)i * n + c] -= lij * a[(size_t)j * n + c];
    }
  }
  float sg = (swaps & 1) ? -1.0f : 1.0f, lad = 0.0f;
  for (int j = 0; j < n; j++) {
    float u = a[(size_t)j * n + j];
    sg *= (u > 0.0f) ? 1.0f : ((u < 0.0f) ? -1.0f : 0.0f);
    lad += logf(fabsf(u));
  }
  *sign_out = sg;
  *lad_out = lad;
}

/* solve_lu (_metal_kernels.py:917-969; kernels _LU_SOLVE_SRC :701-768 and
 * _LU_SOLVE_LG_SRC :849-914, identical arithmetic): LU with partial pivoting
 * where the pivot is the FIRST row whose |a_ij| beats a running maximum that
 * starts at 0 (so an all-zero column keeps row j), full-row swap when the
 * pivot row differs, and, only for a non-zero pivot, the column scaled by the
 * reciprocal 1/pivot followed by the rank-1 update (:717-738). The solve
 * applies the recorded swaps to each right-hand side in order, then a unit-
 * lower forward and an upper backward substitution, each row accumulating
 * its terms in increasing column order and the backward step dividing by
 * U_ii (:741-767). a (n x n) is overwritten with LU; y has n floats. */
static void lu_solve_one(float *a, int n, const float *b, float *x, int m, int *piv, float *y) {
  for (int j = 0; j < n; j++) {
    float max_val = 0.0f;
    int max_row = j;
    for (int i = j; i < n; i++) {
      float v = a[(size_t)i * n + j];
      float av = v < 0 ? -v : v;
      if (av > max_val) { max_val = av; max_row = i; }
    }
    piv[j] = max_row;
    if (max_row != j)
      for (int c = 0; c < n; c++) {
        float tmp = a[(size_t)j * n + c];
        a[(size_t)j * n + c] = a[(size_t)max_row * n + c];
        a[(size_t)max_row * n + c] = tmp;
      }
    float diag = a[(size_t)j * n + j];
    if (diag != 0.0f) {
      float inv_diag = 1.0f / diag;
      for (int i = j + 1; i < n; i++) {
        a[(size_t)i * n + j] *= inv_diag;
        for (int c = j + 1; c < n; c++) a[(size_t)i * n + c] -= a[(size_t)i * n + j] * a[(size_t)j * n + c];
      }
    }
  }
  for (int col = 0; col < m; col++) {
    for (int i = 0; i < n; i++) y[i] = b[(size_t)i * m + col];
    for (int i = 0; i < n; i++) {
      int pi = piv[i];
      if (pi != i) { float tmp = y[i]; y[i] = y[pi]; y[pi] = tmp; }
    }
    for (int i = 1; i < n; i++)
      for (int p = 0; p < i; p++) y[i] -= a[(size_t)i * n + p] * y[p];
    for (int i = n - 1; i >= 0; i--) {
      for (int p = i + 1; p < n; p++) y[i] -= a[(size_t)i * n + p] * y[p];
      y[i] /= a[(size_t)i * n + i];
    }
    for (int i = 0; i < n; i++) x[(size_t)i * m + col] = y[i];
  }
}

/* qr (_metal_kernels.py:641-694; kernels _QR_SRC :319-381 and _QR_TG_SRC
 * :385-473, identical arithmetic): Householder QR of a square matrix. Column
 * j: sigma = sum_{i>=j} r_ij^2 (in order), norm = sqrt(max(sigma, 1e-30)),
 * v = (r_jj + s*norm, r_{j+1,j}, ...) with s = +1 when r_jj >= 0 else -1,
 * tau = 2 / v.v (0 when v.v <= 1e-30); Q <- Q (I - tau v v^T) row by row and
 * R <- (I - tau v v^T) R for the columns right of j, with the products
 * grouped as (tau * dot) * v_i and (tau * v_i) * dot exactly as written
 * (:343-366); then r_jj = -s * norm and the column below it zeroed.
 * lapack_tail: above k = 63 the reference runs LAPACK on the CPU stream
 * (:685-688), whose reflector generator (xLARFG) leaves a column alone when
 * everything below its diagonal is exactly zero (tau = 0, r_jj kept): the
 * last column of a square matrix always. Otherwise both generate the same
 * reflector (beta = -sign(alpha) * norm). */
static void qr_one(const float *A, float *Q, float *R, int n, int lapack_tail) {
  memcpy(R, A, (size_t)n * n * sizeof(float));
  for (int i = 0; i < n; i++)
    for (int j = 0; j < n; j++) Q[(size_t)i * n + j] = (i == j) ? 1.0f : 0.0f;
  for (int j = 0; j < n; j++) {
    if (lapack_tail) {
      int zero_tail = 1;
      for (int i = j + 1; i < n; i++) zero_tail &= (R[(size_t)i * n + j] == 0.0f);
      if (zero_tail) continue;
    }
    float sigma = 0.0f;
    for (int i = j; i < n; i++) {
      float v = R[(size_t)i * n + j];
      sigma += v * v;
    }
    float norm_x = sqrtf(fmaxf(sigma, 1e-30f));
    float x_jj = R[(size_t)j * n + j];
    float sgn = (x_jj >= 0.0f) ? 1.0f : -1.0f;
    float v_head = x_jj + sgn * norm_x;
    float vtv = v_head * v_head;
    for (int i = j + 1; i < n; i++) {
      float vi = R[(size_t)i * n + j];
      vtv += vi * vi;
    }
    float tau = (vtv > 1e-30f) ? (2.0f / vtv) : 0.0f;
    for (int row = 0; row < n; row++) {
      float dot = Q[(size_t)row * n + j] * v_head;
      for (int i = j + 1; i < n; i++) dot += Q[(size_t)row * n + i] * R[(size_t)i * n + j];
      Q[(size_t)row * n + j] -= tau * dot * v_head;
      for (int i = j + 1; i < n; i++) Q[(size_t)row * n + i] -= tau * dot * R[(size_t)i * n + j];
    }
    for (int col = j + 1; col < n; col++) {
      float dot = v_head * R[(size_t)j * n + col];
      for (int i = j + 1; i < n; i++) dot += R[(size_t)i * n + j] * R[(size_t)i * n + col];
      R[(size_t)j * n + col] -= tau * v_head * dot;
      for (int i = j + 1; i < n; i++) R[(size_t)i * n + col] -= tau * R[(size_t)i * n + j] * dot;
    }
    R[(size_t)j * n + j] = -sgn * norm_x;
    for (int i = j + 1; i < n; i++) R[(size_t)i * n + j] = 0.0f;
  }
}

/* ------------------------------------------------------------------------ */
/* Batch driver over host threads                                            */
/* ------------------------------------------------------------------------ */

enum { OP_CHOL = 0, OP_CHOL_SMALL, OP_SOLVE, OP_SOLVE_SMALL, OP_TRIL, OP_TRIU,
       OP_LOGDET, OP_SLOGDET, OP_LU_SOLVE, OP_QR };

typedef struct {
  int op;
  const float *A, *b;
  float *out, *out2, *out3;
  int64_t B;
  int n, m;
  int64_t lo, hi;
} job_t;

static void run_range(job_t *j) {
  const int n = j->n, m = j->m;
  const size_t nn = (size_t)n * n, nm = (size_t)n * m;
  float *work = NULL, *L = NULL, *t = NULL, *y = NULL;
  work = (float *)malloc(nn * sizeof(float) + 16);
  L = (float *)malloc(nn * sizeof(float) + 16);
  t = (float *)malloc((nm ? nm : 1) * sizeof(float) + 16);
  y = (float *)malloc((size_t)(n > ORC_BLOCK ? n : ORC_BLOCK) * sizeof(float) + 16);
  int *ipiv = (int *)malloc((size_t)(n ? n : 1) * sizeof(int));
  for (int64_t i = j->lo; i < j->hi; i++) {
    const float *A = j->A + (size_t)i * nn;
    switch (j->op) {
      case OP_CHOL: /* blocked_cholesky (+ optional logdet), _blocked.py:34 */
      case OP_LOGDET: {
        float *Lo = (j->op == OP_CHOL) ? j->out + (size_t)i * nn : L;
        if (n <= ORC_BLOCK) {
          memcpy(Lo, A, nn * sizeof(float));
          chol_unblocked(Lo, n, n);
          zero_upper(Lo, n, n);
        } else {
          chol_blocked(A, Lo, n, work, y);
        }
        if (j->op == OP_LOGDET) j->out[i] = logdet_from_L(Lo, n, n);
        else if (j->out2) j->out2[i] = logdet_from_L(Lo, n, n);
        break;
      }
      case OP_CHOL_SMALL: { /* _metal_kernels.cholesky, any k, unblocked */
        float *Lo = j->out + (size_t)i * nn;
        memcpy(Lo, A, nn * sizeof(float));
        chol_unblocked(Lo, n, n);
        zero_upper(Lo, n, n);
        break;
      }
      case OP_SOLVE: { /* blocked_solve, _blocked.py:140 */
        const float *b = j->b + (size_t)i * nm;
        float *x = j->out + (size_t)i * nm;
        if (n <= ORC_BLOCK) {
          memcpy(L, A, nn * sizeof(float));
          chol_unblocked(L, n, n);
          trsm_cols(L, n, n, b, x, m, m, 2, work);
        } else {
          chol_blocked(A, L, n, work, y);
          solve_blocked(L, n, b, x, m, t, y);
        }
        if (j->out2) j->out2[i] = logdet_from_L(L, n, n);
        break;
      }
      case OP_SOLVE_SMALL: { /* _metal_kernels.solve, fused, unblocked */
        const float *b = j->b + (size_t)i * nm;
        float *x = j->out + (size_t)i * nm;
        memcpy(L, A, nn * sizeof(float));
        chol_unblocked(L, n, n);
        trsm_cols(L, n, n, b, x, m, m, 2, work);
        if (j->out2) j->out2[i] = logdet_from_L(L, n, n);
        break;
      }
      case OP_TRIL:
      case OP_TRIU: {
        const float *b = j->b + (size_t)i * nm;
        float *x = j->out + (size_t)i * nm;
        trsm_cols(A, n, n, b, x, m, m, j->op == OP_TRIL ? 0 : 1, work);
        break;
      }
      case OP_SLOGDET: {
        memcpy(work, A, nn * sizeof(float));
        slogdet_one(work, n, &j->out[i], &j->out2[i]);
        break;
      }
      case OP_LU_SOLVE: {
        memcpy(work, A, nn * sizeof(float));
        lu_solve_one(work, n, j->b + (size_t)i * nm, j->out + (size_t)i * nm, m, ipiv, y);
        break;
      }
      case OP_QR: {
        qr_one(A, j->out + (size_t)i * nn, j->out2 + (size_t)i * nn, n, n > ORC_QR_SHARED_K_MAX);
        break;
      }
    }
  }
  free(work); free(L); free(t); free(y); free(ipiv);
}

static void *thread_main(void *p) { run_range((job_t *)p); return NULL; }

static int run_parallel(job_t base, int nthreads) {
  if (base.B < 0 || base.n < 0 || base.m < 0) return 1;
  if (base.B == 0) return 0;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 512) nthreads = 512;
  if ((int64_t)nthreads > base.B) nthreads = (int)base.B;
  job_t jobs[512];
  pthread_t th[512];
  for (int t = 0; t < nthreads; t++) {
    jobs[t] = base;
    jobs[t].lo = base.B * t / nthreads;
    jobs[t].hi = base.B * (t + 1) / nthreads;
  }
  for (int t = 1; t < nthreads; t++) pthread_create(&th[t], NULL, thread_main, &jobs[t]);
  run_range(&jobs[0]);
  for (int t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Exported entry points (called through ctypes from oracle/__init__.py)     */
/* ------------------------------------------------------------------------ */

/* cholesky = blocked_cholesky (linalg/__init__.py:49); logdet may be NULL. */
int orc_cholesky(const float *A, float *L, float *logdet, int64_t B, int n, int nthreads) {
  job_t j = {OP_CHOL, A, NULL, L, logdet, NULL, B, n, 0, 0, 0};
  return run_parallel(j, nthreads);
}

/* _metal_kernels.cholesky without the k <= 128 limit (unblocked). */
int orc_cholesky_small(const float *A, float *L, int64_t B, int n, int nthreads) {
  job_t j = {OP_CHOL_SMALL, A, NULL, L, NULL, NULL, B, n, 0, 0, 0};
  return run_parallel(j, nthreads);
}

/* solve = blocked_solve (linalg/__init__.py:48); logdet may be NULL. */
int orc_solve(const float *A, const float *b, float *x, float *logdet, int64_t B, int n, int m, int nthreads) {
  job_t j = {OP_SOLVE, A, b, x, logdet, NULL, B, n, m, 0, 0};
  return run_parallel(j, nthreads);
}

/* _metal_kernels.solve (= solve_cholesky) without the k <= 128 limit. */
int orc_solve_small(const float *A, const float *b, float *x, float *logdet, int64_t B, int n, int m, int nthreads) {
  job_t j = {OP_SOLVE_SMALL, A, b, x, logdet, NULL, B, n, m, 0, 0};
  return run_parallel(j, nthreads);
}

int orc_tril_solve(const float *L, const float *b, float *x, int64_t B, int k, int m, int nthreads) {
  job_t j = {OP_TRIL, L, b, x, NULL, NULL, B, k, m, 0, 0};
  return run_parallel(j, nthreads);
}

int orc_triu_solve(const float *L, const float *b, float *x, int64_t B, int k, int m, int nthreads) {
  job_t j = {OP_TRIU, L, b, x, NULL, NULL, B, k, m, 0, 0};
  return run_parallel(j, nthreads);
}

int orc_logdet_spd(const float *A, float *logdet, int64_t B, int n, int nthreads) {
  job_t j = {OP_LOGDET, A, NULL, logdet, NULL, NULL, B, n, 0, 0, 0};
  return run_parallel(j, nthreads);
}

int orc_slogdet(const float *A, float *sign, float *logabsdet, int64_t B, int n, int nthreads) {
  job_t j = {OP_SLOGDET, A, NULL, sign, logabsdet, NULL, B, n, 0, 0, 0};
  return run_parallel(j, nthreads);
}

/* solve_lu (_metal_kernels.py:917-969) without its k <= 128 limit. */
int orc_lu_solve(const float *A, const float *b, float *x, int64_t B, int n, int m, int nthreads) {
  job_t j = {OP_LU_SOLVE, A, b, x, NULL, NULL, B, n, m, 0, 0};
  return run_parallel(j, nthreads);
}

/* qr (_metal_kernels.py:641-694), every k: the GPU kernels' arithmetic, with
 * LAPACK's zero-tail rule above k = 63 where the reference runs LAPACK. */
int orc_qr(const float *A, float *Q, float *R, int64_t B, int n, int nthreads) {
  job_t j = {OP_QR, A, NULL, Q, R, NULL, B, n, 0, 0, 0};
  return run_parallel(j, nthreads);
}
