// Batched Householder QR of square matrices, Q formed explicitly.
//
// Replaces the reference's qr (src/mlx_addons/linalg/_metal_kernels.py:
// 641-694): a single-thread Metal kernel for k < 12 (_QR_SRC :319-381), a
// threadgroup kernel for 12 <= k <= 63 (_QR_TG_SRC :385-473) and CPU LAPACK
// above (:685-688). The reflector of column j is generated as in the Metal
// kernels (:336-352): norm = sqrt(max(sum_{i>=j} r_ij^2, 1e-30)),
// v = (r_jj + s * norm, r_{j+1,j}, ...) with s = +1 for r_jj >= 0 else -1,
// tau = 2 / v.v (0 when v.v <= 1e-30); Q <- Q (I - tau v v^T) and
// R <- (I - tau v v^T) R right of column j, products grouped as
// (tau * dot) * v_i and (tau * v_i) * dot (:354-366); then r_jj = -s * norm
// and zeros below. Above k = 63, where the reference runs LAPACK, a column
// whose sub-diagonal part is exactly zero is left alone (LAPACK's reflector
// generator returns tau = 0 and keeps r_jj), the last column always; for
// every other column both generate the same reflector. Sums are fused into
// FMAs and the norm is reduced in a different order: results agree with the
// reference to rounding.
//
//  * k <= 32: one warp per matrix; lane l holds column l of R and row l of Q
//    in registers. The reflector (column j, in lane j) is broadcast by
//    shuffles; every lane then forms norm, tau and v itself, its own R-column
//    dot product and update, and its own Q-row dot product and update.
//  * k > 32: one CTA per matrix with R and Q^T in shared memory (row stride
//    k | 1: a thread per R column or per Q row reads conflict-free) up to
//    k = 160, in a per-CTA scratch slot above; warp 0 reduces the norms.
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

constexpr int QW = 4;     // warps per CTA, warp tier
constexpr int QT = 256;   // threads per CTA, CTA tier
constexpr int kQrSmemMaxK = 160;
constexpr int kQrLapackAbove = 63;  // _metal_kernels.py:383, QR_SHARED_K_MAX

__global__ void __launch_bounds__(QW * 32) qr_warp_kernel(const QrParams p) {
  __shared__ float st[QW][32 * 33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = p.k;
  float* S = st[warp];
  const int64_t nw = (int64_t)gridDim.x * QW;
  for (int64_t mat = (int64_t)blockIdx.x * QW + warp; mat < p.batch; mat += nw) {
    const float* A = p.A + mat * (size_t)n * n;
    float r[32], q[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      r[i] = (lane < n && i < n) ? A[(size_t)i * n + lane] : 0.f;
      q[i] = (i == lane) ? 1.f : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j >= n) break;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = (i >= j && i < n) ? __shfl_sync(kFull, r[i], j) : 0.f;
      float sigma = 0.f;
#pragma unroll
      for (int i = j; i < 32; ++i) sigma = fmaf(v[i], v[i], sigma);
      const float norm = sqrtf(fmaxf(sigma, 1e-30f));
      const float sgn = (v[j] >= 0.f) ? 1.f : -1.f;
      const float vh = fmaf(sgn, norm, v[j]);
      float vtv = vh * vh;
#pragma unroll
      for (int i = j + 1; i < 32; ++i) vtv = fmaf(v[i], v[i], vtv);
      const float tau = (vtv > 1e-30f) ? (2.f / vtv) : 0.f;
      v[j] = vh;
      if (lane > j) {  // R column `lane` (zero columns beyond n stay zero)
        float dot = 0.f;
#pragma unroll
        for (int i = j; i < 32; ++i) dot = fmaf(v[i], r[i], dot);
#pragma unroll
        for (int i = j; i < 32; ++i) r[i] = fmaf(-(tau * v[i]), dot, r[i]);
      }
      {  // Q row `lane`
        float dot = 0.f;
#pragma unroll
        for (int i = j; i < 32; ++i) dot = fmaf(q[i], v[i], dot);
        const float td = tau * dot;
#pragma unroll
        for (int i = j; i < 32; ++i) q[i] = fmaf(-td, v[i], q[i]);
      }
      if (lane == j) {
        r[j] = -sgn * norm;
#pragma unroll
        for (int i = j + 1; i < 32; ++i) r[i] = 0.f;
      }
    }
    float* Rm = p.R + mat * (size_t)n * n;
    float* Qm = p.Q + mat * (size_t)n * n;
    if (lane < n) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < n) Rm[(size_t)i * n + lane] = r[i];
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 32; ++i) S[lane * 33 + i] = q[i];
    __syncwarp();
    for (int e = lane; e < n * n; e += 32) {
      const int row = e / n, c = e - row * n;
      Qm[e] = S[row * 33 + c];
    }
    __syncwarp();
  }
}

template <bool SMEM>
__global__ void __launch_bounds__(QT) qr_cta_kernel(const QrParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float sInfo[4];
  const int n = p.k, LD = n | 1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool lapack_tail = n > kQrLapackAbove;
  float* R = SMEM ? sm : p.ws + (size_t)blockIdx.x * 2 * n * LD;
  float* QTm = R + (size_t)n * LD;  // QTm[i][row] = Q[row][i]
  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x) {
    const float* A = p.A + mat * (size_t)n * n;
    __syncthreads();
    for (int e = tid; e < n * n; e += QT) {
      const int i = e / n, c = e - i * n;
      R[(size_t)i * LD + c] = A[e];
      QTm[(size_t)i * LD + c] = (i == c) ? 1.f : 0.f;
    }
    __syncthreads();
    for (int j = 0; j < n; ++j) {
      if (warp == 0) {
        float s = 0.f;
        bool nz = false;
        for (int i = j + 1 + lane; i < n; i += 32) {
          const float t = R[(size_t)i * LD + j];
          s = fmaf(t, t, s);
          nz |= (t != 0.f);
        }
        s = warp_sum(s);
        nz = __any_sync(kFull, nz);
        if (lane == 0) {
          const float x = R[(size_t)j * LD + j];
          const float norm = sqrtf(fmaxf(fmaf(x, x, s), 1e-30f));
          const float sgn = (x >= 0.f) ? 1.f : -1.f;
          const float vh = fmaf(sgn, norm, x);
          const float vtv = fmaf(vh, vh, s);
          sInfo[0] = (vtv > 1e-30f) ? (2.f / vtv) : 0.f;
          sInfo[1] = vh;
          sInfo[2] = -sgn * norm;
          sInfo[3] = (lapack_tail && !nz) ? 1.f : 0.f;
        }
      }
      __syncthreads();
      if (sInfo[3] != 0.f) {  // LAPACK: nothing to annihilate, column kept
        __syncthreads();      // sInfo is rewritten by the next column
        continue;
      }
      const float tau = sInfo[0], vh = sInfo[1];
      for (int w = tid; w < 2 * n; w += QT) {
        if (w < n) {
          const int col = w;
          if (col > j) {
            float dot = vh * R[(size_t)j * LD + col];
            for (int i = j + 1; i < n; ++i) dot = fmaf(R[(size_t)i * LD + j], R[(size_t)i * LD + col], dot);
            R[(size_t)j * LD + col] = fmaf(-(tau * vh), dot, R[(size_t)j * LD + col]);
            for (int i = j + 1; i < n; ++i)
              R[(size_t)i * LD + col] = fmaf(-(tau * R[(size_t)i * LD + j]), dot, R[(size_t)i * LD + col]);
          }
        } else {
          const int row = w - n;
          float dot = QTm[(size_t)j * LD + row] * vh;
          for (int i = j + 1; i < n; ++i) dot = fmaf(QTm[(size_t)i * LD + row], R[(size_t)i * LD + j], dot);
          const float td = tau * dot;
          QTm[(size_t)j * LD + row] = fmaf(-td, vh, QTm[(size_t)j * LD + row]);
          for (int i = j + 1; i < n; ++i)
            QTm[(size_t)i * LD + row] = fmaf(-td, R[(size_t)i * LD + j], QTm[(size_t)i * LD + row]);
        }
      }
      __syncthreads();
      const float rjj = sInfo[2];
      for (int i = j + tid; i < n; i += QT) R[(size_t)i * LD + j] = (i == j) ? rjj : 0.f;
      __syncthreads();
    }
    float* Rm = p.R + mat * (size_t)n * n;
    float* Qm = p.Q + mat * (size_t)n * n;
    for (int e = tid; e < n * n; e += QT) {
      const int row = e / n, c = e - row * n;
      Rm[e] = R[(size_t)row * LD + c];
      Qm[e] = QTm[(size_t)c * LD + row];
    }
  }
}

static size_t qr_cta_smem(int k) { return 2 * (size_t)k * (size_t)(k | 1) * sizeof(float); }

int qr_grid(int64_t batch, int k, int sm_count) {
  (void)k;
  const int64_t cap = (int64_t)sm_count * 2;
  return (int)(batch < cap ? batch : cap);
}

size_t qr_ws_floats(int64_t batch, int k, int sm_count) {
  if (k <= kQrSmemMaxK || batch <= 0) return 0;
  return (size_t)qr_grid(batch, k, sm_count) * 2 * (size_t)k * (size_t)(k | 1);
}

cudaError_t launch_qr(const QrParams& p, int sm_count, cudaStream_t s) {
  if (p.k <= 32) {
    static int cache[64];
    int occ = 0;
    cudaError_t e = kernel_occupancy(qr_warp_kernel, QW * 32, 0, cache, &occ);
    if (e != cudaSuccess) return e;
    const int64_t need = (p.batch + QW - 1) / QW;
    const int64_t cap = (int64_t)sm_count * occ;
    qr_warp_kernel<<<(int)(need < cap ? need : cap), QW * 32, 0, s>>>(p);
    return cudaGetLastError();
  }
  if (p.k <= kQrSmemMaxK) {
    const size_t smem = qr_cta_smem(p.k);
    static int cache[64];
    int occ = 0;
    cudaError_t e = kernel_occupancy(qr_cta_kernel<true>, QT, smem, cache, &occ);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, qr_cta_kernel<true>, QT, smem);
    if (e != cudaSuccess) return e;
    if (occ < 1) occ = 1;
    const int64_t cap = (int64_t)sm_count * occ;
    qr_cta_kernel<true><<<(int)(p.batch < cap ? p.batch : cap), QT, smem, s>>>(p);
    return cudaGetLastError();
  }
  qr_cta_kernel<false><<<qr_grid(p.batch, p.k, sm_count), QT, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace b2c
