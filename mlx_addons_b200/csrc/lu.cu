// Batched sign / log|det| through LU with partial pivoting.
//
// Replaces src/mlx_addons/linalg/_det.py:17-48, where the reference calls
// mx.linalg.lu_factor on the CPU stream (LAPACK getrf) and then forms
//   sign      = (-1)^{#(piv[j] != j)} * prod sign(U_jj)
//   logabsdet = sum log|U_jj|.
// The elimination follows LAPACK xGETF2: the pivot is the FIRST row of
// maximal |a_ij| in column j, rows are swapped only when that pivot is
// non-zero, the column is scaled by the reciprocal (or divided when
// |pivot| < FLT_MIN), then the rank-1 trailing update.
//  * n <= 32: one warp per matrix, one row per lane in registers; the argmax
//    is a butterfly over (|value|, row) with ties to the lower row.
//  * n > 32: one CTA per matrix; the matrix lives in shared memory when it
//    fits (n <= 224) and otherwise in a per-CTA scratch slot.
#include <float.h>

#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

constexpr int kLuSmemMaxN = 224;
constexpr int LT = 256;

__device__ __forceinline__ void argmax_step(float& v, int& idx, float ov, int oi) {
  if (ov > v || (ov == v && oi < idx)) {
    v = ov;
    idx = oi;
  }
}

__global__ void __launch_bounds__(128) slogdet_warp_kernel(const SlogdetParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int n = p.n;
  for (int64_t mat = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); mat < p.batch; mat += nwarps) {
    const float* A = p.A + mat * (size_t)n * n;
    float a[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) a[c] = (lane < n && c < n) ? A[(size_t)lane * n + c] : (c == lane ? 1.f : 0.f);
    int swaps = 0;
    float sg = 1.f, lad = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float v = (lane >= j) ? fabsf(a[j]) : -1.f;
      int idx = lane;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, v, o);
        const int oi = __shfl_xor_sync(kFull, idx, o);
        argmax_step(v, idx, ov, oi);
      }
      const int piv = __shfl_sync(kFull, idx, 0);  // uniform even for NaN input
      const float pv = __shfl_sync(kFull, a[j], piv);
      if (piv != j) {
        ++swaps;
        if (pv != 0.f) {
          const int src = (lane == j) ? piv : (lane == piv ? j : lane);
#pragma unroll
          for (int c = j; c < 32; ++c) a[c] = __shfl_sync(kFull, a[c], src);
        }
      }
      const float u = __shfl_sync(kFull, a[j], j);
      sg *= (u > 0.f) ? 1.f : ((u < 0.f) ? -1.f : 0.f);
      lad += logf(fabsf(u));
      if (u != 0.f) {
        const float ru = 1.f / u;
        const float mult = (fabsf(u) >= FLT_MIN) ? a[j] * ru : a[j] / u;
        if (lane > j) a[j] = mult;
      }
#pragma unroll
      for (int c = j + 1; c < 32; ++c) {
        const float prow = __shfl_sync(kFull, a[c], j);
        // separate multiply and subtract (no FMA contraction), as LAPACK's
        // rank-1 update rounds: an exactly singular input keeps an exact
        // zero pivot
        if (lane > j) a[c] = __fsub_rn(a[c], __fmul_rn(a[j], prow));
      }
    }
    if (lane == 0) {
      if (p.sign) p.sign[mat] = (swaps & 1) ? -sg : sg;
      if (p.logabsdet) p.logabsdet[mat] = lad;
    }
  }
}

template <bool SMEM>
__global__ void __launch_bounds__(LT) slogdet_cta_kernel(const SlogdetParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float sVal[LT / 32];
  __shared__ int sIdx[LT / 32];
  __shared__ int sPiv;
  const int n = p.n;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t nn = (size_t)n * n;
  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x) {
    float* a = SMEM ? sm : p.ws + (size_t)blockIdx.x * nn;
    const float* A = p.A + mat * nn;
    __syncthreads();
    for (size_t e = tid; e < nn; e += LT) a[e] = A[e];
    __syncthreads();
    int swaps = 0;
    float sg = 1.f, lad = 0.f;
    for (int j = 0; j < n; ++j) {
      float v = -1.f;
      int idx = n;
      for (int i = j + tid; i < n; i += LT) {
        const float t = fabsf(a[(size_t)i * n + j]);
        if (t > v) {
          v = t;
          idx = i;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, v, o);
        const int oi = __shfl_xor_sync(kFull, idx, o);
        argmax_step(v, idx, ov, oi);
      }
      if (lane == 0) {
        sVal[warp] = v;
        sIdx[warp] = idx;
      }
      __syncthreads();
      if (tid == 0) {
        float bv = sVal[0];
        int bi = sIdx[0];
        for (int w = 1; w < LT / 32; ++w) argmax_step(bv, bi, sVal[w], sIdx[w]);
        sPiv = (bi < n) ? bi : j;  // all-NaN column: keep the diagonal
      }
      __syncthreads();
      const int piv = sPiv;
      const float pv = a[(size_t)piv * n + j];
      if (pv != 0.f && piv != j) {
        for (int c = j + tid; c < n; c += LT) {
          const float t = a[(size_t)j * n + c];
          a[(size_t)j * n + c] = a[(size_t)piv * n + c];
          a[(size_t)piv * n + c] = t;
        }
      }
      __syncthreads();
      const float u = a[(size_t)j * n + j];
      if (tid == 0) {
        if (piv != j) ++swaps;
        sg *= (u > 0.f) ? 1.f : ((u < 0.f) ? -1.f : 0.f);
        lad += logf(fabsf(u));
      }
      if (u != 0.f) {
        const float ru = 1.f / u;
        const bool recip = fabsf(u) >= FLT_MIN;
        for (int i = j + 1 + tid; i < n; i += LT) {
          const float t = a[(size_t)i * n + j];
          a[(size_t)i * n + j] = recip ? t * ru : t / u;
        }
      }
      __syncthreads();
      for (int i = j + 1 + warp; i < n; i += LT / 32) {
        const float lij = a[(size_t)i * n + j];
        for (int c = j + 1 + lane; c < n; c += 32)
          a[(size_t)i * n + c] = __fsub_rn(a[(size_t)i * n + c], __fmul_rn(lij, a[(size_t)j * n + c]));
      }
      __syncthreads();
    }
    if (tid == 0) {
      if (p.sign) p.sign[mat] = (swaps & 1) ? -sg : sg;
      if (p.logabsdet) p.logabsdet[mat] = lad;
    }
  }
}

int slogdet_grid(int64_t batch, int n, int sm_count) {
  (void)n;
  const int64_t cap = (int64_t)sm_count * 2;
  return (int)(batch < cap ? batch : cap);
}

size_t slogdet_ws_floats(int64_t batch, int n, int sm_count) {
  if (n <= kLuSmemMaxN || batch <= 0) return 0;
  return (size_t)slogdet_grid(batch, n, sm_count) * (size_t)n * n;
}

cudaError_t launch_slogdet(const SlogdetParams& p, int sm_count, cudaStream_t s) {
  if (p.n <= 32) {
    static int cache[64];
    int occ = 0;
    cudaError_t e = kernel_occupancy(slogdet_warp_kernel, 128, 0, cache, &occ);
    if (e != cudaSuccess) return e;
    const int64_t need = (p.batch + 3) / 4;
    const int64_t cap = (int64_t)sm_count * occ;
    slogdet_warp_kernel<<<(int)(need < cap ? need : cap), 128, 0, s>>>(p);
    return cudaGetLastError();
  }
  if (p.n <= kLuSmemMaxN) {
    const size_t smem = (size_t)p.n * p.n * sizeof(float);
    static int cache[64];
    int occ = 0;
    cudaError_t e = kernel_occupancy(slogdet_cta_kernel<true>, LT, smem, cache, &occ);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, slogdet_cta_kernel<true>, LT, smem);
    if (e != cudaSuccess) return e;
    if (occ < 1) occ = 1;
    const int64_t cap = (int64_t)sm_count * occ;
    slogdet_cta_kernel<true><<<(int)(p.batch < cap ? p.batch : cap), LT, smem, s>>>(p);
    return cudaGetLastError();
  }
  slogdet_cta_kernel<false><<<slogdet_grid(p.batch, p.n, sm_count), LT, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace b2c
