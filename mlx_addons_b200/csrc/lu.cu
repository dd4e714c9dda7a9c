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
//    is a butterfly over (|value|, row) with ties to the lower row. For
//    n <= 16 the same elimination runs on 16-lane halves of a warp, two
//    matrices per warp. Both stop after step n - 1: the identity rows past n
//    would only contribute pivots of 1 (sign * 1, log|det| + 0).
//  * n > 32: one CTA per matrix; the matrix lives in shared memory when it
//    fits (n <= 224); above, a blocked right-looking LU (n <= 864) or the
//    unblocked elimination, on a per-CTA scratch slot.
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
      if (j >= n) break;  // warp-uniform
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

// n <= 16: lanes 16 h .. 16 h + 15 of a warp hold matrix 2 w + h, one row
// per lane. The arithmetic per matrix is that of slogdet_warp_kernel; as the
// two halves may pivot differently, the row exchange is done without a
// branch (a lane that keeps its row reads its own value).
__global__ void __launch_bounds__(128) slogdet_half_kernel(const SlogdetParams p) {
  const int lane = threadIdx.x & 31;
  const int sl = lane & 15, base = lane & 16;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int n = p.n;
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); 2 * w < p.batch; w += nwarps) {
    const int64_t mat = 2 * w + (base >> 4);
    const bool valid = mat < p.batch;
    const float* A = p.A + (valid ? mat : 0) * (size_t)n * n;
    float a[16];
#pragma unroll
    for (int c = 0; c < 16; ++c)
      a[c] = (valid && sl < n && c < n) ? A[(size_t)sl * n + c] : (c == sl ? 1.f : 0.f);
    int swaps = 0;
    float sg = 1.f, lad = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j >= n) break;  // warp-uniform
      float v = (sl >= j) ? fabsf(a[j]) : -1.f;
      int idx = sl;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, v, o);
        const int oi = __shfl_xor_sync(kFull, idx, o);
        argmax_step(v, idx, ov, oi);
      }
      const int piv = __shfl_sync(kFull, idx, base);  // the half's lane 0: uniform even for NaN input
      const float pv = __shfl_sync(kFull, a[j], base + piv);
      swaps += (piv != j) ? 1 : 0;
      const bool ex = (piv != j) && (pv != 0.f);
      const int src = base + (ex ? ((sl == j) ? piv : (sl == piv ? j : sl)) : sl);
#pragma unroll
      for (int c = j; c < 16; ++c) a[c] = __shfl_sync(kFull, a[c], src);
      const float u = __shfl_sync(kFull, a[j], base + j);
      sg *= (u > 0.f) ? 1.f : ((u < 0.f) ? -1.f : 0.f);
      lad += logf(fabsf(u));
      if (u != 0.f) {
        const float ru = 1.f / u;
        const float mult = (fabsf(u) >= FLT_MIN) ? a[j] * ru : a[j] / u;
        if (sl > j) a[j] = mult;
      }
#pragma unroll
      for (int c = j + 1; c < 16; ++c) {
        const float prow = __shfl_sync(kFull, a[c], base + j);
        // separate multiply and subtract, as in slogdet_warp_kernel
        if (sl > j) a[c] = __fsub_rn(a[c], __fmul_rn(a[j], prow));
      }
    }
    if (sl == 0 && valid) {
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

// Blocked right-looking LU for matrices too large for one CTA's shared memory
// (kLuSmemMaxN < n <= kLuBlockedMaxN): the matrix lives in a per-CTA scratch
// slot, 32-column panels are factored in shared memory (the xGETF2 steps
// above, on the panel only), U12 = L11^{-1} A12 is formed column by column and
// the trailing matrix updated, A22 -= L21 U12. Row interchanges never move
// data in the slot: a shared-memory map from logical to physical rows takes
// each swap, and every later access goes through it. Every element still
// receives the same rank-1 updates, in the same order and with the same
// separately rounded multiply and subtract, as in the unblocked elimination:
// the pivots, signs and U diagonal are those of xGETF2, bit for bit.
constexpr int LBW = 32;
constexpr int kLuBlockedMaxN = 864;

__device__ __forceinline__ float fsub_mul(float a, float l, float u) { return __fsub_rn(a, __fmul_rn(l, u)); }

static size_t slogdet_blocked_smem(int n) {
  // panel (n x 33) + U12 (32 x n) floats + the row map (n ints) + the panel's zero-pivot flags
  return ((size_t)n * 33 + (size_t)LBW * n) * sizeof(float) + (size_t)(n + LBW) * sizeof(int);
}

// One matrix through the blocked LU, in place in its slot `a`. SOLVE selects
// the elimination of the reference's LU solve kernel (_metal_kernels.py:
// 716-742): the pivot is the first row whose |a| beats a running maximum that
// starts at 0 (a NaN never wins; an all-zero column keeps the diagonal), the
// column is always scaled by the reciprocal, and a zero pivot skips its
// column's scaling and every update that involves it (its multipliers stay
// unscaled in the slot, as in the reference). Otherwise xGETF2 (slogdet).
// Shared memory: P (panel, n x 33), U (U12, 32 x n), rowOf (n), zp (32).
template <bool SOLVE>
__device__ __forceinline__ void lu_blocked_factor(float* a, int n, float* P, float* U, int* rowOf, int* zp,
                                                  int& swaps, float& sg, float& lad) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ int sPiv;
  for (int r = tid; r < n; r += LT) rowOf[r] = r;
  __syncthreads();
  for (int j0 = 0; j0 < n; j0 += LBW) {
    const int bw = min(LBW, n - j0), R = n - j0, tc = n - j0 - bw;
    for (int e = tid; e < R * bw; e += LT) {
      const int r = e / bw, c = e - r * bw;
      P[r * 33 + c] = a[(size_t)rowOf[j0 + r] * n + j0 + c];
    }
    __syncthreads();
    // ---- unblocked elimination of the panel (three barriers per column) ---
    for (int jj = 0; jj < bw; ++jj) {
      if (warp == 0) {  // pivot search by one warp: first maximal |a|
        float v = SOLVE ? 0.f : -1.f;
        int idx = R;
        for (int r = jj + lane; r < R; r += 32) {
          const float t = fabsf(P[r * 33 + jj]);
          if (t > v) {
            v = t;
            idx = r;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(kFull, v, o);
          const int oi = __shfl_xor_sync(kFull, idx, o);
          argmax_step(v, idx, ov, oi);
        }
        // nothing beat the start value (all NaN; for SOLVE also all zero): keep the diagonal
        if (lane == 0) sPiv = (idx < R) ? idx : jj;
      }
      __syncthreads();
      const int piv = sPiv;
      const bool swp = P[piv * 33 + jj] != 0.f && piv != jj;
      if (swp && tid < bw) {
        const float t = P[jj * 33 + tid];
        P[jj * 33 + tid] = P[piv * 33 + tid];
        P[piv * 33 + tid] = t;
      }
      if (tid == 0 && swp) {  // the slot's rows follow through the map
        const int t = rowOf[j0 + jj];
        rowOf[j0 + jj] = rowOf[j0 + piv];
        rowOf[j0 + piv] = t;
      }
      __syncthreads();
      const float u = P[jj * 33 + jj];
      if (tid == 0) {
        if (piv != jj) ++swaps;
        sg *= (u > 0.f) ? 1.f : ((u < 0.f) ? -1.f : 0.f);
        lad += logf(fabsf(u));
        if (SOLVE) zp[jj] = (u == 0.f);
      }
      // scaling of column jj fused with the rank-1 update of the same row
      // (a row's multiplier is used by that row only)
      const float ru = 1.f / u;
      const bool recip = SOLVE || fabsf(u) >= FLT_MIN;
      const int c = jj + 1 + lane;
      if (!SOLVE || u != 0.f) {
        for (int r = jj + 1 + warp; r < R; r += LT / 32) {
          float l = P[r * 33 + jj];
          if (u != 0.f) l = recip ? l * ru : l / u;
          __syncwarp();
          if (lane == 0) P[r * 33 + jj] = l;
          if (c < bw) P[r * 33 + c] = fsub_mul(P[r * 33 + c], l, P[jj * 33 + c]);
        }
      }
      __syncthreads();
    }
    // SOLVE: the factored panel back to the slot (multipliers below, U11 above)
    for (int e = tid; e < (SOLVE ? R * bw : 0); e += LT) {
      const int r = e / bw, c = e - r * bw;
      a[(size_t)rowOf[j0 + r] * n + j0 + c] = P[r * 33 + c];
    }
    if (tc == 0) continue;
    // ---- U12 = L11^{-1} A12 (unit lower), one column per thread -----------
    for (int c = tid; c < tc; c += LT) {
      float u[LBW];
#pragma unroll
      for (int q = 0; q < LBW; ++q) {
        if (q < bw) {
          float t = a[(size_t)rowOf[j0 + q] * n + j0 + bw + c];
#pragma unroll
          for (int pp = 0; pp < q; ++pp)
            if (!SOLVE || !zp[pp]) t = fsub_mul(t, P[q * 33 + pp], u[pp]);
          u[q] = t;
          U[q * tc + c] = t;
          if (SOLVE) a[(size_t)rowOf[j0 + q] * n + j0 + bw + c] = t;
        }
      }
    }
    __syncthreads();
    // ---- A22 -= L21 U12, the rank-1 updates in panel order -----------------
    // a warp takes 4 rows x 64 columns at a time, each lane 4 x 2 elements:
    // 8 independent chains and 8 loads in flight
    {
      const int nrow = n - j0 - bw, nrb = (nrow + 3) / 4, ncp = (tc + 63) / 64;
      for (int it = warp; it < nrb * ncp; it += LT / 32) {
        const int rb = it / ncp, cp = it - rb * ncp;
        float* x[4][2];
        float v[4][2];
        const float* lr[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int i = j0 + bw + 4 * rb + k;
          const bool rv = i < n;
          lr[k] = P + (rv ? i - j0 : 0) * 33;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = 64 * cp + lane + 32 * h;
            x[k][h] = (rv && c < tc) ? a + (size_t)rowOf[i] * n + j0 + bw + c : nullptr;
            v[k][h] = x[k][h] ? *x[k][h] : 0.f;
          }
        }
        const int c0 = 64 * cp + lane, c1 = c0 + 32;
#pragma unroll
        for (int q = 0; q < LBW; ++q) {
          if (q < bw && (!SOLVE || !zp[q])) {
            const float u0 = (c0 < tc) ? U[q * tc + c0] : 0.f, u1 = (c1 < tc) ? U[q * tc + c1] : 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float l = lr[k][q];
              v[k][0] = fsub_mul(v[k][0], l, u0);
              v[k][1] = fsub_mul(v[k][1], l, u1);
            }
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            if (x[k][h]) *x[k][h] = v[k][h];
      }
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(LT, 2) slogdet_blocked_kernel(const SlogdetParams p) {
  extern __shared__ __align__(16) float sm[];
  const int n = p.n;
  const int tid = threadIdx.x;
  float* P = sm;                          // panel rows j0..n-1, stride 33
  float* U = sm + (size_t)n * 33;         // U12: row q at U + q * tc
  int* rowOf = reinterpret_cast<int*>(U + (size_t)LBW * n);  // logical row -> physical row of the slot
  int* zp = rowOf + n;
  float* a = p.ws + (size_t)blockIdx.x * n * n;
  const size_t nn = (size_t)n * n;
  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x) {
    const float* A = p.A + mat * nn;
    __syncthreads();
    for (size_t e = tid; e < nn; e += LT) a[e] = A[e];
    int swaps = 0;
    float sg = 1.f, lad = 0.f;
    lu_blocked_factor<false>(a, n, P, U, rowOf, zp, swaps, sg, lad);
    if (tid == 0) {
      if (p.sign) p.sign[mat] = (swaps & 1) ? -sg : sg;
      if (p.logabsdet) p.logabsdet[mat] = lad;
    }
  }
}

// solve_lu for kLuSmemMaxN < k <= kLuBlockedMaxN: the blocked LU above in its
// SOLVE form, then the substitutions of P A = L U against the right-hand
// sides, MCH at a time in shared memory (column-major, y[q n + i]); rows of
// the slot are read through the row map. Forward: per 32-row block, a GEMV
// with the rows already solved (warps over rows, lanes over columns), then
// the unit-lower 32 x 32 solve in one warp per right-hand side (lane = row,
// the solved value broadcast by shuffle). Backward likewise with U, dividing
// by the diagonal as the reference does (_metal_kernels.py:759-763).
constexpr int MCH = 8;

__global__ void __launch_bounds__(LT, 2) gesv_blocked_kernel(const GesvParams p) {
  extern __shared__ __align__(16) float sm[];
  const int n = p.k, m = p.m;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* P = sm;
  float* U = sm + (size_t)n * 33;
  int* rowOf = reinterpret_cast<int*>(U + (size_t)LBW * n);
  int* zp = rowOf + n;
  float* ys = sm;  // after the factorisation: MCH x n right-hand-side values
  float* a = p.ws + (size_t)blockIdx.x * n * n;
  const size_t nn = (size_t)n * n;
  const int nblk = (n + LBW - 1) / LBW;
  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x) {
    const float* A = p.A + mat * nn;
    __syncthreads();
    for (size_t e = tid; e < nn; e += LT) a[e] = A[e];
    int swaps = 0;
    float sg = 1.f, lad = 0.f;
    lu_blocked_factor<true>(a, n, P, U, rowOf, zp, swaps, sg, lad);
    const float* bm = p.b + mat * (size_t)n * m;
    float* xm = p.x + mat * (size_t)n * m;
    for (int q0 = 0; q0 < m; q0 += MCH) {
      const int mc = min(MCH, m - q0);
      __syncthreads();
      for (int e = tid; e < n * mc; e += LT) {  // y = P b
        const int i = e / mc, q = e - i * mc;
        ys[q * n + i] = bm[(size_t)rowOf[i] * m + q0 + q];
      }
      __syncthreads();
      // forward: y_J -= L[J, :j0] y[:j0], then the unit-lower block solve
      for (int J = 0; J < nblk; ++J) {
        const int j0 = LBW * J, bw = min(LBW, n - j0);
        if (j0 > 0) {
          for (int r = warp; r < bw; r += LT / 32) {
            const float* lrow = a + (size_t)rowOf[j0 + r] * n;
            float s[MCH];
#pragma unroll
            for (int q = 0; q < MCH; ++q) s[q] = 0.f;
            for (int c = lane; c < j0; c += 32) {
              const float l = lrow[c];
#pragma unroll
              for (int q = 0; q < MCH; ++q)
                if (q < mc) s[q] = fmaf(l, ys[q * n + c], s[q]);
            }
#pragma unroll
            for (int q = 0; q < MCH; ++q)
              if (q < mc) {
                const float t = warp_sum(s[q]);
                if (lane == 0) ys[q * n + j0 + r] -= t;
              }
          }
          __syncthreads();
        }
        if (warp < mc) {
          const float* lrow = a + (size_t)rowOf[j0 + min(lane, bw - 1)] * n + j0;
          float lr[LBW];
#pragma unroll
          for (int pp = 0; pp < LBW; ++pp) lr[pp] = (pp < lane && lane < bw) ? lrow[pp] : 0.f;
          float y = (lane < bw) ? ys[warp * n + j0 + lane] : 0.f;
#pragma unroll
          for (int pp = 0; pp < LBW; ++pp) {
            if (pp < bw) {
              const float yp = __shfl_sync(kFull, y, pp);
              if (lane > pp) y = fmaf(-lr[pp], yp, y);
            }
          }
          if (lane < bw) ys[warp * n + j0 + lane] = y;
        }
        __syncthreads();
      }
      // backward: y_J -= U[J, J+1:] x[J+1:], then the upper block solve
      for (int J = nblk - 1; J >= 0; --J) {
        const int j0 = LBW * J, bw = min(LBW, n - j0), c0 = j0 + bw;
        if (c0 < n) {
          for (int r = warp; r < bw; r += LT / 32) {
            const float* urow = a + (size_t)rowOf[j0 + r] * n;
            float s[MCH];
#pragma unroll
            for (int q = 0; q < MCH; ++q) s[q] = 0.f;
            for (int c = c0 + lane; c < n; c += 32) {
              const float u = urow[c];
#pragma unroll
              for (int q = 0; q < MCH; ++q)
                if (q < mc) s[q] = fmaf(u, ys[q * n + c], s[q]);
            }
#pragma unroll
            for (int q = 0; q < MCH; ++q)
              if (q < mc) {
                const float t = warp_sum(s[q]);
                if (lane == 0) ys[q * n + j0 + r] -= t;
              }
          }
          __syncthreads();
        }
        if (warp < mc) {
          const float* urow = a + (size_t)rowOf[j0 + min(lane, bw - 1)] * n + j0;
          float ur[LBW];
#pragma unroll
          for (int pp = 0; pp < LBW; ++pp) ur[pp] = (pp >= lane && pp < bw) ? urow[pp] : 0.f;
          float d = 1.f;  // U[lane][lane]
#pragma unroll
          for (int pp = 0; pp < LBW; ++pp) d = (pp == lane) ? ur[pp] : d;
          float y = (lane < bw) ? ys[warp * n + j0 + lane] : 0.f;
#pragma unroll
          for (int pp = LBW - 1; pp >= 0; --pp) {
            if (pp < bw) {
              if (lane == pp) y = y / d;
              const float xp = __shfl_sync(kFull, y, pp);
              if (lane < pp) y = fmaf(-ur[pp], xp, y);
            }
          }
          if (lane < bw) ys[warp * n + j0 + lane] = y;
        }
        __syncthreads();
      }
      for (int e = tid; e < n * mc; e += LT) {
        const int i = e / mc, q = e - i * mc;
        xm[(size_t)i * m + q0 + q] = ys[q * n + i];
      }
    }
  }
}

static cudaError_t blocked_occupancy(int n, int* occ) {
  static int cache[64];
  cudaError_t e = kernel_occupancy(slogdet_blocked_kernel, LT, slogdet_blocked_smem(n), cache, occ);
  if (e != cudaSuccess) return e;
  // the cache above holds the first size queried; this query is for n
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, slogdet_blocked_kernel, LT, slogdet_blocked_smem(n));
  if (e != cudaSuccess) return e;
  if (*occ < 1) *occ = 1;
  return cudaSuccess;
}

static cudaError_t gesv_blocked_occupancy(int n, int* occ) {
  static int cache[64];
  cudaError_t e = kernel_occupancy(gesv_blocked_kernel, LT, slogdet_blocked_smem(n), cache, occ);
  if (e != cudaSuccess) return e;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, gesv_blocked_kernel, LT, slogdet_blocked_smem(n));
  if (e != cudaSuccess) return e;
  if (*occ < 1) *occ = 1;
  return cudaSuccess;
}

bool gesv_blocked_fits(int k) { return k > kLuSmemMaxN && k <= kLuBlockedMaxN; }

int gesv_blocked_grid(int64_t batch, int k, int sm_count) {
  int occ = 2;
  if (gesv_blocked_occupancy(k, &occ) != cudaSuccess) occ = 2;
  const int64_t cap = (int64_t)sm_count * occ;
  return (int)(batch < cap ? batch : cap);
}

cudaError_t launch_gesv_blocked(const GesvParams& p, int grid, cudaStream_t s) {
  int occ = 1;
  cudaError_t e = gesv_blocked_occupancy(p.k, &occ);
  if (e != cudaSuccess) return e;
  gesv_blocked_kernel<<<grid, LT, slogdet_blocked_smem(p.k), s>>>(p);
  return cudaGetLastError();
}

int slogdet_grid(int64_t batch, int n, int sm_count) {
  int per_sm = 2;
  if (n > kLuSmemMaxN && n <= kLuBlockedMaxN) {
    int occ = 1;
    if (blocked_occupancy(n, &occ) == cudaSuccess) per_sm = occ;
  }
  const int64_t cap = (int64_t)sm_count * per_sm;
  return (int)(batch < cap ? batch : cap);
}

size_t slogdet_ws_floats(int64_t batch, int n, int sm_count) {
  if (n <= kLuSmemMaxN || batch <= 0) return 0;
  return (size_t)slogdet_grid(batch, n, sm_count) * (size_t)n * n;
}

cudaError_t launch_slogdet(const SlogdetParams& p, int sm_count, cudaStream_t s) {
  if (p.n <= 16) {
    static int cache[64];
    int occ = 0;
    cudaError_t e = kernel_occupancy(slogdet_half_kernel, 128, 0, cache, &occ);
    if (e != cudaSuccess) return e;
    const int64_t need = (p.batch + 7) / 8;  // 8 matrices per 4-warp CTA
    const int64_t cap = (int64_t)sm_count * occ;
    slogdet_half_kernel<<<(int)(need < cap ? need : cap), 128, 0, s>>>(p);
    return cudaGetLastError();
  }
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
  if (p.n <= kLuBlockedMaxN) {
    int occ = 1;
    cudaError_t e = blocked_occupancy(p.n, &occ);
    if (e != cudaSuccess) return e;
    slogdet_blocked_kernel<<<slogdet_grid(p.batch, p.n, sm_count), LT, slogdet_blocked_smem(p.n), s>>>(p);
    return cudaGetLastError();
  }
  slogdet_cta_kernel<false><<<slogdet_grid(p.batch, p.n, sm_count), LT, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace b2c
