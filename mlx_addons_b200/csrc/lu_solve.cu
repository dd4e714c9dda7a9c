// Batched A x = b through LU with partial pivoting, for any square A.
//
// Replaces the reference's solve_lu (src/mlx_addons/linalg/_metal_kernels.py:
// 917-969; kernels _LU_SOLVE_SRC :701-768 and _LU_SOLVE_LG_SRC :849-914), one
// Metal thread per matrix with the LU in device memory, with the same
// arithmetic contract:
//  * the pivot of column j is the FIRST row whose |a_ij| beats a running
//    maximum that starts at 0, so NaN never wins and an all-zero column keeps
//    row j (:720-725);
//  * the rows are swapped whenever the pivot row differs (:727-733);
//  * only for a non-zero pivot, the column below it is multiplied by the
//    reciprocal 1/pivot and the rank-1 trailing update follows (:734-738);
//  * each right-hand side gets the recorded swaps in order, a unit-lower
//    forward substitution and an upper backward substitution that divides by
//    U_ii, so a singular U gives inf / NaN exactly where the reference's does.
// The forward substitution accumulates each row's terms in the reference's
// order; the backward one is column-oriented (terms in decreasing column
// order), and products are fused into FMAs: results agree to rounding.
//
//  * k <= 32: one warp per matrix, lane i holds row i in registers. Rows never
//    move: a lane keeps a logical position that the pivot swap exchanges, the
//    argmax breaks ties on that logical position (the reference's "first
//    row"), and since a lane also keeps its own right-hand-side row, the
//    swaps reach b for free. The pivot row is broadcast through shared memory.
//  * 32 < k <= 64: the same with two rows per lane (rows l and 32 + l).
//  * k > 64: one CTA per matrix, LU in shared memory (row stride k | 1, so a
//    column read by consecutive threads is conflict-free) up to k = 224, in a
//    per-CTA scratch slot above; one warp per right-hand side for the
//    substitutions.
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

constexpr int GW = 4;             // warps per CTA, warp tier
constexpr int GT = 256;           // threads per CTA, CTA tier
constexpr int GCH = GT / 32;      // right-hand sides per pass, CTA tier
constexpr int kGesvSmemMaxK = 224;
// Above kGesvSmemMaxK the LU lives in scratch but the pivots and GCH
// right-hand sides stay in shared memory: 36 k bytes.

template <int MC>
__global__ void __launch_bounds__(GW * 32) gesv_warp_kernel(const GesvParams p) {
  __shared__ float st[GW][32 * 33];
  __shared__ __align__(16) float prow[GW][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = p.k, m = p.m;
  float* S = st[warp];
  float* P = prow[warp];
  const int64_t nw = (int64_t)gridDim.x * GW;
  for (int64_t mat = (int64_t)blockIdx.x * GW + warp; mat < p.batch; mat += nw) {
    const float* A = p.A + mat * (size_t)n * n;
    __syncwarp();
    for (int e = lane; e < n * n; e += 32) {
      const int r = e / n, c = e - r * n;
      S[r * 33 + c] = A[e];
    }
    __syncwarp();
    float a[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) a[c] = (lane < n && c < n) ? S[lane * 33 + c] : (c == lane ? 1.f : 0.f);
    int lg = lane;  // logical row of this lane's row
    int own[32];    // own[j]: lane holding logical row j (uniform)
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j >= n) break;
      float v = (lg >= j) ? fabsf(a[j]) : -1.f;
      if (!(v == v)) v = 0.f;  // NaN never beats the running maximum
      int key = lg;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, v, o);
        const int ok = __shfl_xor_sync(kFull, key, o);
        if (ov > v || (ov == v && ok < key)) {
          v = ov;
          key = ok;
        }
      }
      const int pl = __ffs(__ballot_sync(kFull, lg == key)) - 1;
      own[j] = pl;
      if (lg == j) lg = key;
      else if (lane == pl) lg = j;
      const float d = __shfl_sync(kFull, a[j], pl);
      if (d != 0.f) {
        if (lane == pl) {
#pragma unroll
          for (int c4 = ((j + 1) >> 2) << 2; c4 < 32; c4 += 4)
            *reinterpret_cast<float4*>(P + c4) = make_float4(a[c4], a[c4 + 1], a[c4 + 2], a[c4 + 3]);
        }
        __syncwarp();
        if (lg > j) {
          const float l = a[j] * (1.f / d);
          a[j] = l;
#pragma unroll
          for (int c4 = ((j + 1) >> 2) << 2; c4 < 32; c4 += 4) {
            const float4 w = *reinterpret_cast<const float4*>(P + c4);
            if (c4 > j) a[c4] = fmaf(-l, w.x, a[c4]);
            if (c4 + 1 > j) a[c4 + 1] = fmaf(-l, w.y, a[c4 + 1]);
            if (c4 + 2 > j) a[c4 + 2] = fmaf(-l, w.z, a[c4 + 2]);
            if (c4 + 3 > j) a[c4 + 3] = fmaf(-l, w.w, a[c4 + 3]);
          }
        }
        __syncwarp();
      }
    }
    const float* bm = p.b + mat * (size_t)n * m;
    float* xm = p.x + mat * (size_t)n * m;
    for (int q0 = 0; q0 < m; q0 += MC) {
      const int mc = (m - q0) < MC ? (m - q0) : MC;
      float y[MC];
#pragma unroll
      for (int q = 0; q < MC; ++q) y[q] = (lane < n && q < mc) ? bm[(size_t)lane * m + q0 + q] : 0.f;
      // forward, unit lower, logical order
#pragma unroll
      for (int pp = 0; pp < 32; ++pp) {
        if (pp >= n) break;
        const int src = own[pp];
#pragma unroll
        for (int q = 0; q < MC; ++q) {
          const float yp = __shfl_sync(kFull, y[q], src);
          if (lg > pp) y[q] = fmaf(-a[pp], yp, y[q]);
        }
      }
      // backward, upper, dividing by U_pp
#pragma unroll
      for (int pp = 31; pp >= 0; --pp) {
        if (pp >= n) continue;
        const int src = own[pp];
        const bool me = lane == src;
#pragma unroll
        for (int q = 0; q < MC; ++q) {
          const float xv = __shfl_sync(kFull, me ? y[q] / a[pp] : 0.f, src);
          if (me) y[q] = xv;
          else if (lg < pp) y[q] = fmaf(-a[pp], xv, y[q]);
        }
      }
      if (lane < n) {
#pragma unroll
        for (int q = 0; q < MC; ++q)
          if (q < mc) xm[(size_t)lg * m + q0 + q] = y[q];
      }
    }
  }
}

// 33 <= k <= 64: one warp per matrix, lane l holds physical rows l and 32 + l.
// As in the one-row kernel, rows never move: each keeps a logical position,
// the argmax breaks ties on it, and own[j] (shared memory: lane * 2 + slot of
// logical row j) drives the substitutions.
constexpr int GW2 = 4;       // warps per CTA
constexpr int S2 = 65;       // staging row stride (odd: conflict-free row reads)
constexpr int W2_FLOATS = 64 * S2 + 64 + 64;  // staging + pivot row + own[] (ints)

template <int MC>
__global__ void __launch_bounds__(GW2 * 32) gesv_warp2_kernel(const GesvParams p) {
  extern __shared__ __align__(16) float smw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = p.k, m = p.m;
  float* S = smw + warp * W2_FLOATS;
  float* P = S + 64 * S2;                                // pivot row (64 floats)
  int* ownS = reinterpret_cast<int*>(P + 64);            // 64 ints
  const int r1 = 32 + lane;
  const int64_t nw = (int64_t)gridDim.x * GW2;
  for (int64_t mat = (int64_t)blockIdx.x * GW2 + warp; mat < p.batch; mat += nw) {
    const float* A = p.A + mat * (size_t)n * n;
    __syncwarp();
    for (int e = lane; e < n * n; e += 32) {
      const int r = e / n, c = e - r * n;
      S[r * S2 + c] = A[e];
    }
    __syncwarp();
    float a0[64], a1[64];
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      a0[c] = (lane < n && c < n) ? S[lane * S2 + c] : (c == lane ? 1.f : 0.f);
      a1[c] = (r1 < n && c < n) ? S[r1 * S2 + c] : (c == r1 ? 1.f : 0.f);
    }
    int lg0 = lane, lg1 = r1;  // logical rows of this lane's two rows
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      if (j >= n) break;
      float v0 = (lg0 >= j) ? fabsf(a0[j]) : -1.f;
      float v1 = (lg1 >= j) ? fabsf(a1[j]) : -1.f;
      if (!(v0 == v0)) v0 = 0.f;  // NaN never beats the running maximum
      if (!(v1 == v1)) v1 = 0.f;
      float v = v0;
      int key = lg0;
      if (v1 > v || (v1 == v && lg1 < key)) {
        v = v1;
        key = lg1;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, v, o);
        const int ok = __shfl_xor_sync(kFull, key, o);
        if (ov > v || (ov == v && ok < key)) {
          v = ov;
          key = ok;
        }
      }
      const bool m0 = lg0 == key, m1 = lg1 == key;
      const int pl = __ffs(__ballot_sync(kFull, m0 || m1)) - 1;
      const int ps = __shfl_sync(kFull, m1 ? 1 : 0, pl);  // slot of the pivot row in its lane
      if (lane == 0) ownS[j] = 2 * pl + ps;
      const bool piv0 = lane == pl && ps == 0, piv1 = lane == pl && ps == 1;
      if (lg0 == j) lg0 = key;
      else if (piv0) lg0 = j;
      if (lg1 == j) lg1 = key;
      else if (piv1) lg1 = j;
      const float d = __shfl_sync(kFull, ps ? a1[j] : a0[j], pl);
      if (d != 0.f) {
        if (lane == pl) {
#pragma unroll
          for (int c4 = ((j + 1) >> 2) << 2; c4 < 64; c4 += 4)
            *reinterpret_cast<float4*>(P + c4) = ps ? make_float4(a1[c4], a1[c4 + 1], a1[c4 + 2], a1[c4 + 3])
                                                    : make_float4(a0[c4], a0[c4 + 1], a0[c4 + 2], a0[c4 + 3]);
        }
        __syncwarp();
        const float rd = 1.f / d;
        const bool u0 = lg0 > j, u1 = lg1 > j;
        const float l0 = a0[j] * rd, l1 = a1[j] * rd;
        if (u0) a0[j] = l0;
        if (u1) a1[j] = l1;
#pragma unroll
        for (int c4 = ((j + 1) >> 2) << 2; c4 < 64; c4 += 4) {
          const float4 w = *reinterpret_cast<const float4*>(P + c4);
          const float ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int c = c4 + i;
            if (c > j) {
              if (u0) a0[c] = fmaf(-l0, ww[i], a0[c]);
              if (u1) a1[c] = fmaf(-l1, ww[i], a1[c]);
            }
          }
        }
        __syncwarp();
      }
    }
    __syncwarp();
    const float* bm = p.b + mat * (size_t)n * m;
    float* xm = p.x + mat * (size_t)n * m;
    for (int q0 = 0; q0 < m; q0 += MC) {
      const int mc = (m - q0) < MC ? (m - q0) : MC;
      float y0[MC], y1[MC];
#pragma unroll
      for (int q = 0; q < MC; ++q) {
        y0[q] = (lane < n && q < mc) ? bm[(size_t)lane * m + q0 + q] : 0.f;
        y1[q] = (r1 < n && q < mc) ? bm[(size_t)r1 * m + q0 + q] : 0.f;
      }
      // forward, unit lower, logical order
#pragma unroll
      for (int pp = 0; pp < 64; ++pp) {
        if (pp >= n) break;
        const int o = ownS[pp], src = o >> 1, sl = o & 1;
#pragma unroll
        for (int q = 0; q < MC; ++q) {
          const float yp = __shfl_sync(kFull, sl ? y1[q] : y0[q], src);
          if (lg0 > pp) y0[q] = fmaf(-a0[pp], yp, y0[q]);
          if (lg1 > pp) y1[q] = fmaf(-a1[pp], yp, y1[q]);
        }
      }
      // backward, upper, dividing by U_pp
#pragma unroll
      for (int pp = 63; pp >= 0; --pp) {
        if (pp >= n) continue;
        const int o = ownS[pp], src = o >> 1, sl = o & 1;
        const bool me0 = lane == src && sl == 0, me1 = lane == src && sl == 1;
#pragma unroll
        for (int q = 0; q < MC; ++q) {
          const float own = me0 ? y0[q] / a0[pp] : (me1 ? y1[q] / a1[pp] : 0.f);
          const float xv = __shfl_sync(kFull, own, src);
          if (me0) y0[q] = xv;
          else if (lg0 < pp) y0[q] = fmaf(-a0[pp], xv, y0[q]);
          if (me1) y1[q] = xv;
          else if (lg1 < pp) y1[q] = fmaf(-a1[pp], xv, y1[q]);
        }
      }
#pragma unroll
      for (int q = 0; q < MC; ++q)
        if (q < mc) {
          if (lane < n) xm[(size_t)lg0 * m + q0 + q] = y0[q];
          if (r1 < n) xm[(size_t)lg1 * m + q0 + q] = y1[q];
        }
    }
  }
}

template <bool SMEM>
__global__ void __launch_bounds__(GT) gesv_cta_kernel(const GesvParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float sVal[GT / 32];
  __shared__ int sIdx[GT / 32];
  const int n = p.k, m = p.m, LD = n | 1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* a = SMEM ? sm : p.ws + (size_t)blockIdx.x * n * LD;
  int* piv = reinterpret_cast<int*>(SMEM ? sm + (size_t)n * LD : sm);
  float* ys = reinterpret_cast<float*>(piv + n);
  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x) {
    const float* A = p.A + mat * (size_t)n * n;
    __syncthreads();
    for (int e = tid; e < n * n; e += GT) {
      const int r = e / n, c = e - r * n;
      a[(size_t)r * LD + c] = A[e];
    }
    __syncthreads();
    for (int j = 0; j < n; ++j) {
      float v = 0.f;
      int idx = j;
      for (int i = j + tid; i < n; i += GT) {
        const float t = fabsf(a[(size_t)i * LD + j]);
        if (t > v) {
          v = t;
          idx = i;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(kFull, v, o);
        const int oi = __shfl_xor_sync(kFull, idx, o);
        if (ov > v || (ov == v && oi < idx)) {
          v = ov;
          idx = oi;
        }
      }
      if (lane == 0) {
        sVal[warp] = v;
        sIdx[warp] = idx;
      }
      __syncthreads();
      if (tid == 0) {
        float bv = sVal[0];
        int bi = sIdx[0];
        for (int w = 1; w < GT / 32; ++w)
          if (sVal[w] > bv || (sVal[w] == bv && sIdx[w] < bi)) {
            bv = sVal[w];
            bi = sIdx[w];
          }
        piv[j] = bi;
      }
      __syncthreads();
      const int pr = piv[j];
      if (pr != j) {
        for (int c = tid; c < n; c += GT) {
          const float t = a[(size_t)j * LD + c];
          a[(size_t)j * LD + c] = a[(size_t)pr * LD + c];
          a[(size_t)pr * LD + c] = t;
        }
        __syncthreads();
      }
      const float d = a[(size_t)j * LD + j];
      if (d != 0.f) {
        const float inv = 1.f / d;
        for (int i = j + 1 + warp; i < n; i += GT / 32) {
          const float l = a[(size_t)i * LD + j] * inv;
          for (int c = j + 1 + lane; c < n; c += 32)
            a[(size_t)i * LD + c] = fmaf(-l, a[(size_t)j * LD + c], a[(size_t)i * LD + c]);
          __syncwarp();
          if (lane == 0) a[(size_t)i * LD + j] = l;
        }
      }
      __syncthreads();
    }
    // one warp per right-hand side
    const float* bm = p.b + mat * (size_t)n * m;
    float* xm = p.x + mat * (size_t)n * m;
    float* y = ys + (size_t)warp * n;
    for (int q0 = 0; q0 < m; q0 += GCH) {
      const int q = q0 + warp;
      if (q < m) {
        for (int i = lane; i < n; i += 32) y[i] = bm[(size_t)i * m + q];
        __syncwarp();
        if (lane == 0)
          for (int i = 0; i < n; ++i) {
            const int pi = piv[i];
            if (pi != i) {
              const float t = y[i];
              y[i] = y[pi];
              y[pi] = t;
            }
          }
        __syncwarp();
        for (int pp = 0; pp < n; ++pp) {
          const float yp = y[pp];
          for (int i = pp + 1 + lane; i < n; i += 32) y[i] = fmaf(-a[(size_t)i * LD + pp], yp, y[i]);
          __syncwarp();
        }
        for (int pp = n - 1; pp >= 0; --pp) {
          const float xv = y[pp] / a[(size_t)pp * LD + pp];
          for (int i = lane; i < pp; i += 32) y[i] = fmaf(-a[(size_t)i * LD + pp], xv, y[i]);
          __syncwarp();
          if (lane == 0) y[pp] = xv;
          __syncwarp();
        }
        for (int i = lane; i < n; i += 32) xm[(size_t)i * m + q] = y[i];
      }
      __syncwarp();
    }
  }
}

static size_t gesv_cta_smem(int k, bool smem) {
  const size_t ld = (size_t)(k | 1);
  return (smem ? (size_t)k * ld * sizeof(float) : 0) + (size_t)k * sizeof(int) + (size_t)GCH * k * sizeof(float);
}

int gesv_grid(int64_t batch, int k, int sm_count) {
  if (gesv_blocked_fits(k)) return gesv_blocked_grid(batch, k, sm_count);
  const int64_t cap = (int64_t)sm_count * 2;
  return (int)(batch < cap ? batch : cap);
}

size_t gesv_ws_floats(int64_t batch, int k, int sm_count) {
  if (k <= kGesvSmemMaxK || batch <= 0) return 0;
  return (size_t)gesv_grid(batch, k, sm_count) * (size_t)k * (size_t)(k | 1);
}

template <int MC>
static cudaError_t launch_gesv_warp(const GesvParams& p, int sm_count, cudaStream_t s) {
  static int cache[64];
  int occ = 0;
  cudaError_t e = kernel_occupancy(gesv_warp_kernel<MC>, GW * 32, 0, cache, &occ);
  if (e != cudaSuccess) return e;
  const int64_t need = (p.batch + GW - 1) / GW;
  const int64_t cap = (int64_t)sm_count * occ;
  gesv_warp_kernel<MC><<<(int)(need < cap ? need : cap), GW * 32, 0, s>>>(p);
  return cudaGetLastError();
}

template <int MC>
static cudaError_t launch_gesv_warp2(const GesvParams& p, int sm_count, cudaStream_t s) {
  static int cache[64];
  int occ = 0;
  const size_t smem = (size_t)GW2 * W2_FLOATS * sizeof(float);
  cudaError_t e = kernel_occupancy(gesv_warp2_kernel<MC>, GW2 * 32, smem, cache, &occ);
  if (e != cudaSuccess) return e;
  const int64_t need = (p.batch + GW2 - 1) / GW2;
  const int64_t cap = (int64_t)sm_count * occ;
  gesv_warp2_kernel<MC><<<(int)(need < cap ? need : cap), GW2 * 32, smem, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_gesv(const GesvParams& p, int sm_count, cudaStream_t s) {
  if (p.k <= 32) return p.m <= 1 ? launch_gesv_warp<1>(p, sm_count, s) : launch_gesv_warp<4>(p, sm_count, s);
  if (p.k <= 64) return p.m <= 1 ? launch_gesv_warp2<1>(p, sm_count, s) : launch_gesv_warp2<4>(p, sm_count, s);
  if (p.k <= kGesvSmemMaxK) {
    const size_t smem = gesv_cta_smem(p.k, true);
    static int cache[64];
    int occ = 0;
    cudaError_t e = kernel_occupancy(gesv_cta_kernel<true>, GT, smem, cache, &occ);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gesv_cta_kernel<true>, GT, smem);
    if (e != cudaSuccess) return e;
    if (occ < 1) occ = 1;
    const int64_t cap = (int64_t)sm_count * occ;
    gesv_cta_kernel<true><<<(int)(p.batch < cap ? p.batch : cap), GT, smem, s>>>(p);
    return cudaGetLastError();
  }
  if (gesv_blocked_fits(p.k)) return launch_gesv_blocked(p, gesv_grid(p.batch, p.k, sm_count), s);
  const size_t smem = gesv_cta_smem(p.k, false);
  static int cache[64];
  int occ = 0;
  cudaError_t e = kernel_occupancy(gesv_cta_kernel<false>, GT, smem, cache, &occ);
  if (e != cudaSuccess) return e;
  gesv_cta_kernel<false><<<gesv_grid(p.batch, p.k, sm_count), GT, smem, s>>>(p);
  return cudaGetLastError();
}

}  // namespace b2c
