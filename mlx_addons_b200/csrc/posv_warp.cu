// Register-resident batched Cholesky factor + solve for k <= 64.
//
// Replaces the reference's one-thread-per-matrix (tier ST, k <= 32,
// src/mlx_addons/linalg/_metal_kernels.py:26-101) and threadgroup (tier TG,
// 33 <= k <= 80, _metal_kernels.py:147-246) kernels, keeping their
// arithmetic contract: clamped pivot sqrt(max(s, 1e-12)), column scaling by
// 1/L_jj, forward then back substitution, lower triangle of A read only,
// upper triangle of an L output zeroed.
//
// Two designs:
//  * thread tier (k <= 16): one thread owns a whole matrix in registers (a
//    square array up to k = 9, a packed lower triangle above); a CTA stages
//    32..128 consecutive matrices through shared memory so global traffic
//    stays coalesced (the reference's per-thread layout puts neighbouring
//    threads k*k floats apart). With m <= 4 the staging is double-buffered:
//    A and b of the next tile load while this tile is factored and solved.
//    Measured on B200 at k = 16 (B = 10,000, m = 1) this issues a small
//    fraction of the warp tier's instructions per matrix: 8.5 us against
//    14.4 us for the warp tier.
//  * warp tier (17 <= k <= 32; the k <= 64 kernel of posv_warp64.cu takes
//    33..64): lanes own rows. k is padded to KP (16, 32,
//    40..64) with an identity block, which leaves L, x and logdet unchanged.
//    KP <= 32: 32/KP matrices per warp, one row per lane. KP > 32: one matrix
//    per warp, lane l owns rows l and 32 + l. The factorisation is
//    right-looking: each step publishes column j through a double-buffered
//    shared-memory vector (one __syncwarp per step) and every lane applies a
//    rank-1 update to its rows from registers. Each warp stages its next
//    matrix with cp.async while it factors the current one, and only the
//    lower blocks the algorithm reads are fetched (rows 0..31 stop at column
//    31), which saves a quarter of the HBM reads at k = 64.
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

// ---------------------------------------------------------------------------
// Warp tier
// ---------------------------------------------------------------------------

template <int KP>
struct WarpShape {
  static constexpr bool TWO = KP > 32;
  static constexpr int R0 = TWO ? 32 : KP;           // length of the first-row register array
  static constexpr int G = TWO ? 1 : 32 / KP;        // matrices per warp
  static constexpr int NB = TWO ? KP - 32 : 0;       // number of second rows
  static constexpr int S0 = R0 + 4;                  // smem row stride (floats); S0/4 odd
  static constexpr int S1 = KP + 4;                  // smem row stride of second rows; S1/4 odd
  static constexpr int STAGE0 = 32 * S0;
  static constexpr int STAGE1 = TWO ? NB * S1 : 0;
  static constexpr int GS = KP + 4;                  // per-group stride of the column buffer
  static constexpr int CB = TWO ? 68 : G * GS;       // one column buffer (floats)
  static constexpr int CS = KP + 4;                  // chunk-buffer row stride
  static constexpr int CHUNK = G * 8 * CS;
  static constexpr int WARP_FLOATS = STAGE0 + STAGE1 + 2 * CB + CHUNK;
  static_assert(KP % 8 == 0 && KP >= 16 && KP <= 64, "KP");
  static_assert((S0 / 4) % 2 == 1 && (S1 / 4) % 2 == 1, "odd float4 strides keep row reads conflict-free");
};

template <int KP>
__device__ __forceinline__ void warp_stage(const PosvParams& p, int64_t unit, float* st0, float* st1, int lane) {
  using W = WarpShape<KP>;
  const int K = p.k;
  const size_t kk = (size_t)K * K;
  if (p.vec && (K & 3) == 0) {
    const int q4 = K >> 2;
    if (!W::TWO) {
      const int per = K * q4, total = W::G * per;
      for (int f = lane; f < total; f += 32) {
        const int gg = f / per, rem = f - gg * per, r = rem / q4, q = rem - r * q4;
        const int64_t mat = unit * W::G + gg;
        if (mat < p.batch) cp_async16(st0 + (gg * KP + r) * W::S0 + 4 * q, p.A + mat * kk + (size_t)r * K + 4 * q);
      }
    } else {
      const int64_t mat = unit;
      if (mat < p.batch) {
        const float* src = p.A + mat * kk;
        for (int f = lane; f < 256; f += 32) {
          const int r = f >> 3, q = f & 7;
          cp_async16(st0 + r * W::S0 + 4 * q, src + (size_t)r * K + 4 * q);
        }
        const int total = (K - 32) * q4;
        for (int f = lane; f < total; f += 32) {
          const int r = f / q4, q = f - r * q4;
          cp_async16(st1 + r * W::S1 + 4 * q, src + (size_t)(32 + r) * K + 4 * q);
        }
      }
    }
  } else {
    if (!W::TWO) {
      const int per = K * K, total = W::G * per;
      for (int f = lane; f < total; f += 32) {
        const int gg = f / per, rem = f - gg * per, r = rem / K, c = rem - r * K;
        const int64_t mat = unit * W::G + gg;
        if (mat < p.batch) cp_async4(st0 + (gg * KP + r) * W::S0 + c, p.A + mat * kk + rem);
      }
    } else {
      const int64_t mat = unit;
      if (mat < p.batch) {
        const float* src = p.A + mat * kk;
        for (int f = lane; f < 1024; f += 32) {
          const int r = f >> 5, c = f & 31;
          cp_async4(st0 + r * W::S0 + c, src + (size_t)r * K + c);
        }
        const int total = (K - 32) * K;
        for (int f = lane; f < total; f += 32) {
          const int r = f / K, c = f - r * K;
          cp_async4(st1 + r * W::S1 + c, src + (size_t)(32 + r) * K + c);
        }
      }
    }
  }
  cp_async_commit();
}

// Register cap: the fully unrolled code otherwise lets the scheduler hoist
// loads of several steps and climb to 255 registers; 3 (KP > 32) or 4 CTAs of
// 128 threads per SM keeps occupancy at the shared-memory limit.
template <int KP, int MC>
__global__ void __launch_bounds__(128, (KP > 32 ? 3 : 4)) posv_warp_kernel(const PosvParams p) {
  using W = WarpShape<KP>;
  extern __shared__ __align__(16) float smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float* st0 = smem + warp * W::WARP_FLOATS;
  float* st1 = st0 + W::STAGE0;
  float* cbuf = st1 + W::STAGE1;
  float* chunk = cbuf + 2 * W::CB;

  const int K = p.k;
  const size_t kk = (size_t)K * K;
  const int g = W::TWO ? 0 : lane / KP;
  const int r0 = W::TWO ? lane : lane % KP;  // first row owned by this lane
  const int r1 = 32 + lane;                  // second row (KP > 32 only)
  const int seg = W::TWO ? 32 : KP;          // shuffle width
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t nunits = (p.batch + W::G - 1) / W::G;
  int64_t unit = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;

  if (unit < nunits) warp_stage<KP>(p, unit, st0, st1, lane);

  for (; unit < nunits; unit += nwarps) {
    cp_async_wait_all();
    __syncwarp();
    const int64_t mat = unit * W::G + g;
    const bool mvalid = mat < p.batch;

    float a0[W::R0];
    float a1[W::TWO ? KP : 1];
    {
      const float* src = st0 + (g * KP + r0) * W::S0;
#pragma unroll
      for (int c4 = 0; c4 < W::R0; c4 += 4) {
        const float4 v = *reinterpret_cast<const float4*>(src + c4);
        const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = c4 + i;
          a0[c] = (mvalid && r0 < K && c < K) ? vv[i] : (c == r0 ? 1.f : 0.f);
        }
      }
      if (W::TWO) {
        const int rr = lane < W::NB ? lane : W::NB - 1;
        const float* src1 = st1 + rr * W::S1;
#pragma unroll
        for (int c4 = 0; c4 < KP; c4 += 4) {
          const float4 v = *reinterpret_cast<const float4*>(src1 + c4);
          const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int c = c4 + i;
            a1[c] = (mvalid && r1 < K && c < K) ? vv[i] : (c == r1 ? 1.f : 0.f);
          }
        }
      }
    }
    __syncwarp();
    if (unit + nwarps < nunits) warp_stage<KP>(p, unit + nwarps, st0, st1, lane);

    // The first MC right-hand sides are loaded now, so that their global
    // latency overlaps the factorisation.
    float yp0[MC], yp1[MC];
    {
      const float* bm = p.b + (size_t)mat * K * p.m;
#pragma unroll
      for (int q = 0; q < MC; ++q) {
        const bool qok = q < p.m;
        yp0[q] = (mvalid && qok && r0 < K) ? bm[(size_t)r0 * p.m + q] : 0.f;
        yp1[q] = (W::TWO && mvalid && qok && r1 < K) ? bm[(size_t)r1 * p.m + q] : 0.f;
      }
    }

    // ---- right-looking factorisation ------------------------------------
    float inv0 = 1.f, inv1 = 1.f;
#pragma unroll
    for (int j = 0; j < KP; ++j) {
      const float dsrc = (j < W::R0) ? a0[j < W::R0 ? j : 0] : a1[W::TWO ? j : 0];
      const float ajj = __shfl_sync(kFull, dsrc, j & 31, seg);
      float d;
      const float r = clamped_rsqrt(ajj, d);
      float* cb = cbuf + (j & 1) * W::CB;
      float v0 = 0.f, v1 = 0.f;
      if (j < W::R0) {
        const int jj = j < W::R0 ? j : 0;
        v0 = (r0 == j) ? d : a0[jj] * r;
        a0[jj] = v0;
        inv0 = (r0 == j) ? r : inv0;
        cb[(W::TWO ? 0 : g * W::GS) + r0] = v0;
      }
      if (W::TWO) {
        const int jj = W::TWO ? j : 0;
        v1 = (r1 == j) ? d : a1[jj] * r;
        a1[jj] = v1;
        inv1 = (r1 == j) ? r : inv1;
        cb[32 + lane] = v1;
      }
      __syncwarp();
      const float* cbg = cb + (W::TWO ? 0 : g * W::GS);
#pragma unroll
      for (int c4 = ((j + 1) >> 2) << 2; c4 < KP; c4 += 4) {
        const float4 w = *reinterpret_cast<const float4*>(cbg + c4);
        const float ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = c4 + i;
          if (c > j) {
            if (c < W::R0 && j < W::R0) a0[c < W::R0 ? c : 0] = fmaf(-v0, ww[i], a0[c < W::R0 ? c : 0]);
            if (W::TWO) a1[W::TWO ? c : 0] = fmaf(-v1, ww[i], a1[W::TWO ? c : 0]);
          }
        }
      }
    }

    // ---- log-determinant: 2 * sum log L_jj = -2 * sum log(1/L_jj) --------
    if (p.logdet) {
      // rows past k (identity padding) add nothing, even when a NaN in the
      // input has reached them through 0 * NaN in the updates
      float lg = (r0 < K) ? -logf(inv0) : 0.f;
      if (W::TWO && r1 < K) lg -= logf(inv1);
      lg = warp_sum(lg, seg);
      if (r0 == 0 && mvalid) p.logdet[mat] = 2.f * lg;
    }

    // ---- factor output, upper triangle zeroed -----------------------------
    if (p.L && mvalid) {
      float* Lm = p.L + mat * kk;
      if (r0 < K) {
        float* row = Lm + (size_t)r0 * K;
        if (p.vec && (K & 3) == 0) {
#pragma unroll
          for (int c4 = 0; c4 < W::R0; c4 += 4)
            if (c4 < K) {
              float4 v;
              v.x = (c4 + 0 <= r0) ? a0[c4 + 0] : 0.f;
              v.y = (c4 + 1 <= r0) ? a0[c4 + 1] : 0.f;
              v.z = (c4 + 2 <= r0) ? a0[c4 + 2] : 0.f;
              v.w = (c4 + 3 <= r0) ? a0[c4 + 3] : 0.f;
              *reinterpret_cast<float4*>(row + c4) = v;
            }
        } else {
#pragma unroll
          for (int c = 0; c < W::R0; ++c)
            if (c < K) row[c] = (c <= r0) ? a0[c] : 0.f;
        }
        if (W::TWO)
          for (int c = 32; c < K; ++c) row[c] = 0.f;
      }
      if (W::TWO && r1 < K) {
        float* row = Lm + (size_t)r1 * K;
        if (p.vec && (K & 3) == 0) {
#pragma unroll
          for (int c4 = 0; c4 < KP; c4 += 4)
            if (c4 < K) {
              float4 v;
              v.x = (c4 + 0 <= r1) ? a1[W::TWO ? c4 + 0 : 0] : 0.f;
              v.y = (c4 + 1 <= r1) ? a1[W::TWO ? c4 + 1 : 0] : 0.f;
              v.z = (c4 + 2 <= r1) ? a1[W::TWO ? c4 + 2 : 0] : 0.f;
              v.w = (c4 + 3 <= r1) ? a1[W::TWO ? c4 + 3 : 0] : 0.f;
              *reinterpret_cast<float4*>(row + c4) = v;
            }
        } else {
#pragma unroll
          for (int c = 0; c < KP; ++c)
            if (c < K) row[c] = (c <= r1) ? a1[W::TWO ? c : 0] : 0.f;
        }
      }
    }

    // ---- forward + back substitution, MC right-hand sides at a time -------
    for (int q0 = 0; q0 < p.m; q0 += MC) {
      float y0[MC], y1[MC];
      const float* bm = p.b + (size_t)mat * K * p.m;
#pragma unroll
      for (int q = 0; q < MC; ++q) {
        const bool qok = q0 + q < p.m;
        y0[q] = q0 == 0 ? yp0[q] : ((mvalid && qok && r0 < K) ? bm[(size_t)r0 * p.m + q0 + q] : 0.f);
        y1[q] = q0 == 0 ? yp1[q] : ((W::TWO && mvalid && qok && r1 < K) ? bm[(size_t)r1 * p.m + q0 + q] : 0.f);
      }
      // forward: L y = b, column-oriented (lane-local L[r][j])
#pragma unroll
      for (int j = 0; j < KP; ++j) {
#pragma unroll
        for (int q = 0; q < MC; ++q) {
          const float own = (j < 32 || !W::TWO) ? y0[q] * inv0 : y1[q] * inv1;
          const float yj = __shfl_sync(kFull, own, j & 31, seg);
          if (j < W::R0) {
            const int jj = j < W::R0 ? j : 0;
            y0[q] = (r0 == j) ? yj : ((r0 > j) ? fmaf(-a0[jj], yj, y0[q]) : y0[q]);
          }
          if (W::TWO) {
            const int jj = W::TWO ? j : 0;
            y1[q] = (r1 == j) ? yj : ((r1 > j) ? fmaf(-a1[jj], yj, y1[q]) : y1[q]);
          }
        }
      }
      // backward: L^T x = y. Row i of L (held by one lane) is published 8 rows
      // at a time through the chunk buffer; lane r then reads L[i][r].
      float* ch = chunk + (W::TWO ? 0 : g * 8 * W::CS);
#pragma unroll
      for (int c0 = KP - 8; c0 >= 0; c0 -= 8) {
        if (W::TWO && c0 >= 32) {
          const int rr = r1 - c0;
          if (rr >= 0 && rr < 8) {
#pragma unroll
            for (int c4 = 0; c4 < KP; c4 += 4)
              *reinterpret_cast<float4*>(ch + rr * W::CS + c4) =
                  make_float4(a1[W::TWO ? c4 : 0], a1[W::TWO ? c4 + 1 : 0], a1[W::TWO ? c4 + 2 : 0],
                              a1[W::TWO ? c4 + 3 : 0]);
          }
        } else {
          const int rr = r0 - c0;
          if (rr >= 0 && rr < 8) {
#pragma unroll
            for (int c4 = 0; c4 < W::R0; c4 += 4)
              *reinterpret_cast<float4*>(ch + rr * W::CS + c4) =
                  make_float4(a0[c4], a0[c4 + 1], a0[c4 + 2], a0[c4 + 3]);
          }
        }
        __syncwarp();
#pragma unroll
        for (int i = c0 + 7; i >= c0; --i) {
          const float* Lrow = ch + (i - c0) * W::CS;
          const float l0 = Lrow[r0 < i ? r0 : 0];
          const float l1 = (W::TWO && i > 32) ? Lrow[r1 < i ? r1 : 0] : 0.f;
#pragma unroll
          for (int q = 0; q < MC; ++q) {
            const float own = (i < 32 || !W::TWO) ? y0[q] * inv0 : y1[q] * inv1;
            const float xi = __shfl_sync(kFull, own, i & 31, seg);
            if (i < W::R0) y0[q] = (r0 == i) ? xi : ((r0 < i) ? fmaf(-l0, xi, y0[q]) : y0[q]);
            else y0[q] = fmaf(-l0, xi, y0[q]);  // i >= 32: every first row r0 < 32 < i
            if (W::TWO && i >= 32) y1[q] = (r1 == i) ? xi : ((r1 < i) ? fmaf(-l1, xi, y1[q]) : y1[q]);
          }
        }
        __syncwarp();
      }
      if (mvalid) {
        float* xm = p.x + (size_t)mat * K * p.m;
#pragma unroll
        for (int q = 0; q < MC; ++q) {
          if (q0 + q < p.m) {
            if (r0 < K) xm[(size_t)r0 * p.m + q0 + q] = y0[q];
            if (W::TWO && r1 < K) xm[(size_t)r1 * p.m + q0 + q] = y1[q];
          }
        }
      }
    }
  }
  cp_async_wait_all();
}

// ---------------------------------------------------------------------------
// Thread tier (k <= 8)
// ---------------------------------------------------------------------------

// Row-major index of (i, j), j <= i, in a packed lower triangle.
__host__ __device__ constexpr int tri(int i, int j) { return i * (i + 1) / 2 + j; }

template <int K>
struct ThreadTile {
  // threads (= matrices) per CTA: keeps the static smem of the single-buffered
  // kernel under 48 KB and, above k = 8, three double-buffered CTAs per SM
  static constexpr int NT = (K * K <= 36) ? 128 : (K <= 8 ? 64 : 32);
  // Register layout of the factor: square for k <= 9, packed lower triangle
  // above. Both are indexed with compile-time indices only; with these
  // choices nvcc keeps every size in registers (no stack frame).
  static constexpr bool PACKED = K > 9;
};

template <int K, bool PACKED>
struct Factor;
template <int K>
struct Factor<K, false> {
  float v[K][K];
  __device__ __forceinline__ float& operator()(int i, int j) { return v[i][j]; }
};
template <int K>
struct Factor<K, true> {
  float v[K * (K + 1) / 2];
  __device__ __forceinline__ float& operator()(int i, int j) { return v[tri(i, j)]; }
};

template <int K, int MC>
__global__ void __launch_bounds__(ThreadTile<K>::NT) posv_thread_kernel(const PosvParams p) {
  constexpr int NT = ThreadTile<K>::NT;
  constexpr int KK = K * K;
  constexpr int SA = KK | 1;          // odd stride: conflict-free per-thread reads
  constexpr int SB = (K * MC) | 1;
  __shared__ __align__(16) float sA[NT * SA];
  __shared__ __align__(16) float sB[NT * SB];
  const int t = threadIdx.x;
  const int64_t ntiles = (p.batch + NT - 1) / NT;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t m0 = tile * NT;
    const int nmat = (int)((p.batch - m0) < NT ? (p.batch - m0) : NT);
    const float* Ag = p.A + m0 * KK;
    const int nA = nmat * KK;
    __syncthreads();  // previous tile's readers of sA/sB are done
    if (SA == KK && p.vec) {
      const int n4 = nA >> 2;
      for (int e = t; e < n4; e += NT) cp_async16(&sA[4 * e], Ag + 4 * e);
      for (int e = 4 * n4 + t; e < nA; e += NT) cp_async4(&sA[e], Ag + e);
    } else {
      for (int e = t; e < nA; e += NT) {
        const int mm = e / KK, o = e - mm * KK;
        cp_async4(&sA[mm * SA + o], Ag + e);
      }
    }
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();

    const bool valid = t < nmat;
    Factor<K, ThreadTile<K>::PACKED> a;
#pragma unroll
    for (int i = 0; i < K; ++i)
#pragma unroll
      for (int j = 0; j <= i; ++j) a(i, j) = valid ? sA[t * SA + i * K + j] : (i == j ? 1.f : 0.f);

    // left-looking factorisation, the order of _metal_kernels.py:36-50
    float inv[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
      float s = a(j, j);
#pragma unroll
      for (int q = 0; q < j; ++q) s = fmaf(-a(j, q), a(j, q), s);
      float d;
      const float r = clamped_rsqrt(s, d);
      a(j, j) = d;
      inv[j] = r;
#pragma unroll
      for (int i = j + 1; i < K; ++i) {
        float tt = a(i, j);
#pragma unroll
        for (int q = 0; q < j; ++q) tt = fmaf(-a(i, q), a(j, q), tt);
        a(i, j) = tt * r;
      }
    }
    if (p.logdet && valid) {
      float dg[K];
#pragma unroll
      for (int j = 0; j < K; ++j) dg[j] = a(j, j);
      const float lg = sum_log_pos(dg);
      p.logdet[m0 + t] = 2.f * lg;
    }
    if (p.L) {
      __syncthreads();
#pragma unroll
      for (int i = 0; i < K; ++i)
#pragma unroll
        for (int j = 0; j < K; ++j) sA[t * SA + i * K + j] = (j <= i) ? a(i, j <= i ? j : 0) : 0.f;
      __syncthreads();
      float* Lg = p.L + m0 * KK;
      for (int e = t; e < nA; e += NT) {
        const int mm = e / KK, o = e - mm * KK;
        Lg[e] = sA[mm * SA + o];
      }
    }
    for (int q0 = 0; q0 < p.m; q0 += MC) {
      const int mc = (p.m - q0) < MC ? (p.m - q0) : MC;
      const int per = K * mc, nB = nmat * per;
      const float* bg = p.b + m0 * K * p.m;
      __syncthreads();
      for (int e = t; e < nB; e += NT) {
        const int mm = e / per, rem = e - mm * per, r = rem / mc, q = rem - r * mc;
        cp_async4(&sB[mm * SB + r * MC + q], bg + (size_t)mm * K * p.m + (size_t)r * p.m + q0 + q);
      }
      cp_async_commit();
      cp_async_wait_all();
      __syncthreads();
      float y[K][MC];
#pragma unroll
      for (int r = 0; r < K; ++r)
#pragma unroll
        for (int q = 0; q < MC; ++q) y[r][q] = (valid && q < mc) ? sB[t * SB + r * MC + q] : 0.f;
#pragma unroll
      for (int q = 0; q < MC; ++q) {
#pragma unroll
        for (int i = 0; i < K; ++i) {
          float tt = y[i][q];
#pragma unroll
          for (int c = 0; c < i; ++c) tt = fmaf(-a(i, c), y[c][q], tt);
          y[i][q] = tt * inv[i];
        }
#pragma unroll
        for (int i = K - 1; i >= 0; --i) {
          float tt = y[i][q];
#pragma unroll
          for (int c = i + 1; c < K; ++c) tt = fmaf(-a(c, i), y[c][q], tt);
          y[i][q] = tt * inv[i];
        }
      }
      __syncthreads();
#pragma unroll
      for (int r = 0; r < K; ++r)
#pragma unroll
        for (int q = 0; q < MC; ++q) sB[t * SB + r * MC + q] = y[r][q];
      __syncthreads();
      float* xg = p.x + m0 * K * p.m;
      for (int e = t; e < nB; e += NT) {
        const int mm = e / per, rem = e - mm * per, r = rem / mc, q = rem - r * mc;
        xg[(size_t)mm * K * p.m + (size_t)r * p.m + q0 + q] = sB[mm * SB + r * MC + q];
      }
    }
  }
}

// Double-buffered variant for m == MC (every right-hand side in one pass, and
// the staging divisions by K*m are by constants): A and b of a tile arrive in
// one cp.async group, and the next tile's group is in flight while the
// current tile is factored, solved and stored.
template <int K, int MC>
__global__ void __launch_bounds__(ThreadTile<K>::NT) posv_thread_db_kernel(const PosvParams p) {
  constexpr int NT = ThreadTile<K>::NT;
  constexpr int KK = K * K;
  constexpr int SA = KK | 1;
  constexpr int SB = (K * MC) | 1;
  constexpr int BUF = NT * (SA + SB);
  extern __shared__ __align__(16) float smem[];
  const int t = threadIdx.x;
  constexpr int m = MC;  // the launcher picks MC == p.m
  const int64_t ntiles = (p.batch + NT - 1) / NT;

  auto stage = [&](int64_t tile, float* buf) {
    const int64_t m0 = tile * NT;
    const int nmat = (int)((p.batch - m0) < NT ? (p.batch - m0) : NT);
    float* sA = buf;
    float* sB = buf + NT * SA;
    const float* Ag = p.A + m0 * KK;
    const int nA = nmat * KK;
    if (SA == KK && p.vec) {
      const int n4 = nA >> 2;
      for (int e = t; e < n4; e += NT) cp_async16(&sA[4 * e], Ag + 4 * e);
      for (int e = 4 * n4 + t; e < nA; e += NT) cp_async4(&sA[e], Ag + e);
    } else {
      for (int e = t; e < nA; e += NT) {
        const int mm = e / KK, o = e - mm * KK;
        cp_async4(&sA[mm * SA + o], Ag + e);
      }
    }
    const int per = K * m, nB = nmat * per;
    const float* bg = p.b + m0 * per;
    for (int e = t; e < nB; e += NT) {
      const int mm = e / per, rem = e - mm * per, r = rem / m, q = rem - r * m;
      cp_async4(&sB[mm * SB + r * MC + q], bg + e);
    }
  };

  int64_t tile = blockIdx.x;
  int cur = 0;
  if (tile < ntiles) stage(tile, smem);
  cp_async_commit();
  for (; tile < ntiles; tile += gridDim.x, cur ^= 1) {
    float* buf = smem + cur * BUF;
    const int64_t next = tile + gridDim.x;
    if (next < ntiles) stage(next, smem + (cur ^ 1) * BUF);
    cp_async_commit();
    asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    __syncthreads();
    float* sA = buf;
    float* sB = buf + NT * SA;
    const int64_t m0 = tile * NT;
    const int nmat = (int)((p.batch - m0) < NT ? (p.batch - m0) : NT);
    const bool valid = t < nmat;

    Factor<K, ThreadTile<K>::PACKED> a;
#pragma unroll
    for (int i = 0; i < K; ++i)
#pragma unroll
      for (int j = 0; j <= i; ++j) a(i, j) = valid ? sA[t * SA + i * K + j] : (i == j ? 1.f : 0.f);
    float inv[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
      float s = a(j, j);
#pragma unroll
      for (int q = 0; q < j; ++q) s = fmaf(-a(j, q), a(j, q), s);
      float d;
      const float r = clamped_rsqrt(s, d);
      a(j, j) = d;
      inv[j] = r;
#pragma unroll
      for (int i = j + 1; i < K; ++i) {
        float tt = a(i, j);
#pragma unroll
        for (int q = 0; q < j; ++q) tt = fmaf(-a(i, q), a(j, q), tt);
        a(i, j) = tt * r;
      }
    }
    if (p.logdet && valid) {
      float dg[K];
#pragma unroll
      for (int j = 0; j < K; ++j) dg[j] = a(j, j);
      const float lg = sum_log_pos(dg);
      p.logdet[m0 + t] = 2.f * lg;
    }
    float y[K][MC];
#pragma unroll
    for (int r = 0; r < K; ++r)
#pragma unroll
      for (int q = 0; q < MC; ++q) y[r][q] = (valid && q < m) ? sB[t * SB + r * MC + q] : 0.f;
#pragma unroll
    for (int q = 0; q < MC; ++q) {
#pragma unroll
      for (int i = 0; i < K; ++i) {
        float tt = y[i][q];
#pragma unroll
        for (int c = 0; c < i; ++c) tt = fmaf(-a(i, c), y[c][q], tt);
        y[i][q] = tt * inv[i];
      }
#pragma unroll
      for (int i = K - 1; i >= 0; --i) {
        float tt = y[i][q];
#pragma unroll
        for (int c = i + 1; c < K; ++c) tt = fmaf(-a(c, i), y[c][q], tt);
        y[i][q] = tt * inv[i];
      }
    }
    // x and L leave through this tile's buffer, then as coalesced stores
    __syncthreads();
#pragma unroll
    for (int r = 0; r < K; ++r)
#pragma unroll
      for (int q = 0; q < MC; ++q) sB[t * SB + r * MC + q] = y[r][q];
    if (p.L) {
#pragma unroll
      for (int i = 0; i < K; ++i)
#pragma unroll
        for (int j = 0; j < K; ++j) sA[t * SA + i * K + j] = (j <= i) ? a(i, j <= i ? j : 0) : 0.f;
    }
    __syncthreads();
    const int per = K * m, nB = nmat * per;
    float* xg = p.x + m0 * per;
    for (int e = t; e < nB; e += NT) {
      const int mm = e / per, rem = e - mm * per, r = rem / m, q = rem - r * m;
      xg[e] = sB[mm * SB + r * MC + q];
    }
    if (p.L) {
      float* Lg = p.L + m0 * KK;
      const int nA = nmat * KK;
      for (int e = t; e < nA; e += NT) {
        const int mm = e / KK, o = e - mm * KK;
        Lg[e] = sA[mm * SA + o];
      }
    }
    __syncthreads();  // this buffer is refilled by the stage two tiles ahead
  }
  cp_async_wait_all();
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------

template <int KP, int MC>
static cudaError_t launch_warp_t(const PosvParams& p, int sm_count, cudaStream_t s) {
  using W = WarpShape<KP>;
  constexpr int threads = 128;
  const size_t smem = (size_t)(threads / 32) * W::WARP_FLOATS * sizeof(float);
  auto kern = posv_warp_kernel<KP, MC>;
  static int cache[64];
  int occ = 0;
  cudaError_t e = kernel_occupancy(kern, threads, smem, cache, &occ);
  if (e != cudaSuccess) return e;
  const int64_t units = (p.batch + W::G - 1) / W::G;
  const int64_t need = (units + threads / 32 - 1) / (threads / 32);
  const int64_t cap = (int64_t)sm_count * occ;
  const int grid = (int)(need < cap ? need : cap);
  kern<<<grid, threads, smem, s>>>(p);
  return cudaGetLastError();
}

template <int K, int MC>
static cudaError_t launch_thread_t(const PosvParams& p, int sm_count, cudaStream_t s) {
  constexpr int NT = ThreadTile<K>::NT;
  auto kern = posv_thread_kernel<K, MC>;
  static int cache[64];
  int occ = 0;
  cudaError_t e = kernel_occupancy(kern, NT, 0, cache, &occ);
  if (e != cudaSuccess) return e;
  const int64_t tiles = (p.batch + NT - 1) / NT;
  const int64_t cap = (int64_t)sm_count * occ;
  const int grid = (int)(tiles < cap ? tiles : cap);
  kern<<<grid, NT, 0, s>>>(p);
  return cudaGetLastError();
}

template <int K, int MC>
static cudaError_t launch_thread_db_t(const PosvParams& p, int sm_count, cudaStream_t s) {
  constexpr int NT = ThreadTile<K>::NT;
  constexpr int SA = (K * K) | 1, SB = (K * MC) | 1;
  const size_t smem = 2 * (size_t)NT * (SA + SB) * sizeof(float);
  auto kern = posv_thread_db_kernel<K, MC>;
  static int cache[64];
  int occ = 0;
  cudaError_t e = kernel_occupancy(kern, NT, smem, cache, &occ);
  if (e != cudaSuccess) return e;
  const int64_t tiles = (p.batch + NT - 1) / NT;
  const int64_t cap = (int64_t)sm_count * occ;
  const int grid = (int)(tiles < cap ? tiles : cap);
  kern<<<grid, NT, smem, s>>>(p);
  return cudaGetLastError();
}

template <int K>
static cudaError_t launch_thread_k(const PosvParams& p, int sm, cudaStream_t s) {
  switch (p.m) {
    case 1: return launch_thread_db_t<K, 1>(p, sm, s);
    case 2: return launch_thread_db_t<K, 2>(p, sm, s);
    case 3: return launch_thread_db_t<K, 3>(p, sm, s);
    case 4: return launch_thread_db_t<K, 4>(p, sm, s);
    default: break;
  }
  return p.m <= 1 ? launch_thread_t<K, 1>(p, sm, s) : launch_thread_t<K, 4>(p, sm, s);
}

template <int KP>
static cudaError_t launch_warp_k(const PosvParams& p, int sm, cudaStream_t s) {
  return p.m <= 1 ? launch_warp_t<KP, 1>(p, sm, s) : launch_warp_t<KP, 4>(p, sm, s);
}

cudaError_t launch_posv_small(const PosvParams& p, int sm_count, cudaStream_t s) {
  switch (p.k) {
    case 1: return launch_thread_k<1>(p, sm_count, s);
    case 2: return launch_thread_k<2>(p, sm_count, s);
    case 3: return launch_thread_k<3>(p, sm_count, s);
    case 4: return launch_thread_k<4>(p, sm_count, s);
    case 5: return launch_thread_k<5>(p, sm_count, s);
    case 6: return launch_thread_k<6>(p, sm_count, s);
    case 7: return launch_thread_k<7>(p, sm_count, s);
    case 8: return launch_thread_k<8>(p, sm_count, s);
    case 9: return launch_thread_k<9>(p, sm_count, s);
    case 10: return launch_thread_k<10>(p, sm_count, s);
    case 11: return launch_thread_k<11>(p, sm_count, s);
    case 12: return launch_thread_k<12>(p, sm_count, s);
    case 13: return launch_thread_k<13>(p, sm_count, s);
    case 14: return launch_thread_k<14>(p, sm_count, s);
    case 15: return launch_thread_k<15>(p, sm_count, s);
    case 16: return launch_thread_k<16>(p, sm_count, s);
    default: break;
  }
  if (p.k <= 16) return launch_warp_k<16>(p, sm_count, s);
  if (p.k <= 32) return launch_warp_k<32>(p, sm_count, s);
  if (p.k <= 64) return launch_posv_warp64(p, sm_count, s);
  return cudaErrorInvalidValue;
}

}  // namespace b2c
