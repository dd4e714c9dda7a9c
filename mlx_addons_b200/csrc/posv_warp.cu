// Register-resident batched Cholesky factor + solve for k <= 16, and the
// dispatch of k <= 64 over the register tiers.
//
// Replaces the reference's one-thread-per-matrix (tier ST, k <= 32,
// src/mlx_addons/linalg/_metal_kernels.py:26-101) and threadgroup (tier TG,
// 33 <= k <= 80, _metal_kernels.py:147-246) kernels, keeping their
// arithmetic contract: clamped pivot sqrt(max(s, 1e-12)), column scaling by
// 1/L_jj, forward then back substitution, lower triangle of A read only,
// upper triangle of an L output zeroed.
//
// Thread tier (k <= 16): one thread owns a whole matrix in registers (a
// square array up to k = 9, a packed lower triangle above); a CTA stages
// 32..128 consecutive matrices through shared memory so global traffic stays
// coalesced (the reference's per-thread layout puts neighbouring threads
// k*k floats apart). With m <= 4 the staging is double-buffered: A and b of
// the next tile load while this tile is factored and solved. 17 <= k <= 32
// (and k = 16 with m >= 4) run segments of 8 or 16 lanes per matrix
// (posv_seg.cu); 33 <= k <= 64 one warp per matrix (posv_warp64.cu).
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

// ---------------------------------------------------------------------------
// Thread tier (k <= 16)
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

cudaError_t launch_posv_small(const PosvParams& p, int sm_count, cudaStream_t s) {
  // k = 16 with four or more right-hand sides: eight lanes per matrix beat
  // one thread per matrix (measured on B200, B = 10,000, m = 4: 12.3 against
  // 18.5 us); below that the thread tier wins (k = 16, m = 2: 9.7 against
  // 12.1 us; k = 12, m = 4: 8.2 against 12.4 us).
  if (p.k == 16 && p.m >= 4) return launch_posv_seg(p, sm_count, s);
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
  if (p.k <= 32) return launch_posv_seg(p, sm_count, s);
  if (p.k <= 64) return posv_tile_applies(p) ? launch_posv_tile(p, sm_count, s) : launch_posv_warp64(p, sm_count, s);
  return cudaErrorInvalidValue;
}

}  // namespace b2c
