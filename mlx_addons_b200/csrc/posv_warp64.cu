// Register-resident batched Cholesky factor + solve, 33 <= k <= 64.
//
// Replaces the reference's threadgroup tier (src/mlx_addons/linalg/
// _metal_kernels.py:147-246, 33 <= k <= 80), whose factorisation step has a
// serial diagonal on thread 0, two threadgroup barriers per column and a
// single-thread substitution, with the same arithmetic contract: pivot
// sqrt(max(s, 1e-12)), column scaled by 1/L_jj, forward then back
// substitution, lower triangle of A read only, upper triangle of L zeroed.
//
// One warp owns one matrix: lane l holds rows l (columns 0..31) and 32 + l
// (columns 0..KP-1) in registers, k padded to KP in {40, 48, 56, 64} with an
// identity block. Right-looking factorisation: at step j the pivot is
// broadcast by shuffle, each lane scales its two column-j entries, the column
// is published through a double-buffered shared vector (one __syncwarp) and
// each lane applies the rank-1 update to its rows with packed two-wide FMAs
// (fma.rn.f32x2). The substitutions reuse the factor in registers: forward is
// column-oriented on the lane-owned rows; backward publishes 8 rows of L at a
// time, interleaved so that one 64-bit shared load gives a lane L[i][l] and
// L[i][32 + l].
//
// A CTA is 12 warps, one CTA per SM. The warps of a CTA start each matrix
// together (one barrier per round), so the three warps on every SM
// sub-partition walk the same instruction stream and share instruction
// fetches: the unrolled factorisation is several thousand instructions long
// and, unsynchronised, the warps thrash the instruction cache. Each warp
// stages its next matrix with cp.async while it works on the current one and
// fetches only the blocks the algorithm reads (rows 0..31 stop at column 31):
// 12 KB instead of 16 KB of A at k = 64.
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

typedef unsigned long long u64;

__device__ __forceinline__ u64 pk2(float lo, float hi) {
  u64 r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float lo2(u64 v) {
  float lo, hi;
  asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo;
}
__device__ __forceinline__ float hi2(u64 v) {
  float lo, hi;
  asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return hi;
}
// d = a * b + c, two lanes of float32 at once.
__device__ __forceinline__ u64 ffma2(u64 a, u64 b, u64 c) {
  u64 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ void lds128(const float* p, u64& x, u64& y) {
  asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "r"(smem_u32(p)));
}
__device__ __forceinline__ u64 lds64(const float* p) {
  u64 x;
  asm volatile("ld.shared.b64 %0, [%1];" : "=l"(x) : "r"(smem_u32(p)));
  return x;
}

// Element c of a packed row.
template <int N>
__device__ __forceinline__ float getc(const u64 (&a)[N], int c) {
  return (c & 1) ? hi2(a[c >> 1]) : lo2(a[c >> 1]);
}
template <int N>
__device__ __forceinline__ void setc(u64 (&a)[N], int c, float v) {
  a[c >> 1] = (c & 1) ? pk2(lo2(a[c >> 1]), v) : pk2(v, hi2(a[c >> 1]));
}

constexpr int W64_WARPS = 12;

template <int KP>
struct W64 {
  static constexpr int NB = KP - 32;  // bottom rows
  static constexpr int S0 = 36;       // stride of the staged top rows (columns 0..31)
  static constexpr int S1 = KP + 4;   // stride of the staged bottom rows; S1/4 odd
  static constexpr int STAGE = 32 * S0 + NB * S1;
  static constexpr int CBW = 72;      // one column buffer
  static constexpr int CHS = 68;      // row stride of the back-substitution chunk (64 interleaved + pad)
  static constexpr int WARP_FLOATS = STAGE + 2 * CBW + 8 * CHS;
  static_assert(KP % 8 == 0 && KP > 32 && KP <= 64, "KP");
  static_assert((S1 / 4) % 2 == 1, "odd float4 stride keeps row reads conflict-free");
};

template <int KP>
__device__ __forceinline__ void w64_stage(const PosvParams& p, int64_t mat, float* st, int lane, bool fast) {
  using W = W64<KP>;
  if (mat >= p.batch) return;
  const int K = p.k;
  const float* src = p.A + mat * (size_t)K * K;
  float* st1 = st + 32 * W::S0;
  if (fast) {  // K == KP, 16-byte aligned: 16-byte copies, fixed lane pattern
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int r = (lane >> 3) + 4 * t, q = lane & 7;
      cp_async16(st + r * W::S0 + 4 * q, src + r * KP + 4 * q);
    }
    constexpr int Q = KP / 4, TOTAL = W::NB * Q;
#pragma unroll
    for (int f0 = 0; f0 < TOTAL; f0 += 32) {
      const int f = f0 + lane;
      if (f < TOTAL) {
        const int r = f / Q, q = f - r * Q;
        cp_async16(st1 + r * W::S1 + 4 * q, src + (32 + r) * KP + 4 * q);
      }
    }
  } else {
    for (int f = lane; f < 1024; f += 32) {
      const int r = f >> 5, c = f & 31;
      cp_async4(st + r * W::S0 + c, src + (size_t)r * K + c);
    }
    const int total = (K - 32) * K;
    for (int f = lane; f < total; f += 32) {
      const int r = f / K, c = f - r * K;
      cp_async4(st1 + r * W::S1 + c, src + (size_t)(32 + r) * K + c);
    }
  }
}

template <int KP, int MC>
__global__ void __launch_bounds__(W64_WARPS * 32, 1) posv_warp64_kernel(const PosvParams p) {
  using W = W64<KP>;
  constexpr int H0 = 16;      // packed pairs of the top row
  constexpr int H1 = KP / 2;  // packed pairs of the bottom row
  extern __shared__ __align__(16) float smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float* st = smem + warp * W::WARP_FLOATS;
  float* st1 = st + 32 * W::S0;
  float* cbuf = st + W::STAGE;
  float* chunk = cbuf + 2 * W::CBW;

  const int K = p.k;
  const bool fast = (K == KP) && p.vec;
  const int r1 = 32 + lane;
  const int64_t nround = (p.batch + W64_WARPS - 1) / W64_WARPS;

  if ((int64_t)blockIdx.x < nround) {
    w64_stage<KP>(p, (int64_t)blockIdx.x * W64_WARPS + warp, st, lane, fast);
    cp_async_commit();
  }
  for (int64_t rd = blockIdx.x; rd < nround; rd += gridDim.x) {
    __syncthreads();  // the CTA's warps start the round together
    const int64_t mat = rd * W64_WARPS + warp;
    const bool mvalid = mat < p.batch;
    cp_async_wait_all();
    __syncwarp();

    u64 a0[H0], a1[H1];
    if (fast && mvalid) {
      const float* s0 = st + lane * W::S0;
#pragma unroll
      for (int c4 = 0; c4 < 32; c4 += 4) lds128(s0 + c4, a0[c4 / 2], a0[c4 / 2 + 1]);
      const float* s1 = st1 + (lane < W::NB ? lane : W::NB - 1) * W::S1;
#pragma unroll
      for (int c4 = 0; c4 < KP; c4 += 4) lds128(s1 + c4, a1[c4 / 2], a1[c4 / 2 + 1]);
      if (W::NB < 32 && lane >= W::NB) {  // rows beyond KP do not exist: zero rows
#pragma unroll
        for (int h = 0; h < H1; ++h) a1[h] = 0ull;
      }
    } else {
      const float* s0 = st + lane * W::S0;
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        const float x0 = (mvalid && c < K) ? s0[c] : (c == lane ? 1.f : 0.f);
        const float x1 = (mvalid && c + 1 < K) ? s0[c + 1] : (c + 1 == lane ? 1.f : 0.f);
        a0[c / 2] = pk2(x0, x1);
      }
      const float* s1 = st1 + (lane < W::NB ? lane : W::NB - 1) * W::S1;
#pragma unroll
      for (int c = 0; c < KP; c += 2) {
        const bool rowok = mvalid && r1 < K;
        const float x0 = (rowok && c < K) ? s1[c] : (c == r1 ? 1.f : 0.f);
        const float x1 = (rowok && c + 1 < K) ? s1[c + 1] : (c + 1 == r1 ? 1.f : 0.f);
        a1[c / 2] = pk2(x0, x1);
      }
    }
    __syncwarp();
    if (rd + gridDim.x < nround) w64_stage<KP>(p, (rd + gridDim.x) * W64_WARPS + warp, st, lane, fast);
    cp_async_commit();

    // ---- right-looking factorisation ------------------------------------
    float inv0 = 1.f, inv1 = 1.f, d0 = 1.f, d1 = 1.f;
#pragma unroll
    for (int j = 0; j < KP; ++j) {
      const float dsrc = (j < 32) ? getc(a0, j < 32 ? j : 0) : getc(a1, j);
      const float ajj = __shfl_sync(kFull, dsrc, j & 31);
      float d;
      const float r = clamped_rsqrt(ajj, d);
      float v0 = 0.f;
      if (j < 32) {
        const int jj = j < 32 ? j : 0;
        v0 = (lane == j) ? d : getc(a0, jj) * r;
        setc(a0, jj, v0);
        inv0 = (lane == j) ? r : inv0;
        d0 = (lane == j) ? d : d0;
      }
      float v1 = (r1 == j) ? d : getc(a1, j) * r;
      setc(a1, j, v1);
      if (j >= 32) {
        inv1 = (r1 == j) ? r : inv1;
        d1 = (r1 == j) ? d : d1;
      }
      float* cb = cbuf + (j & 1) * W::CBW;
      if (j < 31) cb[lane] = v0;
      cb[32 + lane] = v1;
      __syncwarp();
      const u64 n0 = pk2(-v0, -v0), n1 = pk2(-v1, -v1);
#pragma unroll
      for (int c4 = ((j + 1) >> 2) << 2; c4 < KP; c4 += 4) {
        u64 w01, w23;
        lds128(cb + c4, w01, w23);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int c = c4 + 2 * h;  // pair (c, c+1)
          const u64 w = h ? w23 : w01;
          if (c > j) {  // both columns of the pair are trailing
            if (c < 32 && j < 31) a0[c / 2 < H0 ? c / 2 : 0] = ffma2(n0, w, a0[c / 2 < H0 ? c / 2 : 0]);
            a1[c / 2] = ffma2(n1, w, a1[c / 2]);
          } else if (c + 1 > j) {  // only column c+1
            const float wc = hi2(w);
            if (c + 1 < 32) setc(a0, c + 1 < 32 ? c + 1 : 0, fmaf(-v0, wc, getc(a0, c + 1 < 32 ? c + 1 : 0)));
            setc(a1, c + 1, fmaf(-v1, wc, getc(a1, c + 1)));
          }
        }
      }
    }

    // ---- zero the strict upper triangle kept in registers -----------------
#pragma unroll
    for (int c = 1; c < 32; ++c) setc(a0, c, (c <= lane) ? getc(a0, c) : 0.f);
#pragma unroll
    for (int c = 33; c < KP; ++c) setc(a1, c, (c <= r1) ? getc(a1, c) : 0.f);

    if (p.logdet) {
      float lg = logf(d0) + logf(d1);
      lg = warp_sum(lg);
      if (lane == 0 && mvalid) p.logdet[mat] = 2.f * lg;
    }

    if (p.L && mvalid) {
      float* Lm = p.L + mat * (size_t)K * K;
      if (fast) {
        float* row0 = Lm + (size_t)lane * KP;
#pragma unroll
        for (int c4 = 0; c4 < 32; c4 += 4)
          *reinterpret_cast<float4*>(row0 + c4) = make_float4(lo2(a0[c4 / 2]), hi2(a0[c4 / 2]), lo2(a0[c4 / 2 + 1]),
                                                              hi2(a0[c4 / 2 + 1]));
#pragma unroll
        for (int c4 = 32; c4 < KP; c4 += 4) *reinterpret_cast<float4*>(row0 + c4) = make_float4(0.f, 0.f, 0.f, 0.f);
        if (lane < W::NB) {
          float* row1 = Lm + (size_t)r1 * KP;
#pragma unroll
          for (int c4 = 0; c4 < KP; c4 += 4)
            *reinterpret_cast<float4*>(row1 + c4) = make_float4(lo2(a1[c4 / 2]), hi2(a1[c4 / 2]),
                                                                lo2(a1[c4 / 2 + 1]), hi2(a1[c4 / 2 + 1]));
        }
      } else {
        float* row0 = Lm + (size_t)lane * K;
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (c < K) row0[c] = getc(a0, c);
        for (int c = 32; c < K; ++c) row0[c] = 0.f;
        if (r1 < K) {
          float* row1 = Lm + (size_t)r1 * K;
#pragma unroll
          for (int c = 0; c < KP; ++c)
            if (c < K) row1[c] = getc(a1, c);
        }
      }
    }

    // ---- substitutions, MC right-hand sides at a time ---------------------
    for (int q0 = 0; q0 < p.m; q0 += MC) {
      u64 y[MC];  // (row l, row 32 + l)
      const float* bm = p.b + (size_t)mat * K * p.m;
#pragma unroll
      for (int q = 0; q < MC; ++q) {
        const bool qok = mvalid && q0 + q < p.m;
        y[q] = pk2(qok ? bm[(size_t)lane * p.m + q0 + q] : 0.f,
                   (qok && r1 < K) ? bm[(size_t)r1 * p.m + q0 + q] : 0.f);
      }
      // forward, L y = b: the column j of L below the diagonal is lane-local
#pragma unroll
      for (int j = 0; j < KP; ++j) {
        const u64 lj = pk2(j < 32 ? getc(a0, j < 32 ? j : 0) : 0.f, getc(a1, j));
#pragma unroll
        for (int q = 0; q < MC; ++q) {
          const float own = (j < 32) ? lo2(y[q]) * inv0 : hi2(y[q]) * inv1;
          const float yj = __shfl_sync(kFull, own, j & 31);
          const u64 upd = ffma2(lj, pk2(-yj, -yj), y[q]);  // rows above j see L[r][j] = 0
          if (j < 32) y[q] = (lane == j) ? pk2(yj, hi2(upd)) : upd;
          else y[q] = (r1 == j) ? pk2(lo2(upd), yj) : upd;
        }
      }
      // backward, L^T x = y: row i of L is published 8 rows at a time,
      // element c stored at 2 * (c % 32) + c / 32
#pragma unroll
      for (int c0 = KP - 8; c0 >= 0; c0 -= 8) {
        if (c0 >= 32) {
          const int rr = r1 - c0;
          if (rr >= 0 && rr < 8) {
            float* dst = chunk + rr * W::CHS;
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              const float h0 = (c + 32 < KP) ? getc(a1, c + 32 < KP ? c + 32 : 0) : 0.f;
              const float h1 = (c + 33 < KP) ? getc(a1, c + 33 < KP ? c + 33 : 0) : 0.f;
              *reinterpret_cast<float4*>(dst + 2 * c) = make_float4(getc(a1, c), h0, getc(a1, c + 1), h1);
            }
          }
        } else {
          const int rr = lane - c0;
          if (rr >= 0 && rr < 8) {
            float* dst = chunk + rr * W::CHS;
#pragma unroll
            for (int c = 0; c < 32; c += 2)
              *reinterpret_cast<float4*>(dst + 2 * c) = make_float4(getc(a0, c), 0.f, getc(a0, c + 1), 0.f);
          }
        }
        __syncwarp();
#pragma unroll
        for (int i = c0 + 7; i >= c0; --i) {
          const u64 li = lds64(chunk + (i - c0) * W::CHS + 2 * lane);  // (L[i][l], L[i][32+l])
#pragma unroll
          for (int q = 0; q < MC; ++q) {
            const float own = (i < 32) ? lo2(y[q]) * inv0 : hi2(y[q]) * inv1;
            const float xi = __shfl_sync(kFull, own, i & 31);
            const u64 upd = ffma2(li, pk2(-xi, -xi), y[q]);  // rows below i see L[i][r] = 0
            if (i < 32) y[q] = (lane == i) ? pk2(xi, hi2(upd)) : upd;
            else y[q] = (r1 == i) ? pk2(lo2(upd), xi) : upd;
          }
        }
        __syncwarp();
      }
      if (mvalid) {
        float* xm = p.x + (size_t)mat * K * p.m;
#pragma unroll
        for (int q = 0; q < MC; ++q) {
          if (q0 + q < p.m) {
            xm[(size_t)lane * p.m + q0 + q] = lo2(y[q]);
            if (r1 < K) xm[(size_t)r1 * p.m + q0 + q] = hi2(y[q]);
          }
        }
      }
    }
  }
  cp_async_wait_all();
}

template <int KP, int MC>
static cudaError_t launch_w64_t(const PosvParams& p, int sm_count, cudaStream_t s) {
  using W = W64<KP>;
  constexpr int threads = W64_WARPS * 32;
  const size_t smem = (size_t)W64_WARPS * W::WARP_FLOATS * sizeof(float);
  auto kern = posv_warp64_kernel<KP, MC>;
  static int cache[64];
  int occ = 0;
  cudaError_t e = kernel_occupancy(kern, threads, smem, cache, &occ);
  if (e != cudaSuccess) return e;
  const int64_t rounds = (p.batch + W64_WARPS - 1) / W64_WARPS;
  const int64_t cap = (int64_t)sm_count * occ;
  const int grid = (int)(rounds < cap ? rounds : cap);
  kern<<<grid, threads, smem, s>>>(p);
  return cudaGetLastError();
}

template <int KP>
static cudaError_t launch_w64_k(const PosvParams& p, int sm, cudaStream_t s) {
  return p.m <= 1 ? launch_w64_t<KP, 1>(p, sm, s) : launch_w64_t<KP, 4>(p, sm, s);
}

cudaError_t launch_posv_warp64(const PosvParams& p, int sm_count, cudaStream_t s) {
  if (p.k <= 40) return launch_w64_k<40>(p, sm_count, s);
  if (p.k <= 48) return launch_w64_k<48>(p, sm_count, s);
  if (p.k <= 56) return launch_w64_k<56>(p, sm_count, s);
  return launch_w64_k<64>(p, sm_count, s);
}

}  // namespace b2c
