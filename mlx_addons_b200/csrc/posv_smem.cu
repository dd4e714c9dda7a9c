// Shared-memory tier of the batched Cholesky factor + solve: 65 <= k <= 192
// (to 256 on request), at most 8 right-hand sides.
//
// Same contract as the other tiers and as the reference's blocked algorithm
// (src/mlx_addons/linalg/_blocked.py:34-217): lower triangle of A read,
// pivots clamped to sqrt(1e-12), L written once with its upper triangle
// zeroed when requested, substitutions in the same kernel.
//
// One CTA factors one matrix at a time entirely in shared memory: the lower
// triangle of A as 32 x 32 blocks (row stride 36 floats, so float4 reads of
// 8 consecutive rows hit 8 different bank groups), 36 blocks = 166 KB at
// k = 256, plus the right-hand sides. Nothing is written to or re-read from
// HBM between the load of A and b and the store of x (and L). Right-looking
// by 32-column panels J:
//   1. warp 0 factors the diagonal block in registers (one row per lane);
//   2. all warps form its inverse L_JJ^{-1} (a few columns each), kept
//      swizzled for this panel and, transposed, in the block's unused strict
//      upper triangle for the back substitution;
//   3. tasks over the warps: y_J = L_JJ^{-1} b_J (one task per right-hand
//      side) and the panel solve L_IJ = A_IJ L_JJ^{-T} as 16-row x 32-column
//      register-tiled products with the inverse, in place;
//   4. tasks: the trailing update A_IK -= L_IJ L_KJ^T (J < K <= I), the same
//      16 x 32 tiles, and b_I -= L_IJ y_J (one task per block row).
// A barrier separates the steps. The back substitution walks the blocks
// from the last, one warp per right-hand side: t = y_J - sum_{I>J} L_IJ^T
// x_I, then x_J = L_JJ^{-T} t with the stored inverse.
// Rows past k are an identity block, which no real row ever reads.
#include <stdlib.h>
#include <string.h>

#include "b2c_blocked_common.cuh"
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

namespace {

constexpr int SB = 32;         // block edge
constexpr int SS = 36;         // block row stride (floats)
constexpr int BLKF = SB * SS;  // floats per block
constexpr int SMCH = 8;        // right-hand sides of the fused substitutions

__host__ __device__ constexpr int tri(int nb) { return nb * (nb + 1) / 2; }
__device__ __forceinline__ int boff(int I, int J) { return (tri(I) + J) * BLKF; }

// shared-memory layout (floats) for nb blocks a side
__host__ __device__ constexpr int sm_y(int nb) { return tri(nb) * BLKF; }          // y / x: [q][32 nb]
__host__ __device__ constexpr int sm_inv(int nb) { return sm_y(nb) + SMCH * SB * nb; }  // 32 x 32 inverse
__host__ __device__ constexpr int sm_cb(int nb) { return sm_inv(nb) + 1024; }      // factor32 column buffer
__host__ __device__ constexpr int sm_acc(int nb) { return sm_cb(nb) + 72; }        // back-substitution sums
__host__ __device__ constexpr int sm_floats(int nb) { return sm_acc(nb) + SB * SMCH; }

// acc[i][j] (+|-)= sum_{q<32} A[ty + 4 i][q] B[tx + 8 j][q]; A rows at stride SS;
// B rows at stride SS, or the swizzled 32 x 32 inverse
template <bool SUB, bool SWZ>
__device__ __forceinline__ void tile16(float (&acc)[4][4], const float* A, const float* B, int ty, int tx) {
#pragma unroll 2
  for (int q = 0; q < 32; q += 4) {
    float4 a[4], b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(A + (ty + 4 * i) * SS + q);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      b[j] = *reinterpret_cast<const float4*>(SWZ ? B + inv_off(tx + 8 * j, q) : B + (tx + 8 * j) * SS + q);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float t = acc[i][j];
        if (SUB) {
          t = fmaf(-a[i].x, b[j].x, t);
          t = fmaf(-a[i].y, b[j].y, t);
          t = fmaf(-a[i].z, b[j].z, t);
          t = fmaf(-a[i].w, b[j].w, t);
        } else {
          t = fmaf(a[i].x, b[j].x, t);
          t = fmaf(a[i].y, b[j].y, t);
          t = fmaf(a[i].z, b[j].z, t);
          t = fmaf(a[i].w, b[j].w, t);
        }
        acc[i][j] = t;
      }
  }
}

}  // namespace

template <int NW>
__global__ void __launch_bounds__(NW * 32, 16 / NW) posv_smem_kernel(const PosvParams p) {
  constexpr int NT = NW * 32;
  constexpr int CPW = 32 / NW;  // inverse columns per warp
  extern __shared__ __align__(16) float sm[];
  const int K = p.k, NB = (K + SB - 1) / SB, KP = NB * SB;
  const int m = p.m, mc = m < SMCH ? m : SMCH;  // m <= SMCH on this tier
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ty = lane >> 3, tx = lane & 7;
  float* T = sm;
  float* Y = sm + sm_y(NB);
  float* Li = sm + sm_inv(NB);
  float* cb = sm + sm_cb(NB);
  float* tacc = sm + sm_acc(NB);
  const bool vec = p.vec && (K & 3) == 0;
  const size_t kk = (size_t)K * K;

  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x) {
    const float* A = p.A + mat * kk;
    __syncthreads();  // the previous matrix's readers are done
    // ---- A's lower-triangle blocks (identity beyond k) and b --------------
    for (int e = tid; e < tri(NB) * SB * 8; e += NT) {
      const int b = e >> 8, rr = (e >> 3) & 31, qd = e & 7;
      int I = 0;
      while (tri(I + 1) <= b) ++I;
      const int J = b - tri(I);
      if (I == J && 4 * qd > rr) continue;  // wholly above the diagonal
      const int r = SB * I + rr, c = SB * J + 4 * qd;
      float* dst = T + b * BLKF + rr * SS + 4 * qd;
      if (vec && r < K && c + 3 < K) {
        cp_async16(dst, A + (size_t)r * K + c);
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int cc = c + u;
          dst[u] = (r < K && cc < K) ? __ldg(A + (size_t)r * K + cc) : (r == cc ? 1.f : 0.f);
        }
      }
    }
    cp_async_commit();
    const float* bm = p.b + (size_t)mat * K * m;
    for (int e = tid; e < KP * mc; e += NT) {
      const int q = e / KP, i = e - q * KP;
      Y[e] = (i < K) ? __ldg(bm + (size_t)i * m + q) : 0.f;
    }
    cp_async_wait_all();
    __syncthreads();

    float lg = 0.f;
    for (int J = 0; J < NB; ++J) {
      float* D = T + boff(J, J);
      // ---- 1. diagonal block (warp 0) -------------------------------------
      if (warp == 0) {
        float a[32];
#pragma unroll
        for (int c4 = 0; c4 < 32; c4 += 4) {
          const float4 v = *reinterpret_cast<const float4*>(D + lane * SS + c4);
          a[c4] = v.x;
          a[c4 + 1] = v.y;
          a[c4 + 2] = v.z;
          a[c4 + 3] = v.w;
        }
        float invo = 1.f, dv = 1.f;
        factor32(a, lane, cb, invo, dv);
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (c <= lane) D[lane * SS + c] = (c < lane) ? a[c] : dv;
        if (SB * J + lane < K) lg += logf(dv);
      }
      __syncthreads();
      // ---- 2. inverse X = L_JJ^{-1}: warp w forms columns CPW w .. CPW w + CPW - 1
      {
        float lrow[32];
#pragma unroll
        for (int c4 = 0; c4 < 32; c4 += 4) {
          const float4 v = *reinterpret_cast<const float4*>(D + lane * SS + c4);
          lrow[c4] = v.x;
          lrow[c4 + 1] = v.y;
          lrow[c4 + 2] = v.z;
          lrow[c4 + 3] = v.w;
        }
        float dl = 1.f;
#pragma unroll
        for (int c = 0; c < 32; ++c) dl = (c == lane) ? lrow[c] : dl;
        const float il = 1.f / dl;
        float xs[CPW];
#pragma unroll
        for (int q = 0; q < CPW; ++q) xs[q] = (lane == CPW * warp + q) ? 1.f : 0.f;
#pragma unroll
        for (int pp = 0; pp < 32; ++pp) {
#pragma unroll
          for (int q = 0; q < CPW; ++q) {
            const float xp = __shfl_sync(kFull, xs[q] * il, pp);
            xs[q] = (lane == pp) ? xp : ((lane > pp) ? fmaf(-lrow[pp], xp, xs[q]) : xs[q]);
          }
        }
        // (the transposed copy lands above D's diagonal, which no warp reads)
#pragma unroll
        for (int q = 0; q < CPW; ++q) {
          const int c = CPW * warp + q;
          Li[inv_off(lane, c)] = xs[q];
          if (lane > c) D[c * SS + lane] = xs[q];  // X[lane][c], transposed, above the diagonal
        }
      }
      __syncthreads();
      // ---- 3. y_J = L_JJ^{-1} b_J; L_IJ = A_IJ L_JJ^{-T} (16-row halves) ----
      {
        const int nt = mc + 2 * (NB - 1 - J);
        for (int t = warp; t < nt; t += NW) {
          if (t < mc) {
            float* yq = Y + t * KP + SB * J;
            float y = 0.f;
#pragma unroll
            for (int c4 = 0; c4 < 32; c4 += 4) {
              const float4 l4 = *reinterpret_cast<const float4*>(Li + inv_off(lane, c4));
              y = fmaf(l4.x, yq[c4], y);
              y = fmaf(l4.y, yq[c4 + 1], y);
              y = fmaf(l4.z, yq[c4 + 2], y);
              y = fmaf(l4.w, yq[c4 + 3], y);
            }
            __syncwarp();
            yq[lane] = y;
          } else {
            const int u = t - mc, I = J + 1 + (u >> 1), h = u & 1;
            float* Ab = T + boff(I, J) + 16 * h * SS;
            float acc[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
            tile16<false, true>(acc, Ab, Li, ty, tx);
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int j = 0; j < 4; ++j) Ab[(ty + 4 * i) * SS + tx + 8 * j] = acc[i][j];
          }
        }
      }
      __syncthreads();
      // ---- 4. A_IK -= L_IJ L_KJ^T (J < K <= I); b_I -= L_IJ y_J ---------------
      {
        const int n1 = NB - 1 - J, ntr = n1 * (n1 + 1);  // block pairs x 2 halves
        const int nt = ntr + (mc > 0 ? n1 : 0);
        for (int t = warp; t < nt; t += NW) {
          if (t < ntr) {
            const int u = t >> 1, h = t & 1;
            int i1 = 0;
            while ((i1 + 1) * (i1 + 2) / 2 <= u) ++i1;
            const int I = J + 1 + i1, Kb = J + 1 + (u - i1 * (i1 + 1) / 2);
            float* C = T + boff(I, Kb) + 16 * h * SS;
            const float* Ab = T + boff(I, J) + 16 * h * SS;
            const float* Bb = T + boff(Kb, J);
            float acc[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int j = 0; j < 4; ++j) acc[i][j] = C[(ty + 4 * i) * SS + tx + 8 * j];
            tile16<true, false>(acc, Ab, Bb, ty, tx);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int j = 0; j < 4; ++j) C[(ty + 4 * i) * SS + tx + 8 * j] = acc[i][j];
          } else {
            const int I = J + 1 + (t - ntr);
            const float* Lr = T + boff(I, J) + lane * SS;
            float s[SMCH];
#pragma unroll
            for (int q = 0; q < SMCH; ++q) s[q] = 0.f;
#pragma unroll
            for (int c4 = 0; c4 < 32; c4 += 4) {
              const float4 l4 = *reinterpret_cast<const float4*>(Lr + c4);
#pragma unroll
              for (int q = 0; q < SMCH; ++q) {
                if (q < mc) {
                  const float* yq = Y + q * KP + SB * J + c4;
                  s[q] = fmaf(l4.x, yq[0], s[q]);
                  s[q] = fmaf(l4.y, yq[1], s[q]);
                  s[q] = fmaf(l4.z, yq[2], s[q]);
                  s[q] = fmaf(l4.w, yq[3], s[q]);
                }
              }
            }
#pragma unroll
            for (int q = 0; q < SMCH; ++q)
              if (q < mc) Y[q * KP + SB * I + lane] -= s[q];
          }
        }
      }
      __syncthreads();
    }
    if (warp == 0 && p.logdet) {
      const float l = warp_sum(lg);
      if (lane == 0) p.logdet[mat] = 2.f * l;
    }

    // ---- back substitution: x_J = L_JJ^{-T} (y_J - sum_{I>J} L_IJ^T x_I) ----
    // warp w alone owns right-hand sides w, w + NW, ... (their columns of Y
    // and of tacc), so no CTA barrier is needed and every sum runs in a fixed
    // order
    if (mc > 0) {
      for (int q = warp; q < mc; q += NW) {
        float* yq = Y + q * KP;
        for (int J = NB - 1; J >= 0; --J) {
          float t = yq[SB * J + lane];
          for (int I = J + 1; I < NB; ++I) {
            const float* Lb = T + boff(I, J) + lane;
            const float* xi = yq + SB * I;
#pragma unroll 8
            for (int r = 0; r < SB; ++r) t = fmaf(-Lb[r * SS], xi[r], t);
          }
          tacc[lane * SMCH + q] = t;
          __syncwarp();
          const float* D = T + boff(J, J);
          const float dinv = 1.f / D[lane * SS + lane];
          float x = 0.f;
#pragma unroll 4
          for (int c = 0; c < SB; ++c) {
            // X^T[lane][c] = X[c][lane]: stored at D[lane][c] above the diagonal
            const float w = (c > lane) ? D[lane * SS + c] : ((c == lane) ? dinv : 0.f);
            x = fmaf(w, tacc[c * SMCH + q], x);
          }
          __syncwarp();
          yq[SB * J + lane] = x;
          __syncwarp();
        }
      }
      __syncthreads();
      float* xm = p.x + (size_t)mat * K * m;
      for (int e = tid; e < K * mc; e += NT) {
        const int i = e / mc, q = e - i * mc;
        xm[(size_t)i * m + q] = Y[q * KP + i];
      }
    }
    if (p.L) {
      float* Lm = p.L + mat * kk;
      for (int e = tid; e < K * K; e += NT) {
        const int r = e / K, c = e - r * K;
        Lm[e] = (c > r) ? 0.f : T[boff(r / SB, c / SB) + (r % SB) * SS + (c % SB)];
      }
    }
  }
}

// Used up to k = 192, where two or more CTAs fit an SM and one matrix's
// serial panel steps overlap another's products (measured on B200, B = 2,000:
// 1.35-1.7x the blocked tier for 65 <= k <= 192; 0.93-0.98x at k = 224 and
// 256, one CTA per SM). B2C_SMEM_TIER=all extends it to k = 256, =0 turns it
// off (read per call, so a test can flip it).
static int smem_tier_max_k() {
  const char* t = getenv("B2C_SMEM_TIER");
  if (t && strcmp(t, "0") == 0) return 0;
  if (t && strcmp(t, "all") == 0) return 256;
  return 192;
}

bool smem_tier_fits(int k, int m) { return k >= 1 && k <= smem_tier_max_k() && m <= SMCH; }

bool smem_tier_enabled() { return smem_tier_max_k() > 0; }

static int device_sm_count() {
  static int cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 148;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

static int smem_tier_warps(int nb) { return nb <= 4 ? 4 : (nb <= 6 ? 8 : 16); }

template <int NW>
static cudaError_t launch_smem_t(const PosvParams& p, cudaStream_t s) {
  const int sm_count = device_sm_count();
  const int nb = (p.k + SB - 1) / SB;
  const size_t smem = (size_t)sm_floats(nb) * sizeof(float);
  static int cache[64];
  int occ = 0;
  auto kern = posv_smem_kernel<NW>;
  cudaError_t e = kernel_occupancy(kern, NW * 32, smem, cache, &occ);
  if (e != cudaSuccess) return e;
  // the cache holds the occupancy of the first size queried; this launch's size may differ
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, NW * 32, smem);
  if (e != cudaSuccess) return e;
  if (occ < 1) occ = 1;
  const int64_t cap = (int64_t)sm_count * occ;
  kern<<<(int)(p.batch < cap ? p.batch : cap), NW * 32, smem, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_posv_smem(const PosvParams& p, cudaStream_t s) {
  const int nw = smem_tier_warps((p.k + SB - 1) / SB);
  if (nw == 4) return launch_smem_t<4>(p, s);
  if (nw == 8) return launch_smem_t<8>(p, s);
  return launch_smem_t<16>(p, s);
}

}  // namespace b2c
