// Shared-memory tier of the batched Cholesky factor + solve: 65 <= k <= 256,
// any number of right-hand sides (the first 8 fused
// into the factorisation, the rest in passes of 8 against the factor kept in
// shared memory).
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
// by 32-column panels J, the diagonal block J already factored:
//   A. tasks over the warps: y_J = L_JJ^{-1} b_J (one per right-hand side)
//      and the panel solve L_IJ = A_IJ L_JJ^{-T} (one per block row, lane =
//      row), both by substitution in registers, with L_JJ^T in shared
//      memory for the column broadcasts and 1 / L_jj kept per block;
//   B. look-ahead: warp 0 applies panel J to diagonal block J+1 and factors
//      it (one row per lane) while the other warps run the rest of the
//      trailing update A_IK -= L_IJ L_KJ^T (J < K <= I) as 16 x 32
//      register-tiled products and b_I -= L_IJ y_J.
// A barrier separates A and B, so the serial diagonal factor of one panel
// overlaps the products of the previous one. The back substitution walks the
// blocks from the last, one warp per right-hand side: t = y_J - sum_{I>J}
// L_IJ^T x_I, then L_JJ^T x_J = t by substitution.
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
__host__ __device__ constexpr int sm_lt(int nb) { return sm_y(nb) + SMCH * SB * nb; }   // L_JJ^T (stride SS)
__host__ __device__ constexpr int sm_dinv(int nb) { return sm_lt(nb) + BLKF; }         // 1 / L_jj, all blocks
__host__ __device__ constexpr int sm_cb(int nb) { return sm_dinv(nb) + SB * nb; }      // factor32 column buffer
__host__ __device__ constexpr int sm_floats(int nb) { return sm_cb(nb) + 72; }

// acc[i][j] -= sum_{q<32} A[ty + 4 i][q] B[tx + 8 j][q], rows of A and B at stride SS
__device__ __forceinline__ void tile16_sub(float (&acc)[4][4], const float* A, const float* B, int ty, int tx) {
#pragma unroll 2
  for (int q = 0; q < 32; q += 4) {
    float4 a[4], b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(A + (ty + 4 * i) * SS + q);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      b[j] = *reinterpret_cast<const float4*>(B + (tx + 8 * j) * SS + q);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float t = acc[i][j];
        t = fmaf(-a[i].x, b[j].x, t);
        t = fmaf(-a[i].y, b[j].y, t);
        t = fmaf(-a[i].z, b[j].z, t);
        t = fmaf(-a[i].w, b[j].w, t);
        acc[i][j] = t;
      }
  }
}

// Warp 0: factors diagonal block D in registers (one row per lane); L back
// to D's lower triangle, L^T to Lt, 1 / L_jj to dinv; returns this lane's
// log L_jj for rows below `rows` (0 for the identity rows past k). Kept out
// of line: one copy of the 32-step chain serves every call, so it stays in
// the instruction cache.
__device__ __noinline__ float smem_factor_diag(float* D, float* Lt, float* dinv, float* cb, int rows, int lane) {
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
  // whole rows and columns, no lane-dependent branch: what lands above the
  // diagonal of D and below it in Lt is never read
#pragma unroll
  for (int c = 0; c < 32; ++c) a[c] = (c == lane) ? dv : a[c];
#pragma unroll
  for (int c4 = 0; c4 < 32; c4 += 4)
    *reinterpret_cast<float4*>(D + lane * SS + c4) = make_float4(a[c4], a[c4 + 1], a[c4 + 2], a[c4 + 3]);
#pragma unroll
  for (int c = 0; c < 32; ++c) Lt[c * SS + lane] = a[c];
  dinv[lane] = invo;
  return (lane < rows) ? logf(dv) : 0.f;
}

}  // namespace

template <int NW>
__global__ void __launch_bounds__(NW * 32, 16 / NW) posv_smem_kernel(const PosvParams p) {
  constexpr int NT = NW * 32;
  extern __shared__ __align__(16) float sm[];
  const int K = p.k, NB = (K + SB - 1) / SB, KP = NB * SB;
  const int m = p.m, mc = m < SMCH ? m : SMCH;  // right-hand sides fused into the factorisation
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ty = lane >> 3, tx = lane & 7;
  float* T = sm;
  float* Y = sm + sm_y(NB);
  float* Lt = sm + sm_lt(NB);
  float* dinv = sm + sm_dinv(NB);
  float* cb = sm + sm_cb(NB);
  const bool vec = p.vec && (K & 3) == 0;
  const size_t kk = (size_t)K * K;

  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x) {
    const float* A = p.A + mat * kk;
    __syncthreads();  // the previous matrix's readers are done
    // ---- A's lower-triangle blocks (identity beyond k) and b --------------
    // block b's quad (row rr, columns 4 qd ..) of the lower triangle, by the
    // threads of `first`..NT-1; block 0 first, then the rest, so that warp 0
    // factors block 0 while the other warps stage the others
    auto stage = [&](int b0, int b1, int first) {
      for (int e = tid - first + b0 * SB * 8; e < b1 * SB * 8; e += NT - first) {
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
    };
    stage(0, 1, 0);
    cp_async_wait_all();
    __syncthreads();
    float lg = 0.f;
    const float* bm = p.b + (size_t)mat * K * m;
    if (warp == 0) {
      lg += smem_factor_diag(T + boff(0, 0), Lt, dinv, cb, K, lane);
    } else {
      stage(1, tri(NB), 32);
      for (int e = tid - 32; e < KP * mc; e += NT - 32) {
        const int q = e / KP, i = e - q * KP;
        Y[e] = (i < K) ? __ldg(bm + (size_t)i * m + q) : 0.f;
      }
      cp_async_wait_all();
    }
    __syncthreads();
    for (int J = 0; J < NB; ++J) {
      const float* dJ = dinv + SB * J;
      // ---- A. y_J = L_JJ^{-1} b_J and L_IJ = A_IJ L_JJ^{-T}, by substitution ----
      {
        const int nt = mc + (NB - 1 - J);
        for (int t = warp; t < nt; t += NW) {
          if (t < mc) {  // forward, one right-hand side: lane = row
            const float* D = T + boff(J, J) + lane * SS;
            float lr[32];
#pragma unroll
            for (int c4 = 0; c4 < 32; c4 += 4) {
              const float4 v = *reinterpret_cast<const float4*>(D + c4);
              lr[c4] = v.x;
              lr[c4 + 1] = v.y;
              lr[c4 + 2] = v.z;
              lr[c4 + 3] = v.w;
            }
            float* yq = Y + t * KP + SB * J;
            float y = yq[lane];
            const float di = dJ[lane];
            float yo = 0.f;
#pragma unroll
            for (int pp = 0; pp < 32; ++pp) {
              const float yp = __shfl_sync(kFull, y * di, pp);
              if (lane == pp) yo = yp;
              if (lane > pp) y = fmaf(-lr[pp], yp, y);
            }
            yq[lane] = yo;
          } else {  // panel solve: lane = row of A_IJ, x L_JJ^T = a
            const int I = J + 1 + (t - mc);
            float* Ar = T + boff(I, J) + lane * SS;
            float a[32];
#pragma unroll
            for (int c4 = 0; c4 < 32; c4 += 4) {
              const float4 v = *reinterpret_cast<const float4*>(Ar + c4);
              a[c4] = v.x;
              a[c4 + 1] = v.y;
              a[c4 + 2] = v.z;
              a[c4 + 3] = v.w;
            }
#pragma unroll
            for (int pp = 0; pp < 32; ++pp) {
              a[pp] *= dJ[pp];
              const float xp = a[pp];
#pragma unroll
              for (int c4 = ((pp + 1) >> 2) << 2; c4 < 32; c4 += 4) {  // L[c][pp] = Lt[pp][c]
                const float4 l4 = *reinterpret_cast<const float4*>(Lt + pp * SS + c4);
                const float ll[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
                for (int u = 0; u < 4; ++u)
                  if (c4 + u > pp) a[c4 + u] = fmaf(-xp, ll[u], a[c4 + u]);
              }
            }
#pragma unroll
            for (int c4 = 0; c4 < 32; c4 += 4)
              *reinterpret_cast<float4*>(Ar + c4) = make_float4(a[c4], a[c4 + 1], a[c4 + 2], a[c4 + 3]);
          }
        }
      }
      __syncthreads();
      // ---- B. warp 0: block J+1's update and factor (look-ahead); the other
      //         warps: A_IK -= L_IJ L_KJ^T (J < K <= I, but not block J+1's),
      //         b_I -= L_IJ y_J ----
      {
        const int n1 = NB - 1 - J, ntr = n1 * (n1 + 1);  // block pairs x 2 halves; pair 0 is block J+1's
        if (warp == 0) {
          if (n1 > 0) {
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
              float* C = T + boff(J + 1, J + 1) + 16 * h * SS;
              const float* Ab = T + boff(J + 1, J) + 16 * h * SS;
              const float* Bb = T + boff(J + 1, J);
              float acc[4][4];
#pragma unroll
              for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = C[(ty + 4 * i) * SS + tx + 8 * j];
              tile16_sub(acc, Ab, Bb, ty, tx);
#pragma unroll
              for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) C[(ty + 4 * i) * SS + tx + 8 * j] = acc[i][j];
            }
            __syncwarp();
            lg += smem_factor_diag(T + boff(J + 1, J + 1), Lt, dinv + SB * (J + 1), cb, K - SB * (J + 1), lane);
          }
        } else {
          const int nt = ntr - 2 + (mc > 0 ? n1 : 0);
          for (int t0 = warp - 1; t0 < nt; t0 += NW - 1) {
            const int t = t0 + 2;
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
              tile16_sub(acc, Ab, Bb, ty, tx);
#pragma unroll
              for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) C[(ty + 4 * i) * SS + tx + 8 * j] = acc[i][j];
            } else {
              const int I = J + 1 + (t - ntr);
              const float* Lr = T + boff(I, J) + lane * SS;
              float sacc[SMCH];
#pragma unroll
              for (int q = 0; q < SMCH; ++q) sacc[q] = 0.f;
#pragma unroll
              for (int c4 = 0; c4 < 32; c4 += 4) {
                const float4 l4 = *reinterpret_cast<const float4*>(Lr + c4);
#pragma unroll
                for (int q = 0; q < SMCH; ++q) {
                  if (q < mc) {
                    const float* yq = Y + q * KP + SB * J + c4;
                    sacc[q] = fmaf(l4.x, yq[0], sacc[q]);
                    sacc[q] = fmaf(l4.y, yq[1], sacc[q]);
                    sacc[q] = fmaf(l4.z, yq[2], sacc[q]);
                    sacc[q] = fmaf(l4.w, yq[3], sacc[q]);
                  }
                }
              }
#pragma unroll
              for (int q = 0; q < SMCH; ++q)
                if (q < mc) Y[q * KP + SB * I + lane] -= sacc[q];
            }
          }
        }
      }
      __syncthreads();
    }
    if (warp == 0 && p.logdet) {
      const float l = warp_sum(lg);
      if (lane == 0) p.logdet[mat] = 2.f * l;
    }

    // ---- substitutions with the factor in shared memory ---------------------
    // warp w alone owns right-hand sides w, w + NW, ... of a pass (their
    // columns of Y), so no CTA barrier is needed between blocks and every
    // sum runs in a fixed order.
    // forward, L y = b, for passes after the first (whose y rode along with
    // the factorisation): y_J = L_JJ^{-1} (b_J - sum_{I<J} L_JI y_I)
    auto forward = [&](int nq) {
      for (int q = warp; q < nq; q += NW) {
        float* yq = Y + q * KP;
        for (int J = 0; J < NB; ++J) {
          float y = yq[SB * J + lane], y1 = 0.f, y2 = 0.f, y3 = 0.f;
          for (int I = 0; I < J; ++I) {
            const float* Lr = T + boff(J, I) + lane * SS;
            const float* yi = yq + SB * I;
#pragma unroll
            for (int c4 = 0; c4 < 32; c4 += 4) {
              const float4 l4 = *reinterpret_cast<const float4*>(Lr + c4);
              y = fmaf(-l4.x, yi[c4], y);
              y1 = fmaf(-l4.y, yi[c4 + 1], y1);
              y2 = fmaf(-l4.z, yi[c4 + 2], y2);
              y3 = fmaf(-l4.w, yi[c4 + 3], y3);
            }
          }
          y = (y + y1) + (y2 + y3);
          const float* lr = T + boff(J, J) + lane * SS;
          const float di = dinv[SB * J + lane];
          float yo = 0.f;
#pragma unroll
          for (int pp = 0; pp < 32; ++pp) {
            const float yp = __shfl_sync(kFull, y * di, pp);
            if (lane == pp) yo = yp;
            if (lane > pp) y = fmaf(-lr[pp], yp, y);
          }
          __syncwarp();
          yq[SB * J + lane] = yo;
          __syncwarp();
        }
      }
    };
    // backward, L^T x = y: L_JJ^T x_J = y_J - sum_{I>J} L_IJ^T x_I
    auto backward = [&](int nq) {
      for (int q = warp; q < nq; q += NW) {
        float* yq = Y + q * KP;
        for (int J = NB - 1; J >= 0; --J) {
          float t = yq[SB * J + lane], t1 = 0.f, t2 = 0.f, t3 = 0.f;
          for (int I = J + 1; I < NB; ++I) {
            const float* Lb = T + boff(I, J) + lane;
            const float* xi = yq + SB * I;
#pragma unroll 2
            for (int r = 0; r < SB; r += 4) {
              t = fmaf(-Lb[r * SS], xi[r], t);
              t1 = fmaf(-Lb[(r + 1) * SS], xi[r + 1], t1);
              t2 = fmaf(-Lb[(r + 2) * SS], xi[r + 2], t2);
              t3 = fmaf(-Lb[(r + 3) * SS], xi[r + 3], t3);
            }
          }
          t = (t + t1) + (t2 + t3);
          // column-oriented: x_c final in lane c, then rows above subtract L[c][lane] x_c
          const float* D = T + boff(J, J);
          const float di = dinv[SB * J + lane];
          float xo = 0.f;
#pragma unroll
          for (int c = 31; c >= 0; --c) {
            const float xc = __shfl_sync(kFull, t * di, c);
            if (lane == c) xo = xc;
            if (lane < c) t = fmaf(-D[c * SS + lane], xc, t);
          }
          __syncwarp();
          yq[SB * J + lane] = xo;
          __syncwarp();
        }
      }
    };
    for (int q0 = 0; q0 < m; q0 += SMCH) {
      const int nq = min(SMCH, m - q0);
      if (q0 > 0) {  // the first pass's b was staged with A
        __syncthreads();  // the previous pass's x are stored
        for (int e = tid; e < KP * nq; e += NT) {
          const int q = e / KP, i = e - q * KP;
          Y[e] = (i < K) ? __ldg(bm + (size_t)i * m + q0 + q) : 0.f;
        }
        __syncthreads();
        forward(nq);
      }
      backward(nq);
      __syncthreads();
      float* xm = p.x + (size_t)mat * K * m;
      for (int e = tid; e < K * nq; e += NT) {
        const int i = e / nq, q = e - i * nq;
        xm[(size_t)i * m + q0 + q] = Y[q * KP + i];
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

// The default for k <= 256, where the factor fits one CTA's shared memory
// (measured on B200, B = 2,000: 1.5-2.3x the blocked tier for 65 <= k <= 192,
// 1.14-1.20x at k = 224 and 256, one CTA per SM there). B2C_SMEM_TIER=0
// turns it off (read per call, so a test can flip it); =all is accepted as
// the default.
static int smem_tier_max_k() {
  const char* t = getenv("B2C_SMEM_TIER");
  if (t && strcmp(t, "0") == 0) return 0;
  return 256;
}

bool smem_tier_fits(int k, int m) {
  (void)m;
  return k >= 1 && k <= smem_tier_max_k();
}

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
  if (posv_dag_applies(p)) return launch_posv_dag(p, s);
  const int nw = smem_tier_warps((p.k + SB - 1) / SB);
  if (nw == 4) return launch_smem_t<4>(p, s);
  if (nw == 8) return launch_smem_t<8>(p, s);
  return launch_smem_t<16>(p, s);
}

}  // namespace b2c
