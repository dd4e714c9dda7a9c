// Blocked Cholesky factor + solve for k > 64, register-tiled.
//
// Same contract as the blocked tier it supersedes (posv_blocked.cu, which
// remains the path for k whose panel inverses do not fit shared memory) and as
// the reference's blocked algorithm (src/mlx_addons/linalg/_blocked.py:34-217):
// lower triangle of A read, pivots clamped to sqrt(1e-12), L written once
// with its upper triangle zeroed when requested, substitutions in the same
// kernel.
//
// One CTA of 256 threads factors one matrix at a time (persistent grid, two
// CTAs per SM), left-looking by 32-column panels. For panel J (columns
// j0..j0+31) and each group of up to 256 panel rows:
//   1. P = A[rows, panel] - L[rows, :j0] L[panel, :j0]^T as a register-tiled
//      GEMM: thread (ty, tx) owns rows ty + 32 i (i < 8) and columns tx + 8 j
//      (j < 4); both operands are staged in shared memory 32 columns at a time
//      with cp.async; the strides make every float4 read conflict-free.
//   2. Warp 0 factors the 32x32 diagonal block in registers (right-looking,
//      reference clamp); all 8 warps then form its inverse, 4 columns each, by
//      independent forward substitutions, kept in shared memory (swizzled).
//   3. The remaining panel rows are solved as X = P L_JJ^{-T}, the same
//      register-tiled micro-kernel with the inverse as the second operand.
//   4. The panel is written once.
// The substitutions then use the per-panel inverses: each 32-row block is a
// GEMV over the rows already solved followed by a 32x32 mat-vec with the
// inverse (forward: L_JJ^{-1}; backward: L_JJ^{-T}), one warp per right-hand
// side, instead of a 32-step dependent chain.
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

namespace {

constexpr int T2 = 256;    // threads per CTA
constexpr int RG2 = 256;   // panel rows per group
constexpr int KC2 = 32;    // staged columns of the GEMM operands
constexpr int AS2 = 36;    // row stride of the staged operands (floats)
constexpr int MCB2 = 8;    // max right-hand sides per pass (one per warp)
constexpr int kMaxSmemFloats = 227 * 1024 / 4;

// shared-memory layout (floats)
constexpr int OFF_A = 0;                  // RG2 x AS2: GEMM operand A, then P; solves: RHS + reduction
constexpr int OFF_B = OFF_A + RG2 * AS2;  // 32 x AS2: GEMM operand B
constexpr int OFF_D = OFF_B + 32 * AS2;   // 32 x 36: diagonal block / L_JJ
constexpr int OFF_INV = OFF_D + 32 * 36;  // nblk x 1024: per-panel inverses (swizzled rows of 32)
constexpr int FIXED2 = OFF_INV;

__device__ __forceinline__ int inv_off(int c, int q) { return c * 32 + (((q >> 2) ^ (c & 7)) << 2) + (q & 3); }

// acc[i][j] += sign * sum_kk As[ty + 32 i][kk] * Bs[tx + 8 j][kk] over KC2 columns
template <bool SUB>
__device__ __forceinline__ void tile_mma(float (&acc)[8][4], const float* As, const float* Bs, int ty, int tx) {
#pragma unroll 1
  for (int kk = 0; kk < KC2; kk += 4) {
    float4 a[8], b[4];
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = *reinterpret_cast<const float4*>(As + (ty + 32 * i) * AS2 + kk);
#pragma unroll
    for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(Bs + (tx + 8 * j) * AS2 + kk);
#pragma unroll
    for (int i = 0; i < 8; ++i)
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

// Same as tile_mma, the second operand being a swizzled 32x32 inverse.
__device__ __forceinline__ void tile_mma_inv(float (&acc)[8][4], const float* As, const float* Li, int ty, int tx) {
#pragma unroll 1
  for (int kk = 0; kk < 32; kk += 4) {
    float4 a[8], b[4];
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = *reinterpret_cast<const float4*>(As + (ty + 32 * i) * AS2 + kk);
#pragma unroll
    for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(Li + inv_off(tx + 8 * j, kk));
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float t = acc[i][j];
        t = fmaf(a[i].x, b[j].x, t);
        t = fmaf(a[i].y, b[j].y, t);
        t = fmaf(a[i].z, b[j].z, t);
        t = fmaf(a[i].w, b[j].w, t);
        acc[i][j] = t;
      }
  }
}

// Right-looking factorisation of a 32x32 block held one row per lane.
__device__ __forceinline__ void factor32(float (&a)[32], int lane, float* colbuf, float& inv_own, float& d_own) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float sc = fmaxf(__shfl_sync(kFull, a[j], j), kClamp);
    const float r = rsqrtf(sc);
    const float d = sc * r;
    const float v = (lane == j) ? d : a[j] * r;
    a[j] = v;
    inv_own = (lane == j) ? r : inv_own;
    d_own = (lane == j) ? d : d_own;
    float* cb = colbuf + (j & 1) * 36;
    cb[lane] = v;
    __syncwarp();
#pragma unroll
    for (int c4 = ((j + 1) >> 2) << 2; c4 < 32; c4 += 4) {
      const float4 w = *reinterpret_cast<const float4*>(cb + c4);
      const float ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = c4 + i;
        if (c > j) a[c] = fmaf(-v, ww[i], a[c]);
      }
    }
  }
}

}  // namespace

__global__ void __launch_bounds__(T2, 2) posv_blocked2_kernel(const PosvParams p, int mcb) {
  extern __shared__ __align__(16) float sm[];
  const int K = p.k;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ty = tid >> 3, tx = tid & 7;
  float* As = sm + OFF_A;
  float* Bs = sm + OFF_B;
  float* sD = sm + OFF_D;
  float* sInv = sm + OFF_INV;
  const size_t kk = (size_t)K * K;
  const bool vec = p.vec && (K & 3) == 0;
  const int nblk = (K + 31) / 32;

  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x) {
    const float* A = p.A + mat * kk;
    float* Wm = p.L ? p.L + mat * kk : p.ws + (size_t)blockIdx.x * kk;
    float lgacc = 0.f;
    for (int J = 0; J < nblk; ++J) {
      const int j0 = 32 * J, bw = min(32, K - j0);
      float* Li = sInv + J * 1024;
      for (int rg = j0; rg < K; rg += RG2) {
        // ---- P = A[rows, panel] - L[rows, :j0] L[panel, :j0]^T ----------
        float acc[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = rg + ty + 32 * i;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = tx + 8 * j;
            acc[i][j] = (r < K && c < bw) ? __ldg(A + (size_t)r * K + j0 + c) : 0.f;
          }
        }
        for (int p0 = 0; p0 < j0; p0 += KC2) {
          __syncthreads();  // previous readers of As / Bs are done
          if (vec) {
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              const int f = tid + T2 * t, row = f >> 3, q = f & 7;
              if (rg + row < K) cp_async16(As + row * AS2 + 4 * q, Wm + (size_t)(rg + row) * K + p0 + 4 * q);
            }
            {
              const int row = tid >> 3, q = tid & 7;
              if (row < bw) cp_async16(Bs + row * AS2 + 4 * q, Wm + (size_t)(j0 + row) * K + p0 + 4 * q);
            }
          } else {
            for (int f = tid; f < RG2 * KC2; f += T2) {
              const int row = f >> 5, c = f & 31;
              if (rg + row < K) cp_async4(As + row * AS2 + c, Wm + (size_t)(rg + row) * K + p0 + c);
            }
            for (int f = tid; f < 32 * KC2; f += T2) {
              const int row = f >> 5, c = f & 31;
              if (row < bw) cp_async4(Bs + row * AS2 + c, Wm + (size_t)(j0 + row) * K + p0 + c);
            }
          }
          cp_async_commit();
          cp_async_wait_all();
          __syncthreads();
          tile_mma<true>(acc, As, Bs, ty, tx);
        }
        // ---- P to shared memory (As is free now); diagonal rows to sD -----
        const bool first = (rg == j0);
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) As[(ty + 32 * i) * AS2 + tx + 8 * j] = (tx + 8 * j < bw) ? acc[i][j] : 0.f;
        if (first) {
#pragma unroll
          for (int j = 0; j < 4; ++j) sD[ty * 36 + tx + 8 * j] = acc[0][j];  // row j0 + ty
        }
        __syncthreads();
        // ---- diagonal block: factor (warp 0) and invert (all warps) -----
        if (first) {
          if (warp == 0) {
            float a[32];
#pragma unroll
            for (int c = 0; c < 32; ++c)
              a[c] = (lane < bw && c < bw) ? sD[lane * 36 + c] : (c == lane ? 1.f : 0.f);
            float invo = 1.f, dv = 1.f;
            factor32(a, lane, Bs, invo, dv);  // Bs doubles as the column buffer
            __syncwarp();
#pragma unroll
            for (int c = 0; c < 32; ++c) sD[lane * 36 + c] = (c < lane) ? a[c] : (c == lane ? dv : 0.f);
            if (lane < bw) {
              lgacc += logf(dv);
              float* wr = Wm + (size_t)(j0 + lane) * K + j0;
#pragma unroll
              for (int c = 0; c < 32; ++c)
                if (c < bw) wr[c] = (c < lane) ? a[c] : (c == lane ? dv : 0.f);
              if (p.L)
                for (int c = j0 + bw; c < K; ++c) Wm[(size_t)(j0 + lane) * K + c] = 0.f;
            }
          }
          __syncthreads();
          // inverse X = L_JJ^{-1}; warp w computes columns 4w..4w+3, lane = row
          {
            float lrow[32];
#pragma unroll
            for (int c4 = 0; c4 < 32; c4 += 4) {
              const float4 v = *reinterpret_cast<const float4*>(sD + lane * 36 + c4);
              lrow[c4] = v.x; lrow[c4 + 1] = v.y; lrow[c4 + 2] = v.z; lrow[c4 + 3] = v.w;
            }
            float dl = 1.f;
#pragma unroll
            for (int c = 0; c < 32; ++c) dl = (c == lane) ? lrow[c] : dl;
            const float il = 1.f / dl;
            float xs[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) xs[q] = (lane == 4 * warp + q) ? 1.f : 0.f;
#pragma unroll
            for (int pp = 0; pp < 32; ++pp) {
              // row pp of X is final in lane pp once scaled by 1 / L_pp
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float xp = __shfl_sync(kFull, xs[q] * il, pp);
                xs[q] = (lane == pp) ? xp : ((lane > pp) ? fmaf(-lrow[pp], xp, xs[q]) : xs[q]);
              }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) Li[inv_off(lane, 4 * warp + q)] = xs[q];
          }
          __syncthreads();
        }
        // ---- X = P L_JJ^{-T} for the rows below the diagonal block -------
        float x[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) x[i][j] = 0.f;
        tile_mma_inv(x, As, Li, ty, tx);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = rg + ty + 32 * i;
          if (r >= K || (first && i == 0)) continue;  // diagonal rows hold L_JJ already
          float* wr = Wm + (size_t)r * K + j0;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (tx + 8 * j < bw) wr[tx + 8 * j] = x[i][j];
        }
        __syncthreads();  // W writes visible before the next group / panel
      }
    }
    if (warp == 0 && p.logdet) {
      const float lg = warp_sum(lgacc);
      if (lane == 0) p.logdet[mat] = 2.f * lg;
    }

    // ---- substitutions with the panel inverses ---------------------------
    if (p.m > 0) {
      float* sY = As;                   // mcb x K, column-major per right-hand side
      float* sRed = Bs;                 // 8 x 8 x 32 reduction (Bs and sD)
      const float* bm = p.b + (size_t)mat * K * p.m;
      float* xm = p.x + (size_t)mat * K * p.m;
      for (int q0 = 0; q0 < p.m; q0 += mcb) {
        const int mc = min(mcb, p.m - q0);
        __syncthreads();
        for (int e = tid; e < K * mc; e += T2) {
          const int r = e / mc, q = e - r * mc;
          sY[q * K + r] = bm[(size_t)r * p.m + q0 + q];
        }
        __syncthreads();
        // forward: y_J = Linv_J (b_J - L[J, :j0] y[:j0])
        for (int J = 0; J < nblk; ++J) {
          const int j0 = 32 * J, bw = min(32, K - j0);
          if (j0 > 0) {
            for (int ii = warp; ii < bw; ii += 8) {
              const float* Lr = Wm + (size_t)(j0 + ii) * K;
              float s[MCB2];
#pragma unroll
              for (int q = 0; q < MCB2; ++q) s[q] = 0.f;
              for (int pp = lane; pp < j0; pp += 32) {
                const float l = Lr[pp];
#pragma unroll
                for (int q = 0; q < MCB2; ++q)
                  if (q < mc) s[q] = fmaf(l, sY[q * K + pp], s[q]);
              }
#pragma unroll
              for (int q = 0; q < MCB2; ++q)
                if (q < mc) {
                  const float t = warp_sum(s[q]);
                  if (lane == 0) sY[q * K + j0 + ii] -= t;
                }
            }
            __syncthreads();
          }
          if (warp < mc) {
            const float* Li = sInv + J * 1024;
            const float* t = sY + warp * K + j0;
            float y = 0.f;
#pragma unroll
            for (int q4 = 0; q4 < 32; q4 += 4) {
              const float4 l4 = *reinterpret_cast<const float4*>(Li + inv_off(lane, q4));
              const float t0 = (q4 < bw) ? t[q4] : 0.f, t1 = (q4 + 1 < bw) ? t[q4 + 1] : 0.f;
              const float t2 = (q4 + 2 < bw) ? t[q4 + 2] : 0.f, t3 = (q4 + 3 < bw) ? t[q4 + 3] : 0.f;
              y = fmaf(l4.x, t0, y);
              y = fmaf(l4.y, t1, y);
              y = fmaf(l4.z, t2, y);
              y = fmaf(l4.w, t3, y);
            }
            __syncwarp();
            if (lane < bw) sY[warp * K + j0 + lane] = y;
          }
          __syncthreads();
        }
        // backward: x_J = Linv_J^T (y_J - L[J+1:, J]^T x[J+1:])
        for (int J = nblk - 1; J >= 0; --J) {
          const int j0 = 32 * J, bw = min(32, K - j0);
          if (j0 + 32 < K) {
            float s[MCB2];
#pragma unroll
            for (int q = 0; q < MCB2; ++q) s[q] = 0.f;
            for (int r = j0 + 32 + warp; r < K; r += 8) {
              const float l = Wm[(size_t)r * K + j0 + lane];
#pragma unroll
              for (int q = 0; q < MCB2; ++q)
                if (q < mc) s[q] = fmaf(l, sY[q * K + r], s[q]);
            }
#pragma unroll
            for (int q = 0; q < MCB2; ++q) sRed[(warp * MCB2 + q) * 32 + lane] = s[q];
            __syncthreads();
            if (warp < mc) {
              float t = 0.f;
#pragma unroll
              for (int w = 0; w < 8; ++w) t += sRed[(w * MCB2 + warp) * 32 + lane];
              sY[warp * K + j0 + lane] -= t;
            }
            __syncthreads();
          }
          if (warp < mc) {
            const float* Li = sInv + J * 1024;
            const float* t = sY + warp * K + j0;
            float xv = 0.f;
#pragma unroll
            for (int q = 0; q < 32; ++q) {
              const float tq = (q < bw) ? t[q] : 0.f;
              xv = fmaf(Li[inv_off(q, lane)], tq, xv);
            }
            __syncwarp();
            if (lane < bw) sY[warp * K + j0 + lane] = xv;
          }
          __syncthreads();
        }
        for (int e = tid; e < K * mc; e += T2) {
          const int r = e / mc, q = e - r * mc;
          xm[(size_t)r * p.m + q0 + q] = sY[q * K + r];
        }
      }
    }
    __syncthreads();
  }
}

int blocked2_mcb(int k) {
  int mcb = (RG2 * AS2) / (k > 0 ? k : 1);
  return mcb > MCB2 ? MCB2 : mcb;
}

size_t blocked2_smem_bytes(int k) {
  const int nblk = (k + 31) / 32;
  return (size_t)(FIXED2 + nblk * 1024) * sizeof(float);
}

bool blocked2_fits(int k) {
  return blocked2_mcb(k) >= 1 && blocked2_smem_bytes(k) <= (size_t)kMaxSmemFloats * sizeof(float);
}

cudaError_t launch_posv_blocked2(const PosvParams& p, int grid, cudaStream_t s) {
  static int cache[64];
  int occ = 0;
  cudaError_t e = kernel_occupancy(posv_blocked2_kernel, T2, blocked2_smem_bytes(p.k), cache, &occ);
  if (e != cudaSuccess) return e;
  posv_blocked2_kernel<<<grid, T2, blocked2_smem_bytes(p.k), s>>>(p, blocked2_mcb(p.k));
  return cudaGetLastError();
}

}  // namespace b2c
