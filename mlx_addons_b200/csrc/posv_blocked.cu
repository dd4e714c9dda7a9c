// Blocked Cholesky factor + solve for large k, and the triangular solves.
//
// Replaces the reference's 80-wide blocked algorithm
// (src/mlx_addons/linalg/_blocked.py:34-217), which runs a Python loop of
// O(nblocks^2) separate launches (small potrf kernel, TRSM through
// tril_solve, a full non-symmetric GEMM for the trailing update, two
// concatenate copies of the trailing matrix per block column, then a second
// pass over L for the substitutions), and its tril_solve / triu_solve kernels
// (_metal_kernels.py:103-141, :248-313, :593-638).
//
// One CTA (256 threads) owns one matrix at a time (persistent grid). The
// factorisation is left-looking by 32-column panels:
//   1. panel rows j0..k-1 accumulate A[r, panel] - L[r, :j0] L[panel, :j0]^T,
//      one row per thread in registers; the panel's top rows L[panel, :j0]
//      are staged in shared memory 128 columns at a time and read as float4
//      broadcasts;
//   2. warp 0 factors the 32x32 diagonal block in registers (row per lane,
//      same right-looking step as the warp tier) with the reference's clamp;
//   3. every other panel row is solved against L_JJ^T (TRSM) in registers;
//   4. the panel is written once to L (or to a per-CTA scratch slot).
// Each element of L is written once; A is read once. The substitutions then
// stream L by 32-row blocks: a warp-per-row GEMV with coalesced row reads and
// a warp-level 32x32 triangular solve (forward), and a column-block
// reduction over the rows below plus a transposed 32x32 solve (backward).
// The right-hand sides stay in shared memory for both passes.
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

constexpr int BT = 256;      // threads of the factorisation CTA
constexpr int PW = 32;       // panel width
constexpr int PC = 128;      // staged columns of the panel's top rows
constexpr int SBS = PC + 4;  // row stride of that stage (16-byte rows)
constexpr int SLS = 36;      // row stride of the staged diagonal block
constexpr int MCB = 8;       // max right-hand sides per solve pass
constexpr int kSmemBudgetFloats = 200 * 1024 / 4;

__device__ __forceinline__ float4 ld4(const float* p, bool vec) {
  if (vec) return *reinterpret_cast<const float4*>(p);
  return make_float4(p[0], p[1], p[2], p[3]);
}

// Right-looking factorisation of a 32x32 block held one row per lane
// (rows >= the valid size are identity rows). inv_own receives 1/L_ll.
__device__ __forceinline__ void warp_factor32(float (&a)[32], int lane, float* colbuf, float& inv_own) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float ajj = __shfl_sync(kFull, a[j], j);
    float d;
    const float r = clamped_rsqrt(ajj, d);
    const float v = (lane == j) ? d : a[j] * r;
    a[j] = v;
    inv_own = (lane == j) ? r : inv_own;
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

// ---------------------------------------------------------------------------
// Blocked substitutions on a row-major lower-triangular L (k x k) with the
// right-hand sides in shared memory, column-major per right-hand side:
// sY[q * K + r]. Called by all NT threads of the CTA.
// ---------------------------------------------------------------------------

template <int NT>
__device__ void blocked_forward(const float* Lm, int K, float* sY, int mc, float* sRed) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int j0 = 0; j0 < K; j0 += 32) {
    const int bw = min(32, K - j0);
    if (j0 > 0) {
      for (int ii = warp; ii < bw; ii += NW) {
        const int i = j0 + ii;
        const float* Lr = Lm + (size_t)i * K;
        float s[MCB];
#pragma unroll
        for (int q = 0; q < MCB; ++q) s[q] = 0.f;
        for (int pp = lane; pp < j0; pp += 32) {
          const float l = Lr[pp];
#pragma unroll
          for (int q = 0; q < MCB; ++q)
            if (q < mc) s[q] = fmaf(l, sY[q * K + pp], s[q]);
        }
#pragma unroll
        for (int q = 0; q < MCB; ++q) {
          if (q < mc) {
            const float t = warp_sum(s[q]);
            if (lane == 0) sY[q * K + i] -= t;
          }
        }
      }
      __syncthreads();
    }
    if (warp < mc) {  // one right-hand side per warp at a time
      float lrow[32];
      float dl = 1.f;
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const bool ok = lane < bw && c < bw && c <= lane;
        lrow[c] = ok ? Lm[(size_t)(j0 + lane) * K + j0 + c] : (c == lane ? 1.f : 0.f);
        dl = (c == lane) ? lrow[c] : dl;
      }
      for (int q = warp; q < mc; q += NW) {
        float y = lane < bw ? sY[q * K + j0 + lane] : 0.f;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float t = y / dl;
          y = (lane == c) ? t : y;
          const float yc = __shfl_sync(kFull, y, c);
          if (lane > c) y = fmaf(-lrow[c], yc, y);
        }
        if (lane < bw) sY[q * K + j0 + lane] = y;
      }
    }
    __syncthreads();
  }
}

template <int NT>
__device__ void blocked_backward(const float* Lm, int K, float* sY, int mc, float* sRed) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nblk = (K + 31) / 32;
  for (int jb = nblk - 1; jb >= 0; --jb) {
    const int j0 = jb * 32, bw = min(32, K - j0);
    if (j0 + 32 < K) {
      float s[MCB];
#pragma unroll
      for (int q = 0; q < MCB; ++q) s[q] = 0.f;
      for (int r = j0 + 32 + warp; r < K; r += NW) {
        const float l = Lm[(size_t)r * K + j0 + lane];
#pragma unroll
        for (int q = 0; q < MCB; ++q)
          if (q < mc) s[q] = fmaf(l, sY[q * K + r], s[q]);
      }
      if (NW > 1) {
#pragma unroll
        for (int q = 0; q < MCB; ++q) sRed[(warp * MCB + q) * 32 + lane] = s[q];
        __syncthreads();
        if (warp == 0) {
          for (int q = 0; q < mc; ++q) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < NW; ++w) t += sRed[(w * MCB + q) * 32 + lane];
            sY[q * K + j0 + lane] -= t;
          }
        }
      } else {
        for (int q = 0; q < mc; ++q) sY[q * K + j0 + lane] -= s[q < MCB ? q : 0];
      }
      __syncthreads();
    }
    if (warp < mc) {  // one right-hand side per warp at a time
      float lcol[32];
      float dl = 1.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const bool ok = lane < bw && i < bw && i >= lane;
        lcol[i] = ok ? Lm[(size_t)(j0 + i) * K + j0 + lane] : (i == lane ? 1.f : 0.f);
        dl = (i == lane) ? lcol[i] : dl;
      }
      for (int q = warp; q < mc; q += NW) {
        float y = lane < bw ? sY[q * K + j0 + lane] : 0.f;
#pragma unroll
        for (int i = 31; i >= 0; --i) {
          const float t = y / dl;
          y = (lane == i) ? t : y;
          const float xi = __shfl_sync(kFull, y, i);
          if (lane < i) y = fmaf(-lcol[i], xi, y);
        }
        if (lane < bw) sY[q * K + j0 + lane] = y;
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Factorisation (+ solve) kernel
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(BT, 1) posv_blocked_kernel(const PosvParams p, int mcb) {
  extern __shared__ __align__(16) float sm[];
  const int K = p.k;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* sB = sm;
  float* sL = sB + 32 * SBS;
  float* sInv = sL + 32 * SLS;
  float* sCol = sInv + 32;
  float* sRed = sCol + 72;
  float* sY = sRed + (BT / 32) * MCB * 32;
  const size_t kk = (size_t)K * K;
  const bool vec = p.vec && (K & 3) == 0;

  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x) {
    const float* A = p.A + mat * kk;
    float* Wm = p.L ? p.L + mat * kk : p.ws + (size_t)blockIdx.x * kk;
    float lgacc = 0.f;
    for (int j0 = 0; j0 < K; j0 += PW) {
      const int bw = min(PW, K - j0);
      for (int rg = j0; rg < K; rg += BT) {
        const int r = rg + tid;
        const bool rv = r < K;
        float acc[32];
        if (rv && bw == 32 && vec) {
          const float* ar = A + (size_t)r * K + j0;
#pragma unroll
          for (int c4 = 0; c4 < 32; c4 += 4) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(ar + c4));
            acc[c4] = v.x; acc[c4 + 1] = v.y; acc[c4 + 2] = v.z; acc[c4 + 3] = v.w;
          }
        } else {
          const float* ar = A + (size_t)(rv ? r : 0) * K + j0;
#pragma unroll
          for (int c = 0; c < 32; ++c) acc[c] = (rv && c < bw) ? __ldg(ar + c) : 0.f;
        }
        // acc -= L[r, :j0] L[j0:j0+32, :j0]^T
        for (int p0 = 0; p0 < j0; p0 += PC) {
          const int pc = min(PC, j0 - p0);
          __syncthreads();
          for (int e = tid; e < 32 * pc; e += BT) {
            const int c = e / pc, pp = e - c * pc;
            sB[c * SBS + pp] = (c < bw) ? Wm[(size_t)(j0 + c) * K + p0 + pp] : 0.f;
          }
          __syncthreads();
          if (rv) {
            const float* wr = Wm + (size_t)r * K + p0;
            for (int pp = 0; pp < pc; pp += 4) {
              const float4 lv = ld4(wr + pp, vec);
#pragma unroll
              for (int c = 0; c < 32; ++c) {
                const float4 bv = *reinterpret_cast<const float4*>(sB + c * SBS + pp);
                float t = acc[c];
                t = fmaf(-lv.x, bv.x, t);
                t = fmaf(-lv.y, bv.y, t);
                t = fmaf(-lv.z, bv.z, t);
                t = fmaf(-lv.w, bv.w, t);
                acc[c] = t;
              }
            }
          }
        }
        const bool diagrow = (rg == j0) && (tid < 32);
        if (rg == j0) {
          if (warp == 0) {
            if (lane >= bw) {
#pragma unroll
              for (int c = 0; c < 32; ++c) acc[c] = (c == lane) ? 1.f : 0.f;
            }
            float invo = 1.f;
            warp_factor32(acc, lane, sCol, invo);
#pragma unroll
            for (int c4 = 0; c4 < 32; c4 += 4)
              *reinterpret_cast<float4*>(sL + lane * SLS + c4) = make_float4(acc[c4], acc[c4 + 1], acc[c4 + 2], acc[c4 + 3]);
            sInv[lane] = invo;
            if (lane < bw) lgacc -= logf(invo);  // identity rows past k add nothing
          }
          __syncthreads();
        }
        if (rv && !diagrow) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            float t = acc[c];
#pragma unroll
            for (int q4 = 0; q4 < c; q4 += 4) {
              const float4 l4 = *reinterpret_cast<const float4*>(sL + c * SLS + q4);
              if (q4 + 0 < c) t = fmaf(-acc[q4 + 0], l4.x, t);
              if (q4 + 1 < c) t = fmaf(-acc[q4 + 1 < 32 ? q4 + 1 : 0], l4.y, t);
              if (q4 + 2 < c) t = fmaf(-acc[q4 + 2 < 32 ? q4 + 2 : 0], l4.z, t);
              if (q4 + 3 < c) t = fmaf(-acc[q4 + 3 < 32 ? q4 + 3 : 0], l4.w, t);
            }
            acc[c] = t * sInv[c];
          }
        }
        if (rv) {
          float* wr = Wm + (size_t)r * K + j0;
          if (diagrow) {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (c < bw) wr[c] = (c <= lane) ? acc[c] : 0.f;
            if (p.L)
              for (int c = j0 + bw; c < K; ++c) Wm[(size_t)r * K + c] = 0.f;
          } else if (vec && bw == 32) {
#pragma unroll
            for (int c4 = 0; c4 < 32; c4 += 4)
              *reinterpret_cast<float4*>(wr + c4) = make_float4(acc[c4], acc[c4 + 1], acc[c4 + 2], acc[c4 + 3]);
          } else {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (c < bw) wr[c] = acc[c];
          }
        }
        __syncthreads();
      }
    }
    if (warp == 0 && p.logdet) {
      const float lg = warp_sum(lgacc);
      if (lane == 0) p.logdet[mat] = 2.f * lg;
    }
    if (p.m > 0) {
      const float* bm = p.b + (size_t)mat * K * p.m;
      float* xm = p.x + (size_t)mat * K * p.m;
      for (int q0 = 0; q0 < p.m; q0 += mcb) {
        const int mc = min(mcb, p.m - q0);
        __syncthreads();
        for (int e = tid; e < K * mc; e += BT) {
          const int r = e / mc, q = e - r * mc;
          sY[q * K + r] = bm[(size_t)r * p.m + q0 + q];
        }
        __syncthreads();
        blocked_forward<BT>(Wm, K, sY, mc, sRed);
        blocked_backward<BT>(Wm, K, sY, mc, sRed);
        for (int e = tid; e < K * mc; e += BT) {
          const int r = e / mc, q = e - r * mc;
          xm[(size_t)r * p.m + q0 + q] = sY[q * K + r];
        }
      }
    }
    __syncthreads();
  }
}

static int blocked_mcb(int k) {
  const int fixed = 32 * SBS + 32 * SLS + 32 + 72 + (BT / 32) * MCB * 32;
  const int avail = kSmemBudgetFloats - fixed;
  int mcb = avail / (k > 0 ? k : 1);
  if (mcb > MCB) mcb = MCB;
  return mcb;
}

static size_t blocked_smem_bytes(int k, int mcb) {
  return (size_t)(32 * SBS + 32 * SLS + 32 + 72 + (BT / 32) * MCB * 32 + mcb * k) * sizeof(float);
}

int blocked_grid(int64_t batch, int k, int sm_count) {
  const int64_t cap = (int64_t)sm_count * (blocked2_fits(k) ? blocked2_ctas_per_sm() : 2);
  return (int)(batch < cap ? batch : cap);
}

cudaError_t launch_posv_blocked(const PosvParams& p, int grid, cudaStream_t s) {
  if (smem_tier_enabled() && !blocked2_tensor_cores() && smem_tier_fits(p.k, p.m)) return launch_posv_smem(p, s);
  if (blocked2_fits(p.k)) return launch_posv_blocked2(p, grid, s);
  const int mcb = blocked_mcb(p.k);
  if (mcb < 1) return cudaErrorInvalidValue;
  const size_t smem = blocked_smem_bytes(p.k, mcb);
  static int cache[64];
  int occ = 0;
  cudaError_t e = kernel_occupancy(posv_blocked_kernel, BT, blocked_smem_bytes(64, MCB), cache, &occ);
  if (e != cudaSuccess) return e;
  posv_blocked_kernel<<<grid, BT, smem, s>>>(p, mcb);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Standalone triangular solves (tril_solve / triu_solve)
// ---------------------------------------------------------------------------

template <int NT>
__global__ void __launch_bounds__(NT) trsm_kernel(const TrsmParams p, int mcb) {
  extern __shared__ __align__(16) float sm[];
  const int K = p.k;
  float* sRed = sm;
  float* sY = sRed + (NT / 32) * MCB * 32;
  // work item = (matrix, chunk of mcb right-hand sides): a small batch with
  // many right-hand sides still spreads over the SMs
  const int nchunk = (p.m + mcb - 1) / mcb;
  const int64_t items = p.batch * (int64_t)nchunk;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int64_t mat = it / nchunk;
    const int q0 = (int)(it - mat * nchunk) * mcb;
    const float* Lm = p.L + mat * (size_t)K * K;
    const float* bm = p.b + (size_t)mat * K * p.m;
    float* xm = p.x + (size_t)mat * K * p.m;
    {
      const int mc = min(mcb, p.m - q0);
      __syncthreads();
      for (int e = threadIdx.x; e < K * mc; e += NT) {
        const int r = e / mc, q = e - r * mc;
        sY[q * K + r] = bm[(size_t)r * p.m + q0 + q];
      }
      __syncthreads();
      if (p.transpose) blocked_backward<NT>(Lm, K, sY, mc, sRed);
      else blocked_forward<NT>(Lm, K, sY, mc, sRed);
      for (int e = threadIdx.x; e < K * mc; e += NT) {
        const int r = e / mc, q = e - r * mc;
        xm[(size_t)r * p.m + q0 + q] = sY[q * K + r];
      }
    }
  }
}

template <int NT>
static cudaError_t launch_trsm_t(const TrsmParams& p, int sm_count, cudaStream_t s) {
  const int fixed = (NT / 32) * MCB * 32;
  int mcb = (kSmemBudgetFloats - fixed) / (p.k > 0 ? p.k : 1);
  if (mcb > MCB) mcb = MCB;
  if (mcb < 1) return cudaErrorInvalidValue;
  const size_t smem = (size_t)(fixed + mcb * p.k) * sizeof(float);
  auto kern = trsm_kernel<NT>;
  static int cache[64];
  int occ = 0;
  cudaError_t e = kernel_occupancy(kern, NT, (size_t)(fixed + MCB * 64) * sizeof(float), cache, &occ);
  if (e != cudaSuccess) return e;
  // occupancy at the actual shared-memory size (a pure query)
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, NT, smem);
  if (e != cudaSuccess) return e;
  if (occ < 1) occ = 1;
  const int64_t cap = (int64_t)sm_count * occ;
  const int64_t items = p.batch * (int64_t)((p.m + mcb - 1) / mcb);
  const int grid = (int)(items < cap ? items : cap);
  kern<<<grid, NT, smem, s>>>(p, mcb);
  return cudaGetLastError();
}

cudaError_t launch_trsm(const TrsmParams& p, int sm_count, cudaStream_t s) {
  return p.k <= 32 ? launch_trsm_t<32>(p, sm_count, s) : launch_trsm_t<256>(p, sm_count, s);
}

}  // namespace b2c
