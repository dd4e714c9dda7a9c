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
// broadcast by shuffle (the owner of row j updated it one step early:
// look-ahead), each lane scales its two column-j entries, the column is
// published through a double-buffered shared vector (one __syncwarp) and
// each lane applies the rank-1 update to its rows with packed two-wide FMAs
// (fma.rn.f32x2). The diagonal and its inverse go to shared memory from lane
// 0, and the diagonal and strict upper triangle are then zeroed in registers,
// so both substitutions are select-free: a step never changes its own pivot
// row, each row keeps its running value unscaled and is multiplied by
// 1/L_ii once at the end of the pass. Forward substitution is column-
// oriented on the lane-owned rows; backward publishes 8 rows of L at a time,
// interleaved so that one 64-bit shared load gives a lane L[i][l] and
// L[i][32 + l].
//
// A CTA is 12 warps (168 registers per thread, 172 KB of shared memory), one
// CTA per SM, the register-file limit. Each warp stages its next matrix with
// cp.async while it works on the current one and fetches only the 16-byte
// chunks that hold lower-triangle entries: 8.5 KB of the 16 KB of A at k = 64
// (9 KB in 32-byte sectors), which also cuts the PCIe traffic when A is a
// mapped host buffer. Measured on B200, the column broadcast dominates the shared-
// memory pipe; 16 warps at 128 registers were slower (spills), and a CTA-wide
// barrier per round (to keep warps on the same code) was slower too.
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

constexpr int W64_WARPS = 12;

// Per-warp shared memory (floats). The staged matrix uses 16-byte chunks
// swizzled by row (chunk q of row r at q ^ (r & 7)) wherever a row holds a
// multiple of 8 chunks, else an odd float4 stride; either way 8 consecutive
// rows read at the same column hit 8 different bank groups. The column
// buffer + diagonal buffer of the factorisation and the row chunk of the back
// substitution share one region: their lifetimes do not overlap.
template <int KP>
struct W64 {
  static constexpr int NB = KP - 32;                   // bottom rows
  static constexpr bool SW1 = (KP % 32) == 0;          // swizzled bottom rows
  static constexpr int S1 = SW1 ? KP : KP + 4;         // bottom-row stride
  static constexpr int STAGE = 32 * 32 + NB * S1;
  static constexpr int CBW = 72;                       // one column buffer
  static constexpr int UNION = 8 * 64;                 // chunk; or 2 column buffers + 128 diagonal floats
  static constexpr int WARP_FLOATS = STAGE + UNION;
  static_assert(KP % 8 == 0 && KP > 32 && KP <= 64, "KP");
  static_assert(SW1 || ((S1 / 4) % 2 == 1), "odd float4 stride keeps row reads conflict-free");
  static_assert(2 * CBW + 128 <= UNION, "union");
  // float offset of 16-byte chunk q of staged top row r / bottom row r
  __device__ static __forceinline__ int off0(int r, int q) { return r * 32 + 4 * (q ^ (r & 7)); }
  __device__ static __forceinline__ int off1(int r, int q) {
    return SW1 ? 32 * 32 + r * KP + 4 * (q ^ (r & 7)) : 32 * 32 + r * S1 + 4 * q;
  }
};

template <int KP>
__device__ __forceinline__ void w64_stage(const PosvParams& p, int64_t mat, float* st, int lane, bool chunked) {
  using W = W64<KP>;
  if (mat >= p.batch) return;
  const int K = p.k;
  const float* src = p.A + mat * (size_t)K * K;
  // Only chunks that hold part of the lower triangle are fetched (chunk q of
  // row r when 4q <= r); the staged upper triangle keeps stale values, which
  // the factorisation only ever combines into upper-triangle registers.
  // Rows past k are not staged: the register load reads identity rows for them.
  if (chunked) {  // k % 4 == 0, 16-byte aligned rows: 16-byte copies, fixed lane pattern
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int r = (lane >> 3) + 4 * t, q = lane & 7;
      if (q <= t) cp_async16(st + W::off0(r, q), src + r * K + 4 * q);  // r >> 2 == t
    }
    constexpr int Q = KP / 4, TOTAL = W::NB * Q;
#pragma unroll
    for (int f0 = 0; f0 < TOTAL; f0 += 32) {
      const int f = f0 + lane;
      if (f < TOTAL) {
        const int r = f / Q, q = f - r * Q;
        if (32 + r < K && q <= 8 + (r >> 2)) cp_async16(st + W::off1(r, q), src + (32 + r) * K + 4 * q);
      }
    }
  } else {
    for (int f = lane; f < 1024; f += 32) {
      const int r = f >> 5, c = f & 31;
      if (c <= r) cp_async4(st + W::off0(r, c >> 2) + (c & 3), src + (size_t)r * K + c);
    }
    for (int r = 0; r < K - 32; ++r) {
      const float* row = src + (size_t)(32 + r) * K;
      for (int c = lane; c <= 32 + r; c += 32) cp_async4(st + W::off1(r, c >> 2) + (c & 3), row + c);
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
  float* cbuf = st + W::STAGE;     // factorisation: 2 column buffers
  float* dg = cbuf + 2 * W::CBW;   // dg[2j] = L_jj, dg[2j + 1] = 1 / L_jj
  float* chunk = cbuf;             // back substitution: 8 rows of L

  const int K = p.k;
  const bool fast = (K == KP) && p.vec;
  const bool chunked = (K % 4 == 0) && p.vec;
  const int r1 = 32 + lane;
  const int64_t nround = (p.batch + W64_WARPS - 1) / W64_WARPS;

  if ((int64_t)blockIdx.x < nround) {
    w64_stage<KP>(p, (int64_t)blockIdx.x * W64_WARPS + warp, st, lane, chunked);
    cp_async_commit();
  }
  for (int64_t rd = blockIdx.x; rd < nround; rd += gridDim.x) {
    const int64_t mat = rd * W64_WARPS + warp;
    const bool mvalid = mat < p.batch;
    cp_async_wait_all();
    __syncwarp();

    u64 a0[H0], a1[H1];
    if (fast && mvalid) {
#pragma unroll
      for (int c4 = 0; c4 < 32; c4 += 4) lds128(st + W::off0(lane, c4 / 4), a0[c4 / 2], a0[c4 / 2 + 1]);
      const int rb = lane < W::NB ? lane : W::NB - 1;
#pragma unroll
      for (int c4 = 0; c4 < KP; c4 += 4) lds128(st + W::off1(rb, c4 / 4), a1[c4 / 2], a1[c4 / 2 + 1]);
      if (W::NB < 32 && lane >= W::NB) {  // rows beyond KP do not exist: zero rows
#pragma unroll
        for (int h = 0; h < H1; ++h) a1[h] = 0ull;
      }
    } else {
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        const float* s0 = st + W::off0(lane, c >> 2) + (c & 3);
        const float x0 = (mvalid && c < K) ? s0[0] : (c == lane ? 1.f : 0.f);
        const float x1 = (mvalid && c + 1 < K) ? s0[1] : (c + 1 == lane ? 1.f : 0.f);
        a0[c / 2] = pk2(x0, x1);
      }
      const int rb = lane < W::NB ? lane : W::NB - 1;
#pragma unroll
      for (int c = 0; c < KP; c += 2) {
        const bool rowok = mvalid && r1 < K;
        const float* s1 = st + W::off1(rb, c >> 2) + (c & 3);
        const float x0 = (rowok && c < K) ? s1[0] : (c == r1 ? 1.f : 0.f);
        const float x1 = (rowok && c + 1 < K) ? s1[1] : (c + 1 == r1 ? 1.f : 0.f);
        a1[c / 2] = pk2(x0, x1);
      }
    }
    __syncwarp();
    if (rd + gridDim.x < nround) w64_stage<KP>(p, (rd + gridDim.x) * W64_WARPS + warp, st, lane, chunked);
    cp_async_commit();

    // ---- right-looking factorisation ------------------------------------
    // Look-ahead: the owner of row j+1 updates its own diagonal as soon as its
    // column-j entry is known (dn0 / dn1), so the next pivot broadcast does not
    // wait for the shared-memory column exchange of step j. Every lane computes
    // the pivot's square root and inverse; lane 0 records them in dg.
    float dn0 = 0.f, dn1 = 0.f;
#pragma unroll
    for (int j = 0; j < KP; ++j) {
      const float dsrc = (j == 0) ? getc(a0, 0) : ((j < 32) ? dn0 : dn1);
      const float sc = fmaxf(__shfl_sync(kFull, dsrc, j & 31), kClamp);
      const float r = rsqrtf(sc);
      if (lane == 0) *reinterpret_cast<float2*>(dg + 2 * j) = make_float2(sc * r, r);
      // column j of L for this lane's rows (the owner's own entry is not used)
      float v0 = 0.f;
      if (j < 32) {
        v0 = getc(a0, j < 32 ? j : 0) * r;
        setc(a0, j < 32 ? j : 0, v0);
      }
      const float v1 = getc(a1, j) * r;
      setc(a1, j, v1);
      if (j + 1 < 32) dn0 = fmaf(-v0, v0, getc(a0, j + 1 < 32 ? j + 1 : 0));
      else if (j + 1 < KP) dn1 = fmaf(-v1, v1, getc(a1, j + 1 < KP ? j + 1 : 0));
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
    __syncwarp();
    // diagonal of this lane's rows: row l (dg[2l]) and row 32 + l
    const float2 dt = *reinterpret_cast<const float2*>(dg + 2 * lane);
    const float2 db = (lane < W::NB) ? *reinterpret_cast<const float2*>(dg + 64 + 2 * lane) : make_float2(1.f, 1.f);
    const u64 invp = pk2(dt.y, db.y);

    // ---- zero the diagonal and strict upper triangle kept in registers ---
    // (L then reads 0 wherever a substitution step must leave a row alone)
#pragma unroll
    for (int c = 0; c < 32; ++c) setc(a0, c, (c < lane) ? getc(a0, c) : 0.f);
#pragma unroll
    for (int c = 32; c < KP; ++c) setc(a1, c, (c < r1) ? getc(a1, c) : 0.f);

    if (p.logdet) {
      // rows past k (identity padding) add nothing, even when a NaN in the
      // input has reached them through 0 * NaN in the updates
      float lg = (lane < K ? logf(dt.x) : 0.f) + (r1 < K ? logf(db.x) : 0.f);
      lg = warp_sum(lg);
      if (lane == 0 && mvalid) p.logdet[mat] = 2.f * lg;
    }

    if (p.L && mvalid) {
      float* Lm = p.L + mat * (size_t)K * K;
      float* row0 = Lm + (size_t)lane * K;
      if (fast) {
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
      // the diagonal goes in after the row stores (same thread, program order)
      row0[lane] = dt.x;
      if (r1 < K) Lm[(size_t)r1 * K + r1] = db.x;
    }

    // ---- substitutions, MC right-hand sides at a time ---------------------
    // Each lane keeps its rows' running values unscaled: a step never touches
    // its own pivot row (L[j][j] reads 0), the owner broadcasts value * 1/L_jj,
    // and every row is scaled by its 1/L_ii once at the end of a pass.
    for (int q0 = 0; q0 < p.m; q0 += MC) {
      u64 y[MC];  // (row l, row 32 + l)
      const float* bm = p.b + (size_t)mat * K * p.m;
#pragma unroll
      for (int q = 0; q < MC; ++q) {
        const bool qok = mvalid && q0 + q < p.m;
        y[q] = pk2(qok ? bm[(size_t)lane * p.m + q0 + q] : 0.f,
                   (qok && r1 < K) ? bm[(size_t)r1 * p.m + q0 + q] : 0.f);
      }
      // forward, L y = b: column j of L is lane-local
#pragma unroll
      for (int j = 0; j < KP; ++j) {
        const u64 lj = pk2(j < 32 ? getc(a0, j < 32 ? j : 0) : 0.f, getc(a1, j));
        const float ij = (j < 32) ? dt.y : db.y;
#pragma unroll
        for (int q = 0; q < MC; ++q) {
          const float yj = __shfl_sync(kFull, ((j < 32) ? lo2(y[q]) : hi2(y[q])) * ij, j & 31);
          y[q] = ffma2(lj, pk2(-yj, -yj), y[q]);
        }
      }
#pragma unroll
      for (int q = 0; q < MC; ++q) y[q] = fmul2(y[q], invp);
      // backward, L^T x = y: row i of L is published 8 rows at a time,
      // element c stored at 2 * (c % 32) + c / 32
#pragma unroll
      for (int c0 = KP - 8; c0 >= 0; c0 -= 8) {
        if (c0 >= 32) {
          const int rr = r1 - c0;
          if (rr >= 0 && rr < 8) {
            float* dst = chunk + rr * 64;
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              const float h0 = (c + 32 < KP) ? getc(a1, c + 32 < KP ? c + 32 : 0) : 0.f;
              const float h1 = (c + 33 < KP) ? getc(a1, c + 33 < KP ? c + 33 : 0) : 0.f;
              *reinterpret_cast<float4*>(dst + 4 * ((c >> 1) ^ rr)) = make_float4(getc(a1, c), h0, getc(a1, c + 1), h1);
            }
          }
        } else {
          const int rr = lane - c0;
          if (rr >= 0 && rr < 8) {
            float* dst = chunk + rr * 64;
#pragma unroll
            for (int c = 0; c < 32; c += 2)
              *reinterpret_cast<float4*>(dst + 4 * ((c >> 1) ^ rr)) = make_float4(getc(a0, c), 0.f, getc(a0, c + 1), 0.f);
          }
        }
        __syncwarp();
#pragma unroll
        for (int i = c0 + 7; i >= c0; --i) {
          // (L[i][l], L[i][32 + l]): float 2l of the row, chunk l/2 swizzled by the row
          const u64 li = lds64(chunk + (i - c0) * 64 + 4 * ((lane >> 1) ^ (i - c0)) + 2 * (lane & 1));
          const float ii = (i < 32) ? dt.y : db.y;
#pragma unroll
          for (int q = 0; q < MC; ++q) {
            const float xi = __shfl_sync(kFull, ((i < 32) ? lo2(y[q]) : hi2(y[q])) * ii, i & 31);
            y[q] = ffma2(li, pk2(-xi, -xi), y[q]);
          }
        }
        __syncwarp();
      }
#pragma unroll
      for (int q = 0; q < MC; ++q) y[q] = fmul2(y[q], invp);
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
