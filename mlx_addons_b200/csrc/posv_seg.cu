// Register-resident batched Cholesky factor + solve for small k: S lanes of
// a warp per matrix (S = 16: two matrices per warp, 17 <= k <= 32; S = 8:
// four per warp, used at k = 16 with four or more right-hand sides), the
// k <= 64 design of posv_warp64.cu on a warp segment. Measured on B200
// (B = 10,000, m = 1) against the one-row-per-lane warp kernel it replaced:
// k = 24 18.5 against 43.1 us, k = 30 30.7 against 47.6 us, k = 32 23.4
// against 45.3 us.
//
// Replaces the reference's one-thread-per-matrix tier for k <= 32
// (src/mlx_addons/linalg/_metal_kernels.py:26-72) with the same arithmetic
// contract: pivot sqrt(max(s, 1e-12)), column scaled by 1/L_jj, forward then
// back substitution, lower triangle of A read only, upper triangle of L
// zeroed.
//
// Segment lane s holds rows s (columns 0..S-1) and S + s (columns 0..KP-1)
// in registers as packed column pairs, k padded to KP (a multiple of 8,
// S < KP <= 2S) with an identity block. Right-looking factorisation: at step
// j the pivot comes by shuffle within the segment (the owner of row j
// updated it one step early), each lane scales its two column-j entries, the
// column goes through a double-buffered shared vector and every lane applies
// the rank-1 update with packed two-wide FMAs (fma.rn.f32x2). The diagonal
// and its inverse go to shared memory; the diagonal and strict upper
// triangle are then zeroed in registers, so both substitutions are
// select-free (each row keeps its running value unscaled and is multiplied
// by 1/L_ii once per pass). Backward substitution publishes 8 rows of L at a
// time, interleaved so that one 64-bit shared load gives lane s L[i][s] and
// L[i][S + s].
//
// Each warp stages its next group of matrices with cp.async while it works
// on the current one, fetching only the 16-byte chunks that hold
// lower-triangle entries.
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

namespace {

// Small CTAs (4 warps) with several per SM, so that a batch of a few
// thousand matrices spreads over all SMs in one round.
constexpr int SEG_WARPS = 4;
template <int S>
struct SegOcc {
  static constexpr int MIN_CTAS = S == 8 ? 6 : 4;  // CTAs per SM the register budget allows
};

// Per-segment shared memory (floats). Staged rows use odd float4 strides, so
// 8 consecutive rows read at the same column hit 8 different bank groups.
// The two column buffers + the diagonal of the factorisation and the row
// chunk of the back substitution share one region.
template <int S, int KP>
struct Seg {
  static constexpr int G = 32 / S;             // matrices per warp
  static constexpr int NB = KP - S;            // bottom rows
  static constexpr int S0 = S + 4;             // top-row stride
  static constexpr int S1 = KP + 4;            // bottom-row stride
  static constexpr int STAGE = S * S0 + NB * S1;
  static constexpr int CBW = 2 * S + 4;        // one column buffer: every lane writes rows s and S + s
  static constexpr int FACT = 2 * CBW + 2 * KP;  // 2 column buffers + (L_jj, 1/L_jj) per row
  static constexpr int CHUNK = 8 * 2 * S;      // 8 rows of L, interleaved
  static constexpr int UNION = FACT > CHUNK ? FACT : CHUNK;
  static constexpr int SEG_FLOATS = STAGE + UNION;
  static_assert(S == 8 || S == 16, "S");
  static_assert(KP % 8 == 0 && KP > S && KP <= 2 * S, "KP");
  static_assert((S0 / 4) % 2 == 1 && (S1 / 4) % 2 == 1, "odd float4 strides");
  static_assert(STAGE % 4 == 0 && UNION % 4 == 0 && CBW % 4 == 0, "16-byte alignment");
};

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}

template <int S, int KP>
__device__ __forceinline__ void seg_stage(const PosvParams& p, int64_t mat, float* st, int sl, bool fast, bool pair) {
  using W = Seg<S, KP>;
  if (mat >= p.batch) return;
  const int K = p.k;
  const float* src = p.A + mat * (size_t)K * K;
  // Only chunks that hold part of the lower triangle are fetched; the staged
  // upper triangle keeps stale values, which the factorisation only ever
  // combines into upper-triangle registers.
  if (fast) {  // K == KP, 16-byte aligned rows
    constexpr int Q0 = S / 4, Q1 = KP / 4;
#pragma unroll
    for (int f0 = 0; f0 < S * Q0; f0 += S) {
      const int f = f0 + sl, r = f / Q0, q = f - r * Q0;
      if (4 * q <= r) cp_async16(st + r * W::S0 + 4 * q, src + r * KP + 4 * q);
    }
#pragma unroll
    for (int f0 = 0; f0 < W::NB * Q1; f0 += S) {
      const int f = f0 + sl;
      if (f < W::NB * Q1) {
        const int r = f / Q1, q = f - r * Q1;
        if (4 * q <= S + r) cp_async16(st + S * W::S0 + r * W::S1 + 4 * q, src + (S + r) * KP + 4 * q);
      }
    }
  } else if (pair) {  // even K, 8-byte aligned rows: column pairs (c, c+1) with c <= r
    const int top = (K < S ? K : S), tp = (top + 1) / 2;
    for (int f = sl; f < top * tp; f += S) {
      const int r = f / tp, c = 2 * (f - r * tp);
      if (c <= r) cp_async8(st + r * W::S0 + c, src + (size_t)r * K + c);
    }
    const int nb = K - S, kp = K / 2;
    for (int f = sl; f < nb * kp; f += S) {
      const int r = f / kp, c = 2 * (f - r * kp);
      if (c <= S + r) cp_async8(st + S * W::S0 + r * W::S1 + c, src + (size_t)(S + r) * K + c);
    }
  } else {
    const int top = (K < S ? K : S);
    for (int f = sl; f < top * top; f += S) {
      const int r = f / top, c = f - r * top;
      if (c <= r) cp_async4(st + r * W::S0 + c, src + (size_t)r * K + c);
    }
    const int nb = K - S;
    for (int f = sl; f < nb * K; f += S) {
      const int r = f / K, c = f - r * K;
      if (c <= S + r) cp_async4(st + S * W::S0 + r * W::S1 + c, src + (size_t)(S + r) * K + c);
    }
  }
}

template <int S, int KP, int MC>
__global__ void __launch_bounds__(SEG_WARPS * 32, SegOcc<S>::MIN_CTAS) posv_seg_kernel(const PosvParams p) {
  using W = Seg<S, KP>;
  constexpr int H0 = S / 2;   // packed pairs of the top row
  constexpr int H1 = KP / 2;  // packed pairs of the bottom row
  extern __shared__ __align__(16) float smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = lane / S;      // segment of the warp = matrix of the group
  const int sl = lane % S;     // lane within the segment
  float* st = smem + (warp * W::G + g) * W::SEG_FLOATS;
  float* cbuf = st + W::STAGE;     // factorisation: 2 column buffers
  float* dg = cbuf + 2 * W::CBW;   // dg[2j] = L_jj, dg[2j + 1] = 1 / L_jj
  float* chunk = cbuf;             // back substitution: 8 rows of L

  const int K = p.k;
  const bool fast = (K == KP) && p.vec;
  const bool pair = (K % 2 == 0) && p.vec;  // 8-byte copies of column pairs
  const int r1 = S + sl;
  const int64_t per_round = (int64_t)SEG_WARPS * W::G;
  const int64_t nround = (p.batch + per_round - 1) / per_round;

  if ((int64_t)blockIdx.x < nround) {
    seg_stage<S, KP>(p, (int64_t)blockIdx.x * per_round + warp * W::G + g, st, sl, fast, pair);
    cp_async_commit();
  }
  for (int64_t rd = blockIdx.x; rd < nround; rd += gridDim.x) {
    const int64_t mat = rd * per_round + warp * W::G + g;
    const bool mvalid = mat < p.batch;
    cp_async_wait_all();
    __syncwarp();

    u64 a0[H0], a1[H1];
    if (fast && mvalid) {
#pragma unroll
      for (int c4 = 0; c4 < S; c4 += 4) lds128(st + sl * W::S0 + c4, a0[c4 / 2], a0[c4 / 2 + 1]);
      const int rb = sl < W::NB ? sl : W::NB - 1;
#pragma unroll
      for (int c4 = 0; c4 < KP; c4 += 4) lds128(st + S * W::S0 + rb * W::S1 + c4, a1[c4 / 2], a1[c4 / 2 + 1]);
      if (W::NB < S && sl >= W::NB) {  // rows beyond KP do not exist: zero rows
#pragma unroll
        for (int h = 0; h < H1; ++h) a1[h] = 0ull;
      }
    } else {
#pragma unroll
      for (int c = 0; c < S; c += 2) {
        const float* s0 = st + sl * W::S0 + c;
        const bool rowok = mvalid && sl < K;
        const float x0 = (rowok && c < K) ? s0[0] : (c == sl ? 1.f : 0.f);
        const float x1 = (rowok && c + 1 < K) ? s0[1] : (c + 1 == sl ? 1.f : 0.f);
        a0[c / 2] = pk2(x0, x1);
      }
      const int rb = sl < W::NB ? sl : W::NB - 1;
#pragma unroll
      for (int c = 0; c < KP; c += 2) {
        const bool rowok = mvalid && r1 < K;
        const float* s1 = st + S * W::S0 + rb * W::S1 + c;
        const float x0 = (rowok && c < K) ? s1[0] : (c == r1 ? 1.f : 0.f);
        const float x1 = (rowok && c + 1 < K) ? s1[1] : (c + 1 == r1 ? 1.f : 0.f);
        a1[c / 2] = pk2(x0, x1);
      }
    }
    __syncwarp();
    if (rd + gridDim.x < nround)
      seg_stage<S, KP>(p, (rd + gridDim.x) * per_round + warp * W::G + g, st, sl, fast, pair);
    cp_async_commit();

    // ---- right-looking factorisation ------------------------------------
    // Look-ahead: the owner of row j+1 updates its own diagonal as soon as its
    // column-j entry is known (dn0 / dn1), so the next pivot shuffle does not
    // wait for the shared-memory column exchange of step j.
    float dn0 = 0.f, dn1 = 0.f;
#pragma unroll
    for (int j = 0; j < KP; ++j) {
      const float dsrc = (j == 0) ? getc(a0, 0) : ((j < S) ? dn0 : dn1);
      const float sc = fmaxf(__shfl_sync(kFull, dsrc, j & (S - 1), S), kClamp);
      const float r = rsqrtf(sc);
      if (sl == 0) *reinterpret_cast<float2*>(dg + 2 * j) = make_float2(sc * r, r);
      // column j of L for this lane's rows (the owner's own entry is not used)
      float v0 = 0.f;
      if (j < S) {
        v0 = getc(a0, j < S ? j : 0) * r;
        setc(a0, j < S ? j : 0, v0);
      }
      const float v1 = getc(a1, j) * r;
      setc(a1, j, v1);
      if (j + 1 < S) dn0 = fmaf(-v0, v0, getc(a0, j + 1 < S ? j + 1 : 0));
      else if (j + 1 < KP) dn1 = fmaf(-v1, v1, getc(a1, j + 1 < KP ? j + 1 : 0));
      float* cb = cbuf + (j & 1) * W::CBW;
      if (j < S - 1) cb[sl] = v0;
      cb[S + sl] = v1;
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
            if (c < S && j < S - 1) a0[c / 2 < H0 ? c / 2 : 0] = ffma2(n0, w, a0[c / 2 < H0 ? c / 2 : 0]);
            a1[c / 2] = ffma2(n1, w, a1[c / 2]);
          } else if (c + 1 > j) {  // only column c+1
            const float wc = hi2(w);
            if (c + 1 < S) setc(a0, c + 1 < S ? c + 1 : 0, fmaf(-v0, wc, getc(a0, c + 1 < S ? c + 1 : 0)));
            setc(a1, c + 1, fmaf(-v1, wc, getc(a1, c + 1)));
          }
        }
      }
    }
    __syncwarp();
    // diagonal of this lane's rows: row s and row S + s
    const float2 dt = *reinterpret_cast<const float2*>(dg + 2 * sl);
    const float2 db = (sl < W::NB) ? *reinterpret_cast<const float2*>(dg + 2 * S + 2 * sl) : make_float2(1.f, 1.f);
    const u64 invp = pk2(dt.y, db.y);

    // ---- zero the diagonal and strict upper triangle kept in registers ---
#pragma unroll
    for (int c = 0; c < S; ++c) setc(a0, c, (c < sl) ? getc(a0, c) : 0.f);
#pragma unroll
    for (int c = S; c < KP; ++c) setc(a1, c, (c < r1) ? getc(a1, c) : 0.f);

    if (p.logdet) {
      // rows past k (identity padding) add nothing, even when a NaN in the
      // input has reached them through 0 * NaN in the updates
      float lg = (sl < K ? logf(dt.x) : 0.f) + (r1 < K ? logf(db.x) : 0.f);
      lg = warp_sum(lg, S);
      if (sl == 0 && mvalid) p.logdet[mat] = 2.f * lg;
    }

    if (p.L && mvalid && fast) {  // K == KP, aligned rows: 16-byte stores
      float* Lm = p.L + mat * (size_t)K * K;
      float* row0 = Lm + (size_t)sl * KP;
#pragma unroll
      for (int c4 = 0; c4 < S; c4 += 4)
        *reinterpret_cast<float4*>(row0 + c4) =
            make_float4(lo2(a0[c4 / 2]), hi2(a0[c4 / 2]), lo2(a0[c4 / 2 + 1]), hi2(a0[c4 / 2 + 1]));
#pragma unroll
      for (int c4 = S; c4 < KP; c4 += 4) *reinterpret_cast<float4*>(row0 + c4) = make_float4(0.f, 0.f, 0.f, 0.f);
      if (sl < W::NB) {
        float* row1 = Lm + (size_t)r1 * KP;
#pragma unroll
        for (int c4 = 0; c4 < KP; c4 += 4)
          *reinterpret_cast<float4*>(row1 + c4) =
              make_float4(lo2(a1[c4 / 2]), hi2(a1[c4 / 2]), lo2(a1[c4 / 2 + 1]), hi2(a1[c4 / 2 + 1]));
      }
      // the diagonal goes in after the row stores (same thread, program order)
      row0[sl] = dt.x;
      if (sl < W::NB) Lm[(size_t)r1 * KP + r1] = db.x;
    } else if (p.L && mvalid) {
      float* Lm = p.L + mat * (size_t)K * K;
      if (sl < K) {
        float* row0 = Lm + (size_t)sl * K;
#pragma unroll
        for (int c = 0; c < S; ++c)
          if (c < K) row0[c] = getc(a0, c);
        for (int c = S; c < K; ++c) row0[c] = 0.f;
        row0[sl] = dt.x;  // after the row stores (same thread, program order)
      }
      if (r1 < K) {
        float* row1 = Lm + (size_t)r1 * K;
#pragma unroll
        for (int c = 0; c < KP; ++c)
          if (c < K) row1[c] = getc(a1, c);
        row1[r1] = db.x;
      }
    }

    // ---- substitutions, MC right-hand sides at a time ---------------------
    for (int q0 = 0; q0 < p.m; q0 += MC) {
      u64 y[MC];  // (row s, row S + s)
      const float* bm = p.b + (size_t)mat * K * p.m;
#pragma unroll
      for (int q = 0; q < MC; ++q) {
        const bool qok = mvalid && q0 + q < p.m;
        y[q] = pk2((qok && sl < K) ? bm[(size_t)sl * p.m + q0 + q] : 0.f,
                   (qok && r1 < K) ? bm[(size_t)r1 * p.m + q0 + q] : 0.f);
      }
      // forward, L y = b: column j of L is lane-local
#pragma unroll
      for (int j = 0; j < KP; ++j) {
        const u64 lj = pk2(j < S ? getc(a0, j < S ? j : 0) : 0.f, getc(a1, j));
        const float ij = (j < S) ? dt.y : db.y;
#pragma unroll
        for (int q = 0; q < MC; ++q) {
          const float yj = __shfl_sync(kFull, ((j < S) ? lo2(y[q]) : hi2(y[q])) * ij, j & (S - 1), S);
          y[q] = ffma2(lj, pk2(-yj, -yj), y[q]);
        }
      }
#pragma unroll
      for (int q = 0; q < MC; ++q) y[q] = fmul2(y[q], invp);
      // backward, L^T x = y: rows of L are published 8 at a time, element c
      // of a row stored at 2 * (c % S) + c / S, float4 chunks swizzled by the row
      constexpr int NQ = S / 2;  // float4 chunks per published row
#pragma unroll
      for (int c0 = KP - 8; c0 >= 0; c0 -= 8) {
        const int rr = (c0 >= S ? r1 : sl) - c0;
        if (rr >= 0 && rr < 8) {
          float* dst = chunk + rr * 2 * S;
          const int sw = rr & (NQ - 1);
#pragma unroll
          for (int c = 0; c < S; c += 2) {
            float e0, e1, h0, h1;
            if (c0 >= S) {
              e0 = getc(a1, c);
              e1 = getc(a1, c + 1);
              h0 = (c + S < KP) ? getc(a1, c + S < KP ? c + S : 0) : 0.f;
              h1 = (c + S + 1 < KP) ? getc(a1, c + S + 1 < KP ? c + S + 1 : 0) : 0.f;
            } else {
              e0 = getc(a0, c);
              e1 = getc(a0, c + 1);
              h0 = 0.f;
              h1 = 0.f;
            }
            *reinterpret_cast<float4*>(dst + 4 * ((c >> 1) ^ sw)) = make_float4(e0, h0, e1, h1);
          }
        }
        __syncwarp();
#pragma unroll
        for (int i = c0 + 7; i >= c0; --i) {
          // (L[i][s], L[i][S + s]): float 2s of the row
          const u64 li = lds64(chunk + (i - c0) * 2 * S + 4 * ((sl >> 1) ^ ((i - c0) & (NQ - 1))) + 2 * (sl & 1));
          const float ii = (i < S) ? dt.y : db.y;
#pragma unroll
          for (int q = 0; q < MC; ++q) {
            const float xi = __shfl_sync(kFull, ((i < S) ? lo2(y[q]) : hi2(y[q])) * ii, i & (S - 1), S);
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
            if (sl < K) xm[(size_t)sl * p.m + q0 + q] = lo2(y[q]);
            if (r1 < K) xm[(size_t)r1 * p.m + q0 + q] = hi2(y[q]);
          }
        }
      }
    }
  }
  cp_async_wait_all();
}

template <int S, int KP, int MC>
cudaError_t launch_seg_t(const PosvParams& p, int sm_count, cudaStream_t s) {
  using W = Seg<S, KP>;
  constexpr int threads = SEG_WARPS * 32;
  const size_t smem = (size_t)SEG_WARPS * W::G * W::SEG_FLOATS * sizeof(float);
  auto kern = posv_seg_kernel<S, KP, MC>;
  static int cache[64];
  int occ = 0;
  cudaError_t e = kernel_occupancy(kern, threads, smem, cache, &occ);
  if (e != cudaSuccess) return e;
  const int64_t per_round = (int64_t)SEG_WARPS * W::G;
  const int64_t rounds = (p.batch + per_round - 1) / per_round;
  const int64_t cap = (int64_t)sm_count * occ;
  const int grid = (int)(rounds < cap ? rounds : cap);
  kern<<<grid, threads, smem, s>>>(p);
  return cudaGetLastError();
}

template <int S, int KP>
cudaError_t launch_seg_k(const PosvParams& p, int sm, cudaStream_t s) {
  return p.m <= 1 ? launch_seg_t<S, KP, 1>(p, sm, s) : launch_seg_t<S, KP, 4>(p, sm, s);
}

}  // namespace

cudaError_t launch_posv_seg(const PosvParams& p, int sm_count, cudaStream_t s) {
  if (p.k <= 16) return launch_seg_k<8, 16>(p, sm_count, s);
  if (p.k <= 24) return launch_seg_k<16, 24>(p, sm_count, s);
  if (p.k <= 32) return launch_seg_k<16, 32>(p, sm_count, s);
  return cudaErrorInvalidValue;
}

}  // namespace b2c
