// Register-resident batched Cholesky factor + solve for 33 <= k <= 64 with at
// most one right-hand side: one matrix per warp on a 2-D cyclic layout.
//
// Replaces the reference's threadgroup tier (src/mlx_addons/linalg/
// _metal_kernels.py:147-246, 33 <= k <= 80) for the fused solve and the
// log-determinant, with its arithmetic contract: pivot sqrt(max(s, 1e-12)),
// column scaled by 1/L_jj, forward then back substitution, only the lower
// triangle of A read.
//
// Layout. Lane 8b + a (a in 0..7, b in 0..3) owns rows 8 ri + a and columns
// 4 ci + b of its warp's matrix: slot (ri, ci) exists for ci <= 2 ri + 1, 72
// registers at k = 64 (against 96 for two whole rows per lane), and the
// trailing triangle of every step stays spread over all 32 lanes. k is
// padded to KP = 48 or 64 with an identity block (measured on B200: the
// layouts with an odd number of 8-row blocks, KP = 40 and 56, ran at half
// the speed of KP = 48 and 64 respectively, so k = 33..48 takes KP = 48 and
// k = 49..64 KP = 64).
//
// The trailing matrix is held negated (R = -A), so the published column
// holds L itself and the rank-1 update is R += v_row v_col.
//
// Factorisation (right-looking, KP steps, grouped by column group: the four
// steps of a group update the same slots and share one loop body, every
// register index a compile-time constant). Step j: the lanes of column j
// scale it by 1/L_jj and publish it into a per-warp buffer whose entry
// 12 a + ri holds row 8 ri + a, so the row view (rows 8 ri + a) and the
// column view (columns 4 ci + b, entry 12 (4 (ci & 1) + b) + ci / 2) are both
// 16-byte vector loads from the same 96 floats; rows <= j publish zeros,
// which masks the finished part of the trailing update without selects. Each
// lane forms the next pivot itself from two shuffled values (the diagonal
// slot before the step's update and L[j+1][j]) between its first and its
// other rank-1 FMAs, so no shared-memory round trip sits on the pivot chain.
// With one right-hand side the forward substitution rides along: lane (a, b)
// keeps rows 8 (2 b) + a and 8 (2 b + 1) + a of it. The back substitution
// publishes 8 rows of L at a time and runs column-oriented with one row per
// lane half, the solution values broadcast by shuffle.
//
// A CTA is 12 warps, one CTA per SM (168 registers per thread). Each warp
// stages its next matrix with cp.async while it works on the
// current one and fetches only the 16-byte chunks of the lower triangle, into
// 128-byte aligned rows with the chunks XOR-swizzled by row (each cp.async
// writes whole 128-byte segments, the 2-D register load is free of bank
// conflicts).
#include <cstdlib>

#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

namespace {


__device__ __forceinline__ void st32s(uint32_t a, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
__device__ __forceinline__ void st64s(uint32_t a, float x, float y) {
  asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(a), "f"(x), "f"(y) : "memory");
}
__device__ __forceinline__ void st128s(uint32_t a, float x, float y, float z, float w) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(x), "f"(y), "f"(z), "f"(w) : "memory");
}
__device__ __forceinline__ float ld32s(uint32_t a) {
  float x;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(x) : "r"(a) : "memory");
  return x;
}
__device__ __forceinline__ void ld64s(uint32_t a, float& x, float& y) {
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(x), "=f"(y) : "r"(a) : "memory");
}
__device__ __forceinline__ void ld128s(uint32_t a, float& x, float& y, float& z, float& w) {
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(x), "=f"(y), "=f"(z), "=f"(w) : "r"(a) : "memory");
}
// 1 / sqrt(x) for a normal x (the pivots are clamped to >= 1e-12): the
// hardware approximation alone, without the denormal range handling of
// rsqrtf.
__device__ __forceinline__ float rsqrt_normal(float x) {
  float r;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Width (4, 2, 1) of the vector access that starts at index ri when indices
// t .. n - 1 are covered greedily by 16-, 8- and 4-byte accesses aligned to
// their size; 0 if ri does not start one.
__host__ __device__ constexpr int vec_width(int t, int n, int ri) {
  int r = t;
  while (r < n) {
    const int w = (r % 4 == 0 && r + 3 < n) ? 4 : (r % 2 == 0 && r + 1 < n) ? 2 : 1;
    if (r == ri) return w;
    r += w;
  }
  return 0;
}

template <int KP>
struct TileLayout {
  static constexpr int NB = KP / 8;  // row blocks
  static constexpr int NC = KP / 4;  // column groups
  // Staged matrix: rows 0..31 at 32 floats, rows 32.. at 64 floats, each
  // 128-byte aligned, 16-byte chunk q of row r stored at chunk position
  // (q & 8) | ((q & 7) ^ (r & 7)). A cp.async that fills 8 consecutive chunks
  // of a row then writes one 128-byte segment (one shared-memory wavefront,
  // and each global sector requested once: this matters when A is mapped
  // host memory read across PCIe), and the 2-D register load, lanes
  // (a, b) reading (8 ri + a, 4 ci + b), hits 32 distinct banks.
  __host__ __device__ static constexpr int rowbase(int r) { return r < 32 ? 32 * r : 1024 + 64 * (r - 32); }
  __host__ __device__ static constexpr int chunkpos(int r, int q) { return (q & 8) | ((q & 7) ^ (r & 7)); }
  __host__ __device__ static constexpr int at(int r, int c) { return rowbase(r) + 4 * chunkpos(r, c >> 2) + (c & 3); }
  static constexpr int MAT = rowbase(KP);  // floats of the staged matrix
  static constexpr int STAGE = MAT + KP;   // + its right-hand side
  // Column buffer (floats): entry 12 a + ri is row 8 ri + a of the published
  // column (12 a mod 32 puts the eight row phases in distinct 4-bank groups);
  // entry 96 holds the right-hand-side value of the step's row.
  static constexpr int XS = 12;
  static constexpr int XB = 100;
  static constexpr int NPB = 4;          // one column buffer per step of a group
  static constexpr int DG = 2 * KP;      // per step: s_j, 1 / L_jj
  static constexpr int CHS = 68;         // back substitution: 8 rows of L, row stride
  static constexpr int UNION = (NPB * XB + DG) > 8 * CHS ? (NPB * XB + DG) : 8 * CHS;
  static constexpr int WARP_FLOATS = (STAGE + UNION + 31) / 32 * 32;  // 128-byte aligned warp regions
  static_assert(KP % 8 == 0 && KP > 32 && KP <= 64, "KP");
  static_assert(STAGE % 4 == 0 && WARP_FLOATS % 32 == 0 && XB % 4 == 0, "alignment");
};

// Stage matrix `mat` into `sm`.
template <int KP, int NS>
__device__ __forceinline__ void tile_stage(const PosvParams& p, int64_t mat, float* sm, int lane, bool fast,
                                           bool bfast) {
  using Lay = TileLayout<KP>;
  constexpr int NB = Lay::NB;
  const int K = p.k;
  const float* src = p.A + mat * (size_t)K * K;
  if (fast) {
    // k % 4 == 0 and 16-byte aligned rows: the 16-byte chunks that hold
    // lower-triangle entries (chunk q of row r when 4 q <= r), rows 0..31
    // eight lanes per row and rows 32.. sixteen lanes per row, so each warp
    // instruction asks for whole row prefixes (this matters when A is mapped
    // host memory read across PCIe); the staged upper-triangle entries keep
    // stale values, which only ever reach upper-triangle slots. Rows past k
    // (all of them 32 or more) are identity rows, written as chunks.
    auto dst = [&](int r, int q) { return sm + Lay::rowbase(r) + 4 * Lay::chunkpos(r, q); };
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int r = (lane >> 3) + 4 * t, q = lane & 7;
      if (q <= t) cp_async16(dst(r, q), src + r * K + 4 * q);
    }
    constexpr int Q = KP / 4, TOTAL = (KP - 32) * Q;
#pragma unroll
    for (int f0 = 0; f0 < TOTAL; f0 += 32) {
      const int f = f0 + lane;
      const int r = 32 + f / Q, q = f % Q;
      if (f < TOTAL && q <= (r >> 2)) {
        if (r < K) {
          cp_async16(dst(r, q), src + r * K + 4 * q);
        } else {
          const int d = r - 4 * q;  // position of the diagonal in the chunk
          *reinterpret_cast<float4*>(dst(r, q)) =
              make_float4(d == 0 ? 1.f : 0.f, d == 1 ? 1.f : 0.f, d == 2 ? 1.f : 0.f, d == 3 ? 1.f : 0.f);
        }
      }
    }
  } else {
    // element-wise: lower triangle from A, identity padding past k, zero
    // upper triangle (every slot the register load reads: columns
    // 0 .. 8 (r / 8) + 7 of row r)
    for (int r = 0; r < KP; ++r) {
      const int W = 8 * (r >> 3) + 8;
      for (int c = lane; c < W; c += 32) {
        float* d = sm + Lay::at(r, c);
        if (r < K && c <= r)
          cp_async4(d, src + (size_t)r * K + c);
        else
          *d = (r == c) ? 1.f : 0.f;
      }
    }
  }
  if (NS) {
    float* sb = sm + Lay::MAT;
    const float* bsrc = p.b + mat * (size_t)K;
    if (bfast) {
      if (4 * lane < K)
        cp_async16(sb + 4 * lane, bsrc + 4 * lane);
      else if (lane < KP / 4)
        *reinterpret_cast<float4*>(sb + 4 * lane) = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      for (int r = lane; r < KP; r += 32) {
        if (r < K)
          cp_async4(sb + r, bsrc + r);
        else
          sb[r] = 0.f;
      }
    }
  }
}

// Column group H of the right-looking factorisation: steps j = 4 H .. 4 H + 3
// (rows of block H / 2). On entry r / sv hold pivot j's 1 / L_jj and s_j, and
// D1 the diagonal slot (j+1, j+1) after step j-1's update.
template <int KP, int NS, int H>
__device__ __forceinline__ void tile_group(float (&R)[KP / 8][KP / 4], float (&Y)[KP / 8], float& r, float& sv,
                                           float& D1, uint32_t pb, uint32_t dgb, int lane, int a, int b,
                                           uint32_t rowoff, uint32_t coloff0, uint32_t coloff1) {
  using Lay = TileLayout<KP>;
  constexpr int NB = Lay::NB, NC = Lay::NC;
  constexpr int t = H >> 1, s = H;
  constexpr bool last = (H == NC - 1);
  constexpr int tn = (4 * H + 4) >> 3;  // block of the next group's first row
  // a - 4 (H & 1) compared with jb gives a > j & 7 and a == j & 7 in one compare
  const int ar = a - 4 * (H & 1);
  uint32_t P = pb, dga = dgb + 8 * (4 * H);
  // KP = 64: two steps per loop body, measured on B200 the best trade
  // between the run-time index work of a rolled loop and the
  // instruction-cache misses of a fully unrolled one (k = 64, B = 10,000:
  // 85 us, against 98 / 97 us); KP = 48 with a right-hand side: fully
  // unrolled (48.9 us against 52.2 us with two steps per body; without one
  // the full unroll spills 184 bytes, so that form keeps two steps)
#pragma unroll(KP == 64 || NS == 0 ? 2 : 4)
  for (int jb = 0; jb < 4; ++jb) {
    const int jn = 4 * H + jb + 1;  // next column
    if (lane == 0) st64s(dga, sv, r);  // every lane holds the same values
    // scale column j on its lanes
    const bool wr = (b == jb);
    const float f = wr ? -r : 1.f;
#pragma unroll
    for (int ri = t; ri < NB; ++ri) R[ri][s] *= f;
    float wsrc = R[t][s];
    if constexpr ((H & 1) && t + 1 < NB) wsrc = (jb == 3) ? R[t + 1][s] : wsrc;
    const float W1 = __shfl_sync(kFull, wsrc, 8 * jb + (jn & 7));  // L[j+1][j]
    // publish column j (rows <= j as zeros): entries 12 a + ri, ri >= t
    if (wr) {
      float v[NB];
#pragma unroll
      for (int ri = t; ri < NB; ++ri) v[ri] = R[ri][s];
      v[t] = (ar > jb) ? v[t] : 0.f;
      const uint32_t dst = P + rowoff;
#pragma unroll
      for (int ri = t; ri < NB; ++ri) {
        const int w = vec_width(t, NB, ri);
        if (w == 4)
          st128s(dst + 4 * ri, v[ri], v[ri + 1], v[ri + 2], v[ri + 3]);
        else if (w == 2)
          st64s(dst + 4 * ri, v[ri], v[ri + 1]);
        else if (w == 1)
          st32s(dst + 4 * ri, v[ri]);
      }
    }
    float yv = 0.f;
    if constexpr (NS) {
      // row j's right-hand-side value, kept by lanes (j & 7, every b)
      Y[t] *= (ar == jb) ? -r : 1.f;
      yv = __shfl_sync(kFull, Y[t], 4 * (H & 1) + jb);
    }
    __syncwarp();
    float rv[NB];
    {
      const uint32_t src = P + rowoff;
#pragma unroll
      for (int ri = t; ri < NB; ++ri) {
        const int w = vec_width(t, NB, ri);
        if (w == 4)
          ld128s(src + 4 * ri, rv[ri], rv[ri + 1], rv[ri + 2], rv[ri + 3]);
        else if (w == 2)
          ld64s(src + 4 * ri, rv[ri], rv[ri + 1]);
        else if (w == 1)
          rv[ri] = ld32s(src + 4 * ri);
      }
    }
    // column values of one parity: entries u = ci / 2 of row phase 4 par + b
    auto colquad = [&](const int par, const int u0) {
      const uint32_t src = P + (par ? coloff1 : coloff0);
      float cv[4];
      const int lo = (s - par + 1) >> 1;  // first u with 2 u + par >= s
      const int first = u0 > lo ? u0 : lo;
      const int n = (u0 + 4 < NB ? u0 + 4 : NB) - first;
      if (n <= 0) return;
      if (first == u0 && n == 4)
        ld128s(src + 4 * u0, cv[0], cv[1], cv[2], cv[3]);
      else if (first == u0 + 2 && n == 2)
        ld64s(src + 4 * (u0 + 2), cv[2], cv[3]);
      else {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (u0 + k >= first && u0 + k < first + n) cv[k] = ld32s(src + 4 * (u0 + k));
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int u = u0 + k, c = 2 * u + par;
        if (u < first || u >= first + n) continue;
#pragma unroll
        for (int ri = t; ri < NB; ++ri) {
          if (c > 2 * ri + 1) continue;
          R[ri][c] = fmaf(rv[ri], cv[k], R[ri][c]);
        }
      }
    };
    // the quads holding groups s and s + 1 (the next column) first
    constexpr int pa0 = s & 1, qa0 = ((s >> 1) >> 2) << 2;
    constexpr int pa1 = (s + 1) & 1, qa1 = (((s + 1) >> 1) >> 2) << 2;
    constexpr bool two = !last && !(pa1 == pa0 && qa1 == qa0);
    colquad(pa0, qa0);
    if constexpr (two) colquad(pa1, qa1);
    {
      // pivot j+1 = -(D1 + W1^2) (unused after the last column)
      const float sn = fmaxf(-fmaf(W1, W1, D1), kClamp);
      sv = sn;
      r = rsqrt_normal(sn);
    }
#pragma unroll
    for (int par = 0; par < 2; ++par) {
#pragma unroll
      for (int u0 = 0; u0 < NB; u0 += 4)
        if (!(par == pa0 && u0 == qa0) && !(two && par == pa1 && u0 == qa1)) colquad(par, u0);
    }
    if constexpr (NS) {
      // rows 8 ri + a from the row view just loaded (rows <= j read 0)
#pragma unroll
      for (int ri = t; ri < NB; ++ri) Y[ri] = fmaf(rv[ri], yv, Y[ri]);
    }
    // the diagonal slot (j+2, j+2) after this step's update, for pivot j+2
    float dsrc = R[t][s];
    if constexpr (!last) dsrc = (jb >= 2) ? R[tn][s + 1] : dsrc;
    D1 = __shfl_sync(kFull, dsrc, 8 * ((jn + 1) & 3) + ((jn + 1) & 7));
    P += 4 * Lay::XB;
    dga += 8;
  }
}

template <int KP, int NS, int H>
struct TileGroups {
  __device__ static __forceinline__ void run(float (&R)[KP / 8][KP / 4], float (&Y)[KP / 8], float& r, float& sv,
                                             float& D1, uint32_t pb, uint32_t dgb, int lane, int a, int b,
                                             uint32_t rowoff, uint32_t coloff0, uint32_t coloff1) {
    tile_group<KP, NS, H>(R, Y, r, sv, D1, pb, dgb, lane, a, b, rowoff, coloff0, coloff1);
    TileGroups<KP, NS, H + 1>::run(R, Y, r, sv, D1, pb, dgb, lane, a, b, rowoff, coloff0, coloff1);
  }
};
template <int KP, int NS>
struct TileGroups<KP, NS, KP / 4> {
  __device__ static __forceinline__ void run(float (&)[KP / 8][KP / 4], float (&)[KP / 8], float&, float&, float&,
                                             uint32_t, uint32_t, int, int, int, uint32_t, uint32_t, uint32_t) {}
};

}  // namespace

// 12 warps (12 matrices) per CTA, one CTA per SM: 168 registers per thread.
// Measured on B200 (k = 64, B = 10,000): 85 us, against 102 / 105 us with
// 14 / 10 warps and 117 us with two CTAs of 8.
constexpr int TL_WARPS = 12;

template <int KP, int NS>
__global__ void __launch_bounds__(TL_WARPS * 32, 1) posv_tile_kernel(const PosvParams p, int bvec) {
  using Lay = TileLayout<KP>;
  constexpr int NB = Lay::NB, NC = Lay::NC;
  extern __shared__ __align__(128) float smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int a = lane & 7, b = lane >> 3;
  float* st = smem + warp * Lay::WARP_FLOATS;
  // union region (32-bit shared addresses): the column buffers and the
  // pivots during the factorisation; y by row, then 8 rows of L, during the
  // back substitution
  const uint32_t un = smem_u32(st + Lay::STAGE);
  const uint32_t pb = un;
  const uint32_t dgb = un + 4 * Lay::NPB * Lay::XB;
  const uint32_t zb = un, ch = un;
  const uint32_t rowoff = 4 * Lay::XS * a, coloff0 = 4 * Lay::XS * b, coloff1 = 4 * Lay::XS * (4 + b);

  const int K = p.k;
  const bool fast = (K % 4 == 0) && p.vec;
  const bool bfast = (K % 4 == 0) && bvec;
  // matrix gw + i nw for warp gw = warp * gridDim.x + CTA: every SM gets the
  // same number of matrices to within one (the last round's warps spread
  // over all SMs instead of filling the first ones)
  const int64_t gw = (int64_t)warp * gridDim.x + blockIdx.x;
  const int64_t nw = (int64_t)gridDim.x * TL_WARPS;

  if (gw < p.batch) tile_stage<KP, NS>(p, gw, st, lane, fast, bfast);
  cp_async_commit();

  for (int64_t mat = gw; mat < p.batch; mat += nw) {
    cp_async_wait_all();
    __syncwarp();

    // ---- registers from the staged matrix ---------------------------------
    float R[NB][NC];
    float Y[NB];  // right-hand side, rows 8 ri + a (the same on the four lanes b)
#pragma unroll
    for (int ri = 0; ri < NB; ++ri) {
      const int ro = Lay::rowbase(8 * ri + a) + b;  // row 8 ri + a, (8 ri + a) & 7 = a
#pragma unroll
      for (int ci = 0; ci < NC; ++ci)
        if (ci <= 2 * ri + 1) R[ri][ci] = -st[ro + 4 * ((ci & 8) | ((ci & 7) ^ a))];
    }
    if (NS) {
#pragma unroll
      for (int ri = 0; ri < NB; ++ri) Y[ri] = -st[Lay::MAT + 8 * ri + a];
    }
    __syncwarp();
    if (mat + nw < p.batch) tile_stage<KP, NS>(p, mat + nw, st, lane, fast, bfast);
    cp_async_commit();

    // ---- right-looking factorisation (+ forward substitution) -------------
    float r, sv, D1;
    {
      const float s0 = fmaxf(-__shfl_sync(kFull, R[0][0], 0), kClamp);  // pivot 0 = A_00
      sv = s0;
      r = rsqrt_normal(s0);
      D1 = __shfl_sync(kFull, R[0][0], 9);  // slot (1, 1) before step 0's update
    }
    TileGroups<KP, NS, 0>::run(R, Y, r, sv, D1, pb, dgb, lane, a, b, rowoff, coloff0, coloff1);
    __syncwarp();

    // ---- log-determinant: sum of log(s_j) = 2 sum log(L_jj), rows < k -----
    if (p.logdet) {
      float lg = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = 32 * h + lane;
        if (j < K) lg += logf(ld32s(dgb + 8 * j));
      }
      lg = warp_sum(lg);
      if (lane == 0) p.logdet[mat] = lg;
    }

    if constexpr (NS) {
      // ---- back substitution, L^T x = y ------------------------------------
      // lane l keeps rows l and 32 + l: x_i = y_i / L_ii, then y_c -= L[i][c] x_i
      const bool hi_half = 32 + lane < KP;
      const float r0 = ld32s(dgb + 8 * lane + 4);
      const float r1 = hi_half ? ld32s(dgb + 8 * (32 + lane) + 4) : 1.f;
      __syncwarp();  // column buffers are dead from here; the pivots are read
      if (b == 0) {
#pragma unroll
        for (int ri = 0; ri < NB; ++ri) st32s(zb + 4 * (8 * ri + a), Y[ri]);
      }
      __syncwarp();
      float y0 = ld32s(zb + 4 * lane);
      float y1 = hi_half ? ld32s(zb + 4 * (32 + lane)) : 0.f;
      __syncwarp();
      // the diagonal and upper part of the diagonal blocks read 0
#pragma unroll
      for (int T = 0; T < NB; ++T) {
        R[T][2 * T] = (b >= a) ? 0.f : R[T][2 * T];
        R[T][2 * T + 1] = (4 + b >= a) ? 0.f : R[T][2 * T + 1];
      }
      const uint32_t crow = ch + 4 * (Lay::CHS * a + b);
#pragma unroll
      for (int T = NB - 1; T >= 0; --T) {
        // chunk row a = row 8 T + a of L; the next two column groups read 0
        // (they held the previous chunk's diagonal blocks)
#pragma unroll
        for (int ci = 0; ci < NC; ++ci) {
          if (ci <= 2 * T + 1)
            st32s(crow + 16 * ci, R[T][ci]);
          else if (ci <= 2 * T + 3)
            st32s(crow + 16 * ci, 0.f);
        }
        __syncwarp();
        // rows i = 8 T + 7 .. 8 T; L[i][c] reads 0 for c >= i
        const uint32_t rd = ch + 4 * lane;
#pragma unroll
        for (int ii = 7; ii >= 0; --ii) {
          const uint32_t row = rd + 4 * Lay::CHS * ii;
          if (T >= 4) {  // rows 32 + ...: lane ii + 8 T - 32 owns it
            const float xi = __shfl_sync(kFull, y1 * r1, 8 * T - 32 + ii);
            y0 = fmaf(-ld32s(row), xi, y0);
            y1 = fmaf(-ld32s(row + 4 * 32), xi, y1);
          } else {
            const float xi = __shfl_sync(kFull, y0 * r0, 8 * T + ii);
            y0 = fmaf(-ld32s(row), xi, y0);
          }
        }
        __syncwarp();
      }
      float* xm = p.x + mat * (size_t)K;
      if (lane < K) xm[lane] = y0 * r0;
      if (hi_half && 32 + lane < K) xm[32 + lane] = y1 * r1;
      __syncwarp();  // chunk reads done before the next matrix's column buffers
    }
  }
  cp_async_wait_all();
}

namespace {

template <int KP, int NS>
cudaError_t launch_tile_t(const PosvParams& p, int sm_count, cudaStream_t s) {
  using Lay = TileLayout<KP>;
  constexpr int threads = TL_WARPS * 32;
  const size_t smem = (size_t)TL_WARPS * Lay::WARP_FLOATS * sizeof(float);
  auto kern = posv_tile_kernel<KP, NS>;
  static int cache[64];
  int occ = 0;
  cudaError_t e = kernel_occupancy(kern, threads, smem, cache, &occ);
  if (e != cudaSuccess) return e;
  const int64_t ctas = (p.batch + TL_WARPS - 1) / TL_WARPS;
  const int64_t cap = (int64_t)sm_count * occ;
  const int grid = (int)(ctas < cap ? ctas : cap);
  const int bvec = (p.m == 1 && p.b && (reinterpret_cast<uintptr_t>(p.b) & 15u) == 0) ? 1 : 0;
  kern<<<grid, threads, smem, s>>>(p, bvec);
  return cudaGetLastError();
}

template <int KP>
cudaError_t launch_tile_k(const PosvParams& p, int sm, cudaStream_t s) {
  return p.m == 0 ? launch_tile_t<KP, 0>(p, sm, s) : launch_tile_t<KP, 1>(p, sm, s);
}

}  // namespace

bool posv_tile_applies(const PosvParams& p) {
  const char* e = getenv("B2C_TILE_TIER");
  if (e && e[0] == '0') return false;
  return p.k > 32 && p.k <= 64 && p.m <= 1 && !p.L;
}

cudaError_t launch_posv_tile(const PosvParams& p, int sm_count, cudaStream_t s) {
  if (p.k <= 48) return launch_tile_k<48>(p, sm_count, s);
  return launch_tile_k<64>(p, sm_count, s);
}

}  // namespace b2c
