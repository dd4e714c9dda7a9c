// Blocked Cholesky factor + solve for k > 64, register-tiled.
//
// Same contract as the blocked tier it supersedes (posv_blocked.cu, which
// remains the path for k whose panel inverses do not fit shared memory) and as
// the reference's blocked algorithm (src/mlx_addons/linalg/_blocked.py:34-217):
// lower triangle of A read, pivots clamped to sqrt(1e-12), L written once
// with its upper triangle zeroed when requested, substitutions in the same
// kernel.
//
// One CTA of NT = 128 threads factors one matrix at a time (persistent grid,
// four CTAs per SM: the serial parts of a panel, the 32x32 factor and its
// inverse, of one matrix overlap the GEMMs of the others), left-looking by
// 32-column panels. The rows of panel J (columns j0..j0+31, rows j0..k-1) are
// taken in groups of 128, 64 or 32 rows (the register tile of a thread is
// RI x 4 with RI = 8, 4, 2), so the shrinking panels of the late columns are
// never padded by more than 31 rows. For each group:
//   1. P = A[rows, panel] - L[rows, :j0] L[panel, :j0]^T as a register-tiled
//      GEMM: thread (ty, tx) owns rows ty + (NT/8) i (i < RI) and columns
//      tx + 8 j (j < 4). Both operands are staged in shared memory 32 columns at a
//      time with cp.async, double-buffered: chunk c + 1 loads while chunk c
//      is multiplied, one CTA barrier per chunk. The strides make every
//      float4 read conflict-free.
//   2. First group of the panel: warp 0 factors the 32x32 diagonal block in
//      registers (right-looking, reference clamp); all warps then form its
//      inverse, 32 / (NT/32) columns each, by independent forward substitutions, kept in
//      shared memory (swizzled) for this panel. When right-hand sides follow,
//      the strict lower triangle of the inverse is also stored, transposed,
//      in the strict upper triangle of the diagonal block of L's slot (unused
//      by L; zeroed again at the end when L is an output).
//   3. The panel rows below the diagonal block are solved as X = P L_JJ^{-T},
//      the same micro-kernel with the inverse as the second operand.
//   4. The panel is written once.
// The substitutions then use the panel inverses (reloaded per 32-row block
// from the slot; 1 / L_jj is recomputed bit for bit): each block is a GEMV
// over the rows already solved followed by a 32x32 mat-vec with the inverse
// (forward: L_JJ^{-1}; backward: L_JJ^{-T}), one warp per right-hand side,
// instead of a 32-step dependent chain.
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

namespace {

constexpr int KC2 = 32;    // staged columns of the GEMM operands
constexpr int AS2 = 36;    // row stride of the staged operands (floats)
constexpr int MCB2 = 8;    // max right-hand sides per pass

template <int NT>
struct B2 {
  static constexpr int NW = NT / 32;      // warps
  static constexpr int TY = NT / 8;       // thread rows; a thread's rows are ty + TY i
  static constexpr int RMIN = 32 / TY;    // smallest RI: a first group covers the 32 diagonal rows
  static constexpr int A_FL = 8 * TY * AS2;  // one A-operand buffer (RI = 8)
  static constexpr int B_FL = 32 * AS2;      // one B-operand buffer
  // shared-memory layout (floats)
  static constexpr int OFF_A = 0;                  // 2 x A_FL: GEMM operand A (double-buffered), then P; solves: RHS
  static constexpr int OFF_B = OFF_A + 2 * A_FL;   // 2 x B_FL: GEMM operand B; column buffer; solves: reduction
  static constexpr int OFF_D = OFF_B + 2 * B_FL;   // 32 x 36: diagonal block
  static constexpr int OFF_INV = OFF_D + 32 * 36;  // 1024: inverse of the current diagonal block (swizzled rows)
  static constexpr int OFF_Y = OFF_INV + 1024;     // 2 x 256: y rows of the staged chunk (32 x 8), then t
  static constexpr int SMEM = OFF_Y + 2 * 256;
  static constexpr int CPW = 32 / NW;              // inverse columns per warp
  static constexpr int TV = 256 / NT;              // fused-forward (row, rhs) pairs per thread
  static_assert(NT == 128 || NT == 256, "NT");
  static_assert(NW * MCB2 * 32 <= 2 * B_FL, "reduction buffer");
};

__device__ __forceinline__ int inv_off(int c, int q) { return c * 32 + (((q >> 2) ^ (c & 7)) << 2) + (q & 3); }

// acc[i][j] += sign * sum_kk As[ty + TY i][kk] * Bs[tx + 8 j][kk] over KC2 columns
template <bool SUB, int RI, int TY>
__device__ __forceinline__ void tile_mma(float (&acc)[RI][4], const float* As, const float* Bs, int ty, int tx) {
#pragma unroll 1
  for (int kk = 0; kk < KC2; kk += 4) {
    float4 a[RI], b[4];
#pragma unroll
    for (int i = 0; i < RI; ++i) a[i] = *reinterpret_cast<const float4*>(As + (ty + TY * i) * AS2 + kk);
#pragma unroll
    for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(Bs + (tx + 8 * j) * AS2 + kk);
#pragma unroll
    for (int i = 0; i < RI; ++i)
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
template <int RI, int TY>
__device__ __forceinline__ void tile_mma_inv(float (&acc)[RI][4], const float* As, const float* Li, int ty, int tx) {
#pragma unroll 1
  for (int kk = 0; kk < 32; kk += 4) {
    float4 a[RI], b[4];
#pragma unroll
    for (int i = 0; i < RI; ++i) a[i] = *reinterpret_cast<const float4*>(As + (ty + TY * i) * AS2 + kk);
#pragma unroll
    for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(Li + inv_off(tx + 8 * j, kk));
#pragma unroll
    for (int i = 0; i < RI; ++i)
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

// One row group of panel J: rows rg .. rg + TY RI - 1 (clipped to K).
// fwd: the forward substitution of the first p.m (<= MCB2) right-hand sides
// rides along: for the panel's first group, the (row, right-hand side) pairs
// (j0 + ty + TY t, tx) accumulate t = b - L[row, :j0] y[:j0] from the staged
// B operand (exactly the panel rows' chunks) and the staged rows of y, and
// y_J = L_JJ^{-1} t is written to x (which then holds y).
template <int NT, int RI>
__device__ __noinline__ void panel_group(const PosvParams& p, const float* A, float* Wm, int K, int j0, int rg,
                                            float* sm, bool vec, bool fwd, int64_t mat, float& lgacc) {
  using S = B2<NT>;
  constexpr int TY = S::TY;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ty = tid >> 3, tx = tid & 7;
  const int bw = min(32, K - j0);
  float* sD = sm + S::OFF_D;
  float* Li = sm + S::OFF_INV;
  const bool first = (rg == j0);
  const bool fw = fwd && first;
  const int m = p.m;
  float* ym = p.x + (size_t)mat * K * m;  // y (forward result) lives in x
  float tv[S::TV];                        // t of (row j0 + ty + TY t, right-hand side tx)
#pragma unroll
  for (int t = 0; t < S::TV; ++t) {
    const int r = ty + TY * t;
    tv[t] = (fw && r < bw && tx < m) ? p.b[(size_t)mat * K * m + (size_t)(j0 + r) * m + tx] : 0.f;
  }

  float acc[RI][4];
#pragma unroll
  for (int i = 0; i < RI; ++i) {
    const int r = rg + ty + TY * i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = tx + 8 * j;
      acc[i][j] = (r < K && c < bw) ? __ldg(A + (size_t)r * K + j0 + c) : 0.f;
    }
  }

  // ---- P = A[rows, panel] - L[rows, :j0] L[panel, :j0]^T, double-buffered --
  const int nch = j0 / KC2;
  auto stage = [&](int ch) {
    float* As = sm + S::OFF_A + (ch & 1) * S::A_FL;
    float* Bs = sm + S::OFF_B + (ch & 1) * S::B_FL;
    const int p0 = ch * KC2;
    if (vec) {
#pragma unroll
      for (int t = 0; t < RI; ++t) {
        const int f = tid + NT * t, row = f >> 3, q = f & 7;
        if (rg + row < K) cp_async16(As + row * AS2 + 4 * q, Wm + (size_t)(rg + row) * K + p0 + 4 * q);
      }
#pragma unroll
      for (int t = 0; t < 256 / NT; ++t) {
        const int f = tid + NT * t, row = f >> 3, q = f & 7;
        if (row < bw) cp_async16(Bs + row * AS2 + 4 * q, Wm + (size_t)(j0 + row) * K + p0 + 4 * q);
      }
    } else {
      for (int f = tid; f < TY * RI * KC2; f += NT) {
        const int row = f >> 5, c = f & 31;
        if (rg + row < K) cp_async4(As + row * AS2 + c, Wm + (size_t)(rg + row) * K + p0 + c);
      }
      for (int f = tid; f < 32 * KC2; f += NT) {
        const int row = f >> 5, c = f & 31;
        if (row < bw) cp_async4(Bs + row * AS2 + c, Wm + (size_t)(j0 + row) * K + p0 + c);
      }
    }
    if (fw && tx < m) {
#pragma unroll
      for (int t = 0; t < S::TV; ++t) {
        const int r = ty + TY * t;
        cp_async4(sm + S::OFF_Y + (ch & 1) * 256 + r * 8 + tx, ym + (size_t)(p0 + r) * m + tx);
      }
    }
    cp_async_commit();
  };
  if (nch > 0) {
    __syncthreads();  // the previous group's readers of the operand buffers are done
    stage(0);
    for (int ch = 0; ch < nch; ++ch) {
      cp_async_wait_all();  // chunk ch (the only group in flight)
      __syncthreads();      // chunk ch visible; everyone is past chunk ch - 1
      if (ch + 1 < nch) stage(ch + 1);
      tile_mma<true, RI, TY>(acc, sm + S::OFF_A + (ch & 1) * S::A_FL, sm + S::OFF_B + (ch & 1) * S::B_FL, ty, tx);
      if (fw && tx < m) {  // t -= L[row, chunk] y[chunk][tx]
        const float* Ys = sm + S::OFF_Y + (ch & 1) * 256 + tx;
#pragma unroll
        for (int t = 0; t < S::TV; ++t) {
          const int r = ty + TY * t;
          if (r < bw) {
            const float* Bs = sm + S::OFF_B + (ch & 1) * S::B_FL + r * AS2;
            float v = tv[t];
#pragma unroll
            for (int kk = 0; kk < KC2; kk += 4) {
              const float4 l4 = *reinterpret_cast<const float4*>(Bs + kk);
              v = fmaf(-l4.x, Ys[(kk + 0) * 8], v);
              v = fmaf(-l4.y, Ys[(kk + 1) * 8], v);
              v = fmaf(-l4.z, Ys[(kk + 2) * 8], v);
              v = fmaf(-l4.w, Ys[(kk + 3) * 8], v);
            }
            tv[t] = v;
          }
        }
      }
    }
  }

  // ---- P to shared memory (operand buffer 0); diagonal rows to sD --------
  float* Pm = sm + S::OFF_A;
  float* sT = sm + S::OFF_Y;  // t of the panel (32 x 8), free once the chunks are done
  __syncthreads();
#pragma unroll
  for (int i = 0; i < RI; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) Pm[(ty + TY * i) * AS2 + tx + 8 * j] = (tx + 8 * j < bw) ? acc[i][j] : 0.f;
  if (first) {
#pragma unroll
    for (int i = 0; i < S::RMIN; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sD[(ty + TY * i) * 36 + tx + 8 * j] = acc[i][j];  // row j0 + ty + TY i
  }
  if (fw) {
#pragma unroll
    for (int t = 0; t < S::TV; ++t) {
      const int r = ty + TY * t;
      sT[r * 8 + tx] = (r < bw && tx < m) ? tv[t] : 0.f;
    }
  }
  __syncthreads();

  // ---- diagonal block: factor (warp 0) and invert (all warps) ------------
  if (first) {
    if (warp == 0) {
      float a[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) a[c] = (lane < bw && c < bw) ? sD[lane * 36 + c] : (c == lane ? 1.f : 0.f);
      float invo = 1.f, dv = 1.f;
      factor32(a, lane, sm + S::OFF_B, invo, dv);  // operand buffer B doubles as the column buffer
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 32; ++c) sD[lane * 36 + c] = (c < lane) ? a[c] : (c == lane ? dv : 0.f);
      if (lane < bw) lgacc += logf(dv);
    }
    __syncthreads();
    // L_JJ rows to the slot, coalesced (upper part: zero, or the transposed
    // inverse written below when right-hand sides follow); rows right of the
    // block zeroed when L is an output
    for (int e = tid; e < 1024; e += NT) {
      const int r = e >> 5, c = e & 31;
      if (r < bw && c < bw && (c <= r || p.m == 0)) Wm[(size_t)(j0 + r) * K + j0 + c] = sD[r * 36 + c];
    }
    if (p.L) {
      const int w = K - j0 - bw;
      for (int e = tid; e < bw * w; e += NT) {
        const int r = e / w, c = e - r * w;
        Wm[(size_t)(j0 + r) * K + j0 + bw + c] = 0.f;
      }
    }
    // inverse X = L_JJ^{-1}; warp w computes columns CPW w .. CPW w + CPW - 1, lane = row
    {
      float lrow[32];
#pragma unroll
      for (int c4 = 0; c4 < 32; c4 += 4) {
        const float4 v = *reinterpret_cast<const float4*>(sD + lane * 36 + c4);
        lrow[c4] = v.x;
        lrow[c4 + 1] = v.y;
        lrow[c4 + 2] = v.z;
        lrow[c4 + 3] = v.w;
      }
      float dl = 1.f;
#pragma unroll
      for (int c = 0; c < 32; ++c) dl = (c == lane) ? lrow[c] : dl;
      const float il = 1.f / dl;
      float xs[S::CPW];
#pragma unroll
      for (int q = 0; q < S::CPW; ++q) xs[q] = (lane == S::CPW * warp + q) ? 1.f : 0.f;
#pragma unroll
      for (int pp = 0; pp < 32; ++pp) {
        // row pp of X is final in lane pp once scaled by 1 / L_pp
#pragma unroll
        for (int q = 0; q < S::CPW; ++q) {
          const float xp = __shfl_sync(kFull, xs[q] * il, pp);
          xs[q] = (lane == pp) ? xp : ((lane > pp) ? fmaf(-lrow[pp], xp, xs[q]) : xs[q]);
        }
      }
#pragma unroll
      for (int q = 0; q < S::CPW; ++q) {
        const int c = S::CPW * warp + q;
        Li[inv_off(lane, c)] = xs[q];
        // strict lower triangle, transposed into the unused strict upper
        // triangle of the diagonal block, for the substitutions
        if (p.m > 0 && lane > c && lane < bw) Wm[(size_t)(j0 + c) * K + j0 + lane] = xs[q];
      }
    }
    __syncthreads();
    if (fw && tx < m) {  // y_J = L_JJ^{-1} t
#pragma unroll
      for (int t = 0; t < S::TV; ++t) {
        const int r = ty + TY * t;
        if (r < bw) {
          float y = 0.f;
#pragma unroll
          for (int c4 = 0; c4 < 32; c4 += 4) {
            const float4 l4 = *reinterpret_cast<const float4*>(Li + inv_off(r, c4));
            y = fmaf(l4.x, sT[(c4 + 0) * 8 + tx], y);
            y = fmaf(l4.y, sT[(c4 + 1) * 8 + tx], y);
            y = fmaf(l4.z, sT[(c4 + 2) * 8 + tx], y);
            y = fmaf(l4.w, sT[(c4 + 3) * 8 + tx], y);
          }
          ym[(size_t)(j0 + r) * m + tx] = y;
        }
      }
    }
  }

  // ---- X = P L_JJ^{-T} for the rows below the diagonal block -------------
  float x[RI][4];
#pragma unroll
  for (int i = 0; i < RI; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) x[i][j] = 0.f;
  tile_mma_inv<RI, TY>(x, Pm, Li, ty, tx);
#pragma unroll
  for (int i = 0; i < RI; ++i) {
    const int r = rg + ty + TY * i;
    if (r >= K || (first && i < S::RMIN)) continue;  // diagonal rows hold L_JJ already
    float* wr = Wm + (size_t)r * K + j0;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (tx + 8 * j < bw) wr[tx + 8 * j] = x[i][j];
  }
  __syncthreads();  // W writes and the P / inverse reads are done before the next group
}

// Inverse of diagonal block J, rebuilt in shared memory from the slot in one
// pass: the strict lower triangle was stored transposed in the block's strict
// upper triangle; the diagonal is 1 / L_jj, recomputed exactly as it was
// formed.
template <int NT>
__device__ __forceinline__ void load_block_inverse(const float* Wm, int K, int j0, int bw, float* Li) {
  __syncthreads();  // the previous block's readers of Li are done
  for (int e = threadIdx.x; e < 1024; e += NT) {
    const int r = e >> 5, c = e & 31;  // Li[r][c] sits at slot (j0 + c, j0 + r) when r > c
    float v;
    if (r >= bw || c >= bw) v = (r == c) ? 1.f : 0.f;
    else if (r > c) v = Wm[(size_t)(j0 + c) * K + j0 + r];
    else if (r == c) v = 1.f / Wm[(size_t)(j0 + r) * K + j0 + r];
    else v = 0.f;
    Li[inv_off(r, c)] = v;
  }
  __syncthreads();
}

}  // namespace

template <int NT>
__global__ void __launch_bounds__(NT, 512 / NT) posv_blocked2_kernel(const PosvParams p, int mcb) {
  using S = B2<NT>;
  constexpr int NW = S::NW;
  extern __shared__ __align__(16) float sm[];
  const int K = p.k;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* sInv = sm + S::OFF_INV;
  const size_t kk = (size_t)K * K;
  const bool vec = p.vec && (K & 3) == 0;
  const int nblk = (K + 31) / 32;
  // forward substitution fused into the factorisation when every right-hand
  // side fits one pass; y is kept in x (b_J is read before y_J is written
  // over it, so x may alias b)
  const bool fwd = p.m >= 1 && p.m <= MCB2 && p.m <= mcb;

  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x) {
    const float* A = p.A + mat * kk;
    float* Wm = p.L ? p.L + mat * kk : p.ws + (size_t)blockIdx.x * kk;
    float lgacc = 0.f;
    for (int J = 0; J < nblk; ++J) {
      const int j0 = 32 * J;
      for (int rg = j0; rg < K;) {
        const int nb = (K - rg + S::TY - 1) / S::TY;  // TY-row blocks left in the panel
        if (nb >= 8) {
          panel_group<NT, 8>(p, A, Wm, K, j0, rg, sm, vec, fwd, mat, lgacc);
          rg += 8 * S::TY;
        } else if (nb >= 4) {
          panel_group<NT, 4>(p, A, Wm, K, j0, rg, sm, vec, fwd, mat, lgacc);
          rg += 4 * S::TY;
        } else {
          if constexpr (S::RMIN == 1) {
            if (nb == 1) {
              panel_group<NT, 1>(p, A, Wm, K, j0, rg, sm, vec, fwd, mat, lgacc);
              rg += S::TY;
              continue;
            }
          }
          panel_group<NT, 2>(p, A, Wm, K, j0, rg, sm, vec, fwd, mat, lgacc);
          rg += 2 * S::TY;
        }
      }
    }
    if (warp == 0 && p.logdet) {
      const float lg = warp_sum(lgacc);
      if (lane == 0) p.logdet[mat] = 2.f * lg;
    }

    // ---- substitutions with the panel inverses ---------------------------
    if (p.m > 0) {
      float* sY = sm + S::OFF_A;   // mcb x K, column-major per right-hand side
      float* sRed = sm + S::OFF_B; // NW x 8 x 32 reduction
      const float* bm = p.b + (size_t)mat * K * p.m;
      float* xm = p.x + (size_t)mat * K * p.m;
      for (int q0 = 0; q0 < p.m; q0 += mcb) {
        const int mc = min(mcb, p.m - q0);
        __syncthreads();
        const float* src = fwd ? xm : bm;  // fused: x holds y already
        for (int e = tid; e < K * mc; e += NT) {
          const int r = e / mc, q = e - r * mc;
          sY[q * K + r] = src[(size_t)r * p.m + q0 + q];
        }
        __syncthreads();
        // forward: y_J = Linv_J (b_J - L[J, :j0] y[:j0])
        for (int J = 0; J < (fwd ? 0 : nblk); ++J) {
          const int j0 = 32 * J, bw = min(32, K - j0);
          if (j0 > 0) {
            for (int ii = warp; ii < bw; ii += NW) {
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
          }
          load_block_inverse<NT>(Wm, K, j0, bw, sInv);  // syncs before and after its writes
          for (int q = warp; q < mc; q += NW) {
            const float* t = sY + q * K + j0;
            float y = 0.f;
#pragma unroll
            for (int q4 = 0; q4 < 32; q4 += 4) {
              const float4 l4 = *reinterpret_cast<const float4*>(sInv + inv_off(lane, q4));
              const float t0 = (q4 < bw) ? t[q4] : 0.f, t1 = (q4 + 1 < bw) ? t[q4 + 1] : 0.f;
              const float t2 = (q4 + 2 < bw) ? t[q4 + 2] : 0.f, t3 = (q4 + 3 < bw) ? t[q4 + 3] : 0.f;
              y = fmaf(l4.x, t0, y);
              y = fmaf(l4.y, t1, y);
              y = fmaf(l4.z, t2, y);
              y = fmaf(l4.w, t3, y);
            }
            __syncwarp();
            if (lane < bw) sY[q * K + j0 + lane] = y;
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
#pragma unroll 8
            for (int r = j0 + 32 + warp; r < K; r += NW) {  // unrolled: 8 row loads in flight per warp
              const float l = Wm[(size_t)r * K + j0 + lane];
#pragma unroll
              for (int q = 0; q < MCB2; ++q)
                if (q < mc) s[q] = fmaf(l, sY[q * K + r], s[q]);
            }
#pragma unroll
            for (int q = 0; q < MCB2; ++q) sRed[(warp * MCB2 + q) * 32 + lane] = s[q];
            __syncthreads();
            for (int q = warp; q < mc; q += NW) {
              float t = 0.f;
#pragma unroll
              for (int w = 0; w < NW; ++w) t += sRed[(w * MCB2 + q) * 32 + lane];
              sY[q * K + j0 + lane] -= t;
            }
          }
          load_block_inverse<NT>(Wm, K, j0, bw, sInv);
          for (int q = warp; q < mc; q += NW) {
            const float* t = sY + q * K + j0;
            float xv = 0.f;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const float tq = (c < bw) ? t[c] : 0.f;
              xv = fmaf(sInv[inv_off(c, lane)], tq, xv);
            }
            __syncwarp();
            if (lane < bw) sY[q * K + j0 + lane] = xv;
          }
          __syncthreads();
        }
        for (int e = tid; e < K * mc; e += NT) {
          const int r = e / mc, q = e - r * mc;
          xm[(size_t)r * p.m + q0 + q] = sY[q * K + r];
        }
      }
      if (p.L) {  // the inverses lived in L's strict upper diagonal blocks
        __syncthreads();
        for (int J = 0; J < nblk; ++J) {
          const int j0 = 32 * J, bw = min(32, K - j0);
          for (int e = tid; e < 1024; e += NT) {
            const int r = e >> 5, c = e & 31;
            if (c > r && c < bw) Wm[(size_t)(j0 + r) * K + j0 + c] = 0.f;
          }
        }
      }
    }
    __syncthreads();
  }
}

// CTA size of the blocked tier (128: four CTAs per SM; 256: two).
constexpr int kBlockedNT = 128;

int blocked2_mcb(int k) {
  int mcb = (2 * B2<kBlockedNT>::A_FL) / (k > 0 ? k : 1);
  return mcb > MCB2 ? MCB2 : mcb;
}

size_t blocked2_smem_bytes(int k) {
  (void)k;
  return (size_t)B2<kBlockedNT>::SMEM * sizeof(float);
}

bool blocked2_fits(int k) { return blocked2_mcb(k) >= 1; }

int blocked2_ctas_per_sm() { return 512 / kBlockedNT; }

cudaError_t launch_posv_blocked2(const PosvParams& p, int grid, cudaStream_t s) {
  static int cache[64];
  int occ = 0;
  auto kern = posv_blocked2_kernel<kBlockedNT>;
  cudaError_t e = kernel_occupancy(kern, kBlockedNT, blocked2_smem_bytes(p.k), cache, &occ);
  if (e != cudaSuccess) return e;
  kern<<<grid, kBlockedNT, blocked2_smem_bytes(p.k), s>>>(p, blocked2_mcb(p.k));
  return cudaGetLastError();
}

}  // namespace b2c
