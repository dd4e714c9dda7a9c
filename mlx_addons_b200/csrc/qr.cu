// Batched Householder QR of square matrices, Q formed explicitly.
//
// Replaces the reference's qr (src/mlx_addons/linalg/_metal_kernels.py:
// 641-694): a single-thread Metal kernel for k < 12 (_QR_SRC :319-381), a
// threadgroup kernel for 12 <= k <= 63 (_QR_TG_SRC :385-473) and CPU LAPACK
// above (:685-688). The reflector of column j is generated as in the Metal
// kernels (:336-352): norm = sqrt(max(sum_{i>=j} r_ij^2, 1e-30)),
// v = (r_jj + s * norm, r_{j+1,j}, ...) with s = +1 for r_jj >= 0 else -1,
// tau = 2 / v.v (0 when v.v <= 1e-30); Q <- Q (I - tau v v^T) and
// R <- (I - tau v v^T) R right of column j, products grouped as
// (tau * dot) * v_i and (tau * v_i) * dot (:354-366); then r_jj = -s * norm
// and zeros below. Above k = 63, where the reference runs LAPACK, a column
// whose sub-diagonal part is exactly zero is left alone (LAPACK's reflector
// generator returns tau = 0 and keeps r_jj), the last column always; for
// every other column both generate the same reflector. Sums are fused into
// FMAs and the norm is reduced in a different order: results agree with the
// reference to rounding.
//
//  * k <= 32: one warp per matrix; lane l holds column l of R and row l of Q
//    in registers. The reflector (column j, in lane j) is broadcast by
//    shuffles; every lane then forms norm, tau and v itself, its own R-column
//    dot product and update, and its own Q-row dot product and update.
//  * 33 <= k <= 64: one warp per matrix, R and then Q in registers, two
//    columns per lane (qr_warp64_kernel, below).
//  * k > 64: one CTA per matrix with R and Q^T in shared memory (row stride
//    k | 1: a thread per R column or per Q row reads conflict-free) up to
//    k = 160, in a per-CTA scratch slot above; warp 0 reduces the norms.
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

constexpr int QW = 4;     // warps per CTA, warp tier
constexpr int QT = 256;   // threads per CTA, CTA tier
constexpr int kQrSmemMaxK = 160;
constexpr int kQrLapackAbove = 63;  // _metal_kernels.py:383, QR_SHARED_K_MAX

__global__ void __launch_bounds__(QW * 32) qr_warp_kernel(const QrParams p) {
  __shared__ float st[QW][32 * 33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = p.k;
  float* S = st[warp];
  const int64_t nw = (int64_t)gridDim.x * QW;
  for (int64_t mat = (int64_t)blockIdx.x * QW + warp; mat < p.batch; mat += nw) {
    const float* A = p.A + mat * (size_t)n * n;
    float r[32], q[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      r[i] = (lane < n && i < n) ? A[(size_t)i * n + lane] : 0.f;
      q[i] = (i == lane) ? 1.f : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j >= n) break;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = (i >= j && i < n) ? __shfl_sync(kFull, r[i], j) : 0.f;
      float sigma = 0.f;
#pragma unroll
      for (int i = j; i < 32; ++i) sigma = fmaf(v[i], v[i], sigma);
      const float norm = sqrtf(fmaxf(sigma, 1e-30f));
      const float sgn = (v[j] >= 0.f) ? 1.f : -1.f;
      const float vh = fmaf(sgn, norm, v[j]);
      float vtv = vh * vh;
#pragma unroll
      for (int i = j + 1; i < 32; ++i) vtv = fmaf(v[i], v[i], vtv);
      const float tau = (vtv > 1e-30f) ? (2.f / vtv) : 0.f;
      v[j] = vh;
      if (lane > j) {  // R column `lane` (zero columns beyond n stay zero)
        float dot = 0.f;
#pragma unroll
        for (int i = j; i < 32; ++i) dot = fmaf(v[i], r[i], dot);
#pragma unroll
        for (int i = j; i < 32; ++i) r[i] = fmaf(-(tau * v[i]), dot, r[i]);
      }
      {  // Q row `lane`
        float dot = 0.f;
#pragma unroll
        for (int i = j; i < 32; ++i) dot = fmaf(q[i], v[i], dot);
        const float td = tau * dot;
#pragma unroll
        for (int i = j; i < 32; ++i) q[i] = fmaf(-td, v[i], q[i]);
      }
      if (lane == j) {
        r[j] = -sgn * norm;
#pragma unroll
        for (int i = j + 1; i < 32; ++i) r[i] = 0.f;
      }
    }
    float* Rm = p.R + mat * (size_t)n * n;
    float* Qm = p.Q + mat * (size_t)n * n;
    if (lane < n) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < n) Rm[(size_t)i * n + lane] = r[i];
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 32; ++i) S[lane * 33 + i] = q[i];
    __syncwarp();
    for (int e = lane; e < n * n; e += 32) {
      const int row = e / n, c = e - row * n;
      Qm[e] = S[row * 33 + c];
    }
    __syncwarp();
  }
}

template <bool SMEM>
__global__ void __launch_bounds__(QT) qr_cta_kernel(const QrParams p) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float sInfo[4];
  const int n = p.k, LD = n | 1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool lapack_tail = n > kQrLapackAbove;
  float* R = SMEM ? sm : p.ws + (size_t)blockIdx.x * 2 * n * LD;
  float* QTm = R + (size_t)n * LD;  // QTm[i][row] = Q[row][i]
  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x) {
    const float* A = p.A + mat * (size_t)n * n;
    __syncthreads();
    for (int e = tid; e < n * n; e += QT) {
      const int i = e / n, c = e - i * n;
      R[(size_t)i * LD + c] = A[e];
      QTm[(size_t)i * LD + c] = (i == c) ? 1.f : 0.f;
    }
    __syncthreads();
    for (int j = 0; j < n; ++j) {
      if (warp == 0) {
        float s = 0.f;
        bool nz = false;
        for (int i = j + 1 + lane; i < n; i += 32) {
          const float t = R[(size_t)i * LD + j];
          s = fmaf(t, t, s);
          nz |= (t != 0.f);
        }
        s = warp_sum(s);
        nz = __any_sync(kFull, nz);
        if (lane == 0) {
          const float x = R[(size_t)j * LD + j];
          const float norm = sqrtf(fmaxf(fmaf(x, x, s), 1e-30f));
          const float sgn = (x >= 0.f) ? 1.f : -1.f;
          const float vh = fmaf(sgn, norm, x);
          const float vtv = fmaf(vh, vh, s);
          sInfo[0] = (vtv > 1e-30f) ? (2.f / vtv) : 0.f;
          sInfo[1] = vh;
          sInfo[2] = -sgn * norm;
          sInfo[3] = (lapack_tail && !nz) ? 1.f : 0.f;
        }
      }
      __syncthreads();
      if (sInfo[3] != 0.f) {  // LAPACK: nothing to annihilate, column kept
        __syncthreads();      // sInfo is rewritten by the next column
        continue;
      }
      const float tau = sInfo[0], vh = sInfo[1];
      for (int w = tid; w < 2 * n; w += QT) {
        if (w < n) {
          const int col = w;
          if (col > j) {
            float dot = vh * R[(size_t)j * LD + col];
            for (int i = j + 1; i < n; ++i) dot = fmaf(R[(size_t)i * LD + j], R[(size_t)i * LD + col], dot);
            R[(size_t)j * LD + col] = fmaf(-(tau * vh), dot, R[(size_t)j * LD + col]);
            for (int i = j + 1; i < n; ++i)
              R[(size_t)i * LD + col] = fmaf(-(tau * R[(size_t)i * LD + j]), dot, R[(size_t)i * LD + col]);
          }
        } else {
          const int row = w - n;
          float dot = QTm[(size_t)j * LD + row] * vh;
          for (int i = j + 1; i < n; ++i) dot = fmaf(QTm[(size_t)i * LD + row], R[(size_t)i * LD + j], dot);
          const float td = tau * dot;
          QTm[(size_t)j * LD + row] = fmaf(-td, vh, QTm[(size_t)j * LD + row]);
          for (int i = j + 1; i < n; ++i)
            QTm[(size_t)i * LD + row] = fmaf(-td, R[(size_t)i * LD + j], QTm[(size_t)i * LD + row]);
        }
      }
      __syncthreads();
      const float rjj = sInfo[2];
      for (int i = j + tid; i < n; i += QT) R[(size_t)i * LD + j] = (i == j) ? rjj : 0.f;
      __syncthreads();
    }
    float* Rm = p.R + mat * (size_t)n * n;
    float* Qm = p.Q + mat * (size_t)n * n;
    for (int e = tid; e < n * n; e += QT) {
      const int row = e / n, c = e - row * n;
      Rm[e] = R[(size_t)row * LD + c];
      Qm[e] = QTm[(size_t)c * LD + row];
    }
  }
}

static size_t qr_cta_smem(int k) { return 2 * (size_t)k * (size_t)(k | 1) * sizeof(float); }

// ---- 33 <= k <= 64: one warp per matrix, registers ------------------------
// Lane l owns columns l and 32 + l, rows packed in pairs (u64 of two floats):
// R in phase 1, then Q in phase 2, 2 k registers either way (KP = k padded
// to 40 / 48 / 56 / 64 with an identity block, which no reflector touches).
// Phase 1, column j: its owner (lane j % 32) publishes the column to shared
// memory; every lane reduces the norm (warp sum) and forms s * norm, v_j =
// r_jj + s * norm and tau itself; the owner writes v_j over r_jj (and a 0
// above it when j is odd), so that the column IS the reflector v, pair for
// pair (the rows above it read 0), and records the final r_jj (-s * norm,
// or r_jj itself when LAPACK's zero-tail rule skips the column). Each lane then takes its two columns' dot products with v and
// updates them with packed FMAs (fma.rn.f32x2, two consecutive rows at a
// time); columns at or left of j are left alone, and the reflector stays in
// shared memory for phase 2. Phase 2 forms Q = H_0 H_1 ... H_{k-1} by
// backward accumulation (Q <- H_j Q for j = k-1 .. 0, the same column-wise
// dot and update), which touches only rows >= j at step j. Rounding differs
// from the reference's forward accumulation and grouping; results agree to
// rounding, and the LAPACK zero-tail rule above k = 63 (tau = 0, r_jj kept)
// holds exactly.
// warps per CTA, one CTA per SM: 12 at up to 168 registers a thread; 8 for
// KP = 64, whose 128-register state spills at 168 (measured on B200: k = 64,
// 0.56 ms with 8 warps, 0.78 ms with 12; k = 56, 0.40 ms with 12, 0.46 with 8)
template <int KP>
struct QrWarps {
  static constexpr int N = KP >= 64 ? 8 : 12;
};

typedef unsigned long long qu64;
__device__ __forceinline__ qu64 qpk(float lo, float hi) {
  qu64 r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float qlo(qu64 v) {
  float lo, hi;
  asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo;
}
__device__ __forceinline__ float qhi(qu64 v) {
  float lo, hi;
  asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return hi;
}
__device__ __forceinline__ qu64 qfma2(qu64 a, qu64 b, qu64 c) {
  qu64 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ qu64 qld64(const float* p) {
  qu64 x;
  asm volatile("ld.shared.b64 %0, [%1];" : "=l"(x) : "r"(smem_u32(p)));
  return x;
}
__device__ __forceinline__ void qld128(const float* p, qu64& x, qu64& y) {
  asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void qst64(float* p, qu64 x) {
  asm volatile("st.shared.b64 [%0], %1;" ::"r"(smem_u32(p)), "l"(x) : "memory");
}
template <int NP>
__device__ __forceinline__ float qget(const qu64 (&a)[NP], int i) {
  return (i & 1) ? qhi(a[i >> 1]) : qlo(a[i >> 1]);
}
template <int NP>
__device__ __forceinline__ void qset(qu64 (&a)[NP], int i, float v) {
  a[i >> 1] = (i & 1) ? qpk(qlo(a[i >> 1]), v) : qpk(v, qhi(a[i >> 1]));
}

// The passes over pairs Q0 .. NP-1 of the two register columns and of v
// (shared memory, 16-byte loads of two pairs; Q0 is a multiple of 4). Steps
// go in blocks of 8 columns that share Q0 = 4 * block: one copy of the code
// per block and pass (full unrolling over the steps overflowed the
// instruction cache), and the few pairs above a step's column read zeros.
template <int NP, int Q0>
__device__ __forceinline__ void qdot(const qu64 (&x0)[NP], const qu64 (&x1)[NP], const float* v, qu64& d0, qu64& d1) {
  qu64 e0 = 0ull, e1 = 0ull;
#pragma unroll
  for (int q = Q0; q < NP; q += 2) {
    qu64 va, vb;
    qld128(v + 2 * q, va, vb);
    d0 = qfma2(x0[q], va, d0);
    d1 = qfma2(x1[q], va, d1);
    if (q + 1 < NP) {
      e0 = qfma2(x0[q + 1], vb, e0);
      e1 = qfma2(x1[q + 1], vb, e1);
    }
  }
  d0 = qpk(qlo(d0) + qlo(e0), qhi(d0) + qhi(e0));
  d1 = qpk(qlo(d1) + qlo(e1), qhi(d1) + qhi(e1));
}

template <int NP, int Q0>
__device__ __forceinline__ void qaxpy(qu64 (&x0)[NP], qu64 (&x1)[NP], const float* v, qu64 n0, qu64 n1) {
#pragma unroll
  for (int q = Q0; q < NP; q += 2) {
    qu64 va, vb;
    qld128(v + 2 * q, va, vb);
    x0[q] = qfma2(n0, va, x0[q]);
    x1[q] = qfma2(n1, va, x1[q]);
    if (q + 1 < NP) {
      x0[q + 1] = qfma2(n0, vb, x0[q + 1]);
      x1[q + 1] = qfma2(n1, vb, x1[q + 1]);
    }
  }
}

// rows 2 Q0 .. KP-1 of column x0 or x1 (by `hi`) to v, rows above j as zeros
template <int NP, int Q0>
__device__ __forceinline__ void qpublish(const qu64 (&x0)[NP], const qu64 (&x1)[NP], bool hi, float* v, int j) {
#pragma unroll
  for (int q = Q0; q < NP; ++q) {
    qu64 x = hi ? x1[q] : x0[q];
    if (q < Q0 + 4) x = qpk(2 * q >= j ? qlo(x) : 0.f, 2 * q + 1 >= j ? qhi(x) : 0.f);
    qst64(v + 2 * q, x);
  }
}

template <int KP>
struct QrW64 {
  static constexpr int NP = KP / 2;
  static constexpr int NB = KP / 8;  // blocks of 8 columns
  // reflectors V[j][i]; tau; the final r_jj
  static constexpr int WARP_FLOATS = KP * KP + 2 * KP;
};

// Phase 1 (R) for the columns of block B and the blocks after it.
template <int KP, int B>
struct QrPhase1 {
  static __device__ __forceinline__ void run(qu64 (&r0)[KP / 2], qu64 (&r1)[KP / 2], float* V, float* tu, float* dg,
                                             int n, bool lapack, int lane) {
    constexpr int NP = KP / 2, Q0 = 4 * B, J0 = 8 * B;
    if (J0 >= n) return;
    const int j1 = min(J0 + 8, n);
    for (int j = J0; j < j1; ++j) {
      const int o = j & 31;
      float* Vj = V + j * KP;
      if (lane == o) qpublish<NP, Q0>(r0, r1, j >= 32, Vj, j);
      __syncwarp();
      const float x = Vj[j];
      float t = 0.f;
      bool nz = false;
      if (j + 1 + lane < KP) {
        const float v = Vj[j + 1 + lane];
        t = v * v;
        nz = v != 0.f;
      }
      if (j + 33 + lane < KP) {
        const float v = Vj[j + 33 + lane];
        t = fmaf(v, v, t);
        nz = nz || v != 0.f;
      }
      const float tail = warp_sum(t);
      const bool skip = lapack && !__any_sync(kFull, nz);  // LAPACK: nothing below the diagonal
      const float norm = sqrtf(fmaxf(fmaf(x, x, tail), 1e-30f));
      const float snrm = (x >= 0.f) ? norm : -norm;
      const float vh = x + snrm;
      const float vtv = fmaf(vh, vh, tail);
      const float tau = skip ? 0.f : ((vtv > 1e-30f) ? 2.f / vtv : 0.f);
      __syncwarp();  // every lane has read x before the owner writes v_j over it
      if (lane == o) {
        Vj[j] = vh;
        tu[j] = tau;
        dg[j] = skip ? x : -snrm;
      }
      __syncwarp();
      if (!skip) {
        qu64 d0 = 0ull, d1 = 0ull;
        qdot<NP, Q0>(r0, r1, Vj, d0, d1);
        // columns at or left of j keep their values (left of j they hold reflectors)
        const float f0 = (lane > j) ? tau * (qlo(d0) + qhi(d0)) : 0.f;
        const float f1 = (32 + lane > j) ? tau * (qlo(d1) + qhi(d1)) : 0.f;
        qaxpy<NP, Q0>(r0, r1, Vj, qpk(-f0, -f0), qpk(-f1, -f1));
      }
    }
    QrPhase1<KP, B + 1>::run(r0, r1, V, tu, dg, n, lapack, lane);
  }
};
template <int KP>
struct QrPhase1<KP, KP / 8> {
  static __device__ __forceinline__ void run(qu64 (&)[KP / 2], qu64 (&)[KP / 2], float*, float*, float*, int, bool,
                                             int) {}
};

// Phase 2 (Q <- H_j Q) for the columns of block B, last to first, then the blocks before it.
template <int KP, int B>
struct QrPhase2 {
  static __device__ __forceinline__ void run(qu64 (&q0)[KP / 2], qu64 (&q1)[KP / 2], const float* V, const float* tu,
                                             int n) {
    constexpr int NP = KP / 2, Q0 = 4 * B, J0 = 8 * B;
    for (int j = min(J0 + 8, n) - 1; j >= J0; --j) {
      const float tau = tu[j];
      if (tau == 0.f) continue;
      const float* Vj = V + j * KP;
      qu64 d0 = 0ull, d1 = 0ull;
      qdot<NP, Q0>(q0, q1, Vj, d0, d1);
      const float f0 = tau * (qlo(d0) + qhi(d0)), f1 = tau * (qlo(d1) + qhi(d1));
      qaxpy<NP, Q0>(q0, q1, Vj, qpk(-f0, -f0), qpk(-f1, -f1));
    }
    QrPhase2<KP, B - 1>::run(q0, q1, V, tu, n);
  }
};
template <int KP>
struct QrPhase2<KP, -1> {
  static __device__ __forceinline__ void run(qu64 (&)[KP / 2], qu64 (&)[KP / 2], const float*, const float*, int) {}
};

template <int KP>
__global__ void __launch_bounds__(QrWarps<KP>::N * 32, 1) qr_warp64_kernel(const QrParams p) {
  constexpr int QW64 = QrWarps<KP>::N;
  using W = QrW64<KP>;
  constexpr int NP = W::NP;
  extern __shared__ __align__(16) float smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* V = smem + warp * W::WARP_FLOATS;
  float* tu = V + KP * KP;
  float* dg = tu + KP;
  const int n = p.k;
  const bool lapack = n > kQrLapackAbove;
  const int c0 = lane, c1 = 32 + lane;
  const int64_t nw = (int64_t)gridDim.x * QW64;
  for (int64_t mat = (int64_t)blockIdx.x * QW64 + warp; mat < p.batch; mat += nw) {
    const float* A = p.A + mat * (size_t)n * n;
    qu64 r0[NP], r1[NP];
#pragma unroll
    for (int q = 0; q < NP; ++q) {
      const int i0 = 2 * q, i1 = 2 * q + 1;
      const float a00 = (i0 < n && c0 < n) ? A[(size_t)i0 * n + c0] : (i0 == c0 ? 1.f : 0.f);
      const float a10 = (i1 < n && c0 < n) ? A[(size_t)i1 * n + c0] : (i1 == c0 ? 1.f : 0.f);
      const float a01 = (i0 < n && c1 < n) ? A[(size_t)i0 * n + c1] : (i0 == c1 ? 1.f : 0.f);
      const float a11 = (i1 < n && c1 < n) ? A[(size_t)i1 * n + c1] : (i1 == c1 ? 1.f : 0.f);
      r0[q] = qpk(a00, a10);
      r1[q] = qpk(a01, a11);
    }
    QrPhase1<KP, 0>::run(r0, r1, V, tu, dg, n, lapack, lane);
    __syncwarp();
    // R: strict upper triangle from the registers, r_jj from dg, zeros below
    float* Rm = p.R + mat * (size_t)n * n;
    const float g0 = (c0 < n) ? dg[c0] : 0.f, g1 = (c1 < n) ? dg[c1 < KP ? c1 : 0] : 0.f;
#pragma unroll
    for (int i = 0; i < KP; ++i) {
      if (i < n) {
        if (c0 < n) Rm[(size_t)i * n + c0] = (i < c0) ? qget(r0, i) : (i == c0 ? g0 : 0.f);
        if (c1 < n) Rm[(size_t)i * n + c1] = (i < c1) ? qget(r1, i) : (i == c1 ? g1 : 0.f);
      }
    }
    // Q = H_0 ... H_{n-1}: Q <- H_j Q from the identity
#pragma unroll
    for (int q = 0; q < NP; ++q) {
      r0[q] = qpk(2 * q == c0 ? 1.f : 0.f, 2 * q + 1 == c0 ? 1.f : 0.f);
      r1[q] = qpk(2 * q == c1 ? 1.f : 0.f, 2 * q + 1 == c1 ? 1.f : 0.f);
    }
    QrPhase2<KP, W::NB - 1>::run(r0, r1, V, tu, n);
    float* Qm = p.Q + mat * (size_t)n * n;
#pragma unroll
    for (int i = 0; i < KP; ++i) {
      if (i < n) {
        if (c0 < n) Qm[(size_t)i * n + c0] = qget(r0, i);
        if (c1 < n) Qm[(size_t)i * n + c1] = qget(r1, i);
      }
    }
    __syncwarp();
  }
}

template <int KP>
static cudaError_t launch_qr_w64(const QrParams& p, int sm_count, cudaStream_t s) {
  constexpr int QW64 = QrWarps<KP>::N;
  const size_t smem = (size_t)QW64 * QrW64<KP>::WARP_FLOATS * sizeof(float);
  static int cache[64];
  int occ = 0;
  cudaError_t e = kernel_occupancy(qr_warp64_kernel<KP>, QW64 * 32, smem, cache, &occ);
  if (e != cudaSuccess) return e;
  const int64_t need = (p.batch + QW64 - 1) / QW64;
  const int64_t cap = (int64_t)sm_count * occ;
  qr_warp64_kernel<KP><<<(int)(need < cap ? need : cap), QW64 * 32, smem, s>>>(p);
  return cudaGetLastError();
}

int qr_grid(int64_t batch, int k, int sm_count) {
  (void)k;
  const int64_t cap = (int64_t)sm_count * 2;
  return (int)(batch < cap ? batch : cap);
}

size_t qr_ws_floats(int64_t batch, int k, int sm_count) {
  if (k <= kQrSmemMaxK || batch <= 0) return 0;
  return (size_t)qr_grid(batch, k, sm_count) * 2 * (size_t)k * (size_t)(k | 1);
}

cudaError_t launch_qr(const QrParams& p, int sm_count, cudaStream_t s) {
  if (p.k <= 32) {
    static int cache[64];
    int occ = 0;
    cudaError_t e = kernel_occupancy(qr_warp_kernel, QW * 32, 0, cache, &occ);
    if (e != cudaSuccess) return e;
    const int64_t need = (p.batch + QW - 1) / QW;
    const int64_t cap = (int64_t)sm_count * occ;
    qr_warp_kernel<<<(int)(need < cap ? need : cap), QW * 32, 0, s>>>(p);
    return cudaGetLastError();
  }
  if (p.k <= 40) return launch_qr_w64<40>(p, sm_count, s);
  if (p.k <= 48) return launch_qr_w64<48>(p, sm_count, s);
  if (p.k <= 56) return launch_qr_w64<56>(p, sm_count, s);
  if (p.k <= 64) return launch_qr_w64<64>(p, sm_count, s);
  if (p.k <= kQrSmemMaxK) {
    const size_t smem = qr_cta_smem(p.k);
    static int cache[64];
    int occ = 0;
    cudaError_t e = kernel_occupancy(qr_cta_kernel<true>, QT, smem, cache, &occ);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, qr_cta_kernel<true>, QT, smem);
    if (e != cudaSuccess) return e;
    if (occ < 1) occ = 1;
    const int64_t cap = (int64_t)sm_count * occ;
    qr_cta_kernel<true><<<(int)(p.batch < cap ? p.batch : cap), QT, smem, s>>>(p);
    return cudaGetLastError();
  }
  qr_cta_kernel<false><<<qr_grid(p.batch, p.k, sm_count), QT, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace b2c
