// Task-graph form of the shared-memory tier: batched Cholesky factor + solve
// + logdet for 65 <= k <= 256, m <= 8, A in device memory with k % 4 == 0.
//
// Same contract as the other tiers and as the reference's blocked algorithm
// (src/mlx_addons/linalg/_blocked.py:34-217, the per-block kernels at
// src/mlx_addons/linalg/_metal_kernels.py:147-206): lower triangle of A
// read, pivots clamped to sqrt(1e-12), x = A^{-1} b by the two substitutions,
// logdet = 2 sum log L_jj, L written with its upper triangle zeroed when
// requested.
//
// One CTA owns one matrix at a time (a persistent grid walks the batch).
// The lower triangle of A arrives in shared memory as 32 x 32 blocks, one
// TMA tile load per block (3-D tensor map over (batch, row, column), 128-byte
// swizzle, no multicast), each completing its own mbarrier, so work on the
// first blocks starts while the rest are in flight. The factorisation and
// both substitutions are a task graph over those blocks:
//   P(J)     factor diagonal block J in registers (one row per lane, the
//            next pivot shuffled from its owner one step ahead); L_JJ goes
//            back to the lower triangle, L_JJ^T to the upper one, so that
//            rows of the block serve both substitutions as broadcasts;
//   T(I,J)   L_IJ = A_IJ L_JJ^{-T} by substitution, one row per lane;
//   U(I,K,J) A_IK -= L_IJ L_KJ^T on one 16 x 32 half of block (I,K),
//            register-tiled 4 x 4 per lane;
//   F(J), B(I,J)        forward substitution of the right-hand sides;
//   S(I), G(J,I)        back substitution (z_J += L_IJ^T x_I, then
//                       x_J = L_JJ^{-T} (y_J - z_J)).
// Warps take tasks from a list in a fixed topological order (critical path
// first: T(J+1,J), U(J+1,J+1,J) and P(J+1) lead each panel) through a shared
// counter, and wait for their inputs on events: one mbarrier per (half
// block, panel) step and per substitution step, each completed once per
// matrix by the task that produces it; a waiting warp is suspended by the
// hardware until its event completes. Every input of a task precedes it in the list, so the earliest
// unfinished task always has its inputs ready and the graph cannot stall:
// the waits are bounded all the same (one second of %globaltimer); a wait
// that runs out marks the matrix and the CTA's later ones NaN, sets a device
// flag (b2c_take_device_fault) and ends the CTA after its loads have landed.
// Summation orders are fixed by the graph, so results do not depend on the
// schedule.
#include <cuda.h>  // CUtensorMap and its enums; the encoder comes from the runtime's driver entry point
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

__device__ unsigned int g_dag_fault;

namespace {

constexpr int GB = 32;           // block edge
constexpr int GBF = GB * GB;     // floats per block: 32 rows of 128 bytes
constexpr int GMAXNB = 8;        // k <= 256
constexpr int GMAXTASK = 320;    // 284 at 8 blocks a side

enum : uint32_t { TK_P = 0, TK_T = 1, TK_U = 2, TK_F = 3, TK_B = 4, TK_S = 5, TK_G = 6, TK_W = 7 };

// A task in 13 bits: type, block indices I, K, J (3 bits each), half h.
__host__ __device__ constexpr uint16_t tenc(int type, int I, int K, int J, int h) {
  return (uint16_t)(type | (I << 3) | (K << 6) | (J << 9) | (h << 12));
}
// The task list, built on the host for (blocks a side, rhs or not, warps)
// and passed by value, so a captured launch carries it.
struct DagTasks {
  int n;
  int inject;  // test only: CTA 0 waits on a phase that never completes, every wait limited to 1 ms
  uint16_t t[GMAXTASK];
};

__host__ __device__ constexpr int gtri(int n) { return n * (n + 1) / 2; }
__host__ __device__ constexpr int gblk(int I, int J) { return gtri(I) + J; }

// Float offset of element (r, c) of a block, and of the 16-byte chunk q of
// row r: rows of 128 bytes whose chunks are XOR-swizzled by the row (the
// layout TMA's 128-byte swizzle writes into a 1024-byte aligned block).
__host__ __device__ constexpr int swz(int r, int c) { return r * 32 + ((((c >> 2) ^ r) & 7) << 2) + (c & 3); }
__host__ __device__ constexpr int swq(int r, int q) { return r * 32 + (((q ^ r) & 7) << 2); }

// Task-graph events, each an mbarrier that one task arrives on once per
// matrix (so a waiter uses the matrix's phase parity):
//   ev_blk(I,K,h,J)  half h of block (I,K) has the update of panel J (J < K),
//                    or holds its final L (J == K);
//   ev_y(I,v)        v forward steps applied to right-hand-side block I
//                    (v = I + 1: y_I final);
//   ev_x(I)          x_I final;
//   ev_z(J,v)        v back-substitution terms added to z_J;
//   ev_w(J)          W_J = L_JJ^{-1} formed.
// The tile load of block b completes mbarrier gnev(nb) + b, after the events.
__host__ __device__ constexpr int gnev_blk(int nb) { return nb * (nb + 1) * (nb + 2) / 3; }
__host__ __device__ constexpr int gnev(int nb) { return gnev_blk(nb) + gtri(nb) + nb + nb * nb + nb; }
__host__ __device__ constexpr int ev_blk(int I, int K, int h, int J) {
  return I * (I + 1) * (I + 2) / 3 + K * (K + 1) + 2 * J + h;
}
__host__ __device__ constexpr int ev_y(int nb, int I, int v) { return gnev_blk(nb) + gtri(I) + v - 1; }
__host__ __device__ constexpr int ev_x(int nb, int I) { return gnev_blk(nb) + gtri(nb) + I; }
__host__ __device__ constexpr int ev_z(int nb, int J, int v) { return gnev_blk(nb) + gtri(nb) + nb + J * nb + v - 1; }
__host__ __device__ constexpr int ev_w(int nb, int J) { return gnev_blk(nb) + gtri(nb) + nb + nb * nb + J; }

// The mbarriers a task waits on (three slots) and arrives on (two slots),
// -1 for an unused slot; the kernel and the host's list scheduler both read
// the graph from here.
__host__ __device__ inline void task_waits(uint32_t e, int nb, int (&w)[3]) {
  const int type = e & 7, I = (e >> 3) & 7, K = (e >> 6) & 7, J = (e >> 9) & 7, h = (e >> 12) & 1;
  const int load = gnev(nb);
  w[0] = w[1] = w[2] = -1;
  switch (type) {
    case TK_P:  // every update of the diagonal block, or its tile load
      if (J > 0) {
        w[0] = ev_blk(J, J, 0, J - 1);
        w[1] = ev_blk(J, J, 1, J - 1);
      } else {
        w[0] = load + gblk(0, 0);
      }
      break;
    case TK_W: w[0] = ev_blk(J, J, 0, J); break;
    case TK_T:  // L_JJ, and every update of block (I,J) or its tile load
      w[0] = ev_blk(J, J, 0, J);
      if (J > 0) {
        w[1] = ev_blk(I, J, 0, J - 1);
        w[2] = ev_blk(I, J, 1, J - 1);
      } else {
        w[1] = load + gblk(I, 0);
      }
      break;
    case TK_U:  // L_IJ, L_KJ and the previous update of this half of (I,K)
      w[0] = ev_blk(I, J, 0, J);
      w[1] = ev_blk(K, J, 0, J);
      w[2] = J > 0 ? ev_blk(I, K, h, J - 1) : load + gblk(I, K);
      break;
    case TK_F:  // W_J and every forward update of block J
      w[0] = ev_w(nb, J);
      if (J > 0) w[1] = ev_y(nb, J, J);
      break;
    case TK_B:  // y_J, L_IJ and the previous forward update of block I
      w[0] = ev_y(nb, J, J + 1);
      w[1] = ev_blk(I, J, 0, J);
      if (J > 0) w[2] = ev_y(nb, I, J);
      break;
    case TK_S:  // y_I (formed after W_I) and every back-substitution term of block I
      w[0] = ev_y(nb, I, I + 1);
      if (I < nb - 1) w[1] = ev_z(nb, I, nb - 1 - I);
      break;
    default:  // TK_G: x_I and the previous term of block J
      w[0] = ev_x(nb, I);
      if (I < nb - 1) w[1] = ev_z(nb, J, nb - 1 - I);
      break;
  }
}
__host__ __device__ inline void task_fires(uint32_t e, int nb, int (&f)[2]) {
  const int type = e & 7, I = (e >> 3) & 7, K = (e >> 6) & 7, J = (e >> 9) & 7, h = (e >> 12) & 1;
  f[1] = -1;
  switch (type) {
    case TK_P: f[0] = ev_blk(J, J, 0, J); f[1] = ev_blk(J, J, 1, J); break;
    case TK_W: f[0] = ev_w(nb, J); break;
    case TK_T: f[0] = ev_blk(I, J, 0, J); f[1] = ev_blk(I, J, 1, J); break;
    case TK_U: f[0] = ev_blk(I, K, h, J); break;
    case TK_F: f[0] = ev_y(nb, J, J + 1); break;
    case TK_B: f[0] = ev_y(nb, I, J + 1); break;
    case TK_S: f[0] = ev_x(nb, I); break;
    default: f[0] = ev_z(nb, J, nb - I); break;
  }
}

// Shared-memory layout in floats after the 1024-byte aligned base.
struct GLay {
  int nbt, nev, w, y, z, dinv, ld, cb, bar, ctl, task, total;
};
__host__ __device__ inline GLay glay(int nb, int mc, int nw) {
  GLay L{};
  L.nbt = gtri(nb);
  L.w = L.nbt * GBF;                 // W_J = L_JJ^{-1}, one block per J (right-hand sides only)
  L.y = L.w + (mc > 0 ? nb * GBF : 0);  // right-hand sides, then y: [32 nb][mc]
  L.z = L.y + 32 * nb * mc;          // back-substitution sums, then x: [32 nb][mc]
  L.dinv = L.z + 32 * nb * mc;       // 1 / L_jj
  L.ld = L.dinv + 32 * nb;           // per diagonal block: sum log L_jj
  L.cb = L.ld + GMAXNB;              // per warp: column buffer of P (2 x 32)
  L.nev = gnev(nb);
  L.bar = L.cb + nw * 64;            // mbarriers (8 bytes): the events, then one per block's tile load
  L.ctl = L.bar + 2 * (L.nev + L.nbt);  // int: [0] task counter, [1] abort
  L.task = L.ctl + 4;                // uint16 task list
  L.total = L.task + GMAXTASK / 2;
  return L;
}
__host__ inline size_t gdag_smem_bytes(int nb, int mc, int nw) {
  return (size_t)glay(nb, mc, nw).total * sizeof(float) + 1024;  // + alignment slack
}

__device__ __forceinline__ uint64_t gnow() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
constexpr uint64_t kGWaitNs = 1000000000ull;  // one second

__device__ __forceinline__ void mbar_init1(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_done(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// try_wait that lets the hardware suspend the thread (up to 10 us) until the
// phase completes, so waiting warps take no issue slots.
__device__ __forceinline__ bool mbar_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(10000u)
      : "memory");
  return done != 0;
}
// Warp-uniform bounded wait for an mbarrier phase (a tile load or an event);
// false if the CTA gave up or one second passed (the caller then raises the
// abort flag).
__device__ __forceinline__ bool gwait(uint64_t* bar, uint32_t parity, const int* abort_flag,
                                      uint64_t limit = kGWaitNs) {
  if (__all_sync(kFull, mbar_done(bar, parity))) return true;
  const uint64_t t0 = gnow();
  for (;;) {
    if (__all_sync(kFull, mbar_sleep(bar, parity))) return true;
    if (__any_sync(kFull, *reinterpret_cast<const volatile int*>(abort_flag) != 0)) return false;
    if (__shfl_sync(kFull, (gnow() - t0 > limit) ? 1 : 0, 0)) return false;
  }
}
// One thread: bounded wait used on the abort path before the CTA exits.
__device__ __forceinline__ void gload_settle(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = gnow();
  while (!mbar_done(bar, parity) && gnow() - t0 < kGWaitNs) {
  }
}

// 32 x 32 tile (columns x, rows y) of matrix z through the tensor map; the
// load completes `bar`'s transaction count.
__device__ __forceinline__ void tma_tile(float* dst, const CUtensorMap* tm, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ float grsqrt(float x) {
  float r;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// a[c] -= v * src[c] for c >= C0, on a row held as packed pairs; the 16-byte
// chunk q of src is at src + off(q). Pairs whose both columns are >= C0 take
// one fma.rn.f32x2; a single column C0 (odd) takes a scalar FMA.
template <int C0>
__device__ __forceinline__ void axpy_chunk(u64 (&A2)[16], u64 nv2, float v, int q, u64 w0, u64 w1) {
  const int c = 4 * q;
  if (c >= C0) A2[2 * q] = ffma2(nv2, w0, A2[2 * q]);
  else if (c + 1 >= C0) setc(A2, c + 1, fmaf(-v, hi2(w0), getc(A2, c + 1)));
  if (c + 2 >= C0) A2[2 * q + 1] = ffma2(nv2, w1, A2[2 * q + 1]);
  else if (c + 3 >= C0) setc(A2, c + 3, fmaf(-v, hi2(w1), getc(A2, c + 3)));
}
template <int C0, typename Off>
__device__ __forceinline__ void row_axpy(u64 (&A2)[16], float v, const float* src, Off off) {
  const u64 nv2 = pk2(-v, -v);
#pragma unroll
  for (int q = C0 >> 2; q < 8; ++q) {
    u64 w0, w1;
    lds128(src + off(q), w0, w1);
    axpy_chunk<C0>(A2, nv2, v, q, w0, w1);
  }
}

__device__ __forceinline__ void load_row2(u64 (&A2)[16], const float* blk, int r) {
#pragma unroll
  for (int q = 0; q < 8; ++q) lds128(blk + swq(r, q), A2[2 * q], A2[2 * q + 1]);
}
__device__ __forceinline__ void store_row2(float* blk, int r, const u64 (&A2)[16]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) sts128(blk + swq(r, q), A2[2 * q], A2[2 * q + 1]);
}

// One column step of P (unrolled over j). Lane r's entries of columns >= r
// are dead (the diagonal lives in dg, the upper part is never written back)
// and are updated like the others, so no step needs a lane-dependent
// predicate; nothing flows from them into the lower triangle.
template <int J>
struct PotrfStep {
  __device__ __forceinline__ static void run(u64 (&A2)[16], float& dg, float& sc, float& r, float& dme, float& rme,
                                             float* cb, int lane) {
    const float d = sc * r;
    float v = getc(A2, J) * r;  // L[lane][J] for lanes below J
    if (lane == J) {
      v = d;
      dme = d;
      rme = r;
    }
    setc(A2, J, v);
    if constexpr (J < 31) {
      dg = fmaf(-v, v, dg);
      // the next pivot: row J+1's diagonal after this step, from its owner
      sc = fmaxf(__shfl_sync(kFull, dg, J + 1), kClamp);
      r = grsqrt(sc);
      const float w1 = __shfl_sync(kFull, v, J + 1);  // L[J+1][J]
      setc(A2, J + 1, fmaf(-v, w1, getc(A2, J + 1)));
      if constexpr (J < 30) {
        float* cbj = cb + (J & 1) * 32;
        cbj[lane] = v;
        __syncwarp();
        row_axpy<J + 2>(A2, v, cbj, [](int q) { return 4 * q; });
      }
      PotrfStep<J + 1>::run(A2, dg, sc, r, dme, rme, cb, lane);
    }
  }
};

// P(J): factor the diagonal block D (one row per lane; rows >= `rows` are
// padding and factor as identity). Writes L to the lower triangle, L^T to
// the upper, 1 / L_jj to dinv; returns log L_jj of this lane's row (0 for
// padding rows).
__device__ __noinline__ float task_potrf(float* D, float* dinv, float* cb, int rows, int lane) {
  u64 A2[16];
  load_row2(A2, D, lane);
  const bool pad = lane >= rows;
  float dg = pad ? 1.f : D[swz(lane, lane)];  // this row's diagonal, kept apart from A2
#pragma unroll
  for (int c = 0; c < 32; ++c) setc(A2, c, (pad || c >= lane) ? 0.f : getc(A2, c));
  float sc = fmaxf(__shfl_sync(kFull, dg, 0), kClamp);
  float r = grsqrt(sc);
  float dme = 1.f, rme = 1.f;
  PotrfStep<0>::run(A2, dg, sc, r, dme, rme, cb, lane);
  // row `lane` of L to the lower triangle (whole rows, the diagonal selected
  // in, dead entries above it), then, after the warp barrier, the same values
  // transposed over those dead entries; no lane-dependent branch
#pragma unroll
  for (int c = 0; c < 32; ++c) setc(A2, c, c == lane ? dme : getc(A2, c));
  store_row2(D, lane, A2);
  __syncwarp();
  const int lq = lane >> 2, lr = lane & 3;
#pragma unroll
  for (int c = 0; c < 31; ++c)
    if (c < lane) D[c * 32 + (((lq ^ c) & 7) << 2) + lr] = getc(A2, c);  // swz(c, lane)
  dinv[lane] = rme;
  return pad ? 0.f : logf(dme);
}

template <int PP>
struct TrsmStep {
  __device__ __forceinline__ static void run(u64 (&A2)[16], const float* D, const float* dinv) {
    const float xp = getc(A2, PP) * dinv[PP];
    setc(A2, PP, xp);
    if constexpr (PP < 31) {
      row_axpy<PP + 1>(A2, xp, D, [](int q) { return swq(PP, q); });
      TrsmStep<PP + 1>::run(A2, D, dinv);
    }
  }
};

// T(I,J): X <- X L_JJ^{-T}, one row of X per lane; D is the factored
// diagonal block (row pp's upper part holds L[c][pp], c > pp).
__device__ __forceinline__ void task_trsm(float* X, const float* D, const float* dinv, int lane) {
  u64 A2[16];
  load_row2(A2, X, lane);
  TrsmStep<0>::run(A2, D, dinv);
  store_row2(X, lane, A2);
}

// U: rows 16 h .. 16 h + 15 of C -= (same rows of Aop) Bop^T, as 3xTF32
// m16n8k8 products: four k-steps of 8 by four column tiles of 8 (two when
// `top` marks the upper half of a diagonal block, whose right half lies
// above the diagonal). Lane (g, t) = (lane / 4, lane % 4) holds the
// fragments: A rows g, g + 8, columns t, t + 4 of the k-step; B rows g of
// the column tile, columns t, t + 4; D rows g, g + 8, columns 2t, 2t + 1.
// Every fragment load reads 32 distinct floats from 32 banks.
__device__ __forceinline__ void task_update(float* C, const float* Aop, const float* Bop, int h, bool top, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const int ra = 16 * h + g;
  float acc[4][4];
#pragma unroll
  for (int n = 0; n < 4; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[n][i] = 0.f;
#pragma unroll
  for (int k0 = 0; k0 < 32; k0 += 8) {
    uint32_t ah[4], al[4];
    tf32_split(Aop[swz(ra, k0 + t)], ah[0], al[0]);
    tf32_split(Aop[swz(ra + 8, k0 + t)], ah[1], al[1]);
    tf32_split(Aop[swz(ra, k0 + t + 4)], ah[2], al[2]);
    tf32_split(Aop[swz(ra + 8, k0 + t + 4)], ah[3], al[3]);
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      if (top && n >= 2) continue;
      uint32_t bh0, bl0, bh1, bl1;
      tf32_split(Bop[swz(8 * n + g, k0 + t)], bh0, bl0);
      tf32_split(Bop[swz(8 * n + g, k0 + t + 4)], bh1, bl1);
      mma_tf32(acc[n], al, bh0, bh1);
      mma_tf32(acc[n], ah, bl0, bl1);
      mma_tf32(acc[n], ah, bh0, bh1);
    }
  }
#pragma unroll
  for (int n = 0; n < 4; ++n) {
    if (top && n >= 2) continue;
    float2* p0 = reinterpret_cast<float2*>(C + swz(ra, 8 * n + 2 * t));
    float2* p1 = reinterpret_cast<float2*>(C + swz(ra + 8, 8 * n + 2 * t));
    float2 c0 = *p0, c1 = *p1;
    c0.x -= acc[n][0];
    c0.y -= acc[n][1];
    c1.x -= acc[n][2];
    c1.y -= acc[n][3];
    *p0 = c0;
    *p1 = c1;
  }
}

// W(J): W = L_JJ^{-1} (lower triangular), one column per lane: row r of
// L w = e_lane for r = 0..31, the rows of L broadcast from D. Used by the
// substitutions of the right-hand sides only, so it stays off the
// factorisation's critical path.
__device__ __noinline__ void task_inv(float* Wb, const float* D, const float* dinv, int lane) {
  float w[32];
#pragma unroll
  for (int r = 0; r < 32; ++r) {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int q = 0; 4 * q < r; ++q) {
      const float4 l = *reinterpret_cast<const float4*>(D + swq(r, q));
      if (4 * q + 0 < r) s0 = fmaf(l.x, w[4 * q], s0);
      if (4 * q + 1 < r) s1 = fmaf(l.y, w[4 * q + 1], s1);
      if (4 * q + 2 < r) s2 = fmaf(l.z, w[4 * q + 2], s2);
      if (4 * q + 3 < r) s3 = fmaf(l.w, w[4 * q + 3], s3);
    }
    w[r] = ((r == lane ? 1.f : 0.f) - ((s0 + s1) + (s2 + s3))) * dinv[r];
  }
#pragma unroll
  for (int r = 0; r < 32; ++r) Wb[swz(r, lane)] = w[r];
}

// acc = op(A) B for a 32 x 32 block A (swizzled; transposed when TR) and a
// 32 x 8 right-hand-side block B read through bget(k, n), in 3xTF32
// m16n8k8 products: two row tiles by four k-steps. Lane (g, t) ends with
// rows 16 mt + g and 16 mt + g + 8, columns 2t and 2t + 1 of tile mt.
template <bool TR, typename BGet>
__device__ __forceinline__ void mma_32x8(float (&acc)[2][4], const float* A, BGet bget, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mt][i] = 0.f;
#pragma unroll
  for (int k0 = 0; k0 < 32; k0 += 8) {
    uint32_t bh0, bl0, bh1, bl1;
    tf32_split(bget(k0 + t, g), bh0, bl0);
    tf32_split(bget(k0 + t + 4, g), bh1, bl1);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int r = 16 * mt + g;
      uint32_t ah[4], al[4];
      tf32_split(TR ? A[swz(k0 + t, r)] : A[swz(r, k0 + t)], ah[0], al[0]);
      tf32_split(TR ? A[swz(k0 + t, r + 8)] : A[swz(r + 8, k0 + t)], ah[1], al[1]);
      tf32_split(TR ? A[swz(k0 + t + 4, r)] : A[swz(r, k0 + t + 4)], ah[2], al[2]);
      tf32_split(TR ? A[swz(k0 + t + 4, r + 8)] : A[swz(r + 8, k0 + t + 4)], ah[3], al[3]);
      mma_tf32(acc[mt], al, bh0, bh1);
      mma_tf32(acc[mt], ah, bl0, bl1);
      mma_tf32(acc[mt], ah, bh0, bh1);
    }
  }
}

// Row c of an MC-wide right-hand-side block as registers (16-byte loads when
// MC is a multiple of 4).
template <int MC>
__device__ __forceinline__ void rhs_row(float (&v)[MC], const float* Yr) {
  if constexpr (MC % 4 == 0) {
#pragma unroll
    for (int q = 0; q < MC; q += 4) {
      const float4 t = *reinterpret_cast<const float4*>(Yr + q);
      v[q] = t.x;
      v[q + 1] = t.y;
      v[q + 2] = t.z;
      v[q + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int q = 0; q < MC; ++q) v[q] = Yr[q];
  }
}

// F(J): y_J = W_J b_J (b_J after the forward updates from earlier blocks),
// one row per lane.
template <int MC>
__device__ __forceinline__ void task_fwd(float* Yb, const float* Wb, int lane) {
  if constexpr (MC == 8) {
    float d[2][4];
    mma_32x8<false>(d, Wb, [&](int k, int n) { return Yb[k * 8 + n]; }, lane);
    __syncwarp();  // every lane has read b_J before any lane overwrites it
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      *reinterpret_cast<float2*>(Yb + (16 * mt + g) * 8 + 2 * t) = make_float2(d[mt][0], d[mt][1]);
      *reinterpret_cast<float2*>(Yb + (16 * mt + g + 8) * 8 + 2 * t) = make_float2(d[mt][2], d[mt][3]);
    }
    return;
  }
  float acc[MC];
#pragma unroll
  for (int q = 0; q < MC; ++q) acc[q] = 0.f;
#pragma unroll
  for (int qq = 0; qq < 8; ++qq) {
    const float4 w4 = *reinterpret_cast<const float4*>(Wb + swq(lane, qq));
    const float ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float bv[MC];
      rhs_row<MC>(bv, Yb + (4 * qq + u) * MC);
#pragma unroll
      for (int q = 0; q < MC; ++q) acc[q] = fmaf(ww[u], bv[q], acc[q]);
    }
  }
  __syncwarp();  // every lane has read b_J before any lane overwrites it
#pragma unroll
  for (int q = 0; q < MC; ++q) Yb[lane * MC + q] = acc[q];
}

// B(I,J): y_I -= L_IJ y_J, one row of block I per lane.
template <int MC>
__device__ __forceinline__ void task_fupd(float* YI, const float* YJ, const float* X, int lane) {
  if constexpr (MC == 8) {
    float d[2][4];
    mma_32x8<false>(d, X, [&](int k, int n) { return YJ[k * 8 + n]; }, lane);
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      float2* p0 = reinterpret_cast<float2*>(YI + (16 * mt + g) * 8 + 2 * t);
      float2* p1 = reinterpret_cast<float2*>(YI + (16 * mt + g + 8) * 8 + 2 * t);
      float2 c0 = *p0, c1 = *p1;
      c0.x -= d[mt][0];
      c0.y -= d[mt][1];
      c1.x -= d[mt][2];
      c1.y -= d[mt][3];
      *p0 = c0;
      *p1 = c1;
    }
    return;
  }
  float acc[MC];
#pragma unroll
  for (int q = 0; q < MC; ++q) acc[q] = 0.f;
#pragma unroll
  for (int qq = 0; qq < 8; ++qq) {
    const float4 l4 = *reinterpret_cast<const float4*>(X + swq(lane, qq));
    const float ll[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float yv[MC];
      rhs_row<MC>(yv, YJ + (4 * qq + u) * MC);
#pragma unroll
      for (int q = 0; q < MC; ++q) acc[q] = fmaf(ll[u], yv[q], acc[q]);
    }
  }
#pragma unroll
  for (int q = 0; q < MC; ++q) YI[lane * MC + q] -= acc[q];
}

// S(I): x_I = W_I^T (y_I - z_I), one row of x per lane (column lane of W_I,
// zero above row lane); x_I replaces z_I and goes to global memory.
template <int MC>
__device__ __forceinline__ void task_bwd(const float* Yb, float* Zb, const float* Wb, float* xg, int m, int rows,
                                         int lane) {
  if constexpr (MC == 8) {
    float d[2][4];
    mma_32x8<true>(d, Wb, [&](int k, int n) { return Yb[k * 8 + n] - Zb[k * 8 + n]; }, lane);
    __syncwarp();  // every lane has read z_I before any lane overwrites it
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int r = 16 * mt + g + 8 * hh;
        const float v0 = d[mt][2 * hh], v1 = d[mt][2 * hh + 1];
        *reinterpret_cast<float2*>(Zb + r * 8 + 2 * t) = make_float2(v0, v1);
        if (r < rows) {
          if (2 * t < m) xg[(size_t)r * m + 2 * t] = v0;
          if (2 * t + 1 < m) xg[(size_t)r * m + 2 * t + 1] = v1;
        }
      }
    return;
  }
  float acc[MC];
#pragma unroll
  for (int q = 0; q < MC; ++q) acc[q] = 0.f;
#pragma unroll 8
  for (int c = 0; c < 32; ++c) {
    const float wv = Wb[swz(c, lane)];
    float yv[MC], zv[MC];
    rhs_row<MC>(yv, Yb + c * MC);
    rhs_row<MC>(zv, Zb + c * MC);
#pragma unroll
    for (int q = 0; q < MC; ++q) acc[q] = fmaf(wv, yv[q] - zv[q], acc[q]);
  }
  __syncwarp();  // every lane has read z_I before any lane overwrites it
#pragma unroll
  for (int q = 0; q < MC; ++q) Zb[lane * MC + q] = acc[q];
  if (lane < rows) {
#pragma unroll
    for (int q = 0; q < MC; ++q)
      if (q < m) xg[(size_t)lane * m + q] = acc[q];
  }
}

// G(J,I): z_J += L_IJ^T x_I; lane = row of block J = column of X. The sums
// live apart from y, which forward updates of other blocks may still read.
template <int MC>
__device__ __forceinline__ void task_bupd(float* ZJ, const float* XI, const float* X, int lane) {
  if constexpr (MC == 8) {
    float d[2][4];
    mma_32x8<true>(d, X, [&](int k, int n) { return XI[k * 8 + n]; }, lane);
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      float2* p0 = reinterpret_cast<float2*>(ZJ + (16 * mt + g) * 8 + 2 * t);
      float2* p1 = reinterpret_cast<float2*>(ZJ + (16 * mt + g + 8) * 8 + 2 * t);
      float2 c0 = *p0, c1 = *p1;
      c0.x += d[mt][0];
      c0.y += d[mt][1];
      c1.x += d[mt][2];
      c1.y += d[mt][3];
      *p0 = c0;
      *p1 = c1;
    }
    return;
  }
  float acc[MC];
#pragma unroll
  for (int q = 0; q < MC; ++q) acc[q] = 0.f;
#pragma unroll 8
  for (int c = 0; c < 32; ++c) {
    const float l = X[swz(c, lane)];
    float xv[MC];
    rhs_row<MC>(xv, XI + c * MC);
#pragma unroll
    for (int q = 0; q < MC; ++q) acc[q] = fmaf(l, xv[q], acc[q]);
  }
#pragma unroll
  for (int q = 0; q < MC; ++q) ZJ[lane * MC + q] += acc[q];
}

}  // namespace

template <int NW, int MC>
__global__ void __launch_bounds__(NW * 32, 16 / NW)
    posv_dag_kernel(const PosvParams p, const __grid_constant__ CUtensorMap tmap,
                    const __grid_constant__ DagTasks tl) {
  constexpr int NT = NW * 32;
  extern __shared__ __align__(16) unsigned char g_raw[];
  float* sm = reinterpret_cast<float*>(g_raw + ((1024u - (smem_u32(g_raw) & 1023u)) & 1023u));
  const int K = p.k, NB = (K + GB - 1) / GB, m = p.m;
  const bool rhs = m > 0;
  const GLay L = glay(NB, rhs ? MC : 0, NW);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* T = sm;
  float* Wm = sm + L.w;
  float* Y = sm + L.y;
  float* Z = sm + L.z;
  float* dinv = sm + L.dinv;
  float* ld = sm + L.ld;
  float* cb = sm + L.cb + warp * 64;
  uint64_t* mb = reinterpret_cast<uint64_t*>(sm + L.bar);  // events, then the tile loads
  uint64_t* loads = mb + L.nev;
  int* ctl = reinterpret_cast<int*>(sm + L.ctl);
  uint16_t* tasks = reinterpret_cast<uint16_t*>(sm + L.task);
  const int ntask = tl.n;

  for (int e = tid; e < L.nev; e += NT) mbar_init1(mb + e);
  for (int e = tid; e < ntask; e += NT) tasks[e] = tl.t[e];
  if (tid == 0) {
    for (int b = 0; b < L.nbt; ++b) mbar_init1(loads + b);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  uint32_t it = 0;
  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x, ++it) {
    // the previous matrix's shared-memory reads and writes come before the
    // tile loads that overwrite the blocks
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      for (int I = 0; I < NB; ++I)
        for (int J = 0; J <= I; ++J) {
          const int b = gblk(I, J);
          mbar_expect(loads + b, GBF * 4);
          tma_tile(T + b * GBF, &tmap, GB * J, GB * I, (int)mat, loads + b);
        }
    }
    if (tid < 2) ctl[tid] = 0;
    if (rhs) {
      const float* bm = p.b + (size_t)mat * K * m;
      for (int e = tid; e < 32 * NB * MC; e += NT) {
        const int i = e / MC, q = e - i * MC;
        Y[e] = (i < K && q < m) ? __ldg(bm + (size_t)i * m + q) : 0.f;
        Z[e] = 0.f;
      }
    }
    __syncthreads();
    const uint32_t par = it & 1u;
    int* abort_flag = ctl + 1;

    for (;;) {
      int t = 0;
      if (lane == 0) t = atomicAdd(ctl, 1);
      t = __shfl_sync(kFull, t, 0);
      if (t >= ntask) break;
      if (__shfl_sync(kFull, *reinterpret_cast<volatile int*>(abort_flag), 0)) break;
      const uint32_t e = tasks[t];
      const int type = e & 7, I = (e >> 3) & 7, Kb = (e >> 6) & 7, J = (e >> 9) & 7, h = (e >> 12) & 1;
      int wt[3];
      task_waits(e, NB, wt);
      bool ok = true;
#pragma unroll
      for (int i = 0; i < 3; ++i)
        if (ok && wt[i] >= 0) ok = gwait(mb + wt[i], par, abort_flag, tl.inject ? 1000000ull : kGWaitNs);
      // test only: the first task of CTA 0's first matrix waits for the phase
      // after its block's tile load, which nothing completes in this matrix;
      // nothing is in flight but that CTA's own tile loads
      if (tl.inject && ok && blockIdx.x == 0 && it == 0 && t == 0)
        ok = gwait(loads, par, abort_flag, 1000000ull) && gwait(loads, par ^ 1u, abort_flag, 1000000ull);
      if (!ok) {
        if (lane == 0) atomicOr(abort_flag, 1);
        break;
      }
      switch (type) {
        case TK_P: {
          float lg = task_potrf(T + gblk(J, J) * GBF, dinv + GB * J, cb, min(GB, K - GB * J), lane);
          lg = warp_sum(lg);
          if (lane == 0) ld[J] = lg;
          break;
        }
        case TK_W: task_inv(Wm + J * GBF, T + gblk(J, J) * GBF, dinv + GB * J, lane); break;
        case TK_T: task_trsm(T + gblk(I, J) * GBF, T + gblk(J, J) * GBF, dinv + GB * J, lane); break;
        case TK_U:
          task_update(T + gblk(I, Kb) * GBF, T + gblk(I, J) * GBF, T + gblk(Kb, J) * GBF, h, I == Kb && h == 0, lane);
          break;
        case TK_F: task_fwd<MC>(Y + GB * J * MC, Wm + J * GBF, lane); break;
        case TK_B: task_fupd<MC>(Y + GB * I * MC, Y + GB * J * MC, T + gblk(I, J) * GBF, lane); break;
        case TK_S:
          task_bwd<MC>(Y + GB * I * MC, Z + GB * I * MC, Wm + I * GBF, p.x + ((size_t)mat * K + GB * I) * m, m,
                       min(GB, K - GB * I), lane);
          break;
        default:  // TK_G: z_J += L_IJ^T x_I
          task_bupd<MC>(Z + GB * J * MC, Z + GB * I * MC, T + gblk(I, J) * GBF, lane);
          break;
      }
      if (!ok) {
        if (lane == 0) atomicOr(abort_flag, 1);
        break;
      }
      // publish: the warp's shared-memory writes, then the arrivals (release)
      int ft[2];
      task_fires(e, NB, ft);
      __threadfence_block();
      __syncwarp();
      if (lane == 0) {
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(mb + ft[0])) : "memory");
        if (ft[1] >= 0)
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(mb + ft[1])) : "memory");
      }
    }
    __syncthreads();

    if (*reinterpret_cast<volatile int*>(abort_flag)) {
      // let every tile load of this matrix land, then mark this matrix and
      // every later one of this CTA unfinished: x, logdet (and L) NaN
      if (tid == 0)
        for (int b = 0; b < L.nbt; ++b) gload_settle(loads + b, par);
      const float qnan = __int_as_float(0x7fc00000);
      for (int64_t m2 = mat; m2 < p.batch; m2 += gridDim.x) {
        if (m > 0)
          for (int64_t e = tid; e < (int64_t)K * m; e += NT) p.x[(size_t)m2 * K * m + e] = qnan;
        if (p.L)
          for (int64_t e = tid; e < (int64_t)K * K; e += NT) p.L[(size_t)m2 * K * K + e] = qnan;
        if (p.logdet && tid == 0) p.logdet[m2] = qnan;
      }
      if (tid == 0) atomicOr(&g_dag_fault, 1u);
      __syncthreads();
      break;
    }
    if (tid == 0 && p.logdet) {
      float s = 0.f;
      for (int J = 0; J < NB; ++J) s += ld[J];
      p.logdet[mat] = 2.f * s;
    }
    if (p.L) {
      float* Lm = p.L + (size_t)mat * K * K;
      for (int e = tid; e < K * K; e += NT) {
        const int r = e / K, c = e - r * K;
        Lm[e] = (c > r) ? 0.f : T[gblk(r / GB, c / GB) * GBF + swz(r % GB, c % GB)];
      }
    }
  }
}

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// B2C_SMEM_DAG=0 (read per call) keeps these calls on the barrier-phased
// kernel of posv_smem.cu; B2C_DAG_WARPS=4|8|12|16 overrides the warps per CTA
// and B2C_DAG_AHEAD the schedule's look-ahead (tuning).
bool dag_enabled() {
  const char* t = getenv("B2C_SMEM_DAG");
  return !(t && strcmp(t, "0") == 0);
}

int dag_warps(int nb) {
  const char* t = getenv("B2C_DAG_WARPS");
  if (t) {
    const int w = atoi(t);
    if (w == 4 || w == 8 || w == 12 || w == 16) return w;
  }
  return nb <= 4 ? 4 : (nb <= 6 ? 8 : 12);
}

// The tasks of one matrix in a topological order (panel by panel).
int dag_topo(int nb, bool rhs, uint16_t* out) {
  int n = 0;
  for (int J = 0; J < nb; ++J) {
    out[n++] = tenc(TK_P, J, J, J, 0);
    if (rhs) out[n++] = tenc(TK_W, J, J, J, 0);
    if (rhs) out[n++] = tenc(TK_F, J, J, J, 0);
    for (int I = J + 1; I < nb; ++I) out[n++] = tenc(TK_T, I, J, J, 0);
    for (int K = J + 1; K < nb; ++K)
      for (int I = K; I < nb; ++I) {
        out[n++] = tenc(TK_U, I, K, J, 0);
        out[n++] = tenc(TK_U, I, K, J, 1);
      }
    if (rhs)
      for (int I = J + 1; I < nb; ++I) out[n++] = tenc(TK_B, I, J, J, 0);
  }
  if (rhs)
    for (int I = nb - 1; I >= 0; --I) {
      out[n++] = tenc(TK_S, I, I, I, 0);
      for (int J = I - 1; J >= 0; --J) out[n++] = tenc(TK_G, I, J, J, 0);
    }
  return n;
}

// Orders the tasks for `nw` warps by list scheduling: a simulated warp that
// becomes free takes, among the tasks whose inputs are all scheduled, the
// one ready soonest, breaking ties by the longest path from the task to the
// end of the graph (so the factorisation's chain P -> T -> U -> P leads).
// Durations are rough per-task cycle counts measured on B200. Every task
// comes after its inputs, which is what keeps the kernel free of stalls.
void dag_schedule(int nb, bool rhs, int nw, double ahead, DagTasks& out) {
  uint16_t topo[GMAXTASK];
  const int n = dag_topo(nb, rhs, topo);
  const int nev = gnev(nb);
  std::vector<int> prod(nev + gtri(nb), -1);
  for (int i = 0; i < n; ++i) {
    int f[2];
    task_fires(topo[i], nb, f);
    for (int j = 0; j < 2; ++j)
      if (f[j] >= 0) prod[f[j]] = i;
  }
  std::vector<std::vector<int>> dep(n), succ(n);
  for (int i = 0; i < n; ++i) {
    int w[3];
    task_waits(topo[i], nb, w);
    for (int j = 0; j < 3; ++j)
      if (w[j] >= 0 && w[j] < nev && prod[w[j]] >= 0) {
        dep[i].push_back(prod[w[j]]);
        succ[prod[w[j]]].push_back(i);
      }
  }
  double dur_of[8] = {6000, 3000, 4500, 2000, 1600, 1700, 2000, 3700};  // P T U F B S G W
  if (const char* d = getenv("B2C_DAG_DUR"))  // tuning: eight comma-separated cycle counts
    for (int i = 0; i < 8 && *d; ++i) {
      dur_of[i] = atof(d);
      while (*d && *d != ',') ++d;
      if (*d == ',') ++d;
    }
  std::vector<double> dur(n), bl(n, 0.0), ready(n, 0.0);
  for (int i = 0; i < n; ++i) dur[i] = dur_of[topo[i] & 7];
  for (int i = n - 1; i >= 0; --i) {  // topo order: successors come later
    double mx = 0.0;
    for (int sidx : succ[i]) mx = bl[sidx] > mx ? bl[sidx] : mx;
    bl[i] = dur[i] + mx;
  }
  std::vector<int> left(n);
  std::vector<char> cand(n, 0), done(n, 0);
  for (int i = 0; i < n; ++i) {
    left[i] = (int)dep[i].size();
    if (left[i] == 0) cand[i] = 1;
  }
  std::vector<double> free_at(nw > 0 ? nw : 1, 0.0);
  out.n = n;
  for (int k = 0; k < n; ++k) {
    int wk = 0;
    for (int w = 1; w < (int)free_at.size(); ++w)
      if (free_at[w] < free_at[wk]) wk = w;
    const double tw = free_at[wk];
    // among the tasks ready within `ahead` of this warp, the longest path
    // first (a warp that takes a task early sleeps on its inputs); else the
    // task ready soonest
    int best = -1;
    for (int i = 0; i < n; ++i) {
      if (!cand[i]) continue;
      if (best < 0) { best = i; continue; }
      const bool ni = ready[i] <= tw + ahead, nb_ = ready[best] <= tw + ahead;
      if (ni && nb_) {
        if (bl[i] > bl[best] || (bl[i] == bl[best] && ready[i] < ready[best])) best = i;
      } else if (ni != nb_) {
        if (ni) best = i;
      } else if (ready[i] < ready[best] || (ready[i] == ready[best] && bl[i] > bl[best])) {
        best = i;
      }
    }
    const double start = ready[best] > tw ? ready[best] : tw, end = start + dur[best];
    out.t[k] = topo[best];
    cand[best] = 0;
    done[best] = 1;
    free_at[wk] = end;
    for (int sidx : succ[best]) {
      if (end > ready[sidx]) ready[sidx] = end;
      if (--left[sidx] == 0) cand[sidx] = 1;
    }
  }
  // every input before its consumer, or the panel order (which has that property)
  std::vector<int> pos(n, -1);
  for (int k = 0; k < n; ++k)
    for (int i = 0; i < n; ++i)
      if (topo[i] == out.t[k]) pos[i] = k;
  bool ok = true;
  for (int i = 0; i < n && ok; ++i) {
    ok = pos[i] >= 0;
    for (int d : dep[i]) ok = ok && pos[d] >= 0 && pos[d] < pos[i];
  }
  if (!ok)
    for (int k = 0; k < n; ++k) out.t[k] = topo[k];
}

// Task lists per (blocks a side, rhs, warps), built once.
const DagTasks& dag_tasks(int nb, bool rhs, int nw) {
  static DagTasks cache[GMAXNB + 1][2][17];
  static bool have[GMAXNB + 1][2][17];
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  DagTasks& d = cache[nb][rhs ? 1 : 0][nw];
  if (!have[nb][rhs ? 1 : 0][nw]) {
    const char* a = getenv("B2C_DAG_AHEAD");  // tuning: look-ahead of the schedule, cycles
    dag_schedule(nb, rhs, nw, a ? atof(a) : 0.0, d);
    have[nb][rhs ? 1 : 0][nw] = true;
  }
  return d;
}

int dag_sm_count() {
  static int cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 148;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

template <int NW, int MC>
cudaError_t launch_dag_t(const PosvParams& p, const CUtensorMap& tm, cudaStream_t s) {
  const int nb = (p.k + GB - 1) / GB;
  const size_t smem = gdag_smem_bytes(nb, p.m > 0 ? MC : 0, NW);
  DagTasks tl = dag_tasks(nb, p.m > 0, NW);
  const char* inj = getenv("B2C_DAG_INJECT_TIMEOUT");  // test only, read per call
  tl.inject = (inj && atoi(inj) != 0) ? 1 : 0;
  static int cache[64];
  int occ = 0;
  auto kern = posv_dag_kernel<NW, MC>;
  cudaError_t e = kernel_occupancy(kern, NW * 32, smem, cache, &occ);
  if (e != cudaSuccess) return e;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, NW * 32, smem);
  if (e != cudaSuccess) return e;
  if (occ < 1) occ = 1;
  const int64_t cap = (int64_t)dag_sm_count() * occ;
  kern<<<(int)(p.batch < cap ? p.batch : cap), NW * 32, smem, s>>>(p, tm, tl);
  return cudaGetLastError();
}

template <int MC>
cudaError_t launch_dag_mc(const PosvParams& p, const CUtensorMap& tm, cudaStream_t s) {
  switch (dag_warps((p.k + GB - 1) / GB)) {
    case 4: return launch_dag_t<4, MC>(p, tm, s);
    case 8: return launch_dag_t<8, MC>(p, tm, s);
    case 12: return launch_dag_t<12, MC>(p, tm, s);
    default: return launch_dag_t<16, MC>(p, tm, s);
  }
}

}  // namespace

// Where the task graph takes a call by default, from B200 measurements of
// both forms of the tier (ms, task graph / barrier-phased, B = 1,000 and
// 10,000): at 7 and 8 blocks a side it wins for every m (k = 256, m = 1:
// 0.398 / 0.518 and 3.75 / 4.99; m = 8: 0.459 / 0.553 and 4.24 / 5.33); at
// 3 to 5 blocks it wins with several right-hand sides (k = 80, m = 8: 0.063 /
// 0.072 and 0.611 / 0.636; k = 160, m = 8: 0.180 / 0.196 and 1.60 / 1.67)
// but not with one, where the barrier-phased kernel's cheap single
// substitution and several CTAs per SM are ahead (k = 80, m = 1: 0.057 /
// 0.047 and 0.527 / 0.376; k = 128, m = 1: 0.100 / 0.078); at 6 blocks the
// inverses' 24 KB leave one CTA per SM where the barrier-phased kernel fits
// two (k = 192, m = 8: 0.309 / 0.271). B2C_SMEM_DAG=all takes every k >= 65
// it can (tests use it), =0 none.
bool dag_takes(int nb, int m) {
  const char* t = getenv("B2C_SMEM_DAG");
  if (t && strcmp(t, "all") == 0) return nb >= 3;
  return nb >= 7 || (nb >= 3 && nb <= 5 && m >= 2);
}

bool posv_dag_applies(const PosvParams& p) {
  if (!dag_enabled() || p.k < 65 || p.k > GB * GMAXNB || !dag_takes((p.k + GB - 1) / GB, p.m) || (p.k & 3) != 0 ||
      p.m > 8 || p.batch < 1)
    return false;
  if (p.batch > 0x7fffffffLL || (reinterpret_cast<uintptr_t>(p.A) & 15) != 0 || encode_tiled() == nullptr) return false;
  // tile loads read device memory only (host buffers take the cp.async kernel)
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p.A) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeDevice;
}

cudaError_t launch_posv_dag(const PosvParams& p, cudaStream_t s) {
  CUtensorMap tm;
  const cuuint64_t dims[3] = {(cuuint64_t)p.k, (cuuint64_t)p.k, (cuuint64_t)p.batch};
  const cuuint64_t strides[2] = {(cuuint64_t)p.k * 4, (cuuint64_t)p.k * p.k * 4};
  const cuuint32_t box[3] = {GB, GB, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode_tiled()(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(p.A), dims, strides,
                                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  return p.m > 1 ? launch_dag_mc<8>(p, tm, s) : launch_dag_mc<1>(p, tm, s);
}

// Reads and clears the task-graph kernel's fault flag (synchronises the device).
cudaError_t dag_take_fault(unsigned int* fault) {
  unsigned int f = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&f, g_dag_fault, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  *fault |= f;
  const unsigned int zero = 0;
  return cudaMemcpyToSymbol(g_dag_fault, &zero, sizeof(unsigned int));
}

}  // namespace b2c
