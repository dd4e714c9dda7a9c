// Blocked Cholesky factor + solve for k > 64, panel products on the tensor cores.
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
// taken in groups of 128, 64 or 32 rows (16 RI rows, RI = 8, 4, 2), so the
// shrinking panels of the late columns are never padded by more than 31
// rows. For each group:
//   1. P = A[rows, panel] - L[rows, :j0] L[panel, :j0]^T as 3xTF32
//      mma.sync m16n8k8 tiles (GroupTiles: each warp 2 x 4, 1 x 4 or 2 x 1
//      tiles of the group). Both operands are staged in shared memory 32
//      columns at a time with cp.async, double-buffered: chunk c + 1 loads
//      while chunk c is multiplied, one CTA barrier per chunk. The 36-float
//      row stride makes every fragment load conflict-free.
//   2. First group of the panel: warp 0 factors the 32x32 diagonal block in
//      registers (right-looking, reference clamp); all warps then form its
//      inverse, 32 / (NT/32) columns each, by independent forward substitutions, kept in
//      shared memory (swizzled) for this panel. When right-hand sides follow,
//      the strict lower triangle of the inverse is also stored, transposed,
//      in the strict upper triangle of the diagonal block of L's slot (unused
//      by L; zeroed again at the end when L is an output).
//   3. The panel rows below the diagonal block are solved as X = P L_JJ^{-T},
//      the same tensor-core tiles with the inverse as the second operand.
//   4. The panel is written once.
// The substitutions then use the panel inverses (reloaded per 32-row block
// from the slot; 1 / L_jj is recomputed bit for bit): each block is a GEMV
// over the rows already solved followed by a 32x32 mat-vec with the inverse
// (forward: L_JJ^{-1}; backward: L_JJ^{-T}), one warp per right-hand side,
// instead of a 32-step dependent chain.
//
// Tensor-core form (posv_blocked2_kernel<128, true>, B2C_BLOCKED_GEMM=tc): the two
// panel GEMMs, P = A - L L^T and X = P L_JJ^{-T}, run on the 5th-generation
// tensor cores as 3xTF32 products (hi_a hi_b + hi_a lo_b + lo_a hi_b, where
// hi = tf32(x) rounded to nearest and lo = tf32(x - hi): FP32-level accuracy
// from three TF32 MMAs). Groups are always 128 rows (M = 128, one row per
// thread); the accumulator D (128 x 32 FP32) lives in 32 columns of tensor
// memory. Operand chunks of 16 columns go global -> registers -> shared
// memory, split into hi/lo on the way, in the K-major no-swizzle layout
// (8-row x 16-byte core matrices), double-buffered: thread 0 issues a chunk's
// six MMAs and commits them to that buffer's mbarrier, and the buffer is
// rewritten only after that mbarrier completes, while the next chunk's loads
// are in flight. Every mbarrier wait gives up after one second of global
// time; the CTA then waits (bounded again) for the MMAs it had committed,
// writes NaN to x and logdet of the matrix it was on and of every later one
// of its matrices, sets a fault flag readable from the host
// (blocked_take_fault) and leaves through its normal exit, freeing its
// tensor memory.
#include <stdlib.h>
#include <string.h>

#include <type_traits>

#include "b2c_blocked_common.cuh"
#include "b2c_common.cuh"
#include "b2c_kernels.cuh"

namespace b2c {

// Set (bit 0) by a CTA of the tensor-core kernel whose mbarrier wait timed out.
__device__ unsigned int g_blocked_fault;

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

// Shared-memory layout of the tensor-core form (floats). Chunk buffer b at
// b * BUF: A rows (128 x 16) hi at AHI and lo at ALO, B rows (32 x 16) hi at
// BHI and lo at BLO; the 16-byte unit (row r, column quad q) of an R-row
// operand sits at (q R + r) * 4. After the chunks, the same 40 KB hold the
// operands of X = P L_JJ^{-T}: P (128 x 32) at PHI / PLO, L_JJ^{-1} (32 x 32)
// at IHI / ILO.
struct B2TC {
  static constexpr int NT = 128;
  static constexpr int NW = 4;
  static constexpr int A_FL = B2<128>::A_FL;  // the substitutions' buffer size (right-hand sides per pass)
  static constexpr int BUF = 5632;
  static constexpr int AHI = 0, ALO = 2048, BHI = 4096, BLO = 4864;  // B: 48 rows (32 of L, 16 of y)
  static constexpr int PHI = 0, PLO = 4096, IHI = 8192, ILO = 9216;
  static constexpr int OFF_A = 0;                   // substitutions: right-hand sides (2 A_FL floats)
  static constexpr int OFF_B = 2 * A_FL;            // factor32 column buffer; substitutions: reduction
  static constexpr int OFF_D = 2 * BUF;             // 32 x 36: diagonal block
  static constexpr int OFF_INV = OFF_D + 32 * 36;   // 1024: inverse of the diagonal block (swizzled rows)
  static constexpr int OFF_Y = OFF_INV + 1024;      // 32 x 8: t of the fused forward substitution
  static constexpr int OFF_BAR = OFF_Y + 256;       // three mbarriers, then the tensor-memory address
  static constexpr int SMEM = OFF_BAR + 8;
  static constexpr int TMEM_COLS = 64;              // D: 32 columns of P, 16 of the fused forward
  static_assert(OFF_B + NW * MCB2 * 32 <= OFF_D, "reduction buffer");
  static_assert(IHI + 1024 <= OFF_B && ILO + 1024 <= OFF_D, "inverse operands");
  static_assert(BLO + 768 == BUF, "chunk buffer");
  static_assert((OFF_BAR * 4) % 8 == 0, "mbarrier alignment");
};

// x rounded to TF32 (10 stored mantissa bits), to nearest with ties away
// from zero: add half a unit of the 13th bit, clear the 13 low bits. Integer
// ALU work; the same result as cvt.rna.tf32.f32 for finite x, at a fraction
// of the conversion unit's cost.
__device__ __forceinline__ float to_tf32(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// hi = tf32(v) and lo = tf32(v - hi), stored as 16-byte units
__device__ __forceinline__ void split_store(float4 v, float* hi, float* lo) {
  const float4 h = make_float4(to_tf32(v.x), to_tf32(v.y), to_tf32(v.z), to_tf32(v.w));
  *reinterpret_cast<float4*>(hi) = h;
  *reinterpret_cast<float4*>(lo) =
      make_float4(to_tf32(v.x - h.x), to_tf32(v.y - h.y), to_tf32(v.z - h.z), to_tf32(v.w - h.w));
}

// Shared-memory matrix descriptor, K-major, no swizzle: lbo = byte distance
// between the two core matrices along K of one MMA, sbo = byte distance
// between consecutive 8-row groups; descriptor version 1 (bit 46).
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46);
}

// Instruction descriptors: D in FP32, A and B in TF32, both K-major, M = 128.
// X product: N = 32. Chunk products: A negated (bit 13), N in bits 17..22
// (32, or 48 with the fused forward substitution's columns).
constexpr uint32_t kIdescX = (1u << 4) | (2u << 7) | (2u << 10) | ((32u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescChunk = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 13) | ((128u >> 4) << 24);

__device__ __forceinline__ void umma_tf32(uint32_t tmem, uint32_t idesc, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

// Three TF32 MMAs of one K = 8 step: D (+)= lo_a hi_b + hi_a lo_b + hi_a hi_b.
__device__ __forceinline__ void umma_3xtf32(uint32_t tmem, uint32_t idesc, uint32_t ahi, uint32_t alo, uint32_t a_lbo,
                                            uint32_t bhi, uint32_t blo, uint32_t b_lbo, uint32_t acc) {
  const uint64_t dah = umma_desc(ahi, a_lbo, 128), dal = umma_desc(alo, a_lbo, 128);
  const uint64_t dbh = umma_desc(bhi, b_lbo, 128), dbl = umma_desc(blo, b_lbo, 128);
  umma_tf32(tmem, idesc, dal, dbh, acc);
  umma_tf32(tmem, idesc, dah, dbl, 1u);
  umma_tf32(tmem, idesc, dah, dbh, 1u);
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Limit of every mbarrier wait: one second of global time, 1 ms when a test
// makes a wait run out on purpose (PosvParams::tc_inject).
__device__ __forceinline__ uint64_t wait_limit_ns(const PosvParams& p) {
  return p.tc_inject ? 1000000ull : 1000000000ull;
}

// Wait for the completion of the mbarrier phase with the given parity; false
// after `limit` ns of global time without it.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit) {
  const uint32_t a = smem_u32(bar);
  const uint64_t t0 = global_ns();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if (global_ns() - t0 > limit) return false;
  }
}

// Row (warp 32 + lane) of the 128 x 32 accumulator, one column per register;
// the load and its wait form one statement, so no use can precede the wait.
__device__ __forceinline__ void tmem_ld_row32(uint32_t taddr, float (&d)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int c = 0; c < 32; ++c) d[c] = __uint_as_float(r[c]);
}

// Row (warp 32 + lane), 8 columns from column offset of taddr.
__device__ __forceinline__ void tmem_ld_row8(uint32_t taddr, float (&d)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int c = 0; c < 8; ++c) d[c] = __uint_as_float(r[c]);
}

// Stores of one accumulator row (32 or 8 columns), complete on return.
__device__ __forceinline__ void tmem_st_row32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;\n" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
      "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
      "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_st_row8(uint32_t taddr, const float (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n\t"
      "tcgen05.wait::st.sync.aligned;\n" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
      : "memory");
}

// Four consecutive floats of a row: one 16-byte load when rows are 16-byte
// aligned, else four. L2-coherent (the slot is written by this CTA).
__device__ __forceinline__ float4 ld4_cg(const float* ptr, bool vec) {
  if (vec) return __ldcg(reinterpret_cast<const float4*>(ptr));
  return make_float4(__ldcg(ptr), __ldcg(ptr + 1), __ldcg(ptr + 2), __ldcg(ptr + 3));
}

// The diagonal block's tail, once its factor is in sD and visible to the
// CTA: L_JJ rows to the slot, coalesced (upper part: zero, or the transposed
// inverse written below when right-hand sides follow); rows right of the
// block zeroed when L is an output; the inverse X = L_JJ^{-1} formed by all
// warps into Li; then, for the fused forward substitution, y_J = L_JJ^{-1} t
// with t (32 x 8) in sT. Thread (ty, tx) = (tid / 8, tid % 8) owns the
// (row, right-hand side) pairs (ty + TY t, tx).
template <int NT>
__device__ __forceinline__ void diag_tail(const PosvParams& p, float* Wm, int K, int j0, int bw, const float* sD,
                                          float* Li, const float* sT, bool fw, float* ym) {
  constexpr int NW = NT / 32, CPW = 32 / NW, TV = 256 / NT, TY = NT / 8;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ty = tid >> 3, tx = tid & 7;
  const int m = p.m;
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
    float xs[CPW];
#pragma unroll
    for (int q = 0; q < CPW; ++q) xs[q] = (lane == CPW * warp + q) ? 1.f : 0.f;
#pragma unroll
    for (int pp = 0; pp < 32; ++pp) {
      // row pp of X is final in lane pp once scaled by 1 / L_pp
#pragma unroll
      for (int q = 0; q < CPW; ++q) {
        const float xp = __shfl_sync(kFull, xs[q] * il, pp);
        xs[q] = (lane == pp) ? xp : ((lane > pp) ? fmaf(-lrow[pp], xp, xs[q]) : xs[q]);
      }
    }
#pragma unroll
    for (int q = 0; q < CPW; ++q) {
      const int c = CPW * warp + q;
      Li[inv_off(lane, c)] = xs[q];
      // strict lower triangle, transposed into the unused strict upper
      // triangle of the diagonal block, for the substitutions
      if (p.m > 0 && lane > c && lane < bw) Wm[(size_t)(j0 + c) * K + j0 + lane] = xs[q];
    }
  }
  __syncthreads();
  if (fw && tx < m) {  // y_J = L_JJ^{-1} t
#pragma unroll
    for (int t = 0; t < TV; ++t) {
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

// The chunk products of a group on the tensor cores (NT = 128, four warps):
// the TY RI = 16 RI rows by 32 columns of P split into m16n8 tiles, warp w
// taking MT x NTL of them from row 32 w (RI = 8), 16 w (RI = 4) or 0 with
// column 8 w (RI = 2). Each K = 8 step is three TF32 products (3xTF32: hi hi,
// hi lo, lo hi); the fragment loads of the staged operands (row stride 36)
// read 32 distinct banks.
template <int RI>
struct GroupTiles {
  static constexpr int MT = RI == 4 ? 1 : 2;
  static constexpr int NTL = RI == 2 ? 1 : 4;
  __device__ static int row0(int w) { return RI == 8 ? 32 * w : (RI == 4 ? 16 * w : 0); }
  __device__ static int col0(int w) { return RI == 2 ? 8 * w : 0; }
};

// d += As Bop^T over 32 columns of K, As the staged rows (stride 36), bop(n, k)
// element k of the second operand's row n.
template <int RI, typename BOp>
__device__ __forceinline__ void group_mma(float (&d)[GroupTiles<RI>::MT][GroupTiles<RI>::NTL][4], const float* As,
                                          BOp bop, int warp, int lane) {
  using G = GroupTiles<RI>;
  const int g = lane >> 2, t = lane & 3;
  const int r0 = G::row0(warp), c0 = G::col0(warp);
#pragma unroll
  for (int k0 = 0; k0 < KC2; k0 += 8) {
    uint32_t ah[G::MT][4], al[G::MT][4];
#pragma unroll
    for (int mt = 0; mt < G::MT; ++mt) {
      const float* ar = As + (r0 + 16 * mt + g) * AS2 + k0 + t;
      tf32_split(ar[0], ah[mt][0], al[mt][0]);
      tf32_split(ar[8 * AS2], ah[mt][1], al[mt][1]);
      tf32_split(ar[4], ah[mt][2], al[mt][2]);
      tf32_split(ar[8 * AS2 + 4], ah[mt][3], al[mt][3]);
    }
#pragma unroll
    for (int n = 0; n < G::NTL; ++n) {
      uint32_t bh0, bl0, bh1, bl1;
      tf32_split(bop(c0 + 8 * n + g, k0 + t), bh0, bl0);
      tf32_split(bop(c0 + 8 * n + g, k0 + t + 4), bh1, bl1);
#pragma unroll
      for (int mt = 0; mt < G::MT; ++mt) {
        mma_tf32(d[mt][n], al[mt], bh0, bh1);
        mma_tf32(d[mt][n], ah[mt], bl0, bl1);
        mma_tf32(d[mt][n], ah[mt], bh0, bh1);
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

  // A's panel columns in the tensor-core tile layout: lane (g, t) of warp w
  // holds rows row0 + 16 mt + g (+ 8) and columns col0 + 8 n + 2t (+ 1)
  static_assert(NT == 128, "four warps share a group's tiles");
  using G = GroupTiles<RI>;
  const int tg = lane >> 2, tt = lane & 3;
  float av[G::MT][G::NTL][4], prod[G::MT][G::NTL][4];
#pragma unroll
  for (int mt = 0; mt < G::MT; ++mt)
#pragma unroll
    for (int n = 0; n < G::NTL; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = rg + G::row0(warp) + 16 * mt + tg + 8 * (i >> 1);
        const int c = G::col0(warp) + 8 * n + 2 * tt + (i & 1);
        av[mt][n][i] = (r < K && c < bw) ? __ldg(A + (size_t)r * K + j0 + c) : 0.f;
        prod[mt][n][i] = 0.f;
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
      const float* Bs = sm + S::OFF_B + (ch & 1) * S::B_FL;
      group_mma<RI>(prod, sm + S::OFF_A + (ch & 1) * S::A_FL, [&](int n, int k) { return Bs[n * AS2 + k]; }, warp,
                    lane);
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

  // ---- P = A - products to shared memory (operand buffer 0) --------------
  float* Pm = sm + S::OFF_A;
  float* sT = sm + S::OFF_Y;  // t of the panel (32 x 8), free once the chunks are done
  __syncthreads();
#pragma unroll
  for (int mt = 0; mt < G::MT; ++mt)
#pragma unroll
    for (int n = 0; n < G::NTL; ++n)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int r = G::row0(warp) + 16 * mt + tg + 8 * hh, c = G::col0(warp) + 8 * n + 2 * tt;
        float2 v;
        v.x = (c < bw) ? av[mt][n][2 * hh] - prod[mt][n][2 * hh] : 0.f;
        v.y = (c + 1 < bw) ? av[mt][n][2 * hh + 1] - prod[mt][n][2 * hh + 1] : 0.f;
        *reinterpret_cast<float2*>(Pm + r * AS2 + c) = v;
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
      for (int c = 0; c < 32; ++c) a[c] = (lane < bw && c < bw) ? Pm[lane * AS2 + c] : (c == lane ? 1.f : 0.f);
      float invo = 1.f, dv = 1.f;
      factor32(a, lane, sm + S::OFF_B, invo, dv);  // operand buffer B doubles as the column buffer
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 32; ++c) sD[lane * 36 + c] = (c < lane) ? a[c] : (c == lane ? dv : 0.f);
      if (lane < bw) lgacc += logf(dv);
    }
    __syncthreads();
    diag_tail<NT>(p, Wm, K, j0, bw, sD, Li, sT, fw, ym);
  }

  // ---- X = P L_JJ^{-T} for the rows below the diagonal block -------------
#pragma unroll
  for (int mt = 0; mt < G::MT; ++mt)
#pragma unroll
    for (int n = 0; n < G::NTL; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) prod[mt][n][i] = 0.f;
  group_mma<RI>(prod, Pm, [&](int n, int k) { return Li[inv_off(n, k)]; }, warp, lane);
#pragma unroll
  for (int mt = 0; mt < G::MT; ++mt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int rl = G::row0(warp) + 16 * mt + tg + 8 * hh, r = rg + rl;
      if (r >= K || (first && rl < 32)) continue;  // diagonal rows hold L_JJ already
      float* wr = Wm + (size_t)r * K + j0;
#pragma unroll
      for (int n = 0; n < G::NTL; ++n) {
        const int c = G::col0(warp) + 8 * n + 2 * tt;
        if (c < bw) wr[c] = prod[mt][n][2 * hh];
        if (c + 1 < bw) wr[c + 1] = prod[mt][n][2 * hh + 1];
      }
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


// One 128-row group of panel J on the tensor cores: rows rg .. rg + 127
// (rows at or past K computed on zeros and dropped), thread t owning row
// rg + t. D starts as A's panel columns (tcgen05.st) and the chunk MMAs
// subtract (A operand negated), so D ends as P. With the fused forward
// substitution (first group), the chunk's y rows ride along as B rows 32..39
// (N = 48): D[r][32 + q] starts as b[j0 + r][q] and ends as t. Chunk loads
// run two chunks ahead in two register sets. `pend` / `par` track the three
// mbarriers (bit i: a commit on barrier i not yet waited for / the parity of
// the next phase to wait for), the same in every thread. Returns false, the
// same in every thread, when an mbarrier wait timed out.
__device__ __forceinline__ bool panel_tc(const PosvParams& p, const float* A, float* Wm, int K, int j0, int rg,
                                         float* sm, bool vec, bool fwd, int64_t mat, float& lgacc, uint32_t tmem,
                                         uint32_t& pend, uint32_t& par) {
  using S = B2TC;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bw = min(32, K - j0);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::OFF_BAR);
  float* sD = sm + S::OFF_D;
  float* Li = sm + S::OFF_INV;
  const bool first = (rg == j0);
  const bool fw = fwd && first;
  const int m = p.m;
  float* ym = p.x + (size_t)mat * K * m;  // y (forward result) lives in x
  const int row = rg + tid;
  const bool live = row < K;
  const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);  // this warp's 32 lanes of D
  const uint32_t sbase = smem_u32(sm);
  bool ok = true;
  auto settle = [&](int i) {  // wait for barrier i's outstanding commit, if any
    if ((pend >> i) & 1u) {
      ok = mbar_wait(bars + i, (par >> i) & 1u, wait_limit_ns(p)) && ok;
      pend &= ~(1u << i);
      par ^= 1u << i;
    }
  };

  // this thread's row of A's panel columns (bw is a multiple of 4 when vec)
  float pr[32];
  {
    const float* ar = A + (size_t)row * K + j0;
#pragma unroll
    for (int c4 = 0; c4 < 32; c4 += 4) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (live && vec && c4 < bw) {
        v = __ldg(reinterpret_cast<const float4*>(ar + c4));
      } else if (live && !vec) {
        if (c4 < bw) v.x = __ldg(ar + c4);
        if (c4 + 1 < bw) v.y = __ldg(ar + c4 + 1);
        if (c4 + 2 < bw) v.z = __ldg(ar + c4 + 2);
        if (c4 + 3 < bw) v.w = __ldg(ar + c4 + 3);
      }
      pr[c4] = v.x;
      pr[c4 + 1] = v.y;
      pr[c4 + 2] = v.z;
      pr[c4 + 3] = v.w;
    }
  }
  // fused forward: t of (row j0 + lane, right-hand side q), warp 0
  float tq[8];
#pragma unroll
  for (int q = 0; q < 8; ++q)
    tq[q] = (fw && warp == 0 && lane < bw && q < m) ? p.b[(size_t)mat * K * m + (size_t)(j0 + lane) * m + q] : 0.f;

  // ---- D = [A | b] - L[rows, :j0] [L[panel, :j0] | y[:j0]]^T ----------------
  // chunk ch = columns 16 ch .. 16 ch + 15; A unit f = tid + 128 i (row f / 4,
  // quad f % 4); B unit tid (row tid / 4, quad tid % 4); y element tid
  // (column tid / 8, right-hand side tid % 8)
  const int nch = j0 / 16;
  const uint32_t idesc = kIdescChunk | ((fw ? 48u : 32u) >> 3 << 17);
  float4 a0[4], b0, a1[4], b1;
  float y0 = 0.f, y1 = 0.f;
  auto gload = [&](float4(&ra)[4], float4& rb, float& ry, int ch) {
    const int p0 = ch * 16;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int f = tid + 128 * i, r = f >> 2, q = f & 3;
      ra[i] = (rg + r < K) ? ld4_cg(Wm + (size_t)(rg + r) * K + p0 + 4 * q, vec) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int r = tid >> 2, q = tid & 3;
    rb = (r < bw) ? ld4_cg(Wm + (size_t)(j0 + r) * K + p0 + 4 * q, vec) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (fw) {
      const int kk = tid >> 3, qq = tid & 7;
      ry = (qq < m) ? __ldcg(ym + (size_t)(p0 + kk) * m + qq) : 0.f;
    }
  };
  // chunk ch from registers to buffer ch & 1 (hi / lo), then its six MMAs
  auto chunk = [&](float4(&ra)[4], float4& rb, float& ry, int ch) -> bool {
    const int b = ch & 1;
    float* buf = sm + b * S::BUF;
    settle(b);  // the MMAs that last read buffer b are done
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int f = tid + 128 * i, r = f >> 2, q = f & 3, o = (q * 128 + r) * 4;
      split_store(ra[i], buf + S::AHI + o, buf + S::ALO + o);
    }
    {
      const int r = tid >> 2, q = tid & 3, o = (q * 48 + r) * 4;
      split_store(rb, buf + S::BHI + o, buf + S::BLO + o);
    }
    if (fw) {  // y[p0 + kk][qq] is B element (32 + qq, kk)
      const int kk = tid >> 3, qq = tid & 7, o = ((kk >> 2) * 48 + 32 + qq) * 4 + (kk & 3);
      const float h = to_tf32(ry);
      buf[S::BHI + o] = h;
      buf[S::BLO + o] = to_tf32(ry - h);
    }
    if (ch + 2 < nch) gload(ra, rb, ry, ch + 2);  // two chunks ahead
    fence_async_smem();                           // generic-proxy writes -> tensor-core reads
    tc_fence_before();
    if (__syncthreads_or(!ok)) return false;
    tc_fence_after();
    if (tid == 0) {
      const uint32_t bb = sbase + (uint32_t)(b * S::BUF) * 4u;
#pragma unroll
      for (int s = 0; s < 2; ++s)  // K = 8 per step: quads 2 s, 2 s + 1
        umma_3xtf32(tmem, idesc, bb + (S::AHI + s * 1024) * 4, bb + (S::ALO + s * 1024) * 4, 128 * 16,
                    bb + (S::BHI + s * 384) * 4, bb + (S::BLO + s * 384) * 4, 48 * 16, 1u);
      umma_commit(bars + b);
    }
    pend |= 1u << b;
    return true;
  };
  if (nch > 0) {
    tmem_st_row32(taddr, pr);
    if (fw && warp == 0) tmem_st_row8(taddr + 32, tq);
#pragma unroll
    for (int q = 0; q < 8; ++q) tq[q] = 0.f;  // reloaded from D below; nothing live across the chunks
    gload(a0, b0, y0, 0);
    if (nch > 1) gload(a1, b1, y1, 1);
    for (int ch = 0; ch < nch; ch += 2) {
      if (!chunk(a0, b0, y0, ch)) return false;
      if (ch + 1 < nch && !chunk(a1, b1, y1, ch + 1)) return false;
    }
    settle(0);
    settle(1);
    tc_fence_after();
    tmem_ld_row32(taddr, pr);
    if (fw && warp == 0) tmem_ld_row8(taddr + 32, tq);
    tc_fence_before();
  }
#pragma unroll
  for (int c = 0; c < 32; ++c)
    if (c >= bw) pr[c] = 0.f;
  __syncthreads();  // the chunks' operand buffers are no longer read

  // ---- diagonal block: factor (warp 0, rows in registers), inverse ----------
  if (first) {
    float* sT = sm + S::OFF_Y;
    if (warp == 0) {
      float a[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) a[c] = (lane < bw && c < bw) ? pr[c] : (c == lane ? 1.f : 0.f);
      float invo = 1.f, dv = 1.f;
      factor32(a, lane, sm + S::OFF_B, invo, dv);
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 32; ++c) sD[lane * 36 + c] = (c < lane) ? a[c] : (c == lane ? dv : 0.f);
      if (lane < bw) lgacc += logf(dv);
      if (fw) {
#pragma unroll
        for (int q = 0; q < 8; ++q) sT[lane * 8 + q] = (lane < bw && q < m) ? tq[q] : 0.f;
      }
    }
    __syncthreads();
    diag_tail<128>(p, Wm, K, j0, bw, sD, Li, sT, fw, ym);
  }

  // ---- X = P L_JJ^{-T}: P rows and L_JJ^{-1} as hi / lo operands ----------
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int o = (q * 128 + tid) * 4;
    split_store(make_float4(pr[4 * q], pr[4 * q + 1], pr[4 * q + 2], pr[4 * q + 3]), sm + S::PHI + o, sm + S::PLO + o);
  }
#pragma unroll
  for (int u = tid; u < 256; u += 128) {  // B row n = row n of L_JJ^{-1}
    const int n = u & 31, q = u >> 5, o = (q * 32 + n) * 4;
    split_store(*reinterpret_cast<const float4*>(Li + inv_off(n, 4 * q)), sm + S::IHI + o, sm + S::ILO + o);
  }
  fence_async_smem();
  if (__syncthreads_or(!ok)) return false;
  tc_fence_after();
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < 4; ++s)
      umma_3xtf32(tmem, kIdescX, sbase + (S::PHI + s * 1024) * 4, sbase + (S::PLO + s * 1024) * 4, 128 * 16,
                  sbase + (S::IHI + s * 256) * 4, sbase + (S::ILO + s * 256) * 4, 32 * 16, s ? 1u : 0u);
    umma_commit(bars + 2);
  }
  pend |= 4u;
  settle(2);
  tc_fence_after();
  float x[32];
  tmem_ld_row32(taddr, x);
  tc_fence_before();
  if (live && !(first && tid < 32)) {  // diagonal rows hold L_JJ already
    float* wr = Wm + (size_t)row * K + j0;
#pragma unroll
    for (int c4 = 0; c4 < 32; c4 += 4) {
      if (vec) {
        if (c4 < bw) *reinterpret_cast<float4*>(wr + c4) = make_float4(x[c4], x[c4 + 1], x[c4 + 2], x[c4 + 3]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (c4 + e < bw) wr[c4 + e] = x[c4 + e];
      }
    }
  }
  // slot writes, operand reads and tensor-memory reads are done before the next group
  return !__syncthreads_or(!ok);
}
}  // namespace

template <int NT, bool TC>
__global__ void __launch_bounds__(NT, 512 / NT) posv_blocked2_kernel(const PosvParams p, int mcb) {
  static_assert(!TC || NT == 128, "the tensor-core form runs 128 threads, one per accumulator row");
  using S = typename std::conditional<TC, B2TC, B2<NT>>::type;
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

  // tensor-core form: 64 columns of tensor memory (allocated by warp 0), three
  // mbarriers (chunk buffers 0 and 1, the X product)
  uint32_t tmem = 0, pend = 0, par = 0;
  if constexpr (TC) {
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + B2TC::OFF_BAR + 6);
    if (warp == 0) {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                   "n"(B2TC::TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
#pragma unroll
      for (int i = 0; i < 3; ++i)
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(sm + B2TC::OFF_BAR + 2 * i)));
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tmem = *tslot;
  }

  for (int64_t mat = blockIdx.x; mat < p.batch; mat += gridDim.x) {
    const float* A = p.A + mat * kk;
    float* Wm = p.L ? p.L + mat * kk : p.ws + (size_t)blockIdx.x * kk;
    float lgacc = 0.f;
    if constexpr (TC) {
      bool failed = false;
      if (p.tc_inject && blockIdx.x == 0 && mat == 0) {
        // test only: wait for the X barrier's next phase while nothing is
        // committed to it and no MMA is in flight; the wait runs out
        const bool okw =
            mbar_wait(reinterpret_cast<uint64_t*>(sm + B2TC::OFF_BAR) + 2, (par >> 2) & 1u, wait_limit_ns(p));
        failed = __syncthreads_or(!okw);
      }
      for (int J = 0; J < nblk && !failed; ++J)
        for (int rg = 32 * J; rg < K && !failed; rg += 128)
          failed = !panel_tc(p, A, Wm, K, 32 * J, rg, sm, vec, fwd, mat, lgacc, tmem, pend, par);
      if (failed) {  // the same in every thread
        // let MMAs committed before the timeout finish before the tensor
        // memory is freed (each wait bounded again), then mark this matrix
        // and every later one of this CTA unfinished: x and logdet NaN
        uint64_t* bars = reinterpret_cast<uint64_t*>(sm + B2TC::OFF_BAR);
        for (int i = 0; i < 3; ++i)
          if ((pend >> i) & 1u) mbar_wait(bars + i, (par >> i) & 1u, wait_limit_ns(p));
        pend = 0;
        const float qnan = __int_as_float(0x7fc00000);
        for (int64_t m2 = mat; m2 < p.batch; m2 += gridDim.x) {
          if (p.m > 0)
            for (int64_t e = tid; e < (int64_t)K * p.m; e += NT) p.x[(size_t)m2 * K * p.m + e] = qnan;
          if (p.logdet && tid == 0) p.logdet[m2] = qnan;
        }
        if (tid == 0) atomicOr(&g_blocked_fault, 1u);
        break;
      }
    }
    if constexpr (!TC) {
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
  if constexpr (TC) {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(B2TC::TMEM_COLS));
  }
}

// CTA size of the blocked tier (128: four CTAs per SM; 256: two).
constexpr int kBlockedNT = 128;

int blocked2_mcb(int k) {
  int mcb = (2 * B2<kBlockedNT>::A_FL) / (k > 0 ? k : 1);
  return mcb > MCB2 ? MCB2 : mcb;
}

// Panel GEMMs on FP32 FFMA, the faster form measured at k = 256 and 512;
// B2C_BLOCKED_GEMM=tc selects the tensor-core (3xTF32) form (read per call,
// so a test can flip it).
bool blocked2_tensor_cores() {
  const char* g = getenv("B2C_BLOCKED_GEMM");
  return g && strcmp(g, "tc") == 0;
}

size_t blocked2_smem_bytes(int k) {
  (void)k;
  const int fl = blocked2_tensor_cores() ? B2TC::SMEM : B2<kBlockedNT>::SMEM;
  return (size_t)fl * sizeof(float);
}

// B2C_BLOCKED_LEGACY=1 (read per call; tests and profiles) sends every k of the
// blocked tier to the earlier kernel of posv_blocked.cu, which otherwise serves
// only the k whose panel inverses do not fit here (above 9,216).
bool blocked2_fits(int k) {
  const char* t = getenv("B2C_BLOCKED_LEGACY");
  if (t && t[0] == '1') return false;
  return blocked2_mcb(k) >= 1;
}

int blocked2_ctas_per_sm() { return 512 / kBlockedNT; }

cudaError_t launch_posv_blocked2(const PosvParams& p, int grid, cudaStream_t s) {
  int occ = 0;
  cudaError_t e;
  const size_t smem = blocked2_smem_bytes(p.k);
  if (blocked2_tensor_cores()) {
    static int cache[64];
    auto kern = posv_blocked2_kernel<kBlockedNT, true>;
    e = kernel_occupancy(kern, kBlockedNT, smem, cache, &occ);
    if (e != cudaSuccess) return e;
    // test only (B2C_TC_INJECT_TIMEOUT=1, read per call): CTA 0 times out one
    // wait on purpose, every wait limited to 1 ms
    PosvParams q = p;
    const char* inj = getenv("B2C_TC_INJECT_TIMEOUT");
    q.tc_inject = (inj && inj[0] == '1') ? 1 : 0;
    kern<<<grid, kBlockedNT, smem, s>>>(q, blocked2_mcb(p.k));
  } else {
    static int cache[64];
    auto kern = posv_blocked2_kernel<kBlockedNT, false>;
    e = kernel_occupancy(kern, kBlockedNT, smem, cache, &occ);
    if (e != cudaSuccess) return e;
    kern<<<grid, kBlockedNT, smem, s>>>(p, blocked2_mcb(p.k));
  }
  return cudaGetLastError();
}

// Reads and clears the tensor-core kernel's fault flag (synchronises the
// device): nonzero when one of its mbarrier waits timed out.
cudaError_t blocked_take_fault(unsigned int* fault) {
  cudaError_t e = cudaMemcpyFromSymbol(fault, g_blocked_fault, sizeof(unsigned int));
  if (e != cudaSuccess) return e;
  const unsigned int zero = 0;
  return cudaMemcpyToSymbol(g_blocked_fault, &zero, sizeof(unsigned int));
}

}  // namespace b2c
