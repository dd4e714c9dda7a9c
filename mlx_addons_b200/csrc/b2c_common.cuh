// Shared device helpers for the b2c kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b2c {

// Pivot clamp of the reference: L_jj = sqrt(max(s, 1e-12))
// (src/mlx_addons/linalg/_metal_kernels.py:42, :168).
constexpr float kClamp = 1e-12f;
constexpr unsigned kFull = 0xffffffffu;

struct PosvParams {
  const float* A;      // (batch, k, k)
  const float* b;      // (batch, k, m) or null when m == 0
  float* x;            // (batch, k, m) or null when m == 0
  float* L;            // (batch, k, k) or null
  float* logdet;       // (batch,) or null
  float* ws;           // scratch (blocked tier without L), slot per CTA
  int64_t batch;
  int k;
  int m;
  int vec;             // 1 when A/L/b/x allow 16-byte vector access
  int tc_inject;       // test only: the tensor-core blocked kernel times out one wait (0 otherwise)
};

struct TrsmParams {
  const float* L;
  const float* b;
  float* x;
  int64_t batch;
  int k;
  int m;
  int transpose;       // 0: L x = b, 1: L^T x = b
};

struct GesvParams {
  const float* A;
  const float* b;
  float* x;
  float* ws;           // scratch for matrices that do not fit shared memory
  int64_t batch;
  int k;
  int m;
};

struct QrParams {
  const float* A;
  float* Q;
  float* R;
  float* ws;           // scratch for matrices that do not fit shared memory
  int64_t batch;
  int k;
};

struct SlogdetParams {
  const float* A;
  float* sign;
  float* logabsdet;
  float* ws;           // scratch for matrices that do not fit shared memory
  int64_t batch;
  int n;
};

// 1 / sqrt(max(s, clamp)) refined by one Newton step; d receives the square
// root itself. Relative error about 1 ulp, the same order as IEEE sqrt + div.
__device__ __forceinline__ float clamped_rsqrt(float s, float& d) {
  const float sc = fmaxf(s, kClamp);
  float r = rsqrtf(sc);
  r = r * fmaf(-0.5f * sc * r, r, 1.5f);
  d = sc * r;
  return r;
}

// sum_j log(d[j]) for N Cholesky diagonals, each a positive normal float
// (the clamp keeps them >= 1e-6) or NaN (non-finite input): one log of the
// product of the mantissas in [1, 2), plus ln 2 times the sum of the
// exponents. The product of at most 16 mantissas stays below 2^16, so
// nothing is renormalised; it carries N - 1 roundings, the same order as a
// sum of N separately rounded logs, at the cost of one logf instead of N.
// A NaN diagonal makes the result NaN, as the sum of logs would.
template <int N>
__device__ __forceinline__ float sum_log_pos(const float (&d)[N]) {
  static_assert(N >= 1 && N <= 16, "mantissa product bound");
  float mant = 1.f, nan_carry = 0.f;
  int ex = 0;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const uint32_t bits = __float_as_uint(d[j]);
    ex += (int)(bits >> 23) - 127;
    mant *= __uint_as_float((bits & 0x007fffffu) | 0x3f800000u);
    nan_carry = fmaf(d[j], 0.f, nan_carry);
  }
  return fmaf((float)ex, 0.69314718055994531f, logf(mant)) + nan_carry;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Two float32 lanes in one 64-bit register pair, for the packed
// fma.rn.f32x2 / mul.rn.f32x2 instructions (one issue slot for two FMAs).
typedef unsigned long long u64;

__device__ __forceinline__ u64 pk2(float lo, float hi) {
  u64 r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float lo2(u64 v) {
  float lo, hi;
  asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo;
}
__device__ __forceinline__ float hi2(u64 v) {
  float lo, hi;
  asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return hi;
}
// d = a * b + c, two lanes of float32 at once.
__device__ __forceinline__ u64 ffma2(u64 a, u64 b, u64 c) {
  u64 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ u64 fmul2(u64 a, u64 b) {
  u64 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ void lds128(const float* p, u64& x, u64& y) {
  asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "r"(smem_u32(p)));
}
__device__ __forceinline__ u64 lds64(const float* p) {
  u64 x;
  asm volatile("ld.shared.b64 %0, [%1];" : "=l"(x) : "r"(smem_u32(p)));
  return x;
}

__device__ __forceinline__ void sts128(float* p, u64 x, u64 y) {
  asm volatile("st.shared.v2.b64 [%0], {%1, %2};" ::"r"(smem_u32(p)), "l"(x), "l"(y) : "memory");
}

// Element c of a packed row.
template <int N>
__device__ __forceinline__ float getc(const u64 (&a)[N], int c) {
  return (c & 1) ? hi2(a[c >> 1]) : lo2(a[c >> 1]);
}
template <int N>
__device__ __forceinline__ void setc(u64 (&a)[N], int c, float v) {
  a[c >> 1] = (c & 1) ? pk2(lo2(a[c >> 1]), v) : pk2(v, hi2(a[c >> 1]));
}



// Ampere-style asynchronous global->shared copies (LDGSTS). They need no
// registers and accept any destination layout, which the padded
// bank-conflict-free staging layouts below rely on.
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// 3xTF32 split: hi keeps the top 10 mantissa bits (what a TF32 operand
// carries), lo = x - hi exactly; a*b ~ hi*hi + hi*lo + lo*hi to about fp32
// accuracy.
__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  const uint32_t h = __float_as_uint(x) & 0xffffe000u;
  hi = h;
  lo = __float_as_uint(x - __uint_as_float(h));
}
// d += a * b on the tensor cores: a 16 x 8 (row), b 8 x 8 (col), TF32 in, FP32 accumulate.
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float warp_sum(float v, int width = 32) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    if (o < width) v += __shfl_xor_sync(kFull, v, o, width);
  return v;
}

// Opt a kernel into the device's full dynamic shared memory once per device
// and cache its occupancy for `threads` threads and `smem` bytes, so that
// launches made later (including inside CUDA graph capture) issue no
// attribute calls. `cache` is a per-kernel array indexed by device.
template <typename Kern>
__host__ cudaError_t kernel_occupancy(Kern kern, int threads, size_t smem, int* cache, int* occ) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && cache[dev] > 0) {
    *occ = cache[dev];
    return cudaSuccess;
  }
  int optin = 0;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
  cudaFuncAttributes fa;
  e = cudaFuncGetAttributes(&fa, kern);
  if (e != cudaSuccess) return e;
  // static + dynamic shared memory may not exceed the opt-in limit
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
  if (e != cudaSuccess) return e;
  int o = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kern, threads, smem);
  if (e != cudaSuccess) return e;
  if (o < 1) o = 1;
  if (dev >= 0 && dev < 64) cache[dev] = o;
  *occ = o;
  return cudaSuccess;
}

}  // namespace b2c
