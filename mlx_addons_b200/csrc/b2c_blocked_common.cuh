// Device helpers shared by the CTA-per-matrix Cholesky tiers
// (posv_blocked2.cu, posv_smem.cu).
#pragma once

#include "b2c_common.cuh"

namespace b2c {

// Float offset of element q of row c of a 32 x 32 matrix whose 16-byte
// units are XOR-swizzled by the row: 8 consecutive rows read at the same q
// hit 8 different bank groups.
__device__ __forceinline__ int inv_off(int c, int q) { return c * 32 + (((q >> 2) ^ (c & 7)) << 2) + (q & 3); }

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

}  // namespace b2c
