// Kernel launchers shared between the translation units of libb2c.
#pragma once

#include "b2c_common.cuh"

namespace b2c {

// k <= 64: thread tier (k <= 16), posv_warp.cu; segments of 8 / 16 lanes
// per matrix (17..32, and k = 16 with m >= 4), posv_seg.cu; 33..64: the 2-D
// tile tier (posv_tile.cu) and the two-rows-per-lane warp tier (posv_warp64.cu,
// m >= 2 or an L output).
cudaError_t launch_posv_small(const PosvParams& p, int sm_count, cudaStream_t s);
cudaError_t launch_posv_warp64(const PosvParams& p, int sm_count, cudaStream_t s);
// One matrix per warp on a 2-D cyclic layout for 33..64 with m <= 1 and no L
// output, posv_tile.cu; B2C_TILE_TIER=0 (read per call) routes those calls to
// the two-rows-per-lane kernel of posv_warp64.cu.
bool posv_tile_applies(const PosvParams& p);
cudaError_t launch_posv_tile(const PosvParams& p, int sm_count, cudaStream_t s);
// Segmented form of the two-rows-per-lane design for k <= 32: 8 lanes per
// matrix for k <= 16, 16 lanes for 17..32. posv_seg.cu
cudaError_t launch_posv_seg(const PosvParams& p, int sm_count, cudaStream_t s);

// k > 64 (any k >= 1 accepted): blocked CTA-per-matrix tier. posv_blocked.cu
int blocked_grid(int64_t batch, int k, int sm_count);
cudaError_t launch_posv_blocked(const PosvParams& p, int grid, cudaStream_t s);

// Register-tiled blocked tier used by launch_posv_blocked whenever its
// per-panel inverses fit shared memory (k up to about 1,440). posv_blocked2.cu
bool blocked2_fits(int k);
int blocked2_ctas_per_sm();
// Whether blocked2 runs its panel GEMMs on the tensor cores (B2C_BLOCKED_GEMM=tc).
bool blocked2_tensor_cores();
// Shared-memory tier (posv_smem.cu): the whole lower triangle of one matrix
// in one CTA's shared memory, k <= 256, any m; used by launch_posv_blocked
// unless B2C_SMEM_TIER=0. Needs no scratch.
bool smem_tier_enabled();
bool smem_tier_fits(int k, int m);
cudaError_t launch_posv_smem(const PosvParams& p, cudaStream_t s);
// Task-graph form of the shared-memory tier (posv_dag.cu): by default
// 193 <= k <= 256 with m <= 8, and 65 <= k <= 160 with 2 <= m <= 8 (every
// 65 <= k <= 256, m <= 8 with B2C_SMEM_DAG=all); k % 4 == 0, A in device
// memory; launch_posv_smem takes it whenever it applies.
bool posv_dag_applies(const PosvParams& p);
cudaError_t launch_posv_dag(const PosvParams& p, cudaStream_t s);
// Reads and clears the task-graph kernel's fault flag (ORed into *fault).
cudaError_t dag_take_fault(unsigned int* fault);
// Reads and clears the tensor-core blocked kernel's fault flag.
cudaError_t blocked_take_fault(unsigned int* fault);
cudaError_t launch_posv_blocked2(const PosvParams& p, int grid, cudaStream_t s);

// Triangular solves, any k. posv_blocked.cu
cudaError_t launch_trsm(const TrsmParams& p, int sm_count, cudaStream_t s);

// slogdet, any n. lu.cu
int slogdet_grid(int64_t batch, int n, int sm_count);
size_t slogdet_ws_floats(int64_t batch, int n, int sm_count);
cudaError_t launch_slogdet(const SlogdetParams& p, int sm_count, cudaStream_t s);

// solve_lu (partial-pivot LU solve), k <= kGesvMaxK. lu_solve.cu
constexpr int kGesvMaxK = 4096;
int gesv_grid(int64_t batch, int k, int sm_count);
size_t gesv_ws_floats(int64_t batch, int k, int sm_count);
cudaError_t launch_gesv(const GesvParams& p, int sm_count, cudaStream_t s);
// Blocked LU solve on a per-CTA scratch slot (k x k floats), lu.cu; used by
// launch_gesv for kGesvSmemMaxK < k <= 864.
bool gesv_blocked_fits(int k);
int gesv_blocked_grid(int64_t batch, int k, int sm_count);
cudaError_t launch_gesv_blocked(const GesvParams& p, int grid, cudaStream_t s);

// qr (Householder, Q formed explicitly), k <= kQrMaxK. qr.cu
constexpr int kQrMaxK = 4096;
int qr_grid(int64_t batch, int k, int sm_count);
size_t qr_ws_floats(int64_t batch, int k, int sm_count);
cudaError_t launch_qr(const QrParams& p, int sm_count, cudaStream_t s);

// Sets this thread's b2c_last_error() message; returns code. abi.cu
int set_error(int code, const char* msg);

}  // namespace b2c
