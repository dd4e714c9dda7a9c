/*
 * b2c — batched SPD Cholesky solve for NVIDIA B200 (sm_100a), C ABI.
 *
 * Drop-in boundary for the batched linear-algebra path of
 * guillaume-osmo/mlx-addons (`mlx_addons.linalg`). Every entry point:
 *   - takes plain pointers and sizes; array pointers are DEVICE pointers owned
 *     by the caller (inputs and outputs on the current CUDA device);
 *   - enqueues its kernels on the given stream (a cudaStream_t passed as
 *     void*; NULL = the legacy default stream) and returns without
 *     synchronising;
 *   - returns B2C_OK or an error code and never throws; b2c_last_error()
 *     gives a message for the calling thread;
 *   - allocates nothing: scratch, where an operation needs it, is a caller
 *     buffer sized by b2c_workspace_size().
 *
 * Layouts are those of the reference: float32, row-major, contiguous,
 * A / L of shape (batch, k, k), right-hand sides of shape (batch, k, m).
 * Semantics follow the reference bit for bit where it defines them:
 *   - only the lower triangle of A (and of L) is read;
 *   - a non-positive pivot s is clamped, L_jj = sqrt(max(s, 1e-12)), so no
 *     NaN is produced for non-SPD input (_metal_kernels.py:42,90,168,228);
 *   - the upper triangle of an L output is zeroed (_metal_kernels.py:98-99);
 *   - transpose=1 in b2c_trsm solves L^T x = b with the LOWER factor
 *     (_metal_kernels.py:617-638).
 * Paths cited below are relative to the reference project root.
 */
#ifndef B2C_H_
#define B2C_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define B2C_OK 0
#define B2C_ERR_INVALID_ARGUMENT 1 /* null pointer, negative size, bad flag */
#define B2C_ERR_UNSUPPORTED 2      /* a size this build does not handle */
#define B2C_ERR_WORKSPACE 3        /* workspace missing or too small */
#define B2C_ERR_CUDA 4             /* a CUDA runtime call or launch failed */

/* Operation ids for b2c_workspace_size. */
#define B2C_OP_POSV 0
#define B2C_OP_POTRF 1
#define B2C_OP_TRSM 2
#define B2C_OP_SLOGDET 3
#define B2C_OP_GESV 4
#define B2C_OP_QR 5

/* Library version, (major << 16) | (minor << 8) | patch. */
int b2c_version(void);

/* Message of the last failing call made by this host thread ("" if none). */
const char *b2c_last_error(void);

/* Bytes of scratch `op` needs for (batch, k, m) with L not requested; 0 when
 * the operation runs entirely out of registers and shared memory (b2c_posv /
 * b2c_potrf for k <= 256, the register and shared-memory tiers). Scratch
 * contents need no initialisation. */
size_t b2c_workspace_size(int op, int64_t batch, int k, int m);

/* Fused Cholesky factorisation + forward + back substitution, x = A^{-1} b,
 * with optional factor and log-determinant outputs; one pass over A.
 *   A      (batch, k, k)  input, lower triangle read
 *   b      (batch, k, m)  input (a (batch, k) vector is m = 1)
 *   x      (batch, k, m)  output; may alias b
 *   L      (batch, k, k)  optional output (NULL = not written), upper zeroed
 *   logdet (batch,)       optional output, 2 * sum(log(diag L))
 * Replaces: mlx_addons.linalg.solve = blocked_solve
 *           (src/mlx_addons/linalg/__init__.py:48, _blocked.py:140-217),
 *           solve_cholesky = _metal_kernels.solve (_metal_kernels.py:536-559,
 *           :972), and the L / logdet of cholesky + logdet_spd on the same A
 *           (__init__.py:49, _det.py:100-113) in the same pass.
 * The reference's k <= 128 limit of solve_cholesky is lifted: any k >= 1. */
int b2c_posv(const float *A, const float *b, float *x, float *L, float *logdet,
             int64_t batch, int k, int m, void *workspace, size_t workspace_bytes,
             void *stream);

/* Cholesky factorisation with optional outputs; at least one of L / logdet.
 * Replaces: mlx_addons.linalg.cholesky = blocked_cholesky
 *           (src/mlx_addons/linalg/__init__.py:49, _blocked.py:34-137,
 *           _metal_kernels.py:562-590) with L != NULL, and logdet_spd
 *           (_det.py:51-67, :100-113) with L == NULL. */
int b2c_potrf(const float *A, float *L, float *logdet, int64_t batch, int k,
              void *workspace, size_t workspace_bytes, void *stream);

/* Triangular solve with a lower-triangular L (lower triangle incl. diagonal
 * read, division by the diagonal): transpose = 0 solves L x = b,
 * transpose = 1 solves L^T x = b. x may alias b.
 * Replaces: tril_solve (src/mlx_addons/linalg/_metal_kernels.py:593-614) and
 *           triu_solve (_metal_kernels.py:617-638); the reference's
 *           k <= 128 assertion (:596, :620) is lifted. */
int b2c_trsm(const float *L, const float *b, float *x, int64_t batch, int k,
             int m, int transpose, void *stream);

/* Sign and log|det| of general square matrices through LU with partial
 * pivoting (first maximal |a_ij| as pivot): sign = (-1)^{#swaps} *
 * prod sign(U_jj), logabsdet = sum log|U_jj|; a zero pivot gives sign 0 and
 * logabsdet -inf. Either output may be NULL.
 * Replaces: slogdet / det (src/mlx_addons/linalg/_det.py:17-48, :70-97),
 *           which run LAPACK getrf on the CPU stream (_det.py:30). */
int b2c_slogdet(const float *A, float *sign, float *logabsdet, int64_t batch,
                int n, void *workspace, size_t workspace_bytes, void *stream);

/* A x = b for general square A through LU with partial pivoting: the pivot
 * of column j is the first row whose |a_ij| exceeds a running maximum that
 * starts at 0 (an all-zero column keeps row j), rows are swapped when the
 * pivot row differs, a non-zero pivot's column is scaled by its reciprocal
 * and the trailing matrix updated; each right-hand side is permuted, forward
 * substituted (unit lower) and back substituted dividing by U_ii, so a
 * singular U yields inf / NaN in x like the reference. x may not alias b.
 *   A (batch, k, k), b (batch, k, m), x (batch, k, m)
 * Replaces: solve_lu (src/mlx_addons/linalg/_metal_kernels.py:917-969,
 *           kernels _LU_SOLVE_SRC :701-768, _LU_SOLVE_LG_SRC :849-914);
 *           the reference's k <= 128 assertion (:932) is raised to
 *           k <= 4096 (B2C_ERR_UNSUPPORTED above). */
int b2c_gesv(const float *A, const float *b, float *x, int64_t batch, int k,
             int m, void *workspace, size_t workspace_bytes, void *stream);

/* Householder QR of square matrices, A = Q R with Q formed explicitly.
 * Column j's reflector: norm = sqrt(max(sum_{i>=j} r_ij^2, 1e-30)),
 * v = (r_jj + s norm, r_{j+1,j}, ...), s = +1 if r_jj >= 0 else -1,
 * tau = 2 / v.v (0 if v.v <= 1e-30); r_jj becomes -s norm. For k > 63 a
 * column with an exactly zero sub-diagonal part is left as it is (tau = 0),
 * as LAPACK's reflector generator does.
 *   A (batch, k, k) input; Q, R (batch, k, k) outputs (R upper triangular)
 * Replaces: qr (src/mlx_addons/linalg/_metal_kernels.py:641-694; kernels
 *           _QR_SRC :319-381 for k < 12, _QR_TG_SRC :385-473 for
 *           12 <= k <= 63, CPU LAPACK :685-688 above). k <= 4096. */
int b2c_qr(const float *A, float *Q, float *R, int64_t batch, int k,
           void *workspace, size_t workspace_bytes, void *stream);

/* Device-accessible address of pinned, mapped host memory (the address a
 * kernel may dereference; equal to host_ptr under unified addressing).
 * Returns B2C_ERR_CUDA, leaving *device_ptr NULL, when host_ptr is not
 * page-locked and mapped, so a caller can decide between passing host buffers
 * straight to b2c_posv / b2c_potrf / b2c_slogdet (the kernels then read and
 * write them across PCIe) and staging them through device memory.
 * Plumbing for the host-buffer path; no counterpart in the reference, whose
 * arrays live in unified memory. */
int b2c_host_device_pointer(const void *host_ptr, void **device_ptr);

/* Reads and clears the device fault flags of this library on the current
 * device (synchronises it): *fault = 0 when every kernel finished its work;
 * nonzero = a CTA gave up on a bounded wait (one second) and left the matrix
 * it was on and every later matrix of that CTA (batch indices i, i + grid,
 * ...) unfinished: their x and logdet are NaN, their L incomplete (NaN from
 * the task-graph kernel). Two kernels wait at all, each only on mbarriers of
 * its own CTA: the tensor-core form of the blocked tier (b2c_posv /
 * b2c_potrf / b2c_posv_static_scratch for k > 64 with B2C_BLOCKED_GEMM=tc)
 * and the task-graph form of the shared-memory tier (65 <= k <= 256). Such a
 * kernel still returns normally (no fault, no hang).
 * Failure detection; no counterpart in the reference. */
int b2c_take_device_fault(unsigned int *fault);

/* b2c_posv without caller scratch: the same fused factor + solve (+ logdet)
 * as b2c_posv with L = NULL, for callers that cannot allocate GPU memory when
 * they solve (no cudaMalloc under their allocator, memory partitioned up
 * front, or a plugin host that passes only input and output buffers). Its
 * scratch is a 16 MiB array inside the library, held on every GPU that loads
 * the library until exit: k is limited to 2048 (larger k returns
 * B2C_ERR_UNSUPPORTED) and at most 16 MiB / (4 k^2) matrices are factored
 * at a time. Each call outside stream capture looks up the array's device
 * address in the current context; a call during capture reuses the address
 * of the last call in the same context, so make one call per device and
 * context before capturing (B2C_ERR_CUDA otherwise). All calls share the
 * array: calls that overlap on the GPU race and must be serialised.
 * This entry point has no counterpart in the reference. */
int b2c_posv_static_scratch(const float *A, const float *b, float *x, float *logdet,
                            int64_t batch, int k, int m, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* B2C_H_ */
