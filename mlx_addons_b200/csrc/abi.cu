// extern "C" boundary of libb2c (declared in include/b2c.h).
//
// Validates arguments, picks the tier for (k, m) and launches on the caller's
// stream. No entry point allocates, synchronises or throws; errors come back
// as status codes with a per-thread message.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "b2c.h"
#include "b2c_kernels.cuh"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = '\0';
  return B2C_OK;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(B2C_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};

// SM count of the current device (cached; a benign race writes equal values).
cudaError_t sm_count_current(int* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < kMaxDevices && g_sm_count[dev] > 0) {
    *out = g_sm_count[dev];
    return cudaSuccess;
  }
  int n = 0;
  e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < kMaxDevices) g_sm_count[dev] = n;
  *out = n;
  return cudaSuccess;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Tier override for testing and tuning: B2C_TIER=blocked routes every k to
// the blocked tier (read per call, so a test can flip it).
bool force_blocked() {
  const char* t = getenv("B2C_TIER");
  return t && strcmp(t, "blocked") == 0;
}

bool uses_blocked(int k) { return k > 64 || force_blocked(); }

// The blocked path keeps its factor in a caller workspace unless the
// shared-memory tier takes the call (k <= 256), which needs none. Both the
// size query and the call evaluate this in the same way (the tier switches
// are read per call).
bool posv_needs_workspace(int k, int m) {
  if (!uses_blocked(k)) return false;
  return !(b2c::smem_tier_enabled() && !b2c::blocked2_tensor_cores() && b2c::smem_tier_fits(k, m));
}

constexpr int kMaxK = 1 << 16;

}  // namespace

namespace b2c {
// Records `msg` as this thread's b2c_last_error() message and returns `code`
// (used by entry points defined in other translation units).
int set_error(int code, const char* msg) {
  if (code == B2C_OK) return ok();
  return fail(code, "%s", msg);
}
}  // namespace b2c

extern "C" {

int b2c_version(void) { return (0 << 16) | (1 << 8) | 0; }

int b2c_host_device_pointer(const void* host_ptr, void** device_ptr) {
  if (!device_ptr) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_host_device_pointer: device_ptr is NULL");
  *device_ptr = nullptr;
  if (!host_ptr) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_host_device_pointer: host_ptr is NULL");
  void* d = nullptr;
  cudaError_t e = cudaHostGetDevicePointer(&d, const_cast<void*>(host_ptr), 0);
  if (e != cudaSuccess) {
    cudaGetLastError();  // not mapped host memory: clear the sticky-free error
    return fail(B2C_ERR_CUDA, "b2c_host_device_pointer: not pinned mapped host memory (%s)", cudaGetErrorName(e));
  }
  *device_ptr = d;
  return ok();
}

const char* b2c_last_error(void) { return g_err; }

int b2c_take_device_fault(unsigned int* fault) {
  if (!fault) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_take_device_fault: fault is NULL");
  *fault = 0;
  cudaError_t e = b2c::blocked_take_fault(fault);
  if (e == cudaSuccess) e = b2c::dag_take_fault(fault);
  if (e != cudaSuccess) return cuda_fail(e, "b2c_take_device_fault");
  return ok();
}

size_t b2c_workspace_size(int op, int64_t batch, int k, int m) {
  (void)m;
  if (batch <= 0 || k <= 0 || k > kMaxK) return 0;
  int sm = 0;
  if (sm_count_current(&sm) != cudaSuccess) return 0;
  switch (op) {
    case B2C_OP_POSV:
    case B2C_OP_POTRF:
      if (!posv_needs_workspace(k, op == B2C_OP_POTRF ? 0 : m)) return 0;
      return (size_t)b2c::blocked_grid(batch, k, sm) * (size_t)k * k * sizeof(float);
    case B2C_OP_SLOGDET:
      return b2c::slogdet_ws_floats(batch, k, sm) * sizeof(float);
    case B2C_OP_GESV:
      return b2c::gesv_ws_floats(batch, k, sm) * sizeof(float);
    case B2C_OP_QR:
      return b2c::qr_ws_floats(batch, k, sm) * sizeof(float);
    default:
      return 0;
  }
}

static int posv_impl(const float* A, const float* b, float* x, float* L, float* logdet, int64_t batch, int k,
                     int m, void* workspace, size_t workspace_bytes, void* stream, const char* name) {
  if (batch < 0) return fail(B2C_ERR_INVALID_ARGUMENT, "%s: batch must be >= 0 (got %lld)", name, (long long)batch);
  if (k < 1) return fail(B2C_ERR_INVALID_ARGUMENT, "%s: k must be >= 1 (got %d)", name, k);
  if (k > kMaxK) return fail(B2C_ERR_UNSUPPORTED, "%s: k = %d exceeds %d", name, k, kMaxK);
  if (m < 0) return fail(B2C_ERR_INVALID_ARGUMENT, "%s: m must be >= 0 (got %d)", name, m);
  if (batch == 0) return ok();
  if (!A) return fail(B2C_ERR_INVALID_ARGUMENT, "%s: A is NULL", name);
  if (m > 0 && (!b || !x)) return fail(B2C_ERR_INVALID_ARGUMENT, "%s: b and x must be non-NULL when m > 0", name);
  int sm = 0;
  cudaError_t e = sm_count_current(&sm);
  if (e != cudaSuccess) return cuda_fail(e, name);

  b2c::PosvParams p{};
  p.A = A;
  p.b = b;
  p.x = x;
  p.L = L;
  p.logdet = logdet;
  p.ws = static_cast<float*>(workspace);
  p.batch = batch;
  p.k = k;
  p.m = m;
  p.vec = aligned16(A) && (!L || aligned16(L)) && (!workspace || aligned16(workspace));
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  if (uses_blocked(k)) {
    const int grid = b2c::blocked_grid(batch, k, sm);
    if (!L && posv_needs_workspace(k, m)) {
      const size_t need = (size_t)grid * (size_t)k * k * sizeof(float);
      if (!workspace || workspace_bytes < need)
        return fail(B2C_ERR_WORKSPACE, "%s: k = %d needs %zu workspace bytes (got %zu)", name, k, need,
                    workspace ? workspace_bytes : (size_t)0);
    }
    e = b2c::launch_posv_blocked(p, grid, s);
  } else {
    e = b2c::launch_posv_small(p, sm, s);
  }
  if (e != cudaSuccess) return cuda_fail(e, name);
  return ok();
}

int b2c_posv(const float* A, const float* b, float* x, float* L, float* logdet, int64_t batch, int k, int m,
             void* workspace, size_t workspace_bytes, void* stream) {
  return posv_impl(A, b, x, L, logdet, batch, k, m, workspace, workspace_bytes, stream, "b2c_posv");
}

int b2c_potrf(const float* A, float* L, float* logdet, int64_t batch, int k, void* workspace,
              size_t workspace_bytes, void* stream) {
  if (!L && !logdet && batch > 0)
    return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_potrf: at least one of L and logdet must be non-NULL");
  return posv_impl(A, nullptr, nullptr, L, logdet, batch, k, 0, workspace, workspace_bytes, stream, "b2c_potrf");
}

int b2c_trsm(const float* L, const float* b, float* x, int64_t batch, int k, int m, int transpose, void* stream) {
  if (batch < 0) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_trsm: batch must be >= 0");
  if (k < 1) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_trsm: k must be >= 1 (got %d)", k);
  if (k > kMaxK) return fail(B2C_ERR_UNSUPPORTED, "b2c_trsm: k = %d exceeds %d", k, kMaxK);
  if (m < 0) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_trsm: m must be >= 0");
  if (transpose != 0 && transpose != 1) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_trsm: transpose must be 0 or 1");
  if (batch == 0 || m == 0) return ok();
  if (!L || !b || !x) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_trsm: L, b and x must be non-NULL");
  int sm = 0;
  cudaError_t e = sm_count_current(&sm);
  if (e != cudaSuccess) return cuda_fail(e, "b2c_trsm");
  b2c::TrsmParams p;
  p.L = L;
  p.b = b;
  p.x = x;
  p.batch = batch;
  p.k = k;
  p.m = m;
  p.transpose = transpose;
  e = b2c::launch_trsm(p, sm, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "b2c_trsm");
  return ok();
}

int b2c_slogdet(const float* A, float* sign, float* logabsdet, int64_t batch, int n, void* workspace,
                size_t workspace_bytes, void* stream) {
  if (batch < 0) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_slogdet: batch must be >= 0");
  if (n < 1) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_slogdet: n must be >= 1 (got %d)", n);
  if (n > kMaxK) return fail(B2C_ERR_UNSUPPORTED, "b2c_slogdet: n = %d exceeds %d", n, kMaxK);
  if (batch == 0) return ok();
  if (!A) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_slogdet: A is NULL");
  if (!sign && !logabsdet) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_slogdet: both outputs are NULL");
  int sm = 0;
  cudaError_t e = sm_count_current(&sm);
  if (e != cudaSuccess) return cuda_fail(e, "b2c_slogdet");
  const size_t need = b2c::slogdet_ws_floats(batch, n, sm) * sizeof(float);
  if (need && (!workspace || workspace_bytes < need))
    return fail(B2C_ERR_WORKSPACE, "b2c_slogdet: n = %d needs %zu workspace bytes (got %zu)", n, need,
                workspace ? workspace_bytes : (size_t)0);
  b2c::SlogdetParams p;
  p.A = A;
  p.sign = sign;
  p.logabsdet = logabsdet;
  p.ws = static_cast<float*>(workspace);
  p.batch = batch;
  p.n = n;
  e = b2c::launch_slogdet(p, sm, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "b2c_slogdet");
  return ok();
}

int b2c_gesv(const float* A, const float* b, float* x, int64_t batch, int k, int m, void* workspace,
             size_t workspace_bytes, void* stream) {
  if (batch < 0) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_gesv: batch must be >= 0");
  if (k < 1) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_gesv: k must be >= 1 (got %d)", k);
  if (k > b2c::kGesvMaxK) return fail(B2C_ERR_UNSUPPORTED, "b2c_gesv: k = %d exceeds %d", k, b2c::kGesvMaxK);
  if (m < 0) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_gesv: m must be >= 0 (got %d)", m);
  if (batch == 0 || m == 0) return ok();
  if (!A || !b || !x) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_gesv: A, b and x must be non-NULL");
  if (b == x) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_gesv: x may not alias b");
  int sm = 0;
  cudaError_t e = sm_count_current(&sm);
  if (e != cudaSuccess) return cuda_fail(e, "b2c_gesv");
  const size_t need = b2c::gesv_ws_floats(batch, k, sm) * sizeof(float);
  if (need && (!workspace || workspace_bytes < need))
    return fail(B2C_ERR_WORKSPACE, "b2c_gesv: k = %d needs %zu workspace bytes (got %zu)", k, need,
                workspace ? workspace_bytes : (size_t)0);
  b2c::GesvParams p;
  p.A = A;
  p.b = b;
  p.x = x;
  p.ws = static_cast<float*>(workspace);
  p.batch = batch;
  p.k = k;
  p.m = m;
  e = b2c::launch_gesv(p, sm, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "b2c_gesv");
  return ok();
}

int b2c_qr(const float* A, float* Q, float* R, int64_t batch, int k, void* workspace, size_t workspace_bytes,
           void* stream) {
  if (batch < 0) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_qr: batch must be >= 0");
  if (k < 1) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_qr: k must be >= 1 (got %d)", k);
  if (k > b2c::kQrMaxK) return fail(B2C_ERR_UNSUPPORTED, "b2c_qr: k = %d exceeds %d", k, b2c::kQrMaxK);
  if (batch == 0) return ok();
  if (!A || !Q || !R) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_qr: A, Q and R must be non-NULL");
  if (Q == R) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_qr: Q and R must be distinct");
  int sm = 0;
  cudaError_t e = sm_count_current(&sm);
  if (e != cudaSuccess) return cuda_fail(e, "b2c_qr");
  const size_t need = b2c::qr_ws_floats(batch, k, sm) * sizeof(float);
  if (need && (!workspace || workspace_bytes < need))
    return fail(B2C_ERR_WORKSPACE, "b2c_qr: k = %d needs %zu workspace bytes (got %zu)", k, need,
                workspace ? workspace_bytes : (size_t)0);
  b2c::QrParams p;
  p.A = A;
  p.Q = Q;
  p.R = R;
  p.ws = static_cast<float*>(workspace);
  p.batch = batch;
  p.k = k;
  e = b2c::launch_qr(p, sm, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "b2c_qr");
  return ok();
}

}  // extern "C"
