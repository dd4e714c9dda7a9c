// b2c_posv_static_scratch: the blocked factor + solve without caller scratch.
//
// Some callers cannot allocate GPU memory at the point where they need a
// solve: code running under an allocator that forbids cudaMalloc during
// steady state, embedders whose memory is fully partitioned up front, and
// plugin hosts that hand a library nothing but its input and output buffers.
// b2c_posv needs a caller workspace for k > 64 (one k*k slot per resident
// CTA when L is not requested); this entry point takes its scratch from a
// fixed array inside the library instead and allocates nothing.
//
// The array is a file-scope __device__ variable of kStaticScratchBytes
// (16 MiB): every GPU on which the library's kernels are loaded holds it
// until the process exits. It bounds k at 2048 (one 2048 x 2048 float slot)
// and caps the number of matrices factored at the same time at
// 16 MiB / (4 k^2) (16 at k = 512), so large k run on fewer SMs than
// b2c_posv would use.
//
// Host code cannot pass the array's name to a kernel (in host code it is a
// host-side shadow, not a device address), so the first call on each device
// looks up the device address with cudaGetSymbolAddress, with that device
// current, and caches it; make that first call before any stream capture.
// All calls share the one array and leave their data in it. Nothing in it
// needs clearing: the kernel writes every scratch element before reading it.
// Calls that overlap on the GPU (different streams, or different host
// threads on the same device) race on the array; serialise them.
#include <mutex>

#include "b2c.h"
#include "b2c_kernels.cuh"

namespace {

constexpr size_t kStaticScratchBytes = 16u << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_static_scratch[kStaticScratchBytes / sizeof(float)];

std::mutex g_mu;
void* g_addr[kMaxDevices] = {nullptr};
int g_sms[kMaxDevices] = {0};

int fail(int code, const char* msg) { return b2c::set_error(code, msg); }

}  // namespace

extern "C" int b2c_posv_static_scratch(const float* A, const float* b, float* x, float* logdet, int64_t batch,
                                       int k, int m, void* stream) {
  if (batch < 0 || k < 1 || m < 0) return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_posv_static_scratch: bad size");
  const size_t slot = (size_t)k * k * sizeof(float);
  if (slot > kStaticScratchBytes)
    return fail(B2C_ERR_UNSUPPORTED,
                "b2c_posv_static_scratch: k exceeds 2048, the largest matrix its 16 MiB scratch array holds");
  if (batch == 0) return fail(B2C_OK, "");
  if (!A || (m > 0 && (!b || !x)))
    return fail(B2C_ERR_INVALID_ARGUMENT, "b2c_posv_static_scratch: A, b and x must be non-NULL");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(B2C_ERR_CUDA, "b2c_posv_static_scratch: no current CUDA device");
  void* addr;
  int sms;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[dev]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
      if (e != cudaSuccess) return fail(B2C_ERR_CUDA, "b2c_posv_static_scratch: cudaGetSymbolAddress failed");
      int n = 0;
      e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return fail(B2C_ERR_CUDA, "b2c_posv_static_scratch: device query failed");
      g_sms[dev] = n;
      g_addr[dev] = p;
    }
    addr = g_addr[dev];
    sms = g_sms[dev];
  }
  b2c::PosvParams p;
  p.A = A;
  p.b = b;
  p.x = x;
  p.L = nullptr;
  p.logdet = logdet;
  p.ws = static_cast<float*>(addr);
  p.batch = batch;
  p.k = k;
  p.m = m;
  p.vec = ((reinterpret_cast<uintptr_t>(A) & 15u) == 0) ? 1 : 0;
  int grid = b2c::blocked_grid(batch, k, sms);
  const int slots = (int)(kStaticScratchBytes / slot);
  if (grid > slots) grid = slots;  // one scratch slot per resident CTA
  cudaError_t e = b2c::launch_posv_blocked(p, grid, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(B2C_ERR_CUDA, "b2c_posv_static_scratch: kernel launch failed");
  return fail(B2C_OK, "");
}
