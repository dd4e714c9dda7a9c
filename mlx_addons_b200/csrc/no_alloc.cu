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
// host-side shadow, not a device address). A device address is valid only
// in the context that looked it up, so every call made outside stream
// capture looks it up again with cudaGetSymbolAddress in the current
// context (a cheap host call, which also keeps the address right after the
// device was reset or another context was made current) and records it for
// that context; a call made during stream capture, where the lookup is not
// allowed, uses the address recorded for the current context and fails with
// B2C_ERR_CUDA if there is none, so make one call per device and context
// before capturing. All calls share the one array and leave their data in
// it. Nothing in it needs clearing: the kernel writes every scratch element
// before reading it. Calls that overlap on the GPU (different streams, or
// different host threads on the same device) race on the array; serialise
// them.
#include <mutex>

#include "b2c.h"
#include "b2c_kernels.cuh"

namespace {

constexpr size_t kStaticScratchBytes = 16u << 20;
constexpr int kMaxContexts = 64;

static __device__ __align__(256) float g_static_scratch[kStaticScratchBytes / sizeof(float)];

// The driver's cuCtxGetCurrent, reached through the runtime (no link to the
// driver library): the current context is the key of the recorded addresses.
typedef int (*CtxGetCurrentFn)(void**);

std::mutex g_mu;
CtxGetCurrentFn g_ctx_get = nullptr;
bool g_ctx_get_looked_up = false;
void* g_ctx[kMaxContexts] = {nullptr};
void* g_addr[kMaxContexts] = {nullptr};
int g_nctx = 0;

int fail(int code, const char* msg) { return b2c::set_error(code, msg); }

// Current context handle (nullptr if it cannot be told).
void* current_context() {
  if (!g_ctx_get_looked_up) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_get = reinterpret_cast<CtxGetCurrentFn>(fn);
    g_ctx_get_looked_up = true;
  }
  void* ctx = nullptr;
  if (!g_ctx_get || g_ctx_get(&ctx) != 0) return nullptr;
  return ctx;
}

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
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                cudaSuccess)
    return fail(B2C_ERR_CUDA, "b2c_posv_static_scratch: no current CUDA device");
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) != cudaSuccess)
    return fail(B2C_ERR_CUDA, "b2c_posv_static_scratch: cudaStreamIsCapturing failed");
  void* addr = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    void* ctx = current_context();
    int slot_i = -1;
    for (int i = 0; i < g_nctx; ++i)
      if (g_ctx[i] == ctx) slot_i = i;
    if (cap == cudaStreamCaptureStatusNone) {
      cudaError_t e = cudaGetSymbolAddress(&addr, g_static_scratch);
      if (e != cudaSuccess) return fail(B2C_ERR_CUDA, "b2c_posv_static_scratch: cudaGetSymbolAddress failed");
      if (slot_i < 0 && g_nctx < kMaxContexts) slot_i = g_nctx++;
      if (slot_i >= 0) {
        g_ctx[slot_i] = ctx;
        g_addr[slot_i] = addr;
      }
    } else {
      if (slot_i < 0 || !ctx)
        return fail(B2C_ERR_CUDA,
                    "b2c_posv_static_scratch: called during stream capture before any call outside capture "
                    "in this context");
      addr = g_addr[slot_i];
    }
  }
  b2c::PosvParams p{};
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
  cudaError_t e = b2c::launch_posv_blocked(p, grid, s);
  if (e != cudaSuccess) return fail(B2C_ERR_CUDA, "b2c_posv_static_scratch: kernel launch failed");
  return fail(B2C_OK, "");
}
