// sarr_forward_static: the single-view image forward of sarr_forward with its
// workspace in a file-scope device array of this library, for callers that
// cannot allocate device memory themselves (see include/sarr.h).
//
// Scratch: g_static_scratch, kStaticScratchBytes (8 MiB) per device, which
// holds the workspace of one view with n <= kStaticMaxGaussians (131,072)
// Gaussians and an image of at most 256 x 256 pixels. Nothing in it has to
// start at zero: every byte the call reads is written earlier in the same
// call (the device error word is cleared by the call itself).
//
// Setup: the first call in a CUDA context, with that context current, looks
// up the array's device address with cudaGetSymbolAddress and caches it
// under that context's handle; later calls in the same context reuse it.
// Make that first call before any stream capture begins. A context that is
// destroyed and re-created (cudaDeviceReset) may come back under the same
// handle, so the cache does not survive a device reset: do not reset a
// device between calls. Every call in a context uses the same scratch, so
// calls on one device must not overlap: issue them on one stream, or order
// them.
#include <mutex>

#include "sarr.h"
#include "sarr_internal.h"

namespace {

constexpr int64_t kStaticMaxGaussians = 131072;
constexpr int kStaticMaxSamples = 256;
constexpr size_t kStaticScratchBytes = (size_t)8 * 1024 * 1024;
constexpr int kStaticMaxContexts = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// cuCtxGetCurrent, resolved through the runtime (the library links no
// driver-API import library).
using CtxGetCurrentFn = int (*)(void** ctx);

struct ScratchEntry {
  void* ctx;
  void* ptr;
};

std::mutex g_static_mu;
ScratchEntry g_static_cache[kStaticMaxContexts] = {};
int g_static_used = 0;
CtxGetCurrentFn g_ctx_get_current = nullptr;

// The current context's handle; makes the runtime initialise its context on
// this device first, so that the handle is the one the kernels will run in.
int current_context(void** ctx) {
  if (cudaFree(nullptr) != cudaSuccess) return SARR_ERR_CUDA;
  if (!g_ctx_get_current) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return SARR_ERR_CUDA;
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  }
  *ctx = nullptr;
  if (g_ctx_get_current(ctx) != 0 || !*ctx) return SARR_ERR_CUDA;
  return SARR_OK;
}

// Device address of g_static_scratch in the current context (cached).
int static_scratch(void** out) {
  std::lock_guard<std::mutex> lk(g_static_mu);
  void* ctx = nullptr;
  int st = current_context(&ctx);
  if (st) return st;
  for (int i = 0; i < g_static_used; ++i) {
    if (g_static_cache[i].ctx == ctx) {
      *out = g_static_cache[i].ptr;
      return SARR_OK;
    }
  }
  if (g_static_used == kStaticMaxContexts) return SARR_ERR_CAPACITY;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) return SARR_ERR_CUDA;
  g_static_cache[g_static_used++] = ScratchEntry{ctx, p};
  *out = p;
  return SARR_OK;
}

}  // namespace

extern "C" int sarr_forward_static(const sarr_view* view, int64_t n, const float* means,
                                   const float* cov, int cov_layout, const float* sigma,
                                   const float* sh, int sh_stride, int sh_k, float* image,
                                   sarr_stream_t stream) {
  if (!view || n < 0) return SARR_ERR_ARG;
  if (n > kStaticMaxGaussians || view->range_samples > kStaticMaxSamples ||
      view->azimuth_samples > kStaticMaxSamples)
    return SARR_ERR_CAPACITY;
  size_t need = 0;
  int st = sarr_workspace_size(n, view->range_samples, view->azimuth_samples, 1, 0, &need);
  if (st) return st;
  if (need > kStaticScratchBytes) return SARR_ERR_CAPACITY;
  void* ws = nullptr;
  st = static_scratch(&ws);
  if (st) return st;
  return sarr_forward(view, 1, n, means, cov, cov_layout, sigma, sh, sh_stride, sh_k, image,
                      nullptr, nullptr, ws, kStaticScratchBytes, stream);
}

// The device error word of the static scratch: the same read-and-clear as
// sarr_check_device_errors on a caller workspace (it synchronises the stream).
extern "C" int sarr_check_static_errors(sarr_stream_t stream) {
  void* ws = nullptr;
  const int st = static_scratch(&ws);
  if (st) return st;
  return sarr_check_device_errors(ws, kStaticScratchBytes, stream);
}
