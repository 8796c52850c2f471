// sarr_forward_static: the single-view image forward of sarr_forward with its
// workspace in a file-scope device array of this library, for callers that
// cannot allocate device memory themselves (see include/sarr.h).
//
// Scratch: g_static_scratch, kStaticScratchBytes (6 MiB) per device, which
// holds the workspace of one view with n <= kStaticMaxGaussians (131,072)
// Gaussians and an image of at most 256 x 256 pixels. Nothing in it has to
// start at zero: every byte the call reads is written earlier in the same
// call (the device error word is cleared by the call itself).
//
// Setup: the first call on a device, with that device current, looks up the
// array's device address with cudaGetSymbolAddress and caches it; later calls
// on that device reuse it. Make that first call before any stream capture
// begins. Every call on a device uses the same scratch, so calls on one
// device must not overlap: issue them on one stream, or order them.
#include <mutex>

#include "sarr.h"
#include "sarr_internal.h"

namespace {

constexpr int64_t kStaticMaxGaussians = 131072;
constexpr int kStaticMaxSamples = 256;
constexpr size_t kStaticScratchBytes = (size_t)6 * 1024 * 1024;
constexpr int kStaticMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_static_mu;
void* g_static_ptr[kStaticMaxDevices] = {};

// Device address of g_static_scratch on the current device (cached).
int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SARR_ERR_CUDA;
  if (dev < 0 || dev >= kStaticMaxDevices) return SARR_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) return SARR_ERR_CUDA;
    g_static_ptr[dev] = p;
  }
  *out = g_static_ptr[dev];
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
