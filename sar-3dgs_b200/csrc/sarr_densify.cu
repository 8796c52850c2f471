// Densification and pruning of the Gaussian set (GaussianModel.densify_and_prune,
// gaussian_model.py:433-566) as three passes over the Gaussians instead of
// Python loops: flags and per-block counts, block offsets, and a stable scatter
// into the new arrays (kept Gaussians in order, then the clones, then the two
// halves of every split), so the result is the reference's in content and order.
#include <math.h>
#include <stdint.h>

#include "sarr.h"

namespace sarr {
void count_launches(int k);  // the library's launch counter (sarr_abi.cu)
}

namespace {

constexpr int kDensifyThreads = 1024;

enum : uint8_t { kClone = 1, kSplit = 2, kPrune = 4 };

struct DensifyCounts {
  int64_t blocks;
};

__device__ __forceinline__ int block_excl_scan(int x, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = s_warp[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    s_warp[lane] = wi - w;
    if (lane == 31) s_warp[32] = wi;
  }
  __syncthreads();
  *total = s_warp[32];
  const int r = s_warp[warp] + incl - x;
  __syncthreads();
  return r;
}

// Flags of densify_and_prune (:464-475): scale norm of exp(scales), norm of the
// mean gradient, sigmoid opacity; per-block counts of kept / cloned / split.
__global__ void __launch_bounds__(kDensifyThreads) densify_flags_kernel(
    int64_t n, const float* __restrict__ scales, const float* __restrict__ logits,
    const float* __restrict__ grad_means, float grad_thr, float size_thr, float large_thr,
    float opacity_thr, uint8_t* __restrict__ flags, int* __restrict__ block_counts) {
  __shared__ int s_warp[33];
  const int64_t i = (int64_t)blockIdx.x * kDensifyThreads + threadIdx.x;
  int keep = 0, clone = 0, split = 0;
  if (i < n) {
    const float s0 = expf(scales[3 * i]), s1 = expf(scales[3 * i + 1]), s2 = expf(scales[3 * i + 2]);
    const float snorm = sqrtf(s0 * s0 + s1 * s1 + s2 * s2);
    const float g0 = grad_means[3 * i], g1 = grad_means[3 * i + 1], g2 = grad_means[3 * i + 2];
    const float gnorm = sqrtf(g0 * g0 + g1 * g1 + g2 * g2);
    const bool small = snorm < size_thr, large = snorm > large_thr, high = gnorm > grad_thr;
    const bool low_op = 1.0f / (1.0f + expf(-logits[i])) < opacity_thr;
    clone = small && high;
    split = large && high;
    const bool prune = low_op || large;
    keep = !prune;
    flags[i] = (uint8_t)((clone ? kClone : 0) | (split ? kSplit : 0) | (prune ? kPrune : 0));
  }
  int tot;
  block_excl_scan(keep, s_warp, &tot);
  const int tk = tot;
  block_excl_scan(clone, s_warp, &tot);
  const int tc = tot;
  block_excl_scan(split, s_warp, &tot);
  if (threadIdx.x == 0) {
    block_counts[3 * blockIdx.x] = tk;
    block_counts[3 * blockIdx.x + 1] = tc;
    block_counts[3 * blockIdx.x + 2] = tot;
  }
}

// Exclusive offsets of the block counts (one CTA) and the totals
// counts[0..2] = kept, clones, splits (int64).
__global__ void __launch_bounds__(kDensifyThreads) densify_offsets_kernel(int blocks, int* block_counts,
                                                                          int64_t* counts) {
  __shared__ int s_warp[33];
  int64_t carry[3] = {0, 0, 0};
  for (int b0 = 0; b0 < blocks; b0 += kDensifyThreads) {
    const int b = b0 + threadIdx.x;
    for (int q = 0; q < 3; ++q) {
      const int x = b < blocks ? block_counts[3 * b + q] : 0;
      int tot;
      const int e = block_excl_scan(x, s_warp, &tot);
      if (b < blocks) block_counts[3 * b + q] = (int)(carry[q] + e);
      carry[q] += tot;
    }
  }
  if (threadIdx.x == 0)
    for (int q = 0; q < 3; ++q) counts[q] = carry[q];
}

struct ApplyArgs {
  int64_t n;
  const float *means, *scales, *rot, *logits, *sh, *grad_means;
  int sh_cols;
  const uint8_t* flags;
  const int* block_offsets;
  const int64_t* counts;
  int do_clones, do_splits;
  float *o_means, *o_scales, *o_rot, *o_logits, *o_sh;
  bool vec;  // rotation rows and 16-column SH rows 16-byte aligned: copied as float4
};

__device__ __forceinline__ void copy_row(const ApplyArgs& a, int64_t src, int64_t dst) {
  for (int k = 0; k < 3; ++k) a.o_means[3 * dst + k] = a.means[3 * src + k];
  for (int k = 0; k < 3; ++k) a.o_scales[3 * dst + k] = a.scales[3 * src + k];
  a.o_logits[dst] = a.logits[src];
  if (a.vec) {
    reinterpret_cast<float4*>(a.o_rot)[dst] = reinterpret_cast<const float4*>(a.rot)[src];
    const float4* hs = reinterpret_cast<const float4*>(a.sh) + 4 * src;
    float4* hd = reinterpret_cast<float4*>(a.o_sh) + 4 * dst;
#pragma unroll
    for (int q = 0; q < 4; ++q) hd[q] = hs[q];
    return;
  }
  for (int k = 0; k < 4; ++k) a.o_rot[4 * dst + k] = a.rot[4 * src + k];
  for (int k = 0; k < a.sh_cols; ++k) a.o_sh[(size_t)dst * a.sh_cols + k] = a.sh[(size_t)src * a.sh_cols + k];
}

// Kept Gaussians at their rank; clones (:504-521): mean + grad * 0.01, the
// rest copied; splits (:523-548): two Gaussians with scale log(0.8 exp(s)) and
// mean offsets (0.4 s_x cos a, 0.4 s_y sin a, 0) for a = 0 and pi, in the
// reference's float32 operation order.
__global__ void __launch_bounds__(kDensifyThreads) densify_apply_kernel(const ApplyArgs a) {
  __shared__ int s_warp[33];
  const int64_t i = (int64_t)blockIdx.x * kDensifyThreads + threadIdx.x;
  const uint8_t f = i < a.n ? a.flags[i] : (uint8_t)kPrune;
  const int keep = !(f & kPrune), clone = (f & kClone) != 0, split = (f & kSplit) != 0;
  int tot;
  const int rk = block_excl_scan(keep, s_warp, &tot);
  const int rc = block_excl_scan(clone, s_warp, &tot);
  const int rs = block_excl_scan(split, s_warp, &tot);
  if (i >= a.n) return;
  const int* off = a.block_offsets + 3 * blockIdx.x;
  const int64_t kept = a.counts[0], clones = a.do_clones ? a.counts[1] : 0;
  if (keep) copy_row(a, i, off[0] + rk);
  if (a.do_clones && clone) {
    const int64_t d = kept + off[1] + rc;
    copy_row(a, i, d);
    for (int k = 0; k < 3; ++k)
      a.o_means[3 * d + k] = __fadd_rn(a.means[3 * i + k], __fmul_rn(a.grad_means[3 * i + k], 0.01f));
  }
  if (a.do_splits && split) {
    const int64_t d0 = kept + clones + 2 * (int64_t)(off[2] + rs);
    const float v0 = __fmul_rn(expf(a.scales[3 * i]), 0.8f);
    const float v1 = __fmul_rn(expf(a.scales[3 * i + 1]), 0.8f);
    const float v2 = __fmul_rn(expf(a.scales[3 * i + 2]), 0.8f);
    // cos and sin of 0 and pi as the reference's numpy values, rounded to float
    const float cs[2] = {1.0f, -1.0f}, sn[2] = {0.0f, 1.2246467991473532e-16f};
    for (int h = 0; h < 2; ++h) {
      const int64_t d = d0 + h;
      copy_row(a, i, d);
      const float ox = __fmul_rn(__fmul_rn(v0, 0.5f), cs[h]);
      const float oy = __fmul_rn(__fmul_rn(v1, 0.5f), sn[h]);
      a.o_means[3 * d] = __fadd_rn(a.means[3 * i], ox);
      a.o_means[3 * d + 1] = __fadd_rn(a.means[3 * i + 1], oy);
      a.o_means[3 * d + 2] = __fadd_rn(a.means[3 * i + 2], 0.0f);
      a.o_scales[3 * d] = logf(v0);
      a.o_scales[3 * d + 1] = logf(v1);
      a.o_scales[3 * d + 2] = logf(v2);
    }
  }
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? SARR_OK : SARR_ERR_CUDA; }

}  // namespace

extern "C" int sarr_densify_workspace_size(int64_t n, size_t* bytes) {
  if (!bytes || n < 0) return SARR_ERR_ARG;
  const int64_t blocks = (n + kDensifyThreads - 1) / kDensifyThreads;
  *bytes = (((size_t)n + 255) & ~(size_t)255) + (((size_t)blocks * 12 + 255) & ~(size_t)255) + 256;
  return SARR_OK;
}

extern "C" int sarr_densify_flags(int64_t n, const float* scales_log, const float* opacity_logits,
                                  const float* grad_means, float grad_threshold, float size_threshold,
                                  float large_scale_threshold, float opacity_threshold,
                                  int64_t* counts_out, void* ws, size_t ws_bytes, sarr_stream_t stream) {
  size_t need = 0;
  if (sarr_densify_workspace_size(n, &need) != SARR_OK) return SARR_ERR_ARG;
  if (n == 0) return SARR_OK;
  if (!scales_log || !opacity_logits || !grad_means || !counts_out) return SARR_ERR_ARG;
  if (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255)) return SARR_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int blocks = (int)((n + kDensifyThreads - 1) / kDensifyThreads);
  uint8_t* flags = static_cast<uint8_t*>(ws);
  int* bc = reinterpret_cast<int*>(static_cast<unsigned char*>(ws) + (((size_t)n + 255) & ~(size_t)255));
  densify_flags_kernel<<<blocks, kDensifyThreads, 0, s>>>(n, scales_log, opacity_logits, grad_means,
                                                          grad_threshold, size_threshold,
                                                          large_scale_threshold, opacity_threshold,
                                                          flags, bc);
  densify_offsets_kernel<<<1, kDensifyThreads, 0, s>>>(blocks, bc, counts_out);
  sarr::count_launches(2);
  return cuda_status(cudaGetLastError());
}

extern "C" int sarr_densify_apply(int64_t n, const float* means, const float* scales_log,
                                  const float* rotations, const float* opacity_logits, const float* sh,
                                  int sh_cols, const float* grad_means, const int64_t* counts,
                                  int do_clones, int do_splits, float* out_means, float* out_scales,
                                  float* out_rotations, float* out_opacity_logits, float* out_sh,
                                  void* ws, size_t ws_bytes, sarr_stream_t stream) {
  size_t need = 0;
  if (sarr_densify_workspace_size(n, &need) != SARR_OK || sh_cols < 0) return SARR_ERR_ARG;
  if (n == 0) return SARR_OK;
  if (!means || !scales_log || !rotations || !opacity_logits || (sh_cols && !sh) || !grad_means ||
      !counts || !out_means || !out_scales || !out_rotations || !out_opacity_logits ||
      (sh_cols && !out_sh))
    return SARR_ERR_ARG;
  if (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255)) return SARR_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int blocks = (int)((n + kDensifyThreads - 1) / kDensifyThreads);
  ApplyArgs a;
  a.n = n;
  a.means = means;
  a.scales = scales_log;
  a.rot = rotations;
  a.logits = opacity_logits;
  a.sh = sh;
  a.grad_means = grad_means;
  a.sh_cols = sh_cols;
  a.flags = static_cast<const uint8_t*>(ws);
  a.block_offsets = reinterpret_cast<const int*>(static_cast<const unsigned char*>(ws) +
                                                 (((size_t)n + 255) & ~(size_t)255));
  a.counts = counts;
  a.do_clones = do_clones;
  a.do_splits = do_splits;
  a.o_means = out_means;
  a.o_scales = out_scales;
  a.o_rot = out_rotations;
  a.o_logits = out_opacity_logits;
  a.o_sh = out_sh;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  a.vec = sh_cols == 16 && a16(rotations) && a16(out_rotations) && a16(sh) && a16(out_sh);
  densify_apply_kernel<<<blocks, kDensifyThreads, 0, s>>>(a);
  sarr::count_launches(1);
  return cuda_status(cudaGetLastError());
}
