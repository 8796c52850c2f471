// Training-step kernels around the rasterizer: the Gaussian parameter
// producer (covariance from log-scales and quaternions, transmittance from
// logits) and the combined L1 + D-SSIM loss with its image gradient.
//
//   gaussian_params_kernel   replaces GaussianModel.compute_covariance_full /
//                            compute_covariance and get_opacity
//                            (gaussian_model.py:261-330): one pass over the
//                            Gaussians instead of a Python loop building S.
//   loss_moments_kernel      the 5 windowed moments of CombinedLoss.forward
//                            (losses.py:170-215) per pixel, the SSIM map, the
//                            L1 term, and the per-pixel partial derivatives
//                            of the SSIM map with respect to the moments;
//   loss_grad_kernel         the image gradient: L1 term plus the window
//                            correlation of those partial derivatives;
//   loss_reduce_kernel       deterministic reduction of the per-block sums.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "sarr.h"

namespace {

constexpr int kMaxWindow = 11;

// ---------------------------------------------------------------------------
// producer
// ---------------------------------------------------------------------------
// Sigma = R diag(exp(s))^2 R^T with R from the quaternion (w, x, y, z) as
// Quaternion.to_rotation_matrix writes it (gaussian_model.py:40-51, not
// normalised); transmittance = sigmoid(logit).
__global__ void gaussian_params_kernel(int64_t n, const float* __restrict__ scales,
                                       const float* __restrict__ rot, int cov_layout,
                                       float* __restrict__ cov, const float* __restrict__ logits,
                                       float* __restrict__ sigma) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  if (cov) {
    const float s0 = expf(scales[3 * j]), s1 = expf(scales[3 * j + 1]), s2 = expf(scales[3 * j + 2]);
    const float w = rot[4 * j], x = rot[4 * j + 1], y = rot[4 * j + 2], z = rot[4 * j + 3];
    const float R[3][3] = {{1.0f - 2.0f * (y * y + z * z), 2.0f * (x * y - w * z), 2.0f * (x * z + w * y)},
                           {2.0f * (x * y + w * z), 1.0f - 2.0f * (x * x + z * z), 2.0f * (y * z - w * x)},
                           {2.0f * (x * z - w * y), 2.0f * (y * z + w * x), 1.0f - 2.0f * (x * x + y * y)}};
    const float d[3] = {s0 * s0, s1 * s1, s2 * s2};
    float S[3][3];
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int b = 0; b < 3; ++b) S[a][b] = R[a][0] * d[0] * R[b][0] + R[a][1] * d[1] * R[b][1] + R[a][2] * d[2] * R[b][2];
    if (cov_layout == SARR_COV33) {
      float* o = cov + 9 * j;
#pragma unroll
      for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int b = 0; b < 3; ++b) o[3 * a + b] = S[a][b];
    } else {
      float* o = cov + 6 * j;  // xx yy zz xy xz yz
      o[0] = S[0][0];
      o[1] = S[1][1];
      o[2] = S[2][2];
      o[3] = S[0][1];
      o[4] = S[0][2];
      o[5] = S[1][2];
    }
  }
  if (sigma) sigma[j] = 1.0f / (1.0f + expf(-logits[j]));
}

// ---------------------------------------------------------------------------
// loss
// ---------------------------------------------------------------------------
struct LossParams {
  int V, H, W;
  int window, half;
  float g[kMaxWindow];  // 1-D window weights (the 2-D window is g g^T)
  float l1_weight, ssim_weight;
  int l1_mode;
  float inv_count;      // 1 / (V H W)
};

constexpr int kTileX = 32, kTileY = 16;  // output pixels per CTA
constexpr int kLossThreads = 256;
constexpr int kHaloMax = kMaxWindow / 2;

// Loads rows [y0 - half, y0 + kTileY + half) x columns [x0 - half, x0 + kTileX
// + half) of image `img` (zero outside) into `tile`.
__device__ __forceinline__ void load_halo(const float* __restrict__ img, int H, int W, int y0, int x0,
                                          int half, float* tile, int pitch) {
  const int rows = kTileY + 2 * half, cols = kTileX + 2 * half;
  for (int i = threadIdx.x; i < rows * cols; i += kLossThreads) {
    const int r = i / cols, c = i - r * cols;
    const int y = y0 - half + r, x = x0 - half + c;
    tile[r * pitch + c] = (y >= 0 && y < H && x >= 0 && x < W) ? img[(size_t)y * W + x] : 0.0f;
  }
}

// Weighted L1 factor of losses.py:28-62 (1 for the plain L1).
__device__ __forceinline__ float l1_factor(int mode, float t, float tmax) {
  if (mode == SARR_L1_PLAIN || !(tmax > 0.0f)) return 1.0f;
  const float tn = t / tmax;
  if (mode == SARR_L1_SQUARE) return 1.0f + tn * tn;
  if (mode == SARR_L1_SQRT) return 1.0f + sqrtf(tn + 1e-8f);
  return 1.0f + tn;
}

__global__ void __launch_bounds__(kLossThreads) loss_tmax_kernel(const float* __restrict__ target,
                                                                 int64_t count, float* partial) {
  float m = -INFINITY;
  for (int64_t i = (int64_t)blockIdx.x * kLossThreads + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * kLossThreads)
    m = fmaxf(m, target[i]);
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float s[kLossThreads / 32];
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kLossThreads / 32; ++w) m = fmaxf(m, s[w]);
    partial[blockIdx.x] = m;
  }
}

__global__ void loss_tmax_final_kernel(const float* partial, int n, float* tmax) {
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += 32) m = fmaxf(m, partial[i]);
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (threadIdx.x == 0) *tmax = m;
}

// Per output pixel: the windowed means of p, t, p^2, t^2, p t (zero padding,
// as F.conv2d with padding window/2), the SSIM map value, the L1 term, and
// dm, de2, dept = d ssim / d (mean p, windowed mean of p^2, windowed mean of
// p t), scaled by -ssim_weight / count for the gradient. Per-CTA sums of the
// SSIM map and of the L1 term go to `partial` [2][blocks].
__global__ void __launch_bounds__(kLossThreads) loss_moments_kernel(const LossParams P,
                                                                    const float* __restrict__ pred,
                                                                    const float* __restrict__ target,
                                                                    const float* __restrict__ tmax_p,
                                                                    float* __restrict__ dgrad,
                                                                    float* __restrict__ partial) {
  constexpr int kRowsMax = kTileY + 2 * kHaloMax, kColsMax = kTileX + 2 * kHaloMax;
  __shared__ float s_p[kRowsMax * kColsMax], s_t[kRowsMax * kColsMax];
  __shared__ float s_h[5][kRowsMax * kTileX];  // horizontal pass of the 5 quantities
  __shared__ float s_red[2][kLossThreads / 32];
  const int v = blockIdx.z, y0 = blockIdx.y * kTileY, x0 = blockIdx.x * kTileX;
  const int H = P.H, W = P.W, half = P.half, win = P.window;
  const size_t img = (size_t)v * H * W;
  const int pitch = kTileX + 2 * half;
  load_halo(pred + img, H, W, y0, x0, half, s_p, pitch);
  load_halo(target + img, H, W, y0, x0, half, s_t, pitch);
  __syncthreads();
  const int rows = kTileY + 2 * half;
  for (int i = threadIdx.x; i < rows * kTileX; i += kLossThreads) {
    const int r = i / kTileX, c = i - r * kTileX;
    float a = 0.f, b = 0.f, aa = 0.f, bb = 0.f, ab = 0.f;
    for (int k = 0; k < win; ++k) {
      const float p = s_p[r * pitch + c + k], t = s_t[r * pitch + c + k], g = P.g[k];
      a += g * p;
      b += g * t;
      aa += g * (p * p);
      bb += g * (t * t);
      ab += g * (p * t);
    }
    s_h[0][i] = a;
    s_h[1][i] = b;
    s_h[2][i] = aa;
    s_h[3][i] = bb;
    s_h[4][i] = ab;
  }
  __syncthreads();
  const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
  const float tmax = tmax_p ? *tmax_p : 0.0f;
  const float gs = -P.ssim_weight * P.inv_count;
  float ssim_sum = 0.f, l1_sum = 0.f;
  for (int i = threadIdx.x; i < kTileY * kTileX; i += kLossThreads) {
    const int r = i / kTileX, c = i - r * kTileX;
    const int y = y0 + r, x = x0 + c;
    if (y >= H || x >= W) continue;
    float m[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < win; ++k) {
      const float g = P.g[k];
#pragma unroll
      for (int q = 0; q < 5; ++q) m[q] += g * s_h[q][(r + k) * kTileX + c];
    }
    const float mp = m[0], mt = m[1];
    const float mp2 = mp * mp, mt2 = mt * mt, mpt = mp * mt;
    const float sp = m[2] - mp2, st = m[3] - mt2, spt = m[4] - mpt;
    const float A1 = 2.0f * mpt + C1, A2 = 2.0f * spt + C2;
    const float B1 = mp2 + mt2 + C1, B2 = sp + st + C2;
    const float ssim = (A1 * A2) / (B1 * B2);
    ssim_sum += ssim;
    const float p = s_p[(r + half) * pitch + c + half], t = s_t[(r + half) * pitch + c + half];
    l1_sum += fabsf(p - t) * l1_factor(P.l1_mode, t, tmax);
    if (dgrad) {
      const float inv = 1.0f / (B1 * B2);
      const float d_mp = 2.0f * mt * A2 * inv - ssim * 2.0f * mp / B1;
      const float d_sp = -ssim / B2;
      const float d_spt = 2.0f * A1 * inv;
      const size_t o = img + (size_t)y * W + x, plane = (size_t)P.V * H * W;
      dgrad[o] = gs * (d_mp - 2.0f * mp * d_sp - mt * d_spt);
      dgrad[plane + o] = gs * d_sp;
      dgrad[2 * plane + o] = gs * d_spt;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    ssim_sum += __shfl_xor_sync(0xffffffffu, ssim_sum, o);
    l1_sum += __shfl_xor_sync(0xffffffffu, l1_sum, o);
  }
  if ((threadIdx.x & 31) == 0) {
    s_red[0][threadIdx.x >> 5] = ssim_sum;
    s_red[1][threadIdx.x >> 5] = l1_sum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f, b = 0.f;
    for (int w = 0; w < kLossThreads / 32; ++w) {
      a += s_red[0][w];
      b += s_red[1][w];
    }
    const int blk = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    const int nblk = gridDim.x * gridDim.y * gridDim.z;
    partial[blk] = a;
    partial[nblk + blk] = b;
  }
}

// grad_j = l1_weight * factor * sign(p - t) / count
//        + (K * dm)_j + 2 p_j (K * de2)_j + t_j (K * dept)_j
__global__ void __launch_bounds__(kLossThreads) loss_grad_kernel(const LossParams P,
                                                                 const float* __restrict__ pred,
                                                                 const float* __restrict__ target,
                                                                 const float* __restrict__ tmax_p,
                                                                 const float* __restrict__ dgrad,
                                                                 float* __restrict__ grad) {
  constexpr int kRowsMax = kTileY + 2 * kHaloMax, kColsMax = kTileX + 2 * kHaloMax;
  __shared__ float s_d[3][kRowsMax * kColsMax];
  __shared__ float s_h[3][kRowsMax * kTileX];
  const int v = blockIdx.z, y0 = blockIdx.y * kTileY, x0 = blockIdx.x * kTileX;
  const int H = P.H, W = P.W, half = P.half, win = P.window;
  const size_t img = (size_t)v * H * W, plane = (size_t)P.V * H * W;
  const int pitch = kTileX + 2 * half;
  for (int q = 0; q < 3; ++q) load_halo(dgrad + q * plane + img, H, W, y0, x0, half, s_d[q], pitch);
  __syncthreads();
  const int rows = kTileY + 2 * half;
  for (int i = threadIdx.x; i < rows * kTileX; i += kLossThreads) {
    const int r = i / kTileX, c = i - r * kTileX;
    float a[3] = {0.f, 0.f, 0.f};
    for (int k = 0; k < win; ++k) {
      const float g = P.g[k];
#pragma unroll
      for (int q = 0; q < 3; ++q) a[q] += g * s_d[q][r * pitch + c + k];
    }
#pragma unroll
    for (int q = 0; q < 3; ++q) s_h[q][i] = a[q];
  }
  __syncthreads();
  const float tmax = tmax_p ? *tmax_p : 0.0f;
  for (int i = threadIdx.x; i < kTileY * kTileX; i += kLossThreads) {
    const int r = i / kTileX, c = i - r * kTileX;
    const int y = y0 + r, x = x0 + c;
    if (y >= H || x >= W) continue;
    float a[3] = {0.f, 0.f, 0.f};
    for (int k = 0; k < win; ++k) {
      const float g = P.g[k];
#pragma unroll
      for (int q = 0; q < 3; ++q) a[q] += g * s_h[q][(r + k) * kTileX + c];
    }
    const size_t o = img + (size_t)y * W + x;
    const float p = pred[o], t = target[o];
    const float diff = p - t;
    const float sgn = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
    grad[o] = P.l1_weight * l1_factor(P.l1_mode, t, tmax) * sgn * P.inv_count + a[0] +
              2.0f * p * a[1] + t * a[2];
  }
}

// losses [3] = total, l1, dssim from the per-CTA sums (fixed order).
__global__ void loss_reduce_kernel(const LossParams P, const float* partial, int nblk, float* losses) {
  double ssim = 0.0, l1 = 0.0;
  for (int i = threadIdx.x; i < nblk; i += 32) {
    ssim += partial[i];
    l1 += partial[nblk + i];
  }
  for (int o = 16; o > 0; o >>= 1) {
    ssim += __shfl_xor_sync(0xffffffffu, ssim, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  if (threadIdx.x == 0) {
    const float l1m = (float)(l1 * P.inv_count), dssim = (float)(1.0 - ssim * P.inv_count);
    losses[0] = P.l1_weight * l1m + P.ssim_weight * dssim;
    losses[1] = l1m;
    losses[2] = dssim;
  }
}

struct LossWs {
  size_t dgrad, partial, tmax_partial, tmax, bytes;
};

constexpr int kTmaxBlocks = 256;

LossWs loss_ws(int V, int H, int W) {
  LossWs L;
  const size_t plane = (size_t)V * H * W;
  const size_t blocks = (size_t)((W + kTileX - 1) / kTileX) * ((H + kTileY - 1) / kTileY) * V;
  size_t o = 0;
  L.dgrad = o;
  o += (3 * plane * 4 + 255) & ~(size_t)255;
  L.partial = o;
  o += (2 * blocks * 4 + 255) & ~(size_t)255;
  L.tmax_partial = o;
  o += kTmaxBlocks * 4;
  L.tmax = o;
  o += 256;
  L.bytes = o;
  return L;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? SARR_OK : SARR_ERR_CUDA; }

}  // namespace

extern "C" int sarr_gaussian_params(int64_t n, const float* scales_log, const float* rotations,
                                    float* cov_out, int cov_layout, const float* opacity_logits,
                                    float* opacity_out, sarr_stream_t stream) {
  if (n < 0) return SARR_ERR_ARG;
  if (cov_out && (!scales_log || !rotations)) return SARR_ERR_ARG;
  if (cov_out && cov_layout != SARR_COV6 && cov_layout != SARR_COV33) return SARR_ERR_ARG;
  if (opacity_out && !opacity_logits) return SARR_ERR_ARG;
  if (n == 0 || (!cov_out && !opacity_out)) return SARR_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  gaussian_params_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(n, scales_log, rotations, cov_layout,
                                                                     cov_out, opacity_logits, opacity_out);
  return cuda_status(cudaGetLastError());
}

extern "C" int sarr_loss_workspace_size(int n_images, int height, int width, size_t* bytes) {
  if (!bytes || n_images < 0 || height < 0 || width < 0) return SARR_ERR_ARG;
  *bytes = loss_ws(n_images, height, width).bytes;
  return SARR_OK;
}

extern "C" int sarr_combined_loss(int n_images, int height, int width, const float* pred,
                                  const float* target, float l1_weight, float ssim_weight,
                                  int window_size, int l1_mode, float* losses_out, float* grad_pred,
                                  void* ws, size_t ws_bytes, sarr_stream_t stream) {
  if (n_images < 1 || height < 1 || width < 1 || !pred || !target || !losses_out) return SARR_ERR_ARG;
  if (window_size < 1 || window_size > kMaxWindow || (window_size & 1) == 0) return SARR_ERR_ARG;
  if (l1_mode < SARR_L1_PLAIN || l1_mode > SARR_L1_SQRT) return SARR_ERR_ARG;
  const LossWs L = loss_ws(n_images, height, width);
  if (!ws || ws_bytes < L.bytes || (reinterpret_cast<uintptr_t>(ws) & 255)) return SARR_ERR_WORKSPACE;
  unsigned char* w = static_cast<unsigned char*>(ws);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  LossParams P;
  memset(&P, 0, sizeof(P));
  P.V = n_images;
  P.H = height;
  P.W = width;
  P.window = window_size;
  P.half = window_size / 2;
  // gaussian_kernel (losses.py:65-78): exp(-x^2 / (2 sigma^2)) at integer
  // offsets, sigma = 1.5, normalised to sum 1 (float32 as torch computes it)
  float gsum = 0.0f;
  for (int k = 0; k < window_size; ++k) {
    const float x = (float)(k - window_size / 2);
    P.g[k] = expf(-(x * x) / (2.0f * 1.5f * 1.5f));
    gsum += P.g[k];
  }
  for (int k = 0; k < window_size; ++k) P.g[k] /= gsum;
  P.l1_weight = l1_weight;
  P.ssim_weight = ssim_weight;
  P.l1_mode = l1_mode;
  P.inv_count = (float)(1.0 / ((double)n_images * height * width));

  const float* tmax = nullptr;
  if (l1_mode != SARR_L1_PLAIN) {
    float* tp = reinterpret_cast<float*>(w + L.tmax_partial);
    loss_tmax_kernel<<<kTmaxBlocks, kLossThreads, 0, s>>>(target, (int64_t)n_images * height * width, tp);
    loss_tmax_final_kernel<<<1, 32, 0, s>>>(tp, kTmaxBlocks, reinterpret_cast<float*>(w + L.tmax));
    tmax = reinterpret_cast<const float*>(w + L.tmax);
  }
  const dim3 grid((width + kTileX - 1) / kTileX, (height + kTileY - 1) / kTileY, n_images);
  const int nblk = grid.x * grid.y * grid.z;
  float* dgrad = grad_pred ? reinterpret_cast<float*>(w + L.dgrad) : nullptr;
  float* partial = reinterpret_cast<float*>(w + L.partial);
  loss_moments_kernel<<<grid, kLossThreads, 0, s>>>(P, pred, target, tmax, dgrad, partial);
  if (grad_pred) loss_grad_kernel<<<grid, kLossThreads, 0, s>>>(P, pred, target, tmax, dgrad, grad_pred);
  loss_reduce_kernel<<<1, 32, 0, s>>>(P, partial, nblk, losses_out);
  return cuda_status(cudaGetLastError());
}
