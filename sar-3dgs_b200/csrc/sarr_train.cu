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
//   loss_reduce_kernel       deterministic reduction of the per-block sums;
//   adam_kernel              the Adam update of torch.optim.Adam (the
//                            reference's optimiser, train.py:429-435) over a
//                            flat range of parameters with per-segment
//                            learning rates, so that a bucket of a flat
//                            gradient buffer is updated as soon as its
//                            all-reduce has landed.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "sarr.h"

namespace sarr {
void count_launches(int k);  // the library's launch counter (sarr_abi.cu)
}

namespace {

constexpr int kMaxWindow = 11;

// ---------------------------------------------------------------------------
// producer
// ---------------------------------------------------------------------------
// Sigma = R diag(exp(s))^2 R^T with R from the quaternion (w, x, y, z) as
// Quaternion.to_rotation_matrix writes it (gaussian_model.py:40-51, not
// normalised); transmittance = sigmoid(logit).
__device__ __forceinline__ void gaussian_cov(float l0, float l1, float l2, float w, float x, float y,
                                             float z, float S[3][3]) {
  const float s0 = expf(l0), s1 = expf(l1), s2 = expf(l2);
  const float R[3][3] = {{1.0f - 2.0f * (y * y + z * z), 2.0f * (x * y - w * z), 2.0f * (x * z + w * y)},
                         {2.0f * (x * y + w * z), 1.0f - 2.0f * (x * x + z * z), 2.0f * (y * z - w * x)},
                         {2.0f * (x * z - w * y), 2.0f * (y * z + w * x), 1.0f - 2.0f * (x * x + y * y)}};
  const float d[3] = {s0 * s0, s1 * s1, s2 * s2};
#pragma unroll
  for (int a = 0; a < 3; ++a)
#pragma unroll
    for (int b = 0; b < 3; ++b) S[a][b] = R[a][0] * d[0] * R[b][0] + R[a][1] * d[1] * R[b][1] + R[a][2] * d[2] * R[b][2];
}

// One thread per Gaussian, kParamThreads Gaussians per CTA. `staged`: the
// rows of a full CTA move through shared memory with 16-byte loads and stores
// (all rows of the CTA are contiguous: 3, 4 and 6 or 9 floats per Gaussian),
// so every warp access is coalesced; a partial last CTA, or unaligned
// pointers, read and write per Gaussian.
constexpr int kParamThreads = 256;

__global__ void __launch_bounds__(kParamThreads) gaussian_params_kernel(
    int64_t n, const float* __restrict__ scales, const float* __restrict__ rot, int cov_layout,
    float* __restrict__ cov, const float* __restrict__ logits, float* __restrict__ sigma, bool staged) {
  __shared__ __align__(16) float s_sc[kParamThreads * 3];
  __shared__ __align__(16) float s_cov[kParamThreads * 9];
  const int tid = threadIdx.x;
  const int64_t j0 = (int64_t)blockIdx.x * kParamThreads, j = j0 + tid;
  const bool full = staged && j0 + kParamThreads <= n;  // the same for the whole CTA
  const int cw = cov_layout == SARR_COV33 ? 9 : 6;
  if (cov) {
    float S[3][3];
    if (full) {
      const float4* src = reinterpret_cast<const float4*>(scales + 3 * j0);
      for (int i = tid; i < kParamThreads * 3 / 4; i += kParamThreads)
        reinterpret_cast<float4*>(s_sc)[i] = src[i];
      const float4 q = reinterpret_cast<const float4*>(rot)[j];
      __syncthreads();
      gaussian_cov(s_sc[3 * tid], s_sc[3 * tid + 1], s_sc[3 * tid + 2], q.x, q.y, q.z, q.w, S);
    } else if (j < n) {
      gaussian_cov(scales[3 * j], scales[3 * j + 1], scales[3 * j + 2], rot[4 * j], rot[4 * j + 1],
                   rot[4 * j + 2], rot[4 * j + 3], S);
    }
    float* o = full ? s_cov + cw * tid : cov + cw * j;
    if (full || j < n) {
      if (cw == 9) {
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
          for (int b = 0; b < 3; ++b) o[3 * a + b] = S[a][b];
      } else {  // xx yy zz xy xz yz
        o[0] = S[0][0];
        o[1] = S[1][1];
        o[2] = S[2][2];
        o[3] = S[0][1];
        o[4] = S[0][2];
        o[5] = S[1][2];
      }
    }
    if (full) {
      __syncthreads();
      float4* dst = reinterpret_cast<float4*>(cov + cw * j0);
      for (int i = tid; i < kParamThreads * cw / 4; i += kParamThreads)
        dst[i] = reinterpret_cast<const float4*>(s_cov)[i];
    }
  }
  if (sigma && j < n) sigma[j] = 1.0f / (1.0f + expf(-logits[j]));
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
  bool vec;             // W % 4 == 0 and 16-byte aligned images and workspace (16-byte halo copies)
};

// Loss tiling: a CTA covers kTileX = 32 columns (one per lane) and
// kLossWarps strips of kStrip rows (one strip per warp); each lane walks down
// its column, applying the separable window along the row (from the shared
// memory tile) and then along the column (from the last kWin row sums, kept
// in registers).
constexpr int kTileX = 32;
constexpr int kLossThreads = 128, kLossWarps = kLossThreads / 32;
constexpr int kStrip = 16;                      // rows per warp
constexpr int kTileRows = kLossWarps * kStrip;  // output rows per CTA

// Shared-memory tile of one image: rows [y0 - kHalf, y0 + rows - kHalf),
// columns x0 - kPad + j for j in [0, kTileX + 2 kPad) (kPad = kHalf rounded up
// to 4, so that the interior columns x0 .. x0 + 31 start on a 16-byte
// boundary); only j in [kPad - kHalf, kPad + kTileX + kHalf) is filled.
template <int kHalf>
struct HaloTile {
  static constexpr int kPad = (kHalf + 3) / 4 * 4;
  static constexpr int kPitch = kTileX + 2 * kPad;
};

__device__ __forceinline__ void cp_async4(float* dst, const float* src, bool in) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(in ? 4 : 0) : "memory");
}

__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool in) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(in ? 16 : 0) : "memory");
}

// Fills the tile with cp.async copies (zero-filled outside the image); the
// caller waits with cp_async_wait_all. `vec` (the 32 interior columns lie in
// the image, W % 4 == 0 and `img` is 16-byte aligned): each row's interior
// moves as eight 16-byte copies and only the 2 kHalf halo columns one by one.
template <int kHalf>
__device__ __forceinline__ void load_halo_async(const float* __restrict__ img, int H, int W, int y0,
                                                int x0, int rows, float* tile, bool vec) {
  using HT = HaloTile<kHalf>;
  if (vec) {
    constexpr int kPer = kTileX / 4 + 2 * kHalf;
    for (int it = threadIdx.x; it < rows * kPer; it += kLossThreads) {
      const int r = it / kPer, e = it - r * kPer;
      const int y = y0 - kHalf + r;
      const bool yin = y >= 0 && y < H;
      float* row = tile + r * HT::kPitch;
      if (e < kTileX / 4) {
        cp_async16(row + HT::kPad + 4 * e, yin ? img + (size_t)y * W + x0 + 4 * e : img, yin);
      } else {
        const int h = e - kTileX / 4;
        const int j = h < kHalf ? HT::kPad - kHalf + h : HT::kPad + kTileX + (h - kHalf);
        const int x = x0 - HT::kPad + j;
        const bool in = yin && x >= 0 && x < W;
        cp_async4(row + j, in ? img + (size_t)y * W + x : img, in);
      }
    }
  } else {
    constexpr int kCols = kTileX + 2 * kHalf;
    for (int it = threadIdx.x; it < rows * kCols; it += kLossThreads) {
      const int r = it / kCols, c = it - r * kCols;
      const int y = y0 - kHalf + r, x = x0 - kHalf + c;
      const bool in = y >= 0 && y < H && x >= 0 && x < W;
      cp_async4(tile + r * HT::kPitch + HT::kPad - kHalf + c, in ? img + (size_t)y * W + x : img, in);
    }
  }
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
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
// SSIM map and of the L1 term go to `partial` [2][blocks]. kWin: the (odd)
// window size, so that every window loop unrolls.
template <int kWin>
__global__ void __launch_bounds__(kLossThreads) loss_moments_kernel(const LossParams P,
                                                                    const float* __restrict__ pred,
                                                                    const float* __restrict__ target,
                                                                    const float* __restrict__ tmax_p,
                                                                    float* __restrict__ dgrad,
                                                                    float* __restrict__ partial) {
  constexpr int kHalf = kWin / 2, kIn = kStrip + 2 * kHalf;
  constexpr int kRows = kTileRows + 2 * kHalf, kPitch = HaloTile<kHalf>::kPitch;
  constexpr int kOff = HaloTile<kHalf>::kPad - kHalf;  // tile column of x0 - kHalf
  __shared__ __align__(16) float s_p[kRows * kPitch];
  __shared__ __align__(16) float s_t[kRows * kPitch];
  __shared__ float s_red[2][kLossWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int v = blockIdx.z, y0 = blockIdx.y * kTileRows, x0 = blockIdx.x * kTileX;
  const int H = P.H, W = P.W;
  const size_t img = (size_t)v * H * W, plane = (size_t)P.V * H * W;
  load_halo_async<kHalf>(pred + img, H, W, y0, x0, kRows, s_p, P.vec && x0 + kTileX <= W);
  load_halo_async<kHalf>(target + img, H, W, y0, x0, kRows, s_t, P.vec && x0 + kTileX <= W);
  float g[kWin];
#pragma unroll
  for (int k = 0; k < kWin; ++k) g[k] = P.g[k];
  cp_async_wait_all();
  __syncthreads();
  const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
  const float tmax = tmax_p ? *tmax_p : 0.0f;
  const float gs = -P.ssim_weight * P.inv_count;
  const int x = x0 + lane, rw = warp * kStrip;  // rw: the strip's first row in the tile
  float ssim_sum = 0.f, l1_sum = 0.f;
  float hs[kWin][5];  // row sums of the last kWin input rows (ring)
#pragma unroll
  for (int q = 0; q < kIn; ++q) {
    const float* rp = s_p + (rw + q) * kPitch + kOff + lane;
    const float* rt = s_t + (rw + q) * kPitch + kOff + lane;
    float a = 0.f, b = 0.f, aa = 0.f, bb = 0.f, ab = 0.f;
#pragma unroll
    for (int k = 0; k < kWin; ++k) {
      const float p = rp[k], t = rt[k];
      a += g[k] * p;
      b += g[k] * t;
      aa += g[k] * (p * p);
      bb += g[k] * (t * t);
      ab += g[k] * (p * t);
    }
    float* h = hs[q % kWin];
    h[0] = a;
    h[1] = b;
    h[2] = aa;
    h[3] = bb;
    h[4] = ab;
    if (q < kWin - 1) continue;
    const int o = q - (kWin - 1);  // output row of the strip
    const int y = y0 + rw + o;
    if (y >= H || x >= W) continue;
    float m[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < kWin; ++k)
#pragma unroll
      for (int u = 0; u < 5; ++u) m[u] += g[k] * hs[(o + k) % kWin][u];
    const float mp = m[0], mt = m[1];
    const float mp2 = mp * mp, mt2 = mt * mt, mpt = mp * mt;
    const float sp = m[2] - mp2, st = m[3] - mt2, spt = m[4] - mpt;
    const float A1 = 2.0f * mpt + C1, A2 = 2.0f * spt + C2;
    const float B1 = mp2 + mt2 + C1, B2 = sp + st + C2;
    const float inv = 1.0f / (B1 * B2);
    const float ssim = (A1 * A2) * inv;
    ssim_sum += ssim;
    const float p = s_p[(rw + o + kHalf) * kPitch + kOff + lane + kHalf];
    const float t = s_t[(rw + o + kHalf) * kPitch + kOff + lane + kHalf];
    l1_sum += fabsf(p - t) * l1_factor(P.l1_mode, t, tmax);
    if (dgrad) {
      // 1 / B1 = B2 inv and 1 / B2 = B1 inv
      const float d_mp = 2.0f * mt * A2 * inv - ssim * 2.0f * mp * (B2 * inv);
      const float d_sp = -ssim * (B1 * inv);
      const float d_spt = 2.0f * A1 * inv;
      const size_t oi = img + (size_t)y * W + x;
      dgrad[oi] = gs * (d_mp - 2.0f * mp * d_sp - mt * d_spt);
      dgrad[plane + oi] = gs * d_sp;
      dgrad[2 * plane + oi] = gs * d_spt;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    ssim_sum += __shfl_xor_sync(0xffffffffu, ssim_sum, o);
    l1_sum += __shfl_xor_sync(0xffffffffu, l1_sum, o);
  }
  if (lane == 0) {
    s_red[0][warp] = ssim_sum;
    s_red[1][warp] = l1_sum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f, b = 0.f;
    for (int w = 0; w < kLossWarps; ++w) {
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
template <int kWin>
__global__ void __launch_bounds__(kLossThreads) loss_grad_kernel(const LossParams P,
                                                                 const float* __restrict__ pred,
                                                                 const float* __restrict__ target,
                                                                 const float* __restrict__ tmax_p,
                                                                 const float* __restrict__ dgrad,
                                                                 float* __restrict__ grad) {
  constexpr int kHalf = kWin / 2, kIn = kStrip + 2 * kHalf;
  constexpr int kRows = kTileRows + 2 * kHalf, kPitch = HaloTile<kHalf>::kPitch;
  constexpr int kOff = HaloTile<kHalf>::kPad - kHalf;
  __shared__ __align__(16) float s_d[3][kRows * kPitch];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int v = blockIdx.z, y0 = blockIdx.y * kTileRows, x0 = blockIdx.x * kTileX;
  const int H = P.H, W = P.W;
  const size_t img = (size_t)v * H * W, plane = (size_t)P.V * H * W;
#pragma unroll
  for (int u = 0; u < 3; ++u)
    load_halo_async<kHalf>(dgrad + u * plane + img, H, W, y0, x0, kRows, s_d[u], P.vec && x0 + kTileX <= W);
  float g[kWin];
#pragma unroll
  for (int k = 0; k < kWin; ++k) g[k] = P.g[k];
  cp_async_wait_all();
  __syncthreads();
  const float tmax = tmax_p ? *tmax_p : 0.0f;
  const float l1s = P.l1_weight * P.inv_count;
  const int x = x0 + lane, rw = warp * kStrip;
  float hs[kWin][3];
#pragma unroll
  for (int q = 0; q < kIn; ++q) {
    float a[3] = {0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < kWin; ++k)
#pragma unroll
      for (int u = 0; u < 3; ++u) a[u] += g[k] * s_d[u][(rw + q) * kPitch + kOff + lane + k];
#pragma unroll
    for (int u = 0; u < 3; ++u) hs[q % kWin][u] = a[u];
    if (q < kWin - 1) continue;
    const int o = q - (kWin - 1);
    const int y = y0 + rw + o;
    if (y >= H || x >= W) continue;
    float m[3] = {0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < kWin; ++k)
#pragma unroll
      for (int u = 0; u < 3; ++u) m[u] += g[k] * hs[(o + k) % kWin][u];
    const size_t oi = img + (size_t)y * W + x;
    const float p = pred[oi], t = target[oi];
    const float diff = p - t;
    const float sgn = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
    grad[oi] = l1s * l1_factor(P.l1_mode, t, tmax) * sgn + m[0] + 2.0f * p * m[1] + t * m[2];
  }
}

// losses [3] = total, l1, dssim from the per-CTA sums: thread i adds blocks
// i, i + kReduceThreads, ... in double, then a fixed pairwise tree (the same
// order on every call).
constexpr int kReduceThreads = 1024;

__global__ void __launch_bounds__(kReduceThreads) loss_reduce_kernel(const LossParams P,
                                                                     const float* partial, int nblk,
                                                                     float* losses) {
  __shared__ double s_ssim[kReduceThreads], s_l1[kReduceThreads];
  double ssim = 0.0, l1 = 0.0;
  for (int i = threadIdx.x; i < nblk; i += kReduceThreads) {
    ssim += partial[i];
    l1 += partial[nblk + i];
  }
  s_ssim[threadIdx.x] = ssim;
  s_l1[threadIdx.x] = l1;
  __syncthreads();
  for (int h = kReduceThreads / 2; h > 0; h >>= 1) {
    if ((int)threadIdx.x < h) {
      s_ssim[threadIdx.x] += s_ssim[threadIdx.x + h];
      s_l1[threadIdx.x] += s_l1[threadIdx.x + h];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float l1m = (float)(s_l1[0] * P.inv_count), dssim = (float)(1.0 - s_ssim[0] * P.inv_count);
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
  const size_t blocks = (size_t)((W + kTileX - 1) / kTileX) * ((H + kTileRows - 1) / kTileRows) * V;
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

template <int kWin>
void launch_loss(dim3 grid, cudaStream_t s, const LossParams& P, const float* pred, const float* target,
                 const float* tmax, float* dgrad, float* partial, float* grad_pred) {
  loss_moments_kernel<kWin><<<grid, kLossThreads, 0, s>>>(P, pred, target, tmax, dgrad, partial);
  if (grad_pred) loss_grad_kernel<kWin><<<grid, kLossThreads, 0, s>>>(P, pred, target, tmax, dgrad, grad_pred);
}

// ---------------------------------------------------------------------------
// Adam
// ---------------------------------------------------------------------------
constexpr int kAdamMaxSegments = 8;
constexpr int kAdamThreads = 256;

struct AdamParams {
  int64_t count;
  int nseg;
  int64_t seg_end[kAdamMaxSegments];
  float seg_step[kAdamMaxSegments];  // lr / (1 - beta1^step)
  float beta1, beta2, one_m_beta1, one_m_beta2;
  float bc2_sqrt;                    // sqrt(1 - beta2^step)
  float eps;
};

// One element of torch.optim.Adam's single-tensor update (weight_decay 0, no
// amsgrad): exp_avg.lerp_(grad, 1 - beta1); exp_avg_sq.mul_(beta2)
// .addcmul_(grad, grad, 1 - beta2); denom = sqrt(exp_avg_sq) / bc2_sqrt + eps;
// param.addcdiv_(exp_avg, denom, -step_size).
__device__ __forceinline__ float adam_elem(float p, float g, float& m, float& v, float step_size,
                                           const AdamParams& A) {
  m = __fmaf_rn(A.one_m_beta1, __fsub_rn(g, m), m);
  v = __fadd_rn(__fmul_rn(v, A.beta2), __fmul_rn(__fmul_rn(A.one_m_beta2, g), g));
  const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), A.bc2_sqrt), A.eps);
  return __fadd_rn(p, __fmul_rn(-step_size, __fdiv_rn(m, denom)));
}

__device__ __forceinline__ float adam_step_size(const AdamParams& A, int64_t i) {
  float s = A.seg_step[A.nseg - 1];
  for (int k = A.nseg - 2; k >= 0; --k)
    if (i < A.seg_end[k]) s = A.seg_step[k];
  return s;
}

// Four elements per thread with 16-byte accesses when every array is 16-byte
// aligned; the tail (and unaligned calls) one element per thread.
__global__ void __launch_bounds__(kAdamThreads) adam_kernel(AdamParams A, float* __restrict__ param,
                                                            const float* __restrict__ grad,
                                                            float* __restrict__ m,
                                                            float* __restrict__ v, bool vec) {
  const int64_t t = (int64_t)blockIdx.x * kAdamThreads + threadIdx.x;
  if (vec) {
    const int64_t i = 4 * t;
    if (i + 3 < A.count) {
      float4 p4 = reinterpret_cast<const float4*>(param)[t];
      const float4 g4 = reinterpret_cast<const float4*>(grad)[t];
      float4 m4 = reinterpret_cast<const float4*>(m)[t];
      float4 v4 = reinterpret_cast<const float4*>(v)[t];
      p4.x = adam_elem(p4.x, g4.x, m4.x, v4.x, adam_step_size(A, i), A);
      p4.y = adam_elem(p4.y, g4.y, m4.y, v4.y, adam_step_size(A, i + 1), A);
      p4.z = adam_elem(p4.z, g4.z, m4.z, v4.z, adam_step_size(A, i + 2), A);
      p4.w = adam_elem(p4.w, g4.w, m4.w, v4.w, adam_step_size(A, i + 3), A);
      reinterpret_cast<float4*>(param)[t] = p4;
      reinterpret_cast<float4*>(m)[t] = m4;
      reinterpret_cast<float4*>(v)[t] = v4;
    } else {
      for (int64_t j = i; j < A.count; ++j) {
        float mj = m[j], vj = v[j];
        param[j] = adam_elem(param[j], grad[j], mj, vj, adam_step_size(A, j), A);
        m[j] = mj;
        v[j] = vj;
      }
    }
  } else if (t < A.count) {
    float mj = m[t], vj = v[t];
    param[t] = adam_elem(param[t], grad[t], mj, vj, adam_step_size(A, t), A);
    m[t] = mj;
    v[t] = vj;
  }
}

// Disjoint ranges [begin_k, end_k) of the same flat arrays in one launch
// (grid.y = range), each with its own step size.
struct AdamRanges {
  int n;
  int64_t begin[kAdamMaxSegments], end[kAdamMaxSegments], gbegin[kAdamMaxSegments];
};

__global__ void __launch_bounds__(kAdamThreads) adam_ranges_kernel(AdamParams A, AdamRanges R,
                                                                   float* __restrict__ param,
                                                                   const float* __restrict__ grad,
                                                                   float* __restrict__ m,
                                                                   float* __restrict__ v) {
  const int k = blockIdx.y;
  const int64_t b = R.begin[k], e = R.end[k], gshift = R.gbegin[k] - b;
  const float step_size = A.seg_step[k];
  for (int64_t i = b + (int64_t)blockIdx.x * kAdamThreads + threadIdx.x; i < e;
       i += (int64_t)gridDim.x * kAdamThreads) {
    float mi = m[i], vi = v[i];
    param[i] = adam_elem(param[i], grad[i + gshift], mi, vi, step_size, A);
    m[i] = mi;
    v[i] = vi;
  }
}

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
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool staged = !cov_out || (a16(scales_log) && a16(rotations) && a16(cov_out));
  gaussian_params_kernel<<<(unsigned)((n + kParamThreads - 1) / kParamThreads), kParamThreads, 0, s>>>(
      n, scales_log, rotations, cov_layout, cov_out, opacity_logits, opacity_out, staged);
  sarr::count_launches(1);
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
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  P.vec = (width & 3) == 0 && a16(pred) && a16(target) && a16(ws);

  const float* tmax = nullptr;
  if (l1_mode != SARR_L1_PLAIN) {
    float* tp = reinterpret_cast<float*>(w + L.tmax_partial);
    loss_tmax_kernel<<<kTmaxBlocks, kLossThreads, 0, s>>>(target, (int64_t)n_images * height * width, tp);
    loss_tmax_final_kernel<<<1, 32, 0, s>>>(tp, kTmaxBlocks, reinterpret_cast<float*>(w + L.tmax));
    tmax = reinterpret_cast<const float*>(w + L.tmax);
  }
  const dim3 grid((width + kTileX - 1) / kTileX, (height + kTileRows - 1) / kTileRows, n_images);
  const int nblk = grid.x * grid.y * grid.z;
  float* dgrad = grad_pred ? reinterpret_cast<float*>(w + L.dgrad) : nullptr;
  float* partial = reinterpret_cast<float*>(w + L.partial);
  switch (window_size) {
    case 1: launch_loss<1>(grid, s, P, pred, target, tmax, dgrad, partial, grad_pred); break;
    case 3: launch_loss<3>(grid, s, P, pred, target, tmax, dgrad, partial, grad_pred); break;
    case 5: launch_loss<5>(grid, s, P, pred, target, tmax, dgrad, partial, grad_pred); break;
    case 7: launch_loss<7>(grid, s, P, pred, target, tmax, dgrad, partial, grad_pred); break;
    case 9: launch_loss<9>(grid, s, P, pred, target, tmax, dgrad, partial, grad_pred); break;
    default: launch_loss<11>(grid, s, P, pred, target, tmax, dgrad, partial, grad_pred); break;
  }
  loss_reduce_kernel<<<1, kReduceThreads, 0, s>>>(P, partial, nblk, losses_out);
  sarr::count_launches((l1_mode != SARR_L1_PLAIN ? 2 : 0) + (grad_pred ? 3 : 2));
  return cuda_status(cudaGetLastError());
}

extern "C" int sarr_adam_step(int64_t count, float* param, const float* grad, float* exp_avg,
                              float* exp_avg_sq, int n_segments, const int64_t* segment_end,
                              const float* segment_lr, float beta1, float beta2, float eps,
                              int64_t step, sarr_stream_t stream) {
  if (count < 0 || step < 1 || n_segments < 1 || n_segments > kAdamMaxSegments) return SARR_ERR_ARG;
  if (!segment_end || !segment_lr) return SARR_ERR_ARG;
  if (!(beta1 >= 0.0f && beta1 < 1.0f && beta2 >= 0.0f && beta2 < 1.0f)) return SARR_ERR_ARG;
  if (count == 0) return SARR_OK;
  if (!param || !grad || !exp_avg || !exp_avg_sq) return SARR_ERR_ARG;
  AdamParams A;
  memset(&A, 0, sizeof(A));
  A.count = count;
  A.nseg = n_segments;
  // torch.optim.Adam evaluates the bias corrections in double precision
  const double bc1 = 1.0 - pow((double)beta1, (double)step);
  const double bc2 = 1.0 - pow((double)beta2, (double)step);
  for (int k = 0; k < n_segments; ++k) {
    if (k > 0 && segment_end[k] < segment_end[k - 1]) return SARR_ERR_ARG;
    A.seg_end[k] = segment_end[k];
    A.seg_step[k] = (float)((double)segment_lr[k] / bc1);
  }
  if (segment_end[n_segments - 1] < count) return SARR_ERR_ARG;
  A.beta1 = beta1;
  A.beta2 = beta2;
  A.one_m_beta1 = (float)(1.0 - (double)beta1);
  A.one_m_beta2 = (float)(1.0 - (double)beta2);
  A.bc2_sqrt = (float)sqrt(bc2);
  A.eps = eps;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec = a16(param) && a16(grad) && a16(exp_avg) && a16(exp_avg_sq);
  const int64_t threads = vec ? (count + 3) / 4 : count;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  adam_kernel<<<(unsigned)((threads + kAdamThreads - 1) / kAdamThreads), kAdamThreads, 0, s>>>(
      A, param, grad, exp_avg, exp_avg_sq, vec);
  sarr::count_launches(1);
  return cuda_status(cudaGetLastError());
}

extern "C" int sarr_adam_step_ranges(int n_ranges, const int64_t* range_begin,
                                     const int64_t* range_end, const int64_t* grad_begin,
                                     const float* range_lr, float* param, const float* grad,
                                     float* exp_avg, float* exp_avg_sq, float beta1, float beta2,
                                     float eps, int64_t step, sarr_stream_t stream) {
  if (n_ranges < 1 || n_ranges > kAdamMaxSegments || step < 1) return SARR_ERR_ARG;
  if (!range_begin || !range_end || !grad_begin || !range_lr) return SARR_ERR_ARG;
  if (!(beta1 >= 0.0f && beta1 < 1.0f && beta2 >= 0.0f && beta2 < 1.0f)) return SARR_ERR_ARG;
  if (!param || !grad || !exp_avg || !exp_avg_sq) return SARR_ERR_ARG;
  AdamParams A;
  memset(&A, 0, sizeof(A));
  AdamRanges R;
  memset(&R, 0, sizeof(R));
  const double bc1 = 1.0 - pow((double)beta1, (double)step);
  const double bc2 = 1.0 - pow((double)beta2, (double)step);
  int64_t longest = 0;
  R.n = n_ranges;
  for (int k = 0; k < n_ranges; ++k) {
    if (range_begin[k] < 0 || range_end[k] < range_begin[k] || grad_begin[k] < 0) return SARR_ERR_ARG;
    R.begin[k] = range_begin[k];
    R.end[k] = range_end[k];
    R.gbegin[k] = grad_begin[k];
    A.seg_step[k] = (float)((double)range_lr[k] / bc1);
    if (range_end[k] - range_begin[k] > longest) longest = range_end[k] - range_begin[k];
  }
  if (longest == 0) return SARR_OK;
  A.nseg = n_ranges;
  A.beta1 = beta1;
  A.beta2 = beta2;
  A.one_m_beta1 = (float)(1.0 - (double)beta1);
  A.one_m_beta2 = (float)(1.0 - (double)beta2);
  A.bc2_sqrt = (float)sqrt(bc2);
  A.eps = eps;
  const int64_t blocks = (longest + kAdamThreads - 1) / kAdamThreads;
  const dim3 grid((unsigned)(blocks < 148 * 8 ? blocks : 148 * 8), (unsigned)n_ranges);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  adam_ranges_kernel<<<grid, kAdamThreads, 0, s>>>(A, R, param, grad, exp_avg, exp_avg_sq);
  sarr::count_launches(1);
  return cuda_status(cudaGetLastError());
}
