/*
 * sarr.h - C ABI of the B200 SAR Gaussian-splatting rasterizer (libsarr.so).
 *
 * This library is a drop-in replacement for the native module
 * `cuda_rasterizer_sar` of SAR-3DGS (cuda_rasterizer/rasterizer_impl_v2.cu).
 * Every entry point takes device pointers, plain sizes and a cudaStream_t,
 * never allocates device memory, and returns an int status (SARR_OK == 0).
 * Scratch memory is a caller-provided workspace whose size comes from
 * sarr_workspace_size(); per-view results that a backward pass can reuse
 * live in an optional caller-provided "state" buffer (sarr_state_size()).
 *
 * Semantics that are kept bit-for-bit from the reference rasterizer:
 *   - the image tensor has shape [range_samples, azimuth_samples] but its
 *     memory is laid out as image[c * range_samples + r] (azimuth-major),
 *     c = azimuth pixel, r = range pixel (rasterizer_impl_v2.cu:769, :838);
 *   - each 16x16 tile keeps the first 64 valid Gaussians in index order whose
 *     pixel bbox overlaps the tile's inclusive pixel range (:490-538), and
 *     composites them sorted by (Z_r, index) (:795-807);
 *   - Omega (shadow occlusion) is a side output averaged per Gaussian and never
 *     enters the image (:611-719, :1239-1252);
 *   - the backward reproduces the reference backward_kernel formulas
 *     (:841-1020), including its approximations.
 */
#ifndef SARR_H_
#define SARR_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st *sarr_stream_t;

/* Status codes. */
#define SARR_OK 0
#define SARR_ERR_ARG 1          /* bad argument (null pointer, negative size, bad layout) */
#define SARR_ERR_WORKSPACE 2    /* workspace or state buffer too small or misaligned */
#define SARR_ERR_UNSUPPORTED 3  /* image larger than 2048 x 2048 pixels (128 tiles per axis) */
#define SARR_ERR_CUDA 4         /* a CUDA runtime call or kernel launch failed */
#define SARR_ERR_DEVICE 5       /* a kernel reported an error (bounded wait expired) */
#define SARR_ERR_CAPACITY 6     /* request larger than the static scratch of sarr_forward_static */

/* Covariance input layouts. */
#define SARR_COV6 6   /* [N,6] packed upper triangle xx,yy,zz,xy,xz,yz (cov_3x3_to_6 order) */
#define SARR_COV33 9  /* [N,3,3] full symmetric matrix, row major */

/* Forward/backward flags. */
#define SARR_FLAG_OMEGA 1       /* workspace sizing: forward will compute Omega */
#define SARR_FLAG_ACCUMULATE 2  /* backward: add into the gradient buffers instead of overwriting */
#define SARR_FLAG_TILES_ONLY 4  /* backward: per-tile pass only; rows come from sarr_backward_scatter */
#define SARR_FLAG_RANGE_ROWS 8  /* sarr_backward_scatter: the gradient arrays hold rows [begin, end) only */

/*
 * One radar view. Field meaning and units follow SARRenderParams /
 * SARRasterizationSettings (rasterizer_impl_v2.cu:80-96, :476-488).
 * Angles are in degrees. radar_x and radar_y are accepted but, exactly as in
 * the reference (:1107-1111), the radar position is recomputed from radar_z
 * and the angles.
 */
typedef struct sarr_view {
  float radar_x, radar_y, radar_z;
  float track_angle;
  float incidence_angle;
  float azimuth_angle;
  float range_resolution;
  float azimuth_resolution;
  int32_t range_samples;
  int32_t azimuth_samples;
} sarr_view;

/* Human-readable text for a status code. No reference counterpart. */
const char *sarr_status_string(int status);

/* Library version string. No reference counterpart. */
const char *sarr_version(void);

/*
 * Bytes of workspace needed to process up to `n_views` views of `n` Gaussians
 * per call (views are processed in groups of at most 256 per kernel launch; a
 * smaller workspace than the full request is fine as long as it holds one
 * view: the library then loops over smaller groups). Replaces the ~30
 * per-call cudaMalloc calls of CUDASARRenderer::render
 * (rasterizer_impl_v2.cu:1064-1093) and render_sar_backward (:1434-1463).
 */
int sarr_workspace_size(int64_t n, int range_samples, int azimuth_samples, int n_views,
                        int flags, size_t *bytes);

/*
 * Bytes of one view's forward state (tile lists, sorted tile records and the
 * per-Gaussian tile rectangles) that sarr_backward() can reuse instead of
 * recomputing the forward pipeline. The reference recomputes it
 * (rasterizer_impl_v2.cu:1495-1559).
 */
int sarr_state_size(int64_t n, int range_samples, int azimuth_samples, size_t *bytes);

/*
 * Forward render of n_views views that share (range_samples, azimuth_samples).
 * Replaces render_sar (rasterizer_impl_v2.cu:1618-1662) and
 * render_sar_with_settings (:1664-1699), i.e. CUDASARRenderer::render
 * (:1024-1316), for one view per call or a batch of views.
 *
 *   means   [n,3] float32, cov [n,6] or [n,3,3] float32 (cov_layout),
 *   sigma   [n] float32 (transmittance / opacity after sigmoid),
 *   sh      rows of sh_stride floats, the first sh_k (1..16) used, missing
 *           coefficients read as 0,
 *   images  n_views x (range_samples * azimuth_samples) floats, each image in
 *           the reference's azimuth-major layout,
 *   omega   nullable; n_views x n floats (second output of render_sar),
 *   states  nullable; n_views consecutive buffers of sarr_state_size() bytes
 *           (each 256-byte aligned) receiving the state for sarr_backward(),
 *   ws      workspace from sarr_workspace_size() with SARR_FLAG_OMEGA when
 *           omega is requested, 256-byte aligned.
 */
int sarr_forward(const sarr_view *views, int n_views, int64_t n, const float *means,
                 const float *cov, int cov_layout, const float *sigma, const float *sh,
                 int sh_stride, int sh_k, float *images, float *omega, void *states,
                 void *ws, size_t ws_bytes, sarr_stream_t stream);

/*
 * Gaussian parameters of a training step: replaces
 * GaussianModel.compute_covariance_full / compute_covariance and get_opacity
 * (gaussian_model.py:261-330). For each of the n Gaussians:
 *   cov_out      Sigma = R diag(exp(s))^2 R^T, R from the quaternion
 *                (w, x, y, z) exactly as Quaternion.to_rotation_matrix
 *                builds it (gaussian_model.py:33-55, no normalisation), in
 *                cov_layout (SARR_COV33 [n,3,3] or SARR_COV6 [n,6] in the
 *                rasterizer's xx yy zz xy xz yz order); NULL skips it. The
 *                reference detaches this covariance (no gradient flows back
 *                to scales or rotations); so does this entry point.
 *   opacity_out  sigmoid(opacity_logits); NULL skips it.
 * Inputs scales_log [n,3], rotations [n,4], opacity_logits [n], fp32,
 * contiguous device arrays.
 */
int sarr_gaussian_params(int64_t n, const float *scales_log, const float *rotations,
                         float *cov_out, int cov_layout, const float *opacity_logits,
                         float *opacity_out, sarr_stream_t stream);

/* Weighted-L1 modes of losses.py:28-62 (SARR_L1_PLAIN: the plain mean |p - t|). */
#define SARR_L1_PLAIN 0
#define SARR_L1_LINEAR 1
#define SARR_L1_SQUARE 2
#define SARR_L1_SQRT 3

/* Workspace bytes of sarr_combined_loss for n_images images of height x width. */
int sarr_loss_workspace_size(int n_images, int height, int width, size_t *bytes);

/*
 * CombinedLoss.forward (losses.py:160-219) and its gradient with respect to
 * pred, for n_images images [n_images, height, width] (contiguous fp32):
 *   losses_out [3] (device)  total = l1_weight * L1 + ssim_weight * D-SSIM,
 *                            L1, D-SSIM, each a mean over all pixels of all
 *                            images as the reference computes them for a
 *                            [B, H, W] batch;
 *   grad_pred (nullable)     d total / d pred, the same layout as pred.
 * window_size: odd, <= 11 (the reference's default is 5; Gaussian window of
 * sigma 1.5, zero padding). The loss and its gradient are symmetric under
 * transposing both images, so images in the rasterizer's azimuth-major
 * memory order can be passed as they are. Deterministic (fixed reduction
 * order). No reference counterpart for the fused gradient (the reference
 * differentiates the torch graph).
 */
int sarr_combined_loss(int n_images, int height, int width, const float *pred,
                       const float *target, float l1_weight, float ssim_weight, int window_size,
                       int l1_mode, float *losses_out, float *grad_pred, void *ws, size_t ws_bytes,
                       sarr_stream_t stream);

/*
 * One Adam step over `count` consecutive fp32 parameters: replaces the
 * optimizer.step() of the reference's training step
 * (training/training_pipeline.py:205; torch.optim.Adam built at
 * train.py:429-435 with one learning rate per parameter group, betas and eps
 * at their defaults, no weight decay). Per element, torch.optim.Adam's update:
 *   m = lerp(m, g, 1 - beta1);  v = beta2 v + (1 - beta2) g^2;
 *   p -= lr / (1 - beta1^step) * m / (sqrt(v) / sqrt(1 - beta2^step) + eps),
 * with the bias corrections in double precision as torch evaluates them.
 * Learning rates by segment: element i uses segment_lr[k] for the first k with
 * i < segment_end[k] (host arrays of n_segments <= 8 entries, ends ascending,
 * the last >= count). `step` is the 1-based step count after this update.
 * The arrays are device memory and may be a bucket (sub-range) of flat
 * parameter/gradient/moment buffers.
 */
int sarr_adam_step(int64_t count, float *param, const float *grad, float *exp_avg,
                   float *exp_avg_sq, int n_segments, const int64_t *segment_end,
                   const float *segment_lr, float beta1, float beta2, float eps, int64_t step,
                   sarr_stream_t stream);

/*
 * sarr_adam_step over up to 8 disjoint ranges [range_begin[k], range_end[k])
 * of the flat param / exp_avg / exp_avg_sq arrays in one launch, range k with
 * learning rate range_lr[k] and its gradient at grad[grad_begin[k] + (i -
 * range_begin[k])] (host arrays): the same update, element for element. For
 * a bucket of Gaussians whose parameter groups are not contiguous (their
 * means, opacity and SH rows) and whose gradients are laid out by bucket. No
 * reference counterpart beyond sarr_adam_step's.
 */
int sarr_adam_step_ranges(int n_ranges, const int64_t *range_begin, const int64_t *range_end,
                          const int64_t *grad_begin, const float *range_lr, float *param,
                          const float *grad, float *exp_avg, float *exp_avg_sq, float beta1,
                          float beta2, float eps, int64_t step, sarr_stream_t stream);

/*
 * Densification and pruning (GaussianModel.densify_and_prune,
 * gaussian_model.py:433-566) in two calls, with a host decision between them
 * (the reference's max_gaussians tests, which need the counts):
 *   sarr_densify_flags   per Gaussian: clone = |exp(s)| < size_threshold and
 *                        |grad_mean| > grad_threshold; split = |exp(s)| >
 *                        large_scale_threshold and |grad_mean| >
 *                        grad_threshold; prune = sigmoid(logit) <
 *                        opacity_threshold or |exp(s)| > large_scale_threshold.
 *                        counts_out (device int64 [3]) = kept, clones, splits.
 *   sarr_densify_apply   writes the new set: the kept Gaussians in order,
 *                        then (do_clones) one clone per clone flag with mean
 *                        + 0.01 grad, then (do_splits) two Gaussians per
 *                        split flag with scale log(0.8 exp(s)) and mean
 *                        offsets (0.4 exp(s_x) cos a, 0.4 exp(s_y) sin a, 0)
 *                        for a = 0 and pi (:523-548); output arrays hold kept +
 *                        do_clones * clones + 2 * do_splits * splits rows.
 * Inputs: means [n,3], scales_log [n,3], rotations [n,4], opacity_logits
 * [n], sh [n, sh_cols], grad_means [n,3]; the workspace (from
 * sarr_densify_workspace_size) carries the flags from the first call to the
 * second. Deterministic; no reference counterpart for the split into two calls.
 */
int sarr_densify_workspace_size(int64_t n, size_t *bytes);
int sarr_densify_flags(int64_t n, const float *scales_log, const float *opacity_logits,
                       const float *grad_means, float grad_threshold, float size_threshold,
                       float large_scale_threshold, float opacity_threshold, int64_t *counts_out,
                       void *ws, size_t ws_bytes, sarr_stream_t stream);
int sarr_densify_apply(int64_t n, const float *means, const float *scales_log,
                       const float *rotations, const float *opacity_logits, const float *sh,
                       int sh_cols, const float *grad_means, const int64_t *counts, int do_clones,
                       int do_splits, float *out_means, float *out_scales, float *out_rotations,
                       float *out_opacity_logits, float *out_sh, void *ws, size_t ws_bytes,
                       sarr_stream_t stream);

/*
 * sarr_forward for one view, image only, without a workspace argument: the
 * scratch is an 8 MiB array inside this library, one per device. No
 * counterpart in the reference. It is for callers that cannot allocate
 * device memory: a host whose device memory is all owned by another
 * allocator (a pool reserved at start-up) or a C/C++ caller with no device
 * allocator of its own, for whom cudaMalloc mid-run is not an option (it
 * synchronises the device and can fail under memory pressure).
 *   Limits: n <= 131072 Gaussians, range_samples and azimuth_samples <= 256;
 *           larger requests return SARR_ERR_CAPACITY.
 *   Setup:  the first call in a CUDA context (that context current: the
 *           device's primary context for runtime-API callers) looks up the
 *           scratch's device address once (cudaGetSymbolAddress) and caches it
 *           under the context handle; make that first call before any stream
 *           capture begins. Do not reset the device (cudaDeviceReset) between
 *           calls: the cache does not notice a re-created context.
 *   Zero:   nothing has to start at zero; each call writes every scratch byte
 *           it reads.
 *   Races:  all calls on a device share the scratch; calls on one device
 *           must not overlap (one stream, or ordered by the caller).
 *   Errors: device-side errors of these calls (a bounded wait that expired)
 *           are read with sarr_check_static_errors().
 * Arguments as sarr_forward with n_views = 1, omega = states = NULL. Never
 * allocates device or pinned memory.
 */
int sarr_forward_static(const sarr_view *view, int64_t n, const float *means, const float *cov,
                        int cov_layout, const float *sigma, const float *sh, int sh_stride,
                        int sh_k, float *image, sarr_stream_t stream);

/*
 * Reads and clears the device error word of sarr_forward_static's scratch in
 * the current context (synchronises the stream), as sarr_check_device_errors
 * does for a caller workspace. Returns SARR_OK or SARR_ERR_DEVICE. No
 * counterpart in the reference.
 */
int sarr_check_static_errors(sarr_stream_t stream);

/*
 * Backward of n_views views; the parameter gradients are the SUM over the
 * views (or are added to the buffers with SARR_FLAG_ACCUMULATE).
 * Replaces render_sar_backward (rasterizer_impl_v2.cu:1380-1616) with
 * CUDASARRenderer::backward / backward_kernel (:1318-1377, :841-1020).
 *
 *   grad_images  n_views x (range_samples * azimuth_samples) floats, same
 *                layout as the images (the reference reads grad_output at
 *                pix_c * Nr + pix_r, :905),
 *   states       nullable; the states written by sarr_forward() for these
 *                views and inputs; when null the forward pipeline is recomputed,
 *   grad_means   [n,3]; grad_cov [n,6] (grad_cov_layout SARR_COV6: slots
 *                0,1,3 carry the image-plane rr, cc, rc terms, slots 2,4,5 are
 *                zero, as in the reference :964-969) or [n,3,3] (SARR_COV33,
 *                the cov_6_to_3x3 expansion of the same values);
 *   grad_sigma   [n]; grad_sh [n, grad_sh_cols] with grad_sh_cols in 1..16
 *                (the reference returns 16 columns);
 *   grad_norm    nullable; [n] = ||grad_means[i]||_2, the densification
 *                statistic of GaussianModel.densify_and_prune
 *                (gaussian_model.py:461-466).
 *   flags        SARR_FLAG_ACCUMULATE; SARR_FLAG_TILES_ONLY (n_views <= 256):
 *                only the per-tile pass runs, into ws, and the gradient
 *                arrays are not touched (see sarr_backward_scatter).
 */
int sarr_backward(const sarr_view *views, int n_views, int64_t n, const float *means,
                  const float *cov, int cov_layout, const float *sigma, const float *sh,
                  int sh_stride, int sh_k, const float *grad_images, const void *states,
                  float *grad_means, float *grad_cov, int grad_cov_layout, float *grad_sigma,
                  float *grad_sh, int grad_sh_cols, float *grad_norm, int flags, void *ws,
                  size_t ws_bytes, sarr_stream_t stream);

/*
 * The second half of a backward split in two (no reference counterpart; the
 * reference's backward, rasterizer_impl_v2.cu:1380-1616, is one call): after
 * sarr_backward(..., flags | SARR_FLAG_TILES_ONLY, ws) has run the per-tile
 * pass of n_views <= 256 views into `ws` (which must then hold all of them in
 * one launch group), this writes the dense gradient rows of the Gaussians
 * [begin, end) only, with the same values (and bits) as the single call.
 * Several calls over disjoint ranges produce the whole gradient, so a caller
 * can start reducing one range over GPUs while the next one is written.
 * Arguments: the views, n and states of the SARR_FLAG_TILES_ONLY call; the
 * gradient arrays are the full [n, ...] arrays of sarr_backward (row i at row
 * i), or with SARR_FLAG_RANGE_ROWS arrays of end - begin rows (row i at row
 * i - begin); flags: SARR_FLAG_ACCUMULATE, SARR_FLAG_RANGE_ROWS. The
 * workspace must not be used by another call in between.
 */
int sarr_backward_scatter(const sarr_view *views, int n_views, int64_t n, const void *states,
                          int64_t begin, int64_t end, float *grad_means, float *grad_cov,
                          int grad_cov_layout, float *grad_sigma, float *grad_sh, int grad_sh_cols,
                          float *grad_norm, int flags, void *ws, size_t ws_bytes,
                          sarr_stream_t stream);

/*
 * Test hook: the per-Gaussian intermediate arrays of preprocess_kernel and
 * compute_ranges_kernel (rasterizer_impl_v2.cu:322-470) plus the shadow
 * footprint ranges of build_shadow_tile_list_kernel (:572-597), for one view,
 * computed by the same device code as the production kernels.
 * f32_out: 13 x n floats in the order ipp_r, ipp_c, cov_ipp_rr, cov_ipp_cc,
 * cov_ipp_rc, shadow_x, shadow_y, cov_shadow_xx, cov_shadow_yy,
 * cov_shadow_xy, gaussian_yr, gaussian_z, scattering.
 * i32_out: 10 x n ints: valid, range_min, range_max, azi_min, azi_max,
 * shadow_ok, shadow_c_min, shadow_c_max, shadow_r_min, shadow_r_max.
 */
int sarr_debug_preprocess(const sarr_view *view, int64_t n, const float *means,
                          const float *cov, int cov_layout, const float *sigma,
                          const float *sh, int sh_stride, int sh_k, float *f32_out,
                          int32_t *i32_out, sarr_stream_t stream);

/*
 * Test hook: the capped tile lists of build_tile_gaussian_list_kernel
 * (rasterizer_impl_v2.cu:490-538) and build_shadow_tile_list_kernel
 * (:540-609), and the per-tile depth order used by render_kernel /
 * compute_omega_kernel (:787-807, :674-694), for one view.
 * counts [T] int, lists [T][64] int (index order), sorted [T][64] int
 * (Gaussian ids in compositing order); T = tiles_x * tiles_y,
 * tile id = tile_r * tiles_x + tile_c. Shadow outputs are nullable.
 */
int sarr_debug_tile_lists(const sarr_view *view, int64_t n, const float *means,
                          const float *cov, int cov_layout, const float *sigma,
                          int32_t *counts, int32_t *lists, int32_t *sorted,
                          int32_t *shadow_counts, int32_t *shadow_lists,
                          int32_t *shadow_sorted, void *ws, size_t ws_bytes,
                          sarr_stream_t stream);

/*
 * Test hook: the per-view constants of one view as the kernels see them,
 * written as 30 floats to device memory `out`: radar_x, radar_y, radar_z,
 * track angle [rad], beta [rad], R_c, rho_r, rho_a, Nr, Na, cos(track),
 * sin(track), cos(beta), sin(beta) (the last four evaluated on the device, as
 * the reference's kernels evaluate them, :103-106), then the 16 SH basis
 * values (compute_sh_basis_host, :284-320).
 */
int sarr_debug_view_constants(const sarr_view *view, float *out, sarr_stream_t stream);

/*
 * Test hook (host only, no GPU needed): the tile rectangle this library
 * derives from a clamped pixel bbox [r_min, r_max] x [c_min, c_max]. Tile
 * (tr, tc) is in the rectangle exactly when the reference's hit test of
 * build_tile_gaussian_list_kernel (rasterizer_impl_v2.cu:511-529) passes.
 * Writes tc0, tc1, tr0, tr1 (tc0 > tc1 when no tile is hit).
 */
int sarr_debug_tile_rect(int r_min, int r_max, int c_min, int c_max, int range_samples,
                         int azimuth_samples, int32_t *tc0, int32_t *tc1, int32_t *tr0,
                         int32_t *tr1);

/*
 * Reads and clears the device error word of a workspace (synchronises the
 * stream). Returns SARR_OK or SARR_ERR_DEVICE. No reference counterpart
 * (the reference checks no CUDA error at all).
 */
int sarr_check_device_errors(void *ws, size_t ws_bytes, sarr_stream_t stream);

/* Number of kernels this library has launched in this process. */
int64_t sarr_launch_count(void);

/*
 * Kernel timing (no reference counterpart). While enabled, every kernel
 * launch of this library is bracketed by two CUDA events recorded on the
 * launching stream; sarr_profile_read() waits for them and returns, per
 * kernel kind, the summed device time in milliseconds and the launch count,
 * then clears the record. Kinds are numbered 0 .. SARR_KERNEL_KINDS-1 and
 * named by sarr_kernel_name(). Intended for one device per process.
 */
#define SARR_KERNEL_KINDS 15
int sarr_profile_enable(int enable);
int sarr_profile_read(double *total_ms, int64_t *launches, int n_kinds);
const char *sarr_kernel_name(int kind);

#ifdef __cplusplus
}
#endif

#endif /* SARR_H_ */
