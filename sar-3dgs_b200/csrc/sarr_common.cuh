// Shared device code of the B200 SAR rasterizer: constants, per-view constants,
// the per-Gaussian radar projection, the tile records and the TMA helpers.
//
// Floating-point expressions that decide tile membership, validity and the
// pixel value are written term by term in the same order as the reference
// (cuda_rasterizer/rasterizer_impl_v2.cu), zero terms included: nvcc contracts
// a*b+c into fma, and the rounding of the result depends on which product is
// fused, so the expression trees must be the same for the tile lists to be
// bit-exact. Everything else (data movement, tile selection, sorting,
// reductions) is this library's own design.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sarr {

// Constants fixed by the reference (rasterizer_impl_v2.cu:10-13, :472-474).
constexpr float kEps = 1e-6f;                   // EPSILON
constexpr float kPi = 3.14159265358979323846f;  // PI
constexpr int kTile = 16;                       // BLOCK_X == BLOCK_Y
constexpr int kCap = 64;                        // MAX_GAUSSIANS_PER_TILE
constexpr int kSh = 16;                         // SH_COEFFS_SIZE

// Design constants of this implementation.
constexpr int kBinThreads = 256;                 // threads of a binning CTA
constexpr int kBinPerThread = 4;                 // Gaussians per binning thread
constexpr int kChunk = kBinThreads * kBinPerThread;  // Gaussians per count row
constexpr int kSelectThreads = 128;
constexpr int kScanThreads = 512;                // scan4_kernel (4 tiles per lane)
constexpr int kScan1Threads = 1024;              // scan_kernel (1 tile per lane, few views: more warps per tile column)
#ifndef SARR_PREFIX_CHUNKS
#define SARR_PREFIX_CHUNKS 64
#endif
constexpr int kPrefixChunks = SARR_PREFIX_CHUNKS;  // chunks binned exactly before saturation skipping
// Images of at most this many tiles keep per-(chunk, tile) hit words for the
// first-stage prefix chunks (selection reads hits instead of re-testing
// rectangles).
constexpr int kHitBitsMaxTiles = 1024;
#ifndef SARR_PREFIX_STAGE1
#define SARR_PREFIX_STAGE1 8
#endif
constexpr int kPrefixStage1 = SARR_PREFIX_STAGE1;  // cell-culled calls: chunks of the prefix binned exactly
constexpr int kXCap = kChunk;                    // exactly binned Gaussians listed per skipped chunk
constexpr int kSegMaskMaxTiles = 2048;           // prefix-chunk segment masks up to this many tiles
constexpr int kSegMaskAllMaxTiles = 512;         // segment masks of every chunk up to this many tiles
constexpr int kWarpsPerTile = 8;                 // 8 warps x 32 pixels = one 16x16 tile
constexpr int kMaxTilesAxis = 128;               // images up to 2048 x 2048
constexpr int kMaxViewsPerLaunch = 256;
constexpr int kGatherScanBlock = 4096;           // elements per CTA of the backward's index scan
constexpr uint32_t kEmptyRect = 0x000000FFu;     // tc0 = 255 > tc1 = 0

// Device error bits (workspace error word).
// Cell culling of multi-view launches: a view-independent grid of cells over
// the Gaussian centres; per view, one bit per cell says whether any member
// can reach a tile that is still open after the saturation prefix.
constexpr int kMaxCells = 65536;
constexpr int kCellWords = kMaxCells / 32;
// Cells split the Gaussians of a spatial cell by their bbox bound, so that a
// cell's largest bound stays close to its members' bounds.
constexpr int kHbBuckets = 4;
constexpr int kMaxSpatialCells = kMaxCells / kHbBuckets;
__host__ __device__ __forceinline__ int hb_bucket(float hb) {
  return (int)(hb > 6.0f) + (int)(hb > 8.0f) + (int)(hb > 11.0f);
}
constexpr int kCellMinViews = 8;                 // calls with fewer views bin without cells
constexpr uint32_t kCellAlways = 0xFFFFFFFFu;    // no cell: always tested individually
constexpr uint32_t kCellNever = 0xFFFFFFFEu;     // transmittance < 0.01: never in a list
constexpr float kCellMaxHalfBound = 64.0f;       // larger bbox bounds are never culled

struct SceneGrid {
  int lo_key[3], hi_key[3];  // ordered-int keys of the finite centres' bounding box
  float lo[3];
  float a, inv_a;            // cell edge [m] and its inverse
  int dims[3];
  int ncells;
  float half_diag;           // bound on |member centre - cell centre| [m], with margins
  int valid;                 // 0: no finite centre (no Gaussian is in a cell)
  int nspatial;              // spatial cells (ncells = nspatial * kHbBuckets)
  int block_sums[kMaxCells / 1024];  // member counts per 1024 cells (scan scratch)
  int n_always;              // Gaussians after the prefix that are in no cell
};

// Spatial cells are numbered in blocks of 4 x 4 x 2 grid cells, the blocks in
// x-major order, so that a warp of cell_test_kernel (32 cells) and a bitmap
// word of bin_cand_kernel (8 cells) cover compact pieces of the scene: the
// candidate cells of a view, which lie along the scene's edges in its image,
// gather into fewer warps and words (cell test 0.55 -> 0.49 ms, candidate
// test 0.71 -> 0.68 ms per 1024 sweep views against x-major rows). The grid
// is padded to whole blocks (padding cells have no members).
constexpr int kCellBlock = 32;
__host__ __device__ __forceinline__ int64_t padded_spatial_cells(const int dims[3]) {
  return (int64_t)((dims[0] + 3) / 4) * ((dims[1] + 3) / 4) * ((dims[2] + 1) / 2) * kCellBlock;
}
__host__ __device__ __forceinline__ int spatial_cell(const int dims[3], int ix, int iy, int iz) {
  const int nbx = (dims[0] + 3) / 4, nby = (dims[1] + 3) / 4;
  const int blk = ((iz >> 1) * nby + (iy >> 2)) * nbx + (ix >> 2);
  return blk * kCellBlock + (((iz & 1) * 4 + (iy & 3)) * 4 + (ix & 3));
}

// Order-preserving map of floats to ints (for atomicMin / atomicMax).
__device__ __forceinline__ int ordered_key(float f) {
  const int i = __float_as_int(f);
  return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float key_float(int k) {
  return __int_as_float(k >= 0 ? k : k ^ 0x7FFFFFFF);
}

constexpr int kDevErrTmaTimeout = 1;
constexpr int kDevErrListSlot = 2;

// Per-view values computed on the host exactly as CUDASARRenderer::render
// does (rasterizer_impl_v2.cu:1100-1120).
struct ViewHost {
  float radar_x, radar_y, radar_z;
  float alpha;  // track angle [rad]
  float beta;   // asin(sin(incidence) cos(azimuth)) [rad]
  float Rc;     // scene-centre slant range
  float rho_r, rho_a;
  int Nr, Na;
  float sh_basis[kSh];
};

// ViewHost plus the rotation trig, evaluated on the device with CUDA's
// cosf/sinf like the reference kernels do (:103-106, :128-131), and the
// per-view products of the projection, computed once per view with the same
// operations (and so the same bits) the per-Gaussian code would use.
struct ViewConst {
  ViewHost h;
  float cos_a, sin_a, cos_b, sin_b;
  int tiles_x, tiles_y;
  float cb_sa, cb_ca, sb_ca, sb_sa;      // world_to_radar products
  float half_Nr, half_Na, Rc_rho;        // Nr/2, Na/2, R_c / rho_r
  float J10;                             // 1 / rho_a
  float kXX[6], kYY[6], kZZ[6], kXY[6], kXZ[6], kYZ[6];  // Sigma_r = R Sigma R^T coefficients
  float kcc[6];                          // cov_cc = J10^2 XX (+ zero terms)
  float krc0;                            // J00 * J10
  float inv_rho_r, inv_rho_a;            // fast approximate centre (saturation skipping)
  float center_margin;                   // its error bound [px], with room to spare
};

template <int kViews>
struct ViewHostPackN {
  int n;
  ViewHost v[kViews];
};
using ViewHostPack = ViewHostPackN<kMaxViewsPerLaunch>;
constexpr int kSmallViewPack = 8;  // parameter block of launches of at most 8 views

// One Gaussian of a tile list, as the compositing kernels read it.
// For the image-plane list (mx, my) = (ipp_c, ipp_r) and (cxx, cxy, cyy) =
// (cov_cc, cov_rc, cov_rr): the argument order of compute_gaussian_density_2d
// in render_kernel (:815-819). For the shadow list (mx, my) = (X_r, Y_r) and
// (cxx, cxy, cyy) = (cov_XrXr, cov_XrYr, cov_YrYr) (:701-705).
struct __align__(16) Rec {
  float mx, my;
  float cxx, cxy, cyy;
  float inv_det;  // 1 / (cxx*cyy - cxy*cxy)
  float norm;     // 2*PI*sqrt(det); -1 marks |det| < EPSILON (density is 0)
  float sigma;    // transmittance
  float s_pos;    // max(0, S), S the leaky-ReLU SH scattering (image list only)
  float z;        // Z_r, the depth sort key
  float yr;       // Y_r (backward chain)
  int pos;        // slot of this Gaussian in the index-ordered tile list
};
static_assert(sizeof(Rec) == 48, "Rec must stay 48 bytes (TMA bulk granularity)");

// Radar-frame projection of one Gaussian.
struct Proj {
  float xr, yr, zr;
  float r, c;                    // ipp_r, ipp_c
  float cov_rr, cov_cc, cov_rc;  // image-plane covariance [pixel^2]
  float XX, YY, XY;              // radar-frame covariance block used for the shadow plane
};

__device__ __forceinline__ void load_cov6(const float* __restrict__ p, int layout, float cw[6]) {
  if (layout == 6) {
    cw[0] = p[0]; cw[1] = p[1]; cw[2] = p[2]; cw[3] = p[3]; cw[4] = p[4]; cw[5] = p[5];
  } else {  // [3,3] row major: xx yy zz xy xz yz = [0] [4] [8] [1] [2] [5]
    cw[0] = p[0]; cw[1] = p[4]; cw[2] = p[8]; cw[3] = p[1]; cw[4] = p[2]; cw[5] = p[5];
  }
}

// IEEE single-precision operations that the compiler may neither contract
// nor reassociate. The reference is compiled with nvcc's default FMA
// contraction, so its results depend on which products got fused; the
// expressions below spell out that fusion explicitly (established bit for bit
// against the reference's own kernels on a B200), which makes the results
// independent of how this file's surrounding code is compiled.
__device__ __forceinline__ float mul_(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float sub_(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fma_(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ float div_(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float sqrt_(float a) { return __fsqrt_rn(a); }

// k0 x0 + k1 x1 + ... + k5 x5 left to right: the first product fused into the
// first addition, every later product fused into the running sum.
__device__ __forceinline__ float chain6(const float k[6], const float x[6]) {
  float s = fma_(k[0], x[0], mul_(k[1], x[1]));
#pragma unroll
  for (int i = 2; i < 6; ++i) s = fma_(k[i], x[i], s);
  return s;
}

// Per-view products of the projection (:98-203): R = the world-to-radar
// rotation rows, the coefficients of Sigma_r = R Sigma R^T per output entry,
// and the view-only Jacobian terms. Same operations as the per-Gaussian code
// would perform, so the same bits.
__device__ __forceinline__ void view_derive(ViewConst& v) {
  const float ca = v.cos_a, sa = v.sin_a, cb = v.cos_b, sb = v.sin_b;
  v.cb_sa = mul_(cb, sa);
  v.cb_ca = mul_(cb, ca);
  v.sb_ca = mul_(sb, ca);
  v.sb_sa = mul_(sb, sa);
  v.half_Nr = mul_((float)v.h.Nr, 0.5f);
  v.half_Na = mul_((float)v.h.Na, 0.5f);
  v.Rc_rho = div_(v.h.Rc, v.h.rho_r);
  const float R00 = ca, R01 = sa, R02 = 0.0f;
  const float R10 = v.cb_sa, R11 = -v.cb_ca, R12 = -sb;
  const float R20 = -v.sb_sa, R21 = v.sb_ca, R22 = -cb;
  const float kXX[6] = {mul_(R00, R00), mul_(R01, R01), mul_(R02, R02), mul_(mul_(2.0f, R00), R01),
                        mul_(mul_(2.0f, R00), R02), mul_(mul_(2.0f, R01), R02)};
  const float kYY[6] = {mul_(R10, R10), mul_(R11, R11), mul_(R12, R12), mul_(mul_(2.0f, R10), R11),
                        mul_(mul_(2.0f, R10), R12), mul_(mul_(2.0f, R11), R12)};
  const float kZZ[6] = {mul_(R20, R20), mul_(R21, R21), mul_(R22, R22), mul_(mul_(2.0f, R20), R21),
                        mul_(mul_(2.0f, R20), R22), mul_(mul_(2.0f, R21), R22)};
  const float kXY[6] = {mul_(R00, R10), mul_(R01, R11), mul_(R02, R12), fma_(R00, R11, mul_(R01, R10)),
                        fma_(R00, R12, mul_(R02, R10)), fma_(R01, R12, mul_(R02, R11))};
  const float kXZ[6] = {mul_(R00, R20), mul_(R01, R21), mul_(R02, R22), fma_(R00, R21, mul_(R01, R20)),
                        fma_(R00, R22, mul_(R02, R20)), fma_(R01, R22, mul_(R02, R21))};
  const float kYZ[6] = {mul_(R10, R20), mul_(R11, R21), mul_(R12, R22), fma_(R10, R21, mul_(R11, R20)),
                        fma_(R12, R20, mul_(R10, R22)), fma_(R12, R21, mul_(R11, R22))};
  const float J00 = 0.0f, J11 = 0.0f, J12 = 0.0f;
  const float J10 = div_(1.0f, v.h.rho_a);
  const float kcc[6] = {mul_(J10, J10), mul_(J11, J11), mul_(J12, J12), mul_(mul_(2.0f, J10), J11),
                        mul_(mul_(2.0f, J10), J12), mul_(mul_(2.0f, J11), J12)};
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    v.kXX[i] = kXX[i];
    v.kYY[i] = kYY[i];
    v.kZZ[i] = kZZ[i];
    v.kXY[i] = kXY[i];
    v.kXZ[i] = kXZ[i];
    v.kYZ[i] = kYZ[i];
    v.kcc[i] = kcc[i];
  }
  v.J10 = J10;
  v.krc0 = mul_(J00, J10);
  v.inv_rho_r = 1.0f / v.h.rho_r;
  v.inv_rho_a = 1.0f / v.h.rho_a;
  // the approximate centre's error grows with the magnitude of the cancelling
  // slant-range terms R_min / rho_r and R_c / rho_r (a few ulps of them)
  v.center_margin = 0.25f + 4e-6f * fabsf(v.Rc_rho);
}

// world_to_radar + project_to_ipp (:98-113, :160-174): radar-frame centre and
// image-plane position. Returns R_min.
__device__ __forceinline__ float project_center(const ViewConst& v, float px, float py, float pz,
                                                Proj& o) {
  const float dx = sub_(px, v.h.radar_x);
  const float dy = sub_(py, v.h.radar_y);
  const float dz = sub_(pz, v.h.radar_z);
  o.xr = fma_(v.cos_a, dx, mul_(v.sin_a, dy));
  o.yr = fma_(-v.sin_b, dz, fma_(v.cb_sa, dx, -mul_(v.cb_ca, dy)));
  o.zr = fma_(-v.cos_b, dz, fma_(v.sb_ca, dy, -mul_(v.sb_sa, dx)));
  const float Rmin = sqrt_(add_(fma_(o.yr, o.yr, mul_(o.zr, o.zr)), kEps * kEps));
  o.r = sub_(add_(div_(Rmin, v.h.rho_r), v.half_Nr), v.Rc_rho);
  o.c = add_(div_(o.xr, v.h.rho_a), v.half_Na);
  return Rmin;
}

// transform_covariance_3x3 (:115-158): the six entries of Sigma_r = R Sigma R^T
// in the order XX, YY, ZZ, XY, XZ, YZ. Zero entries of R (R02) are kept as
// terms: they leave finite results unchanged and propagate non-finite inputs
// as the reference does.
__device__ __forceinline__ void radar_cov(const ViewConst& v, const float cw[6], float X6[6]) {
  const float x6[6] = {cw[0], cw[1], cw[2], cw[3], cw[4], cw[5]};  // xx yy zz xy xz yz
  X6[0] = chain6(v.kXX, x6);
  X6[1] = chain6(v.kYY, x6);
  X6[2] = chain6(v.kZZ, x6);
  X6[3] = chain6(v.kXY, x6);
  X6[4] = chain6(v.kXZ, x6);
  X6[5] = chain6(v.kYZ, x6);
}

// compute_jacobian_ipp + project_covariance_ipp + project_covariance_shadow
// (:176-213) from Sigma_r. Zero entries of J (J00, J11, J12) are kept as terms.
__device__ __forceinline__ void image_cov(const ViewConst& v, const float X6[6], float Rmin,
                                          Proj& o) {
  const float J00 = 0.0f, J11 = 0.0f, J12 = 0.0f;
  const float rR = mul_(v.h.rho_r, Rmin);
  const float J01 = div_(o.yr, rR);
  const float J02 = div_(o.zr, rR);
  const float J10 = v.J10;
  const float krr[6] = {mul_(J00, J00), mul_(J01, J01), mul_(J02, J02), mul_(mul_(2.0f, J00), J01),
                        mul_(mul_(2.0f, J00), J02), mul_(mul_(2.0f, J01), J02)};
  const float krc[6] = {v.krc0, mul_(J01, J11), mul_(J02, J12), fma_(J01, J10, mul_(J00, J11)),
                        fma_(J02, J10, mul_(J00, J12)), fma_(J01, J12, mul_(J02, J11))};
  o.cov_rr = chain6(krr, X6);
  o.cov_cc = chain6(v.kcc, X6);
  o.cov_rc = chain6(krc, X6);
  o.XX = X6[0];
  o.YY = X6[1];
  o.XY = X6[3];
}

__device__ __forceinline__ void project_cov(const ViewConst& v, const float cw[6], float Rmin,
                                            Proj& o) {
  float X6[6];
  radar_cov(v, cw, X6);
  image_cov(v, X6, Rmin, o);
}

// A bound valid for every view on the half-widths of the reference's 3-sigma
// bboxes (pixels for the image plane, metres for the shadow footprint).
// Both use std = sqrt(max(a*b / max(det, EPS), EPS)) <= 1/sqrt(1 - rho^2) for
// the correlation rho of two projections of the Gaussian on orthogonal
// directions (image plane: the radar X axis and a Y/Z combination; shadow: X
// and Y). By Wielandt's inequality rho^2 <= ((kappa-1)/(kappa+1))^2 for the
// covariance's condition number kappa, so std^2 <= (kappa+1)^2 / (4 kappa); a
// 1% relative and 1.5 px absolute margin cover the float rounding of the
// reference's own evaluation, which stays far below 1% for kappa <= 2.5e4.
// The eigenvalues come from the closed-form trigonometric solution of the
// symmetric 3x3 eigenproblem; a slack of 1e-5 * lambda_max on both extreme eigenvalues covers its float error.
// +inf for covariances that are not clearly positive definite or have
// kappa > 2.5e4.
__device__ __forceinline__ float view_free_half_bound(const float cw[6]) {
  const float xx = cw[0], yy = cw[1], zz = cw[2], xy = cw[3], xz = cw[4], yz = cw[5];
  const float q = (xx + yy + zz) * (1.0f / 3.0f);
  const float axx = xx - q, ayy = yy - q, azz = zz - q;
  const float p2 = axx * axx + ayy * ayy + azz * azz + 2.0f * (xy * xy + xz * xz + yz * yz);
  float lmax = q, lmin = q;
  if (p2 > 0.0f) {
    const float p = sqrtf(p2 * (1.0f / 6.0f));
    const float inv = 1.0f / p;
    const float bxx = axx * inv, byy = ayy * inv, bzz = azz * inv;
    const float bxy = xy * inv, bxz = xz * inv, byz = yz * inv;
    const float detB = bxx * (byy * bzz - byz * byz) - bxy * (bxy * bzz - byz * bxz) +
                       bxz * (bxy * byz - byy * bxz);
    const float hr = fminf(fmaxf(0.5f * detB, -1.0f), 1.0f);
    const float phi = acosf(hr) * (1.0f / 3.0f);
    lmax = q + 2.0f * p * cosf(phi);
    lmin = q + 2.0f * p * cosf(phi + 2.0943951f);
  }
  const float slack = 1e-5f * fabsf(lmax);
  const float hi = lmax + slack, lo = lmin - slack;
  if (!(lo > 0.0f) || !(hi > 0.0f)) return INFINITY;
  const float kappa = hi / lo;
  if (!(kappa < 2.5e4f)) return INFINITY;
  return 3.0f * ((kappa + 1.0f) / (2.0f * sqrtf(kappa))) * 1.01f + 1.5f;
}

// Centre of a Gaussian in the image plane (pixels) and the shadow plane
// (metres) with fast arithmetic. Its error against project_center is a few
// ulps of the cancelling slant-range terms R_min / rho_r and R_c / rho_r
// (about 0.01 px for a 5 km altitude at 0.2 m), which ViewConst::center_margin
// bounds with room to spare.
__device__ __forceinline__ void approx_center(const ViewConst& v, float px, float py, float pz,
                                              float& r, float& c, float& xr, float& yr) {
  const float dx = px - v.h.radar_x, dy = py - v.h.radar_y, dz = pz - v.h.radar_z;
  xr = v.cos_a * dx + v.sin_a * dy;
  yr = -v.sin_b * dz + (v.cb_sa * dx - v.cb_ca * dy);
  const float zr = -v.cos_b * dz + (v.sb_ca * dy - v.sb_sa * dx);
  const float R2 = yr * yr + zr * zr + kEps * kEps;
  const float Rmin = R2 * rsqrtf(R2);
  r = (Rmin - v.h.Rc) * v.inv_rho_r + v.half_Nr;
  c = xr * v.inv_rho_a + v.half_Na;
}

// The whole per-Gaussian projection of preprocess_kernel (:356-403).
__device__ __forceinline__ void project_gaussian(const ViewConst& v, float px, float py, float pz,
                                                 const float cw[6], Proj& o) {
  const float Rmin = project_center(v, px, py, pz, o);
  project_cov(v, cw, Rmin, o);
}

// preprocess_kernel's validity test (:405-406); the sigma < 0.01 test
// (:351) is applied by the callers before projecting.
__device__ __forceinline__ bool proj_valid(const Proj& o, int Nr, int Na) {
  return (o.r >= 0 && o.r < (float)Nr && o.c >= 0 && o.c < (float)Na);
}

// compute_ranges_kernel for a valid Gaussian (:446-464).
__device__ __forceinline__ void ipp_ranges(const Proj& o, int Nr, int Na, int& r_min, int& r_max,
                                           int& c_min, int& c_max) {
  const float cov_rr = o.cov_rr, cov_cc = o.cov_cc, cov_rc = o.cov_rc;
  float det = fma_(cov_rr, cov_cc, -mul_(cov_rc, cov_rc));
  if (det < kEps) det = kEps;
  const float inv_det = div_(1.0f, det);
  // std_r and std_c of the reference are the same value: cov_rr*cov_cc and
  // cov_cc*cov_rr are equal in IEEE arithmetic.
  const float std_r = sqrt_(fmaxf(mul_(mul_(cov_rr, cov_cc), inv_det), kEps));
  const float std_c = std_r;
  r_min = (int)floorf(fma_(-3.0f, std_r, o.r));
  r_max = (int)ceilf(fma_(3.0f, std_r, o.r));
  c_min = (int)floorf(fma_(-3.0f, std_c, o.c));
  c_max = (int)ceilf(fma_(3.0f, std_c, o.c));
  r_min = max(0, r_min);
  r_max = min(Nr - 1, r_max);
  c_min = max(0, c_min);
  c_max = min(Na - 1, c_max);
}

// build_shadow_tile_list_kernel's footprint of a valid Gaussian (:572-597).
// Returns false when |det| < EPSILON (the reference skips the Gaussian).
__device__ __forceinline__ bool shadow_ranges(const Proj& o, int Nr, int Na, int& r_min, int& r_max,
                                              int& c_min, int& c_max) {
  const float mux = o.xr, muy = o.yr;
  const float cov_xx = o.XX, cov_yy = o.YY, cov_xy = o.XY;
  const float det = fma_(cov_xx, cov_yy, -mul_(cov_xy, cov_xy));
  if (fabsf(det) < kEps) return false;
  const float inv_det = div_(1.0f, det);
  const float std_xy = sqrt_(fmaxf(mul_(mul_(cov_xx, cov_yy), inv_det), kEps));  // std_x == std_y
  c_min = (int)floorf(fma_(-3.0f, std_xy, mux));
  c_max = (int)ceilf(fma_(3.0f, std_xy, mux));
  r_min = (int)floorf(fma_(-3.0f, std_xy, muy));
  r_max = (int)ceilf(fma_(3.0f, std_xy, muy));
  c_min = max(0, c_min);
  c_max = min(Na - 1, c_max);
  r_min = max(0, r_min);
  r_max = min(Nr - 1, r_max);
  return true;
}

// Tiles hit by a pixel bbox, packed as 4 bytes (tc0, tc1, tr0, tr1).
// The reference hit test for tile (tr, tc) (:511-529) is
//   !(r_max < 16 tr || r_min > min(16 tr + 16, Nr) || c_max < 16 tc || c_min > min(16 tc + 16, Na))
// (an inclusive upper pixel bound, so neighbouring tiles overlap by one
// pixel). Solved for the tile index: tr in [ceil((r_min-16)/16), floor(r_max/16)]
// when 0 <= r_max and r_min <= Nr, otherwise no tile.
__host__ __device__ __forceinline__ uint32_t make_rect(int r_min, int r_max, int c_min, int c_max,
                                                       int Nr, int Na) {
  if (r_max < 0 || c_max < 0 || r_min > Nr || c_min > Na) return kEmptyRect;
  const int tr0 = (r_min > 0 ? r_min - 1 : 0) / kTile;
  const int tr1 = r_max / kTile;
  const int tc0 = (c_min > 0 ? c_min - 1 : 0) / kTile;
  const int tc1 = c_max / kTile;
  if (tr0 > tr1 || tc0 > tc1) return kEmptyRect;
  return (uint32_t)tc0 | ((uint32_t)tc1 << 8) | ((uint32_t)tr0 << 16) | ((uint32_t)tr1 << 24);
}

__host__ __device__ __forceinline__ bool rect_has(uint32_t rc, int tx, int ty) {
  const int tc0 = rc & 0xFF, tc1 = (rc >> 8) & 0xFF, tr0 = (rc >> 16) & 0xFF, tr1 = rc >> 24;
  return tx >= tc0 && tx <= tc1 && ty >= tr0 && ty <= tr1;
}

// compute_sh_scattering_with_basis (:236-244). A full 16-coefficient row
// that is 16-byte aligned is read with four 16-byte loads.
__device__ __forceinline__ float sh_scattering(const ViewConst& v, const float* __restrict__ row,
                                               int sh_k) {
  float c[kSh];
  if (sh_k == kSh && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
#pragma unroll
    for (int q = 0; q < kSh / 4; ++q) {
      const float4 x = __ldg(r4 + q);
      c[4 * q] = x.x;
      c[4 * q + 1] = x.y;
      c[4 * q + 2] = x.z;
      c[4 * q + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < kSh; ++i) c[i] = i < sh_k ? row[i] : 0.0f;
  }
  float scattering = mul_(c[0], v.h.sh_basis[0]);
#pragma unroll
  for (int i = 1; i < kSh; i++) scattering = fma_(c[i], v.h.sh_basis[i], scattering);
  const float LEAKY_ALPHA = 0.1f;
  return scattering > 0.0f ? scattering : mul_(LEAKY_ALPHA, scattering);
}

constexpr float kTwoPi = 2.0f * kPi;

// The per-Gaussian constants of compute_gaussian_density_2d (:223-226, :231).
__device__ __forceinline__ void rec_density_consts(Rec& g) {
  const float det = fma_(g.cxx, g.cyy, -mul_(g.cxy, g.cxy));
  if (fabsf(det) < kEps) {
    g.inv_det = 0.0f;
    g.norm = -1.0f;
  } else {
    g.inv_det = div_(1.0f, det);
    g.norm = mul_(kTwoPi, sqrt_(det));
  }
}

// compute_gaussian_density_2d (:215-234) at pixel (px, py) = (pix_c, pix_r).
__device__ __forceinline__ float rec_density(const Rec& g, float px, float py) {
  if (g.norm < 0.0f) return 0.0f;
  const float dx = sub_(px, g.mx);
  const float dy = sub_(py, g.my);
  const float q = fma_(mul_(g.cxx, dy), dy,
                       fma_(mul_(g.cyy, dx), dx, -mul_(mul_(mul_(2.0f, g.cxy), dx), dy)));
  const float exponent = mul_(mul_(-0.5f, q), g.inv_det);
  if (exponent < -20.0f) return 0.0f;
  const float result = div_(expf(exponent), g.norm);
  return fmaxf(result, 0.0f);
}

// ---------------------------------------------------------------------------
// TMA bulk copy (cp.async.bulk, no multicast) and mbarrier helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Global -> shared bulk copy; dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for phase `parity` of the barrier for at most ~2 s of SM clock. On
// expiry it records kDevErrTmaTimeout, waits once more (bounded) so that no
// copy into this CTA's shared memory is left in flight when the caller
// returns, and reports failure.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
  const long long limit = 4000000000LL;
  long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) {
      if (err) atomicOr(err, kDevErrTmaTimeout);
      t0 = clock64();
      while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > limit) break;
      }
      return false;
    }
  }
  return true;
}

// Inclusive prefix sum over the lanes of a full warp.
__device__ __forceinline__ int warp_incl_scan(int x, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  return x;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Warp sums of eight values at once (reduce-scatter butterfly, 9 shuffles
// instead of 40): every lane returns the total of value
// k = 4 * bit4 + 2 * bit3 + bit2 of its lane index. The order of the
// additions is fixed, so the sums are reproducible.
__device__ __forceinline__ float warp_sum8_scatter(const float v[8], int lane) {
  const unsigned full = 0xffffffffu;
  const bool h16 = (lane & 16) != 0, h8 = (lane & 8) != 0, h4 = (lane & 4) != 0;
  float a[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    a[i] = (h16 ? v[4 + i] : v[i]) + __shfl_xor_sync(full, h16 ? v[i] : v[4 + i], 16);
  float b[2];
#pragma unroll
  for (int i = 0; i < 2; ++i)
    b[i] = (h8 ? a[2 + i] : a[i]) + __shfl_xor_sync(full, h8 ? a[i] : a[2 + i], 8);
  float c = (h4 ? b[1] : b[0]) + __shfl_xor_sync(full, h4 ? b[0] : b[1], 4);
  c += __shfl_xor_sync(full, c, 2);
  c += __shfl_xor_sync(full, c, 1);
  return c;
}

}  // namespace sarr
