// C ABI of the B200 SAR rasterizer (declared in include/sarr.h).
//
// Host responsibilities: argument validation, the per-view host math that the
// reference evaluates on the CPU (CUDASARRenderer::render,
// cuda_rasterizer/rasterizer_impl_v2.cu:1100-1120, and compute_sh_basis_host
// :284-320, in float with the C library's sinf/cosf/asinf/tanf so that the
// values are the reference's bits), carving of the caller's workspace and the
// kernel launch sequence on the caller's stream. No device allocation, no
// synchronisation, no host<->device copies on the hot path.
#include <stdint.h>
#include <string.h>

#include <atomic>
#include <cmath>
#include <map>
#include <mutex>
#include <vector>

#include "sarr.h"
#include "sarr_internal.h"

using namespace sarr;

namespace {

std::atomic<int64_t> g_launches{0};

}  // namespace

namespace sarr {
// Launches of the training-step kernels (sarr_train.cu, sarr_densify.cu),
// which are launched without the per-kind profiling hooks.
void count_launches(int k) { g_launches += k; }
}  // namespace sarr

namespace {

// compute_sh_basis_host (rasterizer_impl_v2.cu:284-320): the reference's own
// 16-term basis (terms 9-15 are not the standard real SH); constants :15-24.
void sh_basis_host(float theta, float phi, float* b) {
  const float C0 = 0.28209479177387814f, C1 = 0.4886025119029199f, C2 = 1.0925484305920792f;
  const float C20 = 0.31539156525252005f, C22 = 0.5462742152960396f, C3 = 0.5900435899266435f;
  const float C30 = 0.4570459564643759f;
  const float ct = cosf(theta), st = sinf(theta), cp = cosf(phi), sp = sinf(phi);
  const float ct2 = ct * ct;
  const float s_ct = st * ct;  // sin(theta) cos(theta)
  const float s_cp = st * cp;  // sin(theta) cos(phi)
  b[0] = C0;
  b[1] = C1 * st * sp;
  b[2] = C1 * st * cp;
  b[3] = C1 * ct;
  b[4] = C2 * s_cp * sp;
  b[5] = C2 * s_ct * cp;
  b[6] = C20 * (3.0f * ct2 - 1.0f);
  b[7] = -C2 * s_ct * sp;
  b[8] = -C2 * s_ct * cp;
  const float p3 = 3.0f * ct2 - 1.0f;
  const float p5 = (5.0f * ct2 - 3.0f) * ct;
  b[9] = C22 * st * sp * p3;
  b[10] = C22 * s_cp * p3;
  b[11] = C22 * ct * p3;
  b[12] = C3 * st * sp * p5;
  b[13] = C3 * s_cp * p5;
  const float p15 = (15.0f * ct2 - 6.0f) * ct2 - 1.0f;
  b[14] = C30 * p15;
  b[15] = -C3 * st * sp * p5;
}

// Host view setup of CUDASARRenderer::render (:1100-1120).
void view_host(const sarr_view& in, ViewHost& out) {
  const float track_rad = in.track_angle * 0.017453292519943295f;
  const float incidence_rad = in.incidence_angle * 0.017453292519943295f;
  const float azimuth_rad = in.azimuth_angle * 0.017453292519943295f;
  float sin_beta = sinf(incidence_rad) * cosf(azimuth_rad);
  sin_beta = fmaxf(fminf(sin_beta, 1.0f), -1.0f);
  const float beta_rad = asinf(sin_beta);
  const float tan_beta = tanf(beta_rad);
  const float altitude = in.radar_z;
  out.radar_x = altitude * tan_beta * sinf(track_rad);
  out.radar_y = -altitude * tan_beta * cosf(track_rad);
  out.radar_z = altitude;
  out.Rc = altitude / cosf(beta_rad);
  out.alpha = track_rad;
  out.beta = beta_rad;
  out.rho_r = in.range_resolution;
  out.rho_a = in.azimuth_resolution;
  out.Nr = in.range_samples;
  out.Na = in.azimuth_samples;
  const float theta = beta_rad;
  float phi = track_rad;
  if (phi < 0.0f) phi += 2.0f * kPi;
  sh_basis_host(theta, phi, out.sh_basis);
}

inline bool aligned(const void* p, uintptr_t a) { return ((uintptr_t)p & (a - 1)) == 0; }

int make_dims(const sarr_view* views, int n_views, int64_t n, Dims& d) {
  if (!views || n_views < 1 || n < 0 || n > (int64_t)INT32_MAX) return SARR_ERR_ARG;
  const int Nr = views[0].range_samples, Na = views[0].azimuth_samples;
  if (Nr < 0 || Na < 0) return SARR_ERR_ARG;
  for (int v = 1; v < n_views; ++v)
    if (views[v].range_samples != Nr || views[v].azimuth_samples != Na) return SARR_ERR_ARG;
  d.n = n;
  d.Nr = Nr;
  d.Na = Na;
  d.tiles_x = (Na + kTile - 1) / kTile;
  d.tiles_y = (Nr + kTile - 1) / kTile;
  if (d.tiles_x > kMaxTilesAxis || d.tiles_y > kMaxTilesAxis) return SARR_ERR_UNSUPPORTED;
  d.T = d.tiles_x * d.tiles_y;
  d.C = (int)((n + kChunk - 1) / kChunk);
  return SARR_OK;
}

int check_inputs(int64_t n, const float* means, const float* cov, int cov_layout, const float* sigma,
                 const float* sh, int sh_stride, int sh_k) {
  if (cov_layout != SARR_COV6 && cov_layout != SARR_COV33) return SARR_ERR_ARG;
  if (sh_k < 1 || sh_k > kSh || sh_stride < sh_k) return SARR_ERR_ARG;
  if (n > 0 && (!means || !cov || !sigma || !sh)) return SARR_ERR_ARG;
  if (!aligned(means, 4) || !aligned(cov, 4) || !aligned(sigma, 4) || !aligned(sh, 4)) return SARR_ERR_ARG;
  return SARR_OK;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? SARR_OK : SARR_ERR_CUDA; }

// ---------------------------------------------------------------------------
// launch accounting and optional per-kernel event timing
// ---------------------------------------------------------------------------
enum KernelKind {
  kKindSetup = 0, kKindBin, kKindSelect, kKindSelectShadow, kKindRender, kKindOmegaTile,
  kKindOmegaScatter, kKindBwdTile, kKindBwdScatter, kKindAux, kKindScan, kKindBinSkip,
  kKindBinFinalize, kKindSelectRender, kKindBinCand, kKindCount
};
static_assert(kKindCount == SARR_KERNEL_KINDS, "kernel kinds");

const char* const kKindNames[kKindCount] = {
    "view_setup", "bin_kernel", "select_kernel", "select_kernel_shadow", "render_kernel",
    "omega_tile_kernel", "omega_scatter_kernel", "bwd_tile_kernel", "bwd_scatter_kernel", "aux",
    "scan_kernel", "bin_skip_kernel", "bin_finalize_kernel", "select_render_kernel",
    "bin_cand_kernel"};

struct ProfRecord {
  int kind, device;
  cudaEvent_t start, stop;
};

std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfRecord> g_prof_records;
std::map<int, std::vector<cudaEvent_t>> g_prof_pool;  // free events per device

cudaEvent_t prof_event(int device) {
  auto& pool = g_prof_pool[device];
  if (!pool.empty()) {
    cudaEvent_t e = pool.back();
    pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

// Launches one kernel through `f`, counting it and, while profiling is on,
// bracketing it with events on the launching stream.
template <class F>
cudaError_t run_kernel(int kind, cudaStream_t s, F&& f) {
  ProfRecord rec{kind, 0, nullptr, nullptr};
  bool timed = false;
  {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (g_prof_on && cudaGetDevice(&rec.device) == cudaSuccess) {
      rec.start = prof_event(rec.device);
      rec.stop = prof_event(rec.device);
      timed = rec.start && rec.stop;
    }
  }
  if (timed) cudaEventRecord(rec.start, s);
  const cudaError_t e = f();
  g_launches++;
  if (timed) {
    cudaEventRecord(rec.stop, s);
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof_records.push_back(rec);
  }
  return e;
}

__global__ void fill_kernel(float* p, int64_t count, float value) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count) p[i] = value;
}

__global__ void clear_err_kernel(int* err) { *err = 0; }

cudaError_t fill(float* p, int64_t count, float value, cudaStream_t s) {
  if (count <= 0) return cudaSuccess;
  return run_kernel(kKindAux, s, [&] {
    fill_kernel<<<(unsigned)((count + 255) / 256), 256, 0, s>>>(p, count, value);
    return cudaGetLastError();
  });
}

struct Ws {
  WsLayout L;
  unsigned char* base;
  ViewConst* views;
  int* err;
  int group;
  unsigned char* view_area() const { return base + L.head; }
};

// Cell culling is used when the call qualifies (cells_eligible), the tile
// grid suits the cell binner, and the workspace holds the cell layout for at
// least one view; otherwise the call bins without cells.
static bool use_cells(const Dims& d, int n_views) {
  return cells_eligible(d, n_views) && bin_cell_supported(d);
}

int carve_ws(const Dims& d, void* ws, size_t ws_bytes, int n_views, Ws& w) {
  if (!ws || !aligned(ws, 256)) return SARR_ERR_WORKSPACE;
  w.L = ws_layout(d, use_cells(d, n_views));
  if (w.L.cells && ws_bytes < w.L.head + w.L.per_view) w.L = ws_layout(d, false);
  if (ws_bytes < w.L.head + w.L.per_view) return SARR_ERR_WORKSPACE;
  size_t fit = (ws_bytes - w.L.head) / w.L.per_view;
  int g = n_views < kMaxViewsPerLaunch ? n_views : kMaxViewsPerLaunch;
  if ((size_t)g > fit) g = (int)fit;
  w.group = g;
  w.base = static_cast<unsigned char*>(ws);
  w.views = reinterpret_cast<ViewConst*>(w.base + w.L.viewconst);
  w.err = reinterpret_cast<int*>(w.base + w.L.err);
  return SARR_OK;
}

// view constants of views [g0, g0+gv) into the workspace
cudaError_t setup_views(const sarr_view* views, int g0, int gv, const Ws& w, bool clear_err,
                        cudaStream_t s) {
  ViewHostPack pack;
  memset(&pack, 0, sizeof(pack));
  pack.n = gv;
  for (int v = 0; v < gv; ++v) view_host(views[g0 + v], pack.v[v]);
  return run_kernel(kKindSetup, s, [&] {
    return launch_view_setup(pack, w.views, clear_err ? w.err : nullptr, s);
  });
}

// The view-independent cell grid of a call (cell culling), before its groups.
cudaError_t run_cell_prep(const Dims& d, const Ws& w, const float* means, const float* cov,
                          int cov_layout, const float* sigma, cudaStream_t s) {
  if (!w.L.cells) return cudaSuccess;
  CellPrepArgs cp;
  cp.n = d.n;
  cp.means = means;
  cp.cov = cov;
  cp.cov_layout = cov_layout;
  cp.sigma = sigma;
  cp.grid = reinterpret_cast<SceneGrid*>(w.base + w.L.scene);
  cp.hb = reinterpret_cast<float*>(w.base + w.L.hb);
  cp.cid = reinterpret_cast<uint32_t*>(w.base + w.L.cid);
  cp.cell_hb = reinterpret_cast<int*>(w.base + w.L.cell_hb);
  cp.pstart = (int64_t)kPrefixChunks * kChunk;
  cp.cell_count = reinterpret_cast<int*>(w.base + w.L.cell_count);
  cp.cell_start = reinterpret_cast<int*>(w.base + w.L.cell_start);
  cp.cell_center = reinterpret_cast<float4*>(w.base + w.L.cell_center);
  cp.mem_pos = reinterpret_cast<float4*>(w.base + w.L.mem_pos);
  cp.mem_idx = reinterpret_cast<int*>(w.base + w.L.mem_idx);
  cp.always = reinterpret_cast<int*>(w.base + w.L.always);
  return run_kernel(kKindAux, s, [&] { return launch_cell_prep(cp, s); });
}

// bin + select of the image-plane list (and optionally the shadow list) for a
// group of views. With `fuse` given (an image-only call) and a selection that
// select_render_kernel can take, the image list's selection is not launched:
// its arguments are left in *fuse for that kernel (fuse->views is set only
// then).
cudaError_t run_selection(const Dims& d, const Ws& w, int gv, const float* means, const float* cov,
                          int cov_layout, const float* sigma, const float* sh, int sh_stride,
                          int sh_k, const StateRef& ipp, const StateRef* shr, cudaStream_t s,
                          SelectArgs* fuse = nullptr) {
  BinArgs ba;
  memset(&ba, 0, sizeof(ba));
  ba.views = w.views;
  ba.n = d.n;
  ba.C = d.C;
  ba.means = means;
  ba.cov = cov;
  ba.cov_layout = cov_layout;
  ba.sigma = sigma;
  ba.ipp = ipp;
  if (shr) ba.sh = *shr;
  ba.counts_ipp = w.view_area() + w.L.counts_ipp;
  ba.counts_sh = w.view_area() + w.L.counts_sh;
  ba.counts_vstride = w.L.per_view;
  ba.use_tma = aligned(means, 16) && aligned(cov, 16) && aligned(sigma, 16);
  ba.err = w.err;
  ba.nviews = gv;
  const bool masks = segmask_supported(d);
  ba.segmask = masks ? reinterpret_cast<uint32_t*>(w.view_area() + w.L.segmask_ipp) : nullptr;
  ba.segmask_sh = masks ? reinterpret_cast<uint32_t*>(w.view_area() + w.L.segmask_sh) : nullptr;
  ba.segmask_vstride = w.L.per_view / sizeof(uint32_t);
  // the per-view skipping binner also writes the masks of its chunks when
  // every chunk has room for them (few views: select_kernel then batches the
  // hit segments of all need entries); cell binning lists the exactly binned
  // Gaussians per chunk instead, which costs the many-view forward less
  const bool masks_all = masks && segmask_all_chunks(d) && !w.L.cells && skip_bin_per_warp(d, shr != nullptr);
  ba.skip_masks = masks_all ? 1 : 0;
  ba.xcount = reinterpret_cast<int*>(w.view_area() + w.L.xcount);
  ba.xlist = reinterpret_cast<uint16_t*>(w.view_area() + w.L.xlist);
  ba.x_vstride = w.L.per_view;
  ba.open_ipp = reinterpret_cast<const int*>(w.view_area() + w.L.open_ipp);
  ba.open_sh = reinterpret_cast<const int*>(w.view_area() + w.L.open_sh);
  ba.open_vstride = w.L.per_view / sizeof(int);
  // Enough CTAs to fill the GPU (~8 per SM on 148 SMs): a large launch gets
  // one CTA per chunk covering all views (the chunk is read once); a small
  // one splits the views across CTAs.
  auto views_per_cta = [gv](int chunks) {
    const int target = 148 * 8;
    int split = (target + chunks - 1) / chunks;
    if (split > gv) split = gv;
    if (split < 1) split = 1;
    return (gv + split - 1) / split;
  };
  // The first kPrefixChunks chunks are binned exactly; tiles that they fill
  // with 64 hits are marked saturated, and the remaining chunks skip the
  // covariance projection of Gaussians that can only reach saturated tiles.
  int prefix = d.C > kPrefixChunks ? kPrefixChunks : d.C;
  // One view on the per-view path (the training step): the skipping binner
  // runs one CTA per chunk after the prefix, so its last wave can be nearly
  // empty. The prefix is then widened, up to one CTA per SM of exact binning
  // (which costs about the same as 48), until the remaining chunks fill whole
  // waves. The lists do not depend on the prefix length.
  if (gv == 1 && !w.L.cells && masks_all && d.C > kPrefixChunks) {
    const int wave = skip_bin_wave(d, cov_layout, shr != nullptr, true);
    int sms = 0, dev = 0;
    if (wave > 0 && cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) {
      const int rest = d.C - kPrefixChunks;
      const int waves = (rest + wave - 1) / wave;
      const int p = d.C - (waves - 1) * wave;  // leaves exactly waves - 1 full waves
      if (waves > 1 && p <= sms) prefix = p;
    }
  }
  // Cell-culled calls bin the prefix in two stages: the first
  // kPrefixStage1 chunks exactly, then the rest of the prefix through the
  // skipping binner against the tiles still open after stage 1 (with
  // segment masks, as selection expects for prefix chunks); the lists do not
  // depend on the split.
  const int stage1 = (w.L.cells && masks && kPrefixStage1 > 0 && kPrefixStage1 < prefix &&
                      skip_bin_per_warp(d, shr != nullptr))
                         ? kPrefixStage1
                         : prefix;
  ba.chunk_offset = 0;
  ba.views_per_cta = views_per_cta(stage1);
  // one view per warp in the prefix binner once a CTA holds 8 views or more
  if (ba.views_per_cta >= 8) ba.views_per_cta = (ba.views_per_cta + 7) / 8 * 8;
  // the first stage of a two-stage prefix keeps the hit words of its chunks
  // (image list), which selection reads instead of re-testing rectangles
  const bool hit_words = stage1 < prefix && w.L.hbits != 0 && masks &&
                         prefix_hit_words(d);
  ba.hbits = hit_words ? reinterpret_cast<uint32_t*>(w.view_area() + w.L.hbits) : nullptr;
  ba.hbits_vstride = w.L.per_view / sizeof(uint32_t);
  ba.hbits_to = stage1;
  cudaError_t e = run_kernel(kKindBin, s, [&] {
    return launch_bin(ba, d, stage1, shr != nullptr, false, s);
  });
  if (e != cudaSuccess) return e;
  if (stage1 < prefix) {
    OpenArgs o1;
    o1.tiles_x = d.tiles_x;
    o1.tiles_y = d.tiles_y;
    o1.prefix_chunks = stage1;
    o1.counts[0] = ba.counts_ipp;
    o1.counts[1] = ba.counts_sh;
    o1.counts_vstride = w.L.per_view;
    o1.table[0] = const_cast<int*>(ba.open_ipp);
    o1.table[1] = const_cast<int*>(ba.open_sh);
    o1.table_vstride = ba.open_vstride;
    o1.cand_count = nullptr;
    e = run_kernel(kKindAux, s, [&] { return launch_open_table(o1, gv, shr ? 2 : 1, s); });
    if (e != cudaSuccess) return e;
    BinArgs b2 = ba;
    b2.hbits = nullptr;
    b2.chunk_offset = stage1;
    b2.views_per_cta = views_per_cta(prefix - stage1);
    // whole rounds of one view per warp (a CTA of 12 views left half of its
    // 8 warps idle in the second round)
#ifndef SARR_STAGE2_ROUND_VIEWS
#define SARR_STAGE2_ROUND_VIEWS 1
#endif
    if (SARR_STAGE2_ROUND_VIEWS && b2.views_per_cta > kBinThreads / 32)
      b2.views_per_cta = b2.views_per_cta / (kBinThreads / 32) * (kBinThreads / 32);
    b2.skip_masks = 1;
    b2.xlist = nullptr;  // prefix chunks are read through their segment masks
    b2.xcount = nullptr;
    e = run_kernel(kKindBinSkip, s, [&] {
      return launch_bin(b2, d, prefix - stage1, shr != nullptr, true, s);
    });
    if (e != cudaSuccess) return e;
  }
  if (prefix < d.C) {
    OpenArgs og;
    og.tiles_x = d.tiles_x;
    og.tiles_y = d.tiles_y;
    og.prefix_chunks = prefix;
    og.counts[0] = ba.counts_ipp;
    og.counts[1] = ba.counts_sh;
    og.counts_vstride = w.L.per_view;
    og.table[0] = const_cast<int*>(ba.open_ipp);
    og.table[1] = const_cast<int*>(ba.open_sh);
    og.table_vstride = ba.open_vstride;
    og.cand_count = w.L.cells ? reinterpret_cast<int*>(w.base + w.L.cand_count) : nullptr;
    e = run_kernel(kKindAux, s, [&] { return launch_open_table(og, gv, shr ? 2 : 1, s); });
    if (e != cudaSuccess) return e;
    ba.chunk_offset = prefix;
    if (w.L.cells) {
      CellTestArgs ct;
      ct.views = w.views;
      ct.grid = reinterpret_cast<const SceneGrid*>(w.base + w.L.scene);
      ct.cell_hb = reinterpret_cast<const int*>(w.base + w.L.cell_hb);
      ct.cell_center = reinterpret_cast<const float4*>(w.base + w.L.cell_center);
      ct.open_ipp = ba.open_ipp;
      ct.open_sh = ba.open_sh;
      ct.open_vstride = ba.open_vstride;
      ct.shadow = shr != nullptr;
      ct.bits = reinterpret_cast<uint32_t*>(w.view_area() + w.L.bits);
      ct.bits_vstride = w.L.per_view / sizeof(uint32_t);
      ct.cand_count = og.cand_count;
      ct.cand_words = reinterpret_cast<uint32_t*>(w.view_area() + w.L.cand_words);
      ct.cand_vstride = ct.bits_vstride;
      ct.ipp = ipp;
      ct.sparse_from = (int64_t)prefix * kChunk;
      ct.n = d.n;
      e = run_kernel(kKindAux, s, [&] { return launch_cell_test(ct, d, gv, s); });
      if (e != cudaSuccess) return e;
      ba.chunks = d.C - prefix;
      ba.grid = ct.grid;
      ba.cell_start = reinterpret_cast<const int*>(w.base + w.L.cell_start);
      ba.mem_pos = reinterpret_cast<const float4*>(w.base + w.L.mem_pos);
      ba.mem_idx = reinterpret_cast<const int*>(w.base + w.L.mem_idx);
      ba.always = reinterpret_cast<const int*>(w.base + w.L.always);
      ba.bits = ct.bits;
      ba.bits_vstride = ct.bits_vstride;
      ba.cand_count = ct.cand_count;
      ba.cand_words = ct.cand_words;
      ba.cand_vstride = ct.cand_vstride;

      e = run_kernel(kKindBinCand, s, [&] { return launch_bin_cand(ba, d, shr != nullptr, s); });
      if (e != cudaSuccess) return e;
      e = run_kernel(kKindBinFinalize, s, [&] { return launch_bin_finalize(ba, d, shr != nullptr, s); });
      if (e != cudaSuccess) return e;
    } else {
      ba.views_per_cta = views_per_cta(d.C - prefix);
      e = run_kernel(kKindBinSkip, s, [&] {
        return launch_bin(ba, d, d.C - prefix, shr != nullptr, true, s);
      });
      if (e != cudaSuccess) return e;
    }
  }

  ScanArgs sc;
  sc.T = d.T;
  sc.C = d.C;
  sc.counts = ba.counts_ipp;
  sc.counts_vstride = w.L.per_view;
  sc.st = ipp;
  sc.need = w.view_area() + w.L.need_ipp;
  sc.need_vstride = w.L.per_view;
  sc.need_n = reinterpret_cast<int*>(w.view_area() + w.L.need_n_ipp);
  sc.need_n_vstride = w.L.per_view / sizeof(int);
  e = run_kernel(kKindScan, s, [&] { return launch_scan(sc, gv, s); });
  if (e != cudaSuccess) return e;

  SelectArgs sa;
  memset(&sa, 0, sizeof(sa));
  sa.views = w.views;
  sa.n = d.n;
  sa.C = d.C;
  sa.means = means;
  sa.cov = cov;
  sa.cov_layout = cov_layout;
  sa.sigma = sigma;
  sa.sh = sh;
  sa.sh_stride = sh_stride;
  sa.sh_k = sh_k;
  sa.st = ipp;
  sa.need = sc.need;
  sa.need_vstride = sc.need_vstride;
  sa.need_n = sc.need_n;
  sa.need_n_vstride = sc.need_n_vstride;
  // the skipping binners record each chunk's exactly binned Gaussians, except
  // the CTA-wide variant for very large tile grids
  const bool xlists = prefix < d.C && (w.L.cells || skip_bin_per_warp(d, shr != nullptr));
  sa.xs = ipp;
  sa.segmask = ba.segmask;
  sa.segmask_vstride = ba.segmask_vstride;
  sa.segmask_to = masks_all ? d.C : prefix;
  sa.hbits = ba.hbits;
  sa.hbits_vstride = ba.hbits_vstride;
  sa.hbits_to = ba.hbits_to;
  sa.xlist_from = xlists ? prefix : INT32_MAX;
  sa.xcount = xlists ? ba.xcount : nullptr;
  sa.xlist = xlists ? ba.xlist : nullptr;
  sa.x_vstride = ba.x_vstride;
  sa.err = w.err;
  if (fuse && !shr && select_render_fusable(sa, gv)) {
    *fuse = sa;
    return cudaSuccess;
  }
  e = run_kernel(kKindSelect, s, [&] { return launch_select(sa, d, gv, false, s); });
  if (e != cudaSuccess || !shr) return e;

  sc.counts = ba.counts_sh;
  sc.st = *shr;
  sc.need = w.view_area() + w.L.need_sh;
  sc.need_n = reinterpret_cast<int*>(w.view_area() + w.L.need_n_sh);
  e = run_kernel(kKindScan, s, [&] { return launch_scan(sc, gv, s); });
  if (e != cudaSuccess) return e;
  sa.st = *shr;
  sa.segmask = ba.segmask_sh;
  sa.hbits = nullptr;  // hit words are kept for the image list only
  sa.need = sc.need;
  sa.need_n = sc.need_n;
  e = run_kernel(kKindSelectShadow, s, [&] { return launch_select(sa, d, gv, true, s); });
  return e;
}

// The backward's inverse index of a group's image-plane lists (workspace
// head and the views' entry slices).
BwdIndexArgs bwd_index_args(const Dims& d, const Ws& w, int gv, const StateRef& ipp) {
  BwdIndexArgs ia;
  ia.nviews = gv;
  ia.n = d.n;
  ia.T = d.T;
  ia.ipp = ipp;
  ia.cnt = reinterpret_cast<int*>(w.base + w.L.g_cnt);
  ia.start = reinterpret_cast<int*>(w.base + w.L.g_start);
  ia.bsum = reinterpret_cast<int*>(w.base + w.L.g_bsum);
  ia.entries = reinterpret_cast<uint32_t*>(w.view_area() + w.L.entries);
  ia.entries_vstride = w.L.per_view / sizeof(uint32_t);
  return ia;
}

}  // namespace

extern "C" {

const char* sarr_status_string(int status) {
  switch (status) {
    case SARR_OK: return "ok";
    case SARR_ERR_ARG: return "invalid argument";
    case SARR_ERR_WORKSPACE: return "workspace or state buffer too small or misaligned";
    case SARR_ERR_UNSUPPORTED: return "image larger than 2048 x 2048 pixels is not supported";
    case SARR_ERR_CUDA: return "CUDA launch or runtime error";
    case SARR_ERR_DEVICE: return "device-side error (bounded wait expired)";
    case SARR_ERR_CAPACITY:
      return "request exceeds the static scratch of sarr_forward_static (n <= 131072, image <= 256 x 256)";
    default: return "unknown status";
  }
}

const char* sarr_version(void) { return "sarr 0.1.0 (sm_100a)"; }

int sarr_workspace_size(int64_t n, int range_samples, int azimuth_samples, int n_views, int flags,
                        size_t* bytes) {
  (void)flags;
  if (!bytes || n_views < 1) return SARR_ERR_ARG;
  sarr_view v;
  memset(&v, 0, sizeof(v));
  v.range_samples = range_samples;
  v.azimuth_samples = azimuth_samples;
  Dims d;
  const int st = make_dims(&v, 1, n, d);
  if (st) return st;
  const WsLayout L = ws_layout(d, use_cells(d, n_views));
  const int g = n_views < kMaxViewsPerLaunch ? n_views : kMaxViewsPerLaunch;
  *bytes = L.head + L.per_view * (size_t)g;
  return SARR_OK;
}

int sarr_state_size(int64_t n, int range_samples, int azimuth_samples, size_t* bytes) {
  if (!bytes) return SARR_ERR_ARG;
  sarr_view v;
  memset(&v, 0, sizeof(v));
  v.range_samples = range_samples;
  v.azimuth_samples = azimuth_samples;
  Dims d;
  const int st = make_dims(&v, 1, n, d);
  if (st) return st;
  *bytes = state_layout(d.n, d.T).bytes;
  return SARR_OK;
}

int sarr_forward(const sarr_view* views, int n_views, int64_t n, const float* means, const float* cov,
                 int cov_layout, const float* sigma, const float* sh, int sh_stride, int sh_k,
                 float* images, float* omega, void* states, void* ws, size_t ws_bytes,
                 sarr_stream_t stream) {
  Dims d;
  int st = make_dims(views, n_views, n, d);
  if (st) return st;
  st = check_inputs(n, means, cov, cov_layout, sigma, sh, sh_stride, sh_k);
  if (st) return st;
  const size_t npix = (size_t)d.Nr * d.Na;
  if (npix > 0 && !images) return SARR_ERR_ARG;
  if (states && !aligned(states, 256)) return SARR_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  if (n == 0 || d.T == 0) {
    cudaError_t e = cudaSuccess;
    if (npix > 0) e = cudaMemsetAsync(images, 0, (size_t)n_views * npix * sizeof(float), s);
    if (e == cudaSuccess && omega) e = fill(omega, (int64_t)n_views * n, 1.0f, s);
    return cuda_status(e);
  }

  Ws w;
  st = carve_ws(d, ws, ws_bytes, n_views, w);
  if (st) return st;
  const size_t state_bytes = w.L.st.bytes;
  if (run_cell_prep(d, w, means, cov, cov_layout, sigma, s) != cudaSuccess) return SARR_ERR_CUDA;

  for (int g0 = 0; g0 < n_views; g0 += w.group) {
    const int gv = (n_views - g0) < w.group ? (n_views - g0) : w.group;
    cudaError_t e = setup_views(views, g0, gv, w, g0 == 0, s);
    if (e != cudaSuccess) return SARR_ERR_CUDA;
    StateRef ipp;
    if (states) {
      ipp.base = static_cast<unsigned char*>(states) + (size_t)g0 * state_bytes;
      ipp.vstride = state_bytes;
    } else {
      ipp.base = w.view_area() + w.L.state_ipp;
      ipp.vstride = w.L.per_view;
    }
    ipp.L = w.L.st;
    StateRef shr;
    shr.base = w.view_area() + w.L.state_sh;
    shr.vstride = w.L.per_view;
    shr.L = w.L.st;

    SelectArgs fused;
    fused.views = nullptr;
    e = run_selection(d, w, gv, means, cov, cov_layout, sigma, sh, sh_stride, sh_k, ipp,
                      omega ? &shr : nullptr, s, (!states && !omega) ? &fused : nullptr);
    if (e != cudaSuccess) return SARR_ERR_CUDA;

    TileArgs ta;
    memset(&ta, 0, sizeof(ta));
    ta.views = w.views;
    ta.st = ipp;
    ta.images = images + (size_t)g0 * npix;
    ta.img_vstride = npix;
    ta.err = w.err;
    if (fused.views)
      e = run_kernel(kKindSelectRender, s, [&] { return launch_select_render(fused, ta, d, gv, s); });
    else
      e = run_kernel(kKindRender, s, [&] { return launch_render(ta, d, gv, s); });
    if (e != cudaSuccess) return SARR_ERR_CUDA;

    if (omega) {
      TileArgs to;
      memset(&to, 0, sizeof(to));
      to.views = w.views;
      to.st = shr;
      to.partial = reinterpret_cast<float*>(w.view_area() + w.L.partial_om);
      to.partial_vstride = w.L.per_view / sizeof(float);
      to.err = w.err;
      e = run_kernel(kKindOmegaTile, s, [&] { return launch_omega_tile(to, d, gv, s); });
      if (e != cudaSuccess) return SARR_ERR_CUDA;
      OmegaScatterArgs os;
      os.views = w.views;
      os.n = d.n;
      os.sh = shr;
      os.ipp = ipp;
      os.partial = to.partial;
      os.partial_vstride = to.partial_vstride;
      os.omega = omega + (size_t)g0 * d.n;
      os.omega_vstride = (size_t)d.n;
      e = run_kernel(kKindOmegaScatter, s, [&] { return launch_omega_scatter(os, d, gv, s); });
      if (e != cudaSuccess) return SARR_ERR_CUDA;
    }
  }
  return SARR_OK;
}

int sarr_backward(const sarr_view* views, int n_views, int64_t n, const float* means, const float* cov,
                  int cov_layout, const float* sigma, const float* sh, int sh_stride, int sh_k,
                  const float* grad_images, const void* states, float* grad_means, float* grad_cov,
                  int grad_cov_layout, float* grad_sigma, float* grad_sh, int grad_sh_cols,
                  float* grad_norm, int flags, void* ws, size_t ws_bytes, sarr_stream_t stream) {
  Dims d;
  int st = make_dims(views, n_views, n, d);
  if (st) return st;
  st = check_inputs(n, means, cov, cov_layout, sigma, sh, sh_stride, sh_k);
  if (st) return st;
  if (grad_cov_layout != SARR_COV6 && grad_cov_layout != SARR_COV33) return SARR_ERR_ARG;
  if (grad_sh_cols < 1 || grad_sh_cols > kSh) return SARR_ERR_ARG;
  if (n > 0 && (!grad_means || !grad_cov || !grad_sigma || !grad_sh)) return SARR_ERR_ARG;
  const size_t npix = (size_t)d.Nr * d.Na;
  if (npix > 0 && !grad_images) return SARR_ERR_ARG;
  if (states && !aligned(states, 256)) return SARR_ERR_WORKSPACE;
  const bool acc = (flags & SARR_FLAG_ACCUMULATE) != 0;
  const bool tiles_only = (flags & SARR_FLAG_TILES_ONLY) != 0;
  if (tiles_only && n_views > kMaxViewsPerLaunch) return SARR_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (n == 0) return SARR_OK;
  if (d.T == 0) {
    if (acc || tiles_only) return SARR_OK;
    cudaError_t e = cudaMemsetAsync(grad_means, 0, (size_t)n * 3 * 4, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(grad_cov, 0, (size_t)n * grad_cov_layout * 4, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(grad_sigma, 0, (size_t)n * 4, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(grad_sh, 0, (size_t)n * grad_sh_cols * 4, s);
    if (e == cudaSuccess && grad_norm) e = cudaMemsetAsync(grad_norm, 0, (size_t)n * 4, s);
    return cuda_status(e);
  }

  Ws w;
  st = carve_ws(d, ws, ws_bytes, n_views, w);
  if (st) return st;
  if (tiles_only && w.group < n_views) return SARR_ERR_WORKSPACE;  // one launch group
  const size_t state_bytes = w.L.st.bytes;
  if (!states && run_cell_prep(d, w, means, cov, cov_layout, sigma, s) != cudaSuccess)
    return SARR_ERR_CUDA;

  for (int g0 = 0; g0 < n_views; g0 += w.group) {
    const int gv = (n_views - g0) < w.group ? (n_views - g0) : w.group;
    cudaError_t e = setup_views(views, g0, gv, w, g0 == 0, s);
    if (e != cudaSuccess) return SARR_ERR_CUDA;
    StateRef ipp;
    if (states) {
      ipp.base = const_cast<unsigned char*>(static_cast<const unsigned char*>(states)) + (size_t)g0 * state_bytes;
      ipp.vstride = state_bytes;
    } else {
      ipp.base = w.view_area() + w.L.state_ipp;
      ipp.vstride = w.L.per_view;
    }
    ipp.L = w.L.st;
    if (!states) {
      e = run_selection(d, w, gv, means, cov, cov_layout, sigma, sh, sh_stride, sh_k, ipp, nullptr, s);
      if (e != cudaSuccess) return SARR_ERR_CUDA;
    }
    TileArgs tb;
    memset(&tb, 0, sizeof(tb));
    tb.views = w.views;
    tb.st = ipp;
    tb.images = const_cast<float*>(grad_images) + (size_t)g0 * npix;
    tb.img_vstride = npix;
    tb.partial = reinterpret_cast<float*>(w.view_area() + w.L.partial_bwd);
    tb.partial_vstride = w.L.per_view / sizeof(float);
    tb.err = w.err;
    e = run_kernel(kKindBwdTile, s, [&] { return launch_bwd_tile(tb, d, gv, s); });
    if (e != cudaSuccess) return SARR_ERR_CUDA;
    BwdIndexArgs ia = bwd_index_args(d, w, gv, ipp);
    e = run_kernel(kKindAux, s, [&] { return launch_bwd_index(ia, s); });
    if (e != cudaSuccess) return SARR_ERR_CUDA;
    if (tiles_only) break;  // sarr_backward_scatter writes the rows

    BwdScatterArgs bs;
    bs.views = w.views;
    bs.nviews = gv;
    bs.n = d.n;
    bs.ipp = ipp;
    bs.partial = tb.partial;
    bs.partial_vstride = tb.partial_vstride;
    bs.grad_means = grad_means;
    bs.grad_cov = grad_cov;
    bs.grad_cov_layout = grad_cov_layout;
    bs.grad_sigma = grad_sigma;
    bs.grad_sh = grad_sh;
    bs.grad_sh_cols = grad_sh_cols;
    bs.grad_norm = grad_norm;
    bs.accumulate = (acc || g0 > 0) ? 1 : 0;
    bs.start = ia.start;
    bs.entries = ia.entries;
    bs.entries_vstride = ia.entries_vstride;
    bs.heavy = reinterpret_cast<int*>(w.base + w.L.g_heavy);
    bs.row0 = 0;
    bs.begin = 0;
    bs.end = d.n;
    e = run_kernel(kKindBwdScatter, s, [&] { return launch_bwd_scatter(bs, d, s); });
    if (e != cudaSuccess) return SARR_ERR_CUDA;
  }
  return SARR_OK;
}

int sarr_backward_scatter(const sarr_view* views, int n_views, int64_t n, const void* states,
                          int64_t begin, int64_t end, float* grad_means, float* grad_cov,
                          int grad_cov_layout, float* grad_sigma, float* grad_sh, int grad_sh_cols,
                          float* grad_norm, int flags, void* ws, size_t ws_bytes,
                          sarr_stream_t stream) {
  Dims d;
  int st = make_dims(views, n_views, n, d);
  if (st) return st;
  if (n_views > kMaxViewsPerLaunch) return SARR_ERR_ARG;
  if (begin < 0 || end < begin || end > n) return SARR_ERR_ARG;
  if (grad_cov_layout != SARR_COV6 && grad_cov_layout != SARR_COV33) return SARR_ERR_ARG;
  if (grad_sh_cols < 1 || grad_sh_cols > kSh) return SARR_ERR_ARG;
  if (end > begin && (!grad_means || !grad_cov || !grad_sigma || !grad_sh)) return SARR_ERR_ARG;
  if (states && !aligned(states, 256)) return SARR_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (end == begin) return SARR_OK;
  const bool acc = (flags & SARR_FLAG_ACCUMULATE) != 0;
  if (d.T == 0) {
    if (acc) return SARR_OK;
    const int64_t m = end - begin;
    const int64_t r0 = (flags & SARR_FLAG_RANGE_ROWS) ? 0 : begin;  // first row written
    cudaError_t e = cudaMemsetAsync(grad_means + 3 * r0, 0, (size_t)m * 3 * 4, s);
    if (e == cudaSuccess)
      e = cudaMemsetAsync(grad_cov + grad_cov_layout * r0, 0, (size_t)m * grad_cov_layout * 4, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(grad_sigma + r0, 0, (size_t)m * 4, s);
    if (e == cudaSuccess)
      e = cudaMemsetAsync(grad_sh + (size_t)grad_sh_cols * r0, 0, (size_t)m * grad_sh_cols * 4, s);
    if (e == cudaSuccess && grad_norm) e = cudaMemsetAsync(grad_norm + r0, 0, (size_t)m * 4, s);
    return cuda_status(e);
  }
  Ws w;
  st = carve_ws(d, ws, ws_bytes, n_views, w);
  if (st) return st;
  if (w.group < n_views) return SARR_ERR_WORKSPACE;
  StateRef ipp;
  if (states) {
    ipp.base = const_cast<unsigned char*>(static_cast<const unsigned char*>(states));
    ipp.vstride = w.L.st.bytes;
  } else {
    ipp.base = w.view_area() + w.L.state_ipp;
    ipp.vstride = w.L.per_view;
  }
  ipp.L = w.L.st;
  BwdScatterArgs bs;
  bs.views = w.views;
  bs.nviews = n_views;
  bs.n = d.n;
  bs.ipp = ipp;
  bs.partial = reinterpret_cast<float*>(w.view_area() + w.L.partial_bwd);
  bs.partial_vstride = w.L.per_view / sizeof(float);
  bs.grad_means = grad_means;
  bs.grad_cov = grad_cov;
  bs.grad_cov_layout = grad_cov_layout;
  bs.grad_sigma = grad_sigma;
  bs.grad_sh = grad_sh;
  bs.grad_sh_cols = grad_sh_cols;
  bs.grad_norm = grad_norm;
  bs.accumulate = acc ? 1 : 0;
  const BwdIndexArgs ia = bwd_index_args(d, w, n_views, ipp);
  bs.start = ia.start;
  bs.entries = ia.entries;
  bs.entries_vstride = ia.entries_vstride;
  bs.heavy = reinterpret_cast<int*>(w.base + w.L.g_heavy);
  bs.row0 = (flags & SARR_FLAG_RANGE_ROWS) ? begin : 0;
  bs.begin = begin;
  bs.end = end;
  return cuda_status(run_kernel(kKindBwdScatter, s, [&] { return launch_bwd_scatter(bs, d, s); }));
}

int sarr_debug_preprocess(const sarr_view* view, int64_t n, const float* means, const float* cov,
                          int cov_layout, const float* sigma, const float* sh, int sh_stride,
                          int sh_k, float* f32_out, int32_t* i32_out, sarr_stream_t stream) {
  Dims d;
  int st = make_dims(view, 1, n, d);
  if (st) return st;
  st = check_inputs(n, means, cov, cov_layout, sigma, sh, sh_stride, sh_k);
  if (st) return st;
  if (n > 0 && (!f32_out || !i32_out)) return SARR_ERR_ARG;
  if (n == 0) return SARR_OK;
  DebugPreArgs a;
  view_host(*view, a.vh);
  a.n = n;
  a.means = means;
  a.cov = cov;
  a.cov_layout = cov_layout;
  a.sigma = sigma;
  a.sh = sh;
  a.sh_stride = sh_stride;
  a.sh_k = sh_k;
  a.f32 = f32_out;
  a.i32 = i32_out;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return cuda_status(run_kernel(kKindAux, s, [&] { return launch_debug_preprocess(a, s); }));
}

int sarr_debug_tile_lists(const sarr_view* view, int64_t n, const float* means, const float* cov,
                          int cov_layout, const float* sigma, int32_t* counts, int32_t* lists,
                          int32_t* sorted, int32_t* shadow_counts, int32_t* shadow_lists,
                          int32_t* shadow_sorted, void* ws, size_t ws_bytes, sarr_stream_t stream) {
  Dims d;
  int st = make_dims(view, 1, n, d);
  if (st) return st;
  // SH does not influence the lists; any valid pointer will do.
  st = check_inputs(n, means, cov, cov_layout, sigma, means, 1, 1);
  if (st) return st;
  if (!counts || !lists || !sorted) return SARR_ERR_ARG;
  const bool want_sh = shadow_counts && shadow_lists && shadow_sorted;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (d.T == 0) return SARR_OK;
  if (n == 0) {
    cudaError_t e = cudaMemsetAsync(counts, 0, (size_t)d.T * 4, s);
    if (e == cudaSuccess && want_sh) e = cudaMemsetAsync(shadow_counts, 0, (size_t)d.T * 4, s);
    return cuda_status(e);
  }
  Ws w;
  st = carve_ws(d, ws, ws_bytes, 1, w);
  if (st) return st;
  cudaError_t e = setup_views(view, 0, 1, w, true, s);
  if (e != cudaSuccess) return SARR_ERR_CUDA;
  StateRef ipp{w.view_area() + w.L.state_ipp, w.L.per_view, w.L.st};
  StateRef shr{w.view_area() + w.L.state_sh, w.L.per_view, w.L.st};
  e = run_selection(d, w, 1, means, cov, cov_layout, sigma, means, 1, 1, ipp, &shr, s);
  if (e != cudaSuccess) return SARR_ERR_CUDA;
  DebugListArgs la{d.T, ipp, counts, lists, sorted};
  e = run_kernel(kKindAux, s, [&] { return launch_debug_lists(la, s); });
  if (e == cudaSuccess && want_sh) {
    DebugListArgs lb{d.T, shr, shadow_counts, shadow_lists, shadow_sorted};
    e = run_kernel(kKindAux, s, [&] { return launch_debug_lists(lb, s); });
  }
  return cuda_status(e);
}

int sarr_debug_view_constants(const sarr_view* view, float* out, sarr_stream_t stream) {
  if (!view || !out) return SARR_ERR_ARG;
  ViewHost vh;
  view_host(*view, vh);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return cuda_status(run_kernel(kKindAux, s, [&] { return launch_debug_view(vh, out, s); }));
}

int sarr_debug_tile_rect(int r_min, int r_max, int c_min, int c_max, int range_samples,
                         int azimuth_samples, int32_t* tc0, int32_t* tc1, int32_t* tr0,
                         int32_t* tr1) {
  if (!tc0 || !tc1 || !tr0 || !tr1) return SARR_ERR_ARG;
  const uint32_t rc = make_rect(r_min, r_max, c_min, c_max, range_samples, azimuth_samples);
  *tc0 = rc & 0xFF;
  *tc1 = (rc >> 8) & 0xFF;
  *tr0 = (rc >> 16) & 0xFF;
  *tr1 = rc >> 24;
  return SARR_OK;
}

int sarr_check_device_errors(void* ws, size_t ws_bytes, sarr_stream_t stream) {
  if (!ws || ws_bytes < 256) return SARR_ERR_ARG;
  // The error word sits at a fixed offset, independent of the problem size.
  const size_t off = align256(sizeof(ViewConst) * kMaxViewsPerLaunch);
  if (ws_bytes < off + 4) return SARR_ERR_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int h = 0;
  int* err = reinterpret_cast<int*>(static_cast<unsigned char*>(ws) + off);
  cudaError_t e = cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return SARR_ERR_CUDA;
  if (h != 0) {
    run_kernel(kKindAux, s, [&] {
      clear_err_kernel<<<1, 1, 0, s>>>(err);
      return cudaGetLastError();
    });
    return SARR_ERR_DEVICE;
  }
  return SARR_OK;
}

int64_t sarr_launch_count(void) { return g_launches.load(); }

int sarr_profile_enable(int enable) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof_on = enable != 0;
  return SARR_OK;
}

int sarr_profile_read(double* total_ms, int64_t* launches, int n_kinds) {
  if (!total_ms || !launches || n_kinds < 1) return SARR_ERR_ARG;
  std::vector<ProfRecord> recs;
  {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    recs.swap(g_prof_records);
  }
  for (int k = 0; k < n_kinds; ++k) {
    total_ms[k] = 0.0;
    launches[k] = 0;
  }
  int status = SARR_OK;
  int dev0 = 0;
  cudaGetDevice(&dev0);
  for (const ProfRecord& r : recs) {
    cudaSetDevice(r.device);
    float ms = 0.0f;
    if (cudaEventSynchronize(r.stop) != cudaSuccess ||
        cudaEventElapsedTime(&ms, r.start, r.stop) != cudaSuccess)
      status = SARR_ERR_CUDA;
    if (r.kind < n_kinds) {
      total_ms[r.kind] += ms;
      launches[r.kind] += 1;
    }
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof_pool[r.device].push_back(r.start);
    g_prof_pool[r.device].push_back(r.stop);
  }
  cudaSetDevice(dev0);
  return status;
}

const char* sarr_kernel_name(int kind) {
  return (kind >= 0 && kind < kKindCount) ? kKindNames[kind] : "unknown";
}

}  // extern "C"
