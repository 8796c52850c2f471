// Kernels of the B200 SAR rasterizer.
//
// Forward pipeline per view (replaces preprocess_kernel, compute_ranges_kernel,
// build_tile_gaussian_list_kernel, build_shadow_tile_list_kernel,
// compute_omega_kernel, the host Omega average and render_kernel of
// cuda_rasterizer/rasterizer_impl_v2.cu:322-839, :1239-1252):
//
//   bin_kernel       the first kPrefixChunks chunks of 1024 Gaussians, exactly:
//                    TMA bulk copy of a chunk's means/cov/sigma into shared
//                    memory, projection, validity, pixel bbox -> tile rectangle
//                    (4 bytes per list), and a per-chunk per-tile hit count
//                    built with a 2-D difference array.
//   open_table_kernel  summed-area table of the tiles that the prefix left with
//                    fewer than 64 hits (still open).
//   bin_skip_kernel / bin_cell_kernel
//                    the remaining chunks: Gaussians that can only reach full
//                    tiles get an empty rectangle after a conservative test
//                    (bin_cell_kernel first rejects whole cells of a
//                    view-independent grid); the rest are binned exactly, one
//                    view per warp, and listed per chunk.
//   scan_kernel      per tile, the chunks holding its first 64 hits.
//   select_kernel    one warp per tile: the hits of those chunks in index
//                    order (warp ballots), the selected Gaussians projected
//                    again (SH only for them), ranked by (Z_r, index) and
//                    stored as 48-byte records.
//   render_kernel    one CTA per tile: TMA bulk copy of its sorted records,
//                    front-to-back compositing by 8 x 8 pixel warp blocks (two
//                    pixels per lane) that skip records whose density is 0 on
//                    the whole block.
//   omega_tile_kernel / omega_scatter_kernel
//                    per-pixel Omega walk with per-slot warp reductions, then
//                    a per-Gaussian gather of those partial sums.
//
// Backward (replaces backward_kernel :841-1020): bwd_tile_kernel replays each
// pixel front to back and reduces the 7 per-(pixel, Gaussian) terms over the
// tile with warp shuffles; bwd_scatter_kernel gathers them per Gaussian and
// writes the dense gradient rows, applying the per-Gaussian chain rule once.
// No float atomics: results are deterministic.
#include <algorithm>

#include "sarr_internal.h"

namespace sarr {

// ---------------------------------------------------------------------------
// view setup
// ---------------------------------------------------------------------------
// The pack is a __grid_constant__ parameter: indexed in place, not copied.
// kViews: capacity of the parameter block (the kernel parameters are copied
// per launch, so calls of a few views use a small block).
template <int kViews>
__global__ void view_setup_kernel(const __grid_constant__ ViewHostPackN<kViews> pack,
                                  ViewConst* __restrict__ out, int* err) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (err && v == 0) *err = 0;
  if (v >= pack.n) return;
  ViewConst c;
  c.h = pack.v[v];
  c.cos_a = cosf(c.h.alpha);
  c.sin_a = sinf(c.h.alpha);
  c.cos_b = cosf(c.h.beta);
  c.sin_b = sinf(c.h.beta);
  c.tiles_x = (c.h.Na + kTile - 1) / kTile;
  c.tiles_y = (c.h.Nr + kTile - 1) / kTile;
  view_derive(c);
  out[v] = c;
}

// ---------------------------------------------------------------------------
// binning
// ---------------------------------------------------------------------------
__device__ __forceinline__ void diff_add(int* d, int pitch, uint32_t rc) {
  const int tc0 = rc & 0xFF, tc1 = (rc >> 8) & 0xFF, tr0 = (rc >> 16) & 0xFF, tr1 = rc >> 24;
  if (tc0 > tc1) return;
  atomicAdd(&d[tr0 * pitch + tc0], 1);
  atomicAdd(&d[tr0 * pitch + tc1 + 1], -1);
  atomicAdd(&d[(tr1 + 1) * pitch + tc0], -1);
  atomicAdd(&d[(tr1 + 1) * pitch + tc1 + 1], 1);
}

// Number of open tiles inside a tile rectangle, from the summed-area table
// tab[(tiles_y+1)][pitch] (entry [y][x] counts the open tiles above and left
// of (y, x)). An empty rectangle holds none.
__device__ __forceinline__ int open_in_rect(uint32_t rc, const int* __restrict__ tab, int pitch) {
  if (rc == kEmptyRect) return 0;
  const int tc0 = rc & 0xFF, tc1 = ((rc >> 8) & 0xFF) + 1, tr0 = (rc >> 16) & 0xFF, tr1 = (rc >> 24) + 1;
  return __ldg(tab + tr1 * pitch + tc1) - __ldg(tab + tr0 * pitch + tc1) -
         __ldg(tab + tr1 * pitch + tc0) + __ldg(tab + tr0 * pitch + tc0);
}

// open_in_rect on a table staged in shared memory.
__device__ __forceinline__ int open_in_rect_s(uint32_t rc, const int* tab, int pitch) {
  if (rc == kEmptyRect) return 0;
  const int tc0 = rc & 0xFF, tc1 = ((rc >> 8) & 0xFF) + 1, tr0 = (rc >> 16) & 0xFF, tr1 = (rc >> 24) + 1;
  return tab[tr1 * pitch + tc1] - tab[tr0 * pitch + tc1] - tab[tr1 * pitch + tc0] + tab[tr0 * pitch + tc0];
}

// The view's open-tile tables (image list, then shadow list when `lists` is
// 2) copied into shared memory by the whole CTA; ends with a barrier.
__device__ __forceinline__ void stage_open_tables(int* s_tab, const int* open_ipp, const int* open_sh,
                                                  int size, int lists) {
  for (int e = threadIdx.x; e < size; e += blockDim.x) {
    s_tab[e] = open_ipp[e];
    if (lists > 1) s_tab[size + e] = open_sh[e];
  }
  __syncthreads();
}

// Shared memory for the staged open tables of one view (0: read them from
// global memory instead).
constexpr size_t kOpenStageMaxBytes = 16384;
static size_t open_stage_bytes(int tiles_x, int tiles_y, int lists) {
  const size_t b = (size_t)(tiles_x + 1) * (tiles_y + 1) * 4 * lists;
  return b <= kOpenStageMaxBytes ? b : 0;
}

// ORs `bit` into the mask of every tile of a rectangle.
__device__ __forceinline__ void mark_rect(uint32_t* mask, uint32_t rc, int tiles_x, uint32_t bit) {
  if (rc == kEmptyRect) return;
  const int tc0 = rc & 0xFF, tc1 = (rc >> 8) & 0xFF, tr0 = (rc >> 16) & 0xFF, tr1 = rc >> 24;
  for (int ty = tr0; ty <= tr1; ++ty)
    for (int tx = tc0; tx <= tc1; ++tx) atomicOr(mask + ty * tiles_x + tx, bit);
}

// Writes the round's nonzero hit words of a rectangle's tiles (out[t * 32])
// and clears them. Lanes whose rectangles share a tile may both write its
// word: all ORs of the round are done (the caller synchronises the warp
// before), so every writer writes the same word, and a lane that finds it
// cleared by another has nothing left to write.
__device__ __forceinline__ void flush_hit_words(uint32_t* hw, uint32_t rc, int tiles_x, uint32_t* out) {
  if (rc == kEmptyRect) return;
  const int tc0 = rc & 0xFF, tc1 = (rc >> 8) & 0xFF, tr0 = (rc >> 16) & 0xFF, tr1 = rc >> 24;
  for (int tr = tr0; tr <= tr1; ++tr)
    for (int tc = tc0; tc <= tc1; ++tc) {
      const int t = tr * tiles_x + tc;
      const uint32_t w = hw[t];
      if (w) {
        out[(size_t)t * 32] = w;
        hw[t] = 0;
      }
    }
}

// Tile rectangle of the pixel box centred on (cr, cc) with half-width h,
// clamped like the reference's bboxes.
__device__ __forceinline__ uint32_t bound_rect(float cr, float cc, float h, int Nr, int Na) {
  const int r0 = max(0, (int)floorf(cr - h)), r1 = min(Nr - 1, (int)ceilf(cr + h));
  const int c0 = max(0, (int)floorf(cc - h)), c1 = min(Na - 1, (int)ceilf(cc + h));
  return make_rect(r0, r1, c0, c1, Nr, Na);
}

// Exact per-Gaussian binning of one Gaussian for one view (preprocess_kernel
// + compute_ranges_kernel + the shadow footprint, :322-470, :572-597).
template <bool kShadow>
__device__ __forceinline__ void bin_exact(const ViewConst& vc, const float* s_means, const float* s_cov,
                                          int cs, int j, uint32_t& rc_ipp, uint32_t& rc_sh) {
  const int Nr = vc.h.Nr, Na = vc.h.Na;
  Proj o;
  const float Rmin = project_center(vc, s_means[3 * j], s_means[3 * j + 1], s_means[3 * j + 2], o);
  if (!proj_valid(o, Nr, Na)) return;
  float cw[6], X6[6];
  load_cov6(s_cov + j * cs, cs, cw);
  radar_cov(vc, cw, X6);
  image_cov(vc, X6, Rmin, o);
  int r0, r1, c0, c1;
  ipp_ranges(o, Nr, Na, r0, r1, c0, c1);
  rc_ipp = make_rect(r0, r1, c0, c1, Nr, Na);
  if (kShadow) {
    if (shadow_ranges(o, Nr, Na, r0, r1, c0, c1)) rc_sh = make_rect(r0, r1, c0, c1, Nr, Na);
  }
}

// Stages chunk `base` (gcount Gaussians) of means, covariances (unless
// s_cov is null) and transmittances in shared memory: one TMA bulk copy per
// array when the chunk is full and the arrays are 16-byte aligned, plain
// loads otherwise. Every thread of the CTA calls it; false when the copy
// timed out (error recorded).
__device__ __forceinline__ bool stage_chunk(const BinArgs& a, int64_t base, int gcount, float* s_means,
                                            float* s_cov, float* s_sigma, uint64_t* bar) {
  const int tid = threadIdx.x, cs = a.cov_layout;
  const bool tma = a.use_tma && gcount == kChunk;
  if (tid == 0 && tma) mbar_init(bar, 1);
  __syncthreads();
  bool ok = true;
  if (tma) {
    if (tid == 0) {
      const uint32_t bm = 3u * kChunk * 4u, bc = s_cov ? (uint32_t)cs * kChunk * 4u : 0u, bs = kChunk * 4u;
      mbar_arrive_expect_tx(bar, bm + bc + bs);
      tma_load_1d(s_means, a.means + base * 3, bm, bar);
      if (s_cov) tma_load_1d(s_cov, a.cov + base * cs, bc, bar);
      tma_load_1d(s_sigma, a.sigma + base, bs, bar);
    }
    ok = mbar_wait_bounded(bar, 0, a.err);  // every reader observes the barrier phase
  } else {
    for (int i = tid; i < 3 * gcount; i += blockDim.x) s_means[i] = a.means[base * 3 + i];
    if (s_cov)
      for (int i = tid; i < cs * gcount; i += blockDim.x) s_cov[i] = a.cov[base * cs + i];
    for (int i = tid; i < gcount; i += blockDim.x) s_sigma[i] = a.sigma[base + i];
  }
  return __syncthreads_and(ok);
}

// One CTA per chunk of kChunk Gaussians, all views of the launch: the chunk is
// staged in shared memory once and projected for every view in turn.
//
// kSkip (chunks after the saturation prefix): a tile's list is complete once
// the prefix holds 64 of its hits, so a later Gaussian whose bbox can only
// reach such tiles enters no list and gets an empty rectangle. Stage 1 decides
// that for every Gaussian from a fast approximate centre and a view-independent
// bbox bound (both with margins); only the rest are queued, compacted, and
// binned exactly in stage 2, which keeps the warps of both stages coherent.
#ifndef SARR_BIN_MIN_CTAS
#define SARR_BIN_MIN_CTAS 4
#endif
template <bool kShadow, bool kSkip, int kThreads>
__global__ void __launch_bounds__(kThreads, kThreads == kBinThreads ? SARR_BIN_MIN_CTAS : 1)
    bin_kernel(const BinArgs a) {
  constexpr int kPer = kChunk / kThreads;  // Gaussians per thread
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ uint64_t bar;
  __shared__ int s_qn;
  __shared__ short s_queue[kChunk];

  const int tid = threadIdx.x, lane = tid & 31;
  const int chunk = blockIdx.x + a.chunk_offset;
  const int tiles_x = a.views[0].tiles_x, tiles_y = a.views[0].tiles_y, T = tiles_x * tiles_y;
  const int cs = a.cov_layout;

  float* s_means = reinterpret_cast<float*>(smem_raw);
  float* s_cov = s_means + 3 * kChunk;
  float* s_sigma = s_cov + cs * kChunk;
  int* s_diff_ipp = reinterpret_cast<int*>(s_sigma + kChunk);
  const int pitch = tiles_x + 1;
  const int T1 = (tiles_y + 1) * pitch;
  int* s_diff_sh = s_diff_ipp + T1;
  // segment masks (exact variant, when a.segmask is set): bit s of tile t is
  // set when Gaussians [32 s, 32 s + 32) of the chunk hold a hit of t
  const bool masks = !kSkip && a.segmask != nullptr;
  uint32_t* s_mask_ipp = reinterpret_cast<uint32_t*>(s_diff_ipp + T1 * (kShadow ? 2 : 1));
  uint32_t* s_mask_sh = s_mask_ipp + T;
  // hit words (BinArgs::hbits) of the image list: iteration k of warp w
  // bins segment w + k kThreads / 32 of the chunk, one Gaussian per lane, so
  // each warp ORs one segment's word per tile in its own array
  const bool hits = masks && a.hbits != nullptr && chunk < a.hbits_to;
  uint32_t* s_hw = s_mask_ipp + T * (kShadow ? 2 : 1) + (tid >> 5) * T;

  const int64_t base = (int64_t)chunk * kChunk;
  const int gcount = (int)min((int64_t)kChunk, a.n - base);
  if (!stage_chunk(a, base, gcount, s_means, s_cov, s_sigma, &bar)) return;
  if (hits) {
    for (int i = lane; i < T; i += 32) s_hw[i] = 0;
    __syncwarp();
  }

  float hb[kPer];  // view-independent bbox half-width bounds (kSkip)
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int j = tid + k * kThreads;
    hb[k] = INFINITY;
    if (kSkip && j < gcount) {
      float cw[6];
      load_cov6(s_cov + j * cs, cs, cw);
      hb[k] = view_free_half_bound(cw);
    }
  }

  const int v_begin = blockIdx.y * a.views_per_cta;
  const int v_end = min(a.nviews, v_begin + a.views_per_cta);
  for (int v = v_begin; v < v_end; ++v) {
    const ViewConst& vc = a.views[v];
    const int Nr = vc.h.Nr, Na = vc.h.Na;
    for (int i = tid; i < T1 * (kShadow ? 2 : 1); i += kThreads) s_diff_ipp[i] = 0;
    if (masks)
      for (int i = tid; i < T * (kShadow ? 2 : 1); i += kThreads) s_mask_ipp[i] = 0;
    if (kSkip && tid == 0) s_qn = 0;
    __syncthreads();

    uint32_t* rects_ipp = reinterpret_cast<uint32_t*>(a.ipp.base + v * a.ipp.vstride + a.ipp.L.rects);
    uint32_t* rects_sh =
        kShadow ? reinterpret_cast<uint32_t*>(a.sh.base + v * a.sh.vstride + a.sh.L.rects) : nullptr;
    // every rectangle of the view is written (cell binning marks its state
    // sparse afterwards)
    if (!kSkip && chunk == 0 && tid == 0)
      *reinterpret_cast<int64_t*>(a.ipp.base + v * a.ipp.vstride + a.ipp.L.meta) = INT64_MAX;

    if (kSkip) {
      // stage 1: cheap conservative test for every Gaussian
      const ViewConst vcl = vc;  // local copy: the rect stores below cannot alias it
      const int* open_ipp = a.open_ipp + v * a.open_vstride;
      const int* open_sh = a.open_sh + v * a.open_vstride;
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int j = tid + k * kThreads;
        bool exact = false;
        if (j < gcount) {
          bool skip = s_sigma[j] < 0.01f;  // invalid: empty rectangles either way
          if (!skip && hb[k] <= 64.0f) {
            float r, c, xr, yr;
            approx_center(vcl, s_means[3 * j], s_means[3 * j + 1], s_means[3 * j + 2], r, c, xr, yr);
            const float h = hb[k] + vcl.center_margin;
            skip = open_in_rect(bound_rect(r, c, h, Nr, Na), open_ipp, pitch) == 0;
            if (kShadow && skip) skip = open_in_rect(bound_rect(yr, xr, h, Nr, Na), open_sh, pitch) == 0;
          }
          if (skip) {
            rects_ipp[base + j] = kEmptyRect;
            if (kShadow) rects_sh[base + j] = kEmptyRect;
          }
          exact = !skip;
        }
        const unsigned m = __ballot_sync(0xffffffffu, exact);
        if (m) {
          int slot0 = 0;
          if (lane == 0) slot0 = atomicAdd(&s_qn, __popc(m));
          slot0 = __shfl_sync(0xffffffffu, slot0, 0);
          if (exact) s_queue[slot0 + __popc(m & ((1u << lane) - 1u))] = (short)j;
        }
      }
      __syncthreads();
      // stage 2: the queued Gaussians, exactly
      const int qn = s_qn;
      for (int q = tid; q < qn; q += kThreads) {
        const int j = s_queue[q];
        uint32_t rc_ipp = kEmptyRect, rc_sh = kEmptyRect;
        bin_exact<kShadow>(vcl, s_means, s_cov, cs, j, rc_ipp, rc_sh);
        rects_ipp[base + j] = rc_ipp;
        diff_add(s_diff_ipp, pitch, rc_ipp);
        if (kShadow) {
          rects_sh[base + j] = rc_sh;
          diff_add(s_diff_sh, pitch, rc_sh);
        }
      }
    } else {
      const ViewConst vcl = vc;  // local copy: loaded once for all of this thread's Gaussians
      uint32_t* ghw = hits ? a.hbits + v * a.hbits_vstride + (size_t)chunk * T * 32 : nullptr;
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int j = tid + k * kThreads;
        uint32_t rc_hit = kEmptyRect;
        if (j < gcount) {
          uint32_t rc_ipp = kEmptyRect, rc_sh = kEmptyRect;
          if (!(s_sigma[j] < 0.01f))  // preprocess_kernel: transmittance < 0.01 -> invalid (:351)
            bin_exact<kShadow>(vcl, s_means, s_cov, cs, j, rc_ipp, rc_sh);
          rects_ipp[base + j] = rc_ipp;
          diff_add(s_diff_ipp, pitch, rc_ipp);
          if (masks) mark_rect(s_mask_ipp, rc_ipp, tiles_x, 1u << (j >> 5));
          if (hits) mark_rect(s_hw, rc_ipp, tiles_x, 1u << lane);
          rc_hit = rc_ipp;
          if (kShadow) {
            rects_sh[base + j] = rc_sh;
            diff_add(s_diff_sh, pitch, rc_sh);
            if (masks) mark_rect(s_mask_sh, rc_sh, tiles_x, 1u << (j >> 5));
          }
        }
        if (hits) {
          __syncwarp();
          flush_hit_words(s_hw, rc_hit, tiles_x, ghw + ((tid + k * kThreads) >> 5));
          __syncwarp();  // the words are clear before the next segment's ORs
        }
      }
    }
    __syncthreads();

    // 2-D inclusive prefix of the difference arrays: rows, then columns.
    // Threads [0,128) handle the image-plane list, [128,256) the shadow list.
    {
      const int half = tid >> 7, i = tid & 127;
      if (half == 0 || (kShadow && half == 1)) {
        int* d = half ? s_diff_sh : s_diff_ipp;
        if (i < tiles_y) {
          int run = 0;
          for (int x = 0; x < tiles_x; ++x) {
            run += d[i * pitch + x];
            d[i * pitch + x] = run;
          }
        }
      }
    }
    __syncthreads();
    {
      const int half = tid >> 7, i = tid & 127;
      if (half == 0 || (kShadow && half == 1)) {
        int* d = half ? s_diff_sh : s_diff_ipp;
        if (i < tiles_x) {
          int run = 0;
          for (int y = 0; y < tiles_y; ++y) {
            run += d[y * pitch + i];
            d[y * pitch + i] = run;
          }
        }
      }
    }
    __syncthreads();

    uint8_t* cnt_ipp = a.counts_ipp + v * a.counts_vstride + (size_t)chunk * T;
    uint8_t* cnt_sh = kShadow ? a.counts_sh + v * a.counts_vstride + (size_t)chunk * T : nullptr;
    for (int t = tid; t < T; t += kThreads) {
      const int y = t / tiles_x, x = t - y * tiles_x;
      cnt_ipp[t] = (uint8_t)min(s_diff_ipp[y * pitch + x], 255);
      if (kShadow) cnt_sh[t] = (uint8_t)min(s_diff_sh[y * pitch + x], 255);
    }
    if (masks) {
      uint32_t* m = a.segmask + v * a.segmask_vstride + (size_t)chunk * T;
      for (int t = tid; t < T; t += kThreads) m[t] = s_mask_ipp[t];
      if (kShadow) {
        uint32_t* msh = a.segmask_sh + v * a.segmask_vstride + (size_t)chunk * T;
        for (int t = tid; t < T; t += kThreads) msh[t] = s_mask_sh[t];
      }
    }
    __syncthreads();  // the difference arrays and the queue are reused by the next view
  }
}

// Exact list of view v and chunk c (null when the launch records none), and
// the per-chunk lengths of view v.
__device__ __forceinline__ uint16_t* x_list(const BinArgs& a, int v, int c) {
  if (!a.xlist) return nullptr;
  return reinterpret_cast<uint16_t*>(reinterpret_cast<unsigned char*>(a.xlist) + v * a.x_vstride) +
         (size_t)c * kXCap;
}
__device__ __forceinline__ int* x_count(const BinArgs& a, int v) {
  return reinterpret_cast<int*>(reinterpret_cast<unsigned char*>(a.xcount) + v * a.x_vstride);
}

// Adds one hit to every tile of a rectangle in a warp's tile counters (two
// 16-bit counters per word; a chunk holds at most kChunk hits per tile) and,
// when `mask` is given, ORs `bit` into the tiles' segment masks, in one
// flattened pass over the rectangle's tiles. The OR is atomic when
// kAtomicOr (lanes may OR different bits); otherwise it is a plain
// read-modify-write, exact when every lane between two __syncwarp ORs the
// same bit into masks only its warp writes.
template <bool kAtomicOr>
__device__ __forceinline__ void count_mark_rect(uint32_t* cnt, uint32_t* mask, uint32_t rc,
                                                int tiles_x, uint32_t bit, uint32_t* hw = nullptr,
                                                uint32_t hbit = 0) {
  if (rc == kEmptyRect) return;
  const int tc0 = rc & 0xFF, tc1 = (rc >> 8) & 0xFF, tr0 = (rc >> 16) & 0xFF, tr1 = rc >> 24;
  const int w = tc1 - tc0 + 1, cells = w * (tr1 - tr0 + 1);
  int t = tr0 * tiles_x + tc0, x = 0;
  for (int e = 0; e < cells; ++e) {
    atomicAdd(cnt + (t >> 1), 1u << ((t & 1) << 4));
    if (hw) atomicOr(hw + t, hbit);
    if (mask) {
      if (kAtomicOr) {
        atomicOr(mask + t, bit);
      } else {
        volatile uint32_t* m = mask + t;
        *m = *m | bit;
      }
    }
    if (++x == w) {
      x = 0;
      t += tiles_x - w + 1;
    } else {
      ++t;
    }
  }
}

// Writes a warp's tile counters of one view and chunk as saturating u8 counts
// and clears them for the next view.
__device__ __forceinline__ void flush_counts(uint32_t* cnt, uint8_t* out, int T, int lane) {
  if ((T & 3) == 0) {
    for (int t4 = lane; t4 < (T >> 2); t4 += 32) {
      const uint32_t w0 = cnt[2 * t4], w1 = cnt[2 * t4 + 1];
      const uint32_t c0 = min(w0 & 0xFFFFu, 255u), c1 = min(w0 >> 16, 255u);
      const uint32_t c2 = min(w1 & 0xFFFFu, 255u), c3 = min(w1 >> 16, 255u);
      reinterpret_cast<uint32_t*>(out)[t4] = c0 | (c1 << 8) | (c2 << 16) | (c3 << 24);
    }
  } else {
    for (int t = lane; t < T; t += 32)
      out[t] = (uint8_t)min((cnt[t >> 1] >> ((t & 1) << 4)) & 0xFFFFu, 255u);
  }
  __syncwarp();
  for (int i = lane; i < ((T + 1) >> 1); i += 32) cnt[i] = 0;
  __syncwarp();
}

// Prefix chunks, one view per warp: every Gaussian of the staged chunk is
// binned exactly by the warp of its view (32 per round), its hits counted in
// per-warp 16-bit tile counters and, for the segment masks, the round's bit
// ORed into per-warp tile masks (all lanes of a round OR the same bit, so the
// plain read-modify-write is exact). No CTA barrier inside the view loop.
// Means and transmittances are staged; covariances are read through L1.
template <bool kShadow>
#ifndef SARR_PREFIX_MIN_CTAS
#define SARR_PREFIX_MIN_CTAS 4
#endif
__global__ void __launch_bounds__(kBinThreads, SARR_PREFIX_MIN_CTAS) bin_prefix_kernel(const BinArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ uint64_t bar;
  constexpr int kWarps = kBinThreads / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunk = blockIdx.x + a.chunk_offset;
  const int tiles_x = a.views[0].tiles_x, tiles_y = a.views[0].tiles_y, T = tiles_x * tiles_y;
  const int TW = (T + 1) >> 1;
  const int cs = a.cov_layout;
  const int lists = kShadow ? 2 : 1;
  const bool masks = a.segmask != nullptr;

  float* s_means = reinterpret_cast<float*>(smem_raw);
  float* s_sigma = s_means + 3 * kChunk;
  uint32_t* s_cnt = reinterpret_cast<uint32_t*>(s_sigma + kChunk) + warp * (TW + T) * lists;
  uint32_t* s_cnt_sh = s_cnt + TW;
  uint32_t* s_mask = s_cnt + TW * lists;
  uint32_t* s_mask_sh = s_mask + T;
  // hit words of the current round (image list), after every warp's counters
  const bool hits = a.hbits != nullptr && masks && chunk < a.hbits_to;
  uint32_t* s_hw = reinterpret_cast<uint32_t*>(s_sigma + kChunk) + kWarps * (TW + T) * lists + warp * T;

  const int64_t base = (int64_t)chunk * kChunk;
  const int gcount = (int)min((int64_t)kChunk, a.n - base);
  {
    const bool tma = a.use_tma && gcount == kChunk;
    if (tid == 0 && tma) mbar_init(&bar, 1);
    __syncthreads();
    bool ok = true;
    if (tma) {
      if (tid == 0) {
        mbar_arrive_expect_tx(&bar, 4u * kChunk * 4u);
        tma_load_1d(s_means, a.means + base * 3, 3u * kChunk * 4u, &bar);
        tma_load_1d(s_sigma, a.sigma + base, kChunk * 4u, &bar);
      }
      ok = mbar_wait_bounded(&bar, 0, a.err);
    } else {
      for (int i = tid; i < 3 * gcount; i += kBinThreads) s_means[i] = a.means[base * 3 + i];
      for (int i = tid; i < gcount; i += kBinThreads) s_sigma[i] = a.sigma[base + i];
    }
    if (!__syncthreads_and(ok)) return;
  }
  for (int i = lane; i < (TW + T) * lists; i += 32) s_cnt[i] = 0;
  if (hits)
    for (int i = lane; i < T; i += 32) s_hw[i] = 0;
  __syncwarp();
  const float* cov = a.cov + base * cs;

  const int v_end = min(a.nviews, (int)(blockIdx.y + 1) * a.views_per_cta);
  for (int v = blockIdx.y * a.views_per_cta + warp; v < v_end; v += kWarps) {
    const ViewConst& vg = a.views[v];
    unsigned char* stv = a.ipp.base + v * a.ipp.vstride;
    uint32_t* rects_ipp = reinterpret_cast<uint32_t*>(stv + a.ipp.L.rects) + base;
    uint32_t* rects_sh =
        kShadow ? reinterpret_cast<uint32_t*>(a.sh.base + v * a.sh.vstride + a.sh.L.rects) + base : nullptr;
    // every rectangle of the view is written (cell binning marks its state
    // sparse afterwards)
    if (chunk == 0 && lane == 0) *reinterpret_cast<int64_t*>(stv + a.ipp.L.meta) = INT64_MAX;
    uint32_t* ghw = hits ? a.hbits + v * a.hbits_vstride + (size_t)chunk * T * 32 : nullptr;
    for (int r = 0; r < kChunk / 32; ++r) {
      const int j = r * 32 + lane;
      uint32_t rc_hit = kEmptyRect;
      if (j < gcount) {
        uint32_t rc_ipp = kEmptyRect, rc_sh = kEmptyRect;
        if (!(s_sigma[j] < 0.01f)) {  // preprocess_kernel: transmittance < 0.01 -> invalid (:351)
          Proj o;
          const float Rmin = project_center(vg, s_means[3 * j], s_means[3 * j + 1], s_means[3 * j + 2], o);
          if (proj_valid(o, vg.h.Nr, vg.h.Na)) {
            float cw[6], X6[6];
            load_cov6(cov + j * cs, cs, cw);
            radar_cov(vg, cw, X6);
            image_cov(vg, X6, Rmin, o);
            int r0, r1, c0, c1;
            ipp_ranges(o, vg.h.Nr, vg.h.Na, r0, r1, c0, c1);
            rc_ipp = make_rect(r0, r1, c0, c1, vg.h.Nr, vg.h.Na);
            if (kShadow && shadow_ranges(o, vg.h.Nr, vg.h.Na, r0, r1, c0, c1))
              rc_sh = make_rect(r0, r1, c0, c1, vg.h.Nr, vg.h.Na);
          }
        }
        rects_ipp[j] = rc_ipp;
        count_mark_rect<false>(s_cnt, masks ? s_mask : nullptr, rc_ipp, tiles_x, 1u << r,
                               hits ? s_hw : nullptr, 1u << lane);
        rc_hit = rc_ipp;
        if (kShadow) {
          rects_sh[j] = rc_sh;
          count_mark_rect<false>(s_cnt_sh, masks ? s_mask_sh : nullptr, rc_sh, tiles_x, 1u << r);
        }
      }
      __syncwarp();  // the next round ORs another bit into the same masks
      if (hits) {
        flush_hit_words(s_hw, rc_hit, tiles_x, ghw + r);
        __syncwarp();  // the words are clear before the next round's ORs
      }
    }
    flush_counts(s_cnt, a.counts_ipp + v * a.counts_vstride + (size_t)chunk * T, T, lane);
    if (kShadow) flush_counts(s_cnt_sh, a.counts_sh + v * a.counts_vstride + (size_t)chunk * T, T, lane);
    if (masks) {
      uint32_t* m = a.segmask + v * a.segmask_vstride + (size_t)chunk * T;
      for (int t = lane; t < T; t += 32) {
        m[t] = s_mask[t];
        s_mask[t] = 0;
      }
      if (kShadow) {
        uint32_t* msh = a.segmask_sh + v * a.segmask_vstride + (size_t)chunk * T;
        for (int t = lane; t < T; t += 32) {
          msh[t] = s_mask_sh[t];
          s_mask_sh[t] = 0;
        }
      }
    }
    __syncwarp();
  }
}

// Writes a warp's tile segment masks of one view and chunk and clears them.
// Only nonzero masks are written: select_kernel reads the mask of a (chunk,
// tile) only when the chunk holds hits of the tile.
__device__ __forceinline__ void flush_masks(uint32_t* mask, uint32_t* out, int T, int lane) {
  for (int t = lane; t < T; t += 32) {
    const uint32_t m = mask[t];
    if (m) {
      out[t] = m;
      mask[t] = 0;
    }
  }
  __syncwarp();
}

// Saturation-skipping binning of the chunks after the prefix. The chunk is
// staged once per CTA (with the view-independent bbox bounds); with more than
// four views per CTA each warp then bins whole views alone, with no CTA
// barrier, and with fewer the warps of a view split the chunk into slices.
// A conservative test of every Gaussian (approximate centre, bbox bound,
// open-tile table) writes empty rectangles for those that can only reach
// saturated tiles, the others go to a warp queue that is drained 32 at a time
// by exact binning, and the hits land in per-warp tile counters.
// The covariances are read through L1 rather than staged: each is read once
// for the bound and again only for the exactly binned Gaussians, and the
// smaller shared-memory footprint leaves L1 to cache them (0.76 -> 0.73 ms
// per 1024 sweep views; the single-view forward + backward 6.16k -> 6.35k
// steps/s).
#ifndef SARR_SKIP_COV_SMEM
#define SARR_SKIP_COV_SMEM 0
#endif
template <bool kShadow>
__global__ void __launch_bounds__(kBinThreads, 3) bin_skip_kernel(const BinArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ uint64_t bar;
  __shared__ short s_queue[kBinThreads / 32][64];
  constexpr int kWarps = kBinThreads / 32;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunk = blockIdx.x + a.chunk_offset;
  const int tiles_x = a.views[0].tiles_x, tiles_y = a.views[0].tiles_y, T = tiles_x * tiles_y;
  const int cs = a.cov_layout;
  const int TW = (T + 1) >> 1;

  const int64_t base = (int64_t)chunk * kChunk;
  float* s_means = reinterpret_cast<float*>(smem_raw);
  // the covariances staged (SARR_SKIP_COV_SMEM) or read from global memory
  float* s_cov_st = SARR_SKIP_COV_SMEM ? s_means + 3 * kChunk : nullptr;
  const float* s_cov = SARR_SKIP_COV_SMEM ? s_cov_st : a.cov + base * cs;
  float* s_sigma = s_means + 3 * kChunk + (SARR_SKIP_COV_SMEM ? cs * kChunk : 0);
  float* s_hb = s_sigma + kChunk;
  uint32_t* s_cnt = reinterpret_cast<uint32_t*>(s_hb + kChunk) + warp * TW * (kShadow ? 2 : 1);
  uint32_t* s_cnt_sh = s_cnt + TW;
  // segment masks (when a.skip_masks): bit s of tile t is set when Gaussians
  // [32 s, 32 s + 32) of the chunk hold a hit of t
  const bool masks = a.skip_masks != 0;
  uint32_t* s_mask = reinterpret_cast<uint32_t*>(s_hb + kChunk) + kWarps * TW * (kShadow ? 2 : 1) +
                     warp * T * (kShadow ? 2 : 1);
  uint32_t* s_mask_sh = s_mask + T;

  const int gcount = (int)min((int64_t)kChunk, a.n - base);
  if (!stage_chunk(a, base, gcount, s_means, s_cov_st, s_sigma, &bar)) return;

  for (int i = lane; i < TW * (kShadow ? 2 : 1); i += 32) s_cnt[i] = 0;
  if (masks)
    for (int i = lane; i < T * (kShadow ? 2 : 1); i += 32) s_mask[i] = 0;
  for (int j = tid; j < gcount; j += kBinThreads) {
    float cw[6];
    load_cov6(s_cov + j * cs, cs, cw);
    s_hb[j] = view_free_half_bound(cw);
  }
  __syncthreads();

  const int pitch = tiles_x + 1;
  const unsigned lt_mask = (1u << lane) - 1u;
  short* queue = s_queue[warp];

  // Bins Gaussians [j_lo, j_hi) of the chunk for view v into this warp's
  // counters; the exactly binned ones are listed (index order) in xl[0..).
  // Returns how many were listed.
  auto bin_range = [&](int v, int j_lo, int j_hi, uint16_t* xl) {
    const ViewConst& vg = a.views[v];  // exact binning reads its constants from here (L1)
    const ViewConst vc = vg;            // the stage-1 constants, held in registers
    const int Nr = vc.h.Nr, Na = vc.h.Na;
    uint32_t* rects_ipp = reinterpret_cast<uint32_t*>(a.ipp.base + v * a.ipp.vstride + a.ipp.L.rects) + base;
    uint32_t* rects_sh =
        kShadow ? reinterpret_cast<uint32_t*>(a.sh.base + v * a.sh.vstride + a.sh.L.rects) + base : nullptr;
    const int* open_ipp = a.open_ipp + v * a.open_vstride;
    const int* open_sh = a.open_sh + v * a.open_vstride;
    int xn = 0;
    // exact binning of queue[lane] (every lane with a queued Gaussian)
    auto bin_queued = [&](int j) {
      uint32_t rc_ipp = kEmptyRect, rc_sh = kEmptyRect;
      bin_exact<kShadow>(vg, s_means, s_cov, cs, j, rc_ipp, rc_sh);
      rects_ipp[j] = rc_ipp;
      count_mark_rect<true>(s_cnt, masks ? s_mask : nullptr, rc_ipp, tiles_x, 1u << (j >> 5));
      if (kShadow) {
        rects_sh[j] = rc_sh;
        count_mark_rect<true>(s_cnt_sh, masks ? s_mask_sh : nullptr, rc_sh, tiles_x, 1u << (j >> 5));
      }
      if (xl) xl[xn + lane] = (uint16_t)j;
    };
    int qn = 0;
    for (int j0 = j_lo; j0 < j_hi; j0 += 32) {
      const int j = j0 + lane;
      bool exact = false;
      if (j < j_hi) {
        bool skip = s_sigma[j] < 0.01f;  // invalid: empty rectangles either way
        const float hb = s_hb[j];
        if (!skip && hb <= 64.0f) {
          float r, c, xr, yr;
          approx_center(vc, s_means[3 * j], s_means[3 * j + 1], s_means[3 * j + 2], r, c, xr, yr);
          const float h = hb + vc.center_margin;
          skip = open_in_rect(bound_rect(r, c, h, Nr, Na), open_ipp, pitch) == 0;
          if (kShadow && skip) skip = open_in_rect(bound_rect(yr, xr, h, Nr, Na), open_sh, pitch) == 0;
        }
        if (skip) {
          rects_ipp[j] = kEmptyRect;
          if (kShadow) rects_sh[j] = kEmptyRect;
        }
        exact = !skip;
      }
      const unsigned m = __ballot_sync(0xffffffffu, exact);
      if (exact) queue[qn + __popc(m & lt_mask)] = (short)j;
      qn += __popc(m);
      __syncwarp();
      if (qn >= 32) {
        bin_queued(queue[lane]);
        xn += 32;
        __syncwarp();
        if (lane < qn - 32) queue[lane] = queue[lane + 32];
        qn -= 32;
        __syncwarp();
      }
    }
    if (lane < qn) bin_queued(queue[lane]);
    xn += qn;
    __syncwarp();
    return xn;
  };

  const int vbase = blockIdx.y * a.views_per_cta;
  const int nv_cta = min(a.nviews - vbase, a.views_per_cta);
  if (nv_cta > kWarps / 2) {
    // one view per warp at a time
    for (int v = vbase + warp; v < vbase + nv_cta; v += kWarps) {
      const int xn = bin_range(v, 0, gcount, x_list(a, v, chunk));
      if (a.xlist && lane == 0) x_count(a, v)[chunk] = xn;
      flush_counts(s_cnt, a.counts_ipp + v * a.counts_vstride + (size_t)chunk * T, T, lane);
      if (kShadow) flush_counts(s_cnt_sh, a.counts_sh + v * a.counts_vstride + (size_t)chunk * T, T, lane);
      if (masks) {
        flush_masks(s_mask, a.segmask + v * a.segmask_vstride + (size_t)chunk * T, T, lane);
        if (kShadow) flush_masks(s_mask_sh, a.segmask_sh + v * a.segmask_vstride + (size_t)chunk * T, T, lane);
      }
    }
    return;
  }
  // few views: wpv warps share a view, each binning one contiguous slice of
  // the chunk; then all warps merge the slices' counters, masks and exact
  // lists (in slice order) and write them out
  __shared__ uint16_t s_x[kWarps / 2][kChunk];
  __shared__ int s_xn[kWarps];
  const int wpv = kWarps / nv_cta;
  const int vl = warp / wpv, sl = warp % wpv;
  const bool active = vl < nv_cta;
  const int per = (gcount + wpv * 32 - 1) / (wpv * 32) * 32;
  const int j_lo = min(gcount, sl * per), j_hi = min(gcount, j_lo + per);
  if (active) {
    const int xn = bin_range(vbase + vl, j_lo, j_hi, a.xlist ? s_x[vl] + j_lo : nullptr);
    if (lane == 0) s_xn[warp] = xn;
  }
  __syncthreads();
  if (active && a.xlist) {  // each warp places its own slice
    const int v = vbase + vl;
    int off = 0;
    for (int o = 0; o < sl; ++o) off += s_xn[vl * wpv + o];
    const int n_s = s_xn[warp];
    uint16_t* xl = x_list(a, v, chunk);
    for (int i = lane; i < n_s; i += 32) xl[off + i] = s_x[vl][j_lo + i];
    if (sl == wpv - 1 && lane == 0) x_count(a, v)[chunk] = off + n_s;
  }
  constexpr int kLists = kShadow ? 2 : 1;
  const uint32_t* cnt0 = reinterpret_cast<const uint32_t*>(s_hb + kChunk);  // warp w: + w * TW * kLists
  const uint32_t* mask0 = cnt0 + kWarps * TW * kLists;                     // warp w: + w * T * kLists
  // counters: the 16-bit tile counts of the copies add without carry (a
  // chunk holds 1024 Gaussians), then saturate to u8
  const bool quad = (T & 3) == 0;
  const int per_list = quad ? T / 4 : T;
  for (int it = tid; it < nv_cta * kLists * per_list; it += kBinThreads) {
    const int q = it % per_list, li = (it / per_list) % kLists, v_l = it / (per_list * kLists);
    const int v = vbase + v_l;
    uint8_t* out = (li ? a.counts_sh : a.counts_ipp) + v * a.counts_vstride + (size_t)chunk * T;
    const uint32_t* c = cnt0 + (v_l * wpv) * TW * kLists + li * TW;
    if (quad) {
      uint32_t w0 = 0, w1 = 0;
      for (int o = 0; o < wpv; ++o, c += TW * kLists) {
        w0 += c[2 * q];
        w1 += c[2 * q + 1];
      }
      const uint32_t c0 = min(w0 & 0xFFFFu, 255u), c1 = min(w0 >> 16, 255u);
      const uint32_t c2 = min(w1 & 0xFFFFu, 255u), c3 = min(w1 >> 16, 255u);
      reinterpret_cast<uint32_t*>(out)[q] = c0 | (c1 << 8) | (c2 << 16) | (c3 << 24);
    } else {
      uint32_t w = 0;
      for (int o = 0; o < wpv; ++o, c += TW * kLists) w += c[q >> 1];
      out[q] = (uint8_t)min((w >> ((q & 1) << 4)) & 0xFFFFu, 255u);
    }
  }
  if (masks) {
    for (int it = tid; it < nv_cta * kLists * T; it += kBinThreads) {
      const int t = it % T, li = (it / T) % kLists, v_l = it / (T * kLists);
      const uint32_t* m = mask0 + (v_l * wpv) * T * kLists + li * T + t;
      uint32_t acc = 0;
      for (int o = 0; o < wpv; ++o, m += T * kLists) acc |= *m;
      // only nonzero masks are read (select_kernel reads the mask of a
      // (chunk, tile) only when the chunk holds hits of the tile)
      if (acc) (li ? a.segmask_sh : a.segmask)[(vbase + v_l) * a.segmask_vstride + (size_t)chunk * T + t] = acc;
    }
  }
}

// ---------------------------------------------------------------------------
// cell culling (calls of kCellMinViews views or more)
// ---------------------------------------------------------------------------
// Tile rectangle of the box (cr +- hr) x (cc +- hc), clamped like bound_rect;
// half-widths that are not finite and below 1e6 give the whole image.
__device__ __forceinline__ uint32_t bound_rect2(float cr, float cc, float hr, float hc, int Nr,
                                                int Na) {
  if (!(hr < 1e6f && hc < 1e6f && fabsf(cr) < 1e9f && fabsf(cc) < 1e9f))
    return make_rect(0, Nr - 1, 0, Na - 1, Nr, Na);
  const int r0 = max(0, (int)floorf(cr - hr)), r1 = min(Nr - 1, (int)ceilf(cr + hr));
  const int c0 = max(0, (int)floorf(cc - hc)), c1 = min(Na - 1, (int)ceilf(cc + hc));
  return make_rect(r0, r1, c0, c1, Nr, Na);
}

__global__ void cell_init_kernel(SceneGrid* g, int* cell_hb, int* cell_count) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < kMaxCells) {
    cell_hb[i] = ordered_key(-1.0f);
    cell_count[i] = 0;
  }
  if (i < 3) {
    g->lo_key[i] = ordered_key(INFINITY);
    g->hi_key[i] = ordered_key(-INFINITY);
  }
  if (i == 0) g->n_always = 0;
}

// Bounding box of the finite Gaussian centres.
__global__ void __launch_bounds__(256) scene_bounds_kernel(const float* __restrict__ means,
                                                           int64_t n, SceneGrid* g) {
  float lo[3] = {INFINITY, INFINITY, INFINITY}, hi[3] = {-INFINITY, -INFINITY, -INFINITY};
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x) {
    const float p[3] = {means[3 * j], means[3 * j + 1], means[3 * j + 2]};
    if (isfinite(p[0]) && isfinite(p[1]) && isfinite(p[2])) {
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        lo[k] = fminf(lo[k], p[k]);
        hi[k] = fmaxf(hi[k], p[k]);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    for (int o = 16; o > 0; o >>= 1) {
      lo[k] = fminf(lo[k], __shfl_xor_sync(0xffffffffu, lo[k], o));
      hi[k] = fmaxf(hi[k], __shfl_xor_sync(0xffffffffu, hi[k], o));
    }
  }
  // one set of atomics per CTA (the per-warp ones contended on six words)
  __shared__ float s_lo[8][3], s_hi[8][3];
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      s_lo[warp][k] = lo[k];
      s_hi[warp][k] = hi[k];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      float l = s_lo[0][k], h = s_hi[0][k];
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
        l = fminf(l, s_lo[w][k]);
        h = fmaxf(h, s_hi[w][k]);
      }
      atomicMin(&g->lo_key[k], ordered_key(l));
      atomicMax(&g->hi_key[k], ordered_key(h));
    }
  }
}

// Cell grid over the bounding box: about n / 32 cells, at most kMaxCells.
// Membership uses floor((p - lo) / a) in float; half_diag bounds the distance
// of a member to its cell's centre including those roundings.
__global__ void scene_grid_kernel(SceneGrid* g, int64_t n) {
  if (threadIdx.x != 0) return;
  float lo[3], hi[3], ext[3];
  bool ok = true;
  for (int k = 0; k < 3; ++k) {
    lo[k] = key_float(g->lo_key[k]);
    hi[k] = key_float(g->hi_key[k]);
    ok = ok && (lo[k] <= hi[k]);
    ext[k] = hi[k] - lo[k];
  }
  g->valid = 0;
  g->ncells = 0;
  if (!ok) return;
  const float emax = fmaxf(ext[0], fmaxf(ext[1], ext[2]));
  const float pad = 1e-3f * emax + 1e-6f;
  const float vol = (ext[0] + pad) * (ext[1] + pad) * (ext[2] + pad);
  const int64_t target = max((int64_t)1, min((int64_t)kMaxSpatialCells, n / 64));
  float a = cbrtf(vol / (float)target);
  if (!(a > 0.0f) || !isfinite(a)) a = fmaxf(emax, 1e-6f);
  int dims[3];
  for (int it = 0; it < 200; ++it) {
    for (int k = 0; k < 3; ++k) {
      float t = ceilf(ext[k] / a);
      dims[k] = t < 1.0f ? 1 : (t > 1e6f ? 1000000 : (int)t);
      while ((float)dims[k] * a < ext[k]) ++dims[k];
    }
    if (padded_spatial_cells(dims) <= kMaxSpatialCells) break;
    a *= 1.05f;
  }
  const int64_t prod = padded_spatial_cells(dims);
  if (prod > kMaxSpatialCells) return;  // not reached for finite boxes; no cells then
  float scale = emax + a;
  for (int k = 0; k < 3; ++k) {
    g->lo[k] = lo[k];
    g->dims[k] = dims[k];
    scale += fabsf(lo[k]);
  }
  g->a = a;
  g->inv_a = 1.0f / a;
  g->nspatial = (int)prod;
  g->ncells = (int)prod * kHbBuckets;
  g->half_diag = a * 0.8660254f * 1.0001f + 4e-6f * scale;
  g->valid = 1;
}

// Centres of the spatial cells.
__global__ void __launch_bounds__(256) cell_center_kernel(const SceneGrid* g, float4* center) {
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (!g->valid || c >= g->nspatial) return;
  // the inverse of spatial_cell
  const int nbx = (g->dims[0] + 3) / 4, nby = (g->dims[1] + 3) / 4;
  const int blk = c / kCellBlock, l = c % kCellBlock;
  const int ix = (blk % nbx) * 4 + (l & 3), iy = ((blk / nbx) % nby) * 4 + ((l >> 2) & 3);
  const int iz = (blk / (nbx * nby)) * 2 + (l >> 4);
  center[c] = make_float4(g->lo[0] + ((float)ix + 0.5f) * g->a, g->lo[1] + ((float)iy + 0.5f) * g->a,
                          g->lo[2] + ((float)iz + 0.5f) * g->a, 0.0f);
}

// Per Gaussian: its view-independent bbox bound and cell id, and the largest
// bound of every cell.
__global__ void __launch_bounds__(256) cell_assign_kernel(const CellPrepArgs a) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= a.n) return;
  const SceneGrid& g = *a.grid;
  uint32_t id = kCellAlways;
  float hb = INFINITY;
  if (a.sigma[j] < 0.01f) {
    id = kCellNever;  // preprocess_kernel: invalid (:351)
  } else {
    float cw[6];
    load_cov6(a.cov + j * a.cov_layout, a.cov_layout, cw);
    hb = view_free_half_bound(cw);
    const float x = a.means[3 * j], y = a.means[3 * j + 1], z = a.means[3 * j + 2];
    if (g.valid && hb <= kCellMaxHalfBound && isfinite(x) && isfinite(y) && isfinite(z)) {
      const int ix = min(max((int)floorf((x - g.lo[0]) * g.inv_a), 0), g.dims[0] - 1);
      const int iy = min(max((int)floorf((y - g.lo[1]) * g.inv_a), 0), g.dims[1] - 1);
      const int iz = min(max((int)floorf((z - g.lo[2]) * g.inv_a), 0), g.dims[2] - 1);
      id = (uint32_t)(spatial_cell(g.dims, ix, iy, iz) * kHbBuckets + hb_bucket(hb));
      atomicMax(a.cell_hb + id, ordered_key(hb));
      if (j >= a.pstart) atomicAdd(a.cell_count + id, 1);
    }
  }
  a.hb[j] = hb;
  a.cid[j] = id;
  if (id == kCellAlways && j >= a.pstart) a.always[atomicAdd(&a.grid->n_always, 1)] = (int)j;
}

// Exclusive scan of the cells' member counts into cell_start, in two passes of
// 1024-cell blocks (block scans, then block offsets); the counts become the
// fill cursors.
__device__ __forceinline__ int block_excl_scan_1024(int x, int* s_warp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int incl = warp_incl_scan(x, lane);
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = s_warp[lane];
    s_warp[lane] = warp_incl_scan(w, lane) - w;
  }
  __syncthreads();
  return s_warp[warp] + incl - x;
}

__global__ void __launch_bounds__(1024) cell_scan_blocks_kernel(const CellPrepArgs a) {
  __shared__ int s_warp[32];
  const int c = blockIdx.x * 1024 + threadIdx.x;
  const int x = a.cell_count[c];
  const int excl = block_excl_scan_1024(x, s_warp);
  a.cell_start[c] = excl;
  if (threadIdx.x == 1023) a.grid->block_sums[blockIdx.x] = excl + x;
}

__global__ void __launch_bounds__(1024) cell_scan_offsets_kernel(const CellPrepArgs a) {
  __shared__ int s_off;
  const int c = blockIdx.x * 1024 + threadIdx.x;
  if (threadIdx.x < 32) {
    int sum = 0;
    for (int b = threadIdx.x; b < (int)blockIdx.x; b += 32) sum += a.grid->block_sums[b];
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (threadIdx.x == 0) s_off = sum;
  }
  __syncthreads();
  const int start = a.cell_start[c] + s_off;
  a.cell_start[c] = start;
  a.cell_count[c] = start;
  if (c == kMaxCells - 1) a.cell_start[kMaxCells] = s_off + a.grid->block_sums[gridDim.x - 1];
}

// Member lists: centre and bbox bound of every Gaussian after the prefix,
// grouped by cell (order inside a cell is immaterial: the lists are only
// read to find the Gaussians to bin exactly, which are then ordered per chunk).
__global__ void __launch_bounds__(256) cell_fill_kernel(const CellPrepArgs a) {
  const int64_t j = a.pstart + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= a.n) return;
  const uint32_t id = a.cid[j];
  if (id >= (uint32_t)kMaxCells) return;
  const int pos = atomicAdd(a.cell_count + id, 1);
  a.mem_pos[pos] = make_float4(a.means[3 * j], a.means[3 * j + 1], a.means[3 * j + 2], a.hb[j]);
  a.mem_idx[pos] = (int)j;
}

// Cell bitmap of one view: bit c is set when a member of cell c may reach a
// tile still open after the prefix (either list). A member p of cell c lies
// within half_diag of the cell centre q; R_min and X_r are 1-Lipschitz in the
// world position, so its exact image centre lies within half_diag / rho
// (pixels) of q's, and approximate-centre errors add center_margin at p and q.
template <bool kStaged>
__global__ void __launch_bounds__(256) cell_test_kernel(const CellTestArgs a) {
  // one thread per spatial cell: its centre is projected once and tested
  // with the bound of each of its kHbBuckets cells c = spatial * 4 + bucket
  static_assert(kHbBuckets == 4, "a lane assembles one 4-bit nibble of the cell bitmap");
  extern __shared__ int s_open[];
  const int sc = blockIdx.x * 256 + threadIdx.x, lane = threadIdx.x & 31;
  const int v = blockIdx.y;
  const SceneGrid& g = *a.grid;
  const int tsize = (a.views[v].tiles_x + 1) * (a.views[v].tiles_y + 1);
  if (kStaged)
    stage_open_tables(s_open, a.open_ipp + v * a.open_vstride, a.open_sh + v * a.open_vstride, tsize,
                      a.shadow ? 2 : 1);
  uint32_t nib = 0;
  if (g.valid && sc * kHbBuckets < g.ncells) {
    const ViewConst& vc = a.views[v];
    const int Nr = vc.h.Nr, Na = vc.h.Na, pitch = vc.tiles_x + 1;
    float r = 0.0f, cc = 0.0f, xr = 0.0f, yr = 0.0f;  // the cell centre's image position
    const float dr = g.half_diag * fabsf(vc.inv_rho_r) * 1.0001f;
    const float dc = g.half_diag * fabsf(vc.inv_rho_a) * 1.0001f;
    const float ds = g.half_diag * 1.0001f;
    const int* open_ipp = a.open_ipp + v * a.open_vstride;
    const int* open_sh = a.open_sh + v * a.open_vstride;
    // a larger bound gives a rectangle that contains the smaller one's, so
    // the cell's largest bound is tested first: when it reaches no open tile,
    // neither does any of its buckets (most cells of a view)
    auto reaches_open = [&](float hbm) {
      const float base = hbm + 2.0f * vc.center_margin + 0.02f;
      const uint32_t ri = bound_rect2(r, cc, base + dr, base + dc, Nr, Na);
      bool open = (kStaged ? open_in_rect_s(ri, s_open, pitch) : open_in_rect(ri, open_ipp, pitch)) > 0;
      if (a.shadow && !open) {
        const uint32_t rs = bound_rect2(yr, xr, base + ds, base + ds, Nr, Na);
        open = (kStaged ? open_in_rect_s(rs, s_open + tsize, pitch) : open_in_rect(rs, open_sh, pitch)) > 0;
      }
      return open;
    };
    float hbv[kHbBuckets];
    float hmax = -1.0f;
#pragma unroll
    for (int b = 0; b < kHbBuckets; ++b) {
      hbv[b] = key_float(a.cell_hb[sc * kHbBuckets + b]);
      if (hbv[b] >= 0.0f && hbv[b] > hmax) hmax = hbv[b];
    }
    if (hmax >= 0.0f) {
      const float4 q = a.cell_center[sc];
      approx_center(vc, q.x, q.y, q.z, r, cc, xr, yr);
    }
    if (hmax >= 0.0f && reaches_open(hmax)) {
#pragma unroll
      for (int b = 0; b < kHbBuckets; ++b)
        if (hbv[b] >= 0.0f && (hbv[b] == hmax || reaches_open(hbv[b]))) nib |= 1u << b;
    }
  }
  // word k of the warp's 4 bitmap words holds the nibbles of lanes 8k .. 8k+7
  uint32_t word = nib << (4 * (lane & 7));
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) word |= __shfl_xor_sync(0xffffffffu, word, o);
  if ((lane & 7) == 0) {
    const int wi = sc * kHbBuckets >> 5;
    a.bits[v * a.bits_vstride + wi] = word;
    if (word) a.cand_words[v * a.cand_vstride + atomicAdd(a.cand_count + v, 1)] = (uint32_t)wi;
  }
  unsigned char* xs = a.ipp.base + v * a.ipp.vstride;
  uint32_t* xbits = reinterpret_cast<uint32_t*>(xs + a.ipp.L.xbits);
  const int64_t words = (a.n + 31) / 32;
  for (int64_t i = blockIdx.x * 256 + threadIdx.x; i < words; i += (int64_t)gridDim.x * 256) xbits[i] = 0;
  if (blockIdx.x == 0 && threadIdx.x == 0)
    *reinterpret_cast<int64_t*>(xs + a.ipp.L.meta) = a.sparse_from;
}

// Cell binning, part 1 (per view): the members of the view's candidate cells
// (bit set by cell_test_kernel) go through bin_skip_kernel's per-Gaussian
// test; those it cannot skip, and the Gaussians in no cell, get their bit set
// in the view's exactly-binned bitmap. bin_finalize_kernel bins them.
// Grid: (kCandBlocks + kAlwaysBlocks, views). The first kCandBlocks CTAs'
// warps take the view's nonzero bitmap words (cell_test_kernel's list) in
// turn, a warp the 32 cells of one word; the others take strides of the
// no-cell list. The bits are ORed, so the order of the words does not matter.
constexpr int kCandBlocks = 32;
constexpr int kAlwaysBlocks = 16;

// 32 registers for 8 CTAs per SM: the member gathers are latency-bound
// (0.80 -> 0.71 ms per 1024 sweep views against 45 registers)
#ifndef SARR_CAND_MIN_CTAS
#define SARR_CAND_MIN_CTAS 8
#endif
#define SARR_CAND_BOUNDS __launch_bounds__(kBinThreads, SARR_CAND_MIN_CTAS)
template <bool kShadow, bool kStaged>
__global__ void SARR_CAND_BOUNDS bin_cand_kernel(const BinArgs a) {
  constexpr int kWarps = kBinThreads / 32;
  extern __shared__ int s_open[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int v = blockIdx.y;
  const SceneGrid& g = *a.grid;
  uint32_t* xbits = reinterpret_cast<uint32_t*>(a.ipp.base + v * a.ipp.vstride + a.ipp.L.xbits);
  if ((int)blockIdx.x < kCandBlocks) {
    const int nw = a.cand_count[v];
    // the same for the whole CTA (the staging below synchronises it)
    if (!g.valid || (int)blockIdx.x * kWarps >= nw) return;
    const int tsize = (a.views[v].tiles_x + 1) * (a.views[v].tiles_y + 1);
    if (kStaged)
      stage_open_tables(s_open, a.open_ipp + v * a.open_vstride, a.open_sh + v * a.open_vstride, tsize,
                        kShadow ? 2 : 1);
    const ViewConst vc = a.views[v];
    const int Nr = vc.h.Nr, Na = vc.h.Na, pitch = vc.tiles_x + 1;
    const int* open_ipp = a.open_ipp + v * a.open_vstride;
    const int* open_sh = a.open_sh + v * a.open_vstride;
    const uint32_t* words = a.cand_words + v * a.cand_vstride;
    for (int q = blockIdx.x * kWarps + warp; q < nw; q += kCandBlocks * kWarps) {
      const int word = (int)words[q];
      const uint32_t cand = a.bits[v * a.bits_vstride + word];
      // the members of the word's candidate cells, concatenated, 32 per round:
      // member p of the concatenation belongs to the first lane (cell) whose
      // inclusive member prefix exceeds p
      const int c_l = word * 32 + lane;
      const bool set = (cand >> lane) & 1u;
      const int start_l = set ? a.cell_start[c_l] : 0;
      const int cnt_l = set ? a.cell_start[c_l + 1] - start_l : 0;
      const int incl_l = warp_incl_scan(cnt_l, lane);
      const int total = __shfl_sync(0xffffffffu, incl_l, 31);
      for (int p0 = 0; p0 < total; p0 += 32) {
        const int p = p0 + lane;
        int lo = 0, hi = 31;  // first lane with incl > p
#pragma unroll
        for (int it = 0; it < 5; ++it) {
          const int mid = (lo + hi) >> 1;
          const int im = __shfl_sync(0xffffffffu, incl_l, mid);
          if (im > p) hi = mid; else lo = mid + 1;
        }
        const int owner_start = __shfl_sync(0xffffffffu, start_l, lo);
        const int owner_excl = __shfl_sync(0xffffffffu, incl_l - cnt_l, lo);
        if (p < total) {
          const int m = owner_start + (p - owner_excl);
          const float4 p4 = a.mem_pos[m];
          float r, cc, xr, yr;
          approx_center(vc, p4.x, p4.y, p4.z, r, cc, xr, yr);
          const float h = p4.w + vc.center_margin;
          const uint32_t ri = bound_rect(r, cc, h, Nr, Na);
          bool exact = (kStaged ? open_in_rect_s(ri, s_open, pitch) : open_in_rect(ri, open_ipp, pitch)) != 0;
          if (kShadow && !exact) {
            const uint32_t rs = bound_rect(yr, xr, h, Nr, Na);
            exact = (kStaged ? open_in_rect_s(rs, s_open + tsize, pitch) : open_in_rect(rs, open_sh, pitch)) != 0;
          }
          if (exact) {
            const int j = a.mem_idx[m];
            atomicOr(xbits + (j >> 5), 1u << (j & 31));
          }
        }
      }
    }
  } else {
    const int nwarps = (gridDim.x - kCandBlocks) * kWarps;
    const int na = g.n_always;
    for (int i = ((blockIdx.x - kCandBlocks) * kWarps + warp) * 32 + lane; i < na; i += nwarps * 32) {
      const int j = a.always[i];
      atomicOr(xbits + (j >> 5), 1u << (j & 31));
    }
  }
}

// Cell binning, part 2: one warp per (view, chunk after the prefix). The
// Gaussians whose bits are set are listed in index order and binned exactly
// (32 lanes at a time), and the chunk's tile counts are written.
// 40 registers for 6 CTAs per SM (1.06 -> 1.05 ms per 1024 sweep views;
// 32 registers spill more than the occupancy gains)
#ifndef SARR_FIN_MIN_CTAS
#define SARR_FIN_MIN_CTAS 6
#endif
#define SARR_FIN_BOUNDS __launch_bounds__(kBinThreads, SARR_FIN_MIN_CTAS)
template <bool kShadow>
__global__ void SARR_FIN_BOUNDS bin_finalize_kernel(const BinArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int kWarps = kBinThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int v = blockIdx.y;
  const int tiles_x = a.views[0].tiles_x, tiles_y = a.views[0].tiles_y, T = tiles_x * tiles_y;
  const int TW = (T + 1) >> 1;
  const int cs = a.cov_layout;
  uint32_t* s_cnt = reinterpret_cast<uint32_t*>(smem_raw) + warp * TW * (kShadow ? 2 : 1);
  uint32_t* s_cnt_sh = s_cnt + TW;
  const bool masks = a.skip_masks != 0;
  uint32_t* s_mask = reinterpret_cast<uint32_t*>(smem_raw) + kWarps * TW * (kShadow ? 2 : 1) +
                     warp * T * (kShadow ? 2 : 1);
  uint32_t* s_mask_sh = s_mask + T;
  const int k = blockIdx.x * kWarps + warp;
  if (k >= a.chunks) return;
  const int chunk = a.chunk_offset + k;
  const int64_t base = (int64_t)chunk * kChunk;
  const int gcount = (int)min((int64_t)kChunk, a.n - base);
  const ViewConst& vg = a.views[v];

  for (int i = lane; i < TW * (kShadow ? 2 : 1); i += 32) s_cnt[i] = 0;
  if (masks)
    for (int i = lane; i < T * (kShadow ? 2 : 1); i += 32) s_mask[i] = 0;
  const uint32_t* xbits = reinterpret_cast<const uint32_t*>(a.ipp.base + v * a.ipp.vstride + a.ipp.L.xbits);
  const uint32_t word = base + lane * 32 < a.n ? xbits[(size_t)chunk * 32 + lane] : 0u;
  const int cnt = __popc(word);
  const int excl = warp_incl_scan(cnt, lane) - cnt;
  const int total = __shfl_sync(0xffffffffu, excl + cnt, 31);
  uint16_t* xl = x_list(a, v, chunk);
  if (lane == 0) x_count(a, v)[chunk] = total;
  reinterpret_cast<uint16_t*>(a.ipp.base + v * a.ipp.vstride + a.ipp.L.xoff)[(size_t)chunk * 32 + lane] =
      (uint16_t)excl;
  {
    uint32_t wbits = word;
    int pos = excl;
    while (wbits) {
      xl[pos++] = (uint16_t)(lane * 32 + __ffs(wbits) - 1);
      wbits &= wbits - 1;
    }
  }
  __syncwarp();

  uint32_t* rects_ipp = reinterpret_cast<uint32_t*>(a.ipp.base + v * a.ipp.vstride + a.ipp.L.rects) + base;
  uint32_t* rects_sh =
      kShadow ? reinterpret_cast<uint32_t*>(a.sh.base + v * a.sh.vstride + a.sh.L.rects) + base : nullptr;
  const float* means = a.means + base * 3;
  const float* cov = a.cov + base * cs;
  // the chunk is sparse: the listed Gaussians' rectangles are stored
  // compactly from its first slot, in list order
  for (int i = lane; i < total; i += 32) {
    const int jl = xl[i];
    uint32_t rc_ipp = kEmptyRect, rc_sh = kEmptyRect;
    bin_exact<kShadow>(vg, means, cov, cs, jl, rc_ipp, rc_sh);
    rects_ipp[i] = rc_ipp;
    count_mark_rect<true>(s_cnt, masks ? s_mask : nullptr, rc_ipp, tiles_x, 1u << (jl >> 5));
    if (kShadow) {
      rects_sh[i] = rc_sh;
      count_mark_rect<true>(s_cnt_sh, masks ? s_mask_sh : nullptr, rc_sh, tiles_x, 1u << (jl >> 5));
    }
  }
  // the other Gaussians' rectangles are left unwritten: the state's meta and
  // exactness bits mark them empty
  __syncwarp();
  flush_counts(s_cnt, a.counts_ipp + v * a.counts_vstride + (size_t)chunk * T, T, lane);
  if (kShadow) flush_counts(s_cnt_sh, a.counts_sh + v * a.counts_vstride + (size_t)chunk * T, T, lane);
  if (masks) {
    flush_masks(s_mask, a.segmask + v * a.segmask_vstride + (size_t)chunk * T, T, lane);
    if (kShadow) flush_masks(s_mask_sh, a.segmask_sh + v * a.segmask_vstride + (size_t)chunk * T, T, lane);
  }
}

// Open-tile summed-area table of one list of one view (grid: views x lists).
// A tile is open while the first `prefix_chunks` chunk rows hold fewer than 64
// of its hits; entry [y][x] of the table counts the open tiles (ty, tx) with
// ty < y and tx < x. Built in shared memory with warp scans when it fits
// (kOpenSmemInts), in global memory otherwise.
constexpr int kOpenSmemInts = 8192;

__global__ void __launch_bounds__(256) open_table_kernel(const OpenArgs a) {
  __shared__ int s_tab[kOpenSmemInts];
  const int v = blockIdx.x, list = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tiles_x = a.tiles_x, tiles_y = a.tiles_y, T = tiles_x * tiles_y, pitch = tiles_x + 1;
  if (a.cand_count && list == 0 && tid == 0) a.cand_count[v] = 0;
  const int size = (tiles_y + 1) * pitch;
  const uint8_t* counts = (list ? a.counts[1] : a.counts[0]) + v * a.counts_vstride;
  int* out = (list ? a.table[1] : a.table[0]) + v * a.table_vstride;
  int* tab = size <= kOpenSmemInts ? s_tab : out;
  for (int x = tid; x < pitch; x += 256) tab[x] = 0;
  for (int y = tid; y < tiles_y; y += 256) tab[(y + 1) * pitch] = 0;
  for (int t = tid; t < T; t += 256) {
    int sum = 0;
    // sixteen chunks' counts in flight per step (only sum < kCap matters, and
    // the sum only grows)
    for (int c0 = 0; c0 < a.prefix_chunks && sum < kCap; c0 += 16) {
      int cv[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) cv[u] = c0 + u < a.prefix_chunks ? counts[(size_t)(c0 + u) * T + t] : 0;
#pragma unroll
      for (int u = 0; u < 16; ++u) sum += cv[u];
    }
    const int y = t / tiles_x, x = t - y * tiles_x;
    tab[(y + 1) * pitch + x + 1] = sum < kCap ? 1 : 0;
  }
  __syncthreads();
  // rows: one warp per row, 32 columns per step
  for (int y = warp; y < tiles_y; y += 8) {
    int* row = tab + (y + 1) * pitch + 1;
    int carry = 0;
    for (int x0 = 0; x0 < tiles_x; x0 += 32) {
      const int x = x0 + lane;
      const int val = x < tiles_x ? row[x] : 0;
      const int incl = warp_incl_scan(val, lane) + carry;
      if (x < tiles_x) row[x] = incl;
      carry = __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  __syncthreads();
  // columns: one warp per column
  for (int x = warp; x < tiles_x; x += 8) {
    int carry = 0;
    for (int y0 = 0; y0 < tiles_y; y0 += 32) {
      const int y = y0 + lane;
      int* e = tab + (y + 1) * pitch + x + 1;
      const int val = y < tiles_y ? *e : 0;
      const int incl = warp_incl_scan(val, lane) + carry;
      if (y < tiles_y) *e = incl;
      carry = __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  if (tab == s_tab) {
    __syncthreads();
    for (int i = tid; i < size; i += 256) out[i] = s_tab[i];
  }
}

// Per-tile prefix of the chunk counts, coalesced: one CTA per 32 adjacent
// tiles (lane = tile), each warp summing a contiguous range of chunk rows.
// Emits, per tile, the chunks that hold its first 64 hits in index order as
// (chunk, hits before the chunk, hits in the chunk) and the list length.
__global__ void __launch_bounds__(kScan1Threads) scan_kernel(const ScanArgs a) {
  __shared__ int s_part[kScan1Threads / 32][32];
  __shared__ int s_nneed[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int v = blockIdx.y;
  const int T = a.T;
  const int t = blockIdx.x * 32 + lane;
  const bool live = t < T;
  const uint8_t* counts = a.counts + v * a.counts_vstride;
  const int C = a.C;
  const int per = (C + kScan1Threads / 32 - 1) / (kScan1Threads / 32);
  const int c0 = min(warp * per, C), c1 = min(c0 + per, C);
  int sum = 0;
  if (live)
#pragma unroll 8
    for (int c = c0; c < c1; ++c) sum += counts[(size_t)c * T + t];
  s_part[warp][lane] = sum;
  if (warp == 0) s_nneed[lane] = 0;
  __syncthreads();
  int pre = 0, total = 0;
#pragma unroll
  for (int w = 0; w < kScan1Threads / 32; ++w) {
    const int x = s_part[w][lane];
    pre += (w < warp) ? x : 0;
    total += x;
  }
  unsigned char* st = a.st.base + v * a.st.vstride;
  int4* need = reinterpret_cast<int4*>(a.need + v * a.need_vstride);
  if (live && pre < kCap) {
    // eight chunks' counts in flight per step
    for (int cb = c0; cb < c1 && pre < kCap; cb += 8) {
      int cv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) cv[u] = cb + u < c1 ? counts[(size_t)(cb + u) * T + t] : 0;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (cv[u] > 0 && pre < kCap) {
          const int q = atomicAdd(&s_nneed[lane], 1);
          need[(size_t)t * kCap + q] = make_int4(cb + u, pre, cv[u], 0);
        }
        pre += cv[u];
      }
    }
  }
  __syncthreads();
  if (warp == 0 && live) {
    reinterpret_cast<int*>(st + a.st.L.count)[t] = min(total, kCap);
    a.need_n[v * a.need_n_vstride + t] = s_nneed[lane];
  }
}

// scan_kernel for tile counts that are a multiple of 4: a CTA takes 32
// adjacent tiles of one view, 8 lanes of a warp cover them with 4 tiles each
// (one 32-bit load of their u8 counts per chunk, a 32-byte sector per 8
// lanes), and the chunks are split into kScanSlices slices, four per warp
// (one per 8-lane group). Each slice's sums give every slice the hits before
// it; the slices that start below 64 hits then emit their need entries.
constexpr int kScanTilesPerLane = 4;
constexpr int kScanTilesPerCta = 8 * kScanTilesPerLane;
constexpr int kScanSlices = kScanThreads / 8;

// 40 registers for 3 CTAs (48 warps) per SM: the chunk-row loads are
// latency-bound (0.31 -> 0.24 ms per 1024 sweep views against 42 registers)
#ifndef SARR_SCAN_MIN_CTAS
#define SARR_SCAN_MIN_CTAS 3
#endif
#define SARR_SCAN_BOUNDS __launch_bounds__(kScanThreads, SARR_SCAN_MIN_CTAS)
__global__ void SARR_SCAN_BOUNDS scan4_kernel(const ScanArgs a) {
  __shared__ __align__(16) int s_part[kScanSlices][kScanTilesPerCta];
  __shared__ int s_nneed[kScanTilesPerCta];
  __shared__ __align__(16) int s_total[kScanTilesPerCta];
  const int tid = threadIdx.x, grp = tid & 7, slice = tid >> 3;
  const int v = blockIdx.y;
  const int T = a.T, C = a.C;
  const int tb = blockIdx.x * kScanTilesPerCta + kScanTilesPerLane * grp;  // the lane's first tile
  const bool live = tb < T;
  const uint8_t* counts = a.counts + v * a.counts_vstride;
  const int per = (C + kScanSlices - 1) / kScanSlices;
  const int c0 = min(slice * per, C), c1 = min(c0 + per, C);
  int sum[4] = {0, 0, 0, 0};
  if (live)
#pragma unroll 8
    for (int c = c0; c < c1; ++c) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(counts + (size_t)c * T + tb);
#pragma unroll
      for (int i = 0; i < 4; ++i) sum[i] += (w >> (8 * i)) & 0xFFu;
    }
  *reinterpret_cast<int4*>(&s_part[slice][kScanTilesPerLane * grp]) = make_int4(sum[0], sum[1], sum[2], sum[3]);
  if (tid < kScanTilesPerCta) s_nneed[tid] = 0;
  __syncthreads();
  // the slices' sums become the hits before each slice (one lane per tile)
  if (tid < kScanTilesPerCta) {
    int run = 0;
    for (int q = 0; q < kScanSlices; ++q) {
      const int x = s_part[q][tid];
      s_part[q][tid] = run;
      run += x;
    }
    s_total[tid] = run;
  }
  __syncthreads();
  int pre[4], total[4];
  {
    const int4 x = *reinterpret_cast<const int4*>(&s_part[slice][kScanTilesPerLane * grp]);
    const int4 y = *reinterpret_cast<const int4*>(&s_total[kScanTilesPerLane * grp]);
    pre[0] = x.x, pre[1] = x.y, pre[2] = x.z, pre[3] = x.w;
    total[0] = y.x, total[1] = y.y, total[2] = y.z, total[3] = y.w;
  }
  unsigned char* st = a.st.base + v * a.st.vstride;
  int4* need = reinterpret_cast<int4*>(a.need + v * a.need_vstride);
  auto open = [&]() {
    bool o = false;
#pragma unroll
    for (int i = 0; i < 4; ++i) o = o || pre[i] < kCap;
    return o;
  };
  if (live && open()) {
    // four chunks' words in flight per step
    for (int cb = c0; cb < c1 && open(); cb += 4) {
      uint32_t wv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        wv[u] = cb + u < c1 ? *reinterpret_cast<const uint32_t*>(counts + (size_t)(cb + u) * T + tb) : 0u;
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int cnt = (int)((wv[u] >> (8 * i)) & 0xFFu);
          if (cnt > 0 && pre[i] < kCap) {
            const int q = atomicAdd(&s_nneed[kScanTilesPerLane * grp + i], 1);
            need[(size_t)(tb + i) * kCap + q] = make_int4(cb + u, pre[i], cnt, 0);
          }
          pre[i] += cnt;
        }
    }
  }
  __syncthreads();
  if (slice == 0 && live) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      reinterpret_cast<int*>(st + a.st.L.count)[tb + i] = min(total[i], kCap);
      a.need_n[v * a.need_n_vstride + tb + i] = s_nneed[kScanTilesPerLane * grp + i];
    }
  }
}

// ---------------------------------------------------------------------------
// capped tile selection + tile records
// ---------------------------------------------------------------------------
// The 48-byte record of list slot `slot` of tile t: the listed Gaussian
// projected again in full (SH scattering only for the image list), its
// density constants, transmittance, Z_r, Y_r and slot; the image list also
// stores (Y_r, Z_r) for the backward (kStateYz). Returns Z_r. A list id
// outside [0, n) (only a corrupted workspace can produce one) is reported and
// replaced by 0.
template <bool kShadowList, bool kStateYz = true>
__device__ __forceinline__ float select_record(const SelectArgs& a, const ViewConst& vc,
                                               unsigned char* st, int t, int slot, int* list,
                                               Rec& g) {
  int id = list[slot];
  if (id < 0 || (int64_t)id >= a.n) {
    atomicOr(a.err, kDevErrListSlot);
    id = 0;
    list[slot] = 0;
  }
  float cw[6];
  load_cov6(a.cov + (size_t)id * a.cov_layout, a.cov_layout, cw);
  const float* m = a.means + (size_t)id * 3;
  Proj o;
  project_gaussian(vc, m[0], m[1], m[2], cw, o);
  if (!kShadowList) {
    g.mx = o.c;
    g.my = o.r;
    g.cxx = o.cov_cc;
    g.cxy = o.cov_rc;
    g.cyy = o.cov_rr;
    g.s_pos = fmaxf(0.0f, sh_scattering(vc, a.sh + (size_t)id * a.sh_stride, a.sh_k));
  } else {
    g.mx = o.xr;
    g.my = o.yr;
    g.cxx = o.XX;
    g.cxy = o.XY;
    g.cyy = o.YY;
    g.s_pos = 0.0f;
  }
  rec_density_consts(g);
  g.sigma = a.sigma[id];
  g.z = o.zr;
  g.yr = o.yr;
  g.pos = slot;
  if (!kShadowList && kStateYz) {
    float2* yz = reinterpret_cast<float2*>(st + a.st.L.yz);
    yz[(size_t)t * kCap + slot] = make_float2(o.yr, o.zr);
  }
  return o.zr;
}

// Ranks of `count` slots by (Z_r, slot) into rank_out[slot] when some Z_r is
// NaN: the reference's stable insertion sort on Z_r with strict '>'
// (:795-807) replayed by one thread.
__device__ __forceinline__ void insertion_ranks(const float* z, int count, int* rank_out) {
  int idx[kCap];
  float zv[kCap];
  for (int i = 0; i < count; ++i) {
    idx[i] = i;
    zv[i] = z[i];
  }
  for (int i = 1; i < count; ++i) {
    const int ti = idx[i];
    const float tz = zv[i];
    int j = i - 1;
    while (j >= 0 && zv[j] > tz) {
      idx[j + 1] = idx[j];
      zv[j + 1] = zv[j];
      j--;
    }
    idx[j + 1] = ti;
    zv[j + 1] = tz;
  }
  for (int k = 0; k < count; ++k) rank_out[idx[k]] = k;
}

// Orderable 64-bit key of (Z_r, slot) for a Z_r that is not NaN: the
// float's bits mapped to an unsigned order (-0 taken as +0: the reference's
// comparisons treat them as equal), the slot in the low word; unused slots
// get the largest key.
__device__ __forceinline__ uint64_t zslot_key(float z, int slot, bool used) {
  if (!used) return ~0ull;
  const uint32_t u = __float_as_uint(z + 0.0f);
  const uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((uint64_t)k << 32) | (uint32_t)slot;
}

// Sorted positions of the keys of slots lane and lane + 32 (kN = 64) or of
// slot lane (kN = 32), by a bitonic sorting network across the warp: the
// element at position e = lane + 32 h is key[h]; e's partner in a
// compare-exchange stage (k, j) is e ^ j, in lane ^ j for j < 32 and in the
// same lane for j = 32. Each sorted position then writes its position into
// s_rank[slot]. Keys are distinct (the slot is part of the key).
template <int kN>
__device__ __forceinline__ void warp_sort_ranks(uint64_t key0, uint64_t key1, int lane, int* s_rank) {
  uint64_t key[2] = {key0, key1};
#pragma unroll
  for (int k = 2; k <= kN; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j == 32) {
        const uint64_t lo = key[0] < key[1] ? key[0] : key[1];
        const uint64_t hi = key[0] < key[1] ? key[1] : key[0];
        key[0] = lo;
        key[1] = hi;
      } else {
#pragma unroll
        for (int h = 0; h < kN / 32; ++h) {
          const int e = lane + 32 * h;
          const uint64_t other = __shfl_xor_sync(0xffffffffu, key[h], j);
          const bool take_min = ((e & k) == 0) == ((lane & j) == 0);
          const bool smaller = other < key[h];
          key[h] = (take_min == smaller) ? other : key[h];
        }
      }
    }
  }
#pragma unroll
  for (int h = 0; h < kN / 32; ++h)
    if (key[h] != ~0ull) s_rank[(uint32_t)key[h]] = lane + 32 * h;
}

// Need entries of tile t taken by one warp: q = q0 + qs i, i = 0, 1, ...
// (qs = 1: every entry; qs = 2: one of two warps' share). Lane l holds
// entries i = l and i = l + 32, each with its chunk's exact-list length or
// segment mask in aux (-1: neither). kAllMasks: every chunk has segment
// masks (the per-view path).
struct NeedRegs {
  int4 nd[2];
  int aux[2];
};

template <bool kAllMasks>
__device__ __forceinline__ NeedRegs prefetch_need(const SelectArgs& a, int v, int T, int t, int nneed,
                                                  int lane, int q0, int qs) {
  const int4* need = reinterpret_cast<const int4*>(a.need + v * a.need_vstride) + (size_t)t * kCap;
  const int* xcount = a.xcount ? reinterpret_cast<const int*>(
                                     reinterpret_cast<const unsigned char*>(a.xcount) + v * a.x_vstride)
                               : nullptr;
  NeedRegs r;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int q = q0 + qs * (lane + 32 * h);
    r.nd[h] = make_int4(0, 0, 0, 0);
    r.aux[h] = -1;
    if (q < nneed) {
      r.nd[h] = need[q];
      const int c = r.nd[h].x;
      if (!kAllMasks && xcount && c >= a.xlist_from)
        r.aux[h] = xcount[c];
      else if (a.segmask && c < a.segmask_to)
        r.aux[h] = (int)a.segmask[v * a.segmask_vstride + (size_t)c * T + t];
    }
  }
  return r;
}

// Emit of the need entries in `nr` (entries q0 + qs i of tile (tx, ty)) when
// the chunks after the prefix have exact lists or none: each entry's chunk
// fills list slots [hits before, hits before + needed) with its first
// Gaussians, in index order, whose rectangle holds the tile, taken from the
// chunk's exact list, its segment masks, or all of its rectangles. Warp-wide;
// entries fill disjoint slots, so warps may split them.
__device__ __forceinline__ void emit_entries(const SelectArgs& a, int v, const unsigned char* st,
                                             int t, int T, int tx, int ty, int nneed,
                                             const NeedRegs& nr, int q0, int qs, int* list, int lane,
                                             bool skip_hit_words = false) {
  const uint32_t* rects = reinterpret_cast<const uint32_t*>(st + a.st.L.rects);
  const unsigned lt_mask = (1u << lane) - 1u;
  // chunks from sparse_from on keep only their exactly binned Gaussians'
  // rectangles, compactly in list order (cell binning)
  const unsigned char* xsv = a.xs.base + v * a.xs.vstride;
  const int64_t sparse_from = *reinterpret_cast<const int64_t*>(xsv + a.xs.L.meta);
  for (int i = 0; q0 + qs * i < nneed; ++i) {
    const int hq = i >> 5, src = i & 31;
    int4 nd;
    nd.x = __shfl_sync(0xffffffffu, hq ? nr.nd[1].x : nr.nd[0].x, src);
    nd.y = __shfl_sync(0xffffffffu, hq ? nr.nd[1].y : nr.nd[0].y, src);
    nd.z = __shfl_sync(0xffffffffu, hq ? nr.nd[1].z : nr.nd[0].z, src);
    const int aux = __shfl_sync(0xffffffffu, hq ? nr.aux[1] : nr.aux[0], src);
    const int want = min(nd.z, kCap - nd.y);
    const int64_t b0 = (int64_t)nd.x * kChunk;
    if (a.hbits && a.segmask && nd.x < a.hbits_to && nd.x < a.segmask_to) {
      if (skip_hit_words) continue;  // taken by emit_hit_words
      // the chunk's hit words of the tile, lane r taking word r when the
      // segment mask (aux) marks it; their hits in order are the chunk's
      // hits in index order
      const uint32_t* hw = a.hbits + v * a.hbits_vstride + ((size_t)nd.x * T + t) * 32;
      const uint32_t w = (((uint32_t)aux >> lane) & 1u) ? hw[lane] : 0u;
      const int cnt = __popc(w);
      int rk = warp_incl_scan(cnt, lane) - cnt;
      uint32_t bits = w;
      const int jb = (int)b0 + 32 * lane;
      while (bits && rk < want) {
        list[nd.y + rk] = jb + __ffs(bits) - 1;
        bits &= bits - 1u;
        ++rk;
      }
      continue;
    }
    const int xc = (a.xcount && nd.x >= a.xlist_from) ? aux : -1;
    if (xc >= 0) {
      // only the chunk's exactly binned Gaussians can hit the tile
      const uint16_t* xl = reinterpret_cast<const uint16_t*>(
                               reinterpret_cast<const unsigned char*>(a.xlist) + v * a.x_vstride) +
                           (size_t)nd.x * kXCap;
      const bool compact = b0 >= sparse_from;
      int found = 0;
      for (int i0 = 0; i0 < xc && found < want; i0 += 32) {
        const int i = i0 + lane;
        bool hit = false;
        int j = 0;
        if (i < xc) {
          j = (int)b0 + xl[i];
          hit = rect_has(rects[compact ? b0 + i : j], tx, ty);
        }
        const unsigned m = __ballot_sync(0xffffffffu, hit);
        const int rk = found + __popc(m & lt_mask);
        if (hit && rk < want) list[nd.y + rk] = j;
        found += __popc(m);
      }
      continue;
    }
    const int valid = (int)min((int64_t)kChunk, a.n - b0);
    if (a.segmask && nd.x < a.segmask_to) {
      // only the 32-Gaussian segments that hold hits of the tile, four at a time
      uint32_t segs = (uint32_t)aux;
      int found = 0;
      while (segs && found < want) {
        int sj[4];
        uint32_t rc[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          sj[u] = -1;
          if (segs) {
            sj[u] = (__ffs(segs) - 1) * 32 + lane;
            segs &= segs - 1;
          }
          rc[u] = (sj[u] >= 0 && sj[u] < valid) ? rects[b0 + sj[u]] : kEmptyRect;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (found >= want) break;
          const bool hit = rect_has(rc[u], tx, ty);
          const unsigned m = __ballot_sync(0xffffffffu, hit);
          const int rk = found + __popc(m & lt_mask);
          if (hit && rk < want) list[nd.y + rk] = (int)b0 + sj[u];
          found += __popc(m);
        }
      }
      continue;
    }
    uint4 r4[kChunk / 128];
#pragma unroll
    for (int k = 0; k < kChunk / 128; ++k) {
      const int j = k * 128 + 4 * lane;
      if (j + 3 < valid) {
        r4[k] = __ldg(reinterpret_cast<const uint4*>(rects + b0 + j));
      } else {
        r4[k].x = j < valid ? rects[b0 + j] : kEmptyRect;
        r4[k].y = j + 1 < valid ? rects[b0 + j + 1] : kEmptyRect;
        r4[k].z = j + 2 < valid ? rects[b0 + j + 2] : kEmptyRect;
        r4[k].w = kEmptyRect;
      }
    }
    int found = 0;
#pragma unroll
    for (int k = 0; k < kChunk / 128; ++k) {
      if (found >= want) break;
      const bool h0 = rect_has(r4[k].x, tx, ty), h1 = rect_has(r4[k].y, tx, ty);
      const bool h2 = rect_has(r4[k].z, tx, ty), h3 = rect_has(r4[k].w, tx, ty);
      const int cnt = (int)h0 + (int)h1 + (int)h2 + (int)h3;
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int rk = found + incl - cnt;
      const int j = (int)b0 + k * 128 + 4 * lane;
      if (h0) { if (rk < want) list[nd.y + rk] = j; ++rk; }
      if (h1) { if (rk < want) list[nd.y + rk] = j + 1; ++rk; }
      if (h2) { if (rk < want) list[nd.y + rk] = j + 2; ++rk; }
      if (h3) { if (rk < want) list[nd.y + rk] = j + 3; }
      found += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
}

// The need entries of the chunks that have hit words (chunk < a.hbits_to,
// at most one entry per chunk), all together in chunk order: the pairs
// (chunk, marked segment) are taken 32 per round, one lane each, and a warp
// scan of the words' popcounts numbers the hits in index order. Entries of
// earlier chunks hold every hit before a later chunk's (scan_kernel emits
// entries only while fewer than 64 hits precede the chunk), so a hit's list
// slot is the number of hits before it. Warp-wide; nr holds the entries
// lane and lane + 32 (prefetch_need with q0 = 0, qs = 1).
__device__ __forceinline__ void emit_hit_words(const SelectArgs& a, int v, int t, int T, int nneed,
                                               const NeedRegs& nr, int* list, int lane) {
  const unsigned full = 0xffffffffu;
  // lane c: the segment mask of chunk c's entry (0: none)
  uint32_t mask = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const bool mine = lane + 32 * h < nneed && nr.nd[h].x < a.hbits_to;
    unsigned m = __ballot_sync(full, mine);
    while (m) {
      const int src = __ffs(m) - 1;
      m &= m - 1u;
      const int c = __shfl_sync(full, nr.nd[h].x, src);
      const uint32_t mk = (uint32_t)__shfl_sync(full, nr.aux[h], src);
      if (lane == c) mask = mk;
    }
  }
  const int nseg = __popc(mask);
  const int seg_incl = warp_incl_scan(nseg, lane);
  const int pairs = __shfl_sync(full, seg_incl, 31);
  const uint32_t* hw0 = a.hbits + v * a.hbits_vstride + (size_t)t * 32;
  const size_t chunk_stride = (size_t)T * 32;
  int carry = 0;  // hits numbered so far
  for (int p0 = 0; p0 < pairs && carry < kCap; p0 += 32) {
    const int p = p0 + lane;
    // the pair's chunk: the first lane whose inclusive segment count exceeds p
    int lo = 0, hi = 31;
#pragma unroll
    for (int it = 0; it < 5; ++it) {
      const int mid = (lo + hi) >> 1;
      if (__shfl_sync(full, seg_incl, mid) > p) hi = mid; else lo = mid + 1;
    }
    const int c = lo;
    const int k = p - (__shfl_sync(full, seg_incl, c) - __shfl_sync(full, nseg, c));
    uint32_t mm = __shfl_sync(full, mask, c);
    uint32_t w = 0;
    int r = 0;
    if (p < pairs) {
      for (int i = 0; i < k; ++i) mm &= mm - 1u;  // drop the chunk's first k marked segments
      r = __ffs(mm) - 1;
      w = hw0[c * chunk_stride + r];
    }
    const int cnt = __popc(w);
    const int incl = warp_incl_scan(cnt, lane);
    int rk = carry + incl - cnt;
    const int jb = c * kChunk + 32 * r;
    while (w && rk < kCap) {
      list[rk] = jb + __ffs(w) - 1;
      w &= w - 1u;
      ++rk;
    }
    carry += __shfl_sync(full, incl, 31);
  }
}

// One warp per tile (kSelectThreads / 32 tiles per CTA), no CTA barrier.
//  1. emit: every needed chunk's 1024 rectangles are loaded at once (eight
//     16-byte loads per lane) and its hits are ranked in index order with a
//     warp scan, filling list slots [hits before, hits before + needed);
//  2. the listed Gaussians (two slots per lane) are projected again in full
//     (SH only for them) into 48-byte records;
//  3. each slot's rank by (Z_r, slot) places its record.
template <bool kShadowList, bool kAllMasks>
__global__ void __launch_bounds__(kSelectThreads, 8) select_kernel(const SelectArgs a) {
  constexpr int kWarps = kSelectThreads / 32;
  __shared__ int s_list[kWarps][kCap];
  __shared__ float s_z[kWarps][kCap];
  __shared__ int s_rank[kWarps][kCap];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int v = blockIdx.y;
  const ViewConst& vc = a.views[v];
  const int tiles_x = vc.tiles_x, T = tiles_x * vc.tiles_y;
  const int t = blockIdx.x * kWarps + warp;
  if (t >= T) return;  // warp-uniform; nothing below synchronises the CTA
  const int tx = t % tiles_x, ty = t / tiles_x;
  unsigned char* st = a.st.base + v * a.st.vstride;
  const int count = reinterpret_cast<const int*>(st + a.st.L.count)[t];
  if (count == 0) return;
  const int nneed = a.need_n[v * a.need_n_vstride + t];
  int* list = s_list[warp];
  list[lane] = -1;
  list[lane + 32] = -1;
  __syncwarp();

  // 1. emit
  const NeedRegs nr = prefetch_need<kAllMasks>(a, v, T, t, nneed, lane, 0, 1);
  if constexpr (kAllMasks) {
    const uint32_t* rects = reinterpret_cast<const uint32_t*>(st + a.st.L.rects);
    const unsigned lt_mask = (1u << lane) - 1u;
    // Every chunk has segment masks: the (need entry, hit segment) pairs of
    // all entries, in order, kSelBatch per round with their rectangle loads
    // in flight together.
    constexpr int kSelBatch = 8;
    const unsigned full = 0xffffffffu;
    // (the per-view path keeps every rectangle at its Gaussian's slot)
    auto entry_mask = [&](int q) {
      return (uint32_t)__shfl_sync(full, q >= 32 ? nr.aux[1] : nr.aux[0], q & 31);
    };
    int eq = 0;                        // entry being enumerated
    uint32_t rem = entry_mask(0);      // its segments not yet enumerated
    int cur = -1, found = 0, want = 0, ny = 0;
    bool more = true;
    while (more) {
      uint32_t rc[kSelBatch];
      int jj[kSelBatch], qq[kSelBatch];
#pragma unroll
      for (int b = 0; b < kSelBatch; ++b) {
        while (rem == 0 && eq + 1 < nneed) rem = entry_mask(++eq);
        qq[b] = -1;
        jj[b] = 0;
        rc[b] = kEmptyRect;
        if (rem != 0) {
          const int seg = __ffs(rem) - 1;
          rem &= rem - 1;
          const int cq = __shfl_sync(full, eq >= 32 ? nr.nd[1].x : nr.nd[0].x, eq & 31);
          const int64_t jg = (int64_t)cq * kChunk + seg * 32 + lane;
          qq[b] = eq;
          jj[b] = (int)jg;
          if (jg < a.n) rc[b] = rects[jg];
        }
      }
      more = rem != 0 || eq + 1 < nneed;
#pragma unroll
      for (int b = 0; b < kSelBatch; ++b) {
        const int q = qq[b];
        if (q < 0) break;
        if (q != cur) {
          cur = q;
          found = 0;
          const bool h1 = q >= 32;
          ny = __shfl_sync(full, h1 ? nr.nd[1].y : nr.nd[0].y, q & 31);
          const int z = __shfl_sync(full, h1 ? nr.nd[1].z : nr.nd[0].z, q & 31);
          want = min(z, kCap - ny);
        }
        if (found >= want) continue;
        const bool hit = rect_has(rc[b], tx, ty);
        const unsigned m = __ballot_sync(full, hit);
        const int rk = found + __popc(m & lt_mask);
        if (hit && rk < want) list[ny + rk] = jj[b];
        found += __popc(m);
      }
    }
  } else {
    const bool hw = a.hbits != nullptr && a.segmask != nullptr;
    if (hw) emit_hit_words(a, v, t, T, nneed, nr, list, lane);
    emit_entries(a, v, st, t, T, tx, ty, nneed, nr, 0, 1, list, lane, hw);
  }
  __syncwarp();

  // 2. records of the listed Gaussians (slots lane and lane + 32)
  Rec rec[2];
  bool nan_z = false;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int slot = lane + 32 * h;
    if (slot < count) {
      const float zr = select_record<kShadowList>(a, vc, st, t, slot, list, rec[h]);
      s_z[warp][slot] = zr;
      nan_z = nan_z || (zr != zr);
    }
  }
  __syncwarp();

  // 3. rank by (Z_r, slot): equal to the reference's stable insertion sort on
  // Z_r with strict '>' (:795-807) whenever no Z_r is NaN; with a NaN the
  // insertion sort itself is replayed.
  int rank[2] = {0, 0};
  const float* z = s_z[warp];
  if (__any_sync(0xffffffffu, nan_z)) {
    if (lane == 0) insertion_ranks(z, count, s_rank[warp]);
    __syncwarp();
    rank[0] = s_rank[warp][lane];
    rank[1] = s_rank[warp][lane + 32];
  } else {
    // no NaN: the position of each slot's (Z_r, slot) key in sorted order
    int* sr = s_rank[warp];
    const uint64_t k0 = zslot_key(rec[0].z, lane, lane < count);
    if (count <= 32) {
      warp_sort_ranks<32>(k0, ~0ull, lane, sr);
    } else {
      warp_sort_ranks<64>(k0, zslot_key(rec[1].z, lane + 32, lane + 32 < count), lane, sr);
    }
    __syncwarp();
    rank[0] = sr[lane];
    rank[1] = sr[lane + 32];
  }

  // 4. state (the list length was written by scan_kernel)
  int* st_list = reinterpret_cast<int*>(st + a.st.L.list) + (size_t)t * kCap;
  Rec* st_recs = reinterpret_cast<Rec*>(st + a.st.L.recs) + (size_t)t * kCap;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int slot = lane + 32 * h;
    if (slot < count) {
      st_list[slot] = list[slot];
      st_recs[rank[h]] = rec[h];
    }
  }
}

// Few-view variant of select_kernel, for launches of fewer than
// kSelectCtaMaxViews views whose chunks all have segment masks and keep every
// rectangle at its Gaussian's slot (the per-view path): such a launch has
// only T tiles of work, so one 128-thread CTA takes each tile. Its four warps
// take the need entries in turn (each entry fills its own list slots), one
// thread per slot builds the records and two per slot count the ranks. The
// lists and records are select_kernel's.
constexpr int kSelectCtaMaxViews = 16;

template <bool kShadowList>
__global__ void __launch_bounds__(kSelectThreads) select_cta_kernel(const SelectArgs a) {
  constexpr int kWarps = kSelectThreads / 32;
  static_assert(kSelectThreads == 2 * kCap, "two threads per list slot for the ranks");
  __shared__ int s_list[kCap];
  __shared__ float s_z[kCap];
  __shared__ int s_rank[2][kCap];
  __shared__ int4 s_need[kCap];
  __shared__ uint32_t s_segs[kCap];
  __shared__ int s_nan;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int v = blockIdx.y, t = blockIdx.x;
  const ViewConst& vc = a.views[v];
  const int tiles_x = vc.tiles_x, T = tiles_x * vc.tiles_y;
  const int tx = t % tiles_x, ty = t / tiles_x;
  unsigned char* st = a.st.base + v * a.st.vstride;
  const int count = reinterpret_cast<const int*>(st + a.st.L.count)[t];
  if (count == 0) return;  // the same for the whole CTA
  const int nneed = a.need_n[v * a.need_n_vstride + t];
  const int4* need = reinterpret_cast<const int4*>(a.need + v * a.need_vstride) + (size_t)t * kCap;
  // the need entries and their chunks' segment masks, one thread each
  const uint32_t* masks = a.segmask + v * a.segmask_vstride;
  if (tid < kCap) {
    s_list[tid] = -1;
    if (tid < nneed) {
      const int4 nd = need[tid];
      s_need[tid] = nd;
      s_segs[tid] = masks[(size_t)nd.x * T + t];
    }
  }
  if (tid == 0) s_nan = 0;
  __syncthreads();

  // 1. emit: warp w takes need entries w, w + 4, ...; the hit segments of an
  // entry's chunk four at a time
  const uint32_t* rects = reinterpret_cast<const uint32_t*>(st + a.st.L.rects);
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int q = warp; q < nneed; q += kWarps) {
    const int4 nd = s_need[q];
    uint32_t segs = s_segs[q];
    const int want = min(nd.z, kCap - nd.y);
    const int64_t b0 = (int64_t)nd.x * kChunk;
    int found = 0;
    while (segs && found < want) {
      int64_t sj[4];
      uint32_t rc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        sj[u] = -1;
        if (segs) {
          sj[u] = b0 + (__ffs(segs) - 1) * 32 + lane;
          segs &= segs - 1;
        }
        rc[u] = (sj[u] >= 0 && sj[u] < a.n) ? rects[sj[u]] : kEmptyRect;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (found >= want) break;
        const bool hit = rect_has(rc[u], tx, ty);
        const unsigned m = __ballot_sync(0xffffffffu, hit);
        const int rk = found + __popc(m & lt_mask);
        if (hit && rk < want) s_list[nd.y + rk] = (int)sj[u];
        found += __popc(m);
      }
    }
  }
  __syncthreads();

  // 2. records: thread s builds slot s
  Rec g;
  if (tid < count) {
    const float zr = select_record<kShadowList>(a, vc, st, t, tid, s_list, g);
    s_z[tid] = zr;
    if (zr != zr) s_nan = 1;
  }
  __syncthreads();

  // 3. rank by (Z_r, slot) (see select_kernel): threads s and s + 64 count
  // the smaller keys among slots [0, 32) and [32, 64)
  const bool nan_z = s_nan != 0;
  if (nan_z) {
    if (tid == 0) insertion_ranks(s_z, count, s_rank[0]);
  } else {
    const int slot = tid & (kCap - 1), half = tid >> 6;
    if (slot < count) {
      const float zs = s_z[slot];
      int r = 0;
      const int j1 = min(count, 32 * half + 32);
      for (int j = 32 * half; j < j1; ++j) {
        const float zj = s_z[j];
        r += (zj < zs) || (zj == zs && j < slot);
      }
      s_rank[half][slot] = r;
    }
  }
  __syncthreads();

  // 4. state (the list length was written by scan_kernel)
  if (tid < count) {
    const int rank = nan_z ? s_rank[0][tid] : s_rank[0][tid] + s_rank[1][tid];
    reinterpret_cast<int*>(st + a.st.L.list)[(size_t)t * kCap + tid] = s_list[tid];
    (reinterpret_cast<Rec*>(st + a.st.L.recs) + (size_t)t * kCap)[rank] = g;
  }
}

// ---------------------------------------------------------------------------
// compositing
// ---------------------------------------------------------------------------
// Loads the `count` sorted records of tile t into shared memory with one TMA
// bulk copy. Every thread of the CTA must call it.
__device__ __forceinline__ bool load_tile_recs(Rec* s_rec, uint64_t* bar, const unsigned char* st,
                                               const StateLayout& L, int t, int count, int* err,
                                               bool whole_block) {
  if (threadIdx.x == 0) mbar_init(bar, 1);
  if (whole_block) __syncthreads(); else __syncwarp();
  if (threadIdx.x == 0) {
    const uint32_t bytes = (uint32_t)count * (uint32_t)sizeof(Rec);
    mbar_arrive_expect_tx(bar, bytes);
    tma_load_1d(s_rec, st + L.recs + (size_t)t * kCap * sizeof(Rec), bytes, bar);
  }
  return mbar_wait_bounded(bar, 0, err);
}

// Exponent cutoff of one record for compositing: a pixel whose exponent
// (compute_gaussian_density_2d's -q / (2 det)) is below it has a density
// below 1e-8, in the reference (expf within 2 ulp of exp, the CUDA math
// library's documented bound, and a correctly rounded division by norm) and
// in density_above_cutoff (within 2e-6 relative), and is skipped by the
// compositing, so the pixel may skip it without evaluating the exponential.
// The cutoff is max(-20, ln(1e-8 norm) - 1e-3): below -20 the reference's
// density is 0; below ln(1e-8 norm) - 1e-3 the exact exp is below
// 0.999e-8 norm, and the evaluation errors above and those of logf and of
// the product 1e-8f * norm (both below 1e-6 relative) keep the computed
// density below 1e-8. A NaN from logf leaves the cutoff at -20; an infinite
// norm gives +inf (density 0 or NaN -> 0 there).
__device__ __forceinline__ float density_cutoff(const Rec& g) {
  return fmaxf(-20.0f, logf(mul_(1e-8f, g.norm)) - 1e-3f);
}

// Half-widths (columns, rows) of the box outside which a record's exponent is
// below `cutoff` (< 0). The exponent is -q / (2 det) with
// q = cxx dy^2 + cyy dx^2 - 2 cxy dx dy, and q <= K det implies
// |dx| <= sqrt(K cxx), |dy| <= sqrt(K cyy). The box is taken for
// K = -2.04 cutoff (2 % on q) plus 0.01 px: for correlations
// |cxy| / sqrt(cxx cyy) <= 0.999 the float evaluation of q and det is within
// 0.04 % of exact, so the computed exponent stays below 1.019 cutoff < cutoff
// outside it. Other records: no box (density 0 everywhere when
// |det| < EPSILON; unbounded otherwise, or when cutoff >= -0.01).
__device__ __forceinline__ float2 density_extent(const Rec& g, float cutoff) {
  if (g.norm < 0.0f) return make_float2(-1.0f, -1.0f);
  const float cxx = g.cxx, cyy = g.cyy, cxy = g.cxy;
  const bool bounded = cxx > 0.0f && cyy > 0.0f && cxx < 1e30f && cyy < 1e30f && g.inv_det > 0.0f &&
                       cxy * cxy <= 0.998f * (cxx * cyy) && cutoff < -0.01f;
  if (!bounded) return make_float2(INFINITY, INFINITY);
  const float k = -2.04f * cutoff;
  return make_float2(sqrtf(k * cxx) + 0.01f, sqrtf(k * cyy) + 0.01f);
}

// 2^x with PTX's ex2.approx (relative error below 2^-22 over the range used
// here; subnormal results flushed to zero, which only affects densities far
// below the 1e-8 cut-off).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// -log2(norm) of a record: compute_gaussian_density_2d's division by norm
// becomes an addition to the base-2 exponent.
__device__ __forceinline__ float density_log2_scale(const Rec& g) { return -log2f(g.norm); }

// The exponent of compute_gaussian_density_2d (:215-234) at pixel (px, py),
// evaluated with the reference's operations (so the cut-off boxes of
// density_extent, derived for this evaluation, hold).
__device__ __forceinline__ float density_exponent(const Rec& g, float px, float py) {
  const float dx = sub_(px, g.mx);
  const float dy = sub_(py, g.my);
  const float q = fma_(mul_(g.cxx, dy), dy,
                       fma_(mul_(g.cyy, dx), dx, -mul_(mul_(mul_(2.0f, g.cxy), dx), dy)));
  return mul_(mul_(-0.5f, q), g.inv_det);
}

// compute_gaussian_density_2d of a record whose norm is >= 0 at pixel
// (px, py): exp(exponent) / norm evaluated as 2^(exponent log2(e) -
// log2(norm)) with one ex2.approx (`l2s` = density_log2_scale(g)); relative
// error below 2e-6 against the correctly rounded value for exponents >= -20
// (the fma's rounding of a product below 29 in magnitude, and ex2's own
// error). 0 where the exponent is below the record's cutoff (there the
// reference's density is below 1e-8, and every caller treats such a density
// as no contribution) and where it is NaN (the reference's fmaxf(NaN, 0)).
// Records with norm < 0 have an empty cutoff box and reach no caller.
__device__ __forceinline__ float density_above_cutoff(const Rec& g, float cutoff, float l2s,
                                                      float px, float py) {
  const float exponent = density_exponent(g, px, py);
  if (exponent < cutoff) return 0.0f;
  return fmaxf(ex2_approx(__fmaf_rn(exponent, 1.4426950408889634f, l2s)), 0.0f);
}

// Marks, for the records of one tile (lanes hold records lane and lane + 32),
// those whose cutoff box meets the pixel block [bx0, bx1] x [by0, by1]
// (columns x rows), and stores every record's cutoff and log2 scale in cut[].
// Warp-wide.
__device__ __forceinline__ uint64_t block_hits(const Rec* recs, int count, float2* cut, float bx0,
                                               float bx1, float by0, float by1, int lane) {
  uint64_t hit = 0;
  for (int h = 0; h < (count > 32 ? 2 : 1); ++h) {
    const int k = lane + 32 * h;
    bool in = false;
    if (k < count) {
      const Rec& g = recs[k];
      const float cutoff = density_cutoff(g);
      cut[k] = make_float2(cutoff, density_log2_scale(g));
      const float2 e = density_extent(g, cutoff);
      const float mdx = fmaxf(0.0f, fmaxf(bx0 - g.mx, g.mx - bx1));
      const float mdy = fmaxf(0.0f, fmaxf(by0 - g.my, g.my - by1));
      in = !(mdx > e.x) && !(mdy > e.y);
    }
    hit |= (uint64_t)__ballot_sync(0xffffffffu, in) << (32 * h);
  }
  return hit;
}

// hit[i] bit k: record k's cutoff box meets columns [c0 + 4i, c0 + 4i + 3]
// of rows [r0, r0 + 7]; cut[k] receives record k's cutoff and log2 scale.
// Warp-wide; ends with __syncwarp.
template <int kPix>
__device__ __forceinline__ void quarter_hits(const Rec* s_rec, float2* cut, int count, int r0, int c0,
                                             int lane, uint64_t (&hit)[kPix]) {
#pragma unroll
  for (int i = 0; i < kPix; ++i) hit[i] = 0;
  const float by0 = (float)r0, by1 = (float)(r0 + 7);
  for (int h = 0; h < (count > 32 ? 2 : 1); ++h) {
    const int k = lane + 32 * h;
    bool in[kPix];
#pragma unroll
    for (int i = 0; i < kPix; ++i) in[i] = false;
    if (k < count) {
      const Rec& g = s_rec[k];
      const float cutoff = density_cutoff(g);
      cut[k] = make_float2(cutoff, density_log2_scale(g));
      const float2 e = density_extent(g, cutoff);
      const float mdy = fmaxf(0.0f, fmaxf(by0 - g.my, g.my - by1));
      if (!(mdy > e.y)) {
#pragma unroll
        for (int i = 0; i < kPix; ++i) {
          const float hx0 = (float)(c0 + 4 * i), hx1 = hx0 + 3.0f;
          const float mdx = fmaxf(0.0f, fmaxf(hx0 - g.mx, g.mx - hx1));
          in[i] = !(mdx > e.x);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kPix; ++i)
      hit[i] |= (uint64_t)__ballot_sync(0xffffffffu, in[i]) << (32 * h);
  }
  __syncwarp();
}

// Compositing of one warp's 8 x (4 kPix) pixel block (rows r0 .. r0 + 7,
// columns c0 .. c0 + 4 kPix - 1; the lane's row pr and first column pc0)
// from the tile's `count` sorted records in shared memory, into the lane's
// value / trans / done; `cut` is the warp's scratch for the records' cutoffs.
// Warp-wide.
template <int kPix>
__device__ __forceinline__ void composite_block(const Rec* s_rec, float2* cut, int count, int r0,
                                                int c0, int pr, int pc0, int lane,
                                                float (&value)[kPix], float (&trans)[kPix],
                                                bool (&done)[kPix]) {
  uint64_t hit[kPix];
  quarter_hits<kPix>(s_rec, cut, count, r0, c0, lane, hit);
  // Records in two passes of 32 (32-bit masks): the lane visits, in list
  // order, the records marked for any of its pixels, and each pixel takes
  // those marked for its quarter. A pixel whose transmittance ran out drops
  // its mask (and the lane's pending records are narrowed to the others').
  // A density that is NaN or below 1e-8 (the reference's gamma < 1e-8 skip,
  // and its fmaxf(NaN, 0)) contributes nothing.
  const float fy = (float)pr;
  const float4* recs4 = reinterpret_cast<const float4*>(s_rec);
  float px[kPix];
#pragma unroll
  for (int i = 0; i < kPix; ++i) px[i] = (float)(pc0 + 4 * i);
  for (int h = 0; h < (count > 32 ? 2 : 1); ++h) {
    uint32_t m[kPix];
    uint32_t todo = 0;
#pragma unroll
    for (int i = 0; i < kPix; ++i) {
      m[i] = done[i] ? 0u : (uint32_t)(hit[i] >> (32 * h));
      todo |= m[i];
    }
    while (todo) {
      const int kk = __ffs(todo) - 1;
      todo &= todo - 1u;
      const int k = 32 * h + kk;
      // mx my cxx cxy | cyy inv_det norm sigma | s_pos z yr pos
      const float4 ra = recs4[3 * k], rb = recs4[3 * k + 1], rc = recs4[3 * k + 2];
      const float2 c = cut[k];
      // the row's part of compute_gaussian_density_2d's quadratic form,
      // shared by the lane's pixels (same range row)
      const float dy = sub_(fy, ra.y);
      const float qy = mul_(ra.z, dy);     // cxx * dy
      const float cxy2 = mul_(2.0f, ra.w);
      // (-0.5 q) inv_det and q (-0.5 inv_det) are the same rounding of the
      // same exact product (-0.5 is a power of two) unless a factor is
      // subnormal
      const float nh_inv_det = mul_(-0.5f, rb.y);
#pragma unroll
      for (int i = 0; i < kPix; ++i) {
        if ((m[i] >> kk) & 1u) {
          const float dx = sub_(px[i], ra.x);
          const float q = fma_(qy, dy, fma_(mul_(rb.x, dx), dx, -mul_(mul_(cxy2, dx), dy)));
          const float exponent = mul_(q, nh_inv_det);
          if (!(exponent < c.x)) {
            const float gamma_ipp = ex2_approx(__fmaf_rn(exponent, 1.4426950408889634f, c.y));
            if (gamma_ipp >= 1e-8f) {
              const float sigma = rb.w;
              const float alpha_i = mul_(sigma, gamma_ipp);
              value[i] = fma_(mul_(trans[i], alpha_i), rc.x, value[i]);
              trans[i] = mul_(trans[i], fma_(-sigma, gamma_ipp, 1.0f));
            }
          }
        }
      }
      // a pixel whose transmittance fell below 1e-8 at this record takes no
      // later record (the reference's break after the update); each pixel
      // meets the record once, so one test per record suffices. A finished
      // pixel's transmittance is set to 1 (it is not read again: its mask is
      // cleared), which keeps it out of later tests.
      float tmin = trans[0];
#pragma unroll
      for (int i = 1; i < kPix; ++i) tmin = fminf(tmin, trans[i]);
      if (tmin < 1e-8f) {
#pragma unroll
        for (int i = 0; i < kPix; ++i) {
          if (trans[i] < 1e-8f) {
            trans[i] = 1.0f;
            done[i] = true;
            m[i] = 0u;
          }
        }
        uint32_t keep = 0;
#pragma unroll
        for (int j = 0; j < kPix; ++j) keep |= m[j];
        todo &= keep;
      }
    }
  }
}

// One CTA per tile: the tile's sorted records arrive with one TMA bulk copy;
// warp w composites an 8 x (4 kPix) pixel block, each lane kPix pixels of one
// range row (azimuth columns c, c + 4; lanes along range, contiguous in the
// image). Before compositing, each warp marks, per 8 x 4 half of its block,
// the records whose cutoff box (density_extent) meets that half (one bit per
// record, two ballots): every pixel outside a record's box is skipped by the
// compositing, so visiting only the marked records, in list order, leaves
// each pixel's arithmetic the reference's, record by record.
//
// kPix pixels per lane: 4 for launches of many views (2 warps per tile, each
// an 8 x 16 block: the per-record overheads spread over four pixels; 1.62 ->
// 1.51 ms per 1024 views against 2 pixels), 1 for a few views (8 warps per
// tile, more warps in flight when the grid is small).
template <int kPix>
__global__ void __launch_bounds__(kTile * kTile / kPix) render_kernel(const TileArgs a) {
  constexpr int kWarps = kTile * kTile / kPix / 32;
  __shared__ __align__(16) Rec s_rec[kCap];
  __shared__ float2 s_cut[kWarps][kCap];
  __shared__ uint64_t bar;
  const int v = blockIdx.y, t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ViewConst& vc = a.views[v];
  const int Nr = vc.h.Nr, Na = vc.h.Na, tiles_x = vc.tiles_x;
  const int tx = t % tiles_x, ty = t / tiles_x;
  // warp block: 8 range rows x (4 * kPix) azimuth columns
  const int r0 = ty * kTile + (warp & 1) * 8, c0 = tx * kTile + (warp >> 1) * 4 * kPix;
  const int pr = r0 + (lane & 7), pc0 = c0 + (lane >> 3);
  const unsigned char* st = a.st.base + v * a.st.vstride;
  const int count = reinterpret_cast<const int*>(st + a.st.L.count)[t];

  float value[kPix], trans[kPix];
  bool done[kPix];
#pragma unroll
  for (int i = 0; i < kPix; ++i) {
    value[i] = 0.0f;
    trans[i] = 1.0f;
    done[i] = false;
  }
  if (count > 0) {
    const bool ok = load_tile_recs(s_rec, &bar, st, a.st.L, t, count, a.err, true);
    if (__syncthreads_and(ok))
      composite_block<kPix>(s_rec, s_cut[warp], count, r0, c0, pr, pc0, lane, value, trans, done);
  }
  float* img = a.images + v * a.img_vstride;
  if (pr < Nr) {
#pragma unroll
    for (int i = 0; i < kPix; ++i)
      if (pc0 + 4 * i < Na) img[(size_t)(pc0 + 4 * i) * Nr + pr] = value[i];
  }
}

// Image-only launches of many views: select_kernel's selection and
// render_kernel<4>'s compositing of one tile in one CTA of two warps, the
// tile's list and records kept in shared memory (neither is written to the
// state). Warp w emits need entries w, w + 2, ... (entries fill disjoint list
// slots); thread s builds the record of list slot s; each warp ranks all
// slots by (Z_r, slot) and places its own slots' records; then each warp
// composites its 8 x 16 pixel block as render_kernel<4> does. The records
// and the image equal select_kernel's and render_kernel<4>'s. On one SM the
// dependent gathers of some CTAs' selection overlap other CTAs' compositing.
constexpr int kFusedPix = 4;
constexpr int kFusedThreads = kTile * kTile / kFusedPix;

#ifndef SARR_FUSED_MIN_CTAS
#define SARR_FUSED_MIN_CTAS 18
#endif
__global__ void __launch_bounds__(kFusedThreads, SARR_FUSED_MIN_CTAS)
    select_render_kernel(const SelectArgs sa, const TileArgs ta) {
  constexpr int kPix = kFusedPix;
  static_assert(kFusedThreads == kCap, "one thread per list slot");
  static_assert(kFusedThreads == 64, "two warps: 8-row halves of the tile");
  __shared__ __align__(16) Rec s_rec[kCap];
  __shared__ float2 s_cut[2][kCap];
  __shared__ int s_list[kCap];
  __shared__ float s_z[kCap];
  __shared__ int s_rank[2][kCap];
  const int v = blockIdx.y, t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ViewConst& vc = sa.views[v];
  const int Nr = vc.h.Nr, Na = vc.h.Na, tiles_x = vc.tiles_x, T = tiles_x * vc.tiles_y;
  const int tx = t % tiles_x, ty = t / tiles_x;
  // warp block: 8 range rows x 16 azimuth columns
  const int r0 = ty * kTile + warp * 8, c0 = tx * kTile;
  const int pr = r0 + (lane & 7), pc0 = c0 + (lane >> 3);
  unsigned char* st = sa.st.base + v * sa.st.vstride;
  const int count = reinterpret_cast<const int*>(st + sa.st.L.count)[t];

  float value[kPix], trans[kPix];
  bool done[kPix];
#pragma unroll
  for (int i = 0; i < kPix; ++i) {
    value[i] = 0.0f;
    trans[i] = 1.0f;
    done[i] = false;
  }
  if (count > 0) {  // the same for the whole CTA
    const int nneed = sa.need_n[v * sa.need_n_vstride + t];
    s_list[tid] = -1;
    // the warps take alternate entries (entries with hit words one at a
    // time: emit_hit_words would leave the other warp idle on most tiles)
    const NeedRegs nr = prefetch_need<false>(sa, v, T, t, nneed, lane, warp, 2);
    __syncthreads();
    emit_entries(sa, v, st, t, T, tx, ty, nneed, nr, warp, 2, s_list, lane);
    __syncthreads();

    Rec rec;
    bool nan_z = false;
    if (tid < count) {
      const float zr = select_record<false, false>(sa, vc, st, t, tid, s_list, rec);
      s_z[tid] = zr;
      nan_z = zr != zr;
    }
    // rank by (Z_r, slot), as select_kernel
    int rank = 0;
    if (__syncthreads_or(nan_z)) {
      if (tid == 0) insertion_ranks(s_z, count, s_rank[0]);
      __syncthreads();
      rank = s_rank[0][tid];
    } else {
      int* sr = s_rank[warp];
      const uint64_t k0 = zslot_key(s_z[lane], lane, lane < count);
      if (count <= 32)
        warp_sort_ranks<32>(k0, ~0ull, lane, sr);
      else
        warp_sort_ranks<64>(k0, zslot_key(s_z[lane + 32], lane + 32, lane + 32 < count), lane, sr);
      __syncwarp();
      rank = sr[tid];
    }
    if (tid < count) s_rec[rank] = rec;
    __syncthreads();
    composite_block<kPix>(s_rec, s_cut[warp], count, r0, c0, pr, pc0, lane, value, trans, done);
  }
  float* img = ta.images + v * ta.img_vstride;
  if (pr < Nr) {
#pragma unroll
    for (int i = 0; i < kPix; ++i)
      if (pc0 + 4 * i < Na) img[(size_t)(pc0 + 4 * i) * Nr + pr] = value[i];
  }
}

// Omega per pixel (compute_omega_kernel :696-718): Omega_before of every
// listed Gaussian reached by the pixel is summed over the tile's pixels with
// warp reductions; partial[t][slot] = (sum, pixel count).
__global__ void __launch_bounds__(kWarpsPerTile * 32) omega_tile_kernel(const TileArgs a) {
  __shared__ __align__(16) Rec s_rec[kCap];
  __shared__ float2 s_red[kWarpsPerTile][kCap];
  __shared__ uint64_t bar;
  const int v = blockIdx.y, t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ViewConst& vc = a.views[v];
  const int Nr = vc.h.Nr, Na = vc.h.Na, tiles_x = vc.tiles_x;
  const int tx = t % tiles_x, ty = t / tiles_x;
  const unsigned char* st = a.st.base + v * a.st.vstride;
  const int count = reinterpret_cast<const int*>(st + a.st.L.count)[t];
  if (count == 0) return;
  const bool ok = load_tile_recs(s_rec, &bar, st, a.st.L, t, count, a.err, true);
  if (!__syncthreads_and(ok)) return;

  const int pc = tx * kTile + warp * 2 + (lane >> 4);
  const int pr = ty * kTile + (lane & 15);
  bool alive = pc < Na && pr < Nr;
  const float fx = (float)pc, fy = (float)pr;
  float omega = 1.0f;
  for (int k = 0; k < count; ++k) {
    const unsigned counted = __ballot_sync(0xffffffffu, alive);
    if (counted == 0) {
      if (lane == 0)
        for (int kk = k; kk < count; ++kk) s_red[warp][kk] = make_float2(0.0f, 0.0f);
      break;
    }
    const float before = alive ? omega : 0.0f;
    if (alive) {
      const Rec& g = s_rec[k];
      const float gamma_shadow = rec_density(g, fx, fy);
      const float sigma_i = g.sigma;
      omega = mul_(omega, fma_(-gamma_shadow, sigma_i, 1.0f));
      if (omega < 1e-8f) {
        omega = 0.0f;
        alive = false;
      }
    }
    const float sum = warp_sum(before);
    if (lane == 0) s_red[warp][k] = make_float2(sum, (float)__popc(counted));
  }
  __syncthreads();
  if (tid < count) {
    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int w = 0; w < kWarpsPerTile; ++w) {
      acc.x += s_red[w][tid].x;
      acc.y += s_red[w][tid].y;
    }
    float2* partial = reinterpret_cast<float2*>(a.partial + v * a.partial_vstride);
    partial[(size_t)t * kCap + s_rec[tid].pos] = acc;
  }
}

// Position of Gaussian i in the index-ordered list of tile t, or -1.
__device__ __forceinline__ int list_find(const int* __restrict__ list, int cnt, int i) {
  if (cnt <= 0 || i < list[0] || i > list[cnt - 1]) return -1;
  int lo = 0, hi = cnt - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    const int x = list[mid];
    if (x == i) return mid;
    if (x < i) lo = mid + 1; else hi = mid - 1;
  }
  return -1;
}

// Host-side Omega average (:1239-1252). Every Gaussian of a view starts at
// 1.0 (the reference's value for a Gaussian no pixel reached); then one
// thread per (tile, slot) entry of the view's shadow lists: the thread of the
// Gaussian's first listing tile, in the row-major tile order of its shadow
// rectangle, sums the (Omega, pixel count) partials of every tile that lists
// it, in that order, and writes their quotient. Only listed Gaussians (at most
// 64 per tile) do any work beyond the fill.
__global__ void __launch_bounds__(256) omega_fill_kernel(float* __restrict__ omega, int64_t n,
                                                         int nviews, size_t vstride) {
  const int64_t total = n * nviews;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t v = e / n, i = e - v * n;
    omega[v * vstride + i] = 1.0f;
  }
}

__global__ void __launch_bounds__(256) omega_listed_kernel(const OmegaScatterArgs a) {
  const int v = blockIdx.y;
  const ViewConst& vc = a.views[v];
  const int tiles_x = vc.tiles_x, T = tiles_x * vc.tiles_y;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= T * kCap) return;
  const int t = e / kCap, slot = e - t * kCap;
  const unsigned char* st = a.sh.base + v * a.sh.vstride;
  const int* cnts = reinterpret_cast<const int*>(st + a.sh.L.count);
  if (slot >= cnts[t]) return;
  const int* lists = reinterpret_cast<const int*>(st + a.sh.L.list);
  const int i = lists[(size_t)t * kCap + slot];
  if (i < 0 || (int64_t)i >= a.n) return;
  const uint32_t rc = state_rect(st, a.sh.L, a.ipp.base + v * a.ipp.vstride, a.ipp.L, i);
  const int tc0 = rc & 0xFF, tc1 = (rc >> 8) & 0xFF, tr0 = (rc >> 16) & 0xFF, tr1 = rc >> 24;
  const float2* partial = reinterpret_cast<const float2*>(a.partial + v * a.partial_vstride);
  float sum = 0.0f, c = 0.0f;
  bool first = true;
  for (int ty = tr0; ty <= tr1; ++ty)
    for (int tx = tc0; tx <= tc1; ++tx) {
      const int u = ty * tiles_x + tx;
      const int p = u == t ? slot : list_find(lists + (size_t)u * kCap, cnts[u], i);
      if (p < 0) continue;
      if (first && u != t) return;  // an earlier tile's thread writes this Gaussian
      first = false;
      const float2 q = partial[(size_t)u * kCap + p];
      sum += q.x;
      c += q.y;
    }
  a.omega[v * a.omega_vstride + i] = c > 0.0f ? sum / c : 1.0f;
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
// Per (pixel, Gaussian) terms of backward_kernel (:910-1018), summed over the
// tile: 0 grad_sigma, 1 dL/dpixel * dpixel/dS (times the SH basis later),
// 2..4 grad_cov rr, cc, rc, 5..6 grad_ipp_r, grad_ipp_c.
// Launches of fewer than SARR_BWD_ONE_PART_MIN_VIEWS views split the tile's
// records into kBwdParts consecutive parts, one CTA each (grid.z): the CTA of
// part q replays the transmittance of every pixel through the records before
// its part (the same operations in the same order as the full traversal) and
// computes the gradient terms of its own records, so the per-record sums are
// those of one front-to-back pass; larger launches take a tile in one CTA.
// The per-record constants of bwd_pixel_terms, computed once per record with
// the operations the per-pixel terms would repeat: x = 1 / (det + EPSILON)
// (.cu:973-974: one correctly rounded reciprocal and two products instead of
// two divisions, within 1.5 ulp of the quotients), y = -(cov_cc inv_det) / 2,
// z = -(cov_rr inv_det) / 2, w = 1 where det > EPSILON. det equals the
// record's (fma is symmetric in its factors), so its reciprocal and
// 2 pi sqrt(det) are the record's inv_det and norm.
__device__ __forceinline__ float4 bwd_rec_const(const Rec& g) {
  const float cov_rr = g.cyy, cov_cc = g.cxx, cov_rc = g.cxy;
  const float det = fma_(cov_rr, cov_cc, -mul_(cov_rc, cov_rc));
  const float inv_det = g.inv_det;
  return make_float4(__frcp_rn(add_(det, kEps)), -mul_(mul_(cov_cc, inv_det), 0.5f),
                     -mul_(mul_(cov_rr, inv_det), 0.5f), det > kEps ? 1.0f : 0.0f);
}

// bwd_rec_const of the records [0, count) into rc[] (CTA-wide, then a barrier).
__device__ __forceinline__ void fill_bwd_rec_consts(const Rec* recs, int count, float4* rc) {
  for (int k = threadIdx.x; k < count; k += blockDim.x) rc[k] = bwd_rec_const(recs[k]);
  __syncthreads();
}

// The gradient terms of one pixel for one record (backward_kernel :910-1018,
// written into A[0..6] where the pixel contributes, A untouched otherwise)
// and the pixel's transmittance update; returns whether it contributes.
// `rc`: the record's bwd_rec_const.
__device__ __forceinline__ bool bwd_pixel_terms(const Rec& g, float2 cut, float4 rc, float fx, float fy,
                                                float dL_d_pixel, float& prev_transmittance,
                                                float (&A)[7]) {
  bool contrib = false;
  const float gamma_ipp = density_above_cutoff(g, cut.x, cut.y, fx, fy);
  if (gamma_ipp >= 1e-8f) {
    contrib = true;
    const float sigma_i = g.sigma;
    const float S_i = g.s_pos;
    const float alpha_i = mul_(sigma_i, gamma_ipp);
    const float d_pixel_d_alpha = mul_(prev_transmittance, S_i);
    const float d_pixel_d_S = mul_(prev_transmittance, alpha_i);
    const float g_a = mul_(dL_d_pixel, d_pixel_d_alpha);  // dL/dpixel * dpixel/dalpha
    const float g_as = mul_(g_a, sigma_i);
    A[0] = mul_(g_a, gamma_ipp);
    A[1] = mul_(dL_d_pixel, d_pixel_d_S);
    const float dx = sub_(fx, g.mx);
    const float dy = sub_(fy, g.my);
    const float cov_rr = g.cyy, cov_cc = g.cxx, cov_rc = g.cxy;
    if (rc.w != 0.0f) {  // det > EPSILON
      const float inv_det = g.inv_det;
      // the backward's own exponent pairs cov_cc with dx^2 and cov_rr with dy^2 (:950)
      const float q = fma_(mul_(cov_rr, dy), dy,
                           fma_(mul_(cov_cc, dx), dx, -mul_(mul_(mul_(2.0f, cov_rc), dx), dy)));
      const float exponent = mul_(mul_(-0.5f, q), inv_det);
      if (exponent > -20.0f) {
        // exp(exponent) / norm, as in the density (one ex2.approx)
        const float base_val = ex2_approx(__fmaf_rn(exponent, 1.4426950408889634f, cut.y));
        const float h = mul_(mul_(0.5f, base_val), inv_det);
        const float d_gamma_d_cov_rr = mul_(h, fma_(dy, dy, rc.y));
        const float d_gamma_d_cov_cc = mul_(h, fma_(dx, dx, rc.z));
        const float d_gamma_d_cov_rc = mul_(mul_(mul_(-base_val, inv_det), dx), dy);
        A[2] = mul_(g_as, d_gamma_d_cov_rr);
        A[3] = mul_(g_as, d_gamma_d_cov_cc);
        A[4] = mul_(g_as, d_gamma_d_cov_rc);
      }
    }
    const float inv_det_eps = rc.x;  // 1 / (det + EPSILON) (.cu:973-974)
    const float d_center_dr = mul_(-fma_(cov_rc, dx, -mul_(cov_rr, dy)), inv_det_eps);
    const float d_center_dc = mul_(-fma_(cov_cc, dx, -mul_(cov_rc, dy)), inv_det_eps);
    A[5] = mul_(g_as, d_center_dr);
    A[6] = mul_(g_as, d_center_dc);
    prev_transmittance = mul_(prev_transmittance, fma_(-sigma_i, gamma_ipp, 1.0f));
    if (prev_transmittance < 1e-8f) prev_transmittance = 0.0f;
  }
  return contrib;
}

constexpr int kBwdParts = 4;
constexpr int kBwdPartRecs = kCap / kBwdParts;

__global__ void __launch_bounds__(kWarpsPerTile * 32) bwd_tile_kernel(const TileArgs a) {
  __shared__ __align__(16) Rec s_rec[kCap];
  __shared__ float s_red[kWarpsPerTile][kBwdPartRecs][8];
  __shared__ float2 s_cut[kWarpsPerTile][kCap];
  __shared__ float4 s_rc[kCap];
  __shared__ uint64_t bar;
  const int v = blockIdx.y, t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ViewConst& vc = a.views[v];
  const int Nr = vc.h.Nr, Na = vc.h.Na, tiles_x = vc.tiles_x;
  const int tx = t % tiles_x, ty = t / tiles_x;
  const unsigned char* st = a.st.base + v * a.st.vstride;
  const int count_all = reinterpret_cast<const int*>(st + a.st.L.count)[t];
  const int k_lo = blockIdx.z * kBwdPartRecs;
  if (k_lo >= count_all) return;
  const int count = min(count_all, k_lo + kBwdPartRecs);  // records [0, count) are read
  const bool ok = load_tile_recs(s_rec, &bar, st, a.st.L, t, count, a.err, true);
  if (!__syncthreads_and(ok)) return;
  fill_bwd_rec_consts(s_rec, count, s_rc);

  const int pc = tx * kTile + warp * 2 + (lane >> 4);
  const int pr = ty * kTile + (lane & 15);
  const bool in = pc < Na && pr < Nr;
  const float dL_d_pixel = in ? a.images[v * a.img_vstride + (size_t)pc * Nr + pr] : 0.0f;
  const float fx = (float)pc, fy = (float)pr;
  float prev_transmittance = 1.0f;
  // Records whose cutoff box misses the warp's 2 x 16 pixel block have no
  // contributing pixel there: their sums stay 0.
  for (int e = lane; e < kBwdPartRecs * 8; e += 32) (&s_red[warp][0][0])[e] = 0.0f;
  const float bx0 = (float)(tx * kTile + warp * 2), by0 = (float)(ty * kTile);
  uint64_t todo = block_hits(s_rec, count, s_cut[warp], bx0, bx0 + 1.0f, by0, by0 + 15.0f, lane);
  __syncwarp();

  // transmittance through the records before this part
  uint64_t before = k_lo ? todo & ((1ull << k_lo) - 1ull) : 0ull;
  todo &= ~before;
  while (before) {
    const int k = __ffsll((long long)before) - 1;
    before &= before - 1;
    const Rec& g = s_rec[k];
    if (in) {
      const float2 cut = s_cut[warp][k];
      const float gamma_ipp = density_above_cutoff(g, cut.x, cut.y, fx, fy);
      if (gamma_ipp >= 1e-8f) {
        prev_transmittance = mul_(prev_transmittance, fma_(-g.sigma, gamma_ipp, 1.0f));
        if (prev_transmittance < 1e-8f) prev_transmittance = 0.0f;
      }
    }
  }

  while (todo) {
    const int k = __ffsll((long long)todo) - 1;
    todo &= todo - 1;
    const Rec& g = s_rec[k];
    float A[7] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    bool contrib = false;
    if (in) contrib = bwd_pixel_terms(g, s_cut[warp][k], s_rc[k], fx, fy, dL_d_pixel, prev_transmittance, A);
    if (__any_sync(0xffffffffu, contrib)) {
      const float A8[8] = {A[0], A[1], A[2], A[3], A[4], A[5], A[6], 0.0f};
      const float total = warp_sum8_scatter(A8, lane);
      const int c = 4 * ((lane >> 4) & 1) + 2 * ((lane >> 3) & 1) + ((lane >> 2) & 1);
      if ((lane & 3) == 0 && c < 7) s_red[warp][k - k_lo][c] = total;
    }
  }
  __syncthreads();
  float* partial = a.partial + v * a.partial_vstride;
  for (int e = tid; e < (count - k_lo) * 7; e += kWarpsPerTile * 32) {
    const int kp = e / 7, c = e - kp * 7;
    float acc = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarpsPerTile; ++w) acc += s_red[w][kp][c];
    partial[((size_t)t * kCap + s_rec[k_lo + kp].pos) * 8 + c] = acc;
  }
}

// bwd_tile_kernel for launches of many views: two warps per (tile, part),
// each an 8 x 16 pixel block with four pixels per lane (one range row,
// azimuth columns c, c + 4, c + 8, c + 12, as render_kernel<4>). Per record,
// each lane adds its pixels' terms first, so one warp reduction covers 128
// pixels; per pixel, only the records whose cutoff box meets its 8 x 4
// quarter are visited (the others have density 0 there). The per-record sums
// are those of bwd_tile_kernel up to the order of the additions. kParts is
// the number of record parts (grid.z): launches of many views have CTAs
// enough with one part, which walks each pixel through the tile's records
// once instead of replaying the records before each part.
constexpr int kBwdPix = 4;
constexpr int kBwdManyMinViews = 16;
#ifndef SARR_BWD_ONE_PART_MIN_VIEWS
#define SARR_BWD_ONE_PART_MIN_VIEWS 32
#endif

template <int kParts>
__global__ void __launch_bounds__(kTile * kTile / kBwdPix) bwd_tile4_kernel(const TileArgs a) {
  constexpr int kWarps = kTile * kTile / kBwdPix / 32;
  static_assert(kWarps == 2, "two 8-row halves of the tile");
  constexpr int kPartRecs = kCap / kParts;
  __shared__ __align__(16) Rec s_rec[kCap];
  __shared__ float s_red[kWarps][kPartRecs][8];
  __shared__ float2 s_cut[kWarps][kCap];
  __shared__ float4 s_rc[kCap];
  __shared__ uint64_t bar;
  const int v = blockIdx.y, t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ViewConst& vc = a.views[v];
  const int Nr = vc.h.Nr, Na = vc.h.Na, tiles_x = vc.tiles_x;
  const int tx = t % tiles_x, ty = t / tiles_x;
  const unsigned char* st = a.st.base + v * a.st.vstride;
  const int count_all = reinterpret_cast<const int*>(st + a.st.L.count)[t];
  const int k_lo = blockIdx.z * kPartRecs;
  if (k_lo >= count_all) return;
  const int count = min(count_all, k_lo + kPartRecs);  // records [0, count) are read
  const bool ok = load_tile_recs(s_rec, &bar, st, a.st.L, t, count, a.err, true);
  if (!__syncthreads_and(ok)) return;
  fill_bwd_rec_consts(s_rec, count, s_rc);

  const int r0 = ty * kTile + warp * 8, c0 = tx * kTile;
  const int pr = r0 + (lane & 7), pc0 = c0 + (lane >> 3);
  const float fy = (float)pr;
  float dL[kBwdPix], trans[kBwdPix], fx[kBwdPix];
  bool in[kBwdPix];
  const float* gimg = a.images + v * a.img_vstride;
#pragma unroll
  for (int i = 0; i < kBwdPix; ++i) {
    const int pc = pc0 + 4 * i;
    in[i] = pc < Na && pr < Nr;
    dL[i] = in[i] ? gimg[(size_t)pc * Nr + pr] : 0.0f;
    trans[i] = 1.0f;
    fx[i] = (float)pc;
  }
  for (int e = lane; e < kPartRecs * 8; e += 32) (&s_red[warp][0][0])[e] = 0.0f;
  uint64_t hit[kBwdPix];
  quarter_hits<kBwdPix>(s_rec, s_cut[warp], count, r0, c0, lane, hit);
  uint64_t any = 0;
#pragma unroll
  for (int i = 0; i < kBwdPix; ++i) any |= hit[i];

  // transmittance through the records before this part
  uint64_t before = k_lo ? any & ((1ull << k_lo) - 1ull) : 0ull;
  uint64_t todo = any & ~before;
  while (before) {
    const int k = __ffsll((long long)before) - 1;
    before &= before - 1;
    const Rec& g = s_rec[k];
    const float2 cut = s_cut[warp][k];
#pragma unroll
    for (int i = 0; i < kBwdPix; ++i) {
      if (((hit[i] >> k) & 1ull) && in[i]) {
        const float gamma_ipp = density_above_cutoff(g, cut.x, cut.y, fx[i], fy);
        if (gamma_ipp >= 1e-8f) {
          trans[i] = mul_(trans[i], fma_(-g.sigma, gamma_ipp, 1.0f));
          if (trans[i] < 1e-8f) trans[i] = 0.0f;
        }
      }
    }
  }

  while (todo) {
    const int k = __ffsll((long long)todo) - 1;
    todo &= todo - 1;
    const Rec& g = s_rec[k];
    const float2 cut = s_cut[warp][k];
    const float4 rc = s_rc[k];
    float A[7] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    bool contrib = false;
#pragma unroll
    for (int i = 0; i < kBwdPix; ++i) {
      if (((hit[i] >> k) & 1ull) && in[i]) {
        float Ai[7] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (bwd_pixel_terms(g, cut, rc, fx[i], fy, dL[i], trans[i], Ai)) {
          contrib = true;
#pragma unroll
          for (int j = 0; j < 7; ++j) A[j] = add_(A[j], Ai[j]);
        }
      }
    }
    if (__any_sync(0xffffffffu, contrib)) {
      const float A8[8] = {A[0], A[1], A[2], A[3], A[4], A[5], A[6], 0.0f};
      const float total = warp_sum8_scatter(A8, lane);
      const int c = 4 * ((lane >> 4) & 1) + 2 * ((lane >> 3) & 1) + ((lane >> 2) & 1);
      if ((lane & 3) == 0 && c < 7) s_red[warp][k - k_lo][c] = total;
    }
  }
  __syncthreads();
  float* partial = a.partial + v * a.partial_vstride;
  for (int e = tid; e < (count - k_lo) * 7; e += kWarps * 32) {
    const int kp = e / 7, c = e - kp * 7;
    partial[((size_t)t * kCap + s_rec[k_lo + kp].pos) * 8 + c] = add_(s_red[0][kp][c], s_red[1][kp][c]);
  }
}

// Dense gradient rows. The per-Gaussian chain of backward_kernel (:979-1013)
// is linear in (grad_ipp_r, grad_ipp_c), so it is applied once to the tile sums.
// The backward's inverse index (launch_bwd_index): the list entries of the
// group's image-plane tile lists grouped by Gaussian. A count pass (one
// thread per (view, tile, slot)), an exclusive scan of the counts, and a fill
// pass that places each entry in its Gaussian's range (in any order there;
// bwd_scatter_kernel orders each Gaussian's few entries itself).
__device__ __forceinline__ uint32_t* entry_slot(uint32_t* entries, size_t vstride, int per,
                                                int64_t e) {
  return entries + (size_t)(e / per) * vstride + (size_t)(e % per);
}

template <bool kFill>
__global__ void __launch_bounds__(256) bwd_index_kernel(const BwdIndexArgs a) {
  const int v = blockIdx.y;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= a.T * kCap) return;
  const int t = e / kCap, slot = e - t * kCap;
  const unsigned char* st = a.ipp.base + v * a.ipp.vstride;
  if (slot >= reinterpret_cast<const int*>(st + a.ipp.L.count)[t]) return;
  const int i = reinterpret_cast<const int*>(st + a.ipp.L.list)[(size_t)t * kCap + slot];
  if (i < 0 || (int64_t)i >= a.n) return;
  if (!kFill) {
    atomicAdd(a.cnt + i, 1);
  } else {
    const int64_t pos = (int64_t)a.start[i] + atomicSub(a.cnt + i, 1) - 1;
    *entry_slot(a.entries, a.entries_vstride, a.T * kCap, pos) =
        ((uint32_t)v << 24) | ((uint32_t)t << 6) | (uint32_t)slot;
  }
}

// Exclusive scan of cnt[0, n) into start[0, n] in three passes: block sums
// (kGatherScanBlock elements per CTA, 16 per thread), the scan of the block
// sums by one CTA, and each block's local scan plus its offset.
constexpr int kGatherScanThreads = kGatherScanBlock / 16;
static_assert(kGatherScanThreads == 256, "16 elements per thread, 256 threads");

__device__ __forceinline__ int block_excl_scan256(int x, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int incl = warp_incl_scan(x, lane);
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = lane < 8 ? s_warp[lane] : 0;
    const int wi = warp_incl_scan(w, lane);
    if (lane < 8) s_warp[8 + lane] = wi - w;
    if (lane == 7) s_warp[16] = wi;
  }
  __syncthreads();
  total = s_warp[16];
  return s_warp[8 + warp] + incl - x;
}

__global__ void __launch_bounds__(kGatherScanThreads) gather_scan_sums_kernel(const int* __restrict__ cnt,
                                                                              int64_t n, int* bsum) {
  __shared__ int s_warp[17];
  const int64_t base = (int64_t)blockIdx.x * kGatherScanBlock + threadIdx.x * 16;
  int x = 0;
#pragma unroll
  for (int k = 0; k < 16; ++k)
    if (base + k < n) x += cnt[base + k];
  int total;
  block_excl_scan256(x, s_warp, total);
  if (threadIdx.x == 0) bsum[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kGatherScanThreads) gather_scan_top_kernel(int* bsum, int nb,
                                                                             int* start, int64_t n) {
  __shared__ int s_warp[17];
  int carry = 0;
  for (int b0 = 0; b0 < nb; b0 += kGatherScanThreads) {
    const int b = b0 + threadIdx.x;
    const int x = b < nb ? bsum[b] : 0;
    int total;
    const int ex = block_excl_scan256(x, s_warp, total);
    if (b < nb) bsum[b] = carry + ex;
    carry += total;
    __syncthreads();  // s_warp is reused by the next round
  }
  if (threadIdx.x == 0) {
    bsum[nb] = carry;
    start[n] = carry;
  }
}

__global__ void __launch_bounds__(kGatherScanThreads) gather_scan_apply_kernel(const int* __restrict__ cnt,
                                                                               int64_t n,
                                                                               const int* __restrict__ bsum,
                                                                               int* start) {
  __shared__ int s_warp[17];
  const int64_t base = (int64_t)blockIdx.x * kGatherScanBlock + threadIdx.x * 16;
  int c[16];
  int x = 0;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    c[k] = base + k < n ? cnt[base + k] : 0;
    x += c[k];
  }
  int total;
  int run = bsum[blockIdx.x] + block_excl_scan256(x, s_warp, total);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    if (base + k < n) start[base + k] = run;
    run += c[k];
  }
}

// Dense gradient rows of the Gaussians [begin, end). A Gaussian's list
// entries (from the inverse index) are taken in (view, tile) order -- views
// ascending, the tiles of a view in row-major order -- their per-slot partial
// sums added per view, then the view's chain rule (:979-1013), which is
// linear in (grad_ipp_r, grad_ipp_c), applied once per view and the views'
// contributions summed in view order. Deterministic: no float atomics.
// bwd_scatter_kernel takes the Gaussians with at most kScatterLocalEntries
// entries, one thread each; the others (the lowest-index Gaussians fill most
// tile lists, so they have one entry per listing tile of every view) go to
// bwd_heavy_kernel, one warp each.
constexpr int kScatterLocalEntries = 16;

// One view's contribution: its partial sums A[0..4] and the means chain.
struct ViewContrib {
  float a0, a1, a2, a3, a4, cx, cy, cz;
};

__device__ __forceinline__ ViewContrib bwd_view_contrib(const ViewConst& vc, const float A[7], float2 yzr) {
  ViewContrib o;
  o.a0 = A[0];
  o.a1 = A[1];
  o.a2 = A[2];
  o.a3 = A[3];
  o.a4 = A[4];
  const float rho_r = vc.h.rho_r, rho_a = vc.h.rho_a;
  const float yr = yzr.x, zr = yzr.y;
  const float grad_ipp_r = A[5], grad_ipp_c = A[6];
  const float Rmin = sqrtf(yr * yr + zr * zr + kEps);
  const float d_r_d_yr = yr / (rho_r * Rmin);
  const float d_r_d_zr = zr / (rho_r * Rmin);
  const float grad_xr = grad_ipp_c / rho_a;
  const float grad_yr = grad_ipp_r * d_r_d_yr / rho_r;
  const float grad_zr = grad_ipp_r * d_r_d_zr / rho_r;
  const float cos_a = vc.cos_a, sin_a = vc.sin_a, cos_b = vc.cos_b, sin_b = vc.sin_b;
  const float d_xr_d_xw = cos_a, d_xr_d_yw = sin_a, d_xr_d_zw = 0.0f;
  const float d_yr_d_xw = cos_b * sin_a, d_yr_d_yw = -cos_b * cos_a, d_yr_d_zw = -sin_b;
  const float d_zr_d_xw = -sin_b * sin_a, d_zr_d_yw = sin_b * cos_a, d_zr_d_zw = -cos_b;
  o.cx = grad_xr * d_xr_d_xw + grad_yr * d_yr_d_xw + grad_zr * d_zr_d_xw;
  o.cy = grad_xr * d_xr_d_yw + grad_yr * d_yr_d_yw + grad_zr * d_zr_d_yw;
  o.cz = grad_xr * d_xr_d_zw + grad_yr * d_yr_d_zw + grad_zr * d_zr_d_zw;
  return o;
}

// The 23 gradient sums of a Gaussian, accumulated view by view with the
// same operations on both paths.
struct GradSums {
  float sigma, rr, cc, rc, x, y, z;
  float sh[kSh];
};

__device__ __forceinline__ void grad_add_view(GradSums& g, const ViewContrib& c, const ViewConst& vc) {
  g.sigma = __fadd_rn(g.sigma, c.a0);
#pragma unroll
  for (int k = 0; k < kSh; ++k) g.sh[k] = __fmaf_rn(c.a1, vc.h.sh_basis[k], g.sh[k]);
  g.rr = __fadd_rn(g.rr, c.a2);
  g.cc = __fadd_rn(g.cc, c.a3);
  g.rc = __fadd_rn(g.rc, c.a4);
  g.x = __fadd_rn(g.x, c.cx);
  g.y = __fadd_rn(g.y, c.cy);
  g.z = __fadd_rn(g.z, c.cz);
}

__device__ __forceinline__ void entry_partial(const BwdScatterArgs& a, uint32_t key, float A[7], float2& yzr) {
  const int v = (int)(key >> 24), t = (int)((key >> 6) & 0x3FFFFu), slot = (int)(key & 63u);
  const float* q8 = a.partial + v * a.partial_vstride + ((size_t)t * kCap + slot) * 8;
  const float4 p0 = *reinterpret_cast<const float4*>(q8);
  const float4 p1 = *reinterpret_cast<const float4*>(q8 + 4);
  A[0] = __fadd_rn(A[0], p0.x);
  A[1] = __fadd_rn(A[1], p0.y);
  A[2] = __fadd_rn(A[2], p0.z);
  A[3] = __fadd_rn(A[3], p0.w);
  A[4] = __fadd_rn(A[4], p1.x);
  A[5] = __fadd_rn(A[5], p1.y);
  A[6] = __fadd_rn(A[6], p1.z);
  const unsigned char* st = a.ipp.base + v * a.ipp.vstride;
  yzr = reinterpret_cast<const float2*>(st + a.ipp.L.yz)[(size_t)t * kCap + slot];
}

__device__ __forceinline__ void write_grad_row(const BwdScatterArgs& a, int64_t gi, const GradSums& g) {
  const int64_t i = gi - a.row0;  // the row of Gaussian gi in the gradient arrays
  float gx = g.x, gy = g.y, gz = g.z;
  float* gm = a.grad_means + i * 3;
  if (a.accumulate) {
    gx += gm[0];
    gy += gm[1];
    gz += gm[2];
  }
  gm[0] = gx;
  gm[1] = gy;
  gm[2] = gz;
  if (a.grad_norm) a.grad_norm[i] = sqrtf(gx * gx + gy * gy + gz * gz);
  if (a.grad_cov_layout == 6) {
    float* gc = a.grad_cov + i * 6;
    const float c6[6] = {g.rr, g.cc, 0.f, g.rc, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < 6; ++q) gc[q] = a.accumulate ? gc[q] + c6[q] : c6[q];
  } else {
    float* gc = a.grad_cov + i * 9;
    const float c9[9] = {g.rr, g.rc, 0.f, g.rc, g.cc, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < 9; ++q) gc[q] = a.accumulate ? gc[q] + c9[q] : c9[q];
  }
  a.grad_sigma[i] = a.accumulate ? a.grad_sigma[i] + g.sigma : g.sigma;
  float* gs = a.grad_sh + i * a.grad_sh_cols;
  if (a.grad_sh_cols == kSh && !a.accumulate && ((uintptr_t)gs & 15) == 0) {
    float4* gs4 = reinterpret_cast<float4*>(gs);
#pragma unroll
    for (int q = 0; q < 4; ++q) gs4[q] = make_float4(g.sh[4 * q], g.sh[4 * q + 1], g.sh[4 * q + 2], g.sh[4 * q + 3]);
  } else {
#pragma unroll
    for (int k = 0; k < kSh; ++k)
      if (k < a.grad_sh_cols) gs[k] = a.accumulate ? gs[k] + g.sh[k] : g.sh[k];
  }
}

__device__ __forceinline__ GradSums grad_zero() {
  GradSums g;
  g.sigma = g.rr = g.cc = g.rc = g.x = g.y = g.z = 0.f;
#pragma unroll
  for (int k = 0; k < kSh; ++k) g.sh[k] = 0.f;
  return g;
}

// The entries of one Gaussian in sorted order (keys[0..c) ascending), summed.
template <typename KeyAt>
__device__ __forceinline__ GradSums grad_from_sorted(const BwdScatterArgs& a, int c, KeyAt key_at) {
  GradSums g = grad_zero();
  int cur_v = -1;
  float A[7] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float2 yzr = make_float2(0.f, 0.f);
  for (int q = 0; q < c; ++q) {
    const uint32_t k = key_at(q);
    const int v = (int)(k >> 24);
    if (v != cur_v) {
      if (cur_v >= 0) grad_add_view(g, bwd_view_contrib(a.views[cur_v], A, yzr), a.views[cur_v]);
      cur_v = v;
#pragma unroll
      for (int cc = 0; cc < 7; ++cc) A[cc] = 0.f;
    }
    entry_partial(a, k, A, yzr);
  }
  if (cur_v >= 0) grad_add_view(g, bwd_view_contrib(a.views[cur_v], A, yzr), a.views[cur_v]);
  return g;
}

// Calls of at most kDirectGatherMaxViews views: no inverse index; each
// Gaussian looks itself up in the lists of the tiles its rectangle covers,
// view by view (binary searches in the index-ordered lists), in the same
// (view, tile) order and with the same sums as the indexed path.
constexpr int kDirectGatherMaxViews = 4;

__global__ void __launch_bounds__(256) bwd_gather_kernel(const BwdScatterArgs a) {
  const int64_t i = a.begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.end) return;
  GradSums g = grad_zero();
  for (int v = 0; v < a.nviews; ++v) {
    const ViewConst& vc = a.views[v];
    const int tiles_x = vc.tiles_x;
    const unsigned char* st = a.ipp.base + v * a.ipp.vstride;
    const uint32_t rc = state_rect(st, a.ipp.L, st, a.ipp.L, i);
    const int tc0 = rc & 0xFF, tc1 = (rc >> 8) & 0xFF, tr0 = (rc >> 16) & 0xFF, tr1 = rc >> 24;
    if (tc0 > tc1) continue;
    const int* cnts = reinterpret_cast<const int*>(st + a.ipp.L.count);
    const int* lists = reinterpret_cast<const int*>(st + a.ipp.L.list);
    float A[7] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float2 yzr = make_float2(0.f, 0.f);
    bool hit = false;
    for (int ty = tr0; ty <= tr1; ++ty)
      for (int tx = tc0; tx <= tc1; ++tx) {
        const int t = ty * tiles_x + tx;
        const int p = list_find(lists + (size_t)t * kCap, cnts[t], (int)i);
        if (p >= 0) {
          hit = true;
          entry_partial(a, ((uint32_t)v << 24) | ((uint32_t)t << 6) | (uint32_t)p, A, yzr);
        }
      }
    if (hit) grad_add_view(g, bwd_view_contrib(vc, A, yzr), vc);
  }
  write_grad_row(a, i, g);
}

__global__ void __launch_bounds__(256) bwd_scatter_kernel(const BwdScatterArgs a) {
  const int64_t i = a.begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.end) return;
  const int e0 = a.start[i], c = a.start[i + 1] - e0;
  if (c > kScatterLocalEntries) {
    const int h = atomicAdd(a.heavy, 1);
    a.heavy[1 + h] = (int)i;
    return;
  }
  const int per_view = a.views[0].tiles_x * a.views[0].tiles_y * kCap;
  uint32_t key[kScatterLocalEntries];
  for (int q = 0; q < c; ++q)
    key[q] = *entry_slot(const_cast<uint32_t*>(a.entries), a.entries_vstride, per_view, (int64_t)e0 + q);
  for (int q = 1; q < c; ++q) {  // insertion sort (a Gaussian's keys are distinct)
    const uint32_t x = key[q];
    int r = q - 1;
    while (r >= 0 && key[r] > x) {
      key[r + 1] = key[r];
      --r;
    }
    key[r + 1] = x;
  }
  const GradSums g = grad_from_sorted(a, c, [&](int q) { return key[q]; });
  write_grad_row(a, i, g);
}

// One warp per Gaussian left by bwd_scatter_kernel (8 per CTA, persistent
// over the list). The group's views are taken in blocks of 32, lane l for
// view 32 j + l of block j: the lanes read the Gaussian's entries 32 at a
// time and drop each entry of the block into its view's bucket in shared
// memory; each lane then orders its view's bucket by tile, sums the
// partials and applies the view's chain rule; then 23 lanes, one per output
// sum, add the block's view contributions in view order. A view with more
// than kHeavyViewEntries listing tiles of the Gaussian (a bbox wider than
// ~80 pixels) takes them in order by repeated selection.
constexpr int kHeavyViewEntries = 32;
constexpr int kHeavyWarps = 8;

__device__ __forceinline__ uint32_t entry_at(const BwdScatterArgs& a, int per_view, int64_t e) {
  return a.entries[(size_t)(e / per_view) * a.entries_vstride + (size_t)(e % per_view)];
}

__global__ void __launch_bounds__(kHeavyWarps * 32) bwd_heavy_kernel(const BwdScatterArgs a) {
  __shared__ ViewContrib s_con[kHeavyWarps][32];
  __shared__ int s_has[kHeavyWarps][32];
  __shared__ int s_cnt[kHeavyWarps][32];
  // one bucket row per view of the block, padded so that the lanes, each on
  // its own row at the same position, hit distinct banks
  __shared__ uint32_t s_keys[kHeavyWarps][32][kHeavyViewEntries + 1];
  __shared__ float s_out[kHeavyWarps][23];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int count = a.heavy[0];
  const int nviews = a.nviews;
  const int per_view = a.views[0].tiles_x * a.views[0].tiles_y * kCap;  // >= 64 entries per slice
  uint32_t* keys = s_keys[warp][lane];
  for (int h = blockIdx.x * kHeavyWarps + warp; h < count; h += gridDim.x * kHeavyWarps) {
    const int64_t i = a.heavy[1 + h];
    const int e0 = a.start[i], c = a.start[i + 1] - e0;
    float acc = 0.f;  // output sum `lane` (lanes < 23)
    for (int vb = 0; vb < nviews; vb += 32) {
      const int v = vb + lane;
      s_cnt[warp][lane] = 0;
      __syncwarp();
      {
        // entry e0 + q0 + lane lies in slice `slice` at offset `off`
        int slice = (e0 + lane) / per_view, off = (e0 + lane) % per_view;
        for (int q0 = 0; q0 < c; q0 += 32) {
          if (q0 + lane < c) {
            const uint32_t k = a.entries[(size_t)slice * a.entries_vstride + off];
            const int vr = (int)(k >> 24) - vb;
            if (vr >= 0 && vr < 32) {
              const int p = atomicAdd(&s_cnt[warp][vr], 1);
              if (p < kHeavyViewEntries) s_keys[warp][vr][p] = k;
            }
          }
          off += 32;
          if (off >= per_view) {
            off -= per_view;
            ++slice;
          }
        }
      }
      __syncwarp();
      const int m = s_cnt[warp][lane];
      s_has[warp][lane] = 0;
      if (v < nviews && m > 0) {
        float A[7] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        float2 yzr = make_float2(0.f, 0.f);
        if (m <= kHeavyViewEntries) {
          for (int q = 1; q < m; ++q) {  // insertion sort by tile (a view's keys are distinct)
            const uint32_t x = keys[q];
            int r = q - 1;
            while (r >= 0 && keys[r] > x) {
              keys[r + 1] = keys[r];
              --r;
            }
            keys[r + 1] = x;
          }
          for (int q = 0; q < m; ++q) entry_partial(a, keys[q], A, yzr);
        } else {
          uint32_t last = 0;
          for (int q = 0; q < m; ++q) {
            uint32_t k = 0xFFFFFFFFu;
            for (int r = 0; r < c; ++r) {
              const uint32_t x = entry_at(a, per_view, (int64_t)e0 + r);
              if ((int)(x >> 24) == v && (q == 0 || x > last) && x < k) k = x;
            }
            last = k;
            entry_partial(a, k, A, yzr);
          }
        }
        s_con[warp][lane] = bwd_view_contrib(a.views[v], A, yzr);
        s_has[warp][lane] = 1;
      }
      __syncwarp();
      if (lane < 23) {
        // output sum lane: 0 sigma, 1..16 SH, 17 rr, 18 cc, 19 rc, 20..22 x y z.
        // Every lane takes acc = fma(x, y, acc): y is the view's SH basis value
        // for the SH sums and 1 for the others (x * 1 is exact, so that is
        // acc + x rounded once), so the lanes run one path.
        const int field = lane == 0 ? 0 : (lane <= kSh ? 1 : lane - kSh + 1);  // ViewContrib member
        const int ub = min(32, nviews - vb);
        for (int u = 0; u < ub; ++u) {
          if (!s_has[warp][u]) continue;
          const float x = (&s_con[warp][u].a0)[field];
          const float y = (lane >= 1 && lane <= kSh) ? a.views[vb + u].h.sh_basis[lane - 1] : 1.0f;
          acc = __fmaf_rn(x, y, acc);
        }
      }
      __syncwarp();
    }
    if (lane < 23) s_out[warp][lane] = acc;
    __syncwarp();
    if (lane == 0) {
      GradSums g;
      g.sigma = s_out[warp][0];
#pragma unroll
      for (int k = 0; k < kSh; ++k) g.sh[k] = s_out[warp][1 + k];
      g.rr = s_out[warp][17];
      g.cc = s_out[warp][18];
      g.rc = s_out[warp][19];
      g.x = s_out[warp][20];
      g.y = s_out[warp][21];
      g.z = s_out[warp][22];
      write_grad_row(a, i, g);
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// test hooks
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) debug_preprocess_kernel(const DebugPreArgs a) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.n) return;
  ViewConst vc;
  vc.h = a.vh;
  vc.cos_a = cosf(a.vh.alpha);
  vc.sin_a = sinf(a.vh.alpha);
  vc.cos_b = cosf(a.vh.beta);
  vc.sin_b = sinf(a.vh.beta);
  view_derive(vc);
  const int Nr = a.vh.Nr, Na = a.vh.Na;
  float cw[6];
  load_cov6(a.cov + (size_t)i * a.cov_layout, a.cov_layout, cw);
  const float* m = a.means + (size_t)i * 3;
  Proj o;
  project_gaussian(vc, m[0], m[1], m[2], cw, o);
  const float S = sh_scattering(vc, a.sh + (size_t)i * a.sh_stride, a.sh_k);
  const float f[13] = {o.r, o.c, o.cov_rr, o.cov_cc, o.cov_rc, o.xr, o.yr, o.XX, o.YY, o.XY, o.yr, o.zr, S};
#pragma unroll
  for (int k = 0; k < 13; ++k) a.f32[(size_t)k * a.n + i] = f[k];
  const bool valid = !(a.sigma[i] < 0.01f) && proj_valid(o, Nr, Na);
  int r0 = 0, r1 = 0, c0 = 0, c1 = 0, s_ok = 0, sc0 = 0, sc1 = 0, sr0 = 0, sr1 = 0;
  if (valid) {
    ipp_ranges(o, Nr, Na, r0, r1, c0, c1);
    s_ok = shadow_ranges(o, Nr, Na, sr0, sr1, sc0, sc1) ? 1 : 0;
  }
  const int32_t q[10] = {valid ? 1 : 0, r0, r1, c0, c1, s_ok, sc0, sc1, sr0, sr1};
#pragma unroll
  for (int k = 0; k < 10; ++k) a.i32[(size_t)k * a.n + i] = q[k];
}

__global__ void __launch_bounds__(kCap) debug_lists_kernel(const DebugListArgs a) {
  const int t = blockIdx.x, s = threadIdx.x;
  const unsigned char* st = a.st.base;
  const int cnt = reinterpret_cast<const int*>(st + a.st.L.count)[t];
  const int* list = reinterpret_cast<const int*>(st + a.st.L.list) + (size_t)t * kCap;
  const Rec* recs = reinterpret_cast<const Rec*>(st + a.st.L.recs) + (size_t)t * kCap;
  if (s == 0) a.counts[t] = cnt;
  a.lists[(size_t)t * kCap + s] = s < cnt ? list[s] : -1;
  a.sorted[(size_t)t * kCap + s] = s < cnt ? list[recs[s].pos] : -1;
}

__global__ void debug_view_kernel(const ViewHost vh, float* __restrict__ out) {
  const float f[14] = {vh.radar_x, vh.radar_y, vh.radar_z, vh.alpha, vh.beta, vh.Rc, vh.rho_r,
                       vh.rho_a, (float)vh.Nr, (float)vh.Na, cosf(vh.alpha), sinf(vh.alpha),
                       cosf(vh.beta), sinf(vh.beta)};
  for (int k = 0; k < 14; ++k) out[k] = f[k];
  for (int k = 0; k < kSh; ++k) out[14 + k] = vh.sh_basis[k];
}

// ---------------------------------------------------------------------------
// launch wrappers
// ---------------------------------------------------------------------------
// Dynamic shared memory above the default opt-in limit needs the function
// attribute; the kernels' static shared memory (< 16 KB) counts against the
// same 48 KB.
static bool needs_smem_attr(size_t dynamic_smem) { return dynamic_smem + 16384 > 48 * 1024; }

// Segment masks of the prefix chunks are kept for tile grids up to
// kSegMaskMaxTiles tiles.
bool segmask_supported(const Dims& d) { return d.T <= kSegMaskMaxTiles; }

static size_t bin_smem_bytes(const Dims& d, int cov_layout, bool shadow, bool masks) {
  const size_t stage = (size_t)(3 + cov_layout + 1) * kChunk * sizeof(float);
  const size_t T1 = (size_t)(d.tiles_y + 1) * (d.tiles_x + 1);
  return stage + T1 * sizeof(int) * (shadow ? 2 : 1) +
         (masks ? (size_t)d.T * 4 * (shadow ? 2 : 1) : 0);
}

// Per-warp tile counters of bin_skip_kernel; grids whose counters would not
// fit in kWarpCountBytes use the CTA-wide skipping variant of bin_kernel.
constexpr size_t kWarpCountBytes = 32 * 1024;
static size_t warp_count_bytes(const Dims& d, bool shadow) {
  return (size_t)(kBinThreads / 32) * ((d.T + 1) / 2) * 4 * (shadow ? 2 : 1);
}
bool segmask_all_chunks(const Dims& d) { return d.T <= kSegMaskAllMaxTiles; }

// per-warp segment masks of the skipping binners
static size_t warp_mask_bytes(const Dims& d, bool shadow, bool masks) {
  return masks ? (size_t)(kBinThreads / 32) * d.T * 4 * (shadow ? 2 : 1) : 0;
}

static size_t bin_skip_smem_bytes(const Dims& d, int cov_layout, bool shadow, bool masks) {
  return (size_t)(3 + (SARR_SKIP_COV_SMEM ? cov_layout : 0) + 2) * kChunk * sizeof(float) +
         warp_count_bytes(d, shadow) + warp_mask_bytes(d, shadow, masks);
}

// CTAs of bin_skip_kernel that the whole GPU holds at once (0 if unknown).
int skip_bin_wave(const Dims& d, int cov_layout, bool shadow, bool masks) {
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  const size_t smem = bin_skip_smem_bytes(d, cov_layout, shadow, masks);
  const cudaError_t e =
      shadow ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, bin_skip_kernel<true>, kBinThreads, smem)
             : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, bin_skip_kernel<false>, kBinThreads, smem);
  if (e != cudaSuccess) return 0;
  return sms * per_sm;
}

bool skip_bin_per_warp(const Dims& d, bool shadow) {
  return warp_count_bytes(d, shadow) <= kWarpCountBytes;
}

template <bool kShadow>
static void launch_bin_skip_t(const BinArgs& a, dim3 grid, size_t smem, cudaStream_t s) {
  if (needs_smem_attr(smem))
    cudaFuncSetAttribute(bin_skip_kernel<kShadow>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  bin_skip_kernel<kShadow><<<grid, kBinThreads, smem, s>>>(a);
}

cudaError_t launch_view_setup(const ViewHostPack& pack, ViewConst* out, int* err_to_clear,
                              cudaStream_t s) {
  if (pack.n <= kSmallViewPack) {
    ViewHostPackN<kSmallViewPack> small;
    small.n = pack.n;
    for (int v = 0; v < kSmallViewPack; ++v) small.v[v] = pack.v[v];
    view_setup_kernel<kSmallViewPack><<<1, 32, 0, s>>>(small, out, err_to_clear);
  } else {
    view_setup_kernel<kMaxViewsPerLaunch><<<(pack.n + 31) / 32, 32, 0, s>>>(pack, out, err_to_clear);
  }
  return cudaGetLastError();
}

template <bool kShadow, bool kSkip>
static void launch_bin_t(const BinArgs& a, dim3 grid, size_t smem, size_t hit_bytes_per_warp,
                         cudaStream_t s) {
  // a launch of few CTAs (exact binning of one view's prefix chunks) uses 512
  // threads, two Gaussians each, for a shorter chain per thread; the hit
  // words take one array per warp
  if (!kSkip && grid.x * grid.y < 148) {
    const size_t sm = smem + (512 / 32) * hit_bytes_per_warp;
    if (needs_smem_attr(sm))
      cudaFuncSetAttribute(bin_kernel<kShadow, kSkip, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)sm);
    bin_kernel<kShadow, kSkip, 512><<<grid, 512, sm, s>>>(a);
    return;
  }
  const size_t sm = smem + (kBinThreads / 32) * hit_bytes_per_warp;
  if (needs_smem_attr(sm))
    cudaFuncSetAttribute(bin_kernel<kShadow, kSkip, kBinThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sm);
  bin_kernel<kShadow, kSkip, kBinThreads><<<grid, kBinThreads, sm, s>>>(a);
}

// bin_prefix_kernel: staged means + transmittances, per-warp counters and
// segment masks; larger tile grids use the CTA-wide bin_kernel.
constexpr size_t kPrefixWarpBytes = 48 * 1024;
static size_t prefix_warp_bytes(const Dims& d, bool shadow, bool hits) {
  return (size_t)(kBinThreads / 32) * (((d.T + 1) / 2 + d.T) * (shadow ? 2 : 1) + (hits ? d.T : 0)) * 4;
}

bool prefix_hit_words(const Dims& d) { return d.T <= kHitBitsMaxTiles; }

template <bool kShadow>
static void launch_bin_prefix_t(const BinArgs& a, dim3 grid, size_t smem, cudaStream_t s) {
  if (needs_smem_attr(smem))
    cudaFuncSetAttribute(bin_prefix_kernel<kShadow>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  bin_prefix_kernel<kShadow><<<grid, kBinThreads, smem, s>>>(a);
}

cudaError_t launch_bin(const BinArgs& a, const Dims& d, int chunks, bool shadow, bool skip,
                       cudaStream_t s) {
  const dim3 grid(chunks, (a.nviews + a.views_per_cta - 1) / a.views_per_cta);
  // one view per warp needs views to fill the CTA's warps
  const bool hits = a.hbits != nullptr;
  if (!skip && a.views_per_cta >= kBinThreads / 32 && prefix_warp_bytes(d, shadow, hits) <= kPrefixWarpBytes) {
    const size_t smem = (size_t)4 * kChunk * 4 + prefix_warp_bytes(d, shadow, hits);
    if (shadow) launch_bin_prefix_t<true>(a, grid, smem, s);
    else launch_bin_prefix_t<false>(a, grid, smem, s);
    return cudaGetLastError();
  }
  if (skip && skip_bin_per_warp(d, shadow)) {
    const size_t smem = bin_skip_smem_bytes(d, a.cov_layout, shadow, a.skip_masks != 0);
    if (shadow) launch_bin_skip_t<true>(a, grid, smem, s);
    else launch_bin_skip_t<false>(a, grid, smem, s);
    return cudaGetLastError();
  }
  const bool masks = !skip && a.segmask != nullptr;
  const size_t smem = bin_smem_bytes(d, a.cov_layout, shadow, masks);
  const size_t hw = masks && hits ? (size_t)d.T * 4 : 0;
  if (shadow) {
    if (skip) launch_bin_t<true, true>(a, grid, smem, 0, s);
    else launch_bin_t<true, false>(a, grid, smem, hw, s);
  } else {
    if (skip) launch_bin_t<false, true>(a, grid, smem, 0, s);
    else launch_bin_t<false, false>(a, grid, smem, hw, s);
  }
  return cudaGetLastError();
}

bool bin_cell_supported(const Dims& d) { return warp_count_bytes(d, true) <= kWarpCountBytes; }

cudaError_t launch_bin_cand(const BinArgs& a, const Dims& d, bool shadow, cudaStream_t s) {
  const dim3 grid(kCandBlocks + kAlwaysBlocks, a.nviews);
  const size_t sm = open_stage_bytes(d.tiles_x, d.tiles_y, shadow ? 2 : 1);
  if (shadow) {
    if (sm) bin_cand_kernel<true, true><<<grid, kBinThreads, sm, s>>>(a);
    else bin_cand_kernel<true, false><<<grid, kBinThreads, 0, s>>>(a);
  } else {
    if (sm) bin_cand_kernel<false, true><<<grid, kBinThreads, sm, s>>>(a);
    else bin_cand_kernel<false, false><<<grid, kBinThreads, 0, s>>>(a);
  }
  return cudaGetLastError();
}

template <bool kShadow>
static void launch_bin_finalize_t(const BinArgs& a, dim3 grid, size_t smem, cudaStream_t s) {
  if (needs_smem_attr(smem))
    cudaFuncSetAttribute(bin_finalize_kernel<kShadow>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  bin_finalize_kernel<kShadow><<<grid, kBinThreads, smem, s>>>(a);
}

cudaError_t launch_bin_finalize(const BinArgs& a, const Dims& d, bool shadow, cudaStream_t s) {
  const int warps = kBinThreads / 32;
  const dim3 grid((a.chunks + warps - 1) / warps, a.nviews);
  const size_t smem = warp_count_bytes(d, shadow) + warp_mask_bytes(d, shadow, a.skip_masks != 0);
  if (shadow) launch_bin_finalize_t<true>(a, grid, smem, s);
  else launch_bin_finalize_t<false>(a, grid, smem, s);
  return cudaGetLastError();
}

cudaError_t launch_cell_prep(const CellPrepArgs& a, cudaStream_t s) {
  cell_init_kernel<<<(kMaxCells + 255) / 256, 256, 0, s>>>(a.grid, a.cell_hb, a.cell_count);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t blocks = min((int64_t)148 * 8, (a.n + 255) / 256);
  scene_bounds_kernel<<<(unsigned)max((int64_t)1, blocks), 256, 0, s>>>(a.means, a.n, a.grid);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  scene_grid_kernel<<<1, 32, 0, s>>>(a.grid, a.n);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cell_center_kernel<<<kMaxSpatialCells / 256, 256, 0, s>>>(a.grid, a.cell_center);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cell_assign_kernel<<<(unsigned)((a.n + 255) / 256), 256, 0, s>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cell_scan_blocks_kernel<<<kMaxCells / 1024, 1024, 0, s>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cell_scan_offsets_kernel<<<kMaxCells / 1024, 1024, 0, s>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess || a.n <= a.pstart) return e;
  cell_fill_kernel<<<(unsigned)((a.n - a.pstart + 255) / 256), 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_cell_test(const CellTestArgs& a, const Dims& d, int nviews, cudaStream_t s) {
  const size_t sm = open_stage_bytes(d.tiles_x, d.tiles_y, a.shadow ? 2 : 1);
  if (sm) cell_test_kernel<true><<<dim3(kMaxSpatialCells / 256, nviews), 256, sm, s>>>(a);
  else cell_test_kernel<false><<<dim3(kMaxSpatialCells / 256, nviews), 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_open_table(const OpenArgs& a, int nviews, int nlists, cudaStream_t s) {
  open_table_kernel<<<dim3(nviews, nlists), 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_scan(const ScanArgs& a, int nviews, cudaStream_t s) {
  // four tiles per lane for launches of many views (a few views would leave
  // the GPU with too few CTAs)
  const bool aligned4 = nviews >= 16 && (a.T % kScanTilesPerLane) == 0 &&
                        (reinterpret_cast<uintptr_t>(a.counts) & 3) == 0 && (a.counts_vstride & 3) == 0;
  if (aligned4)
    scan4_kernel<<<dim3((a.T + kScanTilesPerCta - 1) / kScanTilesPerCta, nviews), kScanThreads, 0, s>>>(a);
  else
    scan_kernel<<<dim3((a.T + 31) / 32, nviews), kScan1Threads, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_select(const SelectArgs& a, const Dims& d, int nviews, bool shadow_list,
                          cudaStream_t s) {
  const dim3 grid((d.T + kSelectThreads / 32 - 1) / (kSelectThreads / 32), nviews);
  const bool all = a.segmask && a.segmask_to >= a.C;
  if (all && nviews < kSelectCtaMaxViews) {
    // (every chunk with segment masks: the per-view path, rectangles at their
    // Gaussians' slots)
    if (shadow_list) select_cta_kernel<true><<<dim3(d.T, nviews), kSelectThreads, 0, s>>>(a);
    else select_cta_kernel<false><<<dim3(d.T, nviews), kSelectThreads, 0, s>>>(a);
    return cudaGetLastError();
  }
  if (shadow_list) {
    if (all) select_kernel<true, true><<<grid, kSelectThreads, 0, s>>>(a);
    else select_kernel<true, false><<<grid, kSelectThreads, 0, s>>>(a);
  } else {
    if (all) select_kernel<false, true><<<grid, kSelectThreads, 0, s>>>(a);
    else select_kernel<false, false><<<grid, kSelectThreads, 0, s>>>(a);
  }
  return cudaGetLastError();
}

#ifndef SARR_RENDER_MANY_PIX
#define SARR_RENDER_MANY_PIX 4
#endif
cudaError_t launch_render(const TileArgs& a, const Dims& d, int nviews, cudaStream_t s) {
  constexpr int kMany = SARR_RENDER_MANY_PIX;
  if (nviews >= 16)
    render_kernel<kMany><<<dim3(d.T, nviews), kTile * kTile / kMany, 0, s>>>(a);
  else
    render_kernel<1><<<dim3(d.T, nviews), 256, 0, s>>>(a);
  return cudaGetLastError();
}

#ifndef SARR_FUSE_SELECT_RENDER
#define SARR_FUSE_SELECT_RENDER 1
#endif
bool select_render_fusable(const SelectArgs& a, int nviews) {
  // the many-view compositing (render_kernel<4>) and a selection whose chunks
  // after the prefix have exact lists or none (select_kernel<false, false>)
  const bool all = a.segmask && a.segmask_to >= a.C;
  return SARR_FUSE_SELECT_RENDER && nviews >= 16 && SARR_RENDER_MANY_PIX == kFusedPix && !all;
}

cudaError_t launch_select_render(const SelectArgs& sa, const TileArgs& ta, const Dims& d,
                                 int nviews, cudaStream_t s) {
  select_render_kernel<<<dim3(d.T, nviews), kFusedThreads, 0, s>>>(sa, ta);
  return cudaGetLastError();
}

cudaError_t launch_omega_tile(const TileArgs& a, const Dims& d, int nviews, cudaStream_t s) {
  omega_tile_kernel<<<dim3(d.T, nviews), kWarpsPerTile * 32, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_omega_scatter(const OmegaScatterArgs& a, const Dims& d, int nviews,
                                 cudaStream_t s) {
  const int64_t total = d.n * nviews;
  const unsigned fill_blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16);
  omega_fill_kernel<<<fill_blocks, 256, 0, s>>>(a.omega, d.n, nviews, a.omega_vstride);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  count_launches(1);  // the second kernel of this launch step
  omega_listed_kernel<<<dim3((d.T * kCap + 255) / 256, nviews), 256, 0, s>>>(a);
  return cudaGetLastError();
}

#ifndef SARR_BWD_MANY_PIX
#define SARR_BWD_MANY_PIX 1
#endif
cudaError_t launch_bwd_tile(const TileArgs& a, const Dims& d, int nviews, cudaStream_t s) {
  if (SARR_BWD_MANY_PIX && nviews >= SARR_BWD_ONE_PART_MIN_VIEWS)
    bwd_tile4_kernel<1><<<dim3(d.T, nviews, 1), kTile * kTile / kBwdPix, 0, s>>>(a);
  else if (SARR_BWD_MANY_PIX && nviews >= kBwdManyMinViews)
    bwd_tile4_kernel<kBwdParts><<<dim3(d.T, nviews, kBwdParts), kTile * kTile / kBwdPix, 0, s>>>(a);
  else
    bwd_tile_kernel<<<dim3(d.T, nviews, kBwdParts), kWarpsPerTile * 32, 0, s>>>(a);
  return cudaGetLastError();
}

bool bwd_uses_index(int nviews) { return nviews > kDirectGatherMaxViews; }

cudaError_t launch_bwd_index(const BwdIndexArgs& a, cudaStream_t s) {
  if (!bwd_uses_index(a.nviews)) return cudaSuccess;
  cudaError_t e = cudaMemsetAsync(a.cnt, 0, (size_t)a.n * sizeof(int), s);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)((a.T * kCap + 255) / 256), (unsigned)a.nviews);
  bwd_index_kernel<false><<<grid, 256, 0, s>>>(a);
  const int nb = (int)((a.n + kGatherScanBlock - 1) / kGatherScanBlock);
  gather_scan_sums_kernel<<<nb, kGatherScanThreads, 0, s>>>(a.cnt, a.n, a.bsum);
  gather_scan_top_kernel<<<1, kGatherScanThreads, 0, s>>>(a.bsum, nb, a.start, a.n);
  gather_scan_apply_kernel<<<nb, kGatherScanThreads, 0, s>>>(a.cnt, a.n, a.bsum, a.start);
  bwd_index_kernel<true><<<grid, 256, 0, s>>>(a);
  count_launches(4);  // five kernels in this launch step
  return cudaGetLastError();
}

cudaError_t launch_bwd_scatter(const BwdScatterArgs& a, const Dims& d, cudaStream_t s) {
  (void)d;
  if (a.end <= a.begin) return cudaSuccess;
  const unsigned blocks = (unsigned)((a.end - a.begin + 255) / 256);
  if (!bwd_uses_index(a.nviews)) {
    bwd_gather_kernel<<<blocks, 256, 0, s>>>(a);
    return cudaGetLastError();
  }
  cudaError_t e = cudaMemsetAsync(a.heavy, 0, sizeof(int), s);
  if (e != cudaSuccess) return e;
  bwd_scatter_kernel<<<blocks, 256, 0, s>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  count_launches(1);  // the second kernel of this launch step
  int sms = 148, per_sm = 0, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, bwd_heavy_kernel, kHeavyWarps * 32, 0) !=
          cudaSuccess || per_sm < 1)
    per_sm = 1;
  bwd_heavy_kernel<<<sms * per_sm, kHeavyWarps * 32, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_debug_preprocess(const DebugPreArgs& a, cudaStream_t s) {
  const unsigned blocks = (unsigned)((a.n + 255) / 256);
  debug_preprocess_kernel<<<blocks, 256, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_debug_view(const ViewHost& vh, float* out, cudaStream_t s) {
  debug_view_kernel<<<1, 1, 0, s>>>(vh, out);
  return cudaGetLastError();
}

cudaError_t launch_debug_lists(const DebugListArgs& a, cudaStream_t s) {
  debug_lists_kernel<<<a.T, kCap, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace sarr
