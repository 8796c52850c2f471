// Internal interface between the C ABI layer (sarr_abi.cu) and the kernels
// (sarr_kernels.cu): memory layouts of the per-view state and the workspace,
// kernel argument blocks and launch wrappers.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "sarr_common.cuh"

namespace sarr {

// The library's launch counter (sarr_launch_count), for launch steps that
// issue more than one kernel.
void count_launches(int k);

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Image / tiling geometry of one call (all views of a call share it).
struct Dims {
  int64_t n;
  int Nr, Na;
  int tiles_x, tiles_y, T;
  int C;  // count rows: ceil(n / kChunk)
};

// Per-view forward state. The image-plane list is what the backward reuses;
// the shadow list (same layout, yz unused) only lives in the workspace.
//   rects  [n] u32   tile rectangle of each Gaussian (kEmptyRect when invalid)
//   count  [T] i32   list length (<= 64)
//   list   [T][64]   Gaussian ids in index order (the reference's tile list)
//   yz     [T][64]   (Y_r, Z_r) of list slot s (backward chain)
//   recs   [T][64]   Rec in compositing (Z_r, index) order
//   xbits  [n/32] u32 bit i: Gaussian i was binned exactly (cell binning)
//   xoff   [n/32] u16 per 32-Gaussian word: exactly binned Gaussians of the
//                    chunk in its earlier words
//   meta   int64     first Gaussian from which the chunks are sparse: only
//                    their exactly binned Gaussians have rectangles, stored
//                    compactly from the chunk's first slot in index order
//                    (INT64_MAX: every rectangle is at its Gaussian's slot)
struct StateLayout {
  size_t rects, count, list, yz, recs, xbits, xoff, meta, bytes;
};

__host__ __device__ inline StateLayout state_layout(int64_t n, int T) {
  StateLayout L;
  size_t o = 0;
  L.rects = o;
  o += align256((size_t)n * 4);
  L.count = o;
  o += align256((size_t)T * 4);
  L.list = o;
  o += align256((size_t)T * kCap * 4);
  L.yz = o;
  o += align256((size_t)T * kCap * 8);
  L.recs = o;
  o += align256((size_t)T * kCap * sizeof(Rec));
  L.xbits = o;
  o += align256((size_t)(n + 31) / 32 * 4);
  L.xoff = o;
  o += align256((size_t)(n + 31) / 32 * 2);
  L.meta = o;
  o += 256;
  L.bytes = o;
  return L;
}

// Tile rectangle of Gaussian i in a state whose exactness bits are those of
// `xs` (the image-plane state of the same view).
__device__ __forceinline__ uint32_t state_rect(const unsigned char* st, const StateLayout& L,
                                               const unsigned char* xs, const StateLayout& XL,
                                               int64_t i) {
  const uint32_t* rects = reinterpret_cast<const uint32_t*>(st + L.rects);
  const int64_t sparse_from = *reinterpret_cast<const int64_t*>(xs + XL.meta);
  if (i < sparse_from) return rects[i];
  const uint32_t word = reinterpret_cast<const uint32_t*>(xs + XL.xbits)[i >> 5];
  if (!((word >> (i & 31)) & 1u)) return kEmptyRect;
  const int k = reinterpret_cast<const uint16_t*>(xs + XL.xoff)[i >> 5] +
                __popc(word & ((1u << (i & 31)) - 1u));
  return rects[(i / kChunk) * kChunk + k];
}

// Workspace: [ViewConst x 32][error word][per-view areas x group]
//   per view: counts_ipp [C][T] u8, counts_sh [C][T] u8, need_ipp / need_sh
//   [T][64] int4 and need_n_ipp / need_n_sh [T] i32 (the chunks holding each
//   tile's list, from scan_kernel), open_ipp / open_sh [tiles_y+1][tiles_x+1]
//   i32 (summed-area tables of the tiles still open after the saturation
//   prefix, from open_table_kernel), state_ipp (used when the caller gives no
//   state), state_sh, partial_om [T][64] float2, partial_bwd [T][64][8] float,
//   entries [T][64] u32 (the backward's list entries grouped by Gaussian:
//   the group's views' slices form one array indexed by g_start).
// The head also holds the backward's inverse index of the list entries:
// g_cnt [n], g_start [n + 1] (exclusive scan) and g_bsum (scan block sums).
// With cells (multi-view calls, see kCellMinViews) the head also holds the
// SceneGrid, per-Gaussian bbox bounds hb [n] f32 and cell ids cid [n] u32, the
// per-cell largest bound cell_hb [kMaxCells] (ordered-int keys), the cells'
// member lists (Gaussians after the prefix, cell by cell: cell_start
// [kMaxCells + 1], mem_pos [n] float4 = centre and bound, mem_idx [n]), the
// Gaussians after the prefix that are in no cell (always [n]) and, per view of
// a launch group, the number of nonzero cell-bitmap words (cand_count
// [kMaxViewsPerLaunch]); each view area holds its cell bitmap bits
// [kCellWords] u32, the indices of its nonzero words (cand_words
// [kCellWords] u32) and, for images of at most kHitBitsMaxTiles tiles, the
// hit words of the first kPrefixStage1 chunks (hbits [kPrefixStage1][T][32]
// u32, see BinArgs::hbits).
struct WsLayout {
  size_t viewconst, err, scene, hb, cid, cell_hb, cell_count, cell_start, cell_center, mem_pos, mem_idx,
      always, cand_count, g_cnt, g_start, g_bsum, g_heavy, head;
  size_t counts_ipp, counts_sh, need_ipp, need_sh, need_n_ipp, need_n_sh, open_ipp, open_sh;
  size_t bits, cand_words, hbits, xcount, xlist, segmask_ipp, segmask_sh, state_ipp, state_sh, partial_om, partial_bwd,
      entries, per_view;
  bool cells;
  StateLayout st;
};

// Cell culling applies to calls of at least kCellMinViews views whose
// Gaussians extend past the exactly binned prefix.
__host__ inline bool cells_eligible(const Dims& d, int n_views) {
  return n_views >= kCellMinViews && d.C > kPrefixChunks;
}

__host__ inline WsLayout ws_layout(const Dims& d, bool cells) {
  WsLayout L;
  L.cells = cells;
  L.viewconst = 0;
  L.err = align256(sizeof(ViewConst) * kMaxViewsPerLaunch);
  size_t h = L.err + 256;
  L.scene = L.hb = L.cid = L.cell_hb = L.cell_count = L.cell_start = L.cell_center = 0;
  L.mem_pos = L.mem_idx = L.always = L.cand_count = 0;
  if (cells) {
    L.scene = h;
    h += align256(sizeof(SceneGrid));
    L.hb = h;
    h += align256((size_t)d.n * 4);
    L.cid = h;
    h += align256((size_t)d.n * 4);
    L.cell_hb = h;
    h += align256((size_t)kMaxCells * 4);
    L.cell_count = h;
    h += align256((size_t)kMaxCells * 4);
    L.cell_start = h;
    h += align256((size_t)(kMaxCells + 1) * 4);
    L.cell_center = h;
    h += align256((size_t)kMaxSpatialCells * 16);
    L.mem_pos = h;
    h += align256((size_t)d.n * 16);
    L.mem_idx = h;
    h += align256((size_t)d.n * 4);
    L.always = h;
    h += align256((size_t)d.n * 4);
    L.cand_count = h;
    h += align256((size_t)kMaxViewsPerLaunch * 4);
  }
  // the backward's inverse index: list entries per Gaussian, their offsets
  // (exclusive scan) and the scan's per-block sums
  L.g_cnt = h;
  h += align256((size_t)d.n * 4);
  L.g_start = h;
  h += align256((size_t)(d.n + 1) * 4);
  L.g_bsum = h;
  h += align256((size_t)((d.n + kGatherScanBlock - 1) / kGatherScanBlock + 1) * 4);
  L.g_heavy = h;  // [0]: count, then the Gaussians with many list entries
  h += align256((size_t)(d.n + 1) * 4);
  L.head = h;
  L.st = state_layout(d.n, d.T);
  size_t o = 0;
  L.counts_ipp = o;
  o += align256((size_t)d.C * d.T);
  L.counts_sh = o;
  o += align256((size_t)d.C * d.T);
  L.need_ipp = o;
  o += align256((size_t)d.T * kCap * 16);
  L.need_sh = o;
  o += align256((size_t)d.T * kCap * 16);
  L.need_n_ipp = o;
  o += align256((size_t)d.T * 4);
  L.need_n_sh = o;
  o += align256((size_t)d.T * 4);
  L.open_ipp = o;
  o += align256((size_t)(d.tiles_y + 1) * (d.tiles_x + 1) * 4);
  L.open_sh = o;
  o += align256((size_t)(d.tiles_y + 1) * (d.tiles_x + 1) * 4);
  // Per chunk after the prefix: how many of its Gaussians the skipping binner
  // binned exactly (-1: more than kXCap, or not recorded) and their chunk
  // offsets in index order; select_kernel scans only those.
  // Per chunk and tile: which 32-Gaussian segments of the chunk hold hits of
  // the tile (select_kernel reads only those); for every chunk up to
  // kSegMaskAllMaxTiles tiles, for the prefix chunks otherwise.
  const size_t mchunks = d.T <= kSegMaskAllMaxTiles ? (size_t)d.C : (size_t)kPrefixChunks;
  L.segmask_ipp = o;
  o += align256(mchunks * d.T * 4);
  L.segmask_sh = o;
  o += align256(mchunks * d.T * 4);
  L.xcount = o;
  o += align256((size_t)d.C * 4);
  L.xlist = o;
  o += align256((size_t)d.C * kXCap * 2);
  L.bits = L.cand_words = L.hbits = 0;
  if (cells) {
    L.bits = o;
    o += align256((size_t)kCellWords * 4);
    L.cand_words = o;
    o += align256((size_t)kCellWords * 4);
    if (d.T <= kHitBitsMaxTiles) {
      L.hbits = o;
      o += align256((size_t)kPrefixStage1 * d.T * 32 * 4);
    }
  }
  L.state_ipp = o;
  o += L.st.bytes;
  L.state_sh = o;
  o += L.st.bytes;
  L.partial_om = o;
  o += align256((size_t)d.T * kCap * 8);
  L.partial_bwd = o;
  o += align256((size_t)d.T * kCap * 8 * 4);
  L.entries = o;
  o += align256((size_t)d.T * kCap * 4);
  L.per_view = o;
  return L;
}

// A strided family of per-view state buffers.
struct StateRef {
  unsigned char* base;
  size_t vstride;
  StateLayout L;
};

struct BinArgs {
  const ViewConst* views;
  int nviews;
  int views_per_cta;  // views handled by one CTA (grid.y = ceil(nviews / views_per_cta))
  int chunk_offset;   // first chunk of this launch
  const int* open_ipp;  // open-tile summed-area tables (skip variant), open_vstride ints per view
  const int* open_sh;
  size_t open_vstride;
  uint32_t* segmask;     // segment masks [chunk][T] (null: none)
  int skip_masks;        // the skipping binners write the masks of their chunks too
  // nullable: hit words of the image list [chunk][T][32] (bit l of word r:
  // Gaussian 32 r + l of the chunk hits the tile), written by
  // bin_prefix_kernel for chunks < hbits_to where nonzero
  uint32_t* hbits;
  size_t hbits_vstride;  // words per view
  int hbits_to;
  uint32_t* segmask_sh;
  size_t segmask_vstride;  // words per view
  int* xcount;         // exactly binned Gaussians per chunk (skip variants)
  uint16_t* xlist;     // [C][kXCap] their chunk offsets
  size_t x_vstride;    // bytes per view of both
  // cell variant
  int chunks;          // chunks after the prefix
  const SceneGrid* grid;
  const int* cell_start;
  const float4* mem_pos;
  const int* mem_idx;
  const int* always;
  const uint32_t* bits;  // cell bitmaps, bits_vstride words per view
  size_t bits_vstride;
  const int* cand_count;        // per view: bitmap words with a candidate cell
  const uint32_t* cand_words;   // their indices, cand_vstride words per view
  size_t cand_vstride;
  // exactly-binned bitmaps: the xbits of the image-plane states (ipp)
  int64_t n;
  int C;
  const float* means;
  const float* cov;
  int cov_layout;
  const float* sigma;
  StateRef ipp;  // rects written into ipp.base + v * vstride + L.rects
  StateRef sh;   // used when the shadow list is built
  uint8_t* counts_ipp;
  uint8_t* counts_sh;
  size_t counts_vstride;
  int use_tma;
  int* err;
};

struct CellPrepArgs {
  int64_t n;
  int64_t pstart;  // first Gaussian after the exactly binned prefix
  const float* means;
  const float* cov;
  int cov_layout;
  const float* sigma;
  SceneGrid* grid;
  float* hb;
  uint32_t* cid;
  int* cell_hb;
  int* cell_count;
  int* cell_start;
  float4* cell_center;  // [kMaxSpatialCells] centre of each spatial cell
  float4* mem_pos;
  int* mem_idx;
  int* always;
};

struct CellTestArgs {
  const ViewConst* views;
  const SceneGrid* grid;
  const float4* cell_center;
  const int* cell_hb;
  const int* open_ipp;
  const int* open_sh;
  size_t open_vstride;
  int shadow;
  uint32_t* bits;
  size_t bits_vstride;
  int* cand_count;       // per view: nonzero bitmap words (cleared by open_table_kernel)
  uint32_t* cand_words;  // their indices, in no particular order
  size_t cand_vstride;
  StateRef ipp;          // its xbits are cleared and its meta set (sparse rectangles)
  int64_t sparse_from;   // first Gaussian after the prefix
  int64_t n;
};

struct SelectArgs {
  const ViewConst* views;
  int64_t n;
  int C;
  const float* means;
  const float* cov;
  int cov_layout;
  const float* sigma;
  const float* sh;
  int sh_stride;
  int sh_k;
  StateRef st;
  const unsigned char* need;  // int4 [T][64] per view: chunk, hits before, hits in chunk
  size_t need_vstride;        // bytes
  const int* need_n;          // [T] per view
  size_t need_n_vstride;      // ints
  const uint32_t* segmask;    // segment masks of chunks < segmask_to (null: none)
  size_t segmask_vstride;     // words
  int segmask_to;
  const uint32_t* hbits;      // hit words of chunks < hbits_to (null: none); read
  size_t hbits_vstride;       // only where the segment mask has the word's bit
  int hbits_to;
  StateRef xs;                // image-plane states: exactness bits and meta of the rectangles
  int xlist_from;             // first chunk with an exact list (INT32_MAX: none)
  const int* xcount;
  const uint16_t* xlist;
  size_t x_vstride;           // bytes
  int* err;
};

// Open-tile tables of up to two lists (blockIdx.y selects the list).
struct OpenArgs {
  int tiles_x, tiles_y, prefix_chunks;
  const uint8_t* counts[2];
  size_t counts_vstride;
  int* table[2];
  size_t table_vstride;  // ints
  int* cand_count;       // nullable: per view, cleared here for cell_test_kernel
};

struct ScanArgs {
  int T, C;
  const uint8_t* counts;
  size_t counts_vstride;
  StateRef st;  // receives the list lengths
  unsigned char* need;
  size_t need_vstride;
  int* need_n;
  size_t need_n_vstride;
};

struct TileArgs {
  const ViewConst* views;
  StateRef st;
  float* images;  // render: output; backward: (const) grad images
  size_t img_vstride;
  float* partial;  // omega: float2 [T][64]; backward: float [T][64][8]
  size_t partial_vstride;
  int* err;
};

struct OmegaScatterArgs {
  const ViewConst* views;
  int64_t n;
  StateRef sh;
  StateRef ipp;  // exactness bits of the rectangles
  const float* partial;
  size_t partial_vstride;
  float* omega;
  size_t omega_vstride;
};

struct BwdScatterArgs {
  const ViewConst* views;
  int nviews;
  int64_t n;
  StateRef ipp;
  const float* partial;
  size_t partial_vstride;
  float* grad_means;
  float* grad_cov;
  int grad_cov_layout;
  float* grad_sigma;
  float* grad_sh;
  int grad_sh_cols;
  float* grad_norm;
  int accumulate;
  // the inverse index (launch_bwd_index): Gaussian i's list entries are
  // entries[start[i] .. start[i+1]), entry e at entries + (e / per) *
  // entries_vstride + e % per (per = T * 64), packed view << 24 | tile << 6 | slot
  const int* start;
  const uint32_t* entries;
  size_t entries_vstride;  // u32 per view
  int64_t begin, end;      // the gradient rows written: Gaussians [begin, end)
  int64_t row0;            // Gaussian i's gradient row is i - row0 (0 or begin)
  int* heavy;              // [0]: count, [1..]: Gaussians left to bwd_heavy_kernel
};

// The inverse index of a group's image-plane tile lists for the backward.
struct BwdIndexArgs {
  int nviews;
  int64_t n;
  int T;
  StateRef ipp;
  int* cnt;       // [n], zero on entry, zero again on return
  int* start;     // [n + 1]
  int* bsum;      // [ceil(n / kGatherScanBlock) + 1]
  uint32_t* entries;
  size_t entries_vstride;
};

struct DebugPreArgs {
  ViewHost vh;
  int64_t n;
  const float* means;
  const float* cov;
  int cov_layout;
  const float* sigma;
  const float* sh;
  int sh_stride;
  int sh_k;
  float* f32;
  int32_t* i32;
};

struct DebugListArgs {
  int T;
  StateRef st;
  int32_t* counts;
  int32_t* lists;
  int32_t* sorted;
};

// Launch wrappers; each returns the cudaError_t of the launch.
// view constants of a group (and, when err_to_clear is set, the error word cleared)
cudaError_t launch_view_setup(const ViewHostPack& pack, ViewConst* out, int* err_to_clear,
                              cudaStream_t s);
// bin_kernel over chunks [a.chunk_offset, a.chunk_offset + chunks)
cudaError_t launch_bin(const BinArgs& a, const Dims& d, int chunks, bool shadow, bool skip,
                       cudaStream_t s);
cudaError_t launch_open_table(const OpenArgs& a, int nviews, int nlists, cudaStream_t s);
// view-independent cell grid of one call (four kernels)
cudaError_t launch_cell_prep(const CellPrepArgs& a, cudaStream_t s);
cudaError_t launch_cell_test(const CellTestArgs& a, const Dims& d, int nviews, cudaStream_t s);
// cell binning of the a.chunks chunks from a.chunk_offset: bin_cand_kernel
// (candidate cells' members), then bin_finalize_kernel (per chunk)
cudaError_t launch_bin_cand(const BinArgs& a, const Dims& d, bool shadow, cudaStream_t s);
cudaError_t launch_bin_finalize(const BinArgs& a, const Dims& d, bool shadow, cudaStream_t s);
bool bin_cell_supported(const Dims& d);
// Whether the exact prefix binners can keep hit words (BinArgs::hbits) for
// this tile grid (both bin_prefix_kernel and bin_kernel write them).
bool prefix_hit_words(const Dims& d);
// true when the skipping binner keeps per-warp counters (and records the
// exact lists); false selects its CTA-wide variant
bool skip_bin_per_warp(const Dims& d, bool shadow);
int skip_bin_wave(const Dims& d, int cov_layout, bool shadow, bool masks);
bool segmask_supported(const Dims& d);
bool segmask_all_chunks(const Dims& d);
cudaError_t launch_scan(const ScanArgs& a, int nviews, cudaStream_t s);
cudaError_t launch_select(const SelectArgs& a, const Dims& d, int nviews, bool shadow_list,
                          cudaStream_t s);
cudaError_t launch_render(const TileArgs& a, const Dims& d, int nviews, cudaStream_t s);
// Whether a launch of the image list's selection and compositing may run as
// the one select_render_kernel (image-only calls of many views).
bool select_render_fusable(const SelectArgs& a, int nviews);
cudaError_t launch_select_render(const SelectArgs& sa, const TileArgs& ta, const Dims& d,
                                 int nviews, cudaStream_t s);
cudaError_t launch_omega_tile(const TileArgs& a, const Dims& d, int nviews, cudaStream_t s);
cudaError_t launch_omega_scatter(const OmegaScatterArgs& a, const Dims& d, int nviews,
                                 cudaStream_t s);
cudaError_t launch_bwd_tile(const TileArgs& a, const Dims& d, int nviews, cudaStream_t s);
cudaError_t launch_bwd_scatter(const BwdScatterArgs& a, const Dims& d, cudaStream_t s);
// the inverse index: count entries per Gaussian, scan, fill (five kernels);
// calls of a few views use none (bwd_uses_index)
bool bwd_uses_index(int nviews);
cudaError_t launch_bwd_index(const BwdIndexArgs& a, cudaStream_t s);
cudaError_t launch_debug_preprocess(const DebugPreArgs& a, cudaStream_t s);
cudaError_t launch_debug_lists(const DebugListArgs& a, cudaStream_t s);
cudaError_t launch_debug_view(const ViewHost& vh, float* out, cudaStream_t s);

}  // namespace sarr
