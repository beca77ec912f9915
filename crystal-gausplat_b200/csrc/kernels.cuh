// kernels.cuh — kernel argument blocks and launchers (internal).
#pragma once
#include "common.cuh"

namespace gs {

constexpr int kMaxBatchViews = GSC_MAX_BATCH_VIEWS;

// Preprocess of `nviews` views of one size (the per-Gaussian outputs mean2d ..
// tiles_touched are written only when nviews == 1).
struct PreprocessArgs {
  int64_t n;
  const float* pos;
  const float* log_scale;
  const float* rot;
  const float* logit_opacity;
  const float* sh;
  gsc_raster_config cfg;
  int tiles_x, tiles_y;
  int nviews;
  gsc_camera cams[kMaxBatchViews];
  float* splats_v[kMaxBatchViews];
  // bits(depth) (~0 if the Gaussian emits no pair) << 32 | index; may be null.
  // With view_key: view << 60 | bits(depth) << 28 | index (index < 2^28), the
  // words of all views sorted together by bits [28, 64).
  uint64_t* depth_pairs_v[kMaxBatchViews];
  int view_key;
  // with view_key and depth_compact: view << 56 | (bits(depth) - depth_base,
  // 2^28 - 1 if no pair) << 28 | index, sorted by bits [28, 56 + view bits);
  // the host sets it only when every emitted depth (near_z, far_z] maps below
  // 2^28 - 1
  int depth_compact;
  uint32_t depth_base;
  // contributing-pairs binning: the binning record's mask has bit k for the
  // k-th tile of the rect (row-major) that can contribute (~0 = the whole
  // rect), and the pair count is theirs
  int contributing;
  // if set: the binning record of each Gaussian, 32 B (one sector) that the
  // depth-ordered gathers of the pair counting and the emission read:
  // {x0, y0, rect width, pair count}, {mask low, mask high, 0, 0}
  uint4* bin_v[kMaxBatchViews];
  // if set: per view, += the pairs every Gaussian emits (zeroed by the host)
  unsigned long long* pair_total_v[kMaxBatchViews];
  float* mean2d;
  float* cov2d;
  float* conic;
  float* depth;
  float* radius;
  float* colors;
  float* opacity;
  uint32_t* tiles_touched;
  float* cov3d;
};

struct CompositeFwdArgs {
  const float* splats;
  const uint32_t* vals;
  const uint32_t* ranges;
  int width, height, tiles_x, tiles_y;
  float t_stop, alpha_min, alpha_max, power_cut;
  float bg[3];
  float* image;
  uint32_t* n_contrib;
  float* final_T;
  uint32_t* last;
  unsigned long long* pge;  // if set: += pixel-Gaussian evaluations (tile-list entries visited)
  uint32_t* tile_work;         // if set: per tile, the largest per-pixel `last` (backward list length)
  // Depth-sliced binning: the tile lists come in slices of the depth order and
  // each launch composites one slice on top of the per-pixel state the
  // previous one left (C in image, T in final_T, n_contrib, last). With
  // tile_base (per tile: entries of the earlier slices, the list index of this
  // slice's first entry) null there is one slice.
  uint32_t* tile_base;
  // one bit per tile (done_words 64-bit words per tile row): every pixel
  // stopped (set by a slice, read by the next)
  unsigned long long* tile_done;
  int done_words;
  int first_slice, last_slice;
  // per-tile cut of the slices (tile hint): a first slice sets *open_flag when
  // a tile whose pixels did not all stop has a finite cut (it may have
  // second-slice pairs); mark_done: the last slice also marks its done tiles
  const float* tile_cut;
  unsigned int* open_flag;
  int mark_done;
};

struct CompositeBwdArgs {
  const float* splats;
  const uint32_t* vals;
  const uint32_t* ranges;
  int width, height, tiles_x, tiles_y;
  float alpha_min, alpha_max, power_cut;
  float bg[3];
  const float* dL_dimage;
  const float* image;
  const float* target;
  float l1_scale;
  const float* final_T;
  const uint32_t* last;
  float* grad2d;
  float* loss_sum;
  const uint32_t* tile_order;  // if set: block b composites tile tile_order[b]
};

struct PreprocessBwdArgs {
  int64_t n;
  const float* pos;
  const float* log_scale;
  const float* rot;
  const float* logit_opacity;
  const float* sh;
  gsc_camera cam;
  gsc_raster_config cfg;
  const float* grad2d;
  float* g_pos;
  float* g_log_scale;
  float* g_rot;
  float* g_logit_opacity;
  float* g_sh;
  float* d_mean2d;
  float* d_cov2d;
  float* d_opacity;
  float* d_colors;
  // FULL mode: views summed by one launch (cam / grad2d above are view 0)
  int nviews;
  const float* grad2d_v[kMaxBatchViews];
  gsc_camera cams[kMaxBatchViews];
};

constexpr int kMaxAdamGroups = 8;

struct AdamGroupDev {
  float* param;
  const float* grad;
  float* m;
  float* v;
  int64_t numel;
  float lr;
  float weight_decay;
  float decay;  // 1 - lr * weight_decay
  int vec;      // all four pointers 16-byte aligned
};

struct AdamArgs {
  AdamGroupDev g[kMaxAdamGroups];
  int64_t chunk_end[kMaxAdamGroups];  // inclusive prefix of ceil(numel/4)
  int ngroups;
  float beta1, beta2, eps, bc1, bc2, grad_scale;
};

int launch_preprocess(const PreprocessArgs& a, cudaStream_t stream);
int launch_block_sums(const float* splats, int64_t n, uint32_t* sums, cudaStream_t stream);
int launch_scan_block_sums(const uint32_t* sums, int64_t nb, uint64_t* offsets, uint64_t* total,
                           cudaStream_t stream);
int launch_emit_keys(const float* splats, int64_t n, const uint64_t* offsets, int tiles_x,
                     int tiles_y, uint64_t* keys, uint32_t* vals, cudaStream_t stream);
int launch_tile_ranges(const uint64_t* keys, int64_t n, int32_t num_tiles, uint32_t* ranges,
                       cudaStream_t stream);
// Depth-sliced binning (GSC_BIN_OCCLUDED): at most kMaxSlices slices of the depth order.
constexpr int kMaxSlices = 4;
// Pair count of each 256-position chunk of `order`. With tile_done (one bit
// per tile, done_words 64-bit words per tile row), Gaussians whose listed
// tiles are all done count 0 and get their bit in skip_bits.
int launch_block_sums_gather(const uint4* bins, const uint32_t* order, int64_t n, uint32_t* sums,
                             cudaStream_t stream, const unsigned long long* tile_done = nullptr,
                             int done_words = 0, uint32_t* skip_bits = nullptr);
// 64-bit words per tile row of a tile-done bit set
inline int done_words_of(int tiles_x) { return (tiles_x + 63) / 64; }
// *dst += *src on the device (tracing counters).
int launch_add_u64(const uint64_t* src, unsigned long long* dst, cudaStream_t stream);
// Per tile, the first keep[t] entries of the slices' lists, concatenated;
// *total (device) = their count.
int launch_concat_slices(const uint32_t* const* slice_vals, const uint32_t* const* slice_ranges, int nslices,
                         const uint32_t* keep, int32_t num_tiles, uint32_t* out_vals, uint32_t* out_ranges,
                         uint64_t* total, cudaStream_t stream);
// Per-tile depth cut of occluded binning (a tile hint): the pairs of a view
// are split into the pairs (g, t) with !(depth(g) >= cut[t]) (mode 0: the
// first slice, a depth prefix of every tile's list) and those with
// depth(g) >= cut[t] whose tile is not done (mode 1: the second slice). The
// binning record's third word of its second half holds bits(depth).
struct TileCut {
  const float* cut = nullptr;                  // per tile; null: no cut
  const unsigned long long* done = nullptr;    // mode 1: tile-done bits
  int done_words = 0;
  int mode = 0;
  int tiles_x = 0;
  uint64_t* sub = nullptr;  // per position: the record's passing tiles (records of <= 64 tiles)
  uint32_t* cnt = nullptr;  // per position: number of passing tiles
  const unsigned int* open = nullptr;  // mode 1: 0 if no tile can have a second-slice pair
};
// Pair count of each 256-position chunk of `order` under a tile cut, with
// every position's count and sub-mask (tc.cnt, tc.sub).
int launch_block_sums_cut(const uint4* bins, const uint32_t* order, int64_t n, uint32_t* sums, const TileCut& tc,
                          cudaStream_t stream);
// Next cut of every tile after a view's last slice: done tiles (every pixel
// stopped) get (1 + margin) x the depth of the last entry any pixel used
// (entry keep[t] - 1 of the final list), the others +inf.
int launch_tile_cut_update(const uint32_t* ranges, const uint32_t* vals, const uint32_t* keep,
                           const unsigned long long* done, int done_words, int32_t tiles_x, int32_t num_tiles,
                           const float* splats, float margin, float* cut_out, cudaStream_t stream);
// hist (may be null): the tile sort's digit counts of the tile bits, digit d of
// pass q at hist[(q * 256 + d) * kHistStride]; ranges (may be null): preset to
// {0xFFFFFFFF, 0} for num_tiles tiles; grid_cap (> 0): at most that many blocks.
constexpr int kHistStride = 32;
int launch_emit_tiles(const uint4* bins, const uint32_t* order, int64_t n, const uint64_t* offsets,
                      int tiles_x, uint64_t* pair_out, cudaStream_t stream, uint32_t* hist = nullptr,
                      int hist_passes = 0, uint32_t* ranges = nullptr, int32_t num_tiles = 0,
                      int64_t grid_cap = 0, const uint32_t* skip_bits = nullptr, const TileCut* tc = nullptr);
// Tiles in decreasing order of their work (log-spaced buckets, 4 per
// octave), so that the compositing's last wave holds the short tiles: work
// = range length (ranges given) or tile_work[t].
int launch_tile_order(const uint32_t* ranges, const uint32_t* tile_work, int32_t num_tiles, uint32_t* order,
                      cudaStream_t stream);
// empty ranges {0xFFFFFFFF, 0} -> {0, 0}
int launch_ranges_finish(uint32_t* ranges, int32_t num_tiles, cudaStream_t stream);
// 64-bit keys (tile << 32 | bits(depth)) from the tile ranges and the ids
int launch_make_keys_ranges(const uint32_t* ranges, int32_t num_tiles, const uint32_t* ids, const float* splats,
                            uint64_t* keys, cudaStream_t stream);
int launch_tile_ranges_u32(const uint32_t* tiles, int64_t n, int32_t num_tiles, uint32_t* ranges,
                           cudaStream_t stream);
size_t sort_scratch_bytes(int64_t n, int begin_bit, int end_bit);
// The sort's look-back wait against a predecessor that never publishes (needs
// 2 KB of zeroable scratch); it gives up after spin_limit re-reads.
int launch_lookback_selftest(gsc_ctx* ctx, uint32_t spin_limit, char* scratch);
int launch_sort_pairs(gsc_ctx* ctx, uint64_t* keys, uint32_t* vals, int64_t n, int begin_bit,
                      int end_bit, char* scratch);
size_t sort_scratch_bytes_u32(int64_t n, int begin_bit, int end_bit);
// Stable sort of packed u64 (key << 32 | value) by bits [begin_bit, end_bit) of
// the u64; the sorted words go to hi_out (may be null) / lo_out (low word &
// lo_mask). `pairs` is overwritten.
size_t sort_scratch_bytes_packed(int64_t n, int begin_bit, int end_bit);
// With hist_ready the digit histograms are already in the scratch (zeroed by
// sort_packed_clear, filled by the producer of `pairs`, e.g. emit_tiles, at
// stride kHistStride: sort_packed_hist). With
// `ranges` (begin_bit 32, every tile bit sorted, ranges preset to
// {0xFFFFFFFF, 0} per tile) the last pass also writes each tile's range.
int launch_sort_packed(gsc_ctx* ctx, uint64_t* pairs, int64_t n, int begin_bit, int end_bit, uint32_t* hi_out,
                       uint32_t* lo_out, char* scratch, uint32_t lo_mask = 0xFFFFFFFFu, bool hist_ready = false,
                       uint32_t* ranges = nullptr, uint32_t ntiles = 0, const uint64_t* n_dev = nullptr);
uint32_t* sort_packed_hist(char* scratch, int64_t n, int begin_bit, int end_bit);  // wide digit counts
int sort_packed_clear(gsc_ctx* ctx, int64_t n, int begin_bit, int end_bit, char* scratch);
int launch_sort_pairs_u32(gsc_ctx* ctx, uint32_t* keys, uint32_t* vals, int64_t n, int begin_bit,
                          int end_bit, char* scratch);
int launch_composite_fwd(const CompositeFwdArgs& a, cudaStream_t stream);
int launch_composite_bwd(const CompositeBwdArgs& a, bool full, cudaStream_t stream);
int launch_preprocess_bwd(const PreprocessBwdArgs& a, bool full, cudaStream_t stream);
// FULL mode over the Gaussians with a screen-space gradient in some view only
// (scratch: preprocess_bwd_compact_scratch(n) bytes).
int launch_preprocess_bwd_compact(const PreprocessBwdArgs& a, char* scratch, int num_sms, cudaStream_t stream);
size_t preprocess_bwd_compact_scratch(int64_t n);
int launch_adam(const AdamArgs& a, cudaStream_t stream);
int launch_l1(const float* pred, const float* target, int64_t numel, float scale, float* grad,
              float* loss_sum, int num_sms, cudaStream_t stream);

}  // namespace gs
