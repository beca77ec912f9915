// binning.cu — tile binning: exact key allocation and canonical key emission
// (replacing create_tile_keys, src/metal/kernels/gaussian.metal:315-357, whose
// atomic slot counter gives a nondeterministic order and has no bound check),
// and tile ranges (init_tile_ranges + compute_tile_ranges,
// src/metal/kernels/radix_sort.metal:288-324).
//
// Allocation: preprocess leaves one tiles_touched sum per 256-Gaussian block;
// scan_block_sums_kernel turns them into 64-bit exclusive offsets and the
// total. Emission: each block owns the contiguous key range
// [offset[b], offset[b] + sum[b]) and fills it with coalesced stores, every
// thread locating the Gaussian of its output slot by binary search over the
// block's inclusive scan. Canonical order: Gaussian id, then ty, then tx.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "kernels.cuh"

namespace gs {

// Inclusive scan of one u32 per thread over a 256-thread block.
__device__ __forceinline__ uint32_t block_incl_scan_256(uint32_t v, uint32_t* s_warp) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    uint32_t t = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += t;
  }
  if (lane == 31) s_warp[w] = v;
  __syncthreads();
  uint32_t add = 0;
  for (int k = 0; k < w; k++) add += s_warp[k];
  __syncthreads();
  return v + add;
}

__global__ void __launch_bounds__(1024) scan_block_sums_kernel(const uint32_t* sums, int64_t nb,
                                                                uint64_t* offsets, uint64_t* total) {
  __shared__ uint64_t s_warp[32];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int64_t chunk = (nb + 1023) / 1024;
  const int64_t lo = min(nb, (int64_t)tid * chunk), hi = min(nb, lo + chunk);
  uint64_t mine = 0;
  for (int64_t k = lo; k < hi; k++) mine += sums[k];
  uint64_t v = mine;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    uint64_t t = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += t;
  }
  if (lane == 31) s_warp[w] = v;
  __syncthreads();
  if (w == 0) {
    uint64_t x = s_warp[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      uint64_t t = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += t;
    }
    s_warp[lane] = x;
  }
  __syncthreads();
  uint64_t run = (v - mine) + (w > 0 ? s_warp[w - 1] : 0);
  for (int64_t k = lo; k < hi; k++) {
    offsets[k] = run;
    run += sums[k];
  }
  if (tid == 1023) *total = s_warp[31];
}

__global__ void __launch_bounds__(256) emit_keys_kernel(const float4* __restrict__ splats, int64_t n,
                                                        const uint64_t* __restrict__ offsets,
                                                        int tiles_x, int tiles_y,
                                                        uint64_t* __restrict__ keys,
                                                        uint32_t* __restrict__ vals) {
  __shared__ uint32_t s_incl[256];
  __shared__ int s_x0[256], s_y0[256], s_wx[256];
  __shared__ uint32_t s_depth[256];
  __shared__ uint32_t s_warp[8];
  const int64_t base = (int64_t)blockIdx.x * 256;
  const int64_t i = base + threadIdx.x;
  uint32_t t = 0;
  if (i < n) {
    const float4 s0 = splats[i * 3], s2 = splats[i * 3 + 2];
    t = __float_as_uint(s2.w);
    if (t) {
      int x0, x1, y0, y1;
      tile_bounds(s0.x, s0.y, s2.z, tiles_x, tiles_y, &x0, &x1, &y0, &y1);
      s_x0[threadIdx.x] = x0;
      s_y0[threadIdx.x] = y0;
      s_wx[threadIdx.x] = x1 - x0 + 1;
      s_depth[threadIdx.x] = __float_as_uint(s2.y);
    }
  }
  uint32_t incl = block_incl_scan_256(t, s_warp);
  s_incl[threadIdx.x] = incl;
  __syncthreads();
  const uint32_t total = s_incl[255];
  const uint64_t out = offsets[blockIdx.x];
  for (uint32_t k = threadIdx.x; k < total; k += 256) {
    int lo = 0, hi = 255;  // smallest j with s_incl[j] > k
    while (lo < hi) {
      int mid = (lo + hi) >> 1;
      if (s_incl[mid] > k) hi = mid; else lo = mid + 1;
    }
    const uint32_t excl = lo ? s_incl[lo - 1] : 0u;
    const uint32_t local = k - excl;
    const int wx = s_wx[lo];
    const int ty = s_y0[lo] + (int)(local / (uint32_t)wx);
    const int tx = s_x0[lo] + (int)(local % (uint32_t)wx);
    const uint64_t tile = (uint64_t)(uint32_t)(ty * tiles_x + tx);
    keys[out + k] = (tile << 32) | (uint64_t)s_depth[lo];
    vals[out + k] = (uint32_t)(base + lo);
  }
}

__global__ void __launch_bounds__(256) tile_ranges_kernel(const uint64_t* __restrict__ keys, int64_t n,
                                                          uint32_t num_tiles, uint32_t* __restrict__ ranges) {
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= n) return;
  const uint32_t t = (uint32_t)(keys[i] >> 32);
  const uint32_t prev = i > 0 ? (uint32_t)(keys[i - 1] >> 32) : 0xFFFFFFFFu;
  const uint32_t next = i < n - 1 ? (uint32_t)(keys[i + 1] >> 32) : 0xFFFFFFFFu;
  if (t != prev && t < num_tiles) ranges[(size_t)t * 2] = (uint32_t)i;
  if (t != next && t < num_tiles) ranges[(size_t)t * 2 + 1] = (uint32_t)(i + 1);
}

__global__ void __launch_bounds__(256) block_sums_kernel(const float4* __restrict__ splats, int64_t n,
                                                         uint32_t* __restrict__ sums) {
  __shared__ uint32_t s_warp[8];
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  uint32_t t = i < n ? __float_as_uint(splats[i * 3 + 2].w) : 0u;
  uint32_t incl = block_incl_scan_256(t, s_warp);
  if (threadIdx.x == 255) sums[blockIdx.x] = incl;
}

int launch_block_sums(const float* splats, int64_t n, uint32_t* sums, cudaStream_t stream) {
  if (n == 0) return GSC_OK;
  block_sums_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const float4*>(splats), n, sums);
  GS_CK_LAUNCH("block_sums_kernel");
  return GSC_OK;
}

int launch_scan_block_sums(const uint32_t* sums, int64_t nb, uint64_t* offsets, uint64_t* total,
                           cudaStream_t stream) {
  scan_block_sums_kernel<<<1, 1024, 0, stream>>>(sums, nb, offsets, total);
  GS_CK_LAUNCH("scan_block_sums_kernel");
  return GSC_OK;
}

int launch_emit_keys(const float* splats, int64_t n, const uint64_t* offsets, int tiles_x,
                     int tiles_y, uint64_t* keys, uint32_t* vals, cudaStream_t stream) {
  if (n == 0) return GSC_OK;
  emit_keys_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const float4*>(splats), n, offsets, tiles_x, tiles_y, keys, vals);
  GS_CK_LAUNCH("emit_keys_kernel");
  return GSC_OK;
}

int launch_tile_ranges(const uint64_t* keys, int64_t n, int32_t num_tiles, uint32_t* ranges,
                       cudaStream_t stream) {
  GS_CK(cudaMemsetAsync(ranges, 0, sizeof(uint32_t) * 2 * (size_t)num_tiles, stream));
  if (n == 0) return GSC_OK;
  tile_ranges_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(keys, n, (uint32_t)num_tiles, ranges);
  GS_CK_LAUNCH("tile_ranges_kernel");
  return GSC_OK;
}

// ---------------------------------------------------------------------------
// Depth-first binning for whole-view rasterization.
//
// The sorted (key, value) list that a stable sort of the canonical emission
// by key = tile << 32 | bits(depth) produces is ordered by (tile, depth,
// Gaussian id): a Gaussian emits at most one key per tile, and equal keys
// keep emission (= id) order. The same list comes out of
//   1. a stable sort of the Gaussians by depth bits (N pairs, 32-bit keys),
//   2. emission of (tile, id) pairs in that depth order,
//   3. a stable sort of those pairs by the tile bits only,
// which moves 8-byte pairs through ceil(tile_bits / 8) passes instead of
// 12-byte pairs through ceil((32 + tile_bits) / 8) passes. The emission also
// counts the tile sort's digits (so the sort needs no histogram pass) and
// presets every tile's range to {~0, 0}; the sort's last pass writes the ids
// and the ranges (runs of one tile), ranges_finish_kernel turns the untouched
// {~0, 0} into the reference's empty {0, 0}, and no tile array is kept. The
// 64-bit keys are rebuilt on request from the tile ranges
// (make_keys_ranges_kernel).
// ---------------------------------------------------------------------------

// `bins`: the 32-byte binning records of preprocess ({x0, y0, width, count},
// {mask low, mask high, 0, 0}), gathered in depth order, one sector each.
// True if every tile the Gaussian's binning record lists is marked done (all
// its pixels stopped in an earlier depth slice). tile_done holds one bit per
// tile, `words` 64-bit words per tile row. The record's tiles are, row by row
// of its rectangle, a mask of at most 64 bits (all of them when the mask is
// ~0); each row's part is compared with the done bits of the same tiles.
// Rectangles of more than 64 tiles are never skipped.
__device__ __forceinline__ bool all_tiles_done(uint4 b0, uint4 b1, const unsigned long long* __restrict__ tile_done,
                                               int words) {
  const uint32_t cnt = b0.w, wx = b0.z;
  if (cnt > 64 || wx == 0 || wx > 64) return false;
  uint64_t mk = ((uint64_t)b1.y << 32) | b1.x;
  if (mk == ~0ull) mk = cnt == 64 ? ~0ull : (1ull << cnt) - 1ull;  // every tile of the rect
  const uint64_t row_bits = wx == 64 ? ~0ull : (1ull << wx) - 1ull;
  const int lo = (int)b0.x >> 6, sh = (int)b0.x & 63;
  const unsigned long long* row = tile_done + (size_t)b0.y * words;
  for (; mk; mk = wx == 64 ? 0ull : mk >> wx, row += words) {
    const uint64_t want = mk & row_bits;
    if (!want) continue;
    uint64_t d = row[lo] >> sh;
    if (sh && lo + 1 < words) d |= row[lo + 1] << (64 - sh);
    if (want & ~d) return false;
  }
  return true;
}

// With tile_done (a later depth slice): Gaussians whose tiles are all done
// count 0 pairs, and their bit is set in skip_bits (one bit per position).
__global__ void __launch_bounds__(256) block_sums_gather_kernel(const uint4* __restrict__ bins,
                                                                const uint32_t* __restrict__ order,
                                                                int64_t n, uint32_t* __restrict__ sums,
                                                                const unsigned long long* __restrict__ tile_done,
                                                                int done_words, uint32_t* __restrict__ skip_bits) {
  __shared__ uint32_t s_warp[8];
  const int64_t p = (int64_t)blockIdx.x * 256 + threadIdx.x;
  uint32_t t = 0;
  bool skip = false;
  if (p < n) {
    const uint32_t gid = order[p];
    const uint4 b0 = bins[(size_t)gid * 2];
    t = b0.w;
    if (tile_done && t) {
      skip = all_tiles_done(b0, bins[(size_t)gid * 2 + 1], tile_done, done_words);
      if (skip) t = 0;
    }
  }
  if (skip_bits) {
    const uint32_t bits = __ballot_sync(0xffffffffu, skip);
    if ((threadIdx.x & 31) == 0 && p < n) skip_bits[p >> 5] = bits;
  }
  uint32_t incl = block_incl_scan_256(t, s_warp);
  if (threadIdx.x == 255) sums[blockIdx.x] = incl;
}

// ---- per-tile depth cut (tile hint) -----------------------------------------
__device__ __forceinline__ bool tile_is_done(const unsigned long long* __restrict__ done, int words, int tx, int ty) {
  return (done[(size_t)ty * words + (tx >> 6)] >> (tx & 63)) & 1ull;
}
// Whether pair (Gaussian at depth d, tile (tx, ty)) belongs to the cut's slice.
// A NaN cut puts every pair in the first slice.
__device__ __forceinline__ bool cut_passes(const TileCut& c, float d, int tx, int ty) {
  const float ct = __ldg(c.cut + (size_t)ty * c.tiles_x + tx);
  if (c.mode == 0) return !(d >= ct);
  return d >= ct && !tile_is_done(c.done, c.done_words, tx, ty);
}
// Passing tiles of a binning record of at most 64 tiles: the sub-mask of its
// mask (bit i = tile i of the rect, row-major) and its population count.
__device__ __forceinline__ uint32_t cut_small_record(const TileCut& c, uint4 b0, uint4 b1, uint64_t* sub) {
  const uint32_t cnt = b0.w, wx = b0.z;
  const float d = __uint_as_float(b1.z);
  uint64_t mk = ((uint64_t)b1.y << 32) | b1.x;
  if (mk == ~0ull) mk = cnt == 64 ? ~0ull : (1ull << cnt) - 1ull;  // every tile of the rect
  const uint32_t inv = (65535u + wx) / wx;  // row of a position < 64 by multiply and shift
  uint64_t out = 0;
  for (uint64_t m = mk; m; m &= m - 1ull) {
    const uint32_t i = (uint32_t)(__ffsll((long long)m) - 1);
    const uint32_t ry = (i * inv) >> 16;
    if (cut_passes(c, d, (int)b0.x + (int)(i - ry * wx), (int)b0.y + (int)ry)) out |= 1ull << i;
  }
  *sub = out;
  return (uint32_t)__popcll(out);
}
// Passing tiles of a record of more than 64 tiles (every tile of its rect),
// counted by the whole warp: lane `who`'s record, tiles 32 at a time.
__device__ __forceinline__ uint32_t cut_big_count(const TileCut& c, uint4 b0, float d, int lane) {
  const uint32_t nr = b0.w, wx = b0.z;
  uint32_t k = 0;
  for (uint32_t r0 = 0; r0 < nr; r0 += 32) {
    const uint32_t r = r0 + (uint32_t)lane;
    bool ok = false;
    if (r < nr) {
      const uint32_t ry = r / wx;
      ok = cut_passes(c, d, (int)b0.x + (int)(r - ry * wx), (int)b0.y + (int)ry);
    }
    k += (uint32_t)__popc(__ballot_sync(0xffffffffu, ok));
  }
  return k;
}

// Pair count of each 256-position chunk under a tile cut, with every
// position's passing-tile count and (records of <= 64 tiles) sub-mask. (A
// count in Gaussian order -- records read sequentially, the counts gathered
// in depth order from L2 by a second kernel -- measured slower, and so did
// keeping the gathered records in depth order for the later passes.)
__global__ void __launch_bounds__(256) block_sums_cut_kernel(const uint4* __restrict__ bins,
                                                             const uint32_t* __restrict__ order, int64_t n,
                                                             uint32_t* __restrict__ sums, TileCut tc) {
  __shared__ uint32_t s_warp[8];
  if (tc.open && *(volatile const unsigned int*)tc.open == 0u) {  // no second-slice pair anywhere
    if (threadIdx.x == 0) sums[blockIdx.x] = 0u;
    return;
  }
  const int64_t p = (int64_t)blockIdx.x * 256 + threadIdx.x;
  const int lane = threadIdx.x & 31;
  uint32_t t = 0;
  uint64_t sub = 0;
  uint4 b0 = make_uint4(0u, 0u, 0u, 0u), b1 = b0;
  if (p < n) {
    const uint32_t gid = order[p];
    b0 = bins[(size_t)gid * 2];
    if (b0.w) {
      b1 = bins[(size_t)gid * 2 + 1];
      if (b0.w <= 64) t = cut_small_record(tc, b0, b1, &sub);
    }
  }
  // records of more than 64 tiles: counted by the whole warp, one at a time
  for (uint32_t big = __ballot_sync(0xffffffffu, b0.w > 64u); big; big &= big - 1u) {
    const int who = __ffs(big) - 1;
    uint4 w0;
    w0.x = __shfl_sync(0xffffffffu, b0.x, who);
    w0.y = __shfl_sync(0xffffffffu, b0.y, who);
    w0.z = __shfl_sync(0xffffffffu, b0.z, who);
    w0.w = __shfl_sync(0xffffffffu, b0.w, who);
    const float d = __uint_as_float(__shfl_sync(0xffffffffu, b1.z, who));
    const uint32_t k = cut_big_count(tc, w0, d, lane);
    if (lane == who) t = k;
  }
  if (p < n) {
    tc.sub[p] = sub;
    tc.cnt[p] = t;
  }
  const uint32_t incl = block_incl_scan_256(t, s_warp);
  if (threadIdx.x == 255) sums[blockIdx.x] = incl;
}

constexpr int kEmitMaxPasses = 4;
#ifndef GS_EMIT_FNS
#define GS_EMIT_FNS 1
#endif
constexpr int kOwnWin = 1024;  // outputs per warp window (owner lane per output)

// Position of the k-th (0-based) set bit of m; m has more than k set bits.
__device__ __forceinline__ uint32_t select_bit64(uint64_t m, uint32_t k) {
#if GS_EMIT_FNS
  const uint32_t lo = (uint32_t)m, c = (uint32_t)__popc(lo);
  return k < c ? __fns(lo, 0u, (int)k + 1) : 32u + __fns((uint32_t)(m >> 32), 0u, (int)(k - c) + 1);
#endif
  uint32_t pos = 0;
#pragma unroll
  for (int w = 32; w >= 1; w >>= 1) {
    const uint32_t c = __popcll(m & ((1ull << w) - 1ull));
    if (k >= c) {
      k -= c;
      m >>= w;
      pos += w;
    }
  }
  return pos;
}

__global__ void __launch_bounds__(256) emit_tiles_kernel(const uint4* __restrict__ bins,
                                                         const uint32_t* __restrict__ order, int64_t n,
                                                         const uint64_t* __restrict__ offsets,
                                                         int tiles_x, uint64_t* __restrict__ pair_out,
                                                         uint32_t* __restrict__ hist, int hist_passes,
                                                         uint32_t* __restrict__ ranges, int32_t num_tiles,
                                                         const uint32_t* __restrict__ skip_bits, TileCut tc) {
  __shared__ uint32_t s_hist[kEmitMaxPasses][256];
  __shared__ uint32_t s_incl[256];
  __shared__ int s_x0[256], s_y0[256], s_wx[256];
  __shared__ uint32_t s_inv[256];  // ceil(2^16 / width): row of a test < 64 by multiply and shift
  __shared__ uint32_t s_id[256];
  __shared__ uint64_t s_mask[256];
  __shared__ uint32_t s_warp[8];
  // tile cut: records of more than 64 tiles are emitted warp-cooperatively
  __shared__ uint32_t s_big[256];  // tile count of such a record, else 0
  __shared__ float s_depth[256];
  const bool cut = tc.cut != nullptr;
  const bool live = !(cut && tc.open && *(volatile const unsigned int*)tc.open == 0u);
  __shared__ uint8_t s_own[8][kOwnWin];
  if (ranges)
    for (int64_t r = (int64_t)blockIdx.x * 256 + threadIdx.x; r < num_tiles; r += (int64_t)gridDim.x * 256) {
      ranges[2 * r] = 0xFFFFFFFFu;
      ranges[2 * r + 1] = 0u;
    }
  for (int k = threadIdx.x; k < hist_passes * 256; k += 256) (&s_hist[0][0])[k] = 0u;
  // A block takes chunks of 256 Gaussians (in depth order) in turn, so that
  // its digit counts reach global memory once per block, not per chunk.
  const int64_t nchunks = live ? (n + 255) / 256 : 0;
  for (int64_t chunk = blockIdx.x; chunk < nchunks; chunk += gridDim.x) {
    const int64_t p = chunk * 256 + threadIdx.x;
    uint32_t t = 0;
    s_big[threadIdx.x] = 0u;
    if (p < n) {
      if (cut) {
        t = tc.cnt[p];  // passing tiles, counted by block_sums_cut_kernel
        if (t) {
          const uint32_t gid = order[p];
          const uint4 b0 = bins[(size_t)gid * 2];
          s_x0[threadIdx.x] = (int)b0.x;
          s_y0[threadIdx.x] = (int)b0.y;
          s_wx[threadIdx.x] = (int)b0.z;
          s_inv[threadIdx.x] = (65535u + b0.z) / b0.z;
          s_id[threadIdx.x] = gid;
          if (b0.w <= 64) {
            s_mask[threadIdx.x] = tc.sub[p];
          } else {
            s_big[threadIdx.x] = b0.w;
            s_depth[threadIdx.x] = __uint_as_float(bins[(size_t)gid * 2 + 1].z);
          }
        }
      } else {
        const uint32_t gid = order[p];
        const uint4 b0 = bins[(size_t)gid * 2];
        t = b0.w;
        if (skip_bits && ((skip_bits[p >> 5] >> (p & 31)) & 1u)) t = 0;  // every tile already done
        if (t) {
          const uint4 b1 = bins[(size_t)gid * 2 + 1];
          s_x0[threadIdx.x] = (int)b0.x;
          s_y0[threadIdx.x] = (int)b0.y;
          s_wx[threadIdx.x] = (int)b0.z;
          s_inv[threadIdx.x] = (65535u + b0.z) / b0.z;
          s_id[threadIdx.x] = gid;
          s_mask[threadIdx.x] = ((uint64_t)b1.y << 32) | b1.x;
        }
      }
    }
    uint32_t incl = block_incl_scan_256(t, s_warp);
    s_incl[threadIdx.x] = incl;
    __syncthreads();
    const uint64_t out = offsets[chunk];
    const int wb = threadIdx.x & ~31;
    const uint32_t wend = s_incl[wb + 31];
    const uint32_t wbeg = wb ? s_incl[wb - 1] : 0u;
    // Each warp writes the contiguous output range of its 32 Gaussians, a
    // window of kOwnWin outputs at a time: every lane first marks its
    // Gaussian's outputs of the window with its lane number, then the lanes
    // take the window's outputs 32 at a time and read their owner back.
    const int lane = threadIdx.x & 31;
    uint8_t* own_of = s_own[threadIdx.x >> 5];
    const uint32_t g_end = s_incl[threadIdx.x], g_beg = g_end - t;
    for (uint32_t w0 = wbeg; w0 < wend; w0 += kOwnWin) {
      const uint32_t w1 = min(w0 + (uint32_t)kOwnWin, wend);
      for (uint32_t k = max(g_beg, w0); k < min(g_end, w1); k++) own_of[k - w0] = (uint8_t)lane;
      __syncwarp();
      for (uint32_t k0 = w0; k0 < w1; k0 += 32) {
        const uint32_t k = k0 + lane;
        const int own = k < w1 ? wb + own_of[k - w0] : wb;
        const bool valid = k < w1 && !s_big[own];  // tile-cut records of > 64 tiles: below
        uint32_t tile = 0xFFFFFFFFu;
        if (valid) {
          uint32_t local = k - (own ? s_incl[own - 1] : 0u);
          const uint64_t mk = s_mask[own];
          const uint32_t wx = (uint32_t)s_wx[own];
          uint32_t ry;
          if (mk != ~0ull) {
            local = select_bit64(mk, local);  // local-th contributing tile of the rect (< 64)
            ry = (local * s_inv[own]) >> 16;
          } else {
            ry = local / wx;
          }
          const int ty = s_y0[own] + (int)ry;
          const int tx = s_x0[own] + (int)(local - ry * wx);
          tile = (uint32_t)(ty * tiles_x + tx);
          pair_out[out + k] = ((uint64_t)tile << 32) | (uint64_t)s_id[own];
        }
        // digit counts of the tile sort
        if (valid)
          for (int q = 0; q < hist_passes; q++) atomicAdd(&s_hist[q][(tile >> (8 * q)) & 255u], 1u);
      }
      __syncwarp();
    }
    // tile-cut records of more than 64 tiles: the warp walks each one's rect,
    // 32 tiles at a time, in the order block_sums_cut_kernel counted them
    for (uint32_t big = __ballot_sync(0xffffffffu, s_big[threadIdx.x] != 0u); big; big &= big - 1u) {
      const int g = wb + __ffs(big) - 1;
      const uint32_t nr = s_big[g], wx = (uint32_t)s_wx[g];
      const int x0 = s_x0[g], y0 = s_y0[g];
      const float d = s_depth[g];
      const uint64_t gbase = out + (g ? s_incl[g - 1] : 0u);
      uint32_t run = 0;
      for (uint32_t r0 = 0; r0 < nr; r0 += 32) {
        const uint32_t r = r0 + (uint32_t)lane;
        bool ok = false;
        uint32_t tile = 0;
        if (r < nr) {
          const uint32_t ry = r / wx;
          const int tx = x0 + (int)(r - ry * wx), ty = y0 + (int)ry;
          ok = cut_passes(tc, d, tx, ty);
          tile = (uint32_t)(ty * tiles_x + tx);
        }
        const uint32_t bal = __ballot_sync(0xffffffffu, ok);
        if (ok) {
          pair_out[gbase + run + (uint32_t)__popc(bal & ((1u << lane) - 1u))] = ((uint64_t)tile << 32) | (uint64_t)s_id[g];
          for (int q = 0; q < hist_passes; q++) atomicAdd(&s_hist[q][(tile >> (8 * q)) & 255u], 1u);
        }
        run += (uint32_t)__popc(bal);
      }
    }
    __syncthreads();  // the chunk's shared records are replaced next
  }
  if (hist_passes == 0) return;
  // one counter per 128-byte line (stride kHistStride), so that the blocks'
  // adds spread over the L2 slices
  for (int k = threadIdx.x; k < hist_passes * 256; k += 256) {
    const uint32_t c = (&s_hist[0][0])[k];
    if (c) atomicAdd(&hist[(size_t)k * kHistStride], c);
  }
}

__global__ void __launch_bounds__(256) tile_ranges_u32_kernel(const uint32_t* __restrict__ tiles, int64_t n,
                                                              uint32_t num_tiles, uint32_t* __restrict__ ranges) {
  // four keys per thread: one 16-byte load (tiles is 16-byte aligned) and the two neighbours
  const int64_t i0 = ((int64_t)blockIdx.x * 256 + threadIdx.x) * 4;
  if (i0 >= n) return;
  uint32_t t[6];
  t[0] = i0 > 0 ? tiles[i0 - 1] : 0xFFFFFFFFu;
  if (i0 + 4 <= n) {
    const uint4 v = *reinterpret_cast<const uint4*>(tiles + i0);
    t[1] = v.x; t[2] = v.y; t[3] = v.z; t[4] = v.w;
  } else {
#pragma unroll
    for (int k = 0; k < 4; k++) t[1 + k] = i0 + k < n ? tiles[i0 + k] : 0xFFFFFFFFu;
  }
  t[5] = i0 + 4 < n ? tiles[i0 + 4] : 0xFFFFFFFFu;
#pragma unroll
  for (int k = 1; k <= 4; k++) {
    const uint32_t c = t[k];
    if (c >= num_tiles) continue;  // also the padding past n
    if (c != t[k - 1]) ranges[(size_t)c * 2] = (uint32_t)(i0 + k - 1);
    if (c != t[k + 1]) ranges[(size_t)c * 2 + 1] = (uint32_t)(i0 + k);
  }
}

int launch_block_sums_gather(const uint4* bins, const uint32_t* order, int64_t n, uint32_t* sums,
                             cudaStream_t stream, const unsigned long long* tile_done, int done_words,
                             uint32_t* skip_bits) {
  if (n == 0) return GSC_OK;
  block_sums_gather_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(bins, order, n, sums, tile_done,
                                                                            done_words, skip_bits);
  GS_CK_LAUNCH("block_sums_gather_kernel");
  return GSC_OK;
}

// Final tile lists of depth-sliced binning: tile t keeps the first keep[t]
// entries of its slices' lists, concatenated in slice order (the entries
// that the compositing read; the rest lie behind every pixel's stop).
// keep_scan: one block, exclusive scan of keep into the output ranges.
__global__ void __launch_bounds__(1024) keep_scan_kernel(const uint32_t* __restrict__ keep, int32_t num_tiles,
                                                         uint32_t* __restrict__ out_ranges,
                                                         uint64_t* __restrict__ total) {
  __shared__ uint32_t s_warp[32];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int chunk = (num_tiles + 1023) / 1024;
  const int lo = min(num_tiles, tid * chunk), hi = min(num_tiles, lo + chunk);
  uint32_t mine = 0;
  for (int t = lo; t < hi; t++) mine += keep[t];
  uint32_t v = mine;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t u = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += u;
  }
  if (lane == 31) s_warp[w] = v;
  __syncthreads();
  if (w == 0) {
    uint32_t x = s_warp[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t u = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += u;
    }
    s_warp[lane] = x;
  }
  __syncthreads();
  uint32_t run = (v - mine) + (w > 0 ? s_warp[w - 1] : 0u);
  for (int t = lo; t < hi; t++) {  // empty tiles get the reference's empty range {0, 0}
    const uint32_t k = keep[t];
    out_ranges[2 * (size_t)t] = k ? run : 0u;
    out_ranges[2 * (size_t)t + 1] = k ? run + k : 0u;
    run += k;
  }
  if (tid == 1023) *total = run;
}

struct SliceLists {
  const uint32_t* vals[kMaxSlices];
  const uint32_t* ranges[kMaxSlices];
  int n;
};

// One warp per tile copies its kept entries.
__global__ void __launch_bounds__(256) concat_slices_kernel(SliceLists sl, const uint32_t* __restrict__ keep,
                                                            int32_t num_tiles, const uint32_t* __restrict__ out_ranges,
                                                            uint32_t* __restrict__ out_vals) {
  const int t = (int)(((int64_t)blockIdx.x * 256 + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= num_tiles) return;
  uint32_t left = keep[t];
  uint32_t dst = out_ranges[2 * (size_t)t];
  for (int s = 0; s < sl.n && left; s++) {
    const uint32_t a = sl.ranges[s][2 * (size_t)t], b = sl.ranges[s][2 * (size_t)t + 1];
    const uint32_t take = min(left, b - a);
    for (uint32_t k = lane; k < take; k += 32) out_vals[dst + k] = sl.vals[s][a + k];
    dst += take;
    left -= take;
  }
}

__global__ void add_u64_kernel(const uint64_t* __restrict__ src, unsigned long long* __restrict__ dst) {
  if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(dst, (unsigned long long)*src);
}

int launch_add_u64(const uint64_t* src, unsigned long long* dst, cudaStream_t stream) {
  add_u64_kernel<<<1, 32, 0, stream>>>(src, dst);
  GS_CK_LAUNCH("add_u64_kernel");
  return GSC_OK;
}

int launch_concat_slices(const uint32_t* const* slice_vals, const uint32_t* const* slice_ranges, int nslices,
                         const uint32_t* keep, int32_t num_tiles, uint32_t* out_vals, uint32_t* out_ranges,
                         uint64_t* total, cudaStream_t stream) {
  if (nslices < 1 || nslices > kMaxSlices) {
    set_error("concat_slices: bad slice count");
    return GSC_ERR_INVALID;
  }
  if (num_tiles == 0) return cudaMemsetAsync(total, 0, 8, stream) == cudaSuccess ? GSC_OK : GSC_ERR_CUDA;
  SliceLists sl;
  std::memset(&sl, 0, sizeof sl);
  sl.n = nslices;
  for (int s = 0; s < nslices; s++) {
    sl.vals[s] = slice_vals[s];
    sl.ranges[s] = slice_ranges[s];
  }
  keep_scan_kernel<<<1, 1024, 0, stream>>>(keep, num_tiles, out_ranges, total);
  GS_CK_LAUNCH("keep_scan_kernel");
  const int64_t threads = (int64_t)num_tiles * 32;
  concat_slices_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(sl, keep, num_tiles, out_ranges,
                                                                               out_vals);
  GS_CK_LAUNCH("concat_slices_kernel");
  return GSC_OK;
}

int launch_emit_tiles(const uint4* bins, const uint32_t* order, int64_t n, const uint64_t* offsets,
                      int tiles_x, uint64_t* pair_out, cudaStream_t stream, uint32_t* hist, int hist_passes,
                      uint32_t* ranges, int32_t num_tiles, int64_t grid_cap, const uint32_t* skip_bits,
                      const TileCut* tc) {
  if (n == 0) return GSC_OK;
  if (hist_passes < 0 || hist_passes > kEmitMaxPasses || (hist_passes > 0 && !hist)) {
    set_error("emit_tiles: bad histogram arguments");
    return GSC_ERR_INVALID;
  }
  if (tc && (!tc->cut || !tc->sub || !tc->cnt || skip_bits)) {
    set_error("emit_tiles: a tile cut needs its cut, sub-masks and counts (and no skip bits)");
    return GSC_ERR_INVALID;
  }
  const int64_t chunks = (n + 255) / 256;
  const int64_t grid = grid_cap > 0 ? std::min<int64_t>(chunks, grid_cap) : chunks;
  emit_tiles_kernel<<<(unsigned)grid, 256, 0, stream>>>(bins, order, n, offsets, tiles_x, pair_out, hist,
                                                        hist_passes, ranges, num_tiles, skip_bits,
                                                        tc ? *tc : TileCut());
  GS_CK_LAUNCH("emit_tiles_kernel");
  return GSC_OK;
}

int launch_block_sums_cut(const uint4* bins, const uint32_t* order, int64_t n, uint32_t* sums, const TileCut& tc,
                          cudaStream_t stream) {
  if (n == 0) return GSC_OK;
  if (!tc.cut || !tc.sub || !tc.cnt || (tc.mode == 1 && !tc.done) || tc.tiles_x <= 0) {
    set_error("block_sums_cut: incomplete tile cut");
    return GSC_ERR_INVALID;
  }
  block_sums_cut_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(bins, order, n, sums, tc);
  GS_CK_LAUNCH("block_sums_cut_kernel");
  return GSC_OK;
}

__global__ void __launch_bounds__(256) tile_cut_update_kernel(const uint32_t* __restrict__ ranges,
                                                              const uint32_t* __restrict__ vals,
                                                              const uint32_t* __restrict__ keep,
                                                              const unsigned long long* __restrict__ done,
                                                              int done_words, int32_t tiles_x, int32_t num_tiles,
                                                              const float4* __restrict__ splats, float margin,
                                                              float* __restrict__ cut_out) {
  const int32_t t = (int32_t)(blockIdx.x * 256 + threadIdx.x);
  if (t >= num_tiles) return;
  const uint32_t w = keep[t];
  float c = __int_as_float(0x7f800000);  // +inf: the whole list stays in the first slice
  if (w && tile_is_done(done, done_words, t % tiles_x, t / tiles_x)) {
    const uint32_t gid = vals[ranges[2 * t] + w - 1];
    c = splats[(size_t)gid * 3 + 2].y * (1.0f + margin);  // record word 9: depth
  }
  cut_out[t] = c;
}

int launch_tile_cut_update(const uint32_t* ranges, const uint32_t* vals, const uint32_t* keep,
                           const unsigned long long* done, int done_words, int32_t tiles_x, int32_t num_tiles,
                           const float* splats, float margin, float* cut_out, cudaStream_t stream) {
  if (num_tiles <= 0) return GSC_OK;
  tile_cut_update_kernel<<<(unsigned)((num_tiles + 255) / 256), 256, 0, stream>>>(
      ranges, vals, keep, done, done_words, tiles_x, num_tiles, reinterpret_cast<const float4*>(splats), margin,
      cut_out);
  GS_CK_LAUNCH("tile_cut_update_kernel");
  return GSC_OK;
}

// Tile order for the backward compositing: a counting sort of the tiles by
// work in buckets of a quarter octave (the work's leading bit and the two
// below it), largest first, tiles without work last. One block; the order
// within a bucket is whatever the shared-memory atomics give (every tile is
// composited independently, so it does not change any result).
constexpr int kOrderBuckets = 132;

__global__ void __launch_bounds__(1024) tile_order_kernel(const uint32_t* __restrict__ ranges,
                                                          const uint32_t* __restrict__ tile_work,
                                                          int32_t num_tiles, uint32_t* __restrict__ order) {
  __shared__ uint32_t s_off[kOrderBuckets];
  for (int k = threadIdx.x; k < kOrderBuckets; k += 1024) s_off[k] = 0u;
  __syncthreads();
  auto bucket = [&](int32_t t) -> int {
    const uint32_t w = ranges ? ranges[2 * t + 1] - ranges[2 * t] : tile_work[t];
    if (w == 0) return kOrderBuckets - 1;  // last
    const int msb = 31 - __clz(w);
    const uint32_t frac = msb >= 2 ? (w >> (msb - 2)) & 3u : (w << (2 - msb)) & 3u;
    return kOrderBuckets - 2 - (4 * msb + (int)frac);  // larger work first
  };
  for (int32_t t = threadIdx.x; t < num_tiles; t += 1024) atomicAdd(&s_off[bucket(t)], 1u);
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t run = 0;
    for (int k = 0; k < kOrderBuckets; k++) {
      const uint32_t c = s_off[k];
      s_off[k] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int32_t t = threadIdx.x; t < num_tiles; t += 1024) order[atomicAdd(&s_off[bucket(t)], 1u)] = (uint32_t)t;
}

int launch_tile_order(const uint32_t* ranges, const uint32_t* tile_work, int32_t num_tiles, uint32_t* order,
                      cudaStream_t stream) {
  if (num_tiles <= 0) return GSC_OK;
  tile_order_kernel<<<1, 1024, 0, stream>>>(ranges, tile_work, num_tiles, order);
  GS_CK_LAUNCH("tile_order_kernel");
  return GSC_OK;
}

__global__ void __launch_bounds__(256) ranges_finish_kernel(uint32_t* __restrict__ ranges, int32_t num_tiles) {
  const int64_t t = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (t >= num_tiles) return;
  if (ranges[2 * t] == 0xFFFFFFFFu) ranges[2 * t] = 0u;
}

int launch_ranges_finish(uint32_t* ranges, int32_t num_tiles, cudaStream_t stream) {
  if (num_tiles <= 0) return GSC_OK;
  ranges_finish_kernel<<<(unsigned)((num_tiles + 255) / 256), 256, 0, stream>>>(ranges, num_tiles);
  GS_CK_LAUNCH("ranges_finish_kernel");
  return GSC_OK;
}

// One warp per tile writes the keys of the tile's range.
__global__ void __launch_bounds__(256) make_keys_ranges_kernel(const uint32_t* __restrict__ ranges,
                                                               int32_t num_tiles,
                                                               const uint32_t* __restrict__ ids,
                                                               const float4* __restrict__ splats,
                                                               uint64_t* __restrict__ keys) {
  const int64_t t = ((int64_t)blockIdx.x * 256 + threadIdx.x) >> 5;
  if (t >= num_tiles) return;
  const uint32_t b = ranges[2 * t], e = ranges[2 * t + 1];
  for (uint32_t i = b + (threadIdx.x & 31); i < e; i += 32) {
    const uint32_t depth_bits = __float_as_uint(splats[(size_t)ids[i] * 3 + 2].y);
    keys[i] = ((uint64_t)t << 32) | depth_bits;
  }
}

int launch_make_keys_ranges(const uint32_t* ranges, int32_t num_tiles, const uint32_t* ids, const float* splats,
                            uint64_t* keys, cudaStream_t stream) {
  if (num_tiles <= 0) return GSC_OK;
  make_keys_ranges_kernel<<<(unsigned)(((int64_t)num_tiles * 32 + 255) / 256), 256, 0, stream>>>(
      ranges, num_tiles, ids, reinterpret_cast<const float4*>(splats), keys);
  GS_CK_LAUNCH("make_keys_ranges_kernel");
  return GSC_OK;
}

int launch_tile_ranges_u32(const uint32_t* tiles, int64_t n, int32_t num_tiles, uint32_t* ranges,
                           cudaStream_t stream) {
  GS_CK(cudaMemsetAsync(ranges, 0, sizeof(uint32_t) * 2 * (size_t)num_tiles, stream));
  if (n == 0) return GSC_OK;
  tile_ranges_u32_kernel<<<(unsigned)((n + 1023) / 1024), 256, 0, stream>>>(tiles, n, (uint32_t)num_tiles, ranges);
  GS_CK_LAUNCH("tile_ranges_u32_kernel");
  return GSC_OK;
}


}  // namespace gs
