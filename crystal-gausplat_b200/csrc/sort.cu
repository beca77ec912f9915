// sort.cu — stable LSD radix sort of (u64 key, u32 value) pairs, replacing
// GPURadixSort.sort! (src/metal/gpu_radix_sort.cr:46-200,
// src/metal/kernels/radix_sort.metal:21-281: 4-bit digits, 5 dispatches per
// pass, and a digit-0-only scan that breaks it beyond 512 keys).
//
// Design (onesweep): 8-bit digits over the requested bit range only.
//   1. histogram_kernel reads the keys once and builds the digit histograms of
//      every pass.
//   2. One onesweep_kernel per pass: a CTA takes the next partition of 4096
//      pairs by atomic ticket, ranks its keys stably with warp match/ballot
//      and per-warp digit counters in shared memory, publishes its per-digit
//      counts, resolves its global digit offsets by decoupled look-back over
//      earlier partitions (bounded spin: on give-up it sets the device error
//      word and never writes out of bounds), reorders the tile in shared
//      memory and scatters keys then values with coalesced runs.
// Traffic per pair: 8 B (histogram) + 24 B per pass.
//
// Packed mode (the whole-view binning): a pair travels as one u64, key in the
// high word and value in the low word, sorted by key bits only; scatter runs
// are then twice as long and there is no value phase. The last pass writes
// the two words to separate arrays.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace gs {

namespace {
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kItems = 16;
constexpr int kWarpKeys = 32 * kItems;           // 512
constexpr int kTileKeys = kWarps * kWarpKeys;    // 4096
constexpr uint32_t kFlagAgg = 1u << 30;
constexpr uint32_t kFlagInc = 2u << 30;
constexpr uint32_t kValMask = (1u << 30) - 1u;
constexpr uint32_t kSpinLimit = 1u << 21;
}  // namespace


// Decoupled look-back of partition `part` for digit d: walks the earlier
// partitions' status words back to the nearest inclusive prefix, adding the
// aggregates on the way. A word still 0 (nothing published) is re-read after
// a short sleep, at most spin_limit times; then the wait gives up, sets
// GS_DEVERR_TIMEOUT in *err (read back by gsc_sync) and returns what it has,
// so the kernel always finishes.
__device__ __forceinline__ uint32_t lookback_exclusive(const uint32_t* status, int64_t part, uint32_t d,
                                                       uint32_t spin_limit, uint32_t* err) {
  uint32_t excl = 0, spins = 0;
  int64_t j = part - 1;
  while (j >= 0) {
    const uint32_t s = *(volatile const uint32_t*)(status + (size_t)j * 256 + d);
    const uint32_t flag = s & ~kValMask;
    if (flag == 0) {
      if (++spins > spin_limit) {
        atomicOr(err, GS_DEVERR_TIMEOUT);
        break;
      }
      __nanosleep(32);
      continue;
    }
    excl += s & kValMask;
    if (flag == kFlagInc) break;
    j--;
  }
  return excl;
}

// The look-back wait on a status array whose partition 0 never publishes:
// partition 1's wait must give up after spin_limit re-reads (failure-path
// self-test of gsc_selftest_wait_timeout).
__global__ void __launch_bounds__(256) lookback_selftest_kernel(const uint32_t* status, uint32_t spin_limit,
                                                                uint32_t* err) {
  lookback_exclusive(status, 1, threadIdx.x, spin_limit, err);
}

int launch_lookback_selftest(gsc_ctx* ctx, uint32_t spin_limit, char* scratch) {
  GS_CK(cudaMemsetAsync(scratch, 0, 2 * 256 * 4, ctx->stream));
  lookback_selftest_kernel<<<1, 256, 0, ctx->stream>>>(reinterpret_cast<const uint32_t*>(scratch), spin_limit,
                                                      ctx->err);
  GS_CK_LAUNCH("lookback_selftest_kernel");
  return GSC_OK;
}

template <typename K>
__global__ void __launch_bounds__(256) histogram_kernel(const K* __restrict__ keys, int64_t n,
                                                        int begin_bit, int end_bit, int npass,
                                                        uint32_t* __restrict__ hist) {
  __shared__ uint32_t s_hist[8][256];
  for (int k = threadIdx.x; k < 8 * 256; k += 256) (&s_hist[0][0])[k] = 0;
  __syncthreads();
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (int64_t)gridDim.x * 256) {
    const K key = keys[i];
    for (int p = 0; p < npass; p++) {
      const int shift = begin_bit + 8 * p;
      const int bits = min(8, end_bit - shift);
      const uint32_t d = (uint32_t)(key >> shift) & ((1u << bits) - 1u);
      atomicAdd(&s_hist[p][d], 1u);
    }
  }
  __syncthreads();
  for (int k = threadIdx.x; k < npass * 256; k += 256) {
    const uint32_t c = (&s_hist[0][0])[k];
    if (c) atomicAdd(&hist[k], c);
  }
}

// Exclusive scan of one u32 per thread over 256 threads.
__device__ __forceinline__ uint32_t block_excl_scan_256(uint32_t v, uint32_t* s_warp) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    uint32_t t = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += t;
  }
  if (lane == 31) s_warp[w] = x;
  __syncthreads();
  uint32_t add = 0;
  for (int k = 0; k < w; k++) add += s_warp[k];
  __syncthreads();
  return x - v + add;
}

// MODE: 0 = (key, value) pairs; 1 = packed u64, written packed; 2 = packed
// u64, written split (high word to keys_hi, low word to vals_out).
#ifndef GS_PACKED_MIN_CTAS
#define GS_PACKED_MIN_CTAS 5
#endif
#ifndef GS_PAIR_MIN_CTAS
#define GS_PAIR_MIN_CTAS 5
#endif
// One partition (4096 keys) of a onesweep pass: the CTA takes the next
// ticket; false (nothing done) if it is past the last partition (`parts`).
template <typename K, int MODE>
__device__ __forceinline__ bool onesweep_tile(
    const K* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
    K* __restrict__ keys_out, uint32_t* __restrict__ vals_out, int64_t n, int shift,
    uint32_t digit_mask, const uint32_t* __restrict__ hist, uint32_t* status, uint32_t* ticket,
    int64_t parts, uint32_t* err, uint32_t* __restrict__ keys_hi, uint32_t lo_mask,
    uint32_t* __restrict__ ranges, uint32_t ntiles, int hstride) {
  __shared__ K s_keys[kTileKeys];  // reused for values
  // per-warp digit counters; in pair mode two 16-bit counters per word (a warp
  // ranks at most 512 keys per digit, a tile 4096), which saves the 4 KB that
  // the fifth CTA per SM needs
  constexpr bool kPack16 = MODE == 0;
  __shared__ uint32_t s_whw[kWarps][kPack16 ? 128 : 256];
  unsigned short* s_wh16 = reinterpret_cast<unsigned short*>(&s_whw[0][0]);
  __shared__ uint32_t s_gbase[256];
  __shared__ uint8_t s_dig[MODE == 0 ? kTileKeys : 1];  // pair mode only
  __shared__ uint32_t s_warp[kWarps];
  __shared__ uint32_t s_part;

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (tid == 0) s_part = atomicAdd(ticket, 1u);
  for (int k = tid; k < kWarps * (kPack16 ? 128 : 256); k += kThreads) (&s_whw[0][0])[k] = 0;
  __syncthreads();
  const uint32_t part = s_part;
  if ((int64_t)part >= parts) return false;
  const int64_t tile_base = (int64_t)part * kTileKeys;
  const int64_t warp_base = tile_base + (int64_t)w * kWarpKeys;
  const uint32_t num_valid = (uint32_t)min((int64_t)kTileKeys, n - tile_base);

  // Only the packed digits and ranks stay live across the look-back; keys
  // and values are read again (from L2) when the tile is reordered, which
  // keeps the register count low enough for 4-5 CTAs per SM.
  uint32_t rank[kItems];
  uint32_t dig[kItems / 4];  // four 8-bit digits per register
#pragma unroll
  for (int i = 0; i < kItems / 4; i++) dig[i] = 0;
  // partition-local 32-bit indices: the warp's keys start at wkeys
  const K* __restrict__ wkeys = keys_in + warp_base;
  const int wvalid = (int)max((int64_t)0, min((int64_t)kWarpKeys, n - warp_base));
#pragma unroll
  for (int i = 0; i < kItems; i++) {
    const int li = i * 32 + lane;
    // Pairs past the end take the largest digit (and come last in index
    // order), so they sort behind every valid pair of the tile.
    const uint32_t d = li < wvalid ? ((uint32_t)(wkeys[li] >> shift) & digit_mask) : digit_mask;
    dig[i / 4] |= d << (8 * (i % 4));
  }
  const uint32_t lt_mask = (1u << lane) - 1u;
  const int nbits = 32 - __clz(digit_mask);  // digit width (padding digits 255 agree on these bits)
#pragma unroll
  for (int i = 0; i < kItems; i++) {
    const uint32_t d = (dig[i / 4] >> (8 * (i % 4))) & 255u;
    // Lanes holding the same digit: AND of one ballot per digit bit (constant
    // cost, whatever the number of distinct digits in the warp).
    uint32_t peers = 0xffffffffu;
#pragma unroll
    for (int b = 0; b < 8; b++) {
      if (b < nbits) {
        const uint32_t bit = (d >> b) & 1u;
        const uint32_t bal = __ballot_sync(0xffffffffu, bit);
        peers &= ~(bal ^ (0u - bit));  // bal where the bit is set, ~bal where clear
      }
    }
    const int leader = __ffs(peers) - 1;
    uint32_t b = 0;
    if (lane == leader) {
      if (kPack16) {
        const uint32_t sh = 16u * (d & 1u);
        b = (atomicAdd(&s_whw[w][d >> 1], (uint32_t)__popc(peers) << sh) >> sh) & 0xFFFFu;
      } else {
        b = atomicAdd(&s_whw[w][d], (uint32_t)__popc(peers));
      }
    }
    b = __shfl_sync(0xffffffffu, b, leader);
    rank[i] = (d << 16) | (b + __popc(peers & lt_mask));
  }
  __syncthreads();

  // Thread d owns digit d: warp offsets, tile count, tile-local prefix.
  const uint32_t d = tid;
  uint32_t cnt = 0;
#pragma unroll
  for (int ww = 0; ww < kWarps; ww++) {
    if (kPack16) {
      const uint32_t c = s_wh16[ww * 256 + d];
      s_wh16[ww * 256 + d] = (unsigned short)cnt;
      cnt += c;
    } else {
      const uint32_t c = s_whw[ww][d];
      s_whw[ww][d] = cnt;
      cnt += c;
    }
  }
  const uint32_t valid_cnt = d == digit_mask ? cnt - (kTileKeys - num_valid) : cnt;
  const uint32_t local_excl = block_excl_scan_256(cnt, s_warp);
  // each warp's start within the digit becomes its start within the tile
#pragma unroll
  for (int ww = 0; ww < kWarps; ww++) {
    if (kPack16) s_wh16[ww * 256 + d] = (unsigned short)(s_wh16[ww * 256 + d] + local_excl);
    else s_whw[ww][d] += local_excl;
  }
  const uint32_t gexcl = block_excl_scan_256(hist[(size_t)d * hstride], s_warp);

  // Decoupled look-back.
  uint32_t* my = status + (size_t)part * 256 + d;
  uint32_t excl = 0;
  if (part == 0) {
    *(volatile uint32_t*)my = kFlagInc | valid_cnt;
  } else {
    *(volatile uint32_t*)my = kFlagAgg | valid_cnt;
    excl = lookback_exclusive(status, part, d, kSpinLimit, err);
    *(volatile uint32_t*)my = kFlagInc | ((excl + valid_cnt) & kValMask);
  }
  s_gbase[d] = gexcl + excl - local_excl;  // global position = s_gbase[d] + tile position
  __syncthreads();

#pragma unroll
  for (int i = 0; i < kItems; i++) {
    const int li = i * 32 + lane;
    const uint32_t dd = rank[i] >> 16;
    const uint32_t wbase = kPack16 ? (uint32_t)s_wh16[w * 256 + dd] : s_whw[w][dd];
    const uint32_t pos = wbase + (rank[i] & 0xFFFFu);
    if (li < wvalid) s_keys[pos] = wkeys[li];
    rank[i] = pos;
  }
  __syncthreads();
  for (uint32_t j = tid; j < num_valid; j += kThreads) {
    const K key = s_keys[j];
    const uint32_t dd = (uint32_t)(key >> shift) & digit_mask;
    const uint32_t gpos = s_gbase[dd] + j;
    if (MODE == 0) s_dig[j] = (uint8_t)dd;
    if ((int64_t)gpos >= n) {
      atomicOr(err, GS_DEVERR_BOUNDS);
    } else if (MODE == 2) {
      const uint32_t hi = (uint32_t)((uint64_t)key >> 32);
      if (keys_hi) keys_hi[gpos] = hi;
      vals_out[gpos] = (uint32_t)key & lo_mask;
      if (ranges && hi < ntiles) {
        // Last pass of a sort by the whole high word (the tile): equal tiles
        // share the digit, so a run of one tile in this tile-local order is a
        // run of consecutive output positions; its ends bound the tile's
        // range, and the runs of all partitions merge by min / max.
        if (j == 0 || (uint32_t)((uint64_t)s_keys[j - 1] >> 32) != hi) atomicMin(&ranges[2 * (size_t)hi], gpos);
        if (j + 1 == num_valid || (uint32_t)((uint64_t)s_keys[j + 1] >> 32) != hi)
          atomicMax(&ranges[2 * (size_t)hi + 1], gpos + 1);
      }
    } else {
      keys_out[gpos] = key;
    }
  }
  if (MODE != 0) return true;
  __syncthreads();
  uint32_t* s_vals = reinterpret_cast<uint32_t*>(s_keys);
#pragma unroll
  for (int i = 0; i < kItems; i++) {
    const int li = i * 32 + lane;
    if (li < wvalid) s_vals[rank[i]] = vals_in[warp_base + li];
  }
  __syncthreads();
  for (uint32_t j = tid; j < num_valid; j += kThreads) {
    const uint32_t gpos = s_gbase[s_dig[j]] + j;
    if ((int64_t)gpos < n) vals_out[gpos] = s_vals[j];
  }
  return true;
}


// One onesweep pass; every CTA takes partitions by atomic ticket, so the
// look-back only ever waits on partitions that a running CTA holds. With
// n_dev the key count is known on the device only (the host sizes buffers by
// an upper bound) and PERSIST kernels run a grid of at most what is resident
// at once, each CTA taking partitions until none is left; otherwise the grid
// is the partitions, one per CTA (the loop's live state costs the one-shot
// kernel registers: 15.8 vs 16.8 Gkey/s on the 30M-pair sort).
template <typename K, int MODE = 0, bool PERSIST = false>
__global__ void __launch_bounds__(kThreads, MODE == 0 ? GS_PAIR_MIN_CTAS : GS_PACKED_MIN_CTAS) onesweep_kernel(
    const K* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
    K* __restrict__ keys_out, uint32_t* __restrict__ vals_out, int64_t n, int shift,
    uint32_t digit_mask, const uint32_t* __restrict__ hist, uint32_t* status, uint32_t* ticket,
    uint32_t* err, uint32_t* __restrict__ keys_hi = nullptr, uint32_t lo_mask = 0xFFFFFFFFu,
    uint32_t* __restrict__ ranges = nullptr, uint32_t ntiles = 0, int hstride = 1,
    const uint64_t* __restrict__ n_dev = nullptr) {
  if (!PERSIST) {  // one partition per CTA (grid = partitions; the last ticket is past them)
    onesweep_tile<K, MODE>(keys_in, vals_in, keys_out, vals_out, n, shift, digit_mask, hist, status, ticket,
                           INT64_MAX, err, keys_hi, lo_mask, ranges, ntiles, hstride);
    return;
  }
  if (n_dev) n = (int64_t)*n_dev;
  const int64_t parts = (n + kTileKeys - 1) / kTileKeys;
  while (onesweep_tile<K, MODE>(keys_in, vals_in, keys_out, vals_out, n, shift, digit_mask, hist, status, ticket,
                                parts, err, keys_hi, lo_mask, ranges, ntiles, hstride))
    __syncthreads();  // shared memory is reused by the next partition
}

// Grid of a persistent onesweep pass: the partitions, at most as many CTAs as
// fit on the device at once (the CTAs loop over partitions).
template <typename K, int MODE>
static unsigned onesweep_grid(const gsc_ctx* ctx, int64_t parts) {
  static int per_sm = 0;
  if (per_sm == 0) {
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, onesweep_kernel<K, MODE, true>, kThreads, 0) !=
            cudaSuccess ||
        nb < 1) {
      cudaGetLastError();
      nb = 1;
    }
    per_sm = nb;
  }
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(parts, (int64_t)per_sm * ctx->num_sms));
}

template <typename K>
size_t sort_scratch_bytes_t(int64_t n, int begin_bit, int end_bit) {
  const int npass = (end_bit - begin_bit + 7) / 8;
  const int64_t parts = (n + kTileKeys - 1) / kTileKeys;
  size_t b = align256((size_t)n * sizeof(K)) + align256((size_t)n * 4);
  b += align256((size_t)npass * 256 * 4 + (size_t)npass * parts * 256 * 4 + (size_t)npass * 4);
  return b;
}

size_t sort_scratch_bytes(int64_t n, int begin_bit, int end_bit) {
  return sort_scratch_bytes_t<uint64_t>(n, begin_bit, end_bit);
}
size_t sort_scratch_bytes_u32(int64_t n, int begin_bit, int end_bit) {
  return sort_scratch_bytes_t<uint32_t>(n, begin_bit, end_bit);
}

template <typename K>
static int sort_pairs_t(gsc_ctx* ctx, K* keys, uint32_t* vals, int64_t n, int begin_bit, int end_bit,
                        char* scratch) {
  cudaStream_t stream = ctx->stream;
  if (n <= 1 || end_bit <= begin_bit) return GSC_OK;
  const int npass = (end_bit - begin_bit + 7) / 8;
  const int64_t parts = (n + kTileKeys - 1) / kTileKeys;
  K* alt_keys = reinterpret_cast<K*>(scratch);
  scratch += align256((size_t)n * sizeof(K));
  uint32_t* alt_vals = reinterpret_cast<uint32_t*>(scratch);
  scratch += align256((size_t)n * 4);
  uint32_t* hist = reinterpret_cast<uint32_t*>(scratch);
  uint32_t* status = hist + npass * 256;
  uint32_t* tickets = status + (size_t)npass * parts * 256;
  const size_t meta = (size_t)npass * 256 * 4 + (size_t)npass * parts * 256 * 4 + (size_t)npass * 4;
  GS_CK(cudaMemsetAsync(hist, 0, meta, stream));

  const int64_t hblocks = min((int64_t)ctx->num_sms * 8, (n + 4095) / 4096);
  histogram_kernel<K><<<(unsigned)max((int64_t)1, hblocks), 256, 0, stream>>>(keys, n, begin_bit, end_bit,
                                                                             npass, hist);
  GS_CK_LAUNCH("histogram_kernel");
  K* src_k = keys;
  uint32_t* src_v = vals;
  K* dst_k = alt_keys;
  uint32_t* dst_v = alt_vals;
  for (int p = 0; p < npass; p++) {
    const int shift = begin_bit + 8 * p;
    const int bits = min(8, end_bit - shift);
    onesweep_kernel<K><<<(unsigned)parts, kThreads, 0, stream>>>(
        src_k, src_v, dst_k, dst_v, n, shift, (1u << bits) - 1u, hist + p * 256,
        status + (size_t)p * parts * 256, tickets + p, ctx->err);
    GS_CK_LAUNCH("onesweep_kernel");
    std::swap(src_k, dst_k);
    std::swap(src_v, dst_v);
  }
  if (src_k != keys) {
    GS_CK(cudaMemcpyAsync(keys, src_k, (size_t)n * sizeof(K), cudaMemcpyDeviceToDevice, stream));
    GS_CK(cudaMemcpyAsync(vals, src_v, (size_t)n * 4, cudaMemcpyDeviceToDevice, stream));
  }
  return GSC_OK;
}

int launch_sort_pairs(gsc_ctx* ctx, uint64_t* keys, uint32_t* vals, int64_t n, int begin_bit,
                      int end_bit, char* scratch) {
  return sort_pairs_t<uint64_t>(ctx, keys, vals, n, begin_bit, end_bit, scratch);
}

int launch_sort_pairs_u32(gsc_ctx* ctx, uint32_t* keys, uint32_t* vals, int64_t n, int begin_bit,
                          int end_bit, char* scratch) {
  return sort_pairs_t<uint32_t>(ctx, keys, vals, n, begin_bit, end_bit, scratch);
}

__global__ void __launch_bounds__(256) split_words_kernel(const uint64_t* __restrict__ in, int64_t n,
                                                          uint32_t* __restrict__ hi, uint32_t* __restrict__ lo,
                                                          uint32_t lo_mask) {
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= n) return;
  const uint64_t v = in[i];
  if (hi) hi[i] = (uint32_t)(v >> 32);
  lo[i] = (uint32_t)v & lo_mask;
}

// Packed-sort scratch: the pair-sort layout (alternate words, status words,
// compact histograms, tickets), then the wide histograms that a producer of
// the words fills (one counter per 128-byte line, kHistStride apart).
static size_t wide_hist_bytes(int begin_bit, int end_bit) {
  const int npass = end_bit > begin_bit ? (end_bit - begin_bit + 7) / 8 : 0;
  return align256((size_t)npass * 256 * kHistStride * 4);
}

size_t sort_scratch_bytes_packed(int64_t n, int begin_bit, int end_bit) {
  return sort_scratch_bytes_t<uint64_t>(n, begin_bit, end_bit) + wide_hist_bytes(begin_bit, end_bit);
}

static uint32_t* compact_hist(char* scratch, int64_t n) {
  return reinterpret_cast<uint32_t*>(scratch + align256((size_t)n * 8) + align256((size_t)n * 4));
}

uint32_t* sort_packed_hist(char* scratch, int64_t n, int begin_bit, int end_bit) {
  return reinterpret_cast<uint32_t*>(scratch + sort_scratch_bytes_t<uint64_t>(n, begin_bit, end_bit));
}

int sort_packed_clear(gsc_ctx* ctx, int64_t n, int begin_bit, int end_bit, char* scratch) {
  const int npass = end_bit > begin_bit ? (end_bit - begin_bit + 7) / 8 : 0;
  if (n < 1 || npass == 0) return GSC_OK;
  // compact histograms, status words and tickets, through the wide histograms
  char* from = reinterpret_cast<char*>(compact_hist(scratch, n));
  char* to = reinterpret_cast<char*>(sort_packed_hist(scratch, n, begin_bit, end_bit)) +
             wide_hist_bytes(begin_bit, end_bit);
  GS_CK(cudaMemsetAsync(from, 0, (size_t)(to - from), ctx->stream));
  return GSC_OK;
}

int launch_sort_packed(gsc_ctx* ctx, uint64_t* pairs, int64_t n, int begin_bit, int end_bit, uint32_t* hi_out,
                       uint32_t* lo_out, char* scratch, uint32_t lo_mask, bool hist_ready, uint32_t* ranges,
                       uint32_t ntiles, const uint64_t* n_dev) {
  cudaStream_t stream = ctx->stream;
  if (n <= 0) return GSC_OK;
  const int npass = end_bit > begin_bit ? (end_bit - begin_bit + 7) / 8 : 0;
  if (n_dev && (!hist_ready || npass == 0)) {
    set_error("launch_sort_packed: a device-side count needs producer-counted digits");
    return GSC_ERR_INVALID;
  }
  if (!n_dev && (npass == 0 || (n == 1 && !ranges))) {
    split_words_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(pairs, n, hi_out, lo_out, lo_mask);
    GS_CK_LAUNCH("split_words_kernel");
    return GSC_OK;
  }
  const int64_t parts = (n + kTileKeys - 1) / kTileKeys;
  uint64_t* alt = reinterpret_cast<uint64_t*>(scratch);
  uint32_t* hist = compact_hist(scratch, n);
  uint32_t* status = hist + npass * 256;
  uint32_t* tickets = status + (size_t)npass * parts * 256;
  const int hstride = hist_ready ? kHistStride : 1;
  if (hist_ready) {
    hist = sort_packed_hist(scratch, n, begin_bit, end_bit);
  } else {
    const int rc = sort_packed_clear(ctx, n, begin_bit, end_bit, scratch);
    if (rc != GSC_OK) return rc;
    const int64_t hblocks = min((int64_t)ctx->num_sms * 8, (n + 4095) / 4096);
    histogram_kernel<uint64_t><<<(unsigned)max((int64_t)1, hblocks), 256, 0, stream>>>(pairs, n, begin_bit,
                                                                                      end_bit, npass, hist);
    GS_CK_LAUNCH("histogram_kernel");
  }
  uint64_t* src = pairs;
  uint64_t* dst = alt;
  for (int p = 0; p < npass; p++) {
    const int shift = begin_bit + 8 * p;
    const int bits = min(8, end_bit - shift);
    if (p + 1 < npass) {
      if (n_dev)
        onesweep_kernel<uint64_t, 1, true><<<onesweep_grid<uint64_t, 1>(ctx, parts), kThreads, 0, stream>>>(
            src, nullptr, dst, nullptr, n, shift, (1u << bits) - 1u, hist + (size_t)p * 256 * hstride,
            status + (size_t)p * parts * 256, tickets + p, ctx->err, nullptr, 0xFFFFFFFFu, nullptr, 0, hstride,
            n_dev);
      else
        onesweep_kernel<uint64_t, 1><<<(unsigned)parts, kThreads, 0, stream>>>(
            src, nullptr, dst, nullptr, n, shift, (1u << bits) - 1u, hist + (size_t)p * 256 * hstride,
            status + (size_t)p * parts * 256, tickets + p, ctx->err, nullptr, 0xFFFFFFFFu, nullptr, 0, hstride);
    } else {
      if (n_dev)
        onesweep_kernel<uint64_t, 2, true><<<onesweep_grid<uint64_t, 2>(ctx, parts), kThreads, 0, stream>>>(
            src, nullptr, nullptr, lo_out, n, shift, (1u << bits) - 1u, hist + (size_t)p * 256 * hstride,
            status + (size_t)p * parts * 256, tickets + p, ctx->err, hi_out, lo_mask, ranges, ntiles, hstride,
            n_dev);
      else
        onesweep_kernel<uint64_t, 2><<<(unsigned)parts, kThreads, 0, stream>>>(
            src, nullptr, nullptr, lo_out, n, shift, (1u << bits) - 1u, hist + (size_t)p * 256 * hstride,
            status + (size_t)p * parts * 256, tickets + p, ctx->err, hi_out, lo_mask, ranges, ntiles, hstride);
    }
    GS_CK_LAUNCH("onesweep_kernel");
    std::swap(src, dst);
  }
  return GSC_OK;
}

}  // namespace gs
