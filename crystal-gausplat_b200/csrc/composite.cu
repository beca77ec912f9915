// composite.cu — per-tile alpha compositing, forward and backward.
//
// Forward replaces rasterize_tile (src/metal/kernels/gaussian.metal:364-445)
// over EVERY 16x16 tile (the reference's dispatch covers only
// ceil(tx/16) x ceil(ty/16) of them, rasterizer.cr:332). One CTA of 256
// threads per tile, one pixel per thread; the tile's sorted Gaussians are
// staged 256 at a time into shared memory as packed records (three float4 per
// Gaussian) and every thread walks the batch front to back while T > t_stop.
// The CTA leaves as soon as every pixel is done.
//
// Backward replaces rasterize_backward (gaussian.metal:452-567): batches are
// staged back to front; per Gaussian each thread forms its 9 partials, the
// warp sums them through a shared-memory transpose and lanes 0-8 issue the
// global atomics. The L1 loss
// gradient (src/ops/loss.cr:33-57) is fused into the per-pixel load.
//
// Skip test: a pixel whose power lies below its Gaussian's cut has
// o*G < alpha_min, so it is rejected before the exponential. The cut is
// ln(alpha_min / o) minus a margin far above the exponential's and the
// logarithm's error (pixel_power_cut; ln(alpha_min) minus a margin where the
// whole-tile test has no per-Gaussian threshold), so the accepted set is
// exactly the one the full test gives.
#include "common.cuh"
#include "cull.cuh"
#include "kernels.cuh"

namespace gs {

// Whole-tile rejection (tile_culled) lives in cull.cuh.

// Stable compaction of the batch survivors: returns this thread's slot (or
// -1) and the survivor count; needs a 8-entry shared scratch.
template <int NW = 8>
__device__ __forceinline__ int compact_slot(bool keep, uint32_t* s_cnt, int* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const uint32_t bal = __ballot_sync(0xffffffffu, keep);
  if (lane == 0) s_cnt[w] = __popc(bal);
  __syncthreads();
  int base = 0, tot = 0;
#pragma unroll
  for (int k = 0; k < NW; k++) {
    const int c = (int)s_cnt[k];
    base += k < w ? c : 0;
    tot += c;
  }
  *total = tot;
  return keep ? base + __popc(bal & ((1u << lane) - 1u)) : -1;
}

// Minimum resident CTAs per SM (register budget) of the two kernels.
#ifndef GS_FWD_MIN_CTAS
#define GS_FWD_MIN_CTAS 5
#endif
#ifndef GS_BWD_MIN_CTAS
#define GS_BWD_MIN_CTAS 7
#endif
// Backward: skip, per warp, the entries behind all of its pixels' last
// contributors; send the partials of a Gaussian that at most GS_BWD_DIRECT
// lanes of a warp hit straight to global memory instead of through the
// warp's transpose reduction.
// Forward: the next batch's splat records are fetched into shared memory with
// cp.async while the current batch is composited.
#ifndef GS_FWD_CPASYNC
#define GS_FWD_CPASYNC 1
#endif

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

#ifndef GS_BWD_WARP_HI
#define GS_BWD_WARP_HI 1
#endif
#ifndef GS_BWD_FAST_EXP
#define GS_BWD_FAST_EXP 1
#endif
#ifndef GS_BWD_FAST_OMAX  // opacity bound of the hardware exponential (below alpha_max)
#define GS_BWD_FAST_OMAX 0.98f
#endif
// e^x as 2^(x log2 e) on the hardware's approximate base-2 exponential
// (subnormal results flushed to zero; they lie far below any accepted alpha).
__device__ __forceinline__ float exp_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.44269504088896341f));
  return y;
}
#ifndef GS_BWD_DIRECT
#define GS_BWD_DIRECT 2
#endif

__global__ void __launch_bounds__(256, GS_FWD_MIN_CTAS) composite_fwd_kernel(CompositeFwdArgs a) {
  // Staged batch, one record per surviving list entry:
  //   s0 = {mean.x, mean.y, -A/2, -B}, s1 = {-C/2, opacity, per-Gaussian power cut, -},
  //   s2 = {r, g, b, -} (read only by accepted pixels)
  __shared__ float4 s0[256];
  __shared__ float4 s1[256];
  __shared__ float4 s2[256];
  const int tile = blockIdx.x;
  const int tx = tile % a.tiles_x, ty = tile / a.tiles_x;
  const int tid = threadIdx.x;
  const int x = tx * GS_TILE + (tid & 15), y = ty * GS_TILE + (tid >> 4);
  const bool inside = x < a.width && y < a.height;
  const float pxf = (float)x + 0.5f, pyf = (float)y + 0.5f;
  const uint32_t start = a.ranges[2 * tile], end = a.ranges[2 * tile + 1];
  const float4* __restrict__ splats = reinterpret_cast<const float4*>(a.splats);
  const float t_stop = a.t_stop, amin = a.alpha_min, amax = a.alpha_max, cut = a.power_cut;
  // every power that reaches the exponential lies in [cut, 0]
  const bool short_exp = cut >= -87.0f;

  __shared__ uint32_t s_idx[256];
  __shared__ uint32_t s_cnt[8];
  const float rx0 = tx * GS_TILE + 0.5f, ry0 = ty * GS_TILE + 0.5f;
  const float rx1 = min(tx * GS_TILE + GS_TILE, a.width) - 0.5f;
  const float ry1 = min(ty * GS_TILE + GS_TILE, a.height) - 0.5f;

  const bool sliced = a.tile_base != nullptr;
  const bool first = !sliced || a.first_slice, last_slice = !sliced || a.last_slice;
  const uint32_t base = sliced ? a.tile_base[tile] : 0u;  // list index of this slice's first entry
  const size_t pix = (size_t)y * a.width + x;
  float T = 1.0f, C0 = 0.0f, C1 = 0.0f, C2 = 0.0f;
  uint32_t cnt = 0, lst = 0;
  // a tile whose pixels all stopped in an earlier slice has nothing to add
  const bool tile_skip =
      sliced && !first && ((a.tile_done[(size_t)ty * a.done_words + (tx >> 6)] >> (tx & 63)) & 1ull);
  if (!first && inside && (!tile_skip || last_slice)) {
    T = a.final_T[pix];
    C0 = a.image[pix * 3 + 0];
    C1 = a.image[pix * 3 + 1];
    C2 = a.image[pix * 3 + 2];
    cnt = a.n_contrib[pix];
    lst = a.last[pix];
  }
  bool done = !inside || !(T > t_stop);
#if GS_FWD_CPASYNC
  // Each thread stages the 48-byte record of its own entry of the next batch
  // (s_raw[3 tid .. 3 tid + 2]) and reads it back itself after waiting for
  // its own copies; the entry's id is loaded one batch earlier still.
  __shared__ float4 s_raw[3 * 256];
  uint32_t gid_next = 0;
  if (!tile_skip && start < end) {
    if (start + tid < end) {
      const float4* src = splats + (size_t)a.vals[start + tid] * 3;
      cp_async16(&s_raw[3 * tid], src);
      cp_async16(&s_raw[3 * tid + 1], src + 1);
      cp_async16(&s_raw[3 * tid + 2], src + 2);
    }
    cp_async_commit();
    if (start + 256 + tid < end) gid_next = a.vals[start + 256 + tid];
  }
#endif
  for (uint32_t b = start; b < end && !tile_skip; b += 256) {
    if (__syncthreads_count(done) == 256) break;
    const uint32_t idx = b + tid;
    float4 g0, g1;
    float g2 = 0.0f, pcut = cut;
    bool keep = false;
#if GS_FWD_CPASYNC
    cp_async_wait_all();
#endif
    if (idx < end) {
#if GS_FWD_CPASYNC
      g0 = s_raw[3 * tid];
      g1 = s_raw[3 * tid + 1];
      g2 = s_raw[3 * tid + 2].x;
#else
      const uint32_t gid = a.vals[idx];
      g0 = splats[(size_t)gid * 3];
      g1 = splats[(size_t)gid * 3 + 1];
      g2 = splats[(size_t)gid * 3 + 2].x;
#endif
      const CullGauss cg = cull_prepare(g0, g1.x, g1.y, amin);
      keep = !cull_tile(cg, rx0, rx1, ry0, ry1);
      pcut = pixel_power_cut(cg, cut);
    }
    int m;
    const int slot = compact_slot(keep, s_cnt, &m);
    if (slot >= 0) {
      // conic pre-scaled by powers of two (-A/2, -B, -C/2); the power below is
      // fma(dy dy, -C/2, fma(dx dy, -B, dx dx (-A/2))), the oracle's formula
      s0[slot] = make_float4(g0.x, g0.y, -0.5f * g0.z, -g0.w);
      s1[slot] = make_float4(-0.5f * g1.x, g1.y, pcut, 0.0f);
      s2[slot] = make_float4(g1.z, g1.w, g2, 0.0f);
      s_idx[slot] = idx - start;
    }
#if GS_FWD_CPASYNC
    if (b + 256 < end) {  // the next batch's records, while this one is composited
      if (b + 256 + tid < end) {
        const float4* src = splats + (size_t)gid_next * 3;
        cp_async16(&s_raw[3 * tid], src);
        cp_async16(&s_raw[3 * tid + 1], src + 1);
        cp_async16(&s_raw[3 * tid + 2], src + 2);
      }
      cp_async_commit();
      gid_next = b + 512 + tid < end ? a.vals[b + 512 + tid] : 0u;
    }
#endif
    __syncthreads();
    if (!done) {
      int jl = -1;  // slot of the last accepted entry of this batch
      for (int j = 0; j < m; j++) {
        const float4 q0 = s0[j];
        const float dx = pxf - q0.x, dy = pyf - q0.y;
        const float4 q1 = s1[j];
        const float power = fmaf(dy * dy, q1.x, fmaf(dx * dy, q0.w, dx * dx * q0.z));
        if (power > 0.0f || power < q1.z) continue;
        const float G = short_exp ? gs_expf_pixel(power) : gs_expf(power);
        const float alpha = fminf(amax, q1.y * G);
        if (alpha < amin) continue;
        const float4 c = s2[j];
        const float w = T * alpha;
        C0 = fmaf(w, c.x, C0);
        C1 = fmaf(w, c.y, C1);
        C2 = fmaf(w, c.z, C2);
        T *= (1.0f - alpha);
        cnt++;
        jl = j;
        if (!(T > t_stop)) {
          done = true;
          break;
        }
      }
      if (jl >= 0) lst = base + s_idx[jl] + 1;
    }
  }
#if GS_FWD_CPASYNC
  cp_async_wait_all();  // no copy outlives the loop (an early stop leaves one in flight)
#endif
  if (!last_slice) {
    // hand the state to the next slice; mark the tile if every pixel stopped
    if (tile_skip) {
      if (tid == 0) a.tile_base[tile] = base + (end - start);
      return;
    }
    const bool all_done = __syncthreads_count(done) == 256;
    if (tid == 0) {
      a.tile_base[tile] = base + (end - start);
      if (all_done) atomicOr(&a.tile_done[(size_t)ty * a.done_words + (tx >> 6)], 1ull << (tx & 63));
      // a tile still open with a finite cut may have second-slice pairs
      else if (a.open_flag && a.tile_cut[tile] < __int_as_float(0x7f800000)) atomicOr(a.open_flag, 1u);
    }
    if (!inside) return;
    a.final_T[pix] = T;
    a.image[pix * 3 + 0] = C0;
    a.image[pix * 3 + 1] = C1;
    a.image[pix * 3 + 2] = C2;
    a.n_contrib[pix] = cnt;
    a.last[pix] = lst;
    return;
  }
  if (a.mark_done && !tile_skip) {  // the next tile cut needs to know which tiles stopped
    const bool all_done = __syncthreads_count(done) == 256;
    if (tid == 0 && all_done)
      atomicOr(&a.tile_done[(size_t)ty * a.done_words + (tx >> 6)], 1ull << (tx & 63));
  }
  const uint32_t list_len = base + (end - start);  // the whole tile list, every slice
  if (a.pge) {  // tracing: entries visited before the stop (whole list if never stopped)
    __shared__ unsigned long long s_pge;
    if (tid == 0) s_pge = 0;
    __syncthreads();
    uint32_t visited = !inside ? 0u : (!(T > t_stop) ? lst : list_len);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) visited += __shfl_xor_sync(0xffffffffu, visited, off);
    if ((tid & 31) == 0) atomicAdd(&s_pge, (unsigned long long)visited);
    __syncthreads();
    if (tid == 0) atomicAdd(a.pge, s_pge);
  }
  if (a.tile_work) {  // the backward's list length for this tile: max over pixels of `last`
    __shared__ uint32_t s_work;
    if (tid == 0) s_work = 0u;
    __syncthreads();
    uint32_t v = inside ? lst : 0u;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, off));
    if ((tid & 31) == 0 && v) atomicMax(&s_work, v);
    __syncthreads();
    if (tid == 0) a.tile_work[tile] = s_work;
  }
  if (!inside) return;
  a.image[pix * 3 + 0] = fmaf(T, a.bg[0], C0);
  a.image[pix * 3 + 1] = fmaf(T, a.bg[1], C1);
  a.image[pix * 3 + 2] = fmaf(T, a.bg[2], C2);
  if (a.n_contrib) a.n_contrib[pix] = cnt;
  if (a.final_T) a.final_T[pix] = T;
  if (a.last) a.last[pix] = lst;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// One pixel's backward state.
struct BwdPixel {
  bool inside;
  float pyf;
  float g[3];
  float T;
  float ag;  // (colour behind this Gaussian, incl. background) . g -- the only use of it
  uint32_t hi;
};

// Partials of one pixel for one Gaussian (gaussian.metal:505-566; FULL mode
// adds the conic gradient, the alpha clamp and the corrected running colour).
template <bool FULL>
__device__ __forceinline__ bool bwd_pixel(BwdPixel& P, uint32_t idx, float4 g0, float4 g1, float g2,
                                          float cut, float amin, float amax, float amin_lo, float amin_hi,
                                          bool short_exp, bool fast, float dx, float dxxa, float v[9]) {
  if (!(P.inside && idx < P.hi)) return false;
  // dx and dx dx (-A/2) are shared by the thread's pixels (one column)
  const float dy = P.pyf - g0.y;
  const float power = fmaf(dy * dy, g1.x, fmaf(dx * dy, g0.w, dxxa));  // == forward's power
  if (power > 0.0f || power < cut) return false;
  const float o = g1.y;
  float G, alpha;
#if GS_BWD_FAST_EXP
  if (fast) {
    // o < GS_BWD_FAST_OMAX < alpha_max: o G never reaches the clamp, and G
    // is the hardware exponential (ex2.approx of power * log2 e, about 2e-7
    // relative): the gradients only need to be within tolerance. Where o G
    // falls within 1e-5 of alpha_min the forward's exponential decides
    // instead, so that the accepted set is exactly the forward's.
    G = exp_approx(power);
    alpha = o * G;
    if (alpha < amin_hi) {
      if (alpha < amin_lo) return false;
      G = short_exp ? gs_expf_pixel(power) : gs_expf(power);
      alpha = o * G;
      if (alpha < amin) return false;
    }
  } else
#endif
  {
    // Same exponential and tests as the forward, so the accepted set matches it.
    G = short_exp ? gs_expf_pixel(power) : gs_expf(power);
    alpha = fminf(amax, o * G);
    if (alpha < amin) return false;
  }
  // From here on the gradients only need to be within tolerance, so products
  // and sums are fused (explicit fmaf; the file is built without contraction).
  // T_before = T / (1 - alpha) and dL/dalpha = T_before c.g - (acc / (1 - alpha)).g,
  // with one reciprocal and the running colour kept as acc.g. 1 - alpha lies
  // in [0.01, 1], so the hardware's approximate reciprocal (__fdividef) is
  // accurate to a couple of ulps there; it measured 2 % faster than the
  // correctly rounded one, with the gradient gate unchanged.
  const float inv = __fdividef(1.0f, 1.0f - alpha);
  const float T_before = P.T * inv;
  const float wgt = T_before * alpha;
  const float cg = fmaf(g2, P.g[2], fmaf(g1.w, P.g[1], g1.z * P.g[0]));
  v[6] = fmaf(wgt, P.g[0], v[6]);
  v[7] = fmaf(wgt, P.g[1], v[7]);
  v[8] = fmaf(wgt, P.g[2], v[8]);
  const float dL_dalpha = fmaf(T_before, cg, -P.ag * inv);
  float dL_dG, dL_do;
  if (FULL && !(o * G <= amax)) {
    dL_dG = 0.0f;
    dL_do = 0.0f;
  } else {
    dL_dG = dL_dalpha * o;
    dL_do = dL_dalpha * G;
  }
  const float dL_dpower = dL_dG * G;
  // g0 = {mean, -A/2, -B}, g1.x = -C/2 (pre-scaled conic, see fwd):
  // dpower/dmean = -(2 g0.z dx + g0.w dy, g0.w dx + 2 g1.x dy)
  const float px_ = dL_dpower * dx, py_ = dL_dpower * dy;
  v[0] = fmaf(-2.0f * g0.z, px_, fmaf(-g0.w, py_, v[0]));
  v[1] = fmaf(-2.0f * g1.x, py_, fmaf(-g0.w, px_, v[1]));
  if (FULL) {
    v[2] = fmaf(-0.5f * dx, px_, v[2]);
    v[3] = fmaf(-dx, py_, v[3]);
    v[4] = fmaf(-0.5f * dy, py_, v[4]);
  }
  v[5] += dL_do;
  P.T = T_before;
  P.ag = fmaf(FULL ? wgt : -wgt, cg, P.ag);  // REF keeps gaussian.metal:566
  return true;
}

// 128 threads per tile, two pixels per thread (rows r and r + 8), so each
// warp reduction covers 64 pixels.
constexpr int kBwdPix = 2;                        // pixels per thread
constexpr int kBwdThreads = GS_TILE_PIXELS / kBwdPix;  // 128
constexpr int kBwdWarps = kBwdThreads / 32;
constexpr int kBwdRowStep = GS_TILE / kBwdPix;        // rows between a thread's pixels

template <bool FULL, bool L1>
__global__ void __launch_bounds__(kBwdThreads, GS_BWD_MIN_CTAS) composite_bwd_kernel(CompositeBwdArgs a) {
  __shared__ float4 s0[kBwdThreads];
  __shared__ float4 s1[kBwdThreads];
  __shared__ float2 s2[kBwdThreads];  // {b, per-Gaussian power cut}
  __shared__ uint32_t s_gid[kBwdThreads];
  __shared__ uint32_t s_idx[kBwdThreads];
  __shared__ uint32_t s_cnt[kBwdWarps];
  __shared__ uint32_t s_hi;
  __shared__ float s_loss[kBwdWarps];
  // per-warp transpose buffer of the 9 partials (rows padded to 36 floats)
  __shared__ __align__(16) float s_red[kBwdWarps][9 * 36];
  const int tile = a.tile_order ? (int)a.tile_order[blockIdx.x] : (int)blockIdx.x;
  const int tx = tile % a.tiles_x, ty = tile / a.tiles_x;
  const int tid = threadIdx.x, lane = tid & 31;
  const uint32_t start = a.ranges[2 * tile], end = a.ranges[2 * tile + 1];
  const float4* __restrict__ splats = reinterpret_cast<const float4*>(a.splats);
  const float amin = a.alpha_min, amax = a.alpha_max, cut = a.power_cut;
  const bool short_exp = cut >= -87.0f;
  const float amin_lo = amin * (1.0f - 1e-5f), amin_hi = amin * (1.0f + 1e-5f);  // exact-decision band
  const float fast_omax = fminf(GS_BWD_FAST_OMAX, amax * (1.0f - 1e-5f));

  BwdPixel P[kBwdPix];
  const float pxf = (float)(tx * GS_TILE + (tid & 15)) + 0.5f;  // the thread's pixel column
  float loss = 0.0f;
#pragma unroll
  for (int h = 0; h < kBwdPix; h++) {
    const int x = tx * GS_TILE + (tid & 15), y = ty * GS_TILE + (tid >> 4) + kBwdRowStep * h;
    BwdPixel& Q = P[h];
    Q.inside = x < a.width && y < a.height;
    Q.pyf = (float)y + 0.5f;
    Q.T = 1.0f;
    Q.hi = start;
    Q.g[0] = Q.g[1] = Q.g[2] = 0.0f;
    if (Q.inside) {
      const size_t pix = (size_t)y * a.width + x;
#pragma unroll
      for (int c = 0; c < 3; c++) {
        if (L1) {
          const float diff = a.image[pix * 3 + c] - a.target[pix * 3 + c];
          const float sg = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
          Q.g[c] = sg * a.l1_scale;
          loss += fabsf(diff) * a.l1_scale;
        } else {
          Q.g[c] = a.dL_dimage[pix * 3 + c];
        }
      }
      Q.T = a.final_T[pix];
      Q.hi = FULL ? start + a.last[pix] : end;
    }
    Q.ag = (a.bg[0] * Q.T) * Q.g[0] + (a.bg[1] * Q.T) * Q.g[1] + (a.bg[2] * Q.T) * Q.g[2];
  }

  if (L1 && a.loss_sum) {
    const float l = warp_sum(loss);
    if (lane == 0) s_loss[tid >> 5] = l;
  }
  if (tid == 0) s_hi = start;
  __syncthreads();
  if (L1 && a.loss_sum && tid == 0) {
    float t = 0.0f;
    for (int w = 0; w < kBwdWarps; w++) t += s_loss[w];
    if (t != 0.0f) atomicAdd(a.loss_sum, t);
  }
  if (FULL) {
    uint32_t mh = P[0].hi;
#pragma unroll
    for (int h = 1; h < kBwdPix; h++) mh = max(mh, P[h].hi);
    atomicMax(&s_hi, mh);
  }
  __syncthreads();
  const uint32_t hi = FULL ? s_hi : end;
#if GS_BWD_WARP_HI
  // The warp's own list length: entries at or past every one of its pixels'
  // last contributor are skipped as a block (the per-pixel test stays).
  uint32_t whi = end;
  if (FULL) whi = __reduce_max_sync(0xffffffffu, max(P[0].hi, P[1].hi));
#endif

  const float rx0 = tx * GS_TILE + 0.5f, ry0 = ty * GS_TILE + 0.5f;
  const float rx1 = min(tx * GS_TILE + GS_TILE, a.width) - 0.5f;
  const float ry1 = min(ty * GS_TILE + GS_TILE, a.height) - 0.5f;
  const int red_row = lane / 3, red_part = lane - 3 * (lane / 3);  // reduction roles
  for (int64_t bend = hi; bend > (int64_t)start; bend -= kBwdThreads) {
    const int64_t bstart = max((int64_t)start, bend - kBwdThreads);
    const int mb = (int)(bend - bstart);
    __syncthreads();
    bool keep = false;
    float4 q0, q1;
    float q2 = 0.0f, pcut = cut;
    uint32_t gid = 0;
    if (tid < mb) {
      gid = a.vals[bend - 1 - tid];
      q0 = splats[(size_t)gid * 3];
      q1 = splats[(size_t)gid * 3 + 1];
      q2 = splats[(size_t)gid * 3 + 2].x;
      const CullGauss cg = cull_prepare(q0, q1.x, q1.y, amin);
      keep = !cull_tile(cg, rx0, rx1, ry0, ry1);
      pcut = pixel_power_cut(cg, cut);
    }
    int m;
    const int slot = compact_slot<kBwdWarps>(keep, s_cnt, &m);
    if (slot >= 0) {
      s_gid[slot] = gid;
      s0[slot] = make_float4(q0.x, q0.y, -0.5f * q0.z, -q0.w);
      s1[slot] = make_float4(-0.5f * q1.x, q1.y, q1.z, q1.w);
      s2[slot] = make_float2(q2, pcut);
      s_idx[slot] = (uint32_t)(bend - 1 - tid);
    }
    __syncthreads();
    int j0 = 0;
#if GS_BWD_WARP_HI
    if (FULL) {  // the batch is in descending list order: first slot below whi
      int lo = 0, up = m;
      while (lo < up) {
        const int mid = (lo + up) >> 1;
        if (s_idx[mid] >= whi) lo = mid + 1; else up = mid;
      }
      j0 = lo;
    }
#endif
    for (int j = j0; j < m; j++) {
      const uint32_t idx = s_idx[j];
      const float4 g0 = s0[j];
      const float4 g1 = s1[j];
      const float2 g2 = s2[j];
      float v[9];
#pragma unroll
      for (int k = 0; k < 9; k++) v[k] = 0.0f;
      bool ok = false;
      const float dx = pxf - g0.x, dxxa = dx * dx * g0.z;
      const bool fast = g1.y < fast_omax;  // the same for every lane
#pragma unroll
      for (int h = 0; h < kBwdPix; h++)
        ok |= bwd_pixel<FULL>(P[h], idx, g0, g1, g2.x, g2.y, amin, amax, amin_lo, amin_hi, short_exp, fast, dx,
                              dxxa, v);
      const uint32_t hits = __ballot_sync(0xffffffffu, ok);
#if GS_BWD_DIRECT > 0
      if (hits && __popc(hits) <= GS_BWD_DIRECT) {
        // few lanes hit: their partials go straight to the global sums
        if (ok) {
          float* dst = a.grad2d + (size_t)s_gid[j] * 9;
#pragma unroll
          for (int k = 0; k < 9; k++)
            if (v[k] != 0.0f) atomicAdd(dst + k, v[k]);
        }
      } else
#endif
      if (hits) {
        float* red = s_red[tid >> 5];
#pragma unroll
        for (int k = 0; k < 9; k++) red[k * 36 + lane] = v[k];
        __syncwarp();
        // row k (32 lanes' partials of field k) is summed by lanes 3k..3k+2,
        // three, three and two float4 each (conflict-free: the 8 lanes of a
        // quarter-warp cover 32 distinct banks), then folded into lane 3k
        float r = 0.0f;
        if (lane < 27) {
          const float4* row = reinterpret_cast<const float4*>(red + red_row * 36) + red_part * 3;
          const float4 t0 = row[0], t1 = row[1];
          r = ((t0.x + t0.y) + (t0.z + t0.w)) + ((t1.x + t1.y) + (t1.z + t1.w));
          if (red_part < 2) {
            const float4 t2 = row[2];
            r += (t2.x + t2.y) + (t2.z + t2.w);
          }
        }
        const float r1 = __shfl_down_sync(0xffffffffu, r, 1);
        const float r2 = __shfl_down_sync(0xffffffffu, r, 2);
        if (lane < 27 && red_part == 0) {
          r = (r + r1) + r2;
          if (r != 0.0f) atomicAdd(a.grad2d + (size_t)s_gid[j] * 9 + red_row, r);
        }
        __syncwarp();
      }
    }
  }
}

int launch_composite_fwd(const CompositeFwdArgs& a, cudaStream_t stream) {
  const int tiles = a.tiles_x * a.tiles_y;
  if (tiles == 0) return GSC_OK;
  composite_fwd_kernel<<<tiles, 256, 0, stream>>>(a);
  GS_CK_LAUNCH("composite_fwd_kernel");
  return GSC_OK;
}

int launch_composite_bwd(const CompositeBwdArgs& a, bool full, cudaStream_t stream) {
  const int tiles = a.tiles_x * a.tiles_y;
  if (tiles == 0) return GSC_OK;
  const bool l1 = a.target != nullptr;
  if (full && l1) composite_bwd_kernel<true, true><<<tiles, kBwdThreads, 0, stream>>>(a);
  else if (full) composite_bwd_kernel<true, false><<<tiles, kBwdThreads, 0, stream>>>(a);
  else if (l1) composite_bwd_kernel<false, true><<<tiles, kBwdThreads, 0, stream>>>(a);
  else composite_bwd_kernel<false, false><<<tiles, kBwdThreads, 0, stream>>>(a);
  GS_CK_LAUNCH("composite_bwd_kernel");
  return GSC_OK;
}

}  // namespace gs
