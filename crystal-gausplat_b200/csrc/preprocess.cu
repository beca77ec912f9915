// preprocess.cu — fused per-Gaussian forward: scale exp, quaternion, 3-D
// covariance, EWA projection with culling, conic, radius, tile count, SH
// colour and opacity sigmoid (src/metal/kernels/gaussian.metal:90-308,
// src/gaussian_splatting/gaussian.cr:119-142, rasterizer.cr:110-171).
//
// One thread per Gaussian, 128 per block. The 192-byte SH rows of a block are
// staged through shared memory with coalesced float4 loads, into rows padded
// to 13 float4 so that the per-thread float4 reads are free of bank conflicts.
//
// Binning record (32 bytes per Gaussian and view): {x0, y0, rect width, pair
// count}, {tile mask low, high, bits(depth), 0}.
//
// Packed splat record (12 floats, private to this library):
//   s0 = {mean.x, mean.y, conic.xx, conic.xy}
//   s1 = {conic.yy, opacity (0 if culled or det <= 0), r, g}
//   s2 = {b, depth, radius, bits(tiles_touched)}
#include "cull.cuh"
#include "geometry.cuh"
#include "kernels.cuh"

namespace gs {

constexpr int kPreThreads = 128;

// The two halves of contributing-pairs binning's per-tile test for tile
// column tx of a row (see row_extent): its pixel-centre span [rx0, rx1]
// reaches right of xl, and starts left of xr.
__device__ __forceinline__ bool row_tile_right_ok(const RowCull& rc, int tx, int width, float xl) {
  const float rx1 = min(tx * GS_TILE + GS_TILE, width) - 0.5f;
  return rx1 - rc.mx >= xl;
}
__device__ __forceinline__ bool row_tile_left_ok(const RowCull& rc, int tx, float xr) {
  const float rx0 = tx * GS_TILE + 0.5f;
  return rx0 - rc.mx <= xr;
}
constexpr int kShRow = 13;  // float4 per staged SH row (12 used + 1 pad)

// One Gaussian per thread; a.nviews views per launch. The camera-independent
// terms (scales, quaternion, 3-D covariance, opacity, the staged SH row) are
// formed once and every view's record, mask and depth word are written to that
// view's buffers.
#ifndef GS_PRE_MIN_CTAS
#define GS_PRE_MIN_CTAS 8
#endif
__global__ void __launch_bounds__(kPreThreads, GS_PRE_MIN_CTAS) preprocess_kernel(PreprocessArgs a) {
  __shared__ float4 s_sh[kPreThreads * kShRow];
  const int64_t base = (int64_t)blockIdx.x * kPreThreads;
  const int64_t i = base + threadIdx.x;
  const int64_t n = a.n;
  const gsc_raster_config& cfg = a.cfg;

  // Coalesced staging of this block's SH coefficients (48 floats each).
  {
    const int64_t cnt = min((int64_t)kPreThreads, n - base);
    const float4* src = reinterpret_cast<const float4*>(a.sh + base * 48);
    for (int k = threadIdx.x; k < cnt * 12; k += kPreThreads) s_sh[(k / 12) * kShRow + k % 12] = src[k];
  }
  __syncthreads();

  float p[3] = {0.0f, 0.0f, 0.0f}, c3[6] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f}, o = 0.0f;
  if (i < n) {
    p[0] = a.pos[i * 3]; p[1] = a.pos[i * 3 + 1]; p[2] = a.pos[i * 3 + 2];
    const float s[3] = {gs_expf(a.log_scale[i * 3]), gs_expf(a.log_scale[i * 3 + 1]),
                        gs_expf(a.log_scale[i * 3 + 2])};
    float4 q4 = reinterpret_cast<const float4*>(a.rot)[i];
    float q[4], qn;
    load_quat(q4, cfg.mode, q, &qn);
    float R[3][3];
    quat_to_R(q[0], q[1], q[2], q[3], R);
    cov3d_of(s, R, c3);
    o = gs_sigmoid(a.logit_opacity[i]);
    if (a.cov3d) {
#pragma unroll
      for (int k = 0; k < 6; k++) a.cov3d[i * 6 + k] = c3[k];
    }
    if (a.opacity) a.opacity[i] = o;
  }
  const float4* shrow = s_sh + threadIdx.x * kShRow;

  for (int v = 0; v < a.nviews; v++) {
    const gsc_camera& cam = a.cams[v];
    const bool stage_out = a.nviews == 1;  // the per-Gaussian outputs of the stage entry point
    uint32_t tiles = 0;
    float col_b = 0.0f, depth_o = 0.0f, radius_o = 0.0f;
    uint32_t nt = 0;  // contributing tiles of this thread's Gaussian (contributing-pairs binning)
    uint64_t mask_o = ~0ull;
    int rx_o = 0, ry_o = 0, rw_o = 1;
    if (i < n) {
      Projected pr;
      project(p, c3, cam, cfg, &pr);

      // colour
      float d[3], len;
      view_dir(p, cam, d, &len);
      float b[16];
      sh_basis_hi(d[0], d[1], d[2], b);
      float raw[3];
      sh_eval([&](int k) { return reinterpret_cast<const float*>(shrow)[k]; }, d[0], d[1], d[2], b,
              cfg.sh_degree, cfg.mode, raw);
      float col[3];
#pragma unroll
      for (int c = 0; c < 3; c++) col[c] = fmaxf(0.0f, raw[c] + 0.5f);

      float px = -1000.0f, py = -1000.0f, depth = 0.0f, radius = 0.0f;
      int x0 = 0, x1 = -1, y0 = 0, y1 = -1;
      if (pr.visible) {
        px = pr.px; py = pr.py; depth = pr.zc; radius = pr.r;
        if (pr.r > 0.0f && pr.zc > 0.0f) {
          tile_bounds(px, py, pr.r, a.tiles_x, a.tiles_y, &x0, &x1, &y0, &y1);
          if (x1 >= x0 && y1 >= y0) tiles = (uint32_t)((x1 - x0 + 1) * (y1 - y0 + 1));
        }
      }
      const float o_eff = (pr.visible && pr.det > 0.0f) ? o : 0.0f;
      const float4 g0 = make_float4(px, py, pr.A, pr.B);
      // Contributing-pairs binning: the rect's tiles (<= 64) that meet the
      // ellipse, row by row (bit = row-major position in the rect).
      if (a.contributing) {
        uint64_t mask = ~0ull;
        if (tiles > 0 && tiles <= 64) {
          const RowCull rc = row_cull_prepare(g0, pr.Cc, o_eff, cfg.alpha_min);
          if (rc.kind != 0) {
            mask = 0ull;
            const int wx = x1 - x0 + 1;
            for (int ty = y0, bit = 0; ty <= y1; ty++, bit += wx) {
              float ry0, ry1, xl = 0.0f, xr = -1.0f, rx0, rx1;
              tile_pixel_rect(x0, ty, cam.width, cam.height, &rx0, &rx1, &ry0, &ry1);
              if (!(rc.kind == 2 && row_extent(rc, ry0, ry1, &xl, &xr))) continue;
              // A tile tx of the row survives iff rx1(tx) - mx >= xl and
              // rx0(tx) - mx <= xr. Both sides are monotone in tx, so the
              // survivors are one run [ta, tb]: estimate its ends, then move
              // them with the exact per-tile tests (usually no step).
              int ta = x0, tb = x1;
              if (!row_tile_right_ok(rc, ta, cam.width, xl)) {
                ta = min(max((int)ceilf((xl + rc.mx - 15.5f) * 0.0625f), x0), x1 + 1);
                while (ta > x0 && row_tile_right_ok(rc, ta - 1, cam.width, xl)) ta--;
                while (ta <= x1 && !row_tile_right_ok(rc, ta, cam.width, xl)) ta++;
              }
              if (!row_tile_left_ok(rc, tb, xr)) {
                tb = max(min((int)floorf((xr + rc.mx - 0.5f) * 0.0625f), x1), x0 - 1);
                while (tb < x1 && row_tile_left_ok(rc, tb + 1, xr)) tb++;
                while (tb >= x0 && !row_tile_left_ok(rc, tb, xr)) tb--;
              }
              if (ta <= tb) {
                const int len = tb - ta + 1;
                const uint64_t run = len >= 64 ? ~0ull : (1ull << len) - 1ull;
                mask |= run << (bit + (ta - x0));
              }
            }
          } else {
            mask = tiles == 64 ? ~0ull : (1ull << tiles) - 1ull;
          }
          nt = (uint32_t)__popcll(mask);
        } else {
          nt = tiles;
        }
        mask_o = mask;
      }
      if (tiles) {
        rx_o = x0;
        ry_o = y0;
        rw_o = x1 - x0 + 1;
      }
      float4* sp = reinterpret_cast<float4*>(a.splats_v[v]) + i * 3;
      sp[0] = g0;
      sp[1] = make_float4(pr.Cc, o_eff, col[0], col[1]);
      col_b = col[2]; depth_o = depth; radius_o = radius;

      if (stage_out) {
        if (a.mean2d) { a.mean2d[i * 2] = px; a.mean2d[i * 2 + 1] = py; }
        if (a.depth) a.depth[i] = depth;
        if (a.radius) a.radius[i] = radius;
        if (a.cov2d) { a.cov2d[i * 3] = pr.a; a.cov2d[i * 3 + 1] = pr.b; a.cov2d[i * 3 + 2] = pr.c; }
        if (a.conic) { a.conic[i * 3] = pr.A; a.conic[i * 3 + 1] = pr.B; a.conic[i * 3 + 2] = pr.Cc; }
        if (a.colors) { a.colors[i * 3] = col[0]; a.colors[i * 3 + 1] = col[1]; a.colors[i * 3 + 2] = col[2]; }
        if (a.tiles_touched) a.tiles_touched[i] = tiles;
      }
    }

    const uint32_t emit = a.contributing ? nt : tiles;
    if (a.pair_total_v[v]) {  // the view's pair count (occluded binning counts only its first slices)
      const uint32_t ws = __reduce_add_sync(0xffffffffu, i < n ? emit : 0u);
      if ((threadIdx.x & 31) == 0 && ws) atomicAdd(a.pair_total_v[v], (unsigned long long)ws);
    }
    if (i < n) {
      reinterpret_cast<float4*>(a.splats_v[v])[i * 3 + 2] =
          make_float4(col_b, depth_o, radius_o, __uint_as_float(emit));
      if (a.bin_v[v]) {
        a.bin_v[v][2 * i] = make_uint4((uint32_t)rx_o, (uint32_t)ry_o, (uint32_t)rw_o, emit);
        a.bin_v[v][2 * i + 1] = make_uint4((uint32_t)mask_o, (uint32_t)(mask_o >> 32), __float_as_uint(depth_o), 0u);
      }
      if (a.depth_pairs_v[v]) {
        uint64_t word;
        if (a.view_key && a.depth_compact) {
          const uint64_t kb = emit ? __float_as_uint(depth_o) - a.depth_base : 0x0FFFFFFFu;
          word = ((uint64_t)v << 56) | (kb << 28) | (uint64_t)i;
        } else {
          const uint64_t kb = emit ? __float_as_uint(depth_o) : 0xFFFFFFFFu;
          word = a.view_key ? ((uint64_t)v << 60) | (kb << 28) | (uint64_t)i : (kb << 32) | (uint64_t)i;
        }
        a.depth_pairs_v[v][i] = word;
      }
    }
  }
}

int launch_preprocess(const PreprocessArgs& a, cudaStream_t stream) {
  if (a.n == 0) return GSC_OK;
  const int64_t blocks = (a.n + kPreThreads - 1) / kPreThreads;
  preprocess_kernel<<<(unsigned)blocks, kPreThreads, 0, stream>>>(a);
  GS_CK_LAUNCH("preprocess_kernel");
  return GSC_OK;
}

}  // namespace gs
