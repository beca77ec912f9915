// preprocess.cu — fused per-Gaussian forward: scale exp, quaternion, 3-D
// covariance, EWA projection with culling, conic, radius, tile count, SH
// colour and opacity sigmoid (src/metal/kernels/gaussian.metal:90-308,
// src/gaussian_splatting/gaussian.cr:119-142, rasterizer.cr:110-171).
//
// One thread per Gaussian, 128 per block. The 192-byte SH rows of a block are
// staged through shared memory with coalesced float4 loads, into rows padded
// to 13 float4 so that the per-thread float4 reads are free of bank conflicts.
//
// Packed splat record (12 floats, private to this library):
//   s0 = {mean.x, mean.y, conic.xx, conic.xy}
//   s1 = {conic.yy, opacity (0 if culled or det <= 0), r, g}
//   s2 = {b, depth, radius, bits(tiles_touched)}
#include "geometry.cuh"
#include "kernels.cuh"

namespace gs {

constexpr int kPreThreads = 128;
constexpr int kShRow = 13;  // float4 per staged SH row (12 used + 1 pad)

__global__ void __launch_bounds__(kPreThreads) preprocess_kernel(PreprocessArgs a) {
  __shared__ float4 s_sh[kPreThreads * kShRow];
  const int64_t base = (int64_t)blockIdx.x * kPreThreads;
  const int64_t i = base + threadIdx.x;
  const int64_t n = a.n;
  const gsc_camera& cam = a.cam;
  const gsc_raster_config& cfg = a.cfg;

  // Coalesced staging of this block's SH coefficients (48 floats each).
  {
    const int64_t cnt = min((int64_t)kPreThreads, n - base);
    const float4* src = reinterpret_cast<const float4*>(a.sh + base * 48);
    for (int k = threadIdx.x; k < cnt * 12; k += kPreThreads) s_sh[(k / 12) * kShRow + k % 12] = src[k];
  }
  __syncthreads();

  uint32_t tiles = 0;
  if (i < n) {
    const float p[3] = {a.pos[i * 3], a.pos[i * 3 + 1], a.pos[i * 3 + 2]};
    const float s[3] = {gs_expf(a.log_scale[i * 3]), gs_expf(a.log_scale[i * 3 + 1]),
                        gs_expf(a.log_scale[i * 3 + 2])};
    float4 q4 = reinterpret_cast<const float4*>(a.rot)[i];
    float q[4], qn;
    load_quat(q4, cfg.mode, q, &qn);
    float R[3][3];
    quat_to_R(q[0], q[1], q[2], q[3], R);
    float c3[6];
    cov3d_of(s, R, c3);
    Projected pr;
    project(p, c3, cam, cfg, &pr);

    // colour
    float d[3], len;
    view_dir(p, cam, d, &len);
    float b[16];
    sh_basis_hi(d[0], d[1], d[2], b);
    float shv[48];
#pragma unroll
    for (int q = 0; q < 12; q++) {
      const float4 v = s_sh[threadIdx.x * kShRow + q];
      shv[4 * q] = v.x; shv[4 * q + 1] = v.y; shv[4 * q + 2] = v.z; shv[4 * q + 3] = v.w;
    }
    float raw[3];
    sh_eval([&](int k) { return shv[k]; }, d[0], d[1], d[2], b, cfg.sh_degree, cfg.mode, raw);
    float col[3];
#pragma unroll
    for (int c = 0; c < 3; c++) col[c] = fmaxf(0.0f, raw[c] + 0.5f);
    const float o = gs_sigmoid(a.logit_opacity[i]);

    float px = -1000.0f, py = -1000.0f, depth = 0.0f, radius = 0.0f;
    if (pr.visible) {
      px = pr.px; py = pr.py; depth = pr.zc; radius = pr.r;
      if (pr.r > 0.0f && pr.zc > 0.0f) {
        int x0, x1, y0, y1;
        tile_bounds(px, py, pr.r, a.tiles_x, a.tiles_y, &x0, &x1, &y0, &y1);
        if (x1 >= x0 && y1 >= y0) tiles = (uint32_t)((x1 - x0 + 1) * (y1 - y0 + 1));
      }
    }
    const float o_eff = (pr.visible && pr.det > 0.0f) ? o : 0.0f;
    float4* sp = reinterpret_cast<float4*>(a.splats) + i * 3;
    sp[0] = make_float4(px, py, pr.A, pr.B);
    sp[1] = make_float4(pr.Cc, o_eff, col[0], col[1]);
    sp[2] = make_float4(col[2], depth, radius, __uint_as_float(tiles));

    if (a.mean2d) { a.mean2d[i * 2] = px; a.mean2d[i * 2 + 1] = py; }
    if (a.depth) a.depth[i] = depth;
    if (a.radius) a.radius[i] = radius;
    if (a.cov2d) { a.cov2d[i * 3] = pr.a; a.cov2d[i * 3 + 1] = pr.b; a.cov2d[i * 3 + 2] = pr.c; }
    if (a.conic) { a.conic[i * 3] = pr.A; a.conic[i * 3 + 1] = pr.B; a.conic[i * 3 + 2] = pr.Cc; }
    if (a.colors) { a.colors[i * 3] = col[0]; a.colors[i * 3 + 1] = col[1]; a.colors[i * 3 + 2] = col[2]; }
    if (a.opacity) a.opacity[i] = o;
    if (a.tiles_touched) a.tiles_touched[i] = tiles;
    if (a.depth_keys) {
      a.depth_keys[i] = tiles ? __float_as_uint(depth) : 0xFFFFFFFFu;
      a.order[i] = (uint32_t)i;
    }
    if (a.cov3d) {
#pragma unroll
      for (int k = 0; k < 6; k++) a.cov3d[i * 6 + k] = c3[k];
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
