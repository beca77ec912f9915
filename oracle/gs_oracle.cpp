// gs_oracle.cpp — CPU restatement of crystal-gausplat's rasterizer hot path.
//
// TEST INFRASTRUCTURE ONLY (the checker for libgsplat_cuda.so; never linked
// into the product). Parity unpinned by the reference's own tests (it has
// none for this path); pinned here by known-answer tests and float64 finite
// differences in tests/. Every function cites the reference lines it restates.
//
// Build: oracle/Makefile (-O2 -ffp-contract=off -fno-fast-math -fopenmp).
#include "gs_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

// Spherical-harmonics constants, gaussian.metal:11-28.
const float SH_C0 = 0.28209479177387814f;
const float SH_C1 = 0.4886025119029199f;
const float SH_C2[5] = {1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                        -1.0925484305920792f, 0.5462742152960396f};
const float SH_C3[7] = {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                        0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f,
                        -0.5900435899266435f};
const int TILE = 16;  // gaussian.metal:31

int g_threads = 1;
int g_exact_sums = 1;  // screen-space gradient sums in double (see gso_composite_backward)

inline float bits_to_float(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline uint32_t float_to_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}

// 2^j for j in [-126, 127], exact.
inline float pow2i(int j) { return bits_to_float((uint32_t)(j + 127) << 23); }

// float -> int with truncation toward zero (C `int(f)`, gaussian.metal:338-341),
// saturated to +-1e9 first so that out-of-range values are defined identically
// on every target.
inline int trunc_sat(float f) {
  f = std::fmax(f, -1.0e9f);
  f = std::fmin(f, 1.0e9f);
  return (int)f;
}

struct Proj {
  bool visible;
  float xc, yc, zc;     // camera-space position
  float px, py;         // mean2d
  float J00, J02, J11, J12;
  float C[6];           // cov_cam upper: 00 01 02 11 12 22
  float a, b, c;        // cov2d with low-pass (xx, xy, yy)
  float det;
  float r;              // radius
  float A, B, Cc;       // conic (0 if det <= 0)
};

// quat_to_matrix, gaussian.metal:64-82. q = (w, x, y, z).
inline void quat_to_R(float w, float x, float y, float z, float R[3][3]) {
  R[0][0] = 1.0f - 2.0f * (y * y + z * z);
  R[0][1] = 2.0f * (x * y - z * w);
  R[0][2] = 2.0f * (x * z + y * w);
  R[1][0] = 2.0f * (x * y + z * w);
  R[1][1] = 1.0f - 2.0f * (x * x + z * z);
  R[1][2] = 2.0f * (y * z - x * w);
  R[2][0] = 2.0f * (x * z - y * w);
  R[2][1] = 2.0f * (y * z + x * w);
  R[2][2] = 1.0f - 2.0f * (x * x + y * y);
}

// Quaternion as used by the given mode: REF uses it as stored (the host
// normalize_rotations! never reaches GPU tensors, gaussian.cr:274-296);
// FULL normalises (a zero quaternion becomes the identity).
inline void load_quat(const float* q, int mode, float out[4], float* norm) {
  float w = q[0], x = q[1], y = q[2], z = q[3];
  if (mode == GSC_MODE_FULL) {
    float n = std::sqrt(((w * w + x * x) + y * y) + z * z);
    *norm = n;
    if (n > 0.0f) {
      w = w / n; x = x / n; y = y / n; z = z / n;
    } else {
      w = 1.0f; x = 0.0f; y = 0.0f; z = 0.0f;
    }
  } else {
    *norm = 1.0f;
  }
  out[0] = w; out[1] = x; out[2] = y; out[3] = z;
}

// compute_cov3d, gaussian.metal:90-131: Sigma = R diag(s^2) R^T, upper triangle.
inline void cov3d_of(const float s[3], const float R[3][3], float cov[6]) {
  float s2[3] = {s[0] * s[0], s[1] * s[1], s[2] * s[2]};
  int k = 0;
  for (int i = 0; i < 3; i++)
    for (int j = i; j < 3; j++)
      cov[k++] = (R[i][0] * s2[0] * R[j][0] + R[i][1] * s2[1] * R[j][1]) + R[i][2] * s2[2] * R[j][2];
}

inline float sym3(const float c[6], int i, int j) {
  static const int idx[3][3] = {{0, 1, 2}, {1, 3, 4}, {2, 4, 5}};
  return c[idx[i][j]];
}

// project_gaussians, gaussian.metal:138-249, with the row-major view matrix
// the host intends (camera.cr:185-187) and the symmetric camera covariance.
inline void project(const float p[3], const float cov3[6], const gsc_camera* cam,
                    const gsc_raster_config* cfg, Proj* o) {
  const float* W = cam->view;
  o->xc = ((W[0] * p[0] + W[1] * p[1]) + W[2] * p[2]) + W[3];
  o->yc = ((W[4] * p[0] + W[5] * p[1]) + W[6] * p[2]) + W[7];
  o->zc = ((W[8] * p[0] + W[9] * p[1]) + W[10] * p[2]) + W[11];
  o->visible = false;
  o->r = 0.0f;
  o->A = o->B = o->Cc = 0.0f;
  o->a = o->b = o->c = 0.0f;
  if (o->zc <= cfg->near_z || o->zc > cfg->far_z) return;
  float xn = o->xc / o->zc, yn = o->yc / o->zc;
  if (std::fabs(xn) > cam->tan_fov_x * cfg->fov_cull || std::fabs(yn) > cam->tan_fov_y * cfg->fov_cull)
    return;
  o->visible = true;
  o->px = cam->fx * xn + cam->cx;
  o->py = cam->fy * yn + cam->cy;
  float z2 = o->zc * o->zc;
  o->J00 = cam->fx / o->zc;
  o->J02 = -cam->fx * o->xc / z2;
  o->J11 = cam->fy / o->zc;
  o->J12 = -cam->fy * o->yc / z2;
  // cov_cam = V Sigma V^T, V = rows 0..2 of the view rotation.
  float V[3][3] = {{W[0], W[1], W[2]}, {W[4], W[5], W[6]}, {W[8], W[9], W[10]}};
  float T[3][3];
  for (int i = 0; i < 3; i++)
    for (int k = 0; k < 3; k++)
      T[i][k] = (V[i][0] * sym3(cov3, 0, k) + V[i][1] * sym3(cov3, 1, k)) + V[i][2] * sym3(cov3, 2, k);
  int q = 0;
  for (int i = 0; i < 3; i++)
    for (int j = i; j < 3; j++) o->C[q++] = (T[i][0] * V[j][0] + T[i][1] * V[j][1]) + T[i][2] * V[j][2];
  const float C00 = o->C[0], C01 = o->C[1], C02 = o->C[2], C11 = o->C[3], C12 = o->C[4], C22 = o->C[5];
  const float J00 = o->J00, J02 = o->J02, J11 = o->J11, J12 = o->J12;
  float xx = J00 * J00 * C00 + 2.0f * J00 * J02 * C02 + J02 * J02 * C22;
  float xy = J00 * J11 * C01 + J00 * J12 * C02 + J02 * J11 * C12 + J02 * J12 * C22;
  float yy = J11 * J11 * C11 + 2.0f * J11 * J12 * C12 + J12 * J12 * C22;
  xx += cfg->lowpass;
  yy += cfg->lowpass;
  o->a = xx; o->b = xy; o->c = yy;
  float det = xx * yy - xy * xy;
  o->det = det;
  float trace = xx + yy;
  float lambda_max = 0.5f * (trace + std::sqrt(std::fmax(0.0f, trace * trace - 4.0f * det)));
  o->r = std::ceil(3.0f * std::sqrt(lambda_max));
  if (det > 0.0f) {
    // Inverse covariance exactly as rasterize_tile computes it (gaussian.metal:412-418).
    float inv_det = 1.0f / det;
    o->A = yy * inv_det;
    o->B = -xy * inv_det;
    o->Cc = xx * inv_det;
  }
}

struct ShBasis {
  float b[16];
};

// View direction (gaussian.metal:268-273): normalize(campos - pos).
inline void view_dir(const float p[3], const gsc_camera* cam, float v[3], float d[3], float* len) {
  v[0] = cam->campos[0] - p[0];
  v[1] = cam->campos[1] - p[1];
  v[2] = cam->campos[2] - p[2];
  float l = std::sqrt((v[0] * v[0] + v[1] * v[1]) + v[2] * v[2]);
  *len = l;
  d[0] = v[0] / l; d[1] = v[1] / l; d[2] = v[2] / l;
}

// Real SH basis with the reference constants and sign convention
// (gaussian.metal:279-300 for degrees 0-2; degree 3 completes it with SH_C3).
inline void sh_basis(float x, float y, float z, ShBasis* B) {
  float xx = x * x, yy = y * y, zz = z * z;
  float xy = x * y, yz = y * z, xz = x * z;
  B->b[0] = SH_C0;
  B->b[1] = -y; B->b[2] = z; B->b[3] = -x;  // times SH_C1 applied on the sum
  B->b[4] = SH_C2[0] * xy;
  B->b[5] = SH_C2[1] * yz;
  B->b[6] = SH_C2[2] * (2.0f * zz - xx - yy);
  B->b[7] = SH_C2[3] * xz;
  B->b[8] = SH_C2[4] * (xx - yy);
  B->b[9] = SH_C3[0] * y * (3.0f * xx - yy);
  B->b[10] = SH_C3[1] * xy * z;
  B->b[11] = SH_C3[2] * y * (4.0f * zz - xx - yy);
  B->b[12] = SH_C3[3] * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
  B->b[13] = SH_C3[4] * x * (4.0f * zz - xx - yy);
  B->b[14] = SH_C3[5] * z * (xx - yy);
  B->b[15] = SH_C3[6] * x * (xx - 3.0f * yy);
}

// eval_sh (gaussian.metal:256-308). raw[c] = value before "+0.5, max 0".
inline void sh_eval(const float* sh, const ShBasis& B, int degree, int mode, float raw[3]) {
  for (int c = 0; c < 3; c++) {
    float r = 0.0f;
    r += SH_C0 * sh[0 * 3 + c];
    if (degree >= 1)
      r += SH_C1 * (B.b[1] * sh[1 * 3 + c] + B.b[2] * sh[2 * 3 + c] - (-B.b[3]) * sh[3 * 3 + c]);
    if (degree >= 2 && (mode == GSC_MODE_FULL || c == 0)) {
      float t = B.b[4] * sh[4 * 3 + c] + B.b[5] * sh[5 * 3 + c] + B.b[6] * sh[6 * 3 + c] +
                B.b[7] * sh[7 * 3 + c] + B.b[8] * sh[8 * 3 + c];
      r += t;
    }
    if (degree >= 3 && mode == GSC_MODE_FULL) {
      float t = B.b[9] * sh[9 * 3 + c] + B.b[10] * sh[10 * 3 + c] + B.b[11] * sh[11 * 3 + c] +
                B.b[12] * sh[12 * 3 + c] + B.b[13] * sh[13 * 3 + c] + B.b[14] * sh[14 * 3 + c] +
                B.b[15] * sh[15 * 3 + c];
      r += t;
    }
    raw[c] = r;
  }
}

// Partial derivatives of the real SH basis (reference constants) with respect
// to the unit view direction; zero where basis k does not depend on a component.
inline void sh_basis_derivs(float x, float y, float z, float DX[16], float DY[16], float DZ[16]) {
  const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
  for (int k = 0; k < 16; k++) DX[k] = DY[k] = DZ[k] = 0.0f;
  DY[1] = -SH_C1;
  DZ[2] = SH_C1;
  DX[3] = -SH_C1;
  DX[4] = SH_C2[0] * y; DY[4] = SH_C2[0] * x;
  DY[5] = SH_C2[1] * z; DZ[5] = SH_C2[1] * y;
  DX[6] = SH_C2[2] * (-2.0f * x); DY[6] = SH_C2[2] * (-2.0f * y); DZ[6] = SH_C2[2] * (4.0f * z);
  DX[7] = SH_C2[3] * z; DZ[7] = SH_C2[3] * x;
  DX[8] = SH_C2[4] * (2.0f * x); DY[8] = SH_C2[4] * (-2.0f * y);
  DX[9] = SH_C3[0] * (6.0f * xy); DY[9] = SH_C3[0] * (3.0f * xx - 3.0f * yy);
  DX[10] = SH_C3[1] * yz; DY[10] = SH_C3[1] * xz; DZ[10] = SH_C3[1] * xy;
  DX[11] = SH_C3[2] * (-2.0f * xy); DY[11] = SH_C3[2] * (4.0f * zz - xx - 3.0f * yy); DZ[11] = SH_C3[2] * (8.0f * yz);
  DX[12] = SH_C3[3] * (-6.0f * xz); DY[12] = SH_C3[3] * (-6.0f * yz);
  DZ[12] = SH_C3[3] * (6.0f * zz - 3.0f * xx - 3.0f * yy);
  DX[13] = SH_C3[4] * (4.0f * zz - 3.0f * xx - yy); DY[13] = SH_C3[4] * (-2.0f * xy); DZ[13] = SH_C3[4] * (8.0f * xz);
  DX[14] = SH_C3[5] * (2.0f * xz); DY[14] = SH_C3[5] * (-2.0f * yz); DZ[14] = SH_C3[5] * (xx - yy);
  DX[15] = SH_C3[6] * (3.0f * xx - 3.0f * yy); DY[15] = SH_C3[6] * (-6.0f * xy);
}

// Gaussian3D#opacity, gaussian.cr:132-142.
inline float sigmoid(float x) { return 1.0f / (1.0f + gso_expf(-x)); }

inline void tile_bounds(float px, float py, float r, int tiles_x, int tiles_y, int* x0, int* x1,
                        int* y0, int* y1) {
  // gaussian.metal:338-341, with tiles_x/tiles_y = ceil(W/16), ceil(H/16).
  *x0 = std::max(0, trunc_sat(px - r) / TILE);
  *x1 = std::min(tiles_x - 1, trunc_sat(px + r) / TILE);
  *y0 = std::max(0, trunc_sat(py - r) / TILE);
  *y1 = std::min(tiles_y - 1, trunc_sat(py + r) / TILE);
}

}  // namespace

extern "C" {

// The reference's rasterizer constants (gaussian.metal:160,174,227-228,
// 400,425-426; trainer.cr:186), as gsc_raster_config_default fills them, so
// that a CPU-only caller (the benchmark's reference arm) needs nothing from
// the CUDA library.
void gso_raster_config_default(gsc_raster_config* cfg) {
  cfg->mode = GSC_MODE_FULL;
  cfg->sh_degree = 3;
  cfg->t_stop = 1e-3f;
  cfg->alpha_min = 1.0f / 255.0f;
  cfg->alpha_max = 0.99f;
  cfg->lowpass = 0.3f;
  cfg->fov_cull = 1.3f;
  cfg->near_z = 0.01f;
  cfg->far_z = 1000.0f;
  cfg->background[0] = cfg->background[1] = cfg->background[2] = 0.0f;
  cfg->binning = GSC_BIN_OCCLUDED;
}

float gso_expf(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return INFINITY;
  if (x < -103.97208404541015625f) return 0.0f;
  // Cody & Waite (1980) reduction: x = k ln2 + r, |r| <= ln2/2.
  float k = std::rint(x * 1.44269502162933349609375f);
  float r = std::fma(-k, 0.693145751953125f, x);
  r = std::fma(-k, 1.428606765330187045e-06f, r);
  // e^r by its Taylor series to degree 7 (truncation < 1e-8 relative).
  float p = 1.98412698412698412698e-4f;   // 1/7!
  p = std::fma(p, r, 1.38888888888888888889e-3f);  // 1/6!
  p = std::fma(p, r, 8.33333333333333333333e-3f);  // 1/5!
  p = std::fma(p, r, 4.16666666666666666667e-2f);  // 1/4!
  p = std::fma(p, r, 1.66666666666666666667e-1f);  // 1/3!
  p = std::fma(p, r, 0.5f);
  p = std::fma(p, r, 1.0f);
  p = std::fma(p, r, 1.0f);
  int ki = (int)k;
  if (ki > 127) return p * pow2i(127) * pow2i(ki - 127);
  if (ki < -126) return p * pow2i(ki + 64) * pow2i(-64);
  return p * pow2i(ki);
}

void gso_set_threads(int nthreads) { g_threads = nthreads < 1 ? 1 : nthreads; }
void gso_set_exact_sums(int on) { g_exact_sums = on ? 1 : 0; }

void gso_preprocess(const gsc_gaussians* g, const gsc_camera* cam, const gsc_raster_config* cfg,
                    float* mean2d, float* cov2d, float* conic, float* depth, float* radius,
                    float* colors, float* opacity, uint32_t* tiles_touched, float* cov3d) {
  const int64_t n = g->count;
  const int tiles_x = (cam->width + TILE - 1) / TILE, tiles_y = (cam->height + TILE - 1) / TILE;
#pragma omp parallel for num_threads(g_threads) schedule(static)
  for (int64_t i = 0; i < n; i++) {
    const float* p = g->position + i * 3;
    const float* ls = g->log_scale + i * 3;
    // Gaussian3D#scale (gaussian.cr:119-129), done per Gaussian.
    float s[3] = {gso_expf(ls[0]), gso_expf(ls[1]), gso_expf(ls[2])};
    float q[4], qn;
    load_quat(g->rotation + i * 4, cfg->mode, q, &qn);
    float R[3][3];
    quat_to_R(q[0], q[1], q[2], q[3], R);
    float c3[6];
    cov3d_of(s, R, c3);
    if (cov3d) std::memcpy(cov3d + i * 6, c3, sizeof c3);
    Proj pr;
    project(p, c3, cam, cfg, &pr);
    if (pr.visible) {
      if (mean2d) { mean2d[i * 2] = pr.px; mean2d[i * 2 + 1] = pr.py; }
      if (depth) depth[i] = pr.zc;
      if (radius) radius[i] = pr.r;
      if (cov2d) { cov2d[i * 3] = pr.a; cov2d[i * 3 + 1] = pr.b; cov2d[i * 3 + 2] = pr.c; }
      if (conic) { conic[i * 3] = pr.A; conic[i * 3 + 1] = pr.B; conic[i * 3 + 2] = pr.Cc; }
      if (tiles_touched) {
        uint32_t t = 0;
        if (pr.r > 0.0f && pr.zc > 0.0f) {
          int x0, x1, y0, y1;
          tile_bounds(pr.px, pr.py, pr.r, tiles_x, tiles_y, &x0, &x1, &y0, &y1);
          if (x1 >= x0 && y1 >= y0) t = (uint32_t)((x1 - x0 + 1) * (y1 - y0 + 1));
        }
        tiles_touched[i] = t;
      }
    } else {
      // Culled sentinels, gaussian.metal:161-166.
      if (mean2d) { mean2d[i * 2] = -1000.0f; mean2d[i * 2 + 1] = -1000.0f; }
      if (depth) depth[i] = 0.0f;
      if (radius) radius[i] = 0.0f;
      if (cov2d) { cov2d[i * 3] = 0.0f; cov2d[i * 3 + 1] = 0.0f; cov2d[i * 3 + 2] = 0.0f; }
      if (conic) { conic[i * 3] = 0.0f; conic[i * 3 + 1] = 0.0f; conic[i * 3 + 2] = 0.0f; }
      if (tiles_touched) tiles_touched[i] = 0;
    }
    if (colors) {
      float v[3], d[3], len;
      view_dir(p, cam, v, d, &len);
      ShBasis B;
      sh_basis(d[0], d[1], d[2], &B);
      float raw[3];
      sh_eval(g->sh + i * 48, B, cfg->sh_degree, cfg->mode, raw);
      for (int c = 0; c < 3; c++) colors[i * 3 + c] = std::fmax(0.0f, raw[c] + 0.5f);
    }
    if (opacity) opacity[i] = sigmoid(g->logit_opacity[i]);
  }
}

int64_t gso_emit_keys(int64_t n, const float* mean2d, const float* depth, const float* radius,
                      int32_t tiles_x, int32_t tiles_y, uint64_t* keys, uint32_t* vals,
                      int64_t capacity) {
  int64_t m = 0;
  for (int64_t i = 0; i < n; i++) {
    float px = mean2d[i * 2], py = mean2d[i * 2 + 1], r = radius[i], d = depth[i];
    if (r <= 0.0f || d <= 0.0f) continue;  // gaussian.metal:335
    int x0, x1, y0, y1;
    tile_bounds(px, py, r, tiles_x, tiles_y, &x0, &x1, &y0, &y1);
    uint64_t dbits = float_to_bits(d);
    for (int ty = y0; ty <= y1; ty++)
      for (int tx = x0; tx <= x1; tx++) {
        if (keys) {
          if (m >= capacity) return -1;
          uint64_t tile = (uint64_t)(uint32_t)(ty * tiles_x + tx);
          keys[m] = (tile << 32) | dbits;
          vals[m] = (uint32_t)i;
        }
        m++;
      }
  }
  return m;
}

void gso_sort_pairs(int64_t n, uint64_t* keys, uint32_t* vals, int begin_bit, int end_bit) {
  // A stable comparison sort by the key bits [begin_bit, end_bit): the
  // (masked key, original position) records are ordered lexicographically,
  // which is the stable order. Chunks are sorted on the OpenMP threads and
  // merged pairwise (std::merge keeps the left run first on ties, and the
  // positions make every record distinct anyway).
  const uint64_t mask = (end_bit - begin_bit >= 64) ? ~0ull : (((1ull << (end_bit - begin_bit)) - 1ull));
  struct Rec {
    uint64_t k;
    int64_t i;
    bool operator<(const Rec& o) const { return k < o.k || (k == o.k && i < o.i); }
  };
  std::vector<Rec> a(n), b(n);
#pragma omp parallel for num_threads(g_threads) schedule(static)
  for (int64_t i = 0; i < n; i++) a[i] = Rec{(keys[i] >> begin_bit) & mask, i};
  int parts = 1;
  while (parts < g_threads && parts < 64 && (int64_t)parts * 65536 < n) parts *= 2;
  std::vector<int64_t> cut(parts + 1);
  for (int p = 0; p <= parts; p++) cut[p] = n * p / parts;
#pragma omp parallel for num_threads(g_threads) schedule(static)
  for (int p = 0; p < parts; p++) std::sort(a.begin() + cut[p], a.begin() + cut[p + 1]);
  for (int w = 1; w < parts; w *= 2) {
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int p = 0; p < parts; p += 2 * w) {
      const int64_t lo = cut[p], mid = cut[std::min(p + w, parts)], hi = cut[std::min(p + 2 * w, parts)];
      std::merge(a.begin() + lo, a.begin() + mid, a.begin() + mid, a.begin() + hi, b.begin() + lo);
    }
    std::swap(a, b);
  }
  std::vector<uint64_t> k2(n);
  std::vector<uint32_t> v2(n);
#pragma omp parallel for num_threads(g_threads) schedule(static)
  for (int64_t i = 0; i < n; i++) { k2[i] = keys[a[i].i]; v2[i] = vals[a[i].i]; }
  std::memcpy(keys, k2.data(), n * 8);
  std::memcpy(vals, v2.data(), n * 4);
}

void gso_tile_ranges(int64_t n, const uint64_t* keys, int32_t num_tiles, uint32_t* ranges) {
  // init_tile_ranges + compute_tile_ranges, radix_sort.metal:288-324.
  std::memset(ranges, 0, sizeof(uint32_t) * 2 * (size_t)num_tiles);
  for (int64_t i = 0; i < n; i++) {
    uint32_t t = (uint32_t)(keys[i] >> 32);
    uint32_t prev = i > 0 ? (uint32_t)(keys[i - 1] >> 32) : 0xFFFFFFFFu;
    uint32_t next = i < n - 1 ? (uint32_t)(keys[i + 1] >> 32) : 0xFFFFFFFFu;
    if (t != prev && t < (uint32_t)num_tiles) ranges[t * 2] = (uint32_t)i;
    if (t != next && t < (uint32_t)num_tiles) ranges[t * 2 + 1] = (uint32_t)(i + 1);
  }
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Compositing
// ---------------------------------------------------------------------------
namespace {

struct PixelEval {
  bool ok;   // passes det / power / alpha tests
  float dx, dy, A, B, C, power, G, alpha;
};

// Per-pixel Gaussian evaluation of rasterize_tile (gaussian.metal:403-426),
// inverse covariance recomputed from cov2d per pixel as the reference does.
inline PixelEval eval_gauss(float pxf, float pyf, const float* mean2d, const float* cov2d,
                            const float* opacity, uint32_t gid, const gsc_raster_config* cfg) {
  PixelEval e;
  e.ok = false;
  float mx = mean2d[gid * 2], my = mean2d[gid * 2 + 1];
  e.dx = pxf - mx;
  e.dy = pyf - my;
  float cxx = cov2d[gid * 3], cxy = cov2d[gid * 3 + 1], cyy = cov2d[gid * 3 + 2];
  float det = cxx * cyy - cxy * cxy;
  if (det <= 0.0f) return e;
  float inv_det = 1.0f / det;
  e.A = cyy * inv_det;
  e.B = -cxy * inv_det;
  e.C = cxx * inv_det;
  // fma(dy dy, -C/2, fma(dx dy, -B, dx dx (-A/2))): the scalings are exact
  e.power = std::fma(e.dy * e.dy, -0.5f * e.C, std::fma(e.dx * e.dy, -e.B, e.dx * e.dx * (-0.5f * e.A)));
  if (e.power > 0.0f) return e;
  e.G = gso_expf(e.power);
  e.alpha = std::fmin(cfg->alpha_max, opacity[gid] * e.G);
  if (e.alpha < cfg->alpha_min) return e;
  e.ok = true;
  return e;
}

}  // namespace

extern "C" {

void gso_composite_forward(int32_t width, int32_t height, const uint32_t* ranges,
                           const uint32_t* vals, const float* mean2d, const float* cov2d,
                           const float* opacity, const float* colors,
                           const gsc_raster_config* cfg, float* image, uint32_t* n_contrib,
                           float* final_T, uint32_t* last) {
  const int tiles_x = (width + TILE - 1) / TILE, tiles_y = (height + TILE - 1) / TILE;
#pragma omp parallel for num_threads(g_threads) schedule(dynamic, 4)
  for (int t = 0; t < tiles_x * tiles_y; t++) {
    int tx = t % tiles_x, ty = t / tiles_x;
    uint32_t start = ranges[t * 2], end = ranges[t * 2 + 1];
    for (int ly = 0; ly < TILE; ly++)
      for (int lx = 0; lx < TILE; lx++) {
        int x = tx * TILE + lx, y = ty * TILE + ly;
        if (x >= width || y >= height) continue;
        float pxf = (float)x + 0.5f, pyf = (float)y + 0.5f;
        float C[3] = {0.0f, 0.0f, 0.0f};
        float T = 1.0f;
        uint32_t cnt = 0, lst = 0;
        for (uint32_t i = start; i < end && T > cfg->t_stop; i++) {
          uint32_t gid = vals[i];
          PixelEval e = eval_gauss(pxf, pyf, mean2d, cov2d, opacity, gid, cfg);
          if (!e.ok) continue;
          const float w = T * e.alpha;
          for (int c = 0; c < 3; c++) C[c] = std::fma(w, colors[gid * 3 + c], C[c]);
          T *= (1.0f - e.alpha);
          cnt++;
          lst = i - start + 1;
        }
        size_t pix = (size_t)y * width + x;
        for (int c = 0; c < 3; c++) image[pix * 3 + c] = std::fma(T, cfg->background[c], C[c]);
        if (n_contrib) n_contrib[pix] = cnt;
        if (final_T) final_T[pix] = T;
        if (last) last[pix] = lst;
      }
  }
}

// rasterize_tile (gaussian.metal:364-445) with the reference's own
// expression forms, for bounding the fused forms above against it: the
// inverse covariance recomputed per pixel, power = -0.5 (dx dx inv_xx +
// 2 dx dy inv_xy + dy dy inv_yy) summed left to right (gaussian.metal:421),
// colour += (T alpha) c and colour += T background without fused
// multiply-adds (gaussian.metal:430, 436). The exponential is this project's
// (the reference's fast-math Metal exp is not specified to the bit).
void gso_composite_forward_literal(int32_t width, int32_t height, const uint32_t* ranges,
                                   const uint32_t* vals, const float* mean2d, const float* cov2d,
                                   const float* opacity, const float* colors,
                                   const gsc_raster_config* cfg, float* image, uint32_t* n_contrib,
                                   float* final_T) {
  const int tiles_x = (width + TILE - 1) / TILE, tiles_y = (height + TILE - 1) / TILE;
#pragma omp parallel for num_threads(g_threads) schedule(dynamic, 4)
  for (int t = 0; t < tiles_x * tiles_y; t++) {
    const int tx = t % tiles_x, ty = t / tiles_x;
    const uint32_t start = ranges[t * 2], end = ranges[t * 2 + 1];
    for (int ly = 0; ly < TILE; ly++)
      for (int lx = 0; lx < TILE; lx++) {
        const int x = tx * TILE + lx, y = ty * TILE + ly;
        if (x >= width || y >= height) continue;
        const float px = (float)x + 0.5f, py = (float)y + 0.5f;
        float col[3] = {0.0f, 0.0f, 0.0f};
        float T = 1.0f;
        uint32_t cnt = 0;
        for (uint32_t i = start; i < end && T > cfg->t_stop; i++) {
          const uint32_t gid = vals[i];
          const float dx = px - mean2d[gid * 2], dy = py - mean2d[gid * 2 + 1];
          const float cxx = cov2d[gid * 3], cxy = cov2d[gid * 3 + 1], cyy = cov2d[gid * 3 + 2];
          const float det = cxx * cyy - cxy * cxy;
          if (det <= 0.0f) continue;
          const float inv_det = 1.0f / det;
          const float inv_xx = cyy * inv_det, inv_xy = -cxy * inv_det, inv_yy = cxx * inv_det;
          const float q = dx * dx * inv_xx + 2.0f * dx * dy * inv_xy + dy * dy * inv_yy;
          const float power = -0.5f * q;
          if (power > 0.0f) continue;
          const float alpha = std::fmin(cfg->alpha_max, opacity[gid] * gso_expf(power));
          if (alpha < cfg->alpha_min) continue;
          const float w = T * alpha;
          for (int c = 0; c < 3; c++) {
            const float term = w * colors[gid * 3 + c];
            col[c] = col[c] + term;
          }
          T *= (1.0f - alpha);
          cnt++;
        }
        const size_t pix = (size_t)y * width + x;
        for (int c = 0; c < 3; c++) {
          const float bg = T * cfg->background[c];
          image[pix * 3 + c] = col[c] + bg;
        }
        if (n_contrib) n_contrib[pix] = cnt;
        if (final_T) final_T[pix] = T;
      }
  }
}

void gso_composite_backward(int32_t width, int32_t height, const uint32_t* ranges,
                            const uint32_t* vals, const float* mean2d, const float* cov2d,
                            const float* opacity, const float* colors,
                            const gsc_raster_config* cfg, const float* dL_dimage,
                            const float* image, const float* target, float l1_scale,
                            const float* final_T, const uint32_t* last, float* grad2d,
                            double* loss_sum) {
  const int tiles_x = (width + TILE - 1) / TILE, tiles_y = (height + TILE - 1) / TILE;
  const bool full = cfg->mode == GSC_MODE_FULL;
  // The per-pixel terms are fp32 (the reference's per-thread arithmetic).
  // By default (gso_set_exact_sums(1)) their sum per Gaussian and field is
  // accumulated in double and rounded once: the exact sum of those terms,
  // independent of the order in which threads add. With 0 they are added in
  // fp32 as they come, like the reference's fp32 atomics in an unspecified
  // order (gaussian.metal:503-566); that spread of fp32 summation orders is
  // what the parity tests compare the kernels' own spread with.
  int64_t n_gauss = 0;
  for (int t = 0; g_exact_sums && t < tiles_x * tiles_y; t++)
    for (uint32_t i = ranges[t * 2]; i < ranges[t * 2 + 1]; i++) n_gauss = std::max<int64_t>(n_gauss, vals[i] + 1);
  std::vector<double> acc2d((size_t)n_gauss * 9, 0.0);
  double loss = 0.0;
#pragma omp parallel for num_threads(g_threads) schedule(dynamic, 4) reduction(+ : loss)
  for (int t = 0; t < tiles_x * tiles_y; t++) {
    int tx = t % tiles_x, ty = t / tiles_x;
    uint32_t start = ranges[t * 2], end = ranges[t * 2 + 1];
    for (int ly = 0; ly < TILE; ly++)
      for (int lx = 0; lx < TILE; lx++) {
        int x = tx * TILE + lx, y = ty * TILE + ly;
        if (x >= width || y >= height) continue;
        size_t pix = (size_t)y * width + x;
        float pxf = (float)x + 0.5f, pyf = (float)y + 0.5f;
        float g[3];
        for (int c = 0; c < 3; c++) {
          if (target) {
            // Loss.l1_with_grad, loss.cr:47-52, fused.
            float diff = image[pix * 3 + c] - target[pix * 3 + c];
            float sg = diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f);
            g[c] = sg * l1_scale;
            loss += (double)(std::fabs(diff) * l1_scale);
          } else {
            g[c] = dL_dimage[pix * 3 + c];
          }
        }
        float T = final_T[pix];
        float acc[3];
        for (int c = 0; c < 3; c++) acc[c] = cfg->background[c] * T;
        // FULL: from the last contributor the forward evaluated; REF: whole
        // list (gaussian.metal:503).
        int64_t hi = full ? (int64_t)start + (int64_t)last[pix] : (int64_t)end;
        for (int64_t i = hi - 1; i >= (int64_t)start; i--) {
          uint32_t gid = vals[i];
          PixelEval e = eval_gauss(pxf, pyf, mean2d, cov2d, opacity, gid, cfg);
          if (!e.ok) continue;
          const float* c = colors + gid * 3;
          float o = opacity[gid];
          float T_before = T / (1.0f - e.alpha);
          float dc[3];
          for (int k = 0; k < 3; k++) dc[k] = T_before * e.alpha * g[k];
          float dL_dalpha = 0.0f;
          for (int k = 0; k < 3; k++) dL_dalpha += (T_before * (c[k] - acc[k] / T)) * g[k];
          float dL_dG, dL_do;
          if (full && !(o * e.G <= cfg->alpha_max)) {
            dL_dG = 0.0f;  // alpha clamped at alpha_max: no gradient through o*G
            dL_do = 0.0f;
          } else {
            dL_dG = dL_dalpha * o;
            dL_do = dL_dalpha * e.G;
          }
          float dL_dpower = dL_dG * e.G;
          float dmx = dL_dpower * (e.A * e.dx + e.B * e.dy);
          float dmy = dL_dpower * (e.B * e.dx + e.C * e.dy);
          float vals9[9] = {dmx, dmy, 0.0f, 0.0f, 0.0f, dL_do, dc[0], dc[1], dc[2]};
          if (full) {
            vals9[2] = dL_dpower * (-0.5f * e.dx * e.dx);
            vals9[3] = dL_dpower * (-e.dx * e.dy);
            vals9[4] = dL_dpower * (-0.5f * e.dy * e.dy);
          }
          if (g_exact_sums) {
            double* gd = acc2d.data() + (size_t)gid * 9;
            for (int k = 0; k < 9; k++) {
#pragma omp atomic
              gd[k] += (double)vals9[k];
            }
          } else {
            float* gf = grad2d + (size_t)gid * 9;
            for (int k = 0; k < 9; k++) {
#pragma omp atomic
              gf[k] += vals9[k];
            }
          }
          T = T_before;
          for (int k = 0; k < 3; k++) {
            float contrib = T_before * e.alpha * c[k];
            acc[k] = full ? acc[k] + contrib : acc[k] - contrib;  // REF keeps gaussian.metal:566
          }
        }
      }
  }
  for (size_t i = 0; i < acc2d.size(); i++) grad2d[i] += (float)acc2d[i];
  if (loss_sum) *loss_sum += loss;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Preprocess backward, loss, optimiser, whole view
// ---------------------------------------------------------------------------
extern "C" {

void gso_preprocess_backward(const gsc_gaussians* g, const gsc_camera* cam,
                             const gsc_raster_config* cfg, const float* grad2d,
                             const gsc_gaussian_grads* grads, float* d_mean2d, float* d_cov2d,
                             float* d_opacity, float* d_colors) {
  const int64_t n = g->count;
  const bool full = cfg->mode == GSC_MODE_FULL;
  const float* W = cam->view;
  const float fx = cam->fx, fy = cam->fy;
#pragma omp parallel for num_threads(g_threads) schedule(static)
  for (int64_t i = 0; i < n; i++) {
    const float* gd = grad2d + i * 9;
    const float dmx = gd[0], dmy = gd[1], dA = gd[2], dB = gd[3], dC = gd[4], dop = gd[5];
    const float dcol[3] = {gd[6], gd[7], gd[8]};
    if (d_mean2d) { d_mean2d[i * 2] = dmx; d_mean2d[i * 2 + 1] = dmy; }
    if (d_opacity) d_opacity[i] = dop;
    if (d_colors) for (int c = 0; c < 3; c++) d_colors[i * 3 + c] = dcol[c];
    if (d_cov2d) for (int c = 0; c < 3; c++) d_cov2d[i * 3 + c] = 0.0f;
    const float* p = g->position + i * 3;
    // Opacity sigmoid chain, trainer.cr:234-241.
    float o = sigmoid(g->logit_opacity[i]);
    grads->logit_opacity[i] += dop * o * (1.0f - o);
    if (!full) {
      // project_backward!, rasterizer.cr:395-427 (position through the mean only).
      float xc = W[0] * p[0] + W[1] * p[1] + W[2] * p[2] + W[3];
      float yc = W[4] * p[0] + W[5] * p[1] + W[6] * p[2] + W[7];
      float zc = W[8] * p[0] + W[9] * p[1] + W[10] * p[2] + W[11];
      if (!(zc <= cfg->near_z)) {
        float z2 = zc * zc;
        float dL_dcx = dmx * fx / zc;
        float dL_dcy = dmy * fy / zc;
        float dL_dcz = dmx * (-fx * xc / z2) + dmy * (-fy * yc / z2);
        for (int j = 0; j < 3; j++)
          grads->position[i * 3 + j] += dL_dcx * W[j] + dL_dcy * W[4 + j] + dL_dcz * W[8 + j];
      }
      // sh_backward!, rasterizer.cr:442-448 (DC only, divided by C0).
      for (int c = 0; c < 3; c++) grads->sh[i * 48 + c] += dcol[c] / SH_C0;
      continue;
    }
    bool any = false;
    for (int k = 0; k < 9; k++) any = any || gd[k] != 0.0f;
    if (!any) continue;
    // ---- recompute the forward ----
    const float* ls = g->log_scale + i * 3;
    float s[3] = {gso_expf(ls[0]), gso_expf(ls[1]), gso_expf(ls[2])};
    const float* qr = g->rotation + i * 4;
    float q[4], qnorm;
    load_quat(qr, cfg->mode, q, &qnorm);
    float R[3][3];
    quat_to_R(q[0], q[1], q[2], q[3], R);
    float c3[6];
    cov3d_of(s, R, c3);
    Proj pr;
    project(p, c3, cam, cfg, &pr);
    if (!pr.visible) continue;
    float dp[3] = {0.0f, 0.0f, 0.0f};
    // ---- colour -> SH coefficients and view direction ----
    {
      float v[3], d[3], len;
      view_dir(p, cam, v, d, &len);
      ShBasis B;
      sh_basis(d[0], d[1], d[2], &B);
      float raw[3];
      sh_eval(g->sh + i * 48, B, cfg->sh_degree, cfg->mode, raw);
      const float x = d[0], y = d[1], z = d[2];
      const int deg = cfg->sh_degree;
      const int ncoef = (deg + 1) * (deg + 1);
      float basis[16];
      basis[0] = SH_C0;
      basis[1] = SH_C1 * -y; basis[2] = SH_C1 * z; basis[3] = SH_C1 * -x;
      for (int k = 4; k < 16; k++) basis[k] = B.b[k];
      const float* sh = g->sh + i * 48;
      float w[3];
      for (int c = 0; c < 3; c++) {
        w[c] = raw[c] + 0.5f > 0.0f ? dcol[c] : 0.0f;  // max(0, .) mask
        if (w[c] == 0.0f) continue;
        for (int k = 0; k < ncoef; k++) grads->sh[i * 48 + k * 3 + c] += basis[k] * w[c];
      }
      // Direction gradient, one coefficient at a time: t_k = sum_c w_c S(k,c)
      // times the partial derivatives of basis k.
      float DX[16], DY[16], DZ[16];
      sh_basis_derivs(x, y, z, DX, DY, DZ);
      float gx = 0.0f, gy = 0.0f, gz = 0.0f;
      for (int k = 1; k < ncoef; k++) {
        const float t = w[0] * sh[k * 3] + w[1] * sh[k * 3 + 1] + w[2] * sh[k * 3 + 2];
        gx += t * DX[k];
        gy += t * DY[k];
        gz += t * DZ[k];
      }
      // d = v/|v|, v = campos - p
      float dd = x * gx + y * gy + z * gz;
      dp[0] -= (gx - x * dd) / len;
      dp[1] -= (gy - y * dd) / len;
      dp[2] -= (gz - z * dd) / len;
    }
    // ---- conic -> cov2d ----
    float da = 0.0f, db = 0.0f, dc2 = 0.0f;
    if (pr.det > 0.0f) {
      const float A = pr.A, B = pr.B, C = pr.Cc;
      float P00 = A * A * dA + A * B * dB + B * B * dC;
      float P01 = A * B * dA + (A * C + B * B) * (0.5f * dB) + B * C * dC;
      float P11 = B * B * dA + B * C * dB + C * C * dC;
      da = -P00;
      db = -2.0f * P01;
      dc2 = -P11;
    }
    if (d_cov2d) { d_cov2d[i * 3] = da; d_cov2d[i * 3 + 1] = db; d_cov2d[i * 3 + 2] = dc2; }
    // ---- cov2d = J C J^T -> cov_cam C and Jacobian J ----
    float Jm[2][3] = {{pr.J00, 0.0f, pr.J02}, {0.0f, pr.J11, pr.J12}};
    float Gc[2][2] = {{da, 0.5f * db}, {0.5f * db, dc2}};
    float Cm[3][3];
    for (int a = 0; a < 3; a++)
      for (int b2 = 0; b2 < 3; b2++) Cm[a][b2] = sym3(pr.C, a, b2);
    float GJ[2][3];  // Gc J
    for (int a = 0; a < 2; a++)
      for (int k = 0; k < 3; k++) GJ[a][k] = Gc[a][0] * Jm[0][k] + Gc[a][1] * Jm[1][k];
    float dCm[3][3];  // J^T Gc J
    for (int k = 0; k < 3; k++)
      for (int l = 0; l < 3; l++) dCm[k][l] = Jm[0][k] * GJ[0][l] + Jm[1][k] * GJ[1][l];
    float dJ[2][3];  // 2 Gc J C
    for (int a = 0; a < 2; a++)
      for (int k = 0; k < 3; k++)
        dJ[a][k] = 2.0f * (GJ[a][0] * Cm[0][k] + GJ[a][1] * Cm[1][k] + GJ[a][2] * Cm[2][k]);
    const float xc = pr.xc, yc = pr.yc, zc = pr.zc;
    const float z2 = zc * zc, z3 = z2 * zc;
    float dxc = dJ[0][2] * (-fx / z2);
    float dyc = dJ[1][2] * (-fy / z2);
    float dzc = dJ[0][0] * (-fx / z2) + dJ[0][2] * (2.0f * fx * xc / z3) + dJ[1][1] * (-fy / z2) +
                dJ[1][2] * (2.0f * fy * yc / z3);
    // ---- mean2d -> camera-space position ----
    dxc += dmx * fx / zc;
    dyc += dmy * fy / zc;
    dzc += -(dmx * fx * xc + dmy * fy * yc) / z2;
    const float V[3][3] = {{W[0], W[1], W[2]}, {W[4], W[5], W[6]}, {W[8], W[9], W[10]}};
    for (int j = 0; j < 3; j++) dp[j] += V[0][j] * dxc + V[1][j] * dyc + V[2][j] * dzc;
    for (int j = 0; j < 3; j++) grads->position[i * 3 + j] += dp[j];
    // ---- C = V Sigma V^T -> Sigma ----
    float VtD[3][3];
    for (int a = 0; a < 3; a++)
      for (int l = 0; l < 3; l++) VtD[a][l] = V[0][a] * dCm[0][l] + V[1][a] * dCm[1][l] + V[2][a] * dCm[2][l];
    float dS[3][3];
    for (int a = 0; a < 3; a++)
      for (int b2 = 0; b2 < 3; b2++) dS[a][b2] = VtD[a][0] * V[0][b2] + VtD[a][1] * V[1][b2] + VtD[a][2] * V[2][b2];
    // ---- Sigma = M M^T, M = R diag(s) ----
    float M[3][3];
    for (int a = 0; a < 3; a++)
      for (int j = 0; j < 3; j++) M[a][j] = R[a][j] * s[j];
    float dM[3][3];
    for (int a = 0; a < 3; a++)
      for (int j = 0; j < 3; j++) dM[a][j] = 2.0f * (dS[a][0] * M[0][j] + dS[a][1] * M[1][j] + dS[a][2] * M[2][j]);
    float dR[3][3];
    for (int j = 0; j < 3; j++) {
      float ds = dM[0][j] * R[0][j] + dM[1][j] * R[1][j] + dM[2][j] * R[2][j];
      grads->log_scale[i * 3 + j] += ds * s[j];
      for (int a = 0; a < 3; a++) dR[a][j] = dM[a][j] * s[j];
    }
    // ---- R(q) -> q ----
    const float w = q[0], x = q[1], y = q[2], z = q[3];
    float dqw = 2.0f * (-z * dR[0][1] + y * dR[0][2] + z * dR[1][0] - x * dR[1][2] - y * dR[2][0] + x * dR[2][1]);
    float dqx = 2.0f * (y * dR[0][1] + z * dR[0][2] + y * dR[1][0] - 2.0f * x * dR[1][1] - w * dR[1][2] +
                        z * dR[2][0] + w * dR[2][1] - 2.0f * x * dR[2][2]);
    float dqy = 2.0f * (-2.0f * y * dR[0][0] + x * dR[0][1] + w * dR[0][2] + x * dR[1][0] + z * dR[1][2] -
                        w * dR[2][0] + z * dR[2][1] - 2.0f * y * dR[2][2]);
    float dqz = 2.0f * (-2.0f * z * dR[0][0] - w * dR[0][1] + x * dR[0][2] + w * dR[1][0] - 2.0f * z * dR[1][1] +
                        y * dR[1][2] + x * dR[2][0] + y * dR[2][1]);
    // through q/|q|
    float dot = w * dqw + x * dqx + y * dqy + z * dqz;
    if (qnorm > 0.0f) {
      grads->rotation[i * 4 + 0] += (dqw - w * dot) / qnorm;
      grads->rotation[i * 4 + 1] += (dqx - x * dot) / qnorm;
      grads->rotation[i * 4 + 2] += (dqy - y * dot) / qnorm;
      grads->rotation[i * 4 + 3] += (dqz - z * dot) / qnorm;
    }
  }
}

void gso_l1_loss_grad(int64_t numel, const float* pred, const float* target, float scale,
                      float* grad, double* loss_sum) {
  // Loss.l1_with_grad, src/ops/loss.cr:33-57.
  double loss = 0.0;
  for (int64_t i = 0; i < numel; i++) {
    float diff = pred[i] - target[i];
    loss += (double)(std::fabs(diff) * scale);
    grad[i] = (diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f)) * scale;
  }
  if (loss_sum) *loss_sum += loss;
}

// ---- contributing-pairs binning ----------------------------------------------

// ln x for positive finite float x by frexp and the atanh series through
// s^13, in a fixed order of +, *, / (identical bits on every IEEE float
// implementation).
static float log_series(float x) {
  int e;
  float m = std::frexp(x, &e);
  if (m < 0.70710678f) {
    m *= 2.0f;
    e -= 1;
  }
  const float s = (m - 1.0f) / (m + 1.0f), s2 = s * s;
  float p = 1.0f / 13.0f;
  const float inv[] = {1.0f / 11.0f, 1.0f / 9.0f, 1.0f / 7.0f, 1.0f / 5.0f, 1.0f / 3.0f, 1.0f};
  for (float c : inv) p = p * s2 + c;
  return (float)e * 0.69314718f + 2.0f * s * p;
}

// Row form used by contributing-pairs binning: the ellipse q <= thr cut by the
// tile's row strip projects to one x interval [xl, xr] (from the leftmost and
// rightmost points of the ellipse clamped into the strip), widened by
// 1e-2 px + 2e-3 of the half-width (and the strip's reach likewise); the tile
// survives iff its pixel-centre span meets it.
static bool row_culled(float mx, float my, float A, float B, float C, float o, float rx0, float rx1,
                       float ry0, float ry1, float alpha_min) {
  if (!std::isfinite(mx) || !std::isfinite(my)) return false;
  if (!(o > 0.0f)) return o == 0.0f && std::isfinite(A) && std::isfinite(B) && std::isfinite(C);
  if (!(A > 0.0f && C > 0.0f) || !std::isfinite(A) || !std::isfinite(B) || !std::isfinite(C)) return false;
  const float rho = std::fabs(B) / std::sqrt(A * C);
  if (!(1.0f - rho >= 1e-3f)) return false;
  const float cut = log_series(alpha_min / o) - 1e-4f;
  if (cut >= 0.0f) return true;
  const float thr = -2.0f * cut * (1.0f + 2e-3f) + 2e-3f;
  const float det = A * C - B * B;
  if (!(det > 0.0f)) return false;
  const float xe = std::sqrt(thr * C / det), ye0 = std::sqrt(thr * A / det);
  const float dyl = B * std::sqrt(thr / (C * det));
  const float pad = 1e-2f + 2e-3f * xe;
  const float ye = ye0 + 1e-2f + 2e-3f * ye0;
  const float y0 = ry0 - my, y1 = ry1 - my;
  if (y0 > ye || y1 < -ye) return true;
  const float a = std::fmax(y0, -ye), b = std::fmin(y1, ye);
  const float dl = std::fmin(std::fmax(dyl, a), b), dr = std::fmin(std::fmax(-dyl, a), b);
  const float Dl = std::fmax(0.0f, A * thr - det * dl * dl);
  const float Dr = std::fmax(0.0f, A * thr - det * dr * dr);
  const float xl = (-B * dl - std::sqrt(Dl)) / A - pad;
  const float xr = (-B * dr + std::sqrt(Dr)) / A + pad;
  return !(rx1 - mx >= xl && rx0 - mx <= xr);
}

int64_t gso_contributing_lists(int32_t W, int32_t H, int64_t m, const uint64_t* keys,
                               const uint32_t* vals, const float* mean2d, const float* conic,
                               const float* opacity, const uint32_t* tiles_touched,
                               float alpha_min, uint64_t* out_keys, uint32_t* out_vals) {
  const int tiles_x = (W + 15) / 16;
  // keep flags on the OpenMP threads, then an ordered compaction
  std::vector<uint8_t> keep_flag(m);
#pragma omp parallel for num_threads(g_threads) schedule(dynamic, 65536)
  for (int64_t i = 0; i < m; i++) {
    const uint32_t id = vals[i];
    const uint32_t tile = (uint32_t)(keys[i] >> 32);
    bool keep = tiles_touched[id] > 64;
    if (!keep) {
      const int tx = (int)(tile % (uint32_t)tiles_x), ty = (int)(tile / (uint32_t)tiles_x);
      const float rx0 = tx * 16 + 0.5f, ry0 = ty * 16 + 0.5f;
      const float rx1 = std::min(tx * 16 + 16, W) - 0.5f, ry1 = std::min(ty * 16 + 16, H) - 0.5f;
      keep = !row_culled(mean2d[2 * id], mean2d[2 * id + 1], conic[3 * id], conic[3 * id + 1],
                         conic[3 * id + 2], opacity[id], rx0, rx1, ry0, ry1, alpha_min);
    }
    keep_flag[i] = keep;
  }
  int64_t k = 0;
  for (int64_t i = 0; i < m; i++) {
    if (keep_flag[i]) {
      out_keys[k] = keys[i];
      out_vals[k] = vals[i];
      k++;
    }
  }
  return k;
}

// ---- losses beyond L1 -------------------------------------------------------

// Gaussian window of Loss#gaussian_window (loss.cr:262-281), sigma 1.5: fp32
// exp, fp32 row-major sum, each value divided by it. 1D (two_d false) for the
// separable form.
static std::vector<float> ssim_window(int win, bool two_d) {
  const int c = win / 2, n = two_d ? win * win : win;
  std::vector<float> w(n);
  for (int i = 0; i < n; i++) {
    const int dx = (two_d ? i % win : i) - c, dy = two_d ? i / win - c : 0;
    w[i] = gso_expf((float)(-(dx * dx + dy * dy)) / (2.0f * 1.5f * 1.5f));
  }
  float sum = 0.0f;
  for (int i = 0; i < n; i++) sum += w[i];
  for (int i = 0; i < n; i++) w[i] = w[i] / sum;
  return w;
}

void gso_loss_grad(const float* pred, const float* target, int32_t H, int32_t W, int32_t C,
                   int32_t win, int32_t mode, float w_l1, float w_ssim, float* grad,
                   float* ssim_map, float* out) {
  // Loss.ssim (loss.cr:117-186) per valid pixel and channel; REF literally
  // (2D window, means then variances), FULL separably with moments
  // blur(x), blur(y), blur(x^2), blur(y^2), blur(xy) and the analytic gradient
  // dSum S/dx_q = blur(A) + 2 x_q blur(B) + y_q blur(C).
  const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
  const int pad = win / 2, vw = W - 2 * pad, vh = H - 2 * pad;
  const bool any = vw > 0 && vh > 0, full = mode == GSC_MODE_FULL;
  const int64_t numel = (int64_t)H * W * C, plane = (int64_t)H * W;
  const float n_f = (float)numel, count_f = any ? (float)((int64_t)vw * vh * C) : 0.0f;
  auto at = [&](const float* img, int y, int x, int c) { return img[((int64_t)y * W + x) * C + c]; };
  const std::vector<float> w2 = ssim_window(win, true), g = ssim_window(win, false);
  const bool need_abc = full && grad && w_ssim != 0.0f && any;
  std::vector<float> abc(need_abc ? 3 * numel : 0, 0.0f);
  double ssum = 0.0;
  for (int c = 0; c < C && any; c++)
    for (int y = pad; y < H - pad; y++)
      for (int x = pad; x < W - pad; x++) {
        float S;
        if (!full) {
          float mu_x = 0.0f, mu_y = 0.0f, sx = 0.0f, sy = 0.0f, sxy = 0.0f;
          for (int wy = 0; wy < win; wy++)
            for (int wx = 0; wx < win; wx++) {
              const float w = w2[wy * win + wx];
              mu_x += w * at(pred, y - pad + wy, x - pad + wx, c);
              mu_y += w * at(target, y - pad + wy, x - pad + wx, c);
            }
          for (int wy = 0; wy < win; wy++)
            for (int wx = 0; wx < win; wx++) {
              const float w = w2[wy * win + wx];
              const float px = at(pred, y - pad + wy, x - pad + wx, c);
              const float py = at(target, y - pad + wy, x - pad + wx, c);
              sx += w * (px - mu_x) * (px - mu_x);
              sy += w * (py - mu_y) * (py - mu_y);
              sxy += w * (px - mu_x) * (py - mu_y);
            }
          const float num = (2.0f * mu_x * mu_y + C1) * (2.0f * sxy + C2);
          const float den = (mu_x * mu_x + mu_y * mu_y + C1) * (sx + sy + C2);
          S = num / den;
        } else {
          float m[5] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
          for (int k = 0; k < win; k++) {
            float h[5] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
            for (int j = 0; j < win; j++) {
              const float p = at(pred, y - pad + k, x - pad + j, c);
              const float t = at(target, y - pad + k, x - pad + j, c);
              h[0] += g[j] * p;
              h[1] += g[j] * t;
              h[2] += g[j] * (p * p);
              h[3] += g[j] * (t * t);
              h[4] += g[j] * (p * t);
            }
            for (int q = 0; q < 5; q++) m[q] += g[k] * h[q];
          }
          const float mu_x = m[0], mu_y = m[1];
          const float sxx = m[2] - mu_x * mu_x, syy = m[3] - mu_y * mu_y, sxy = m[4] - mu_x * mu_y;
          const float n1 = 2.0f * mu_x * mu_y + C1, n2 = 2.0f * sxy + C2;
          const float d1 = mu_x * mu_x + mu_y * mu_y + C1, d2 = sxx + syy + C2;
          const float dd = d1 * d2;
          S = (n1 * n2) / dd;
          if (need_abc) {
            const float dmu = 2.0f * mu_y * n2 / dd - 2.0f * mu_x * S / d1;
            const float dsxx = -S / d2;
            const float dsxy = 2.0f * n1 / dd;
            const int64_t o = (int64_t)y * W + x;
            abc[(0 * C + c) * plane + o] = dmu - 2.0f * mu_x * dsxx - mu_y * dsxy;
            abc[(1 * C + c) * plane + o] = dsxx;
            abc[(2 * C + c) * plane + o] = dsxy;
          }
        }
        ssum += (double)S;
        if (ssim_map) ssim_map[((int64_t)y * W + x) * C + c] = S;
      }
  // Gradient (loss.cr:33-57, 194-216, 227-249) and the L1 sum.
  auto abc_at = [&](int j, int c, int y, int x) -> float {
    if (y < pad || y >= H - pad || x < pad || x >= W - pad) return 0.0f;
    return abc[(j * C + c) * plane + (int64_t)y * W + x];
  };
  double l1 = 0.0;
  for (int y = 0; y < H; y++)
    for (int x = 0; x < W; x++)
      for (int c = 0; c < C; c++) {
        const int64_t e = ((int64_t)y * W + x) * C + c;
        const float p = pred[e], t = target[e], diff = p - t;
        l1 += (double)std::fabs(diff);
        if (!grad) continue;
        float sd;
        if (need_abc) {
          float b[3] = {0.0f, 0.0f, 0.0f};
          for (int k = 0; k < win; k++) {
            float h[3] = {0.0f, 0.0f, 0.0f};
            for (int j = 0; j < win; j++)
              for (int q = 0; q < 3; q++) h[q] += g[j] * abc_at(q, c, y - pad + k, x - pad + j);
            for (int q = 0; q < 3; q++) b[q] += g[k] * h[q];
          }
          const float dS = b[0] + 2.0f * p * b[1] + t * b[2];
          sd = -(dS / count_f);
        } else if (full) {
          sd = 0.0f;  // no valid pixel (or no SSIM term): SSIM is the constant 0
        } else {
          sd = 2.0f * diff / n_f;
        }
        const float l1d = (diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f)) / n_f;
        grad[e] = w_l1 * l1d + w_ssim * sd;
      }
  const float ssim = count_f > 0.0f ? (float)(ssum / (double)count_f) : 0.0f;
  const float l1v = n_f > 0.0f ? (float)(l1 / (double)n_f) : 0.0f;
  out[0] = w_l1 * l1v + w_ssim * (1.0f - ssim);
  out[1] = l1v;
  out[2] = ssim;
}

void gso_mse_loss_grad(const float* pred, const float* target, int64_t numel, float* grad,
                       float* out) {
  // Loss.mse_with_grad, loss.cr:83-105 (sum in double).
  double s = 0.0;
  for (int64_t i = 0; i < numel; i++) {
    const float diff = pred[i] - target[i];
    s += (double)(diff * diff);
    if (grad) grad[i] = 2.0f * diff / (float)numel;
  }
  const float v = numel > 0 ? (float)(s / (double)numel) : 0.0f;
  out[0] = v;
  out[1] = v;
  out[2] = 0.0f;
}

// ---- 8-bit images -> targets ------------------------------------------------

void gso_image_to_target(const uint8_t* src, int32_t sw, int32_t sh, int32_t sc, float* dst,
                         int32_t dw, int32_t dh, int32_t dc) {
  // ImageIO.resize (image_io.cr:289-335), then byte / 255 (image_io.cr:83-97).
  const bool same = sw == dw && sh == dh;
  const float scale_x = (float)sw / (float)dw, scale_y = (float)sh / (float)dh;
  for (int y = 0; y < dh; y++)
    for (int x = 0; x < dw; x++) {
      float* out = dst + ((int64_t)y * dw + x) * dc;
      if (same) {
        for (int c = 0; c < dc; c++) out[c] = (float)src[((int64_t)y * sw + x) * sc + c] / 255.0f;
        continue;
      }
      float sx = ((float)x + 0.5f) * scale_x - 0.5f, sy = ((float)y + 0.5f) * scale_y - 0.5f;
      sx = std::min(std::max(sx, 0.0f), (float)(sw - 1));
      sy = std::min(std::max(sy, 0.0f), (float)(sh - 1));
      const int x0 = std::min(std::max((int)sx, 0), sw - 1), y0 = std::min(std::max((int)sy, 0), sh - 1);
      const int x1 = std::min(x0 + 1, sw - 1), y1 = std::min(y0 + 1, sh - 1);
      const float fx = sx - (float)x0, fy = sy - (float)y0;
      for (int c = 0; c < dc; c++) {
        const float v00 = src[((int64_t)y0 * sw + x0) * sc + c], v10 = src[((int64_t)y0 * sw + x1) * sc + c];
        const float v01 = src[((int64_t)y1 * sw + x0) * sc + c], v11 = src[((int64_t)y1 * sw + x1) * sc + c];
        const float v0 = v00 * (1.0f - fx) + v10 * fx;
        const float v1 = v01 * (1.0f - fx) + v11 * fx;
        const float v = v0 * (1.0f - fy) + v1 * fy;
        out[c] = (float)(uint8_t)std::min(std::max(v, 0.0f), 255.0f) / 255.0f;
      }
    }
}

// ---- densification -------------------------------------------------------

// SplitMix64 finaliser (Steele, Lea & Flood 2014) as a counter-based hash:
// U(seed, index, draw) = top 24 bits of mix(seed ^ mix(8 * index + draw)) / 2^24.
static uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static float hash_u01(uint64_t seed, uint64_t idx, uint32_t draw) {
  const uint64_t h = mix64(seed ^ mix64(idx * 8ull + draw));
  return (float)(h >> 40) * (1.0f / 16777216.0f);
}

void gso_grad_accumulate(const float* d, int32_t stride, int64_t n, float* accum, int32_t* count) {
  // GradientAccumulator#accumulate, trainer.cr:86-99: norm of the 2D mean gradient.
  for (int64_t i = 0; i < n; i++) {
    const float gx = d[i * stride], gy = d[i * stride + 1];
    accum[i] += std::sqrt(gx * gx + gy * gy);
    count[i] += 1;
  }
}

void gso_densify_plan(const gsc_gaussians* g, const float* accum, const int32_t* count,
                      float grad_thr, float size_thr, float op_thr, uint8_t* flags, int64_t* counts) {
  // densify_and_prune!, trainer.cr:296-325: average gradient (GradientAccumulator#average,
  // trainer.cr:101-110), largest exp(log_scale), sigmoid(logit) against the thresholds.
  counts[0] = counts[1] = counts[2] = 0;
  for (int64_t i = 0; i < g->count; i++) {
    const float avg = count[i] == 0 ? 0.0f : accum[i] / (float)count[i];
    const float* ls = g->log_scale + i * 3;
    const float s0 = gso_expf(ls[0]), s1 = gso_expf(ls[1]), s2 = gso_expf(ls[2]);
    const float ms = std::fmax(s0, std::fmax(s1, s2));
    uint8_t f = 0;
    if (avg > grad_thr) f |= ms > size_thr ? GSC_DENSIFY_SPLIT : GSC_DENSIFY_CLONE;
    if (sigmoid(g->logit_opacity[i]) < op_thr) f |= GSC_DENSIFY_PRUNE;
    flags[i] = f;
    const bool split = f & GSC_DENSIFY_SPLIT, clone = f & GSC_DENSIFY_CLONE;
    counts[0] += !split && !(f & GSC_DENSIFY_PRUNE);
    counts[1] += clone;
    counts[2] += split;
  }
  // Gaussian3D#remove! never empties the set (gaussian.cr:234-235).
  if (g->count > 0 && counts[0] + counts[1] + counts[2] == 0) {
    for (int64_t i = 0; i < g->count; i++) flags[i] &= (uint8_t)~GSC_DENSIFY_PRUNE;
    counts[0] = g->count;
  }
}

static void densify_row(const gsc_gaussians* g, int64_t i, const gsc_gaussians_out* o, int64_t d,
                        const float p[3], const float l[3]) {
  for (int k = 0; k < 3; k++) {
    o->position[d * 3 + k] = p[k];
    o->log_scale[d * 3 + k] = l[k];
  }
  for (int k = 0; k < 4; k++) o->rotation[d * 4 + k] = g->rotation[i * 4 + k];
  o->logit_opacity[d] = g->logit_opacity[i];
  for (int k = 0; k < 48; k++) o->sh[d * 48 + k] = g->sh[i * 48 + k];
}

void gso_densify_apply(const gsc_gaussians* g, const uint8_t* flags, const gsc_gaussians_out* o,
                       float clone_noise, float ln_split, uint64_t seed) {
  // Output [kept][clones][split halves 1][split halves 2], each in index order.
  // Clone noise: add_position_noise!, trainer.cr:375-386. Split: split_gaussians!,
  // trainer.cr:332-370. Pruning (remove!, gaussian.cr:233-266) acts on original indices.
  int64_t nk = 0, nc = 0, ns = 0;
  for (int64_t i = 0; i < g->count; i++) {
    const uint8_t f = flags[i];
    nk += !(f & GSC_DENSIFY_SPLIT) && !(f & GSC_DENSIFY_PRUNE);
    nc += (f & GSC_DENSIFY_CLONE) != 0;
    ns += (f & GSC_DENSIFY_SPLIT) != 0;
  }
  int64_t ik = 0, ic = nk, is = nk + nc;
  for (int64_t i = 0; i < g->count; i++) {
    const uint8_t f = flags[i];
    const float* p = g->position + i * 3;
    const float* l = g->log_scale + i * 3;
    if (!(f & GSC_DENSIFY_SPLIT) && !(f & GSC_DENSIFY_PRUNE)) densify_row(g, i, o, ik++, p, l);
    if (f & GSC_DENSIFY_CLONE) {
      float q[3];
      for (int k = 0; k < 3; k++)
        q[k] = p[k] + (hash_u01(seed, (uint64_t)i, k) - 0.5f) * 2.0f * clone_noise;
      densify_row(g, i, o, ic++, q, l);
    }
    if (f & GSC_DENSIFY_SPLIT) {
      const float l2[3] = {l[0] - ln_split, l[1] - ln_split, l[2] - ln_split};
      for (int h = 0; h < 2; h++) {
        const float offset = gso_expf(l2[0]) * 0.5f * (h == 0 ? 1.0f : -1.0f);
        float q[3];
        for (int k = 0; k < 3; k++)
          q[k] = p[k] + offset * (hash_u01(seed, (uint64_t)i, 3 + 3 * h + k) - 0.5f);
        densify_row(g, i, o, is + h * ns, q, l2);
      }
      is++;
    }
  }
}

}  // extern "C"

namespace {
// Float32#**(Int32) of the reference's Crystal host (adam.cr:129-130): the
// LLVM powi intrinsic, at run time compiler-rt's __powisf2 -- binary
// exponentiation in fp32, lowest exponent bit first.
float powi_f32(float a, int b) {
  const bool recip = b < 0;
  float r = 1.0f;
  for (;;) {
    if (b & 1) r *= a;
    b /= 2;
    if (b == 0) break;
    a *= a;
  }
  return recip ? 1.0f / r : r;
}
}  // namespace

extern "C" {

float gso_powi_f32(float a, int32_t b) { return powi_f32(a, b); }

void gso_adam_step(const gsc_adam_group* groups, int32_t ngroups, float beta1, float beta2,
                   float eps, int32_t step, float grad_scale) {
  // Adam#step / update_adam! / apply_weight_decay!, src/optim/adam.cr:86-176.
  // Bias corrections 1 - beta^t in fp32, with beta^t as Float32#**(Int32)
  // evaluates it (adam.cr:129-130; see powi_f32).
  const float bc1 = 1.0f - powi_f32(beta1, step);
  const float bc2 = 1.0f - powi_f32(beta2, step);
  for (int gi = 0; gi < ngroups; gi++) {
    const gsc_adam_group& G = groups[gi];
    const float decay = 1.0f - G.lr * G.weight_decay;
#pragma omp parallel for num_threads(g_threads) schedule(static)
    for (int64_t i = 0; i < G.numel; i++) {
      float p = G.param[i];
      if (G.weight_decay > 0.0f) p = p * decay;
      float gr = G.grad[i] * grad_scale;
      float m = beta1 * G.m[i] + (1.0f - beta1) * gr;
      float v = beta2 * G.v[i] + (1.0f - beta2) * gr * gr;
      float mh = m / bc1;
      float vh = v / bc2;
      p = p - G.lr * mh / (std::sqrt(vh) + eps);
      G.m[i] = m;
      G.v[i] = v;
      G.param[i] = p;
    }
  }
}

int64_t gso_render_view(const gsc_gaussians* g, const gsc_camera* cam,
                        const gsc_raster_config* cfg, float* image, const float* target,
                        float l1_scale, const gsc_gaussian_grads* grads, double* loss_sum) {
  const int64_t n = g->count;
  const int W = cam->width, H = cam->height;
  const int tiles_x = (W + TILE - 1) / TILE, tiles_y = (H + TILE - 1) / TILE;
  std::vector<float> mean2d(n * 2), cov2d(n * 3), depth(n), radius(n), colors(n * 3), opac(n);
  gso_preprocess(g, cam, cfg, mean2d.data(), cov2d.data(), nullptr, depth.data(), radius.data(),
                 colors.data(), opac.data(), nullptr, nullptr);
  int64_t m = gso_emit_keys(n, mean2d.data(), depth.data(), radius.data(), tiles_x, tiles_y,
                            nullptr, nullptr, 0);
  std::vector<uint64_t> keys(m);
  std::vector<uint32_t> vals(m);
  gso_emit_keys(n, mean2d.data(), depth.data(), radius.data(), tiles_x, tiles_y, keys.data(),
                vals.data(), m);
  gso_sort_pairs(m, keys.data(), vals.data(), 0, 64);
  std::vector<uint32_t> ranges((size_t)tiles_x * tiles_y * 2);
  gso_tile_ranges(m, keys.data(), tiles_x * tiles_y, ranges.data());
  std::vector<float> fT((size_t)W * H);
  std::vector<uint32_t> last((size_t)W * H);
  gso_composite_forward(W, H, ranges.data(), vals.data(), mean2d.data(), cov2d.data(), opac.data(),
                        colors.data(), cfg, image, nullptr, fT.data(), last.data());
  if (target && grads) {
    std::vector<float> g2d(n * 9, 0.0f);
    gso_composite_backward(W, H, ranges.data(), vals.data(), mean2d.data(), cov2d.data(),
                           opac.data(), colors.data(), cfg, nullptr, image, target, l1_scale,
                           fT.data(), last.data(), g2d.data(), loss_sum);
    gso_preprocess_backward(g, cam, cfg, g2d.data(), grads, nullptr, nullptr, nullptr, nullptr);
  }
  return m;
}

}  // extern "C"
