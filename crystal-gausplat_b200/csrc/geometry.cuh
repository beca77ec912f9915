// geometry.cuh — per-Gaussian math shared by the preprocess forward and
// backward kernels: quaternion -> rotation, 3-D covariance, EWA projection and
// spherical-harmonics colour. Operation order is written out explicitly (the
// library is compiled without FMA contraction) and follows
// src/metal/kernels/gaussian.metal:64-308, with the view matrix read
// row-major as the host intends (src/gaussian_splatting/camera.cr:185-187).
#pragma once
#include "common.cuh"

namespace gs {

struct Projected {
  bool visible;
  float xc, yc, zc;
  float px, py;
  float J00, J02, J11, J12;
  float C[6];      // camera-space covariance, upper: 00 01 02 11 12 22
  float a, b, c;   // cov2d with low-pass (xx, xy, yy)
  float det;
  float r;
  float A, B, Cc;  // inverse cov2d, zero when det <= 0
};

// quat_to_matrix, gaussian.metal:64-82; q = (w, x, y, z).
__device__ __forceinline__ void quat_to_R(float w, float x, float y, float z, float R[3][3]) {
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

// GSC_MODE_REF uses the stored quaternion (host normalize_rotations! is a
// no-op for GPU tensors, gaussian.cr:274-296); GSC_MODE_FULL normalises it.
__device__ __forceinline__ void load_quat(float4 q4, int mode, float q[4], float* norm) {
  float w = q4.x, x = q4.y, y = q4.z, z = q4.w;
  if (mode == GSC_MODE_FULL) {
    float n = sqrtf(((w * w + x * x) + y * y) + z * z);
    *norm = n;
    if (n > 0.0f) {
      w = w / n; x = x / n; y = y / n; z = z / n;
    } else {
      w = 1.0f; x = 0.0f; y = 0.0f; z = 0.0f;
    }
  } else {
    *norm = 1.0f;
  }
  q[0] = w; q[1] = x; q[2] = y; q[3] = z;
}

// compute_cov3d, gaussian.metal:90-131.
__device__ __forceinline__ void cov3d_of(const float s[3], const float R[3][3], float cov[6]) {
  float s2[3] = {s[0] * s[0], s[1] * s[1], s[2] * s[2]};
  int k = 0;
#pragma unroll
  for (int i = 0; i < 3; i++)
#pragma unroll
    for (int j = i; j < 3; j++)
      cov[k++] = (R[i][0] * s2[0] * R[j][0] + R[i][1] * s2[1] * R[j][1]) + R[i][2] * s2[2] * R[j][2];
}

__device__ __forceinline__ float sym3(const float c[6], int i, int j) {
  // (i,j) -> upper-triangle index; i, j are compile-time after unrolling.
  int lo = i < j ? i : j, hi = i < j ? j : i;
  int idx = lo == 0 ? hi : (lo == 1 ? 2 + hi : 5);
  return c[idx];
}

// project_gaussians, gaussian.metal:138-249.
__device__ __forceinline__ void project(const float p[3], const float cov3[6], const gsc_camera& cam,
                                        const gsc_raster_config& cfg, Projected* o) {
  const float* W = cam.view;
  o->xc = ((W[0] * p[0] + W[1] * p[1]) + W[2] * p[2]) + W[3];
  o->yc = ((W[4] * p[0] + W[5] * p[1]) + W[6] * p[2]) + W[7];
  o->zc = ((W[8] * p[0] + W[9] * p[1]) + W[10] * p[2]) + W[11];
  o->visible = false;
  o->r = 0.0f;
  o->A = o->B = o->Cc = 0.0f;
  o->a = o->b = o->c = 0.0f;
  o->px = o->py = 0.0f;
  if (o->zc <= cfg.near_z || o->zc > cfg.far_z) return;
  float xn = o->xc / o->zc, yn = o->yc / o->zc;
  if (fabsf(xn) > cam.tan_fov_x * cfg.fov_cull || fabsf(yn) > cam.tan_fov_y * cfg.fov_cull) return;
  o->visible = true;
  o->px = cam.fx * xn + cam.cx;
  o->py = cam.fy * yn + cam.cy;
  float z2 = o->zc * o->zc;
  o->J00 = cam.fx / o->zc;
  o->J02 = -cam.fx * o->xc / z2;
  o->J11 = cam.fy / o->zc;
  o->J12 = -cam.fy * o->yc / z2;
  const float V[3][3] = {{W[0], W[1], W[2]}, {W[4], W[5], W[6]}, {W[8], W[9], W[10]}};
  float T[3][3];
#pragma unroll
  for (int i = 0; i < 3; i++)
#pragma unroll
    for (int k = 0; k < 3; k++)
      T[i][k] = (V[i][0] * sym3(cov3, 0, k) + V[i][1] * sym3(cov3, 1, k)) + V[i][2] * sym3(cov3, 2, k);
  int q = 0;
#pragma unroll
  for (int i = 0; i < 3; i++)
#pragma unroll
    for (int j = i; j < 3; j++) o->C[q++] = (T[i][0] * V[j][0] + T[i][1] * V[j][1]) + T[i][2] * V[j][2];
  const float C00 = o->C[0], C01 = o->C[1], C02 = o->C[2], C11 = o->C[3], C12 = o->C[4], C22 = o->C[5];
  const float J00 = o->J00, J02 = o->J02, J11 = o->J11, J12 = o->J12;
  float xx = J00 * J00 * C00 + 2.0f * J00 * J02 * C02 + J02 * J02 * C22;
  float xy = J00 * J11 * C01 + J00 * J12 * C02 + J02 * J11 * C12 + J02 * J12 * C22;
  float yy = J11 * J11 * C11 + 2.0f * J11 * J12 * C12 + J12 * J12 * C22;
  xx += cfg.lowpass;
  yy += cfg.lowpass;
  o->a = xx; o->b = xy; o->c = yy;
  float det = xx * yy - xy * xy;
  o->det = det;
  float trace = xx + yy;
  float lambda_max = 0.5f * (trace + sqrtf(fmaxf(0.0f, trace * trace - 4.0f * det)));
  o->r = ceilf(3.0f * sqrtf(lambda_max));
  if (det > 0.0f) {
    // Inverse covariance as rasterize_tile computes it per pixel (gaussian.metal:412-418).
    float inv_det = 1.0f / det;
    o->A = yy * inv_det;
    o->B = -xy * inv_det;
    o->Cc = xx * inv_det;
  }
}

// normalize(campos - pos), gaussian.metal:268-269.
__device__ __forceinline__ void view_dir(const float p[3], const gsc_camera& cam, float d[3], float* len) {
  float v0 = cam.campos[0] - p[0], v1 = cam.campos[1] - p[1], v2 = cam.campos[2] - p[2];
  float l = sqrtf((v0 * v0 + v1 * v1) + v2 * v2);
  *len = l;
  d[0] = v0 / l; d[1] = v1 / l; d[2] = v2 / l;
}

// SH basis b[4..15] (degrees 2 and 3) with the reference constants;
// degrees 0 and 1 are applied inline as gaussian.metal:279-287 does.
__device__ __forceinline__ void sh_basis_hi(float x, float y, float z, float b[16]) {
  const ShConsts K = sh_consts();
  float xx = x * x, yy = y * y, zz = z * z;
  float xy = x * y, yz = y * z, xz = x * z;
  b[4] = K.c2[0] * xy;
  b[5] = K.c2[1] * yz;
  b[6] = K.c2[2] * (2.0f * zz - xx - yy);
  b[7] = K.c2[3] * xz;
  b[8] = K.c2[4] * (xx - yy);
  b[9] = K.c3[0] * y * (3.0f * xx - yy);
  b[10] = K.c3[1] * xy * z;
  b[11] = K.c3[2] * y * (4.0f * zz - xx - yy);
  b[12] = K.c3[3] * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
  b[13] = K.c3[4] * x * (4.0f * zz - xx - yy);
  b[14] = K.c3[5] * z * (xx - yy);
  b[15] = K.c3[6] * x * (xx - 3.0f * yy);
}

// eval_sh, gaussian.metal:256-308 (raw = value before "+0.5, max 0").
// sh points at the 48 coefficients of one Gaussian (k*3 + c).
template <typename ShRead>
__device__ __forceinline__ void sh_eval(ShRead S, float x, float y, float z, const float b[16],
                                        int degree, int mode, float raw[3]) {
#pragma unroll
  for (int c = 0; c < 3; c++) {
    float r = 0.0f;
    r += kShC0 * S(0 * 3 + c);
    if (degree >= 1) r += kShC1 * (-y * S(1 * 3 + c) + z * S(2 * 3 + c) - x * S(3 * 3 + c));
    if (degree >= 2 && (mode == GSC_MODE_FULL || c == 0)) {
      float t = b[4] * S(4 * 3 + c) + b[5] * S(5 * 3 + c) + b[6] * S(6 * 3 + c) + b[7] * S(7 * 3 + c) +
                b[8] * S(8 * 3 + c);
      r += t;
    }
    if (degree >= 3 && mode == GSC_MODE_FULL) {
      float t = b[9] * S(9 * 3 + c) + b[10] * S(10 * 3 + c) + b[11] * S(11 * 3 + c) +
                b[12] * S(12 * 3 + c) + b[13] * S(13 * 3 + c) + b[14] * S(14 * 3 + c) +
                b[15] * S(15 * 3 + c);
      r += t;
    }
    raw[c] = r;
  }
}

// Partial derivatives of the real SH basis with respect to the unit view
// direction (k = 1..15); zero where basis k does not depend on a component.
__device__ __forceinline__ void sh_basis_derivs(float x, float y, float z, float DX[16], float DY[16],
                                                float DZ[16]) {
  const ShConsts K = sh_consts();
  const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
#pragma unroll
  for (int k = 0; k < 16; k++) DX[k] = DY[k] = DZ[k] = 0.0f;
  DY[1] = -kShC1;
  DZ[2] = kShC1;
  DX[3] = -kShC1;
  DX[4] = K.c2[0] * y; DY[4] = K.c2[0] * x;
  DY[5] = K.c2[1] * z; DZ[5] = K.c2[1] * y;
  DX[6] = K.c2[2] * (-2.0f * x); DY[6] = K.c2[2] * (-2.0f * y); DZ[6] = K.c2[2] * (4.0f * z);
  DX[7] = K.c2[3] * z; DZ[7] = K.c2[3] * x;
  DX[8] = K.c2[4] * (2.0f * x); DY[8] = K.c2[4] * (-2.0f * y);
  DX[9] = K.c3[0] * (6.0f * xy); DY[9] = K.c3[0] * (3.0f * xx - 3.0f * yy);
  DX[10] = K.c3[1] * yz; DY[10] = K.c3[1] * xz; DZ[10] = K.c3[1] * xy;
  DX[11] = K.c3[2] * (-2.0f * xy); DY[11] = K.c3[2] * (4.0f * zz - xx - 3.0f * yy); DZ[11] = K.c3[2] * (8.0f * yz);
  DX[12] = K.c3[3] * (-6.0f * xz); DY[12] = K.c3[3] * (-6.0f * yz);
  DZ[12] = K.c3[3] * (6.0f * zz - 3.0f * xx - 3.0f * yy);
  DX[13] = K.c3[4] * (4.0f * zz - 3.0f * xx - yy); DY[13] = K.c3[4] * (-2.0f * xy); DZ[13] = K.c3[4] * (8.0f * xz);
  DX[14] = K.c3[5] * (2.0f * xz); DY[14] = K.c3[5] * (-2.0f * yz); DZ[14] = K.c3[5] * (xx - yy);
  DX[15] = K.c3[6] * (3.0f * xx - 3.0f * yy); DY[15] = K.c3[6] * (-6.0f * xy);
}

}  // namespace gs
