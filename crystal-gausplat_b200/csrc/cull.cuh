// cull.cuh — exact whole-tile rejection of a Gaussian, shared by the
// compositing kernels and by contributing-pairs binning in preprocess.
#pragma once
#include "common.cuh"

namespace gs {

// Natural log of a positive finite float: x = m 2^e with m in [1/sqrt 2,
// sqrt 2), ln x = e ln 2 + 2 atanh(s), s = (m - 1)/(m + 1), |s| <= 0.1716,
// by its odd power series through s^13 (truncation below 1e-11). Only +, *, /
// in a fixed order (no contraction), so every IEEE implementation returns the
// same bits; the error is a few ulp, far inside the margins below.
__device__ __forceinline__ float gs_logf_series(float x) {
  int e;
  float m = frexpf(x, &e);
  if (m < 0.70710678f) {
    m *= 2.0f;
    e -= 1;
  }
  const float s = (m - 1.0f) / (m + 1.0f), s2 = s * s;
  float p = 1.0f / 13.0f;
  p = p * s2 + 1.0f / 11.0f;
  p = p * s2 + 1.0f / 9.0f;
  p = p * s2 + 1.0f / 7.0f;
  p = p * s2 + 1.0f / 5.0f;
  p = p * s2 + 1.0f / 3.0f;
  p = p * s2 + 1.0f;
  return (float)e * 0.69314718f + 2.0f * s * p;
}

// Whole-tile rejection. True only if NO pixel centre of the tile's rectangle
// [rx0, rx1] x [ry0, ry1] can pass the alpha test for this Gaussian. The
// minimum of the Mahalanobis form q(d) = d^T conic d over the rectangle (zero
// if the mean is inside, else attained on an edge) is compared with the
// opacity-aware threshold
//     o * exp(-q/2) < alpha_min  <=>  q > -2 ln(alpha_min / o).
// Both this fp32 evaluation and the per-pixel fp32 one have relative error
// <= 10 eps / (1 - rho) + 2 eps, rho = |B| / sqrt(AC) (each term of the form
// is within 5 eps, and |A dx^2| + |2 B dx dy| + |C dy^2| <= 2 q / (1 - rho)),
// i.e. <= 6.1e-4 each once 1 - rho >= 1e-3; the cull is refused below that,
// and the threshold is raised by 2e-3 relative + 2e-3 absolute and lowered in
// ln by 1e-4 (covering the exponential and the product o * G). The edge
// minimiser dy* = -B dx / C, computed as dx * (-B / C), is a point of the edge
// whose form exceeds the edge minimum by C (rounding of dy*)^2 only, orders of
// magnitude below the margin. Non-finite or non-positive-definite inputs are
// never culled. The set of Gaussians that reach the per-pixel loop therefore
// changes, but not the result.
//
// cull_prepare does the per-Gaussian part (logarithm, square root, ratios)
// once; cull_tile tests one rectangle with products and clamps.
struct CullGauss {
  float A, B, C, mx, my, nbc, nba, thr;
  float cut;  // ln(alpha_min / o) - 1e-4 (kind 2 only)
  int kind;  // 0: never culled, 1: culled everywhere, 2: test each tile
};

__device__ __forceinline__ CullGauss cull_prepare(float4 g0, float conic_c, float o, float alpha_min) {
  CullGauss g;
  g.kind = 0;
  if (!isfinite(g0.x) || !isfinite(g0.y)) return g;
  if (!(o > 0.0f)) {
    g.kind = (o == 0.0f && isfinite(g0.z) && isfinite(g0.w) && isfinite(conic_c)) ? 1 : 0;
    return g;
  }
  const float A = g0.z, B = g0.w, C = conic_c;
  if (!(A > 0.0f && C > 0.0f) || !isfinite(A) || !isfinite(B) || !isfinite(C)) return g;
  const float rho = fabsf(B) / sqrtf(A * C);
  if (!(1.0f - rho >= 1e-3f)) return g;
  const float cut = gs_logf_series(alpha_min / o) - 1e-4f;
  if (cut >= 0.0f) {  // o < alpha_min: alpha = o*G <= o never reaches alpha_min
    g.kind = 1;
    return g;
  }
  g.A = A; g.B = B; g.C = C;
  g.mx = g0.x; g.my = g0.y;
  g.cut = cut;
  g.nbc = -B / C;
  g.nba = -B / A;
  g.thr = -2.0f * cut * (1.0f + 2e-3f) + 2e-3f;
  g.kind = 2;
  return g;
}

__device__ __forceinline__ float cull_form(const CullGauss& g, float dx, float dy) {
  return g.A * dx * dx + 2.0f * g.B * dx * dy + g.C * dy * dy;
}

__device__ __forceinline__ bool cull_tile(const CullGauss& g, float rx0, float rx1, float ry0, float ry1) {
  if (g.kind != 2) return g.kind == 1;
  const float x0 = rx0 - g.mx, x1 = rx1 - g.mx, y0 = ry0 - g.my, y1 = ry1 - g.my;
  if (x0 <= 0.0f && x1 >= 0.0f && y0 <= 0.0f && y1 >= 0.0f) return false;  // mean inside
  float qmin = INFINITY;
#pragma unroll
  for (int e = 0; e < 2; e++) {  // edges x = x0, x1
    const float dx = e ? x1 : x0;
    qmin = fminf(qmin, cull_form(g, dx, fminf(fmaxf(dx * g.nbc, y0), y1)));
  }
#pragma unroll
  for (int e = 0; e < 2; e++) {  // edges y = y0, y1
    const float dy = e ? y1 : y0;
    qmin = fminf(qmin, cull_form(g, fminf(fmaxf(dy * g.nba, x0), x1), dy));
  }
  return qmin > g.thr;
}

// Per-pixel skip threshold of one Gaussian: a pixel whose power is below it
// has o * G < alpha_min (G = gs_expf(power) is within 2 ulp of e^power and
// the threshold sits 1.1e-3 below ln(alpha_min / o), far beyond the few-ulp
// error of the logarithm), so it is rejected before the exponential with the
// accepted set unchanged. `fallback` (ln alpha_min minus a margin, valid for
// every opacity <= 1) is used where the cull has no per-Gaussian threshold.
__device__ __forceinline__ float pixel_power_cut(const CullGauss& g, float fallback) {
  return g.kind == 2 ? fmaxf(g.cut - 1e-3f, fallback) : fallback;
}

// g0 = {mean.x, mean.y, conic.xx, conic.xy}, conic_c = conic.yy, o = opacity.
__device__ __forceinline__ bool tile_culled(float4 g0, float conic_c, float o, float rx0, float rx1,
                                            float ry0, float ry1, float alpha_min) {
  return cull_tile(cull_prepare(g0, conic_c, o, alpha_min), rx0, rx1, ry0, ry1);
}

// Row form of the same test, for contributing-pairs binning. The region that
// can pass the alpha test is inside the ellipse q(d) <= thr (thr as above).
// Its intersection with a horizontal strip dy in [y0, y1] is convex, so its x
// projection is one interval [xl, xr]: xl is the left boundary x(dy) = (-B dy -
// sqrt(A thr - det dy^2)) / A (convex in dy) at its minimiser clamped into the
// strip, i.e. the ellipse's leftmost point dy_l = B sqrt(thr / (C det)), and xr
// likewise at -dy_l. A tile of the row survives iff its pixel-centre span
// [rx0, rx1] meets [xl, xr]. The interval is widened by 1e-2 px + 2e-3 of the
// ellipse's half-width sqrt(thr C / det), and the strip's reach by the same
// share of its half-height, which covers the rounding of this evaluation (the
// cancellation in A thr - det dy^2 contributes at most sqrt(2 eps thr / A), a
// sixth of that share); the culled set is therefore a subset of the exact one.
struct RowCull {
  float mx, my, A, B, det, thr, dyl, ye, pad;
  int kind;  // 0: never culled, 1: culled everywhere, 2: test each row
};

__device__ __forceinline__ RowCull row_cull_prepare(float4 g0, float conic_c, float o, float alpha_min) {
  const CullGauss c = cull_prepare(g0, conic_c, o, alpha_min);
  RowCull r;
  r.kind = c.kind;
  if (c.kind != 2) return r;
  r.mx = c.mx; r.my = c.my; r.A = c.A; r.B = c.B; r.thr = c.thr;
  r.det = c.A * c.C - c.B * c.B;
  if (!(r.det > 0.0f)) {
    r.kind = 0;
    return r;
  }
  const float xe = sqrtf(r.thr * c.C / r.det), ye = sqrtf(r.thr * c.A / r.det);
  r.dyl = c.B * sqrtf(r.thr / (c.C * r.det));
  r.pad = 1e-2f + 2e-3f * xe;
  r.ye = ye + 1e-2f + 2e-3f * ye;
  return r;
}

// Interval [xl, xr] (relative to the mean, widened) of the strip of pixel-centre
// rows [ry0, ry1]; false if the strip misses the ellipse.
__device__ __forceinline__ bool row_extent(const RowCull& r, float ry0, float ry1, float* xl, float* xr) {
  const float y0 = ry0 - r.my, y1 = ry1 - r.my;
  if (y0 > r.ye || y1 < -r.ye) return false;
  const float a = fmaxf(y0, -r.ye), b = fminf(y1, r.ye);
  const float dl = fminf(fmaxf(r.dyl, a), b), dr = fminf(fmaxf(-r.dyl, a), b);
  const float Dl = fmaxf(0.0f, r.A * r.thr - r.det * dl * dl);
  const float Dr = fmaxf(0.0f, r.A * r.thr - r.det * dr * dr);
  *xl = (-r.B * dl - sqrtf(Dl)) / r.A - r.pad;
  *xr = (-r.B * dr + sqrtf(Dr)) / r.A + r.pad;
  return true;
}

// Pixel-centre rectangle of tile (tx, ty) in a width x height image.
__device__ __forceinline__ void tile_pixel_rect(int tx, int ty, int width, int height, float* rx0, float* rx1,
                                                float* ry0, float* ry1) {
  *rx0 = tx * GS_TILE + 0.5f;
  *ry0 = ty * GS_TILE + 0.5f;
  *rx1 = min(tx * GS_TILE + GS_TILE, width) - 0.5f;
  *ry1 = min(ty * GS_TILE + GS_TILE, height) - 0.5f;
}

}  // namespace gs
