// ssim.cu — SSIM and the combined L1 + SSIM loss on the device
// (Loss.ssim / ssim_loss_with_grad / combined_with_grad / mse_with_grad,
// src/ops/loss.cr:59-249), which the reference runs as serial host loops.
//
// Two arithmetic modes:
//  REF  — the reference's literal SSIM: 2D Gaussian window (sigma 1.5,
//         normalised by its fp32 sum), valid region only, two-pass local
//         variance, per-pixel summation in window order; its gradient is the
//         reference's surrogate 2 (pred - target) / n (loss.cr:194-216).
//  FULL — the same definition with the window applied separably (the 2D
//         window is the outer product of the normalised 1D one) and the
//         analytic gradient of the mean SSIM. With the local moments
//         mu, m_xx = blur(x^2), m_xy = blur(x y), every valid pixel p gives
//         A = dS/dmu_x, B = dS/dm_xx, C = dS/dm_xy, and
//         dSum S / dx_q = blur(A)(q) + 2 x_q blur(B)(q) + y_q blur(C)(q).
//
// Layout: images are [H, W, C] row-major fp32, C <= 4. Each CTA owns a 16x16
// tile of output pixels and stages the tile plus its halo (pad = window/2 on
// each side) in shared memory; block partial sums are double and reduced in a
// fixed order, so results are reproducible run to run.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace gs {

constexpr int kSsimTile = 16;
constexpr int kSsimMaxWin = 15;
constexpr int kSsimMaxSpan = kSsimTile + kSsimMaxWin - 1;  // 30
constexpr int kSsimMaxC = 4;

struct SsimArgs {
  const float* pred;
  const float* target;
  int H, W, C, win, pad;
  int full;              // 1: FULL (separable + analytic gradient), 0: REF
  float* map;            // nullable [H, W, C]: per-pixel SSIM on the valid region
  float* abc;            // FULL: [3][C][H][W] A, B, C maps on the valid region
  double* ssim_part;     // per-block sum of S
  float* grad;           // nullable [H, W, C], written
  double* l1_part;       // per-block sum of |pred - target|
  float w_l1, w_ssim;    // grad = w_l1 * sign / n + w_ssim * d(ssim loss)
  float n_f, count_f;    // numel, number of valid (pixel, channel) terms
};

__device__ __forceinline__ float ssim_c1() { return 0.01f * 0.01f; }
__device__ __forceinline__ float ssim_c2() { return 0.03f * 0.03f; }

// Reference window (loss.cr:262-281): exp(-(dx^2 + dy^2) / (2 sigma^2)), fp32
// sum in row-major order, each value divided by it. The 1D window of the
// separable form is built the same way from exp(-d^2 / (2 sigma^2)).
__device__ void build_window(float* s_w, int win, bool two_d) {
  const int c = win / 2, n = two_d ? win * win : win;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int dx = (two_d ? i % win : i) - c, dy = two_d ? i / win - c : 0;
    s_w[i] = gs_expf((float)(-(dx * dx + dy * dy)) / (2.0f * 1.5f * 1.5f));
  }
  __syncthreads();
  __shared__ float s_sum;
  if (threadIdx.x == 0) {
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum += s_w[i];
    s_sum = sum;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) s_w[i] = s_w[i] / s_sum;
  __syncthreads();
}

// Fixed-order block sum of one double per thread (256 threads).
__device__ __forceinline__ double block_sum_d(double v, double* s_red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x == 0)
    for (int w = 0; w < 8; w++) t += s_red[w];
  return t;
}

// Stage rows [y0, y0+span) x cols [x0, x0+span) of channel c (zero outside the image).
__device__ __forceinline__ void stage_tile(const float* img, const SsimArgs& a, int c, int y0, int x0, int span,
                                           float* s) {
  for (int i = threadIdx.x; i < span * span; i += 256) {
    const int r = i / span, q = i % span, y = y0 + r, x = x0 + q;
    s[i] = (y < a.H && x < a.W) ? img[((int64_t)y * a.W + x) * a.C + c] : 0.0f;
  }
}

__global__ void __launch_bounds__(256) ssim_ref_kernel(SsimArgs a) {
  __shared__ float s_w[kSsimMaxWin * kSsimMaxWin];
  __shared__ float s_p[kSsimMaxSpan * kSsimMaxSpan];
  __shared__ float s_t[kSsimMaxSpan * kSsimMaxSpan];
  __shared__ double s_red[8];
  build_window(s_w, a.win, true);
  const int span = kSsimTile + 2 * a.pad;
  const int tx = threadIdx.x % kSsimTile, ty = threadIdx.x / kSsimTile;
  const int x0 = blockIdx.x * kSsimTile, y0 = blockIdx.y * kSsimTile;  // tile's window origin
  const int x = a.pad + x0 + tx, y = a.pad + y0 + ty;                    // output pixel
  const bool valid = x < a.W - a.pad && y < a.H - a.pad;
  const int ws = a.win;
  double acc = 0.0;
  for (int c = 0; c < a.C; c++) {
    __syncthreads();
    stage_tile(a.pred, a, c, y0, x0, span, s_p);
    stage_tile(a.target, a, c, y0, x0, span, s_t);
    __syncthreads();
    if (!valid) continue;
    // loss.cr:146-179, literally: means, then variances about them.
    float mu_x = 0.0f, mu_y = 0.0f, sx = 0.0f, sy = 0.0f, sxy = 0.0f;
    for (int wy = 0; wy < ws; wy++)
      for (int wx = 0; wx < ws; wx++) {
        const float w = s_w[wy * ws + wx];
        const int k = (ty + wy) * span + tx + wx;
        mu_x += w * s_p[k];
        mu_y += w * s_t[k];
      }
    for (int wy = 0; wy < ws; wy++)
      for (int wx = 0; wx < ws; wx++) {
        const float w = s_w[wy * ws + wx];
        const int k = (ty + wy) * span + tx + wx;
        const float px = s_p[k], py = s_t[k];
        sx += w * (px - mu_x) * (px - mu_x);
        sy += w * (py - mu_y) * (py - mu_y);
        sxy += w * (px - mu_x) * (py - mu_y);
      }
    const float num = (2.0f * mu_x * mu_y + ssim_c1()) * (2.0f * sxy + ssim_c2());
    const float den = (mu_x * mu_x + mu_y * mu_y + ssim_c1()) * (sx + sy + ssim_c2());
    const float S = num / den;
    acc += (double)S;
    if (a.map) a.map[((int64_t)y * a.W + x) * a.C + c] = S;
  }
  const double t = block_sum_d(acc, s_red);
  if (threadIdx.x == 0) a.ssim_part[blockIdx.y * gridDim.x + blockIdx.x] = t;
}

__global__ void __launch_bounds__(256) ssim_full_fwd_kernel(SsimArgs a) {
  __shared__ float s_g[kSsimMaxWin];
  __shared__ float s_p[kSsimMaxSpan * kSsimMaxSpan];
  __shared__ float s_t[kSsimMaxSpan * kSsimMaxSpan];
  __shared__ float s_h[5][kSsimMaxSpan * kSsimTile];
  __shared__ double s_red[8];
  build_window(s_g, a.win, false);
  const int span = kSsimTile + 2 * a.pad;
  const int tx = threadIdx.x % kSsimTile, ty = threadIdx.x / kSsimTile;
  const int x0 = blockIdx.x * kSsimTile, y0 = blockIdx.y * kSsimTile;
  const int x = a.pad + x0 + tx, y = a.pad + y0 + ty;
  const bool valid = x < a.W - a.pad && y < a.H - a.pad;
  const int ws = a.win;
  const int64_t plane = (int64_t)a.H * a.W;
  double acc = 0.0;
  for (int c = 0; c < a.C; c++) {
    __syncthreads();
    stage_tile(a.pred, a, c, y0, x0, span, s_p);
    stage_tile(a.target, a, c, y0, x0, span, s_t);
    __syncthreads();
    // Horizontal pass: span rows x 16 output columns, five moments.
    for (int i = threadIdx.x; i < span * kSsimTile; i += 256) {
      const int r = i / kSsimTile, q = i % kSsimTile;
      float hx = 0.0f, hy = 0.0f, hxx = 0.0f, hyy = 0.0f, hxy = 0.0f;
      for (int k = 0; k < ws; k++) {
        const float g = s_g[k], p = s_p[r * span + q + k], t = s_t[r * span + q + k];
        hx += g * p;
        hy += g * t;
        hxx += g * (p * p);
        hyy += g * (t * t);
        hxy += g * (p * t);
      }
      s_h[0][i] = hx; s_h[1][i] = hy; s_h[2][i] = hxx; s_h[3][i] = hyy; s_h[4][i] = hxy;
    }
    __syncthreads();
    if (!valid) continue;
    float m[5] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    for (int k = 0; k < ws; k++) {
      const float g = s_g[k];
      const int i = (ty + k) * kSsimTile + tx;
#pragma unroll
      for (int j = 0; j < 5; j++) m[j] += g * s_h[j][i];
    }
    const float mu_x = m[0], mu_y = m[1];
    const float sxx = m[2] - mu_x * mu_x, syy = m[3] - mu_y * mu_y, sxy = m[4] - mu_x * mu_y;
    const float n1 = 2.0f * mu_x * mu_y + ssim_c1(), n2 = 2.0f * sxy + ssim_c2();
    const float d1 = mu_x * mu_x + mu_y * mu_y + ssim_c1(), d2 = sxx + syy + ssim_c2();
    const float dd = d1 * d2;
    const float S = (n1 * n2) / dd;
    acc += (double)S;
    if (a.map) a.map[((int64_t)y * a.W + x) * a.C + c] = S;
    if (a.abc) {
      // Partials holding the central moments, then the chain to (mu_x, m_xx, m_xy).
      const float dmu = 2.0f * mu_y * n2 / dd - 2.0f * mu_x * S / d1;
      const float dsxx = -S / d2;
      const float dsxy = 2.0f * n1 / dd;
      const float A = dmu - 2.0f * mu_x * dsxx - mu_y * dsxy;
      const int64_t o = (int64_t)y * a.W + x;
      a.abc[(0 * a.C + c) * plane + o] = A;
      a.abc[(1 * a.C + c) * plane + o] = dsxx;
      a.abc[(2 * a.C + c) * plane + o] = dsxy;
    }
  }
  const double t = block_sum_d(acc, s_red);
  if (threadIdx.x == 0) a.ssim_part[blockIdx.y * gridDim.x + blockIdx.x] = t;
}

// Gradient of the combined loss over every pixel (16x16 tiles of the whole
// image) and the per-block L1 sums. FULL: blurs A, B, C (zero off the valid
// region) separably. REF: the reference's surrogate 2 (p - t) / n.
__global__ void __launch_bounds__(256) loss_grad_kernel(SsimArgs a) {
  __shared__ float s_g[kSsimMaxWin];
  __shared__ float s_m[3][kSsimMaxSpan * kSsimMaxSpan];
  __shared__ float s_h[3][kSsimMaxSpan * kSsimTile];
  __shared__ double s_red[8];
  const bool full = a.abc != nullptr;  // FULL with a valid region and an SSIM term
  if (full) build_window(s_g, a.win, false);
  const int span = kSsimTile + 2 * a.pad;
  const int tx = threadIdx.x % kSsimTile, ty = threadIdx.x / kSsimTile;
  const int x = blockIdx.x * kSsimTile + tx, y = blockIdx.y * kSsimTile + ty;
  const bool inside = x < a.W && y < a.H;
  const int ws = a.win;
  const int64_t plane = (int64_t)a.H * a.W;
  double l1 = 0.0;
  for (int c = 0; c < a.C; c++) {
    float dS = 0.0f;
    if (full) {
      __syncthreads();
      const int ya = blockIdx.y * kSsimTile - a.pad, xa = blockIdx.x * kSsimTile - a.pad;
      for (int i = threadIdx.x; i < span * span; i += 256) {
        const int r = i / span, q = i % span, yy = ya + r, xx = xa + q;
        const bool v = yy >= a.pad && yy < a.H - a.pad && xx >= a.pad && xx < a.W - a.pad;
        const int64_t o = (int64_t)yy * a.W + xx;
#pragma unroll
        for (int j = 0; j < 3; j++) s_m[j][i] = v ? a.abc[(j * a.C + c) * plane + o] : 0.0f;
      }
      __syncthreads();
      for (int i = threadIdx.x; i < span * kSsimTile; i += 256) {
        const int r = i / kSsimTile, q = i % kSsimTile;
        float h[3] = {0.0f, 0.0f, 0.0f};
        for (int k = 0; k < ws; k++) {
          const float g = s_g[k];
#pragma unroll
          for (int j = 0; j < 3; j++) h[j] += g * s_m[j][r * span + q + k];
        }
#pragma unroll
        for (int j = 0; j < 3; j++) s_h[j][i] = h[j];
      }
      __syncthreads();
      if (inside) {
        float b[3] = {0.0f, 0.0f, 0.0f};
        for (int k = 0; k < ws; k++) {
          const float g = s_g[k];
#pragma unroll
          for (int j = 0; j < 3; j++) b[j] += g * s_h[j][(ty + k) * kSsimTile + tx];
        }
        const int64_t e = ((int64_t)y * a.W + x) * a.C + c;
        const float p = a.pred[e], t = a.target[e];
        dS = b[0] + 2.0f * p * b[1] + t * b[2];
      }
    }
    if (!inside) continue;
    const int64_t e = ((int64_t)y * a.W + x) * a.C + c;
    const float p = a.pred[e], t = a.target[e];
    const float diff = p - t;
    l1 += (double)fabsf(diff);
    if (!a.grad) continue;
    const float l1d = (diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f)) / a.n_f;
    // FULL without a valid region: SSIM is the constant 0.
    const float sd = full ? -(dS / a.count_f) : (a.full ? 0.0f : 2.0f * diff / a.n_f);
    a.grad[e] = a.w_l1 * l1d + a.w_ssim * sd;
  }
  const double tsum = block_sum_d(l1, s_red);
  if (threadIdx.x == 0) a.l1_part[blockIdx.y * gridDim.x + blockIdx.x] = tsum;
}

// out[0] = w_l1 * L1 + w_ssim * (1 - SSIM), out[1] = L1 (mean |p - t|),
// out[2] = SSIM (mean over the valid terms, 0 when there are none).
__global__ void __launch_bounds__(256) loss_finalize_kernel(const double* ssim_part, int64_t ns,
                                                            const double* l1_part, int64_t nl, float n_f,
                                                            float count_f, float w_l1, float w_ssim,
                                                            float* out) {
  __shared__ double s_red[8];
  double s = 0.0, l = 0.0;
  for (int64_t i = threadIdx.x; i < ns; i += 256) s += ssim_part[i];
  for (int64_t i = threadIdx.x; i < nl; i += 256) l += l1_part[i];
  const double ts = block_sum_d(s, s_red);
  __syncthreads();
  const double tl = block_sum_d(l, s_red);
  if (threadIdx.x == 0) {
    const float ssim = count_f > 0.0f ? (float)(ts / (double)count_f) : 0.0f;
    const float l1v = n_f > 0.0f ? (float)(tl / (double)n_f) : 0.0f;
    out[0] = w_l1 * l1v + w_ssim * (1.0f - ssim);
    out[1] = l1v;
    out[2] = ssim;
  }
}

__global__ void __launch_bounds__(256) mse_kernel(const float* __restrict__ pred, const float* __restrict__ target,
                                                  int64_t numel, float denom, float* __restrict__ grad,
                                                  double* __restrict__ part) {
  __shared__ double s_red[8];
  double acc = 0.0;
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < numel; i += (int64_t)gridDim.x * 256) {
    const float diff = pred[i] - target[i];
    acc += (double)(diff * diff);
    if (grad) grad[i] = 2.0f * diff / denom;  // loss.cr:83-105
  }
  const double t = block_sum_d(acc, s_red);
  if (threadIdx.x == 0) part[blockIdx.x] = t;
}

}  // namespace gs

using namespace gs;

namespace {

int loss_common(gsc_ctx* ctx, const float* pred, const float* target, int32_t H, int32_t W, int32_t C,
                int32_t win, int32_t mode, float w_l1, float w_ssim, float* grad, float* ssim_map, float* out) {
  GS_REQUIRE(ctx && pred && target && out, "loss: null pointer");
  GS_REQUIRE(H > 0 && W > 0 && C >= 1 && C <= kSsimMaxC, "loss: image must be [H, W, C] with 1 <= C <= 4");
  GS_REQUIRE(win >= 1 && win <= kSsimMaxWin && (win & 1), "loss: window size must be odd and <= 15");
  GS_REQUIRE(mode == GSC_MODE_FULL || mode == GSC_MODE_REF, "loss: bad mode");
  SsimArgs a{};
  a.pred = pred; a.target = target;
  a.H = H; a.W = W; a.C = C; a.win = win; a.pad = win / 2;
  a.full = mode == GSC_MODE_FULL;
  a.map = ssim_map;
  a.grad = grad;
  a.w_l1 = w_l1; a.w_ssim = w_ssim;
  const int64_t numel = (int64_t)H * W * C;
  const int vw = W - 2 * a.pad, vh = H - 2 * a.pad;
  const bool any = vw > 0 && vh > 0;
  a.n_f = (float)numel;
  a.count_f = any ? (float)((int64_t)vw * vh * C) : 0.0f;
  const dim3 gv(any ? (vw + kSsimTile - 1) / kSsimTile : 0, any ? (vh + kSsimTile - 1) / kSsimTile : 0);
  const dim3 gi((W + kSsimTile - 1) / kSsimTile, (H + kSsimTile - 1) / kSsimTile);
  const int64_t nsp = (int64_t)gv.x * gv.y, nlp = (int64_t)gi.x * gi.y;
  const bool need_abc = a.full && grad && w_ssim != 0.0f && any;
  const size_t b_s = align256((size_t)std::max<int64_t>(nsp, 1) * 8), b_l = align256((size_t)nlp * 8);
  const size_t b_abc = need_abc ? align256((size_t)3 * numel * 4) : 0;
  int rc = scratch_reserve(ctx, b_s + b_l + b_abc);
  if (rc) return rc;
  a.ssim_part = reinterpret_cast<double*>(scratch_base(ctx));
  a.l1_part = reinterpret_cast<double*>(scratch_base(ctx) + b_s);
  a.abc = need_abc ? reinterpret_cast<float*>(scratch_base(ctx) + b_s + b_l) : nullptr;
  if (nsp > 0) {
    if (a.full)
      ssim_full_fwd_kernel<<<gv, 256, 0, ctx->stream>>>(a);
    else
      ssim_ref_kernel<<<gv, 256, 0, ctx->stream>>>(a);
    GS_CK_LAUNCH("ssim_fwd_kernel");
  }
  loss_grad_kernel<<<gi, 256, 0, ctx->stream>>>(a);
  GS_CK_LAUNCH("loss_grad_kernel");
  loss_finalize_kernel<<<1, 256, 0, ctx->stream>>>(a.ssim_part, nsp, a.l1_part, nlp, a.n_f, a.count_f, w_l1,
                                                   w_ssim, out);
  GS_CK_LAUNCH("loss_finalize_kernel");
  return GSC_OK;
}

}  // namespace

extern "C" {

GSC_API int gsc_ssim_loss_grad(gsc_ctx* ctx, const float* pred, const float* target, int32_t height,
                               int32_t width, int32_t channels, int32_t window_size, int32_t mode, float* grad,
                               float* ssim_map, float* out) {
  return loss_common(ctx, pred, target, height, width, channels, window_size, mode, 0.0f, 1.0f, grad, ssim_map,
                     out);
}

GSC_API int gsc_combined_loss_grad(gsc_ctx* ctx, const float* pred, const float* target, int32_t height,
                                   int32_t width, int32_t channels, float lambda_ssim, int32_t mode, float* grad,
                                   float* out) {
  return loss_common(ctx, pred, target, height, width, channels, 11, mode, 1.0f - lambda_ssim, lambda_ssim, grad,
                     nullptr, out);
}

GSC_API int gsc_mse_loss_grad(gsc_ctx* ctx, const float* pred, const float* target, int64_t numel, float* grad,
                              float* out) {
  GS_REQUIRE(ctx && pred && target && out && numel >= 0, "gsc_mse_loss_grad: bad argument");
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((int64_t)ctx->num_sms * 4, (numel + 255) / 256));
  int rc = scratch_reserve(ctx, align256((size_t)blocks * 8));
  if (rc) return rc;
  double* part = reinterpret_cast<double*>(scratch_base(ctx));
  mse_kernel<<<(unsigned)blocks, 256, 0, ctx->stream>>>(pred, target, numel, (float)numel, grad, part);
  GS_CK_LAUNCH("mse_kernel");
  loss_finalize_kernel<<<1, 256, 0, ctx->stream>>>(part, 0, part, blocks, (float)numel, 0.0f, 1.0f, 0.0f, out);
  GS_CK_LAUNCH("loss_finalize_kernel");
  return GSC_OK;
}

}  // extern "C"
