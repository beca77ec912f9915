// preprocess_bwd.cu — per-Gaussian backward from screen-space gradients to
// the 59 trainable floats, replacing the host loops project_backward!,
// sh_backward!, covariance_backward! (src/gaussian_splatting/rasterizer.cr:375-460)
// and the sigmoid chain of Trainer#apply_gradients! (trainer.cr:218-255).
//
// GSC_MODE_REF restates those loops literally (position through the mean
// only, DC SH gradient dL/dc / C0, nothing for scale and rotation).
// GSC_MODE_FULL is the analytic chain: conic -> cov2d -> (camera covariance,
// EWA Jacobian) -> 3-D covariance -> (log-scale, normalised quaternion), mean
// -> position, colour -> SH coefficients and position through the view
// direction, opacity -> logit. Gradients ACCUMULATE into the caller's buffers
// so several views can be summed before the optimiser step.
#include "geometry.cuh"
#include "kernels.cuh"

namespace gs {

// GSC_MODE_REF: the reference's host loops (rasterizer.cr:395-448, trainer.cr:234-241).
__global__ void __launch_bounds__(128) preprocess_bwd_ref_kernel(PreprocessBwdArgs a) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.n) return;
  const gsc_camera& cam = a.cam;
  const gsc_raster_config& cfg = a.cfg;
  const float* W = cam.view;
  const float fx = cam.fx, fy = cam.fy;
  float gv[9];
#pragma unroll
  for (int k = 0; k < 9; k++) gv[k] = a.grad2d[i * 9 + k];
  const float dmx = gv[0], dmy = gv[1], dop = gv[5];
  const float dcol[3] = {gv[6], gv[7], gv[8]};
  if (a.d_mean2d) { a.d_mean2d[i * 2] = dmx; a.d_mean2d[i * 2 + 1] = dmy; }
  if (a.d_opacity) a.d_opacity[i] = dop;
  if (a.d_colors) { a.d_colors[i * 3] = dcol[0]; a.d_colors[i * 3 + 1] = dcol[1]; a.d_colors[i * 3 + 2] = dcol[2]; }
  if (a.d_cov2d) { a.d_cov2d[i * 3] = 0.0f; a.d_cov2d[i * 3 + 1] = 0.0f; a.d_cov2d[i * 3 + 2] = 0.0f; }
  bool any = false;
#pragma unroll
  for (int k = 0; k < 9; k++) any = any || gv[k] != 0.0f;
  if (!any) return;
  const float p[3] = {a.pos[i * 3], a.pos[i * 3 + 1], a.pos[i * 3 + 2]};
  const float o = gs_sigmoid(a.logit_opacity[i]);
  a.g_logit_opacity[i] += dop * o * (1.0f - o);
    const float xc = W[0] * p[0] + W[1] * p[1] + W[2] * p[2] + W[3];
    const float yc = W[4] * p[0] + W[5] * p[1] + W[6] * p[2] + W[7];
    const float zc = W[8] * p[0] + W[9] * p[1] + W[10] * p[2] + W[11];
    if (!(zc <= cfg.near_z)) {
      const float z2 = zc * zc;
      const float dL_dcx = dmx * fx / zc;
      const float dL_dcy = dmy * fy / zc;
      const float dL_dcz = dmx * (-fx * xc / z2) + dmy * (-fy * yc / z2);
#pragma unroll
      for (int j = 0; j < 3; j++)
        a.g_pos[i * 3 + j] += dL_dcx * W[j] + dL_dcy * W[4 + j] + dL_dcz * W[8 + j];
    }
#pragma unroll
    for (int c = 0; c < 3; c++) a.g_sh[i * 48 + c] += dcol[c] / kShC0;
    }

// GSC_MODE_FULL. 128 Gaussians per block; the SH rows, then the SH-gradient
// rows, of the block are moved through shared memory with coalesced float4
// accesses (rows padded to 13 float4), so the 192-byte-strided per-Gaussian
// rows never hit DRAM as scattered requests.
constexpr int kPbThreads = 128;
constexpr int kRowF4 = 13;

__device__ __forceinline__ void stage_rows(float4* s4, const float* g, int64_t base, int cnt) {
  const float4* src = reinterpret_cast<const float4*>(g + base * 48);
  for (int k = threadIdx.x; k < cnt * 12; k += kPbThreads) s4[(k / 12) * kRowF4 + k % 12] = src[k];
}

__device__ __forceinline__ void unstage_rows(const float4* s4, float* g, int64_t base, int cnt) {
  float4* dst = reinterpret_cast<float4*>(g + base * 48);
  for (int k = threadIdx.x; k < cnt * 12; k += kPbThreads) dst[k] = s4[(k / 12) * kRowF4 + k % 12];
}

__global__ void __launch_bounds__(kPbThreads) preprocess_bwd_full_kernel(PreprocessBwdArgs a) {
  __shared__ float4 s4[kPbThreads * kRowF4];
  const int64_t base = (int64_t)blockIdx.x * kPbThreads;
  const int64_t i = base + threadIdx.x;
  const int cnt = (int)min((int64_t)kPbThreads, a.n - base);
  const bool valid = i < a.n;
  const gsc_camera& cam = a.cam;
  const gsc_raster_config& cfg = a.cfg;
  const float* W = cam.view;
  const float fx = cam.fx, fy = cam.fy;
  float gv[9];
#pragma unroll
  for (int k = 0; k < 9; k++) gv[k] = valid ? a.grad2d[i * 9 + k] : 0.0f;
  const float dmx = gv[0], dmy = gv[1], dA = gv[2], dB = gv[3], dC = gv[4], dop = gv[5];
  const float dcol[3] = {gv[6], gv[7], gv[8]};
  if (valid) {
    if (a.d_mean2d) { a.d_mean2d[i * 2] = dmx; a.d_mean2d[i * 2 + 1] = dmy; }
    if (a.d_opacity) a.d_opacity[i] = dop;
    if (a.d_colors) { a.d_colors[i * 3] = dcol[0]; a.d_colors[i * 3 + 1] = dcol[1]; a.d_colors[i * 3 + 2] = dcol[2]; }
    if (a.d_cov2d) { a.d_cov2d[i * 3] = 0.0f; a.d_cov2d[i * 3 + 1] = 0.0f; a.d_cov2d[i * 3 + 2] = 0.0f; }
  }
  bool any = false;
#pragma unroll
  for (int k = 0; k < 9; k++) any = any || gv[k] != 0.0f;
  // every term below is linear in grad2d: blocks without gradients are done
  if (!__syncthreads_or(any)) return;
  stage_rows(s4, a.sh, base, cnt);
  __syncthreads();

  float b[16];
  float w[3] = {0.0f, 0.0f, 0.0f};
  int ncoef = 0;
  if (any) {
    const float p[3] = {a.pos[i * 3], a.pos[i * 3 + 1], a.pos[i * 3 + 2]};
    const float o = gs_sigmoid(a.logit_opacity[i]);
    a.g_logit_opacity[i] += dop * o * (1.0f - o);
    const float s[3] = {gs_expf(a.log_scale[i * 3]), gs_expf(a.log_scale[i * 3 + 1]),
                        gs_expf(a.log_scale[i * 3 + 2])};
    const float4 q4 = reinterpret_cast<const float4*>(a.rot)[i];
    float q[4], qnorm;
    load_quat(q4, cfg.mode, q, &qnorm);
    float R[3][3];
    quat_to_R(q[0], q[1], q[2], q[3], R);
    float c3[6];
    cov3d_of(s, R, c3);
    Projected pr;
    project(p, c3, cam, cfg, &pr);
    any = pr.visible;
    if (any) {
      float dp[3] = {0.0f, 0.0f, 0.0f};
      // ---- colour -> view direction (SH rows from shared memory) ----
      {
        const float* row = reinterpret_cast<const float*>(s4 + threadIdx.x * kRowF4);
        float d[3], len;
        view_dir(p, cam, d, &len);
        sh_basis_hi(d[0], d[1], d[2], b);
        float raw[3];
        sh_eval([&](int k) { return row[k]; }, d[0], d[1], d[2], b, cfg.sh_degree, cfg.mode, raw);
        const float x = d[0], y = d[1], z = d[2];
        ncoef = (cfg.sh_degree + 1) * (cfg.sh_degree + 1);
        b[0] = kShC0;
        b[1] = kShC1 * -y; b[2] = kShC1 * z; b[3] = kShC1 * -x;
#pragma unroll
        for (int c = 0; c < 3; c++) w[c] = raw[c] + 0.5f > 0.0f ? dcol[c] : 0.0f;
        float DX[16], DY[16], DZ[16];
        sh_basis_derivs(x, y, z, DX, DY, DZ);
        float gx = 0.0f, gy = 0.0f, gz = 0.0f;
#pragma unroll
        for (int k = 1; k < 16; k++) {
          if (k >= ncoef) break;
          const float t = w[0] * row[k * 3] + w[1] * row[k * 3 + 1] + w[2] * row[k * 3 + 2];
          gx += t * DX[k];
          gy += t * DY[k];
          gz += t * DZ[k];
        }
        const float dd = x * gx + y * gy + z * gz;
        dp[0] -= (gx - x * dd) / len;
        dp[1] -= (gy - y * dd) / len;
        dp[2] -= (gz - z * dd) / len;
      }
      // ---- conic -> cov2d ----
      float da = 0.0f, db = 0.0f, dc2 = 0.0f;
      if (pr.det > 0.0f) {
        const float A = pr.A, B = pr.B, C = pr.Cc;
        const float P00 = A * A * dA + A * B * dB + B * B * dC;
        const float P01 = A * B * dA + (A * C + B * B) * (0.5f * dB) + B * C * dC;
        const float P11 = B * B * dA + B * C * dB + C * C * dC;
        da = -P00;
        db = -2.0f * P01;
        dc2 = -P11;
      }
      if (a.d_cov2d) { a.d_cov2d[i * 3] = da; a.d_cov2d[i * 3 + 1] = db; a.d_cov2d[i * 3 + 2] = dc2; }

      // ---- cov2d = J C J^T ----
      const float Jm[2][3] = {{pr.J00, 0.0f, pr.J02}, {0.0f, pr.J11, pr.J12}};
      const float Gc[2][2] = {{da, 0.5f * db}, {0.5f * db, dc2}};
      float GJ[2][3];
    #pragma unroll
      for (int r = 0; r < 2; r++)
    #pragma unroll
        for (int k = 0; k < 3; k++) GJ[r][k] = Gc[r][0] * Jm[0][k] + Gc[r][1] * Jm[1][k];
      float dCm[3][3];
    #pragma unroll
      for (int k = 0; k < 3; k++)
    #pragma unroll
        for (int l = 0; l < 3; l++) dCm[k][l] = Jm[0][k] * GJ[0][l] + Jm[1][k] * GJ[1][l];
      float dJ[2][3];
    #pragma unroll
      for (int r = 0; r < 2; r++)
    #pragma unroll
        for (int k = 0; k < 3; k++)
          dJ[r][k] = 2.0f * (GJ[r][0] * sym3(pr.C, 0, k) + GJ[r][1] * sym3(pr.C, 1, k) + GJ[r][2] * sym3(pr.C, 2, k));
      const float xc = pr.xc, yc = pr.yc, zc = pr.zc;
      const float z2 = zc * zc, z3 = z2 * zc;
      float dxc = dJ[0][2] * (-fx / z2);
      float dyc = dJ[1][2] * (-fy / z2);
      float dzc = dJ[0][0] * (-fx / z2) + dJ[0][2] * (2.0f * fx * xc / z3) + dJ[1][1] * (-fy / z2) +
                  dJ[1][2] * (2.0f * fy * yc / z3);
      dxc += dmx * fx / zc;
      dyc += dmy * fy / zc;
      dzc += -(dmx * fx * xc + dmy * fy * yc) / z2;
      const float V[3][3] = {{W[0], W[1], W[2]}, {W[4], W[5], W[6]}, {W[8], W[9], W[10]}};
    #pragma unroll
      for (int j = 0; j < 3; j++) dp[j] += V[0][j] * dxc + V[1][j] * dyc + V[2][j] * dzc;
    #pragma unroll
      for (int j = 0; j < 3; j++) a.g_pos[i * 3 + j] += dp[j];

      // ---- C = V Sigma V^T -> Sigma ----
      float VtD[3][3];
    #pragma unroll
      for (int r = 0; r < 3; r++)
    #pragma unroll
        for (int l = 0; l < 3; l++) VtD[r][l] = V[0][r] * dCm[0][l] + V[1][r] * dCm[1][l] + V[2][r] * dCm[2][l];
      float dS[3][3];
    #pragma unroll
      for (int r = 0; r < 3; r++)
    #pragma unroll
        for (int c = 0; c < 3; c++) dS[r][c] = VtD[r][0] * V[0][c] + VtD[r][1] * V[1][c] + VtD[r][2] * V[2][c];

      // ---- Sigma = M M^T, M = R diag(s) ----
      float M[3][3];
    #pragma unroll
      for (int r = 0; r < 3; r++)
    #pragma unroll
        for (int j = 0; j < 3; j++) M[r][j] = R[r][j] * s[j];
      float dM[3][3];
    #pragma unroll
      for (int r = 0; r < 3; r++)
    #pragma unroll
        for (int j = 0; j < 3; j++) dM[r][j] = 2.0f * (dS[r][0] * M[0][j] + dS[r][1] * M[1][j] + dS[r][2] * M[2][j]);
      float dR[3][3];
    #pragma unroll
      for (int j = 0; j < 3; j++) {
        const float ds = dM[0][j] * R[0][j] + dM[1][j] * R[1][j] + dM[2][j] * R[2][j];
        a.g_log_scale[i * 3 + j] += ds * s[j];
    #pragma unroll
        for (int r = 0; r < 3; r++) dR[r][j] = dM[r][j] * s[j];
      }

      // ---- R(q) -> q -> stored quaternion ----
      const float w = q[0], x = q[1], y = q[2], z = q[3];
      const float dqw = 2.0f * (-z * dR[0][1] + y * dR[0][2] + z * dR[1][0] - x * dR[1][2] - y * dR[2][0] + x * dR[2][1]);
      const float dqx = 2.0f * (y * dR[0][1] + z * dR[0][2] + y * dR[1][0] - 2.0f * x * dR[1][1] - w * dR[1][2] +
                                z * dR[2][0] + w * dR[2][1] - 2.0f * x * dR[2][2]);
      const float dqy = 2.0f * (-2.0f * y * dR[0][0] + x * dR[0][1] + w * dR[0][2] + x * dR[1][0] + z * dR[1][2] -
                                w * dR[2][0] + z * dR[2][1] - 2.0f * y * dR[2][2]);
      const float dqz = 2.0f * (-2.0f * z * dR[0][0] - w * dR[0][1] + x * dR[0][2] + w * dR[1][0] - 2.0f * z * dR[1][1] +
                                y * dR[1][2] + x * dR[2][0] + y * dR[2][1]);
      const float dot = w * dqw + x * dqx + y * dqy + z * dqz;
      if (qnorm > 0.0f) {
        a.g_rot[i * 4 + 0] += (dqw - w * dot) / qnorm;
        a.g_rot[i * 4 + 1] += (dqx - x * dot) / qnorm;
        a.g_rot[i * 4 + 2] += (dqy - y * dot) / qnorm;
        a.g_rot[i * 4 + 3] += (dqz - z * dot) / qnorm;
      }
    }
  }
  // ---- SH coefficients: read-modify-write of the block's gradient rows ----
  __syncthreads();
  stage_rows(s4, a.g_sh, base, cnt);
  __syncthreads();
  if (any) {
    float* row = reinterpret_cast<float*>(s4 + threadIdx.x * kRowF4);
#pragma unroll
    for (int c = 0; c < 3; c++) {
      if (w[c] == 0.0f) continue;
#pragma unroll
      for (int k = 0; k < 16; k++)
        if (k < ncoef) row[k * 3 + c] += b[k] * w[c];
    }
  }
  __syncthreads();
  unstage_rows(s4, a.g_sh, base, cnt);
}

int launch_preprocess_bwd(const PreprocessBwdArgs& a, bool full, cudaStream_t stream) {
  if (a.n == 0) return GSC_OK;
  const unsigned blocks = (unsigned)((a.n + 127) / 128);
  if (full) preprocess_bwd_full_kernel<<<blocks, kPbThreads, 0, stream>>>(a);
  else preprocess_bwd_ref_kernel<<<blocks, 128, 0, stream>>>(a);
  GS_CK_LAUNCH("preprocess_bwd_kernel");
  return GSC_OK;
}

}  // namespace gs
