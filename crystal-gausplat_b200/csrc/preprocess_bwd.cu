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
#include <algorithm>

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

// The FULL chain of Gaussian i over the views whose bit is set in view_mask
// (their grad2d rows); `row` is its SH row, `grow` its SH-gradient row (in
// shared or global memory), every other gradient goes to global memory.
__device__ __forceinline__ void pbwd_full_gaussian(const PreprocessBwdArgs& a, int64_t i, const float* row,
                                                   float* grow, uint32_t view_mask) {
  const gsc_raster_config& cfg = a.cfg;
  const int nv = a.nviews;
    const float p[3] = {a.pos[i * 3], a.pos[i * 3 + 1], a.pos[i * 3 + 2]};
    const float o = gs_sigmoid(a.logit_opacity[i]);
    const float s[3] = {gs_expf(a.log_scale[i * 3]), gs_expf(a.log_scale[i * 3 + 1]),
                        gs_expf(a.log_scale[i * 3 + 2])};
    const float4 q4 = reinterpret_cast<const float4*>(a.rot)[i];
    float q[4], qnorm;
    load_quat(q4, cfg.mode, q, &qnorm);
    float R[3][3];
    quat_to_R(q[0], q[1], q[2], q[3], R);
    float c3[6];
    cov3d_of(s, R, c3);
    const int ncoef = (cfg.sh_degree + 1) * (cfg.sh_degree + 1);
    float dop = 0.0f;
    float dp[3] = {0.0f, 0.0f, 0.0f};
    float dS[3][3] = {{0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f}};
    bool visible_any = false;
    for (int v = 0; v < nv; v++) {
      if (!((view_mask >> v) & 1u)) continue;
      const float* gv = a.grad2d_v[v] + i * 9;
      const float dmx = gv[0], dmy = gv[1], dA = gv[2], dB = gv[3], dC = gv[4];
      const float dcol[3] = {gv[6], gv[7], gv[8]};
      dop += gv[5];
      const gsc_camera& cam = a.cams[v];
      const float* W = cam.view;
      const float fx = cam.fx, fy = cam.fy;
      Projected pr;
      project(p, c3, cam, cfg, &pr);
      if (!pr.visible) continue;
      visible_any = true;
      float vdp[3] = {0.0f, 0.0f, 0.0f};
      // ---- colour -> view direction and SH coefficients ----
      {
        float b[16];
        float d[3], len;
        view_dir(p, cam, d, &len);
        sh_basis_hi(d[0], d[1], d[2], b);
        float raw[3];
        sh_eval([&](int k) { return row[k]; }, d[0], d[1], d[2], b, cfg.sh_degree, cfg.mode, raw);
        const float x = d[0], y = d[1], z = d[2];
        b[0] = kShC0;
        b[1] = kShC1 * -y; b[2] = kShC1 * z; b[3] = kShC1 * -x;
        float w[3];
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
        vdp[0] -= (gx - x * dd) / len;
        vdp[1] -= (gy - y * dd) / len;
        vdp[2] -= (gz - z * dd) / len;
#pragma unroll
        for (int c = 0; c < 3; c++) {
          if (w[c] == 0.0f) continue;
#pragma unroll
          for (int k = 0; k < 16; k++)
            if (k < ncoef) grow[k * 3 + c] += b[k] * w[c];
        }
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
      if (a.d_cov2d && nv == 1) { a.d_cov2d[i * 3] = da; a.d_cov2d[i * 3 + 1] = db; a.d_cov2d[i * 3 + 2] = dc2; }

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
      for (int j = 0; j < 3; j++) dp[j] += vdp[j] + (V[0][j] * dxc + V[1][j] * dyc + V[2][j] * dzc);

      // ---- C = V Sigma V^T -> Sigma ----
      float VtD[3][3];
#pragma unroll
      for (int r = 0; r < 3; r++)
#pragma unroll
        for (int l = 0; l < 3; l++) VtD[r][l] = V[0][r] * dCm[0][l] + V[1][r] * dCm[1][l] + V[2][r] * dCm[2][l];
#pragma unroll
      for (int r = 0; r < 3; r++)
#pragma unroll
        for (int c = 0; c < 3; c++) dS[r][c] += VtD[r][0] * V[0][c] + VtD[r][1] * V[1][c] + VtD[r][2] * V[2][c];
    }
    a.g_logit_opacity[i] += dop * o * (1.0f - o);
    if (visible_any) {
#pragma unroll
      for (int j = 0; j < 3; j++) a.g_pos[i * 3 + j] += dp[j];
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

// One Gaussian per thread, `nviews` views (camera + grad2d each) per launch.
// The camera-independent terms (scales, rotation, 3-D covariance) are formed
// once; per view the position gradient and the symmetric covariance gradient
// dSigma are summed (the scale and rotation gradients are linear in dSigma),
// the SH gradient goes straight into the staged gradient row, and every
// gradient row is read and written once per launch. Dynamic shared memory:
// the SH rows and the SH-gradient rows of the block.
// 4 CTAs per SM (its shared memory allows no more): at most 128 registers.
// Reading the SH rows from global memory instead of staging them (half the
// shared memory) measured slower at 4 and 5 CTAs per SM (0.297 / 0.295 vs
// 0.279 ms per view), and at 6 CTAs the registers spill.
__global__ void __launch_bounds__(kPbThreads, 4) preprocess_bwd_full_kernel(PreprocessBwdArgs a) {
  extern __shared__ float4 s_dyn[];
  float4* s_par = s_dyn;                         // SH rows
  float4* s_grd = s_dyn + kPbThreads * kRowF4;   // SH-gradient rows
  const int64_t base = (int64_t)blockIdx.x * kPbThreads;
  const int64_t i = base + threadIdx.x;
  const int cnt = (int)min((int64_t)kPbThreads, a.n - base);
  const bool valid = i < a.n;
  const int nv = a.nviews;
  bool any = false;
  for (int v = 0; v < nv; v++) {
    if (!valid) break;
    const float* gv = a.grad2d_v[v] + i * 9;
#pragma unroll
    for (int k = 0; k < 9; k++) any = any || gv[k] != 0.0f;
  }
  if (valid && nv == 1) {  // screen-space views of a single-view call
    const float* gv = a.grad2d_v[0] + i * 9;
    if (a.d_mean2d) { a.d_mean2d[i * 2] = gv[0]; a.d_mean2d[i * 2 + 1] = gv[1]; }
    if (a.d_opacity) a.d_opacity[i] = gv[5];
    if (a.d_colors) { a.d_colors[i * 3] = gv[6]; a.d_colors[i * 3 + 1] = gv[7]; a.d_colors[i * 3 + 2] = gv[8]; }
    if (a.d_cov2d) { a.d_cov2d[i * 3] = 0.0f; a.d_cov2d[i * 3 + 1] = 0.0f; a.d_cov2d[i * 3 + 2] = 0.0f; }
  }
  // every term below is linear in grad2d: blocks without gradients are done
  if (!__syncthreads_or(any)) return;
  stage_rows(s_par, a.sh, base, cnt);
  stage_rows(s_grd, a.g_sh, base, cnt);
  __syncthreads();

  if (any) {
    const float* row = reinterpret_cast<const float*>(s_par + threadIdx.x * kRowF4);
    float* grow = reinterpret_cast<float*>(s_grd + threadIdx.x * kRowF4);
    pbwd_full_gaussian(a, i, row, grow, 0xFFFFFFFFu);
  }
  __syncthreads();
  unstage_rows(s_grd, a.g_sh, base, cnt);
}

// Batched backward over the active Gaussians only. A few per cent of the
// Gaussians of a view receive a screen-space gradient (the rest are culled
// or occluded), so one thread per Gaussian left most lanes of a warp idle
// through each view's chain. pbwd_active_kernel lists every Gaussian with a
// nonzero grad2d row in some view (id, mask of those views) in any order;
// pbwd_compact_kernel runs the chain of the listed Gaussians over their
// masked views, reading the SH and SH-gradient rows in place. Each Gaussian's
// arithmetic is that of preprocess_bwd_full_kernel (a view whose grad2d row is
// zero adds only zeros there).
__global__ void __launch_bounds__(256) pbwd_active_kernel(PreprocessBwdArgs a, uint2* __restrict__ list,
                                                          uint32_t* __restrict__ count) {
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  uint32_t mask = 0;
  if (i < a.n) {
    for (int v = 0; v < a.nviews; v++) {
      const float* gv = a.grad2d_v[v] + i * 9;
      bool nz = false;
#pragma unroll
      for (int k = 0; k < 9; k++) nz = nz || gv[k] != 0.0f;
      mask |= (uint32_t)nz << v;
    }
  }
  const uint32_t bal = __ballot_sync(0xffffffffu, mask != 0u);
  if (!bal) return;
  const int lane = threadIdx.x & 31;
  uint32_t base = 0;
  if (lane == 0) base = atomicAdd(count, (uint32_t)__popc(bal));
  base = __shfl_sync(0xffffffffu, base, 0);
  if (mask) list[base + __popc(bal & ((1u << lane) - 1u))] = make_uint2((uint32_t)i, mask);
}

__global__ void __launch_bounds__(kPbThreads, 4) pbwd_compact_kernel(PreprocessBwdArgs a,
                                                                     const uint2* __restrict__ list,
                                                                     const uint32_t* __restrict__ count) {
  const uint32_t cnt = *count;
  for (uint32_t t = blockIdx.x * kPbThreads + threadIdx.x; t < cnt; t += gridDim.x * kPbThreads) {
    const uint2 e = list[t];
    const int64_t i = e.x;
    pbwd_full_gaussian(a, i, a.sh + i * 48, a.g_sh + i * 48, e.y);
  }
}

int launch_preprocess_bwd_compact(const PreprocessBwdArgs& a, char* scratch, int num_sms, cudaStream_t stream) {
  if (a.n == 0) return GSC_OK;
  if (a.n >= (1ll << 32) || a.nviews < 1 || a.nviews > kMaxBatchViews) {
    set_error("preprocess_bwd_compact: bad size");
    return GSC_ERR_INVALID;
  }
  uint32_t* count = reinterpret_cast<uint32_t*>(scratch);
  uint2* list = reinterpret_cast<uint2*>(scratch + 256);
  GS_CK(cudaMemsetAsync(count, 0, 4, stream));
  pbwd_active_kernel<<<(unsigned)((a.n + 255) / 256), 256, 0, stream>>>(a, list, count);
  GS_CK_LAUNCH("pbwd_active_kernel");
  const int64_t grid = std::min<int64_t>((a.n + kPbThreads - 1) / kPbThreads, (int64_t)num_sms * 8);
  pbwd_compact_kernel<<<(unsigned)grid, kPbThreads, 0, stream>>>(a, list, count);
  GS_CK_LAUNCH("pbwd_compact_kernel");
  return GSC_OK;
}

size_t preprocess_bwd_compact_scratch(int64_t n) { return 256 + (size_t)n * 8; }

constexpr size_t kPbSmem = 2 * (size_t)kPbThreads * kRowF4 * sizeof(float4);

int launch_preprocess_bwd(const PreprocessBwdArgs& a, bool full, cudaStream_t stream) {
  if (a.n == 0) return GSC_OK;
  const unsigned blocks = (unsigned)((a.n + 127) / 128);
  if (full) {
    static bool attr_set[64] = {};
    int dev = 0;
    GS_CK(cudaGetDevice(&dev));
    if (dev < 64 && !attr_set[dev]) {
      GS_CK(cudaFuncSetAttribute(preprocess_bwd_full_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kPbSmem));
      attr_set[dev] = true;
    }
    preprocess_bwd_full_kernel<<<blocks, kPbThreads, kPbSmem, stream>>>(a);
  }
  else preprocess_bwd_ref_kernel<<<blocks, 128, 0, stream>>>(a);
  GS_CK_LAUNCH("preprocess_bwd_kernel");
  return GSC_OK;
}

}  // namespace gs
