// densify.cu — densification and pruning on the device, replacing the host
// loops of Trainer#densify_and_prune! / split_gaussians! /
// add_position_noise! (src/gaussian_splatting/trainer.cr:293-392),
// GradientAccumulator (trainer.cr:77-123) and Gaussian3D#clone_gaussians /
// concat! / remove! / reset_opacity! (gaussian.cr:150-271).
//
// The new set is built by one compaction: per 256-Gaussian block, the kept /
// cloned / split counts are scanned (three exclusive scans over the blocks),
// and every thread writes its Gaussian to up to three destinations:
//   [kept originals][clones][first split halves][second split halves],
// each group in original index order. Random offsets come from a
// counter-based hash (SplitMix64 finaliser) of (seed, index, draw), so the
// result is reproducible and identical in the CPU oracle; the reference uses
// an unseeded host RNG.
#include <cstring>

#include "common.cuh"
#include "kernels.cuh"

namespace gs {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Uniform in [0, 1) with 24 random bits.
__device__ __forceinline__ float hash_u01(uint64_t seed, uint64_t idx, uint32_t draw) {
  const uint64_t h = mix64(seed ^ mix64(idx * 8ull + draw));
  return (float)(h >> 40) * (1.0f / 16777216.0f);
}

__global__ void __launch_bounds__(256) grad_accumulate_kernel(const float* __restrict__ d, int stride, int64_t n,
                                                              float* __restrict__ accum, int32_t* __restrict__ count) {
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= n) return;
  const float gx = d[i * stride], gy = d[i * stride + 1];
  accum[i] += sqrtf(gx * gx + gy * gy);
  count[i] += 1;
}

__device__ __forceinline__ uint32_t densify_flags(const float* ls, float logit, float accum, int32_t count,
                                                  float grad_thr, float size_thr, float op_thr) {
  const float avg = count == 0 ? 0.0f : accum / (float)count;
  const float s0 = gs_expf(ls[0]), s1 = gs_expf(ls[1]), s2 = gs_expf(ls[2]);
  const float max_scale = fmaxf(s0, fmaxf(s1, s2));
  uint32_t f = 0;
  if (avg > grad_thr) f |= max_scale > size_thr ? GSC_DENSIFY_SPLIT : GSC_DENSIFY_CLONE;
  if (gs_sigmoid(logit) < op_thr) f |= GSC_DENSIFY_PRUNE;
  return f;
}

__global__ void __launch_bounds__(256) densify_plan_kernel(const float* __restrict__ log_scale,
                                                           const float* __restrict__ logit,
                                                           const float* __restrict__ accum,
                                                           const int32_t* __restrict__ count, int64_t n,
                                                           float grad_thr, float size_thr, float op_thr,
                                                           uint8_t* __restrict__ flags) {
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= n) return;
  flags[i] = (uint8_t)densify_flags(log_scale + i * 3, logit[i], accum[i], count[i], grad_thr, size_thr, op_thr);
}

__device__ __forceinline__ void categories(uint32_t f, bool* keep, bool* clone, bool* split) {
  *split = f & GSC_DENSIFY_SPLIT;
  *clone = f & GSC_DENSIFY_CLONE;
  *keep = !(*split) && !(f & GSC_DENSIFY_PRUNE);
}

// Per-block counts of kept / cloned / split Gaussians: bc[k * nb + b].
__global__ void __launch_bounds__(256) densify_count_kernel(const uint8_t* __restrict__ flags, int64_t n,
                                                            int64_t nb, uint32_t* __restrict__ bc) {
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  bool keep = false, clone = false, split = false;
  if (i < n) categories(flags[i], &keep, &clone, &split);
  const int k = __syncthreads_count(keep), c = __syncthreads_count(clone), s = __syncthreads_count(split);
  if (threadIdx.x == 0) {
    bc[blockIdx.x] = (uint32_t)k;
    bc[nb + blockIdx.x] = (uint32_t)c;
    bc[2 * nb + blockIdx.x] = (uint32_t)s;
  }
}

// Exclusive position of this thread's `pred` within its block.
__device__ __forceinline__ uint32_t block_rank(bool pred, uint32_t* s_w) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const uint32_t bal = __ballot_sync(0xffffffffu, pred);
  __syncthreads();
  if (lane == 0) s_w[w] = __popc(bal);
  __syncthreads();
  uint32_t base = 0;
  for (int k = 0; k < w; k++) base += s_w[k];
  return base + __popc(bal & ((1u << lane) - 1u));
}

struct DensifyApplyArgs {
  const float* pos;
  const float* ls;
  const float* rot;
  const float* logit;
  const float* sh;
  const uint8_t* flags;
  int64_t n, nb;
  const uint64_t* off;  // exclusive block offsets [3][nb]
  int64_t n_keep, n_clone, n_split;
  float* o_pos;
  float* o_ls;
  float* o_rot;
  float* o_logit;
  float* o_sh;
  float clone_noise, ln_split;
  uint64_t seed;
};

__device__ __forceinline__ void copy_row(const DensifyApplyArgs& a, int64_t i, int64_t d, const float p[3],
                                         const float l[3]) {
#pragma unroll
  for (int k = 0; k < 3; k++) {
    a.o_pos[d * 3 + k] = p[k];
    a.o_ls[d * 3 + k] = l[k];
  }
  reinterpret_cast<float4*>(a.o_rot)[d] = reinterpret_cast<const float4*>(a.rot)[i];
  a.o_logit[d] = a.logit[i];
  const float4* src = reinterpret_cast<const float4*>(a.sh + i * 48);
  float4* dst = reinterpret_cast<float4*>(a.o_sh + d * 48);
#pragma unroll
  for (int k = 0; k < 12; k++) dst[k] = src[k];
}

__global__ void __launch_bounds__(256) densify_apply_kernel(DensifyApplyArgs a) {
  __shared__ uint32_t s_w[8];
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  bool keep = false, clone = false, split = false;
  if (i < a.n) categories(a.flags[i], &keep, &clone, &split);
  const uint32_t rk = block_rank(keep, s_w);
  const uint32_t rc = block_rank(clone, s_w);
  const uint32_t rs = block_rank(split, s_w);
  if (i >= a.n) return;
  const float p[3] = {a.pos[i * 3], a.pos[i * 3 + 1], a.pos[i * 3 + 2]};
  const float l[3] = {a.ls[i * 3], a.ls[i * 3 + 1], a.ls[i * 3 + 2]};
  if (keep) copy_row(a, i, (int64_t)a.off[blockIdx.x] + rk, p, l);
  if (clone) {
    // add_position_noise!: (U - 0.5) * 2 * scale per axis (trainer.cr:375-386)
    float q[3];
#pragma unroll
    for (int k = 0; k < 3; k++) q[k] = p[k] + (hash_u01(a.seed, (uint64_t)i, k) - 0.5f) * 2.0f * a.clone_noise;
    copy_row(a, i, a.n_keep + (int64_t)a.off[a.nb + blockIdx.x] + rc, q, l);
  }
  if (split) {
    // split_gaussians!: log_scale -= ln 1.6; offset exp(new log_scale.x) * 0.5 * (+-1),
    // position += offset * (U - 0.5) per axis (trainer.cr:332-370)
    const float l2[3] = {l[0] - a.ln_split, l[1] - a.ln_split, l[2] - a.ln_split};
    const int64_t base = a.n_keep + a.n_clone + (int64_t)a.off[2 * a.nb + blockIdx.x] + rs;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const float offset = gs_expf(l2[0]) * 0.5f * (h == 0 ? 1.0f : -1.0f);
      float q[3];
#pragma unroll
      for (int k = 0; k < 3; k++) q[k] = p[k] + offset * (hash_u01(a.seed, (uint64_t)i, 3 + 3 * h + k) - 0.5f);
      copy_row(a, i, base + h * a.n_split, q, l2);
    }
  }
}

// Gaussian3D#remove! never empties the set (gaussian.cr:234-235): when every
// Gaussian would be pruned, nothing is.
__global__ void __launch_bounds__(256) clear_prune_kernel(uint8_t* __restrict__ flags, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i < n) flags[i] &= (uint8_t)~GSC_DENSIFY_PRUNE;
}

__global__ void __launch_bounds__(256) fill_kernel(float* __restrict__ x, int64_t n, float v) {
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i < n) x[i] = v;
}

}  // namespace gs

using namespace gs;

namespace {

// Block counts + three exclusive scans in ctx scratch; returns the totals on the host.
int densify_scan(gsc_ctx* ctx, const uint8_t* flags, int64_t n, uint64_t** off, int64_t totals[3]) {
  const int64_t nb = (n + 255) / 256;
  const size_t need = align256((size_t)nb * 3 * 4) + align256((size_t)nb * 3 * 8) + 256;
  int rc = scratch_reserve(ctx, need);
  if (rc) return rc;
  uint32_t* bc = reinterpret_cast<uint32_t*>(scratch_base(ctx));
  uint64_t* o = reinterpret_cast<uint64_t*>(scratch_base(ctx) + align256((size_t)nb * 3 * 4));
  uint64_t* tot = reinterpret_cast<uint64_t*>(scratch_base(ctx) + align256((size_t)nb * 3 * 4) +
                                              align256((size_t)nb * 3 * 8));
  densify_count_kernel<<<(unsigned)nb, 256, 0, ctx->stream>>>(flags, n, nb, bc);
  GS_CK_LAUNCH("densify_count_kernel");
  for (int k = 0; k < 3; k++) {
    rc = launch_scan_block_sums(bc + k * nb, nb, o + k * nb, tot + k, ctx->stream);
    if (rc) return rc;
  }
  GS_CK(cudaMemcpyAsync(ctx->pinned, tot, 24, cudaMemcpyDeviceToHost, ctx->stream));
  GS_CK(cudaStreamSynchronize(ctx->stream));
  uint64_t t[3];
  std::memcpy(t, ctx->pinned, 24);
  for (int k = 0; k < 3; k++) totals[k] = (int64_t)t[k];
  *off = o;
  return GSC_OK;
}

}  // namespace

extern "C" {

GSC_API int gsc_grad_accumulate(gsc_ctx* ctx, const float* dmean2d, int32_t stride, int64_t n, float* accum,
                                int32_t* count) {
  GS_REQUIRE(ctx && n >= 0 && stride >= 2, "gsc_grad_accumulate: bad argument");
  if (n == 0) return GSC_OK;
  GS_REQUIRE(dmean2d && accum && count, "gsc_grad_accumulate: null pointer");
  grad_accumulate_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(dmean2d, stride, n, accum, count);
  GS_CK_LAUNCH("grad_accumulate_kernel");
  return GSC_OK;
}

GSC_API int gsc_densify_plan(gsc_ctx* ctx, const gsc_gaussians* g, const float* accum, const int32_t* count,
                             float grad_threshold, float size_threshold, float opacity_threshold, uint8_t* flags,
                             int64_t* counts) {
  GS_REQUIRE(ctx && g && counts, "gsc_densify_plan: null argument");
  GS_REQUIRE(g->count >= 0 && g->count < (1ll << 31), "gsc_densify_plan: bad count");
  counts[0] = counts[1] = counts[2] = 0;
  const int64_t n = g->count;
  if (n == 0) return GSC_OK;
  GS_REQUIRE(g->log_scale && g->logit_opacity && accum && count && flags, "gsc_densify_plan: null pointer");
  densify_plan_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(
      g->log_scale, g->logit_opacity, accum, count, n, grad_threshold, size_threshold, opacity_threshold, flags);
  GS_CK_LAUNCH("densify_plan_kernel");
  uint64_t* off = nullptr;
  int rc = densify_scan(ctx, flags, n, &off, counts);
  if (rc || counts[0] + counts[1] + counts[2] > 0) return rc;
  clear_prune_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(flags, n);
  GS_CK_LAUNCH("clear_prune_kernel");
  counts[0] = n;
  return GSC_OK;
}

GSC_API int gsc_densify_apply(gsc_ctx* ctx, const gsc_gaussians* g, const uint8_t* flags,
                              const gsc_gaussians_out* out, float clone_noise, float ln_split, uint64_t seed) {
  GS_REQUIRE(ctx && g && out, "gsc_densify_apply: null argument");
  GS_REQUIRE(g->count >= 0 && g->count < (1ll << 31), "gsc_densify_apply: bad count");
  const int64_t n = g->count;
  if (n == 0) return GSC_OK;
  GS_REQUIRE(g->position && g->log_scale && g->rotation && g->logit_opacity && g->sh && flags,
             "gsc_densify_apply: null input pointer");
  GS_REQUIRE(out->position && out->log_scale && out->rotation && out->logit_opacity && out->sh,
             "gsc_densify_apply: null output pointer");
  GS_REQUIRE(((uintptr_t)g->rotation & 15u) == 0 && ((uintptr_t)g->sh & 15u) == 0 &&
                 ((uintptr_t)out->rotation & 15u) == 0 && ((uintptr_t)out->sh & 15u) == 0,
             "gsc_densify_apply: rotation and sh must be 16-byte aligned");
  uint64_t* off = nullptr;
  int64_t totals[3];
  int rc = densify_scan(ctx, flags, n, &off, totals);
  if (rc) return rc;
  DensifyApplyArgs a;
  std::memset(&a, 0, sizeof a);
  a.pos = g->position; a.ls = g->log_scale; a.rot = g->rotation; a.logit = g->logit_opacity; a.sh = g->sh;
  a.flags = flags;
  a.n = n;
  a.nb = (n + 255) / 256;
  a.off = off;
  a.n_keep = totals[0]; a.n_clone = totals[1]; a.n_split = totals[2];
  a.o_pos = out->position; a.o_ls = out->log_scale; a.o_rot = out->rotation; a.o_logit = out->logit_opacity;
  a.o_sh = out->sh;
  a.clone_noise = clone_noise;
  a.ln_split = ln_split;
  a.seed = seed;
  densify_apply_kernel<<<(unsigned)a.nb, 256, 0, ctx->stream>>>(a);
  GS_CK_LAUNCH("densify_apply_kernel");
  return GSC_OK;
}

GSC_API int gsc_reset_opacity(gsc_ctx* ctx, float* logit_opacity, int64_t n, float value) {
  GS_REQUIRE(ctx && n >= 0 && (n == 0 || logit_opacity), "gsc_reset_opacity: bad argument");
  if (n == 0) return GSC_OK;
  fill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(logit_opacity, n, value);
  GS_CK_LAUNCH("fill_kernel");
  return GSC_OK;
}

}  // extern "C"
