// optim.cu — fused Adam over every parameter group in one launch
// (Adam#step / update_adam! / apply_weight_decay!, src/optim/adam.cr:86-176,
// which copies each tensor to the host and loops serially), and the L1 loss
// gradient (Loss.l1_with_grad, src/ops/loss.cr:33-57).
//
// Adam: each thread owns 4 consecutive floats of one group (float4 loads and
// stores when the group's pointers are 16-byte aligned and the chunk is
// whole). HBM traffic: 16 B read (p, g, m, v) + 12 B written per float.
#include "common.cuh"
#include "kernels.cuh"

namespace gs {

__device__ __forceinline__ void adam_one(float& p, float gr, float& m, float& v, const AdamArgs& a,
                                         const AdamGroupDev& G) {
  if (G.weight_decay > 0.0f) p = p * G.decay;
  gr = gr * a.grad_scale;
  m = a.beta1 * m + (1.0f - a.beta1) * gr;
  v = a.beta2 * v + (1.0f - a.beta2) * gr * gr;
  const float mh = m / a.bc1;
  const float vh = v / a.bc2;
  p = p - G.lr * mh / (sqrtf(vh) + a.eps);
}

__global__ void __launch_bounds__(256) adam_kernel(AdamArgs a) {
  const int64_t chunk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (chunk >= a.chunk_end[a.ngroups - 1]) return;
  int gi = 0;
  while (chunk >= a.chunk_end[gi]) gi++;
  const AdamGroupDev& G = a.g[gi];
  const int64_t first = (chunk - (gi ? a.chunk_end[gi - 1] : 0)) * 4;
  const int64_t cnt = min((int64_t)4, G.numel - first);
  if (G.vec && cnt == 4) {
    float4 p = *reinterpret_cast<float4*>(G.param + first);
    const float4 g = *reinterpret_cast<const float4*>(G.grad + first);
    float4 m = *reinterpret_cast<float4*>(G.m + first);
    float4 v = *reinterpret_cast<float4*>(G.v + first);
    adam_one(p.x, g.x, m.x, v.x, a, G);
    adam_one(p.y, g.y, m.y, v.y, a, G);
    adam_one(p.z, g.z, m.z, v.z, a, G);
    adam_one(p.w, g.w, m.w, v.w, a, G);
    *reinterpret_cast<float4*>(G.param + first) = p;
    *reinterpret_cast<float4*>(G.m + first) = m;
    *reinterpret_cast<float4*>(G.v + first) = v;
  } else {
    for (int64_t k = first; k < first + cnt; k++) {
      float p = G.param[k], m = G.m[k], v = G.v[k];
      adam_one(p, G.grad[k], m, v, a, G);
      G.param[k] = p;
      G.m[k] = m;
      G.v[k] = v;
    }
  }
}

int launch_adam(const AdamArgs& a, cudaStream_t stream) {
  const int64_t chunks = a.chunk_end[a.ngroups - 1];
  if (chunks == 0) return GSC_OK;
  adam_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, stream>>>(a);
  GS_CK_LAUNCH("adam_kernel");
  return GSC_OK;
}

__global__ void __launch_bounds__(256) l1_kernel(const float* __restrict__ pred, const float* __restrict__ target,
                                                 int64_t numel, float scale, float* __restrict__ grad,
                                                 float* loss_sum) {
  __shared__ float s_w[8];
  float loss = 0.0f;
  for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < numel; i += (int64_t)gridDim.x * 256) {
    const float diff = pred[i] - target[i];
    loss += fabsf(diff) * scale;
    grad[i] = (diff > 0.0f ? 1.0f : (diff < 0.0f ? -1.0f : 0.0f)) * scale;
  }
  if (!loss_sum) return;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) loss += __shfl_xor_sync(0xffffffffu, loss, off);
  if ((threadIdx.x & 31) == 0) s_w[threadIdx.x >> 5] = loss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int w = 0; w < 8; w++) t += s_w[w];
    atomicAdd(loss_sum, t);
  }
}

int launch_l1(const float* pred, const float* target, int64_t numel, float scale, float* grad,
              float* loss_sum, int num_sms, cudaStream_t stream) {
  if (numel == 0) return GSC_OK;
  const int64_t blocks = min((int64_t)num_sms * 8, (numel + 255) / 256);
  l1_kernel<<<(unsigned)blocks, 256, 0, stream>>>(pred, target, numel, scale, grad, loss_sum);
  GS_CK_LAUNCH("l1_kernel");
  return GSC_OK;
}

}  // namespace gs
