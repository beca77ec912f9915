// dp.cu — fused gradient exchange + Adam for view-sharded data parallelism.
//
// Rank r owns the float4 chunks [C r / P, C (r + 1) / P) of the concatenated
// parameter groups. Per chunk: the P gradient chunks are loaded from the P
// ranks' arenas over NVLink (peer pointers) and summed in rank order, Adam
// (Adam#step, src/optim/adam.cr:127-176) updates the shard's parameters and
// this rank's moments, and the new parameter chunk is stored into every
// rank's parameter arena. Per rank this moves the shard's gradients in once
// from each peer and its parameters out once to each peer -- the bytes of a
// reduce-scatter plus an all-gather -- with the optimiser arithmetic done once
// per element instead of on every replica.
//
// With NVLink multicast addresses of the two arenas (an NVSwitch multicast
// object bound to every rank's arena) the same kernel sums a gradient chunk
// with one multimem.ld_reduce (the switch reads the ranks' copies and adds
// them) and writes the new parameter chunk with one multimem.st (the switch
// writes it into every replica): per NVLink direction a rank then moves
// (1 + 1/P) arenas instead of 2 (P - 1)/P.
#include <cmath>
#include <cstring>

#include "common.cuh"
#include "kernels.cuh"

namespace gs {

struct DpBarrierDev {
  int nranks, rank;
  uint32_t* flags[GSC_DP_MAX_RANKS];
  uint32_t epoch;
  uint64_t timeout_ns;
};

struct DpArgsDev {
  int nranks, rank;
  float* peer_grads[GSC_DP_MAX_RANKS];
  float* peer_params[GSC_DP_MAX_RANKS];
  float* m;
  float* v;
  int ngroups;
  int64_t offset[8];
  int64_t numel[8];
  int64_t chunk_end[8];  // inclusive prefix of ceil(numel / 4)
  float lr[8], weight_decay[8], decay[8];
  float beta1, beta2, eps, bc1, bc2, grad_scale;
  int64_t chunk_lo, chunk_hi;  // this rank's shard
  const uint32_t* err;         // the context's error word: skip all work after a failed barrier
  float* mc_grads;             // multicast addresses (both or neither)
  float* mc_params;
};

// Sum over every rank's copy, added by the NVSwitch (fp32).
__device__ __forceinline__ float4 mc_sum4(const float* addr) {
  float4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(addr) : "memory");
  return r;
}
__device__ __forceinline__ float mc_sum1(const float* addr) {
  float r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(r) : "l"(addr) : "memory");
  return r;
}
// One store that lands in every rank's copy.
__device__ __forceinline__ void mc_store4(float* addr, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};"
               ::"l"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}
__device__ __forceinline__ void mc_store1(float* addr, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ float dp_adam(float p, float g, float& m, float& v, const DpArgsDev& a, int gi) {
  if (a.weight_decay[gi] > 0.0f) p = p * a.decay[gi];
  g = g * a.grad_scale;
  m = a.beta1 * m + (1.0f - a.beta1) * g;
  v = a.beta2 * v + (1.0f - a.beta2) * g * g;
  const float mh = m / a.bc1;
  const float vh = v / a.bc2;
  return p - a.lr[gi] * mh / (sqrtf(vh) + a.eps);
}

template <bool MC>
__global__ void __launch_bounds__(256) dp_adam_kernel(DpArgsDev a) {
  const int64_t chunk = a.chunk_lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (chunk >= a.chunk_hi) return;
  // a cross-rank barrier before this launch gave up: the peers' gradients
  // may be incomplete, so touch no peer memory (the host reads the error)
  if (*(volatile const uint32_t*)a.err & GS_DEVERR_TIMEOUT) return;
  int gi = 0;
  while (chunk >= a.chunk_end[gi]) gi++;
  const int64_t first = (chunk - (gi ? a.chunk_end[gi - 1] : 0)) * 4;
  const int64_t cnt = min((int64_t)4, a.numel[gi] - first);
  const int64_t off = a.offset[gi] + first;  // float index in every arena
  if (cnt == 4) {
    float4 g;
    if (MC) {
      g = mc_sum4(a.mc_grads + off);
    } else {
      g = *reinterpret_cast<const float4*>(a.peer_grads[0] + off);
      for (int p = 1; p < a.nranks; p++) {
        const float4 h = *reinterpret_cast<const float4*>(a.peer_grads[p] + off);
        g.x += h.x; g.y += h.y; g.z += h.z; g.w += h.w;
      }
    }
    float4 pr = *reinterpret_cast<const float4*>(a.peer_params[a.rank] + off);  // local replica
    float4 m = *reinterpret_cast<float4*>(a.m + off);
    float4 v = *reinterpret_cast<float4*>(a.v + off);
    pr.x = dp_adam(pr.x, g.x, m.x, v.x, a, gi);
    pr.y = dp_adam(pr.y, g.y, m.y, v.y, a, gi);
    pr.z = dp_adam(pr.z, g.z, m.z, v.z, a, gi);
    pr.w = dp_adam(pr.w, g.w, m.w, v.w, a, gi);
    *reinterpret_cast<float4*>(a.m + off) = m;
    *reinterpret_cast<float4*>(a.v + off) = v;
    if (MC) mc_store4(a.mc_params + off, pr);
    else
      for (int p = 0; p < a.nranks; p++) *reinterpret_cast<float4*>(a.peer_params[p] + off) = pr;
  } else {
    for (int64_t k = 0; k < cnt; k++) {
      float g;
      if (MC) {
        g = mc_sum1(a.mc_grads + off + k);
      } else {
        g = a.peer_grads[0][off + k];
        for (int p = 1; p < a.nranks; p++) g += a.peer_grads[p][off + k];
      }
      float m = a.m[off + k], v = a.v[off + k];
      const float pr = dp_adam(a.peer_params[a.rank][off + k], g, m, v, a, gi);
      a.m[off + k] = m;
      a.v[off + k] = v;
      if (MC) mc_store1(a.mc_params + off + k, pr);
      else
        for (int p = 0; p < a.nranks; p++) a.peer_params[p][off + k] = pr;
    }
  }
}

// Cross-rank barrier over peer-addressable flag arrays: rank r stores
// `epoch` into slot r of every peer's array (release, system scope, after a
// system fence so that this rank's earlier writes -- its gradients, or the
// parameter shards it stored into the peers -- are visible first), then waits
// until every peer's slot of its own array has reached `epoch` (acquire). The
// wait is bounded by timeout_ns of the GPU's global timer; on expiry the
// kernel sets GS_DEVERR_TIMEOUT in the context's error word and returns.
__global__ void dp_barrier_kernel(DpBarrierDev b, uint32_t* err) {
  const int p = threadIdx.x;
  if (p >= b.nranks || p == b.rank) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(b.flags[p] + b.rank), "r"(b.epoch) : "memory");
  const uint32_t* mine = b.flags[b.rank] + p;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if ((int32_t)(v - b.epoch) >= 0) return;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > b.timeout_ns) {
      atomicOr(err, GS_DEVERR_TIMEOUT);
      return;
    }
    __nanosleep(256);
  }
}

}  // namespace gs

using namespace gs;

extern "C" GSC_API int gsc_dp_barrier(gsc_ctx* ctx, const gsc_dp_barrier_args* in) {
  GS_REQUIRE(ctx && in, "gsc_dp_barrier: null argument");
  GS_REQUIRE(in->nranks >= 1 && in->nranks <= GSC_DP_MAX_RANKS && in->rank >= 0 && in->rank < in->nranks,
             "gsc_dp_barrier: bad nranks/rank");
  GS_REQUIRE(in->timeout_us >= 1 && in->timeout_us <= 600000000, "gsc_dp_barrier: timeout_us must be 1 us .. 600 s");
  if (in->nranks == 1) return GSC_OK;
  DpBarrierDev b;
  std::memset(&b, 0, sizeof b);
  b.nranks = in->nranks;
  b.rank = in->rank;
  for (int p = 0; p < in->nranks; p++) {
    GS_REQUIRE(in->peer_flags[p] && ((uintptr_t)in->peer_flags[p] & 3u) == 0,
               "gsc_dp_barrier: null or misaligned flag array");
    b.flags[p] = in->peer_flags[p];
  }
  b.epoch = in->epoch;
  b.timeout_ns = (uint64_t)in->timeout_us * 1000ull;
  StageScope sc(ctx, GSC_STAGE_ADAM);  // part of the exchange + optimiser step
  sc.kernels(1);
  dp_barrier_kernel<<<1, 32, 0, ctx->stream>>>(b, ctx->err);
  GS_CK_LAUNCH("dp_barrier_kernel");
  return GSC_OK;
}

extern "C" GSC_API int gsc_dp_adam_step(gsc_ctx* ctx, const gsc_dp_adam_args* in) {
  GS_REQUIRE(ctx && in, "gsc_dp_adam_step: null argument");
  GS_REQUIRE(in->nranks >= 1 && in->nranks <= GSC_DP_MAX_RANKS && in->rank >= 0 && in->rank < in->nranks,
             "gsc_dp_adam_step: bad nranks/rank");
  GS_REQUIRE(in->ngroups >= 1 && in->ngroups <= 8, "gsc_dp_adam_step: 1..8 groups");
  GS_REQUIRE(in->step >= 1, "gsc_dp_adam_step: step must be >= 1");
  GS_REQUIRE(in->m && in->v, "gsc_dp_adam_step: null moments");
  DpArgsDev a;
  std::memset(&a, 0, sizeof a);
  a.nranks = in->nranks;
  a.rank = in->rank;
  for (int p = 0; p < in->nranks; p++) {
    GS_REQUIRE(in->peer_grads[p] && in->peer_params[p], "gsc_dp_adam_step: null peer pointer");
    GS_REQUIRE(((uintptr_t)in->peer_grads[p] & 15u) == 0 && ((uintptr_t)in->peer_params[p] & 15u) == 0,
               "gsc_dp_adam_step: arenas must be 16-byte aligned");
    a.peer_grads[p] = in->peer_grads[p];
    a.peer_params[p] = in->peer_params[p];
  }
  GS_REQUIRE(((uintptr_t)in->m & 15u) == 0 && ((uintptr_t)in->v & 15u) == 0,
             "gsc_dp_adam_step: moments must be 16-byte aligned");
  a.m = in->m;
  a.v = in->v;
  GS_REQUIRE(!in->mc_grads == !in->mc_params, "gsc_dp_adam_step: give both multicast addresses or neither");
  GS_REQUIRE(((uintptr_t)in->mc_grads & 15u) == 0 && ((uintptr_t)in->mc_params & 15u) == 0,
             "gsc_dp_adam_step: multicast addresses must be 16-byte aligned");
  a.mc_grads = in->mc_grads;
  a.mc_params = in->mc_params;
  a.ngroups = in->ngroups;
  int64_t run = 0;
  for (int i = 0; i < in->ngroups; i++) {
    GS_REQUIRE(in->offset[i] >= 0 && in->offset[i] % 4 == 0 && in->numel[i] >= 0,
               "gsc_dp_adam_step: group offsets must be non-negative multiples of 4");
    a.offset[i] = in->offset[i];
    a.numel[i] = in->numel[i];
    a.lr[i] = in->lr[i];
    a.weight_decay[i] = in->weight_decay[i];
    a.decay[i] = 1.0f - in->lr[i] * in->weight_decay[i];
    run += (in->numel[i] + 3) / 4;
    a.chunk_end[i] = run;
  }
  a.beta1 = in->beta1; a.beta2 = in->beta2; a.eps = in->eps; a.grad_scale = in->grad_scale;
  a.bc1 = 1.0f - powi_f32(in->beta1, in->step);  // fp32, as adam.cr:129-130
  a.bc2 = 1.0f - powi_f32(in->beta2, in->step);
  a.chunk_lo = run * in->rank / in->nranks;
  a.chunk_hi = run * (in->rank + 1) / in->nranks;
  a.err = ctx->err;
  const int64_t n = a.chunk_hi - a.chunk_lo;
  if (n <= 0) return GSC_OK;
  StageScope sc(ctx, GSC_STAGE_ADAM);
  sc.kernels(1);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (a.mc_grads) dp_adam_kernel<true><<<blocks, 256, 0, ctx->stream>>>(a);
  else dp_adam_kernel<false><<<blocks, 256, 0, ctx->stream>>>(a);
  GS_CK_LAUNCH("dp_adam_kernel");
  return GSC_OK;
}
