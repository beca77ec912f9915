// common.cuh — shared device helpers and the context layout of libgsplat_cuda.so.
//
// Floating-point contract (all kernels): built with --fmad=false,
// -prec-div=true, -prec-sqrt=true, -ftz=false, so every fp32 expression is
// evaluated as written with IEEE rounding; the only fused operations are
// explicit __fmaf_rn calls. The exponential is gs_expf below, not expf, so
// the results of preprocess, binning and forward compositing are a pure
// function of the documented operation order.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/gsplat_cuda.h"

#define GS_TILE 16
#define GS_TILE_PIXELS 256

// Device error word bits (gsc_ctx::err), read back by gsc_sync.
#define GS_DEVERR_TIMEOUT 1u
#define GS_DEVERR_BOUNDS 2u

namespace gs {

constexpr float kShC0 = 0.28209479177387814f;
constexpr float kShC1 = 0.4886025119029199f;

struct ShConsts {
  float c2[5];
  float c3[7];
};

// Spherical-harmonics constants, src/metal/kernels/gaussian.metal:11-28.
__device__ __forceinline__ ShConsts sh_consts() {
  ShConsts k = {{1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f,
                 -1.0925484305920792f, 0.5462742152960396f},
                {-0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
                 0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f,
                 -0.5900435899266435f}};
  return k;
}

// beta^step of Adam's bias correction as the reference evaluates it:
// `@beta1 ** state.step` (src/optim/adam.cr:129-130) is Float32#**(Int32),
// which Crystal lowers to LLVM's powi intrinsic; with a run-time exponent
// that is compiler-rt's __powisf2, binary exponentiation in fp32 (the
// result is multiplied by the running square for each set bit of the
// exponent, lowest bit first, and the square is updated after each bit).
inline float powi_f32(float a, int b) {
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

__device__ __forceinline__ float pow2i(int j) { return __int_as_float((j + 127) << 23); }

// exp(x) in fp32: Cody & Waite (1980) reduction x = k ln2 + r with ln 2
// split into a 16-bit head and a tail, e^r by its Taylor series to degree 7
// in Horner form with fused multiply-adds, then an exact scale by 2^k
// (two steps in the subnormal range). Max error about 1 ulp over the
// normal range; identical results on any IEEE target that runs the same
// operations.
__device__ __forceinline__ float gs_expf(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x < -103.97208404541015625f) return 0.0f;
  float k = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  float r = __fmaf_rn(-k, 0.693145751953125f, x);
  r = __fmaf_rn(-k, 1.428606765330187045e-06f, r);
  float p = 1.98412698412698412698e-4f;
  p = __fmaf_rn(p, r, 1.38888888888888888889e-3f);
  p = __fmaf_rn(p, r, 8.33333333333333333333e-3f);
  p = __fmaf_rn(p, r, 4.16666666666666666667e-2f);
  p = __fmaf_rn(p, r, 1.66666666666666666667e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int ki = (int)k;
  if (ki > 127) return p * pow2i(127) * pow2i(ki - 127);
  if (ki < -126) return p * pow2i(ki + 64) * pow2i(-64);
  return p * pow2i(ki);
}

// gs_expf for x in [-103.97, 0] (or NaN): the same operations without the
// range tests, so it returns exactly what gs_expf returns on that range.
__device__ __forceinline__ float gs_expf_nonpos(float x) {
  float k = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  float r = __fmaf_rn(-k, 0.693145751953125f, x);
  r = __fmaf_rn(-k, 1.428606765330187045e-06f, r);
  float p = 1.98412698412698412698e-4f;
  p = __fmaf_rn(p, r, 1.38888888888888888889e-3f);
  p = __fmaf_rn(p, r, 8.33333333333333333333e-3f);
  p = __fmaf_rn(p, r, 4.16666666666666666667e-2f);
  p = __fmaf_rn(p, r, 1.66666666666666666667e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ki = (int)k;
  if (ki < -126) return p * pow2i(ki + 64) * pow2i(-64);
  return p * pow2i(ki);
}

// gs_expf for x in [-87, 0]: the same operations without the range tests and
// without the subnormal step (2^k stays normal there), so it returns exactly
// what gs_expf returns on that range.
__device__ __forceinline__ float gs_expf_pixel(float x) {
  float k = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  float r = __fmaf_rn(-k, 0.693145751953125f, x);
  r = __fmaf_rn(-k, 1.428606765330187045e-06f, r);
  float p = 1.98412698412698412698e-4f;
  p = __fmaf_rn(p, r, 1.38888888888888888889e-3f);
  p = __fmaf_rn(p, r, 8.33333333333333333333e-3f);
  p = __fmaf_rn(p, r, 4.16666666666666666667e-2f);
  p = __fmaf_rn(p, r, 1.66666666666666666667e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  return p * pow2i((int)k);
}

__device__ __forceinline__ float gs_sigmoid(float x) { return 1.0f / (1.0f + gs_expf(-x)); }

// C `int(f)` (truncation toward zero) after saturating to +-1e9, so that
// out-of-range values are defined the same way on every target.
__device__ __forceinline__ int trunc_sat(float f) {
  f = fmaxf(f, -1.0e9f);
  f = fminf(f, 1.0e9f);
  return (int)f;
}

// Tile bounds of a splat, src/metal/kernels/gaussian.metal:338-341 with
// tiles_x = ceil(W/16), tiles_y = ceil(H/16).
__device__ __forceinline__ void tile_bounds(float px, float py, float r, int tiles_x, int tiles_y,
                                            int* x0, int* x1, int* y0, int* y1) {
  *x0 = max(0, trunc_sat(px - r) / GS_TILE);
  *x1 = min(tiles_x - 1, trunc_sat(px + r) / GS_TILE);
  *y0 = max(0, trunc_sat(py - r) / GS_TILE);
  *y1 = min(tiles_y - 1, trunc_sat(py + r) / GS_TILE);
}

}  // namespace gs

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

// A device allocation that grows on demand and never shrinks.
struct GsBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
};

struct gsc_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  int num_sms = 148;
  GsBuf scratch;              // per-call temporary storage (sort double buffer, ...)
  // depth-sliced binning bins two views at once, on `stream` and on `bin2`,
  // each with its own scratch (cur_scratch: the one of the stream in use)
  GsBuf scratch_alt;
  GsBuf* cur_scratch = nullptr;
  cudaStream_t bin2 = nullptr;
  cudaEvent_t bin2_ev[2] = {};
  GsBuf batch_pairs;          // batched forward: every view's packed depth words
  GsBuf batch_order;          // batched forward: every view's depth order
  // batched forward: compositing of view v on `side` overlaps the binning of
  // view v + 1 on `stream` (created on first use)
  cudaStream_t side = nullptr;
  cudaEvent_t side_ev[GSC_MAX_BATCH_VIEWS + 1] = {};
  // depth-sliced binning: per view, "slice binned" (stream -> side) and
  // "slice composited" (side -> stream)
  cudaEvent_t bin_ev[GSC_MAX_BATCH_VIEWS] = {};
  cudaEvent_t comp_ev[GSC_MAX_BATCH_VIEWS] = {};
  uint32_t* err = nullptr;    // device error word (+2: PGE, +4 / +6: binned / kept pairs, u64)
  void* pinned = nullptr;     // 4 KB pinned host staging for small readbacks
  // tracing
  bool profiling = false;
  int64_t kernels = 0;
  // pairs binned / kept in the final lists by whole-view forwards while
  // profiling: host-known counts here, device-known ones at err + 4 / err + 6
  uint64_t prof_binned = 0, prof_kept = 0;
  std::vector<cudaEvent_t> ev_pool;
  struct Mark { int stage; cudaEvent_t a, b; };
  std::vector<Mark> marks;
  int64_t calls[GSC_STAGE_COUNT] = {};
  int64_t stage_kernels[GSC_STAGE_COUNT] = {};
  double ms[GSC_STAGE_COUNT] = {};
};

namespace gs {
// Brackets one stage invocation with CUDA events (when profiling) and counts
// its kernel launches (always).
struct StageScope {
  gsc_ctx* ctx;
  int stage;
  cudaEvent_t a = nullptr;
  StageScope(gsc_ctx* c, int s);
  ~StageScope();
  void kernels(int k);
};
}  // namespace gs

namespace gs {

void set_error(const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);
int ensure(gsc_ctx* ctx, GsBuf* b, size_t bytes);
// Scratch carve-out: returns a 256-byte-aligned pointer inside ctx->scratch,
// growing it (which invalidates earlier carve-outs of the same call) first.
int scratch_reserve(gsc_ctx* ctx, size_t bytes);
inline char* scratch_base(gsc_ctx* ctx) {
  return (char*)(ctx->cur_scratch ? ctx->cur_scratch->ptr : ctx->scratch.ptr);
}
inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace gs

#define GS_CK(call)                                            \
  do {                                                         \
    cudaError_t _e = (call);                                   \
    if (_e != cudaSuccess) return gs::cuda_fail(_e, #call);    \
  } while (0)

#define GS_CK_LAUNCH(name)                                     \
  do {                                                         \
    cudaError_t _e = cudaGetLastError();                       \
    if (_e != cudaSuccess) return gs::cuda_fail(_e, name);     \
  } while (0)

#define GS_REQUIRE(cond, msg)                                  \
  do {                                                         \
    if (!(cond)) {                                             \
      gs::set_error(msg);                                      \
      return GSC_ERR_INVALID;                                  \
    }                                                          \
  } while (0)
