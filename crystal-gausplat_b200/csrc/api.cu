// api.cu — the extern "C" boundary of libgsplat_cuda.so (include/gsplat_cuda.h):
// context, memory, stage entry points, and whole-view orchestration mirroring
// Rasterizer.forward / Rasterizer.backward (src/gaussian_splatting/rasterizer.cr:48-104).
#include <cmath>
#include <cstring>
#include <string>

#include "common.cuh"
#include "kernels.cuh"

namespace gs {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int cuda_fail(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  if (e == cudaErrorMemoryAllocation) return GSC_ERR_NOMEM;
  return GSC_ERR_CUDA;
}

int ensure(gsc_ctx* ctx, GsBuf* b, size_t bytes) {
  if (bytes <= b->bytes && b->ptr) return GSC_OK;
  if (b->ptr) {
    // The old buffer may still be read by queued work on this stream.
    GS_CK(cudaStreamSynchronize(ctx->stream));
    GS_CK(cudaFree(b->ptr));
    b->ptr = nullptr;
    b->bytes = 0;
  }
  size_t want = bytes + bytes / 4 + 256;
  cudaError_t e = cudaMalloc(&b->ptr, want);
  if (e != cudaSuccess) {
    cudaGetLastError();
    b->ptr = nullptr;
    e = cudaMalloc(&b->ptr, bytes ? bytes : 256);
    if (e != cudaSuccess) {
      b->ptr = nullptr;
      return cuda_fail(e, "cudaMalloc");
    }
    want = bytes ? bytes : 256;
  }
  b->bytes = want;
  return GSC_OK;
}

int scratch_reserve(gsc_ctx* ctx, size_t bytes) {
  return ensure(ctx, ctx->cur_scratch ? ctx->cur_scratch : &ctx->scratch, bytes);
}

static float power_cut_of(float alpha_min) {
  if (!(alpha_min > 0.0f)) return -INFINITY;
  return (float)(std::log((double)alpha_min) - 1e-3);
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

static int read_u64(gsc_ctx* ctx, const uint64_t* dptr, uint64_t* out) {
  GS_CK(cudaMemcpyAsync(ctx->pinned, dptr, 8, cudaMemcpyDeviceToHost, ctx->stream));
  GS_CK(cudaStreamSynchronize(ctx->stream));
  std::memcpy(out, ctx->pinned, 8);
  return GSC_OK;
}

static int tile_bits_of(int num_tiles) {
  int b = 0;
  while ((1ll << b) < (long long)num_tiles) b++;
  return b;
}

}  // namespace gs

using namespace gs;

struct gsc_frame {
  gsc_ctx* ctx = nullptr;
  GsBuf splats, depth_pairs, depth_keys, order, pairs, block_sums, offsets, total, tiles, keys, vals, ranges, image, final_T,
      last, n_contrib, grad2d, bins, tile_order, tile_work;
  // depth-sliced binning (GSC_BIN_OCCLUDED)
  GsBuf slice_vals[kMaxSlices], slice_ranges[kMaxSlices], skip_bits, tile_done, tile_base, pair_total;
  // per-tile depth cut of the slices (gsc_frame_set_tile_hint): the caller's
  // array of tiles floats, read when valid, rewritten by every occluded forward
  float* tile_hint = nullptr;
  int64_t tile_hint_count = 0;
  bool tile_hint_valid = false;
  GsBuf cut_sub, cut_cnt, open_flag;
  bool count_pending = false;  // the lists' length is on the device (the final ranges' end)
  bool keys_valid = false;  // `keys` rebuilt from (tiles, vals) on request
  int64_t n = 0, num_keys = 0;
  int width = 0, height = 0, tiles_x = 0, tiles_y = 0;
  float* image_ptr = nullptr;  // image the last forward wrote (caller's or frame's)
  const uint32_t* order_ptr = nullptr;  // depth order of the last forward (own buffer or a batch's)
  bool has_forward = false;
  bool has_grad2d = false;  // a backward left grad2d for this forward
};

extern "C" {

GSC_API int gsc_version(void) { return GSC_VERSION; }

GSC_API const char* gsc_last_error(void) { return g_last_error.c_str(); }

GSC_API void gsc_raster_config_default(gsc_raster_config* cfg) {
  if (!cfg) return;
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

GSC_API int gsc_init(int device, gsc_ctx** out) {
  GS_REQUIRE(out, "gsc_init: out is null");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    cudaGetLastError();
    set_error("gsc_init: no CUDA device");
    return GSC_ERR_NODEVICE;
  }
  if (device < 0 || device >= count) {
    set_error("gsc_init: device index out of range");
    return GSC_ERR_NODEVICE;
  }
  GS_CK(cudaSetDevice(device));
  gsc_ctx* ctx = new gsc_ctx();
  ctx->device = device;
  cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
  e = cudaMalloc(&ctx->err, 64);
  if (e == cudaSuccess) e = cudaMemset(ctx->err, 0, 64);
  if (e == cudaSuccess) e = cudaMallocHost(&ctx->pinned, 4096);
  if (e != cudaSuccess) {
    int rc = cuda_fail(e, "gsc_init");
    if (ctx->err) cudaFree(ctx->err);
    delete ctx;
    return rc;
  }
  *out = ctx;
  return GSC_OK;
}

GSC_API int gsc_destroy(gsc_ctx* ctx) {
  if (!ctx) return GSC_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->scratch.ptr) cudaFree(ctx->scratch.ptr);
  if (ctx->scratch_alt.ptr) cudaFree(ctx->scratch_alt.ptr);
  if (ctx->bin2) {
    cudaStreamSynchronize(ctx->bin2);
    for (auto& e : ctx->bin2_ev)
      if (e) cudaEventDestroy(e);
    cudaStreamDestroy(ctx->bin2);
  }
  if (ctx->batch_pairs.ptr) cudaFree(ctx->batch_pairs.ptr);
  if (ctx->batch_order.ptr) cudaFree(ctx->batch_order.ptr);
  if (ctx->side) {
    cudaStreamSynchronize(ctx->side);
    for (auto& e : ctx->side_ev)
      if (e) cudaEventDestroy(e);
    cudaStreamDestroy(ctx->side);
  }
  if (ctx->err) cudaFree(ctx->err);
  if (ctx->pinned) cudaFreeHost(ctx->pinned);
  delete ctx;
  return GSC_OK;
}

GSC_API int gsc_set_stream(gsc_ctx* ctx, void* stream) {
  GS_REQUIRE(ctx, "gsc_set_stream: null context");
  ctx->stream = (cudaStream_t)stream;
  return GSC_OK;
}

GSC_API int gsc_sync(gsc_ctx* ctx) {
  GS_REQUIRE(ctx, "gsc_sync: null context");
  GS_CK(cudaStreamSynchronize(ctx->stream));
  GS_CK(cudaMemcpyAsync(ctx->pinned, ctx->err, 4, cudaMemcpyDeviceToHost, ctx->stream));
  GS_CK(cudaStreamSynchronize(ctx->stream));
  uint32_t flags;
  std::memcpy(&flags, ctx->pinned, 4);
  if (flags) {
    GS_CK(cudaMemsetAsync(ctx->err, 0, 4, ctx->stream));
    GS_CK(cudaStreamSynchronize(ctx->stream));
    if (flags & GS_DEVERR_TIMEOUT) {
      set_error("a bounded device-side wait gave up (look-back timeout)");
      return GSC_ERR_TIMEOUT;
    }
    set_error("a device-side bounds check failed");
    return GSC_ERR_CUDA;
  }
  return GSC_OK;
}

GSC_API int gsc_selftest_wait_timeout(gsc_ctx* ctx, int32_t spin_limit) {
  GS_REQUIRE(ctx, "gsc_selftest_wait_timeout: null context");
  GS_REQUIRE(spin_limit >= 1 && spin_limit <= 100000, "gsc_selftest_wait_timeout: spin_limit must be 1..100000");
  const int rc = scratch_reserve(ctx, 2 * 256 * 4);
  if (rc != GSC_OK) return rc;
  return launch_lookback_selftest(ctx, (uint32_t)spin_limit, scratch_base(ctx));
}

GSC_API int gsc_alloc(gsc_ctx* ctx, size_t bytes, void** out) {
  GS_REQUIRE(ctx && out, "gsc_alloc: null argument");
  *out = nullptr;
  cudaError_t e = cudaMalloc(out, bytes ? bytes : 1);
  if (e != cudaSuccess) {
    *out = nullptr;
    return cuda_fail(e, "gsc_alloc");
  }
  return GSC_OK;
}

GSC_API int gsc_free(gsc_ctx* ctx, void* ptr) {
  GS_REQUIRE(ctx, "gsc_free: null context");
  if (ptr) GS_CK(cudaFree(ptr));
  return GSC_OK;
}

GSC_API int gsc_memcpy_h2d(gsc_ctx* ctx, void* dst, const void* src, size_t bytes) {
  GS_REQUIRE(ctx && (bytes == 0 || (dst && src)), "gsc_memcpy_h2d: null argument");
  GS_CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  GS_CK(cudaStreamSynchronize(ctx->stream));
  return GSC_OK;
}

GSC_API int gsc_memcpy_d2h(gsc_ctx* ctx, void* dst, const void* src, size_t bytes) {
  GS_REQUIRE(ctx && (bytes == 0 || (dst && src)), "gsc_memcpy_d2h: null argument");
  GS_CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  GS_CK(cudaStreamSynchronize(ctx->stream));
  return GSC_OK;
}

GSC_API int gsc_memset(gsc_ctx* ctx, void* dst, int value, size_t bytes) {
  GS_REQUIRE(ctx && (bytes == 0 || dst), "gsc_memset: null argument");
  GS_CK(cudaMemsetAsync(dst, value, bytes, ctx->stream));
  return GSC_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Stages
// ---------------------------------------------------------------------------
namespace gs {

static int check_gaussians(const gsc_gaussians* g) {
  GS_REQUIRE(g, "null gaussians");
  GS_REQUIRE(g->count >= 0 && g->count < (1ll << 31), "gaussian count out of range [0, 2^31)");
  if (g->count == 0) return GSC_OK;
  GS_REQUIRE(g->position && g->log_scale && g->rotation && g->logit_opacity && g->sh,
             "null gaussian parameter pointer");
  GS_REQUIRE(aligned16(g->rotation) && aligned16(g->sh), "rotation and sh must be 16-byte aligned");
  return GSC_OK;
}

static int check_view(const gsc_camera* cam, const gsc_raster_config* cfg) {
  GS_REQUIRE(cam && cfg, "null camera or config");
  GS_REQUIRE(cam->width > 0 && cam->height > 0 && cam->width <= 65536 && cam->height <= 65536,
             "camera width/height out of range");
  GS_REQUIRE(cfg->mode == GSC_MODE_FULL || cfg->mode == GSC_MODE_REF, "unknown mode");
  GS_REQUIRE(cfg->sh_degree >= 0 && cfg->sh_degree <= 3, "sh_degree must be 0..3");
  GS_REQUIRE(cfg->binning == GSC_BIN_REFERENCE || cfg->binning == GSC_BIN_CONTRIBUTING ||
                 cfg->binning == GSC_BIN_OCCLUDED,
             "unknown binning");
  return GSC_OK;
}

static int do_preprocess(gsc_ctx* ctx, const gsc_gaussians* g, const gsc_camera* cam,
                         const gsc_raster_config* cfg, const gsc_projected* o, uint32_t* block_sums,
                         uint64_t* depth_pairs = nullptr) {
  PreprocessArgs a;
  std::memset(&a, 0, sizeof a);
  a.n = g->count;
  a.pos = g->position; a.log_scale = g->log_scale; a.rot = g->rotation;
  a.logit_opacity = g->logit_opacity; a.sh = g->sh;
  a.cfg = *cfg;
  a.tiles_x = (cam->width + GS_TILE - 1) / GS_TILE;
  a.tiles_y = (cam->height + GS_TILE - 1) / GS_TILE;
  a.nviews = 1;
  a.cams[0] = *cam;
  a.splats_v[0] = o->splats;
  (void)block_sums;
  a.depth_pairs_v[0] = depth_pairs;
  a.mean2d = o->mean2d; a.cov2d = o->cov2d; a.conic = o->conic; a.depth = o->depth;
  a.radius = o->radius; a.colors = o->colors; a.opacity = o->opacity;
  a.tiles_touched = o->tiles_touched; a.cov3d = o->cov3d;
  StageScope sc(ctx, GSC_STAGE_PREPROCESS);
  sc.kernels(g->count ? 1 : 0);
  return launch_preprocess(a, ctx->stream);
}

// Scan the per-block tile counts into offsets and read the total back.
static int do_scan(gsc_ctx* ctx, int64_t n, const uint32_t* sums, uint64_t* offsets, uint64_t* total,
                   uint64_t* host_total) {
  *host_total = 0;
  if (n == 0) return GSC_OK;
  int rc;
  {
    StageScope sc(ctx, GSC_STAGE_SCAN);
    sc.kernels(1);
    rc = launch_scan_block_sums(sums, (n + 255) / 256, offsets, total, ctx->stream);
  }
  if (rc) return rc;
  return read_u64(ctx, total, host_total);
}

static void fill_fwd(CompositeFwdArgs* a, const float* splats, const uint32_t* vals, const uint32_t* ranges,
                     int W, int H, const gsc_raster_config* cfg) {
  std::memset(a, 0, sizeof *a);
  a->splats = splats; a->vals = vals; a->ranges = ranges;
  a->width = W; a->height = H;
  a->tiles_x = (W + GS_TILE - 1) / GS_TILE; a->tiles_y = (H + GS_TILE - 1) / GS_TILE;
  a->t_stop = cfg->t_stop; a->alpha_min = cfg->alpha_min; a->alpha_max = cfg->alpha_max;
  a->power_cut = power_cut_of(cfg->alpha_min);
  for (int c = 0; c < 3; c++) a->bg[c] = cfg->background[c];
}

static void fill_bwd(CompositeBwdArgs* a, const float* splats, const uint32_t* vals, const uint32_t* ranges,
                     int W, int H, const gsc_raster_config* cfg) {
  std::memset(a, 0, sizeof *a);
  a->splats = splats; a->vals = vals; a->ranges = ranges;
  a->width = W; a->height = H;
  a->tiles_x = (W + GS_TILE - 1) / GS_TILE; a->tiles_y = (H + GS_TILE - 1) / GS_TILE;
  a->alpha_min = cfg->alpha_min; a->alpha_max = cfg->alpha_max;
  a->power_cut = power_cut_of(cfg->alpha_min);
  for (int c = 0; c < 3; c++) a->bg[c] = cfg->background[c];
}

static int do_preprocess_bwd(gsc_ctx* ctx, const gsc_gaussians* g, const gsc_camera* cam,
                             const gsc_raster_config* cfg, const float* grad2d,
                             const gsc_gaussian_grads* gr, const gsc_grads2d* g2d) {
  PreprocessBwdArgs a;
  std::memset(&a, 0, sizeof a);
  a.n = g->count;
  a.pos = g->position; a.log_scale = g->log_scale; a.rot = g->rotation;
  a.logit_opacity = g->logit_opacity; a.sh = g->sh;
  a.cam = *cam; a.cfg = *cfg;
  a.grad2d = grad2d;
  a.nviews = 1;
  a.cams[0] = *cam;
  a.grad2d_v[0] = grad2d;
  a.g_pos = gr->position; a.g_log_scale = gr->log_scale; a.g_rot = gr->rotation;
  a.g_logit_opacity = gr->logit_opacity; a.g_sh = gr->sh;
  if (g2d) {
    a.d_mean2d = g2d->mean2d; a.d_cov2d = g2d->cov2d; a.d_opacity = g2d->opacity; a.d_colors = g2d->colors;
  }
  StageScope sc(ctx, GSC_STAGE_PREPROCESS_BWD);
  sc.kernels(g->count ? 1 : 0);
  return launch_preprocess_bwd(a, cfg->mode == GSC_MODE_FULL, ctx->stream);
}

static int check_grads(const gsc_gaussian_grads* gr) {
  GS_REQUIRE(gr && gr->position && gr->log_scale && gr->rotation && gr->logit_opacity && gr->sh,
             "null gradient pointer");
  return GSC_OK;
}

}  // namespace gs

#define GS_TRY(expr)          \
  do {                        \
    int _rc = (expr);         \
    if (_rc != GSC_OK) return _rc; \
  } while (0)

extern "C" {

GSC_API int gsc_preprocess(gsc_ctx* ctx, const gsc_gaussians* g, const gsc_camera* cam,
                           const gsc_raster_config* cfg, const gsc_projected* out) {
  GS_REQUIRE(ctx && out, "gsc_preprocess: null argument");
  GS_TRY(check_gaussians(g));
  GS_TRY(check_view(cam, cfg));
  GS_REQUIRE(g->count == 0 || (out->splats && aligned16(out->splats)),
             "gsc_preprocess: splats must be non-null and 16-byte aligned");
  return do_preprocess(ctx, g, cam, cfg, out, nullptr);
}

GSC_API int gsc_bin(gsc_ctx* ctx, int64_t n, const float* splats, int32_t tiles_x, int32_t tiles_y,
                    uint64_t* keys, uint32_t* values, int64_t capacity, int64_t* num_keys) {
  GS_REQUIRE(ctx && num_keys, "gsc_bin: null argument");
  GS_REQUIRE(n >= 0 && n < (1ll << 31), "gsc_bin: n out of range");
  GS_REQUIRE(tiles_x > 0 && tiles_y > 0, "gsc_bin: bad tile grid");
  *num_keys = 0;
  if (n == 0) return GSC_OK;
  GS_REQUIRE(splats && aligned16(splats), "gsc_bin: splats must be non-null and 16-byte aligned");
  const int64_t nb = (n + 255) / 256;
  GS_TRY(scratch_reserve(ctx, align256(nb * 4) + align256(nb * 8) + 256));
  uint32_t* sums = (uint32_t*)scratch_base(ctx);
  uint64_t* offsets = (uint64_t*)(scratch_base(ctx) + align256(nb * 4));
  uint64_t* total = (uint64_t*)(scratch_base(ctx) + align256(nb * 4) + align256(nb * 8));
  {
    StageScope sc(ctx, GSC_STAGE_SCAN);
    sc.kernels(1);
    GS_TRY(launch_block_sums(splats, n, sums, ctx->stream));
  }
  uint64_t m = 0;
  GS_TRY(do_scan(ctx, n, sums, offsets, total, &m));
  *num_keys = (int64_t)m;
  if ((int64_t)m > capacity) {
    set_error("gsc_bin: key count " + std::to_string(m) + " exceeds capacity " + std::to_string(capacity));
    return GSC_ERR_CAPACITY;
  }
  if (m == 0) return GSC_OK;
  GS_REQUIRE(keys && values, "gsc_bin: null keys/values");
  StageScope sc(ctx, GSC_STAGE_EMIT);
  sc.kernels(1);
  return launch_emit_keys(splats, n, offsets, tiles_x, tiles_y, keys, values, ctx->stream);
}

GSC_API int gsc_sort_pairs_u64(gsc_ctx* ctx, uint64_t* keys, uint32_t* values, int64_t n,
                               int begin_bit, int end_bit) {
  GS_REQUIRE(ctx, "gsc_sort_pairs_u64: null context");
  GS_REQUIRE(n >= 0 && n < (1ll << 30), "gsc_sort_pairs_u64: n must be in [0, 2^30)");
  GS_REQUIRE(begin_bit >= 0 && end_bit <= 64 && begin_bit <= end_bit, "gsc_sort_pairs_u64: bad bit range");
  if (n <= 1 || begin_bit == end_bit) return GSC_OK;
  GS_REQUIRE(keys && values, "gsc_sort_pairs_u64: null keys/values");
  GS_TRY(scratch_reserve(ctx, sort_scratch_bytes(n, begin_bit, end_bit)));
  StageScope sc(ctx, GSC_STAGE_SORT);
  sc.kernels(1 + (end_bit - begin_bit + 7) / 8);
  return launch_sort_pairs(ctx, keys, values, n, begin_bit, end_bit, scratch_base(ctx));
}

GSC_API int gsc_tile_ranges(gsc_ctx* ctx, const uint64_t* sorted_keys, int64_t n, int32_t num_tiles,
                            uint32_t* ranges) {
  GS_REQUIRE(ctx && ranges && num_tiles > 0, "gsc_tile_ranges: bad argument");
  GS_REQUIRE(n >= 0 && (n == 0 || sorted_keys), "gsc_tile_ranges: bad keys");
  StageScope sc(ctx, GSC_STAGE_RANGES);
  sc.kernels(n ? 1 : 0);
  return launch_tile_ranges(sorted_keys, n, num_tiles, ranges, ctx->stream);
}

GSC_API int gsc_composite_forward(gsc_ctx* ctx, const float* splats, const uint32_t* values,
                                  const uint32_t* ranges, int32_t width, int32_t height,
                                  const gsc_raster_config* cfg, float* image, uint32_t* n_contrib,
                                  float* final_T, uint32_t* last) {
  GS_REQUIRE(ctx && cfg && ranges && image && width > 0 && height > 0, "gsc_composite_forward: bad argument");
  GS_REQUIRE(!splats || aligned16(splats), "gsc_composite_forward: splats must be 16-byte aligned");
  CompositeFwdArgs a;
  fill_fwd(&a, splats, values, ranges, width, height, cfg);
  a.image = image; a.n_contrib = n_contrib; a.final_T = final_T; a.last = last;
  StageScope sc(ctx, GSC_STAGE_COMPOSITE_FWD);
  sc.kernels(1);
  return launch_composite_fwd(a, ctx->stream);
}

GSC_API int gsc_composite_backward(gsc_ctx* ctx, const float* splats, const uint32_t* values,
                                   const uint32_t* ranges, int32_t width, int32_t height,
                                   const gsc_raster_config* cfg, const float* dL_dimage,
                                   const float* image, const float* target, float l1_scale,
                                   const float* final_T, const uint32_t* last, float* grad2d,
                                   float* loss_sum) {
  GS_REQUIRE(ctx && cfg && ranges && final_T && grad2d && width > 0 && height > 0,
             "gsc_composite_backward: bad argument");
  GS_REQUIRE(target ? (image != nullptr) : (dL_dimage != nullptr),
             "gsc_composite_backward: need dL_dimage, or image and target");
  GS_REQUIRE(cfg->mode != GSC_MODE_FULL || last, "gsc_composite_backward: FULL mode needs `last`");
  CompositeBwdArgs a;
  fill_bwd(&a, splats, values, ranges, width, height, cfg);
  a.dL_dimage = dL_dimage; a.image = image; a.target = target; a.l1_scale = l1_scale;
  a.final_T = final_T; a.last = last; a.grad2d = grad2d; a.loss_sum = loss_sum;
  StageScope sc(ctx, GSC_STAGE_COMPOSITE_BWD);
  sc.kernels(1);
  return launch_composite_bwd(a, cfg->mode == GSC_MODE_FULL, ctx->stream);
}

GSC_API int gsc_preprocess_backward(gsc_ctx* ctx, const gsc_gaussians* g, const gsc_camera* cam,
                                    const gsc_raster_config* cfg, const float* grad2d,
                                    const gsc_gaussian_grads* grads, const gsc_grads2d* g2d) {
  GS_REQUIRE(ctx, "gsc_preprocess_backward: null context");
  GS_TRY(check_gaussians(g));
  GS_TRY(check_view(cam, cfg));
  GS_TRY(check_grads(grads));
  GS_REQUIRE(g->count == 0 || grad2d, "gsc_preprocess_backward: null grad2d");
  return do_preprocess_bwd(ctx, g, cam, cfg, grad2d, grads, g2d);
}

GSC_API int gsc_l1_loss_grad(gsc_ctx* ctx, const float* pred, const float* target, int64_t numel,
                             float scale, float* grad, float* loss_sum) {
  GS_REQUIRE(ctx && numel >= 0 && (numel == 0 || (pred && target && grad)), "gsc_l1_loss_grad: bad argument");
  StageScope sc(ctx, GSC_STAGE_L1);
  sc.kernels(numel ? 1 : 0);
  return launch_l1(pred, target, numel, scale, grad, loss_sum, ctx->num_sms, ctx->stream);
}

GSC_API int gsc_adam_step(gsc_ctx* ctx, const gsc_adam_group* groups, int32_t ngroups, float beta1,
                          float beta2, float eps, int32_t step, float grad_scale) {
  GS_REQUIRE(ctx && groups && ngroups > 0 && ngroups <= kMaxAdamGroups, "gsc_adam_step: 1..8 groups");
  GS_REQUIRE(step >= 1, "gsc_adam_step: step must be >= 1");
  AdamArgs a;
  std::memset(&a, 0, sizeof a);
  a.ngroups = ngroups;
  a.beta1 = beta1; a.beta2 = beta2; a.eps = eps; a.grad_scale = grad_scale;
  // 1 - beta^t in fp32 as the reference (adam.cr:129-130)
  a.bc1 = 1.0f - powi_f32(beta1, step);
  a.bc2 = 1.0f - powi_f32(beta2, step);
  int64_t run = 0;
  for (int i = 0; i < ngroups; i++) {
    const gsc_adam_group& G = groups[i];
    GS_REQUIRE(G.numel >= 0 && (G.numel == 0 || (G.param && G.grad && G.m && G.v)), "gsc_adam_step: bad group");
    AdamGroupDev& d = a.g[i];
    d.param = G.param; d.grad = G.grad; d.m = G.m; d.v = G.v; d.numel = G.numel;
    d.lr = G.lr; d.weight_decay = G.weight_decay;
    d.decay = 1.0f - G.lr * G.weight_decay;
    d.vec = aligned16(G.param) && aligned16(G.grad) && aligned16(G.m) && aligned16(G.v);
    run += (G.numel + 3) / 4;
    a.chunk_end[i] = run;
  }
  StageScope sc(ctx, GSC_STAGE_ADAM);
  sc.kernels(run ? 1 : 0);
  return launch_adam(a, ctx->stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Whole-view orchestration
// ---------------------------------------------------------------------------
extern "C" {

GSC_API int gsc_frame_create(gsc_ctx* ctx, gsc_frame** out) {
  GS_REQUIRE(ctx && out, "gsc_frame_create: null argument");
  gsc_frame* f = new gsc_frame();
  f->ctx = ctx;
  *out = f;
  return GSC_OK;
}

GSC_API int gsc_frame_set_tile_hint(gsc_frame* f, float* cut, int64_t count, int32_t valid) {
  GS_REQUIRE(f, "gsc_frame_set_tile_hint: null frame");
  GS_REQUIRE(((uintptr_t)cut & 3u) == 0, "gsc_frame_set_tile_hint: misaligned cut array");
  GS_REQUIRE(!cut || count > 0, "gsc_frame_set_tile_hint: empty cut array");
  f->tile_hint = cut;
  f->tile_hint_count = cut ? count : 0;
  f->tile_hint_valid = cut && valid;
  return GSC_OK;
}

GSC_API int gsc_frame_destroy(gsc_frame* f) {
  if (!f) return GSC_OK;
  cudaStreamSynchronize(f->ctx->stream);
  GsBuf* bufs[] = {&f->splats, &f->depth_pairs, &f->pairs, &f->depth_keys, &f->order, &f->block_sums, &f->offsets, &f->total,
                   &f->tiles, &f->keys, &f->vals, &f->ranges, &f->image, &f->final_T, &f->last,
                   &f->n_contrib, &f->grad2d, &f->bins, &f->tile_order, &f->tile_work,
                   &f->skip_bits, &f->tile_done, &f->tile_base, &f->pair_total, &f->cut_sub, &f->cut_cnt,
                   &f->open_flag};
  for (GsBuf* b : bufs)
    if (b->ptr) cudaFree(b->ptr);
  for (int k = 0; k < kMaxSlices; k++) {
    if (f->slice_vals[k].ptr) cudaFree(f->slice_vals[k].ptr);
    if (f->slice_ranges[k].ptr) cudaFree(f->slice_ranges[k].ptr);
  }
  delete f;
  return GSC_OK;
}

}  // extern "C"

namespace {

// Whole-view forward in three phases, so that several views can share the
// preprocess launch and a single host readback of their key counts:
//   forward_prepare   -- buffers and frame fields (no GPU work)
//   forward_sort_scan -- depth sort, per-block pair counts, scan (device only)
//   forward_bin       -- emission, tile sort, ranges, given the pair count
//   forward_composite -- compositing (on a side stream in a batched forward)
int forward_prepare(gsc_ctx* ctx, gsc_frame* f, const gsc_gaussians* g, const gsc_camera* cam,
                    const gsc_raster_config* cfg, float* image) {
  GS_REQUIRE(ctx && f && f->ctx == ctx, "gsc_rasterize_forward: bad context/frame");
  GS_TRY(check_gaussians(g));
  GS_TRY(check_view(cam, cfg));
  const int64_t n = g->count;
  const int W = cam->width, H = cam->height;
  const int tx = (W + GS_TILE - 1) / GS_TILE, ty = (H + GS_TILE - 1) / GS_TILE;
  const int64_t nb = (n + 255) / 256;
  const size_t npix = (size_t)W * H;
  f->has_forward = false;
  f->has_grad2d = false;
  GS_REQUIRE(!f->tile_hint || (int64_t)tx * ty <= f->tile_hint_count,
             "gsc_rasterize_forward: the frame's tile cut array is shorter than the view's tiles");
  f->n = n; f->width = W; f->height = H; f->tiles_x = tx; f->tiles_y = ty;
  GS_TRY(ensure(ctx, &f->splats, (size_t)n * 48 + 48));
  GS_TRY(ensure(ctx, &f->depth_pairs, (size_t)n * 8 + 8));
  GS_TRY(ensure(ctx, &f->depth_keys, (size_t)n * 4 + 4));
  GS_TRY(ensure(ctx, &f->order, (size_t)n * 4 + 4));
  GS_TRY(ensure(ctx, &f->block_sums, (size_t)nb * 4 + 4));
  GS_TRY(ensure(ctx, &f->offsets, (size_t)nb * 8 + 8));
  GS_TRY(ensure(ctx, &f->total, 8));
  GS_TRY(ensure(ctx, &f->ranges, (size_t)tx * ty * 8));
  GS_TRY(ensure(ctx, &f->final_T, npix * 4));
  GS_TRY(ensure(ctx, &f->last, npix * 4));
  GS_TRY(ensure(ctx, &f->n_contrib, npix * 4));
  GS_TRY(ensure(ctx, &f->bins, (size_t)n * 32 + 32));
  if (!image) {
    GS_TRY(ensure(ctx, &f->image, npix * 12));
    image = (float*)f->image.ptr;
  }
  f->image_ptr = image;
  f->order_ptr = (const uint32_t*)f->order.ptr;
  f->keys_valid = false;
  f->count_pending = false;
  return GSC_OK;
}

const uint4* frame_bins(const gsc_frame* f) { return (const uint4*)f->bins.ptr; }

// count_n >= 0: the pair counts and offsets cover depth positions [0, count_n)
// only (occluded binning counts its later slices itself).
int forward_sort_scan(gsc_ctx* ctx, gsc_frame* f, bool sort_depth = true, int64_t count_n = -1,
                      const TileCut* tc = nullptr) {
  const int64_t n = f->n;
  // 1. stable sort of the Gaussians by depth (non-emitting ones carry ~0 and
  //    sink); packed (depth << 32 | index) words, split into keys and order
  //    (a batched forward has sorted every view's words together already)
  if (n > 0 && sort_depth) {
    GS_TRY(scratch_reserve(ctx, sort_scratch_bytes_packed(n, 32, 64)));
    StageScope sc(ctx, GSC_STAGE_SORT);
    sc.kernels(n > 1 ? 1 + 4 : 1);
    GS_TRY(launch_sort_packed(ctx, (uint64_t*)f->depth_pairs.ptr, n, 32, 64, (uint32_t*)f->depth_keys.ptr,
                              (uint32_t*)f->order.ptr, scratch_base(ctx)));
  }
  // 2. exact allocation in depth order: per-block pair counts and their scan
  if (n == 0) return GSC_OK;
  const int64_t cn = count_n >= 0 ? std::min(count_n, n) : n;
  if (cn == 0) return cudaMemsetAsync(f->total.ptr, 0, 8, ctx->stream) == cudaSuccess ? GSC_OK : GSC_ERR_CUDA;
  {
    StageScope sc(ctx, GSC_STAGE_SCAN);
    sc.kernels(1);
    if (tc)
      GS_TRY(launch_block_sums_cut(frame_bins(f), f->order_ptr, cn, (uint32_t*)f->block_sums.ptr, *tc, ctx->stream));
    else
      GS_TRY(launch_block_sums_gather(frame_bins(f), f->order_ptr, cn, (uint32_t*)f->block_sums.ptr, ctx->stream));
  }
  StageScope sc(ctx, GSC_STAGE_SCAN);
  sc.kernels(1);
  return launch_scan_block_sums((const uint32_t*)f->block_sums.ptr, (cn + 255) / 256, (uint64_t*)f->offsets.ptr,
                                (uint64_t*)f->total.ptr, ctx->stream);
}

int forward_bin(gsc_ctx* ctx, gsc_frame* f, const gsc_raster_config* cfg, uint64_t m) {
  (void)cfg;
  const int64_t n = f->n;
  const int tx = f->tiles_x, ty = f->tiles_y;
  if (m >= (1ull << 30)) {
    set_error("gsc_rasterize_forward: " + std::to_string(m) + " keys exceed the 2^30 limit");
    return GSC_ERR_CAPACITY;
  }
  f->num_keys = (int64_t)m;
  if (ctx->profiling) {
    ctx->prof_binned += m;
    ctx->prof_kept += m;
  }
  GS_TRY(ensure(ctx, &f->tiles, (size_t)m * 4 + 4));
  GS_TRY(ensure(ctx, &f->vals, (size_t)m * 4 + 4));
  uint32_t* tiles = (uint32_t*)f->tiles.ptr;
  uint32_t* vals = (uint32_t*)f->vals.ptr;
  uint32_t* ranges = (uint32_t*)f->ranges.ptr;
  const int32_t T = tx * ty;
  const int tb = tile_bits_of(T);
  if (m > 1 && tb > 0) {
    // Emission also counts the sort's digits and presets the ranges; the
    // last sort pass writes the values and the ranges (no tile array).
    GS_TRY(ensure(ctx, &f->pairs, (size_t)m * 8 + 8));
    uint64_t* pairs = (uint64_t*)f->pairs.ptr;
    GS_TRY(scratch_reserve(ctx, sort_scratch_bytes_packed((int64_t)m, 32, 32 + tb)));
    char* scratch = scratch_base(ctx);
    {
      StageScope sc(ctx, GSC_STAGE_EMIT);
      sc.kernels(1);
      GS_TRY(sort_packed_clear(ctx, (int64_t)m, 32, 32 + tb, scratch));
      GS_TRY(launch_emit_tiles(frame_bins(f), f->order_ptr, n, (const uint64_t*)f->offsets.ptr, tx, pairs,
                               ctx->stream, sort_packed_hist(scratch, (int64_t)m, 32, 32 + tb), (tb + 7) / 8,
                               ranges, T, (int64_t)ctx->num_sms * 32));
    }
    {
      // 3. stable sort of the packed (tile << 32 | id) words by the tile bits
      StageScope sc(ctx, GSC_STAGE_SORT);
      sc.kernels((tb + 7) / 8);
      GS_TRY(launch_sort_packed(ctx, pairs, (int64_t)m, 32, 32 + tb, nullptr, vals, scratch, 0xFFFFFFFFu, true,
                                ranges, (uint32_t)T));
    }
    StageScope sc(ctx, GSC_STAGE_RANGES);
    sc.kernels(1);
    return launch_ranges_finish(ranges, T, ctx->stream);
  }
  if (m) {
    GS_TRY(ensure(ctx, &f->pairs, (size_t)m * 8 + 8));
    uint64_t* pairs = (uint64_t*)f->pairs.ptr;
    {
      StageScope sc(ctx, GSC_STAGE_EMIT);
      sc.kernels(1);
      GS_TRY(launch_emit_tiles(frame_bins(f), f->order_ptr, n, (const uint64_t*)f->offsets.ptr, tx, pairs,
                               ctx->stream));
    }
    // 3. a single pair or a single tile: nothing to sort, split the words
    GS_TRY(scratch_reserve(ctx, sort_scratch_bytes_packed((int64_t)m, 32, 32 + tb)));
    StageScope sc(ctx, GSC_STAGE_SORT);
    sc.kernels(tb > 0 && m > 1 ? 1 + (tb + 7) / 8 : 1);
    GS_TRY(launch_sort_packed(ctx, pairs, (int64_t)m, 32, 32 + tb, tiles, vals, scratch_base(ctx)));
  }
  {
    StageScope sc(ctx, GSC_STAGE_RANGES);
    sc.kernels(m ? 1 : 0);
    GS_TRY(launch_tile_ranges_u32(tiles, (int64_t)m, T, ranges, ctx->stream));
  }
  return GSC_OK;
}

int forward_composite(gsc_ctx* ctx, gsc_frame* f, const gsc_raster_config* cfg, uint32_t* n_contrib,
                      float* final_T) {
  const int W = f->width, H = f->height;
  const size_t npix = (size_t)W * H;
  CompositeFwdArgs a;
  fill_fwd(&a, (const float*)f->splats.ptr, (const uint32_t*)f->vals.ptr, (const uint32_t*)f->ranges.ptr, W, H,
           cfg);
  a.image = f->image_ptr;
  a.final_T = (float*)f->final_T.ptr;
  a.last = (uint32_t*)f->last.ptr;
  a.n_contrib = (uint32_t*)f->n_contrib.ptr;
  if (ctx->profiling) a.pge = reinterpret_cast<unsigned long long*>(ctx->err + 2);
  const int32_t T = f->tiles_x * f->tiles_y;
  GS_TRY(ensure(ctx, &f->tile_work, (size_t)T * 4 + 4));
  a.tile_work = (uint32_t*)f->tile_work.ptr;
  {
    // The forward keeps the row-major tile order (its last wave overlaps the
    // next view's binning in a batched forward). It leaves the backward's
    // order: longest backward lists first, so that the backward's last wave
    // holds the short ones; the length is the tile's max of `last` (the full
    // mode's backward starts there), the whole list in the reference mode.
    StageScope sc(ctx, GSC_STAGE_COMPOSITE_FWD);
    sc.kernels(2);
    GS_TRY(launch_composite_fwd(a, ctx->stream));
    const bool full = cfg->mode == GSC_MODE_FULL;
    GS_TRY(ensure(ctx, &f->tile_order, (size_t)T * 4 + 4));
    GS_TRY(launch_tile_order(full ? nullptr : (const uint32_t*)f->ranges.ptr, full ? a.tile_work : nullptr, T,
                             (uint32_t*)f->tile_order.ptr, ctx->stream));
  }
  if (n_contrib)
    GS_CK(cudaMemcpyAsync(n_contrib, f->n_contrib.ptr, npix * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  if (final_T)
    GS_CK(cudaMemcpyAsync(final_T, f->final_T.ptr, npix * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  f->has_forward = true;
  return GSC_OK;
}

// ---- depth-sliced binning (GSC_BIN_OCCLUDED) --------------------------------
//
// The depth order of a view is cut into slices (positions in multiples of
// 256). Slice s is binned (pair counts, emission, tile sort) and composited
// on top of the per-pixel state of slices < s; the compositing marks the
// tiles whose pixels have all stopped, and the next slice's pair counting
// and emission drop the Gaussians whose listed tiles are all marked. Within
// a tile the slices' lists, concatenated in slice order, are the tile's
// contributing list up to its saturation point (every Gaussian before it
// kept) and a subset after it, so every pixel sees the same entries in the
// same order up to its stop and the results equal the unsliced ones bit for
// bit. The frame keeps, per tile, the first tile_work[t] (the largest `last`)
// entries, which is all that the backward reads.
#ifndef GS_OCC_FRAC1
#define GS_OCC_FRAC1 0.2
#endif
#ifndef GS_OCC_FRAC2
#define GS_OCC_FRAC2 1.0
#endif
#ifndef GS_OCC_FRAC3
#define GS_OCC_FRAC3 1.0
#endif

// Depth-sliced binning applies to views of more than one tile (the one-tile
// case has no tile sort to save).
bool occlusion_binning(const gsc_raster_config* cfg, const gsc_frame* f) {
  return cfg->binning == GSC_BIN_OCCLUDED && (int64_t)f->tiles_x * f->tiles_y > 1;
}

// Slice boundaries (depth-order positions) of n Gaussians: [0 = p0 < p1 < ... = n].
int occlusion_slices(int64_t n, int64_t* p) {
  const double frac[kMaxSlices - 1] = {GS_OCC_FRAC1, GS_OCC_FRAC2, GS_OCC_FRAC3};
  int S = 0;
  p[0] = 0;
  for (int k = 0; k < kMaxSlices - 1; k++) {
    int64_t b = (int64_t)(frac[k] * (double)n);
    b = (b + 255) / 256 * 256;
    if (b >= n) break;
    if (b > p[S]) p[++S] = b;
  }
  p[++S] = n;
  return S;
}

// The depth positions the whole-view pair counting covers: every slice but
// the last (which counts its own pairs), or everything with one slice.
int64_t occlusion_count_end(int S, const int64_t* p) { return S >= 2 ? p[S - 1] : p[S]; }

// Per-tile cut (a valid tile hint): two slices that both span every depth
// position, the first holding each tile's pairs in front of its cut, the
// second the rest of the tiles whose pixels did not all stop.
#ifndef GS_TILE_HINT_MARGIN
#define GS_TILE_HINT_MARGIN 0.005f
#endif
bool tile_cut_mode(const gsc_frame* f) { return f->tile_hint && f->tile_hint_valid && f->n > 0; }

int tile_cut_slices(int64_t n, int64_t* p) {
  p[0] = 0;
  p[1] = n;
  p[2] = n;
  return 2;
}

// The cut of slice `mode` (0 or 1) of frame f, with its per-position buffers.
int tile_cut_of(gsc_ctx* ctx, gsc_frame* f, int mode, TileCut* tc) {
  GS_TRY(ensure(ctx, &f->cut_sub, (size_t)f->n * 8 + 8));
  GS_TRY(ensure(ctx, &f->cut_cnt, (size_t)f->n * 4 + 4));
  GS_TRY(ensure(ctx, &f->open_flag, 16));
  tc->cut = f->tile_hint;
  tc->mode = mode;
  tc->tiles_x = f->tiles_x;
  tc->sub = (uint64_t*)f->cut_sub.ptr;
  tc->cnt = (uint32_t*)f->cut_cnt.ptr;
  if (mode == 1) {
    tc->done = (const unsigned long long*)f->tile_done.ptr;
    tc->done_words = done_words_of(f->tiles_x);
    tc->open = (const unsigned int*)f->open_flag.ptr;
  }
  return GSC_OK;
}

// One readback per batch: each view's pair total (from preprocess) and the
// pair counts before its slice boundaries (from the whole-view scan), turned
// into up[v][s], slice s's pair count before the skip test.
int read_slice_counts(gsc_ctx* ctx, gsc_frame* const* frames, int nviews, const int* S,
                      const int64_t (*p)[kMaxSlices + 1], uint64_t* m, uint64_t (*up)[kMaxSlices]) {
  uint64_t* pin = (uint64_t*)ctx->pinned;  // [slot k][view], slot 0 = totals
  for (int v = 0; v < nviews; v++) {
    const gsc_frame* f = frames[v];
    GS_CK(cudaMemcpyAsync(pin + v, f->pair_total.ptr, 8, cudaMemcpyDeviceToHost, ctx->stream));
    for (int k = 1; k < S[v]; k++) {
      // boundary k < S - 1 from the offsets; the last one is the scan's total
      const uint64_t* src = k + 1 < S[v] ? (const uint64_t*)f->offsets.ptr + p[v][k] / 256
                                         : (const uint64_t*)f->total.ptr;
      GS_CK(cudaMemcpyAsync(pin + GSC_MAX_BATCH_VIEWS * k + v, src, 8, cudaMemcpyDeviceToHost, ctx->stream));
    }
  }
  GS_CK(cudaStreamSynchronize(ctx->stream));
  for (int v = 0; v < nviews; v++) {
    m[v] = pin[v];
    uint64_t prev = 0;
    for (int k = 0; k < S[v]; k++) {
      const uint64_t at = k + 1 < S[v] ? pin[GSC_MAX_BATCH_VIEWS * (k + 1) + v] : m[v];
      up[v][k] = at - prev;
      prev = at;
    }
  }
  return GSC_OK;
}

// Binning of slice s of frame f on ctx->stream. Slice 0 uses the whole-view
// offsets (its pair count `m0` is exact and known on the host); a later slice
// counts again with the skip test and sorts with a device-side count, its
// buffers sized by the upper bound `m_up`.
int sliced_bin(gsc_ctx* ctx, gsc_frame* f, int s, const int64_t* p, uint64_t m_up) {
  const bool cutm = tile_cut_mode(f);
  const int64_t n_s = cutm ? f->n : p[s + 1] - p[s];
  const int tx = f->tiles_x, ty = f->tiles_y;
  const int32_t T = tx * ty;
  const int tb = tile_bits_of(T);
  const uint32_t* order = cutm ? f->order_ptr : f->order_ptr + p[s];
  TileCut tc;
  if (cutm) GS_TRY(tile_cut_of(ctx, f, s, &tc));
  GS_TRY(ensure(ctx, &f->slice_vals[s], (size_t)m_up * 4 + 4));
  GS_TRY(ensure(ctx, &f->slice_ranges[s], (size_t)T * 8));
  uint32_t* vals = (uint32_t*)f->slice_vals[s].ptr;
  uint32_t* ranges = (uint32_t*)f->slice_ranges[s].ptr;
  const uint64_t* offsets = (const uint64_t*)f->offsets.ptr + (cutm ? 0 : p[s] / 256);
  const uint64_t* n_dev = nullptr;
  const uint32_t* skip = nullptr;
  if (s > 0 && n_s > 0) {
    StageScope sc(ctx, GSC_STAGE_SCAN);
    sc.kernels(2);
    if (cutm)
      GS_TRY(launch_block_sums_cut(frame_bins(f), order, n_s, (uint32_t*)f->block_sums.ptr, tc, ctx->stream));
    else
      GS_TRY(launch_block_sums_gather(frame_bins(f), order, n_s, (uint32_t*)f->block_sums.ptr, ctx->stream,
                                      (const unsigned long long*)f->tile_done.ptr, done_words_of(tx),
                                      (uint32_t*)f->skip_bits.ptr));
    GS_TRY(launch_scan_block_sums((const uint32_t*)f->block_sums.ptr, (n_s + 255) / 256, (uint64_t*)f->offsets.ptr,
                                  (uint64_t*)f->total.ptr, ctx->stream));
    offsets = (const uint64_t*)f->offsets.ptr;
    n_dev = (const uint64_t*)f->total.ptr;
    if (!cutm) skip = (const uint32_t*)f->skip_bits.ptr;
    if (ctx->profiling)
      GS_TRY(launch_add_u64(n_dev, reinterpret_cast<unsigned long long*>(ctx->err + 4), ctx->stream));
  } else if (s == 0 && ctx->profiling) {
    ctx->prof_binned += m_up;
  }
  if (m_up == 0 || n_s == 0) {
    GS_CK(cudaMemsetAsync(ranges, 0, (size_t)T * 8, ctx->stream));
    return GSC_OK;
  }
  GS_TRY(ensure(ctx, &f->pairs, (size_t)m_up * 8 + 8));
  uint64_t* pairs = (uint64_t*)f->pairs.ptr;
  GS_TRY(scratch_reserve(ctx, sort_scratch_bytes_packed((int64_t)m_up, 32, 32 + tb)));
  char* scratch = scratch_base(ctx);
  {
    StageScope sc(ctx, GSC_STAGE_EMIT);
    sc.kernels(1);
    GS_TRY(sort_packed_clear(ctx, (int64_t)m_up, 32, 32 + tb, scratch));
    GS_TRY(launch_emit_tiles(frame_bins(f), order, n_s, offsets, tx, pairs, ctx->stream,
                             sort_packed_hist(scratch, (int64_t)m_up, 32, 32 + tb), (tb + 7) / 8, ranges, T,
                             (int64_t)ctx->num_sms * 32, skip, cutm ? &tc : nullptr));
  }
  {
    StageScope sc(ctx, GSC_STAGE_SORT);
    sc.kernels((tb + 7) / 8);
    GS_TRY(launch_sort_packed(ctx, pairs, (int64_t)m_up, 32, 32 + tb, nullptr, vals, scratch, 0xFFFFFFFFu, true,
                              ranges, (uint32_t)T, n_dev));
  }
  StageScope sc(ctx, GSC_STAGE_RANGES);
  sc.kernels(1);
  return launch_ranges_finish(ranges, T, ctx->stream);
}

// Compositing of slice s of frame f on ctx->stream; the last slice also
// builds the frame's final lists and the backward's tile order.
int sliced_composite(gsc_ctx* ctx, gsc_frame* f, const gsc_raster_config* cfg, int s, int S) {
  const int32_t T = f->tiles_x * f->tiles_y;
  const size_t done_bytes = (size_t)f->tiles_y * done_words_of(f->tiles_x) * 8;
  const bool cutm = tile_cut_mode(f);
  if (s == 0) {
    GS_CK(cudaMemsetAsync(f->tile_done.ptr, 0, done_bytes, ctx->stream));
    GS_CK(cudaMemsetAsync(f->tile_base.ptr, 0, (size_t)T * 4, ctx->stream));
    if (cutm) GS_CK(cudaMemsetAsync(f->open_flag.ptr, 0, 4, ctx->stream));
  }
  CompositeFwdArgs a;
  fill_fwd(&a, (const float*)f->splats.ptr, (const uint32_t*)f->slice_vals[s].ptr,
           (const uint32_t*)f->slice_ranges[s].ptr, f->width, f->height, cfg);
  a.image = f->image_ptr;
  a.final_T = (float*)f->final_T.ptr;
  a.last = (uint32_t*)f->last.ptr;
  a.n_contrib = (uint32_t*)f->n_contrib.ptr;
  a.tile_base = (uint32_t*)f->tile_base.ptr;
  a.tile_done = (unsigned long long*)f->tile_done.ptr;
  a.done_words = done_words_of(f->tiles_x);
  a.first_slice = s == 0;
  a.last_slice = s == S - 1;
  const bool last = s == S - 1;
  if (cutm && !last) {
    a.tile_cut = f->tile_hint;
    a.open_flag = (unsigned int*)f->open_flag.ptr;
  }
  a.mark_done = last && f->tile_hint != nullptr;  // the next cut needs the stopped tiles
  if (last) {
    if (ctx->profiling) a.pge = reinterpret_cast<unsigned long long*>(ctx->err + 2);
    GS_TRY(ensure(ctx, &f->tile_work, (size_t)T * 4 + 4));
    a.tile_work = (uint32_t*)f->tile_work.ptr;
  }
  {
    StageScope sc(ctx, GSC_STAGE_COMPOSITE_FWD);
    sc.kernels(1);
    GS_TRY(launch_composite_fwd(a, ctx->stream));
  }
  if (!last) return GSC_OK;
  // final lists: per tile the entries up to its largest `last`
  {
    const uint32_t* sv[kMaxSlices];
    const uint32_t* sr[kMaxSlices];
    for (int k = 0; k < S; k++) {
      sv[k] = (const uint32_t*)f->slice_vals[k].ptr;
      sr[k] = (const uint32_t*)f->slice_ranges[k].ptr;
    }
    StageScope sc(ctx, GSC_STAGE_RANGES);
    sc.kernels(f->tile_hint ? 3 : 2);
    GS_TRY(launch_concat_slices(sv, sr, S, a.tile_work, T, (uint32_t*)f->vals.ptr, (uint32_t*)f->ranges.ptr,
                                (uint64_t*)f->total.ptr, ctx->stream));
    if (ctx->profiling)
      GS_TRY(launch_add_u64((const uint64_t*)f->total.ptr, reinterpret_cast<unsigned long long*>(ctx->err + 6),
                            ctx->stream));
    if (f->tile_hint)  // the cut of this view's next forward
      GS_TRY(launch_tile_cut_update((const uint32_t*)f->ranges.ptr, (const uint32_t*)f->vals.ptr, a.tile_work,
                                    (const unsigned long long*)f->tile_done.ptr, done_words_of(f->tiles_x),
                                    f->tiles_x, T, (const float*)f->splats.ptr, GS_TILE_HINT_MARGIN, f->tile_hint,
                                    ctx->stream));
  }
  const bool full = cfg->mode == GSC_MODE_FULL;
  GS_TRY(ensure(ctx, &f->tile_order, (size_t)T * 4 + 4));
  {
    StageScope sc(ctx, GSC_STAGE_COMPOSITE_FWD);
    sc.kernels(1);
    GS_TRY(launch_tile_order(full ? nullptr : (const uint32_t*)f->ranges.ptr, full ? a.tile_work : nullptr, T,
                             (uint32_t*)f->tile_order.ptr, ctx->stream));
  }
  f->has_forward = true;
  f->count_pending = true;
  f->keys_valid = false;
  return GSC_OK;
}

// Depth-sliced forward of `nviews` frames whose depth orders and whole-view
// pair counts (per-chunk offsets; m[v] in total) are ready. up[v][s]: the
// pair count of slice s before the skip test (exact for s = 0). Binning runs
// on the caller's stream, compositing on the side stream, slice by slice
// across the views, so that view v's compositing overlaps the binning of the
// next views and slice s + 1 of a view waits only for its own slice s.
#ifndef GS_BIN_STREAMS
#define GS_BIN_STREAMS 2
#endif
int forward_sliced(gsc_ctx* ctx, gsc_frame* const* frames, int nviews, const gsc_raster_config* cfg,
                   const int64_t (*p)[kMaxSlices + 1], const int* S, const uint64_t (*up)[kMaxSlices]) {
  if (!ctx->side) {
    GS_CK(cudaStreamCreateWithFlags(&ctx->side, cudaStreamNonBlocking));
    for (auto& e : ctx->side_ev) GS_CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  if (!ctx->bin_ev[0])
    for (int v = 0; v < GSC_MAX_BATCH_VIEWS; v++) {
      GS_CK(cudaEventCreateWithFlags(&ctx->bin_ev[v], cudaEventDisableTiming));
      GS_CK(cudaEventCreateWithFlags(&ctx->comp_ev[v], cudaEventDisableTiming));
    }
  for (int v = 0; v < nviews; v++) {
    gsc_frame* f = frames[v];
    const int32_t T = f->tiles_x * f->tiles_y;
    uint64_t mmax = 0;
    for (int s = 0; s < S[v]; s++) mmax = std::max(mmax, up[v][s]);
    GS_TRY(ensure(ctx, &f->tile_done, (size_t)f->tiles_y * done_words_of(f->tiles_x) * 8 + 16));
    GS_TRY(ensure(ctx, &f->tile_base, (size_t)T * 4 + 4));
    GS_TRY(ensure(ctx, &f->skip_bits, (size_t)(f->n + 31) / 32 * 4 + 4));
    // the final lists hold at most every pair of the view
    uint64_t total = 0;
    for (int s = 0; s < S[v]; s++) total += up[v][s];
    GS_TRY(ensure(ctx, &f->vals, (size_t)total * 4 + 4));
    GS_TRY(ensure(ctx, &f->pairs, (size_t)mmax * 8 + 8));
    f->num_keys = (int64_t)total;
  }
  cudaStream_t main_stream = ctx->stream;
  // views alternate between two binning streams (each with its own sort
  // scratch), so the latency-bound sorts of two views overlap
  // Under per-stage tracing everything runs in order on the caller's stream,
  // so that each stage's events time that stage alone.
  const bool serial = ctx->profiling;
  const int nbin = GS_BIN_STREAMS > 1 && nviews > 1 && !serial ? 2 : 1;
  cudaStream_t bin_stream[2] = {main_stream, main_stream};
  if (nbin == 2) {
    if (!ctx->bin2) {
      GS_CK(cudaStreamCreateWithFlags(&ctx->bin2, cudaStreamNonBlocking));
      for (auto& e : ctx->bin2_ev) GS_CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    bin_stream[1] = ctx->bin2;
    GS_CK(cudaEventRecord(ctx->bin2_ev[0], main_stream));  // bin2 follows the caller's earlier work
    GS_CK(cudaStreamWaitEvent(ctx->bin2, ctx->bin2_ev[0], 0));
  }
  int Smax = 0;
  for (int v = 0; v < nviews; v++) Smax = std::max(Smax, S[v]);
  int rc = GSC_OK;
  for (int s = 0; s < Smax && rc == GSC_OK; s++) {
    for (int v = 0; v < nviews && rc == GSC_OK; v++) {
      if (s >= S[v]) continue;
      gsc_frame* f = frames[v];
      const int lane = v % nbin;
      cudaStream_t bs = bin_stream[lane];
      ctx->stream = bs;
      ctx->cur_scratch = lane ? &ctx->scratch_alt : &ctx->scratch;
      if (s > 0) GS_CK(cudaStreamWaitEvent(bs, ctx->comp_ev[v], 0));
      rc = sliced_bin(ctx, f, s, p[v], up[v][s]);
      if (rc) break;
      GS_CK(cudaEventRecord(ctx->bin_ev[v], bs));
      GS_CK(cudaStreamWaitEvent(ctx->side, ctx->bin_ev[v], 0));
      cudaStream_t cs = serial ? bs : ctx->side;
      ctx->stream = cs;
      ctx->cur_scratch = nullptr;
      rc = sliced_composite(ctx, f, cfg, s, S[v]);
      GS_CK(cudaEventRecord(ctx->comp_ev[v], cs));
    }
  }
  ctx->stream = main_stream;
  ctx->cur_scratch = nullptr;
  // the caller's stream waits for every compositing and the second binning stream
  GS_CK(cudaEventRecord(ctx->side_ev[GSC_MAX_BATCH_VIEWS], ctx->side));
  GS_CK(cudaStreamWaitEvent(main_stream, ctx->side_ev[GSC_MAX_BATCH_VIEWS], 0));
  if (nbin == 2) {
    GS_CK(cudaEventRecord(ctx->bin2_ev[1], ctx->bin2));
    GS_CK(cudaStreamWaitEvent(main_stream, ctx->bin2_ev[1], 0));
  }
  return rc;
}

// Compact batched depth keys: an emitted depth z lies in (max(near_z, 0),
// far_z], so bits(z) - bits(max(near_z, 0)) is in [1, span]; usable when the
// span leaves 2^28 - 1 free for the Gaussians that emit nothing.
bool depth_compact_base(const gsc_raster_config* cfg, uint32_t* base) {
  const float lo = cfg->near_z > 0.0f ? cfg->near_z : 0.0f;
  const float hi = cfg->far_z;
  if (!(hi > lo) || !std::isfinite(hi)) return false;
  uint32_t blo, bhi;
  std::memcpy(&blo, &lo, 4);
  std::memcpy(&bhi, &hi, 4);
  if (bhi - blo >= 0x0FFFFFFFu) return false;
  *base = blo;
  return true;
}

// One preprocess launch for the frames (all of one image size).
int forward_preprocess(gsc_ctx* ctx, gsc_frame* const* frames, const gsc_camera* cams, int k,
                       const gsc_gaussians* g, const gsc_raster_config* cfg, uint64_t* batch_words = nullptr) {
  PreprocessArgs a;
  std::memset(&a, 0, sizeof a);
  a.n = g->count;
  a.pos = g->position; a.log_scale = g->log_scale; a.rot = g->rotation;
  a.logit_opacity = g->logit_opacity; a.sh = g->sh;
  a.cfg = *cfg;
  a.tiles_x = frames[0]->tiles_x;
  a.tiles_y = frames[0]->tiles_y;
  a.nviews = k;
  for (int v = 0; v < k; v++) {
    a.cams[v] = cams[v];
    a.splats_v[v] = (float*)frames[v]->splats.ptr;
    a.depth_pairs_v[v] = batch_words ? batch_words + (size_t)v * g->count : (uint64_t*)frames[v]->depth_pairs.ptr;
    a.bin_v[v] = (uint4*)frames[v]->bins.ptr;
  }
  a.view_key = batch_words != nullptr;
  a.depth_compact = a.view_key && depth_compact_base(cfg, &a.depth_base);
  a.contributing = cfg->binning != GSC_BIN_REFERENCE;
  if (occlusion_binning(cfg, frames[0]))
    for (int v = 0; v < k; v++) {
      GS_TRY(ensure(ctx, &frames[v]->pair_total, 8));
      GS_CK(cudaMemsetAsync(frames[v]->pair_total.ptr, 0, 8, ctx->stream));
      a.pair_total_v[v] = (unsigned long long*)frames[v]->pair_total.ptr;
    }
  StageScope sc(ctx, GSC_STAGE_PREPROCESS);
  sc.kernels(g->count ? 1 : 0);
  return launch_preprocess(a, ctx->stream);
}

}  // namespace

extern "C" {

GSC_API int gsc_rasterize_forward(gsc_ctx* ctx, gsc_frame* f, const gsc_gaussians* g,
                                  const gsc_camera* cam, const gsc_raster_config* cfg, float* image,
                                  uint32_t* n_contrib, float* final_T, int64_t* num_rendered) {
  GS_TRY(forward_prepare(ctx, f, g, cam, cfg, image));
  if (occlusion_binning(cfg, f) && g->count) {
    // the depth-sliced path of the batched call, with one view
    GS_TRY(forward_preprocess(ctx, &f, cam, 1, g, cfg));
    int S[1];
    int64_t bounds[1][kMaxSlices + 1];
    uint64_t up[1][kMaxSlices], m = 0;
    TileCut tc0;
    const bool cutm = tile_cut_mode(f);
    if (cutm) GS_TRY(tile_cut_of(ctx, f, 0, &tc0));
    S[0] = cutm ? tile_cut_slices(f->n, bounds[0]) : occlusion_slices(f->n, bounds[0]);
    GS_TRY(forward_sort_scan(ctx, f, true, occlusion_count_end(S[0], bounds[0]), cutm ? &tc0 : nullptr));
    GS_TRY(read_slice_counts(ctx, &f, 1, S, bounds, &m, up));
    if (num_rendered) *num_rendered = (int64_t)m;
    GS_TRY(forward_sliced(ctx, &f, 1, cfg, bounds, S, up));
    if (n_contrib)
      GS_CK(cudaMemcpyAsync(n_contrib, f->n_contrib.ptr, (size_t)f->width * f->height * 4, cudaMemcpyDeviceToDevice,
                            ctx->stream));
    if (final_T)
      GS_CK(cudaMemcpyAsync(final_T, f->final_T.ptr, (size_t)f->width * f->height * 4, cudaMemcpyDeviceToDevice,
                            ctx->stream));
    return GSC_OK;
  }
  GS_TRY(forward_preprocess(ctx, &f, cam, 1, g, cfg));
  GS_TRY(forward_sort_scan(ctx, f));
  uint64_t m = 0;
  if (f->n) GS_TRY(read_u64(ctx, (const uint64_t*)f->total.ptr, &m));
  if (num_rendered) *num_rendered = (int64_t)m;
  GS_TRY(forward_bin(ctx, f, cfg, m));
  return forward_composite(ctx, f, cfg, n_contrib, final_T);
}

GSC_API int gsc_rasterize_forward_batch(gsc_ctx* ctx, gsc_frame* const* frames, const gsc_camera* cams,
                                        int32_t nviews, const gsc_gaussians* g, const gsc_raster_config* cfg,
                                        float* const* images, int64_t* num_rendered) {
  GS_REQUIRE(ctx && frames && cams, "gsc_rasterize_forward_batch: null argument");
  GS_REQUIRE(nviews >= 1 && nviews <= GSC_MAX_BATCH_VIEWS, "gsc_rasterize_forward_batch: nviews out of range");
  for (int v = 0; v < nviews; v++) {
    GS_REQUIRE(cams[v].width == cams[0].width && cams[v].height == cams[0].height,
               "gsc_rasterize_forward_batch: the views must share one image size");
    for (int u = 0; u < v; u++)
      GS_REQUIRE(frames[u] != frames[v], "gsc_rasterize_forward_batch: a frame appears twice");
    GS_TRY(forward_prepare(ctx, frames[v], g, &cams[v], cfg, images ? images[v] : nullptr));
  }
  const int64_t n = g->count;
  const bool batched_depth = nviews > 1 && n > 1 && n < (1ll << 28);
  uint32_t* order = nullptr;
  if (!batched_depth) GS_TRY(forward_preprocess(ctx, frames, cams, nviews, g, cfg));
  if (batched_depth) {
    // One depth sort for the whole batch: view << 60 | bits(depth) << 28 |
    // index words sorted by bits [28, 64), i.e. by view, then depth; view v's
    // order is the v-th run of n indices. With the compact depth keys the
    // words are view << 56 | (bits(depth) - bits(near)) << 28 | index and the
    // sort takes 4 passes instead of 5.
    const int64_t total = (int64_t)nviews * n;
    GS_TRY(ensure(ctx, &ctx->batch_pairs, (size_t)total * 8));
    GS_TRY(ensure(ctx, &ctx->batch_order, (size_t)total * 4));
    uint64_t* words = (uint64_t*)ctx->batch_pairs.ptr;
    order = (uint32_t*)ctx->batch_order.ptr;
    GS_TRY(forward_preprocess(ctx, frames, cams, nviews, g, cfg, words));
    {
      uint32_t base;
      int end_bit = 64;
      if (depth_compact_base(cfg, &base)) {
        int vb = 0;
        while ((1 << vb) < nviews) vb++;
        end_bit = 56 + vb;
      }
      GS_TRY(scratch_reserve(ctx, sort_scratch_bytes_packed(total, 28, end_bit)));
      StageScope sc(ctx, GSC_STAGE_SORT);
      sc.kernels(1 + (end_bit - 28 + 7) / 8);
      GS_TRY(launch_sort_packed(ctx, words, total, 28, end_bit, nullptr, order, scratch_base(ctx), 0x0FFFFFFFu));
    }
  }
  // depth-sliced binning counts the pairs of its first slices here (the last
  // slice counts its own), the view's total comes from preprocess
  const bool occl = occlusion_binning(cfg, frames[0]);
  int S[GSC_MAX_BATCH_VIEWS] = {};
  int64_t bounds[GSC_MAX_BATCH_VIEWS][kMaxSlices + 1] = {};
  TileCut tc0[GSC_MAX_BATCH_VIEWS];
  bool cutm[GSC_MAX_BATCH_VIEWS] = {};
  for (int v = 0; v < nviews && occl; v++) {
    cutm[v] = tile_cut_mode(frames[v]);
    if (cutm[v]) GS_TRY(tile_cut_of(ctx, frames[v], 0, &tc0[v]));
    S[v] = cutm[v] ? tile_cut_slices(frames[v]->n, bounds[v]) : occlusion_slices(frames[v]->n, bounds[v]);
  }
  for (int v = 0; v < nviews; v++) {
    if (batched_depth) frames[v]->order_ptr = order + (size_t)v * n;
    GS_TRY(forward_sort_scan(ctx, frames[v], !batched_depth, occl ? occlusion_count_end(S[v], bounds[v]) : -1,
                             cutm[v] ? &tc0[v] : nullptr));
  }
  // one readback of every view's pair count (and, for depth-sliced binning,
  // of the pair counts before each slice boundary)
  uint64_t m[GSC_MAX_BATCH_VIEWS] = {};
  uint64_t up[GSC_MAX_BATCH_VIEWS][kMaxSlices] = {};
  if (g->count && occl) {
    GS_TRY(read_slice_counts(ctx, frames, nviews, S, bounds, m, up));
  } else if (g->count) {
    uint64_t* pin = (uint64_t*)ctx->pinned;
    for (int v = 0; v < nviews; v++)
      GS_CK(cudaMemcpyAsync(pin + v, frames[v]->total.ptr, 8, cudaMemcpyDeviceToHost, ctx->stream));
    GS_CK(cudaStreamSynchronize(ctx->stream));
    std::memcpy(m, ctx->pinned, 8 * (size_t)nviews);
  }
  if (occl && g->count) {
    for (int v = 0; v < nviews; v++)
      if (num_rendered) num_rendered[v] = (int64_t)m[v];
    return forward_sliced(ctx, frames, nviews, cfg, bounds, S, up);
  }
  // Binning of view v on the caller's stream, its compositing on the side
  // stream, so that it overlaps the binning of view v + 1 (every view has its
  // own frame buffers; the sort scratch is used by the caller's stream only).
  if (!ctx->side) {
    GS_CK(cudaStreamCreateWithFlags(&ctx->side, cudaStreamNonBlocking));
    for (auto& e : ctx->side_ev) GS_CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  cudaStream_t main_stream = ctx->stream;
  int rc = GSC_OK;
  for (int v = 0; v < nviews && rc == GSC_OK; v++) {
    if (num_rendered) num_rendered[v] = (int64_t)m[v];
    rc = forward_bin(ctx, frames[v], cfg, m[v]);
    if (rc) break;
    GS_CK(cudaEventRecord(ctx->side_ev[v], main_stream));
    GS_CK(cudaStreamWaitEvent(ctx->side, ctx->side_ev[v], 0));
    ctx->stream = ctx->side;
    rc = forward_composite(ctx, frames[v], cfg, nullptr, nullptr);
    ctx->stream = main_stream;
  }
  // the caller's stream waits for every compositing
  GS_CK(cudaEventRecord(ctx->side_ev[GSC_MAX_BATCH_VIEWS], ctx->side));
  GS_CK(cudaStreamWaitEvent(main_stream, ctx->side_ev[GSC_MAX_BATCH_VIEWS], 0));
  return rc;
}

GSC_API int gsc_rasterize_backward(gsc_ctx* ctx, gsc_frame* f, const gsc_gaussians* g,
                                   const gsc_camera* cam, const gsc_raster_config* cfg,
                                   const float* dL_dimage, const float* target, float l1_scale,
                                   float* loss_sum, const gsc_gaussian_grads* grads,
                                   const gsc_grads2d* g2d) {
  GS_REQUIRE(ctx && f && f->ctx == ctx, "gsc_rasterize_backward: bad context/frame");
  GS_REQUIRE(f->has_forward, "gsc_rasterize_backward: no forward on this frame");
  GS_TRY(check_gaussians(g));
  GS_TRY(check_view(cam, cfg));
  if (grads) GS_TRY(check_grads(grads));  // NULL: stop after the composite backward
  GS_REQUIRE(g->count == f->n && cam->width == f->width && cam->height == f->height,
             "gsc_rasterize_backward: gaussians/camera differ from the frame's forward");
  GS_REQUIRE((dL_dimage != nullptr) != (target != nullptr),
             "gsc_rasterize_backward: exactly one of dL_dimage / target");
  const int64_t n = f->n;
  GS_TRY(ensure(ctx, &f->grad2d, (size_t)n * 36 + 4));
  float* grad2d = (float*)f->grad2d.ptr;
  GS_CK(cudaMemsetAsync(grad2d, 0, (size_t)n * 36, ctx->stream));
  CompositeBwdArgs a;
  fill_bwd(&a, (const float*)f->splats.ptr, (const uint32_t*)f->vals.ptr, (const uint32_t*)f->ranges.ptr,
           f->width, f->height, cfg);
  a.dL_dimage = dL_dimage;
  a.image = f->image_ptr;
  a.target = target;
  a.l1_scale = l1_scale;
  a.final_T = (const float*)f->final_T.ptr;
  a.last = (const uint32_t*)f->last.ptr;
  a.grad2d = grad2d;
  a.loss_sum = loss_sum;
  {
    StageScope sc(ctx, GSC_STAGE_COMPOSITE_BWD);
    a.tile_order = (const uint32_t*)f->tile_order.ptr;  // the forward's work order
    sc.kernels(1);
    GS_TRY(launch_composite_bwd(a, cfg->mode == GSC_MODE_FULL, ctx->stream));
  }
  f->has_grad2d = true;
  if (!grads) return GSC_OK;
  return do_preprocess_bwd(ctx, g, cam, cfg, grad2d, grads, g2d);
}

// The batched preprocess backward runs over the Gaussians that received a
// screen-space gradient only (preprocess_bwd.cu).
#ifndef GS_PBWD_COMPACT
#define GS_PBWD_COMPACT 1
#endif

GSC_API int gsc_rasterize_backward_batch(gsc_ctx* ctx, gsc_frame* const* frames, const gsc_camera* cams,
                                         int32_t nviews, const gsc_gaussians* g,
                                         const gsc_raster_config* cfg, const gsc_gaussian_grads* grads) {
  GS_REQUIRE(ctx && frames && cams, "gsc_rasterize_backward_batch: null argument");
  GS_REQUIRE(nviews >= 1 && nviews <= GSC_MAX_BATCH_VIEWS, "gsc_rasterize_backward_batch: nviews out of range");
  GS_TRY(check_gaussians(g));
  GS_TRY(check_grads(grads));
  for (int v = 0; v < nviews; v++) {
    const gsc_frame* f = frames[v];
    GS_REQUIRE(f && f->ctx == ctx && f->has_grad2d, "gsc_rasterize_backward_batch: frame without a backward");
    GS_TRY(check_view(&cams[v], cfg));
    GS_REQUIRE(f->n == g->count && cams[v].width == f->width && cams[v].height == f->height,
               "gsc_rasterize_backward_batch: gaussians/camera differ from the frame's forward");
  }
  if (cfg->mode != GSC_MODE_FULL) {  // the reference's per-view host loops
    for (int v = 0; v < nviews; v++)
      GS_TRY(do_preprocess_bwd(ctx, g, &cams[v], cfg, (const float*)frames[v]->grad2d.ptr, grads, nullptr));
    return GSC_OK;
  }
  PreprocessBwdArgs a;
  std::memset(&a, 0, sizeof a);
  a.n = g->count;
  a.pos = g->position; a.log_scale = g->log_scale; a.rot = g->rotation;
  a.logit_opacity = g->logit_opacity; a.sh = g->sh;
  a.cfg = *cfg;
  a.cam = cams[0];
  a.grad2d = (const float*)frames[0]->grad2d.ptr;
  a.nviews = nviews;
  for (int v = 0; v < nviews; v++) {
    a.cams[v] = cams[v];
    a.grad2d_v[v] = (const float*)frames[v]->grad2d.ptr;
  }
  a.g_pos = grads->position; a.g_log_scale = grads->log_scale; a.g_rot = grads->rotation;
  a.g_logit_opacity = grads->logit_opacity; a.g_sh = grads->sh;
#if GS_PBWD_COMPACT
  GS_TRY(scratch_reserve(ctx, preprocess_bwd_compact_scratch(g->count)));
  StageScope sc(ctx, GSC_STAGE_PREPROCESS_BWD);
  sc.kernels(g->count ? 2 : 0);
  return launch_preprocess_bwd_compact(a, scratch_base(ctx), ctx->num_sms, ctx->stream);
#else
  StageScope sc(ctx, GSC_STAGE_PREPROCESS_BWD);
  sc.kernels(g->count ? 1 : 0);
  return launch_preprocess_bwd(a, true, ctx->stream);
#endif
}

GSC_API int gsc_frame_get(gsc_frame* f, int which, void** ptr, int64_t* count) {
  GS_REQUIRE(f && ptr, "gsc_frame_get: null argument");
  const int64_t npix = (int64_t)f->width * f->height;
  if (f->count_pending && (which == GSC_FRAME_KEYS || which == GSC_FRAME_VALUES)) {
    // the final lists' length, left on the device by the list build
    uint64_t cnt = 0;
    GS_TRY(read_u64(f->ctx, (const uint64_t*)f->total.ptr, &cnt));
    f->num_keys = (int64_t)cnt;
    f->count_pending = false;
  }
  void* p = nullptr;
  int64_t c = 0;
  switch (which) {
    case GSC_FRAME_SPLATS: p = f->splats.ptr; c = f->n * 12; break;
    case GSC_FRAME_KEYS:
      if (!f->keys_valid) {
        GS_TRY(ensure(f->ctx, &f->keys, (size_t)f->num_keys * 8 + 8));
        GS_TRY(launch_make_keys_ranges((const uint32_t*)f->ranges.ptr, f->tiles_x * f->tiles_y,
                                       (const uint32_t*)f->vals.ptr, (const float*)f->splats.ptr,
                                       (uint64_t*)f->keys.ptr, f->ctx->stream));
        f->keys_valid = true;
      }
      p = f->keys.ptr;
      c = f->num_keys;
      break;
    case GSC_FRAME_VALUES: p = f->vals.ptr; c = f->num_keys; break;
    case GSC_FRAME_RANGES: p = f->ranges.ptr; c = (int64_t)f->tiles_x * f->tiles_y * 2; break;
    case GSC_FRAME_IMAGE: p = f->image_ptr; c = npix * 3; break;
    case GSC_FRAME_FINAL_T: p = f->final_T.ptr; c = npix; break;
    case GSC_FRAME_LAST: p = f->last.ptr; c = npix; break;
    case GSC_FRAME_N_CONTRIB: p = f->n_contrib.ptr; c = npix; break;
    case GSC_FRAME_GRAD2D: p = f->grad2d.ptr; c = f->n * 9; break;
    default: set_error("gsc_frame_get: unknown item"); return GSC_ERR_INVALID;
  }
  *ptr = p;
  if (count) *count = c;
  return GSC_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Tracing
// ---------------------------------------------------------------------------
namespace gs {

static cudaEvent_t take_event(gsc_ctx* ctx) {
  if (!ctx->ev_pool.empty()) {
    cudaEvent_t e = ctx->ev_pool.back();
    ctx->ev_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return e;
}

StageScope::StageScope(gsc_ctx* c, int s) : ctx(c), stage(s) {
  ctx->calls[stage]++;
  if (ctx->profiling) {
    a = take_event(ctx);
    if (a) cudaEventRecord(a, ctx->stream);
  }
}

StageScope::~StageScope() {
  if (!a) return;
  cudaEvent_t b = take_event(ctx);
  if (!b) return;
  cudaEventRecord(b, ctx->stream);
  ctx->marks.push_back({stage, a, b});
}

void StageScope::kernels(int k) {
  ctx->kernels += k;
  ctx->stage_kernels[stage] += k;
}

}  // namespace gs

extern "C" {

GSC_API int gsc_profile_enable(gsc_ctx* ctx, int on) {
  GS_REQUIRE(ctx, "gsc_profile_enable: null context");
  ctx->profiling = on != 0;
  return GSC_OK;
}

GSC_API int gsc_profile_read(gsc_ctx* ctx, double* ms, int64_t* calls, int64_t* kernels, int reset) {
  GS_REQUIRE(ctx, "gsc_profile_read: null context");
  GS_CK(cudaStreamSynchronize(ctx->stream));
  for (auto& m : ctx->marks) {
    float t = 0.0f;
    if (cudaEventElapsedTime(&t, m.a, m.b) == cudaSuccess) ctx->ms[m.stage] += t;
    else cudaGetLastError();
    ctx->ev_pool.push_back(m.a);
    ctx->ev_pool.push_back(m.b);
  }
  ctx->marks.clear();
  for (int s = 0; s < GSC_STAGE_COUNT; s++) {
    if (ms) ms[s] = ctx->ms[s];
    if (calls) calls[s] = ctx->calls[s];
    if (kernels) kernels[s] = ctx->stage_kernels[s];
    if (reset) {
      ctx->ms[s] = 0.0;
      ctx->calls[s] = 0;
      ctx->stage_kernels[s] = 0;
    }
  }
  return GSC_OK;
}

GSC_API int64_t gsc_kernel_count(gsc_ctx* ctx) { return ctx ? ctx->kernels : 0; }

GSC_API int gsc_profile_pairs(gsc_ctx* ctx, uint64_t* out, int reset) {
  GS_REQUIRE(ctx && out, "gsc_profile_pairs: null argument");
  GS_CK(cudaMemcpyAsync(ctx->pinned, ctx->err + 4, 16, cudaMemcpyDeviceToHost, ctx->stream));
  GS_CK(cudaStreamSynchronize(ctx->stream));
  uint64_t dev[2];
  std::memcpy(dev, ctx->pinned, 16);
  out[0] = ctx->prof_binned + dev[0];
  out[1] = ctx->prof_kept + dev[1];
  if (reset) {
    GS_CK(cudaMemsetAsync(ctx->err + 4, 0, 16, ctx->stream));
    GS_CK(cudaStreamSynchronize(ctx->stream));
    ctx->prof_binned = ctx->prof_kept = 0;
  }
  return GSC_OK;
}

GSC_API int gsc_profile_pge(gsc_ctx* ctx, uint64_t* out, int reset) {
  GS_REQUIRE(ctx && out, "gsc_profile_pge: null argument");
  GS_CK(cudaMemcpyAsync(ctx->pinned, ctx->err + 2, 8, cudaMemcpyDeviceToHost, ctx->stream));
  GS_CK(cudaStreamSynchronize(ctx->stream));
  std::memcpy(out, ctx->pinned, 8);
  if (reset) {
    GS_CK(cudaMemsetAsync(ctx->err + 2, 0, 8, ctx->stream));
    GS_CK(cudaStreamSynchronize(ctx->stream));
  }
  return GSC_OK;
}

}  // extern "C"
