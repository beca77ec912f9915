/*
 * gsplat_cuda.h — C ABI of libgsplat_cuda.so, the sm_100a (B200) Gaussian-splatting
 * rasterizer hot path of crystal-gausplat.
 *
 * The library replaces, for this path only, the Metal backend that the Crystal
 * host reaches through its `lib` FFI blocks:
 *   src/core/buffer.cr:201-211      (lib MetalFFI: buffers)
 *   src/metal/device.cr:205-231     (lib MetalDeviceFFI: device, queue)
 *   src/metal/dispatch.cr:237-254   (lib MetalDispatchFFI: encoders, dispatch)
 *   src/metal/bridge.mm:361-482     (extern "C" gs_* implementation)
 * and the kernels they launch (src/metal/kernels/gaussian.metal,
 * src/metal/kernels/radix_sort.metal) plus the host loops on the same path
 * (src/gaussian_splatting/rasterizer.cr:375-460, src/optim/adam.cr:127-176,
 * src/ops/loss.cr:33-57).
 *
 * Conventions
 *  - Every entry point returns GSC_OK (0) or a negative GSC_ERR_* code; the
 *    message of the last failure on the calling thread is gsc_last_error().
 *    No C++ exception crosses this boundary.
 *  - All array pointers are DEVICE pointers owned by the caller (from
 *    gsc_alloc, cudaMalloc or a torch tensor) unless a parameter says "host".
 *    Layouts are the reference's: row-major fp32, u64 keys, u32 ids,
 *    u32 tile ranges [T,2] (src/gaussian_splatting/rasterizer_context.cr:17-36).
 *  - Work is enqueued asynchronously on the context's stream (gsc_set_stream);
 *    gsc_sync() waits and reports device-side errors (bounded spin timeouts).
 *  - One gsc_ctx per device per host thread; a context is not thread-safe.
 */
#ifndef GSPLAT_CUDA_H
#define GSPLAT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define GSC_API __attribute__((visibility("default")))
#else
#define GSC_API
#endif

#define GSC_VERSION 1

/* ---- status codes ---------------------------------------------------- */
#define GSC_OK 0
#define GSC_ERR_INVALID (-1)  /* bad argument (null pointer, negative size, ...) */
#define GSC_ERR_CUDA (-2)     /* a CUDA runtime call failed */
#define GSC_ERR_CAPACITY (-3) /* output buffer too small (e.g. key capacity) */
#define GSC_ERR_TIMEOUT (-4)  /* a bounded device-side wait gave up */
#define GSC_ERR_NOMEM (-5)    /* device allocation failed */
#define GSC_ERR_NODEVICE (-6) /* no CUDA device / device index out of range */
#define GSC_ERR_UNSUPPORTED (-7)

/* ---- arithmetic modes -------------------------------------------------
 * GSC_MODE_FULL : mathematically complete 3DGS forward/backward with the
 *                 reference's constants: SH evaluated to cfg.sh_degree (<= 3),
 *                 normalised quaternions, analytic gradients for all 59
 *                 floats per Gaussian.
 * GSC_MODE_REF  : the reference's literal per-thread arithmetic:
 *                 truncated SH (gaussian.metal:283-302), quaternion as given,
 *                 backward over the whole tile list with the reference's
 *                 running-colour update (gaussian.metal:503-566), host chain
 *                 of rasterizer.cr:375-460 (position via the mean only, DC
 *                 SH gradient dL/dc / C0, nothing for scale/rotation/cov2d). */
#define GSC_MODE_FULL 0
#define GSC_MODE_REF 1

/* Camera block. Byte-for-byte the reference's CameraParamsGPU
 * (src/gaussian_splatting/rasterizer.cr:467-500, 176 bytes, packed), so the
 * Crystal host can keep build_camera_params (rasterizer.cr:502-531).
 * view: world_to_camera, ROW-major (camera.cr:185-187): x_cam = view[0..3]·[p,1].
 * proj is carried for layout compatibility and not read. */
typedef struct gsc_camera {
  float view[16];
  float proj[16];
  float fx, fy, cx, cy;
  int32_t width, height;
  float tan_fov_x, tan_fov_y; /* tan of half field of view (camera.cr:39-45) */
  float campos[3];            /* camera centre in world space (camera.cr:133-137) */
  float _pad;
} gsc_camera;

/* Rasterizer constants. gsc_raster_config_default() fills the reference
 * values (gaussian.metal:160,174,227-228,400,425-426; trainer.cr:186). */
typedef struct gsc_raster_config {
  int32_t mode;      /* GSC_MODE_FULL or GSC_MODE_REF */
  int32_t sh_degree; /* 0..3, reference SH_DEGREE = 3 (gaussian.cr:14) */
  float t_stop;      /* stop while T > t_stop fails: 1e-3 */
  float alpha_min;   /* skip alpha < alpha_min: 1/255 */
  float alpha_max;   /* alpha = min(alpha_max, o*G): 0.99 */
  float lowpass;     /* added to the cov2d diagonal: 0.3 */
  float fov_cull;    /* cull |x/z| > fov_cull * tan_fov_x: 1.3 */
  float near_z;      /* cull z <= near_z: 0.01 */
  float far_z;       /* cull z > far_z: 1000 */
  float background[3];
  int32_t binning;   /* GSC_BIN_*: tile lists of the whole-view calls (default OCCLUDED) */
} gsc_raster_config;

/* Tile lists built by gsc_rasterize_forward. REFERENCE: every tile of each
 * Gaussian's square 3-sigma rectangle (create_tile_keys,
 * gaussian.metal:315-357), bit-identical to the reference's sorted keys,
 * values and ranges. CONTRIBUTING: the same lists without the (tile,
 * Gaussian) pairs that the exact whole-tile test proves can never pass the
 * alpha test at any pixel of the tile (Gaussians with more than 64 tiles keep
 * all of theirs); images, n_contrib, final_T and gradients are bit-identical
 * to REFERENCE, with fewer pairs to emit, sort and scan. The stage entry
 * point gsc_bin always builds the reference lists. */
#define GSC_BIN_REFERENCE 0
#define GSC_BIN_CONTRIBUTING 1
/* OCCLUDED: the contributing lists binned and composited in slices of the
 * depth order; a Gaussian all of whose tiles are already opaque (every pixel
 * stopped at T <= t_stop in an earlier slice) is not binned. The frame's
 * final lists are, per tile, the contributing list up to the largest `last`
 * of the tile's pixels (the entries the backward reads). Images, n_contrib,
 * final_T, last and gradients are bit-identical to CONTRIBUTING and
 * REFERENCE; *num_rendered reports the contributing pairs before occlusion
 * and gsc_frame_get's count the final lists. */
#define GSC_BIN_OCCLUDED 2

/* The trainable state of Gaussian3D (src/gaussian_splatting/gaussian.cr:19-37):
 * position [N,3], log_scale [N,3], rotation [N,4] (w,x,y,z),
 * logit_opacity [N,1], sh_coeffs [N,16,3] (coefficient-major, channel-minor). */
typedef struct gsc_gaussians {
  const float* position;
  const float* log_scale;
  const float* rotation;
  const float* logit_opacity;
  const float* sh;
  int64_t count;
} gsc_gaussians;

/* Gradients with the same shapes as gsc_gaussians; kernels ACCUMULATE (+=)
 * into them, so the caller zeroes them once per step (Variable#zero_grad!,
 * src/autograd/variable.cr:86-88). d_logit_opacity is dL/dlogit
 * (trainer.cr:234-241 sigmoid chain applied). */
typedef struct gsc_gaussian_grads {
  float* position;
  float* log_scale;
  float* rotation;
  float* logit_opacity;
  float* sh;
} gsc_gaussian_grads;

/* Per-view outputs of preprocess. `splats` is required (12 floats per
 * Gaussian, private packed layout used by binning and compositing); every
 * other pointer may be NULL. They mirror RasterizerContext
 * (rasterizer_context.cr:17-23): mean2d [N,2], cov2d [N,3] (xx,xy,yy, with
 * the low-pass), conic [N,3] (inverse cov2d: xx,xy,yy), depth [N],
 * radius [N], colors [N,3], opacity [N], tiles_touched [N] (u32), cov3d [N,6]. */
typedef struct gsc_projected {
  float* splats;
  float* mean2d;
  float* cov2d;
  float* conic;
  float* depth;
  float* radius;
  float* colors;
  float* opacity;
  uint32_t* tiles_touched;
  float* cov3d;
} gsc_projected;

/* Per-Gaussian screen-space gradients in the reference's RasterizerGradients
 * shapes (rasterizer_context.cr:133-140). Any pointer may be NULL. */
typedef struct gsc_grads2d {
  float* mean2d;  /* [N,2] */
  float* cov2d;   /* [N,3] (zero in GSC_MODE_REF, as gaussian.metal:464 never writes it) */
  float* opacity; /* [N]   dL/d(sigmoid opacity) */
  float* colors;  /* [N,3] */
} gsc_grads2d;

/* One Adam parameter group (src/optim/adam.cr:86-110 loops over these). */
typedef struct gsc_adam_group {
  float* param;
  const float* grad;
  float* m;
  float* v;
  int64_t numel;
  float lr;
  float weight_decay; /* decoupled (AdamW), 0 = plain Adam (adam.cr:112-125) */
} gsc_adam_group;

/* ---- context ---------------------------------------------------------- */
GSC_API int gsc_version(void);
GSC_API const char* gsc_last_error(void);
GSC_API void gsc_raster_config_default(gsc_raster_config* cfg);

typedef struct gsc_ctx gsc_ctx;
typedef struct gsc_frame gsc_frame;

/* Replaces gs_init_device (bridge.mm:17-49): 0 ok, GSC_ERR_NODEVICE. */
GSC_API int gsc_init(int device, gsc_ctx** out);
GSC_API int gsc_destroy(gsc_ctx* ctx);
/* Use `stream` (a cudaStream_t; NULL = legacy default) for all later work. */
GSC_API int gsc_set_stream(gsc_ctx* ctx, void* stream);
/* Wait for the stream; returns GSC_ERR_TIMEOUT if a device wait gave up. */
GSC_API int gsc_sync(gsc_ctx* ctx);

/* Failure-path self-test, with no counterpart in the reference: runs the
 * sort's bounded look-back wait (the only device-side wait on the
 * single-GPU path) against a predecessor that never publishes, so the wait
 * gives up after spin_limit (1..100000) re-reads and the kernel finishes;
 * the next gsc_sync returns GSC_ERR_TIMEOUT and clears the flag, and the
 * context stays usable. */
GSC_API int gsc_selftest_wait_timeout(gsc_ctx* ctx, int32_t spin_limit);

/* ---- memory (replaces gs_create_buffer / gs_buffer_* , bridge.mm:131-146) */
GSC_API int gsc_alloc(gsc_ctx* ctx, size_t bytes, void** out);
GSC_API int gsc_free(gsc_ctx* ctx, void* ptr);
GSC_API int gsc_memcpy_h2d(gsc_ctx* ctx, void* dst, const void* host_src, size_t bytes);
GSC_API int gsc_memcpy_d2h(gsc_ctx* ctx, void* host_dst, const void* src, size_t bytes);
GSC_API int gsc_memset(gsc_ctx* ctx, void* dst, int value, size_t bytes);

/* ---- stages ----------------------------------------------------------- */

/* Fused compute_cov3d + project_gaussians + eval_sh + opacity sigmoid + tile
 * count (gaussian.metal:90-308, gaussian.cr:119-142). One thread per Gaussian. */
GSC_API int gsc_preprocess(gsc_ctx* ctx, const gsc_gaussians* g, const gsc_camera* cam,
                           const gsc_raster_config* cfg, const gsc_projected* out);

/* create_tile_keys (gaussian.metal:315-357) with exact allocation: a scan of
 * tiles_touched, then each Gaussian writes its keys in canonical order
 * (Gaussian id, then ty, then tx). key = tile_id << 32 | float_bits(depth),
 * value = Gaussian id. *num_keys (host) receives the total; GSC_ERR_CAPACITY
 * if it exceeds `capacity` (nothing is written then). */
GSC_API int gsc_bin(gsc_ctx* ctx, int64_t n, const float* splats, int32_t tiles_x, int32_t tiles_y,
                    uint64_t* keys, uint32_t* values, int64_t capacity, int64_t* num_keys);

/* GPURadixSort.sort!(keys, values, n) (src/metal/gpu_radix_sort.cr:46-57):
 * in-place STABLE ascending sort of (u64 key, u32 value) pairs by the key
 * bits [begin_bit, end_bit) (0, 64 = whole key). Onesweep LSD radix,
 * 8-bit digits. Scratch comes from the context. */
GSC_API int gsc_sort_pairs_u64(gsc_ctx* ctx, uint64_t* keys, uint32_t* values, int64_t n,
                               int begin_bit, int end_bit);

/* Allocation-free variant of gsc_sort_pairs_u64, with no counterpart in the
 * reference. For callers that cannot allocate device memory (a host whose own
 * pool owns all device memory, a thread that must not take the driver's
 * allocation locks, a caller without a gsc_ctx): same stable sort and
 * arguments, but the scratch is a fixed device array inside the library
 * (about 3.7 MB per GPU, held until exit), so n <= GSC_STATIC_SORT_MAX_PAIRS;
 * larger n returns GSC_ERR_INVALID. Work is queued on `stream` (a
 * cudaStream_t, NULL = legacy default). The first call on a device may load
 * the library's device code (CUDA lazy loading), which reserves the array,
 * and looks up its address once: make it during initialisation, outside
 * real-time threads and before any stream capture. cudaDeviceReset is not
 * supported while the library is in use. All calls share the array: calls
 * whose GPU work overlaps race. */
#define GSC_STATIC_SORT_MAX_PAIRS 262144
GSC_API int gsc_sort_pairs_u64_static(uint64_t* keys, uint32_t* values, int64_t n, int begin_bit,
                                      int end_bit, void* stream);
/* Device-side status of the last gsc_sort_pairs_u64_static on this device
 * (no reference counterpart, no allocation): waits for `stream`, then returns
 * GSC_OK, GSC_ERR_TIMEOUT (a bounded look-back wait gave up) or GSC_ERR_CUDA
 * (a bounds check failed), and clears the status. The output of a sort whose
 * status is not GSC_OK is not sorted. */
GSC_API int gsc_sort_pairs_u64_static_status(void* stream);

/* GPURadixSort.compute_tile_ranges! (gpu_radix_sort.cr:204-233,
 * radix_sort.metal:288-324): ranges[t] = [first, last+1) of tile t in the
 * sorted keys, (0,0) for empty tiles. */
GSC_API int gsc_tile_ranges(gsc_ctx* ctx, const uint64_t* sorted_keys, int64_t n, int32_t num_tiles,
                            uint32_t* ranges);

/* rasterize_tile (gaussian.metal:364-445) over every 16x16 tile.
 * image [H,W,3]; n_contrib [H,W] u32 (Gaussians that contributed);
 * final_T [H,W]; last [H,W] u32 (tile-list position after the last
 * contributor, for the backward; may be NULL in GSC_MODE_REF). */
GSC_API int gsc_composite_forward(gsc_ctx* ctx, const float* splats, const uint32_t* values,
                                  const uint32_t* ranges, int32_t width, int32_t height,
                                  const gsc_raster_config* cfg, float* image, uint32_t* n_contrib,
                                  float* final_T, uint32_t* last);

/* rasterize_backward (gaussian.metal:452-567). Accumulates into grad2d
 * [N,9] = (dmean.x, dmean.y, dconic.xx, dconic.xy, dconic.yy, dopacity,
 * dcolor.r, dcolor.g, dcolor.b). If `target` is non-NULL the pixel gradient
 * is the L1 gradient sign(image - target) * l1_scale (loss.cr:33-57, fused)
 * and dL_dimage is ignored; `loss_sum` (device float, may be NULL) then
 * receives += sum |image - target| * l1_scale. */
GSC_API int gsc_composite_backward(gsc_ctx* ctx, const float* splats, const uint32_t* values,
                                   const uint32_t* ranges, int32_t width, int32_t height,
                                   const gsc_raster_config* cfg, const float* dL_dimage,
                                   const float* image, const float* target, float l1_scale,
                                   const float* final_T, const uint32_t* last, float* grad2d,
                                   float* loss_sum);

/* project_backward! + sh_backward! + covariance_backward! + the sigmoid chain
 * (rasterizer.cr:375-460, trainer.cr:218-255), as one kernel. Reads grad2d
 * [N,9] from gsc_composite_backward, accumulates into `grads` and writes the
 * optional screen-space views into `g2d`. */
GSC_API int gsc_preprocess_backward(gsc_ctx* ctx, const gsc_gaussians* g, const gsc_camera* cam,
                                    const gsc_raster_config* cfg, const float* grad2d,
                                    const gsc_gaussian_grads* grads, const gsc_grads2d* g2d);

/* Loss.l1_with_grad (src/ops/loss.cr:33-57): grad = sign(pred - target) * scale,
 * *loss_sum (device) += sum |pred - target| * scale. scale = 1/numel matches
 * the reference. */
GSC_API int gsc_l1_loss_grad(gsc_ctx* ctx, const float* pred, const float* target, int64_t numel,
                             float scale, float* grad, float* loss_sum);

/* Adam#step (src/optim/adam.cr:86-176) over all groups in one launch.
 * `step` is the 1-based step count after increment (AdamState#step);
 * every gradient is multiplied by grad_scale first (1/views for a view mean). */
GSC_API int gsc_adam_step(gsc_ctx* ctx, const gsc_adam_group* groups, int32_t ngroups, float beta1,
                          float beta2, float eps, int32_t step, float grad_scale);

/* Data-parallel exchange + optimiser step for view-sharded training, with no
 * reference counterpart (the reference trains one view at a time on one
 * device, trainer.cr:178-215). One kernel per rank: for its 1/nranks shard of
 * the flat parameter arena it sums the ranks' gradient arenas with NVLink
 * peer loads (rank order 0..nranks-1), applies Adam#step to the shard
 * (adam.cr:127-176) and stores the new parameters into every rank's
 * parameter arena with peer stores. It replaces all-reduce + a replicated
 * Adam. All pointers must be device pointers valid in this process (peer
 * pointers from CUDA IPC or symmetric memory); every rank's gradients must be
 * complete before the call and the peers must not read parameters until every
 * rank's call has finished (the caller fences both with a cross-rank
 * barrier). Groups are [offset, offset + numel) float ranges of the arenas;
 * offsets must be multiples of 4.
 * mc_grads / mc_params (optional, both or neither): NVLink multicast
 * addresses of the gradient and parameter arenas (an NVSwitch multicast
 * object bound to every rank's arena, e.g. torch symmetric memory's
 * multicast_ptr), 16-byte aligned. With them the shard's gradient sum is one
 * multimem.ld_reduce per float4 (the switch adds the ranks' values in fp32,
 * in an order of its own) and each new parameter float4 is one multimem.st
 * that lands in every replica: per NVLink direction a rank moves
 * (1 + 1/nranks) arenas instead of 2 (nranks - 1)/nranks. */
#define GSC_DP_MAX_RANKS 8
typedef struct gsc_dp_adam_args {
  int32_t nranks;
  int32_t rank;
  float* peer_grads[GSC_DP_MAX_RANKS];
  float* peer_params[GSC_DP_MAX_RANKS];
  float* m; /* this rank's first-moment arena (only its shard is read/written) */
  float* v; /* this rank's second-moment arena */
  int32_t ngroups;
  int64_t offset[8];
  int64_t numel[8];
  float lr[8];
  float weight_decay[8];
  float beta1, beta2, eps;
  int32_t step;
  float grad_scale;
  float* mc_grads;
  float* mc_params;
} gsc_dp_adam_args;
GSC_API int gsc_dp_adam_step(gsc_ctx* ctx, const gsc_dp_adam_args* args);

/* Cross-rank barrier for the fused exchange (no reference counterpart; it
 * replaces an unbounded device barrier). peer_flags[p] is rank p's array of
 * nranks uint32 words in peer-addressable memory (CUDA IPC or symmetric
 * memory), zero-initialised once. Rank `rank` publishes `epoch` into slot
 * `rank` of every peer's array after a system-scope fence (its earlier writes
 * become visible to the peers first), then waits until every peer's slot of
 * its own array has reached `epoch`. Every rank passes the same epoch, one
 * greater on each call. The wait is bounded by timeout_us (1 .. 600e6): on
 * expiry the kernel sets the context's timeout flag and returns, a
 * following gsc_dp_adam_step skips its work (no peer memory is touched), and
 * gsc_sync returns GSC_ERR_TIMEOUT. nranks == 1 is a no-op. */
typedef struct gsc_dp_barrier_args {
  int32_t nranks;
  int32_t rank;
  uint32_t* peer_flags[GSC_DP_MAX_RANKS];
  uint32_t epoch;
  int32_t timeout_us;
} gsc_dp_barrier_args;
GSC_API int gsc_dp_barrier(gsc_ctx* ctx, const gsc_dp_barrier_args* args);

/* ---- losses beyond L1 (src/ops/loss.cr:59-249) --------------------------
 * Images are [height, width, channels] fp32 row-major, 1 <= channels <= 4.
 * `out` is a DEVICE array of 3 floats: {loss, mean |pred - target|, SSIM}.
 * SSIM (Loss.ssim, loss.cr:117-186) is the mean over the valid region (pixels
 * at least window/2 from every border) and channels of the local SSIM with a
 * Gaussian window of sigma 1.5 and C1 = 0.01^2, C2 = 0.03^2; 0 when the image
 * has no valid pixel. GSC_MODE_REF evaluates it literally (2D window,
 * two-pass variance); GSC_MODE_FULL applies the same window separably.
 * Partial sums are double and reduced in a fixed order. */

/* Loss.ssim_loss_with_grad (loss.cr:189-216): loss = 1 - SSIM. grad
 * (nullable, written): REF = the reference's surrogate 2 (pred - target) / n;
 * FULL = the exact gradient of 1 - SSIM. ssim_map (nullable, [H, W, C]) gets
 * the per-pixel SSIM on the valid region; other entries are left as they are. */
GSC_API int gsc_ssim_loss_grad(gsc_ctx* ctx, const float* pred, const float* target,
                               int32_t height, int32_t width, int32_t channels,
                               int32_t window_size, int32_t mode, float* grad, float* ssim_map,
                               float* out);

/* Loss.combined_with_grad (loss.cr:227-249), window 11: loss =
 * (1 - lambda) * L1 + lambda * (1 - SSIM); grad (nullable, written) =
 * (1 - lambda) * sign(pred - target) / n + lambda * d(1 - SSIM) (as above). */
GSC_API int gsc_combined_loss_grad(gsc_ctx* ctx, const float* pred, const float* target,
                                   int32_t height, int32_t width, int32_t channels,
                                   float lambda_ssim, int32_t mode, float* grad, float* out);

/* Loss.mse_with_grad (loss.cr:83-105): out[0] = out[1] = mean (pred - target)^2,
 * grad (nullable, written) = 2 (pred - target) / numel. Loss.psnr
 * (loss.cr:291-296) is 10 log10(max^2 / out[0]) on the host. */
GSC_API int gsc_mse_loss_grad(gsc_ctx* ctx, const float* pred, const float* target,
                              int64_t numel, float* grad, float* out);

/* ---- training targets from 8-bit images ---------------------------------
 * ImageIO.resize (src/utils/image_io.cr:289-335: bilinear, pixel centres,
 * clamped, each value clamped to [0, 255] and truncated to a byte) to
 * width x height when the sizes differ, then Image#to_tensor's byte / 255
 * (image_io.cr:83-97), keeping the first `channels` of `src_channels`
 * (RGBA -> RGB). src: device [src_height, src_width, src_channels] u8;
 * dst: device [height, width, channels] fp32. */
GSC_API int gsc_image_to_target(gsc_ctx* ctx, const uint8_t* src, int32_t src_width,
                                int32_t src_height, int32_t src_channels, float* dst,
                                int32_t width, int32_t height, int32_t channels);

/* ---- densification (Trainer#densify_and_prune!, trainer.cr:293-392) ---- */

/* GradientAccumulator#accumulate (trainer.cr:86-99): for every i,
 * accum[i] += |dL/dmean2d_i| and count[i] += 1. Row i of dmean2d starts at
 * dmean2d + i * stride (stride 2 for an [N,2] array, 9 for a frame's grad2d). */
GSC_API int gsc_grad_accumulate(gsc_ctx* ctx, const float* dmean2d, int32_t stride, int64_t n,
                                float* accum, int32_t* count);

#define GSC_DENSIFY_CLONE 1u
#define GSC_DENSIFY_SPLIT 2u
#define GSC_DENSIFY_PRUNE 4u

/* The decisions of densify_and_prune! (trainer.cr:296-325): average gradient
 * accum/count (0 when count is 0) above grad_threshold -> split if the largest
 * exp(log_scale) exceeds size_threshold, else clone; sigmoid(logit) below
 * opacity_threshold -> prune. flags[i] gets GSC_DENSIFY_* bits (a split
 * Gaussian is never also kept). counts (host, 3 values) = {kept originals,
 * clones, splits}; the new set has kept + clones + 2 * splits Gaussians.
 * As Gaussian3D#remove! (gaussian.cr:233-235), a plan that would leave no
 * Gaussian prunes none. */
GSC_API int gsc_densify_plan(gsc_ctx* ctx, const gsc_gaussians* g, const float* accum,
                             const int32_t* count, float grad_threshold, float size_threshold,
                             float opacity_threshold, uint8_t* flags, int64_t* counts);

/* Output parameter arrays of a new Gaussian set (same layouts as gsc_gaussians). */
typedef struct gsc_gaussians_out {
  float* position;
  float* log_scale;
  float* rotation;
  float* logit_opacity;
  float* sh;
} gsc_gaussians_out;

/* Builds the densified set in the order [kept originals][clones][first split
 * halves][second split halves], every group in original index order (the
 * reference's concat!/remove! order, with its pruning applied to the original
 * indices). Clones: position += (U - 0.5) * 2 * clone_noise per axis
 * (trainer.cr:375-386). Split halves: log_scale -= ln_split (ln 1.6 in the
 * reference), position += exp(new log_scale.x) * 0.5 * (+1 | -1) * (U - 0.5)
 * per axis (trainer.cr:332-370). U in [0,1) is a counter-based hash of
 * (seed, index, draw), identical on every device and in the CPU oracle. */
GSC_API int gsc_densify_apply(gsc_ctx* ctx, const gsc_gaussians* g, const uint8_t* flags,
                              const gsc_gaussians_out* out, float clone_noise, float ln_split,
                              uint64_t seed);

/* Gaussian3D#reset_opacity! (gaussian.cr:269-271): logit_opacity[i] = value. */
GSC_API int gsc_reset_opacity(gsc_ctx* ctx, float* logit_opacity, int64_t n, float value);

/* ---- whole-view orchestration (Rasterizer.forward/backward,
 *      src/gaussian_splatting/rasterizer.cr:48-104) ----------------------- */

/* A frame holds the per-view state kept between forward and backward
 * (RasterizerContext): splats, keys, values, ranges, per-pixel final_T / last,
 * the rendered image and grad2d. Buffers grow on demand and are reused. */
GSC_API int gsc_frame_create(gsc_ctx* ctx, gsc_frame** out);
GSC_API int gsc_frame_destroy(gsc_frame* frame);

/* Per-tile depth cut for occluded binning (GSC_BIN_OCCLUDED), no reference
 * counterpart: `cut` is a DEVICE array of `count` floats owned by the caller,
 * one per view (pass NULL to unbind); it must stay allocated while bound, and
 * a forward whose tiles_x * tiles_y exceeds `count` fails with
 * GSC_ERR_INVALID before any work. Every occluded forward on
 * this frame while it is bound rewrites it with the view's next cut: for
 * each tile whose pixels all stopped, 1.005 x the depth of the last list
 * entry any of its pixels used, else +inf. With `valid` nonzero the forward
 * reads it: the first slice holds, per tile, the pairs of Gaussians in front
 * of the tile's cut, and the second slice the remaining pairs of the tiles
 * whose pixels did not all stop. Each tile's list is then still its depth
 * order cut at its saturation point, so images, per-pixel outputs, lists and
 * gradients are the same bit for bit whatever the cut holds. Only the work
 * changes: a cut from the same view's previous forward (training revisits
 * its views) leaves the first slice close to the pairs that are kept. The
 * binding is per frame; a caller that renders several views on one frame
 * binds each view's array before its forward. */
GSC_API int gsc_frame_set_tile_hint(gsc_frame* frame, float* cut, int64_t count, int32_t valid);

/* preprocess -> bin -> sort -> ranges -> composite. `image` [H,W,3] may be
 * NULL (the frame's own buffer is used); n_contrib / final_T may be NULL.
 * *num_rendered (host, may be NULL) = number of keys (ctx.num_rendered). */
GSC_API int gsc_rasterize_forward(gsc_ctx* ctx, gsc_frame* frame, const gsc_gaussians* g,
                                  const gsc_camera* cam, const gsc_raster_config* cfg, float* image,
                                  uint32_t* n_contrib, float* final_T, int64_t* num_rendered);

/* gsc_rasterize_forward of up to GSC_MAX_BATCH_VIEWS views of one image size
 * into distinct frames, with one preprocess pass over the Gaussians for all of
 * them (parameters read once) and one host readback of the pair counts.
 * images[k] (or images itself) may be NULL: frame k's own image buffer.
 * num_rendered (host, may be NULL) gets nviews counts. Results are those of
 * the single-view call, bit for bit. */
GSC_API int gsc_rasterize_forward_batch(gsc_ctx* ctx, gsc_frame* const* frames, const gsc_camera* cams,
                                        int32_t nviews, const gsc_gaussians* g,
                                        const gsc_raster_config* cfg, float* const* images,
                                        int64_t* num_rendered);

/* Largest number of views gsc_rasterize_backward_batch sums in one pass. */
#define GSC_MAX_BATCH_VIEWS 8

/* composite backward -> preprocess backward for the frame's last forward.
 * Exactly one of dL_dimage / target is non-NULL (target = fused L1 with
 * l1_scale, loss accumulated into the device float *loss_sum if non-NULL).
 * Gradients accumulate into `grads`; `g2d` (may be NULL) gets screen-space views. */
GSC_API int gsc_rasterize_backward(gsc_ctx* ctx, gsc_frame* frame, const gsc_gaussians* g,
                                   const gsc_camera* cam, const gsc_raster_config* cfg,
                                   const float* dL_dimage, const float* target, float l1_scale,
                                   float* loss_sum, const gsc_gaussian_grads* grads,
                                   const gsc_grads2d* g2d);

/* With grads == NULL, gsc_rasterize_backward stops after the composite
 * backward and leaves the screen-space gradients (GSC_FRAME_GRAD2D) in the
 * frame. gsc_rasterize_backward_batch then runs the preprocess backward of
 * up to GSC_MAX_BATCH_VIEWS such frames in one pass: each Gaussian's
 * parameters and gradient row are read once and the views' contributions are
 * summed before they are added to `grads` (equal to calling the single-view
 * backward per frame up to the order of the fp32 sums). cams[k] is frame k's
 * camera; g and cfg are those of the frames' forwards. */
GSC_API int gsc_rasterize_backward_batch(gsc_ctx* ctx, gsc_frame* const* frames, const gsc_camera* cams,
                                         int32_t nviews, const gsc_gaussians* g,
                                         const gsc_raster_config* cfg, const gsc_gaussian_grads* grads);

/* Frame internals (device pointers, valid until the next forward on the frame). */
#define GSC_FRAME_SPLATS 0
#define GSC_FRAME_KEYS 1
#define GSC_FRAME_VALUES 2
#define GSC_FRAME_RANGES 3
#define GSC_FRAME_IMAGE 4
#define GSC_FRAME_FINAL_T 5
#define GSC_FRAME_LAST 6
#define GSC_FRAME_N_CONTRIB 7
#define GSC_FRAME_GRAD2D 8
GSC_API int gsc_frame_get(gsc_frame* frame, int which, void** ptr, int64_t* count);

/* ---- tracing (no reference counterpart: the reference times whole
 *      self-test loops with Time.instant, src/main.cr:871-1061) -----------
 * When enabled, every stage brackets its kernels with CUDA events on the
 * context's stream; gsc_profile_read syncs the stream and returns, per
 * stage, the summed device milliseconds, the number of stage invocations
 * and the number of kernels launched. */
#define GSC_STAGE_PREPROCESS 0
#define GSC_STAGE_SCAN 1
#define GSC_STAGE_EMIT 2
#define GSC_STAGE_SORT 3
#define GSC_STAGE_RANGES 4
#define GSC_STAGE_COMPOSITE_FWD 5
#define GSC_STAGE_COMPOSITE_BWD 6
#define GSC_STAGE_PREPROCESS_BWD 7
#define GSC_STAGE_ADAM 8
#define GSC_STAGE_L1 9
#define GSC_STAGE_COUNT 10
GSC_API int gsc_profile_enable(gsc_ctx* ctx, int on);
GSC_API int gsc_profile_read(gsc_ctx* ctx, double* ms, int64_t* calls, int64_t* kernels, int reset);
/* Kernels launched by this context since creation (counted whether or not
 * profiling is on). */
GSC_API int64_t gsc_kernel_count(gsc_ctx* ctx);
/* Pixel-Gaussian evaluations counted by whole-view forwards while profiling
 * was enabled: per pixel, the tile-list entries up to the transmittance stop
 * (the whole list if the pixel never stopped). */
GSC_API int gsc_profile_pge(gsc_ctx* ctx, uint64_t* out, int reset);
/* (Tile, Gaussian) pairs of whole-view forwards while profiling was enabled:
 * out[0] = pairs emitted and sorted (with GSC_BIN_OCCLUDED, what the depth
 * slices binned), out[1] = pairs kept in the frames' final lists. */
GSC_API int gsc_profile_pairs(gsc_ctx* ctx, uint64_t* out, int reset);

#ifdef __cplusplus
}
#endif
#endif /* GSPLAT_CUDA_H */
