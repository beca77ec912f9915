/*
 * gs_oracle.h — CPU restatement of crystal-gausplat's rasterizer hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for libgsplat_cuda.so:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load it. The product path never calls it.
 *
 * Parity is UNPINNED by the reference itself: the reference is Crystal +
 * Metal (macOS only), has no CPU rasterizer (rasterizer.cr:54,87 raise without
 * Metal) and ships no golden vectors for this path. This oracle restates the
 * per-thread arithmetic of src/metal/kernels/gaussian.metal and the host math
 * of src/gaussian_splatting/ (*.cr), src/optim/adam.cr and src/ops/loss.cr, and is
 * pinned by known-answer tests and float64 finite differences (tests/).
 *
 * Floating point: IEEE fp32, no contraction (-ffp-contract=off), IEEE
 * division and sqrt, and gso_expf (below) instead of libm expf, so the fp32
 * results of the documented operation order are reproducible bit for bit.
 */
#ifndef GS_ORACLE_H
#define GS_ORACLE_H
#include <stdint.h>
#include "../include/gsplat_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* exp(x) in fp32: Cody–Waite reduction by ln 2 (hi/lo split), degree-7
 * Taylor polynomial in Horner form with fused multiply-adds, scale by 2^k. */
float gso_expf(float x);

/* The reference's rasterizer constants (same values as gsc_raster_config_default). */
void gso_raster_config_default(gsc_raster_config* cfg);

void gso_set_threads(int nthreads);
/* 1 (default): composite-backward sums accumulated in double, rounded once;
 * 0: added in fp32 as they come (the reference's atomics, some order). */
void gso_set_exact_sums(int on);

/* Fused preprocess. Any output may be NULL. */
void gso_preprocess(const gsc_gaussians* g, const gsc_camera* cam, const gsc_raster_config* cfg,
                    float* mean2d, float* cov2d, float* conic, float* depth, float* radius,
                    float* colors, float* opacity, uint32_t* tiles_touched, float* cov3d);

/* Canonical key emission; returns the key count, or -1 if > capacity
 * (keys/vals may be NULL to only count). */
int64_t gso_emit_keys(int64_t n, const float* mean2d, const float* depth, const float* radius,
                      int32_t tiles_x, int32_t tiles_y, uint64_t* keys, uint32_t* vals,
                      int64_t capacity);

/* Contributing-pairs binning (GSC_BIN_CONTRIBUTING): drops from sorted
 * reference lists every (tile, Gaussian) pair that the exact whole-tile test
 * rejects, except for Gaussians whose rectangle has more than 64 tiles; the
 * order of the rest is kept. Returns the number of pairs written. */
int64_t gso_contributing_lists(int32_t width, int32_t height, int64_t m, const uint64_t* keys,
                               const uint32_t* vals, const float* mean2d, const float* conic,
                               const float* opacity, const uint32_t* tiles_touched,
                               float alpha_min, uint64_t* out_keys, uint32_t* out_vals);

/* Stable ascending sort of (key, value) pairs by key bits [begin_bit, end_bit). */
void gso_sort_pairs(int64_t n, uint64_t* keys, uint32_t* vals, int begin_bit, int end_bit);

void gso_tile_ranges(int64_t n, const uint64_t* keys, int32_t num_tiles, uint32_t* ranges);

void gso_composite_forward(int32_t width, int32_t height, const uint32_t* ranges,
                           const uint32_t* vals, const float* mean2d, const float* cov2d,
                           const float* opacity, const float* colors,
                           const gsc_raster_config* cfg, float* image, uint32_t* n_contrib,
                           float* final_T, uint32_t* last);

/* rasterize_tile with the reference's literal expression forms (unfused
 * power and colour sums); the same arguments as gso_composite_forward
 * without `last`. */
void gso_composite_forward_literal(int32_t width, int32_t height, const uint32_t* ranges,
                                   const uint32_t* vals, const float* mean2d, const float* cov2d,
                                   const float* opacity, const float* colors,
                                   const gsc_raster_config* cfg, float* image, uint32_t* n_contrib,
                                   float* final_T);

/* grad2d [N,9] accumulated (+=). dL_dimage or (image, target, l1_scale). */
void gso_composite_backward(int32_t width, int32_t height, const uint32_t* ranges,
                            const uint32_t* vals, const float* mean2d, const float* cov2d,
                            const float* opacity, const float* colors,
                            const gsc_raster_config* cfg, const float* dL_dimage,
                            const float* image, const float* target, float l1_scale,
                            const float* final_T, const uint32_t* last, float* grad2d,
                            double* loss_sum);

void gso_preprocess_backward(const gsc_gaussians* g, const gsc_camera* cam,
                             const gsc_raster_config* cfg, const float* grad2d,
                             const gsc_gaussian_grads* grads, float* d_mean2d, float* d_cov2d,
                             float* d_opacity, float* d_colors);

void gso_l1_loss_grad(int64_t numel, const float* pred, const float* target, float scale,
                      float* grad, double* loss_sum);

/* beta^b as the reference's Float32#**(Int32) (binary exponentiation in fp32). */
float gso_powi_f32(float a, int32_t b);
void gso_adam_step(const gsc_adam_group* groups, int32_t ngroups, float beta1, float beta2,
                   float eps, int32_t step, float grad_scale);

/* Losses (loss.cr:59-249); same contract as gsc_ssim_loss_grad /
 * gsc_combined_loss_grad / gsc_mse_loss_grad, `out` a host array of 3. */
void gso_loss_grad(const float* pred, const float* target, int32_t height, int32_t width,
                   int32_t channels, int32_t window_size, int32_t mode, float w_l1, float w_ssim,
                   float* grad, float* ssim_map, float* out);
void gso_mse_loss_grad(const float* pred, const float* target, int64_t numel, float* grad,
                       float* out);

/* ImageIO.resize + Image#to_tensor (image_io.cr:83-97, 289-335); same
 * contract as gsc_image_to_target. */
void gso_image_to_target(const uint8_t* src, int32_t sw, int32_t sh, int32_t sc, float* dst,
                         int32_t dw, int32_t dh, int32_t dc);

/* Densification (trainer.cr:77-123, 293-392); same contract as
 * gsc_grad_accumulate / gsc_densify_plan / gsc_densify_apply. */
void gso_grad_accumulate(const float* dmean2d, int32_t stride, int64_t n, float* accum,
                         int32_t* count);
void gso_densify_plan(const gsc_gaussians* g, const float* accum, const int32_t* count,
                      float grad_threshold, float size_threshold, float opacity_threshold,
                      uint8_t* flags, int64_t* counts);
void gso_densify_apply(const gsc_gaussians* g, const uint8_t* flags, const gsc_gaussians_out* out,
                       float clone_noise, float ln_split, uint64_t seed);

/* Whole view: forward (and backward with fused L1 when target != NULL), on the
 * reference tile lists (images and gradients do not depend on the binning).
 * Allocates its own intermediates. Returns the number of keys. */
int64_t gso_render_view(const gsc_gaussians* g, const gsc_camera* cam,
                        const gsc_raster_config* cfg, float* image, const float* target,
                        float l1_scale, const gsc_gaussian_grads* grads, double* loss_sum);

#ifdef __cplusplus
}
#endif
#endif
