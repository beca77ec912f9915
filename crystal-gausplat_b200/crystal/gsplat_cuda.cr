# gsplat_cuda.cr -- the Crystal `lib` binding of libgsplat_cuda.so
# (include/gsplat_cuda.h), for the reference's host code.
#
# A maintainer drops this file into src/gaussian_splatting/ of
# skuznetsov/crystal-gausplat and routes the rasterizer path to it instead of
# the Metal FFI blocks it replaces for this path:
#   src/core/buffer.cr:201-211      lib MetalFFI           (buffers)
#   src/metal/device.cr:205-231     lib MetalDeviceFFI     (device, queue)
#   src/metal/dispatch.cr:237-254   lib MetalDispatchFFI   (encoders, dispatch)
#   src/gaussian_splatting/rasterizer.cr:28-45  (the kernel names it dispatches)
#   src/metal/gpu_radix_sort.cr:26-40           (the sort pipelines it builds)
# Every `fun` below has the name, argument count and argument types of the
# C declaration (checked against the header by tests/test_crystal_binding.py).
# Device pointers are plain pointers; allocate with `alloc` or any CUDA
# allocator.

@[Link(ldflags: "-L#{__DIR__}/../../crystal-gausplat_b200 -lgsplat_cuda -Wl,-rpath,#{__DIR__}/../../crystal-gausplat_b200")]
lib GSCuda
  OK               =  0
  ERR_INVALID      = -1
  ERR_CUDA         = -2
  ERR_CAPACITY     = -3
  ERR_TIMEOUT      = -4
  ERR_NOMEM        = -5
  ERR_NODEVICE     = -6
  ERR_UNSUPPORTED  = -7

  MODE_FULL        = 0
  MODE_REF         = 1
  BIN_REFERENCE    = 0
  BIN_CONTRIBUTING = 1
  BIN_OCCLUDED     = 2
  MAX_BATCH_VIEWS  = 8
  DP_MAX_RANKS     = 8
  STATIC_SORT_MAX_PAIRS = 262144

  FRAME_SPLATS    = 0
  FRAME_KEYS      = 1
  FRAME_VALUES    = 2
  FRAME_RANGES    = 3
  FRAME_IMAGE     = 4
  FRAME_FINAL_T   = 5
  FRAME_LAST      = 6
  FRAME_N_CONTRIB = 7
  FRAME_GRAD2D    = 8

  DENSIFY_CLONE = 1_u32
  DENSIFY_SPLIT = 2_u32
  DENSIFY_PRUNE = 4_u32

  # Byte-for-byte the reference's packed CameraParamsGPU (rasterizer.cr:467-500).
  @[Packed]
  struct Camera
    view : StaticArray(Float32, 16)
    proj : StaticArray(Float32, 16)
    fx : Float32
    fy : Float32
    cx : Float32
    cy : Float32
    width : Int32
    height : Int32
    tan_fov_x : Float32
    tan_fov_y : Float32
    campos : StaticArray(Float32, 3)
    pad : Float32
  end

  struct RasterConfig
    mode : Int32
    sh_degree : Int32
    t_stop : Float32
    alpha_min : Float32
    alpha_max : Float32
    lowpass : Float32
    fov_cull : Float32
    near_z : Float32
    far_z : Float32
    background : StaticArray(Float32, 3)
    binning : Int32
  end

  struct Gaussians
    position : Float32*
    log_scale : Float32*
    rotation : Float32*
    logit_opacity : Float32*
    sh : Float32*
    count : Int64
  end

  struct GaussianGrads
    position : Float32*
    log_scale : Float32*
    rotation : Float32*
    logit_opacity : Float32*
    sh : Float32*
  end

  struct Projected
    splats : Float32*
    mean2d : Float32*
    cov2d : Float32*
    conic : Float32*
    depth : Float32*
    radius : Float32*
    colors : Float32*
    opacity : Float32*
    tiles_touched : UInt32*
    cov3d : Float32*
  end

  struct Grads2D
    mean2d : Float32*
    cov2d : Float32*
    opacity : Float32*
    colors : Float32*
  end

  struct AdamGroup
    param : Float32*
    grad : Float32*
    m : Float32*
    v : Float32*
    numel : Int64
    lr : Float32
    weight_decay : Float32
  end

  struct DpAdamArgs
    nranks : Int32
    rank : Int32
    peer_grads : StaticArray(Float32*, 8)
    peer_params : StaticArray(Float32*, 8)
    m : Float32*
    v : Float32*
    ngroups : Int32
    offset : StaticArray(Int64, 8)
    numel : StaticArray(Int64, 8)
    lr : StaticArray(Float32, 8)
    weight_decay : StaticArray(Float32, 8)
    beta1 : Float32
    beta2 : Float32
    eps : Float32
    step : Int32
    grad_scale : Float32
    mc_grads : Float32*
    mc_params : Float32*
  end

  struct DpBarrierArgs
    nranks : Int32
    rank : Int32
    peer_flags : StaticArray(UInt32*, 8)
    epoch : UInt32
    timeout_us : Int32
  end

  struct GaussiansOut
    position : Float32*
    log_scale : Float32*
    rotation : Float32*
    logit_opacity : Float32*
    sh : Float32*
  end

  type Ctx = Void*
  type Frame = Void*

  # context (gs_init_device, bridge.mm:17-49)
  fun version = gsc_version : Int32
  fun last_error = gsc_last_error : UInt8*
  fun config_default = gsc_raster_config_default(cfg : RasterConfig*) : Void
  fun init = gsc_init(device : Int32, out : Ctx*) : Int32
  fun destroy = gsc_destroy(ctx : Ctx) : Int32
  fun set_stream = gsc_set_stream(ctx : Ctx, stream : Void*) : Int32
  fun sync = gsc_sync(ctx : Ctx) : Int32
  fun selftest_wait_timeout = gsc_selftest_wait_timeout(ctx : Ctx, spin_limit : Int32) : Int32

  # memory (gs_create_buffer / gs_buffer_*, bridge.mm:131-146)
  fun alloc = gsc_alloc(ctx : Ctx, bytes : LibC::SizeT, out : Void**) : Int32
  fun free = gsc_free(ctx : Ctx, ptr : Void*) : Int32
  fun memcpy_h2d = gsc_memcpy_h2d(ctx : Ctx, dst : Void*, host_src : Void*, bytes : LibC::SizeT) : Int32
  fun memcpy_d2h = gsc_memcpy_d2h(ctx : Ctx, host_dst : Void*, src : Void*, bytes : LibC::SizeT) : Int32
  fun memset = gsc_memset(ctx : Ctx, dst : Void*, value : Int32, bytes : LibC::SizeT) : Int32

  # stages (gaussian.metal kernels, radix_sort.metal, gpu_radix_sort.cr)
  fun preprocess = gsc_preprocess(ctx : Ctx, g : Gaussians*, cam : Camera*, cfg : RasterConfig*,
                                  out : Projected*) : Int32
  fun bin = gsc_bin(ctx : Ctx, n : Int64, splats : Float32*, tiles_x : Int32, tiles_y : Int32,
                    keys : UInt64*, values : UInt32*, capacity : Int64, num_keys : Int64*) : Int32
  fun sort_pairs_u64 = gsc_sort_pairs_u64(ctx : Ctx, keys : UInt64*, values : UInt32*, n : Int64,
                                          begin_bit : Int32, end_bit : Int32) : Int32
  fun sort_pairs_u64_static = gsc_sort_pairs_u64_static(keys : UInt64*, values : UInt32*, n : Int64,
                                                        begin_bit : Int32, end_bit : Int32,
                                                        stream : Void*) : Int32
  fun sort_pairs_u64_static_status = gsc_sort_pairs_u64_static_status(stream : Void*) : Int32
  fun tile_ranges = gsc_tile_ranges(ctx : Ctx, sorted_keys : UInt64*, n : Int64, num_tiles : Int32,
                                    ranges : UInt32*) : Int32
  fun composite_forward = gsc_composite_forward(ctx : Ctx, splats : Float32*, values : UInt32*,
                                                ranges : UInt32*, width : Int32, height : Int32,
                                                cfg : RasterConfig*, image : Float32*,
                                                n_contrib : UInt32*, final_t : Float32*,
                                                last : UInt32*) : Int32
  fun composite_backward = gsc_composite_backward(ctx : Ctx, splats : Float32*, values : UInt32*,
                                                  ranges : UInt32*, width : Int32, height : Int32,
                                                  cfg : RasterConfig*, dl_dimage : Float32*,
                                                  image : Float32*, target : Float32*,
                                                  l1_scale : Float32, final_t : Float32*,
                                                  last : UInt32*, grad2d : Float32*,
                                                  loss_sum : Float32*) : Int32
  fun preprocess_backward = gsc_preprocess_backward(ctx : Ctx, g : Gaussians*, cam : Camera*,
                                                    cfg : RasterConfig*, grad2d : Float32*,
                                                    grads : GaussianGrads*, g2d : Grads2D*) : Int32
  fun l1_loss_grad = gsc_l1_loss_grad(ctx : Ctx, pred : Float32*, target : Float32*, numel : Int64,
                                      scale : Float32, grad : Float32*, loss_sum : Float32*) : Int32
  fun adam_step = gsc_adam_step(ctx : Ctx, groups : AdamGroup*, ngroups : Int32, beta1 : Float32,
                                beta2 : Float32, eps : Float32, step : Int32,
                                grad_scale : Float32) : Int32
  fun dp_adam_step = gsc_dp_adam_step(ctx : Ctx, args : DpAdamArgs*) : Int32
  fun dp_barrier = gsc_dp_barrier(ctx : Ctx, args : DpBarrierArgs*) : Int32

  # losses (loss.cr:59-296)
  fun ssim_loss_grad = gsc_ssim_loss_grad(ctx : Ctx, pred : Float32*, target : Float32*,
                                          height : Int32, width : Int32, channels : Int32,
                                          window_size : Int32, mode : Int32, grad : Float32*,
                                          ssim_map : Float32*, out : Float32*) : Int32
  fun combined_loss_grad = gsc_combined_loss_grad(ctx : Ctx, pred : Float32*, target : Float32*,
                                                  height : Int32, width : Int32, channels : Int32,
                                                  lambda_ssim : Float32, mode : Int32,
                                                  grad : Float32*, out : Float32*) : Int32
  fun mse_loss_grad = gsc_mse_loss_grad(ctx : Ctx, pred : Float32*, target : Float32*, numel : Int64,
                                        grad : Float32*, out : Float32*) : Int32

  # training targets (image_io.cr:83-97, 289-335)
  fun image_to_target = gsc_image_to_target(ctx : Ctx, src : UInt8*, src_width : Int32,
                                            src_height : Int32, src_channels : Int32,
                                            dst : Float32*, width : Int32, height : Int32,
                                            channels : Int32) : Int32

  # densification (trainer.cr:86-99, 293-392; gaussian.cr:269-271)
  fun grad_accumulate = gsc_grad_accumulate(ctx : Ctx, dmean2d : Float32*, stride : Int32, n : Int64,
                                            accum : Float32*, count : Int32*) : Int32
  fun densify_plan = gsc_densify_plan(ctx : Ctx, g : Gaussians*, accum : Float32*, count : Int32*,
                                      grad_threshold : Float32, size_threshold : Float32,
                                      opacity_threshold : Float32, flags : UInt8*,
                                      counts : Int64*) : Int32
  fun densify_apply = gsc_densify_apply(ctx : Ctx, g : Gaussians*, flags : UInt8*,
                                        out : GaussiansOut*, clone_noise : Float32,
                                        ln_split : Float32, seed : UInt64) : Int32
  fun reset_opacity = gsc_reset_opacity(ctx : Ctx, logit_opacity : Float32*, n : Int64,
                                        value : Float32) : Int32

  # whole-view calls (Rasterizer.forward / .backward, rasterizer.cr:48-104)
  fun frame_create = gsc_frame_create(ctx : Ctx, out : Frame*) : Int32
  fun frame_destroy = gsc_frame_destroy(frame : Frame) : Int32
  fun frame_set_tile_hint = gsc_frame_set_tile_hint(frame : Frame, cut : Float32*, count : Int64, valid : Int32) : Int32
  fun rasterize_forward = gsc_rasterize_forward(ctx : Ctx, frame : Frame, g : Gaussians*,
                                                cam : Camera*, cfg : RasterConfig*, image : Float32*,
                                                n_contrib : UInt32*, final_t : Float32*,
                                                num_rendered : Int64*) : Int32
  fun rasterize_forward_batch = gsc_rasterize_forward_batch(ctx : Ctx, frames : Frame*, cams : Camera*,
                                                            nviews : Int32, g : Gaussians*,
                                                            cfg : RasterConfig*, images : Float32**,
                                                            num_rendered : Int64*) : Int32
  # grads = nil: stop after the compositing backward (screen-space gradients stay in the frame)
  fun rasterize_backward = gsc_rasterize_backward(ctx : Ctx, frame : Frame, g : Gaussians*,
                                                  cam : Camera*, cfg : RasterConfig*,
                                                  dl_dimage : Float32*, target : Float32*,
                                                  l1_scale : Float32, loss_sum : Float32*,
                                                  grads : GaussianGrads*, g2d : Grads2D*) : Int32
  fun rasterize_backward_batch = gsc_rasterize_backward_batch(ctx : Ctx, frames : Frame*,
                                                              cams : Camera*, nviews : Int32,
                                                              g : Gaussians*, cfg : RasterConfig*,
                                                              grads : GaussianGrads*) : Int32
  fun frame_get = gsc_frame_get(frame : Frame, which : Int32, ptr : Void**, count : Int64*) : Int32

  # tracing
  fun profile_enable = gsc_profile_enable(ctx : Ctx, on : Int32) : Int32
  fun profile_read = gsc_profile_read(ctx : Ctx, ms : Float64*, calls : Int64*, kernels : Int64*,
                                      reset : Int32) : Int32
  fun kernel_count = gsc_kernel_count(ctx : Ctx) : Int64
  fun profile_pge = gsc_profile_pge(ctx : Ctx, out : UInt64*, reset : Int32) : Int32
  fun profile_pairs = gsc_profile_pairs(ctx : Ctx, out : UInt64*, reset : Int32) : Int32
end
