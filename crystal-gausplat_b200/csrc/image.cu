// image.cu — 8-bit images to fp32 training targets on the device: the
// bilinear resize of ImageIO.resize (src/utils/image_io.cr:289-335), rounded
// back to bytes as there, fused with Image#to_tensor's byte / 255
// (image_io.cr:83-97) and a channel selection (RGBA -> RGB). Only the bytes
// cross PCIe; one thread per output pixel, all channels.
#include "common.cuh"
#include "kernels.cuh"

namespace gs {

struct ImageArgs {
  const uint8_t* src;
  int sw, sh, sc;
  float* dst;
  int dw, dh, dc;
  float scale_x, scale_y;
};

__global__ void __launch_bounds__(256) image_to_target_kernel(ImageArgs a) {
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= (int64_t)a.dw * a.dh) return;
  const int x = (int)(i % a.dw), y = (int)(i / a.dw);
  float* out = a.dst + i * a.dc;
  if (a.sw == a.dw && a.sh == a.dh) {  // ImageIO.resize returns the image unchanged
    const uint8_t* p = a.src + i * a.sc;
    for (int c = 0; c < a.dc; c++) out[c] = (float)p[c] / 255.0f;
    return;
  }
  float sx = ((float)x + 0.5f) * a.scale_x - 0.5f;
  float sy = ((float)y + 0.5f) * a.scale_y - 0.5f;
  sx = fminf(fmaxf(sx, 0.0f), (float)(a.sw - 1));
  sy = fminf(fmaxf(sy, 0.0f), (float)(a.sh - 1));
  const int x0 = min(max((int)sx, 0), a.sw - 1), y0 = min(max((int)sy, 0), a.sh - 1);
  const int x1 = min(x0 + 1, a.sw - 1), y1 = min(y0 + 1, a.sh - 1);
  const float fx = sx - (float)x0, fy = sy - (float)y0;
  const uint8_t* r0 = a.src + (int64_t)y0 * a.sw * a.sc;
  const uint8_t* r1 = a.src + (int64_t)y1 * a.sw * a.sc;
  for (int c = 0; c < a.dc; c++) {
    const float v00 = r0[x0 * a.sc + c], v10 = r0[x1 * a.sc + c];
    const float v01 = r1[x0 * a.sc + c], v11 = r1[x1 * a.sc + c];
    const float v0 = v00 * (1.0f - fx) + v10 * fx;
    const float v1 = v01 * (1.0f - fx) + v11 * fx;
    const float v = v0 * (1.0f - fy) + v1 * fy;
    const uint8_t b = (uint8_t)fminf(fmaxf(v, 0.0f), 255.0f);  // clamp, then truncate
    out[c] = (float)b / 255.0f;
  }
}

}  // namespace gs

using namespace gs;

extern "C" {

GSC_API int gsc_image_to_target(gsc_ctx* ctx, const uint8_t* src, int32_t src_width, int32_t src_height,
                                int32_t src_channels, float* dst, int32_t width, int32_t height,
                                int32_t channels) {
  GS_REQUIRE(ctx && src && dst, "gsc_image_to_target: null pointer");
  GS_REQUIRE(src_width > 0 && src_height > 0 && width > 0 && height > 0, "gsc_image_to_target: empty image");
  GS_REQUIRE(src_channels >= 1 && src_channels <= 4 && channels >= 1 && channels <= src_channels,
             "gsc_image_to_target: channels must satisfy 1 <= channels <= src_channels <= 4");
  ImageArgs a;
  a.src = src; a.sw = src_width; a.sh = src_height; a.sc = src_channels;
  a.dst = dst; a.dw = width; a.dh = height; a.dc = channels;
  a.scale_x = (float)src_width / (float)width;
  a.scale_y = (float)src_height / (float)height;
  const int64_t n = (int64_t)width * height;
  image_to_target_kernel<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(a);
  GS_CK_LAUNCH("image_to_target_kernel");
  return GSC_OK;
}

}  // extern "C"
