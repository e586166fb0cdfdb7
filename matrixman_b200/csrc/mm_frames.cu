// Frame preprocessing on the device: uint8 BGR frames -> the model's float32
// NCHW input, as the reference prepares each frame on the CPU
// (demo/yolo_helpers.py:53-56): cv2.resize(INTER_LINEAR) to the model size,
// BGR -> RGB, CHW, float32 / 255.
//
// The resize is OpenCV's 8-bit bilinear fixed-point algorithm (OpenCV 4.x, the
// cv2 the reference calls), restated: per output column dx the source
// coordinate fx = (float)((dx + 0.5) * scale_x - 0.5) (double arithmetic, then
// float), sx = floor(fx), fx -= sx; columns left of the image or at/after its
// last column clamp to it with fx = 0; weights round((1 - fx) * 2048) and
// round(fx * 2048) (round half to even).  Rows use the same weights without
// the clamp (the two source rows are clamped to the image instead).  The
// horizontal pass sums S[sx] * a0 + S[sx + 1] * a1 in integers; the vertical
// pass combines two such rows as
//   ((b0 * (h0 >> 4)) >> 16) + ((b1 * (h1 >> 4)) >> 16) + 2) >> 2,
// saturated to 0..255.  scale_x = 1 / (out_w / in_w) in double.
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "mm_common.cuh"

namespace mm {

struct ResizeTap {
  int s0, s1, w0, w1;
};

__device__ __forceinline__ ResizeTap resize_tap(int d, double scale, int n, bool clamp_weight) {
  const float f0 = (float)__dsub_rn(__dmul_rn((double)d + 0.5, scale), 0.5);
  int s = (int)floorf(f0);
  float f = __fsub_rn(f0, (float)s);
  if (clamp_weight) {
    if (s < 0) {
      f = 0.f;
      s = 0;
    }
    if (s >= n - 1) {
      f = 0.f;
      s = n - 1;
    }
  }
  ResizeTap t;
  t.w0 = __float2int_rn(__fmul_rn(__fsub_rn(1.f, f), 2048.f));
  t.w1 = __float2int_rn(__fmul_rn(f, 2048.f));
  t.s0 = min(max(s, 0), n - 1);
  t.s1 = min(max(s + 1, 0), n - 1);
  return t;
}

__global__ void preprocess_bgr8_kernel(const uint8_t* __restrict__ frames, int64_t n, int h, int w,
                                       float* __restrict__ out, int64_t os0, int64_t os1, int64_t os2,
                                       int64_t os3, int oh, int ow, double scale_x, double scale_y) {
  const int64_t total = n * oh * ow;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int dx = (int)(i % ow);
    const int64_t t = i / ow;
    const int dy = (int)(t % oh);
    const int64_t img = t / oh;
    const ResizeTap tx = resize_tap(dx, scale_x, w, true);
    const ResizeTap ty = resize_tap(dy, scale_y, h, false);
    const uint8_t* f = frames + img * (int64_t)h * w * 3;
    const uint8_t* r0 = f + (int64_t)ty.s0 * w * 3;
    const uint8_t* r1 = f + (int64_t)ty.s1 * w * 3;
    float* o = out + img * os0 + dy * os2 + dx * os3;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const int h0 = r0[tx.s0 * 3 + c] * tx.w0 + r0[tx.s1 * 3 + c] * tx.w1;
      const int h1 = r1[tx.s0 * 3 + c] * tx.w0 + r1[tx.s1 * 3 + c] * tx.w1;
      int v = (((ty.w0 * (h0 >> 4)) >> 16) + ((ty.w1 * (h1 >> 4)) >> 16) + 2) >> 2;
      v = v < 0 ? 0 : (v > 255 ? 255 : v);
      o[(2 - c) * os1] = __fdiv_rn((float)v, 255.f);  // BGR -> RGB
    }
  }
}

}  // namespace mm

using namespace mm;

extern "C" int mm_preprocess_bgr8(const uint8_t* frames, int64_t n, int64_t h, int64_t w,
                                  const mm_tensor_t* out, void* stream) {
  int rc;
  if ((rc = validate(out, "mm_preprocess_bgr8 output", MM_F32)) != MM_OK) return rc;
  if (n < 0 || h <= 0 || w <= 0 || h > 0x7fffffffLL || w > 0x7fffffffLL)
    return fail(MM_ERR_INVALID, "mm_preprocess_bgr8: bad frame size");
  if (out->ndim != 4 || out->size[0] != n || out->size[1] != 3 || out->size[2] <= 0 || out->size[3] <= 0)
    return fail(MM_ERR_INVALID, "mm_preprocess_bgr8: output must be [N, 3, out_h, out_w]");
  if (out->size[2] > 0x7fffffffLL || out->size[3] > 0x7fffffffLL)
    return fail(MM_ERR_UNSUPPORTED, "mm_preprocess_bgr8: output too large");
  if (n == 0) return MM_OK;
  if (frames == nullptr) return fail(MM_ERR_INVALID, "mm_preprocess_bgr8: null frames");
  const int oh = (int)out->size[2], ow = (int)out->size[3];
  const double scale_x = 1.0 / ((double)ow / (double)w);
  const double scale_y = 1.0 / ((double)oh / (double)h);
  const int64_t total = n * oh * ow;
  cudaStream_t s = resolve_stream(stream);
  preprocess_bgr8_kernel<<<grid_for(total, 256, (int64_t)sm_count() * 16), 256, 0, s>>>(
      frames, n, (int)h, (int)w, (float*)out->data, out->stride[0], out->stride[1], out->stride[2],
      out->stride[3], oh, ow, scale_x, scale_y);
  MM_LAUNCH_CHECK("mm_preprocess_bgr8 launch");
  return MM_OK;
}
