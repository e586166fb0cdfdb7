// tcgen05 3xTF32 implicit-GEMM convolution (placeholder until the kernel lands).
#include "mm_common.cuh"

using namespace mm;

extern "C" int mm_conv2d_tc(const mm_tensor_t* x, const float* w_hi, const float* w_lo, int k_out,
                            int c_in, int r, int s, int c_pad, int k_pad, const float* bias,
                            const mm_tensor_t* residual, const mm_conv_params_t* p,
                            const mm_tensor_t* y, void* stream) {
  return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: tensor-core path not built");
}
