// Training-path kernels: the backward and optimiser ops of a small model's
// training step (ReLU / log-softmax / NLL backward, Adam's update), which the
// reference runs on its OpenGL backend only
// (drivers/matrixman/backends/opengl/dispatch.py:171-179 lerp_, :264-290
// addcmul_ / addcdiv_, :299 sqrt, :377-382 threshold_backward, :463-479
// log-softmax backward and NLL forward / backward).
//
// Arithmetic follows ATen's CPU kernels for float32 as they are compiled
// (their vectorised loops contract a multiply and an add into one FMA):
//   threshold_backward: self <= threshold ? 0 : grad
//   addcmul:  fma(value * t1, t2, self)
//   addcdiv:  self + (value * t1) / t2
//   lerp:     |w| < 0.5 ? fma(w, end - self, self) : fma(w - 1, end - self, end)
//   sqrt:     correctly rounded (torch's CPU sqrt is within 1 ulp of it)
//   log-softmax backward: grad - exp(output) * sum(grad along dim)
//   NLL: loss = -sum(w[t] * x[i, t]) (/ sum(w[t]) for the mean), ignored rows
//        skipped; gradient -(w[t]) * g (g / total_weight for the mean).
// Sums accumulate in double (ATen's CPU loops sum floats, so totals may differ
// in the last bits).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <string>

#include "mm_common.cuh"

namespace mm {

template <int OP>
__device__ __forceinline__ float pw3_apply(float x, float a, float b, float s) {
  if (OP == MM_PW3_THRESHOLD_BACKWARD) return a <= s ? 0.f : x;
  if (OP == MM_PW3_ADDCMUL) return __fmaf_rn(__fmul_rn(s, a), b, x);
  if (OP == MM_PW3_ADDCDIV) return __fadd_rn(x, __fdiv_rn(__fmul_rn(s, a), b));
  if (OP == MM_PW3_LERP) {
    const bool small = fabsf(s) < 0.5f;
    const float coeff = small ? s : __fsub_rn(s, 1.f);
    return __fmaf_rn(coeff, __fsub_rn(a, x), small ? x : a);
  }
  return __fsqrt_rn(x);  // MM_PW3_SQRT
}

// Not __restrict__: the in-place forms pass y == x.
template <int OP>
__global__ void pointwise3_kernel(const float* x, const float* a, const float* b, float* y, int64_t n,
                                  DevGeom gx, DevGeom ga, DevGeom gb, DevGeom gy, float s) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    y[dev_offset(i, gy)] = pw3_apply<OP>(x[dev_offset(i, gx)], a[dev_offset(i, ga)], b[dev_offset(i, gb)], s);
  }
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per (outer, inner) line of a contiguous [outer, len, inner] view.
__global__ void log_softmax_backward_kernel(const float* __restrict__ g, const float* __restrict__ o,
                                            float* __restrict__ y, int64_t lines, int64_t len,
                                            int64_t inner) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < lines; r += nwarps) {
    const int64_t outer = r / inner, in = r - outer * inner;
    const int64_t base = outer * len * inner + in;
    double sum = 0.0;
    for (int64_t k = lane; k < len; k += 32) sum += (double)g[base + k * inner];
    const float fs = (float)warp_sum(sum);
    for (int64_t k = lane; k < len; k += 32) {
      const int64_t idx = base + k * inner;
      y[idx] = __fsub_rn(g[idx], __fmul_rn(expf(o[idx]), fs));
    }
  }
}

struct NllArgs {
  const float* x;
  int64_t xs0, xs1;
  const int64_t* t;
  int64_t ts0;
  const float* w;  // null: every class weighs 1
  int64_t ws0;
  int64_t n, classes, ignore;
};

__device__ __forceinline__ bool nll_row(const NllArgs& a, int64_t i, int64_t* cls, float* wt) {
  const int64_t c = a.t[i * a.ts0];
  if (c == a.ignore || c < 0 || c >= a.classes) return false;  // range checked on the host
  *cls = c;
  *wt = a.w ? a.w[c * a.ws0] : 1.f;
  return true;
}

// reduction none: out[i] = -(w[t] * x[i, t]), 0 for an ignored row.
__global__ void nll_loss_rows_kernel(NllArgs a, float* __restrict__ out, int64_t os0) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < a.n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t c;
    float wt;
    out[i * os0] = nll_row(a, i, &c, &wt) ? -__fmul_rn(a.x[i * a.xs0 + c * a.xs1], wt) : 0.f;
  }
}

// reduction sum / mean: one block; total_weight = sum of w[t] over kept rows.
__global__ void nll_loss_total_kernel(NllArgs a, int mean, float* __restrict__ out,
                                      float* __restrict__ total) {
  __shared__ double sl[32], sw[32];
  double l = 0.0, wsum = 0.0;
  for (int64_t i = threadIdx.x; i < a.n; i += blockDim.x) {
    int64_t c;
    float wt;
    if (!nll_row(a, i, &c, &wt)) continue;
    l += (double)__fmul_rn(a.x[i * a.xs0 + c * a.xs1], wt);
    wsum += (double)wt;
  }
  l = warp_sum(l);
  wsum = warp_sum(wsum);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sl[warp] = l;
    sw[warp] = wsum;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    l = lane < nw ? sl[lane] : 0.0;
    wsum = lane < nw ? sw[lane] : 0.0;
    l = warp_sum(l);
    wsum = warp_sum(wsum);
    if (lane == 0) {
      const float tw = (float)wsum;
      float v = (float)(0.0 - l);  // +0 when nothing is summed, as ATen
      if (mean) v = __fdiv_rn(v, tw);
      out[0] = v;
      total[0] = tw;
    }
  }
}

// grad_input (zero-filled before) at [i, t[i]].
__global__ void nll_loss_backward_kernel(NllArgs a, int reduction, const float* __restrict__ go,
                                         int64_t gs0, const float* __restrict__ total,
                                         float* __restrict__ gi, int64_t gis0, int64_t gis1) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < a.n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t c;
    float wt;
    if (!nll_row(a, i, &c, &wt)) continue;
    float v;
    if (reduction == 0) {
      v = __fmul_rn(-wt, go[i * gs0]);
    } else {
      const float g = reduction == 1 ? __fdiv_rn(go[0], total[0]) : go[0];
      v = a.w ? __fmul_rn(wt, -g) : -g;
    }
    gi[i * gis0 + c * gis1] = v;
  }
}

static int nll_setup(const mm_tensor_t* x, const mm_tensor_t* t, const mm_tensor_t* w, int64_t ignore,
                     NllArgs* a, const char* who) {
  int rc;
  if ((rc = validate(x, who, MM_F32)) != MM_OK) return rc;
  if ((rc = validate(t, who, MM_I64)) != MM_OK) return rc;
  if (x->ndim != 2 || t->ndim != 1 || t->size[0] != x->size[0])
    return fail(MM_ERR_UNSUPPORTED, std::string(who) + ": input must be [N, C] and target [N]");
  a->x = (const float*)x->data;
  a->xs0 = x->stride[0];
  a->xs1 = x->stride[1];
  a->t = (const int64_t*)t->data;
  a->ts0 = t->stride[0];
  a->w = nullptr;
  a->ws0 = 0;
  if (w != nullptr) {
    if ((rc = validate(w, who, MM_F32)) != MM_OK) return rc;
    if (w->ndim != 1 || w->size[0] != x->size[1])
      return fail(MM_ERR_INVALID, std::string(who) + ": weight must be [C]");
    a->w = (const float*)w->data;
    a->ws0 = w->stride[0];
  }
  a->n = x->size[0];
  a->classes = x->size[1];
  a->ignore = ignore;
  return MM_OK;
}

}  // namespace mm

using namespace mm;

#define MM_VALIDATE(t, name, dt)     \
  do {                               \
    int _rc = validate(t, name, dt); \
    if (_rc != MM_OK) return _rc;    \
  } while (0)

extern "C" int mm_pointwise3(int op, const mm_tensor_t* x, const mm_tensor_t* a, const mm_tensor_t* b,
                             const mm_tensor_t* y, double scalar, void* stream) {
  MM_VALIDATE(x, "mm_pointwise3 self", MM_F32);
  MM_VALIDATE(a, "mm_pointwise3 operand 1", MM_F32);
  MM_VALIDATE(b, "mm_pointwise3 operand 2", MM_F32);
  MM_VALIDATE(y, "mm_pointwise3 output", MM_F32);
  const mm_tensor_t* ops[4] = {x, a, b, y};
  Geom g[4];
  int rc = collapse(4, ops, g);
  if (rc != MM_OK) return rc;
  const int64_t n = numel(y);
  if (n == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  const unsigned grid = grid_for(n, 256, (int64_t)sm_count() * 8);
  const float fs = (float)scalar;
#define MM_PW3_CASE(OP)                                                                     \
  case OP:                                                                                  \
    pointwise3_kernel<OP><<<grid, 256, 0, s>>>((const float*)x->data, (const float*)a->data, \
                                               (const float*)b->data, (float*)y->data, n,   \
                                               to_dev(g[0]), to_dev(g[1]), to_dev(g[2]),    \
                                               to_dev(g[3]), fs);                           \
    break;
  switch (op) {
    MM_PW3_CASE(MM_PW3_THRESHOLD_BACKWARD)
    MM_PW3_CASE(MM_PW3_ADDCMUL)
    MM_PW3_CASE(MM_PW3_ADDCDIV)
    MM_PW3_CASE(MM_PW3_LERP)
    MM_PW3_CASE(MM_PW3_SQRT)
    default:
      return fail(MM_ERR_UNSUPPORTED, "mm_pointwise3: unknown op " + std::to_string(op));
  }
#undef MM_PW3_CASE
  MM_LAUNCH_CHECK("mm_pointwise3 launch");
  return MM_OK;
}

extern "C" int mm_log_softmax_backward(const mm_tensor_t* grad, const mm_tensor_t* output, int dim,
                                       const mm_tensor_t* y, void* stream) {
  MM_VALIDATE(grad, "mm_log_softmax_backward grad", MM_F32);
  MM_VALIDATE(output, "mm_log_softmax_backward output", MM_F32);
  MM_VALIDATE(y, "mm_log_softmax_backward result", MM_F32);
  const int nd = y->ndim;
  if (dim < 0 || dim >= (nd ? nd : 1)) return fail(MM_ERR_INVALID, "mm_log_softmax_backward: dim out of range");
  const mm_tensor_t* ts[3] = {grad, output, y};
  for (const mm_tensor_t* t : ts) {
    if (t->ndim != nd) return fail(MM_ERR_INVALID, "mm_log_softmax_backward: shapes differ");
    int64_t expect = 1;
    for (int i = nd - 1; i >= 0; --i) {
      if (t->size[i] != y->size[i]) return fail(MM_ERR_INVALID, "mm_log_softmax_backward: shapes differ");
      if (t->size[i] != 1 && t->stride[i] != expect)
        return fail(MM_ERR_UNSUPPORTED, "mm_log_softmax_backward: operands must be contiguous");
      expect *= t->size[i];
    }
  }
  int64_t outer = 1, inner = 1;
  const int64_t len = nd ? y->size[dim] : 1;
  for (int i = 0; i < dim; ++i) outer *= y->size[i];
  for (int i = dim + 1; i < nd; ++i) inner *= y->size[i];
  const int64_t lines = outer * inner;
  if (lines == 0 || len == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  const unsigned grid = grid_for(lines * 32, 256, (int64_t)sm_count() * 8);
  log_softmax_backward_kernel<<<grid, 256, 0, s>>>((const float*)grad->data, (const float*)output->data,
                                                   (float*)y->data, lines, len, inner);
  MM_LAUNCH_CHECK("mm_log_softmax_backward launch");
  return MM_OK;
}

extern "C" int mm_nll_loss(const mm_tensor_t* input, const mm_tensor_t* target, const mm_tensor_t* weight,
                           int reduction, int64_t ignore_index, const mm_tensor_t* out,
                           const mm_tensor_t* total_weight, void* stream) {
  NllArgs a;
  int rc = nll_setup(input, target, weight, ignore_index, &a, "mm_nll_loss");
  if (rc != MM_OK) return rc;
  MM_VALIDATE(out, "mm_nll_loss output", MM_F32);
  if (reduction < 0 || reduction > 2) return fail(MM_ERR_INVALID, "mm_nll_loss: reduction must be 0, 1 or 2");
  cudaStream_t s = resolve_stream(stream);
  if (reduction == 0) {
    if (out->ndim != 1 || out->size[0] != a.n) return fail(MM_ERR_INVALID, "mm_nll_loss: output must be [N]");
    if (a.n == 0) return MM_OK;
    nll_loss_rows_kernel<<<grid_for(a.n, 256, (int64_t)sm_count() * 8), 256, 0, s>>>(a, (float*)out->data,
                                                                                      out->stride[0]);
  } else {
    MM_VALIDATE(total_weight, "mm_nll_loss total_weight", MM_F32);
    if (numel(out) != 1 || numel(total_weight) != 1)
      return fail(MM_ERR_INVALID, "mm_nll_loss: output and total_weight must hold one value");
    nll_loss_total_kernel<<<1, 1024, 0, s>>>(a, reduction == 1, (float*)out->data, (float*)total_weight->data);
  }
  MM_LAUNCH_CHECK("mm_nll_loss launch");
  return MM_OK;
}

extern "C" int mm_nll_loss_backward(const mm_tensor_t* grad_output, const mm_tensor_t* input,
                                    const mm_tensor_t* target, const mm_tensor_t* weight, int reduction,
                                    int64_t ignore_index, const mm_tensor_t* total_weight,
                                    const mm_tensor_t* grad_input, void* stream) {
  NllArgs a;
  int rc = nll_setup(input, target, weight, ignore_index, &a, "mm_nll_loss_backward");
  if (rc != MM_OK) return rc;
  MM_VALIDATE(grad_output, "mm_nll_loss_backward grad_output", MM_F32);
  MM_VALIDATE(grad_input, "mm_nll_loss_backward grad_input", MM_F32);
  if (reduction < 0 || reduction > 2)
    return fail(MM_ERR_INVALID, "mm_nll_loss_backward: reduction must be 0, 1 or 2");
  if (grad_input->ndim != 2 || grad_input->size[0] != a.n || grad_input->size[1] != a.classes ||
      grad_input->stride[1] != 1 || grad_input->stride[0] != a.classes)
    return fail(MM_ERR_INVALID, "mm_nll_loss_backward: grad_input must be contiguous [N, C]");
  if (reduction == 0 ? (grad_output->ndim != 1 || grad_output->size[0] != a.n) : numel(grad_output) != 1)
    return fail(MM_ERR_INVALID, "mm_nll_loss_backward: grad_output has the wrong shape");
  const float* tw = nullptr;
  if (reduction == 1) {
    MM_VALIDATE(total_weight, "mm_nll_loss_backward total_weight", MM_F32);
    if (numel(total_weight) != 1) return fail(MM_ERR_INVALID, "mm_nll_loss_backward: total_weight must hold one value");
    tw = (const float*)total_weight->data;
  }
  cudaStream_t s = resolve_stream(stream);
  const int64_t n = a.n * a.classes;
  if (n == 0) return MM_OK;
  MM_CUDA(cudaMemsetAsync(grad_input->data, 0, (size_t)n * sizeof(float), s), "mm_nll_loss_backward: zero");
  nll_loss_backward_kernel<<<grid_for(a.n, 256, (int64_t)sm_count() * 8), 256, 0, s>>>(
      a, reduction, (const float*)grad_output->data, reduction == 0 ? grad_output->stride[0] : 0, tw,
      (float*)grad_input->data, grad_input->stride[0], grad_input->stride[1]);
  MM_LAUNCH_CHECK("mm_nll_loss_backward launch");
  return MM_OK;
}
