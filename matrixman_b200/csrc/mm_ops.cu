// Memory-bound operators of libmatrixman_b200: elementwise, fill/arange,
// strided copy/cat, eval BatchNorm, softmax, pooling (generic max, fused SPPF
// chain, avg, adaptive avg), reductions, nearest upsample, the YOLO detect
// decode and the tf32 weight split.
//
// Layout policy: every kernel takes full strides; the host collapses the
// iteration space first so dense tensors (NCHW or NHWC) run a flat,
// 128-bit vectorised loop and only genuinely strided views pay for index
// decomposition.  Grids are sized in multiples of the SM count and loops are
// grid-strided.
#include <cuda_runtime.h>
#include <math.h>
#include <algorithm>
#include <stdint.h>

#include <string>

#include "mm_common.cuh"

namespace mm {

// ---------------------------------------------------------------------------
// Scalar math.  Transcendentals use CUDA's libm expf / exp (double) directly.
// ---------------------------------------------------------------------------

// Standalone activations are evaluated in double precision and rounded once,
// which keeps them within a few ulp of torch's CPU kernels (the tolerance the
// backend promises for activations).
__device__ __forceinline__ float silu_accurate(float x) {
  double d = (double)x;
  return (float)(d / (1.0 + exp(-d)));
}
__device__ __forceinline__ float sigmoid_accurate(float x) {
  double d = (double)x;
  return (float)(1.0 / (1.0 + exp(-d)));
}

template <int OP>
__device__ __forceinline__ float unary_apply(float x, float a, float b) {
  if (OP == MM_UNARY_COPY) return x;
  if (OP == MM_UNARY_SILU) return silu_accurate(x);
  if (OP == MM_UNARY_RELU) return (x != x) ? x : (x > 0.f ? x : 0.f);
  if (OP == MM_UNARY_SIGMOID) return sigmoid_accurate(x);
  if (OP == MM_UNARY_ADD_SCALAR) return x + a;
  if (OP == MM_UNARY_MUL_SCALAR) return x * a;
  if (OP == MM_UNARY_DIV_SCALAR) return __fdiv_rn(x, a);
  if (OP == MM_UNARY_NEG) return -x;
  if (OP == MM_UNARY_CLAMP) return (x != x) ? x : fminf(fmaxf(x, a), b);
  return x;
}

template <int OP>
__device__ __forceinline__ float binary_apply(float x, float y, float alpha) {
  if (OP == MM_BINARY_ADD) return fmaf(y, alpha, x);
  if (OP == MM_BINARY_SUB) return fmaf(y, -alpha, x);
  if (OP == MM_BINARY_MUL) return x * y;
  return __fdiv_rn(x, y);
}

// ---------------------------------------------------------------------------
// Elementwise kernels
// ---------------------------------------------------------------------------

template <int OP>
__global__ void unary_flat_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n,
                                  float a, float b) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  bool vec = ((((uintptr_t)x) | ((uintptr_t)y)) & 15) == 0;
  if (vec) {
    int64_t n4 = n >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float4* y4 = reinterpret_cast<float4*>(y);
    for (int64_t i = tid; i < n4; i += nth) {
      float4 v = x4[i];
      v.x = unary_apply<OP>(v.x, a, b);
      v.y = unary_apply<OP>(v.y, a, b);
      v.z = unary_apply<OP>(v.z, a, b);
      v.w = unary_apply<OP>(v.w, a, b);
      y4[i] = v;
    }
    for (int64_t i = (n4 << 2) + tid; i < n; i += nth) y[i] = unary_apply<OP>(x[i], a, b);
  } else {
    for (int64_t i = tid; i < n; i += nth) y[i] = unary_apply<OP>(x[i], a, b);
  }
}

template <int OP>
__global__ void unary_strided_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n,
                                     DevGeom gx, DevGeom gy, float a, float b) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < n; i += nth) {
    y[dev_offset(i, gy)] = unary_apply<OP>(x[dev_offset(i, gx)], a, b);
  }
}

template <int OP>
__global__ void binary_flat_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                   float* __restrict__ y, int64_t n, float alpha) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  bool vec = ((((uintptr_t)a) | ((uintptr_t)b) | ((uintptr_t)y)) & 15) == 0;
  if (vec) {
    int64_t n4 = n >> 2;
    for (int64_t i = tid; i < n4; i += nth) {
      float4 u = reinterpret_cast<const float4*>(a)[i];
      float4 v = reinterpret_cast<const float4*>(b)[i];
      float4 r;
      r.x = binary_apply<OP>(u.x, v.x, alpha);
      r.y = binary_apply<OP>(u.y, v.y, alpha);
      r.z = binary_apply<OP>(u.z, v.z, alpha);
      r.w = binary_apply<OP>(u.w, v.w, alpha);
      reinterpret_cast<float4*>(y)[i] = r;
    }
    for (int64_t i = (n4 << 2) + tid; i < n; i += nth) y[i] = binary_apply<OP>(a[i], b[i], alpha);
  } else {
    for (int64_t i = tid; i < n; i += nth) y[i] = binary_apply<OP>(a[i], b[i], alpha);
  }
}

template <int OP>
__global__ void binary_strided_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                      float* __restrict__ y, int64_t n, DevGeom ga, DevGeom gb,
                                      DevGeom gy, float alpha) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < n; i += nth) {
    y[dev_offset(i, gy)] = binary_apply<OP>(a[dev_offset(i, ga)], b[dev_offset(i, gb)], alpha);
  }
}

template <typename T>
__global__ void fill_kernel(T* __restrict__ y, int64_t n, DevGeom gy, T value) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < n; i += nth) y[dev_offset(i, gy)] = value;
}

template <typename T>
__global__ void arange_kernel(T* __restrict__ y, int64_t n, int64_t stride, double start,
                              double step) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < n; i += nth) y[i * stride] = (T)(start + (double)i * step);
}

template <typename T>
__global__ void copy_strided_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n,
                                    DevGeom gx, DevGeom gy) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < n; i += nth) y[dev_offset(i, gy)] = x[dev_offset(i, gx)];
}

// Copy of rows: y[r*ys + c] = x[r*xs + c] for c < cols, with cols % 4 == 0 and
// 16-byte aligned rows (NHWC channel slices: cat / split materialisation).
// One warp per row (grid-stride over rows), lanes stride over the row's
// float4s: coalesced 16-byte accesses, no per-element index division.
// Row copy (concatenation into NHWC channel slices): rows x cols4 float4
// elements over a flat index, so short rows leave no lane idle; each thread
// has four independent loads in flight before its stores.
__global__ void copy_rows_vec4_kernel(const float* __restrict__ x, float* __restrict__ y,
                                      int64_t rows, int cols4, int64_t xs, int64_t ys) {
  pdl_wait();
  const int64_t total = rows * cols4;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e0 < total; e0 += 4 * nth) {
    float4 v[4];
    int64_t dofs[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t e = e0 + u * nth;
      dofs[u] = -1;
      if (e < total) {
        const int64_t r = e / cols4;
        const int64_t c = e - r * cols4;
        v[u] = __ldg(reinterpret_cast<const float4*>(x + r * xs) + c);
        dofs[u] = r * ys + 4 * c;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (dofs[u] >= 0) *reinterpret_cast<float4*>(y + dofs[u]) = v[u];
  }
}

// ---------------------------------------------------------------------------
// BatchNorm (eval): y = x * alpha[c] + beta[c] with alpha = w / sqrt(var+eps),
// beta = b - mean*alpha (the same factorisation torch's CPU kernel uses).
// ---------------------------------------------------------------------------

__global__ void bn_eval_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n,
                               DevGeom gx, DevGeom gy, DevGeom gc, const float* __restrict__ mean,
                               const float* __restrict__ var, const float* __restrict__ w,
                               const float* __restrict__ b, float eps) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < n; i += nth) {
    int64_t c = dev_offset(i, gc);
    float invstd = 1.0f / sqrtf(var[c] + eps);
    float alpha = (w ? w[c] : 1.0f) * invstd;
    float beta = (b ? b[c] : 0.0f) - mean[c] * alpha;
    y[dev_offset(i, gy)] = x[dev_offset(i, gx)] * alpha + beta;
  }
}

// ---------------------------------------------------------------------------
// Softmax along one dim: one warp per row, three passes (max, sum, write).
// Row elements are at base + j*dstride; rows enumerated through `grow`.
// ---------------------------------------------------------------------------

__global__ void softmax_rows_kernel(const float* __restrict__ x, float* __restrict__ y,
                                    int64_t rows, int64_t len, DevGeom grx, DevGeom gry,
                                    int64_t xds, int64_t yds, int log_mode) {
  int lane = threadIdx.x & 31;
  int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = warp; r < rows; r += nwarps) {
    const float* xr = x + dev_offset(r, grx);
    float* yr = y + dev_offset(r, gry);
    float m = -INFINITY;
    for (int64_t j = lane; j < len; j += 32) m = fmaxf(m, xr[j * xds]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    double s = 0.0;
    for (int64_t j = lane; j < len; j += 32) s += exp((double)xr[j * xds] - (double)m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (log_mode) {
      double ls = log(s);
      for (int64_t j = lane; j < len; j += 32)
        yr[j * yds] = (float)((double)xr[j * xds] - (double)m - ls);
    } else {
      double inv = 1.0 / s;
      for (int64_t j = lane; j < len; j += 32)
        yr[j * yds] = (float)(exp((double)xr[j * xds] - (double)m) * inv);
    }
  }
}

// ---------------------------------------------------------------------------
// Pooling over dims (2,3) of a rank-4 tensor with arbitrary strides.
// ---------------------------------------------------------------------------

struct Pool4 {
  int64_t n, c, h, w, oh, ow;
  int64_t xs[4], ys[4];
};

__global__ void max_pool2d_kernel(const float* __restrict__ x, float* __restrict__ y, Pool4 p,
                                  int kh, int kw, int sh, int sw, int ph, int pw, int dh, int dw) {
  int64_t total = p.n * p.c * p.oh * p.ow;
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < total; i += nth) {
    // Channel-fastest enumeration keeps NHWC accesses coalesced; NCHW views
    // still hit every element exactly once.
    int64_t t = i;
    int64_t c = t % p.c; t /= p.c;
    int64_t ox = t % p.ow; t /= p.ow;
    int64_t oy = t % p.oh; t /= p.oh;
    int64_t n = t;
    const float* xb = x + n * p.xs[0] + c * p.xs[1];
    float best = -INFINITY;
    int64_t y0 = oy * sh - ph, x0 = ox * sw - pw;
    for (int a = 0; a < kh; ++a) {
      int64_t iy = y0 + (int64_t)a * dh;
      if (iy < 0 || iy >= p.h) continue;
      for (int bb = 0; bb < kw; ++bb) {
        int64_t ix = x0 + (int64_t)bb * dw;
        if (ix < 0 || ix >= p.w) continue;
        float v = xb[iy * p.xs[2] + ix * p.xs[3]];
        if (v > best || v != v) best = v;
        if (best != best) break;
      }
      if (best != best) break;
    }
    y[n * p.ys[0] + c * p.ys[1] + oy * p.ys[2] + ox * p.ys[3]] = best;
  }
}

__global__ void avg_pool2d_kernel(const float* __restrict__ x, float* __restrict__ y, Pool4 p,
                                  int kh, int kw, int sh, int sw, int ph, int pw,
                                  int count_include_pad, int divisor_override) {
  int64_t total = p.n * p.c * p.oh * p.ow;
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < total; i += nth) {
    int64_t t = i;
    int64_t c = t % p.c; t /= p.c;
    int64_t ox = t % p.ow; t /= p.ow;
    int64_t oy = t % p.oh; t /= p.oh;
    int64_t n = t;
    // torch semantics: the window is clipped to [-pad, size+pad) for the
    // divisor, then to the image for the sum.
    int64_t hstart = oy * sh - ph, wstart = ox * sw - pw;
    int64_t hend = hstart + kh, wend = wstart + kw;
    if (hend > p.h + ph) hend = p.h + ph;
    if (wend > p.w + pw) wend = p.w + pw;
    int64_t pool_size = (hend - hstart) * (wend - wstart);
    if (hstart < 0) hstart = 0;
    if (wstart < 0) wstart = 0;
    if (hend > p.h) hend = p.h;
    if (wend > p.w) wend = p.w;
    const float* xb = x + n * p.xs[0] + c * p.xs[1];
    float s = 0.f;
    for (int64_t iy = hstart; iy < hend; ++iy)
      for (int64_t ix = wstart; ix < wend; ++ix) s += xb[iy * p.xs[2] + ix * p.xs[3]];
    int64_t div;
    if (divisor_override > 0) div = divisor_override;
    else if (count_include_pad) div = pool_size;
    else div = (hend - hstart) * (wend - wstart);
    y[n * p.ys[0] + c * p.ys[1] + oy * p.ys[2] + ox * p.ys[3]] = s / (float)div;
  }
}

__global__ void adaptive_avg_pool2d_kernel(const float* __restrict__ x, float* __restrict__ y,
                                           Pool4 p) {
  int64_t total = p.n * p.c * p.oh * p.ow;
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < total; i += nth) {
    int64_t t = i;
    int64_t c = t % p.c; t /= p.c;
    int64_t ox = t % p.ow; t /= p.ow;
    int64_t oy = t % p.oh; t /= p.oh;
    int64_t n = t;
    int64_t h0 = (oy * p.h) / p.oh, h1 = ((oy + 1) * p.h + p.oh - 1) / p.oh;
    int64_t w0 = (ox * p.w) / p.ow, w1 = ((ox + 1) * p.w + p.ow - 1) / p.ow;
    const float* xb = x + n * p.xs[0] + c * p.xs[1];
    float s = 0.f;
    for (int64_t iy = h0; iy < h1; ++iy)
      for (int64_t ix = w0; ix < w1; ++ix) s += xb[iy * p.xs[2] + ix * p.xs[3]];
    y[n * p.ys[0] + c * p.ys[1] + oy * p.ys[2] + ox * p.ys[3]] = s / (float)((h1 - h0) * (w1 - w0));
  }
}

// Fused SPPF chain.  pool5 applied k times with -inf padding equals the
// (4k+1)x(4k+1) window clipped to the image, so y1/y2/y3 are the 5/9/13
// windows of x.  Each block stages a (TH+12)x(TW+12) halo tile of one
// channel group in shared memory, runs separable row maxima of width 5/9/13,
// then column maxima.  Max is exact, so the result is bit-identical to three
// chained pools; NaNs propagate.
constexpr int SPPF_TH = 8, SPPF_TW = 8, SPPF_CG = 8, SPPF_HALO = 6;

__device__ __forceinline__ float nanmax(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fc00000) : fmaxf(a, b);
}

__global__ void sppf_kernel(const float* __restrict__ x, float* __restrict__ y1,
                            float* __restrict__ y2, float* __restrict__ y3, Pool4 p, Pool4 q2,
                            Pool4 q3, int64_t tiles_w, int64_t tiles_h, int64_t cgroups) {
  constexpr int HH = SPPF_TH + 2 * SPPF_HALO, WW = SPPF_TW + 2 * SPPF_HALO;
  __shared__ float tile[HH][WW][SPPF_CG];
  __shared__ float rmax[3][HH][SPPF_TW][SPPF_CG];
  int64_t b = blockIdx.x;
  int64_t tw = b % tiles_w; b /= tiles_w;
  int64_t th = b % tiles_h; b /= tiles_h;
  int64_t cg = b % cgroups; b /= cgroups;
  int64_t n = b;
  int64_t oy0 = th * SPPF_TH, ox0 = tw * SPPF_TW, c0 = cg * SPPF_CG;
  int tid = threadIdx.x;
  for (int i = tid; i < HH * WW * SPPF_CG; i += blockDim.x) {
    int cc = i % SPPF_CG;
    int xx = (i / SPPF_CG) % WW;
    int yy = i / (SPPF_CG * WW);
    int64_t iy = oy0 + yy - SPPF_HALO, ix = ox0 + xx - SPPF_HALO, c = c0 + cc;
    float v = -INFINITY;
    if (iy >= 0 && iy < p.h && ix >= 0 && ix < p.w && c < p.c)
      v = x[n * p.xs[0] + c * p.xs[1] + iy * p.xs[2] + ix * p.xs[3]];
    tile[yy][xx][cc] = v;
  }
  __syncthreads();
  for (int i = tid; i < HH * SPPF_TW * SPPF_CG; i += blockDim.x) {
    int cc = i % SPPF_CG;
    int xx = (i / SPPF_CG) % SPPF_TW;
    int yy = i / (SPPF_CG * SPPF_TW);
    int cx = xx + SPPF_HALO;
    float m5 = -INFINITY;
    for (int d = -2; d <= 2; ++d) m5 = nanmax(m5, tile[yy][cx + d][cc]);
    float m9 = m5;
    for (int d = 3; d <= 4; ++d) m9 = nanmax(m9, nanmax(tile[yy][cx - d][cc], tile[yy][cx + d][cc]));
    float m13 = m9;
    for (int d = 5; d <= 6; ++d) m13 = nanmax(m13, nanmax(tile[yy][cx - d][cc], tile[yy][cx + d][cc]));
    rmax[0][yy][xx][cc] = m5;
    rmax[1][yy][xx][cc] = m9;
    rmax[2][yy][xx][cc] = m13;
  }
  __syncthreads();
  for (int i = tid; i < SPPF_TH * SPPF_TW * SPPF_CG; i += blockDim.x) {
    int cc = i % SPPF_CG;
    int xx = (i / SPPF_CG) % SPPF_TW;
    int yy = i / (SPPF_CG * SPPF_TW);
    int64_t oy = oy0 + yy, ox = ox0 + xx, c = c0 + cc;
    if (oy >= p.h || ox >= p.w || c >= p.c) continue;
    int cy = yy + SPPF_HALO;
    float a5 = -INFINITY, a9 = -INFINITY, a13 = -INFINITY;
    for (int d = -2; d <= 2; ++d) a5 = nanmax(a5, rmax[0][cy + d][xx][cc]);
    for (int d = -4; d <= 4; ++d) a9 = nanmax(a9, rmax[1][cy + d][xx][cc]);
    for (int d = -6; d <= 6; ++d) a13 = nanmax(a13, rmax[2][cy + d][xx][cc]);
    y1[n * p.ys[0] + c * p.ys[1] + oy * p.ys[2] + ox * p.ys[3]] = a5;
    y2[n * q2.ys[0] + c * q2.ys[1] + oy * q2.ys[2] + ox * q2.ys[3]] = a9;
    y3[n * q3.ys[0] + c * q3.ys[1] + oy * q3.ys[2] + ox * q3.ys[3]] = a13;
  }
}

// SPPF on whole small images: one block per (image, group of SPPF_CG
// channels) holds the image in shared memory and runs SPPF's definition --
// three chained 5x5 stride-1 max-pools with -inf padding -- as row and column
// passes between two buffers, writing each pool's result to its slice.  The
// input is read once (the tiled kernel re-reads 6.25x for its halos at 20 x 20).
__global__ void sppf_image_kernel(const float* __restrict__ x, float* __restrict__ y1,
                                  float* __restrict__ y2, float* __restrict__ y3, Pool4 p, Pool4 q2,
                                  Pool4 q3, int cgroups) {
  pdl_wait();
  extern __shared__ float sp_buf[];
  const int H = (int)p.h, W = (int)p.w, HW = H * W;
  float* a = sp_buf;                    // [H][W][SPPF_CG]
  float* b = sp_buf + HW * SPPF_CG;
  const int n = blockIdx.x / cgroups;
  const int c0 = (blockIdx.x - n * cgroups) * SPPF_CG;
  const int total = HW * SPPF_CG;
  for (int e = threadIdx.x; e < total; e += blockDim.x) {
    const int cc = e % SPPF_CG, pix = e / SPPF_CG;
    const int yy = pix / W, xx = pix - yy * W;
    const int c = c0 + cc;
    a[e] = c < p.c ? x[n * p.xs[0] + c * p.xs[1] + yy * p.xs[2] + xx * p.xs[3]] : 0.f;
  }
  __syncthreads();
  for (int round = 0; round < 3; ++round) {
    for (int e = threadIdx.x; e < total; e += blockDim.x) {  // rows: a -> b
      const int cc = e % SPPF_CG, pix = e / SPPF_CG;
      const int yy = pix / W, xx = pix - yy * W;
      float m = -INFINITY;
#pragma unroll
      for (int d = -2; d <= 2; ++d) {
        const int xs = xx + d;
        if (xs >= 0 && xs < W) m = nanmax(m, a[(yy * W + xs) * SPPF_CG + cc]);
      }
      b[e] = m;
    }
    __syncthreads();
    float* yo = round == 0 ? y1 : round == 1 ? y2 : y3;
    const Pool4& q = round == 0 ? p : round == 1 ? q2 : q3;
    for (int e = threadIdx.x; e < total; e += blockDim.x) {  // columns: b -> a, store
      const int cc = e % SPPF_CG, pix = e / SPPF_CG;
      const int yy = pix / W, xx = pix - yy * W;
      float m = -INFINITY;
#pragma unroll
      for (int d = -2; d <= 2; ++d) {
        const int ys = yy + d;
        if (ys >= 0 && ys < H) m = nanmax(m, b[(ys * W + xx) * SPPF_CG + cc]);
      }
      a[e] = m;
      const int c = c0 + cc;
      if (c < p.c) yo[n * q.ys[0] + c * q.ys[1] + yy * q.ys[2] + xx * q.ys[3]] = m;
    }
    __syncthreads();
  }
}

// The same whole-image SPPF on channels-last tensors with 16-byte aligned
// pixels, four channels (one float4) per element: a block holds CG4 float4 of
// every pixel, each thread computes the (row, column) of its elements once and
// reuses them in all seven passes, and every shared-memory and global access
// moves a float4.  Same passes, same comparisons, same results as
// sppf_image_kernel.
constexpr int SPPF4_THREADS = 256, SPPF4_MAXE = 6;  // elements per thread: <= 6 (48 KB)

__device__ __forceinline__ float4 nanmax4(float4 a, float4 b) {
  return make_float4(nanmax(a.x, b.x), nanmax(a.y, b.y), nanmax(a.z, b.z), nanmax(a.w, b.w));
}

template <int CG4>
__global__ void __launch_bounds__(SPPF4_THREADS) sppf_image_v4_kernel(
    const float* __restrict__ x, float* __restrict__ y1, float* __restrict__ y2, float* __restrict__ y3,
    Pool4 p, Pool4 q2, Pool4 q3, int cgroups) {
  pdl_wait();
  extern __shared__ float4 sp4_buf[];
  const int H = (int)p.h, W = (int)p.w, total = H * W * CG4;
  float4* a = sp4_buf;  // [H][W][CG4]
  float4* b = sp4_buf + total;
  const int n = blockIdx.x / cgroups;
  const int c0 = (blockIdx.x - n * cgroups) * 4 * CG4;
  int ey[SPPF4_MAXE], ex[SPPF4_MAXE];
#pragma unroll
  for (int k = 0; k < SPPF4_MAXE; ++k) {
    const int e = threadIdx.x + k * SPPF4_THREADS;
    const int pix = e / CG4;
    ey[k] = pix / W;
    ex[k] = pix - ey[k] * W;
    if (e < total) {
      const int c = c0 + 4 * (e % CG4);
      a[e] = __ldg(reinterpret_cast<const float4*>(x + n * p.xs[0] + c + ey[k] * p.xs[2] + ex[k] * p.xs[3]));
    }
  }
  __syncthreads();
  for (int round = 0; round < 3; ++round) {
#pragma unroll
    for (int k = 0; k < SPPF4_MAXE; ++k) {  // rows: a -> b
      const int e = threadIdx.x + k * SPPF4_THREADS;
      if (e < total) {
        const int cc = e % CG4;
        float4 m = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
#pragma unroll
        for (int d = -2; d <= 2; ++d) {
          const int xs = ex[k] + d;
          if (xs >= 0 && xs < W) m = nanmax4(m, a[(ey[k] * W + xs) * CG4 + cc]);
        }
        b[e] = m;
      }
    }
    __syncthreads();
    float* yo = round == 0 ? y1 : round == 1 ? y2 : y3;
    const int64_t ys0 = round == 0 ? p.ys[0] : round == 1 ? q2.ys[0] : q3.ys[0];
    const int64_t ys2 = round == 0 ? p.ys[2] : round == 1 ? q2.ys[2] : q3.ys[2];
    const int64_t ys3 = round == 0 ? p.ys[3] : round == 1 ? q2.ys[3] : q3.ys[3];
#pragma unroll
    for (int k = 0; k < SPPF4_MAXE; ++k) {  // columns: b -> a, store
      const int e = threadIdx.x + k * SPPF4_THREADS;
      if (e < total) {
        const int cc = e % CG4;
        float4 m = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
#pragma unroll
        for (int d = -2; d <= 2; ++d) {
          const int ys = ey[k] + d;
          if (ys >= 0 && ys < H) m = nanmax4(m, b[(ys * W + ex[k]) * CG4 + cc]);
        }
        a[e] = m;
        *reinterpret_cast<float4*>(yo + n * ys0 + c0 + 4 * cc + ey[k] * ys2 + ex[k] * ys3) = m;
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Reduction (sum/mean) over a dim mask: one warp per output element.
// ---------------------------------------------------------------------------

__global__ void reduce_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t nout,
                              int64_t nred, DevGeom gkeep_x, DevGeom gkeep_y, DevGeom gred,
                              int mean) {
  int lane = threadIdx.x & 31;
  int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t o = warp; o < nout; o += nwarps) {
    const float* xb = x + dev_offset(o, gkeep_x);
    double s = 0.0;
    for (int64_t j = lane; j < nred; j += 32) s += (double)xb[dev_offset(j, gred)];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) {
      if (mean) s /= (double)nred;
      y[dev_offset(o, gkeep_y)] = (float)s;
    }
  }
}

// ---------------------------------------------------------------------------
// Nearest upsampling with torch's source-index rule:
//   src = min(floor(dst * scale), in - 1), scale = 1/user_scale or in/out (fp32)
// ---------------------------------------------------------------------------

__device__ __forceinline__ int64_t nearest_src(int64_t dst, int64_t in, int64_t out, float scale) {
  if (out == in) return dst;
  if (out == 2 * in) return dst >> 1;
  int64_t s = (int64_t)floorf((float)dst * scale);
  return s < in - 1 ? s : in - 1;
}

__global__ void upsample_nearest_kernel(const float* __restrict__ x, float* __restrict__ y,
                                        Pool4 p, float scale_h, float scale_w) {
  int64_t total = p.n * p.c * p.oh * p.ow;
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < total; i += nth) {
    int64_t t = i;
    int64_t c = t % p.c; t /= p.c;
    int64_t ox = t % p.ow; t /= p.ow;
    int64_t oy = t % p.oh; t /= p.oh;
    int64_t n = t;
    int64_t iy = nearest_src(oy, p.h, p.oh, scale_h);
    int64_t ix = nearest_src(ox, p.w, p.ow, scale_w);
    y[n * p.ys[0] + c * p.ys[1] + oy * p.ys[2] + ox * p.ys[3]] =
        x[n * p.xs[0] + c * p.xs[1] + iy * p.xs[2] + ix * p.xs[3]];
  }
}

// NHWC fast path (channel stride 1, C % 4 == 0, aligned): one float4 per thread.
__global__ void upsample_nearest_nhwc4_kernel(const float* __restrict__ x, float* __restrict__ y,
                                              Pool4 p, float scale_h, float scale_w) {
  int64_t c4 = p.c >> 2;
  int64_t total = p.n * p.oh * p.ow * c4;
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < total; i += nth) {
    int64_t t = i;
    int64_t c = (t % c4) * 4; t /= c4;
    int64_t ox = t % p.ow; t /= p.ow;
    int64_t oy = t % p.oh; t /= p.oh;
    int64_t n = t;
    int64_t iy = nearest_src(oy, p.h, p.oh, scale_h);
    int64_t ix = nearest_src(ox, p.w, p.ow, scale_w);
    float4 v = *reinterpret_cast<const float4*>(x + n * p.xs[0] + c + iy * p.xs[2] + ix * p.xs[3]);
    *reinterpret_cast<float4*>(y + n * p.ys[0] + c + oy * p.ys[2] + ox * p.ys[3]) = v;
  }
}

// Exact 2x nearest upsample of NHWC float4 rows (output = 2 x input in both
// dimensions, where the source index is dst >> 1): each thread reads one input
// float4 and writes the 2 x 2 output block; blockIdx.y walks input rows.
__global__ void upsample2x_nhwc4_kernel(const float* __restrict__ x, float* __restrict__ y, Pool4 p) {
  pdl_wait();
  const int c4 = (int)(p.c >> 2);
  const int row_elems = (int)p.w * c4;
  for (int64_t row = blockIdx.y; row < p.n * p.h; row += gridDim.y) {
    const int64_t n = row / p.h, iy = row - n * p.h;
    const float* xr = x + n * p.xs[0] + iy * p.xs[2];
    float* yr = y + n * p.ys[0] + 2 * iy * p.ys[2];
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < row_elems; e += gridDim.x * blockDim.x) {
      const int ix = e / c4, c = (e - ix * c4) * 4;
      const float4 v = *reinterpret_cast<const float4*>(xr + ix * p.xs[3] + c);
      float* o = yr + 2 * ix * p.ys[3] + c;
      *reinterpret_cast<float4*>(o) = v;
      *reinterpret_cast<float4*>(o + p.ys[3]) = v;
      *reinterpret_cast<float4*>(o + p.ys[2]) = v;
      *reinterpret_cast<float4*>(o + p.ys[2] + p.ys[3]) = v;
    }
  }
}

// ---------------------------------------------------------------------------
// YOLOv8 detect decode (DFL + dist2bbox + sigmoid), one thread per (image,
// anchor).  Box: softmax over reg_max bins per side (max-subtracted, fp32
// expf), expectation with weights 0..reg_max-1; lt/rb distances give
// x1y1 = c - lt, x2y2 = c + rb; output (cx, cy, w, h) * stride.
// ---------------------------------------------------------------------------

struct DecodeLevel {
  const float* base;
  int64_t sn, sh, sw, sc;  // strides of [B, H, W, C] (C = 4*reg_max + nc)
  int64_t h, w;
  int64_t anchor0;
  float stride;
};

struct DecodeArgs {
  DecodeLevel lv[4];
  int nlevels;
  int reg_max;
  int nc;
  int64_t batch, anchors;
  float* out;
  int64_t on, oc, oa;  // out strides of [B, 4+nc, A]
};

__global__ void yolo_decode_kernel(DecodeArgs a) {
  int64_t total = a.batch * a.anchors;
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < total; i += nth) {
    int64_t n = i / a.anchors;
    int64_t an = i - n * a.anchors;
    int l = 0;
    while (l + 1 < a.nlevels && an >= a.lv[l + 1].anchor0) ++l;
    const DecodeLevel& L = a.lv[l];
    int64_t local = an - L.anchor0;
    int64_t yy = local / L.w, xx = local - yy * L.w;
    const float* f = L.base + n * L.sn + yy * L.sh + xx * L.sw;
    float dist[4];
    for (int side = 0; side < 4; ++side) {
      const float* lg = f + (int64_t)side * a.reg_max * L.sc;
      float m = -INFINITY;
      for (int k = 0; k < a.reg_max; ++k) m = fmaxf(m, lg[k * L.sc]);
      float s = 0.f, e = 0.f;
      for (int k = 0; k < a.reg_max; ++k) {
        float p = expf(lg[k * L.sc] - m);
        s += p;
        e += p * (float)k;
      }
      dist[side] = e / s;
    }
    float ax = (float)xx + 0.5f, ay = (float)yy + 0.5f;
    float x1 = ax - dist[0], y1 = ay - dist[1];
    float x2 = ax + dist[2], y2 = ay + dist[3];
    float* o = a.out + n * a.on + an * a.oa;
    o[0 * a.oc] = (x1 + x2) * 0.5f * L.stride;
    o[1 * a.oc] = (y1 + y2) * 0.5f * L.stride;
    o[2 * a.oc] = (x2 - x1) * L.stride;
    o[3 * a.oc] = (y2 - y1) * L.stride;
    const float* cl = f + (int64_t)4 * a.reg_max * L.sc;
    for (int k = 0; k < a.nc; ++k) {
      float v = cl[k * L.sc];
      o[(4 + k) * a.oc] = 1.0f / (1.0f + expf(-v));
    }
  }
}

// The same decode for the layout the prepared YOLO head writes: NHWC feature
// rows (channel stride 1, 16-byte aligned), 16 distribution bins, nc a
// multiple of 4.  One thread per anchor, blockIdx.y = image; a warp covers 32
// consecutive pixels of one level, i.e. one contiguous block of rows, and each
// phase issues its float4 loads back to back so every line is fetched once.
// Loading one box side (4 float4) at a time keeps the kernel at 64 registers,
// so 8 CTAs fit per SM instead of 4: 15 % faster at YOLOv8n batch 64 (0.76 of
// the HBM copy rate) than holding all 16 box float4 at once.
// The arithmetic is the generic kernel's, in the same order (same results).
__global__ void __launch_bounds__(128, 8) yolo_decode_rows_kernel(DecodeArgs a) {
  pdl_wait();
  const int an = (int)(blockIdx.x * blockDim.x + threadIdx.x);
  if (an >= (int)a.anchors) return;
  int l = 0;
  while (l + 1 < a.nlevels && an >= (int)a.lv[l + 1].anchor0) ++l;
  const DecodeLevel& L = a.lv[l];
  const int local = an - (int)L.anchor0;
  const int yy = local / (int)L.w, xx = local - yy * (int)L.w;
  const float ax = (float)xx + 0.5f, ay = (float)yy + 0.5f;
  for (int64_t n = blockIdx.y; n < a.batch; n += gridDim.y) {
    const float4* f = reinterpret_cast<const float4*>(L.base + n * L.sn + yy * L.sh + xx * L.sw);
    float dist[4];
#pragma unroll
    for (int side = 0; side < 4; ++side) {
      float4 v[16];  // (only this side's four are loaded: 63 registers, 8 CTAs per SM)
#pragma unroll
      for (int j = 4 * side; j < 4 * side + 4; ++j) v[j] = __ldg(f + j);
      const float lg[16] = {v[4 * side].x,     v[4 * side].y,     v[4 * side].z,     v[4 * side].w,
                            v[4 * side + 1].x, v[4 * side + 1].y, v[4 * side + 1].z, v[4 * side + 1].w,
                            v[4 * side + 2].x, v[4 * side + 2].y, v[4 * side + 2].z, v[4 * side + 2].w,
                            v[4 * side + 3].x, v[4 * side + 3].y, v[4 * side + 3].z, v[4 * side + 3].w};
      float m = -INFINITY;
#pragma unroll
      for (int k = 0; k < 16; ++k) m = fmaxf(m, lg[k]);
      float s = 0.f, e = 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        float p = expf(lg[k] - m);
        s += p;
        e += p * (float)k;
      }
      dist[side] = e / s;
    }
    float x1 = ax - dist[0], y1 = ay - dist[1];
    float x2 = ax + dist[2], y2 = ay + dist[3];
    float* o = a.out + n * a.on + (int64_t)an * a.oa;
    o[0 * a.oc] = (x1 + x2) * 0.5f * L.stride;
    o[1 * a.oc] = (y1 + y2) * 0.5f * L.stride;
    o[2 * a.oc] = (x2 - x1) * L.stride;
    o[3 * a.oc] = (y2 - y1) * L.stride;
    const float4* cl = f + 16;
    for (int k4 = 0; k4 < a.nc / 4; k4 += 5) {
      float4 c[5];
      const int cnt = min(5, a.nc / 4 - k4);
#pragma unroll
      for (int j = 0; j < 5; ++j)
        if (j < cnt) c[j] = __ldg(cl + k4 + j);
#pragma unroll
      for (int j = 0; j < 5; ++j) {
        if (j < cnt) {
          float* oc = o + (int64_t)(4 + 4 * (k4 + j)) * a.oc;
          oc[0] = 1.0f / (1.0f + expf(-c[j].x));
          oc[a.oc] = 1.0f / (1.0f + expf(-c[j].y));
          oc[2 * a.oc] = 1.0f / (1.0f + expf(-c[j].z));
          oc[3 * a.oc] = 1.0f / (1.0f + expf(-c[j].w));
        }
      }
    }
  }
}

// tf32 split: hi = x with the 13 low mantissa bits cleared, lo = x - hi (exact).
__global__ void tf32_split_kernel(const float* __restrict__ src, float* __restrict__ hi,
                                  float* __restrict__ lo, int64_t n) {
  int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < n; i += nth) {
    float v = src[i];
    float h = __uint_as_float(__float_as_uint(v) & 0xffffe000u);
    hi[i] = h;
    lo[i] = v - h;
  }
}

// ---------------------------------------------------------------------------
// Host helpers
// ---------------------------------------------------------------------------

static int pool4(const mm_tensor_t* x, const mm_tensor_t* y, Pool4* p, const char* name) {
  if (x->ndim != 4 || y->ndim != 4)
    return fail(MM_ERR_UNSUPPORTED, std::string(name) + ": expects rank-4 [N,C,H,W] tensors");
  if (x->size[0] != y->size[0] || x->size[1] != y->size[1])
    return fail(MM_ERR_INVALID, std::string(name) + ": batch/channel mismatch");
  p->n = x->size[0];
  p->c = x->size[1];
  p->h = x->size[2];
  p->w = x->size[3];
  p->oh = y->size[2];
  p->ow = y->size[3];
  for (int i = 0; i < 4; ++i) {
    p->xs[i] = x->stride[i];
    p->ys[i] = y->stride[i];
  }
  return MM_OK;
}

static bool is_flat(const Geom& g) { return g.nd == 0 || (g.nd == 1 && g.stride[0] == 1); }

}  // namespace mm

using namespace mm;

#define MM_VALIDATE(t, name, dt)                 \
  do {                                           \
    int _rc = validate(t, name, dt);             \
    if (_rc != MM_OK) return _rc;                \
  } while (0)

template <int OP>
static void launch_unary(const mm_tensor_t* x, const mm_tensor_t* y, const Geom* g, int64_t n,
                         float a, float b, cudaStream_t s) {
  int block = 256;
  unsigned grid = grid_for((n + 3) / 4, block, (int64_t)sm_count() * 8);
  if (is_flat(g[0]) && is_flat(g[1])) {
    unary_flat_kernel<OP><<<grid, block, 0, s>>>((const float*)x->data, (float*)y->data, n, a, b);
  } else {
    grid = grid_for(n, block, (int64_t)sm_count() * 8);
    unary_strided_kernel<OP><<<grid, block, 0, s>>>((const float*)x->data, (float*)y->data, n,
                                                    to_dev(g[0]), to_dev(g[1]), a, b);
  }
}

extern "C" int mm_unary(int op, const mm_tensor_t* x, const mm_tensor_t* y, double a, double b,
                        void* stream) {
  MM_VALIDATE(x, "mm_unary input", MM_F32);
  MM_VALIDATE(y, "mm_unary output", MM_F32);
  const mm_tensor_t* ops[2] = {x, y};
  Geom g[2];
  int rc = collapse(2, ops, g);
  if (rc != MM_OK) return rc;
  int64_t n = numel(x);
  if (n == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  float fa = (float)a, fb = (float)b;
  switch (op) {
    case MM_UNARY_COPY: launch_unary<MM_UNARY_COPY>(x, y, g, n, fa, fb, s); break;
    case MM_UNARY_SILU: launch_unary<MM_UNARY_SILU>(x, y, g, n, fa, fb, s); break;
    case MM_UNARY_RELU: launch_unary<MM_UNARY_RELU>(x, y, g, n, fa, fb, s); break;
    case MM_UNARY_SIGMOID: launch_unary<MM_UNARY_SIGMOID>(x, y, g, n, fa, fb, s); break;
    case MM_UNARY_ADD_SCALAR: launch_unary<MM_UNARY_ADD_SCALAR>(x, y, g, n, fa, fb, s); break;
    case MM_UNARY_MUL_SCALAR: launch_unary<MM_UNARY_MUL_SCALAR>(x, y, g, n, fa, fb, s); break;
    case MM_UNARY_DIV_SCALAR: launch_unary<MM_UNARY_DIV_SCALAR>(x, y, g, n, fa, fb, s); break;
    case MM_UNARY_NEG: launch_unary<MM_UNARY_NEG>(x, y, g, n, fa, fb, s); break;
    case MM_UNARY_CLAMP: launch_unary<MM_UNARY_CLAMP>(x, y, g, n, fa, fb, s); break;
    default: return fail(MM_ERR_UNSUPPORTED, "mm_unary: unknown op " + std::to_string(op));
  }
  MM_LAUNCH_CHECK("mm_unary launch");
  return MM_OK;
}

template <int OP>
static void launch_binary(const mm_tensor_t* a, const mm_tensor_t* b, const mm_tensor_t* y,
                          const Geom* g, int64_t n, float alpha, cudaStream_t s) {
  int block = 256;
  if (is_flat(g[0]) && is_flat(g[1]) && is_flat(g[2])) {
    unsigned grid = grid_for((n + 3) / 4, block, (int64_t)sm_count() * 8);
    binary_flat_kernel<OP><<<grid, block, 0, s>>>((const float*)a->data, (const float*)b->data,
                                                  (float*)y->data, n, alpha);
  } else {
    unsigned grid = grid_for(n, block, (int64_t)sm_count() * 8);
    binary_strided_kernel<OP><<<grid, block, 0, s>>>((const float*)a->data, (const float*)b->data,
                                                     (float*)y->data, n, to_dev(g[0]),
                                                     to_dev(g[1]), to_dev(g[2]), alpha);
  }
}

extern "C" int mm_binary(int op, const mm_tensor_t* a, const mm_tensor_t* b, const mm_tensor_t* y,
                         double alpha, void* stream) {
  MM_VALIDATE(a, "mm_binary lhs", MM_F32);
  MM_VALIDATE(b, "mm_binary rhs", MM_F32);
  MM_VALIDATE(y, "mm_binary output", MM_F32);
  const mm_tensor_t* ops[3] = {a, b, y};
  Geom g[3];
  int rc = collapse(3, ops, g);
  if (rc != MM_OK) return rc;
  int64_t n = numel(y);
  if (n == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  float fa = (float)alpha;
  switch (op) {
    case MM_BINARY_ADD: launch_binary<MM_BINARY_ADD>(a, b, y, g, n, fa, s); break;
    case MM_BINARY_SUB: launch_binary<MM_BINARY_SUB>(a, b, y, g, n, fa, s); break;
    case MM_BINARY_MUL: launch_binary<MM_BINARY_MUL>(a, b, y, g, n, fa, s); break;
    case MM_BINARY_DIV: launch_binary<MM_BINARY_DIV>(a, b, y, g, n, fa, s); break;
    default: return fail(MM_ERR_UNSUPPORTED, "mm_binary: unknown op " + std::to_string(op));
  }
  MM_LAUNCH_CHECK("mm_binary launch");
  return MM_OK;
}

extern "C" int mm_fill(const mm_tensor_t* y, double value, void* stream) {
  MM_VALIDATE(y, "mm_fill output", -1);
  const mm_tensor_t* ops[1] = {y};
  Geom g[1];
  int rc = collapse(1, ops, g);
  if (rc != MM_OK) return rc;
  int64_t n = numel(y);
  if (n == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  unsigned grid = grid_for(n, 256, (int64_t)sm_count() * 8);
  if (y->dtype == MM_F32)
    fill_kernel<float><<<grid, 256, 0, s>>>((float*)y->data, n, to_dev(g[0]), (float)value);
  else
    fill_kernel<int64_t><<<grid, 256, 0, s>>>((int64_t*)y->data, n, to_dev(g[0]), (int64_t)value);
  MM_LAUNCH_CHECK("mm_fill launch");
  return MM_OK;
}

extern "C" int mm_arange(const mm_tensor_t* y, double start, double step, void* stream) {
  MM_VALIDATE(y, "mm_arange output", -1);
  if (y->ndim != 1) return fail(MM_ERR_UNSUPPORTED, "mm_arange: output must be rank 1");
  int64_t n = y->size[0];
  if (n == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  unsigned grid = grid_for(n, 256, (int64_t)sm_count() * 8);
  if (y->dtype == MM_F32)
    arange_kernel<float><<<grid, 256, 0, s>>>((float*)y->data, n, y->stride[0], start, step);
  else
    arange_kernel<int64_t><<<grid, 256, 0, s>>>((int64_t*)y->data, n, y->stride[0], start, step);
  MM_LAUNCH_CHECK("mm_arange launch");
  return MM_OK;
}

// Both operands with their dimensions reordered by the output's memory order
// (largest stride first, ties keep logical order), so that channel slices of
// channels-last buffers collapse to [pixels, channels] rows.
static void memory_order(const mm_tensor_t* x, const mm_tensor_t* y, mm_tensor_t* xo,
                         mm_tensor_t* yo) {
  *xo = *x;
  *yo = *y;
  int perm[MM_MAX_DIMS];
  for (int i = 0; i < y->ndim; ++i) perm[i] = i;
  for (int i = 1; i < y->ndim; ++i) {  // insertion sort, stable
    int p = perm[i], j = i - 1;
    while (j >= 0 && y->stride[perm[j]] < y->stride[p]) {
      perm[j + 1] = perm[j];
      --j;
    }
    perm[j + 1] = p;
  }
  for (int i = 0; i < y->ndim; ++i) {
    xo->size[i] = x->size[perm[i]];
    xo->stride[i] = x->stride[perm[i]];
    yo->size[i] = y->size[perm[i]];
    yo->stride[i] = y->stride[perm[i]];
  }
}

static int copy_impl(const mm_tensor_t* x_in, const mm_tensor_t* y_in, cudaStream_t s) {
  if (x_in->dtype != y_in->dtype) return fail(MM_ERR_UNSUPPORTED, "mm_copy: dtype mismatch");
  mm_tensor_t xo, yo;
  if (x_in->ndim != y_in->ndim) return fail(MM_ERR_INVALID, "mm_copy: rank mismatch");
  memory_order(x_in, y_in, &xo, &yo);
  const mm_tensor_t* x = &xo;
  const mm_tensor_t* y = &yo;
  const mm_tensor_t* ops[2] = {x, y};
  Geom g[2];
  int rc = collapse(2, ops, g);
  if (rc != MM_OK) return rc;
  int64_t n = numel(x);
  if (n == 0) return MM_OK;
  size_t es = x->dtype == MM_F32 ? 4 : 8;
  if (is_flat(g[0]) && is_flat(g[1])) {
    // Dense copies run on the SMs (as one row of the row-copy kernel), not on
    // a copy engine: a device-to-device cudaMemcpyAsync waits in the copy
    // engine's queue behind host transfers issued earlier on other streams
    // (the next batch's upload), which would hold up the forward behind it.
    const int64_t bytes = n * (int64_t)es;
    if (bytes % 16 == 0 && bytes / 16 <= 0x7fffffffLL &&
        ((((uintptr_t)x->data) | ((uintptr_t)y->data)) & 15) == 0) {
      const int64_t cols4 = bytes / 16;
      int64_t blocks = (cols4 + 4 * 256 - 1) / (4 * 256);
      const int64_t cap = (int64_t)sm_count() * 16;
      if (blocks > cap) blocks = cap;
      if (blocks < 1) blocks = 1;
      MM_CUDA(launch_pdl(copy_rows_vec4_kernel, dim3((unsigned)blocks), dim3(256), 0, s, (const float*)x->data,
                         (float*)y->data, (int64_t)1, (int)cols4, (int64_t)0, (int64_t)0),
              "mm_copy launch");
      MM_LAUNCH_CHECK("mm_copy launch");
      return MM_OK;
    }
    MM_CUDA(cudaMemcpyAsync(y->data, x->data, bytes, cudaMemcpyDeviceToDevice, s), "mm_copy");
    return MM_OK;
  }
  // Row copies (channel slices of NHWC buffers): rank-2 collapsed geometry
  // with unit inner stride, 16-byte aligned.
  if (x->dtype == MM_F32 && g[0].nd == 2 && g[0].stride[1] == 1 && g[1].stride[1] == 1 &&
      g[0].size[1] % 4 == 0 && g[0].stride[0] % 4 == 0 && g[1].stride[0] % 4 == 0 &&
      ((((uintptr_t)x->data) | ((uintptr_t)y->data)) & 15) == 0) {
    const int64_t rows = g[0].size[0];
    const int64_t cols4 = g[0].size[1] / 4;
    if (cols4 > 0x7fffffff) return fail(MM_ERR_UNSUPPORTED, "mm_copy: row too long");
    const int64_t elems = rows * cols4;
    int64_t blocks = (elems + 4 * 256 - 1) / (4 * 256);
    const int64_t cap = (int64_t)sm_count() * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    MM_CUDA(launch_pdl(copy_rows_vec4_kernel, dim3((unsigned)blocks), dim3(256), 0, s, (const float*)x->data,
                       (float*)y->data, rows, (int)cols4, g[0].stride[0], g[1].stride[0]),
            "mm_copy launch");
    MM_LAUNCH_CHECK("mm_copy launch");
    return MM_OK;
  }
  unsigned grid = grid_for(n, 256, (int64_t)sm_count() * 8);
  if (x->dtype == MM_F32)
    copy_strided_kernel<float><<<grid, 256, 0, s>>>((const float*)x->data, (float*)y->data, n,
                                                    to_dev(g[0]), to_dev(g[1]));
  else
    copy_strided_kernel<int64_t><<<grid, 256, 0, s>>>((const int64_t*)x->data, (int64_t*)y->data,
                                                      n, to_dev(g[0]), to_dev(g[1]));
  MM_LAUNCH_CHECK("mm_copy launch");
  return MM_OK;
}

extern "C" int mm_copy(const mm_tensor_t* x, const mm_tensor_t* y, void* stream) {
  MM_VALIDATE(x, "mm_copy input", -1);
  MM_VALIDATE(y, "mm_copy output", -1);
  return copy_impl(x, y, resolve_stream(stream));
}

extern "C" int mm_cat(const mm_tensor_t* const* inputs, int n, int dim, const mm_tensor_t* y,
                      void* stream) {
  MM_VALIDATE(y, "mm_cat output", -1);
  if (n <= 0) return fail(MM_ERR_INVALID, "mm_cat: no inputs");
  if (dim < 0 || dim >= y->ndim) return fail(MM_ERR_INVALID, "mm_cat: dim out of range");
  cudaStream_t s = resolve_stream(stream);
  int64_t offset = 0;
  for (int i = 0; i < n; ++i) {
    const mm_tensor_t* x = inputs[i];
    MM_VALIDATE(x, "mm_cat input", y->dtype);
    if (x->ndim != y->ndim) return fail(MM_ERR_INVALID, "mm_cat: rank mismatch");
    for (int d = 0; d < y->ndim; ++d)
      if (d != dim && x->size[d] != y->size[d]) return fail(MM_ERR_INVALID, "mm_cat: shape mismatch");
    mm_tensor_t slot = *y;
    slot.size[dim] = x->size[dim];
    size_t es = y->dtype == MM_F32 ? 4 : 8;
    slot.data = (char*)y->data + offset * y->stride[dim] * es;
    offset += x->size[dim];
    if (offset > y->size[dim]) return fail(MM_ERR_INVALID, "mm_cat: inputs exceed output");
    int rc = copy_impl(x, &slot, s);
    if (rc != MM_OK) return rc;
  }
  if (offset != y->size[dim]) return fail(MM_ERR_INVALID, "mm_cat: inputs do not fill output");
  return MM_OK;
}

extern "C" int mm_batch_norm(const mm_tensor_t* x, const float* mean, const float* var,
                             const float* weight, const float* bias, double eps,
                             const mm_tensor_t* y, void* stream) {
  MM_VALIDATE(x, "mm_batch_norm input", MM_F32);
  MM_VALIDATE(y, "mm_batch_norm output", MM_F32);
  if (x->ndim < 2) return fail(MM_ERR_UNSUPPORTED, "mm_batch_norm: rank must be >= 2");
  if (mean == nullptr || var == nullptr) return fail(MM_ERR_INVALID, "mm_batch_norm: missing stats");
  int64_t n = numel(x);
  if (n == 0) return MM_OK;
  // Channel index geometry: stride 1 along dim 1, 0 elsewhere.
  mm_tensor_t ct = *x;
  for (int i = 0; i < ct.ndim; ++i) ct.stride[i] = (i == 1) ? 1 : 0;
  Geom gx, gy, gc;
  gx.nd = gy.nd = gc.nd = x->ndim;
  for (int i = 0; i < x->ndim; ++i) {
    gx.size[i] = gy.size[i] = gc.size[i] = x->size[i];
    gx.stride[i] = x->stride[i];
    gy.stride[i] = y->stride[i];
    gc.stride[i] = ct.stride[i];
  }
  cudaStream_t s = resolve_stream(stream);
  unsigned grid = grid_for(n, 256, (int64_t)sm_count() * 8);
  bn_eval_kernel<<<grid, 256, 0, s>>>((const float*)x->data, (float*)y->data, n, to_dev(gx),
                                      to_dev(gy), to_dev(gc), mean, var, weight, bias, (float)eps);
  MM_LAUNCH_CHECK("mm_batch_norm launch");
  return MM_OK;
}

extern "C" int mm_softmax(const mm_tensor_t* x, int dim, int log_mode, const mm_tensor_t* y,
                          void* stream) {
  MM_VALIDATE(x, "mm_softmax input", MM_F32);
  MM_VALIDATE(y, "mm_softmax output", MM_F32);
  if (x->ndim == 0) {
    // Scalar softmax: exp(0) / 1 = 1, log-softmax = 0.
    return mm_fill(y, log_mode ? 0.0 : 1.0, stream);
  }
  if (dim < 0 || dim >= x->ndim) return fail(MM_ERR_INVALID, "mm_softmax: dim out of range");
  int64_t len = x->size[dim];
  int64_t n = numel(x);
  if (n == 0) return MM_OK;
  int64_t rows = n / len;
  // Row geometry: all dims except `dim`.
  mm_tensor_t rx = *x, ry = *y;
  rx.size[dim] = 1;
  ry.size[dim] = 1;
  const mm_tensor_t* ops[2] = {&rx, &ry};
  Geom g[2];
  int rc = collapse(2, ops, g);
  if (rc != MM_OK) return rc;
  cudaStream_t s = resolve_stream(stream);
  unsigned grid = grid_for(rows * 32, 256, (int64_t)sm_count() * 16);
  softmax_rows_kernel<<<grid, 256, 0, s>>>((const float*)x->data, (float*)y->data, rows, len,
                                           to_dev(g[0]), to_dev(g[1]), x->stride[dim],
                                           y->stride[dim], log_mode);
  MM_LAUNCH_CHECK("mm_softmax launch");
  return MM_OK;
}

extern "C" int mm_max_pool2d(const mm_tensor_t* x, int kh, int kw, int sh, int sw, int ph, int pw,
                             int dh, int dw, const mm_tensor_t* y, void* stream) {
  MM_VALIDATE(x, "mm_max_pool2d input", MM_F32);
  MM_VALIDATE(y, "mm_max_pool2d output", MM_F32);
  if (kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 || dh <= 0 || dw <= 0 || ph < 0 || pw < 0)
    return fail(MM_ERR_INVALID, "mm_max_pool2d: invalid window");
  Pool4 p;
  int rc = pool4(x, y, &p, "mm_max_pool2d");
  if (rc != MM_OK) return rc;
  int64_t total = p.n * p.c * p.oh * p.ow;
  if (total == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  max_pool2d_kernel<<<grid_for(total, 256, (int64_t)sm_count() * 8), 256, 0, s>>>(
      (const float*)x->data, (float*)y->data, p, kh, kw, sh, sw, ph, pw, dh, dw);
  MM_LAUNCH_CHECK("mm_max_pool2d launch");
  return MM_OK;
}

extern "C" int mm_sppf_pool(const mm_tensor_t* x, const mm_tensor_t* y1, const mm_tensor_t* y2,
                            const mm_tensor_t* y3, void* stream) {
  MM_VALIDATE(x, "mm_sppf_pool input", MM_F32);
  MM_VALIDATE(y1, "mm_sppf_pool y1", MM_F32);
  MM_VALIDATE(y2, "mm_sppf_pool y2", MM_F32);
  MM_VALIDATE(y3, "mm_sppf_pool y3", MM_F32);
  Pool4 p, q2, q3;
  int rc = pool4(x, y1, &p, "mm_sppf_pool");
  if (rc == MM_OK) rc = pool4(x, y2, &q2, "mm_sppf_pool");
  if (rc == MM_OK) rc = pool4(x, y3, &q3, "mm_sppf_pool");
  if (rc != MM_OK) return rc;
  if (p.oh != p.h || p.ow != p.w || q2.oh != p.h || q2.ow != p.w || q3.oh != p.h || q3.ow != p.w)
    return fail(MM_ERR_INVALID, "mm_sppf_pool: outputs must match the input's spatial size");
  // Channels-last tensors with 16-byte aligned pixels: the float4 kernel, 4 *
  // CG4 channels per block (CG4 = 2 when the channel count allows it).
  {
    auto v4_ok = [](const mm_tensor_t* t) {
      return t->stride[1] == 1 && t->stride[0] % 4 == 0 && t->stride[2] % 4 == 0 && t->stride[3] % 4 == 0 &&
             (((uintptr_t)t->data) & 15) == 0;
    };
    const int cg4 = p.c % 8 == 0 ? 2 : 1;
    const int64_t total = p.h * p.w * cg4;
    const int64_t blocks = p.n * (p.c / (4 * cg4));
    if (p.c % 4 == 0 && v4_ok(x) && v4_ok(y1) && v4_ok(y2) && v4_ok(y3) &&
        total <= (int64_t)SPPF4_THREADS * SPPF4_MAXE && 2 * total * 16 <= 48 * 1024 && blocks > 0 &&
        blocks <= 0x7fffffffLL) {
      cudaStream_t s = resolve_stream(stream);
      const size_t bytes = (size_t)(2 * total * 16);
      const int cgroups = (int)(p.c / (4 * cg4));
      cudaError_t e = cg4 == 2
          ? launch_pdl(sppf_image_v4_kernel<2>, dim3((unsigned)blocks), dim3(SPPF4_THREADS), bytes, s,
                       (const float*)x->data, (float*)y1->data, (float*)y2->data, (float*)y3->data, p, q2, q3,
                       cgroups)
          : launch_pdl(sppf_image_v4_kernel<1>, dim3((unsigned)blocks), dim3(SPPF4_THREADS), bytes, s,
                       (const float*)x->data, (float*)y1->data, (float*)y2->data, (float*)y3->data, p, q2, q3,
                       cgroups);
      MM_CUDA(e, "mm_sppf_pool launch");
      MM_LAUNCH_CHECK("mm_sppf_pool launch");
      return MM_OK;
    }
  }
  int64_t cgroups = (p.c + SPPF_CG - 1) / SPPF_CG;
  {
    // Whole image per block when two copies of it fit in 48 KB of shared memory.
    const int64_t bytes = 2 * p.h * p.w * SPPF_CG * (int64_t)sizeof(float);
    const int64_t blocks = p.n * cgroups;
    if (bytes <= 48 * 1024 && blocks > 0 && blocks <= 0x7fffffffLL) {
      cudaStream_t s = resolve_stream(stream);
      MM_CUDA(launch_pdl(sppf_image_kernel, dim3((unsigned)blocks), dim3(256), (size_t)bytes, s,
                         (const float*)x->data, (float*)y1->data, (float*)y2->data, (float*)y3->data, p,
                         q2, q3, (int)cgroups),
              "mm_sppf_pool launch");
      MM_LAUNCH_CHECK("mm_sppf_pool launch");
      return MM_OK;
    }
  }
  int64_t tiles_w = (p.w + SPPF_TW - 1) / SPPF_TW, tiles_h = (p.h + SPPF_TH - 1) / SPPF_TH;
  int64_t blocks = p.n * cgroups * tiles_h * tiles_w;
  if (blocks == 0) return MM_OK;
  if (blocks > 0x7fffffffLL) return fail(MM_ERR_UNSUPPORTED, "mm_sppf_pool: tensor too large");
  cudaStream_t s = resolve_stream(stream);
  sppf_kernel<<<(unsigned)blocks, 256, 0, s>>>((const float*)x->data, (float*)y1->data,
                                                (float*)y2->data, (float*)y3->data, p, q2, q3,
                                                tiles_w, tiles_h, cgroups);
  MM_LAUNCH_CHECK("mm_sppf_pool launch");
  return MM_OK;
}

extern "C" int mm_avg_pool2d(const mm_tensor_t* x, int kh, int kw, int sh, int sw, int ph, int pw,
                             int count_include_pad, int divisor_override, const mm_tensor_t* y,
                             void* stream) {
  MM_VALIDATE(x, "mm_avg_pool2d input", MM_F32);
  MM_VALIDATE(y, "mm_avg_pool2d output", MM_F32);
  if (kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 || ph < 0 || pw < 0)
    return fail(MM_ERR_INVALID, "mm_avg_pool2d: invalid window");
  Pool4 p;
  int rc = pool4(x, y, &p, "mm_avg_pool2d");
  if (rc != MM_OK) return rc;
  int64_t total = p.n * p.c * p.oh * p.ow;
  if (total == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  avg_pool2d_kernel<<<grid_for(total, 256, (int64_t)sm_count() * 8), 256, 0, s>>>(
      (const float*)x->data, (float*)y->data, p, kh, kw, sh, sw, ph, pw, count_include_pad,
      divisor_override);
  MM_LAUNCH_CHECK("mm_avg_pool2d launch");
  return MM_OK;
}

extern "C" int mm_adaptive_avg_pool2d(const mm_tensor_t* x, const mm_tensor_t* y, void* stream) {
  MM_VALIDATE(x, "mm_adaptive_avg_pool2d input", MM_F32);
  MM_VALIDATE(y, "mm_adaptive_avg_pool2d output", MM_F32);
  Pool4 p;
  int rc = pool4(x, y, &p, "mm_adaptive_avg_pool2d");
  if (rc != MM_OK) return rc;
  if (p.oh <= 0 || p.ow <= 0) return fail(MM_ERR_INVALID, "mm_adaptive_avg_pool2d: empty output");
  int64_t total = p.n * p.c * p.oh * p.ow;
  if (total == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  adaptive_avg_pool2d_kernel<<<grid_for(total, 256, (int64_t)sm_count() * 8), 256, 0, s>>>(
      (const float*)x->data, (float*)y->data, p);
  MM_LAUNCH_CHECK("mm_adaptive_avg_pool2d launch");
  return MM_OK;
}

extern "C" int mm_reduce(const mm_tensor_t* x, uint32_t dim_mask, int mean, const mm_tensor_t* y,
                         void* stream) {
  MM_VALIDATE(x, "mm_reduce input", MM_F32);
  MM_VALIDATE(y, "mm_reduce output", MM_F32);
  if (y->ndim != x->ndim) return fail(MM_ERR_INVALID, "mm_reduce: output must keep reduced dims");
  mm_tensor_t kx = *x, ky = *y, red = *x;
  int64_t nred = 1, nout = 1;
  for (int i = 0; i < x->ndim; ++i) {
    if (dim_mask & (1u << i)) {
      if (y->size[i] != 1) return fail(MM_ERR_INVALID, "mm_reduce: reduced dim must have size 1");
      nred *= x->size[i];
      kx.size[i] = 1;
      ky.size[i] = 1;
    } else {
      if (y->size[i] != x->size[i]) return fail(MM_ERR_INVALID, "mm_reduce: shape mismatch");
      nout *= x->size[i];
      red.size[i] = 1;
    }
  }
  if (nout == 0) return MM_OK;
  const mm_tensor_t* kops[2] = {&kx, &ky};
  Geom gk[2];
  int rc = collapse(2, kops, gk);
  if (rc != MM_OK) return rc;
  const mm_tensor_t* rops[1] = {&red};
  Geom gr[1];
  rc = collapse(1, rops, gr);
  if (rc != MM_OK) return rc;
  cudaStream_t s = resolve_stream(stream);
  if (nred == 0) return mm_fill(y, mean ? NAN : 0.0, stream);
  reduce_kernel<<<grid_for(nout * 32, 256, (int64_t)sm_count() * 16), 256, 0, s>>>(
      (const float*)x->data, (float*)y->data, nout, nred, to_dev(gk[0]), to_dev(gk[1]),
      to_dev(gr[0]), mean);
  MM_LAUNCH_CHECK("mm_reduce launch");
  return MM_OK;
}

extern "C" int mm_upsample_nearest2d(const mm_tensor_t* x, double scale_h, double scale_w,
                                     const mm_tensor_t* y, void* stream) {
  MM_VALIDATE(x, "mm_upsample_nearest2d input", MM_F32);
  MM_VALIDATE(y, "mm_upsample_nearest2d output", MM_F32);
  Pool4 p;
  int rc = pool4(x, y, &p, "mm_upsample_nearest2d");
  if (rc != MM_OK) return rc;
  int64_t total = p.n * p.c * p.oh * p.ow;
  if (total == 0) return MM_OK;
  if (p.h == 0 || p.w == 0) return fail(MM_ERR_INVALID, "mm_upsample_nearest2d: empty input");
  // torch: scale = user scale given ? (float)(1/scale) : (float)in/out.
  float fh = scale_h > 0 ? (float)(1.0 / scale_h) : (float)p.h / (float)p.oh;
  float fw = scale_w > 0 ? (float)(1.0 / scale_w) : (float)p.w / (float)p.ow;
  cudaStream_t s = resolve_stream(stream);
  bool nhwc4 = x->stride[1] == 1 && y->stride[1] == 1 && p.c % 4 == 0 &&
               p.xs[2] % 4 == 0 && p.xs[3] % 4 == 0 && p.ys[2] % 4 == 0 && p.ys[3] % 4 == 0 &&
               p.xs[0] % 4 == 0 && p.ys[0] % 4 == 0 &&
               ((((uintptr_t)x->data) | ((uintptr_t)y->data)) & 15) == 0;
  if (nhwc4 && p.oh == 2 * p.h && p.ow == 2 * p.w && p.w * (p.c / 4) <= 0x7fffffffLL) {
    const int64_t row_elems = p.w * (p.c / 4);
    const dim3 grid((unsigned)std::min<int64_t>((row_elems + 255) / 256, 1024),
                    (unsigned)std::min<int64_t>(p.n * p.h, 65535));
    MM_CUDA(launch_pdl(upsample2x_nhwc4_kernel, grid, dim3(256), 0, s, (const float*)x->data,
                       (float*)y->data, p),
            "mm_upsample_nearest2d launch");
  } else if (nhwc4) {
    upsample_nearest_nhwc4_kernel<<<grid_for(total / 4, 256, (int64_t)sm_count() * 8), 256, 0, s>>>(
        (const float*)x->data, (float*)y->data, p, fh, fw);
  } else {
    upsample_nearest_kernel<<<grid_for(total, 256, (int64_t)sm_count() * 8), 256, 0, s>>>(
        (const float*)x->data, (float*)y->data, p, fh, fw);
  }
  MM_LAUNCH_CHECK("mm_upsample_nearest2d launch");
  return MM_OK;
}

extern "C" int mm_yolo_decode(const mm_tensor_t* const* feats, const float* strides, int nlevels,
                              int reg_max, int nc, const mm_tensor_t* out, void* stream) {
  MM_VALIDATE(out, "mm_yolo_decode output", MM_F32);
  if (nlevels <= 0 || nlevels > 4) return fail(MM_ERR_UNSUPPORTED, "mm_yolo_decode: 1..4 levels");
  if (reg_max <= 0 || nc < 0) return fail(MM_ERR_INVALID, "mm_yolo_decode: bad reg_max/nc");
  if (out->ndim != 3 || out->size[1] != 4 + nc)
    return fail(MM_ERR_INVALID, "mm_yolo_decode: output must be [B, 4+nc, A]");
  DecodeArgs a;
  a.nlevels = nlevels;
  a.reg_max = reg_max;
  a.nc = nc;
  a.batch = out->size[0];
  int64_t anchors = 0;
  for (int l = 0; l < nlevels; ++l) {
    const mm_tensor_t* f = feats[l];
    MM_VALIDATE(f, "mm_yolo_decode feature", MM_F32);
    // Feature tensors come as logical [B, C, H, W] views.
    if (f->ndim != 4 || f->size[0] != a.batch || f->size[1] != 4 * reg_max + nc)
      return fail(MM_ERR_INVALID, "mm_yolo_decode: feature must be [B, 4*reg_max+nc, H, W]");
    DecodeLevel& L = a.lv[l];
    L.base = (const float*)f->data;
    L.sn = f->stride[0];
    L.sc = f->stride[1];
    L.sh = f->stride[2];
    L.sw = f->stride[3];
    L.h = f->size[2];
    L.w = f->size[3];
    L.anchor0 = anchors;
    L.stride = strides[l];
    anchors += L.h * L.w;
  }
  if (out->size[2] != anchors) return fail(MM_ERR_INVALID, "mm_yolo_decode: anchor count mismatch");
  a.anchors = anchors;
  a.out = (float*)out->data;
  a.on = out->stride[0];
  a.oc = out->stride[1];
  a.oa = out->stride[2];
  int64_t total = a.batch * anchors;
  if (total == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  bool rows = reg_max == 16 && nc % 4 == 0 && anchors < 0x7fffffffLL;
  for (int l = 0; l < nlevels && rows; ++l) {
    const DecodeLevel& L = a.lv[l];
    rows = L.sc == 1 && ((uintptr_t)L.base & 15) == 0 && L.sw % 4 == 0 && L.sh % 4 == 0 &&
           L.sn % 4 == 0;
  }
  if (rows) {
    const dim3 grid((unsigned)((anchors + 127) / 128), (unsigned)std::min<int64_t>(a.batch, 65535));
    MM_CUDA(launch_pdl(yolo_decode_rows_kernel, grid, dim3(128), 0, s, a), "mm_yolo_decode launch");
    MM_LAUNCH_CHECK("mm_yolo_decode launch");
    return MM_OK;
  }
  yolo_decode_kernel<<<grid_for(total, 128, (int64_t)sm_count() * 16), 128, 0, s>>>(a);
  MM_LAUNCH_CHECK("mm_yolo_decode launch");
  return MM_OK;
}

extern "C" int mm_tf32_split(const float* src, float* hi, float* lo, int64_t n, void* stream) {
  if (n <= 0) return MM_OK;
  if (!src || !hi || !lo) return fail(MM_ERR_INVALID, "mm_tf32_split: null pointer");
  cudaStream_t s = resolve_stream(stream);
  tf32_split_kernel<<<grid_for(n, 256, (int64_t)sm_count() * 8), 256, 0, s>>>(src, hi, lo, n);
  MM_LAUNCH_CHECK("mm_tf32_split launch");
  return MM_OK;
}
