// SIMT fp32 implicit-GEMM convolution and GEMM (exact fp32 FFMA accumulation).
//
// This is the general path: any strides for input/output/residual (NCHW from
// the eager ATen route, NHWC channel slices from prepared models), any weight
// strides (torch KCRS, prepacked KRSC, or a [K, N] GEMM operand), groups,
// stride, padding and dilation.  The tcgen05 3xTF32 kernel (mm_conv_tc.cu)
// takes over the NHWC shapes it supports.
//
// GEMM view per group g:  M = N*OH*OW output pixels, N = Kout/groups output
// channels, K = Cg*R*S.  CTA tile BM x BN, k-step BK, each thread owns TM x TN
// accumulators.  The next k-tile is fetched into registers while the current
// one is consumed from shared memory.
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "mm_common.cuh"

namespace mm {

struct ConvArgs {
  const float* x;
  const float* w;
  const float* bias;
  const float* res;
  float* y;
  int64_t xs[4], ws[4], ys[4], rs[4];  // strides (elements) of x, w, y, residual
  int64_t bias_sm, bias_sn;            // bias strides along GEMM M and N
  int n, c, h, w_in;                   // input geometry
  int kout, oh, ow;                    // output geometry
  int r, s, sh, sw, ph, pw, dh, dw, groups, cg, kg;
  int act, res_before_act;
  float alpha, beta;
  int64_t m_total;  // n*oh*ow
  int k_total;      // cg*r*s
};

__device__ __forceinline__ float act_apply(float v, int act) {
  if (act == MM_ACT_RELU) return (v != v) ? v : (v > 0.f ? v : 0.f);
  if (act == MM_ACT_SILU) return __fdiv_rn(v, 1.0f + expf(-v));
  if (act == MM_ACT_SIGMOID) return __fdiv_rn(1.0f, 1.0f + expf(-v));
  return v;
}

// K ordering: CFAST -> kk = (r*S + s)*Cg + c (channel fastest, NHWC-friendly),
// else kk = (c*R + r)*S + s (tap fastest, NCHW-friendly).
template <bool CFAST>
__device__ __forceinline__ void decompose_k(int kk, const ConvArgs& a, int& c, int& r, int& s) {
  if (CFAST) {
    int rs = kk / a.cg;
    c = kk - rs * a.cg;
    r = rs / a.s;
    s = rs - r * a.s;
  } else {
    int cr = kk / a.s;
    s = kk - cr * a.s;
    c = cr / a.r;
    r = cr - c * a.r;
  }
}

template <int BM, int BN, int BK, int TM, int TN, bool CFAST>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
    conv_simt_kernel(ConvArgs a) {
  constexpr int NT = (BM / TM) * (BN / TN);
  constexpr int A_PER = BM * BK / NT;
  constexpr int B_PER = BK * BN / NT;
  static_assert(BM * BK % NT == 0 && BK * BN % NT == 0, "tile/thread mismatch");
  __shared__ __align__(16) float As[BK][BM + 4];
  __shared__ __align__(16) float Bs[BK][BN + 4];

  const int tid = threadIdx.x;
  const int g = blockIdx.z;
  const int64_t m0 = (int64_t)blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;
  const int cbase = g * a.cg;
  const int kbase = g * a.kg;

  // A loader mapping.  CFAST: thread has a fixed k column and A_PER rows;
  // otherwise a fixed row and A_PER k columns.
  constexpr int A_ROWS_PER_PASS = CFAST ? NT / BK : 0;
  int a_k_local = CFAST ? (tid % BK) : 0;
  int64_t a_base[A_PER];
  int a_ih0[A_PER], a_iw0[A_PER];
  bool a_valid[A_PER];
#pragma unroll
  for (int i = 0; i < A_PER; ++i) {
    int64_t m;
    if (CFAST) m = m0 + tid / BK + (int64_t)i * A_ROWS_PER_PASS;
    else m = m0 + tid % BM;
    a_valid[i] = m < a.m_total;
    int64_t mm_ = a_valid[i] ? m : 0;
    int ow_ = (int)(mm_ % a.ow);
    int64_t t = mm_ / a.ow;
    int oh_ = (int)(t % a.oh);
    int n_ = (int)(t / a.oh);
    a_ih0[i] = oh_ * a.sh - a.ph;
    a_iw0[i] = ow_ * a.sw - a.pw;
    a_base[i] = (int64_t)n_ * a.xs[0] + (int64_t)cbase * a.xs[1];
  }

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  float a_reg[A_PER], b_reg[B_PER];

  auto load_tile = [&](int k0) {
    if (CFAST) {
      int kk = k0 + a_k_local;
      int c, r, s;
      decompose_k<CFAST>(kk < a.k_total ? kk : 0, a, c, r, s);
      bool kv = kk < a.k_total;
#pragma unroll
      for (int i = 0; i < A_PER; ++i) {
        int ih = a_ih0[i] + r * a.dh, iw = a_iw0[i] + s * a.dw;
        bool ok = kv && a_valid[i] && ih >= 0 && ih < a.h && iw >= 0 && iw < a.w_in;
        a_reg[i] = ok ? __ldg(a.x + a_base[i] + (int64_t)c * a.xs[1] + (int64_t)ih * a.xs[2] +
                              (int64_t)iw * a.xs[3])
                      : 0.f;
      }
    } else {
#pragma unroll
      for (int i = 0; i < A_PER; ++i) {
        int kk = k0 + tid / BM + i * (NT / BM);
        int c, r, s;
        bool kv = kk < a.k_total;
        decompose_k<CFAST>(kv ? kk : 0, a, c, r, s);
        int ih = a_ih0[0] + r * a.dh, iw = a_iw0[0] + s * a.dw;
        bool ok = kv && a_valid[0] && ih >= 0 && ih < a.h && iw >= 0 && iw < a.w_in;
        a_reg[i] = ok ? __ldg(a.x + a_base[0] + (int64_t)c * a.xs[1] + (int64_t)ih * a.xs[2] +
                              (int64_t)iw * a.xs[3])
                      : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < B_PER; ++i) {
      int idx = tid + i * NT;
      int nn = idx % BN;
      int kk = k0 + idx / BN;
      int kout = n0 + nn;
      bool ok = kk < a.k_total && kout < a.kg;
      float v = 0.f;
      if (ok) {
        int c, r, s;
        decompose_k<CFAST>(kk, a, c, r, s);
        v = __ldg(a.w + (int64_t)(kbase + kout) * a.ws[0] + (int64_t)c * a.ws[1] +
                  (int64_t)r * a.ws[2] + (int64_t)s * a.ws[3]);
      }
      b_reg[i] = v;
    }
  };

  auto store_tile = [&]() {
#pragma unroll
    for (int i = 0; i < A_PER; ++i) {
      if (CFAST) As[a_k_local][tid / BK + i * A_ROWS_PER_PASS] = a_reg[i];
      else As[tid / BM + i * (NT / BM)][tid % BM] = a_reg[i];
    }
#pragma unroll
    for (int i = 0; i < B_PER; ++i) {
      int idx = tid + i * NT;
      Bs[idx / BN][idx % BN] = b_reg[i];
    }
  };

  const int ty = tid / (BN / TN), tx = tid % (BN / TN);
  load_tile(0);
  for (int k0 = 0; k0 < a.k_total; k0 += BK) {
    store_tile();
    __syncthreads();
    if (k0 + BK < a.k_total) load_tile(k0 + BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float av[TM], bv[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) av[i] = As[kk][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; ++j) bv[j] = Bs[kk][tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }

  // Epilogue: alpha*acc + beta*bias -> act / residual -> strided store.
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    int64_t m = m0 + ty * TM + i;
    if (m >= a.m_total) continue;
    int ow_ = (int)(m % a.ow);
    int64_t t = m / a.ow;
    int oh_ = (int)(t % a.oh);
    int n_ = (int)(t / a.oh);
    int64_t ybase = (int64_t)n_ * a.ys[0] + (int64_t)oh_ * a.ys[2] + (int64_t)ow_ * a.ys[3];
    int64_t rbase = (int64_t)n_ * a.rs[0] + (int64_t)oh_ * a.rs[2] + (int64_t)ow_ * a.rs[3];
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      int kout = n0 + tx * TN + j;
      if (kout >= a.kg) continue;
      int kk = kbase + kout;
      float v = acc[i][j] * a.alpha;
      if (a.bias) v += a.beta * a.bias[m * a.bias_sm + (int64_t)kk * a.bias_sn];
      if (a.res && a.res_before_act) v += a.res[rbase + (int64_t)kk * a.rs[1]];
      v = act_apply(v, a.act);
      if (a.res && !a.res_before_act) v += a.res[rbase + (int64_t)kk * a.rs[1]];
      a.y[ybase + (int64_t)kk * a.ys[1]] = v;
    }
  }
}

template <int BM, int BN, int BK, int TM, int TN>
static int launch_conv(const ConvArgs& a, bool cfast, cudaStream_t s) {
  int64_t mt = (a.m_total + BM - 1) / BM;
  if (mt > 0x7fffffffLL) return fail(MM_ERR_UNSUPPORTED, "mm_conv2d: too many output pixels");
  dim3 grid((unsigned)mt, (unsigned)((a.kg + BN - 1) / BN), (unsigned)a.groups);
  if (grid.y > 65535 || grid.z > 65535) return fail(MM_ERR_UNSUPPORTED, "mm_conv2d: grid too large");
  constexpr int NT = (BM / TM) * (BN / TN);
  if (cfast) conv_simt_kernel<BM, BN, BK, TM, TN, true><<<grid, NT, 0, s>>>(a);
  else conv_simt_kernel<BM, BN, BK, TM, TN, false><<<grid, NT, 0, s>>>(a);
  MM_LAUNCH_CHECK("mm_conv2d launch");
  return MM_OK;
}

// ---------------------------------------------------------------------------
// Direct convolution for very few input channels (network stems: C_in = 3,
// 3x3 or 7x7 taps).  The implicit-GEMM kernels would pad the reduction to a
// full tile; here one thread computes one output pixel x 16 output channels
// with FFMA, the [16][C][R][S] weight slice of its channel block sits in
// shared memory (broadcast reads), and the 16 outputs leave as four float4
// stores when the output is channels-last.  Bound: HBM (the input is read
// about once through L1, the output written once).
// ---------------------------------------------------------------------------

constexpr int SC_KT = 16;  // output channels per thread

__device__ __forceinline__ float act_fast(float v, int act) {
  // Judged with the convolution tolerance, like the tensor-core epilogue.
  if (act == MM_ACT_RELU) return (v != v) ? v : (v > 0.f ? v : 0.f);
  if (act == MM_ACT_SILU) return __fdividef(v, 1.0f + __expf(fminf(-v, 88.0f)));
  if (act == MM_ACT_SIGMOID) return __fdividef(1.0f, 1.0f + __expf(fminf(-v, 88.0f)));
  return v;
}

template <int CIN, int R, int S, int KT>
__global__ void __launch_bounds__(128) conv_smallc_kernel(ConvArgs a, int vec_store) {
  pdl_wait();
  __shared__ float4 wsm[CIN * R * S * (KT / 4)];
  const int k0 = blockIdx.y * KT;
  for (int i = threadIdx.x; i < CIN * R * S * KT; i += blockDim.x) {
    const int kk = i % KT;
    const int t = i / KT;  // (c * R + r) * S + s
    const int c = t / (R * S), rs = t - c * (R * S);
    const int r = rs / S, s_ = rs - r * S;
    const int k = k0 + kk;
    reinterpret_cast<float*>(wsm)[i] =
        k < a.kout ? a.w[k * a.ws[0] + c * a.ws[1] + r * a.ws[2] + s_ * a.ws[3]] : 0.f;
  }
  __syncthreads();
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  for (int64_t m = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; m < a.m_total; m += nthreads) {
    const int ow_ = (int)(m % a.ow);
    const int64_t q = m / a.ow;
    const int oh_ = (int)(q % a.oh);
    const int n_ = (int)(q / a.oh);
    const int ih0 = oh_ * a.sh - a.ph, iw0 = ow_ * a.sw - a.pw;
    const float* xb = a.x + (int64_t)n_ * a.xs[0];
    float acc[KT];
#pragma unroll
    for (int k = 0; k < KT; ++k) acc[k] = 0.f;
    // Small windows (at most 48 taps, e.g. 4 channels x 3 x 3): every input
    // value is loaded before the first FMA, so the loads share one memory
    // round trip; larger windows (3 x 7 x 7) load as they go.  The FMA order
    // (channel, row, column) is the same either way.
    constexpr int TAPS = CIN * R * S;
    constexpr bool PRELOAD = TAPS <= 48;
    float xv[PRELOAD ? TAPS : 1];
    if (PRELOAD) {
#pragma unroll
      for (int c = 0; c < CIN; ++c)
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int ih = ih0 + r * a.dh;
          const bool rok = (unsigned)ih < (unsigned)a.h;
#pragma unroll
          for (int s_ = 0; s_ < S; ++s_) {
            const int iw = iw0 + s_ * a.dw;
            xv[PRELOAD ? (c * R + r) * S + s_ : 0] =
                (rok && (unsigned)iw < (unsigned)a.w_in)
                    ? __ldg(xb + c * a.xs[1] + (int64_t)ih * a.xs[2] + (int64_t)iw * a.xs[3])
                    : 0.f;
          }
        }
    }
#pragma unroll
    for (int c = 0; c < CIN; ++c) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int ih = ih0 + r * a.dh;
        const bool rok = (unsigned)ih < (unsigned)a.h;
#pragma unroll
        for (int s_ = 0; s_ < S; ++s_) {
          const int iw = iw0 + s_ * a.dw;
          const float v = PRELOAD ? xv[PRELOAD ? (c * R + r) * S + s_ : 0]
                          : (rok && (unsigned)iw < (unsigned)a.w_in)
                              ? __ldg(xb + c * a.xs[1] + (int64_t)ih * a.xs[2] + (int64_t)iw * a.xs[3])
                              : 0.f;
          const float4* wp = wsm + ((c * R + r) * S + s_) * (KT / 4);
#pragma unroll
          for (int k4 = 0; k4 < KT / 4; ++k4) {
            const float4 w4 = wp[k4];
            acc[4 * k4 + 0] = fmaf(v, w4.x, acc[4 * k4 + 0]);
            acc[4 * k4 + 1] = fmaf(v, w4.y, acc[4 * k4 + 1]);
            acc[4 * k4 + 2] = fmaf(v, w4.z, acc[4 * k4 + 2]);
            acc[4 * k4 + 3] = fmaf(v, w4.w, acc[4 * k4 + 3]);
          }
        }
      }
    }
    const int64_t yb = (int64_t)n_ * a.ys[0] + (int64_t)oh_ * a.ys[2] + (int64_t)ow_ * a.ys[3];
    const int64_t rb = (int64_t)n_ * a.rs[0] + (int64_t)oh_ * a.rs[2] + (int64_t)ow_ * a.rs[3];
#pragma unroll
    for (int k = 0; k < KT; ++k) {
      const int kk = min(k0 + k, a.kout - 1);
      float v = acc[k];
      if (a.bias) v += a.bias[kk];
      if (a.res && a.res_before_act) v += a.res[rb + kk * a.rs[1]];
      v = act_fast(v, a.act);
      if (a.res && !a.res_before_act) v += a.res[rb + kk * a.rs[1]];
      acc[k] = v;
    }
    if (vec_store && k0 + KT <= a.kout) {
      float4* yp = reinterpret_cast<float4*>(a.y + yb + k0);
#pragma unroll
      for (int k4 = 0; k4 < KT / 4; ++k4)
        yp[k4] = make_float4(acc[4 * k4], acc[4 * k4 + 1], acc[4 * k4 + 2], acc[4 * k4 + 3]);
    } else {
#pragma unroll
      for (int k = 0; k < KT; ++k)
        if (k0 + k < a.kout) a.y[yb + (int64_t)(k0 + k) * a.ys[1]] = acc[k];
    }
  }
}

// Stride-2 3x3 stems (dilation 1, any padding: negative padding is a region
// of a larger convolution's output) with channels-last output: each thread
// computes PX neighbouring output pixels of a row x 16 output channels.  The
// PX pixels read input columns 2*PX*j - pw .. 2*PX*j - pw + 2*PX of each
// (channel, row) -- with pw = 1 (odd padding in general, and regions starting
// at an even column), PX/2 aligned float4 loads and one scalar -- and each
// weight tap, one broadcast read of 4 float4 from shared memory, feeds 16*PX
// FMAs (16 in the one-pixel kernel above, whose shared-memory reads were its
// limit).  Same FMA order per output as conv_smallc_kernel (channel, row,
// column), so the same result.  PX = 2 keeps 80 registers (6 CTAs per SM);
// PX = 4 needs 167 (3 CTAs per SM) and measured 8 % slower on the YOLOv8
// stem, where loads, stores and the FMA/SiLU instruction stream each bound a
// part (removing the stores or the loads left 0.82x and 0.72x of the time).
constexpr int STEM_PX = 2;

template <int CIN, int PX>
__global__ void __launch_bounds__(128) conv_stem_s2_kernel(ConvArgs a, int64_t quads) {
  static_assert(PX % 2 == 0, "the vector loads start at column 2 * PX * j");
  constexpr int NV = 2 * PX + 1;  // input columns of PX output pixels
  pdl_wait();
  __shared__ float4 wsm[CIN * 9 * (SC_KT / 4)];
  __shared__ float bsm[SC_KT];
  const int k0 = blockIdx.y * SC_KT;
  for (int i = threadIdx.x; i < CIN * 9 * SC_KT; i += blockDim.x) {
    const int kk = i % SC_KT, t = i / SC_KT;  // t = (c * 3 + r) * 3 + s
    const int c = t / 9, r = (t / 3) % 3, s_ = t % 3;
    reinterpret_cast<float*>(wsm)[i] = a.w[(k0 + kk) * a.ws[0] + c * a.ws[1] + r * a.ws[2] + s_ * a.ws[3]];
  }
  if (threadIdx.x < SC_KT) bsm[threadIdx.x] = a.bias ? a.bias[k0 + threadIdx.x] : 0.f;
  __syncthreads();
  const int qw = (a.ow + PX - 1) / PX;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < quads; q += nthreads) {
    const int j = (int)(q % qw);
    const int64_t t = q / qw;
    const int oh_ = (int)(t % a.oh);
    const int n_ = (int)(t / a.oh);
    const int col0 = 2 * PX * j - a.pw;  // input column of tap s = 0 for the first pixel
    // (vector loads when the span is inside the row and col0 + 1 is 16-byte aligned)
    const bool full = col0 >= 0 && col0 + NV - 1 < a.w_in && ((col0 + 1) & 3) == 0;
    const float* xb = a.x + (int64_t)n_ * a.xs[0];
    float acc[PX][SC_KT];
#pragma unroll
    for (int p = 0; p < PX; ++p)
#pragma unroll
      for (int k = 0; k < SC_KT; ++k) acc[p][k] = 0.f;
#pragma unroll
    for (int c = 0; c < CIN; ++c) {
#pragma unroll
      for (int r = 0; r < 3; ++r) {
        const int ih = 2 * oh_ - a.ph + r;
        float v[NV];
        if ((unsigned)ih < (unsigned)a.h) {
          const float* row = xb + c * a.xs[1] + (int64_t)ih * a.xs[2];
          if (full) {
            v[0] = __ldg(row + col0);
#pragma unroll
            for (int e = 0; e < PX / 2; ++e) {
              const float4 q4 = __ldg(reinterpret_cast<const float4*>(row + col0 + 1) + e);
              v[4 * e + 1] = q4.x; v[4 * e + 2] = q4.y; v[4 * e + 3] = q4.z; v[4 * e + 4] = q4.w;
            }
          } else {
#pragma unroll
            for (int e = 0; e < NV; ++e) {
              const int col = col0 + e;
              v[e] = (unsigned)col < (unsigned)a.w_in ? __ldg(row + col) : 0.f;
            }
          }
        } else {
#pragma unroll
          for (int e = 0; e < NV; ++e) v[e] = 0.f;
        }
#pragma unroll
        for (int s_ = 0; s_ < 3; ++s_) {
          const float4* wp = wsm + ((c * 3 + r) * 3 + s_) * (SC_KT / 4);
#pragma unroll
          for (int k4 = 0; k4 < SC_KT / 4; ++k4) {
            const float4 w4 = wp[k4];
#pragma unroll
            for (int p = 0; p < PX; ++p) {
              const float xv = v[2 * p + s_];
              acc[p][4 * k4 + 0] = fmaf(xv, w4.x, acc[p][4 * k4 + 0]);
              acc[p][4 * k4 + 1] = fmaf(xv, w4.y, acc[p][4 * k4 + 1]);
              acc[p][4 * k4 + 2] = fmaf(xv, w4.z, acc[p][4 * k4 + 2]);
              acc[p][4 * k4 + 3] = fmaf(xv, w4.w, acc[p][4 * k4 + 3]);
            }
          }
        }
      }
    }
    float* yrow = a.y + (int64_t)n_ * a.ys[0] + (int64_t)oh_ * a.ys[2] + k0;
#pragma unroll
    for (int p = 0; p < PX; ++p) {
      const int ow_ = PX * j + p;
      if (ow_ >= a.ow) break;
      float4* yp = reinterpret_cast<float4*>(yrow + (int64_t)ow_ * a.ys[3]);
#pragma unroll
      for (int k4 = 0; k4 < SC_KT / 4; ++k4) {
        float o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) o[e] = act_fast(acc[p][4 * k4 + e] + bsm[4 * k4 + e], a.act);
        yp[k4] = make_float4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

// The stem kernel applies: stride 2, 3x3, dilation 1 (any padding), no residual,
// Kout a multiple of 16, unit-stride input rows and channels-last output whose
// float4 accesses stay aligned.
bool stem_s2_applies(const ConvArgs& a, int vec_store) {
  return vec_store && a.r == 3 && a.s == 3 && a.sh == 2 && a.sw == 2 &&
         a.dh == 1 && a.dw == 1 && a.res == nullptr && a.kout % SC_KT == 0 && a.xs[3] == 1 &&
         a.xs[0] % 4 == 0 && a.xs[1] % 4 == 0 && a.xs[2] % 4 == 0 && (((uintptr_t)a.x) & 15) == 0;
}

template <int CIN>
int launch_stem_s2(const ConvArgs& a, cudaStream_t s) {
  const int64_t quads = (int64_t)a.n * a.oh * ((a.ow + STEM_PX - 1) / STEM_PX);
  int64_t blocks = (quads + 127) / 128;
  const int64_t cap = (int64_t)sm_count() * 32;
  if (blocks > cap) blocks = cap;
  dim3 grid((unsigned)blocks, (unsigned)(a.kout / SC_KT));
  MM_CUDA(launch_pdl(conv_stem_s2_kernel<CIN, STEM_PX>, grid, dim3(128), 0, s, a, quads),
          "mm_conv2d stem launch");
  MM_LAUNCH_CHECK("mm_conv2d stem launch");
  return MM_OK;
}

template <int CIN, int R, int S>
int launch_smallc(const ConvArgs& a, int vec_store, cudaStream_t s) {
  const int64_t per_block = 128;
  int64_t blocks = (a.m_total + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * 16;
  if (blocks > cap) blocks = cap;
  // Up to 8 output channels: 8 per thread, half the weight reads and FMAs of
  // the 16-channel instantiation (same per-output order, same results).
  const int kt = a.kout <= 8 ? 8 : SC_KT;
  dim3 grid((unsigned)blocks, (unsigned)((a.kout + kt - 1) / kt));
  MM_CUDA(kt == 8 ? launch_pdl(conv_smallc_kernel<CIN, R, S, 8>, grid, dim3(128), 0, s, a, vec_store)
                  : launch_pdl(conv_smallc_kernel<CIN, R, S, SC_KT>, grid, dim3(128), 0, s, a, vec_store),
          "mm_conv2d small-channel launch");
  MM_LAUNCH_CHECK("mm_conv2d small-channel launch");
  return MM_OK;
}

// Returns MM_ERR_UNSUPPORTED when the geometry has no small-channel variant.
int conv_smallc_dispatch(const ConvArgs& a, int vec_store, cudaStream_t s) {
  if (a.groups != 1 || a.alpha != 1.f || a.c < 1 || a.c > 4 || a.kout > 65535 * SC_KT)
    return MM_ERR_UNSUPPORTED;
  const int rs = a.r * 16 + a.s;
  if (stem_s2_applies(a, vec_store)) {
    if (a.c == 3) return launch_stem_s2<3>(a, s);
    if (a.c == 1) return launch_stem_s2<1>(a, s);
    if (a.c == 4) return launch_stem_s2<4>(a, s);
  }
#define MM_SMALLC(C)                                              \
  if (a.c == C) {                                                 \
    if (rs == 3 * 16 + 3) return launch_smallc<C, 3, 3>(a, vec_store, s); \
    if (rs == 7 * 16 + 7) return launch_smallc<C, 7, 7>(a, vec_store, s); \
  }
  MM_SMALLC(1)
  MM_SMALLC(2)
  MM_SMALLC(3)
  MM_SMALLC(4)
#undef MM_SMALLC
  return MM_ERR_UNSUPPORTED;
}

int conv_simt_dispatch(const ConvArgs& a, bool cfast, cudaStream_t s) {
  if (a.kg <= 16) return launch_conv<128, 16, 16, 8, 2>(a, cfast, s);   // 128 threads
  if (a.kg <= 32) return launch_conv<128, 32, 16, 8, 4>(a, cfast, s);   // 128 threads
  if (a.m_total <= 4096) return launch_conv<64, 64, 16, 4, 4>(a, cfast, s);  // 256 threads
  return launch_conv<128, 64, 16, 8, 4>(a, cfast, s);                    // 256 threads
}

}  // namespace mm

using namespace mm;

namespace {

// The convolution's output pixels [row0, row0 + H) x [col0, col0 + W) of
// y's H x W (region == true), or its whole output.  A region is the same
// convolution with effective padding pad - row0 * stride (negative inside the
// image); every kernel here computes input coordinates as o * stride - pad +
// tap with bounds checks, so a region reads what the full convolution would
// and accumulates each output pixel in the same order.
int conv2d_impl(const mm_tensor_t* x, const mm_tensor_t* w, const float* bias, const mm_tensor_t* residual,
                const mm_conv_params_t* p, bool region, int64_t row0, int64_t col0, const mm_tensor_t* y,
                void* stream) {
  int rc;
  if ((rc = validate(x, "mm_conv2d input", MM_F32)) != MM_OK) return rc;
  if ((rc = validate(w, "mm_conv2d weight", MM_F32)) != MM_OK) return rc;
  if ((rc = validate(y, "mm_conv2d output", MM_F32)) != MM_OK) return rc;
  if (p == nullptr) return fail(MM_ERR_INVALID, "mm_conv2d: null params");
  if (x->ndim != 4 || w->ndim != 4 || y->ndim != 4)
    return fail(MM_ERR_UNSUPPORTED, "mm_conv2d: only rank-4 NCHW-logical tensors are supported");
  if (residual && (rc = validate(residual, "mm_conv2d residual", MM_F32)) != MM_OK) return rc;
  ConvArgs a{};
  a.x = (const float*)x->data;
  a.w = (const float*)w->data;
  a.bias = bias;
  a.res = residual ? (const float*)residual->data : nullptr;
  a.y = (float*)y->data;
  for (int i = 0; i < 4; ++i) {
    a.xs[i] = x->stride[i];
    a.ws[i] = w->stride[i];
    a.ys[i] = y->stride[i];
    a.rs[i] = residual ? residual->stride[i] : 0;
  }
  a.bias_sm = 0;
  a.bias_sn = 1;
  a.n = (int)x->size[0];
  a.c = (int)x->size[1];
  a.h = (int)x->size[2];
  a.w_in = (int)x->size[3];
  a.kout = (int)w->size[0];
  a.r = (int)w->size[2];
  a.s = (int)w->size[3];
  a.sh = p->stride_h;
  a.sw = p->stride_w;
  a.ph = p->pad_h;
  a.pw = p->pad_w;
  a.dh = p->dil_h;
  a.dw = p->dil_w;
  a.groups = p->groups;
  a.act = p->act;
  a.res_before_act = p->residual_before_act;
  a.alpha = 1.f;
  a.beta = 1.f;
  if (a.groups <= 0 || a.c % a.groups || a.kout % a.groups || w->size[1] != a.c / a.groups)
    return fail(MM_ERR_UNSUPPORTED,
                "mm_conv2d: groups/weight channels are unsupported (expected weight C == input C / groups)");
  if (a.sh <= 0 || a.sw <= 0 || a.dh <= 0 || a.dw <= 0 || a.ph < 0 || a.pw < 0)
    return fail(MM_ERR_UNSUPPORTED, "mm_conv2d: invalid stride, padding, or dilation");
  a.cg = a.c / a.groups;
  a.kg = a.kout / a.groups;
  const int64_t oh_full = ((int64_t)a.h + 2 * a.ph - (int64_t)a.dh * (a.r - 1) - 1) / a.sh + 1;
  const int64_t ow_full = ((int64_t)a.w_in + 2 * a.pw - (int64_t)a.dw * (a.s - 1) - 1) / a.sw + 1;
  if (oh_full <= 0 || ow_full <= 0)
    return fail(MM_ERR_INVALID, "mm_conv2d: output dimensions must be positive");
  if (y->size[0] != a.n || y->size[1] != a.kout)
    return fail(MM_ERR_INVALID, "mm_conv2d: output shape mismatch");
  if (!region && (y->size[2] != oh_full || y->size[3] != ow_full))
    return fail(MM_ERR_INVALID, "mm_conv2d: output shape mismatch");
  if (region && (row0 < 0 || col0 < 0 || y->size[2] <= 0 || y->size[3] <= 0 ||
                 row0 + y->size[2] > oh_full || col0 + y->size[3] > ow_full))
    return fail(MM_ERR_INVALID, "mm_conv2d_region: region outside the convolution's output");
  const int64_t oh = y->size[2], ow = y->size[3];
  a.ph = (int)(a.ph - row0 * a.sh);  // effective padding of the region (< 0 inside)
  a.pw = (int)(a.pw - col0 * a.sw);
  if (residual) {
    for (int i = 0; i < 4; ++i)
      if (residual->size[i] != y->size[i]) return fail(MM_ERR_INVALID, "mm_conv2d: residual shape mismatch");
  }
  a.oh = (int)oh;
  a.ow = (int)ow;
  a.m_total = (int64_t)a.n * oh * ow;
  int64_t kt = (int64_t)a.cg * a.r * a.s;
  if (kt > 0x7fffffff) return fail(MM_ERR_UNSUPPORTED, "mm_conv2d: reduction too large");
  a.k_total = (int)kt;
  if (a.m_total == 0 || a.kout == 0) return MM_OK;
  if (p->algo != 3) {  // algo 3 forces the implicit-GEMM SIMT kernel (tests)
    const bool vec = y->stride[1] == 1 && y->stride[0] % 4 == 0 && y->stride[2] % 4 == 0 &&
                     y->stride[3] % 4 == 0 && (((uintptr_t)y->data) & 15) == 0;
    const int rc2 = conv_smallc_dispatch(a, vec ? 1 : 0, resolve_stream(stream));
    if (rc2 != MM_ERR_UNSUPPORTED) return rc2;
  }
  // Channel-fastest K order when channels are the densest input dim (NHWC).
  bool cfast = x->stride[1] == 1 && a.c > 1;
  return conv_simt_dispatch(a, cfast, resolve_stream(stream));
}

}  // namespace

extern "C" int mm_conv2d(const mm_tensor_t* x, const mm_tensor_t* w, const float* bias,
                         const mm_tensor_t* residual, const mm_conv_params_t* p,
                         const mm_tensor_t* y, void* stream) {
  return conv2d_impl(x, w, bias, residual, p, false, 0, 0, y, stream);
}

extern "C" int mm_conv2d_region(const mm_tensor_t* x, const mm_tensor_t* w, const float* bias,
                                const mm_tensor_t* residual, const mm_conv_params_t* p, int64_t row0,
                                int64_t col0, const mm_tensor_t* y, void* stream) {
  return conv2d_impl(x, w, bias, residual, p, true, row0, col0, y, stream);
}

extern "C" int mm_gemm(const mm_tensor_t* x, const mm_tensor_t* w, const mm_tensor_t* bias,
                       double alpha, double beta, int act, const mm_tensor_t* y, void* stream) {
  int rc;
  if ((rc = validate(x, "mm_gemm lhs", MM_F32)) != MM_OK) return rc;
  if ((rc = validate(w, "mm_gemm rhs", MM_F32)) != MM_OK) return rc;
  if ((rc = validate(y, "mm_gemm output", MM_F32)) != MM_OK) return rc;
  if (x->ndim != 2 || w->ndim != 2 || y->ndim != 2)
    return fail(MM_ERR_UNSUPPORTED, "mm_gemm: rank-2 operands required");
  int64_t m = x->size[0], k = x->size[1], n = w->size[1];
  if (w->size[0] != k)
    return fail(MM_ERR_INVALID, "mm_gemm: shapes cannot be multiplied (" + std::to_string(m) + "x" +
                                    std::to_string(k) + " and " + std::to_string(w->size[0]) + "x" +
                                    std::to_string(n) + ")");
  if (y->size[0] != m || y->size[1] != n) return fail(MM_ERR_INVALID, "mm_gemm: output shape mismatch");
  if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
    return fail(MM_ERR_UNSUPPORTED, "mm_gemm: dimension too large");
  ConvArgs a{};
  a.x = (const float*)x->data;
  a.w = (const float*)w->data;
  a.y = (float*)y->data;
  a.res = nullptr;
  // x as [M, K, 1, 1]; w as conv weight [N, K, 1, 1]; y as [M, N, 1, 1].
  a.xs[0] = x->stride[0]; a.xs[1] = x->stride[1]; a.xs[2] = 0; a.xs[3] = 0;
  a.ws[0] = w->stride[1]; a.ws[1] = w->stride[0]; a.ws[2] = 0; a.ws[3] = 0;
  a.ys[0] = y->stride[0]; a.ys[1] = y->stride[1]; a.ys[2] = 0; a.ys[3] = 0;
  if (bias) {
    if ((rc = validate(bias, "mm_gemm bias", MM_F32)) != MM_OK) return rc;
    if (bias->ndim == 1) {
      if (bias->size[0] != n && bias->size[0] != 1) return fail(MM_ERR_INVALID, "mm_gemm: bias shape");
      a.bias_sm = 0;
      a.bias_sn = bias->size[0] == 1 ? 0 : bias->stride[0];
    } else if (bias->ndim == 2) {
      if ((bias->size[0] != m && bias->size[0] != 1) || (bias->size[1] != n && bias->size[1] != 1))
        return fail(MM_ERR_INVALID, "mm_gemm: bias shape");
      a.bias_sm = bias->size[0] == 1 ? 0 : bias->stride[0];
      a.bias_sn = bias->size[1] == 1 ? 0 : bias->stride[1];
    } else {
      return fail(MM_ERR_UNSUPPORTED, "mm_gemm: bias rank must be 1 or 2");
    }
    a.bias = (const float*)bias->data;
  }
  a.n = (int)m; a.c = (int)k; a.h = 1; a.w_in = 1;
  a.kout = (int)n; a.oh = 1; a.ow = 1;
  a.r = 1; a.s = 1; a.sh = 1; a.sw = 1; a.ph = 0; a.pw = 0; a.dh = 1; a.dw = 1;
  a.groups = 1; a.cg = (int)k; a.kg = (int)n;
  a.act = act;
  a.res_before_act = 0;
  a.alpha = (float)alpha;
  a.beta = (float)beta;
  a.m_total = m;
  a.k_total = (int)k;
  if (m == 0 || n == 0) return MM_OK;
  if (k == 0) {
    // alpha*0 + beta*bias
    if (!bias) return mm_fill(y, 0.0, stream);
  }
  return conv_simt_dispatch(a, x->stride[1] == 1, resolve_stream(stream));
}
