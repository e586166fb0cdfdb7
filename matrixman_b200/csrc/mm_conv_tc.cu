// tcgen05 implicit-GEMM convolution with a 3xTF32 split (fp32-accurate).
//
// GEMM view:  D[M = N*OH*OW pixels, N = Kout] = A[M, K] * B[K, N], K ordered
// (tap r, tap s, channel c) with channels padded to C_pad (multiple of 32).
//
// Persistent CTAs (one per SM) walk a static list of 128-pixel x BN-channel
// tiles.  Warp roles:
//   * warps 0-7 (A producers): gather 128 pixel rows x 32 channels per k-block
//     with 16-byte loads (zero for padding taps, out-of-range pixels and padded
//     channels), prefetching the next k-block into registers while the current
//     one is split into a tf32 high part (round to nearest) and the exact fp32
//     remainder and stored into 128B-swizzled K-major stage buffers;
//   * warp 8 (TMA): prepacked [K_pad][R*S*C_pad] weight hi/lo planes, one 2-D
//     tiled load each per stage (no multicast);
//   * warp 9 (MMA): one thread issues, per 8-wide k step, three
//     tcgen05.mma.kind::tf32 (A_hi*B_hi + A_hi*B_lo + A_lo*B_hi) into one of two
//     TMEM period buffers; every `period` k-blocks the buffer is handed over;
//   * warps 10-13 (accumulator): add each finished period into an fp32 total
//     kept in TMEM with round-to-nearest adds -- the tensor core's own
//     accumulation rounds toward zero, so long reductions inside TMEM drift by
//     ~K * 2^-24 -- and, after the last period, apply bias, activation and the
//     optional residual and store the NHWC output (possibly a channel slice of
//     a concat buffer).  This overlaps the epilogue of one tile with the MMAs
//     of the next.
//
// Every wait is bounded: on timeout the kernel records an error code in
// g_tc_error (read with mm_kernel_error), stops issuing work, waits for its
// in-flight MMAs and bulk copies, frees its TMEM and returns; other CTAs see
// the code and stop as well.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>
#include <unordered_map>

#include "mm_common.cuh"

namespace mm {

__device__ int g_tc_error = 0;

constexpr int TC_BM = 128;        // pixels per tile (MMA M)
constexpr int TC_BK = 32;         // channels per k-block (128 bytes of fp32)
constexpr uint32_t TC_SPIN_LIMIT = 1u << 26;

enum TcError { TC_ERR_NONE = 0, TC_ERR_WAIT_A = 1, TC_ERR_WAIT_B = 2, TC_ERR_WAIT_EMPTY = 3,
               TC_ERR_WAIT_ACC = 4 };

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool tc_error_raised() {
  return *reinterpret_cast<volatile int*>(&g_tc_error) != 0;
}

// Bounded wait; returns false (and records `code`) after TC_WAIT_NS, or at
// once when another CTA has already recorded an error, so a stuck pipeline
// ends the whole grid within a fraction of a second.
constexpr uint64_t TC_WAIT_NS = 200ull * 1000 * 1000;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1; i < TC_SPIN_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 0) {
      if (tc_error_raised()) return false;
      if (global_ns() - t0 > TC_WAIT_NS) break;
    }
    if (i > 64) __nanosleep(32);
  }
  atomicCAS(&g_tc_error, 0, code);
  return false;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128B swizzle, 8-row groups 1024 B
// apart (stride byte offset), sm_100 descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);        // start address
  d |= (uint64_t)1 << 16;                        // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;              // stride byte offset
  d |= (uint64_t)1 << 46;                        // descriptor version
  d |= (uint64_t)2 << 61;                        // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::tf32, fp32 accumulate, K-major A and B.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4)                      // D format: f32
         | (2u << 7)                    // A format: tf32
         | (2u << 10)                   // B format: tf32
         | ((uint32_t)(n >> 3) << 17)   // N / 8
         | ((uint32_t)(m >> 4) << 24);  // M / 16
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  uint32_t mask = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(mask)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float tc_act(float v, int act) {
  if (act == MM_ACT_RELU) return (v != v) ? v : (v > 0.f ? v : 0.f);
  if (act == MM_ACT_SILU) return __fdiv_rn(v, 1.0f + expf(-v));
  if (act == MM_ACT_SIGMOID) return __fdiv_rn(1.0f, 1.0f + expf(-v));
  return v;
}

// tf32 high part rounded to nearest (ties away); the remainder x - hi is exact
// in fp32 and at most half a tf32 ulp of x.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__device__ __forceinline__ float4 split_hi(float4 v) {
  return make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
}

struct TcArgs {
  const float* x;
  int64_t xs0, xs2, xs3;  // NHWC pixel strides (channel stride is 1)
  float* y;
  int64_t ys0, ys2, ys3;
  const float* res;
  int64_t rs0, rs2, rs3;
  const float* bias;
  int h, w, c;
  int oh, ow, kout;
  int r, s, sh, sw, ph, pw, dh, dw;
  int64_t m_total;
  int kb_total;  // r * s * (c_pad / 32)
  int cb;        // c_pad / 32
  int bn;        // N tile: multiple of 16, <= 128
  int n_tiles;   // ceil(kout / bn)
  int64_t tiles; // m tiles * n tiles
  int stages;
  int period;    // k-blocks accumulated in TMEM before promotion to the fp32 total
  int act, res_before_act;
  int vec_store;  // output rows 16-byte aligned: float4 stores
  uint32_t tmem_cols;
};

// Warp roles of the persistent kernel.
constexpr int TC_A_WARPS = 8;                 // warps 0-7: A producers
constexpr int TC_WARP_TMA = 8;                // warp 8: weight TMA
constexpr int TC_WARP_MMA = 9;                // warp 9: MMA issue + TMEM owner
                                              // warps 10-13: promotion + epilogue
constexpr int TC_V2_THREADS = 14 * 32;
constexpr int TC_A_ROWS = TC_BM / (TC_A_WARPS * 32 / 8);  // rows per producer thread (4)

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}

__global__ void __launch_bounds__(TC_V2_THREADS, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap wmap_hi,
                   const __grid_constant__ CUtensorMap wmap_lo, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int S = a.stages;
  const uint32_t a_bytes = TC_BM * 128;
  const uint32_t b_bytes = (uint32_t)a.bn * 128;
  const uint32_t stage_bytes = 2 * a_bytes + 2 * b_bytes;
  uint64_t* bars = (uint64_t*)(smem + (size_t)S * stage_bytes);
  uint64_t* full_a = bars;            // S: 256 producer arrivals
  uint64_t* full_b = bars + S;        // S: TMA transaction bytes
  uint64_t* empty = bars + 2 * S;     // S: MMA commit frees the stage
  uint64_t* buf_full = bars + 3 * S;  // 2: MMA commit, a period is in TMEM
  uint64_t* buf_free = bars + 3 * S + 2;  // 2: 128 promotion arrivals
  uint64_t* drain = bars + 3 * S + 4;     // 1: MMA error path waits for its MMAs
  uint32_t* tmem_slot = (uint32_t*)(bars + 3 * S + 5);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  __shared__ int s_skip;
  if (threadIdx.x == 0) s_skip = tc_error_raised() ? 1 : 0;
  __syncthreads();
  if (s_skip) return;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_a[i], TC_A_WARPS * 32);
      mbar_init(&full_b[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&buf_full[i], 1);
      mbar_init(&buf_free[i], 128);
    }
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == TC_WARP_MMA) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(a.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: period buffers at [0, bn) and [bn, 2 bn), fp32 total at [2 bn, 3 bn).
  const int KB = a.kb_total;
  const int NP = (KB + a.period - 1) / a.period;

  if (warp < TC_A_WARPS) {
    // ---------------- A producers: gather, split, store (register prefetch) --------------
    const int t = threadIdx.x;
    const int j = t & 7;
    const int row0 = t >> 3;  // 0..31; rows row0 + 32 i
    const uint32_t swz = (uint32_t)((j ^ (row0 & 7)) << 4);
    int64_t g = 0;  // global k-block counter across tiles
    bool alive = true;
    for (int64_t tile = blockIdx.x; tile < a.tiles && alive; tile += gridDim.x) {
      const int64_t m0 = (tile / a.n_tiles) * TC_BM;
      int64_t base[TC_A_ROWS];
      int ih0[TC_A_ROWS], iw0[TC_A_ROWS];
      bool rowok[TC_A_ROWS];
#pragma unroll
      for (int i = 0; i < TC_A_ROWS; ++i) {
        const int64_t m = m0 + row0 + 32 * i;
        rowok[i] = m < a.m_total;
        const int64_t mm_ = rowok[i] ? m : 0;
        const int ow_ = (int)(mm_ % a.ow);
        const int64_t q = mm_ / a.ow;
        const int oh_ = (int)(q % a.oh);
        base[i] = (q / a.oh) * a.xs0;
        ih0[i] = oh_ * a.sh - a.ph;
        iw0[i] = ow_ * a.sw - a.pw;
      }
      float4 nxt[TC_A_ROWS];
      auto fetch = [&](int kb, float4* v) {
        const int tap = kb / a.cb;
        const int cbk = kb - tap * a.cb;
        const int kr = tap / a.s, ks = tap - kr * a.s;
        const int c = cbk * TC_BK + j * 4;
#pragma unroll
        for (int i = 0; i < TC_A_ROWS; ++i) {
          const int ih = ih0[i] + kr * a.dh, iw = iw0[i] + ks * a.dw;
          const bool ok = rowok[i] && c < a.c && ih >= 0 && ih < a.h && iw >= 0 && iw < a.w;
          v[i] = ok ? __ldg(reinterpret_cast<const float4*>(a.x + base[i] + (int64_t)ih * a.xs2 +
                                                             (int64_t)iw * a.xs3 + c))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      };
      fetch(0, nxt);
      for (int kb = 0; kb < KB; ++kb, ++g) {
        float4 cur[TC_A_ROWS];
#pragma unroll
        for (int i = 0; i < TC_A_ROWS; ++i) cur[i] = nxt[i];
        if (kb + 1 < KB) fetch(kb + 1, nxt);  // next loads in flight while storing this block
        const int st = (int)(g % S);
        if (!mbar_wait(&empty[st], (uint32_t)((g / S) & 1) ^ 1u, TC_ERR_WAIT_EMPTY)) {
          alive = false;
          break;
        }
        uint8_t* ahi = smem + (size_t)st * stage_bytes;
        uint8_t* alo = ahi + a_bytes;
#pragma unroll
        for (int i = 0; i < TC_A_ROWS; ++i) {
          const uint32_t off = (uint32_t)(row0 + 32 * i) * 128u + swz;
          const float4 hv = split_hi(cur[i]);
          *reinterpret_cast<float4*>(ahi + off) = hv;
          *reinterpret_cast<float4*>(alo + off) =
              make_float4(cur[i].x - hv.x, cur[i].y - hv.y, cur[i].z - hv.z, cur[i].w - hv.w);
        }
        fence_proxy_async_smem();
        mbar_arrive(&full_a[st]);
      }
    }
  } else if (warp == TC_WARP_TMA) {
    // ---------------- weights via TMA ----------------
    if (lane == 0) {
      int64_t g = 0;
      bool alive = true;
      for (int64_t tile = blockIdx.x; tile < a.tiles && alive; tile += gridDim.x) {
        const int n0 = (int)(tile % a.n_tiles) * a.bn;
        for (int kb = 0; kb < KB; ++kb, ++g) {
          const int st = (int)(g % S);
          if (!mbar_wait(&empty[st], (uint32_t)((g / S) & 1) ^ 1u, TC_ERR_WAIT_EMPTY)) {
            alive = false;
            break;
          }
          uint8_t* bhi = smem + (size_t)st * stage_bytes + 2 * a_bytes;
          mbar_arrive_expect_tx(&full_b[st], 2 * b_bytes);
          tma_load_2d(bhi, &wmap_hi, &full_b[st], kb * TC_BK, n0);
          tma_load_2d(bhi + b_bytes, &wmap_lo, &full_b[st], kb * TC_BK, n0);
        }
      }
      // Bulk copies must not outlive the CTA's shared memory.
      for (int64_t k = (g > S ? g - S : 0); k < g; ++k)
        mbar_wait(&full_b[k % S], (uint32_t)((k / S) & 1), TC_ERR_WAIT_B);
    }
  } else if (warp == TC_WARP_MMA) {
    // ---------------- MMA issue: periods into two TMEM buffers ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32(TC_BM, a.bn);
      int64_t g = 0, pc = 0;
      bool alive = true;
      for (int64_t tile = blockIdx.x; tile < a.tiles && alive; tile += gridDim.x) {
        for (int p = 0; p < NP && alive; ++p, ++pc) {
          const int b = (int)(pc & 1);
          if (!mbar_wait(&buf_free[b], (uint32_t)((pc >> 1) & 1) ^ 1u, TC_ERR_WAIT_ACC)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(b * a.bn);
          const int kb_end = min(KB, (p + 1) * a.period);
          for (int kb = p * a.period; kb < kb_end; ++kb, ++g) {
            const int st = (int)(g % S);
            const uint32_t par = (uint32_t)((g / S) & 1);
            if (!mbar_wait(&full_a[st], par, TC_ERR_WAIT_A) ||
                !mbar_wait(&full_b[st], par, TC_ERR_WAIT_B)) {
              alive = false;
              break;
            }
            tc_fence_after();
            const uint32_t ahi = smem_addr(smem + (size_t)st * stage_bytes);
            const uint32_t alo = ahi + a_bytes;
            const uint32_t bhi = alo + a_bytes;
            const uint32_t blo = bhi + b_bytes;
#pragma unroll
            for (int k = 0; k < TC_BK / 8; ++k) {
              const uint64_t dah = smem_desc_sw128(ahi + 32 * k), dal = smem_desc_sw128(alo + 32 * k);
              const uint64_t dbh = smem_desc_sw128(bhi + 32 * k), dbl = smem_desc_sw128(blo + 32 * k);
              mma_tf32(d, dah, dbh, idesc, (kb > p * a.period || k > 0) ? 1u : 0u);
              mma_tf32(d, dah, dbl, idesc, 1u);
              mma_tf32(d, dal, dbh, idesc, 1u);
            }
            mma_commit(&empty[st]);
          }
          mma_commit(&buf_full[b]);  // arrives once the period's MMAs have completed
        }
      }
      if (!alive) {
        // Error path: make sure no MMA still writes TMEM before it is freed.
        mma_commit(drain);
        mbar_wait(drain, 0u, TC_ERR_WAIT_ACC);
      }
    }
  } else {
    // ---------------- promotion (fp32 RN adds) + epilogue ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t total = lane_base + (uint32_t)(2 * a.bn);
    int64_t pc = 0;
    bool alive = true;
    for (int64_t tile = blockIdx.x; tile < a.tiles && alive; tile += gridDim.x) {
      const int64_t m0 = (tile / a.n_tiles) * TC_BM;
      const int n0 = (int)(tile % a.n_tiles) * a.bn;
      const int64_t m = m0 + q * 32 + lane;
      const bool rv = m < a.m_total;
      int64_t ybase = 0, rbase = 0;
      if (rv) {
        const int ow_ = (int)(m % a.ow);
        const int64_t qq = m / a.ow;
        const int oh_ = (int)(qq % a.oh);
        const int64_t n_ = qq / a.oh;
        ybase = n_ * a.ys0 + (int64_t)oh_ * a.ys2 + (int64_t)ow_ * a.ys3;
        rbase = n_ * a.rs0 + (int64_t)oh_ * a.rs2 + (int64_t)ow_ * a.rs3;
      }
      for (int p = 0; p < NP; ++p, ++pc) {
        const int b = (int)(pc & 1);
        if (!mbar_wait(&buf_full[b], (uint32_t)((pc >> 1) & 1), TC_ERR_WAIT_ACC)) {
          alive = false;
          break;
        }
        tc_fence_after();
        const bool last = p == NP - 1;
        const uint32_t buf = lane_base + (uint32_t)(b * a.bn);
        for (int c0 = 0; c0 < a.bn; c0 += 16) {
          float v[16];
          tmem_ld16(buf + (uint32_t)c0, v);
          if (p > 0) {
            float tv[16];
            tmem_ld16(total + (uint32_t)c0, tv);
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = __fadd_rn(v[e], tv[e]);
          }
          if (!last) {
            tmem_st16(total + (uint32_t)c0, v);
            continue;
          }
          if (!rv || g_tc_error != 0) continue;
#pragma unroll
          for (int gq = 0; gq < 4; ++gq) {
            const int ch = n0 + c0 + 4 * gq;
            if (ch >= a.kout) break;
            float o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int cc = ch + e;
              float val = v[4 * gq + e];
              if (cc < a.kout) {
                if (a.bias) val += a.bias[cc];
                if (a.res && a.res_before_act) val += a.res[rbase + cc];
                val = tc_act(val, a.act);
                if (a.res && !a.res_before_act) val += a.res[rbase + cc];
              }
              o[e] = val;
            }
            if (a.vec_store && ch + 3 < a.kout) {
              *reinterpret_cast<float4*>(a.y + ybase + ch) = make_float4(o[0], o[1], o[2], o[3]);
            } else {
              for (int e = 0; e < 4 && ch + e < a.kout; ++e) a.y[ybase + ch + e] = o[e];
            }
          }
        }
        if (!last) asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        mbar_arrive(&buf_free[b]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == TC_WARP_MMA) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(a.tmem_cols)
                 : "memory");
  }
}

}  // namespace mm

using namespace mm;

namespace {

struct MapKey {
  const void* ptr;
  int64_t ktot, kpad;
  int bn;
  int device;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && ktot == o.ktot && kpad == o.kpad && bn == o.bn && device == o.device;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.ptr) ^ (size_t)(k.ktot * 1315423911ull) ^ (size_t)(k.bn << 7) ^
           (size_t)k.device;
  }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// 2-D tensor map over a [kpad rows][ktot cols] fp32 weight plane, box
// {32 cols (128 bytes), bn rows}, 128B swizzle.  Rows beyond kpad read as 0.
int weight_map(const float* w, int64_t ktot, int64_t kpad, int bn, CUtensorMap* out) {
  int dev = 0;
  cudaGetDevice(&dev);
  MapKey key{w, ktot, kpad, bn, dev};
  {
    std::lock_guard<std::mutex> g(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return MM_OK;
    }
  }
  // The driver entry point is resolved through the runtime so the library does
  // not link libcuda (it must load on hosts without a driver).
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn encode = nullptr;
  if (encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
      return fail(MM_ERR_CUDA, "mm_conv2d_tc: cuTensorMapEncodeTiled entry point unavailable");
    encode = (EncodeFn)fn;
  }
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)ktot, (cuuint64_t)kpad};
  cuuint64_t strides[1] = {(cuuint64_t)ktot * 4};
  cuuint32_t box[2] = {32, (cuuint32_t)bn};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)w, dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MM_ERR_CUDA, "mm_conv2d_tc: cuTensorMapEncodeTiled failed (CUresult " +
                                 std::to_string((int)r) + ")");
  std::lock_guard<std::mutex> g(g_map_mu);
  g_maps[key] = map;
  *out = map;
  return MM_OK;
}

bool aligned16(const void* p) { return (((uintptr_t)p) & 15) == 0; }

bool nhwc_ok(const mm_tensor_t* t) {
  return t->ndim == 4 && t->stride[1] == 1 && t->stride[0] % 4 == 0 && t->stride[2] % 4 == 0 &&
         t->stride[3] % 4 == 0 && aligned16(t->data);
}

}  // namespace

extern "C" int mm_conv2d_tc(const mm_tensor_t* x, const float* w_hi, const float* w_lo, int k_out,
                            int c_in, int r, int s, int c_pad, int k_pad, const float* bias,
                            const mm_tensor_t* residual, const mm_conv_params_t* p,
                            const mm_tensor_t* y, void* stream) {
  int rc;
  if ((rc = validate(x, "mm_conv2d_tc input", MM_F32)) != MM_OK) return rc;
  if ((rc = validate(y, "mm_conv2d_tc output", MM_F32)) != MM_OK) return rc;
  if (residual && (rc = validate(residual, "mm_conv2d_tc residual", MM_F32)) != MM_OK) return rc;
  if (p == nullptr || w_hi == nullptr || w_lo == nullptr)
    return fail(MM_ERR_INVALID, "mm_conv2d_tc: null weights or params");
  if (p->groups != 1) return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: grouped convolution");
  if (!nhwc_ok(x))
    return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: input must be a 16-byte aligned NHWC view");
  if (y->ndim != 4 || y->stride[1] != 1 || (residual && (residual->ndim != 4 || residual->stride[1] != 1)))
    return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: output/residual must be NHWC views");
  if (x->size[1] != c_in || c_in % 4 != 0)
    return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: input channels must match and be a multiple of 4");
  if (c_pad % TC_BK != 0 || c_pad < c_in || k_pad % 16 != 0 || k_pad < k_out || k_out <= 0)
    return fail(MM_ERR_INVALID, "mm_conv2d_tc: bad weight padding");
  if (!aligned16(w_hi) || !aligned16(w_lo)) return fail(MM_ERR_INVALID, "mm_conv2d_tc: weights unaligned");
  if (p->stride_h <= 0 || p->stride_w <= 0 || p->dil_h <= 0 || p->dil_w <= 0 || p->pad_h < 0 ||
      p->pad_w < 0 || r <= 0 || s <= 0)
    return fail(MM_ERR_INVALID, "mm_conv2d_tc: invalid geometry");
  const int64_t n = x->size[0], h = x->size[2], w = x->size[3];
  const int64_t oh = (h + 2 * p->pad_h - (int64_t)p->dil_h * (r - 1) - 1) / p->stride_h + 1;
  const int64_t ow = (w + 2 * p->pad_w - (int64_t)p->dil_w * (s - 1) - 1) / p->stride_w + 1;
  if (oh <= 0 || ow <= 0) return fail(MM_ERR_INVALID, "mm_conv2d_tc: empty output");
  if (y->size[0] != n || y->size[1] != k_out || y->size[2] != oh || y->size[3] != ow)
    return fail(MM_ERR_INVALID, "mm_conv2d_tc: output shape mismatch");
  if (residual) {
    for (int i = 0; i < 4; ++i)
      if (residual->size[i] != y->size[i]) return fail(MM_ERR_INVALID, "mm_conv2d_tc: residual shape");
  }
  if (h > 0x7fffffff || w > 0x7fffffff) return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: too large");
  const int64_t m_total = n * oh * ow;
  if (m_total == 0) return MM_OK;

  TcArgs a{};
  a.x = (const float*)x->data;
  a.xs0 = x->stride[0]; a.xs2 = x->stride[2]; a.xs3 = x->stride[3];
  a.y = (float*)y->data;
  a.ys0 = y->stride[0]; a.ys2 = y->stride[2]; a.ys3 = y->stride[3];
  a.res = residual ? (const float*)residual->data : nullptr;
  if (residual) { a.rs0 = residual->stride[0]; a.rs2 = residual->stride[2]; a.rs3 = residual->stride[3]; }
  a.bias = bias;
  a.h = (int)h; a.w = (int)w; a.c = c_in;
  a.oh = (int)oh; a.ow = (int)ow; a.kout = k_out;
  a.r = r; a.s = s; a.sh = p->stride_h; a.sw = p->stride_w; a.ph = p->pad_h; a.pw = p->pad_w;
  a.dh = p->dil_h; a.dw = p->dil_w;
  a.m_total = m_total;
  a.cb = c_pad / TC_BK;
  a.kb_total = r * s * a.cb;
  // N tiles of at most 128 channels, balanced (e.g. 144 -> 2 x 80, 256 -> 2 x 128).
  {
    const int ntiles = (k_out + 127) / 128;
    const int per = (k_out + ntiles - 1) / ntiles;
    a.bn = ((per + 15) / 16) * 16;
  }
  a.n_tiles = (k_out + a.bn - 1) / a.bn;
  a.period = 4;
  a.act = p->act;
  a.res_before_act = p->residual_before_act;
  a.vec_store = nhwc_ok(y) ? 1 : 0;
  // Two period buffers plus the fp32 total: 3 * bn columns (power of two >= 32).
  uint32_t cols = 32;
  while (cols < (uint32_t)(3 * a.bn)) cols <<= 1;
  a.tmem_cols = cols;
  const int64_t ktot = (int64_t)r * s * c_pad;
  const size_t stage_bytes = 2 * (size_t)TC_BM * 128 + 2 * (size_t)a.bn * 128;
  const size_t budget = 200 * 1024;
  int stages = (int)((budget - 2048) / stage_bytes);
  if (stages > 6) stages = 6;
  if (stages < 2) stages = 2;
  a.stages = stages;
  const size_t smem = 1024 + (size_t)stages * stage_bytes + (3 * stages + 5) * 8 + 16;

  CUtensorMap mhi, mlo;
  if ((rc = weight_map(w_hi, ktot, k_pad, a.bn, &mhi)) != MM_OK) return rc;
  if ((rc = weight_map(w_lo, ktot, k_pad, a.bn, &mlo)) != MM_OK) return rc;

  static thread_local size_t configured = 0;
  if (configured < smem) {
    MM_CUDA(cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem),
            "mm_conv2d_tc: shared memory attribute");
    configured = smem;
  }
  const int64_t mt = (m_total + TC_BM - 1) / TC_BM;
  a.tiles = mt * a.n_tiles;
  // Persistent CTAs: one per SM (the shared-memory footprint allows one).
  const int64_t ctas = a.tiles < (int64_t)sm_count() ? a.tiles : (int64_t)sm_count();
  conv_tc_kernel<<<(unsigned)ctas, TC_V2_THREADS, smem, resolve_stream(stream)>>>(mhi, mlo, a);
  MM_LAUNCH_CHECK("mm_conv2d_tc launch");
  return MM_OK;
}

extern "C" int mm_kernel_error(int device, int* code_out, int clear) {
  if (code_out == nullptr) return fail(MM_ERR_INVALID, "mm_kernel_error: null output");
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != device) MM_CUDA(cudaSetDevice(device), "cudaSetDevice");
  int code = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&code, g_tc_error, sizeof(int));
  if (e == cudaSuccess && clear && code != 0) {
    int zero = 0;
    e = cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int));
  }
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "mm_kernel_error");
  *code_out = code;
  return MM_OK;
}
