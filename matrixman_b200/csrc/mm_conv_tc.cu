// tcgen05 implicit-GEMM convolution with a 3xTF32 split (fp32-accurate).
//
// GEMM view:  D[M = N*OH*OW pixels, N = Kout] = A[M, K] * B[K, N], K ordered
// (tap r, tap s, channel c) with channels padded to C_pad (multiple of 32).
//
// Persistent CTAs (one per SM) walk a static list of 128-pixel x BN-channel
// tiles (BN <= 80).  A sub-block is 32 channels of one tap; a k-block is
// KSUB (1 or 2, a template parameter) consecutive sub-blocks, the unit that
// every warp role hands on -- each k-block costs every role a fixed chain of
// barrier waits, copies and MMA issues, so deep reductions run two
// sub-blocks per k-block.  A stage holds the k-block's A tiles (128 pixel rows
// x 128 B each) and, per sub-block, the adjacent B hi and B lo weight tiles
// (BN rows x 128 B each) in shared memory.  The exact remainders of the A
// tiles go to a separate, shorter ring of TMEM lo slots (32 columns per
// sub-block), so the shared-memory pipeline is as deep as shared memory
// allows rather than as TMEM allows.  Warp roles (15 warps, at most four per
// SM sub-partition, so 128 registers per thread):
//   * warps 0-3 (A producers, one per TMEM lane quarter): in the TMA modes
//     they read their 32 rows x 32 channels of each A tile and write the exact
//     remainder x - tf32(x) into a TMEM lo slot with tcgen05.st; in the
//     gather mode they first fetch the tiles with 16-byte cp.async (zero-fill
//     for padding taps, rows past the end and padded channels);
//   * warp 4 (TMA): prepacked [K_pad][R*S*C_pad] weight hi/lo planes, one 2-D
//     tiled load each per sub-block, and the A tiles in the TMA modes;
//   * warp 5 (hi MMAs): A (fp32 in shared memory, which the tensor core reads
//     as tf32 -- the high part of the split) times [B hi | B lo] as one
//     N = 2 BN tcgen05.mma.kind::tf32 per 8 channels, so each A slice is read
//     from shared memory once for both products.  The [hi*hi | hi*lo] sums
//     alternate between two period buffers handed over every `period` k-blocks;
//   * warp 6 (lo MMAs): A lo (TMEM) times B hi, accumulated over a whole tile
//     (~2^-11 of the result); its commits free the stage and the lo slot.
//     Two issuing warps: tcgen05.mma issue from one thread takes about as
//     long as MMAs of these shapes run;
//   * warps 7-14 (accumulator, two per lane quarter): add each finished
//     period's hi*hi + hi*lo into an fp32 total held in registers with
//     round-to-nearest adds -- the tensor core's own accumulation rounds
//     toward zero, so long reductions inside TMEM drift by ~K * 2^-24 -- then
//     add the lo*hi sum and apply bias (staged in shared memory), activation
//     and the optional residual, and store the NHWC output (possibly a channel
//     slice of a concat buffer).  The epilogue of one tile overlaps the MMAs
//     of the next.
// The MMA issue warps and the TMA warp run their loops and waits on all 32
// lanes (warp-uniform state); one elected lane issues.
//
// Stage and phase counters advance incrementally (no divisions in the
// per-k-block paths), and per-row input offsets are computed once per tile.
//
// Every wait is bounded: on timeout the kernel records an error code in
// g_tc_error (read with mm_kernel_error), stops issuing work, waits for its
// in-flight MMAs and bulk copies, frees its TMEM and returns; other CTAs see
// the code and stop as well.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>
#include <cstdlib>
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
               TC_ERR_WAIT_ACC = 4, TC_ERR_DRAIN = 5 };

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

// Non-blocking test of a phase.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or about `ns` nanoseconds pass, instead of polling.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(ns)
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

// Bounded wait; returns false (and records `code`) after g_tc_wait_ns
// (200 ms unless a test shortened it with mm_debug_tc_fault), or soon after
// another CTA has recorded an error, so a stuck pipeline ends the whole grid
// within a fraction of a second.
constexpr uint64_t TC_WAIT_NS = 200ull * 1000 * 1000;
__device__ unsigned long long g_tc_wait_ns = TC_WAIT_NS;
// Test hook (mm_debug_tc_fault): CTA 0 issues nothing for its first k-block,
// so a wait for that stage runs out and the error path runs.
__device__ int g_tc_drop_first_load = 0;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1; i < TC_SPIN_LIMIT; ++i) {
    if (mbar_try_wait_sleep(bar, parity, 1000u)) return true;
    if ((i & 63) == 0) {
      if (tc_error_raised()) return false;
      if (global_ns() - t0 > *reinterpret_cast<volatile unsigned long long*>(&g_tc_wait_ns)) break;
    }
  }
  atomicCAS(&g_tc_error, 0, code);
  return false;
}

// Wait for this CTA's own asynchronous work (bulk copies in flight, MMAs
// committed) on the error path: it ignores the error flag -- no bulk copy may
// land in shared memory after the CTA exits, and no MMA may write TMEM after
// it is freed -- and gives up only after TC_WAIT_NS (recording TC_ERR_DRAIN).
__device__ __forceinline__ bool mbar_drain_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1; i < TC_SPIN_LIMIT; ++i) {
    if (mbar_try_wait_sleep(bar, parity, 1000u)) return true;
    if ((i & 63) == 0 && global_ns() - t0 > TC_WAIT_NS) break;
  }
  atomicCAS(&g_tc_error, 0, (int)TC_ERR_DRAIN);
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

// The same descriptor split into its halves: the high word is a constant
// (stride byte offset, version, swizzle mode); the low word holds the start
// address and the leading byte offset, so stepping along K (32 bytes) adds 2.
constexpr uint32_t TC_DESC_HI = (uint32_t)(1024 >> 4) | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint32_t smem_desc_lo(uint32_t addr) {
  return ((addr >> 4) & 0x3FFFu) | (1u << 16);
}
__device__ __forceinline__ uint64_t desc_of(uint32_t lo) {
  return ((uint64_t)TC_DESC_HI << 32) | lo;
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

// tf32 high part rounded to nearest (ties away); the remainder x - hi is exact
// in fp32 and at most half a tf32 ulp of x.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// The same rounding with two integer operations: adding half a tf32 ulp to
// the magnitude bits and clearing the 13 low mantissa bits rounds to nearest,
// ties away from zero, for every finite value (the carry propagates into the
// exponent exactly like a mantissa overflow).  Infinities and NaNs are not
// preserved (an input that holds them makes the convolution non-finite
// anyway).  Same formula as the host-side weight prepack.
__device__ __forceinline__ float tf32_rna_int(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

__device__ __forceinline__ float4 split_hi(float4 v) {
  return make_float4(tf32_rna_int(v.x), tf32_rna_int(v.y), tf32_rna_int(v.z), tf32_rna_int(v.w));
}

// Division of n < 2^31 by a runtime divisor d as a multiply and shift:
// with s = ceil(log2 d) and m = ceil(2^(31+s) / d), floor(n * m / 2^(31+s))
// equals floor(n / d) (the rounding error of m stays below 1/d).
struct FastDiv {
  uint32_t d, m, s;
};

__host__ __device__ inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f;
  f.d = d;
  f.s = 0;
  while ((1u << f.s) < d) ++f.s;
  f.m = (uint32_t)(((1ull << (31 + f.s)) + d - 1) / d);
  return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  return (uint32_t)(((uint64_t)n * f.m) >> (31 + f.s));
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
  int m_total;    // output pixels (fits in 31 bits; checked on the host)
  int sb_total;   // 32-channel sub-blocks of the reduction: r * s * (c_pad / 32)
  int ksub;       // sub-blocks per k-block (1 or 2; a template parameter of the kernel)
  int kb_total;   // k-blocks per tile: ceil(sb_total / ksub)
  int cb;         // c_pad / 32
  int bn;         // N tile: multiple of 16, <= TC_MAX_BN
  int n_tiles;    // ceil(kout / bn)
  int amode;      // how A tiles arrive: TC_A_GATHER, TC_A_FLAT or TC_A_RECT
  int tw, th;     // TC_A_RECT: output tile of th rows x tw columns (th * tw = 128)
  int ntw, nth;   // TC_A_RECT: tiles across one output image
  int64_t mtiles; // pixel tiles
  int64_t tiles;  // mtiles * n_tiles
  int stages;     // shared-memory pipeline depth (A + B hi + B lo stages)
  int lo_slots;   // TMEM lo slots (2..TC_MAX_LO, ksub * 32 columns each), a ring of its own
  int xbuf;       // lo*hi tile-sum buffers (2: the next tile's sum overlaps the epilogue)
  int epi_groups; // 2: two groups of 4 epilogue warps take alternate tiles (needs one hi*hi
                  // period per tile, xbuf == 2 and bn <= 48, so each group owns its buffers)
  int period;     // k-blocks of hi products accumulated in TMEM before promotion
  int act, res_before_act;
  int vec_store;  // output rows 16-byte aligned: float4 stores
  int stg_chunks; // > 0: the epilogue stages rows in shared memory and writes them with TMA
                  // stores (this many 16-channel chunks per epilogue warp); 0: direct stores
  int res_vec;    // residual rows 16-byte aligned: float4 loads
  FastDiv div_ow, div_oh, div_img, div_ntw;  // output width, height; rectangles per image, per row
};

// How the 128-pixel x 32-channel A tile of a k-block reaches shared memory.
constexpr int TC_A_GATHER = 0;  // producer warps, 16-byte cp.async per pixel row (any geometry)
constexpr int TC_A_FLAT = 1;    // one 2-D TMA load: 1x1, stride 1, no padding, uniform pixels
constexpr int TC_A_RECT = 2;    // one 4-D TMA load of a th x tw output-pixel rectangle
                                // (conv strides become TMA traversal strides)

// Warp roles of the persistent kernel.
// 15 warps: with at most four warps per SM sub-partition each thread may hold
// 128 registers (the epilogue keeps a tile row's fp32 total in registers).
constexpr int TC_A_WARPS = 4;      // warps 0-3: A producers (one per TMEM lane quarter)
constexpr int TC_A_HALVES = 8 / TC_A_WARPS;  // 16-channel halves of a sub-block per producer warp
constexpr int TC_WARP_TMA = TC_A_WARPS;       // TMA (weights; A in the TMA modes)
constexpr int TC_WARP_HI = TC_A_WARPS + 1;    // A hi * [B hi | B lo] MMA issue + TMEM owner
constexpr int TC_WARP_LO = TC_A_WARPS + 2;    // A lo * B hi MMA issue
constexpr int TC_WARP_EPI = TC_A_WARPS + 3;   // 8 warps: promotion + epilogue (2 per lane quarter)
constexpr int TC_EPI_WARPS = 8;
constexpr int TC_EPI_CHUNKS = 3;   // 16-column chunks per epilogue warp (bn <= 96)
constexpr int TC_THREADS = (TC_WARP_EPI + TC_EPI_WARPS) * 32;
constexpr uint32_t TC_TMEM_COLS = 512;
constexpr int TC_LO_COLS = 32;     // TMEM columns per sub-block in a lo slot
constexpr uint32_t TC_A_BYTES = TC_BM * TC_BK * 4;  // one A tile: 128 rows x 128 B
constexpr int TC_MAX_BN = 80;      // N tile limit (5-6 accumulator widths of bn columns + lo slots)
constexpr int TC_MAX_STAGES = 12;  // shared-memory stages (A + B hi + B lo)
constexpr int TC_MAX_LO = 4;       // TMEM lo slots
constexpr int TC_MAX_BIAS = 2048;  // output channels whose bias is staged in shared memory

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

// tcgen05.ld of 16 columns without the completion wait (callers batch loads
// and issue one tcgen05.wait::ld).
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// MMA with the A operand (128 x 8 tf32) read from tensor memory.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                            uint32_t idesc, uint32_t accumulate) {
  uint32_t mask = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate), "r"(mask)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(bar))
      : "memory");
}

// TMA stores of a staged box (bulk-group completion), the group commit and the
// waits for this thread's groups: `.read` returns once the source shared
// memory may be reused, the plain form once the global writes are done.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_addr(src)), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int x, int y,
                                             int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_addr(src)), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Epilogue staging: each epilogue warp owns stg_chunks boxes of 32 rows x 16
// channels (64-byte rows, 64-byte swizzle: 16-byte chunk c of row r sits at
// chunk c ^ ((r >> 1) & 3), which spreads a warp's row writes over all banks).
constexpr uint32_t TC_STG_BOX = 32 * 64;

// Shared-memory layout of one CTA (offsets from the 1024-aligned base).  A
// stage holds the ksub A tiles of a k-block (128 pixel rows x 128 B each,
// 128-byte swizzle), then per sub-block the adjacent B hi and lo tiles (bn
// rows x 128 B each); every tile offset is a multiple of 1024 bytes, as the
// swizzled layout requires.
struct TcSmem {
  uint32_t a_bytes, stage_bytes, stg, bias, bars;
  int stages;
  __host__ __device__ static TcSmem make(int bn, int ksub, int stages, int kout, int stg_chunks) {
    TcSmem l;
    l.stages = stages;
    l.a_bytes = (uint32_t)ksub * TC_A_BYTES;
    l.stage_bytes = l.a_bytes + (uint32_t)ksub * 2u * (uint32_t)bn * 128u;
    l.stg = (uint32_t)stages * l.stage_bytes;           // epilogue staging (1024-aligned)
    l.bias = l.stg + (uint32_t)TC_EPI_WARPS * (uint32_t)stg_chunks * TC_STG_BOX;  // kout floats, 16-byte padded
    l.bars = l.bias + (((uint32_t)kout * 4u + 15u) & ~15u);
    return l;
  }
  // mbarriers: full_x[S], full_b[S], fenced[S], empty[S], lo_full[TC_MAX_LO],
  // lo_empty[TC_MAX_LO], hh_full[2], hh_free[2], cross_full[2],
  // cross_free[2], drain[3] (two used); then the TMEM slot.
  __host__ __device__ int n_bars() const { return 4 * stages + 2 * TC_MAX_LO + 11; }
  __host__ __device__ size_t bytes() const { return 1024 + bars + (size_t)n_bars() * 8 + 16; }
};

// Origin of pixel tile `mt`: flat tiles start at pixel m0; rectangles at
// (image n, output row oh0, output column ow0).
struct TcTile {
  int m0, n, oh0, ow0;
};

__device__ __forceinline__ TcTile tc_tile(const TcArgs& a, int mt) {
  TcTile t;
  if (a.amode == TC_A_RECT) {
    const int per_img = a.nth * a.ntw;
    t.n = (int)fdiv((uint32_t)mt, a.div_img);
    const int rem = mt - t.n * per_img;
    const int ty = (int)fdiv((uint32_t)rem, a.div_ntw);
    t.oh0 = ty * a.th;
    t.ow0 = (rem - ty * a.ntw) * a.tw;
    t.m0 = 0;
  } else {
    t.m0 = mt * TC_BM;
    t.n = t.oh0 = t.ow0 = 0;
  }
  return t;
}

// Output coordinates of tile row `row`; false when the row is outside the
// output (last flat tile, or a rectangle overhanging the image edge).
__device__ __forceinline__ bool tc_row(const TcArgs& a, const TcTile& t, int row, int& n, int& oh,
                                       int& ow) {
  if (a.amode == TC_A_RECT) {
    const int ry = row / a.tw;
    n = t.n;
    oh = t.oh0 + ry;
    ow = t.ow0 + (row - ry * a.tw);
    return oh < a.oh && ow < a.ow;
  }
  const int m = t.m0 + row;
  if (m >= a.m_total) return false;
  const uint32_t q = fdiv((uint32_t)m, a.div_ow);
  ow = (int)((uint32_t)m - q * (uint32_t)a.ow);
  n = (int)fdiv(q, a.div_oh);
  oh = (int)(q - (uint32_t)n * (uint32_t)a.oh);
  return true;
}

// Byte offset of 16-byte chunk j of row `row` in a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t sw128_off(int row, int j) {
  return (uint32_t)(row * 128 + ((j ^ (row & 7)) << 4));
}

// The lowest active lane of the warp: the one thread that issues a warp's
// MMAs and commits (tcgen05.commit tracks the MMAs of the issuing thread).
__device__ __forceinline__ bool elect_one() {
  uint32_t leader;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 l;\n\t"
      "elect.sync l|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(leader));
  return leader != 0;
}

// Bounded wait by a whole warp, with one outcome for all lanes.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int code) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, code));
}

// One MMA issuer warp.  ROLE 0 (hi) reads the A tile straight from shared
// memory -- for fp32 data the tensor core uses the value truncated to tf32,
// which is the high part of the split -- and multiplies it by the adjacent
// B hi and B lo tiles as one N = 2 bn operand, producing [hi*hi | hi*lo] in a
// period buffer that the promotion warps fold into the fp32 total every
// `period` k-blocks (two buffers alternate).  ROLE 1 (lo) reads the exact
// remainder x - trunc(x) that the producer warps wrote into a TMEM lo slot
// and multiplies it by B hi into a per-tile buffer: its sum is ~2^-11 of the
// result, so the tensor core's round-toward-zero accumulation leaves no
// measurable drift there.  Both issuers commit to the stage's `empty`
// barrier; the lo issuer also frees the lo slot.  All 32 lanes run the loop
// and the waits (its state stays warp-uniform); one elected lane issues.
struct TcBars {
  uint64_t *full_x, *full_b, *fenced, *empty, *lo_full, *lo_empty;
  uint64_t *hh_full, *hh_free, *cross_full, *cross_free, *drain;
};

template <int ROLE, int KS>
__device__ __forceinline__ void tc_issue(const TcArgs& a, uint8_t* smem, const TcSmem& L,
                                         uint32_t tmem, const TcBars& B) {
  const int S = a.stages, KB = a.kb_total, LS = a.lo_slots;
  const int NP = (KB + a.period - 1) / a.period;
  const uint32_t slot_cols = (uint32_t)(TC_LO_COLS * KS);
  const uint32_t acc0 = slot_cols * (uint32_t)LS;
  const uint32_t bpair = 2u * (uint32_t)a.bn * 128u;  // one sub-block's B hi + B lo bytes
  const uint32_t idesc = idesc_tf32(TC_BM, ROLE == 0 ? 2 * a.bn : a.bn);
  const bool gather = a.amode == TC_A_GATHER;
  int64_t pc = 0, tc = 0;
  int st = 0;         // A/B stage of the next k-block
  uint32_t par = 0;   // its fill phase parity
  int ls = 0;         // lo slot of the next k-block (ROLE 1)
  uint32_t lpar = 0;  // its fill phase parity
  bool alive = true;
  for (int64_t tile = blockIdx.x; tile < a.tiles && alive; tile += gridDim.x, ++tc) {
    const int xb = a.xbuf == 2 ? (int)(tc & 1) : 0;
    const uint32_t xpar = (uint32_t)((a.xbuf == 2 ? tc >> 1 : tc) & 1);
    uint32_t d = tmem + acc0 + (uint32_t)((4 + xb) * a.bn);
    if (ROLE == 1) {
      if (!warp_wait(&B.cross_free[xb], xpar ^ 1u, TC_ERR_WAIT_ACC)) {
        alive = false;
        break;
      }
      tc_fence_after();
    }
    for (int p = 0; p < NP && alive; ++p) {
      if (ROLE == 0) {
        const int b = (int)(pc & 1);
        if (!warp_wait(&B.hh_free[b], (uint32_t)((pc >> 1) & 1) ^ 1u, TC_ERR_WAIT_ACC)) {
          alive = false;
          break;
        }
        tc_fence_after();
        d = tmem + acc0 + (uint32_t)(b * 2 * a.bn);
      }
      const int kb_begin = p * a.period;
      const int kb_end = min(KB, kb_begin + a.period);
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        // hi: the A tile in shared memory -- TMA modes: full_x (which carries
        // the weights too); gather mode: `fenced`, which every producer thread
        // signals after a proxy fence over its cp.async data, and full_b.
        // lo: the lo slot (its producers waited for full_x first), and full_b
        // in the gather mode.
        bool ok;
        if (ROLE == 0)
          ok = warp_wait(gather ? &B.fenced[st] : &B.full_x[st], par, TC_ERR_WAIT_A);
        else
          ok = warp_wait(&B.lo_full[ls], lpar, TC_ERR_WAIT_A);
        if (!ok || (gather && !warp_wait(&B.full_b[st], par, TC_ERR_WAIT_B))) {
          alive = false;
          break;
        }
        tc_fence_after();
        const uint32_t stage = smem_addr(smem + (size_t)st * L.stage_bytes);
        const bool first = ROLE == 0 ? kb == kb_begin : kb == 0;
        const int nsub = min(KS, a.sb_total - kb * KS);
        if (elect_one()) {
          const uint32_t b_lo0 = smem_desc_lo(stage + L.a_bytes);  // B hi, then B lo (bn rows each)
          const uint32_t a_lo0 = smem_desc_lo(stage);
          const uint32_t lo_col = tmem + (uint32_t)ls * slot_cols;
#pragma unroll
          for (int j = 0; j < KS; ++j) {
            if (j < nsub) {
              // (one A tile is 16 KB = 1024 descriptor units; a B pair 2 bn x 128 B)
              const uint32_t bd = b_lo0 + (uint32_t)j * (bpair >> 4);
              const uint32_t ad = a_lo0 + (uint32_t)j * (TC_A_BYTES >> 4);
#pragma unroll
              for (int k = 0; k < TC_BK / 8; ++k) {
                const uint32_t acc = (first && j == 0 && k == 0) ? 0u : 1u;
                if (ROLE == 1)
                  mma_tf32_ts(d, lo_col + (uint32_t)(j * TC_LO_COLS + 8 * k), desc_of(bd + 2 * k), idesc,
                              acc);
                else
                  mma_tf32(d, desc_of(ad + 2 * k), desc_of(bd + 2 * k), idesc, acc);
              }
            }
          }
          mma_commit(&B.empty[st]);
          if (ROLE == 1) mma_commit(&B.lo_empty[ls]);
        }
        if (++st == S) {
          st = 0;
          par ^= 1u;
        }
        if (ROLE == 1 && ++ls == LS) {
          ls = 0;
          lpar ^= 1u;
        }
      }
      if (ROLE == 0 && alive) {
        if (elect_one()) mma_commit(&B.hh_full[pc & 1]);  // arrives once the period's MMAs complete
        ++pc;
      }
    }
    if (ROLE == 1 && alive) {
      if (elect_one()) mma_commit(&B.cross_full[xb]);
    }
  }
  if (__any_sync(0xffffffffu, !alive || tc_error_raised())) {
    // Error path: no MMA of this warp may still write TMEM when it is freed.
    if (elect_one()) mma_commit(&B.drain[ROLE]);
    __syncwarp();
    mbar_drain_wait(&B.drain[ROLE], 0u);
  }
}

// Epilogue of one 16-column chunk of an output row: bias (shared memory),
// residual (read-only path, RM 1 = added before the activation, 2 = after),
// activation, store.  Activation and residual mode are template parameters,
// so the 16 element chains carry no branches and interleave.  The fused
// activation is judged with the convolution's tolerance (max |diff| / max
// |ref| <= 1e-4), so the fast exponential and division (a few ulp) are used;
// the standalone activation kernels keep correctly rounded arithmetic.  The
// exponent is clamped so the denominator stays finite (x / (1 + e^88) is 0 to
// fp32).  Measured alternatives, per YOLOv8n bs64 forward: an exponential and
// reciprocal on the FMA pipe (range reduction, polynomial, Newton steps;
// about 25 instructions per element) 8 % slower; packed f32x2 arithmetic for
// pairs of elements 1 % slower; four accumulator buffers per ring instead of
// two, no change.  Without the activation the forward took 5 % less time:
// the epilogue of the 1x1 layers over few channels sets their pace.
template <int ACT>
__device__ __forceinline__ float tc_act_t(float v) {
  if (ACT == MM_ACT_RELU) return (v != v) ? v : (v > 0.f ? v : 0.f);
  if (ACT == MM_ACT_SILU) return __fdividef(v, 1.0f + __expf(fminf(-v, 88.0f)));
  if (ACT == MM_ACT_SIGMOID) return __fdividef(1.0f, 1.0f + __expf(fminf(-v, 88.0f)));
  return v;
}

template <int ACT, int RM, int J>
__device__ __forceinline__ void tc_finish_chunk(const TcArgs& a, float (&tot)[TC_EPI_CHUNKS * 16],
                                                int h, int nchunk, int n0, const float* bias_s,
                                                float* yrow, const float* rrow) {
  const int c = a.epi_groups == 2 ? J : h + 2 * J;
  const int cb0 = n0 + 16 * c;
  if (c >= nchunk || cb0 >= a.kout) return;
  if (cb0 + 16 <= a.kout) {
    float rv[16];
    if (RM != 0) {
      if (a.res_vec) {
#pragma unroll
        for (int v4 = 0; v4 < 4; ++v4) {
          const float4 t = __ldg(reinterpret_cast<const float4*>(rrow + cb0) + v4);
          rv[4 * v4] = t.x; rv[4 * v4 + 1] = t.y; rv[4 * v4 + 2] = t.z; rv[4 * v4 + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) rv[e] = __ldg(rrow + cb0 + e);
      }
    }
#pragma unroll
    for (int v4 = 0; v4 < 4; ++v4) {
      const float4 b = *reinterpret_cast<const float4*>(bias_s + cb0 + 4 * v4);
      const float bb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 4 * v4 + e;
        float val = tot[16 * J + i] + bb[e];
        if (RM == 1) val += rv[i];
        val = tc_act_t<ACT>(val);
        if (RM == 2) val += rv[i];
        tot[16 * J + i] = val;
      }
    }
    if (a.vec_store) {
#pragma unroll
      for (int v4 = 0; v4 < 4; ++v4)
        reinterpret_cast<float4*>(yrow + cb0)[v4] =
            make_float4(tot[16 * J + 4 * v4], tot[16 * J + 4 * v4 + 1], tot[16 * J + 4 * v4 + 2],
                        tot[16 * J + 4 * v4 + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) yrow[cb0 + e] = tot[16 * J + e];
    }
    return;
  }
  // Last, partial chunk of an output width that is not a multiple of 16.
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int cc = cb0 + e;
    if (cc < a.kout) {
      float val = tot[16 * J + e] + bias_s[cc];
      if (RM == 1) val += __ldg(rrow + cc);
      val = tc_act_t<ACT>(val);
      if (RM == 2) val += __ldg(rrow + cc);
      yrow[cc] = val;
    }
  }
}

template <int ACT, int RM>
__device__ __forceinline__ void tc_finish_row(const TcArgs& a, float (&tot)[TC_EPI_CHUNKS * 16],
                                              int h, int nchunk, int n0, const float* bias_s,
                                              float* yrow, const float* rrow) {
  tc_finish_chunk<ACT, RM, 0>(a, tot, h, nchunk, n0, bias_s, yrow, rrow);
  tc_finish_chunk<ACT, RM, 1>(a, tot, h, nchunk, n0, bias_s, yrow, rrow);
  tc_finish_chunk<ACT, RM, 2>(a, tot, h, nchunk, n0, bias_s, yrow, rrow);
}

// The same epilogue arithmetic into this warp's staging box J (row r of 32)
// instead of global memory.  Channels past kout get no bias or residual; the
// TMA store clips them.  `rrow` is null for rows outside the output (the
// store clips those rows too).
template <int ACT, int RM, int J>
__device__ __forceinline__ void tc_stage_chunk(const TcArgs& a, float (&tot)[TC_EPI_CHUNKS * 16],
                                               int h, int nchunk, int n0, const float* bias_s,
                                               const float* rrow, uint8_t* stg, int r) {
  const int c = a.epi_groups == 2 ? J : h + 2 * J;
  const int cb0 = n0 + 16 * c;
  if (c >= nchunk || cb0 >= a.kout) return;
  const bool full = cb0 + 16 <= a.kout;
  float rv[16];
  if (RM != 0) {
    if (rrow != nullptr && full && a.res_vec) {
#pragma unroll
      for (int v4 = 0; v4 < 4; ++v4) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(rrow + cb0) + v4);
        rv[4 * v4] = t.x; rv[4 * v4 + 1] = t.y; rv[4 * v4 + 2] = t.z; rv[4 * v4 + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) rv[e] = (rrow != nullptr && cb0 + e < a.kout) ? __ldg(rrow + cb0 + e) : 0.f;
    }
  }
  uint8_t* row = stg + J * TC_STG_BOX + r * 64;
#pragma unroll
  for (int v4 = 0; v4 < 4; ++v4) {
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = 4 * v4 + e;
      float val = tot[16 * J + i] + (full || cb0 + i < a.kout ? bias_s[cb0 + i] : 0.f);
      if (RM == 1) val += rv[i];
      val = tc_act_t<ACT>(val);
      if (RM == 2) val += rv[i];
      o[e] = val;
    }
    *reinterpret_cast<float4*>(row + ((v4 ^ ((r >> 1) & 3)) << 4)) = make_float4(o[0], o[1], o[2], o[3]);
  }
}

template <int ACT, int RM>
__device__ __forceinline__ void tc_stage_row(const TcArgs& a, float (&tot)[TC_EPI_CHUNKS * 16],
                                             int h, int nchunk, int n0, const float* bias_s,
                                             const float* rrow, uint8_t* stg, int r) {
  tc_stage_chunk<ACT, RM, 0>(a, tot, h, nchunk, n0, bias_s, rrow, stg, r);
  tc_stage_chunk<ACT, RM, 1>(a, tot, h, nchunk, n0, bias_s, rrow, stg, r);
  tc_stage_chunk<ACT, RM, 2>(a, tot, h, nchunk, n0, bias_s, rrow, stg, r);
}

// One instantiation per activation and residual mode (RM 0 none, 1 added
// before the activation, 2 after): each carries a single epilogue, which keeps
// the code that the producer, TMA and MMA warps run beside it small.
template <int ACT, int RM, int KS>
__global__ void __launch_bounds__(TC_THREADS, 1)
    conv_tc_kernel(const __grid_constant__ CUtensorMap wmap_hi,
                   const __grid_constant__ CUtensorMap wmap_lo,
                   const __grid_constant__ CUtensorMap amap,
                   const __grid_constant__ CUtensorMap ymap, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int S = a.stages;
  const TcSmem L = TcSmem::make(a.bn, KS, S, a.kout, a.stg_chunks);
  float* bias_s = (float*)(smem + L.bias);
  const uint32_t b_bytes = (uint32_t)a.bn * 128;
  uint64_t* bars = (uint64_t*)(smem + L.bars);
  TcBars B;
  B.full_x = bars;                 // S: A tile (and, in the TMA modes, the B tiles)
  B.full_b = bars + S;             // S: B tiles in the gather mode (TMA transaction bytes)
  B.fenced = bars + 2 * S;         // S: gather mode, the A tile visible to the tensor core
                                   //    (one arrival per producer thread, after a proxy fence)
  B.empty = bars + 3 * S;          // S: one commit per issuer frees the stage
  uint64_t* rest = bars + 4 * S;
  B.lo_full = rest;                // LO: lo slot written (one arrival per producer thread)
  B.lo_empty = rest + TC_MAX_LO;   // LO: the lo issuer's commit frees the slot
  rest += 2 * TC_MAX_LO;
  B.hh_full = rest;                // 2: [hi*hi | hi*lo] period complete in TMEM
  B.hh_free = rest + 2;            // 2: one arrival per promotion thread
  B.cross_full = rest + 4;         // 2: lo*hi tile sum complete
  B.cross_free = rest + 6;         // 2: one arrival per epilogue thread
  B.drain = rest + 8;              // 3: issuer error paths wait for their MMAs
  uint64_t* full_x = B.full_x;
  uint64_t* full_b = B.full_b;
  uint64_t* empty = B.empty;
  uint64_t* hh_full = B.hh_full;
  uint64_t* hh_free = B.hh_free;
  uint64_t* cross_full = B.cross_full;
  uint64_t* cross_free = B.cross_free;
  uint32_t* tmem_slot = (uint32_t*)(bars + L.n_bars());
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  __shared__ int s_skip;
  if (threadIdx.x == 0) s_skip = tc_error_raised() ? 1 : 0;
  __syncthreads();
  if (s_skip) return;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      // Gather mode: every producer thread's cp.async completion arrives
      // (.noinc); TMA modes: the TMA thread's arrive + transaction bytes.
      mbar_init(&full_x[i], a.amode == TC_A_GATHER ? TC_A_WARPS * 32 : 1);
      mbar_init(&full_b[i], 1);
      mbar_init(&B.fenced[i], TC_A_WARPS * 32);
      mbar_init(&empty[i], 2);
    }
    for (int i = 0; i < TC_MAX_LO; ++i) {
      mbar_init(&B.lo_full[i], TC_A_WARPS * 32);
      mbar_init(&B.lo_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&hh_full[i], 1);
      mbar_init(&hh_free[i], 32 * (a.epi_groups == 2 ? TC_EPI_WARPS / 2 : TC_EPI_WARPS));
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&cross_full[i], 1);
      mbar_init(&cross_free[i], 32 * (a.epi_groups == 2 ? TC_EPI_WARPS / 2 : TC_EPI_WARPS));
    }
    for (int i = 0; i < 3; ++i) mbar_init(&B.drain[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == TC_WARP_HI) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(TC_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent launch: the set-up above (barriers, TMEM, both
  // independent of earlier kernels' results) overlaps the previous kernel's
  // tail; the next convolution may be scheduled from here on (its CTAs take an
  // SM only as one of ours leaves, one CTA per SM), and nothing below reads an
  // input or writes the output before every earlier kernel has completed.
  // Both instructions do nothing in a launch without the attribute.
  if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // TMEM columns: lo slots at [32 l, 32 l + 32); from acc0 = 32 LO two period
  // buffers of 2 bn columns ([hi*hi | hi*lo], [acc0, acc0 + 4 bn)), then xbuf
  // lo*hi tile sums of bn columns.
  const int LS = a.lo_slots;
  const uint32_t slot_cols = (uint32_t)(TC_LO_COLS * KS);
  const uint32_t acc0 = slot_cols * (uint32_t)LS;
  const int KB = a.kb_total;
  const int NP = (KB + a.period - 1) / a.period;
  const int64_t my_tiles = a.tiles > blockIdx.x ? (a.tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t total = my_tiles * KB;

  if (warp < TC_A_WARPS) {
    // ---------------- A producers ----------------
    // Warp w owns TMEM lane quarter q = w % 4 (tile rows 32 q .. 32 q + 31) and
    // TC_A_HALVES 16-channel halves, from half0, of every 32-channel sub-block.
    const int q = warp & 3;
    const int half0 = (warp >> 2) * TC_A_HALVES;
    const uint32_t tm_rows = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t stage0 = smem_addr(smem);
    int st = 0;
    uint32_t par = 0;
    int lo_slot = 0;     // lo slot of the k-block being split
    uint32_t lo_par = 0;  // its fill phase parity
    int kbt = 0;        // the k-block's index within its tile
    // Remainder of this warp's 32 rows x 16 channels of each of the `nsub`
    // sub-blocks of stage `st` into lo slot `lo_slot` once the lo issuer has
    // freed it; false on a timeout.
    auto split_into_slot = [&](int nsub) -> bool {
      if (!mbar_wait(&B.lo_empty[lo_slot], lo_par ^ 1u, TC_ERR_WAIT_EMPTY)) return false;
      tc_fence_after();
      const uint32_t tile_s = stage0 + (uint32_t)st * L.stage_bytes;
#pragma unroll
      for (int j = 0; j < KS; ++j) {
        if (j >= nsub) break;
#pragma unroll
        for (int hh = 0; hh < TC_A_HALVES; ++hh) {
          const int half = half0 + hh;
          float lo[16];
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            float4 v;
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                         : "r"(tile_s + (uint32_t)j * TC_A_BYTES + sw128_off(q * 32 + lane, half * 4 + c4)));
            lo[4 * c4 + 0] = v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
            lo[4 * c4 + 1] = v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
            lo[4 * c4 + 2] = v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
            lo[4 * c4 + 3] = v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
          }
          tmem_st16(tm_rows + (uint32_t)lo_slot * slot_cols + (uint32_t)(j * TC_LO_COLS + half * 16), lo);
        }
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&B.lo_full[lo_slot]);
      if (++lo_slot == LS) {
        lo_slot = 0;
        lo_par ^= 1u;
      }
      return true;
    };
    if (a.amode == TC_A_GATHER) {
      // Gather: 16-byte cp.async of this warp's 32 rows x 64 B per half into the
      // swizzled A tile, zero-filled for padding taps, rows outside the output
      // and padded channels, run `ahead` k-blocks in front of the split.
      const int lrow = lane >> 2;
      const int lchunk = lane & 3;
      const int ahead = S - 1;  // k-blocks loaded beyond the one being split
      int64_t ltile = blockIdx.x;
      int lkb = 0;                    // the load cursor's k-block within its tile
      int lkr = 0, lks = 0, lcb = 0;  // and its next sub-block (tap row, tap column, channel block)
      int lst = 0;
      uint32_t lpar = 0;
      int roff[4];  // element offsets (the input spans < 2^31 elements; checked on the host)
      int ih0[4], iw0[4];
      auto setup_rows = [&]() {
        const TcTile t = tc_tile(a, (int)(ltile / a.n_tiles));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          int n_ = 0, oh_ = 0, ow_ = 0;
          const bool ok = tc_row(a, t, q * 32 + lrow + 8 * i, n_, oh_, ow_);
          // Rows outside the output get a coordinate that fails the bounds test.
          ih0[i] = ok ? oh_ * a.sh - a.ph : -0x40000000;
          iw0[i] = ow_ * a.sw - a.pw;
          roff[i] = ok ? n_ * (int)a.xs0 + ih0[i] * (int)a.xs2 + iw0[i] * (int)a.xs3 : 0;
        }
      };
      bool alive = true;
      // Issue the copies of the load cursor's k-block and advance the cursor.
      auto load_next = [&]() -> bool {
        if (!mbar_wait(&empty[lst], lpar ^ 1u, TC_ERR_WAIT_EMPTY)) return false;
        const int nsub = min(KS, a.sb_total - lkb * KS);
        const uint32_t tile_s = stage0 + (uint32_t)lst * L.stage_bytes;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
          if (j >= nsub) break;
          const int dy = lkr * a.dh, dx = lks * a.dw;
          const int cbase = lcb * TC_BK;
#pragma unroll
          for (int hh = 0; hh < TC_A_HALVES; ++hh) {
            const int half = half0 + hh;
            const int lane_c = half * 16 + lchunk * 4;
            const bool cok = cbase + lane_c < a.c;
            const int koff = dy * (int)a.xs2 + dx * (int)a.xs3 + cbase + lane_c;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int row = q * 32 + lrow + 8 * i;
              const bool ok = cok && (unsigned)(ih0[i] + dy) < (unsigned)a.h &&
                              (unsigned)(iw0[i] + dx) < (unsigned)a.w;
              const float* src = a.x + (ok ? roff[i] + koff : 0);
              asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;" ::"r"(
                               tile_s + (uint32_t)j * TC_A_BYTES + sw128_off(row, half * 4 + lchunk)),
                           "l"(src), "r"(ok ? 16 : 0)
                           : "memory");
            }
          }
          if (++lcb == a.cb) {
            lcb = 0;
            if (++lks == a.s) {
              lks = 0;
              ++lkr;
            }
          }
        }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(
                         smem_addr(&full_x[lst]))
                     : "memory");
        if (++lst == S) {
          lst = 0;
          lpar ^= 1u;
        }
        if (++lkb == KB) {
          lkb = 0;
          lkr = lks = lcb = 0;
          ltile += gridDim.x;
          if (ltile < a.tiles) setup_rows();
        }
        return true;
      };
      if (total > 0) setup_rows();
      int64_t issued = 0;
      for (int64_t g = 0; g < total && alive; ++g) {
        // k-block g must be in flight; later k-blocks are issued while their
        // stage is already free (lane 0 tests, the warp follows; every lane
        // then takes the barrier itself, which succeeds at once).
        while (alive && issued <= g) {
          alive = load_next();
          ++issued;
        }
        while (alive && issued < total && issued < g + ahead &&
               __shfl_sync(0xffffffffu, mbar_test(&empty[lst], lpar ^ 1u) ? 1 : 0, 0)) {
          alive = load_next();
          ++issued;
        }
        if (!alive) break;
        if (!mbar_wait(&full_x[st], par, TC_ERR_WAIT_A)) break;
        // The gathered tile was written through the generic proxy: fence, then
        // let the hi issuer read it.
        fence_proxy_async_smem();
        mbar_arrive(&B.fenced[st]);
        if (!split_into_slot(min(KS, a.sb_total - kbt * KS))) break;
        if (++st == S) {
          st = 0;
          par ^= 1u;
        }
        if (++kbt == KB) kbt = 0;
      }
      // No copy may land in shared memory after the CTA has exited.
      asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
      // TMA modes: the A tile arrives by TMA; only the remainder is computed.
      for (int64_t g = 0; g < total; ++g) {
        if (!mbar_wait(&full_x[st], par, TC_ERR_WAIT_A)) break;
        if (!split_into_slot(min(KS, a.sb_total - kbt * KS))) break;
        if (++st == S) {
          st = 0;
          par ^= 1u;
        }
        if (++kbt == KB) kbt = 0;
      }
    }
  } else if (warp == TC_WARP_TMA) {
    // ---------------- TMA: weights, and the A tile in the TMA modes ----------------
    // The whole warp runs the loop and the waits; one elected lane issues.
    {
      int64_t g = 0;
      int st = 0;
      uint32_t par = 0;
      bool alive = true;
      // Test hook (mm_debug_tc_fault): CTA 0 issues nothing for its first
      // k-block, so the waits for that stage run out.
      const bool dropped = blockIdx.x == 0 && *reinterpret_cast<volatile int*>(&g_tc_drop_first_load) != 0;
      for (int64_t tile = blockIdx.x; tile < a.tiles && alive; tile += gridDim.x) {
        const TcTile t = tc_tile(a, (int)(tile / a.n_tiles));
        const int n0 = (int)(tile % a.n_tiles) * a.bn;
        int kr = 0, ks = 0, cbk = 0;
        for (int kb = 0; kb < KB; ++kb, ++g) {
          if (!warp_wait(&empty[st], par ^ 1u, TC_ERR_WAIT_EMPTY)) {
            alive = false;
            break;
          }
          const int nsub = min(KS, a.sb_total - kb * KS);
          if (!(dropped && g == 0) && elect_one()) {
            uint8_t* stage = smem + (size_t)st * L.stage_bytes;
            // TMA modes: A and both weight tiles complete on full_x; gather
            // mode: the weights on full_b (A arrives by the producers' cp.async).
            const bool gmode = a.amode == TC_A_GATHER;
            uint64_t* bbar = gmode ? &full_b[st] : &full_x[st];
            mbar_arrive_expect_tx(bbar, (uint32_t)nsub * ((gmode ? 0u : TC_A_BYTES) + 2u * b_bytes));
            int r_ = kr, s_ = ks, c_ = cbk;
#pragma unroll
            for (int j = 0; j < KS; ++j) {
              if (j >= nsub) break;
              uint8_t* at = stage + (size_t)j * TC_A_BYTES;
              uint8_t* bt = stage + L.a_bytes + (size_t)j * 2 * b_bytes;
              if (a.amode == TC_A_FLAT) {
                tma_load_2d(at, &amap, &full_x[st], c_ * TC_BK, t.m0);
              } else if (a.amode == TC_A_RECT) {
                // Taps outside the image read as zero (TMA out-of-bounds fill).
                tma_load_4d(at, &amap, &full_x[st], c_ * TC_BK, t.ow0 * a.sw - a.pw + s_ * a.dw,
                            t.oh0 * a.sh - a.ph + r_ * a.dh, t.n);
              }
              const int sb = kb * KS + j;
              tma_load_2d(bt, &wmap_hi, bbar, sb * TC_BK, n0);
              tma_load_2d(bt + b_bytes, &wmap_lo, bbar, sb * TC_BK, n0);
              if (++c_ == a.cb) {
                c_ = 0;
                if (++s_ == a.s) {
                  s_ = 0;
                  ++r_;
                }
              }
            }
          }
          __syncwarp();
          if (++st == S) {
            st = 0;
            par ^= 1u;
          }
#pragma unroll
          for (int j = 0; j < KS; ++j) {
            if (j >= nsub) break;
            if (++cbk == a.cb) {
              cbk = 0;
              if (++ks == a.s) {
                ks = 0;
                ++kr;
              }
            }
          }
        }
      }
      // Bulk copies must not outlive the CTA's shared memory.
      for (int64_t k = (g > S ? g - S : 0); k < g; ++k) {
        if (k == 0 && dropped) continue;  // (nothing was issued for it)
        const uint32_t kp = (uint32_t)((k / S) & 1);
        if (a.amode == TC_A_GATHER)
          mbar_drain_wait(&full_b[k % S], kp);
        else
          mbar_drain_wait(&full_x[k % S], kp);
      }
    }
  } else if (warp == TC_WARP_HI) {
    tc_issue<0, KS>(a, smem, L, tmem, B);
  } else if (warp == TC_WARP_LO) {
    tc_issue<1, KS>(a, smem, L, tmem, B);
  } else if (warp >= TC_WARP_EPI) {
    // ---------------- promotion (fp32 RN adds) + epilogue ----------------
    // Two warps per TMEM lane quarter; warp half h owns the 16-column chunks
    // h, h + 2, h + 4 of the tile.  The fp32 total of a tile lives in
    // registers (one output row per thread), indexed with compile-time
    // offsets only.
    // Split mode: warp half h owns chunks h, h + 2, h + 4 of every tile.
    // Group mode: group g (warps g*4 .. g*4+3) owns all chunks of every other
    // tile, so two tiles' epilogues overlap.
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const bool grp = a.epi_groups == 2;
    const int eg = (warp - TC_WARP_EPI) >> 2;
    const int h = grp ? 0 : eg;
    const int cstep = grp ? 1 : 2;
    const int tstep = grp ? 2 : 1;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const int nchunk = a.bn >> 4;
    uint8_t* stg = smem + L.stg + (size_t)(warp - TC_WARP_EPI) * a.stg_chunks * TC_STG_BOX;
    // The bias may be the output of an earlier kernel in the stream, so it is
    // staged only after griddepcontrol.wait, by the epilogue warps that read
    // it (named barrier 1 over their 256 threads).
    for (int i = threadIdx.x - TC_WARP_EPI * 32; i < a.kout; i += TC_EPI_WARPS * 32)
      bias_s[i] = a.bias ? a.bias[i] : 0.f;
    asm volatile("bar.sync 1, %0;" ::"n"(TC_EPI_WARPS * 32) : "memory");
    int64_t tc = grp ? eg : 0;
    bool alive = true;
    for (int64_t tile = blockIdx.x + tc * gridDim.x; tile < a.tiles && alive;
         tile += tstep * (int64_t)gridDim.x, tc += tstep) {
      float tot[TC_EPI_CHUNKS * 16];
      int64_t pc = tc * NP;  // this tile's first period
      const int xb = a.xbuf == 2 ? (int)(tc & 1) : 0;
      const uint32_t xpar = (uint32_t)((a.xbuf == 2 ? tc >> 1 : tc) & 1);
      const uint32_t cross = lane_base + acc0 + (uint32_t)((4 + xb) * a.bn);
      for (int p = 0; p < NP; ++p, ++pc) {
        const int b = (int)(pc & 1);  // (in group mode NP == 1: buffer = tile parity = group)
        if (!mbar_wait(&hh_full[b], (uint32_t)((pc >> 1) & 1), TC_ERR_WAIT_ACC)) {
          alive = false;
          break;
        }
        tc_fence_after();
        const uint32_t buf = lane_base + acc0 + (uint32_t)(b * 2 * a.bn);
#pragma unroll
        for (int j = 0; j < TC_EPI_CHUNKS; ++j) {
          const int c = h + cstep * j;
          if (c < nchunk) {
            uint32_t u[16], w[16];  // hi*hi, hi*lo
            tmem_ld16_nowait(buf + (uint32_t)(16 * c), u);
            tmem_ld16_nowait(buf + (uint32_t)(a.bn + 16 * c), w);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float v = __fadd_rn(__uint_as_float(u[e]), __uint_as_float(w[e]));
              tot[16 * j + e] = p == 0 ? v : __fadd_rn(tot[16 * j + e], v);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&hh_free[b]);
      }
      if (!alive) break;
      if (!mbar_wait(&cross_full[xb], xpar, TC_ERR_WAIT_ACC)) {
        alive = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < TC_EPI_CHUNKS; ++j) {
        const int c = h + cstep * j;
        if (c < nchunk) {
          uint32_t u[16];  // lo*hi
          tmem_ld16_nowait(cross + (uint32_t)(16 * c), u);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) tot[16 * j + e] = __fadd_rn(tot[16 * j + e], __uint_as_float(u[e]));
        }
      }
      tc_fence_before();
      mbar_arrive(&cross_free[xb]);

      const TcTile t = tc_tile(a, (int)(tile / a.n_tiles));
      const int n0 = (int)(tile % a.n_tiles) * a.bn;
      int n_ = 0, oh_ = 0, ow_ = 0;
      const bool valid = tc_row(a, t, q * 32 + lane, n_, oh_, ow_);
      if (a.stg_chunks > 0) {
        // Staged: the warp writes its 32 rows into its boxes, then lane 0
        // stores each box with TMA (rows and channels outside the output are
        // clipped by the tensor map).  Before the boxes are rewritten, the
        // warp's previous stores must have read them.
        if (lane == 0) bulk_wait_read();
        __syncwarp();
        const float* rrow =
            RM != 0 && valid ? a.res + ((int64_t)n_ * a.rs0 + (int64_t)oh_ * a.rs2 + (int64_t)ow_ * a.rs3)
                             : nullptr;
        tc_stage_row<ACT, RM>(a, tot, h, nchunk, n0, bias_s, rrow, stg, lane);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          int sx = 0, sy = 0;  // first pixel of the warp's 32 rows
          bool inside;
          if (a.amode == TC_A_RECT) {
            const int r0 = q * 32;
            sy = t.oh0 + r0 / a.tw;
            sx = t.ow0 + (a.tw >= 32 ? r0 % a.tw : 0);
            inside = sx < a.ow && sy < a.oh;
          } else {
            sy = t.m0 + q * 32;
            inside = sy < a.m_total;
          }
          if (inside) {
#pragma unroll
            for (int j = 0; j < TC_EPI_CHUNKS; ++j) {
              const int c = grp ? j : h + 2 * j;
              if (c < nchunk && n0 + 16 * c < a.kout) {
                if (a.amode == TC_A_RECT)
                  tma_store_4d(&ymap, stg + j * TC_STG_BOX, n0 + 16 * c, sx, sy, t.n);
                else
                  tma_store_2d(&ymap, stg + j * TC_STG_BOX, n0 + 16 * c, sy);
              }
            }
          }
          bulk_commit();
        }
        continue;
      }
      if (!valid) continue;
      float* yrow = a.y + ((int64_t)n_ * a.ys0 + (int64_t)oh_ * a.ys2 + (int64_t)ow_ * a.ys3);
      const float* rrow =
          RM != 0 ? a.res + ((int64_t)n_ * a.rs0 + (int64_t)oh_ * a.rs2 + (int64_t)ow_ * a.rs3)
                  : nullptr;
      tc_finish_row<ACT, RM>(a, tot, h, nchunk, n0, bias_s, yrow, rrow);
    }
    // No store may still read the staging boxes when the CTA exits.
    if (a.stg_chunks > 0 && lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == TC_WARP_HI) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TC_TMEM_COLS)
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

// cuTensorMapEncodeTiled, resolved through the runtime so the library does
// not link libcuda (it must load on hosts without a driver).
// `estr` (traversal strides, default 1): a box dimension of b elements with
// traversal stride t brings ceil(b / t) elements, stored densely.
int encode_tiled(const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                 const cuuint32_t* box, CUtensorMap* out, const cuuint32_t* estr = nullptr,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
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
  const cuuint32_t ones[5] = {1, 1, 1, 1, 1};
  CUresult r = encode(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, (void*)base, dims,
                      strides, box, estr ? estr : ones, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MM_ERR_CUDA, "mm_conv2d_tc: cuTensorMapEncodeTiled failed (CUresult " +
                                 std::to_string((int)r) + ")");
  return MM_OK;
}

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
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)ktot, (cuuint64_t)kpad};
  const cuuint64_t strides[1] = {(cuuint64_t)ktot * 4};
  const cuuint32_t box[2] = {32, (cuuint32_t)bn};
  int rc = encode_tiled(w, 2, dims, strides, box, &map);
  if (rc != MM_OK) return rc;
  std::lock_guard<std::mutex> g(g_map_mu);
  g_maps[key] = map;
  *out = map;
  return MM_OK;
}

bool aligned16(const void* p) { return (((uintptr_t)p) & 15) == 0; }

// Dynamic shared memory one CTA may request on the current device: the
// opt-in maximum minus the kernel's static shared memory.
using TcKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                          const TcArgs);
constexpr int TC_VARIANTS = 24;  // 4 activations x 3 residual modes x 2 k-block widths

template <int ACT, int KS>
TcKernel tc_kernel_rm(int rm) {
  return rm == 1 ? conv_tc_kernel<ACT, 1, KS> : rm == 2 ? conv_tc_kernel<ACT, 2, KS> : conv_tc_kernel<ACT, 0, KS>;
}

template <int KS>
TcKernel tc_kernel_ks(int act, int rm) {
  switch (act) {
    case MM_ACT_RELU: return tc_kernel_rm<MM_ACT_RELU, KS>(rm);
    case MM_ACT_SILU: return tc_kernel_rm<MM_ACT_SILU, KS>(rm);
    case MM_ACT_SIGMOID: return tc_kernel_rm<MM_ACT_SIGMOID, KS>(rm);
    default: return tc_kernel_rm<MM_ACT_NONE, KS>(rm);
  }
}

// Variant v = 2 * (3 * act + rm) + (ksub == 2); activation codes other than
// the four named ones apply no activation.
TcKernel tc_kernel(int v) {
  const int ks2 = v & 1, act = (v >> 1) / 3, rm = (v >> 1) % 3;
  return ks2 ? tc_kernel_ks<2>(act, rm) : tc_kernel_ks<1>(act, rm);
}

int tc_smem_limit(int dev, size_t* out) {
  static size_t cached[256] = {};
  if (dev < 0 || dev >= 256) return fail(MM_ERR_INVALID, "mm_conv2d_tc: device index");
  if (cached[dev] == 0) {
    int optin = 0;
    MM_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev),
            "mm_conv2d_tc: shared memory limit");
    size_t static_smem = 0;
    for (int v = 0; v < TC_VARIANTS; ++v) {
      cudaFuncAttributes fa;
      MM_CUDA(cudaFuncGetAttributes(&fa, tc_kernel(v)), "mm_conv2d_tc: kernel attributes");
      if (fa.sharedSizeBytes > static_smem) static_smem = fa.sharedSizeBytes;
    }
    if ((size_t)optin <= static_smem) return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: shared memory");
    cached[dev] = (size_t)optin - static_smem;
  }
  *out = cached[dev];
  return MM_OK;
}

bool nhwc_ok(const mm_tensor_t* t) {
  return t->ndim == 4 && t->stride[1] == 1 && t->stride[0] % 4 == 0 && t->stride[2] % 4 == 0 &&
         t->stride[3] % 4 == 0 && aligned16(t->data);
}

// The convolution's output pixels [row0, row0 + H) x [col0, col0 + W) of
// y's H x W (region == true), or its whole output (region == false, y must be
// the full output).  A region is the same convolution with effective padding
// pad - row0 * stride (negative inside the image): every A mode computes its
// input coordinates as o * stride - pad + tap and reads taps outside the
// image as zero, so a region reads exactly the rows and columns the full
// convolution would, and each output pixel is accumulated in the same order.
int conv2d_tc_impl(const mm_tensor_t* x, const float* w_hi, const float* w_lo, int k_out, int c_in, int r,
                   int s, int c_pad, int k_pad, const float* bias, const mm_tensor_t* residual,
                   const mm_conv_params_t* p, bool region, int64_t row0, int64_t col0, const mm_tensor_t* y,
                   void* stream) {
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
  const int64_t oh_full = (h + 2 * p->pad_h - (int64_t)p->dil_h * (r - 1) - 1) / p->stride_h + 1;
  const int64_t ow_full = (w + 2 * p->pad_w - (int64_t)p->dil_w * (s - 1) - 1) / p->stride_w + 1;
  if (oh_full <= 0 || ow_full <= 0) return fail(MM_ERR_INVALID, "mm_conv2d_tc: empty output");
  if (y->size[0] != n || y->size[1] != k_out)
    return fail(MM_ERR_INVALID, "mm_conv2d_tc: output shape mismatch");
  if (!region && (y->size[2] != oh_full || y->size[3] != ow_full))
    return fail(MM_ERR_INVALID, "mm_conv2d_tc: output shape mismatch");
  if (region && (row0 < 0 || col0 < 0 || y->size[2] <= 0 || y->size[3] <= 0 ||
                 row0 + y->size[2] > oh_full || col0 + y->size[3] > ow_full))
    return fail(MM_ERR_INVALID, "mm_conv2d_tc_region: region outside the convolution's output");
  const int64_t oh = y->size[2], ow = y->size[3];
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
  a.r = r; a.s = s; a.sh = p->stride_h; a.sw = p->stride_w;
  a.ph = (int)(p->pad_h - row0 * p->stride_h);  // effective padding of the region (< 0 inside)
  a.pw = (int)(p->pad_w - col0 * p->stride_w);
  a.dh = p->dil_h; a.dw = p->dil_w;
  if (m_total > 0x7fffffffLL - TC_BM) return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: too many output pixels");
  {
    // The A producers address the input with 32-bit element offsets: the
    // furthest element any view coordinate (including padding taps, which are
    // never read) can name must stay below 2^31.
    const int64_t span = (n - 1) * x->stride[0] + (h + 2 * (int64_t)p->pad_h + (int64_t)p->dil_h * r) * x->stride[2] +
                         (w + 2 * (int64_t)p->pad_w + (int64_t)p->dil_w * s) * x->stride[3] + c_pad;
    if (span > 0x7fffffffLL || x->stride[2] > 0x7fffffffLL || x->stride[3] > 0x7fffffffLL)
      return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: input too large for 32-bit offsets");
  }
  if (k_out > TC_MAX_BIAS) return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: too many output channels");
  a.m_total = (int)m_total;
  a.cb = c_pad / TC_BK;
  a.sb_total = r * s * a.cb;
  // N tiles of at most TC_MAX_BN channels, balanced (128 -> 2 x 64, 144 -> 2 x 80).
  {
    const int ntiles = (k_out + TC_MAX_BN - 1) / TC_MAX_BN;
    const int per = (k_out + ntiles - 1) / ntiles;
    a.bn = ((per + 15) / 16) * 16;
  }
  a.n_tiles = (k_out + a.bn - 1) / a.bn;
  // Sub-blocks per k-block: every k-block costs each warp role a fixed chain
  // of barrier waits, copies and MMA issues, so reductions of at least four
  // 32-channel sub-blocks run two per k-block (measured 4-11 % faster on the
  // 3x3 layers of YOLOv8n at batch 64; one per k-block stays faster for
  // reductions of one or two sub-blocks, where a tile then has two k-blocks
  // to overlap instead of one).
  a.ksub = a.sb_total >= 4 ? 2 : 1;
  if (const char* env = std::getenv("MATRIXMAN_TC_KSUB")) {
    const int v = std::atoi(env);
    if (v == 1 || v == 2) a.ksub = v;
  }
  while (a.ksub > 1 && a.ksub / 2 >= a.sb_total) a.ksub /= 2;  // no k-block of padding only
  a.kb_total = (a.sb_total + a.ksub - 1) / a.ksub;
  // Promotion period: at most 12 sub-blocks (48 MMAs per accumulator),
  // balanced over the tile (18 -> 2 x 9, 36 -> 3 x 12).  The tensor core's
  // truncating accumulation biases one period's sum by up to ~2.5e-6 relative
  // (all-positive data); promotion into the fp32 total keeps that bias from
  // growing with the reduction length.
  {
    const int pmax = 12 / a.ksub;
    const int np = (a.kb_total + pmax - 1) / pmax;
    a.period = (a.kb_total + np - 1) / np;
  }
  a.act = p->act;
  a.res_before_act = p->residual_before_act;
  a.vec_store = nhwc_ok(y) ? 1 : 0;
  a.res_vec = residual && nhwc_ok(residual) ? 1 : 0;
  // How A tiles arrive (see TC_A_*).  Rectangles are chosen when they cover
  // at least 60 % of their area with output pixels: TMA loads beat the gather
  // mode by enough that a 20-pixel-wide output (best cover 62.5 %) runs about
  // 30 % faster as rectangles despite the idle rows.
  a.amode = TC_A_GATHER;
  a.tw = a.th = a.ntw = a.nth = 1;
  {
    const bool stride1 = p->stride_h == 1 && p->stride_w == 1;
    // TMA traversal strides go up to 8; the box spans tw * stride input columns.
    const bool strided_ok = p->stride_h <= 8 && p->stride_w <= 8;
    const bool uniform = x->stride[2] == w * x->stride[3] && x->stride[0] == h * x->stride[2];
    if (!region && stride1 && r == 1 && s == 1 && p->pad_h == 0 && p->pad_w == 0 && uniform &&
        n * h * w <= 0x7fffffffLL) {
      a.amode = TC_A_FLAT;
    } else if (strided_ok) {
      double best = 0.0;
      for (int tw = 128; tw >= 4; tw /= 2) {
        const int th = TC_BM / tw;
        if (tw * p->stride_w > 256 || th * p->stride_h > 256) continue;
        const int64_t ntw = (ow + tw - 1) / tw, nth = (oh + th - 1) / th;
        const double eff = (double)(oh * ow) / (double)(ntw * tw * nth * th);
        if (eff > best + 1e-9) {
          best = eff;
          a.tw = tw;
          a.th = th;
          a.ntw = (int)ntw;
          a.nth = (int)nth;
        }
      }
      if (best >= 0.6 && (int64_t)n * a.ntw * a.nth <= 0x7fffffffLL) a.amode = TC_A_RECT;
    }
  }
  // A tensor map for the TMA modes (a map the driver rejects falls back to
  // the gather mode).
  CUtensorMap amap;
  memset(&amap, 0, sizeof(amap));
  if (a.amode == TC_A_FLAT) {
    // [pixels][C] rows; channels past C and pixels past the end read as zero.
    const cuuint64_t dims[2] = {(cuuint64_t)c_in, (cuuint64_t)(n * h * w)};
    const cuuint64_t strides[1] = {(cuuint64_t)x->stride[3] * 4};
    const cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)TC_BM};
    if (encode_tiled(x->data, 2, dims, strides, box, &amap) != MM_OK) a.amode = TC_A_GATHER;
  } else if (a.amode == TC_A_RECT) {
    // {C, W, H, N}; coordinates outside the image (padding taps) read as zero.
    const cuuint64_t dims[4] = {(cuuint64_t)c_in, (cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)n};
    const cuuint64_t strides[3] = {(cuuint64_t)x->stride[3] * 4, (cuuint64_t)x->stride[2] * 4,
                                   (cuuint64_t)x->stride[0] * 4};
    const cuuint32_t box[4] = {(cuuint32_t)TC_BK, (cuuint32_t)(a.tw * p->stride_w),
                               (cuuint32_t)(a.th * p->stride_h), 1};
    const cuuint32_t estr[4] = {1, (cuuint32_t)p->stride_w, (cuuint32_t)p->stride_h, 1};
    if (encode_tiled(x->data, 4, dims, strides, box, &amap, estr) != MM_OK) a.amode = TC_A_GATHER;
  }

  a.div_ow = make_fastdiv((uint32_t)a.ow);
  a.div_oh = make_fastdiv((uint32_t)a.oh);
  a.div_img = make_fastdiv((uint32_t)(a.ntw * a.nth));
  a.div_ntw = make_fastdiv((uint32_t)a.ntw);
  a.mtiles = a.amode == TC_A_RECT ? n * (int64_t)a.ntw * a.nth : (m_total + TC_BM - 1) / TC_BM;
  a.tiles = a.mtiles * a.n_tiles;
  // Stages: TMEM holds S lo stages of 32 columns, two [hi*hi | hi*lo] period
  // buffers of 2 bn columns and xbuf lo*hi tile sums of bn columns; shared
  // memory holds S (A + B hi + B lo) stages, the bias and the barriers.
  int dev = 0;
  MM_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  size_t smem_limit = 0;
  if ((rc = tc_smem_limit(dev, &smem_limit)) != MM_OK) return rc;
  // Output tensor map for the staged TMA-store epilogue: a 4-D {K, W, H, N}
  // map (box: 16 channels x one warp's 32 pixels of a rectangle) for
  // rectangle tiles, a 2-D {K, pixels} map (box 16 x 32) for flat tiles when
  // the output pixels are uniformly strided.  Otherwise rows are stored
  // directly.
  const int nchunk = a.bn / 16;
  CUtensorMap ymap;
  memset(&ymap, 0, sizeof(ymap));
  bool staged = false;
  // (A 16-channel tile gains nothing from staging: one box per warp.)
  if (nhwc_ok(y) && a.bn >= 32) {
    if (a.amode == TC_A_RECT) {
      const cuuint64_t dims[4] = {(cuuint64_t)k_out, (cuuint64_t)ow, (cuuint64_t)oh, (cuuint64_t)n};
      const cuuint64_t strides[3] = {(cuuint64_t)y->stride[3] * 4, (cuuint64_t)y->stride[2] * 4,
                                     (cuuint64_t)y->stride[0] * 4};
      const cuuint32_t box[4] = {16, (cuuint32_t)(a.tw >= 32 ? 32 : a.tw),
                                 (cuuint32_t)(a.tw >= 32 ? 1 : 32 / a.tw), 1};
      staged = encode_tiled(y->data, 4, dims, strides, box, &ymap, nullptr,
                            CU_TENSOR_MAP_SWIZZLE_64B) == MM_OK;
    } else if (y->stride[2] == ow * y->stride[3] && y->stride[0] == oh * y->stride[2]) {
      const cuuint64_t dims[2] = {(cuuint64_t)k_out, (cuuint64_t)m_total};
      const cuuint64_t strides[1] = {(cuuint64_t)y->stride[3] * 4};
      const cuuint32_t box[2] = {16, 32};
      staged = encode_tiled(y->data, 2, dims, strides, box, &ymap, nullptr,
                            CU_TENSOR_MAP_SWIZZLE_64B) == MM_OK;
    }
  }
  // Staging per epilogue warp: its chunks of one tile (all of them when the
  // two-group epilogue may be chosen, bn <= 48; half of them otherwise).
  const int stg_bound = staged ? (a.bn <= 16 * TC_EPI_CHUNKS ? nchunk : (nchunk + 1) / 2) : 0;
  // TMEM: lo slots of 32 columns, two [hi*hi | hi*lo] period buffers of 2 bn
  // columns and xbuf lo*hi tile sums of bn columns.  Two tile sums (the next
  // tile's sum overlaps the epilogue) when at least two lo slots still fit,
  // else one; as many lo slots as fit, up to TC_MAX_LO.  Shared memory: as
  // many A + B stages as fit (the lo ring no longer bounds them).
  a.xbuf = 0;
  // (fewer sub-blocks per k-block when TMEM cannot hold two slots of the
  // requested width)
  for (; a.xbuf == 0 && a.ksub >= 1; a.ksub /= 2) {
    for (int xbuf = 2; xbuf >= 1 && a.xbuf == 0; --xbuf) {
      const int free_cols = (int)TC_TMEM_COLS - (4 + xbuf) * a.bn;
      const int slots = free_cols / (TC_LO_COLS * a.ksub);
      if (slots >= 2) {
        a.xbuf = xbuf;
        a.lo_slots = slots < TC_MAX_LO ? slots : TC_MAX_LO;
      }
    }
    if (a.xbuf != 0) break;
  }
  if (a.xbuf == 0) return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: N tile too wide");
  a.kb_total = (a.sb_total + a.ksub - 1) / a.ksub;
  {
    const int pmax = 12 / a.ksub;
    const int np = (a.kb_total + pmax - 1) / pmax;
    a.period = (a.kb_total + np - 1) / np;
  }
  if (const char* lo_env = std::getenv("MATRIXMAN_TC_LO_SLOTS")) {
    const int v = std::atoi(lo_env);
    if (v >= 2 && v <= a.lo_slots) a.lo_slots = v;
  }
  int max_stages = TC_MAX_STAGES;
  if (const char* st_env = std::getenv("MATRIXMAN_TC_STAGES")) {
    const int v = std::atoi(st_env);
    if (v >= 2 && v <= TC_MAX_STAGES) max_stages = v;
  }
  int stages = 0;
  for (int st = max_stages; st >= 2; --st) {
    if (TcSmem::make(a.bn, a.ksub, st, k_out, stg_bound).bytes() <= smem_limit) {
      stages = st;
      break;
    }
  }
  if (stages == 0) return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: N tile too wide");
  a.stages = stages;
  a.epi_groups = (a.period >= a.kb_total && a.xbuf == 2 && a.bn <= 16 * TC_EPI_CHUNKS) ? 2 : 1;
  a.stg_chunks = staged ? (a.epi_groups == 2 ? nchunk : (nchunk + 1) / 2) : 0;
  const int64_t ktot = (int64_t)r * s * c_pad;
  size_t smem = TcSmem::make(a.bn, a.ksub, stages, k_out, a.stg_chunks).bytes();

  CUtensorMap mhi, mlo;
  if ((rc = weight_map(w_hi, ktot, k_pad, a.bn, &mhi)) != MM_OK) return rc;
  if ((rc = weight_map(w_lo, ktot, k_pad, a.bn, &mlo)) != MM_OK) return rc;
  // The kernel owns all 512 TMEM columns, so a second resident CTA on an SM
  // would stall in tcgen05.alloc until the first exits: pad the shared-memory
  // request whenever the occupancy calculator allows more than one CTA.
  const int variant = 2 * (3 * (a.act >= 0 && a.act <= MM_ACT_SIGMOID ? a.act : MM_ACT_NONE) +
                           (a.res ? (a.res_before_act ? 1 : 2) : 0)) +
                      (a.ksub == 2 ? 1 : 0);
  const TcKernel kernel = tc_kernel(variant);
  {
    static size_t configured[256][TC_VARIANTS] = {};
    static size_t min_smem[256][TC_VARIANTS] = {};
    std::lock_guard<std::mutex> g(g_map_mu);
    if (dev < 0 || dev >= 256) return fail(MM_ERR_INVALID, "mm_conv2d_tc: device index");
    if (configured[dev][variant] == 0) {
      const size_t full = smem_limit;
      MM_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)full),
              "mm_conv2d_tc: shared memory attribute");
      configured[dev][variant] = full;
      for (size_t req = 16 * 1024; req <= full; req += 4096) {
        int blocks = 0;
        MM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, TC_THREADS, req),
                "mm_conv2d_tc: occupancy");
        if (blocks <= 1) {
          min_smem[dev][variant] = req;
          break;
        }
      }
      if (min_smem[dev][variant] == 0) min_smem[dev][variant] = full;
    }
    if (smem < min_smem[dev][variant]) smem = min_smem[dev][variant];
    if (smem > configured[dev][variant]) return fail(MM_ERR_UNSUPPORTED, "mm_conv2d_tc: shared memory");
  }
  // Persistent CTAs: one per SM, launched as a programmatic dependent of the
  // previous kernel in the stream (launch_pdl).
  const int64_t ctas = a.tiles < (int64_t)sm_count() ? a.tiles : (int64_t)sm_count();
  MM_CUDA(launch_pdl(kernel, dim3((unsigned)ctas), dim3(TC_THREADS), smem, resolve_stream(stream), mhi, mlo,
                     amap, ymap, a),
          "mm_conv2d_tc launch");
  MM_LAUNCH_CHECK("mm_conv2d_tc launch");
  return MM_OK;
}

}  // namespace

extern "C" int mm_conv2d_tc(const mm_tensor_t* x, const float* w_hi, const float* w_lo, int k_out,
                            int c_in, int r, int s, int c_pad, int k_pad, const float* bias,
                            const mm_tensor_t* residual, const mm_conv_params_t* p,
                            const mm_tensor_t* y, void* stream) {
  return conv2d_tc_impl(x, w_hi, w_lo, k_out, c_in, r, s, c_pad, k_pad, bias, residual, p, false, 0, 0, y,
                        stream);
}

extern "C" int mm_conv2d_tc_region(const mm_tensor_t* x, const float* w_hi, const float* w_lo, int k_out,
                                   int c_in, int r, int s, int c_pad, int k_pad, const float* bias,
                                   const mm_tensor_t* residual, const mm_conv_params_t* p, int64_t row0,
                                   int64_t col0, const mm_tensor_t* y, void* stream) {
  return conv2d_tc_impl(x, w_hi, w_lo, k_out, c_in, r, s, c_pad, k_pad, bias, residual, p, true, row0, col0,
                        y, stream);
}

// Test hook for the bounded-wait error path (no counterpart in the
// reference): sets the budget of the kernel's waits on `device` (wait_ns <= 0:
// the default 200 ms) and whether CTA 0 leaves its first k-block unissued, for
// every later launch on that device.
extern "C" int mm_debug_tc_fault(int device, int64_t wait_ns, int drop_first_load) {
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != device) MM_CUDA(cudaSetDevice(device), "cudaSetDevice");
  const unsigned long long ns = wait_ns > 0 ? (unsigned long long)wait_ns : (unsigned long long)TC_WAIT_NS;
  const int drop = drop_first_load ? 1 : 0;
  cudaError_t e = cudaMemcpyToSymbol(g_tc_wait_ns, &ns, sizeof(ns));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_tc_drop_first_load, &drop, sizeof(drop));
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "mm_debug_tc_fault");
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
