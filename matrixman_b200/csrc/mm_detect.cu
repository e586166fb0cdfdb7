// Detection postprocessing on the device: the reduction the reference runs as
// an OpenGL shader (best class per anchor), and confidence filtering + box
// conversion + per-class greedy NMS, which the reference runs on the CPU.
//
//   mm_detect_reduce: [B, 4+C, A] -> [B, 6, A] = (cx, cy, w, h, best score,
//     best class); the best score starts at -1 and a class replaces it only
//     when strictly greater (first maximum wins), as in the reference shader
//     (backends/opengl/ops/postprocessing.py:35-52).
//   mm_detect_nms: per image, anchors whose best score (first maximum over the
//     classes, as torch's max/argmax) is >= conf_thr become candidates with
//     corner boxes (cx - w/2, cy - h/2, cx + w/2, cy + h/2) clamped to
//     [0, width-1] x [0, height-1]; candidates are ordered by score
//     (descending; equal scores by class, then anchor index), and greedy NMS
//     keeps a candidate unless an earlier kept candidate of the same class
//     overlaps it
//     with IoU > iou_thr (a candidate is kept only when IoU <= iou_thr, so a NaN
//     IoU suppresses) -- the reference's per-class loop
//     (demo/yolo_helpers.py:59-89, 91-137) restated as one pass over all
//     classes, with its fp32 arithmetic in the same order (no contraction).
//     Within a class this order is the reference's (score, then input order);
//     across classes it is the order of the reference's final sort of the kept
//     detections by score (yolo_helpers.py:128), stable over its class-by-class
//     list, so the kept list is already in output order.  The first max_det
//     kept detections (x1, y1, x2, y2, score, class) go to dets[b];
//     counts[b] = their number.
//
// One CTA per image sorts its candidates' keys and holds their boxes and
// classes in shared memory (at most MM_DETECT_MAX_CANDIDATES of them).  An
// image with more candidates runs a second, slower pass over the whole image
// in global memory (detect_nms_large_kernel) with the same result, so the
// number of candidates is not limited.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>

#include "mm_common.cuh"

namespace mm {

constexpr int DET_CAP = MM_DETECT_MAX_CANDIDATES;
constexpr int DET_SORT = 16384;  // power of two >= DET_CAP: the sort's length limit
static_assert(DET_SORT >= DET_CAP && DET_CAP < 32768, "candidate indices are int16");
constexpr int DET_THREADS = 1024;

struct DetArgs {
  const float* pred;
  int64_t ps0, ps1, ps2;  // strides of [B, 4+C, A]
  int64_t batch, anchors;
  int classes;
  float conf_thr, iou_thr, xmax, ymax;  // xmax = width - 1, ymax = height - 1
  int max_det;
  int abits;  // anchor bits of a sort key (32 - class bits); 0: keys do not fit, every
              // image with candidates takes the global-memory pass
  float* dets;
  int64_t ds0, ds1, ds2;  // strides of [B, max_det, 6]
  int32_t* counts;
};

__global__ void detect_reduce_kernel(const float* __restrict__ pred, int64_t ps0, int64_t ps1,
                                     int64_t ps2, float* __restrict__ out, int64_t os0, int64_t os1,
                                     int64_t os2, int64_t batch, int64_t anchors, int classes) {
  const int64_t total = batch * anchors;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / anchors, a = i - b * anchors;
    const float* p = pred + b * ps0 + a * ps2;
    float* o = out + b * os0 + a * os2;
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k * os1] = p[k * ps1];
    float best = -1.0f;
    int best_cls = 0;
    for (int c = 0; c < classes; ++c) {
      const float s = p[(4 + c) * ps1];
      if (s > best) {
        best = s;
        best_cls = c;
      }
    }
    o[4 * os1] = best;
    o[5 * os1] = (float)best_cls;
  }
}

// Workspace of mm_detect_nms: device memory the caller provides, laid out by
// det_work_layout (every part 256-byte aligned).
struct DetWork {
  float4* box;               // [B, A] clamped corner boxes of candidate anchors
  float2* sc;                // [B, A] (best score, class as int bits) of candidate anchors
  unsigned long long* keys;  // [B, DET_CAP] sort keys of the candidates, in arrival order
  float* score;              // [B, DET_CAP] candidate scores in NMS order
  int* keep;                 // [B, DET_CAP] NMS positions of the kept candidates
  int* count;                // [B] candidates per image; zeroed before the candidate pass
};

__host__ __device__ inline size_t det_align(size_t v) { return (v + 255) & ~(size_t)255; }

// Largest batch * anchors the workspace arithmetic accepts: 2^40 anchors in
// all (16 TiB of boxes) keeps every size below 2^48 bytes, far from size_t
// overflow, and above any real detection batch.
constexpr int64_t DET_MAX_BATCH_ANCHORS = (int64_t)1 << 40;

inline bool det_sizes_ok(int64_t batch, int64_t anchors) {
  return batch >= 0 && anchors >= 0 && batch <= 0x7fffffffLL && anchors <= 0x7fffffffLL &&
         (batch == 0 || anchors <= DET_MAX_BATCH_ANCHORS / batch);
}

// Byte offsets of the workspace parts (DetWork order); returns the total size.
__host__ __device__ inline size_t det_work_layout(int64_t batch, int64_t anchors, size_t off[6]) {
  const size_t ba = (size_t)batch * (size_t)anchors, bc = (size_t)batch * DET_CAP;
  const size_t part[6] = {ba * 16, ba * 8, bc * 8, bc * 4, bc * 4, (size_t)batch * 4};
  size_t o = 0;
  for (int i = 0; i < 6; ++i) {
    off[i] = o;
    o = det_align(o + part[i]);
  }
  return o;
}

// torch.maximum / torch.minimum: NaN if either operand is NaN.
__device__ __forceinline__ float tmax(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fc00000) : fmaxf(a, b);
}
__device__ __forceinline__ float tmin(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fc00000) : fminf(a, b);
}

__device__ __forceinline__ float clampf_keep_nan(float v, float hi) {
  return v < 0.f ? 0.f : (v > hi ? hi : v);
}

// Corner box of an anchor: (cx - w/2, cy - h/2, cx + w/2, cy + h/2) clamped
// to [0, xmax] x [0, ymax], in the reference's operation order (w / 2 exact).
__device__ __forceinline__ float4 det_box(const DetArgs& a, const float* pb, int anchor) {
  const float* p = pb + (int64_t)anchor * a.ps2;
  const float cx = p[0], cy = p[a.ps1], w = p[2 * a.ps1], h = p[3 * a.ps1];
  const float hw = __fmul_rn(w, 0.5f), hh = __fmul_rn(h, 0.5f);
  return make_float4(clampf_keep_nan(__fsub_rn(cx, hw), a.xmax), clampf_keep_nan(__fsub_rn(cy, hh), a.ymax),
                     clampf_keep_nan(__fadd_rn(cx, hw), a.xmax), clampf_keep_nan(__fadd_rn(cy, hh), a.ymax));
}

// High half of a sort key: ascending = descending score.  The score's bits
// are mapped to an unsigned integer that orders as the floats do (after -0
// becomes +0, so equal scores give equal halves); NaN scores never reach here
// (they fail the filter).
__device__ __forceinline__ unsigned det_score_key(float score) {
  unsigned u = __float_as_uint(__fadd_rn(score, 0.f));
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ~u;
}

// Sort key of a candidate: ascending keys = descending score, then ascending
// class, then ascending anchor index (the low half holds the class above the
// anchor's abits bits; the host picks abits so that both fit).
__device__ __forceinline__ unsigned long long det_key(float score, int cls, int anchor, int abits) {
  return ((unsigned long long)det_score_key(score) << 32) | ((unsigned long long)(unsigned)cls << abits) |
         (unsigned)anchor;
}

// 1. Candidates, grid-wide: per anchor the best class (first maximum), the
// confidence filter and the clamped corner box.  A candidate's box and score
// go to the workspace at its anchor; its sort key is appended to the image's
// key list (one atomic per warp).
__global__ void detect_candidates_kernel(DetArgs a, DetWork w) {
  const int lane = threadIdx.x & 31;
  for (int64_t b = blockIdx.y; b < a.batch; b += gridDim.y) {
    const float* pb = a.pred + b * a.ps0;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x; base < a.anchors;
         base += (int64_t)gridDim.x * blockDim.x) {
      const int64_t an = base + threadIdx.x;
      bool cand = false;
      float best = 0.f;
      int bc = 0;
      if (an < a.anchors) {
        const float* p = pb + an * a.ps2;
        best = p[4 * a.ps1];
        for (int c = 1; c < a.classes; ++c) {
          const float v = p[(4 + c) * a.ps1];
          if (v > best) {
            best = v;
            bc = c;
          }
        }
        cand = best >= a.conf_thr;
      }
      const unsigned m = __ballot_sync(0xffffffffu, cand);
      if (m == 0u) continue;
      const int leader = __ffs(m) - 1;
      int slot = 0;
      if (lane == leader) slot = atomicAdd(w.count + b, __popc(m));
      slot = __shfl_sync(0xffffffffu, slot, leader) + __popc(m & ((1u << lane) - 1u));
      if (cand) {
        const int64_t i = b * a.anchors + an;
        w.box[i] = det_box(a, pb, (int)an);
        w.sc[i] = make_float2(best, __int_as_float(bc));
        if (slot < DET_CAP && a.abits > 0) w.keys[b * DET_CAP + slot] = det_key(best, bc, (int)an, a.abits);
      }
    }
  }
}

// Shared memory of the NMS pass: the sort keys first, then (over them) the
// boxes and classes in NMS order, a class of -1 marking a suppressed one.
constexpr size_t DET_SMEM = (size_t)DET_CAP * (16 + 2);
static_assert((size_t)DET_CAP * 16 >= (size_t)DET_SORT * 8, "the keys lie inside the box array");
constexpr int DET_PER_THREAD = (DET_CAP + DET_THREADS - 1) / DET_THREADS;

// 2.-4. Per image, one CTA: sort, greedy NMS, output.
__global__ void __launch_bounds__(DET_THREADS) detect_nms_kernel(DetArgs a, DetWork w) {
  extern __shared__ __align__(16) uint8_t det_raw[];
  unsigned long long* key = reinterpret_cast<unsigned long long*>(det_raw);
  float4* box = reinterpret_cast<float4*>(det_raw);
  int16_t* cls = reinterpret_cast<int16_t*>(det_raw + (size_t)DET_CAP * 16);
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  const int n = w.count[b];
  if (n > DET_CAP || (a.abits == 0 && n > 0)) {
    if (tid == 0) a.counts[b] = -n;  // left to detect_nms_large_kernel
    return;
  }

  // 2. Bitonic sort of the keys (padding keys, all ones, sort last).
  int P = 1;
  while (P < n) P <<= 1;
  const unsigned long long* kb = w.keys + b * DET_CAP;
  for (int i = tid; i < P; i += DET_THREADS) key[i] = i < n ? kb[i] : ~0ull;
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int t = tid; t < (P >> 1); t += DET_THREADS) {
        const int i = ((t & ~(j - 1)) << 1) | (t & (j - 1));  // lower slot of the pair
        const int l = i | j;
        const unsigned long long x = key[i], y = key[l];
        if ((i & k) == 0 ? x > y : x < y) {
          key[i] = y;
          key[l] = x;
        }
      }
      __syncthreads();
    }
  }

  // Boxes and classes into shared memory in NMS order (over the keys: every
  // thread takes its keys' anchors first), scores into the workspace.
  unsigned an[DET_PER_THREAD];
#pragma unroll
  for (int k = 0; k < DET_PER_THREAD; ++k) {
    const int j = tid + k * DET_THREADS;
    an[k] = j < n ? (unsigned)key[j] & (unsigned)((1ull << a.abits) - 1ull) : 0u;
  }
  __syncthreads();
  const float4* wb = w.box + b * a.anchors;
  const float2* ws = w.sc + b * a.anchors;
  float* wscore = w.score + b * DET_CAP;
#pragma unroll
  for (int k = 0; k < DET_PER_THREAD; ++k) {
    const int j = tid + k * DET_THREADS;
    if (j < n) {
      const float2 v = ws[an[k]];
      box[j] = wb[an[k]];
      cls[j] = (int16_t)__float_as_int(v.y);
      wscore[j] = v.x;
    }
  }
  __syncthreads();

  // 3. Greedy NMS in score order, suppressing within a class only.  Kept
  // candidates are final once kept (only earlier kept ones suppress), so the
  // pass ends after max_det of them.  i and nk are computed alike by every
  // thread.
  float* db = a.dets + b * a.ds0;
  int* keep = w.keep + b * DET_CAP;
  int i = 0, nk = 0;
  while (nk < a.max_det) {
    // The next live position >= i: the lowest bit of a warp ballot.  Positions
    // below it are settled, and this pass only writes positions above it.
    while (i < n) {
      const unsigned m = __ballot_sync(0xffffffffu, i + lane < n && cls[i + lane] >= 0);
      if (m != 0u) {
        i += __ffs(m) - 1;
        break;
      }
      i += 32;
    }
    if (i >= n) break;
    const float4 cb = box[i];
    const int ccls = cls[i];
    if (tid == 0) {
      float* o = db + (int64_t)nk * a.ds1;
      o[0] = cb.x;
      o[a.ds2] = cb.y;
      o[2 * a.ds2] = cb.z;
      o[3 * a.ds2] = cb.w;
      o[5 * a.ds2] = (float)ccls;
      keep[nk] = i;
    }
    ++nk;
    const float carea = __fmul_rn(__fsub_rn(cb.z, cb.x), __fsub_rn(cb.w, cb.y));
    for (int j = i + 1 + tid; j < n; j += DET_THREADS) {
      if (cls[j] != ccls) continue;
      const float4 rb = box[j];
      const float xx1 = tmax(rb.x, cb.x), yy1 = tmax(rb.y, cb.y);
      const float xx2 = tmin(rb.z, cb.z), yy2 = tmin(rb.w, cb.w);
      float iw = __fsub_rn(xx2, xx1), ih = __fsub_rn(yy2, yy1);
      iw = iw < 0.f ? 0.f : iw;
      ih = ih < 0.f ? 0.f : ih;
      const float inter = __fmul_rn(iw, ih);
      const float rarea = __fmul_rn(__fsub_rn(rb.z, rb.x), __fsub_rn(rb.w, rb.y));
      float den = __fsub_rn(__fadd_rn(carea, rarea), inter);
      den = den < 1e-12f ? 1e-12f : den;
      const float iou = __fdiv_rn(inter, den);
      if (!(iou <= a.iou_thr)) cls[j] = -1;
    }
    __syncthreads();
    ++i;
  }
  __syncthreads();

  // 4. Scores of the kept detections (rows 0..nk-1 hold the rest already).
  for (int r = tid; r < nk; r += DET_THREADS) db[(int64_t)r * a.ds1 + 4 * a.ds2] = wscore[keep[r]];
  if (tid == 0) a.counts[b] = nk;
}

// 5. Images with more candidates than the shared-memory pass holds
// (detect_nms_kernel left counts[b] = -n): greedy NMS over the whole image in
// global memory, one CTA per image (the others return at once).  The CTA marks
// the image's candidates again (class -1 for the other anchors, whose
// workspace entries the candidate pass did not write), then each round finds
// the next candidate in NMS order -- the smallest (score key, class), then
// the smallest anchor among the live ones with it: two block reductions --
// keeps it and removes it and the later candidates of its class that overlap
// it with IoU > iou_thr.  Same order, arithmetic and output as
// detect_nms_kernel, without a limit on candidates, classes or anchors.

// Minimum of v over the CTA (DET_THREADS threads), returned to every thread.
__device__ __forceinline__ unsigned long long det_block_min(unsigned long long v, unsigned long long* red,
                                                            unsigned long long* out) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, v, o);
    v = other < v ? other : v;
  }
  if (lane == 0) red[wid] = v;
  __syncthreads();
  if (wid == 0) {
    v = lane < DET_THREADS / 32 ? red[lane] : ~0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, v, o);
      v = other < v ? other : v;
    }
    if (lane == 0) *out = v;
  }
  __syncthreads();
  return *out;
}

__global__ void __launch_bounds__(DET_THREADS) detect_nms_large_kernel(DetArgs a, DetWork w) {
  const int64_t b = blockIdx.x;
  if (a.counts[b] >= 0) return;
  const int tid = threadIdx.x;
  const float* pb = a.pred + b * a.ps0;
  float2* sc = w.sc + b * a.anchors;
  float4* bx = w.box + b * a.anchors;
  for (int64_t an = tid; an < a.anchors; an += DET_THREADS) {
    const float* p = pb + an * a.ps2;
    float best = p[4 * a.ps1];
    int bc = 0;
    for (int c = 1; c < a.classes; ++c) {
      const float v = p[(4 + c) * a.ps1];
      if (v > best) {
        best = v;
        bc = c;
      }
    }
    if (best >= a.conf_thr) {
      bx[an] = det_box(a, pb, (int)an);
      sc[an] = make_float2(best, __int_as_float(bc));
    } else {
      sc[an] = make_float2(0.f, __int_as_float(-1));
    }
  }
  __syncthreads();
  __shared__ unsigned long long red[DET_THREADS / 32];
  __shared__ unsigned long long s_min;
  float* db = a.dets + b * a.ds0;
  int nk = 0;
  while (nk < a.max_det) {
    unsigned long long mk = ~0ull;
    for (int64_t an = tid; an < a.anchors; an += DET_THREADS) {
      const float2 v = sc[an];
      const int c = __float_as_int(v.y);
      if (c >= 0) {
        const unsigned long long k = ((unsigned long long)det_score_key(v.x) << 32) | (unsigned)c;
        mk = k < mk ? k : mk;
      }
    }
    const unsigned long long key = det_block_min(mk, red, &s_min);
    if (key == ~0ull) break;
    // The smallest anchor with this score and class (its reduction may start
    // only after every thread has read s_min: the first barrier inside).
    unsigned long long ma = ~0ull;
    for (int64_t an = tid; an < a.anchors; an += DET_THREADS) {
      const float2 v = sc[an];
      const int c = __float_as_int(v.y);
      if (c >= 0 && (((unsigned long long)det_score_key(v.x) << 32) | (unsigned)c) == key) {
        ma = (unsigned long long)an < ma ? (unsigned long long)an : ma;
      }
    }
    const int i = (int)det_block_min(ma, red, &s_min);
    const float4 cb = bx[i];
    const float2 cv = sc[i];
    const int ccls = __float_as_int(cv.y);
    if (tid == 0) {
      float* o = db + (int64_t)nk * a.ds1;
      o[0] = cb.x;
      o[a.ds2] = cb.y;
      o[2 * a.ds2] = cb.z;
      o[3 * a.ds2] = cb.w;
      o[4 * a.ds2] = cv.x;
      o[5 * a.ds2] = (float)ccls;
    }
    ++nk;
    __syncthreads();  // every thread has read the kept candidate's entries
    const float carea = __fmul_rn(__fsub_rn(cb.z, cb.x), __fsub_rn(cb.w, cb.y));
    for (int64_t an = tid; an < a.anchors; an += DET_THREADS) {
      const float2 v = sc[an];
      if (__float_as_int(v.y) != ccls) continue;
      if (an == i) {
        sc[an].y = __int_as_float(-1);
        continue;
      }
      const float4 rb = bx[an];
      const float xx1 = tmax(rb.x, cb.x), yy1 = tmax(rb.y, cb.y);
      const float xx2 = tmin(rb.z, cb.z), yy2 = tmin(rb.w, cb.w);
      float iw = __fsub_rn(xx2, xx1), ih = __fsub_rn(yy2, yy1);
      iw = iw < 0.f ? 0.f : iw;
      ih = ih < 0.f ? 0.f : ih;
      const float inter = __fmul_rn(iw, ih);
      const float rarea = __fmul_rn(__fsub_rn(rb.z, rb.x), __fsub_rn(rb.w, rb.y));
      float den = __fsub_rn(__fadd_rn(carea, rarea), inter);
      den = den < 1e-12f ? 1e-12f : den;
      const float iou = __fdiv_rn(inter, den);
      if (!(iou <= a.iou_thr)) sc[an].y = __int_as_float(-1);
    }
    __syncthreads();
  }
  if (tid == 0) a.counts[b] = nk;
}

}  // namespace mm

using namespace mm;

extern "C" int mm_detect_reduce(const mm_tensor_t* pred, const mm_tensor_t* out, void* stream) {
  int rc;
  if ((rc = validate(pred, "mm_detect_reduce prediction", MM_F32)) != MM_OK) return rc;
  if ((rc = validate(out, "mm_detect_reduce output", MM_F32)) != MM_OK) return rc;
  if (pred->ndim != 3 || pred->size[1] < 5)
    return fail(MM_ERR_INVALID, "mm_detect_reduce: prediction must be [B, 4+classes, anchors]");
  if (out->ndim != 3 || out->size[0] != pred->size[0] || out->size[1] != 6 || out->size[2] != pred->size[2])
    return fail(MM_ERR_INVALID, "mm_detect_reduce: output must be [B, 6, anchors]");
  if (pred->size[1] - 4 > 0x7fffffffLL) return fail(MM_ERR_UNSUPPORTED, "mm_detect_reduce: too many classes");
  const int64_t total = pred->size[0] * pred->size[2];
  if (total == 0) return MM_OK;
  cudaStream_t s = resolve_stream(stream);
  detect_reduce_kernel<<<grid_for(total, 256, (int64_t)sm_count() * 8), 256, 0, s>>>(
      (const float*)pred->data, pred->stride[0], pred->stride[1], pred->stride[2], (float*)out->data,
      out->stride[0], out->stride[1], out->stride[2], pred->size[0], pred->size[2],
      (int)(pred->size[1] - 4));
  MM_LAUNCH_CHECK("mm_detect_reduce launch");
  return MM_OK;
}

extern "C" int mm_detect_nms_workspace_size(int64_t batch, int64_t anchors, size_t* bytes) {
  if (bytes == nullptr || batch < 0 || anchors < 0)
    return fail(MM_ERR_INVALID, "mm_detect_nms_workspace_size: bad arguments");
  if (!det_sizes_ok(batch, anchors))
    return fail(MM_ERR_UNSUPPORTED, "mm_detect_nms_workspace_size: batch x anchors too large");
  size_t off[6];
  *bytes = det_work_layout(batch, anchors, off);
  return MM_OK;
}

extern "C" int mm_detect_nms(const mm_tensor_t* pred, float conf_thr, float iou_thr, float width,
                             float height, int max_det, const mm_tensor_t* dets, int32_t* counts,
                             void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = validate(pred, "mm_detect_nms prediction", MM_F32)) != MM_OK) return rc;
  if ((rc = validate(dets, "mm_detect_nms detections", MM_F32)) != MM_OK) return rc;
  if (pred->ndim != 3 || pred->size[1] < 5)
    return fail(MM_ERR_INVALID, "mm_detect_nms: prediction must be [B, 4+classes, anchors]");
  if (max_det < 0 || dets->ndim != 3 || dets->size[0] != pred->size[0] || dets->size[1] != max_det ||
      dets->size[2] != 6)
    return fail(MM_ERR_INVALID, "mm_detect_nms: detections must be [B, max_det, 6]");
  if (counts == nullptr && pred->size[0] > 0) return fail(MM_ERR_INVALID, "mm_detect_nms: null counts");
  if (pred->size[1] - 4 > 32767 || !det_sizes_ok(pred->size[0], pred->size[2]))
    return fail(MM_ERR_UNSUPPORTED, "mm_detect_nms: too many classes, images or anchors");
  if (pred->size[0] == 0) return MM_OK;
  size_t off[6];
  const size_t need = det_work_layout(pred->size[0], pred->size[2], off);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(MM_ERR_INVALID, "mm_detect_nms: workspace smaller than mm_detect_nms_workspace_size");
  if (((uintptr_t)workspace & 255u) != 0u)
    return fail(MM_ERR_INVALID, "mm_detect_nms: workspace must be 256-byte aligned");
  DetArgs a;
  a.pred = (const float*)pred->data;
  a.ps0 = pred->stride[0]; a.ps1 = pred->stride[1]; a.ps2 = pred->stride[2];
  a.batch = pred->size[0];
  a.anchors = pred->size[2];
  a.classes = (int)(pred->size[1] - 4);
  a.conf_thr = conf_thr;
  a.iou_thr = iou_thr;
  a.xmax = width - 1.0f;
  a.ymax = height - 1.0f;
  a.max_det = max_det;
  {
    int cbits = 0;  // bits of the largest class index
    while ((1ll << cbits) < (long long)a.classes) ++cbits;
    a.abits = a.anchors <= (1ll << (32 - cbits)) ? 32 - cbits : 0;
  }
  a.dets = (float*)dets->data;
  a.ds0 = dets->stride[0]; a.ds1 = dets->stride[1]; a.ds2 = dets->stride[2];
  a.counts = counts;
  uint8_t* base = (uint8_t*)workspace;
  DetWork w;
  w.box = (float4*)(base + off[0]);
  w.sc = (float2*)(base + off[1]);
  w.keys = (unsigned long long*)(base + off[2]);
  w.score = (float*)(base + off[3]);
  w.keep = (int*)(base + off[4]);
  w.count = (int*)(base + off[5]);
  {
    // Once per device; host threads may race here, which only repeats the
    // (idempotent) attribute call.
    static std::atomic<bool> configured[256];
    int dev = 0;
    MM_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev >= 0 && dev < 256 && !configured[dev].load(std::memory_order_acquire)) {
      MM_CUDA(cudaFuncSetAttribute(detect_nms_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)DET_SMEM),
              "mm_detect_nms: shared memory attribute");
      configured[dev].store(true, std::memory_order_release);
    }
  }
  cudaStream_t s = resolve_stream(stream);
  MM_CUDA(cudaMemsetAsync(w.count, 0, (size_t)a.batch * sizeof(int), s), "mm_detect_nms: clear counts");
  const int64_t xblocks = std::min<int64_t>((a.anchors + 255) / 256, 1024);
  const dim3 grid((unsigned)std::max<int64_t>(xblocks, 1), (unsigned)std::min<int64_t>(a.batch, 65535));
  detect_candidates_kernel<<<grid, 256, 0, s>>>(a, w);
  MM_LAUNCH_CHECK("mm_detect_nms candidate launch");
  detect_nms_kernel<<<(unsigned)a.batch, DET_THREADS, DET_SMEM, s>>>(a, w);
  MM_LAUNCH_CHECK("mm_detect_nms launch");
  detect_nms_large_kernel<<<(unsigned)a.batch, DET_THREADS, 0, s>>>(a, w);
  MM_LAUNCH_CHECK("mm_detect_nms large-image launch");
  return MM_OK;
}

// ---------------------------------------------------------------------------
// mm_detect_nms_static: the same detection NMS for callers that may not
// allocate device memory -- a plugin inside a host application that owns all
// GPU memory and forbids cudaMalloc after start-up, or a real-time loop whose
// memory is fixed before it starts.  Its workspace is this file's static device
// array instead of a caller buffer.  Every GPU that loads the library holds
// the array until the process exits, and all calls on a GPU share it.
static __device__ __align__(256) uint8_t det_static_work[MM_DETECT_STATIC_WORK_BYTES];

namespace {
std::mutex det_static_mu;
// Device address of det_static_work per device, with the context it was
// looked up in: a device reset (cudaDeviceReset) makes a new context in
// which the module, and so the array, is loaded again at another address.
void* det_static_addr[256] = {};
void* det_static_ctx[256] = {};

// The calling thread's current CUDA context (cuCtxGetCurrent through the
// runtime's driver entry point, so the library does not link libcuda).
int current_context(void** ctx) {
  using GetCtxFn = int (*)(void**);
  static GetCtxFn get_ctx = nullptr;
  if (get_ctx == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        fn == nullptr || q != cudaDriverEntryPointSuccess)
      return fail(MM_ERR_CUDA, "mm_detect_nms_static: cuCtxGetCurrent entry point unavailable");
    get_ctx = (GetCtxFn)fn;
  }
  *ctx = nullptr;
  if (get_ctx(ctx) != 0 || *ctx == nullptr)
    return fail(MM_ERR_STATE, "mm_detect_nms_static: no current CUDA context");
  return MM_OK;
}
}  // namespace

extern "C" int mm_detect_nms_static(const mm_tensor_t* pred, float conf_thr, float iou_thr,
                                    float width, float height, int max_det, const mm_tensor_t* dets,
                                    int32_t* counts, void* stream) {
  int rc;
  if ((rc = validate(pred, "mm_detect_nms_static prediction", MM_F32)) != MM_OK) return rc;
  if (pred->ndim == 3 && pred->size[0] > 0) {
    if (!det_sizes_ok(pred->size[0], pred->size[2]))
      return fail(MM_ERR_UNSUPPORTED, "mm_detect_nms_static: too many images or anchors");
    size_t off[6];
    const size_t need = det_work_layout(pred->size[0], pred->size[2], off);
    if (need > (size_t)MM_DETECT_STATIC_WORK_BYTES)
      return fail(MM_ERR_UNSUPPORTED,
                  "mm_detect_nms_static: " + std::to_string(pred->size[0]) + " images of " +
                      std::to_string(pred->size[2]) + " anchors need " + std::to_string(need) +
                      " bytes of scratch, more than its fixed " +
                      std::to_string((size_t)MM_DETECT_STATIC_WORK_BYTES) +
                      "; split the batch or call mm_detect_nms with a workspace");
  }
  int dev = 0;
  MM_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= 256) return fail(MM_ERR_UNSUPPORTED, "mm_detect_nms_static: device index above 255");
  // The first call on a device (with that device current) makes sure the
  // runtime's context exists (cudaSetDevice initialises it), then looks up
  // the array's device address in it (the name itself is only a host-side
  // stand-in); later calls reuse the address while that context lives.
  MM_CUDA(cudaSetDevice(dev), "mm_detect_nms_static: context");
  void* ctx = nullptr;
  if ((rc = current_context(&ctx)) != MM_OK) return rc;
  void* work = nullptr;
  {
    std::lock_guard<std::mutex> lock(det_static_mu);
    if (det_static_addr[dev] == nullptr || det_static_ctx[dev] != ctx) {
      void* addr = nullptr;
      MM_CUDA(cudaGetSymbolAddress(&addr, det_static_work), "mm_detect_nms_static: static scratch address");
      det_static_addr[dev] = addr;
      det_static_ctx[dev] = ctx;
    }
    work = det_static_addr[dev];
  }
  return mm_detect_nms(pred, conf_thr, iou_thr, width, height, max_det, dets, counts, work,
                       (size_t)MM_DETECT_STATIC_WORK_BYTES, stream);
}
