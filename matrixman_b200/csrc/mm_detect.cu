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
//     (descending; equal scores by anchor index), and greedy NMS keeps a
//     candidate unless an earlier kept candidate of the same class overlaps it
//     with IoU > iou_thr (a candidate is kept only when IoU <= iou_thr, so a NaN
//     IoU suppresses) -- the reference's per-class loop
//     (demo/yolo_helpers.py:59-89, 91-137) restated as one pass over all
//     classes, with its fp32 arithmetic in the same order (no contraction).
//     The first max_det kept detections (x1, y1, x2, y2, score, class), in
//     descending score order, go to dets[b]; counts[b] = their number.
//
// One CTA per image holds its candidates' scores, classes and anchors in
// shared memory (at most MM_DETECT_MAX_CANDIDATES); their boxes are recomputed
// from the prediction (L2-resident) where needed.  An image with more
// candidates is not processed and reports counts[b] = -(number of candidates).
#include <cuda_runtime.h>
#include <stdint.h>

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

// Candidate arrays in dynamic shared memory.
struct DetSmem {
  float* score;    // [DET_CAP]
  int* anchor;     // [DET_CAP]
  int16_t* cls;    // [DET_CAP]
  int16_t* keep;   // [DET_CAP] kept candidates in order
  int16_t* ord;    // [DET_SORT] sort order
  uint8_t* sup;    // [DET_CAP] suppressed flags
};

__host__ __device__ constexpr size_t det_smem_bytes() {
  return (size_t)DET_CAP * (4 + 4 + 2 + 2 + 1) + (size_t)DET_SORT * 2 + 64;
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

// a before b in the NMS order: higher score first, then lower anchor index.
__device__ __forceinline__ bool det_before(const DetSmem& s, int a, int b) {
  return s.score[a] > s.score[b] || (s.score[a] == s.score[b] && s.anchor[a] < s.anchor[b]);
}

// Sort slot x belongs strictly after slot y (-1 = padding, after every candidate).
__device__ __forceinline__ bool det_after(const DetSmem& s, int x, int y) {
  if (x < 0) return y >= 0;
  if (y < 0) return false;
  return det_before(s, y, x);
}

__global__ void __launch_bounds__(DET_THREADS) detect_nms_kernel(DetArgs a) {
  extern __shared__ __align__(16) uint8_t det_raw[];
  __shared__ int s_count;
  DetSmem s;
  s.score = reinterpret_cast<float*>(det_raw);
  s.anchor = reinterpret_cast<int*>(s.score + DET_CAP);
  s.cls = reinterpret_cast<int16_t*>(s.anchor + DET_CAP);
  s.keep = s.cls + DET_CAP;
  s.ord = s.keep + DET_CAP;
  s.sup = reinterpret_cast<uint8_t*>(s.ord + DET_SORT);
  const int64_t b = blockIdx.x;
  const int tid = threadIdx.x;
  if (tid == 0) s_count = 0;
  __syncthreads();

  // 1. Candidates: best class (first maximum), confidence filter, corner boxes.
  const float* pb = a.pred + b * a.ps0;
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
      const int slot = atomicAdd(&s_count, 1);
      if (slot < DET_CAP) {
        s.score[slot] = best;
        s.cls[slot] = (int16_t)bc;
        s.anchor[slot] = (int)an;
      }
    }
  }
  __syncthreads();
  const int count = s_count;
  if (count > DET_CAP) {
    if (tid == 0) a.counts[b] = -count;
    return;
  }
  const int n = count;

  // 2. Bitonic sort of the candidate order (padding entries sort last).
  int P = 1;
  while (P < n) P <<= 1;
  for (int i = tid; i < P; i += DET_THREADS) {
    s.ord[i] = (int16_t)(i < n ? i : -1);
    if (i < n) s.sup[i] = 0;
  }
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < P; i += DET_THREADS) {
        const int l = i ^ j;
        if (l > i) {
          const int ai = s.ord[i], al = s.ord[l];
          const bool up = (i & k) == 0;  // this pair's segment sorts in NMS order
          if (up ? det_after(s, ai, al) : det_after(s, al, ai)) {
            s.ord[i] = (int16_t)al;
            s.ord[l] = (int16_t)ai;
          }
        }
      }
      __syncthreads();
    }
  }

  // 3. Greedy NMS in score order, suppressing within a class only.  Kept
  // candidates are final once kept (only earlier kept ones suppress), so the
  // pass ends after max_det of them.  nk is counted by every thread alike.
  int i = 0, nk = 0;
  while (nk < a.max_det) {
    // uniform: every thread reads the same flags (a padding slot, which the sort
    // never leaves among the first n, would count as suppressed)
    while (i < n && (s.ord[i] < 0 || s.sup[s.ord[i]])) ++i;
    if (i >= n) break;
    const int c = s.ord[i];
    if (tid == 0) s.keep[nk] = (int16_t)c;
    ++nk;
    const float4 cb = det_box(a, pb, s.anchor[c]);
    const float cx1 = cb.x, cy1 = cb.y, cx2 = cb.z, cy2 = cb.w;
    const float carea = __fmul_rn(__fsub_rn(cx2, cx1), __fsub_rn(cy2, cy1));
    const int ccls = s.cls[c];
    for (int j = i + 1 + tid; j < n; j += DET_THREADS) {
      const int r = s.ord[j];
      if (r < 0 || s.sup[r] || s.cls[r] != ccls) continue;
      const float4 rb = det_box(a, pb, s.anchor[r]);
      const float xx1 = tmax(rb.x, cx1), yy1 = tmax(rb.y, cy1);
      const float xx2 = tmin(rb.z, cx2), yy2 = tmin(rb.w, cy2);
      float iw = __fsub_rn(xx2, xx1), ih = __fsub_rn(yy2, yy1);
      iw = iw < 0.f ? 0.f : iw;
      ih = ih < 0.f ? 0.f : ih;
      const float inter = __fmul_rn(iw, ih);
      const float rarea = __fmul_rn(__fsub_rn(rb.z, rb.x), __fsub_rn(rb.w, rb.y));
      float den = __fsub_rn(__fadd_rn(carea, rarea), inter);
      den = den < 1e-12f ? 1e-12f : den;
      const float iou = __fdiv_rn(inter, den);
      if (!(iou <= a.iou_thr)) s.sup[r] = 1;
    }
    __syncthreads();
    ++i;
  }
  __syncthreads();

  // 4. The first max_det kept detections, in descending score order.
  const int kept = nk;
  float* db = a.dets + b * a.ds0;
  for (int r = tid; r < kept; r += DET_THREADS) {
    const int c = s.keep[r];
    float* o = db + r * a.ds1;
    const float4 box = det_box(a, pb, s.anchor[c]);
    o[0] = box.x;
    o[a.ds2] = box.y;
    o[2 * a.ds2] = box.z;
    o[3 * a.ds2] = box.w;
    o[4 * a.ds2] = s.score[c];
    o[5 * a.ds2] = (float)s.cls[c];
  }
  if (tid == 0) a.counts[b] = kept;
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

extern "C" int mm_detect_nms(const mm_tensor_t* pred, float conf_thr, float iou_thr, float width,
                             float height, int max_det, const mm_tensor_t* dets, int32_t* counts,
                             void* stream) {
  int rc;
  if ((rc = validate(pred, "mm_detect_nms prediction", MM_F32)) != MM_OK) return rc;
  if ((rc = validate(dets, "mm_detect_nms detections", MM_F32)) != MM_OK) return rc;
  if (pred->ndim != 3 || pred->size[1] < 5)
    return fail(MM_ERR_INVALID, "mm_detect_nms: prediction must be [B, 4+classes, anchors]");
  if (max_det < 0 || dets->ndim != 3 || dets->size[0] != pred->size[0] || dets->size[1] != max_det ||
      dets->size[2] != 6)
    return fail(MM_ERR_INVALID, "mm_detect_nms: detections must be [B, max_det, 6]");
  if (counts == nullptr && pred->size[0] > 0) return fail(MM_ERR_INVALID, "mm_detect_nms: null counts");
  if (pred->size[1] - 4 > 32767 || pred->size[0] > 0x7fffffffLL || pred->size[2] > 0x7fffffffLL)
    return fail(MM_ERR_UNSUPPORTED, "mm_detect_nms: too many classes, images or anchors");
  if (pred->size[0] == 0) return MM_OK;
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
  a.dets = (float*)dets->data;
  a.ds0 = dets->stride[0]; a.ds1 = dets->stride[1]; a.ds2 = dets->stride[2];
  a.counts = counts;
  const size_t smem = det_smem_bytes();
  {
    static bool configured[256] = {};
    int dev = 0;
    MM_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev >= 0 && dev < 256 && !configured[dev]) {
      MM_CUDA(cudaFuncSetAttribute(detect_nms_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)smem),
              "mm_detect_nms: shared memory attribute");
      configured[dev] = true;
    }
  }
  cudaStream_t s = resolve_stream(stream);
  detect_nms_kernel<<<(unsigned)a.batch, DET_THREADS, smem, s>>>(a);
  MM_LAUNCH_CHECK("mm_detect_nms launch");
  return MM_OK;
}
