"""Per-op CPU restatement (torch CPU fp32 / NumPy) -- test infrastructure only.

Each function states the semantics of one op on MatrixMan's tensor path and
cites the reference implementation it follows.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def conv2d(x, w, b=None, stride=1, padding=0, dilation=1, groups=1):
    """NCHW direct convolution (reference generic kernel conv2d_nchw,
    backends/cuda/gpumatrix.py:989; checked against torch in
    diagnostics/matrixman_conv_demo.py:57-70)."""
    return F.conv2d(x, w, b, stride, padding, dilation, groups)


def conv2d_loops(x: np.ndarray, w: np.ndarray, b=None, stride=(1, 1), padding=(0, 0),
                 dilation=(1, 1), groups=1) -> np.ndarray:
    """Loop-nest convolution with the index rule of reference_conv2d
    (backends/cuda/conv2d.py:13-46); float64 accumulation.  Small cases only."""
    n, c, h, wd = x.shape
    k, cg, r, s = w.shape
    oh = (h + 2 * padding[0] - dilation[0] * (r - 1) - 1) // stride[0] + 1
    ow = (wd + 2 * padding[1] - dilation[1] * (s - 1) - 1) // stride[1] + 1
    out = np.zeros((n, k, oh, ow), dtype=np.float64)
    kg = k // groups
    for bi in range(n):
        for ko in range(k):
            g = ko // kg
            for oy in range(oh):
                for ox in range(ow):
                    acc = 0.0 if b is None else float(b[ko])
                    for ci in range(cg):
                        for ky in range(r):
                            iy = oy * stride[0] - padding[0] + ky * dilation[0]
                            if iy < 0 or iy >= h:
                                continue
                            for kx in range(s):
                                ix = ox * stride[1] - padding[1] + kx * dilation[1]
                                if 0 <= ix < wd:
                                    acc += float(x[bi, g * cg + ci, iy, ix]) * float(w[ko, ci, ky, kx])
                    out[bi, ko, oy, ox] = acc
    return out.astype(np.float32)


def batch_norm_eval(x, mean, var, weight, bias, eps=1e-5):
    """Eval BatchNorm ((x-mean)/sqrt(var+eps)*w+b), batch_norm_inference
    (backends/cuda/gpumatrix.py:3945-4010), known answer in
    backends/cuda/batch_norm.py:9-22."""
    return F.batch_norm(x, mean, var, weight, bias, False, 0.0, eps)


def silu(x):
    """x * sigmoid(x) (backends/cuda/gpumatrix.py:4012; backends/cuda/silu.py:9-11)."""
    return F.silu(x)


def sigmoid(x):
    """1 / (1 + exp(-x)) (backends/cuda/gpumatrix.py:581)."""
    return torch.sigmoid(x)


def relu(x):
    """max(x, 0) with NaN passthrough (OpenGL-only in the reference:
    backends/opengl/ops/activation.py:278-306, 334-393)."""
    return F.relu(x)


def softmax(x, dim):
    """Stable softmax along dim (matrix_softmax, backends/cuda/gpumatrix.py:784-931)."""
    return torch.softmax(x, dim)


def softmax_exact(x: torch.Tensor, dim: int) -> torch.Tensor:
    """Correctly rounded fp32 softmax computed in float64 (the exact reference
    against which ulp distances are measured)."""
    xd = x.double()
    e = torch.exp(xd - xd.amax(dim, keepdim=True))
    return (e / e.sum(dim, keepdim=True)).float()


def log_softmax(x, dim):
    return torch.log_softmax(x, dim)


def max_pool2d(x, kernel, stride=None, padding=0, dilation=1, ceil_mode=False):
    """Max pooling with -inf padding (max_pool2d_5x5_s1_p2,
    backends/cuda/gpumatrix.py:74-169 for 5x5; generic window semantics of
    backends/opengl/ops/pooling.py:47-69 and 105-190)."""
    return F.max_pool2d(x, kernel, stride, padding, dilation, ceil_mode)


def sppf_chain(x):
    """Three chained 5x5/s1/p2 max pools (the SPPF block)."""
    y1 = F.max_pool2d(x, 5, 1, 2)
    y2 = F.max_pool2d(y1, 5, 1, 2)
    y3 = F.max_pool2d(y2, 5, 1, 2)
    return y1, y2, y3


def avg_pool2d(x, kernel, stride=None, padding=0, ceil_mode=False, count_include_pad=True,
               divisor_override=None):
    return F.avg_pool2d(x, kernel, stride, padding, ceil_mode, count_include_pad, divisor_override)


def adaptive_avg_pool2d(x, size):
    return F.adaptive_avg_pool2d(x, size)


def mean(x, dims, keepdim=False):
    """mean over dims (backends/opengl/ops/reduction.py:136-221)."""
    return x.mean(dims, keepdim=keepdim)


def upsample_nearest(x, size=None, scale_factor=None):
    """Nearest upsampling.  For integer output sizes the reference's index rule
    is y = oy*H//Ho (backends/cuda/upsample.py:9-14); torch's rule with the
    size ratio agrees on integer scale factors."""
    return F.interpolate(x, size=size, scale_factor=scale_factor, mode="nearest")


def nearest_reference(values: np.ndarray, oh: int, ow: int) -> np.ndarray:
    """Integer nearest index rule of backends/cuda/upsample.py:9-14."""
    ih, iw = values.shape[-2:]
    ys = (np.arange(oh) * ih // oh).astype(np.int64)
    xs = (np.arange(ow) * iw // ow).astype(np.int64)
    return values[:, :, ys[:, None], xs[None, :]]


def addmm(bias, a, b, beta=1.0, alpha=1.0):
    """beta*bias + alpha*(a @ b) (backends/opengl/ops/matmul.py:262-281)."""
    return torch.addmm(bias, a, b, beta=beta, alpha=alpha)


def fold_conv_bn(w, b, mean, var, gamma, beta, eps):
    """BN folding of preparation.py:385-392: scale = gamma/sqrt(var+eps),
    W' = W*scale, b' = (b - mean)*scale + beta."""
    scale = gamma / torch.sqrt(var + eps)
    return w * scale.reshape(-1, 1, 1, 1), (b - mean) * scale + beta


def yolo_decode(feats, strides, reg_max=16, nc=80):
    """DFL + dist2bbox + sigmoid of the YOLOv8 head over per-level
    [B, 4*reg_max+nc, H, W] features (PreparedCudaDFL chain,
    preparation.py:222-268, followed by the anchor decode)."""
    from workloads.yolov8 import DFL, dist2bbox, make_anchors
    b = feats[0].shape[0]
    no = 4 * reg_max + nc
    flat = torch.cat([f.reshape(b, no, -1) for f in feats], 2)
    anchors, stride_t = make_anchors(feats, strides)
    box, cls = flat.split((4 * reg_max, nc), 1)
    dfl = DFL(reg_max)
    dbox = dist2bbox(dfl(box), anchors.transpose(0, 1).unsqueeze(0), dim=1) * stride_t.transpose(0, 1)
    return torch.cat((dbox, cls.sigmoid()), 1)


def detect_reduce(pred: torch.Tensor) -> torch.Tensor:
    """[B, 4+classes, anchors] -> [B, 6, anchors]: the box rows, the best class
    score (starting at -1; a class replaces it only when strictly greater) and
    its class index as float.  Restates the reference's detection-reduction
    shader (drivers/matrixman/backends/opengl/ops/postprocessing.py:35-52),
    batched."""
    p = pred.to(torch.float32)
    best = torch.full((p.shape[0], p.shape[2]), -1.0)
    cls = torch.zeros((p.shape[0], p.shape[2]))
    for c in range(p.shape[1] - 4):
        s = p[:, 4 + c]
        better = s > best
        best = torch.where(better, s, best)
        cls = torch.where(better, torch.full_like(cls, float(c)), cls)
    return torch.cat((p[:, :4], best[:, None], cls[:, None]), 1)


def _greedy_nms(boxes: torch.Tensor, scores: torch.Tensor, iou_threshold: float) -> list[int]:
    """Greedy NMS with the reference's fallback arithmetic
    (demo/yolo_helpers.py:70-89): keep the best remaining box, drop the rest
    unless IoU <= threshold.  Equal scores keep their input order."""
    keep = []
    order = torch.sort(scores, descending=True, stable=True).indices
    x1, y1, x2, y2 = boxes.unbind(1)
    areas = (x2 - x1) * (y2 - y1)
    while order.numel():
        cur = order[0]
        keep.append(int(cur))
        if order.numel() == 1:
            break
        rest = order[1:]
        xx1 = torch.maximum(x1[rest], x1[cur])
        yy1 = torch.maximum(y1[rest], y1[cur])
        xx2 = torch.minimum(x2[rest], x2[cur])
        yy2 = torch.minimum(y2[rest], y2[cur])
        inter = (xx2 - xx1).clamp_min(0) * (yy2 - yy1).clamp_min(0)
        iou = inter / (areas[cur] + areas[rest] - inter).clamp_min(1e-12)
        order = rest[iou <= iou_threshold]
    return keep


def detections(pred: torch.Tensor, width: int, height: int, conf_threshold: float,
               iou_threshold: float) -> torch.Tensor:
    """One image's [4+classes, anchors] prediction -> [n, 6] detections
    (x1, y1, x2, y2, score, class) in descending score order: best class by
    max/argmax (first maximum), score >= conf_threshold, corner boxes clamped to
    [0, width-1] x [0, height-1], NMS per class.  Restates the reference's
    detections() (demo/yolo_helpers.py:91-137)."""
    p = pred.to(torch.float32).t()
    boxes, scores = p[:, :4], p[:, 4:]
    conf, cls = scores.max(dim=1).values, scores.argmax(dim=1)
    keep = conf >= conf_threshold
    if not keep.any():
        return torch.zeros((0, 6))
    boxes, conf, cls = boxes[keep], conf[keep], cls[keep]
    cx, cy, w, h = boxes.unbind(1)
    conv = torch.stack(((cx - w / 2).clamp(0, width - 1), (cy - h / 2).clamp(0, height - 1),
                        (cx + w / 2).clamp(0, width - 1), (cy + h / 2).clamp(0, height - 1)), 1)
    selected = []
    for c in cls.unique(sorted=True).tolist():
        idx = torch.nonzero(cls == c, as_tuple=False).flatten()
        selected.extend(int(idx[k]) for k in _greedy_nms(conv[idx], conf[idx], iou_threshold))
    sel = torch.tensor(selected, dtype=torch.long)
    sel = sel[torch.sort(conf[sel], descending=True, stable=True).indices]
    return torch.cat((conv[sel], conf[sel, None], cls[sel, None].to(torch.float32)), 1)


def _resize_taps(dst: int, src: int, clamp_weight: bool):
    """Source offsets and 11-bit weights of OpenCV's bilinear 8-bit resize along
    one axis: f = float((d + 0.5) * scale - 0.5) with scale = 1 / (dst / src) in
    double, s = floor(f), f -= s; with clamp_weight (columns) s < 0 or s >= src-1
    clamp s with f = 0; weights round-half-even((1 - f) * 2048), (f * 2048)."""
    scale = 1.0 / (dst / src)
    s0 = np.zeros(dst, np.int64)
    w = np.zeros((dst, 2), np.int64)
    for d in range(dst):
        f = np.float32((d + 0.5) * scale - 0.5)
        s = int(np.floor(f))
        f = np.float32(f - np.float32(s))
        if clamp_weight and s < 0:
            f, s = np.float32(0.0), 0
        if clamp_weight and s >= src - 1:
            f, s = np.float32(0.0), src - 1
        s0[d] = s
        w[d, 0] = int(np.rint(np.float32(np.float32(1.0) - f) * np.float32(2048.0)))
        w[d, 1] = int(np.rint(f * np.float32(2048.0)))
    return s0, w


def resize_linear_u8(src: np.ndarray, out_h: int, out_w: int) -> np.ndarray:
    """cv2.resize(src, (out_w, out_h), interpolation=INTER_LINEAR) for uint8
    [H, W, C] images: OpenCV 4.x's fixed-point bilinear algorithm (the cv2 that
    demo/yolo_helpers.py:54 calls; restated, pinned against cv2 outputs by
    tests/golden/preprocess_vectors.npz).  Horizontal pass in integers, then
    rows combined as ((b0*(h0>>4))>>16) + ((b1*(h1>>4))>>16) + 2) >> 2."""
    h, w = src.shape[:2]
    xs, xw = _resize_taps(out_w, w, True)
    ys, yw = _resize_taps(out_h, h, False)
    s = src.astype(np.int64)
    x1 = np.minimum(xs + 1, w - 1)
    hor = s[:, xs] * xw[None, :, 0, None] + s[:, x1] * xw[None, :, 1, None]
    r0 = hor[np.clip(ys, 0, h - 1)]
    r1 = hor[np.clip(ys + 1, 0, h - 1)]
    b0, b1 = yw[:, 0][:, None, None], yw[:, 1][:, None, None]
    out = (((b0 * (r0 >> 4)) >> 16) + ((b1 * (r1 >> 4)) >> 16) + 2) >> 2
    return np.clip(out, 0, 255).astype(np.uint8)


def preprocess_frame(frame: np.ndarray, image_size: int) -> torch.Tensor:
    """uint8 BGR [H, W, 3] -> [1, 3, S, S] float32 RGB / 255: the reference's
    preprocess_frame (demo/yolo_helpers.py:53-56) with the resize restated."""
    rgb = resize_linear_u8(frame, image_size, image_size)[:, :, ::-1]
    return torch.from_numpy(np.ascontiguousarray(rgb)).permute(2, 0, 1).contiguous().to(torch.float32).div_(255.0).unsqueeze(0)
