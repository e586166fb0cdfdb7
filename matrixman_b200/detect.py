"""Detection postprocessing on the device.

``reduce_detection_output`` is the reference's GPU reduction
(``backends/opengl/ops/postprocessing.py:87-119``, public as
``matrixman.gpu_postprocess_detection``, ``backend.py:263-266``): a
``[B, 4+classes, anchors]`` prediction becomes ``[B, 6, anchors]`` =
(cx, cy, w, h, best score, best class) on the device.  The reference takes
B = 1 only; here any batch works.

``postprocess_detections`` goes further: confidence filter, box conversion and
per-class NMS run on the device too (the reference runs them on the CPU,
``demo/yolo_helpers.py:91-161``), so only the kept detections cross PCIe --
``max_det`` x 24 bytes per image instead of the 2.82 MB raw prediction.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib, audit, ops, runtime
from .tensor import MatrixManTensor

# Candidates per image the shared-memory NMS pass holds
# (MM_DETECT_MAX_CANDIDATES in include/matrixman_b200.h); images with more take
# a global-memory pass, so this is a speed boundary, not a limit.
MAX_CANDIDATES = 12288


def _check_prediction(pred) -> tuple[int, int, int]:
    if not isinstance(pred, MatrixManTensor):
        raise TypeError("MatrixMan: detection postprocessing needs a MatrixMan tensor")
    if pred.dtype != torch.float32:
        raise TypeError("MatrixMan: detection postprocessing supports float32 predictions only")
    shape = tuple(int(v) for v in pred.shape)
    if len(shape) != 3 or shape[1] < 5:
        raise ValueError("MatrixMan: detection prediction must be [B, 4+classes, anchors]")
    return shape


def reduce_detection_output(pred: MatrixManTensor) -> MatrixManTensor:
    """[B, 4+classes, anchors] -> [B, 6, anchors]: box, best score, best class
    (the score starts at -1; a class replaces it only when strictly greater)."""
    b, _, a = _check_prediction(pred)
    out = ops.empty(pred.runtime, (b, 6, a))
    ops._launch("mm_detect_reduce", ops._p(pred.desc()), ops._p(out.desc()), pred.runtime.stream)
    return out


def postprocess_detections(pred: MatrixManTensor, width: int, height: int,
                           conf_threshold: float = 0.25, iou_threshold: float = 0.45,
                           names: dict | None = None, max_det: int = 300) -> list[list[tuple]]:
    """Per image of ``pred`` ([B, 4+classes, anchors], cx/cy/w/h boxes then
    class scores): the detections the reference's ``detections()`` returns --
    ``(box [x1, y1, x2, y2], score, class, name)`` in descending score order --
    computed on the device.  Candidates are anchors whose best class score is
    >= ``conf_threshold``; boxes are clamped to [0, width-1] x [0, height-1];
    NMS is per class with IoU > ``iou_threshold`` suppressing.  At most
    ``max_det`` detections per image are returned; the number of candidates
    is not limited."""
    b, _, _ = _check_prediction(pred)
    if max_det <= 0:
        raise ValueError("MatrixMan: max_det must be positive")
    rt = pred.runtime
    # One block holds the detections and, after them, the per-image counts
    # (int32), so a single copy reads both back.
    n_det = b * int(max_det) * 6
    block = rt.new_storage(n_det + max(b, 1), torch.float32)
    dets = MatrixManTensor._from_owner(block, (b, int(max_det), 6), 0, (int(max_det) * 6, 6, 1))
    ws_bytes = ctypes.c_size_t(0)
    _lib.check(rt.lib.mm_detect_nms_workspace_size(b, int(pred.shape[2]), ctypes.byref(ws_bytes)),
               "detection workspace size")
    work = rt.new_storage(max(ws_bytes.value, 1), torch.uint8)
    ops._launch("mm_detect_nms", ops._p(pred.desc()), float(conf_threshold), float(iou_threshold),
                float(width), float(height), int(max_det), ops._p(dets.desc()),
                ctypes.c_void_p(block.pointer + n_det * 4), ctypes.c_void_p(work.pointer), ws_bytes.value,
                rt.stream)
    flat = torch.empty(n_det + b, dtype=torch.float32)
    if b:
        rt.download(block.pointer, flat)
    audit.record("explicit_readback", flat)
    host_counts = flat[n_det:].view(torch.int32).tolist()
    host = flat[:n_det].view(b, int(max_det), 6)
    names = names or {}
    result = []
    for i in range(b):
        n = host_counts[i]
        if n < 0 or n > max_det:
            raise RuntimeError(f"MatrixMan: detection count {n} of image {i} is out of range")
        result.append([(row[:4], row[4], int(row[5]), names.get(int(row[5]), str(int(row[5]))))
                       for row in host[i, :n].tolist()])
    return result
