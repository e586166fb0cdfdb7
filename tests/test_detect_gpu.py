"""Detection postprocessing on the device against the CPU oracle (pinned to
the reference's detections() by tests/golden/detect_vectors.npz)."""

import numpy as np
import pytest
import torch

from oracle import ops as O
from oracle.tolerance import bit_exact

pytestmark = pytest.mark.gpu

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden" / "detect_vectors.npz"


def gen(seed):
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def as_tensor(dets):
    return torch.tensor([d[0] + [d[1], float(d[2])] for d in dets], dtype=torch.float32).reshape(-1, 6)


def test_detect_reduce_matches_oracle(mm):
    p = torch.rand(3, 24, 777, generator=gen(1)) * 4 - 2   # includes rows below -1
    p[1, 4:, 5] = -3.0                                      # no class above -1: score -1, class 0
    p[2, 7, 9] = p[2, 9, 9] = 5.0                           # tie: first maximum wins
    y = mm.gpu_postprocess_detection(mm.to_device(p)).cpu()
    assert bit_exact(y, O.detect_reduce(p))


def test_nms_matches_reference_vectors(mm):
    d = np.load(GOLDEN)
    for name in ("small", "many_classes", "tight_iou"):
        pred = torch.from_numpy(d[f"prediction_{name}"])
        width, height, conf, iou = d[f"params_{name}"].tolist()
        want = torch.from_numpy(d[f"detections_{name}"])
        batch = torch.cat((pred, pred), 0)
        got = mm.postprocess_detections(mm.to_device(batch), int(width), int(height), conf, iou,
                                        max_det=4096)
        assert len(got) == 2
        for g in got:
            assert bit_exact(as_tensor(g), want), name


def test_nms_strided_view_and_max_det(mm):
    d = np.load(GOLDEN)
    pred = torch.from_numpy(d["prediction_small"])
    width, height, conf, iou = d["params_small"].tolist()
    want = torch.from_numpy(d["detections_small"])
    # [B, anchors, 4+classes] on the device, viewed as [B, 4+classes, anchors]
    view = mm.to_device(pred.transpose(1, 2).contiguous()).transpose(1, 2)
    got = mm.postprocess_detections(view, int(width), int(height), conf, iou, max_det=10)
    assert bit_exact(as_tensor(got[0]), want[:10])


@pytest.mark.parametrize("max_det", [300, 20000])
def test_nms_beyond_shared_memory_capacity(mm, max_det):
    """Images with more candidates than the shared-memory NMS pass holds
    (12288) take the global-memory pass: same detections as the oracle, in the
    same order, bit for bit.  Image 0 has 20000 candidates over 3 classes with
    overlapping boxes and repeated scores; image 1 (about 7000 candidates,
    repeated scores too) stays on the shared-memory pass in the same call.
    Equal scores come out by class, then anchor, in both passes."""
    g = gen(2)
    a = 20000
    p = torch.empty(2, 7, a)
    p[:, 0:2] = torch.rand(2, 2, a, generator=g) * 1300 - 10
    p[:, 2:4] = torch.rand(2, 2, a, generator=g) * 120 + 4
    p[:, 4:] = torch.rand(2, 3, a, generator=g)
    p[0, 4:] = (p[0, 4:] * 64).floor() / 64 * 0.7 + 0.3  # every anchor a candidate, ties
    p[1, 4:] = (p[1, 4:] * 64).floor() / 64 * 0.35
    got = mm.postprocess_detections(mm.to_device(p), 1280, 1280, 0.3, 0.45, max_det=max_det)
    for i in range(2):
        want = O.detections(p[i], 1280, 1280, 0.3, 0.45)[:max_det]
        assert len(got[i]) == len(want)
        assert bit_exact(as_tensor(got[i]), want)


@pytest.mark.parametrize("batch,size", [(3, 256), (1, 640)])
def test_yolo_output_postprocessed_on_device(mm, batch, size):
    """The prepared YOLOv8n output, post-processed on the device, equals the
    oracle applied to the read-back output, image by image (at 640 x 640 the
    random-init model puts all 8400 anchors above the threshold)."""
    import workloads as W
    prepared = mm.prepare(W.yolov8_model("n"))
    with torch.no_grad():
        y = prepared(mm.to_device(W.yolo_input(batch, size=size)))
    got = mm.postprocess_detections(y, size, size, 0.3, 0.5, max_det=12288)
    host = y.cpu()
    assert len(got) == batch
    for i in range(batch):
        want = O.detections(host[i], size, size, 0.3, 0.5)
        assert bit_exact(as_tensor(got[i]), want)


def test_nms_workspace_contract(mm):
    """mm_detect_nms rejects a workspace that is too small or not 256-byte
    aligned (host-side checks, before any launch); max_det = 0 keeps nothing."""
    import ctypes
    from matrixman_b200 import _lib, ops
    pred = mm.to_device(torch.rand(2, 6, 500, generator=gen(3)))
    rt = pred.runtime
    need = ctypes.c_size_t(0)
    _lib.check(rt.lib.mm_detect_nms_workspace_size(2, 500, ctypes.byref(need)))
    work = rt.new_storage(need.value + 256, torch.uint8)
    counts = rt.new_storage(2, torch.int32)

    def call(max_det, ptr, nbytes):
        dets = ops.empty(rt, (2, max_det, 6))
        return rt.lib.mm_detect_nms(ops._p(pred.desc()), 0.25, 0.45, 640.0, 640.0, max_det,
                                    ops._p(dets.desc()), ctypes.c_void_p(counts.pointer),
                                    ctypes.c_void_p(ptr), nbytes, rt.stream)

    assert call(5, work.pointer, need.value - 1) == _lib.MM_ERR_INVALID
    assert call(5, work.pointer + 16, need.value) == _lib.MM_ERR_INVALID
    assert call(0, work.pointer, need.value) == _lib.MM_OK
    host = torch.full((2,), -7, dtype=torch.int32)
    rt.download(counts.pointer, host)
    assert host.tolist() == [0, 0]
