"""mm_detect_nms_static: the detection NMS entry point that allocates no device
memory, for callers that are not allowed to (a plugin inside an application
that owns all GPU memory, a real-time loop whose memory is fixed up front).

It is checked through the C-ABI against mm_detect_nms with a caller-provided
workspace, bit for bit, on two calls in a row: the static scratch keeps the
first call's contents, so the second call (fewer candidates) would show any
state that leaks between calls.  This file is collected last so that a run
stopping at its first failure has run every other test already.
"""

import ctypes

import numpy as np
import pytest
import torch

from matrixman_b200 import _lib, ops
from oracle.tolerance import bit_exact

pytestmark = pytest.mark.gpu

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden" / "detect_vectors.npz"


def _nms(rt, pred, conf, iou, width, height, max_det, static):
    """One C-ABI call; returns (dets of the kept rows per image, counts)."""
    b = int(pred.shape[0])
    dets = ops.empty(rt, (b, max_det, 6))
    counts = rt.new_storage(b, torch.int32)
    args = [ops._p(pred.desc()), conf, iou, float(width), float(height), max_det, ops._p(dets.desc()),
            ctypes.c_void_p(counts.pointer)]
    work = None
    if static:
        status = rt.lib.mm_detect_nms_static(*args, rt.stream)
    else:
        nbytes = ctypes.c_size_t(0)
        _lib.check(rt.lib.mm_detect_nms_workspace_size(b, int(pred.shape[2]), ctypes.byref(nbytes)))
        work = rt.new_storage(nbytes.value, torch.uint8)
        status = rt.lib.mm_detect_nms(*args, ctypes.c_void_p(work.pointer), nbytes.value, rt.stream)
    _lib.check(status, "mm_detect_nms_static" if static else "mm_detect_nms")
    host_counts = torch.empty(b, dtype=torch.int32)
    rt.download(counts.pointer, host_counts)
    host = dets.cpu()  # synchronises: the workspace is released only after this
    del work
    return [host[i, :max(int(host_counts[i]), 0)] for i in range(b)], host_counts


def _inputs(mm):
    g = torch.Generator()
    g.manual_seed(7)
    big = torch.rand(2, 84, 8400, generator=g)       # every anchor is a candidate at 0.25
    big[:, :4] *= 640.0
    d = np.load(GOLDEN)
    small = torch.from_numpy(d["prediction_small"]).repeat(3, 1, 1)
    w, h, conf, iou = d["params_small"].tolist()
    return [(mm.to_device(big), 0.25, 0.45, 640, 640, 300),
            (mm.to_device(small), conf, iou, int(w), int(h), 100)]


def test_static_scratch_matches_workspace_entry_point(mm):
    for pred, conf, iou, w, h, max_det in _inputs(mm):  # two calls in a row on the static scratch
        rt = pred.runtime
        got, got_counts = _nms(rt, pred, conf, iou, w, h, max_det, static=True)
        want, want_counts = _nms(rt, pred, conf, iou, w, h, max_det, static=False)
        assert torch.equal(got_counts, want_counts)
        assert int(got_counts.min()) > 0
        for g_rows, w_rows in zip(got, want):
            assert bit_exact(g_rows, w_rows)


def test_static_scratch_rejects_batches_above_its_size(mm):
    pred = mm.to_device(torch.zeros(11, 84, 8400))     # 11 images of 640 x 640 need > 4 MiB
    with pytest.raises(NotImplementedError, match="scratch"):
        _nms(pred.runtime, pred, 0.25, 0.45, 640, 640, 10, static=True)
