"""Generate the golden vectors that pin the detection-postprocessing oracle.

Run where the reference checkout is importable:

    REFERENCE_ROOT=/path/to/MatrixMan python tests/golden/make_detect_golden.py

It imports the reference's host-side helpers (demo/yolo_helpers.py) and records,
for seeded [1, 4+classes, anchors] predictions with clustered boxes (so that
NMS suppresses) and distinct scores:

* the output of the reference's detections() (demo/yolo_helpers.py:91-137):
  corner boxes, scores and classes of the kept detections in order;
* a consistency check, asserted here: the reference's reduced_detections()
  (demo/yolo_helpers.py:140-161) applied to oracle.ops.detect_reduce of the
  same prediction gives the same detections -- the reduction the reference
  computes in its shader feeds its own decoder unchanged.

Output: tests/golden/detect_vectors.npz (prediction_<case>, detections_<case>,
and the width, height and thresholds of each case).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

CASES = {
    # name: (anchors, classes, width, height, conf, iou, seed)
    "small": (600, 3, 320, 256, 0.30, 0.45, 101),
    "many_classes": (2100, 20, 640, 640, 0.25, 0.50, 102),
    "tight_iou": (900, 4, 640, 480, 0.20, 0.10, 103),
}


def make_prediction(anchors: int, classes: int, width: int, height: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    centers = torch.rand(12, 2, generator=g) * torch.tensor([width, height])
    which = torch.randint(0, 12, (anchors,), generator=g)
    cxcy = centers[which] + torch.randn(anchors, 2, generator=g) * 12
    wh = 20 + torch.rand(anchors, 2, generator=g) * 80
    scores = torch.rand(anchors, classes, generator=g) * 0.3
    boost = torch.rand(anchors, generator=g) < 0.3
    scores[boost, torch.randint(0, classes, (int(boost.sum()),), generator=g)] += 0.6
    pred = torch.cat((cxcy, wh, scores), 1).t().contiguous()[None]
    return pred.to(torch.float32)


def main() -> None:
    ref_root = os.environ.get("REFERENCE_ROOT")
    if not ref_root:
        raise SystemExit("set REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, ref_root)
    from demo import yolo_helpers as ref  # noqa: E402

    from oracle import ops as O

    out = {}
    for name, (anchors, classes, width, height, conf, iou, seed) in CASES.items():
        pred = make_prediction(anchors, classes, width, height, seed)
        dets, _ = ref.detections(pred, width, height, {}, conf, iou)
        reduced, _ = ref.reduced_detections(O.detect_reduce(pred), width, height, {}, conf, iou)
        assert [(d[0], d[1], d[2]) for d in dets] == [(d[0], d[1], d[2]) for d in reduced], name
        arr = np.array([list(d[0]) + [d[1], float(d[2])] for d in dets], dtype=np.float32).reshape(-1, 6)
        out[f"prediction_{name}"] = pred.numpy()
        out[f"detections_{name}"] = arr
        out[f"params_{name}"] = np.array([width, height, conf, iou], dtype=np.float64)
        print(f"{name}: {arr.shape[0]} detections")
    np.savez_compressed(HERE / "detect_vectors.npz", **out)


if __name__ == "__main__":
    main()
