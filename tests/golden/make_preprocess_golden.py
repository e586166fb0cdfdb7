"""Generate the golden vectors that pin the frame-preprocessing oracle.

Run where the reference checkout and cv2 are importable:

    REFERENCE_ROOT=/path/to/MatrixMan python tests/golden/make_preprocess_golden.py

For seeded uint8 BGR frames of several sizes it records the reference's own
preprocess_frame (demo/yolo_helpers.py:53-56: cv2.resize INTER_LINEAR, BGR ->
RGB, CHW, / 255) at several model sizes, stored as the uint8 resized RGB image
(the float result is exactly that / 255).

Output: tests/golden/preprocess_vectors.npz (frame_<case>, rgb_<case>, size_<case>).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

CASES = {
    # name: (height, width, image_size, seed)
    "down_wide": (90, 160, 64, 201),      # 16:9 downscale (non-integer in y)
    "up_small": (17, 29, 48, 202),        # upscale in both axes (border clamps)
    "mixed": (37, 53, 40, 203),           # up in y, down in x
    "square": (64, 64, 64, 204),          # identity size
    "odd": (101, 77, 96, 205),
}


def main() -> None:
    ref_root = os.environ.get("REFERENCE_ROOT")
    if not ref_root:
        raise SystemExit("set REFERENCE_ROOT to the reference checkout")
    sys.path.insert(0, ref_root)
    from demo import yolo_helpers as ref  # noqa: E402

    out = {}
    for name, (h, w, size, seed) in CASES.items():
        frame = np.random.default_rng(seed).integers(0, 256, size=(h, w, 3), dtype=np.uint8)
        t = ref.preprocess_frame(frame, size)                       # [1, 3, S, S] float32
        rgb = np.rint(t[0].permute(1, 2, 0).numpy() * 255.0).astype(np.uint8)
        assert np.array_equal(rgb.astype(np.float32) / np.float32(255.0), t[0].permute(1, 2, 0).numpy())
        out[f"frame_{name}"] = frame
        out[f"rgb_{name}"] = rgb
        out[f"size_{name}"] = np.array([size])
    np.savez_compressed(HERE / "preprocess_vectors.npz", **out)
    print("cases:", ", ".join(CASES))


if __name__ == "__main__":
    main()
