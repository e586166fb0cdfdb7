"""Frame preprocessing on the device against the CPU oracle (pinned to the
reference's preprocess_frame by tests/golden/preprocess_vectors.npz)."""

import numpy as np
import pytest
import torch

from oracle import ops as O
from oracle.tolerance import bit_exact

pytestmark = pytest.mark.gpu

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden" / "preprocess_vectors.npz"


def test_preprocess_matches_reference_vectors(mm):
    d = np.load(GOLDEN)
    for name in ("down_wide", "up_small", "mixed", "square", "odd"):
        size = int(d[f"size_{name}"][0])
        got = mm.preprocess_frames(d[f"frame_{name}"], size).cpu()
        assert bit_exact(got, O.preprocess_frame(d[f"frame_{name}"], size)), name


def test_preprocess_batch_of_hd_frames(mm):
    rng = np.random.default_rng(7)
    frames = rng.integers(0, 256, size=(2, 1080, 1920, 3), dtype=np.uint8)
    pinned = mm.pinned_empty((1080, 1920, 3), dtype=torch.uint8)
    got = mm.preprocess_frames(frames, 640).cpu()
    assert got.shape == (2, 3, 640, 640)
    for i in range(2):
        assert bit_exact(got[i:i + 1], O.preprocess_frame(frames[i], 640))
    pinned.copy_(torch.from_numpy(frames[1]))   # page-locked source: asynchronous upload
    y = mm.preprocess_frames(pinned, 640).cpu()
    assert bit_exact(y, O.preprocess_frame(frames[1], 640))


def test_preprocess_rectangular_size_and_errors(mm):
    frame = np.random.default_rng(8).integers(0, 256, size=(50, 70, 3), dtype=np.uint8)
    got = mm.preprocess_frames(torch.from_numpy(frame), (32, 48)).cpu()
    want = torch.from_numpy(np.ascontiguousarray(O.resize_linear_u8(frame, 32, 48)[:, :, ::-1])) \
        .permute(2, 0, 1).to(torch.float32).div_(255.0)[None]
    assert bit_exact(got, want)
    with pytest.raises(TypeError):
        mm.preprocess_frames(frame.astype(np.float32), 32)
    with pytest.raises(ValueError):
        mm.preprocess_frames(frame[:, :, :2], 32)
