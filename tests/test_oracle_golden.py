"""The CPU oracle reproduces every golden vector recorded from the reference."""

import hashlib
import json

import numpy as np
import torch

from oracle import ops as O
from oracle.tolerance import bit_exact, max_rel_err

from .conftest import GOLDEN


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def test_conv_arange_known_answer(golden):
    g = golden
    y = O.conv2d(t(g["conv_arange_x"]), t(g["conv_arange_w"]), t(g["conv_arange_b"]), 1, 1)
    assert tuple(y.shape) == (1, 3, 4, 6)  # geometry asserted by the reference (conv2d.py:53-57)
    assert max_rel_err(y, t(g["conv_arange_y"])) < 1e-6
    loops = O.conv2d_loops(g["conv_arange_x"], g["conv_arange_w"], g["conv_arange_b"], (1, 1), (1, 1))
    assert np.array_equal(loops, g["conv_arange_y"])


def test_conv_grouped_known_answer(golden):
    g = golden
    y = O.conv2d(t(g["conv_grouped_x"]), t(g["conv_grouped_w"]), None, 2, 1, 1, 8)
    assert max_rel_err(y, t(g["conv_grouped_y"])) < 1e-6
    loops = O.conv2d_loops(g["conv_grouped_x"], g["conv_grouped_w"], None, (2, 2), (1, 1), (1, 1), 8)
    assert np.array_equal(loops, g["conv_grouped_y"])


def demo_inputs(i, golden):
    shapes = [((1, 3, 320, 320), (4, 3, 3, 3), 2, 1, False), ((1, 4, 320, 320), (5, 4, 3, 3), 1, 1, False),
              ((1, 4, 320, 320), (6, 4, 1, 1), 1, 0, False), ((1, 4, 320, 320), (6, 4, 1, 1), 1, 0, True)]
    shape, wshape, s, p, has_b = shapes[i]
    torch.manual_seed(1000 + shape[1] + wshape[0] + s * 10 + p)
    x = torch.randn(shape) * 0.25
    w = torch.randn(wshape) * 0.25
    b = torch.randn((wshape[0],)) * 0.1 if has_b else None
    digest = hashlib.sha256(x.numpy().tobytes()).digest()
    assert digest == golden[f"conv_demo{i}_x_sha256"].tobytes(), "seeded regeneration drifted"
    return x, w, b, s, p


def test_conv_demo_cases(golden):
    for i in range(4):
        x, w, b, s, p = demo_inputs(i, golden)
        assert torch.equal(w, t(golden[f"conv_demo{i}_w"]))
        y = O.conv2d(x, w, b, s, p).reshape(-1)
        idx = t(golden[f"conv_demo{i}_y_idx"])
        assert max_rel_err(y[idx], t(golden[f"conv_demo{i}_y_val"])) < 1e-6


def test_nearest_reference_cases(golden):
    for name, size in (("exact", (4, 6)), ("nonint", (5, 7)), ("multi", (8, 8))):
        x = golden[f"nearest_{name}_x"]
        expected = golden[f"nearest_{name}_y"]
        assert np.array_equal(O.nearest_reference(x, *size), expected)
        if name != "nonint":
            # torch's rule coincides with the integer rule for integer ratios
            assert bit_exact(O.upsample_nearest(t(x), size=size), t(expected))


def test_batch_norm_known_answer(golden):
    g = golden
    y = O.batch_norm_eval(t(g["bn_x"]), t(g["bn_mean"]), t(g["bn_var"]), t(g["bn_w"]), t(g["bn_b"]), 1e-5)
    assert max_rel_err(y, t(g["bn_y"])) < 1e-6


def test_silu_known_answer(golden):
    from oracle.tolerance import max_ulp
    y = O.silu(t(golden["silu_x"]))
    assert max_ulp(y, t(golden["silu_y"])) <= 2


def test_dfl_softmax_demo(golden):
    x = t(golden["dfl_softmax_x"])
    y = O.softmax(x.transpose(1, 2), 1)
    assert bit_exact(y.contiguous(), t(golden["dfl_softmax_y"]))


def test_maxpool_cases(golden):
    for name in ("random_128x20x20", "random_small", "all_negative", "padding_edge"):
        y = O.max_pool2d(t(golden[f"maxpool_{name}_x"]), 5, 1, 2)
        assert bit_exact(y, t(golden[f"maxpool_{name}_y"]))
        y1, _, _ = O.sppf_chain(t(golden[f"maxpool_{name}_x"]))
        assert bit_exact(y1, t(golden[f"maxpool_{name}_y"]))


def test_fold_matches_reference_fold_pair(golden):
    from matrixman_b200.preparation import fold_conv_bn
    from torch import nn
    for has_bias in (0, 1):
        k = f"fold_bias{has_bias}"
        conv = nn.Conv2d(3, 4, 3, padding=1, bias=bool(has_bias))
        bn = nn.BatchNorm2d(4, eps=float(golden[k + "_eps"][0]))
        with torch.no_grad():
            conv.weight.copy_(t(golden[k + "_w"]))
            if has_bias:
                conv.bias.copy_(t(golden[k + "_b"]))
            bn.running_mean.copy_(t(golden[k + "_mean"]))
            bn.running_var.copy_(t(golden[k + "_var"]))
            bn.weight.copy_(t(golden[k + "_gamma"]))
            bn.bias.copy_(t(golden[k + "_beta"]))
        w, b = fold_conv_bn(conv, bn.eval())
        assert bit_exact(w, t(golden[k + "_w_folded"]))
        assert bit_exact(b, t(golden[k + "_b_folded"]))
        wo, bo = O.fold_conv_bn(conv.weight.detach(), conv.bias.detach() if has_bias else torch.zeros(4),
                                bn.running_mean, bn.running_var, bn.weight.detach(), bn.bias.detach(), bn.eps)
        assert bit_exact(wo, t(golden[k + "_w_folded"]))
        assert bit_exact(bo, t(golden[k + "_b_folded"]))


def test_metadata_helpers_match_reference():
    import importlib
    T = importlib.import_module("matrixman_b200.tensor")
    cases = json.loads((GOLDEN / "metadata_cases.json").read_text())
    for c in cases["infer_view_shape"]:
        assert list(T.infer_view_shape(c["shape"], c["request"])) == c["result"]
    for c in cases["expand_shape_strides"]:
        s, st = T.expand_shape_strides(c["shape"], c["strides"], c["request"])
        assert [list(s), list(st)] == c["result"]
    for c in cases["unsqueeze_shape_strides"]:
        s, st = T.unsqueeze_shape_strides(c["shape"], c["strides"], c["dim"])
        assert [list(s), list(st)] == c["result"]


DETECT_CASES = ("small", "many_classes", "tight_iou")


def test_detections_oracle_matches_reference_vectors():
    """oracle.detections reproduces the reference's detections() output
    (tests/golden/make_detect_golden.py) exactly: boxes, scores, classes, order."""
    d = np.load(GOLDEN / "detect_vectors.npz")
    for name in DETECT_CASES:
        pred = torch.from_numpy(d[f"prediction_{name}"])
        width, height, conf, iou = d[f"params_{name}"].tolist()
        got = O.detections(pred[0], int(width), int(height), conf, iou)
        want = torch.from_numpy(d[f"detections_{name}"])
        assert got.shape == want.shape, name
        assert bit_exact(got, want), name


def test_detect_reduce_oracle_semantics():
    """First maximum wins; the score starts at -1 (all-below -1 keeps class 0, score -1)."""
    p = torch.tensor([[[1.0], [2.0], [3.0], [4.0], [0.5], [0.7], [0.7], [0.1]]])
    r = O.detect_reduce(p)
    assert r[0, :, 0].tolist() == [1.0, 2.0, 3.0, 4.0, 0.699999988079071, 1.0]
    q = torch.tensor([[[0.0], [0.0], [1.0], [1.0], [-3.0], [-2.0]]])
    assert O.detect_reduce(q)[0, 4:, 0].tolist() == [-1.0, 0.0]


def test_preprocess_oracle_matches_reference_vectors():
    """oracle.preprocess_frame reproduces the reference's preprocess_frame
    (cv2 INTER_LINEAR resize, BGR -> RGB, / 255) bit for bit."""
    d = np.load(GOLDEN / "preprocess_vectors.npz")
    for name in ("down_wide", "up_small", "mixed", "square", "odd"):
        size = int(d[f"size_{name}"][0])
        got = O.preprocess_frame(d[f"frame_{name}"], size)
        want = torch.from_numpy(d[f"rgb_{name}"]).permute(2, 0, 1).to(torch.float32).div_(255.0)[None]
        assert bit_exact(got, want), name
