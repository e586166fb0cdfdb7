"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a container where the reference checkout is importable:

    REFERENCE_ROOT=/path/to/MatrixMan python tests/golden/make_golden.py

It imports the reference package ``drivers.matrixman`` (CPU-only parts; its
device backends are never initialised) and records the outputs of the
reference's own host-side functions on the reference's own test inputs:

* ``reference_conv2d`` loop nest (drivers/matrixman/backends/cuda/conv2d.py:13-46)
  on its arange known-answer case (conv2d.py:49-57) and grouped multiplier-2
  case (conv2d.py:88-103);
* ``nearest_reference`` (backends/cuda/upsample.py:9-14) on its exact-2x,
  non-integer and multi-channel cases (upsample.py:44-58);
* the BatchNorm known answer (backends/cuda/batch_norm.py:9-22) and the SiLU
  known answer (backends/cuda/silu.py:9-11), evaluated with the formulas
  those files state;
* ``_fold_pair`` (preparation.py:360-398) on the toy Conv+BN module of
  diagnostics/cuda_prepare_diagnostic.py:13-24 (seed 7, with and without bias);
* the view-metadata helpers ``infer_view_shape`` / ``expand_shape_strides`` /
  ``unsqueeze_shape_strides`` (tensor.py:161-268) on a table of cases;
* torch-CPU expectations for the conv demo cases
  (diagnostics/matrixman_conv_demo.py:48-103, seeds 1000+C+K+10s+p), the DFL
  softmax demo (diagnostics/matrixman_softmax_demo.py:12-27, seed 20260829) and
  the max-pool cases of diagnostics/cuda_maxpool_diagnostic.py (seeded here,
  the reference leaves them unseeded).

Outputs: tests/golden/reference_vectors.npz and tests/golden/metadata_cases.json.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

HERE = Path(__file__).resolve().parent


def main() -> int:
    root = os.environ.get("REFERENCE_ROOT")
    if not root or not Path(root, "drivers", "matrixman").is_dir():
        print("set REFERENCE_ROOT to the MatrixMan checkout", file=sys.stderr)
        return 2
    sys.path.insert(0, root)
    import importlib
    ref_tensor = importlib.import_module("drivers.matrixman.tensor")
    from drivers.matrixman.backends.cuda.conv2d import reference_conv2d
    from drivers.matrixman.backends.cuda.upsample import nearest_reference
    from drivers.matrixman.preparation import PreparationReport, _fold_pair, _module_alias_counts

    out: dict[str, np.ndarray] = {}

    # conv known answers (conv2d.py:49-57, 88-103)
    x = np.arange(1, 1 + 2 * 4 * 5, dtype=np.float32).reshape(1, 2, 4, 5)
    w = np.arange(1, 1 + 3 * 2 * 3 * 2, dtype=np.float32).reshape(3, 2, 3, 2) / 10
    b = np.array([0.5, -1.0, 2.0], dtype=np.float32)
    out["conv_arange_x"], out["conv_arange_w"], out["conv_arange_b"] = x, w, b
    out["conv_arange_y"] = reference_conv2d(x, w, b)
    xg = np.empty((1, 8, 16, 16), dtype=np.float32)
    for ch in range(8):
        xg[0, ch] = ch * 100.0 + np.arange(256, dtype=np.float32).reshape(16, 16)
    wg = np.empty((16, 1, 3, 3), dtype=np.float32)
    for oc in range(16):
        wg[oc, 0] = (oc + 1) * np.arange(1, 10, dtype=np.float32).reshape(3, 3) / 10.0
    out["conv_grouped_x"], out["conv_grouped_w"] = xg, wg
    out["conv_grouped_y"] = reference_conv2d(xg, wg, None, stride=(2, 2), padding=(1, 1), groups=8)

    # conv demo cases (matrixman_conv_demo.py:48-103)
    demo = [((1, 3, 320, 320), (4, 3, 3, 3), 2, 1, False), ((1, 4, 320, 320), (5, 4, 3, 3), 1, 1, False),
            ((1, 4, 320, 320), (6, 4, 1, 1), 1, 0, False), ((1, 4, 320, 320), (6, 4, 1, 1), 1, 0, True)]
    for i, (shape, wshape, s, p, has_b) in enumerate(demo):
        torch.manual_seed(1000 + shape[1] + wshape[0] + s * 10 + p)
        xc = torch.randn(shape) * 0.25
        wc = torch.randn(wshape) * 0.25
        bc = torch.randn((wshape[0],)) * 0.1 if has_b else None
        # Inputs are regenerated from the seed by the tests; the fixture keeps
        # their SHA-256 and a fixed sample of the expected output.
        yc = F.conv2d(xc, wc, bc, stride=s, padding=p).numpy()
        idx = np.random.RandomState(i).choice(yc.size, 4096, replace=False)
        out[f"conv_demo{i}_x_sha256"] = np.frombuffer(
            hashlib.sha256(xc.numpy().tobytes()).digest(), dtype=np.uint8)
        out[f"conv_demo{i}_w"] = wc.numpy()
        if bc is not None:
            out[f"conv_demo{i}_b"] = bc.numpy()
        out[f"conv_demo{i}_y_idx"] = idx.astype(np.int64)
        out[f"conv_demo{i}_y_val"] = yc.reshape(-1)[idx]
        out[f"conv_demo{i}_geom"] = np.array([s, p], dtype=np.int64)

    # nearest (upsample.py:44-58)
    ex = np.arange(1, 13, dtype=np.float32).reshape(1, 2, 2, 3)
    ni = np.arange(1, 13, dtype=np.float32).reshape(1, 1, 3, 4)
    mc = np.empty((1, 24, 4, 4), dtype=np.float32)
    for ch in range(24):
        mc[0, ch] = ch * 1000.0 + np.arange(16, dtype=np.float32).reshape(4, 4)
    out["nearest_exact_x"], out["nearest_exact_y"] = ex, nearest_reference(ex, 4, 6)
    out["nearest_nonint_x"], out["nearest_nonint_y"] = ni, nearest_reference(ni, 5, 7)
    out["nearest_multi_x"], out["nearest_multi_y"] = mc, nearest_reference(mc, 8, 8)

    # BatchNorm / SiLU known answers (batch_norm.py:9-22, silu.py:9-11)
    bx = np.arange(1, 25, dtype=np.float32).reshape(1, 3, 2, 4)
    mean = np.array([2.0, 8.0, 20.0], dtype=np.float32)
    var = np.array([1.0, 4.0, 9.0], dtype=np.float32)
    gam = np.array([1.0, 0.5, 2.0], dtype=np.float32)
    bet = np.array([0.0, -1.0, 3.0], dtype=np.float32)
    out["bn_x"], out["bn_mean"], out["bn_var"], out["bn_w"], out["bn_b"] = bx, mean, var, gam, bet
    out["bn_y"] = ((bx - mean.reshape(1, 3, 1, 1)) / np.sqrt(var.reshape(1, 3, 1, 1) + 1e-5)
                   * gam.reshape(1, 3, 1, 1) + bet.reshape(1, 3, 1, 1)).astype(np.float32)
    sv = np.array([-8.0, -2.0, -0.5, 0.0, 0.5, 2.0, 8.0], dtype=np.float32)
    out["silu_x"], out["silu_y"] = sv, (sv / (1.0 + np.exp(-sv))).astype(np.float32)

    # DFL softmax demo (matrixman_softmax_demo.py:12-27)
    torch.manual_seed(20260829)
    base = torch.randn((1, 4, 16, 84))
    out["dfl_softmax_x"] = base.numpy()
    out["dfl_softmax_y"] = torch.softmax(base.transpose(1, 2), dim=1).contiguous().numpy()

    # max-pool cases (cuda_maxpool_diagnostic.py), seeded here
    g = torch.Generator().manual_seed(4242)
    cases = {
        "random_128x20x20": torch.randn(1, 128, 20, 20, generator=g),
        "random_small": torch.randn(1, 3, 7, 9, generator=g),
        "all_negative": -torch.rand(1, 4, 6, 8, generator=g),
        "padding_edge": torch.tensor([[[[-9.0, -8.0], [-7.0, -6.0]]]]),
    }
    for name, src in cases.items():
        out[f"maxpool_{name}_x"] = src.numpy()
        out[f"maxpool_{name}_y"] = F.max_pool2d(src, 5, 1, 2).numpy()

    # _fold_pair on the prepare diagnostic's toy module (seed 7)
    class Conv(nn.Module):
        def __init__(self, bias):
            super().__init__()
            self.conv = nn.Conv2d(3, 4, 3, padding=1, bias=bias)
            self.bn = nn.BatchNorm2d(4)
            self.act = nn.SiLU()

        def forward(self, t):
            return self.act(self.bn(self.conv(t)))

    torch.manual_seed(7)
    for has_bias in (False, True):
        m = Conv(has_bias).eval()
        with torch.no_grad():
            m.bn.running_mean.copy_(torch.randn(4) * 0.1)
            m.bn.running_var.copy_(torch.rand(4) + 0.5)
            m.bn.weight.copy_(torch.rand(4) + 0.5)
            m.bn.bias.copy_(torch.randn(4) * 0.1)
        key = f"fold_bias{int(has_bias)}"
        out[key + "_w"] = m.conv.weight.detach().numpy().copy()
        if has_bias:
            out[key + "_b"] = m.conv.bias.detach().numpy().copy()
        out[key + "_mean"] = m.bn.running_mean.numpy().copy()
        out[key + "_var"] = m.bn.running_var.numpy().copy()
        out[key + "_gamma"] = m.bn.weight.detach().numpy().copy()
        out[key + "_beta"] = m.bn.bias.detach().numpy().copy()
        out[key + "_eps"] = np.array([m.bn.eps], dtype=np.float64)
        report = PreparationReport()
        _fold_pair(m, report, _module_alias_counts(m))
        assert report.folded == 1
        out[key + "_w_folded"] = m.conv.weight.detach().numpy().copy()
        out[key + "_b_folded"] = m.conv.bias.detach().numpy().copy()

    np.savez_compressed(HERE / "reference_vectors.npz", **out)

    # view-metadata helpers (tensor.py:161-268)
    meta = {"infer_view_shape": [], "expand_shape_strides": [], "unsqueeze_shape_strides": []}
    for shape, req in [((2, 3, 4), (6, 4)), ((2, 3, 4), (-1,)), ((2, 3, 4), (2, -1)), ((1, 144, 8400), (1, 4, 16, -1)),
                       ((5,), (5, 1)), ((2, 3, 4), (4, -1, 3))]:
        meta["infer_view_shape"].append({"shape": shape, "request": req,
                                         "result": list(ref_tensor.infer_view_shape(shape, req))})
    for shape, strides, req in [((3, 1), (1, 1), (3, 4)), ((1, 4), (4, 1), (2, 3, 4)), ((2, 1, 5), (5, 5, 1), (2, 7, 5)),
                                ((4,), (1,), (-1,)), ((1,), (1,), (2, 3, 1))]:
        s, st = ref_tensor.expand_shape_strides(shape, strides, req)
        meta["expand_shape_strides"].append({"shape": shape, "strides": strides, "request": req,
                                             "result": [list(s), list(st)]})
    for shape, strides, dim in [((2, 3), (3, 1), 0), ((2, 3), (3, 1), 2), ((2, 3), (3, 1), -1), ((4, 5, 6), (30, 6, 1), 1)]:
        s, st = ref_tensor.unsqueeze_shape_strides(shape, strides, dim)
        meta["unsqueeze_shape_strides"].append({"shape": shape, "strides": strides, "dim": dim,
                                                "result": [list(s), list(st)]})
    (HERE / "metadata_cases.json").write_text(json.dumps(meta, indent=1))
    print(f"wrote {len(out)} arrays to {HERE / 'reference_vectors.npz'}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
