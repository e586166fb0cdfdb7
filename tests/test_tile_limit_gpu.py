"""Convolutions split into output regions (the CUDA mapping of tileLimit)
give the same result as one launch, bit for bit: the region entry points read
the input the whole convolution would read and accumulate every output pixel
in the same order.  Tensor-core, SIMT and stem paths, with and without a
residual, and a prepared model in a fresh process under MATRIXMAN_TILE_LIMIT."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch
import torch.nn.functional as F
from torch import nn

from matrixman_b200 import ops
from matrixman_b200.preparation import PreparedConv2d
from oracle import ops as O
from oracle.tolerance import CONV_GEMM_REL, bit_exact, max_rel_err

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def gen(seed):
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def nhwc(mm, t):
    return mm.to_device(t.permute(0, 2, 3, 1).contiguous()).permute(0, 3, 1, 2)


def _conv(c, k, ksz, stride, seed):
    g = gen(seed)
    conv = nn.Conv2d(c, k, ksz, stride, ksz // 2)
    with torch.no_grad():
        conv.weight.copy_(torch.randn(conv.weight.shape, generator=g) / (c * ksz * ksz) ** 0.5)
        conv.bias.copy_(torch.randn(k, generator=g) * 0.1)
    return conv


@pytest.mark.parametrize("c,k,ksz,stride,h,w,cap,residual", [
    (64, 48, 3, 1, 37, 45, 16, False),   # rectangle tiles, ragged regions
    (32, 32, 3, 2, 40, 41, 7, False),    # stride 2, odd cap
    (64, 64, 1, 1, 33, 33, 10, True),    # 1x1: regions leave the flat TMA mode; residual
    (16, 80, 3, 1, 20, 24, 9, True),     # 16 channels, wide N tile, residual
])
def test_tc_regions_equal_one_launch(mm, c, k, ksz, stride, h, w, cap, residual):
    conv = _conv(c, k, ksz, stride, c + k + h)
    unit = PreparedConv2d(conv, 2)
    x = torch.rand(2, c, h, w, generator=gen(h * w)) * 2 - 1
    xd = nhwc(mm, x)
    rt = xd.runtime
    wv, b, tc = unit.device_weights(rt)
    hi, lo, c_pad, k_pad = tc
    oh, ow = ops.conv_output_hw(h, w, ksz, ksz, unit.stride, unit.padding, unit.dilation)
    shape = (2, k, oh, ow)
    res = None
    if residual:
        res = nhwc(mm, torch.randn(shape, generator=gen(5)))
    outs = []
    for tile_cap in (None, cap):
        out = ops.empty(rt, shape, (oh * ow * k, 1, ow * k, k))
        assert ops.conv_tc(xd, hi, lo, k, c, ksz, ksz, c_pad, k_pad, b, unit.stride, unit.padding,
                           unit.dilation, 2, res, False, out, tile_cap=tile_cap)
        outs.append(out.cpu())
    assert len(ops.conv_regions(oh, ow, cap)) > 1
    assert bit_exact(outs[1], outs[0])
    ref = F.silu(O.conv2d(x, conv.weight.detach(), conv.bias.detach(), stride, ksz // 2))
    if residual:
        ref = ref + res.cpu()
    assert max_rel_err(outs[0], ref) < CONV_GEMM_REL


@pytest.mark.parametrize("c,k,ksz,stride,h,w,cap,layout,groups", [
    (3, 16, 3, 2, 64, 66, 8, "nhwc", 1),    # stem kernel, even region columns (vector loads)
    (3, 16, 3, 2, 64, 66, 7, "nhwc", 1),    # stem kernel, odd region columns (scalar loads)
    (3, 16, 3, 2, 30, 31, 5, "nchw", 1),    # one-pixel small-channel kernel
    (8, 16, 3, 1, 21, 19, 6, "nchw", 2),    # grouped: SIMT implicit GEMM
    (3, 64, 7, 2, 40, 40, 6, "nhwc", 1),    # 7x7 stem
])
def test_simt_regions_equal_one_launch(mm, c, k, ksz, stride, h, w, cap, layout, groups):
    g = gen(c * k + h)
    x = torch.rand(2, c, h, w, generator=g) * 2 - 1
    wt = torch.randn(k, c // groups, ksz, ksz, generator=g) / (c * ksz * ksz) ** 0.5
    bias = torch.randn(k, generator=g) * 0.1
    xd = mm.to_device(x)
    pad = ksz // 2
    oh, ow = ops.conv_output_hw(h, w, ksz, ksz, (stride, stride), (pad, pad), (1, 1))
    strides = (oh * ow * k, 1, ow * k, k) if layout == "nhwc" else None
    outs = [ops.convolution(xd, wt, bias, stride, pad, 1, groups, act=2, out_strides=strides,
                            tile_cap=cap_).cpu() for cap_ in (None, cap)]
    assert len(ops.conv_regions(oh, ow, cap)) > 1
    assert bit_exact(outs[1], outs[0])
    ref = F.silu(O.conv2d(x, wt, bias, stride, pad, 1, groups))
    assert max_rel_err(outs[0], ref) < CONV_GEMM_REL


def test_prepared_model_under_a_tile_limit_in_a_fresh_process():
    """MATRIXMAN_TILE_LIMIT=24 (read at init, then locked): a prepared YOLOv8n
    at 128 x 128, whose stem (64 x 64) and first stages exceed 24 x 24, runs
    its convolutions as region launches and matches the CPU oracle."""
    code = (
        "import json, torch, matrixman_b200 as mm, workloads as W\n"
        "from matrixman_b200 import telemetry\n"
        "from oracle.models import run_cpu\n"
        "from oracle.tolerance import max_rel_err\n"
        "mm.init()\n"
        "model = W.yolov8_model('n')\n"
        "x = W.yolo_input(2, size=128)\n"
        "ref = run_cpu(model, x)\n"
        "p = mm.prepare(model)\n"
        "with torch.no_grad():\n"
        "    ys = [p(mm.to_device(x)).cpu() for _ in range(3)]\n"
        "print(json.dumps({'limit': mm.config.tile_limit, 'err': max(max_rel_err(y, ref) for y in ys),\n"
        "                  'tc_regions': telemetry.launches['mm_conv2d_tc_region'],\n"
        "                  'simt_regions': telemetry.launches['mm_conv2d_region']}))\n")
    env = dict(os.environ, MATRIXMAN_TILE_LIMIT="24", PYTHONPATH=str(ROOT))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, cwd=ROOT,
                         timeout=600)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-4000:]
    res = json.loads([l for l in out.stdout.splitlines() if l.startswith("{")][-1])
    assert res["limit"] == 24
    assert res["tc_regions"] > 0 and res["simt_regions"] > 0
    assert res["err"] < CONV_GEMM_REL, res
