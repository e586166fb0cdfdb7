"""Per-op parity of the B200 kernels against the CPU oracle (through the C ABI).

Bars: conv/GEMM max relative error <= 1e-4 (the
reference's relative_max); activations within 4 ulp of torch CPU; softmax
within 1 ulp of the correctly rounded value (torch's own CPU softmax is up to
~30 ulp away from it, see test_softmax_*); max-pool, cat, upsample, copies
bit-exact.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import ops as O
from oracle.tolerance import CONV_GEMM_REL, ULP_BAR, bit_exact, max_rel_err, max_ulp

pytestmark = pytest.mark.gpu


def gen(seed):
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def dev(mm, t):
    return mm.to_device(t.contiguous())


def nhwc(mm, t):
    """Upload as a channels-last view (logical NCHW)."""
    x = mm.to_device(t.permute(0, 2, 3, 1).contiguous())
    return x.permute(0, 3, 1, 2)


# ---------------------------------------------------------------- convolution

def test_conv_known_answers(mm, golden):
    g = golden
    x, w, b = (torch.from_numpy(g[k]) for k in ("conv_arange_x", "conv_arange_w", "conv_arange_b"))
    y = F.conv2d(dev(mm, x), w, b, 1, 1).cpu()
    assert max_rel_err(y, torch.from_numpy(g["conv_arange_y"])) < CONV_GEMM_REL
    x, w = torch.from_numpy(g["conv_grouped_x"]), torch.from_numpy(g["conv_grouped_w"])
    y = F.conv2d(dev(mm, x), w, None, 2, 1, 1, 8).cpu()
    assert max_rel_err(y, torch.from_numpy(g["conv_grouped_y"])) < CONV_GEMM_REL


def test_conv_demo_cases_against_golden(mm, golden):
    from tests.test_oracle_golden import demo_inputs
    for i in range(4):
        x, w, b, s, p = demo_inputs(i, golden)
        y = F.conv2d(dev(mm, x), w, b, stride=s, padding=p).cpu().reshape(-1)
        idx = torch.from_numpy(golden[f"conv_demo{i}_y_idx"])
        assert max_rel_err(y[idx], torch.from_numpy(golden[f"conv_demo{i}_y_val"])) < CONV_GEMM_REL


def test_config1_conv(mm):
    from workloads import conv1_case
    x, w = conv1_case(0)
    y = F.conv2d(dev(mm, x), w, None, 1, 1).cpu()
    assert max_rel_err(y, O.conv2d(x, w, None, 1, 1)) < CONV_GEMM_REL


@pytest.mark.parametrize("c,k,ksz,stride,pad,dil,groups,hw,n", [
    (3, 16, 3, 2, 1, 1, 1, 64, 2),
    (16, 32, 3, 2, 1, 1, 1, 40, 2),
    (32, 32, 1, 1, 0, 1, 1, 33, 3),
    (64, 64, 3, 1, 1, 1, 1, 20, 2),
    (48, 80, 3, 1, 1, 1, 1, 17, 1),
    (64, 64, 3, 1, 2, 2, 1, 19, 1),
    (8, 16, 3, 2, 1, 1, 8, 16, 1),
    (12, 24, 5, 1, 2, 1, 3, 11, 2),
    (3, 64, 7, 2, 3, 1, 1, 56, 1),
    (3, 20, 3, 2, 1, 1, 1, 31, 1),   # stem with a partial second 16-channel group
    (4, 16, 3, 1, 1, 1, 1, 70, 2),   # stride-1 stem, partial tiles
    (1, 8, 3, 2, 0, 1, 1, 67, 1),    # one channel, no padding
    (2, 32, 3, 1, 0, 1, 1, 9, 3),    # tiny images, two channel groups
])
def test_conv_shapes_nchw_and_nhwc(mm, c, k, ksz, stride, pad, dil, groups, hw, n):
    g = gen(c * 100 + k)
    x = torch.rand(n, c, hw, hw + 1, generator=g) * 2 - 1
    w = torch.randn(k, c // groups, ksz, ksz, generator=g) * (1.0 / (c // groups * ksz * ksz) ** 0.5)
    b = torch.randn(k, generator=g) * 0.1
    ref = O.conv2d(x, w, b, stride, pad, dil, groups)
    y1 = F.conv2d(dev(mm, x), w, b, stride, pad, dil, groups).cpu()
    assert max_rel_err(y1, ref) < CONV_GEMM_REL
    y2 = F.conv2d(nhwc(mm, x), w, b, stride, pad, dil, groups).cpu()
    assert max_rel_err(y2, ref) < CONV_GEMM_REL


@pytest.mark.parametrize("c,k,h,w,n", [
    (3, 16, 64, 65, 2),    # odd input width: a partial last quad of output columns
    (3, 48, 31, 33, 1),    # three 16-channel groups, odd sizes
    (1, 16, 67, 67, 1),
    (2, 32, 9, 12, 3),     # tiny images: every quad touches an edge
    (3, 16, 640, 640, 1),  # the YOLOv8 stem
])
def test_stride2_stem_kernel(mm, c, k, h, w, n):
    """Stride-2 3x3 stems with channels-last output run the 4-pixel stem
    kernel (prepared convolution); NCHW output runs the one-pixel kernel
    (eager F.conv2d).  Both accumulate each output in the same order, so
    they agree bit for bit; both are within the convolution tolerance of the
    oracle, with and without the fused SiLU."""
    from matrixman_b200.preparation import PreparedConv2d
    g = gen(c * 1000 + k + h)
    x = torch.rand(n, c, h, w, generator=g) * 2 - 1
    conv = torch.nn.Conv2d(c, k, 3, 2, 1)
    with torch.no_grad():
        conv.weight.copy_(torch.randn(k, c, 3, 3, generator=g) * (1.0 / (c * 9) ** 0.5))
        conv.bias.copy_(torch.randn(k, generator=g) * 0.1)
        xd = mm.to_device(x)
        y_stem = PreparedConv2d(conv, 0)(xd).cpu()
        y_silu = PreparedConv2d(conv, 2)(xd).cpu()
        y_pixel = F.conv2d(dev(mm, x), conv.weight, conv.bias, 2, 1).cpu()
    ref = O.conv2d(x, conv.weight.detach(), conv.bias.detach(), 2, 1)
    assert bit_exact(y_stem, y_pixel)
    assert max_rel_err(y_stem, ref) < CONV_GEMM_REL
    assert max_rel_err(y_silu, ref * torch.sigmoid(ref)) < CONV_GEMM_REL


def test_conv_empty_and_unsupported(mm):
    x = dev(mm, torch.randn(1, 4, 8, 8))
    with pytest.raises(NotImplementedError):
        torch.ops.aten.convolution.default(x, torch.randn(4, 4, 3, 3), None, [1, 1], [1, 1], [1, 1],
                                           True, [0, 0], 1)
    with pytest.raises(NotImplementedError):
        F.conv2d(x, torch.randn(4, 3, 3, 3), None, 1, 1)  # channels do not match groups
    with pytest.raises(ValueError):
        F.conv2d(dev(mm, torch.randn(1, 4, 2, 2)), torch.randn(4, 4, 5, 5))  # output would be empty


# ---------------------------------------------------------------- GEMM

@pytest.mark.parametrize("m,k,n", [(256, 784, 512), (32, 512, 1000), (7, 13, 5), (1, 64, 3)])
def test_linear_and_addmm(mm, m, k, n):
    g = gen(m + k + n)
    x = torch.randn(m, k, generator=g)
    lin = torch.nn.Linear(k, n)
    with torch.no_grad():
        y = lin(dev(mm, x)).cpu()
        ref = lin(x)
    assert max_rel_err(y, ref) < CONV_GEMM_REL
    a, bm = torch.randn(m, k, generator=g), torch.randn(k, n, generator=g)
    bias = torch.randn(n, generator=g)
    y = torch.addmm(bias, dev(mm, a), bm, beta=0.5, alpha=2.0).cpu()
    assert max_rel_err(y, O.addmm(bias, a, bm, 0.5, 2.0)) < CONV_GEMM_REL
    y = torch.mm(dev(mm, a), dev(mm, bm)).cpu()
    assert max_rel_err(y, a @ bm) < CONV_GEMM_REL
    with pytest.raises(RuntimeError):
        torch.mm(dev(mm, a), dev(mm, torch.randn(k + 1, n)))


# ---------------------------------------------------------------- elementwise

def special_values():
    return torch.tensor([-88.0, -20.0, -8.0, -2.0, -0.5, -1e-30, 0.0, 1e-30, 0.5, 2.0, 8.0, 20.0,
                         88.0, 100.0, float("inf"), -float("inf")])


@pytest.mark.parametrize("name,fn", [("silu", F.silu), ("sigmoid", torch.sigmoid), ("relu", F.relu)])
def test_activations_ulp(mm, name, fn, golden):
    g = gen(7)
    x = torch.cat([torch.randn(1 << 18, generator=g) * 6, special_values()])
    y = fn(dev(mm, x)).cpu()
    ref = fn(x)
    finite = torch.isfinite(ref)
    assert max_ulp(y[finite], ref[finite]) <= ULP_BAR
    assert bit_exact(y[~finite], ref[~finite])  # inf/nan in the same places (silu(-inf) = nan)
    if name == "silu":
        kat = F.silu(dev(mm, torch.from_numpy(golden["silu_x"]))).cpu()
        assert max_ulp(kat, torch.from_numpy(golden["silu_y"])) <= ULP_BAR


def test_inplace_activation_on_strided_view(mm):
    g = gen(8)
    base = torch.randn(2, 6, 5, 7, generator=g)
    d = dev(mm, base)
    view = d[:, 1:4]          # channel slice (non-contiguous)
    F.silu(view, inplace=True)
    F.relu_(d[:, 4:])
    out = d.cpu()
    ref = base.clone()
    ref[:, 1:4] = F.silu(ref[:, 1:4])
    ref[:, 4:] = F.relu(ref[:, 4:])
    assert max_ulp(out, ref) <= ULP_BAR


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
def test_binary_broadcast_and_scalars(mm, op):
    g = gen(9)
    a = torch.randn(4, 3, 8, 9, generator=g)
    b = torch.randn(1, 3, 1, 9, generator=g) + 3.0
    f = {"add": torch.add, "sub": torch.sub, "mul": torch.mul, "div": torch.div}[op]
    y = f(dev(mm, a), dev(mm, b)).cpu()
    assert bit_exact(y, f(a, b))
    y = f(dev(mm, a), 2.5).cpu()
    assert bit_exact(y, f(a, 2.5))
    if op in ("add", "sub"):
        y = f(dev(mm, a), dev(mm, b), alpha=0.75).cpu()
        assert max_ulp(y, f(a, b, alpha=0.75)) <= 1
    d = dev(mm, a)
    getattr(d, op + "_")(dev(mm, b))
    assert bit_exact(d.cpu(), f(a, b))


def test_nhwc_elementwise_keeps_layout(mm):
    g = gen(10)
    a = torch.randn(2, 8, 5, 6, generator=g)
    x = nhwc(mm, a)
    y = x + x
    assert y.stride() == x.stride()
    assert bit_exact(y.cpu(), a + a)


# ---------------------------------------------------------------- softmax

@pytest.mark.parametrize("shape,dim", [((256, 10), 1), ((32, 1000), 1), ((2, 16, 4, 840), 1),
                                       ((3, 5, 7), 0), ((4, 64, 33), 2), ((1,), 0)])
def test_softmax_ulp(mm, shape, dim):
    g = gen(11)
    x = torch.randn(shape, generator=g) * 3
    y = torch.softmax(dev(mm, x), dim).cpu()
    exact = O.softmax_exact(x, dim)
    assert max_ulp(y, exact) <= 1
    torch_cpu = O.softmax(x, dim)
    # torch's CPU kernel is itself up to tens of ulp from exact; the device
    # result must never be further from torch than torch is from exact + 1 ulp.
    assert max_ulp(y, torch_cpu) <= max_ulp(torch_cpu, exact) + 1
    ly = torch.log_softmax(dev(mm, x), dim).cpu()
    assert max_rel_err(ly, O.log_softmax(x, dim)) < 1e-5


def test_dfl_softmax_demo(mm, golden):
    base = torch.from_numpy(golden["dfl_softmax_x"])
    y = torch.ops.aten._softmax.default(dev(mm, base).transpose(1, 2), 1, False).cpu()
    assert max_ulp(y, O.softmax_exact(base.transpose(1, 2), 1)) <= 1
    assert torch.allclose(y, torch.from_numpy(golden["dfl_softmax_y"]), atol=1e-6, rtol=1e-5)


# ---------------------------------------------------------------- pooling / resize / reductions

def test_maxpool_golden_cases_bit_exact(mm, golden):
    for name in ("random_128x20x20", "random_small", "all_negative", "padding_edge"):
        x = torch.from_numpy(golden[f"maxpool_{name}_x"])
        y, idx = F.max_pool2d(dev(mm, x), 5, 1, 2, 1, False, True)
        assert bit_exact(y.cpu(), torch.from_numpy(golden[f"maxpool_{name}_y"]))
        assert tuple(idx.shape) == (0,)


def test_maxpool_storage_offset(mm):
    from matrixman_b200.tensor import MatrixManTensor
    src = torch.randn(1, 2, 6, 6, generator=gen(12))
    base = dev(mm, torch.cat((torch.zeros(1), src.reshape(-1))))
    view = MatrixManTensor._from_owner(base._owner, src.shape, 1, (72, 36, 6, 1))
    y = F.max_pool2d(view, 5, 1, 2)
    assert bit_exact(y.cpu(), F.max_pool2d(src, 5, 1, 2))


@pytest.mark.parametrize("k,s,p,d,ceil", [(3, 2, 1, 1, False), (2, 2, 0, 1, True), (3, 1, 1, 2, False),
                                          (5, 3, 2, 1, True)])
def test_maxpool_generic_bit_exact(mm, k, s, p, d, ceil):
    x = torch.randn(2, 5, 17, 14, generator=gen(k * 10 + s))
    x[0, 0, 3, 3] = float("nan")
    ref = F.max_pool2d(x, k, s, p, d, ceil)
    assert bit_exact(F.max_pool2d(dev(mm, x), k, s, p, d, ceil).cpu(), ref)
    assert bit_exact(F.max_pool2d(nhwc(mm, x), k, s, p, d, ceil).cpu(), ref)


def test_sppf_fused_chain_bit_exact(mm):
    import ctypes
    from matrixman_b200 import ops
    x = torch.randn(2, 40, 20, 23, generator=gen(13))
    x[1, 7, 5, 5] = float("nan")
    d = nhwc(mm, x)
    outs = [ops.empty(d.runtime, x.shape, d._logical_strides) for _ in range(3)]
    ops._launch("mm_sppf_pool", ctypes.byref(d.desc()), *(ctypes.byref(o.desc()) for o in outs),
                d.runtime.stream)
    for o, r in zip(outs, O.sppf_chain(x)):
        assert bit_exact(o.cpu(), r)
    # a partial channel group and a tiny image
    x = torch.randn(1, 12, 7, 9, generator=gen(31))
    d = nhwc(mm, x)
    outs = [ops.empty(d.runtime, x.shape, d._logical_strides) for _ in range(3)]
    ops._launch("mm_sppf_pool", ctypes.byref(d.desc()), *(ctypes.byref(o.desc()) for o in outs),
                d.runtime.stream)
    for o, r in zip(outs, O.sppf_chain(x)):
        assert bit_exact(o.cpu(), r)


@pytest.mark.parametrize("k,s,p,ceil,cip,div", [(2, 2, 0, False, True, None), (3, 2, 1, True, False, None),
                                                (3, 1, 1, False, True, 5)])
def test_avg_pool(mm, k, s, p, ceil, cip, div):
    x = torch.randn(2, 4, 11, 9, generator=gen(14))
    ref = F.avg_pool2d(x, k, s, p, ceil, cip, div)
    y = F.avg_pool2d(dev(mm, x), k, s, p, ceil, cip, div).cpu()
    assert max_rel_err(y, ref) < 1e-6


def test_adaptive_avg_and_mean(mm):
    x = torch.randn(4, 16, 7, 7, generator=gen(15))
    assert max_rel_err(F.adaptive_avg_pool2d(dev(mm, x), (1, 1)).cpu(), F.adaptive_avg_pool2d(x, (1, 1))) < 1e-6
    assert max_rel_err(F.adaptive_avg_pool2d(dev(mm, x), (3, 2)).cpu(), F.adaptive_avg_pool2d(x, (3, 2))) < 1e-6
    assert max_rel_err(dev(mm, x).mean((-1, -2), keepdim=True).cpu(), x.mean((-1, -2), keepdim=True)) < 1e-6
    assert max_rel_err(nhwc(mm, x).mean((2, 3)).cpu(), x.mean((2, 3))) < 1e-6
    assert max_rel_err(dev(mm, x).sum(1).cpu(), x.sum(1)) < 1e-6


def test_upsample_golden_and_scales(mm, golden):
    for name, size in (("exact", (4, 6)), ("nonint", (5, 7)), ("multi", (8, 8))):
        x = torch.from_numpy(golden[f"nearest_{name}_x"])
        y = F.interpolate(dev(mm, x), size=size, mode="nearest").cpu()
        assert bit_exact(y, F.interpolate(x, size=size, mode="nearest"))
        if name != "nonint":
            assert np.array_equal(y.numpy(), golden[f"nearest_{name}_y"])
    x = torch.randn(2, 8, 20, 20, generator=gen(16))
    for sf in (2.0, 3.0):
        ref = F.interpolate(x, scale_factor=sf, mode="nearest")
        assert bit_exact(F.interpolate(nhwc(mm, x), scale_factor=sf, mode="nearest").cpu(), ref)
        assert bit_exact(F.interpolate(dev(mm, x), scale_factor=sf, mode="nearest").cpu(), ref)


def test_batch_norm_eval(mm, golden):
    g = golden
    t = {k: torch.from_numpy(g[k]) for k in ("bn_x", "bn_mean", "bn_var", "bn_w", "bn_b", "bn_y")}
    y = F.batch_norm(dev(mm, t["bn_x"]), t["bn_mean"], t["bn_var"], t["bn_w"], t["bn_b"], False, 0.1, 1e-5).cpu()
    assert max_rel_err(y, t["bn_y"]) < 1e-6
    bn = torch.nn.BatchNorm2d(16).eval()
    from workloads import randomize_bn
    randomize_bn(bn, 3)
    x = torch.randn(3, 16, 9, 9, generator=gen(17))
    with torch.no_grad():
        assert max_rel_err(bn(nhwc(mm, x)).cpu(), bn(x)) < 1e-6
    with pytest.raises(NotImplementedError):
        F.batch_norm(dev(mm, x), bn.running_mean, bn.running_var, training=True)


@pytest.mark.parametrize("nc,hw,batch,layout", [
    (80, (8, 4, 2), 3, "nhwc"),   # 84 anchors per image: 32-anchor chunks straddle levels and images
    (5, (6, 3), 2, "nchw"),       # generic strides, small class count
    (12, (5, 3), 2, "nhwc"),      # row kernel with a partial group of class loads
])
def test_yolo_decode_matches_oracle(mm, nc, hw, batch, layout):
    import ctypes
    from matrixman_b200 import _lib, ops
    g = gen(nc + batch)
    reg_max = 16
    no = 4 * reg_max + nc
    strides = [8.0 * 2 ** i for i in range(len(hw))]
    feats = [torch.randn(batch, no, s, s, generator=g) * 3 for s in hw]
    ref = O.yolo_decode(feats, strides, reg_max, nc)
    devs = [nhwc(mm, f) if layout == "nhwc" else dev(mm, f) for f in feats]
    anchors = sum(s * s for s in hw)
    out = ops.empty(devs[0].runtime, (batch, 4 + nc, anchors))
    descs = [d.desc() for d in devs]
    arr = (ctypes.POINTER(_lib.MMTensor) * len(descs))(*[ctypes.pointer(d) for d in descs])
    st = (ctypes.c_float * len(strides))(*strides)
    ops._launch("mm_yolo_decode", arr, st, len(devs), reg_max, nc, ctypes.byref(out.desc()),
                devs[0].runtime.stream)
    assert max_rel_err(out.cpu(), ref) < CONV_GEMM_REL
