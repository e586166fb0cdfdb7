"""Parity of the tcgen05 3xTF32 convolution (prepared units) with the CPU
oracle, across the geometries YOLOv8 / ResNet use plus edge cases."""

import pytest
import torch
from torch import nn

from matrixman_b200 import _lib
from matrixman_b200.preparation import PreparedConv2d
from oracle import ops as O
from oracle.tolerance import CONV_GEMM_REL, max_rel_err

pytestmark = pytest.mark.gpu

ACTS = {0: lambda t: t, 1: torch.relu, 2: torch.nn.functional.silu}


def gen(seed):
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def nhwc(mm, t):
    return mm.to_device(t.permute(0, 2, 3, 1).contiguous()).permute(0, 3, 1, 2)


def run_case(mm, n, c, k, ksz, stride, pad, hw, act=2, residual=None, seed=0):
    g = gen(seed)
    conv = nn.Conv2d(c, k, ksz, stride, pad, bias=True)
    with torch.no_grad():
        conv.weight.copy_(torch.randn(conv.weight.shape, generator=g) / (c * ksz * ksz) ** 0.5)
        conv.bias.copy_(torch.randn(k, generator=g) * 0.1)
    unit = PreparedConv2d(conv, act)
    assert unit.tc_eligible
    x = torch.rand(n, c, hw, hw + 3, generator=g) * 2 - 1
    ref = ACTS[act](O.conv2d(x, conv.weight.detach(), conv.bias.detach(), stride, pad))
    res_dev = None
    if residual is not None:
        r = torch.randn(ref.shape, generator=g)
        res_dev = nhwc(mm, r)
        if residual == "before":
            ref = ACTS[act](O.conv2d(x, conv.weight.detach(), conv.bias.detach(), stride, pad) + r)
        else:
            ref = ref + r
    from matrixman_b200 import telemetry
    before = telemetry.launches["mm_conv2d_tc"]
    y = unit(nhwc(mm, x), residual=res_dev, residual_before_act=residual == "before")
    assert telemetry.launches["mm_conv2d_tc"] == before + 1, "tensor-core path did not run"
    err = max_rel_err(y.cpu(), ref)
    assert err < CONV_GEMM_REL, f"max relative error {err:.3g}"
    return err


@pytest.mark.parametrize("n,c,k,ksz,stride,pad,hw", [
    (2, 16, 32, 3, 2, 1, 40),     # YOLO downsample
    (2, 32, 32, 3, 1, 1, 20),     # bottleneck 3x3
    (1, 64, 64, 1, 1, 0, 33),     # 1x1
    (1, 48, 80, 3, 1, 1, 17),     # detect class branch width
    (1, 4, 5, 3, 1, 1, 64),       # config-1 channel counts (C padded to 32)
    (1, 20, 24, 3, 1, 1, 16),     # last channel block: 3 of 4 eight-channel steps
    (2, 40, 32, 3, 2, 1, 18),     # second channel block holds 8 channels (1 step)
    (1, 128, 144, 1, 1, 0, 12),   # K not a multiple of 16 tile
    (1, 96, 576, 3, 2, 1, 10),    # K > 256: three N tiles
    (3, 256, 256, 3, 1, 1, 7),    # deep layer
    (2, 128, 128, 3, 1, 1, 20),   # 20 x 23 output: rectangles covering ~62 % (idle rows clipped)
    (1, 64, 64, 7, 2, 3, 23),     # 7x7 stride 2
])
def test_tc_conv_geometries(mm, n, c, k, ksz, stride, pad, hw):
    run_case(mm, n, c, k, ksz, stride, pad, hw, act=2, seed=c * 7 + k)


@pytest.mark.parametrize("act", [0, 1, 2])
@pytest.mark.parametrize("residual", [None, "before", "after"])
def test_tc_conv_epilogues(mm, act, residual):
    run_case(mm, 2, 32, 48, 3, 1, 1, 15, act=act, residual=residual, seed=act * 3 + len(str(residual)))


def test_tc_precision_is_fp32_class(mm):
    """3xTF32 must be far below the 1e-4 bar (plain tf32 would be ~1e-3)."""
    err = run_case(mm, 1, 64, 64, 3, 1, 1, 32, act=0, seed=5)
    assert err < 1e-5


@pytest.mark.parametrize("act", [2, 3])
def test_tc_fused_activation_accuracy(mm, act):
    """The fused SiLU / sigmoid element by element: the same 1x1 convolution
    (identity weights, inputs spread over [-100, 100]) with and without the
    activation; every activated element is within 1e-5 relative of the
    double-precision activation of the un-activated output (absolute 1e-30
    where it underflows).  The bar covers the fast exponential's documented
    error, 2 + 1.173 |x| ulp (about 6e-6 relative at |x| = 88), and the fast
    division's 2 ulp."""
    c = 32
    conv = nn.Conv2d(c, c, 1, 1, 0, bias=True)
    with torch.no_grad():
        conv.weight.copy_(torch.eye(c).reshape(c, c, 1, 1))
        conv.bias.zero_()
    x = torch.linspace(-100.0, 100.0, 4 * 64 * 64 * c).reshape(4, c, 64, 64)
    x[0, 0, 0, :8] = torch.tensor([0.0, -0.0, 1e-30, -1e-30, 80.5, -80.5, 87.0, -87.0])
    xd = nhwc(mm, x)
    with torch.no_grad():
        pre = PreparedConv2d(conv, 0)(xd).cpu().double()
        y = PreparedConv2d(conv, act)(xd).cpu().double()
    ref = pre * torch.sigmoid(pre) if act == 2 else torch.sigmoid(pre)
    err = (y - ref).abs()
    bad = err > 1e-5 * ref.abs() + 1e-30
    i = int(torch.argmax((err / (ref.abs() + 1e-30)).flatten()))
    assert not bool(bad.any()), (int(bad.sum()), float(pre.flatten()[i]), float(y.flatten()[i]),
                                 float(ref.flatten()[i]))


def test_tc_channel_slices_in_and_out(mm):
    from matrixman_b200 import ops
    from matrixman_b200.preparation import _channel_slice
    g = gen(9)
    conv = nn.Conv2d(16, 32, 3, 1, 1)
    unit = PreparedConv2d(conv, 2)
    big = torch.randn(2, 48, 9, 11, generator=g)
    xd = nhwc(mm, big)
    xin = _channel_slice(xd, 16, 32)
    out_buf = ops.empty(xd.runtime, (2, 96, 9, 11), (96 * 9 * 11, 1, 11 * 96, 96))
    ops.fill_(out_buf, 0.0)
    unit(xin, out=_channel_slice(out_buf, 32, 64))
    y = out_buf.cpu()
    ref = torch.nn.functional.silu(O.conv2d(big[:, 16:32], conv.weight.detach(), conv.bias.detach(), 1, 1))
    assert max_rel_err(y[:, 32:64], ref) < CONV_GEMM_REL
    assert torch.count_nonzero(y[:, :32]) == 0 and torch.count_nonzero(y[:, 64:]) == 0


def test_tc_matches_simt_path(mm):
    import matrixman_b200 as matrixman
    g = gen(11)
    conv = nn.Conv2d(64, 64, 3, 1, 1)
    unit = PreparedConv2d(conv, 2)
    x = nhwc(mm, torch.randn(2, 64, 20, 20, generator=g))
    y_tc = unit(x).cpu()
    old = matrixman.config.conv_algo
    matrixman.config.conv_algo = "simt"
    try:
        y_simt = unit(x).cpu()
    finally:
        matrixman.config.conv_algo = old
    assert max_rel_err(y_tc, y_simt) < 1e-5


def test_tc_deep_reduction_drift_bounded(mm):
    """All-positive data is the worst case for the tensor core's truncating
    accumulation (every partial sum moves toward zero).  Each period (at most 12
    k-blocks) is promoted into an fp32 total with round-to-nearest adds, so the
    bias is that of one period and must not grow with the reduction length:
    144 k-blocks against 36 on the same data distribution."""
    drifts = {}
    for c, seed in ((512, 21), (128, 24)):
        g = gen(seed)
        k = 64
        conv = nn.Conv2d(c, k, 3, 1, 1, bias=False)
        with torch.no_grad():
            conv.weight.copy_(torch.rand(conv.weight.shape, generator=g) / (c * 9))
        unit = PreparedConv2d(conv, 0)
        x = torch.rand(1, c, 12, 12, generator=g)
        ref = O.conv2d(x, conv.weight.detach(), None, 1, 1)
        y = unit(nhwc(mm, x)).cpu()
        err = max_rel_err(y, ref)
        assert err < 5e-6, f"C={c}: max relative error {err:.3g}"
        # mean signed relative deviation: the truncation bias of one period
        drifts[c] = ((y - ref) / ref.abs().clamp_min(1e-30)).mean().item()
        assert abs(drifts[c]) < 3e-6, f"C={c}: mean drift {drifts[c]:.3g}"
    assert abs(drifts[512]) < 1.25 * abs(drifts[128]) + 2e-7, f"drift grows with K: {drifts}"


@pytest.mark.parametrize("m,k,n,act", [
    (256, 784, 512, 1),    # MLP layer 1 (K padded to 800)
    (256, 256, 10, 0),     # MLP head: N not a multiple of 4 (scalar stores)
    (32, 512, 1000, 0),    # ResNet-18 fc: 13 N tiles
    (1, 64, 48, 2),        # single row
    (300, 128, 96, 0),     # ragged M (3 tiles, last partial)
])
def test_tc_linear(mm, m, k, n, act):
    from matrixman_b200 import telemetry
    from matrixman_b200.preparation import PreparedLinear
    g = gen(m + k + n)
    lin = nn.Linear(k, n)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(n, k, generator=g) / k ** 0.5)
        lin.bias.copy_(torch.randn(n, generator=g) * 0.1)
    unit = PreparedLinear(lin, act)
    assert unit.tc_eligible
    x = torch.randn(m, k, generator=g)
    ref = ACTS[act](O.addmm(lin.bias.detach(), x, lin.weight.detach().t()))
    before = telemetry.launches["mm_conv2d_tc"]
    y = unit(mm.to_device(x))
    assert telemetry.launches["mm_conv2d_tc"] == before + 1, "tensor-core GEMM did not run"
    err = max_rel_err(y.cpu(), ref)
    assert err < 1e-5, f"max relative error {err:.3g}"


def test_tc_linear_unaligned_rows_fall_back(mm):
    """K % 4 != 0 cannot be read with 16-byte copies: the SIMT GEMM runs."""
    from matrixman_b200 import telemetry
    from matrixman_b200.preparation import PreparedLinear
    g = gen(3)
    lin = nn.Linear(30, 7)
    unit = PreparedLinear(lin, 0)
    assert not unit.tc_eligible
    x = torch.randn(5, 30, generator=g)
    before = telemetry.launches["mm_conv2d_tc"]
    y = unit(mm.to_device(x)).cpu()
    assert telemetry.launches["mm_conv2d_tc"] == before
    assert max_rel_err(y, O.addmm(lin.bias.detach(), x, lin.weight.detach().t())) < CONV_GEMM_REL


def test_no_kernel_error_recorded(mm):
    import ctypes
    code = ctypes.c_int(-1)
    _lib.check(_lib.load().mm_kernel_error(0, ctypes.byref(code), 0))
    assert code.value == 0


@pytest.mark.parametrize("gather", [False, True])
def test_tc_bounded_wait_runs_out_and_recovers(mm, gather):
    """A device-side wait that runs out: with the test hook, CTA 0 leaves its
    first k-block unissued and the wait budget is 1 ms, so a wait for that
    stage gives up.  The kernel records an error code, finishes its own
    in-flight copies and MMAs, frees its tensor memory and returns (the stream
    synchronises; nothing hangs); the next launch with the defaults gives
    correct results.  gather=True uses a 3 x 3 output, which no 128-pixel
    rectangle covers well, so the producers gather A with cp.async;
    gather=False a 32 x 40 output fetched by TMA rectangles."""
    import ctypes
    import time
    from matrixman_b200 import runtime
    lib = _lib.load()
    dev = runtime.current_device()
    rt = runtime.get_runtime(dev)
    g = gen(91)
    conv = nn.Conv2d(64, 64, 3, 1, 1, bias=True)
    with torch.no_grad():
        conv.weight.copy_(torch.randn(conv.weight.shape, generator=g) / 24.0)
    unit = PreparedConv2d(conv, 2)
    x = torch.rand(4, 64, 3, 3, generator=g) * 2 - 1 if gather else \
        torch.rand(4, 64, 32, 40, generator=g) * 2 - 1
    ref = ACTS[2](O.conv2d(x, conv.weight.detach(), conv.bias.detach(), 1, 1))
    xd = nhwc(mm, x)
    code = ctypes.c_int(-1)
    with torch.no_grad():
        assert max_rel_err(unit(xd).cpu(), ref) < CONV_GEMM_REL
        _lib.check(lib.mm_kernel_error(dev, ctypes.byref(code), 1))
        assert code.value == 0
        _lib.check(lib.mm_debug_tc_fault(dev, 1_000_000, 1))
        try:
            t0 = time.perf_counter()
            unit(xd)
            rt.synchronize(timeout_ms=30_000)
            elapsed = time.perf_counter() - t0
            _lib.check(lib.mm_kernel_error(dev, ctypes.byref(code), 1))
        finally:
            _lib.check(lib.mm_debug_tc_fault(dev, 0, 0))
        assert code.value in (1, 2, 3, 4), f"expected a wait error code, got {code.value}"
        assert elapsed < 5.0
        y = unit(xd).cpu()
        _lib.check(lib.mm_kernel_error(dev, ctypes.byref(code), 0))
    assert code.value == 0
    assert max_rel_err(y, ref) < CONV_GEMM_REL
