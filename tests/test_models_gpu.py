"""Whole-model parity on the device against the unprepared CPU fp32 oracle
(max relative error <= 1e-4, the reference's relative_max measure)."""

import pytest
import torch

import workloads as W
from oracle.models import run_cpu
from oracle.tolerance import CONV_GEMM_REL, max_rel_err

pytestmark = pytest.mark.gpu


def _check(mm, model, x, prepared=True, calls=3):
    ref = run_cpu(model, x)
    target = mm.prepare(model) if prepared else model
    with torch.no_grad():
        for _ in range(calls):  # eager warm-up, graph capture, replay
            y = target(mm.to_device(x)).cpu()
            err = max_rel_err(y, ref)
            assert err < CONV_GEMM_REL, f"max relative error {err:.3g}"
    return target


def test_mlp_bs256(mm):
    model = W.mlp_model()
    x = W.mlp_input(256)
    _check(mm, model, x, prepared=False, calls=1)
    p = _check(mm, model, x)
    rep = p._matrixman_preparation_report
    assert rep.linear_units_prepared == 3


def test_resnet18_bs32(mm):
    model = W.resnet18_model()
    x = W.resnet18_input(32)
    p = _check(mm, model, x)
    rep = p._matrixman_preparation_report
    assert rep.folded == 20 and rep.remaining_batch_norm_modules == 0
    assert rep.block_units_prepared["BasicBlock"] == 8


def test_resnet18_unprepared_eager(mm):
    model = W.resnet18_model()
    x = W.resnet18_input(2, size=96)
    _check(mm, model, x, prepared=False, calls=1)


@pytest.mark.parametrize("batch", [1, 2])
def test_yolov8n_prepared(mm, batch):
    model = W.yolov8_model("n")
    x = W.yolo_input(batch)
    p = _check(mm, model, x)
    rep = p._matrixman_preparation_report
    assert rep.folded == 57 and rep.detection_head_prepared == 1


def test_yolov8n_neck_concatenations_in_place(mm):
    """The prepared YOLOv8 writes its four neck concatenations in place: a
    prepared forward launches no concatenation copy, and matches the oracle
    at a size whose levels are not powers of two (odd P5)."""
    from matrixman_b200 import telemetry
    model = W.yolov8_model("n")
    x = W.yolo_input(2, seed=21, size=352)
    p = mm.prepare(model)
    assert p._matrixman_preparation_report.block_units_prepared["YOLOv8 in-place neck"] == 1
    ref = run_cpu(model, x)
    with torch.no_grad():
        before = telemetry.launches["mm_cat"]
        y = p(mm.to_device(x)).cpu()  # eager (first call)
        assert telemetry.launches["mm_cat"] == before
    assert max_rel_err(y, ref) < CONV_GEMM_REL


def test_yolov8n_prepared_bs64(mm):
    """The benchmark's own configuration: YOLOv8n 640x640 at 64 images, eager
    forward, graph capture and graph replay, each against the CPU oracle."""
    model = W.yolov8_model("n")
    x = W.yolo_input(64, seed=1000)
    _check(mm, model, x, calls=3)


def test_yolov8m_prepared_bs8(mm):
    """A batch-8 slice of the YOLOv8m bs256 configuration (eager + graph)."""
    model = W.yolov8_model("m")
    x = W.yolo_input(8, seed=7)
    _check(mm, model, x, calls=2)


def test_parameter_cache_reuploads_after_inplace_edit(mm):
    """An in-place edit of a CPU weight bumps its version, and the next eager
    call uploads it again (reference backends/cuda/backend.py:241-294); an
    unchanged weight is served from the cache."""
    from matrixman_b200 import runtime
    g = torch.Generator().manual_seed(11)
    conv = torch.nn.Conv2d(8, 16, 3, padding=1, bias=True).eval()
    x = torch.rand(2, 8, 24, 24, generator=g) * 2 - 1
    rt = runtime.get_runtime(runtime.current_device())
    with torch.no_grad():
        xd = mm.to_device(x)
        y1 = conv(xd).cpu()
        size1 = rt.parameter_cache_size()
        y1b = conv(xd).cpu()
        assert rt.parameter_cache_size() == size1
        assert torch.equal(y1, y1b)
        conv.weight.mul_(-2.0)
        conv.bias.add_(0.5)
        y2 = conv(xd).cpu()
        ref2 = conv(x)
    assert max_rel_err(y1, torch.nn.functional.conv2d(x, conv.weight / -2.0, conv.bias - 0.5,
                                                      padding=1)) < CONV_GEMM_REL
    assert max_rel_err(y2, ref2) < CONV_GEMM_REL
    assert not torch.allclose(y1, y2)


def test_yolov8n_unprepared_eager(mm):
    model = W.yolov8_model("n")
    x = W.yolo_input(1, size=320)
    _check(mm, model, x, prepared=False, calls=1)


def test_yolov8m_prepared_bs1(mm):
    model = W.yolov8_model("m")
    x = W.yolo_input(1)
    _check(mm, model, x, calls=2)


def test_auto_prepare_lazy(mm):
    model = W.yolov8_model("n")
    lazy = mm.auto_prepare(model)
    x = W.yolo_input(1, size=320)
    ref = run_cpu(model, x)
    with torch.no_grad():
        y = lazy(mm.to_device(x)).cpu()
    assert max_rel_err(y, ref) < CONV_GEMM_REL


@pytest.mark.parametrize("chunks", [1, 2, 3, 4])
def test_infer_pipeline_matches_serial(mm, chunks):
    """Overlapped upload / forward / readback gives the serial path's values."""
    import workloads as W
    model = W.yolov8_model("n")
    prepared = mm.prepare(model)
    x = mm.pinned_empty((5, 3, 256, 256))
    x.copy_(W.yolo_input(5, size=256))
    with torch.no_grad():
        ref = prepared(mm.to_device(x)).cpu()
        y = mm.infer(prepared, x, chunks=chunks)
        y2 = mm.infer(prepared, x, chunks=chunks)  # graph replay path
    assert y.shape == ref.shape
    assert max_rel_err(y, ref) < 1e-6
    assert torch.equal(y, y2)


def test_infer_explicit_sizes(mm):
    """Uneven explicit slices give the serial values; bad sizes are rejected."""
    import workloads as W
    prepared = mm.prepare(W.yolov8_model("n"))
    x = mm.pinned_empty((7, 3, 256, 256))
    x.copy_(W.yolo_input(7, size=256))
    with torch.no_grad():
        ref = prepared(mm.to_device(x)).cpu()
        y = mm.infer(prepared, x, sizes=[1, 2, 3, 1])
        assert max_rel_err(y, ref) < 1e-6
        for bad in ([3, 3], [7, 0], [8, -1], []):
            with pytest.raises(ValueError):
                mm.infer(prepared, x, sizes=bad)


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_infer_stream_matches_serial(mm, depth):
    """The streaming API yields, in order, exactly the serial results of each
    batch (batches of different sizes and contents, several in flight)."""
    model = W.yolov8_model("n")
    prepared = mm.prepare(model)
    batches = []
    for i, n in enumerate((3, 3, 1, 4, 3)):
        x = mm.pinned_empty((n, 3, 256, 256))
        x.copy_(W.yolo_input(n, seed=70 + i, size=256))
        batches.append(x)
    with torch.no_grad():
        refs = [prepared(mm.to_device(x)).cpu() for x in batches]
        outs = [y.clone() for y in mm.infer_stream(prepared, batches, depth=depth)]
    assert len(outs) == len(refs)
    for y, ref in zip(outs, refs):
        assert y.shape == ref.shape
        assert torch.equal(y, ref)
    with pytest.raises(ValueError):
        list(mm.infer_stream(prepared, batches, depth=0))
