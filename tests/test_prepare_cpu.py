"""matrixman.prepare on the host: folding, module replacement, copy semantics
and error behaviour (no device needed: weights upload lazily on first use)."""

import pytest
import torch
from torch import nn

import matrixman_b200 as matrixman
import workloads as W
from matrixman_b200.preparation import (
    PreparedBasicBlock,
    PreparedC2f,
    PreparedConv2d,
    PreparedDetect,
    PreparedLinear,
    PreparedSPPF,
)


def _inner(p):
    return p.module if hasattr(p, "module") and isinstance(p.module, nn.Module) else p


def test_yolov8n_structure():
    model = W.yolov8_model("n")
    p = matrixman.prepare(model)
    rep = p._matrixman_preparation_report
    assert rep.conv_bn_pairs_found == 57 and rep.folded == 57
    assert rep.remaining_batch_norm_modules == 0
    assert rep.block_units_prepared["C2f"] == 8 and rep.block_units_prepared["SPPF"] == 1
    assert rep.detection_head_prepared == 1
    assert rep.conv_units_prepared == 63  # every convolution of the model (DFL excluded)
    inner = _inner(p)
    assert isinstance(inner.b2, PreparedC2f) and isinstance(inner.b9, PreparedSPPF)
    assert isinstance(inner.detect, PreparedDetect) and isinstance(inner.b0, PreparedConv2d)
    # deepcopy: the original keeps its BatchNorms
    assert isinstance(model.b0.bn, nn.BatchNorm2d)


def test_yolov8m_structure():
    p = matrixman.prepare(W.yolov8_model("m"))
    rep = p._matrixman_preparation_report
    assert rep.conv_units_prepared == 83 and rep.remaining_batch_norm_modules == 0


def test_resnet18_and_mlp_structure():
    p = matrixman.prepare(W.resnet18_model())
    rep = p._matrixman_preparation_report
    assert rep.folded == 20 and rep.block_units_prepared["BasicBlock"] == 8
    inner = _inner(p).model
    assert isinstance(inner.layer2[0], PreparedBasicBlock) and isinstance(inner.fc, PreparedLinear)
    assert isinstance(inner.conv1, PreparedConv2d) and isinstance(inner.relu, nn.Identity)
    p = matrixman.prepare(W.mlp_model())
    seq = _inner(p).model
    assert [type(m).__name__ for m in seq] == ["Flatten", "PreparedLinear", "Identity", "PreparedLinear",
                                               "Identity", "PreparedLinear"]
    assert seq[1].act == 1 and seq[5].act == 0


def test_inplace_and_training_rejected():
    m = W.yolov8_model("n")
    p = matrixman.prepare(m, inplace=True)
    assert isinstance(_inner(p).b0, PreparedConv2d)
    with pytest.raises(ValueError, match="eval"):
        matrixman.prepare(W.yolov8_model("n").train())
    with pytest.raises(NotImplementedError):
        matrixman.prepare(W.mlp_model(), training=True)
    with pytest.raises(TypeError):
        matrixman.prepare(object())


def test_prepared_units_reject_cpu_inputs():
    p = matrixman.prepare(W.mlp_model())
    with pytest.raises(RuntimeError, match="MatrixMan"):
        with torch.no_grad():
            p(torch.randn(2, 1, 28, 28))


def test_fold_equivalence_on_cpu():
    """Folded weights give the unfolded result on the CPU (prepare diagnostic,
    diagnostics/cuda_prepare_diagnostic.py:25-38)."""
    from matrixman_b200.preparation import fold_conv_bn
    torch.manual_seed(7)
    conv = nn.Conv2d(3, 4, 3, padding=1)
    bn = nn.BatchNorm2d(4).eval()
    W.randomize_bn(bn, 1)
    x = torch.randn(2, 3, 12, 12)
    w, b = fold_conv_bn(conv, bn)
    with torch.no_grad():
        assert torch.allclose(bn(conv(x)), nn.functional.conv2d(x, w, b, padding=1), atol=1e-5, rtol=1e-5)


def test_tf32_split_is_exact_and_round_nearest():
    from matrixman_b200.preparation import tf32_round_nearest
    g = torch.Generator().manual_seed(0)
    x = torch.randn(100000, generator=g) * torch.exp(torch.randn(100000, generator=g) * 5)
    hi = tf32_round_nearest(x)
    lo = x - hi
    assert torch.all((hi.view(torch.int32) & 0x1FFF) == 0)
    assert torch.equal(hi + lo, x)  # the split is exact
    ulp = torch.ldexp(torch.ones_like(x), torch.frexp(x)[1] - 11)  # tf32 ulp of |x|
    assert torch.all(lo.abs() <= ulp / 2)


def test_prepacked_layouts():
    conv = nn.Conv2d(8, 16, 3, padding=1, bias=False)
    unit = PreparedConv2d(conv, 2)
    assert tuple(unit.weight_krsc.shape) == (16, 3, 3, 8)
    assert torch.equal(unit.weight_krsc, conv.weight.detach().permute(0, 2, 3, 1))
    assert torch.equal(unit.bias, torch.zeros(16))
