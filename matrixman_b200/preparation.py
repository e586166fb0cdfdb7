"""``matrixman.prepare`` / ``matrixman.auto_prepare``: inference preparation.

Reference: drivers/matrixman/preparation.py.  What is kept:

* ``prepare(model, *, backend=None, inplace=False, diagnostics=False,
  training=False)`` returns a prepared **deepcopy** unless ``inplace``
  (preparation.py:488-526, 582-601), requires ``model.eval()``, and records a
  ``PreparationReport`` on the result (preparation.py:271-304).
* Conv+BN folding with the same arithmetic as ``_fold_pair``
  (preparation.py:360-398): ``scale = gamma / sqrt(var + eps)``,
  ``W' = W * scale``, ``b' = (b - mean) * scale + beta``, computed once on the CPU.
* ``auto_prepare`` returns a lazy wrapper that prepares on the first
  MatrixMan eval/no-grad call, cached by a model signature
  (preparation.py:22-114).

What is new (B200 design):

* Folding also covers ``Conv2d -> BatchNorm2d`` neighbours in ``nn.Sequential``
  and torchvision ResNet blocks (``convK``/``bnK``), which the reference left
  unfolded (it only matched modules named Conv/DWConv).
* Modules are replaced by prepared units that keep activations channels-last
  (NHWC) on the device and fuse bias + activation + residual into the
  convolution epilogue: ``PreparedConv2d`` (Conv+BN+SiLU/ReLU),
  ``PreparedC2f`` (concat written in place, bottleneck shortcut fused),
  ``PreparedSPPF`` (one fused 5/9/13 pooling kernel into the concat buffer),
  ``PreparedDetect`` (box/class branches write one feature buffer per level;
  DFL + dist2bbox + sigmoid in one kernel), ``PreparedBasicBlock`` (ResNet),
  ``PreparedLinear`` (GEMM + bias + ReLU).
* Weights are prepacked to KRSC (and to tf32 hi/lo planes for the tcgen05
  kernel) and uploaded once per device.
* With ``config.cuda_graphs`` the prepared forward is captured into a CUDA
  graph per (device, input shape) and replayed.
"""

from __future__ import annotations

import time
from collections import Counter
from copy import deepcopy
from dataclasses import dataclass, field
from weakref import WeakKeyDictionary

import torch
from torch import nn

from . import _lib, ops
from .config import config
from .tensor import MatrixManTensor, channels_last_strides, contiguous_strides

_MARKER = "_matrixman_preparation_kind"
_AUTO_CACHE: WeakKeyDictionary = WeakKeyDictionary()

ACT_OF = {nn.SiLU: _lib.ACT_SILU, nn.ReLU: _lib.ACT_RELU, nn.Sigmoid: _lib.ACT_SIGMOID,
          nn.Identity: _lib.ACT_NONE}


def _act_code(module) -> int | None:
    if module is None:
        return _lib.ACT_NONE
    for cls, code in ACT_OF.items():
        if type(module) is cls:
            return code
    return None


# ---------------------------------------------------------------------------
# Report
# ---------------------------------------------------------------------------

@dataclass
class PreparationReport:
    backend: str = "cuda"
    conv_bn_pairs_found: int = 0
    folded: int = 0
    skipped: int = 0
    original_batch_norm_modules: int = 0
    remaining_batch_norm_modules: int = 0
    conv_units_prepared: int = 0
    linear_units_prepared: int = 0
    block_units_prepared: Counter = field(default_factory=Counter)
    detection_head_prepared: int = 0
    skip_reasons: Counter = field(default_factory=Counter)

    def print(self) -> None:
        print(f"MatrixMan {self.backend.upper()} preparation (B200, inference-only)")
        print(f"  Conv+BN pairs found: {self.conv_bn_pairs_found}")
        print(f"  folded: {self.folded}")
        print(f"  skipped: {self.skipped}")
        print(f"  original BatchNorm modules: {self.original_batch_norm_modules}")
        print(f"  remaining BatchNorm modules: {self.remaining_batch_norm_modules}")
        print(f"  prepared conv units: {self.conv_units_prepared}")
        print(f"  prepared linear units: {self.linear_units_prepared}")
        for name, n in sorted(self.block_units_prepared.items()):
            print(f"  prepared {name} blocks: {n}")
        print(f"  detection heads prepared: {self.detection_head_prepared}")
        if self.skip_reasons:
            print("  skip reasons:")
            for reason, n in sorted(self.skip_reasons.items()):
                print(f"    {reason}: {n}")


# ---------------------------------------------------------------------------
# BatchNorm folding
# ---------------------------------------------------------------------------

def fold_conv_bn(conv: nn.Conv2d, bn: nn.BatchNorm2d) -> tuple[torch.Tensor, torch.Tensor]:
    """Folded (weight, bias); same arithmetic as the reference's _fold_pair."""
    with torch.no_grad():
        mean = bn.running_mean.detach()
        conv_bias = torch.zeros_like(mean) if conv.bias is None else conv.bias.detach()
        gamma = torch.ones_like(mean) if bn.weight is None else bn.weight.detach()
        beta = torch.zeros_like(mean) if bn.bias is None else bn.bias.detach()
        scale = gamma / torch.sqrt(bn.running_var.detach() + bn.eps)
        weight = conv.weight.detach() * scale.reshape(-1, 1, 1, 1)
        bias = (conv_bias - mean) * scale + beta
    return weight, bias


def _foldable(conv, bn, aliases, report) -> bool:
    report.conv_bn_pairs_found += 1
    reason = None
    if aliases[id(conv)] > 1 or aliases[id(bn)] > 1:
        reason = "shared_module_alias"
    elif conv.weight.dtype != torch.float32 or bn.running_mean is None or bn.running_var is None:
        reason = "unsupported_dtype_or_missing_running_stats"
    elif conv.weight.device.type != "cpu" or bn.running_mean.device.type != "cpu":
        reason = "non_cpu_parameter_device"
    elif conv.out_channels != bn.num_features:
        reason = "channel_count_mismatch"
    elif bn.training:
        reason = "batch_norm_training"
    if reason is not None:
        report.skipped += 1
        report.skip_reasons[reason] += 1
        return False
    return True


def _apply_fold(conv: nn.Conv2d, bn: nn.BatchNorm2d, report) -> None:
    w, b = fold_conv_bn(conv, bn)
    conv.weight = nn.Parameter(w, requires_grad=False)
    conv.bias = nn.Parameter(b, requires_grad=False)
    report.folded += 1


_RESNET_CLASSES = {"ResNet", "BasicBlock", "Bottleneck"}


def _is_torchvision_resnet(module) -> bool:
    return (type(module).__name__ in _RESNET_CLASSES
            and type(module).__module__.startswith("torchvision.models"))


def _fold_all(model: nn.Module, report: PreparationReport, aliases: Counter) -> None:
    for module in model.modules():
        # (1) Ultralytics-style Conv/DWConv: .conv + .bn (reference rule).
        conv, bn = getattr(module, "conv", None), getattr(module, "bn", None)
        if isinstance(conv, nn.Conv2d) and isinstance(bn, nn.BatchNorm2d) and \
                type(module).__name__ in {"Conv", "DWConv"}:
            if _foldable(conv, bn, aliases, report):
                _apply_fold(conv, bn, report)
                module.bn = nn.Identity()
            continue
        # (2) torchvision ResNet naming: convK feeds bnK only.
        if _is_torchvision_resnet(module):
            for k in ("1", "2", "3"):
                c, b = getattr(module, "conv" + k, None), getattr(module, "bn" + k, None)
                if isinstance(c, nn.Conv2d) and isinstance(b, nn.BatchNorm2d):
                    if _foldable(c, b, aliases, report):
                        _apply_fold(c, b, report)
                        setattr(module, "bn" + k, nn.Identity())
        # (3) Sequential neighbours.
        if isinstance(module, nn.Sequential):
            keys = list(module._modules.keys())
            for i in range(len(keys) - 1):
                c, b = module._modules[keys[i]], module._modules[keys[i + 1]]
                if isinstance(c, nn.Conv2d) and isinstance(b, nn.BatchNorm2d):
                    if _foldable(c, b, aliases, report):
                        _apply_fold(c, b, report)
                        module._modules[keys[i + 1]] = nn.Identity()


# ---------------------------------------------------------------------------
# Prepared units
# ---------------------------------------------------------------------------

def _copy_routing_attrs(dst: nn.Module, src: nn.Module | None) -> None:
    """Keep graph-routing metadata (Ultralytics stores `f`, `i`, `type`, `np` on layers)."""
    if src is None:
        return
    for key, value in src.__dict__.items():
        if not key.startswith("_") and key != "training" and not hasattr(dst, key):
            try:
                setattr(dst, key, value)
            except Exception:
                pass


def _nhwc(shape) -> tuple:
    return channels_last_strides(shape)


def _channel_slice(buf: MatrixManTensor, start: int, stop: int) -> MatrixManTensor:
    shape = list(buf.shape)
    shape[1] = stop - start
    return MatrixManTensor._from_owner(buf._owner, tuple(shape),
                                       buf._storage_offset + start * buf._logical_strides[1],
                                       buf._logical_strides)


def tf32_round_nearest(x: torch.Tensor) -> torch.Tensor:
    """Round fp32 values to tf32 (10-bit mantissa), nearest with ties away from
    zero: add half a tf32 ulp to the magnitude bits, then clear the 13 low bits
    (a carry into the exponent is the correct rounding).  Finite inputs only."""
    bits = x.contiguous().view(torch.int32)
    rounded = (bits + 0x1000) & -8192
    return rounded.view(torch.float32)


class PreparedConv2d(nn.Module):
    """Conv2d (+ folded BN) + activation (+ residual) as one fused kernel.

    Weights are prepacked KRSC ([K, R, S, C] contiguous) and uploaded once per
    device.  Outputs are channels-last unless the caller passes ``out``
    (e.g. a channel slice of a concat buffer).
    """

    def __init__(self, conv: nn.Conv2d, act: int, weight=None, bias=None, source=None):
        super().__init__()
        w = (conv.weight if weight is None else weight).detach().to(torch.float32)
        b = conv.bias if bias is None else bias
        self.out_channels, self.in_per_group, self.kh, self.kw = (int(v) for v in w.shape)
        self.in_channels = int(conv.in_channels)
        self.stride = tuple(conv.stride)
        self.padding = tuple(conv.padding) if not isinstance(conv.padding, str) else None
        if self.padding is None:
            raise NotImplementedError("MatrixMan/CUDA: string padding is not supported by prepare")
        self.dilation = tuple(conv.dilation)
        self.groups = int(conv.groups)
        self.act = int(act)
        self.register_buffer("weight_krsc", w.permute(0, 2, 3, 1).contiguous(), persistent=True)
        self.register_buffer("bias", (b.detach().to(torch.float32).contiguous() if b is not None
                                      else torch.zeros(self.out_channels)), persistent=True)
        self._device_weights: dict[int, tuple] = {}
        _copy_routing_attrs(self, source)

    def extra_repr(self) -> str:
        act = {0: "none", 1: "relu", 2: "silu", 3: "sigmoid"}[self.act]
        return (f"{self.in_channels}, {self.out_channels}, kernel=({self.kh}, {self.kw}), "
                f"stride={self.stride}, padding={self.padding}, groups={self.groups}, act={act}")

    @property
    def tc_eligible(self) -> bool:
        """The tcgen05 kernel covers ungrouped convolutions with C % 4 == 0."""
        return self.groups == 1 and self.in_channels % 4 == 0

    def tc_planes(self) -> tuple[torch.Tensor, torch.Tensor, int, int]:
        """[K_pad, R*S*C_pad] tf32 high part and fp32 remainder of the weights
        (C padded to a multiple of 32, K to a multiple of 16, zeros)."""
        k, r, s, c = (int(v) for v in self.weight_krsc.shape)
        c_pad = (c + 31) // 32 * 32
        k_pad = (k + 15) // 16 * 16
        packed = torch.zeros(k_pad, r, s, c_pad, dtype=torch.float32)
        packed[:k, :, :, :c] = self.weight_krsc
        packed = packed.reshape(k_pad, r * s * c_pad).contiguous()
        hi = tf32_round_nearest(packed)
        lo = packed - hi
        return hi.contiguous(), lo.contiguous(), c_pad, k_pad

    def device_weights(self, rt):
        entry = self._device_weights.get(rt.index)
        if entry is None:
            w_store = rt.upload(self.weight_krsc, kind=_lib.POOL_PARAMETER, sync=True)
            k, r, s, c = (int(v) for v in self.weight_krsc.shape)
            w_view = MatrixManTensor(w_store, (k, c, r, s), 0, (r * s * c, 1, s * c, c))
            b_store = rt.upload(self.bias, kind=_lib.POOL_PARAMETER, sync=True)
            b_view = MatrixManTensor(b_store, (k,), 0, (1,))
            tc = None
            if self.tc_eligible:
                hi, lo, c_pad, k_pad = self.tc_planes()
                hs = rt.upload(hi, kind=_lib.POOL_PARAMETER, sync=True)
                ls = rt.upload(lo, kind=_lib.POOL_PARAMETER, sync=True)
                tc = (MatrixManTensor(hs, tuple(hi.shape), 0, (hi.shape[1], 1)),
                      MatrixManTensor(ls, tuple(lo.shape), 0, (lo.shape[1], 1)), c_pad, k_pad)
            entry = (w_view, b_view, tc)
            self._device_weights[rt.index] = entry
        return entry

    def forward(self, x, out=None, residual=None, residual_before_act=False):
        if not isinstance(x, MatrixManTensor):
            raise RuntimeError("PreparedConv2d requires a MatrixMan CUDA tensor")
        w, b, tc = self.device_weights(x.runtime)
        if out is None:
            n, _, h, wd = (int(v) for v in x.shape)
            oh, ow = ops.conv_output_hw(h, wd, self.kh, self.kw, self.stride, self.padding,
                                        self.dilation)
            shape = (n, self.out_channels, oh, ow)
            out = ops.empty(x.runtime, shape, _nhwc(shape))
        if tc is not None and config.convAlgo != "simt" and not config.cudaDisableSpecializedConv:
            hi, lo, c_pad, k_pad = tc
            if ops.conv_tc(x, hi, lo, self.out_channels, self.in_channels, self.kh, self.kw, c_pad,
                           k_pad, b, self.stride, self.padding, self.dilation, self.act, residual,
                           residual_before_act, out):
                return out
            if config.convAlgo == "tc":
                raise NotImplementedError("MatrixMan/CUDA: conv_algo='tc' but this convolution's "
                                          "layout is not covered by the tensor-core kernel")
        return ops.convolution(x, w, b, self.stride, self.padding, self.dilation, self.groups,
                               act=self.act, residual=residual,
                               residual_before_act=residual_before_act, out=out)


class PreparedLinear(nn.Module):
    """Linear (+ ReLU/SiLU) as one GEMM with a fused epilogue.

    The GEMM runs on the tcgen05 3xTF32 kernel as a 1x1 convolution over the
    [M, K] row-major activation (one "pixel" per row) when K % 4 == 0 and the
    rows are 16-byte aligned; otherwise on the SIMT GEMM (reference semantics
    of addmm: backends/opengl/ops/matmul.py:262-281)."""

    def __init__(self, linear: nn.Linear, act: int = _lib.ACT_NONE, source=None):
        super().__init__()
        self.in_features = int(linear.in_features)
        self.out_features = int(linear.out_features)
        self.act = int(act)
        self.register_buffer("weight_kn", linear.weight.detach().t().contiguous().to(torch.float32))
        self.register_buffer("bias", linear.bias.detach().to(torch.float32).contiguous()
                             if linear.bias is not None else torch.zeros(self.out_features))
        self._device_weights: dict[int, tuple] = {}
        _copy_routing_attrs(self, source)

    @property
    def tc_eligible(self) -> bool:
        return self.in_features % 4 == 0

    def tc_planes(self) -> tuple[torch.Tensor, torch.Tensor, int, int]:
        """[N_pad, K_pad] tf32 high part and fp32 remainder of W (zero padded)."""
        n, k = self.out_features, self.in_features
        k_pad = (k + 31) // 32 * 32
        n_pad = (n + 15) // 16 * 16
        packed = torch.zeros(n_pad, k_pad, dtype=torch.float32)
        packed[:n, :k] = self.weight_kn.t()
        hi = tf32_round_nearest(packed)
        return hi.contiguous(), (packed - hi).contiguous(), k_pad, n_pad

    def device_weights(self, rt):
        entry = self._device_weights.get(rt.index)
        if entry is None:
            ws = rt.upload(self.weight_kn, kind=_lib.POOL_PARAMETER, sync=True)
            bs = rt.upload(self.bias, kind=_lib.POOL_PARAMETER, sync=True)
            tc = None
            if self.tc_eligible:
                hi, lo, k_pad, n_pad = self.tc_planes()
                hs = rt.upload(hi, kind=_lib.POOL_PARAMETER, sync=True)
                ls = rt.upload(lo, kind=_lib.POOL_PARAMETER, sync=True)
                tc = (MatrixManTensor(hs, tuple(hi.shape), 0, (hi.shape[1], 1)),
                      MatrixManTensor(ls, tuple(lo.shape), 0, (lo.shape[1], 1)), k_pad, n_pad)
            entry = (MatrixManTensor(ws, tuple(self.weight_kn.shape), 0,
                                     contiguous_strides(tuple(self.weight_kn.shape))),
                     MatrixManTensor(bs, (self.out_features,), 0, (1,)), tc)
            self._device_weights[rt.index] = entry
        return entry

    def _gemm_tc(self, x2: MatrixManTensor, bias: MatrixManTensor, tc) -> MatrixManTensor | None:
        m, k = (int(v) for v in x2.shape)
        rs, cs = x2._logical_strides
        if cs != 1:
            return None
        hi, lo, k_pad, n_pad = tc
        n = self.out_features
        out = ops.empty(x2.runtime, (m, n))
        x4 = MatrixManTensor(x2._owner, (m, k, 1, 1), x2._storage_offset, (rs, 1, rs, rs))
        y4 = MatrixManTensor(out._owner, (m, n, 1, 1), out._storage_offset, (n, 1, n, n))
        if ops.conv_tc(x4, hi, lo, n, k, 1, 1, k_pad, n_pad, bias, (1, 1), (0, 0), (1, 1), self.act,
                       None, False, y4):
            return out
        return None

    def forward(self, x):
        if not isinstance(x, MatrixManTensor):
            raise RuntimeError("PreparedLinear requires a MatrixMan CUDA tensor")
        w, b, tc = self.device_weights(x.runtime)
        lead = tuple(int(v) for v in x.shape[:-1])
        x2 = x
        if x.dim() != 2:
            x2 = x.reshape(-1, self.in_features)
        y = None
        if tc is not None and config.convAlgo != "simt" and not config.cudaDisableSpecializedConv:
            y = self._gemm_tc(x2, b, tc)
        if y is None:
            y = ops.gemm(x2, w, b, act=self.act)
        if x.dim() != 2:
            y = y.view(*lead, self.out_features)
        return y


def _conv_unit(module) -> PreparedConv2d | None:
    """Ultralytics-style Conv (conv, bn=Identity after folding, act)."""
    conv, bn, act = getattr(module, "conv", None), getattr(module, "bn", None), getattr(module, "act", None)
    if not isinstance(conv, nn.Conv2d) or not isinstance(bn, nn.Identity):
        return None
    code = _act_code(act)
    if code is None:
        return None
    return PreparedConv2d(conv, code, source=module)


class PreparedC2f(nn.Module):
    """C2f: cv1 -> split -> n bottlenecks -> concat -> cv2, with the concat
    buffer written in place by every producer and the bottleneck shortcut
    fused into its second convolution."""

    def __init__(self, module, cv1: PreparedConv2d, cv2: PreparedConv2d, blocks, source=None):
        super().__init__()
        self.c = int(module.c)
        self.cv1 = cv1
        self.cv2 = cv2
        self.m = nn.ModuleList(blocks)  # each: (cv1, cv2, add)
        self.shortcut = [bool(getattr(b, "add", False)) for b in module.m]
        _copy_routing_attrs(self, source)

    @property
    def out_channels(self) -> int:
        return self.cv2.out_channels

    def forward(self, x, out=None):
        n_, _, h, w = (int(v) for v in x.shape)
        k = len(self.m)
        c = self.c
        shape = (n_, (2 + k) * c, h, w)
        buf = ops.empty(x.runtime, shape, _nhwc(shape))
        self.cv1(x, out=_channel_slice(buf, 0, 2 * c))
        for i, blk in enumerate(self.m):
            inp = _channel_slice(buf, (1 + i) * c, (2 + i) * c)
            t = blk.cv1(inp)
            blk.cv2(t, out=_channel_slice(buf, (2 + i) * c, (3 + i) * c),
                    residual=inp if self.shortcut[i] else None)
        return self.cv2(buf, out=out)


class _BottleneckPair(nn.Module):
    def __init__(self, cv1, cv2):
        super().__init__()
        self.cv1 = cv1
        self.cv2 = cv2


class PreparedSPPF(nn.Module):
    """SPPF: cv1 into slice 0 of the concat buffer, then one fused kernel
    writes the three chained 5x5 max-pools into slices 1..3, then cv2."""

    def __init__(self, cv1: PreparedConv2d, cv2: PreparedConv2d, source=None):
        super().__init__()
        self.cv1 = cv1
        self.cv2 = cv2
        _copy_routing_attrs(self, source)

    @property
    def out_channels(self) -> int:
        return self.cv2.out_channels

    def forward(self, x, out=None):
        n_, _, h, w = (int(v) for v in x.shape)
        c = self.cv1.out_channels
        shape = (n_, 4 * c, h, w)
        buf = ops.empty(x.runtime, shape, _nhwc(shape))
        s0 = _channel_slice(buf, 0, c)
        self.cv1(x, out=s0)
        s1, s2, s3 = (_channel_slice(buf, i * c, (i + 1) * c) for i in (1, 2, 3))
        ops._launch("mm_sppf_pool", ops._p(s0.desc()), ops._p(s1.desc()), ops._p(s2.desc()),
                    ops._p(s3.desc()), x.runtime.stream)
        return self.cv2(buf, out=out)


class PreparedDetect(nn.Module):
    """YOLOv8 decoupled head: per level the box and class branches write one
    [B, H, W, 4*reg_max + nc] buffer; one kernel decodes all levels into
    [B, 4 + nc, A] (DFL softmax/expectation, dist2bbox, stride, sigmoid)."""

    def __init__(self, module, box_branches, cls_branches, source=None):
        super().__init__()
        self.nc = int(module.nc)
        self.reg_max = int(module.reg_max)
        self.nl = int(module.nl)
        self.box = nn.ModuleList([nn.ModuleList(b) for b in box_branches])
        self.cls = nn.ModuleList([nn.ModuleList(c) for c in cls_branches])
        self.strides = [float(s) for s in torch.as_tensor(module.stride).flatten().tolist()]
        _copy_routing_attrs(self, source)

    def forward(self, xs):
        feats = []
        nb = 4 * self.reg_max
        for i in range(self.nl):
            x = xs[i]
            n_, _, h, w = (int(v) for v in x.shape)
            shape = (n_, nb + self.nc, h, w)
            buf = ops.empty(x.runtime, shape, _nhwc(shape))
            b = x
            for j, conv in enumerate(self.box[i]):
                b = conv(b, out=_channel_slice(buf, 0, nb) if j == len(self.box[i]) - 1 else None)
            c = x
            for j, conv in enumerate(self.cls[i]):
                c = conv(c, out=_channel_slice(buf, nb, nb + self.nc) if j == len(self.cls[i]) - 1 else None)
            feats.append(buf)
        n_ = int(feats[0].shape[0])
        anchors = sum(int(f.shape[2]) * int(f.shape[3]) for f in feats)
        out = ops.empty(feats[0].runtime, (n_, 4 + self.nc, anchors))
        import ctypes
        descs = [f.desc() for f in feats]
        arr = (ctypes.POINTER(_lib.MMTensor) * len(descs))(*[ctypes.pointer(d) for d in descs])
        strides = (ctypes.c_float * len(feats))(*self.strides[:len(feats)])
        ops._launch("mm_yolo_decode", arr, strides, len(feats), self.reg_max, self.nc,
                    ops._p(out.desc()), out.runtime.stream)
        return out


class PreparedBasicBlock(nn.Module):
    """torchvision BasicBlock: relu(bn2(conv2(relu(bn1(conv1 x)))) + identity)
    as two fused convolutions (residual + ReLU in the second epilogue)."""

    def __init__(self, conv1: PreparedConv2d, conv2: PreparedConv2d, downsample, source=None):
        super().__init__()
        self.conv1 = conv1
        self.conv2 = conv2
        self.downsample = downsample
        _copy_routing_attrs(self, source)

    def forward(self, x):
        identity = x if self.downsample is None else self.downsample(x)
        t = self.conv1(x)
        return self.conv2(t, residual=identity, residual_before_act=True)


class PreparedResBottleneck(nn.Module):
    """torchvision Bottleneck (1x1 -> 3x3 -> 1x1, expansion 4) with fused epilogues."""

    def __init__(self, conv1, conv2, conv3, downsample, source=None):
        super().__init__()
        self.conv1, self.conv2, self.conv3 = conv1, conv2, conv3
        self.downsample = downsample
        _copy_routing_attrs(self, source)

    def forward(self, x):
        identity = x if self.downsample is None else self.downsample(x)
        return self.conv3(self.conv2(self.conv1(x)), residual=identity, residual_before_act=True)


class PreparedYOLOv8(nn.Module):
    """Whole-model forward of a YOLOv8-architecture detector (backbone
    b0..b9, PAN neck n12..n21 with nearest 2x upsamples and four
    concatenations, Detect head) with every concatenation written in place:
    each of the four neck concat buffers is allocated before its first
    producer runs, and the producers -- the C2f and SPPF outputs, the two
    upsamples and the two stride-2 neck convolutions -- write their channel
    slices of it directly; consumers read those slices as views.  The
    unprepared forward materialises each concatenation with a copy.

    Concatenation layout (channels, in torch.cat order):
      cat12 = [up(p5) | p4] at P4, cat15 = [up(n12) | p3] at P3,
      cat18 = [n16(n15) | n12] at P4, cat21 = [n19(n18) | p5] at P5."""

    def __init__(self, model: nn.Module, source=None):
        super().__init__()
        self.m = model
        up = model.up
        self.scale = float(up.scale_factor if not isinstance(up.scale_factor, tuple) else up.scale_factor[0])
        _copy_routing_attrs(self, source)

    @staticmethod
    def eligible(model: nn.Module) -> bool:
        names = ("b0", "b1", "b2", "b3", "b4", "b5", "b6", "b7", "b8", "b9", "up", "n12", "n15",
                 "n16", "n18", "n19", "n21", "detect")
        if type(model).__name__ != "YOLOv8" or not all(hasattr(model, n) for n in names):
            return False
        convs = ("b0", "b1", "b3", "b5", "b7", "n16", "n19")
        c2fs = ("b2", "b4", "b6", "b8", "n12", "n15", "n18", "n21")
        up = model.up
        return (all(isinstance(getattr(model, n), PreparedConv2d) for n in convs)
                and all(isinstance(getattr(model, n), PreparedC2f) for n in c2fs)
                and isinstance(model.b9, PreparedSPPF) and isinstance(model.detect, PreparedDetect)
                and isinstance(up, nn.Upsample) and up.mode == "nearest" and up.size is None
                and up.scale_factor is not None
                and float(up.scale_factor if not isinstance(up.scale_factor, tuple)
                          else up.scale_factor[0]) == 2.0)

    def __getattr__(self, name):
        # The wrapped model's layers stay reachable (prepared.b2, .detect, ...).
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(self._modules["m"], name)

    def _up(self, x, out):
        n_, c, h, w = (int(v) for v in x.shape)
        return ops.upsample_nearest2d(x, (int(h * self.scale), int(w * self.scale)), self.scale,
                                      self.scale, out=out)

    def forward(self, x):
        m = self.m
        c_p3, c_p4, c_p5 = m.b4.out_channels, m.b6.out_channels, m.b9.out_channels
        c_n12, c_n16, c_n19 = m.n12.out_channels, m.n16.out_channels, m.n19.out_channels
        rt = x.runtime

        def cat_buffer(like, channels):
            n_, _, h, w = (int(v) for v in like.shape)
            shape = (n_, channels, h, w)
            return ops.empty(rt, shape, _nhwc(shape))

        t = m.b3(m.b2(m.b1(m.b0(x))))
        cat15 = cat_buffer(t, c_n12 + c_p3)
        p3 = m.b4(t, out=_channel_slice(cat15, c_n12, c_n12 + c_p3))
        t = m.b5(p3)
        cat12 = cat_buffer(t, c_p5 + c_p4)
        p4 = m.b6(t, out=_channel_slice(cat12, c_p5, c_p5 + c_p4))
        t = m.b8(m.b7(p4))
        cat21 = cat_buffer(t, c_n19 + c_p5)
        p5 = m.b9(t, out=_channel_slice(cat21, c_n19, c_n19 + c_p5))
        self._up(p5, _channel_slice(cat12, 0, c_p5))
        cat18 = cat_buffer(cat12, c_n16 + c_n12)
        n12 = m.n12(cat12, out=_channel_slice(cat18, c_n16, c_n16 + c_n12))
        self._up(n12, _channel_slice(cat15, 0, c_n12))
        n15 = m.n15(cat15)
        m.n16(n15, out=_channel_slice(cat18, 0, c_n16))
        n18 = m.n18(cat18)
        m.n19(n18, out=_channel_slice(cat21, 0, c_n19))
        n21 = m.n21(cat21)
        return m.detect([n15, n18, n21])


def _downsample_unit(ds):
    """Sequential(Conv2d, Identity-after-fold) -> PreparedConv2d (no act)."""
    if ds is None:
        return None
    mods = [m for m in ds if not isinstance(m, nn.Identity)] if isinstance(ds, nn.Sequential) else [ds]
    if len(mods) == 1 and isinstance(mods[0], nn.Conv2d):
        return PreparedConv2d(mods[0], _lib.ACT_NONE)
    return None


# ---------------------------------------------------------------------------
# Module replacement
# ---------------------------------------------------------------------------

def _replace(parent: nn.Module, report: PreparationReport, aliases: Counter) -> None:
    for name, module in list(parent.named_children()):
        cls = type(module).__name__
        if aliases[id(module)] > 1:
            report.skip_reasons["shared_module_alias"] += 1
            _replace(module, report, aliases)
            continue
        prepared = None
        if cls in {"Conv", "DWConv"}:
            prepared = _conv_unit(module)
            if prepared is not None:
                report.conv_units_prepared += 1
        elif cls == "C2f" and hasattr(module, "cv1") and hasattr(module, "m"):
            cv1, cv2 = _conv_unit(module.cv1), _conv_unit(module.cv2)
            blocks = []
            ok = cv1 is not None and cv2 is not None
            for b in module.m:
                b1, b2 = _conv_unit(getattr(b, "cv1", None)), _conv_unit(getattr(b, "cv2", None))
                if b1 is None or b2 is None:
                    ok = False
                    break
                blocks.append(_BottleneckPair(b1, b2))
            if ok:
                prepared = PreparedC2f(module, cv1, cv2, blocks, source=module)
                report.conv_units_prepared += 2 + 2 * len(blocks)
                report.block_units_prepared["C2f"] += 1
        elif cls == "SPPF":
            cv1, cv2 = _conv_unit(module.cv1), _conv_unit(module.cv2)
            pool = getattr(module, "m", None)
            if cv1 is not None and cv2 is not None and isinstance(pool, nn.MaxPool2d) and \
                    _pair(pool.kernel_size) == (5, 5) and _pair(pool.stride) == (1, 1) and \
                    _pair(pool.padding) == (2, 2) and _pair(pool.dilation) == (1, 1) and not pool.ceil_mode:
                prepared = PreparedSPPF(cv1, cv2, source=module)
                report.conv_units_prepared += 2
                report.block_units_prepared["SPPF"] += 1
        elif cls == "Detect" and hasattr(module, "cv2") and hasattr(module, "cv3"):
            boxes, clss = [], []
            ok = True
            for i in range(int(module.nl)):
                bseq, cseq = [], []
                for seq, dst in ((module.cv2[i], bseq), (module.cv3[i], cseq)):
                    for m in seq:
                        if type(m).__name__ in {"Conv", "DWConv"}:
                            u = _conv_unit(m)
                        elif isinstance(m, nn.Conv2d):
                            u = PreparedConv2d(m, _lib.ACT_NONE)
                        else:
                            u = None
                        if u is None:
                            ok = False
                            break
                        dst.append(u)
                boxes.append(bseq)
                clss.append(cseq)
            dfl = getattr(module, "dfl", None)
            if ok and dfl is not None and int(getattr(module, "reg_max", 0)) > 1:
                prepared = PreparedDetect(module, boxes, clss, source=module)
                report.detection_head_prepared += 1
                report.conv_units_prepared += sum(len(b) + len(c) for b, c in zip(boxes, clss))
        elif _is_torchvision_resnet(module) and cls == "BasicBlock":
            c1 = PreparedConv2d(module.conv1, _lib.ACT_RELU) if isinstance(module.bn1, nn.Identity) else None
            c2 = PreparedConv2d(module.conv2, _lib.ACT_RELU) if isinstance(module.bn2, nn.Identity) else None
            ds = _downsample_unit(module.downsample)
            if c1 is not None and c2 is not None and (module.downsample is None or ds is not None):
                prepared = PreparedBasicBlock(c1, c2, ds, source=module)
                report.conv_units_prepared += 2 + (ds is not None)
                report.block_units_prepared["BasicBlock"] += 1
        elif _is_torchvision_resnet(module) and cls == "Bottleneck":
            convs = []
            for k in ("1", "2", "3"):
                bn = getattr(module, "bn" + k)
                convs.append(PreparedConv2d(getattr(module, "conv" + k), _lib.ACT_RELU)
                             if isinstance(bn, nn.Identity) else None)
            ds = _downsample_unit(module.downsample)
            if all(convs) and (module.downsample is None or ds is not None):
                prepared = PreparedResBottleneck(*convs, ds, source=module)
                report.conv_units_prepared += 3 + (ds is not None)
                report.block_units_prepared["Bottleneck"] += 1
        if prepared is not None:
            setattr(parent, name, prepared)
            continue
        _replace(module, report, aliases)
    # Containers: fuse Conv2d/Linear with a following activation.
    if isinstance(parent, nn.Sequential):
        keys = list(parent._modules.keys())
        i = 0
        while i < len(keys):
            m = parent._modules[keys[i]]
            nxt = parent._modules[keys[i + 1]] if i + 1 < len(keys) else None
            code = _act_code(nxt) if nxt is not None and not isinstance(nxt, nn.Identity) else None
            if isinstance(m, nn.Conv2d) and aliases[id(m)] <= 1:
                parent._modules[keys[i]] = PreparedConv2d(m, code if code is not None else _lib.ACT_NONE)
                report.conv_units_prepared += 1
                if code is not None:
                    parent._modules[keys[i + 1]] = nn.Identity()
                    i += 1
            elif isinstance(m, nn.Linear) and aliases[id(m)] <= 1:
                parent._modules[keys[i]] = PreparedLinear(m, code if code is not None else _lib.ACT_NONE)
                report.linear_units_prepared += 1
                if code is not None:
                    parent._modules[keys[i + 1]] = nn.Identity()
                    i += 1
            i += 1
    # torchvision ResNet root: conv1 -> bn1 -> relu is a fixed sequence.
    if _is_torchvision_resnet(parent) and type(parent).__name__ == "ResNet":
        if isinstance(parent.conv1, nn.Conv2d) and isinstance(parent.bn1, nn.Identity):
            parent.conv1 = PreparedConv2d(parent.conv1, _lib.ACT_RELU)
            parent.relu = nn.Identity()
            report.conv_units_prepared += 1
        if isinstance(parent.fc, nn.Linear):
            parent.fc = PreparedLinear(parent.fc)
            report.linear_units_prepared += 1


def _pair(v):
    return tuple(v) if isinstance(v, (tuple, list)) else (v, v)


# ---------------------------------------------------------------------------
# CUDA-graph execution of a prepared model
# ---------------------------------------------------------------------------

def _tensors_in(obj):
    if isinstance(obj, MatrixManTensor):
        yield obj
    elif isinstance(obj, (list, tuple)):
        for o in obj:
            yield from _tensors_in(o)
    elif isinstance(obj, dict):
        for o in obj.values():
            yield from _tensors_in(o)


def _map_tensors(obj, fn):
    if isinstance(obj, MatrixManTensor):
        return fn(obj)
    if isinstance(obj, list):
        return [_map_tensors(o, fn) for o in obj]
    if isinstance(obj, tuple):
        return tuple(_map_tensors(o, fn) for o in obj)
    if isinstance(obj, dict):
        return {k: _map_tensors(v, fn) for k, v in obj.items()}
    return obj


class _GraphEntry:
    def __init__(self):
        self.calls = 0
        self.graph = None
        self.static_input = None
        self.static_output = None


class GraphedForward:
    """Runs a prepared forward eagerly once per input signature (uploads,
    kernel selection, allocation), captures it into a CUDA graph on the
    second call, and replays it afterwards.  Inputs are copied into the
    graph's static input buffer; outputs are returned as fresh tensors
    (``copy_outputs=True``) or as the graph's static buffers, valid until the
    next call."""

    def __init__(self, forward, copy_outputs: bool = True):
        self.forward = forward
        self.copy_outputs = copy_outputs
        self.entries: dict[tuple, _GraphEntry] = {}

    def _key(self, x: MatrixManTensor):
        return (x.runtime.index, tuple(x.shape), x._logical_strides)

    def __call__(self, x, *args, **kwargs):
        if (not config.cudaGraphs or args or kwargs or not isinstance(x, MatrixManTensor)
                or torch.is_grad_enabled() and x.requires_grad):
            return self.forward(x, *args, **kwargs)
        key = self._key(x)
        entry = self.entries.setdefault(key, _GraphEntry())
        rt = x.runtime
        if entry.graph is None:
            entry.calls += 1
            if entry.calls < 2:
                return self.forward(x)
            static_in = ops.empty(rt, x.shape, x._logical_strides)
            ops.copy_into(x, static_in)
            rt.synchronize()
            rt.capture_begin()
            try:
                static_out = self.forward(static_in)
            except Exception:
                try:
                    rt.capture_end()
                except Exception:
                    pass
                raise
            entry.graph = rt.capture_end()
            entry.static_input = static_in
            entry.static_output = static_out
        else:
            if x.element_ptr != entry.static_input.element_ptr:
                ops.copy_into(x, entry.static_input)
        entry.graph.replay()
        if self.copy_outputs:
            return _map_tensors(entry.static_output, lambda t: ops.clone(t))
        return entry.static_output

    def release(self) -> None:
        for e in self.entries.values():
            if e.graph is not None:
                e.graph.destroy()
        self.entries.clear()


class PreparedModel(nn.Module):
    """Wrapper returned by ``prepare`` when graphs are enabled; delegates
    attribute access to the prepared module."""

    def __init__(self, module: nn.Module):
        super().__init__()
        self.module = module
        self._graphed = GraphedForward(module.forward)

    def forward(self, x, *args, **kwargs):
        return self._graphed(x, *args, **kwargs)

    def __getattr__(self, name):
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(self._modules["module"], name)


# ---------------------------------------------------------------------------
# Public entry points
# ---------------------------------------------------------------------------

def _alias_counts(model: nn.Module) -> Counter:
    counts: Counter = Counter()
    for _name, m in model.named_modules(remove_duplicate=False):
        counts[id(m)] += 1
    return counts


def _prepare_model(model: nn.Module, *, inplace: bool, diagnostics: bool) -> nn.Module:
    if not isinstance(model, nn.Module):
        raise TypeError("matrixman.prepare requires a torch.nn.Module")
    if model.training:
        raise ValueError("matrixman.prepare_cuda requires model.eval(); training BatchNorm is not foldable")
    if getattr(model, _MARKER, None):
        return model
    target = model if inplace else deepcopy(model)
    report = PreparationReport(
        original_batch_norm_modules=sum(isinstance(m, nn.BatchNorm2d) for m in target.modules()))
    _fold_all(target, report, _alias_counts(target))
    if config.preparedExecution:
        _replace(target, report, _alias_counts(target))
        if PreparedYOLOv8.eligible(target):
            target = PreparedYOLOv8(target, source=target)
            report.block_units_prepared["YOLOv8 in-place neck"] += 1
    report.remaining_batch_norm_modules = sum(isinstance(m, nn.BatchNorm2d) for m in target.modules())
    target.eval()
    if diagnostics:
        report.print()
    result = PreparedModel(target) if config.cudaGraphs else target
    result.eval()
    object.__setattr__(result, "_matrixman_preparation_report", report)
    object.__setattr__(result, _MARKER, "explicit" if inplace else "explicit-copy")
    return result


def prepare(model: nn.Module, *, backend: str | None = None, inplace: bool = False,
            diagnostics: bool = False, training: bool = False) -> nn.Module:
    """Prepare an eval model for the B200 backend (see module docstring)."""
    if training:
        raise NotImplementedError("matrixman training preparation requires the OpenGL backend, "
                                  "which is unavailable on this build")
    name = str(backend or "cuda").strip().lower()
    if name == "opengl":
        raise NotImplementedError("MatrixMan/B200 provides the CUDA backend only")
    if name != "cuda":
        raise ValueError("matrixman.prepare supports backend='cuda' or backend='opengl'")
    return _prepare_model(model, inplace=inplace, diagnostics=diagnostics)


def prepare_cuda(model: nn.Module, *, inplace: bool = False, diagnostics: bool = False):
    return prepare(model, backend="cuda", inplace=inplace, diagnostics=diagnostics)


def prepare_opengl(model: nn.Module, *, inplace: bool = False, diagnostics: bool = False):
    raise NotImplementedError("MatrixMan/B200 provides the CUDA backend only")


def _model_signature(model: nn.Module) -> tuple:
    params = tuple((n, id(p), int(p._version), int(p.data_ptr()), tuple(p.shape))
                   for n, p in model.named_parameters(remove_duplicate=False))
    bufs = tuple((n, id(b), int(b._version), int(b.data_ptr()), tuple(b.shape))
                 for n, b in model.named_buffers(remove_duplicate=False))
    mods = tuple((n, type(m).__qualname__, m.training) for n, m in model.named_modules())
    return mods, params, bufs


class LazyPreparedModel(nn.Module):
    """Prepares on the first MatrixMan eval/no-grad call (reference preparation.py:75-114)."""

    def __init__(self, model: nn.Module):
        super().__init__()
        if not isinstance(model, nn.Module):
            raise TypeError("matrixman.auto_prepare requires a torch.nn.Module")
        self.model = model

    def forward(self, *args, **kwargs):
        x = args[0] if args else kwargs.get("x")
        if not isinstance(x, MatrixManTensor) or getattr(self.model, _MARKER, None) \
                or config.disableAutoPrepare or self.model.training or torch.is_grad_enabled():
            return self.model(*args, **kwargs)
        sig = _model_signature(self.model)
        entry = _AUTO_CACHE.get(self.model)
        if entry is None or entry[0] != sig:
            t0 = time.perf_counter()
            prepared = prepare(self.model)
            object.__setattr__(prepared, _MARKER, "lazy")
            _AUTO_CACHE[self.model] = (sig, prepared)
            if config.debug or config.trace:
                print(f"[MatrixMan] auto-prepare: prepared in {(time.perf_counter() - t0) * 1e3:.1f} ms")
            entry = _AUTO_CACHE[self.model]
        return entry[1](*args, **kwargs)


def auto_prepare(model: nn.Module) -> LazyPreparedModel:
    if isinstance(model, LazyPreparedModel):
        return model
    return LazyPreparedModel(model)
