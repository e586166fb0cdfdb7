"""YOLOv8-architecture detection model in plain PyTorch (fp32, NCHW).

Written from the public description of the architecture (scaling rule,
block table and head layout); it does not use or reproduce Ultralytics code.
Module class names and attribute names (Conv.conv/.bn/.act, C2f.c/.cv1/.cv2/.m,
Bottleneck.cv1/.cv2/.add, SPPF.cv1/.cv2/.m, Detect.nc/.nl/.reg_max/.stride/
.cv2/.cv3/.dfl, DFL.conv/.c1) follow the public Ultralytics layout so that
``matrixman.prepare`` recognises the same structures it would in an
Ultralytics model.

Scaling: channels = ceil(min(c, max_ch) * width / 8) * 8,
repeats = max(round(n * depth), 1).  n: width 0.25, depth 0.33, max_ch 1024;
m: width 0.75, depth 0.67, max_ch 768.

In eval mode ``forward`` returns the decoded predictions ``[B, 4 + nc, A]``
(xywh boxes in input pixels, then class probabilities) with
A = (H/8)(W/8) + (H/16)(W/16) + (H/32)(W/32).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

SCALES = {
    "n": (0.33, 0.25, 1024),
    "s": (0.33, 0.50, 1024),
    "m": (0.67, 0.75, 768),
    "l": (1.00, 1.00, 512),
    "x": (1.00, 1.25, 512),
}


def _ch(c: int, width: float, max_ch: int) -> int:
    return int(math.ceil(min(c, max_ch) * width / 8) * 8)


def _reps(n: int, depth: float) -> int:
    return max(round(n * depth), 1)


class Conv(nn.Module):
    """Conv2d (no bias) -> BatchNorm2d -> SiLU, padding k//2."""

    def __init__(self, c1: int, c2: int, k: int = 1, s: int = 1, act: bool = True):
        super().__init__()
        self.conv = nn.Conv2d(c1, c2, k, s, k // 2, bias=False)
        self.bn = nn.BatchNorm2d(c2, eps=1e-3, momentum=0.03)
        self.act = nn.SiLU() if act else nn.Identity()

    def forward(self, x):
        return self.act(self.bn(self.conv(x)))


class Bottleneck(nn.Module):
    """Two 3x3 Convs with an optional identity shortcut (added after the activation)."""

    def __init__(self, c1: int, c2: int, shortcut: bool = True):
        super().__init__()
        self.cv1 = Conv(c1, c2, 3)
        self.cv2 = Conv(c2, c2, 3)
        self.add = shortcut and c1 == c2

    def forward(self, x):
        y = self.cv2(self.cv1(x))
        return x + y if self.add else y


class C2f(nn.Module):
    """1x1 Conv to 2c channels, split in halves, n bottlenecks chained on the
    last half (each output kept), concat of (2+n)c channels, 1x1 Conv to c2."""

    def __init__(self, c1: int, c2: int, n: int = 1, shortcut: bool = False):
        super().__init__()
        self.c = c2 // 2
        self.cv1 = Conv(c1, 2 * self.c, 1)
        self.cv2 = Conv((2 + n) * self.c, c2, 1)
        self.m = nn.ModuleList(Bottleneck(self.c, self.c, shortcut) for _ in range(n))

    def forward(self, x):
        parts = list(self.cv1(x).chunk(2, 1))
        for m in self.m:
            parts.append(m(parts[-1]))
        return self.cv2(torch.cat(parts, 1))


class SPPF(nn.Module):
    """1x1 Conv to c1/2, three chained 5x5/s1/p2 max-pools, concat of the four, 1x1 Conv."""

    def __init__(self, c1: int, c2: int, k: int = 5):
        super().__init__()
        c_ = c1 // 2
        self.cv1 = Conv(c1, c_, 1)
        self.cv2 = Conv(c_ * 4, c2, 1)
        self.m = nn.MaxPool2d(kernel_size=k, stride=1, padding=k // 2)

    def forward(self, x):
        y = [self.cv1(x)]
        for _ in range(3):
            y.append(self.m(y[-1]))
        return self.cv2(torch.cat(y, 1))


class DFL(nn.Module):
    """Distribution focal loss integral: softmax over c1 bins, expectation with
    fixed weights 0..c1-1 as a 1x1 convolution."""

    def __init__(self, c1: int = 16):
        super().__init__()
        self.c1 = c1
        self.conv = nn.Conv2d(c1, 1, 1, bias=False).requires_grad_(False)
        with torch.no_grad():
            self.conv.weight.copy_(torch.arange(c1, dtype=torch.float32).view(1, c1, 1, 1))

    def forward(self, x):
        b, _, a = x.shape
        return self.conv(x.view(b, 4, self.c1, a).transpose(2, 1).softmax(1)).view(b, 4, a)


def make_anchors(feats, strides, offset: float = 0.5):
    """Anchor centres (x + 0.5, y + 0.5) per level, row-major, with per-anchor stride."""
    points, stride_t = [], []
    for f, s in zip(feats, strides):
        _, _, h, w = f.shape
        dev = f.device
        sx = torch.arange(w, dtype=torch.float32, device=dev) + offset
        sy = torch.arange(h, dtype=torch.float32, device=dev) + offset
        gy, gx = torch.meshgrid(sy, sx, indexing="ij")
        points.append(torch.stack((gx, gy), -1).view(-1, 2))
        stride_t.append(torch.full((h * w, 1), float(s), dtype=torch.float32, device=dev))
    return torch.cat(points), torch.cat(stride_t)


def dist2bbox(distance, anchor_points, dim: int = 1):
    """Left-top / right-bottom distances -> (cx, cy, w, h)."""
    lt, rb = distance.chunk(2, dim)
    x1y1 = anchor_points - lt
    x2y2 = anchor_points + rb
    return torch.cat(((x1y1 + x2y2) / 2, x2y2 - x1y1), dim)


class Detect(nn.Module):
    """Decoupled head over P3/P4/P5 with DFL box regression."""

    def __init__(self, nc: int = 80, ch=(), strides=(8.0, 16.0, 32.0)):
        super().__init__()
        self.nc = nc
        self.nl = len(ch)
        self.reg_max = 16
        self.no = nc + 4 * self.reg_max
        self.register_buffer("stride", torch.tensor(strides, dtype=torch.float32))
        c2 = max(16, ch[0] // 4, 4 * self.reg_max)
        c3 = max(ch[0], min(nc, 100))
        self.cv2 = nn.ModuleList(
            nn.Sequential(Conv(x, c2, 3), Conv(c2, c2, 3), nn.Conv2d(c2, 4 * self.reg_max, 1)) for x in ch)
        self.cv3 = nn.ModuleList(
            nn.Sequential(Conv(x, c3, 3), Conv(c3, c3, 3), nn.Conv2d(c3, nc, 1)) for x in ch)
        self.dfl = DFL(self.reg_max)

    def forward(self, x):
        x = list(x)
        for i in range(self.nl):
            x[i] = torch.cat((self.cv2[i](x[i]), self.cv3[i](x[i])), 1)
        b = x[0].shape[0]
        flat = torch.cat([xi.reshape(b, self.no, -1) for xi in x], 2)
        anchors, stride_t = make_anchors(x, self.stride.tolist())
        box, cls = flat.split((4 * self.reg_max, self.nc), 1)
        dbox = dist2bbox(self.dfl(box), anchors.transpose(0, 1).unsqueeze(0), dim=1) * stride_t.transpose(0, 1)
        return torch.cat((dbox, cls.sigmoid()), 1)


class YOLOv8(nn.Module):
    """Backbone (Conv/C2f/SPPF), PAN neck (nearest 2x upsample + concat), Detect head."""

    def __init__(self, variant: str = "n", nc: int = 80):
        super().__init__()
        depth, width, max_ch = SCALES[variant]
        c = lambda v: _ch(v, width, max_ch)  # noqa: E731
        r = lambda v: _reps(v, depth)  # noqa: E731
        self.variant = variant
        self.b0 = Conv(3, c(64), 3, 2)
        self.b1 = Conv(c(64), c(128), 3, 2)
        self.b2 = C2f(c(128), c(128), r(3), True)
        self.b3 = Conv(c(128), c(256), 3, 2)
        self.b4 = C2f(c(256), c(256), r(6), True)
        self.b5 = Conv(c(256), c(512), 3, 2)
        self.b6 = C2f(c(512), c(512), r(6), True)
        self.b7 = Conv(c(512), c(1024), 3, 2)
        self.b8 = C2f(c(1024), c(1024), r(3), True)
        self.b9 = SPPF(c(1024), c(1024), 5)
        self.up = nn.Upsample(scale_factor=2.0, mode="nearest")
        self.n12 = C2f(c(1024) + c(512), c(512), r(3), False)
        self.n15 = C2f(c(512) + c(256), c(256), r(3), False)
        self.n16 = Conv(c(256), c(256), 3, 2)
        self.n18 = C2f(c(256) + c(512), c(512), r(3), False)
        self.n19 = Conv(c(512), c(512), 3, 2)
        self.n21 = C2f(c(512) + c(1024), c(1024), r(3), False)
        self.detect = Detect(nc, (c(256), c(512), c(1024)))

    def forward(self, x):
        x = self.b1(self.b0(x))
        p3 = self.b4(self.b3(self.b2(x)))
        p4 = self.b6(self.b5(p3))
        p5 = self.b9(self.b8(self.b7(p4)))
        n12 = self.n12(torch.cat((self.up(p5), p4), 1))
        n15 = self.n15(torch.cat((self.up(n12), p3), 1))
        n18 = self.n18(torch.cat((self.n16(n15), n12), 1))
        n21 = self.n21(torch.cat((self.n19(n18), p5), 1))
        return self.detect([n15, n18, n21])


def conv_count(model: nn.Module) -> int:
    return sum(isinstance(m, nn.Conv2d) for m in model.modules()) - sum(
        isinstance(m, DFL) for m in model.modules())


def macs_per_image(model: nn.Module, h: int = 640, w: int = 640) -> int:
    """Multiply-accumulates of every Conv2d for one image (DFL excluded)."""
    total = 0
    hooks = []

    def hook(mod, inp, out):
        nonlocal total
        if isinstance(mod, nn.Conv2d) and not isinstance(getattr(mod, "_dfl_parent", None), DFL):
            k = mod.kernel_size[0] * mod.kernel_size[1] * (mod.in_channels // mod.groups)
            total += out.numel() // out.shape[0] * k
    for m in model.modules():
        if isinstance(m, DFL):
            m.conv._dfl_parent = m
        if isinstance(m, nn.Conv2d):
            hooks.append(m.register_forward_hook(hook))
    with torch.no_grad():
        model(torch.zeros(1, 3, h, w))
    for hk in hooks:
        hk.remove()
    return total
