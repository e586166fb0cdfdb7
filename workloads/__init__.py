"""Synthetic workloads of the benchmark configurations (user-side models).

Every builder is seeded; no dataset or checkpoint is used (none is
available offline).  Configurations:

* ``conv1``  -- single conv [1,4,320,320] * [5,4,3,3], s1 p1, no bias, x ~ U[-1,1],
  weight Kaiming-uniform (the reference's conv demo shape).
* ``mlp``    -- Flatten, Linear 784-512-256-10 with ReLU, softmax; batch 256,
  inputs N(0,1) clipped to [-3,3].
* ``resnet18`` -- torchvision ResNet-18 (random init), BN running_mean ~ N(0, 0.1^2),
  running_var ~ U(0.5, 1.5), gamma 1, beta 0, softmax head; inputs U[0,1]
  normalised with the ImageNet mean/std; batch 32, 224x224.
* ``yolov8n`` / ``yolov8m`` -- YOLOv8-architecture detectors, 640x640 U[0,1]
  inputs, BN statistics randomised as above.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .yolov8 import YOLOv8

IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def _gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    return g


def randomize_bn(model: nn.Module, seed: int) -> nn.Module:
    g = _gen(seed)
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, nn.BatchNorm2d):
                m.running_mean.copy_(torch.randn(m.num_features, generator=g) * 0.1)
                m.running_var.copy_(torch.rand(m.num_features, generator=g) + 0.5)
                if m.weight is not None:
                    m.weight.fill_(1.0)
                if m.bias is not None:
                    m.bias.fill_(0.0)
    return model


class Softmaxed(nn.Module):
    """model followed by softmax over dim 1."""

    def __init__(self, model: nn.Module):
        super().__init__()
        self.model = model

    def forward(self, x):
        return F.softmax(self.model(x), dim=1)


# -- config 1: single conv ---------------------------------------------------

def conv1_case(seed: int = 0):
    g = _gen(seed)
    x = torch.rand(1, 4, 320, 320, generator=g) * 2 - 1
    w = torch.empty(5, 4, 3, 3)
    torch.manual_seed(seed)
    conv = nn.Conv2d(4, 5, 3, 1, 1, bias=False)
    w.copy_(conv.weight.detach())
    return x, w


# -- config 2: MLP ---------------------------------------------------------------

def mlp_model(seed: int = 1) -> nn.Module:
    torch.manual_seed(seed)
    body = nn.Sequential(nn.Flatten(), nn.Linear(784, 512), nn.ReLU(), nn.Linear(512, 256), nn.ReLU(),
                         nn.Linear(256, 10))
    return Softmaxed(body).eval()


def mlp_input(batch: int = 256, seed: int = 11) -> torch.Tensor:
    return torch.randn(batch, 1, 28, 28, generator=_gen(seed)).clamp_(-3, 3)


# -- config 3: ResNet-18 -----------------------------------------------------------

def resnet18_model(seed: int = 2) -> nn.Module:
    import torchvision
    torch.manual_seed(seed)
    m = torchvision.models.resnet18(weights=None)
    randomize_bn(m, seed + 100)
    return Softmaxed(m).eval()


def resnet18_input(batch: int = 32, seed: int = 12, size: int = 224) -> torch.Tensor:
    x = torch.rand(batch, 3, size, size, generator=_gen(seed))
    mean = torch.tensor(IMAGENET_MEAN).view(1, 3, 1, 1)
    std = torch.tensor(IMAGENET_STD).view(1, 3, 1, 1)
    return ((x - mean) / std).contiguous()


# -- configs 4/5: YOLOv8 --------------------------------------------------------------

def yolov8_model(variant: str = "n", seed: int = 3, nc: int = 80) -> nn.Module:
    torch.manual_seed(seed)
    m = YOLOv8(variant, nc)
    randomize_bn(m, seed + 100)
    return m.eval()


def yolo_input(batch: int = 1, seed: int = 13, size: int = 640) -> torch.Tensor:
    return torch.rand(batch, 3, size, size, generator=_gen(seed))


def macs_per_sample(model: nn.Module, sample: torch.Tensor) -> int:
    """Multiply-accumulates of every Conv2d and Linear for one input sample
    (a batch-1 CPU tensor), counted with forward hooks (the YOLOv8 DFL's fixed
    1x1 convolution excluded, as in ``yolov8.macs_per_image``)."""
    from .yolov8 import DFL
    total = 0
    hooks = []
    dfl_convs = {id(m.conv) for m in model.modules() if isinstance(m, DFL)}

    def hook(mod, inp, out):
        nonlocal total
        if id(mod) in dfl_convs:
            return
        if isinstance(mod, nn.Conv2d):
            k = mod.kernel_size[0] * mod.kernel_size[1] * (mod.in_channels // mod.groups)
            total += out.numel() // out.shape[0] * k
        elif isinstance(mod, nn.Linear):
            total += out.numel() // out.shape[0] * mod.in_features
    for m in model.modules():
        if isinstance(m, (nn.Conv2d, nn.Linear)):
            hooks.append(m.register_forward_hook(hook))
    with torch.no_grad():
        model(sample)
    for hk in hooks:
        hk.remove()
    return total
