"""Tolerance checks used by the parity tests -- test infrastructure only.

* ``max_rel_err``: max|actual - expected| / max|expected| per tensor -- the
  reference's ``relative_max`` (diagnostics/matrixman_yolo_backend_compare.py:244);
  bar 1e-4 for conv/GEMM and whole models.
* ``max_ulp``: largest distance in units in the last place (fp32), with
  ulp(e) = spacing(|e|); bar 4 for activations/softmax.
* bit-exact comparisons use ``torch.equal`` on the raw values (NaN positions
  compared separately).
"""

from __future__ import annotations

import numpy as np
import torch

CONV_GEMM_REL = 1e-4
ULP_BAR = 4


def max_rel_err(actual: torch.Tensor, expected: torch.Tensor) -> float:
    a = actual.detach().double()
    e = expected.detach().double()
    denom = e.abs().max().item()
    diff = (a - e).abs().max().item()
    if denom == 0.0:
        return diff
    return diff / denom


def ulp_distance(actual: torch.Tensor, expected: torch.Tensor) -> np.ndarray:
    a = actual.detach().float().numpy().astype(np.float64)
    e = expected.detach().float().numpy().astype(np.float32)
    sp = np.spacing(np.abs(e)).astype(np.float64)
    return np.abs(a - e.astype(np.float64)) / sp


def max_ulp(actual: torch.Tensor, expected: torch.Tensor) -> float:
    d = ulp_distance(actual, expected)
    return float(d.max()) if d.size else 0.0


def bit_exact(actual: torch.Tensor, expected: torch.Tensor) -> bool:
    a = actual.detach()
    e = expected.detach()
    if a.shape != e.shape or a.dtype != e.dtype:
        return False
    an, en = torch.isnan(a), torch.isnan(e)
    if not torch.equal(an, en):
        return False
    return torch.equal(torch.where(an, torch.zeros_like(a), a), torch.where(en, torch.zeros_like(e), e))
