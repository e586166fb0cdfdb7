"""Whole-workload CPU runs (unprepared, BatchNorm unfolded) -- test
infrastructure and the timed CPU baseline only.

The reference treats stock PyTorch CPU fp32 as ground truth for whole models
(diagnostics/matrixman_yolo_backend_compare.py:219-264 compares per-module
dumps against it with allclose(1e-4) and the relative_max measure).
"""

from __future__ import annotations

import os
import time

import torch


def run_cpu(model: torch.nn.Module, x: torch.Tensor, threads: int | None = None) -> torch.Tensor:
    if threads is not None:
        torch.set_num_threads(int(threads))
    with torch.no_grad():
        return model.eval()(x)


def time_cpu(model: torch.nn.Module, x: torch.Tensor, iters: int = 3, warmup: int = 1,
             threads: int | None = None) -> dict:
    """Median wall time of `iters` forwards after `warmup` (time.perf_counter)."""
    if threads is not None:
        torch.set_num_threads(int(threads))
    model = model.eval()
    times = []
    with torch.no_grad():
        for _ in range(warmup):
            model(x)
        for _ in range(iters):
            t0 = time.perf_counter()
            model(x)
            times.append(time.perf_counter() - t0)
    times.sort()
    return {"median_s": times[len(times) // 2], "times_s": times,
            "threads": torch.get_num_threads(), "cpu_count": os.cpu_count()}


def cpu_model_name() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"
