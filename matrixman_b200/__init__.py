"""matrixman_b200 -- B200-native (sm_100a) implementation of MatrixMan's
PrivateUse1 tensor-op backend.

Drop-in for the public API of ``drivers.matrixman`` (reference
drivers/matrixman/__init__.py:8-96): ``import matrixman_b200 as matrixman``.
Tensors live on the ``matrixman`` device, results come back only through
``.cpu()``, unsupported ops raise, and ``prepare`` folds BatchNorm and prepacks
weights for the tcgen05 / SIMT kernels in libmatrixman_b200.so.
"""

from __future__ import annotations

import sys
import types

from . import config as _config_module
from .api import (
    debug_enabled,
    device_count,
    get_backend,
    gpu_postprocess_detection,
    init,
    pinned_empty,
    prefer,
    randn,
    raw_texture,
    reset_unsupported_report,
    shutdown,
    synchronize,
    tensor,
    to_device,
    to_gm45,
    unsupported_report,
)
from .pipeline import infer, infer_stream
from .detect import postprocess_detections
from .frames import preprocess_frames
from .preparation import auto_prepare, prepare, prepare_cuda, prepare_opengl
from .tensor import Gm45Tensor, MatrixManTensor, install_tensor_method, is_matrixman_tensor

config = _config_module.config
set_profiling = _config_module.set_profiling
set_tracing = _config_module.set_trace
set_trace = _config_module.set_trace


def is_gm45_tensor(value) -> bool:
    import warnings
    warnings.warn("is_gm45_tensor() is deprecated; use is_matrixman_tensor() instead",
                  DeprecationWarning, stacklevel=2)
    return is_matrixman_tensor(value)


def profile_enabled() -> bool:
    from . import telemetry as profiling
    return profiling.enabled()


def profile_report(frame_count: int | None = None) -> str:
    from . import telemetry as profiling
    return profiling.report(frame_count)


def profile_reset() -> None:
    from . import telemetry as profiling
    profiling.reset()


def select_backend():
    return get_backend()


class _MatrixManModule(types.ModuleType):
    """Module attribute assignments for profile/trace update the configuration
    (reference __init__.py:36-61)."""

    def __getattribute__(self, name):
        if name == "profile":
            return _config_module.profile_mode()
        if name == "profiling":
            return _config_module.config.profiling
        if name == "trace":
            return _config_module.config.trace
        return super().__getattribute__(name)

    def __setattr__(self, name, value):
        if name == "profile":
            _config_module.config._set("profile", value)
            return
        if name == "profiling":
            _config_module.set_profiling(value)
            return
        if name == "trace":
            _config_module.set_trace(value)
            return
        super().__setattr__(name, value)


sys.modules[__name__].__class__ = _MatrixManModule

__all__ = [
    "infer",
    "infer_stream",
    "postprocess_detections",
    "preprocess_frames",
    "MatrixManTensor", "Gm45Tensor", "auto_prepare", "config", "debug_enabled", "device_count",
    "gpu_postprocess_detection", "init", "install_tensor_method", "is_gm45_tensor",
    "is_matrixman_tensor", "prefer", "prepare", "prepare_cuda", "prepare_opengl", "profile",
    "profile_enabled", "profile_report", "profile_reset", "profiling", "randn", "raw_texture",
    "reset_unsupported_report", "select_backend", "set_profiling", "set_trace", "set_tracing",
    "shutdown", "synchronize", "tensor", "to_device", "to_gm45", "trace", "unsupported_report",
]
