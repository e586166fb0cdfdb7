"""ATen factory kernels for the ``matrixman`` PrivateUse1 key.

Same role as drivers/matrixman/backends/cuda/factories.py:76-269 (registered
with ``torch.library.Library("aten", "IMPL", "PrivateUse1")``): factories
that receive no MatrixMan tensor argument (``torch.empty(..., device=
"matrixman")``, ``torch.arange(..., device="matrixman")``, the empty
placeholders batch_norm creates) reach these kernels instead of
``__torch_dispatch__``.
"""

from __future__ import annotations

import math

import torch

_library = None


def _runtime(device):
    from .runtime import get_runtime
    dev = torch.device(device) if device is not None else torch.device("matrixman", 0)
    return get_runtime(dev.index or 0)


def _dtype(dtype, storage_only: bool = False):
    """float32/int64 for computed factories; any dtype for empty storage."""
    dtype = torch.float32 if dtype is None else dtype
    if not storage_only and dtype not in (torch.float32, torch.int64):
        raise NotImplementedError(f"MatrixMan/CUDA: unsupported factory dtype {dtype}")
    return dtype


def _empty_memory_format(size, dtype=None, layout=None, device=None, pin_memory=None,
                         memory_format=None):
    from . import ops
    from .tensor import channels_last_strides, contiguous_strides
    shape = tuple(int(s) for s in size)
    strides = (channels_last_strides(shape) if memory_format is torch.channels_last and len(shape) == 4
               else contiguous_strides(shape))
    return ops.empty(_runtime(device), shape, strides, _dtype(dtype, storage_only=True))


def _empty_strided(size, stride, dtype=None, layout=None, device=None, pin_memory=None):
    from . import ops
    return ops.empty(_runtime(device), tuple(int(s) for s in size), tuple(int(s) for s in stride),
                     _dtype(dtype, storage_only=True))


def _full(size, fill_value, dtype=None, layout=None, device=None, pin_memory=None):
    from . import ops
    return ops.full(_runtime(device), tuple(int(s) for s in size), float(fill_value), _dtype(dtype))


def _arange_start_step(start, end, step=1, dtype=None, layout=None, device=None, pin_memory=None):
    from . import ops
    if dtype is None:
        is_int = all(isinstance(v, int) for v in (start, end, step))
        dtype = torch.int64 if is_int else torch.float32
    n = max(int(math.ceil((float(end) - float(start)) / float(step))), 0)
    out = ops.empty(_runtime(device), (n,), None, _dtype(dtype))
    if n:
        ops.arange_into(out, start, step)
    return out


def _arange(end, dtype=None, layout=None, device=None, pin_memory=None):
    return _arange_start_step(0, end, 1, dtype, layout, device, pin_memory)


def _arange_start(start, end, dtype=None, layout=None, device=None, pin_memory=None):
    return _arange_start_step(start, end, 1, dtype, layout, device, pin_memory)


def install_privateuse1_factory_kernels() -> None:
    global _library
    if _library is not None:
        return
    lib = torch.library.Library("aten", "IMPL", "PrivateUse1")
    lib.impl("empty.memory_format", _empty_memory_format)
    lib.impl("empty_strided", _empty_strided)
    lib.impl("full", _full)
    lib.impl("arange", _arange)
    lib.impl("arange.start", _arange_start)
    lib.impl("arange.start_step", _arange_start_step)
    _library = lib
