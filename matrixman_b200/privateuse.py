"""PrivateUse1 registration of the ``matrixman`` device.

Same contract as drivers/matrixman/privateuse.py:39-60 (rename
``privateuseone`` -> ``matrixman`` and register a device module), except that
the device module reports the real number of CUDA devices, so ``matrixman:0``
.. ``matrixman:7`` address the eight B200s of one node.  The C++ hooks /
DeviceGuard extension (csrc/privateuse1_hooks.cpp, replacing
native/autograd_privateuse1.cpp) is loaded from the in-tree build.
"""

from __future__ import annotations

import importlib.util
from pathlib import Path

import torch

_registered = False
_native = None


class MatrixManDeviceModule:
    """Device module exposed as ``torch.matrixman``."""

    @staticmethod
    def is_available() -> bool:
        from . import runtime
        return runtime.device_count() > 0

    @staticmethod
    def device_count() -> int:
        from . import runtime
        return runtime.device_count()

    @staticmethod
    def current_device() -> int:
        from . import runtime
        return runtime.current_device()

    @staticmethod
    def set_device(index) -> None:
        from . import runtime
        runtime.set_device(int(index))

    @staticmethod
    def synchronize(device=None) -> None:
        from . import runtime
        idx = runtime.current_device() if device is None else torch.device(device).index or 0
        runtime.get_runtime(idx).synchronize()

    @staticmethod
    def is_initialized() -> bool:
        return True

    @staticmethod
    def _is_in_bad_fork() -> bool:
        return False

    @staticmethod
    def manual_seed_all(seed: int) -> None:
        del seed

    @staticmethod
    def get_amp_supported_dtype():
        return [torch.float32]


def register_privateuse1_backend() -> None:
    global _registered
    if _registered:
        return
    current = torch._C._get_privateuse1_backend_name()
    if current == "privateuseone":
        torch.utils.rename_privateuse1_backend("matrixman")
    elif current != "matrixman":
        raise RuntimeError(f"PrivateUse1 is already registered as {current!r}, not 'matrixman'")
    try:
        torch._register_device_module("matrixman", MatrixManDeviceModule)
    except RuntimeError:
        if not hasattr(torch, "matrixman"):
            raise
    _registered = True


_devices: dict[int, torch.device] = {}


def device_for(index: int) -> torch.device:
    dev = _devices.get(index)
    if dev is None:
        dev = torch.device("matrixman", int(index))
        _devices[index] = dev
    return dev


def register_native_hooks() -> bool:
    """Load the in-tree C++ hooks extension and register it with torch."""
    global _native
    if _native is not None:
        return True
    from . import _lib
    _lib.load()  # the hooks resolve mm_* symbols from the global namespace
    libdir = Path(__file__).resolve().parent / "_lib"
    candidates = sorted(libdir.glob("_matrixman_hooks*.so"))
    if not candidates:
        raise RuntimeError("MatrixMan/B200: C++ PrivateUse1 hooks not built; run "
                           "`python -m matrixman_b200.build`")
    spec = importlib.util.spec_from_file_location("_matrixman_hooks", candidates[0])
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    module.register_hooks()
    # The guard's stream waits are bounded like every other host wait.
    from .config import config
    module.set_wait_timeout_ms(int(config.waitTimeoutMs))
    _native = module
    return True
