"""Backend-neutral public functions (reference drivers/matrixman/backend.py:78-266).

``init/shutdown/prefer/tensor/to_device/randn`` keep the reference's names,
argument meaning and errors.  The device is a B200 addressed as
``matrixman:<index>``; ``to_device`` accepts an optional ``device`` index so
data-parallel replicas can place batch slices on other GPUs.
"""

from __future__ import annotations

import warnings

import torch

from . import runtime
from .config import config, set_preferred_backend
from .factories import install_privateuse1_factory_kernels
from .tensor import MatrixManTensor, contiguous_strides


class Backend:
    """Selected-backend record (reference backend.py:8-50); only CUDA exists here."""

    name = "cuda"

    def device_info(self, index: int = 0) -> dict:
        rt = runtime.get_runtime(index)
        return {"backend": "CUDA", "device": rt.info["name"],
                "compute_capability": rt.info["compute_capability"],
                "memory_mib": rt.info["memory_mib"], "sm_count": rt.info["sm_count"]}

    def synchronize(self, index: int | None = None) -> None:
        runtime.get_runtime(index).synchronize()


_backend: Backend | None = None


def _banner(rt) -> None:
    if config.trace or config.debug:
        print("MatrixMan CUDA runtime (B200):")
        print(f"  device: {rt.index} {rt.info['name']} (sm_{rt.info['compute_capability'].replace('.', '')},"
              f" {rt.info['sm_count']} SMs, {rt.info['memory_mib']} MiB)")
        print(f"  sync policy: {config.resolved_sync_policy}")
        print(f"  activation pool: {config.activationPool}; scratch pool: {config.scratchPool}")
        print(f"  cuda graphs: {'enabled' if config.cudaGraphs else 'disabled'}")


def active_backend() -> Backend | None:
    return _backend


def get_backend() -> Backend:
    global _backend
    if _backend is None:
        if config.backend not in ("auto", "cuda"):
            raise RuntimeError(f"MatrixMan backend {config.backend!r} is unavailable on this build")
        install_privateuse1_factory_kernels()
        from .privateuse import register_native_hooks
        register_native_hooks()  # C++ DeviceGuard + hooks (indexing, pin_memory)
        rt = runtime.get_runtime(runtime.current_device())
        _banner(rt)
        _backend = Backend()
    return _backend


def init() -> None:
    get_backend()


def shutdown() -> None:
    global _backend
    runtime.shutdown()
    _backend = None


def prefer(name: str):
    requested = str(name).strip().lower()
    if requested not in {"auto", "cuda", "opengl"}:
        raise ValueError("MatrixMan backend must be 'auto', 'cuda', or 'opengl'")
    if requested == "opengl":
        raise RuntimeError("MatrixMan/B200 provides the CUDA backend only; the OpenGL backend is "
                           "unavailable on this build")
    current = active_backend()
    set_preferred_backend(requested)
    return current


def _device_index(device) -> int:
    if device is None:
        return runtime.current_device()
    if isinstance(device, int):
        return device
    dev = torch.device(device)
    if dev.type not in ("matrixman", "privateuseone"):
        raise RuntimeError("MatrixMan/CUDA: tensor only creates tensors on the MatrixMan device")
    return dev.index or 0


def tensor(data, *, device=None) -> MatrixManTensor:
    """Upload CPU data (float32/int64, contiguous) to a matrixman device."""
    get_backend()
    idx = _device_index(device)
    if not isinstance(data, torch.Tensor):
        data = torch.tensor(data, dtype=torch.float32)
    rt = runtime.get_runtime(idx)
    owner = rt.upload(data)
    return MatrixManTensor._from_owner(owner, tuple(data.shape), 0, contiguous_strides(tuple(data.shape)))


def to_device(data, device=None) -> MatrixManTensor:
    return tensor(data, device=device)


def to_gm45(data):
    warnings.warn("matrixman.to_gm45() is deprecated; use matrixman.to_device() instead",
                  DeprecationWarning, stacklevel=2)
    return to_device(data)


def randn(*shape: int, seed: int | None = None) -> MatrixManTensor:
    generator = torch.Generator(device="cpu")
    if seed is not None:
        generator.manual_seed(seed)
    if len(shape) == 1:
        shape = (shape[0], shape[0])
    return tensor(torch.randn(shape, dtype=torch.float32, generator=generator))


def pinned_empty(shape, dtype=torch.float32) -> torch.Tensor:
    """A CPU tensor in page-locked memory (cudaHostAlloc), freed with the tensor.

    Uploads from such buffers are asynchronous copy-engine transfers."""
    import ctypes
    import weakref

    from . import _lib
    lib = _lib.load()
    shape = tuple(int(s) for s in shape)
    n = 1
    for s in shape:
        n *= s
    nbytes = max(n, 1) * torch.empty((), dtype=dtype).element_size()
    ptr = ctypes.c_void_p()
    _lib.check(lib.mm_host_alloc_pinned(nbytes, ctypes.byref(ptr)), "pinned host allocation")
    buf = (ctypes.c_uint8 * nbytes).from_address(ptr.value)
    t = torch.frombuffer(buf, dtype=dtype, count=max(n, 1))[:n].view(shape)
    weakref.finalize(buf, lib.mm_host_free_pinned, ctypes.c_void_p(ptr.value))
    t._matrixman_pinned_buffer = buf  # keeps the mapping alive with the tensor
    return t


def synchronize(device=None) -> None:
    runtime.get_runtime(_device_index(device)).synchronize()


def device_count() -> int:
    return runtime.device_count()


def debug_enabled() -> bool:
    return bool(config.debug)


def unsupported_report() -> dict:
    return {}


def reset_unsupported_report() -> None:
    return None


def raw_texture(data):
    raise NotImplementedError("MatrixMan/CUDA: raw_texture is an OpenGL-only diagnostic")


def gpu_postprocess_detection(value):
    """[B, 4+classes, anchors] -> [B, 6, anchors] on the device (box, best
    score, best class); see ``matrixman_b200.detect``."""
    from .detect import reduce_detection_output

    return reduce_detection_output(value)
