"""Per-device runtime: device init, the runtime stream, storage owners, copies,
the parameter cache and CUDA-graph capture, on top of libmatrixman_b200.

Replaces the Python side of the reference's CudaExecutionBackend
(drivers/matrixman/backends/cuda/gpumatrix.py:4549-5100) and the storage
owner / parameter cache of the CUDA backend façade
(drivers/matrixman/backends/cuda/backend.py:60-96, 241-294).
"""

from __future__ import annotations

import ctypes
import threading
import weakref

import torch

from . import _lib
from .config import config

_runtimes: dict[int, "DeviceRuntime"] = {}
_lock = threading.Lock()
_current_device = threading.local()

DTYPE_CODES = {torch.float32: _lib.MM_F32, torch.int64: _lib.MM_I64}


class _ElementSize(dict):
    """Bytes per element for any torch dtype (storage-only tensors such as the
    uint8 placeholders ATen's batch_norm composite allocates)."""

    def __missing__(self, dtype):
        size = torch.empty((), dtype=dtype).element_size()
        self[dtype] = size
        return size


ELEMENT_SIZE = _ElementSize({torch.float32: 4, torch.int64: 8})


def any_initialized() -> bool:
    return bool(_runtimes)


def device_count() -> int:
    lib = _lib.load(required=False)
    if lib is None:
        return 0
    n = ctypes.c_int(0)
    if lib.mm_device_count(ctypes.byref(n)) != _lib.MM_OK:
        return 0
    return int(n.value)


def current_device() -> int:
    return int(getattr(_current_device, "index", 0))


def set_device(index: int) -> None:
    _current_device.index = int(index)
    if index in _runtimes:
        _lib.call("mm_set_device", int(index))
        _active_device.index = int(index)


# Stream -> device of every initialised runtime; launches make the stream's
# device current before enqueuing, so tensors of several devices can be used
# from one thread (whole-model replicas).
_stream_device: dict[int, int] = {}
_active_device = threading.local()


def activate_stream(stream) -> None:
    """Make the CUDA device that owns `stream` current on this thread."""
    dev = _stream_device.get(stream)
    if dev is not None and getattr(_active_device, "index", -1) != dev:
        _lib.call("mm_set_device", dev)
        _active_device.index = dev


def get_runtime(index: int | None = None) -> "DeviceRuntime":
    index = current_device() if index is None else int(index)
    rt = _runtimes.get(index)
    if rt is None:
        with _lock:
            rt = _runtimes.get(index)
            if rt is None:
                rt = DeviceRuntime(index)
                _runtimes[index] = rt
    return rt


def initialized_runtimes() -> list["DeviceRuntime"]:
    return list(_runtimes.values())


def shutdown(index: int | None = None) -> None:
    with _lock:
        targets = list(_runtimes) if index is None else [int(index)]
        for i in targets:
            rt = _runtimes.pop(i, None)
            if rt is not None:
                rt.close()


class DeviceStorage:
    """Owns one arena block on one device (the reference's CudaTensorOwner).

    ``layout.numel`` / ``layout.kind`` keep the reference's owner attributes
    (backends/cuda/backend.py:22-27, 60-96) so metadata checks read the same.
    """

    class _Layout:
        __slots__ = ("numel", "kind")

        def __init__(self, numel: int):
            self.numel = numel
            self.kind = "cuda_linear"

    __slots__ = ("runtime", "pointer", "nbytes", "dtype", "kind", "layout", "_released",
                 "__weakref__", "keepalive")

    def __init__(self, runtime: "DeviceRuntime", pointer: int, nbytes: int, dtype: torch.dtype,
                 kind: int):
        self.runtime = runtime
        self.pointer = int(pointer)
        self.nbytes = int(nbytes)
        self.dtype = dtype
        self.kind = kind
        self.layout = DeviceStorage._Layout(nbytes // ELEMENT_SIZE[dtype])
        self._released = False
        self.keepalive = None

    @property
    def device_index(self) -> int:
        return self.runtime.index

    @property
    def storage_description(self) -> str:
        return f"cuda_ptr=0x{self.pointer:x}, device={self.runtime.index}"

    def release(self) -> None:
        if self._released or self.pointer == 0:
            return
        self._released = True
        rt = self.runtime
        if rt.closed:
            return
        rt.free(self.pointer)

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class DeviceRuntime:
    """One CUDA device: runtime stream, arena, parameter cache."""

    def __init__(self, index: int):
        lib = _lib.load()
        self.lib = lib
        self.index = int(index)
        _lib.check(lib.mm_init(self.index), f"initialise device {self.index}")
        s = ctypes.c_void_p()
        _lib.check(lib.mm_runtime_stream(self.index, ctypes.byref(s)), "runtime stream")
        self.stream = s.value
        _stream_device[self.stream] = self.index
        _active_device.index = -1  # mm_init may have changed the current device
        info = _lib.MMDeviceInfo()
        _lib.check(lib.mm_device_info(self.index, ctypes.byref(info)), "device info")
        self.info = {
            "name": info.name.decode(),
            "compute_capability": f"{info.cc_major}.{info.cc_minor}",
            "sm_count": int(info.sm_count),
            "memory_mib": int(info.total_bytes // (1 << 20)),
        }
        policy = config.resolved_sync_policy
        _lib.check(lib.mm_pool_configure(
            self.index,
            1 if policy == "safe" else 0,
            1 if config.activationPool == "deferred" else 0,
            1 if config.scratchPool == "deferred" else 0,
            1 if config.cudaDisableAllocPool else 0,
        ), "configure pool")
        self.closed = False
        self._param_cache: dict[tuple, tuple] = {}
        self.capturing = False
        self.launch_count = 0

    # -- memory ----------------------------------------------------------
    def alloc(self, nbytes: int, kind: int = _lib.POOL_ACTIVATION, stream=None) -> int:
        """Arena block ordered on ``stream`` (default: the runtime stream);
        under the safe sync policy a reused block makes that stream wait for
        the block's release event."""
        out = ctypes.c_void_p()
        _lib.check(self.lib.mm_alloc(self.index, max(int(nbytes), 1), kind,
                                     self.stream if stream is None else stream,
                                     ctypes.byref(out)), "allocate")
        return int(out.value)

    def free(self, pointer: int) -> None:
        _lib.check(self.lib.mm_free(ctypes.c_void_p(pointer), self.stream), "free")

    def new_storage(self, numel: int, dtype: torch.dtype = torch.float32,
                    kind: int = _lib.POOL_ACTIVATION, stream=None) -> DeviceStorage:
        nbytes = max(int(numel), 1) * ELEMENT_SIZE[dtype]
        return DeviceStorage(self, self.alloc(nbytes, kind, stream), nbytes, dtype, kind)

    def pool_stats(self) -> dict:
        st = _lib.MMPoolStats()
        _lib.check(self.lib.mm_pool_stats(self.index, ctypes.byref(st)), "pool stats")
        return st.as_dict()

    def trim(self) -> None:
        _lib.check(self.lib.mm_pool_trim(self.index), "trim pool")

    # -- copies ------------------------------------------------------------
    def upload(self, data: torch.Tensor, kind: int = _lib.POOL_ACTIVATION,
               sync: bool = False) -> DeviceStorage:
        """Copy a contiguous CPU tensor into a new arena block."""
        if data.device.type != "cpu":
            raise RuntimeError("MatrixMan/CUDA: tensor upload requires a CPU tensor")
        if data.dtype not in DTYPE_CODES:
            raise TypeError(f"MatrixMan/CUDA: unsupported tensor dtype {data.dtype}; "
                            "only float32 is supported")
        if not data.is_contiguous():
            raise RuntimeError("MatrixMan/CUDA: tensor upload requires a contiguous tensor")
        storage = self.new_storage(data.numel(), data.dtype, kind)
        nbytes = data.numel() * data.element_size()
        flag = ctypes.c_int(0)
        self.lib.mm_host_is_pinned(ctypes.c_void_p(data.data_ptr()), ctypes.byref(flag))
        pinned = bool(flag.value)
        # A pageable source is staged by the driver before the call returns; a
        # pinned source is read asynchronously, so the owner keeps it alive.
        if pinned and not sync:
            storage.keepalive = data
        _lib.check(self.lib.mm_memcpy_h2d(ctypes.c_void_p(storage.pointer),
                                          ctypes.c_void_p(data.data_ptr()), nbytes,
                                          self.stream, 1 if sync else 0),
                   "host-to-device copy")
        return storage

    def download(self, pointer: int, out: torch.Tensor) -> None:
        """Copy device bytes into a contiguous CPU tensor and wait (bounded)."""
        nbytes = out.numel() * out.element_size()
        _lib.check(self.lib.mm_memcpy_d2h(ctypes.c_void_p(out.data_ptr()),
                                          ctypes.c_void_p(pointer), nbytes, self.stream, 0),
                   "device-to-host copy")
        self.synchronize()

    def copy_d2d(self, dst: int, src: int, nbytes: int) -> None:
        _lib.check(self.lib.mm_memcpy_d2d(ctypes.c_void_p(dst), ctypes.c_void_p(src), nbytes,
                                          self.stream), "device-to-device copy")

    def synchronize(self, timeout_ms: int | None = None) -> None:
        timeout = config.waitTimeoutMs if timeout_ms is None else int(timeout_ms)
        _lib.check(self.lib.mm_stream_sync(self.stream, timeout), "synchronize")

    # -- parameters ----------------------------------------------------------
    @staticmethod
    def _param_key(value: torch.Tensor) -> tuple:
        return (
            int(value.untyped_storage().data_ptr()),
            int(value.storage_offset()),
            tuple(int(s) for s in value.shape),
            tuple(int(s) for s in value.stride()),
            str(value.dtype),
        )

    def parameter(self, value: torch.Tensor) -> tuple[DeviceStorage, tuple]:
        """Device copy of a CPU parameter, cached by storage identity + version.

        Returns (storage, strides) where strides describe the uploaded layout
        (the CPU tensor's own strides relative to its first element, or
        contiguous strides when the source is not dense).  Mirrors
        _cached_parameter / _parameter_cache_key (backends/cuda/backend.py:241-294).
        """
        if not isinstance(value, torch.Tensor) or value.device.type != "cpu":
            raise RuntimeError("MatrixMan/CUDA: parameters must be CPU tensors for upload")
        if value.dtype != torch.float32:
            raise NotImplementedError("MatrixMan/CUDA: parameters must be float32")
        key = self._param_key(value)
        version = int(value._version)
        entry = self._param_cache.get(key)
        if entry is not None and entry[1] == version:
            return entry[2], entry[3]
        if entry is not None:
            self.synchronize()
            entry[2].release()
        src = value.detach()
        if src.is_contiguous():
            strides = tuple(int(s) for s in src.stride())
            data = src
        else:
            data = src.contiguous()
            strides = tuple(int(s) for s in data.stride())
        storage = self.upload(data, kind=_lib.POOL_PARAMETER, sync=True)
        # Keep the source tensor alive so a recycled CPU allocation can never
        # match a stale key.
        self._param_cache[key] = (value, version, storage, strides)
        return storage, strides

    def parameter_cache_size(self) -> int:
        return len(self._param_cache)

    # -- graphs --------------------------------------------------------------
    def capture_begin(self) -> None:
        _lib.check(self.lib.mm_graph_capture_begin(self.index, self.stream), "begin graph capture")
        self.capturing = True

    def capture_end(self) -> "CudaGraph":
        handle = ctypes.c_void_p()
        try:
            _lib.check(self.lib.mm_graph_capture_end(self.index, self.stream, ctypes.byref(handle)),
                       "end graph capture")
        finally:
            self.capturing = False
        return CudaGraph(self, handle.value)

    def close(self) -> None:
        if self.closed:
            return
        try:
            self.synchronize()
        except Exception:
            pass
        self._param_cache.clear()
        self.closed = True
        self.lib.mm_shutdown(self.index)


class CudaGraph:
    """An instantiated CUDA graph plus its private arena pool."""

    def __init__(self, runtime: DeviceRuntime, handle: int):
        self.runtime = runtime
        self.handle = handle
        self._finalizer = weakref.finalize(self, CudaGraph._destroy, runtime, handle)

    @staticmethod
    def _destroy(runtime: DeviceRuntime, handle: int) -> None:
        if handle and not runtime.closed:
            runtime.lib.mm_graph_destroy(ctypes.c_void_p(handle))

    def replay(self) -> None:
        _lib.check(self.runtime.lib.mm_graph_launch(ctypes.c_void_p(self.handle),
                                                    self.runtime.stream), "graph launch")

    def destroy(self) -> None:
        self._finalizer()


class PinnedHostPool:
    """Page-locked host blocks for readback results, reused across calls.

    ``.cpu()`` returns ordinary CPU tensors; backing them with cached
    page-locked blocks lets the copy engine write them at full link speed (no
    driver bounce buffer, no first-touch page faults on a fresh allocation).
    A block returns to the cache when the last tensor or view over it is
    freed; at most ``config.readbackCacheMb`` stays cached, the rest is freed.
    """

    GRANULE = 1 << 21

    def __init__(self):
        self._free: dict[int, list[int]] = {}
        self._cached = 0
        self._lock = threading.Lock()

    def empty(self, shape, dtype: torch.dtype) -> torch.Tensor | None:
        cap = int(config.readbackCacheMb) << 20
        n = 1
        for v in shape:
            n *= int(v)
        nbytes = max(n, 1) * ELEMENT_SIZE[dtype]
        size = (nbytes + self.GRANULE - 1) // self.GRANULE * self.GRANULE
        if cap == 0 or size > cap:
            return None
        lib = _lib.load()
        ptr = None
        with self._lock:
            blocks = self._free.get(size)
            if blocks:
                ptr = blocks.pop()
                self._cached -= size
        if ptr is None:
            out = ctypes.c_void_p()
            if lib.mm_host_alloc_pinned(size, ctypes.byref(out)) != _lib.MM_OK or not out.value:
                return None
            ptr = int(out.value)
        buf = (ctypes.c_uint8 * size).from_address(ptr)
        t = torch.frombuffer(buf, dtype=dtype, count=max(n, 1))[:n].view(tuple(int(v) for v in shape))
        weakref.finalize(buf, self._release, ptr, size)
        return t

    def _release(self, ptr: int, size: int) -> None:
        try:
            cap = int(config.readbackCacheMb) << 20
            with self._lock:
                if self._cached + size <= cap:
                    self._free.setdefault(size, []).append(ptr)
                    self._cached += size
                    return
            _lib.load().mm_host_free_pinned(ctypes.c_void_p(ptr))
        except Exception:
            pass

    def trim(self) -> None:
        with self._lock:
            blocks = [p for lst in self._free.values() for p in lst]
            self._free.clear()
            self._cached = 0
        lib = _lib.load()
        for p in blocks:
            lib.mm_host_free_pinned(ctypes.c_void_p(p))

    @property
    def cached_bytes(self) -> int:
        return self._cached


pinned_pool = PinnedHostPool()


def host_empty(shape, dtype: torch.dtype) -> torch.Tensor:
    """CPU tensor for a readback: pooled page-locked memory when available."""
    t = pinned_pool.empty(shape, dtype)
    return t if t is not None else torch.empty(tuple(shape), dtype=dtype)


class Timer:
    """CUDA-event timer on a runtime stream (gpumatrix.py:4785-4816)."""

    def __init__(self, runtime: DeviceRuntime):
        self.runtime = runtime
        lib = runtime.lib
        self._start = ctypes.c_void_p()
        self._stop = ctypes.c_void_p()
        _lib.check(lib.mm_event_create(ctypes.byref(self._start), 1), "event create")
        _lib.check(lib.mm_event_create(ctypes.byref(self._stop), 1), "event create")

    def start(self) -> None:
        _lib.check(self.runtime.lib.mm_event_record(self._start, self.runtime.stream), "event record")

    def stop(self) -> None:
        _lib.check(self.runtime.lib.mm_event_record(self._stop, self.runtime.stream), "event record")

    def elapsed_ms(self) -> float:
        _lib.check(self.runtime.lib.mm_event_sync(self._stop, config.waitTimeoutMs), "event sync")
        ms = ctypes.c_float()
        _lib.check(self.runtime.lib.mm_event_elapsed_ms(self._start, self._stop, ctypes.byref(ms)),
                   "event elapsed")
        return float(ms.value)

    def __del__(self):
        try:
            self.runtime.lib.mm_event_destroy(self._start)
            self.runtime.lib.mm_event_destroy(self._stop)
        except Exception:
            pass
