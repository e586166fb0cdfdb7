"""ctypes binding of libmatrixman_b200.so (the C ABI in include/matrixman_b200.h).

The library is loaded from ``matrixman_b200/_lib/`` (built in-tree by
``python -m matrixman_b200.build``).  There is no fallback: if the library is
missing, every device operation raises.  Status codes map onto the exception
types the reference backend raises (drivers/matrixman/backends/cuda/gpumatrix.py:4508-4518
for driver errors, backends/cuda/backend.py for argument errors).
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

MM_MAX_DIMS = 6
MM_OK = 0
MM_ERR_INVALID = 1
MM_ERR_UNSUPPORTED = 2
MM_ERR_OOM = 3
MM_ERR_CUDA = 4
MM_ERR_TIMEOUT = 5
MM_ERR_STATE = 6

MM_F32 = 0
MM_I64 = 1

MM_IPC_HANDLE_BYTES = 64
POOL_ACTIVATION = 0
POOL_SCRATCH = 1
POOL_PARAMETER = 2

ACT_NONE, ACT_RELU, ACT_SILU, ACT_SIGMOID = 0, 1, 2, 3

(UNARY_COPY, UNARY_SILU, UNARY_RELU, UNARY_SIGMOID, UNARY_ADD_SCALAR, UNARY_MUL_SCALAR,
 UNARY_DIV_SCALAR, UNARY_NEG, UNARY_CLAMP) = range(9)
BINARY_ADD, BINARY_SUB, BINARY_MUL, BINARY_DIV = range(4)
PW3_THRESHOLD_BACKWARD, PW3_ADDCMUL, PW3_ADDCDIV, PW3_LERP, PW3_SQRT = range(5)

LIB_DIR = Path(__file__).resolve().parent / "_lib"
LIB_PATH = LIB_DIR / "libmatrixman_b200.so"


class MMTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("size", ctypes.c_int64 * MM_MAX_DIMS),
        ("stride", ctypes.c_int64 * MM_MAX_DIMS),
    ]


class MMDeviceInfo(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char * 256),
        ("cc_major", ctypes.c_int32),
        ("cc_minor", ctypes.c_int32),
        ("sm_count", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("total_bytes", ctypes.c_int64),
        ("free_bytes", ctypes.c_int64),
    ]


class MMPoolStats(ctypes.Structure):
    _fields_ = [
        ("live_bytes", ctypes.c_int64 * 3),
        ("cached_bytes", ctypes.c_int64 * 3),
        ("pending_bytes", ctypes.c_int64 * 3),
        ("peak_live_bytes", ctypes.c_int64 * 3),
        ("alloc_calls", ctypes.c_int64 * 3),
        ("pool_hits", ctypes.c_int64 * 3),
        ("device_mallocs", ctypes.c_int64),
        ("device_frees", ctypes.c_int64),
        ("oom_recoveries", ctypes.c_int64),
        ("capture_pools", ctypes.c_int64),
    ]

    def as_dict(self) -> dict:
        kinds = ("activation", "scratch", "parameter")
        out = {}
        for field in ("live_bytes", "cached_bytes", "pending_bytes", "peak_live_bytes",
                      "alloc_calls", "pool_hits"):
            arr = getattr(self, field)
            out[field] = {k: int(arr[i]) for i, k in enumerate(kinds)}
        for field in ("device_mallocs", "device_frees", "oom_recoveries", "capture_pools"):
            out[field] = int(getattr(self, field))
        return out


class MMConvParams(ctypes.Structure):
    _fields_ = [
        ("stride_h", ctypes.c_int32), ("stride_w", ctypes.c_int32),
        ("pad_h", ctypes.c_int32), ("pad_w", ctypes.c_int32),
        ("dil_h", ctypes.c_int32), ("dil_w", ctypes.c_int32),
        ("groups", ctypes.c_int32),
        ("act", ctypes.c_int32),
        ("residual_before_act", ctypes.c_int32),
        ("algo", ctypes.c_int32),
    ]


_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t
_d = ctypes.c_double
_u32 = ctypes.c_uint32
_T = ctypes.POINTER(MMTensor)
_TT = ctypes.POINTER(ctypes.POINTER(MMTensor))
_fp = ctypes.c_void_p  # float* passed as address

# name -> argtypes (restype is always int)
SIGNATURES = {
    "mm_abi_version": [],
    "mm_last_error": [ctypes.c_char_p, _sz],
    "mm_device_count": [ctypes.POINTER(_i)],
    "mm_device_info": [_i, ctypes.POINTER(MMDeviceInfo)],
    "mm_init": [_i],
    "mm_shutdown": [_i],
    "mm_set_device": [_i],
    "mm_runtime_stream": [_i, ctypes.POINTER(_vp)],
    "mm_stream_create": [_i, ctypes.POINTER(_vp)],
    "mm_stream_destroy": [_vp],
    "mm_stream_sync": [_vp, _i64],
    "mm_stream_query": [_vp, ctypes.POINTER(_i)],
    "mm_event_create": [ctypes.POINTER(_vp), _i],
    "mm_event_destroy": [_vp],
    "mm_event_record": [_vp, _vp],
    "mm_event_sync": [_vp, _i64],
    "mm_stream_wait_event": [_vp, _vp],
    "mm_event_elapsed_ms": [_vp, _vp, ctypes.POINTER(ctypes.c_float)],
    "mm_pool_configure": [_i, _i, _i, _i, _i],
    "mm_alloc": [_i, _sz, _i, _vp, ctypes.POINTER(_vp)],
    "mm_free": [_vp, _vp],
    "mm_pool_trim": [_i],
    "mm_pool_stats": [_i, ctypes.POINTER(MMPoolStats)],
    "mm_debug_fail_alloc_after": [_i, _i64],
    "mm_host_arena_create": [_i64, _i, ctypes.POINTER(_vp)],
    "mm_host_arena_destroy": [_vp],
    "mm_host_arena_alloc": [_vp, _sz, _i, ctypes.POINTER(_vp)],
    "mm_host_arena_free": [_vp, _vp],
    "mm_host_arena_complete": [_vp, _i64],
    "mm_host_arena_generation": [_vp, ctypes.POINTER(_i64)],
    "mm_host_arena_fail_after": [_vp, _i64],
    "mm_host_arena_stats": [_vp, ctypes.POINTER(MMPoolStats)],
    "mm_memcpy_h2d": [_vp, _vp, _sz, _vp, _i],
    "mm_memcpy_d2h": [_vp, _vp, _sz, _vp, _i],
    "mm_memcpy_d2d": [_vp, _vp, _sz, _vp],
    "mm_memcpy_peer": [_vp, _i, _vp, _i, _sz, _vp],
    "mm_enable_peer_access": [_i, _i],
    "mm_host_alloc_pinned": [_sz, ctypes.POINTER(_vp)],
    "mm_host_free_pinned": [_vp],
    "mm_host_is_pinned": [_vp, ctypes.POINTER(_i)],
    "mm_graph_capture_begin": [_i, _vp],
    "mm_graph_capture_end": [_i, _vp, ctypes.POINTER(_vp)],
    "mm_graph_launch": [_vp, _vp],
    "mm_graph_destroy": [_vp],
    "mm_unary": [_i, _T, _T, _d, _d, _vp],
    "mm_binary": [_i, _T, _T, _T, _d, _vp],
    "mm_fill": [_T, _d, _vp],
    "mm_arange": [_T, _d, _d, _vp],
    "mm_copy": [_T, _T, _vp],
    "mm_cat": [_TT, _i, _i, _T, _vp],
    "mm_batch_norm": [_T, _fp, _fp, _fp, _fp, _d, _T, _vp],
    "mm_softmax": [_T, _i, _i, _T, _vp],
    "mm_max_pool2d": [_T, _i, _i, _i, _i, _i, _i, _i, _i, _T, _vp],
    "mm_sppf_pool": [_T, _T, _T, _T, _vp],
    "mm_avg_pool2d": [_T, _i, _i, _i, _i, _i, _i, _i, _i, _T, _vp],
    "mm_adaptive_avg_pool2d": [_T, _T, _vp],
    "mm_reduce": [_T, _u32, _i, _T, _vp],
    "mm_upsample_nearest2d": [_T, _d, _d, _T, _vp],
    "mm_conv2d": [_T, _T, _fp, _T, ctypes.POINTER(MMConvParams), _T, _vp],
    "mm_conv2d_tc": [_T, _fp, _fp, _i, _i, _i, _i, _i, _i, _fp, _T,
                     ctypes.POINTER(MMConvParams), _T, _vp],
    "mm_conv2d_region": [_T, _T, _fp, _T, ctypes.POINTER(MMConvParams), _i64, _i64, _T, _vp],
    "mm_conv2d_tc_region": [_T, _fp, _fp, _i, _i, _i, _i, _i, _i, _fp, _T,
                            ctypes.POINTER(MMConvParams), _i64, _i64, _T, _vp],
    "mm_tf32_split": [_fp, _fp, _fp, _i64, _vp],
    "mm_ipc_alloc": [_i, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _vp],
    "mm_ipc_free": [_i, _vp],
    "mm_ipc_open": [_i, _vp, ctypes.POINTER(ctypes.c_void_p)],
    "mm_ipc_close": [_i, _vp],
    "mm_kernel_error": [_i, ctypes.POINTER(_i), _i],
    "mm_debug_tc_fault": [_i, _i64, _i],
    "mm_gemm": [_T, _T, _T, _d, _d, _i, _T, _vp],
    "mm_yolo_decode": [_TT, ctypes.POINTER(ctypes.c_float), _i, _i, _i, _T, _vp],
    "mm_detect_reduce": [_T, _T, _vp],
    "mm_detect_nms": [_T, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float, _i, _T, _vp,
                      _vp, ctypes.c_size_t, _vp],
    "mm_detect_nms_workspace_size": [_i64, _i64, ctypes.POINTER(ctypes.c_size_t)],
    "mm_detect_nms_static": [_T, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float, _i, _T,
                             _vp, _vp],
    "mm_preprocess_bgr8": [_vp, _i64, _i64, _i64, _T, _vp],
    "mm_pointwise3": [_i, _T, _T, _T, _T, _d, _vp],
    "mm_log_softmax_backward": [_T, _T, _i, _T, _vp],
    "mm_nll_loss": [_T, _T, _T, _i, _i64, _T, _T, _vp],
    "mm_nll_loss_backward": [_T, _T, _T, _T, _i, _i64, _T, _T, _vp],
}


class MatrixManNativeError(RuntimeError):
    """Base for errors raised from the native runtime."""


class DeviceTimeoutError(TimeoutError):
    """A bounded device wait gave up."""


_lib = None
_load_error: str | None = None


def library_path() -> Path:
    return Path(os.environ.get("MATRIXMAN_B200_LIB", str(LIB_PATH)))


def load(required: bool = True):
    """Load the native library once; raise loudly if it is unavailable."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    path = library_path()
    try:
        lib = ctypes.CDLL(str(path), mode=ctypes.RTLD_GLOBAL)
    except OSError as exc:
        _load_error = f"{path}: {exc}"
        if required:
            raise RuntimeError(
                "MatrixMan/B200: native library libmatrixman_b200.so is not available "
                f"({_load_error}); build it with `python -m matrixman_b200.build`"
            ) from exc
        return None
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_int
    if lib.mm_abi_version() != 1:
        raise RuntimeError("MatrixMan/B200: ABI version mismatch of libmatrixman_b200.so")
    _lib = lib
    return lib


def last_error() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(4096)
    lib.mm_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, action: str = "") -> None:
    """Map a native status code onto the reference's exception conventions."""
    if status == MM_OK:
        return
    message = last_error()
    prefix = f"MatrixMan/CUDA: {action}: " if action else "MatrixMan/CUDA: "
    text = prefix + message
    if status == MM_ERR_INVALID:
        raise ValueError(text)
    if status == MM_ERR_UNSUPPORTED:
        raise NotImplementedError(text)
    if status == MM_ERR_OOM:
        raise MemoryError(text)
    if status == MM_ERR_TIMEOUT:
        raise DeviceTimeoutError(text)
    raise MatrixManNativeError(text)


def call(name: str, *args, action: str | None = None) -> None:
    lib = load()
    check(getattr(lib, name)(*args), action or name)


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def make_tensor(ptr: int, shape, strides, dtype: int = MM_F32) -> MMTensor:
    t = MMTensor()
    t.data = ptr
    t.dtype = dtype
    nd = len(shape)
    if nd > MM_MAX_DIMS:
        raise NotImplementedError(f"MatrixMan/CUDA: tensor rank {nd} exceeds {MM_MAX_DIMS}")
    t.ndim = nd
    for i in range(nd):
        t.size[i] = int(shape[i])
        t.stride[i] = int(strides[i])
    return t
