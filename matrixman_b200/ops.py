"""Operator implementations behind the ATen dispatch table.

Each function validates its arguments with the reference's error conventions
(RuntimeError for wrong device/storage, NotImplementedError for unsupported
op/dtype/shape, ValueError for invalid arguments -- drivers/matrixman/
backends/cuda/backend.py:296-1456), allocates outputs from the activation
pool, and launches one native kernel on the device's runtime stream.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from . import telemetry as profiling
from .config import config
from .runtime import DeviceRuntime, activate_stream, get_runtime
from .tensor import (
    MatrixManTensor,
    broadcast_shapes,
    contiguous_strides,
    dense_strides_like,
    is_channels_last,
    is_dense,
    numel,
    readback_tensor,
)

F32 = torch.float32


def _lib_handle():
    return _lib.load()


def _runtime_of(*tensors) -> DeviceRuntime:
    rt = None
    for t in tensors:
        if isinstance(t, MatrixManTensor):
            if rt is None:
                rt = t.runtime
            elif t.runtime is not rt:
                raise RuntimeError("MatrixMan/CUDA: expected all tensors to be on the same "
                                   f"matrixman device, found {rt.index} and {t.runtime.index}")
    if rt is None:
        rt = get_runtime()
    return rt


def require_mm(t, op: str) -> MatrixManTensor:
    if not isinstance(t, MatrixManTensor):
        raise RuntimeError(f"MatrixMan/CUDA: {op} requires a CUDA-backed MatrixManTensor")
    return t


def require_f32(t, op: str) -> None:
    if t.dtype != F32:
        raise NotImplementedError(f"MatrixMan/CUDA: {op} supports float32 tensors only")


def empty(rt: DeviceRuntime, shape, strides=None, dtype=F32, kind=_lib.POOL_ACTIVATION) -> MatrixManTensor:
    shape = tuple(int(s) for s in shape)
    strides = tuple(strides) if strides is not None else contiguous_strides(shape)
    span = (sum((s - 1) * st for s, st in zip(shape, strides)) + 1) if numel(shape) else 1
    owner = rt.new_storage(span, dtype, kind)
    return MatrixManTensor(owner, shape, 0, strides)


def empty_like(t: MatrixManTensor, shape=None) -> MatrixManTensor:
    shape = tuple(t.shape) if shape is None else tuple(shape)
    if tuple(shape) == tuple(t.shape):
        strides = dense_strides_like(shape, t._logical_strides)
    else:
        strides = contiguous_strides(shape)
    return empty(t.runtime, shape, strides, t.dtype)


def _launch(name: str, *args) -> None:
    lib = _lib_handle()
    activate_stream(args[-1])
    token = profiling.launch_times.begin(name, args[-1]) if profiling.gpu_timing_enabled() else None
    status = getattr(lib, name)(*args)
    if status != _lib.MM_OK:
        _lib.check(status, name)
    if token is not None:
        profiling.launch_times.end(token)
    profiling.count_launch(name)
    if config.cudaDisableAsyncQueue or config.cudaDebug:
        get_runtime().synchronize()


def _p(desc: _lib.MMTensor):
    return ctypes.byref(desc)


def _stream(t: MatrixManTensor):
    return t.runtime.stream


# ---------------------------------------------------------------------------
# Copies and materialisation
# ---------------------------------------------------------------------------

def copy_into(src: MatrixManTensor, dst: MatrixManTensor) -> MatrixManTensor:
    if tuple(src.shape) != tuple(dst.shape):
        src = expand_view(src, dst.shape)
    _launch("mm_copy", _p(src.desc()), _p(dst.desc()), _stream(dst))
    return dst


def materialize(t: MatrixManTensor, strides=None) -> MatrixManTensor:
    out = empty(t.runtime, t.shape, strides if strides is not None else contiguous_strides(t.shape), t.dtype)
    return copy_into(t, out)


def clone(t: MatrixManTensor, memory_format=None) -> MatrixManTensor:
    if memory_format is torch.contiguous_format:
        strides = contiguous_strides(t.shape)
    elif memory_format is torch.channels_last and t.dim() == 4:
        from .tensor import channels_last_strides
        strides = channels_last_strides(t.shape)
    else:
        strides = dense_strides_like(t.shape, t._logical_strides)
    return materialize(t, strides)


def expand_view(t: MatrixManTensor, shape) -> MatrixManTensor:
    from .tensor import expand_shape_strides
    s, st = expand_shape_strides(t.shape, t._logical_strides, shape)
    return MatrixManTensor._from_owner(t._owner, s, t._storage_offset, st)


def upload_cpu_into(src: torch.Tensor, dst: MatrixManTensor) -> MatrixManTensor:
    """``dst.copy_(cpu_tensor)``: upload then device copy into dst's layout."""
    if src.dtype != dst.dtype:
        raise NotImplementedError("MatrixMan/CUDA: copy_ does not convert dtypes")
    staged = dst.runtime.upload(src.detach().contiguous())
    tmp = MatrixManTensor(staged, tuple(src.shape), 0, contiguous_strides(src.shape))
    return copy_into(tmp, dst)


# ---------------------------------------------------------------------------
# Elementwise
# ---------------------------------------------------------------------------

_UNARY = {
    "silu": _lib.UNARY_SILU,
    "relu": _lib.UNARY_RELU,
    "sigmoid": _lib.UNARY_SIGMOID,
    "neg": _lib.UNARY_NEG,
}


def unary(name: str, x, out: MatrixManTensor | None = None, a: float = 0.0, b: float = 0.0,
          code: int | None = None) -> MatrixManTensor:
    x = require_mm(x, name)
    require_f32(x, name)
    y = out if out is not None else empty_like(x)
    op = _UNARY[name] if code is None else code
    _launch("mm_unary", op, _p(x.desc()), _p(y.desc()), float(a), float(b), _stream(x))
    return y


def _as_scalar(v):
    if isinstance(v, (int, float, bool)):
        return float(v)
    if isinstance(v, torch.Tensor) and not isinstance(v, MatrixManTensor) and v.dim() == 0:
        return float(v.item())
    return None


def binary(kind: str, a, b, alpha=1, out: MatrixManTensor | None = None) -> MatrixManTensor:
    sa, sb = _as_scalar(a), _as_scalar(b)
    alpha = float(alpha)
    if sa is not None and sb is not None:
        raise RuntimeError(f"MatrixMan/CUDA: {kind} requires a MatrixMan tensor operand")
    if sb is not None:
        x = require_mm(a, kind)
        require_f32(x, kind)
        y = out if out is not None else empty_like(x)
        if kind == "add":
            code, s = _lib.UNARY_ADD_SCALAR, sb * alpha
        elif kind == "sub":
            code, s = _lib.UNARY_ADD_SCALAR, -sb * alpha
        elif kind == "mul":
            code, s = _lib.UNARY_MUL_SCALAR, sb
        else:
            code, s = _lib.UNARY_DIV_SCALAR, sb
        _launch("mm_unary", code, _p(x.desc()), _p(y.desc()), s, 0.0, _stream(x))
        return y
    if sa is not None:
        # scalar (op) tensor
        x = require_mm(b, kind)
        require_f32(x, kind)
        if kind == "add" and alpha == 1.0:
            return binary("add", x, sa, 1.0, out)
        if kind == "mul":
            return binary("mul", x, sa, 1.0, out)
        return _scalar_first(kind, sa, x, alpha, out)
    a = require_mm(a, kind)
    b = require_mm(b, kind)
    require_f32(a, kind)
    require_f32(b, kind)
    _runtime_of(a, b)
    shape = broadcast_shapes(tuple(a.shape), tuple(b.shape))
    if out is not None:
        if tuple(out.shape) != shape:
            raise RuntimeError(f"MatrixMan/CUDA: output with shape {tuple(out.shape)} doesn't "
                               f"match the broadcast shape {shape}")
        y = out
    else:
        like = a if tuple(a.shape) == shape else (b if tuple(b.shape) == shape else None)
        y = empty_like(like) if like is not None else empty(a.runtime, shape)
    ea = expand_view(a, shape) if tuple(a.shape) != shape else a
    eb = expand_view(b, shape) if tuple(b.shape) != shape else b
    code = {"add": _lib.BINARY_ADD, "sub": _lib.BINARY_SUB, "mul": _lib.BINARY_MUL,
            "div": _lib.BINARY_DIV}[kind]
    _launch("mm_binary", code, _p(ea.desc()), _p(eb.desc()), _p(y.desc()), alpha, _stream(a))
    return y


def _scalar_first(kind, s, x, alpha, out):
    """s (op) alpha*x for a scalar left operand."""
    # Materialise the scalar as an expanded constant and reuse the binary path.
    const = full(x.runtime, (), s)
    return binary(kind, expand_view(const, x.shape), x, alpha, out)


def full(rt: DeviceRuntime, shape, value, dtype=F32, strides=None) -> MatrixManTensor:
    t = empty(rt, shape, strides, dtype)
    if numel(t.shape):
        _launch("mm_fill", _p(t.desc()), float(value), rt.stream)
    return t


def fill_(t: MatrixManTensor, value) -> MatrixManTensor:
    require_mm(t, "fill_")
    v = _as_scalar(value)
    if v is None:
        raise NotImplementedError("MatrixMan/CUDA: fill_ supports scalar values only")
    _launch("mm_fill", _p(t.desc()), v, _stream(t))
    return t


def arange_into(out: MatrixManTensor, start, step) -> MatrixManTensor:
    _launch("mm_arange", _p(out.desc()), float(start), float(step), _stream(out))
    return out


# ---------------------------------------------------------------------------
# cat / stack
# ---------------------------------------------------------------------------

def cat(tensors, dim=0) -> MatrixManTensor:
    tensors = [t for t in tensors]
    if not tensors:
        raise RuntimeError("MatrixMan/CUDA: cat expects a non-empty tensor list")
    # torch skips legacy empty 1-D inputs of size (0,)
    tensors = [t for t in tensors if not (t.dim() == 1 and t.shape[0] == 0)] or tensors[:1]
    for t in tensors:
        require_mm(t, "cat")
    rt = _runtime_of(*tensors)
    ref = tensors[0]
    rank = ref.dim()
    d = int(dim) + rank if int(dim) < 0 else int(dim)
    if d < 0 or d >= rank:
        raise IndexError("MatrixMan/CUDA: cat dimension is out of range")
    for t in tensors:
        if t.dim() != rank or any(t.shape[i] != ref.shape[i] for i in range(rank) if i != d):
            raise RuntimeError("MatrixMan/CUDA: cat inputs must match except in the cat dimension")
        if t.dtype != ref.dtype:
            raise NotImplementedError("MatrixMan/CUDA: cat requires one dtype")
    shape = list(ref.shape)
    shape[d] = sum(int(t.shape[d]) for t in tensors)
    if rank == 4 and all(is_channels_last(t.shape, t._logical_strides) and is_dense(t.shape, t._logical_strides)
                         for t in tensors):
        from .tensor import channels_last_strides
        strides = channels_last_strides(shape)
    else:
        strides = contiguous_strides(shape)
    y = empty(rt, shape, strides, ref.dtype)
    descs = [t.desc() for t in tensors]
    arr = (ctypes.POINTER(_lib.MMTensor) * len(descs))(*[ctypes.pointer(x) for x in descs])
    _launch("mm_cat", arr, len(descs), d, _p(y.desc()), rt.stream)
    return y


def stack(tensors, dim=0) -> MatrixManTensor:
    from .tensor import unsqueeze_shape_strides
    tensors = list(tensors)
    if not tensors:
        raise RuntimeError("MatrixMan/CUDA: stack expects a non-empty tensor list")
    rank = tensors[0].dim()
    d = int(dim) + rank + 1 if int(dim) < 0 else int(dim)
    views = []
    for t in tensors:
        require_mm(t, "stack")
        if tuple(t.shape) != tuple(tensors[0].shape):
            raise RuntimeError("MatrixMan/CUDA: stack expects each tensor to be equal size")
        s, st = unsqueeze_shape_strides(t.shape, t._logical_strides, d)
        views.append(MatrixManTensor._from_owner(t._owner, s, t._storage_offset, st))
    shape = list(views[0].shape)
    shape[d] = len(views)
    y = empty(_runtime_of(*tensors), shape, contiguous_strides(shape), tensors[0].dtype)
    descs = [v.desc() for v in views]
    arr = (ctypes.POINTER(_lib.MMTensor) * len(descs))(*[ctypes.pointer(x) for x in descs])
    _launch("mm_cat", arr, len(descs), d, _p(y.desc()), y.runtime.stream)
    return y


# ---------------------------------------------------------------------------
# Parameters (CPU tensors uploaded once and cached; or device tensors)
# ---------------------------------------------------------------------------

def device_operand(rt: DeviceRuntime, value, name: str) -> MatrixManTensor:
    """A MatrixMan view of a parameter given as a CPU tensor or a device tensor."""
    if isinstance(value, MatrixManTensor):
        if value.runtime is not rt:
            raise RuntimeError(f"MatrixMan/CUDA: {name} is on another matrixman device")
        return value
    if not isinstance(value, torch.Tensor):
        raise RuntimeError(f"MatrixMan/CUDA: {name} must be a tensor")
    if value.device.type != "cpu":
        raise RuntimeError(f"MatrixMan/CUDA: {name} must be a CPU tensor for upload")
    if value.dtype != F32:
        raise NotImplementedError(f"MatrixMan/CUDA: {name} must be float32")
    storage, strides = rt.parameter(value)
    return MatrixManTensor(storage, tuple(value.shape), 0, strides)


def _pair(v, label):
    if isinstance(v, (tuple, list)):
        vals = tuple(int(x) for x in v)
        if len(vals) == 1:
            vals = vals * 2
    else:
        vals = (int(v), int(v))
    if len(vals) != 2:
        raise NotImplementedError(f"MatrixMan/CUDA: convolution {label} must contain two values")
    return vals


def conv_output_hw(h, w, r, s, stride, padding, dilation):
    oh = (h + 2 * padding[0] - dilation[0] * (r - 1) - 1) // stride[0] + 1
    ow = (w + 2 * padding[1] - dilation[1] * (s - 1) - 1) // stride[1] + 1
    return oh, ow


_FROM_CONFIG = object()


def conv_tile_cap(cap=_FROM_CONFIG):
    """Largest output extent (rows and columns) of one convolution launch.

    The reference's ``tileLimit`` bounds the physical tile one convolution pass
    renders into (drivers/matrixman/config.py:305-314, consumed only by the
    OpenGL convolution, backends/opengl/convolution.py:1299; its CUDA backend
    runs every convolution as one launch).  Here a limit the user sets (through
    MATRIXMAN_TILE_LIMIT or a Python override) caps each launch at limit x
    limit output pixels; the default value (256, reported as in the reference)
    and ``auto`` keep one launch per convolution, as the reference's CUDA
    backend does.  ``cap`` overrides the setting (None: no cap)."""
    if cap is _FROM_CONFIG:
        value = config.tileLimit
        if value == "auto" or config.source("tileLimit") == "default":
            return None
        return int(value)
    return None if cap is None else int(cap)


def conv_regions(oh: int, ow: int, cap) -> list[tuple[int, int, int, int]]:
    """(row0, col0, rows, cols) regions covering an oh x ow output, row-major,
    at most cap x cap pixels each; one region when cap is None or the output
    fits."""
    if cap is None or (oh <= cap and ow <= cap):
        return [(0, 0, oh, ow)]
    if cap <= 0:
        raise ValueError("MatrixMan: tile limit must be positive")
    return [(r0, c0, min(cap, oh - r0), min(cap, ow - c0))
            for r0 in range(0, oh, cap) for c0 in range(0, ow, cap)]


def _region_view(t: MatrixManTensor, r0: int, c0: int, rows: int, cols: int) -> MatrixManTensor:
    """Rows [r0, r0 + rows) and columns [c0, c0 + cols) of an N, C, H, W view."""
    st = t._logical_strides
    shape = (int(t.shape[0]), int(t.shape[1]), rows, cols)
    return MatrixManTensor._from_owner(t._owner, shape, t._storage_offset + r0 * st[2] + c0 * st[3], st)


def convolution(x, weight, bias, stride, padding, dilation, groups, *, act=_lib.ACT_NONE,
                residual=None, residual_before_act=False, out=None, out_strides=None,
                tile_cap=_FROM_CONFIG) -> MatrixManTensor:
    x = require_mm(x, "convolution")
    if x.dtype != F32 or x.dim() != 4:
        raise NotImplementedError("MatrixMan/CUDA: only float32 NCHW convolution is implemented")
    rt = x.runtime
    w = device_operand(rt, weight, "convolution weight")
    if w.dim() != 4:
        raise NotImplementedError("MatrixMan/CUDA: convolution weights must be shaped K,C,R,S")
    b = None
    if bias is not None:
        b = device_operand(rt, bias, "convolution bias")
        if b.dim() != 1 or int(b.shape[0]) != int(w.shape[0]):
            raise ValueError("MatrixMan/CUDA: convolution bias length must equal output channels")
        if b._logical_strides[0] != 1:
            b = materialize(b)
    n, c, h, wd = (int(v) for v in x.shape)
    k, wc, r, s = (int(v) for v in w.shape)
    groups = int(groups)
    stride = _pair(stride, "stride")
    padding = _pair(padding, "padding")
    dilation = _pair(dilation, "dilation")
    if groups <= 0 or c % groups or k % groups or wc != c // groups:
        raise NotImplementedError(
            "MatrixMan/CUDA: convolution groups/weight channels are unsupported "
            "(expected weight C == input C / groups)")
    if min(stride + dilation) <= 0 or min(padding) < 0:
        raise NotImplementedError("MatrixMan/CUDA: invalid convolution stride, padding, or dilation")
    oh, ow = conv_output_hw(h, wd, r, s, stride, padding, dilation)
    if oh <= 0 or ow <= 0:
        raise ValueError("MatrixMan/CUDA: convolution output dimensions must be positive")
    shape = (n, k, oh, ow)
    if out is None:
        if out_strides is None:
            from .tensor import channels_last_strides
            out_strides = channels_last_strides(shape) if (
                x.dim() == 4 and is_channels_last(x.shape, x._logical_strides)) else contiguous_strides(shape)
        out = empty(rt, shape, out_strides)
    params = _lib.MMConvParams(stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1],
                               groups, int(act), 1 if residual_before_act else 0, 0)
    bias_ptr = ctypes.c_void_p(b.element_ptr) if b is not None else None
    regions = conv_regions(oh, ow, conv_tile_cap(tile_cap))
    if len(regions) == 1:
        res_desc = residual.desc() if residual is not None else None
        _launch("mm_conv2d", _p(x.desc()), _p(w.desc()), bias_ptr,
                _p(res_desc) if res_desc is not None else None,
                ctypes.byref(params), _p(out.desc()), rt.stream)
        return out
    for r0, c0, rows, cols in regions:
        y = _region_view(out, r0, c0, rows, cols)
        res_desc = _region_view(residual, r0, c0, rows, cols).desc() if residual is not None else None
        _launch("mm_conv2d_region", _p(x.desc()), _p(w.desc()), bias_ptr,
                _p(res_desc) if res_desc is not None else None, ctypes.byref(params),
                ctypes.c_int64(r0), ctypes.c_int64(c0), _p(y.desc()), rt.stream)
    return out


def conv_tc(x: MatrixManTensor, w_hi: MatrixManTensor, w_lo: MatrixManTensor, k_out: int, c_in: int,
            r: int, s: int, c_pad: int, k_pad: int, bias, stride, padding, dilation, act,
            residual, residual_before_act, out: MatrixManTensor, tile_cap=_FROM_CONFIG) -> bool:
    """tcgen05 3xTF32 convolution on prepacked hi/lo weight planes.

    Returns False (nothing launched) when the geometry or layout is outside
    what the tensor-core kernel covers; the caller then runs mm_conv2d.  An
    output larger than the tile cap (conv_tile_cap) runs as several region
    launches with the same result."""
    params = _lib.MMConvParams(stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1],
                               1, int(act), 1 if residual_before_act else 0, 2)
    lib = _lib_handle()
    stream = x.runtime.stream
    activate_stream(stream)
    bias_ptr = ctypes.c_void_p(bias.element_ptr) if bias is not None else None
    oh, ow = int(out.shape[2]), int(out.shape[3])
    regions = conv_regions(oh, ow, conv_tile_cap(tile_cap))
    for i, (r0, c0, rows, cols) in enumerate(regions):
        whole = len(regions) == 1
        y = out if whole else _region_view(out, r0, c0, rows, cols)
        res = residual if whole or residual is None else _region_view(residual, r0, c0, rows, cols)
        res_desc = res.desc() if res is not None else None
        name = "mm_conv2d_tc" if whole else "mm_conv2d_tc_region"
        token = profiling.launch_times.begin(name, stream) if profiling.gpu_timing_enabled() else None
        args = (_p(x.desc()), ctypes.c_void_p(w_hi.element_ptr), ctypes.c_void_p(w_lo.element_ptr),
                int(k_out), int(c_in), int(r), int(s), int(c_pad), int(k_pad), bias_ptr,
                _p(res_desc) if res_desc is not None else None, ctypes.byref(params))
        if whole:
            status = lib.mm_conv2d_tc(*args, _p(y.desc()), stream)
        else:
            status = lib.mm_conv2d_tc_region(*args, ctypes.c_int64(r0), ctypes.c_int64(c0), _p(y.desc()),
                                             stream)
        if status == _lib.MM_ERR_UNSUPPORTED and i == 0:
            if token is not None:
                profiling.launch_times.end(token)
                profiling.launch_times.records.pop()
            return False
        _lib.check(status, name)
        if token is not None:
            profiling.launch_times.end(token)
        profiling.count_launch(name)
    if config.cudaDisableAsyncQueue or config.cudaDebug:
        x.runtime.synchronize()
        check_kernel_error(x.runtime.index)
    return True


def check_kernel_error(device: int) -> None:
    """Raise if a device-side bounded wait gave up (the kernel returned early)."""
    code = ctypes.c_int(0)
    _lib.check(_lib_handle().mm_kernel_error(int(device), ctypes.byref(code), 1), "kernel status")
    if code.value:
        raise _lib.MatrixManNativeError(
            f"MatrixMan/CUDA: a tensor-core kernel stopped after a bounded wait (code {code.value})")


def gemm(x, w_kn, bias=None, alpha=1.0, beta=1.0, act=_lib.ACT_NONE, out=None) -> MatrixManTensor:
    """out[M,N] = act(alpha * x @ w_kn + beta * bias) (addmm / mm / linear)."""
    x = require_mm(x, "mm")
    require_f32(x, "mm")
    rt = x.runtime
    w = device_operand(rt, w_kn, "mm rhs")
    if x.dim() != 2 or w.dim() != 2:
        raise NotImplementedError("MatrixMan/CUDA: mm supports 2D float32 tensors only")
    m, k = (int(v) for v in x.shape)
    k2, n = (int(v) for v in w.shape)
    if k != k2:
        raise RuntimeError(f"MatrixMan/CUDA: mm shapes cannot be multiplied ({m}x{k} and {k2}x{n})")
    bdesc = None
    if bias is not None:
        bt = device_operand(rt, bias, "addmm bias")
        if bt.dim() == 0:
            bt = expand_view(bt, (n,))
        bdesc = bt.desc()
    if out is None:
        out = empty(rt, (m, n))
    _launch("mm_gemm", _p(x.desc()), _p(w.desc()), _p(bdesc) if bdesc is not None else None,
            float(alpha), float(beta), int(act), _p(out.desc()), rt.stream)
    return out


# ---------------------------------------------------------------------------
# Normalisation, softmax, pooling, resize, reductions
# ---------------------------------------------------------------------------

def batch_norm_eval(x, weight, bias, running_mean, running_var, eps) -> MatrixManTensor:
    x = require_mm(x, "BatchNorm")
    require_f32(x, "BatchNorm")
    if x.dim() < 2:
        raise NotImplementedError("MatrixMan/CUDA: BatchNorm supports rank >= 2 tensors only")
    rt = x.runtime
    c = int(x.shape[1])

    def param(v, name, default):
        if v is None:
            v = torch.full((c,), default, dtype=F32)
        t = device_operand(rt, v, f"BatchNorm {name}")
        if tuple(t.shape) != (c,):
            raise NotImplementedError(f"MatrixMan/CUDA: BatchNorm {name} must be shape [{c}]")
        return t if t._logical_strides == (1,) else materialize(t)

    if running_mean is None or running_var is None:
        raise NotImplementedError("MatrixMan/CUDA: BatchNorm requires running statistics in eval mode")
    if float(eps) < 0:
        raise ValueError("MatrixMan/CUDA: BatchNorm epsilon must be non-negative")
    mean = param(running_mean, "running_mean", 0.0)
    var = param(running_var, "running_var", 1.0)
    w = param(weight, "weight", 1.0)
    b = param(bias, "bias", 0.0)
    y = empty_like(x)
    _launch("mm_batch_norm", _p(x.desc()), ctypes.c_void_p(mean.element_ptr),
            ctypes.c_void_p(var.element_ptr), ctypes.c_void_p(w.element_ptr),
            ctypes.c_void_p(b.element_ptr), float(eps), _p(y.desc()), rt.stream)
    return y


def softmax(x, dim, log=False) -> MatrixManTensor:
    x = require_mm(x, "softmax")
    require_f32(x, "softmax")
    rank = x.dim()
    d = int(dim)
    if rank == 0:
        d = 0
    elif d < 0:
        d += rank
    if rank and (d < 0 or d >= rank):
        raise IndexError("MatrixMan/CUDA: softmax dimension is out of range")
    y = empty_like(x)
    _launch("mm_softmax", _p(x.desc()), d, 1 if log else 0, _p(y.desc()), _stream(x))
    return y


def pool_output_size(size, k, s, p, d, ceil_mode):
    numer = size + 2 * p - d * (k - 1) - 1 + (s - 1 if ceil_mode else 0)
    out = numer // s + 1
    if ceil_mode and (out - 1) * s >= size + p:
        out -= 1
    return out


def max_pool2d(x, kernel_size, stride=None, padding=0, dilation=1, ceil_mode=False) -> MatrixManTensor:
    x = require_mm(x, "max_pool2d")
    require_f32(x, "max_pool2d")
    if x.dim() not in (3, 4):
        raise NotImplementedError("MatrixMan/CUDA: max_pool2d supports 3-D/4-D tensors")
    squeeze = x.dim() == 3
    if squeeze:
        x = _unsqueeze0(x)
    kh, kw = _pair(kernel_size, "kernel")
    sh, sw = _pair(stride if (stride is not None and stride != []) else (kh, kw), "stride")
    ph, pw = _pair(padding, "padding")
    dh, dw = _pair(dilation, "dilation")
    if ph > kh // 2 or pw > kw // 2:
        raise ValueError("MatrixMan/CUDA: pad should be at most half of effective kernel size")
    n, c, h, w = (int(v) for v in x.shape)
    oh = pool_output_size(h, kh, sh, ph, dh, ceil_mode)
    ow = pool_output_size(w, kw, sw, pw, dw, ceil_mode)
    if oh <= 0 or ow <= 0:
        raise ValueError("MatrixMan/CUDA: max_pool2d output size is too small")
    y = empty(x.runtime, (n, c, oh, ow), _out_strides_like(x, (n, c, oh, ow)))
    _launch("mm_max_pool2d", _p(x.desc()), kh, kw, sh, sw, ph, pw, dh, dw, _p(y.desc()), _stream(x))
    return _squeeze0(y) if squeeze else y


def _out_strides_like(x, shape):
    from .tensor import channels_last_strides
    if len(shape) == 4 and is_channels_last(x.shape, x._logical_strides) and is_dense(x.shape, x._logical_strides):
        return channels_last_strides(shape)
    return contiguous_strides(shape)


def _unsqueeze0(x):
    from .tensor import unsqueeze_shape_strides
    s, st = unsqueeze_shape_strides(x.shape, x._logical_strides, 0)
    return MatrixManTensor._from_owner(x._owner, s, x._storage_offset, st)


def _squeeze0(x):
    return MatrixManTensor._from_owner(x._owner, tuple(x.shape)[1:], x._storage_offset,
                                       tuple(x._logical_strides)[1:])


def avg_pool2d(x, kernel_size, stride=None, padding=0, ceil_mode=False, count_include_pad=True,
               divisor_override=None) -> MatrixManTensor:
    x = require_mm(x, "avg_pool2d")
    require_f32(x, "avg_pool2d")
    squeeze = x.dim() == 3
    if squeeze:
        x = _unsqueeze0(x)
    if x.dim() != 4:
        raise NotImplementedError("MatrixMan/CUDA: avg_pool2d supports 3-D/4-D tensors")
    kh, kw = _pair(kernel_size, "kernel")
    sh, sw = _pair(stride if (stride is not None and stride != []) else (kh, kw), "stride")
    ph, pw = _pair(padding, "padding")
    n, c, h, w = (int(v) for v in x.shape)
    oh = pool_output_size(h, kh, sh, ph, 1, ceil_mode)
    ow = pool_output_size(w, kw, sw, pw, 1, ceil_mode)
    shape = (n, c, oh, ow)
    y = empty(x.runtime, shape, _out_strides_like(x, shape))
    _launch("mm_avg_pool2d", _p(x.desc()), kh, kw, sh, sw, ph, pw, 1 if count_include_pad else 0,
            int(divisor_override or 0), _p(y.desc()), _stream(x))
    return _squeeze0(y) if squeeze else y


def adaptive_avg_pool2d(x, output_size) -> MatrixManTensor:
    x = require_mm(x, "adaptive_avg_pool2d")
    require_f32(x, "adaptive_avg_pool2d")
    squeeze = x.dim() == 3
    if squeeze:
        x = _unsqueeze0(x)
    oh, ow = _pair(output_size, "output_size")
    n, c, h, w = (int(v) for v in x.shape)
    shape = (n, c, oh, ow)
    y = empty(x.runtime, shape, _out_strides_like(x, shape))
    _launch("mm_adaptive_avg_pool2d", _p(x.desc()), _p(y.desc()), _stream(x))
    return _squeeze0(y) if squeeze else y


def reduce(x, dims, keepdim=False, mean=True) -> MatrixManTensor:
    x = require_mm(x, "mean" if mean else "sum")
    require_f32(x, "mean" if mean else "sum")
    rank = x.dim()
    if dims is None or (isinstance(dims, (list, tuple)) and len(dims) == 0):
        dims = list(range(rank))
    if isinstance(dims, int):
        dims = [dims]
    mask = 0
    for d in dims:
        d = int(d) + rank if int(d) < 0 else int(d)
        if d < 0 or d >= rank:
            raise IndexError("MatrixMan/CUDA: reduction dimension is out of range")
        mask |= 1 << d
    keep_shape = tuple(1 if (mask >> i) & 1 else int(x.shape[i]) for i in range(rank))
    y = empty(x.runtime, keep_shape)
    _launch("mm_reduce", _p(x.desc()), mask, 1 if mean else 0, _p(y.desc()), _stream(x))
    if keepdim:
        return y
    shape = tuple(int(x.shape[i]) for i in range(rank) if not (mask >> i) & 1)
    return MatrixManTensor._from_owner(y._owner, shape, 0, contiguous_strides(shape))


def upsample_nearest2d(x, output_size, scales_h=None, scales_w=None,
                       out: MatrixManTensor | None = None) -> MatrixManTensor:
    """Nearest upsample; ``out`` (optional) is a view to write into, e.g. a
    channel slice of a concatenation buffer."""
    x = require_mm(x, "upsample_nearest2d")
    require_f32(x, "upsample_nearest2d")
    if x.dim() != 4:
        raise NotImplementedError("MatrixMan/CUDA: upsample_nearest2d supports 4-D tensors")
    n, c, h, w = (int(v) for v in x.shape)
    if output_size is None:
        if scales_h is None or scales_w is None:
            raise ValueError("MatrixMan/CUDA: upsample_nearest2d needs output_size or scales")
        oh, ow = int(math.floor(h * scales_h)), int(math.floor(w * scales_w))
    else:
        oh, ow = (int(v) for v in output_size)
    shape = (n, c, oh, ow)
    if out is not None:
        if tuple(int(v) for v in out.shape) != shape:
            raise ValueError("MatrixMan/CUDA: upsample_nearest2d output view has the wrong shape")
        y = out
    else:
        y = empty(x.runtime, shape, _out_strides_like(x, shape))
    _launch("mm_upsample_nearest2d", _p(x.desc()), float(scales_h or 0.0), float(scales_w or 0.0),
            _p(y.desc()), _stream(x))
    return y


# ---------------------------------------------------------------------------
# Training path: backward passes and Adam's element-wise update (the reference
# has these on its OpenGL backend only, backends/opengl/dispatch.py:171-179,
# :264-290, :299, :377-382, :463-479).
# ---------------------------------------------------------------------------
def pointwise3(code: int, x, a=None, b=None, scalar=0.0, out: MatrixManTensor | None = None,
               name: str = "pointwise") -> MatrixManTensor:
    """y = op(x, a, b; scalar), a and b broadcast; ``out`` may be ``x`` (in-place)."""
    x = require_mm(x, name)
    a = x if a is None else require_mm(a, name)
    b = x if b is None else require_mm(b, name)
    for t in (x, a, b):
        require_f32(t, name)
    _runtime_of(x, a, b)
    shape = broadcast_shapes(broadcast_shapes(tuple(x.shape), tuple(a.shape)), tuple(b.shape))
    if out is not None and tuple(out.shape) != shape:
        raise RuntimeError(f"MatrixMan/CUDA: {name}: output with shape {tuple(out.shape)} doesn't "
                           f"match the broadcast shape {shape}")
    y = out if out is not None else (empty_like(x) if tuple(x.shape) == shape else empty(x.runtime, shape))
    ex, ea, eb = (expand_view(t, shape) if tuple(t.shape) != shape else t for t in (x, a, b))
    _launch("mm_pointwise3", int(code), _p(ex.desc()), _p(ea.desc()), _p(eb.desc()), _p(y.desc()),
            float(scalar), _stream(x))
    return y


def log_softmax_backward(grad, output, dim) -> MatrixManTensor:
    grad = require_mm(grad, "log_softmax_backward")
    output = require_mm(output, "log_softmax_backward")
    require_f32(grad, "log_softmax_backward")
    require_f32(output, "log_softmax_backward")
    if tuple(grad.shape) != tuple(output.shape):
        raise RuntimeError("MatrixMan/CUDA: log_softmax_backward needs equal shapes")
    rank = grad.dim()
    d = int(dim) + (rank if int(dim) < 0 else 0)
    if rank and not 0 <= d < rank:
        raise IndexError("MatrixMan/CUDA: log_softmax_backward dimension is out of range")
    dense = contiguous_strides(tuple(grad.shape))
    g = grad if tuple(grad._logical_strides) == dense else materialize(grad)
    o = output if tuple(output._logical_strides) == dense else materialize(output)
    y = empty(grad.runtime, tuple(grad.shape))
    _launch("mm_log_softmax_backward", _p(g.desc()), _p(o.desc()), max(d, 0), _p(y.desc()), _stream(grad))
    return y


_REDUCTIONS = (0, 1, 2)


def _nll_operands(x, target, weight, reduction, ignore_index, op):
    x = require_mm(x, op)
    require_f32(x, op)
    if x.dim() != 2:
        raise NotImplementedError(f"MatrixMan/CUDA: {op} supports input [N, C] and target [N]")
    if int(reduction) not in _REDUCTIONS:
        raise RuntimeError(f"MatrixMan/CUDA: {op} unsupported reduction={reduction}")
    rt = x.runtime
    if isinstance(target, MatrixManTensor):
        host_target = None
    elif isinstance(target, torch.Tensor) and target.device.type == "cpu":
        host_target = target
    else:
        raise RuntimeError(f"MatrixMan/CUDA: {op} requires a tensor target")
    if target.dtype != torch.int64 or target.dim() != 1 or target.shape[0] != x.shape[0]:
        raise RuntimeError(f"MatrixMan/CUDA: {op} requires an int64 target [N] for input [N, C]")
    if host_target is not None:
        target = MatrixManTensor(rt.upload(host_target.contiguous()), tuple(host_target.shape), 0,
                                 contiguous_strides(tuple(host_target.shape)))
    w = None
    if weight is not None:
        w = device_operand(rt, weight, f"{op} weight")
        if tuple(w.shape) != (int(x.shape[1]),):
            raise RuntimeError(f"MatrixMan/CUDA: {op} weight must be [C]")
    return x, target, w, host_target


def _check_targets(values: torch.Tensor, classes: int, ignore_index: int, op: str) -> None:
    bad = (values != int(ignore_index)) & ((values < 0) | (values >= classes))
    if bool(bad.any()):
        raise RuntimeError(f"MatrixMan/CUDA: {op} target contains an out-of-range class index")


def nll_loss(x, target, weight=None, reduction=1, ignore_index=-100):
    """nll_loss_forward: (output, total_weight).  Targets are checked on the
    host (a device target is read back first), as the reference does."""
    x, target, w, host_target = _nll_operands(x, target, weight, reduction, ignore_index, "nll_loss_forward")
    values = host_target if host_target is not None else readback_tensor(target)
    _check_targets(values, int(x.shape[1]), ignore_index, "nll_loss_forward")
    rt = x.runtime
    total = full(rt, (), 0.0)
    out = empty(rt, (int(x.shape[0]),) if int(reduction) == 0 else ())
    _launch("mm_nll_loss", _p(x.desc()), _p(target.desc()), _p(w.desc()) if w is not None else None,
            int(reduction), int(ignore_index), _p(out.desc()), _p(total.desc()), _stream(x))
    return out, total


def nll_loss_backward(grad_output, x, target, weight, reduction, ignore_index, total_weight):
    x, target, w, _ = _nll_operands(x, target, weight, reduction, ignore_index, "nll_loss_backward")
    rt = x.runtime
    go = device_operand(rt, grad_output, "nll_loss_backward grad_output")
    tw = device_operand(rt, total_weight, "nll_loss_backward total_weight")
    gi = empty(rt, tuple(x.shape))
    _launch("mm_nll_loss_backward", _p(go.desc()), _p(x.desc()), _p(target.desc()),
            _p(w.desc()) if w is not None else None, int(reduction), int(ignore_index), _p(tw.desc()),
            _p(gi.desc()), _stream(x))
    return gi
