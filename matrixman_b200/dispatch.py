"""ATen routing for ``MatrixManTensor`` (the reference's dispatch.py:36-416).

The reference walks an ``if`` chain of 22 CUDA ops and raises
``NotImplementedError("MatrixMan/CUDA: <op> not implemented")`` for anything
else (dispatch.py:413-415).  Here the routing is a dict from OpOverload to
handler, covering the reference's CUDA ops plus the ops that only its OpenGL
backend had (addmm, relu, mean.dim, generic/avg/adaptive pooling,
log_softmax) and the view ops needed by torchvision/Ultralytics-style models.
Unsupported ops still raise, naming the op; there is never a CPU fallback.
``_to_copy`` to the CPU is the only readback path (dispatch.py:40-70).
"""

from __future__ import annotations

import torch

from . import ops
from . import telemetry as profiling
from .tensor import (
    MatrixManTensor,
    contiguous_strides,
    expand_shape_strides,
    infer_view_shape,
    readback_tensor,
    unsqueeze_shape_strides,
    view_strides,
)

aten = torch.ops.aten
_HANDLERS: dict = {}


def _register(*overloads):
    def deco(fn):
        for o in overloads:
            _HANDLERS[o] = fn
        return fn
    return deco


def _operator_name(func) -> str:
    names = {
        aten.convolution.default: "Conv2D",
        aten.native_batch_norm.default: "BatchNorm",
        aten.add.Tensor: "Add",
        aten.mm.default: "MatMul",
        aten.cat.default: "Cat",
        aten._softmax.default: "Softmax",
        aten.upsample_nearest2d.default: "UpsampleNearest2D",
        aten.max_pool2d_with_indices.default: "MaxPool2D",
    }
    return names.get(func, str(func))


def handle_torch_dispatch(cls, func, types, args=(), kwargs=None):
    kwargs = kwargs or {}
    handler = _HANDLERS.get(func)
    if handler is None:
        raise NotImplementedError(f"MatrixMan/CUDA: {_operator_name(func)} not implemented")
    if profiling.dispatch_enabled():
        with profiling.dispatch_scope(str(func)):
            return handler(*args, **kwargs)
    return handler(*args, **kwargs)


def _view(t: MatrixManTensor, shape, strides, offset=None) -> MatrixManTensor:
    return MatrixManTensor._from_owner(t._owner, shape, t._storage_offset if offset is None else offset,
                                       strides)


def _norm_dim(d, rank):
    d = int(d)
    if rank == 0:
        if d in (0, -1):
            return 0
    if d < 0:
        d += rank
    if d < 0 or d >= max(rank, 1):
        raise IndexError(f"MatrixMan/CUDA: dimension {d} is out of range for rank {rank}")
    return d


# ---------------------------------------------------------------------------
# Readback and copies
# ---------------------------------------------------------------------------

@_register(aten._to_copy.default)
def _to_copy(source, dtype=None, layout=None, device=None, pin_memory=None, non_blocking=False,
             memory_format=None):
    if not isinstance(source, MatrixManTensor):
        raise RuntimeError("MatrixMan: _to_copy requires a MatrixManTensor source")
    if dtype is not None and dtype != source.dtype:
        raise NotImplementedError("MatrixMan CPU readback does not support dtype conversion")
    if layout not in (None, torch.strided):
        raise NotImplementedError("MatrixMan CPU readback supports strided layout only")
    if pin_memory:
        raise NotImplementedError("MatrixMan CPU readback does not support pin_memory")
    target = torch.device(device) if device is not None else source.device
    if target.type == "cpu":
        if memory_format not in (None, torch.preserve_format):
            raise NotImplementedError("MatrixMan CPU readback supports preserve_format only")
        return readback_tensor(source)
    if target.type == "matrixman":
        if (target.index or 0) != source.runtime.index:
            raise NotImplementedError("MatrixMan/CUDA: cross-device copies use matrixman.replicas")
        return ops.clone(source, memory_format)
    raise NotImplementedError("MatrixMan only supports explicit MatrixMan-to-CPU transfer")


@_register(aten.clone.default)
def _clone(x, memory_format=None):
    return ops.clone(x, memory_format)


@_register(aten.copy_.default)
def _copy_(dst, src, non_blocking=False):
    if isinstance(dst, MatrixManTensor):
        if isinstance(src, MatrixManTensor):
            return ops.copy_into(src, dst)
        if isinstance(src, torch.Tensor):
            return ops.upload_cpu_into(src, dst)
    raise NotImplementedError("MatrixMan/CUDA: copy_ into a CPU tensor; use .cpu() for readback")


@_register(aten.detach.default, aten.alias.default, aten.lift_fresh.default)
def _detach(x):
    return _view(x, tuple(x.shape), x._logical_strides)


# ---------------------------------------------------------------------------
# Metadata-only views
# ---------------------------------------------------------------------------

@_register(aten.view.default, aten._unsafe_view.default, aten._reshape_alias.default,
           aten.reshape.default)
def _view_op(x, size, *rest):
    shape = infer_view_shape(x.shape, size)
    strides = view_strides(x.shape, x._logical_strides, shape)
    if strides is None:
        raise RuntimeError(
            "MatrixMan/CUDA: view size is not compatible with input tensor's size and stride "
            "(at least one dimension spans across two contiguous subspaces). Use .reshape(...) "
            "instead.")
    return _view(x, shape, strides)


@_register(aten.unsqueeze.default)
def _unsqueeze(x, dim):
    s, st = unsqueeze_shape_strides(x.shape, x._logical_strides, dim)
    return _view(x, s, st)


@_register(aten.squeeze.dim, aten.squeeze.dims, aten.squeeze.default)
def _squeeze(x, dim=None):
    rank = x.dim()
    if dim is None:
        dims = set(range(rank))
    elif isinstance(dim, (list, tuple)):
        dims = {_norm_dim(d, rank) for d in dim}
    else:
        dims = {_norm_dim(dim, rank)}
    shape, strides = [], []
    for i, (s, st) in enumerate(zip(x.shape, x._logical_strides)):
        if i in dims and s == 1:
            continue
        shape.append(int(s))
        strides.append(int(st))
    return _view(x, tuple(shape), tuple(strides))


@_register(aten.transpose.int)
def _transpose(x, dim0, dim1):
    rank = x.dim()
    d0, d1 = _norm_dim(dim0, rank), _norm_dim(dim1, rank)
    shape, strides = list(x.shape), list(x._logical_strides)
    shape[d0], shape[d1] = shape[d1], shape[d0]
    strides[d0], strides[d1] = strides[d1], strides[d0]
    return _view(x, tuple(shape), tuple(strides))


@_register(aten.t.default)
def _t(x):
    if x.dim() < 2:
        return _view(x, tuple(x.shape), x._logical_strides)
    return _transpose(x, 0, 1)


@_register(aten.permute.default)
def _permute(x, dims):
    rank = x.dim()
    order = [_norm_dim(d, rank) for d in dims]
    if sorted(order) != list(range(rank)):
        raise RuntimeError("MatrixMan/CUDA: permute dims must be a permutation")
    return _view(x, tuple(int(x.shape[d]) for d in order), tuple(x._logical_strides[d] for d in order))


@_register(aten.expand.default)
def _expand(x, size, implicit=False):
    s, st = expand_shape_strides(x.shape, x._logical_strides, size)
    return _view(x, s, st)


@_register(aten.slice.Tensor)
def _slice(x, dim=0, start=None, end=None, step=1):
    rank = x.dim()
    d = _norm_dim(dim, rank)
    size = int(x.shape[d])
    step = int(step)
    if step <= 0:
        raise ValueError("MatrixMan/CUDA: slice step must be positive")
    start = 0 if start is None else int(start)
    end = size if end is None else int(end)
    if start < 0:
        start += size
    if end < 0:
        end += size
    start = min(max(start, 0), size)
    end = min(max(end, start), size)
    length = (end - start + step - 1) // step
    shape, strides = list(x.shape), list(x._logical_strides)
    offset = x._storage_offset + start * strides[d]
    shape[d] = length
    strides[d] = strides[d] * step
    return _view(x, tuple(shape), tuple(strides), offset if length > 0 else x._storage_offset)


@_register(aten.select.int)
def _select(x, dim, index):
    rank = x.dim()
    d = _norm_dim(dim, rank)
    size = int(x.shape[d])
    i = int(index)
    if i < 0:
        i += size
    if i < 0 or i >= size:
        raise IndexError("MatrixMan/CUDA: select index out of range")
    shape = tuple(int(s) for j, s in enumerate(x.shape) if j != d)
    strides = tuple(int(s) for j, s in enumerate(x._logical_strides) if j != d)
    return _view(x, shape, strides, x._storage_offset + i * x._logical_strides[d])


@_register(aten.split.Tensor)
def _split(x, split_size, dim=0):
    d = _norm_dim(dim, x.dim())
    size = int(x.shape[d])
    split_size = int(split_size)
    if split_size <= 0:
        raise ValueError("MatrixMan/CUDA: split size must be positive")
    sizes = [min(split_size, size - s) for s in range(0, size, split_size)] or [0]
    return _split_with_sizes(x, sizes, d)


@_register(aten.split_with_sizes.default)
def _split_with_sizes(x, split_sizes, dim=0):
    d = _norm_dim(dim, x.dim())
    if sum(int(s) for s in split_sizes) != int(x.shape[d]):
        raise RuntimeError("MatrixMan/CUDA: split_with_sizes sizes must sum to the dimension")
    out, start = [], 0
    for s in split_sizes:
        out.append(_slice(x, d, start, start + int(s)))
        start += int(s)
    return tuple(out)


@_register(aten.unbind.int)
def _unbind(x, dim=0):
    d = _norm_dim(dim, x.dim())
    return tuple(_select(x, d, i) for i in range(int(x.shape[d])))


@_register(aten.as_strided_.default)
def _as_strided_(x, size, stride, storage_offset=None):
    """In-place restride.  Only metadata-equivalent requests are accepted
    (same sizes; strides may differ only on size-1 dims), which is what ATen's
    adaptive_avg_pool2d composite issues for 1x1 channels-last outputs."""
    size = tuple(int(s) for s in size)
    stride = tuple(int(s) for s in stride)
    same_offset = storage_offset is None or int(storage_offset) == x._storage_offset
    if size == tuple(x.shape) and same_offset and all(
            s == 1 or a == b for s, a, b in zip(size, stride, x._logical_strides)):
        return x
    raise NotImplementedError("MatrixMan/CUDA: as_strided_ that changes the memory layout is "
                              "not implemented")


@_register(aten.as_strided.default)
def _as_strided(x, size, stride, storage_offset=None):
    off = x._storage_offset if storage_offset is None else int(storage_offset)
    return MatrixManTensor._from_owner(x._owner, tuple(int(s) for s in size), off,
                                       tuple(int(s) for s in stride))


# ---------------------------------------------------------------------------
# Compute
# ---------------------------------------------------------------------------

@_register(aten.convolution.default)
def _convolution(x, weight, bias, stride, padding, dilation, transposed, output_padding, groups):
    if bool(transposed) or any(int(v) for v in output_padding):
        raise NotImplementedError(
            "MatrixMan/CUDA: transposed convolution and output padding are not implemented")
    return ops.convolution(x, weight, bias, stride, padding, dilation, groups)


@_register(aten.addmm.default)
def _addmm(bias, mat1, mat2, beta=1, alpha=1):
    return ops.gemm(mat1, mat2, bias, alpha=float(alpha), beta=float(beta))


@_register(aten.mm.default)
def _mm(a, b):
    return ops.gemm(a, b)


@_register(aten._softmax.default)
def _softmax(x, dim, half_to_float=False):
    return ops.softmax(x, dim, log=False)


@_register(aten._log_softmax.default)
def _log_softmax(x, dim, half_to_float=False):
    return ops.softmax(x, dim, log=True)


# -- training path (backward passes, Adam's update) --------------------------
from . import _lib as _native_lib  # noqa: E402


def _scalar_arg(v, op):
    if isinstance(v, torch.Tensor) and not isinstance(v, MatrixManTensor) and v.numel() == 1:
        return float(v.item())
    if isinstance(v, (int, float, bool)):
        return float(v)
    raise RuntimeError(f"MatrixMan/CUDA: {op} needs a numeric scalar")


@_register(aten.threshold_backward.default)
def _threshold_backward(grad_output, self, threshold):
    if tuple(grad_output.shape) != tuple(self.shape):
        raise RuntimeError("MatrixMan/CUDA: threshold_backward requires equal shapes")
    return ops.pointwise3(_native_lib.PW3_THRESHOLD_BACKWARD, grad_output, self, grad_output,
                          _scalar_arg(threshold, "threshold_backward"), name="threshold_backward")


@_register(aten._log_softmax_backward_data.default)
def _log_softmax_backward(grad_output, output, dim, input_dtype):
    return ops.log_softmax_backward(grad_output, output, dim)


@_register(aten.nll_loss_forward.default)
def _nll_loss_forward(self, target, weight, reduction, ignore_index):
    return ops.nll_loss(self, target, weight, reduction, ignore_index)


@_register(aten.nll_loss_backward.default)
def _nll_loss_backward(grad_output, self, target, weight, reduction, ignore_index, total_weight):
    return ops.nll_loss_backward(grad_output, self, target, weight, reduction, ignore_index, total_weight)


def _pw3_inplace(code, self, a, b, s, name):
    return ops.pointwise3(code, self, a, b, s, out=self, name=name)


@_register(aten.addcmul.default)
def _addcmul(self, tensor1, tensor2, *, value=1):
    return ops.pointwise3(_native_lib.PW3_ADDCMUL, self, tensor1, tensor2, _scalar_arg(value, "addcmul"),
                          name="addcmul")


@_register(aten.addcmul_.default)
def _addcmul_(self, tensor1, tensor2, *, value=1):
    return _pw3_inplace(_native_lib.PW3_ADDCMUL, self, tensor1, tensor2, _scalar_arg(value, "addcmul_"),
                        "addcmul_")


@_register(aten.addcdiv.default)
def _addcdiv(self, tensor1, tensor2, *, value=1):
    return ops.pointwise3(_native_lib.PW3_ADDCDIV, self, tensor1, tensor2, _scalar_arg(value, "addcdiv"),
                          name="addcdiv")


@_register(aten.addcdiv_.default)
def _addcdiv_(self, tensor1, tensor2, *, value=1):
    return _pw3_inplace(_native_lib.PW3_ADDCDIV, self, tensor1, tensor2, _scalar_arg(value, "addcdiv_"),
                        "addcdiv_")


@_register(aten.lerp.Scalar)
def _lerp(self, end, weight):
    return ops.pointwise3(_native_lib.PW3_LERP, self, end, None, _scalar_arg(weight, "lerp"), name="lerp")


@_register(aten.lerp_.Scalar)
def _lerp_(self, end, weight):
    return _pw3_inplace(_native_lib.PW3_LERP, self, end, None, _scalar_arg(weight, "lerp_"), "lerp_")


@_register(aten.sqrt.default)
def _sqrt(self):
    return ops.pointwise3(_native_lib.PW3_SQRT, self, name="sqrt")


@_register(aten.sqrt_.default)
def _sqrt_(self):
    return _pw3_inplace(_native_lib.PW3_SQRT, self, None, None, 0.0, "sqrt_")


@_register(aten.relu.default)
def _relu(x):
    return ops.unary("relu", x)


@_register(aten.relu_.default)
def _relu_(x):
    ops.unary("relu", x, out=x)
    return x


@_register(aten.silu.default)
def _silu(x):
    return ops.unary("silu", x)


@_register(aten.silu_.default)
def _silu_(x):
    ops.unary("silu", x, out=x)
    return x


@_register(aten.sigmoid.default)
def _sigmoid(x):
    return ops.unary("sigmoid", x)


@_register(aten.sigmoid_.default)
def _sigmoid_(x):
    ops.unary("sigmoid", x, out=x)
    return x


@_register(aten.neg.default)
def _neg(x):
    return ops.unary("neg", x)


@_register(aten.hardtanh.default, aten.clamp.default)
def _clamp(x, min_val=None, max_val=None):
    lo = -float("inf") if min_val is None else float(min_val)
    hi = float("inf") if max_val is None else float(max_val)
    return ops.unary("clamp", x, a=lo, b=hi, code=8)


@_register(aten.add.Tensor, aten.add.Scalar)
def _add(a, b, alpha=1):
    return ops.binary("add", a, b, alpha)


@_register(aten.add_.Tensor, aten.add_.Scalar)
def _add_(a, b, alpha=1):
    return ops.binary("add", a, b, alpha, out=a)


@_register(aten.sub.Tensor, aten.sub.Scalar)
def _sub(a, b, alpha=1):
    return ops.binary("sub", a, b, alpha)


@_register(aten.sub_.Tensor)
def _sub_(a, b, alpha=1):
    return ops.binary("sub", a, b, alpha, out=a)


@_register(aten.rsub.Scalar, aten.rsub.Tensor)
def _rsub(a, b, alpha=1):
    return ops.binary("sub", b, a, alpha)


@_register(aten.mul.Tensor, aten.mul.Scalar)
def _mul(a, b):
    return ops.binary("mul", a, b)


@_register(aten.mul_.Tensor, aten.mul_.Scalar)
def _mul_(a, b):
    return ops.binary("mul", a, b, out=a)


@_register(aten.div.Tensor, aten.div.Scalar)
def _div(a, b):
    return ops.binary("div", a, b)


@_register(aten.div_.Tensor, aten.div_.Scalar)
def _div_(a, b):
    return ops.binary("div", a, b, out=a)


@_register(aten.cat.default)
def _cat(tensors, dim=0):
    return ops.cat(tensors, dim)


@_register(aten.stack.default)
def _stack(tensors, dim=0):
    return ops.stack(tensors, dim)


@_register(aten.fill_.Scalar)
def _fill_(x, value):
    return ops.fill_(x, value)


@_register(aten.zero_.default)
def _zero_(x):
    return ops.fill_(x, 0.0)


@_register(aten.upsample_nearest2d.default)
def _upsample_nearest2d(x, output_size, scales_h=None, scales_w=None):
    return ops.upsample_nearest2d(x, output_size, scales_h, scales_w)


@_register(aten.upsample_nearest2d.vec)
def _upsample_nearest2d_vec(x, output_size, scale_factors):
    sh = sw = None
    if scale_factors is not None:
        sh, sw = (float(s) for s in scale_factors)
    return ops.upsample_nearest2d(x, output_size, sh, sw)


@_register(aten.max_pool2d_with_indices.default)
def _max_pool2d_with_indices(x, kernel_size, stride=(), padding=0, dilation=1, ceil_mode=False):
    values = ops.max_pool2d(x, kernel_size, stride, padding, dilation, ceil_mode)
    # Indices are not materialised on the device (reference dispatch.py:356-357).
    return values, torch.empty((0,), dtype=torch.int64, device="cpu")


@_register(aten.max_pool2d.default)
def _max_pool2d(x, kernel_size, stride=(), padding=0, dilation=1, ceil_mode=False):
    return ops.max_pool2d(x, kernel_size, stride, padding, dilation, ceil_mode)


@_register(aten.avg_pool2d.default)
def _avg_pool2d(x, kernel_size, stride=(), padding=0, ceil_mode=False, count_include_pad=True,
                divisor_override=None):
    return ops.avg_pool2d(x, kernel_size, stride, padding, ceil_mode, count_include_pad,
                          divisor_override)


@_register(aten._adaptive_avg_pool2d.default, aten.adaptive_avg_pool2d.default)
def _adaptive_avg_pool2d(x, output_size):
    return ops.adaptive_avg_pool2d(x, output_size)


@_register(aten.mean.dim)
def _mean_dim(x, dim, keepdim=False, dtype=None):
    if dtype is not None and dtype != torch.float32:
        raise NotImplementedError("MatrixMan/CUDA: mean supports float32 only")
    return ops.reduce(x, dim, keepdim, mean=True)


@_register(aten.mean.default)
def _mean(x, dtype=None):
    return ops.reduce(x, None, False, mean=True)


@_register(aten.sum.dim_IntList)
def _sum_dim(x, dim, keepdim=False, dtype=None):
    return ops.reduce(x, dim, keepdim, mean=False)


@_register(aten.native_batch_norm.default)
def _native_batch_norm(x, weight, bias, running_mean, running_var, training, momentum, eps):
    if bool(training):
        raise NotImplementedError("MatrixMan/CUDA: BatchNorm training mode is not implemented")
    out = ops.batch_norm_eval(x, weight, bias, running_mean, running_var, eps)
    empty = torch.empty((0,), dtype=torch.float32)
    return out, empty, empty


@_register(aten._native_batch_norm_legit_no_training.default)
def _bn_legit_no_training(x, weight, bias, running_mean, running_var, momentum, eps):
    out = ops.batch_norm_eval(x, weight, bias, running_mean, running_var, eps)
    empty = torch.empty((0,), dtype=torch.float32)
    return out, empty, empty


# ---------------------------------------------------------------------------
# Factories reached through a MatrixMan tensor argument
# ---------------------------------------------------------------------------

def _factory_runtime(x, device):
    if device is not None:
        dev = torch.device(device)
        if dev.type != "matrixman":
            raise NotImplementedError("MatrixMan/CUDA: factory on another device")
        from .runtime import get_runtime
        return get_runtime(dev.index or 0)
    return x.runtime


def _check_dtype(dtype, x):
    dtype = x.dtype if dtype is None else dtype
    if dtype not in (torch.float32, torch.int64):
        raise NotImplementedError(f"MatrixMan/CUDA: unsupported dtype {dtype}")
    return dtype


@_register(aten.new_full.default)
def _new_full(x, size, fill_value, dtype=None, layout=None, device=None, pin_memory=None):
    rt = _factory_runtime(x, device)
    return ops.full(rt, tuple(int(s) for s in size), float(fill_value), _check_dtype(dtype, x))


@_register(aten.new_zeros.default)
def _new_zeros(x, size, dtype=None, layout=None, device=None, pin_memory=None):
    return _new_full(x, size, 0.0, dtype, layout, device, pin_memory)


@_register(aten.new_ones.default)
def _new_ones(x, size, dtype=None, layout=None, device=None, pin_memory=None):
    return _new_full(x, size, 1.0, dtype, layout, device, pin_memory)


@_register(aten.new_empty.default)
def _new_empty(x, size, dtype=None, layout=None, device=None, pin_memory=None):
    rt = _factory_runtime(x, device)
    return ops.empty(rt, tuple(int(s) for s in size), None, _check_dtype(dtype, x))


@_register(aten.new_empty_strided.default)
def _new_empty_strided(x, size, stride, dtype=None, layout=None, device=None, pin_memory=None):
    rt = _factory_runtime(x, device)
    return ops.empty(rt, tuple(int(s) for s in size), tuple(int(s) for s in stride), _check_dtype(dtype, x))


@_register(aten.empty_like.default)
def _empty_like(x, dtype=None, layout=None, device=None, pin_memory=None, memory_format=None):
    rt = _factory_runtime(x, device)
    dtype = _check_dtype(dtype, x)
    if memory_format is torch.contiguous_format:
        strides = contiguous_strides(x.shape)
    else:
        from .tensor import dense_strides_like
        strides = dense_strides_like(x.shape, x._logical_strides)
    return ops.empty(rt, tuple(x.shape), strides, dtype)


@_register(aten.zeros_like.default)
def _zeros_like(x, dtype=None, layout=None, device=None, pin_memory=None, memory_format=None):
    y = _empty_like(x, dtype, layout, device, pin_memory, memory_format)
    return ops.fill_(y, 0.0)


@_register(aten.ones_like.default)
def _ones_like(x, dtype=None, layout=None, device=None, pin_memory=None, memory_format=None):
    y = _empty_like(x, dtype, layout, device, pin_memory, memory_format)
    return ops.fill_(y, 1.0)


@_register(aten.full_like.default)
def _full_like(x, fill_value, dtype=None, layout=None, device=None, pin_memory=None,
               memory_format=None):
    y = _empty_like(x, dtype, layout, device, pin_memory, memory_format)
    return ops.fill_(y, fill_value)


@_register(aten.arange.out, aten.arange.start_out)
def _arange_out(*args, out=None, **kwargs):
    if out is None:
        raise RuntimeError("MatrixMan/CUDA: malformed arange.out arguments")
    vals = [float(a) for a in args]
    if len(vals) == 1:
        start, end, step = 0.0, vals[0], 1.0
    elif len(vals) == 2:
        start, end, step = vals[0], vals[1], 1.0
    else:
        start, end, step = vals[0], vals[1], vals[2]
    import math
    n = max(int(math.ceil((end - start) / step)), 0)
    if tuple(out.shape) != (n,):
        raise RuntimeError(f"MatrixMan/CUDA: arange.out expects out of shape ({n},)")
    return ops.arange_into(out, start, step)
