"""``MatrixManTensor``: the PrivateUse1 wrapper subclass and its metadata rules.

Mirrors drivers/matrixman/tensor.py of the reference: a wrapper subclass made
with ``_make_wrapper_subclass`` on the ``matrixman`` device that holds an
owner (here a ``runtime.DeviceStorage``), an element storage offset and
logical strides (tensor.py:307-350), routes every ATen op to the dispatch
module (tensor.py:352-359), and supports only explicit readback to the CPU
(tensor.py:76-158).  Unlike the reference, views may carry any non-negative
strides: prepared models keep activations channels-last (NHWC) under the
logical NCHW shape, and channel slices of concat buffers are zero-copy views.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .privateuse import device_for, register_privateuse1_backend

register_privateuse1_backend()


# ---------------------------------------------------------------------------
# Shape / stride helpers (own implementations of the rules torch applies).
# ---------------------------------------------------------------------------

def numel(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


def contiguous_strides(shape) -> tuple[int, ...]:
    strides = []
    acc = 1
    for size in reversed(tuple(shape)):
        strides.append(acc)
        acc *= max(int(size), 1)
    return tuple(reversed(strides))


def channels_last_strides(shape) -> tuple[int, ...]:
    """Strides of an NHWC buffer viewed with logical NCHW shape."""
    n, c, h, w = (int(s) for s in shape)
    c1, w1, h1 = max(c, 1), max(w, 1), max(h, 1)
    return (h1 * w1 * c1, 1, w1 * c1, c1)


def max_storage_index(shape, strides) -> int:
    if numel(shape) == 0:
        return 0
    return sum((int(s) - 1) * int(st) for s, st in zip(shape, strides))


def is_contiguous(shape, strides) -> bool:
    """torch's definition: size-1 dims may carry any stride."""
    expected = 1
    for size, stride in zip(reversed(tuple(shape)), reversed(tuple(strides))):
        if size == 1:
            continue
        if stride != expected:
            return False
        expected *= size
    return True


def dense_strides_like(shape, strides) -> tuple[int, ...]:
    """Strides of a dense tensor with the same dim ordering as `strides`.

    Equivalent in intent to torch's preserve_format for non-overlapping dense
    inputs (channels-last stays channels-last); any other input gets
    contiguous strides.
    """
    shape = tuple(int(s) for s in shape)
    strides = tuple(int(s) for s in strides)
    if len(shape) == 4 and is_dense(shape, strides) and is_channels_last(shape, strides):
        return channels_last_strides(shape)
    return contiguous_strides(shape)


def is_dense(shape, strides) -> bool:
    """Non-overlapping and dense (every element of a span of numel used once)."""
    dims = [(int(st), int(sz)) for sz, st in zip(shape, strides) if int(sz) != 1]
    dims.sort(key=lambda p: p[0])
    expected = 1
    for st, sz in dims:
        if sz == 0:
            return True
        if st != expected:
            return False
        expected *= sz
    return True


def is_channels_last(shape, strides) -> bool:
    if len(shape) != 4:
        return False
    n, c, h, w = (int(s) for s in shape)
    exp = channels_last_strides(shape)
    for size, st, e in zip((n, c, h, w), strides, exp):
        if size != 1 and int(st) != e:
            return False
    return c > 1 or h * w > 1


def infer_view_shape(input_shape, requested_shape) -> tuple[int, ...]:
    """Resolve one -1 entry (same rule as reference tensor.py:161-186)."""
    requested = [int(s) for s in requested_shape]
    unknown = [i for i, s in enumerate(requested) if s == -1]
    if len(unknown) > 1 or any(s < -1 for s in requested):
        raise ValueError("MatrixMan view accepts at most one -1 dimension")
    total = numel(input_shape)
    known = numel([s for s in requested if s != -1])
    if unknown:
        if known == 0 or total % known:
            raise ValueError("MatrixMan view cannot infer a compatible dimension")
        requested[unknown[0]] = total // known
    if numel(requested) != total:
        raise ValueError("MatrixMan view must preserve the number of elements")
    return tuple(requested)


def view_strides(old_shape, old_strides, new_shape):
    """Strides for viewing (old_shape, old_strides) as new_shape, or None.

    Same feasibility rule as torch's view: dims of the new shape must map onto
    groups of old dims that are mutually contiguous.
    """
    old_shape = [int(s) for s in old_shape]
    old_strides = [int(s) for s in old_strides]
    new_shape = [int(s) for s in new_shape]
    if numel(old_shape) == 0:
        return contiguous_strides(new_shape)
    new_strides = [0] * len(new_shape)
    view_d = len(new_shape) - 1
    chunk_base_stride = old_strides[-1] if old_strides else 1
    tensor_numel = 1
    view_numel = 1
    for tensor_d in range(len(old_shape) - 1, -1, -1):
        tensor_numel *= old_shape[tensor_d]
        if tensor_d == 0 or (old_shape[tensor_d - 1] != 1 and
                             old_strides[tensor_d - 1] != tensor_numel * chunk_base_stride):
            while view_d >= 0 and (view_numel < tensor_numel or new_shape[view_d] == 1):
                new_strides[view_d] = view_numel * chunk_base_stride
                view_numel *= new_shape[view_d]
                view_d -= 1
            if view_numel != tensor_numel:
                return None
            if tensor_d > 0:
                chunk_base_stride = old_strides[tensor_d - 1]
                tensor_numel = 1
                view_numel = 1
    if view_d != -1:
        return None
    return tuple(new_strides)


def expand_shape_strides(input_shape, input_strides, requested_shape):
    """Expanded shape/strides without touching storage (torch expand rules)."""
    src = [int(s) for s in input_shape]
    st = [int(s) for s in input_strides]
    req = [int(s) for s in requested_shape]
    if len(req) < len(src):
        raise ValueError("MatrixMan expand cannot remove dimensions")
    lead = len(req) - len(src)
    out_shape, out_strides = [], []
    for i, r in enumerate(req):
        if i < lead:
            if r < 0:
                raise ValueError("MatrixMan expand does not allow -1 on prepended dimensions")
            out_shape.append(r)
            out_strides.append(0)
            continue
        size, stride = src[i - lead], st[i - lead]
        target = size if r == -1 else r
        if target < 0:
            raise ValueError("MatrixMan expand sizes must be non-negative or -1")
        if size != target:
            if size != 1:
                raise ValueError(f"MatrixMan expand cannot change dimension {i - lead} "
                                 f"from {size} to {target}")
            stride = 0
        out_shape.append(target)
        out_strides.append(stride)
    return tuple(out_shape), tuple(out_strides)


def unsqueeze_shape_strides(input_shape, input_strides, dim):
    shape = tuple(int(s) for s in input_shape)
    strides = tuple(int(s) for s in input_strides)
    rank = len(shape)
    d = int(dim)
    if d < 0:
        d += rank + 1
    if d < 0 or d > rank:
        raise IndexError("MatrixMan unsqueeze dimension is out of range")
    inserted = 1 if d == rank else strides[d] * shape[d]
    return shape[:d] + (1,) + shape[d:], strides[:d] + (inserted,) + strides[d:]


def broadcast_shapes(*shapes) -> tuple[int, ...]:
    rank = max(len(s) for s in shapes)
    out = []
    for i in range(rank):
        size = 1
        for s in shapes:
            j = i - (rank - len(s))
            if j < 0:
                continue
            d = int(s[j])
            if d == 1:
                continue
            if size != 1 and size != d:
                raise RuntimeError(f"MatrixMan/CUDA: shapes {shapes} are not broadcastable")
            size = d
        out.append(size)
    return tuple(out)


# ---------------------------------------------------------------------------
# The wrapper subclass.
# ---------------------------------------------------------------------------

class MatrixManTensor(torch.Tensor):
    """Wrapper around a device storage owner (reference tensor.py:307-367)."""

    @staticmethod
    def __new__(cls, owner, shape, storage_offset=0, logical_strides=None):
        shape = tuple(int(s) for s in shape)
        strides = tuple(logical_strides) if logical_strides is not None else contiguous_strides(shape)
        return torch.Tensor._make_wrapper_subclass(
            cls, shape, strides=strides, storage_offset=int(storage_offset),
            dtype=owner.dtype, layout=torch.strided,
            device=device_for(owner.device_index), requires_grad=False,
        )

    def __init__(self, owner, shape, storage_offset=0, logical_strides=None):
        self._owner = owner
        self._storage_offset = int(storage_offset)
        self._logical_strides = tuple(int(s) for s in (
            logical_strides if logical_strides is not None else contiguous_strides(shape)))

    @staticmethod
    def _from_owner(owner, shape, storage_offset=0, logical_strides=None):
        shape = tuple(int(s) for s in shape)
        strides = tuple(int(s) for s in (logical_strides if logical_strides is not None
                                          else contiguous_strides(shape)))
        if len(strides) != len(shape):
            raise RuntimeError("MatrixMan tensor logical strides must match shape rank")
        if any(s < 0 for s in strides):
            raise RuntimeError("MatrixMan tensor strides must be non-negative")
        if storage_offset < 0 or (numel(shape) > 0 and
                                  storage_offset + max_storage_index(shape, strides) >= owner.layout.numel):
            raise RuntimeError("MatrixMan tensor view storage offset is outside owner storage")
        return MatrixManTensor(owner, shape, storage_offset, strides)

    # -- C ABI view ---------------------------------------------------------
    @property
    def element_ptr(self) -> int:
        from .runtime import ELEMENT_SIZE
        return self._owner.pointer + self._storage_offset * ELEMENT_SIZE[self.dtype]

    def desc(self) -> _lib.MMTensor:
        return _lib.make_tensor(self.element_ptr, self.shape, self._logical_strides,
                                _lib.MM_F32 if self.dtype == torch.float32 else _lib.MM_I64)

    @property
    def runtime(self):
        return self._owner.runtime

    def requires_grad_(self, requires_grad=True):
        if requires_grad:
            from .privateuse import register_native_hooks
            register_native_hooks()
        return torch.Tensor.requires_grad_(self, requires_grad)

    @classmethod
    def __torch_dispatch__(cls, func, types, args=(), kwargs=None):
        from . import dispatch
        return dispatch.handle_torch_dispatch(cls, func, types, args, kwargs)

    def __repr__(self):
        return (f"MatrixManTensor(shape={tuple(self.shape)}, dtype={self.dtype}, device={self.device}, "
                f"{self._owner.storage_description}, storage={self._owner.layout.kind}, "
                f"offset={self._storage_offset}, strides={self._logical_strides})")


Gm45Tensor = MatrixManTensor


def is_matrixman_tensor(value) -> bool:
    return isinstance(value, MatrixManTensor)


# ---------------------------------------------------------------------------
# Readback (reference tensor.py:76-158): explicit, synchronising, exact values.
# ---------------------------------------------------------------------------

def readback_tensor(tensor: MatrixManTensor) -> torch.Tensor:
    """Copy a MatrixMan tensor to an ordinary CPU tensor (waits, bounded)."""
    if not isinstance(tensor, MatrixManTensor):
        raise TypeError("MatrixMan CPU readback requires a MatrixManTensor")
    if tensor.dtype not in (torch.float32, torch.int64):
        raise NotImplementedError(
            f"MatrixMan CPU readback supports float32 and int64 only, got {tensor.dtype}")
    from . import audit
    audit.record("explicit_readback", tensor)
    shape = tuple(int(s) for s in tensor.shape)
    strides = tensor._logical_strides
    rt = tensor.runtime
    n = numel(shape)
    if n == 0:
        return torch.empty(shape, dtype=tensor.dtype)
    from .runtime import host_empty
    if is_contiguous(shape, strides):
        out = host_empty(shape, tensor.dtype)
        rt.download(tensor.element_ptr, out)
        return out
    if is_dense(shape, strides):
        # Dense permutation (e.g. NHWC): copy the span, keep the strides.
        flat = host_empty((n,), tensor.dtype)
        rt.download(tensor.element_ptr, flat)
        return torch.as_strided(flat, shape, strides)
    # Sliced / expanded views: gather on the device into a contiguous block.
    from . import ops
    dense = ops.materialize(tensor)
    out = host_empty(shape, tensor.dtype)
    rt.download(dense.element_ptr, out)
    return out


def install_tensor_method() -> None:
    """Install the historical Tensor.gm45() upload convenience (reference tensor.py:290-297)."""
    def upload(value):
        from .api import to_device
        return to_device(value)
    setattr(torch.Tensor, "gm45", upload)
