"""Whole-model replicas on several devices of one node.

MatrixMan runs one process-global backend on one device (one context on
device 0, ``backends/cuda/gpumatrix.py:4555``; threading model in
``backends/opengl/runtime.py:122-135``).  Inference over a batch shards
naturally: images are independent, so each device runs the whole prepared
model on a contiguous slice of the batch, parameters are uploaded once per
device, and nothing crosses devices during the forward.  The only exchange is
the final gather of the per-replica outputs:

* ``ReplicaSet`` (one process, several devices): replicas are enqueued on
  each device's stream back to back and run concurrently; their outputs are
  copied into one buffer on the root device with copy-engine peer copies
  (NVLink when peer access is available), ordered by cross-device events.
* ``PeerGather`` (one process per device, e.g. under torchrun): rank 0's
  gather buffers are shared through CUDA IPC and every rank writes its rows
  with copy-engine copies over NVLink on a side stream, so a step's gather
  overlaps the next step's forward and uses no SMs.
* ``gather_to_root`` (one process per device): rank outputs travel to rank 0
  with point-to-point sends over the process group (NCCL over NVLink for
  device memory, gloo for CPU tensors in tests).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, ops, runtime
from .tensor import MatrixManTensor, contiguous_strides


def batch_slices(batch: int, parts: int) -> list[tuple[int, int]]:
    """Contiguous [start, end) slices of `batch` over `parts` replicas; the
    first `batch % parts` replicas take one extra image."""
    if parts <= 0:
        raise ValueError("MatrixMan: replica count must be positive")
    if batch < 0:
        raise ValueError("MatrixMan: batch size must be non-negative")
    base, extra = divmod(int(batch), int(parts))
    out, start = [], 0
    for r in range(parts):
        n = base + (1 if r < extra else 0)
        out.append((start, start + n))
        start += n
    return out


def _dense(t: MatrixManTensor) -> MatrixManTensor:
    if tuple(t._logical_strides) == contiguous_strides(tuple(int(v) for v in t.shape)):
        return t
    return ops.materialize(t)


def _leaves(value):
    if isinstance(value, (tuple, list)):
        out = []
        for v in value:
            out.extend(_leaves(v))
        return out
    return [value]


def _rebuild(template, leaves):
    it = iter(leaves)

    def walk(v):
        if isinstance(v, (tuple, list)):
            return type(v)(walk(x) for x in v)
        return next(it)

    return walk(template)


class _Event:
    def __init__(self, device: int):
        runtime.set_device(device)
        self.handle = ctypes.c_void_p()
        _lib.check(_lib.load().mm_event_create(ctypes.byref(self.handle), 0), "event create")

    def __del__(self):
        try:
            _lib.load().mm_event_destroy(self.handle)
        except Exception:
            pass


class ReplicaSet:
    """Run a prepared model on several devices, one batch slice each.

    ``model`` is prepared once (BN folded, weights prepacked); the prepared
    module caches its device weights and CUDA graphs per device, so one
    object serves every replica.  Calling the set with a CPU batch (pinned
    memory makes the uploads asynchronous) returns the outputs of the whole
    batch as MatrixMan tensors on the root device (``devices[0]``)."""

    def __init__(self, model: torch.nn.Module, devices=None, *, prepared: bool = False):
        from .api import get_backend
        from .preparation import prepare

        get_backend()
        self.devices = [int(d) for d in (devices if devices is not None
                                         else range(runtime.device_count()))]
        if not self.devices:
            raise RuntimeError("MatrixMan/CUDA: no devices available for replicas")
        if len(set(self.devices)) != len(self.devices):
            raise ValueError("MatrixMan: replica devices must be distinct")
        self.model = model if prepared else prepare(model)
        self.root = self.devices[0]
        lib = _lib.load()
        self.peer = {}
        for d in self.devices:
            runtime.get_runtime(d)
        for d in self.devices[1:]:
            # Without peer access cudaMemcpyPeerAsync stages through the host:
            # still correct, just slower.
            self.peer[d] = lib.mm_enable_peer_access(self.root, d) == _lib.MM_OK
        self._events = {d: _Event(d) for d in self.devices}
        runtime.set_device(self.root)

    def forward_slices(self, x: torch.Tensor):
        """Upload and run every slice; returns [(device, start, end, output)]."""
        from .api import to_device

        if not isinstance(x, torch.Tensor) or x.device.type != "cpu":
            raise TypeError("MatrixMan: ReplicaSet expects a CPU batch tensor")
        x = x.contiguous()
        results = []
        with torch.no_grad():
            for d, (s, e) in zip(self.devices, batch_slices(int(x.shape[0]), len(self.devices))):
                if s == e:
                    continue
                runtime.set_device(d)
                results.append((d, s, e, self.model(to_device(x[s:e], device=d))))
        return results

    def gather(self, results, batch: int):
        """Copy the replicas' outputs into root-device buffers (batch-major)."""
        if not results:
            raise ValueError("MatrixMan: empty batch")
        lib = _lib.load()
        rt0 = runtime.get_runtime(self.root)
        template = results[0][3]
        per_leaf = [_leaves(r[3]) for r in results]
        gathered = []
        for li, leaf in enumerate(_leaves(template)):
            if not isinstance(leaf, MatrixManTensor):
                raise NotImplementedError("MatrixMan: replica outputs must be MatrixMan tensors")
            shape = (int(batch),) + tuple(int(v) for v in leaf.shape[1:])
            runtime.set_device(self.root)
            out = ops.empty(rt0, shape, contiguous_strides(shape))
            # The block is stream-ordered on the root stream: the copies issued on
            # the other devices' streams start only after the root reaches here.
            root_ev = self._events[self.root].handle
            _lib.check(lib.mm_event_record(root_ev, rt0.stream), "event record")
            for d in {r[0] for r in results if r[0] != self.root}:
                _lib.check(lib.mm_stream_wait_event(runtime.get_runtime(d).stream, root_ev),
                           "stream wait")
            row_bytes = 4
            for v in shape[1:]:
                row_bytes *= v
            for (d, s, e, _), leaves in zip(results, per_leaf):
                y = leaves[li]
                if tuple(y.shape[1:]) != shape[1:] or int(y.shape[0]) != e - s:
                    raise RuntimeError("MatrixMan: replica outputs disagree in shape")
                runtime.set_device(d)
                y = _dense(y)
                rt = y.runtime
                dst = out.element_ptr + s * row_bytes
                if d == self.root:
                    rt.copy_d2d(dst, y.element_ptr, (e - s) * row_bytes)
                    continue
                # Issued on the source stream: ordered after the replica's forward,
                # and the arena reuses y's block only after the copy.
                _lib.check(lib.mm_memcpy_peer(ctypes.c_void_p(dst), self.root,
                                              ctypes.c_void_p(y.element_ptr), d,
                                              (e - s) * row_bytes, rt.stream), "peer copy")
                ev = self._events[d].handle
                _lib.check(lib.mm_event_record(ev, rt.stream), "event record")
                _lib.check(lib.mm_stream_wait_event(rt0.stream, ev), "stream wait")
            gathered.append(out)
        runtime.set_device(self.root)
        return _rebuild(template, gathered)

    def __call__(self, x: torch.Tensor):
        return self.gather(self.forward_slices(x), int(x.shape[0]))

    def synchronize(self) -> None:
        for d in self.devices:
            runtime.get_runtime(d).synchronize()


class _CudaArrayView:
    """Exposes a MatrixMan device buffer to torch (``__cuda_array_interface__``)
    so a process group can send or receive it in place."""

    def __init__(self, t: MatrixManTensor):
        if not t.is_contiguous() or t.dtype != torch.float32:
            raise NotImplementedError("MatrixMan: only dense float32 outputs can be gathered")
        self.__cuda_array_interface__ = {
            "shape": tuple(int(v) for v in t.shape),
            "typestr": "<f4",
            "data": (int(t.element_ptr), False),
            "version": 3,
            "strides": None,
            "stream": None,
        }


def _as_torch(t):
    if isinstance(t, MatrixManTensor):
        return torch.as_tensor(_CudaArrayView(t), device=torch.device("cuda", t.runtime.index))
    return t


def gather_to_root(local, batch_sizes: list[int], group=None, root: int = 0):
    """Gather every rank's batch-major output on rank `root`.

    ``local`` is this rank's output (a dense MatrixMan tensor on the rank's
    device, or a CPU tensor with the gloo backend); ``batch_sizes[r]`` is
    rank r's slice size.  Returns the concatenated batch on `root` (a MatrixMan
    tensor on its device, or a CPU tensor) and None elsewhere.  Every rank
    takes the same steps; the transfers are point-to-point sends to `root`."""
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    if len(batch_sizes) != world:
        raise ValueError("MatrixMan: one batch size per rank is required")
    if int(local.shape[0]) != int(batch_sizes[rank]):
        raise ValueError("MatrixMan: local output does not match this rank's batch size")
    on_device = isinstance(local, MatrixManTensor)
    if on_device:
        local = _dense(local)
    stream_ctx = (torch.cuda.stream(torch.cuda.ExternalStream(local.runtime.stream,
                                                              device=local.runtime.index))
                  if on_device else None)
    tail = tuple(int(v) for v in local.shape[1:])
    row = 1
    for v in tail:
        row *= v
    out = None
    p2p = []
    if rank == root:
        total = sum(int(b) for b in batch_sizes)
        if on_device:
            rt = local.runtime
            out = ops.empty(rt, (total,) + tail, contiguous_strides((total,) + tail))
        else:
            out = torch.empty((total,) + tail, dtype=local.dtype)
        start = 0
        for r, b in enumerate(batch_sizes):
            view = out[start:start + b] if not on_device else MatrixManTensor(
                out._owner, (b,) + tail, out._storage_offset + start * row,
                contiguous_strides((b,) + tail))
            if r == rank:
                if on_device:
                    ops.copy_into(local, view)
                else:
                    view.copy_(local)
            elif b > 0:
                p2p.append((r, view))
            start += b
    if stream_ctx is not None:
        stream_ctx.__enter__()
    try:
        ops_list = []
        if rank == root:
            for r, view in p2p:
                ops_list.append(dist.P2POp(dist.irecv, _as_torch(view), r, group))
        elif int(batch_sizes[rank]) > 0:
            ops_list.append(dist.P2POp(dist.isend, _as_torch(local), root, group))
        if ops_list:
            for req in dist.batch_isend_irecv(ops_list):
                req.wait()
    finally:
        if stream_ctx is not None:
            stream_ctx.__exit__(None, None, None)
    return out


class _IpcBlock(runtime.DeviceStorage):
    """A gather buffer allocated for sharing with other processes (CUDA IPC);
    freed with mm_ipc_free instead of returning to the arena."""

    __slots__ = ()

    def release(self) -> None:
        if self._released or self.pointer == 0:
            return
        self._released = True
        if self.runtime.closed:
            return
        _lib.load().mm_ipc_free(self.runtime.index, ctypes.c_void_p(self.pointer))


class PeerGather:
    """Gather of every rank's batch-major output into one buffer on the root's
    GPU by copy engines, one process per GPU (e.g. under torchrun).

    The root allocates ``slots`` gather buffers and exports them through CUDA
    IPC; every rank opens them once.  ``push(local)`` copies this rank's dense
    output into its rows of the current slot with ``cudaMemcpyAsync`` on a copy
    stream of the rank's own, ordered after the output's producer by an event.
    The copies use copy engines over NVLink, not SMs, so they overlap the next
    forward (a process-group collective would occupy SMs that the persistent
    convolution kernels expect to have).  A pushed output stays referenced
    until its copy has completed.  ``collect()`` waits for this rank's copies,
    then meets the other ranks at a process-group barrier; on the root it
    returns the gathered batch of the last push, valid until the next
    ``collect()``.  Every rank takes the same steps in the same order."""

    def __init__(self, tail_shape, batch_sizes: list[int], group=None, root: int = 0,
                 slots: int = 2, device: int | None = None):
        self.group = group
        self.root = int(root)
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if len(batch_sizes) != self.world:
            raise ValueError("MatrixMan: one batch size per rank is required")
        if slots < 1:
            raise ValueError("MatrixMan: at least one gather slot is required")
        self.tail = tuple(int(v) for v in tail_shape)
        self.sizes = [int(b) for b in batch_sizes]
        self.total = sum(self.sizes)
        self.offsets = [sum(self.sizes[:r]) for r in range(self.world)]
        row = 1
        for v in self.tail:
            row *= v
        self.row_bytes = row * 4
        self.device = runtime.current_device() if device is None else int(device)
        self.rt = runtime.get_runtime(self.device)
        lib = _lib.load()
        self.lib = lib
        nbytes = max(self.total * self.row_bytes, 1)
        self.blocks: list[_IpcBlock] = []
        handles = []
        if self.rank == self.root:
            for _ in range(slots):
                ptr = ctypes.c_void_p()
                h = ctypes.create_string_buffer(_lib.MM_IPC_HANDLE_BYTES)
                _lib.check(lib.mm_ipc_alloc(self.device, nbytes, ctypes.byref(ptr), h), "gather buffer")
                self.blocks.append(_IpcBlock(self.rt, ptr.value, nbytes, torch.float32,
                                             _lib.POOL_ACTIVATION))
                handles.append(h.raw)
        obj = [handles]
        dist.broadcast_object_list(obj, src=self.root, group=group)
        if self.rank == self.root:
            self.dst = [b.pointer for b in self.blocks]
        else:
            self.dst = []
            for raw in obj[0]:
                ptr = ctypes.c_void_p()
                _lib.check(lib.mm_ipc_open(self.device, ctypes.create_string_buffer(raw, len(raw)),
                                           ctypes.byref(ptr)), "open gather buffer")
                self.dst.append(ptr.value)
        s = ctypes.c_void_p()
        _lib.check(lib.mm_stream_create(self.device, ctypes.byref(s)), "copy stream")
        self.copy_stream = s.value
        self.ready = [_Event(self.device) for _ in range(slots)]
        self.done = [_Event(self.device) for _ in range(slots)]
        self.kept: list = [None] * slots
        self.slot = 0
        self.last = -1
        runtime.set_device(self.device)

    def push(self, local: MatrixManTensor) -> None:
        if not isinstance(local, MatrixManTensor):
            raise TypeError("MatrixMan: PeerGather pushes MatrixMan tensors")
        if tuple(int(v) for v in local.shape) != (self.sizes[self.rank],) + self.tail:
            raise ValueError("MatrixMan: local output does not match this rank's slice shape")
        lib = self.lib
        s = self.slot
        if self.kept[s] is not None:
            # The copy that last used this slot must be done before its source
            # block may return to the arena.
            _lib.check(lib.mm_event_sync(self.done[s].handle, runtime.config.waitTimeoutMs),
                       "gather copy wait")
            self.kept[s] = None
        local = _dense(local)
        _lib.check(lib.mm_event_record(self.ready[s].handle, local.runtime.stream), "event record")
        _lib.check(lib.mm_stream_wait_event(self.copy_stream, self.ready[s].handle), "stream wait")
        nbytes = self.sizes[self.rank] * self.row_bytes
        if nbytes:
            dst = self.dst[s] + self.offsets[self.rank] * self.row_bytes
            _lib.check(lib.mm_memcpy_d2d(ctypes.c_void_p(dst), ctypes.c_void_p(local.element_ptr),
                                         nbytes, self.copy_stream), "gather copy")
        _lib.check(lib.mm_event_record(self.done[s].handle, self.copy_stream), "event record")
        self.kept[s] = local
        self.last = s
        self.slot = (s + 1) % len(self.dst)

    def join(self, stream) -> None:
        """Make `stream` wait for this rank's last copy (device-side)."""
        if self.last >= 0:
            _lib.check(self.lib.mm_stream_wait_event(stream, self.done[self.last].handle), "stream wait")

    def collect(self):
        """Wait for this rank's copies, meet the other ranks; the root gets the
        gathered batch of the last push (None elsewhere)."""
        _lib.check(self.lib.mm_stream_sync(self.copy_stream, runtime.config.waitTimeoutMs),
                   "gather copies")
        for i in range(len(self.kept)):
            self.kept[i] = None
        _barrier(self.group, self.device)
        if self.rank != self.root or self.last < 0:
            return None
        block = self.blocks[self.last]
        shape = (self.total,) + self.tail
        return MatrixManTensor(block, shape, 0, contiguous_strides(shape))

    def close(self) -> None:
        """Unmap (other ranks) after a final collect; the root frees its
        buffers when they are garbage-collected."""
        if self.rank != self.root:
            for p in self.dst:
                self.lib.mm_ipc_close(self.device, ctypes.c_void_p(p))
            self.dst = []
        if self.copy_stream:
            self.lib.mm_stream_destroy(ctypes.c_void_p(self.copy_stream))
            self.copy_stream = None


def _barrier(group, device: int) -> None:
    """Process-group barrier; with NCCL an all-reduce of a CUDA tensor on the
    rank's own device (dist.barrier would place its tensor on the default
    accelerator, which is the matrixman device once the backend is up)."""
    try:
        nccl = dist.get_backend(group) == "nccl"
    except Exception:
        nccl = False
    if nccl:
        t = torch.zeros(1, device=torch.device("cuda", device))
        dist.all_reduce(t, group=group)
        torch.cuda.synchronize(device)
    else:
        dist.barrier(group=group)
