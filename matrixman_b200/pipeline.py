"""Batch inference with uploads, compute and readbacks overlapped.

The reference's flow is strictly serial: upload (``to_device``), forward,
explicit ``.cpu()`` readback (``backends/cuda/backend.py:146-157``,
``tensor.py:76-158``).  ``infer`` keeps that contract -- CPU batch in, CPU
result out, values identical to ``model(to_device(x)).cpu()`` -- but splits the
batch into chunks that travel on three streams of the device: host-to-device
copies on an upload stream, the prepared forward on the runtime stream, and
device-to-host copies on a readback stream, ordered by events.  While chunk k
computes, chunk k+1 uploads and chunk k-1 reads back (the two copy directions
use separate copy engines).  From page-locked host memory
(``matrixman.pinned_empty``) every copy is asynchronous.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib, runtime
from .tensor import MatrixManTensor, contiguous_strides

_aux_streams: dict[int, tuple[int, int]] = {}


def _streams(rt) -> tuple[int, int]:
    s = _aux_streams.get(rt.index)
    if s is None:
        lib = _lib.load()
        up, down = ctypes.c_void_p(), ctypes.c_void_p()
        runtime.set_device(rt.index)
        _lib.check(lib.mm_stream_create(rt.index, ctypes.byref(up)), "stream create")
        _lib.check(lib.mm_stream_create(rt.index, ctypes.byref(down)), "stream create")
        s = (up.value, down.value)
        _aux_streams[rt.index] = s
    return s


class _Events:
    def __init__(self, n: int):
        lib = _lib.load()
        self.handles = []
        for _ in range(n):
            h = ctypes.c_void_p()
            _lib.check(lib.mm_event_create(ctypes.byref(h), 0), "event create")
            self.handles.append(h)

    def __getitem__(self, i):
        return self.handles[i]

    def close(self):
        lib = _lib.load()
        for h in self.handles:
            lib.mm_event_destroy(h)
        self.handles = []


def ramp_slices(batch: int, chunks: int) -> list[tuple[int, int]]:
    """[start, end) slices of ``batch`` for ``infer``: sizes in proportion
    1, 2, ..., n-1, then a shorter last slice (ceil(2(n-1)/3)); 64 images in 4
    chunks -> 8, 16, 24, 16.  A forward costs a fixed overhead plus a per-image
    term, and every forward but the first waits only for its own upload: a
    small first slice starts the first forward early, growing slices keep each
    upload ahead of the forward before it, and a shorter last slice shortens the
    final readback.  Measured on YOLOv8n bs64: 10.5 ms against 11.3 ms for four
    equal slices."""
    if batch <= 0:
        return []
    n = max(1, min(int(chunks), int(batch)))
    if n == 1:
        return [(0, int(batch))]
    w = list(range(1, n)) + [max(1, -(-2 * (n - 1) // 3))]
    total = sum(w)
    sizes = [max(1, (int(batch) * wi) // total) for wi in w]
    # distribute the remainder (or excess) over the largest slices
    diff = int(batch) - sum(sizes)
    order = sorted(range(n), key=lambda i: -w[i])
    i = 0
    while diff != 0:
        j = order[i % n]
        if diff > 0:
            sizes[j] += 1
            diff -= 1
        elif sizes[j] > 1:
            sizes[j] -= 1
            diff += 1
        i += 1
    out, start = [], 0
    for v in sizes:
        out.append((start, start + v))
        start += v
    return out


def infer(model, x: torch.Tensor, chunks: int = 4, device=None, sizes=None) -> torch.Tensor:
    """``model(to_device(x)).cpu()`` for a CPU batch ``x``, with the batch split
    into ``chunks`` slices (``ramp_slices``) whose uploads, forwards and
    readbacks overlap.

    ``sizes`` (optional) gives the slice sizes explicitly: positive integers
    summing to the batch; it overrides ``chunks``.  ``model`` should be a
    prepared module (``matrixman.prepare``); its output must be one tensor with
    the batch as its first dimension.  The result is a CPU tensor (in pooled
    page-locked memory when available)."""
    from .api import _device_index, get_backend

    get_backend()
    if not isinstance(x, torch.Tensor) or x.device.type != "cpu":
        raise TypeError("MatrixMan: infer expects a CPU batch tensor")
    if x.dtype != torch.float32:
        raise TypeError("MatrixMan: infer supports float32 input only")
    if x.dim() < 1 or x.shape[0] == 0:
        raise ValueError("MatrixMan: infer needs a non-empty batch")
    x = x.contiguous()
    rt = runtime.get_runtime(_device_index(device))
    runtime.set_device(rt.index)
    lib = _lib.load()
    up, down = _streams(rt)
    if sizes is not None:
        sizes = [int(v) for v in sizes]
        if not sizes or any(v <= 0 for v in sizes) or sum(sizes) != int(x.shape[0]):
            raise ValueError("MatrixMan: infer sizes must be positive and sum to the batch")
        slices, start = [], 0
        for v in sizes:
            slices.append((start, start + v))
            start += v
    else:
        slices = ramp_slices(int(x.shape[0]), int(chunks))
    ev = _Events(3 * len(slices))
    row = x[0].numel()
    keep = []
    out = None
    try:
        with torch.no_grad():
            # All input blocks first: they are ordered on the runtime stream, so
            # one event after the allocations lets the upload stream write
            # them without waiting for any forward enqueued later.
            inputs = []
            for s, e in slices:
                shape = (e - s,) + tuple(int(v) for v in x.shape[1:])
                inputs.append((shape, rt.new_storage((e - s) * row, torch.float32)))
            _lib.check(lib.mm_event_record(ev[0], rt.stream), "event record")
            _lib.check(lib.mm_stream_wait_event(up, ev[0]), "stream wait")
            for k, ((s, e), (shape, storage)) in enumerate(zip(slices, inputs)):
                src = x.data_ptr() + s * row * 4
                _lib.check(lib.mm_memcpy_h2d(ctypes.c_void_p(storage.pointer), ctypes.c_void_p(src),
                                             (e - s) * row * 4, up, 0), "host-to-device copy")
                _lib.check(lib.mm_event_record(ev[3 * k + 1], up), "event record")
            for k, ((s, e), (shape, storage)) in enumerate(zip(slices, inputs)):
                _lib.check(lib.mm_stream_wait_event(rt.stream, ev[3 * k + 1]), "stream wait")
                xd = MatrixManTensor._from_owner(storage, shape, 0, contiguous_strides(shape))
                y = model(xd)
                if not isinstance(y, MatrixManTensor):
                    raise NotImplementedError("MatrixMan: infer needs a model with one tensor output")
                if tuple(y._logical_strides) != contiguous_strides(tuple(int(v) for v in y.shape)):
                    from . import ops
                    y = ops.materialize(y)
                if out is None:
                    out = runtime.host_empty((int(x.shape[0]),) + tuple(int(v) for v in y.shape[1:]),
                                             torch.float32)
                yrow = 1
                for v in y.shape[1:]:
                    yrow *= int(v)
                _lib.check(lib.mm_event_record(ev[3 * k + 2], rt.stream), "event record")
                _lib.check(lib.mm_stream_wait_event(down, ev[3 * k + 2]), "stream wait")
                _lib.check(lib.mm_memcpy_d2h(ctypes.c_void_p(out.data_ptr() + s * yrow * 4),
                                             ctypes.c_void_p(y.element_ptr), (e - s) * yrow * 4,
                                             down, 0), "device-to-host copy")
                # Device blocks are released only after the readback stream is
                # done with them (below).
                keep.append((xd, y))
        _lib.check(lib.mm_stream_sync(ctypes.c_void_p(down), runtime.config.waitTimeoutMs), "synchronize")
    finally:
        try:
            lib.mm_stream_sync(ctypes.c_void_p(down), runtime.config.waitTimeoutMs)
            lib.mm_stream_sync(ctypes.c_void_p(up), runtime.config.waitTimeoutMs)
        finally:
            ev.close()
    del keep
    return out


def infer_stream(model, batches, device=None, depth: int = 2):
    """Pipelined inference over a sequence of CPU batches: yields
    ``model(to_device(x)).cpu()`` for each batch ``x`` of ``batches``, in
    order.

    Whole batches travel on three streams: batch k+1 uploads (upload stream)
    while batch k computes (runtime stream) and batch k-1 reads back
    (readback stream), so a stream of batches pays one upload and one readback
    of latency in all, not per batch, and each forward runs at the full batch
    size.  Up to ``depth`` batches beyond the one being returned stay in
    flight, so the upload of a batch is enqueued well before the forward of the
    batch ahead of it ends (with depth 1 it would wait for the previous
    readback).  Batches should be in page-locked memory (``matrixman.pinned_empty``)
    for the copies to be asynchronous.  ``model`` is a prepared module with one
    batch-major tensor output.  Each yielded result is a CPU tensor (pooled
    page-locked memory when available) that stays valid after the next batch
    is submitted."""
    from .api import _device_index, get_backend

    if int(depth) < 1:
        raise ValueError("MatrixMan: infer_stream depth must be at least 1")
    get_backend()
    rt = runtime.get_runtime(_device_index(device))
    runtime.set_device(rt.index)
    lib = _lib.load()
    up, down = _streams(rt)
    safe_reuse = runtime.config.resolved_sync_policy == "safe"
    pending = []  # (event after readback, host output, device blocks kept alive)
    events = []
    # Input blocks: a ring of depth + 1 per input size, each reused only after
    # the forward that read it (its `consumed` event).  A block freed to the
    # arena would carry a release event at the tail of the runtime stream --
    # after the forward just submitted -- and the next upload into it could not
    # overlap that forward.
    rings: dict[int, list] = {}
    uses: dict[int, int] = {}

    def _event(track=True):
        h = ctypes.c_void_p()
        _lib.check(lib.mm_event_create(ctypes.byref(h), 0), "event create")
        if track:
            events.append(h)
        return h

    def _finish(item):
        done, out, _keep, evs = item
        _lib.check(lib.mm_event_sync(done, runtime.config.waitTimeoutMs), "readback wait")
        for h in evs:  # this batch's events are no longer waited on
            lib.mm_event_destroy(h)
        return out

    try:
        with torch.no_grad():
            for x in batches:
                if not isinstance(x, torch.Tensor) or x.device.type != "cpu" or x.dtype != torch.float32:
                    raise TypeError("MatrixMan: infer_stream expects float32 CPU batches")
                if x.dim() < 1 or x.shape[0] == 0:
                    raise ValueError("MatrixMan: infer_stream needs non-empty batches")
                x = x.contiguous()
                n = int(x.shape[0])
                row = x[0].numel()
                shape = (n,) + tuple(int(v) for v in x.shape[1:])
                uploaded, computed, done = _event(False), _event(False), _event(False)
                ring = rings.setdefault(n * row, [])
                use = uses.get(n * row, 0)
                uses[n * row] = use + 1
                if len(ring) <= int(depth):
                    if safe_reuse:
                        # Ordered on the upload stream: a block reused from the
                        # arena makes it wait for that block's release only.
                        storage = rt.new_storage(n * row, torch.float32, stream=up)
                    else:
                        # Stream-ordered reuse only: the upload waits for the
                        # point of the runtime stream where it was allocated.
                        storage = rt.new_storage(n * row, torch.float32)
                        allocated = _event()
                        _lib.check(lib.mm_event_record(allocated, rt.stream), "event record")
                        _lib.check(lib.mm_stream_wait_event(up, allocated), "stream wait")
                    ring.append((storage, _event()))
                storage, consumed = ring[use % len(ring)]
                if use >= len(ring):
                    _lib.check(lib.mm_stream_wait_event(up, consumed), "stream wait")
                _lib.check(lib.mm_memcpy_h2d(ctypes.c_void_p(storage.pointer), ctypes.c_void_p(x.data_ptr()),
                                             n * row * 4, up, 0), "host-to-device copy")
                _lib.check(lib.mm_event_record(uploaded, up), "event record")
                _lib.check(lib.mm_stream_wait_event(rt.stream, uploaded), "stream wait")
                xd = MatrixManTensor._from_owner(storage, shape, 0, contiguous_strides(shape))
                y = model(xd)
                if not isinstance(y, MatrixManTensor):
                    raise NotImplementedError("MatrixMan: infer_stream needs a model with one tensor output")
                if tuple(y._logical_strides) != contiguous_strides(tuple(int(v) for v in y.shape)):
                    from . import ops
                    y = ops.materialize(y)
                out = runtime.host_empty((n,) + tuple(int(v) for v in y.shape[1:]), torch.float32)
                _lib.check(lib.mm_event_record(consumed, rt.stream), "event record")
                _lib.check(lib.mm_event_record(computed, rt.stream), "event record")
                _lib.check(lib.mm_stream_wait_event(down, computed), "stream wait")
                _lib.check(lib.mm_memcpy_d2h(ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(y.element_ptr),
                                             out.numel() * 4, down, 0), "device-to-host copy")
                _lib.check(lib.mm_event_record(done, down), "event record")
                # The input and output blocks go back to the arena only after
                # their readback (the host waits for `done` first).
                pending.append((done, out, (xd, y), (uploaded, computed, done)))
                if len(pending) > int(depth):
                    yield _finish(pending.pop(0))
            while pending:
                yield _finish(pending.pop(0))
    finally:
        try:
            lib.mm_stream_sync(ctypes.c_void_p(down), runtime.config.waitTimeoutMs)
            lib.mm_stream_sync(ctypes.c_void_p(up), runtime.config.waitTimeoutMs)
        finally:
            for item in pending:
                for h in item[3]:
                    lib.mm_event_destroy(h)
            pending.clear()
            rt.synchronize()  # the ring's blocks may return to the arena now
            rings.clear()
            for h in events:
                lib.mm_event_destroy(h)
