"""Tensor plumbing on the device: upload/readback layouts, views, cat/split/
stack, factories, explicit failure, runtime waits and the device arena."""

import ctypes

import pytest
import torch

import matrixman_b200
from oracle.tolerance import bit_exact

pytestmark = pytest.mark.gpu


def gen(seed):
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def test_roundtrip_and_device(mm):
    x = torch.randn(3, 4, 5, generator=gen(1))
    d = mm.to_device(x)
    assert d.device.type == "matrixman" and mm.is_matrixman_tensor(d)
    assert bit_exact(d.cpu(), x)
    assert bit_exact(d.to("cpu"), x)
    with pytest.raises(NotImplementedError):
        d.to(torch.float64)
    with pytest.raises(NotImplementedError):
        torch.ops.aten._to_copy.default(d, device="cpu", pin_memory=True)


def test_views_readback(mm):
    x = torch.randn(4, 6, 8, generator=gen(2))
    d = mm.to_device(x)
    cases = [
        (d.transpose(0, 2), x.transpose(0, 2)),
        (d[:, 2:5, ::2], x[:, 2:5, ::2]),
        (d.permute(2, 0, 1), x.permute(2, 0, 1)),
        (d.unsqueeze(1).expand(4, 3, 6, 8), x.unsqueeze(1).expand(4, 3, 6, 8)),
        (d.view(24, 8), x.view(24, 8)),
        (d.reshape(-1), x.reshape(-1)),
        (d[1], x[1]),
        (d.select(2, 3), x.select(2, 3)),
    ]
    for got, ref in cases:
        assert tuple(got.shape) == tuple(ref.shape)
        assert bit_exact(got.cpu(), ref.contiguous())
    with pytest.raises(RuntimeError, match="view size is not compatible"):
        d.transpose(0, 1).view(-1)


def test_cat_split_stack_bit_exact(mm):
    g = gen(3)
    a, b, c = (torch.randn(2, k, 5, 6, generator=g) for k in (3, 4, 5))
    y = torch.cat([mm.to_device(a), mm.to_device(b), mm.to_device(c)], 1).cpu()
    assert bit_exact(y, torch.cat([a, b, c], 1))
    y = torch.cat([mm.to_device(a), mm.to_device(a)], 0).cpu()
    assert bit_exact(y, torch.cat([a, a], 0))
    parts = mm.to_device(torch.cat([a, b, c], 1)).chunk(3, 1)
    ref = torch.cat([a, b, c], 1).chunk(3, 1)
    for p, r in zip(parts, ref):
        assert bit_exact(p.cpu(), r.contiguous())
    s = torch.stack([mm.to_device(a), mm.to_device(a * 2)], 2).cpu()
    assert bit_exact(s, torch.stack([a, a * 2], 2))


def test_nhwc_cat_channel_slices(mm):
    g = gen(4)
    a, b = torch.randn(2, 8, 5, 6, generator=g), torch.randn(2, 4, 5, 6, generator=g)
    an = mm.to_device(a.permute(0, 2, 3, 1).contiguous()).permute(0, 3, 1, 2)
    bn = mm.to_device(b.permute(0, 2, 3, 1).contiguous()).permute(0, 3, 1, 2)
    y = torch.cat([an, bn], 1)
    assert y.is_contiguous(memory_format=torch.channels_last)
    assert bit_exact(y.cpu(), torch.cat([a, b], 1))


def test_factories(mm):
    z = torch.zeros(3, 4, device="matrixman")
    assert bit_exact(z.cpu(), torch.zeros(3, 4))
    e = torch.empty(2, 2, device="matrixman")
    assert e.device.type == "matrixman"
    r = torch.arange(10, dtype=torch.float32, device="matrixman")
    assert bit_exact(r.cpu(), torch.arange(10, dtype=torch.float32))
    r = torch.arange(2, 11, 3, device="matrixman")
    assert torch.equal(r.cpu(), torch.arange(2, 11, 3))
    d = mm.to_device(torch.ones(2, 3))
    f = d.new_full((4,), 2.5)
    assert bit_exact(f.cpu(), torch.full((4,), 2.5))
    d.fill_(7.0)
    assert bit_exact(d.cpu(), torch.full((2, 3), 7.0))
    assert bit_exact(torch.zeros_like(d).cpu(), torch.zeros(2, 3))


def test_unsupported_op_raises_with_name(mm):
    d = mm.to_device(torch.randn(4, 4))
    with pytest.raises(NotImplementedError, match="MatrixMan/CUDA: .*not implemented"):
        torch.linalg.inv(d)
    with pytest.raises(NotImplementedError):
        torch.cumsum(d, 0)


def test_bounded_wait_and_stream_query(mm):
    from matrixman_b200 import _lib, runtime
    rt = runtime.get_runtime(0)
    lib = _lib.load()
    done = ctypes.c_int(0)
    rt.synchronize()
    _lib.check(lib.mm_stream_query(rt.stream, ctypes.byref(done)))
    assert done.value == 1
    # Queue a large copy and ask for a 0 ms wait: either it is already done or
    # the wait reports a timeout without blocking; the context stays usable.
    big = mm.to_device(torch.zeros(64 << 20))
    from matrixman_b200 import ops
    ops.clone(big)
    status = lib.mm_stream_sync(rt.stream, 0)
    assert status in (_lib.MM_OK, _lib.MM_ERR_TIMEOUT)
    rt.synchronize()


def test_device_arena_reuse_and_oom_injection(mm):
    from matrixman_b200 import _lib, runtime
    rt = runtime.get_runtime(0)
    rt.synchronize()
    before = rt.pool_stats()
    a = mm.to_device(torch.zeros(1000))
    ptr = a._owner.pointer
    del a
    b = mm.to_device(torch.zeros(1000))
    assert b._owner.pointer == ptr  # same size class reused
    after = rt.pool_stats()
    assert after["pool_hits"]["activation"] > before["pool_hits"]["activation"]
    lib = _lib.load()
    _lib.check(lib.mm_debug_fail_alloc_after(0, 0))
    try:
        with pytest.raises(MemoryError):
            mm.to_device(torch.zeros(123_457_000))
    finally:
        _lib.check(lib.mm_debug_fail_alloc_after(0, -1))
    assert bit_exact(mm.to_device(torch.ones(5)).cpu(), torch.ones(5))


def test_graph_capture_pool_and_replay(mm):
    from matrixman_b200 import ops, runtime
    rt = runtime.get_runtime(0)
    x = torch.randn(16, 32, generator=gen(5))
    d = mm.to_device(x)
    rt.synchronize()
    rt.capture_begin()
    y = (d * 2.0 + 1.0)
    z = torch.relu(y)
    graph = rt.capture_end()
    static_in, static_out = d, z
    for k in range(3):
        xk = torch.randn(16, 32, generator=gen(10 + k))
        ops.copy_into(mm.to_device(xk), static_in)
        graph.replay()
        assert bit_exact(static_out.cpu(), torch.relu(xk * 2.0 + 1.0))
    graph.destroy()


def test_native_hooks_register(mm):
    from matrixman_b200.privateuse import register_native_hooks
    assert register_native_hooks()
    assert torch.matrixman.device_count() >= 1
    d = mm.to_device(torch.ones(2))
    d.requires_grad_(True)
    assert d.requires_grad
