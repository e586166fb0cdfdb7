"""Pool state machine of the caching arena, exercised on the host-backed
instance (same policy code as the device arena, simulated events)."""

import ctypes

import pytest

from matrixman_b200 import _lib


class HostArena:
    def __init__(self, capacity=0, deferred=False):
        self.lib = _lib.load()
        self.h = ctypes.c_void_p()
        _lib.check(self.lib.mm_host_arena_create(capacity, int(deferred), ctypes.byref(self.h)))

    def alloc(self, n, kind=_lib.POOL_ACTIVATION):
        p = ctypes.c_void_p()
        _lib.check(self.lib.mm_host_arena_alloc(self.h, n, kind, ctypes.byref(p)), "alloc")
        return p.value

    def free(self, p):
        _lib.check(self.lib.mm_host_arena_free(self.h, ctypes.c_void_p(p)), "free")

    def complete(self):
        g = ctypes.c_int64()
        self.lib.mm_host_arena_generation(self.h, ctypes.byref(g))
        self.lib.mm_host_arena_complete(self.h, g.value)

    def stats(self):
        s = _lib.MMPoolStats()
        self.lib.mm_host_arena_stats(self.h, ctypes.byref(s))
        return s.as_dict()

    def fail_after(self, n):
        self.lib.mm_host_arena_fail_after(self.h, n)

    def close(self):
        self.lib.mm_host_arena_destroy(self.h)


def test_safe_pool_reuses_same_size_class():
    a = HostArena()
    p = a.alloc(1000)
    a.free(p)
    q = a.alloc(900)  # same 512-byte class (1024)
    assert q == p
    st = a.stats()
    assert st["pool_hits"]["activation"] == 1
    assert st["device_mallocs"] == 1
    a.close()


def test_pools_are_separate():
    a = HostArena()
    p = a.alloc(4096, _lib.POOL_ACTIVATION)
    a.free(p)
    q = a.alloc(4096, _lib.POOL_SCRATCH)
    assert q != p
    a.close()


def test_deferred_pool_waits_for_completion():
    a = HostArena(deferred=True)
    p = a.alloc(2048)
    a.free(p)
    assert a.stats()["pending_bytes"]["activation"] == 2048
    q = a.alloc(2048)  # release not complete yet -> fresh block
    assert q != p
    a.complete()
    r = a.alloc(2048)
    assert r == p
    assert a.stats()["pending_bytes"]["activation"] == 0
    a.close()


def test_parameters_are_never_pooled():
    a = HostArena()
    p = a.alloc(4096, _lib.POOL_PARAMETER)
    a.free(p)
    st = a.stats()
    assert st["cached_bytes"]["parameter"] == 0
    assert st["device_frees"] == 1
    a.close()


def test_oom_recovery_drains_then_raises():
    a = HostArena(capacity=8192)
    p1 = a.alloc(4096)
    a.free(p1)  # 4096 cached
    # 8192 does not fit next to the cached block: the arena drains the cache,
    # retries and succeeds.
    p2 = a.alloc(8192)
    st = a.stats()
    assert st["oom_recoveries"] == 1 and st["cached_bytes"]["activation"] == 0
    with pytest.raises(MemoryError, match="out of device memory"):
        a.alloc(4096)
    a.free(p2)
    a.close()


def test_fault_injection_after_n_allocations():
    a = HostArena()
    a.fail_after(2)
    a.alloc(100)
    a.alloc(200000)
    with pytest.raises(MemoryError):
        a.alloc(300000)
    a.close()


def test_double_free_is_an_error():
    a = HostArena()
    p = a.alloc(100)
    a.free(p)
    with pytest.raises(ValueError, match="double free"):
        a.free(p)
    a.close()


def test_size_classes_bound_waste():
    a = HostArena()
    sizes = [1, 511, 512, 513, 4095, 1 << 20, (1 << 20) + 1, 3_000_000, 123_456_789]
    for s in sizes:
        p = a.alloc(s)
        a.free(p)
    st = a.stats()
    assert st["cached_bytes"]["activation"] <= sum(max(512, int(s * 1.125) + 512) for s in sizes)
    a.close()
