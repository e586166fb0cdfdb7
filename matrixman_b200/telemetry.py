"""Profiling counters and reports (``matrixman.profile_report`` / ``profile_reset``).

Covers what the reference's CUDA profiler (backends/cuda/profiling.py:17-80,
489-665) and frontend profiler (frontend_profiling.py:84-227) report:
kernel launches per entry point, pool statistics, host time per ATen op, and
-- when ``gpu_timing`` is on -- device time per op measured with CUDA events.
"""

from __future__ import annotations

import time
from collections import Counter, defaultdict
from contextlib import contextmanager

from .config import config

launches: Counter = Counter()
dispatch_seconds: defaultdict = defaultdict(float)
dispatch_calls: Counter = Counter()


def enabled() -> bool:
    return bool(config._values["profile"] or config._values["cudaProfile"])


def dispatch_enabled() -> bool:
    return bool(config._values["profile"] or config._values["profileDispatch"])


def count_launch(name: str) -> None:
    launches[name] += 1


def total_launches() -> int:
    return int(sum(launches.values()))


@contextmanager
def dispatch_scope(op: str):
    t0 = time.perf_counter()
    try:
        yield
    finally:
        dispatch_seconds[op] += time.perf_counter() - t0
        dispatch_calls[op] += 1


class LaunchTimes:
    """CUDA-event bracket around every native launch on its own stream
    (enabled by ``config.gpu_timing``; eager execution only -- a captured
    graph has no host-side launches to bracket)."""

    def __init__(self):
        self.records: list[tuple[str, object, object, object]] = []

    def begin(self, name: str, stream) -> object:
        import ctypes
        from . import _lib
        lib = _lib.load()
        e0, e1 = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(lib.mm_event_create(ctypes.byref(e0), 1), "event create")
        _lib.check(lib.mm_event_create(ctypes.byref(e1), 1), "event create")
        _lib.check(lib.mm_event_record(e0, stream), "event record")
        return (name, e0, e1, stream)

    def end(self, token) -> None:
        from . import _lib
        lib = _lib.load()
        _lib.check(lib.mm_event_record(token[2], token[3]), "event record")
        self.records.append(token)

    def summary(self) -> dict:
        """{entry point: {"launches": n, "ms": total}} (synchronises)."""
        import ctypes
        from . import _lib
        lib = _lib.load()
        out: dict = {}
        for name, e0, e1, _s in self.records:
            _lib.check(lib.mm_event_sync(e1, config.waitTimeoutMs), "event sync")
            ms = ctypes.c_float()
            _lib.check(lib.mm_event_elapsed_ms(e0, e1, ctypes.byref(ms)), "event elapsed")
            rec = out.setdefault(name, {"launches": 0, "ms": 0.0, "each_ms": []})
            rec["launches"] += 1
            rec["ms"] += float(ms.value)
            rec["each_ms"].append(float(ms.value))
            lib.mm_event_destroy(e0)
            lib.mm_event_destroy(e1)
        self.records.clear()
        return out


launch_times = LaunchTimes()


def gpu_timing_enabled() -> bool:
    return bool(config._values["gpuTiming"])


def reset() -> None:
    launches.clear()
    dispatch_seconds.clear()
    dispatch_calls.clear()
    launch_times.records.clear()


def report(frame_count: int | None = None) -> str:
    from . import runtime
    lines = ["MatrixMan/B200 profile", "======================"]
    lines.append(f"kernel launches: {total_launches()}")
    for name, n in launches.most_common():
        lines.append(f"  {name:<28} {n}")
    if dispatch_calls:
        lines.append("ATen dispatch (host time):")
        for op, secs in sorted(dispatch_seconds.items(), key=lambda kv: -kv[1]):
            per = secs / max(dispatch_calls[op], 1) * 1e6
            lines.append(f"  {op:<48} calls={dispatch_calls[op]:<6} total={secs*1e3:9.3f} ms "
                         f"avg={per:8.1f} us")
    for rt in runtime.initialized_runtimes():
        st = rt.pool_stats()
        lines.append(f"device {rt.index} pool: live={st['live_bytes']} cached={st['cached_bytes']} "
                     f"pending={st['pending_bytes']} peak={st['peak_live_bytes']} "
                     f"mallocs={st['device_mallocs']} hits={st['pool_hits']}")
    if frame_count:
        lines.append(f"frames: {frame_count}, launches/frame: {total_launches() / frame_count:.1f}")
    text = "\n".join(lines)
    print(text)
    return text
