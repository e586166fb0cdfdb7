"""CPU-materialisation audit (reference drivers/matrixman/audit.py:21-141).

When ``config.audit_cpu_leaks`` is set, every explicit readback is counted
with the tensor's shape so that unexpected device-to-host traffic inside a
model loop shows up in ``audit.report()``.
"""

from __future__ import annotations

from collections import Counter

from .config import config

events: Counter = Counter()
bytes_read: Counter = Counter()


def record(kind: str, tensor=None) -> None:
    if not config._values["auditCpuLeaks"]:
        return
    events[kind] += 1
    if tensor is not None:
        bytes_read[kind] += int(tensor.numel()) * int(tensor.element_size())


def reset() -> None:
    events.clear()
    bytes_read.clear()


def report() -> dict:
    return {"events": dict(events), "bytes": dict(bytes_read)}
