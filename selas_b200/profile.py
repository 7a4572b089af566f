"""Per-kernel timing with CUDA events, for the roofline numbers bench.py reports.

When enabled, every launch made through ``selas_b200.ops`` is bracketed by a pair of CUDA events on
the launching stream and tagged with its kernel family and its algorithmic work (FLOPs for the
GEMM and attention, minimum bytes moved for the memory-bound kernels). ``collect()`` synchronises
and sums, per family, the event-measured time, the launches and the work.
"""

from __future__ import annotations

import contextlib

import torch

_enabled = False
_records: list = []


def enable() -> None:
    global _enabled, _records
    _enabled = True
    _records = []


def disable() -> None:
    global _enabled
    _enabled = False


def enabled() -> bool:
    return _enabled


@contextlib.contextmanager
def region(kind: str, flops: float = 0.0, nbytes: float = 0.0):
    if not _enabled:
        yield
        return
    s = torch.cuda.current_stream()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s)
    try:
        yield
    finally:
        e1.record(s)
        _records.append((kind, flops, nbytes, e0, e1))


def collect() -> dict[str, dict]:
    torch.cuda.synchronize()
    out: dict[str, dict] = {}
    for kind, flops, nbytes, e0, e1 in _records:
        d = out.setdefault(kind, {"ms": 0.0, "launches": 0, "flops": 0.0, "bytes": 0.0})
        d["ms"] += e0.elapsed_time(e1)
        d["launches"] += 1
        d["flops"] += flops
        d["bytes"] += nbytes
    return out
