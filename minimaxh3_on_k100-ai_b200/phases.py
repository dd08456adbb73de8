"""Device-time breakdown of a step by phase (profiling aid for bench.py).

The block code calls ``mark(name)`` at the start of each phase (norm, projection
+ send, exchange wait, attention, ...).  Outside ``record`` that is a no-op; under
``record`` each mark records a CUDA event on the current stream, and the time
from one mark to the next is charged to the earlier mark's phase.  Recording is
for eager steps only (never inside CUDA-graph capture).
"""
from __future__ import annotations

from typing import Callable

import torch

_MARKS: list | None = None


def mark(name: str) -> None:
    if _MARKS is not None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        _MARKS.append((name, ev))


def record(fn: Callable[[], object]) -> dict[str, float]:
    """Run ``fn`` with marks on; return {phase: total ms} (device time between
    consecutive marks, summed over every occurrence of the phase)."""
    global _MARKS
    _MARKS = []
    try:
        fn()
        mark("end")
        torch.cuda.synchronize()
        marks = _MARKS
    finally:
        _MARKS = None
    totals: dict[str, float] = {}
    for (name, ev), (_, nxt) in zip(marks, marks[1:]):
        totals[name] = totals.get(name, 0.0) + ev.elapsed_time(nxt)
    return totals
