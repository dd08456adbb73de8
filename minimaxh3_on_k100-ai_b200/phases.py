"""Device-time breakdown of a step by phase (profiling aid for bench.py).

The block code calls ``mark(name)`` at the start of each phase (norm, projection
+ send, exchange wait, attention, ...).  Outside ``record`` / ``capturing`` that
is a no-op.  Under ``record`` (an eager step) each mark records a CUDA event on
the current stream, and the time from one mark to the next is charged to the
earlier mark's phase.  Under ``capturing`` (inside CUDA-graph capture) only the
named phases are marked, each by an event record node at its start and at the
next mark: after a replay of the graph the events hold that replay's times, so
``totals`` gives the phases' device time inside the replayed step itself.
"""
from __future__ import annotations

import contextlib
from typing import Callable, Iterable

import torch

_MARKS: list | None = None
_ONLY: frozenset | None = None     # under capturing(): the phases to time
_EXTERNAL = False                  # event record nodes in a captured graph


def mark(name: str) -> None:
    if _MARKS is None:
        return
    if _ONLY is not None:
        closes_open_phase = bool(_MARKS) and _MARKS[-1][0] in _ONLY
        if name not in _ONLY and not closes_open_phase:
            return
    ev = torch.cuda.Event(enable_timing=True, external=_EXTERNAL)
    ev.record()
    _MARKS.append((name, ev))


def totals(marks: list, only: Iterable[str] | None = None) -> dict[str, float]:
    """{phase: total ms} from recorded marks (device time from each mark to the
    next, summed over every occurrence of the phase; with ``only``, just those)."""
    keep = None if only is None else set(only)
    out: dict[str, float] = {}
    for (name, ev), (_, nxt) in zip(marks, marks[1:]):
        if keep is None or name in keep:
            out[name] = out.get(name, 0.0) + ev.elapsed_time(nxt)
    return out


def record(fn: Callable[[], object]) -> dict[str, float]:
    """Run ``fn`` eagerly with marks on; return {phase: total ms}."""
    global _MARKS
    _MARKS = []
    try:
        fn()
        mark("end")
        torch.cuda.synchronize()
        marks = _MARKS
    finally:
        _MARKS = None
    return totals(marks)


@contextlib.contextmanager
def capturing(only: Iterable[str] | None = None):
    """Inside CUDA-graph capture: time the phases named in ``only`` (None: every
    phase).  Yields the list that collects the marks (pass it to ``totals`` after
    a replay)."""
    global _MARKS, _ONLY, _EXTERNAL
    marks: list = []
    _MARKS, _ONLY, _EXTERNAL = marks, (None if only is None else frozenset(only)), True
    try:
        yield marks
        mark("end")
    finally:
        _MARKS, _ONLY, _EXTERNAL = None, None, False
