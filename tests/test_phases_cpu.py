"""Host logic of the step's phase marks (phases.py) on CPU, with a stand-in for
CUDA events: which marks are recorded under ``capturing`` (only the named phases
and the mark that closes each), and how ``totals`` charges the time between marks."""
import pytest
import torch

import h3b200  # noqa: F401  (puts the package on the path)
from h3b200 import phases


class _FakeEvent:
    clock = 0.0

    def __init__(self, enable_timing=False, external=False):
        self.external = external
        self.t = None

    def record(self, stream=None):
        _FakeEvent.clock += 1.0
        self.t = _FakeEvent.clock

    def elapsed_time(self, other):
        return other.t - self.t


@pytest.fixture
def fake_events(monkeypatch):
    _FakeEvent.clock = 0.0
    monkeypatch.setattr(torch.cuda, "Event", _FakeEvent)


def test_capturing_marks_only_named_phases_and_their_ends(fake_events):
    with phases.capturing(("attention",)) as marks:
        for name in ("norm1", "qkv", "attention", "out_proj", "gate_up", "attention", "down"):
            phases.mark(name)
    names = [n for n, _ in marks]
    assert names == ["attention", "out_proj", "attention", "down"]
    assert all(ev.external for _, ev in marks)            # event record nodes in a graph
    assert phases.totals(marks, ("attention",)) == {"attention": 2.0}
    phases.mark("after")                                   # outside: a no-op
    assert len(marks) == 4


def test_capturing_closes_a_phase_left_open(fake_events):
    with phases.capturing(("attention",)) as marks:
        phases.mark("qkv")
        phases.mark("attention")
    assert [n for n, _ in marks] == ["attention", "end"]
    assert phases.totals(marks, ("attention",)) == {"attention": 1.0}


def test_record_charges_every_phase(fake_events, monkeypatch):
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)

    def step():
        for name in ("a", "b", "a"):
            phases.mark(name)
    assert phases.record(step) == {"a": 2.0, "b": 1.0}


def test_capturing_every_phase(fake_events):
    with phases.capturing() as marks:
        for name in ("norm1", "attention", "norm1", "down"):
            phases.mark(name)
    assert [n for n, _ in marks] == ["norm1", "attention", "norm1", "down", "end"]
    assert phases.totals(marks) == {"norm1": 2.0, "attention": 1.0, "down": 1.0}
