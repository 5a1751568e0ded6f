"""Scheduling of deferred owner-compute batches (host logic only; the kernels
are covered by the GPU tests in test_dist_gpu.py)."""

import pytest

from dtensor_muon_b200.parallel import owner_compute as oc


class _Spec:
    def __init__(self, name, nbytes=1):
        self.name, self.nbytes = name, nbytes


@pytest.fixture
def calls(monkeypatch):
    out = []
    monkeypatch.setattr(oc, "_run_phases", lambda ws, specs: out.append((ws, [s.name for s in specs])))
    return out


def test_immediate_outside_deferred(calls):
    ws = object()
    oc._enqueue(ws, [_Spec("a"), _Spec("b")])
    assert calls == [(ws, ["a"]), (ws, ["b"])]


def test_deferred_runs_all_batches_together_at_exit(calls):
    ws1, ws2 = object(), object()
    with oc.deferred():
        oc._enqueue(ws1, [_Spec("a")])
        oc._enqueue(ws2, [_Spec("x")])
        oc._enqueue(ws1, [_Spec("b"), _Spec("c")])
        assert calls == []
    assert calls == [(ws1, ["a", "b", "c"]), (ws2, ["x"])]
    assert "pending" not in oc._DEFER and not oc._DEFER.get("on")


def test_nested_deferred_flushes_only_at_outermost_exit(calls):
    ws = object()
    with oc.deferred():
        with oc.deferred():
            oc._enqueue(ws, [_Spec("a")])
        assert calls == []
        oc._enqueue(ws, [_Spec("b")])
    assert calls == [(ws, ["a", "b"])]


def test_queue_flushes_when_over_the_byte_cap(calls, monkeypatch):
    monkeypatch.setattr(oc, "MAX_DEFERRED_BYTES", 10)
    ws = object()
    with oc.deferred():
        oc._enqueue(ws, [_Spec("a", 6)])
        assert calls == []
        oc._enqueue(ws, [_Spec("b", 6)])
        assert calls == [(ws, ["a", "b"])]
        oc._enqueue(ws, [_Spec("c", 1)])
    assert calls == [(ws, ["a", "b"]), (ws, ["c"])]


def test_exception_drops_the_queue(calls):
    ws = object()
    with pytest.raises(RuntimeError):
        with oc.deferred():
            oc._enqueue(ws, [_Spec("a")])
            raise RuntimeError("step failed")
    assert calls == []
    assert "pending" not in oc._DEFER and not oc._DEFER.get("on")
