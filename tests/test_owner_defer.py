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


def test_pipeline_issue_order_uses_per_batch_signals():
    """One barrier per step; batch j's owner work waits only for batch j's
    arrivals, and its apply only for batch j's completion."""
    log = []

    class WS:
        SIGNAL_SLOTS = 256

        def buffer(self, n):
            return "buf", "peers"

        def barrier(self):
            log.append("barrier")

        def next_signal_epoch(self):
            return 7

        def signal(self, slot, epoch):
            log.append(f"signal{slot}@{epoch}")

        def wait(self, slot, epoch):
            log.append(f"wait{slot}@{epoch}")

    class Spec:
        def __init__(self, n):
            self.n, self.nbytes = n, 10

        def place(self, b):
            pass

        def pack(self, peers):
            log.append(f"pack{self.n}")

        def compute(self, buf):
            log.append(f"compute{self.n}")

        def apply(self, peers):
            log.append(f"apply{self.n}")

    oc._run_phases(WS(), [Spec(0), Spec(1)])
    assert log == ["barrier", "pack0", "signal0@7", "pack1", "signal2@7",
                   "wait0@7", "compute0", "signal1@7", "wait2@7", "compute1", "signal3@7",
                   "wait1@7", "apply0", "wait3@7", "apply1"]
