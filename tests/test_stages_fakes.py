"""StageBoundaries host logic with fake control pages and slots (no GPU), in
the style of the reference's tests/test_vpp_resources.py: objects built with
object.__new__ and SimpleNamespace collaborators."""

from types import SimpleNamespace

import pytest

from qwen_infra_b200.vpp import native as NV
from qwen_infra_b200.vpp.stages import StageBoundaries


def _bare(timeout=5.0):
    t = object.__new__(StageBoundaries)
    t.timeout = timeout
    t.failed = t.closed = False
    t.backend = "p2p"
    t.ctrl_in, t.ctrl_out = {}, {}
    return t


def test_waiting_for_a_credit_keeps_granting_to_peers():
    """A rank blocked on its own credit must keep serving grants, or two ranks
    waiting for each other's credits deadlock."""
    t = _bare()
    calls = []
    t.progress = lambda: calls.append("progress")
    attempts = iter([NV.TransportTimeout("slice"), NV.TransportTimeout("slice"), 2])

    def attempt(_slice):
        v = next(attempts)
        if isinstance(v, Exception):
            raise v
        return v

    assert t._wait_progressing("credit", attempt) == 2
    assert calls == ["progress", "progress"]


def test_wait_deadline_flags_failure_on_every_edge():
    t = _bare(timeout=0.05)
    flagged = []
    t.ctrl_in = {1: SimpleNamespace(fail=lambda: flagged.append("in"))}
    t.ctrl_out = {0: SimpleNamespace(fail=lambda: flagged.append("out"))}
    t.progress = lambda: None

    def never(_slice):
        raise NV.TransportTimeout("slice")

    with pytest.raises(NV.TransportTimeout):
        t._wait_progressing("publication", never)
    assert t.failed and sorted(flagged) == ["in", "out"]


def test_peer_failure_propagates_immediately():
    t = _bare()
    t.progress = lambda: None

    def peer_gone(_slice):
        raise NV.PeerFailed("peer")

    with pytest.raises(NV.PeerFailed):
        t._wait_progressing("credit", peer_gone)
    assert t.failed


def test_grants_follow_consumption_order_and_slot_budget():
    """Destination slots are granted strictly in the rank's receive order and
    never beyond the three physical slots."""
    t = _bare()
    # rank 1 of 3 receives stage 1 (edge 0 -> 1) and stage 4 (edge 3 -> 4)
    t.in_edges = {1: None, 4: None}
    t.dst_leases = NV.PhysicalLeases(3)
    t.layout = NV.BoundaryLayout(64, 7, 3, 256)
    t.epoch, t.capacity = 1, 64
    t.dst_rings = {1: NV.SlotRing(NV.DESTINATION, t.layout, 1, 0), 4: NV.SlotRing(NV.DESTINATION, t.layout, 1, 3)}
    t.grant_seq = {1: 0, 4: 0}
    t.grants, t.dst_busy = {}, [None] * 3
    granted = []
    t.ctrl_in = {s: SimpleNamespace(grant=lambda seq, p, s=s: granted.append((s, seq, p))) for s in (1, 4)}
    t._reap = lambda: None
    t.set_order([(0, 1), (1, 1), (0, 4), (2, 1), (1, 4), (3, 1)])
    assert granted == [(1, 0, 0), (1, 1, 1), (4, 0, 2)]
    assert t.schedule[t.sched_pos] == (2, 1)  # the next grant waits for a slot
