"""StageBoundaries host logic with fake control pages and slots (no GPU), in
the style of the reference's tests/test_vpp_resources.py: objects built with
object.__new__ and SimpleNamespace collaborators."""

from types import SimpleNamespace

import pytest

from qwen_infra_b200.vpp import native as NV
from qwen_infra_b200.vpp import stages as ST
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
    t.dst_leases = ST._SharedSlots(3, t.in_edges)
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


def test_edge_layout_grants_up_to_the_ring_on_each_edge():
    """Edge-owned slots (the reference's comparison layout): each incoming
    edge owns 7 physical slots, physical slot = edge base + ring slot, so
    grants run ahead up to 7 per edge independently of the other edge."""
    t = _bare()
    t.in_edges = {1: None, 4: None}
    t.dst_leases = ST._EdgeSlots(3, t.in_edges)
    assert t.dst_leases.count == 14
    t.layout = NV.BoundaryLayout(64, 7, 3, 256)
    t.epoch, t.capacity = 1, 64
    t.dst_rings = {1: NV.SlotRing(NV.DESTINATION, t.layout, 1, 0), 4: NV.SlotRing(NV.DESTINATION, t.layout, 1, 3)}
    t.grant_seq = {1: 0, 4: 0}
    t.grants, t.dst_busy = {}, [None] * 14
    granted = []
    t.ctrl_in = {s: SimpleNamespace(grant=lambda seq, p, s=s: granted.append((s, seq, p))) for s in (1, 4)}
    t._reap = lambda: None
    t.set_order([(b, 1) for b in range(9)] + [(b, 4) for b in range(2)])
    assert granted == [(1, q, q) for q in range(7)]  # edge 1 stops at its 7 ring slots
    # retire sequence 0 of edge 1: its slot (physical 0) comes back, the next grant proceeds
    p, ticket = t.grants.pop((1, 0))
    t.dst_rings[1].transition(ticket, NV.OP_TRANSFER_RECORDED)
    t.dst_rings[1].transition(ticket, NV.OP_CONSUMER_RECORDED)
    t.dst_rings[1].transition(ticket, NV.OP_CONSUMER_COMPLETE)
    t.dst_leases.give_back(p, ticket)
    t.progress()
    assert granted[7] == (1, 7, 0)
    assert t.dst_leases.peak == 7


def test_resource_layout_rules():
    with pytest.raises(ValueError):
        StageBoundaries(0, 2, "cpu", 64, 256, backend="nccl", resource_layout="rank")
    with pytest.raises(ValueError):
        StageBoundaries(0, 2, "cpu", 64, 256, resource_layout="ring")


def test_edge_layout_sender_waits_for_its_ring_slot():
    """A sender 7 messages ahead on edge-owned slots must wait for slot
    seq % 7 to come back (it is the ring slot itself), not fail."""
    t = _bare(timeout=0.2)
    t.out_edges = {0: None}
    t.src_leases = ST._EdgeSlots(2, t.out_edges)
    t.layout = NV.BoundaryLayout(64, 7, 2, 256)
    t.epoch, t.capacity = 1, 64
    t.src_rings = {0: NV.SlotRing(NV.SOURCE, t.layout, 1, 0)}
    t.out_seq = {0: 0}
    t.src_busy = [None] * 7
    t.src_current = {}
    t.stats = dict(slot_waits=0)
    t.src_arena = __import__("torch").zeros((7, 2, 64, 256))
    reaped = []
    t._reap = lambda: reaped.append(1)
    t.closed = t.failed = False
    for seq in range(7):
        t.prepare_send(seq, 0, 8)
        t.out_seq[0] += 1
    with pytest.raises(NV.TransportTimeout):  # slot 0 still held: a bounded wait, then the deadline
        t.prepare_send(7, 0, 8)
    assert reaped and t.stats["slot_waits"] == 1
