"""Host side of the stage-boundary transport (no GPU): the C++ wire codec
against headers recorded from the reference codec, the slot-generation state
machine (the reference's known-answer lifecycle, tests/slot_pool.cpp:15-71),
and the shared-memory credit / publication protocol across two processes."""

import json
import multiprocessing as mp
import re
import subprocess
import uuid
from pathlib import Path

import sys

import pytest

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))
import __graft_entry__  # noqa: E402  (spawned test processes register the package too)

__graft_entry__.load_package()
from qwen_infra_b200.vpp import native as NV  # noqa: E402
GOLDEN = json.loads((REPO / "tests/golden/wire_headers.json").read_text())


def test_codec_reproduces_reference_headers():
    for case in GOLDEN["encoded"]:
        lay = NV.BoundaryLayout(case["cap"], case["slots"], 4, 5120)
        d = lay.make(case["epoch"], case["batch"], case["seq"], case["src"], case["rows"])
        wire = lay.encode(d)
        assert wire.hex() == case["wire"]
        back = lay.decode(wire)
        assert (back.batch_id, back.edge_sequence, back.valid_tokens) == (case["batch"], case["seq"], case["rows"])


def test_codec_rejects_what_the_reference_rejects():
    args = dict(fold_edge=(2048, 7, 1, 3, 1), last_stage=(2048, 7, 1, 7, 1), zero_epoch=(2048, 7, 0, 0, 1),
                over_capacity=(2048, 7, 1, 0, 2049), zero_capacity=(0, 7, 1, 0, 0), eight_slots=(2048, 8, 1, 0, 1))
    for name, rejected in GOLDEN["rejected"].items():
        cap, slots, epoch, src, rows = args[name]
        if rejected:
            with pytest.raises(NV.BoundaryError):
                NV.BoundaryLayout(cap, slots, 4).make(epoch, 0, 0, src, rows)
    assert NV.BoundaryLayout(2048, 7).budget() == GOLDEN["budget_2048_7"]


def test_match_rejects_other_batch_epoch_sequence_or_edge():
    lay = NV.BoundaryLayout(2048, 2)
    for stage in (0, 1, 2, 4, 5, 6):
        wire = lay.encode(lay.make(1, 12, 0, stage, 513))
        assert lay.match(wire, 1, 12, 0, stage).valid_tokens == 513
        for bad in ((1, 13, 0, stage), (2, 12, 0, stage), (1, 12, 1, stage)):
            with pytest.raises(NV.BoundaryError):
                lay.match(wire, *bad)
    corrupt = bytearray(lay.encode(lay.make(1, 12, 0, 0, 513)))
    corrupt[0] ^= 1
    with pytest.raises(NV.BoundaryError):
        lay.decode(bytes(corrupt))


@pytest.mark.parametrize("ranks", [2, 3, 8])
def test_generalised_edges(ranks):
    edges = [s for s in range(2 * ranks - 1) if s != ranks - 1]
    assert [NV.edge_index(ranks, s, s + 1) for s in edges] == list(range(2 * ranks - 2))
    with pytest.raises(NV.BoundaryError):
        NV.edge_index(ranks, ranks - 1, ranks)  # the local fold is not a wire edge
    lay = NV.BoundaryLayout(64, 7, ranks, 256)
    assert sum(lay.budget()) == 2 * (2 * ranks - 2) * 7 * lay.capacity * 256 * 2 * 2


def test_slot_lifecycle_known_answers():
    lay = NV.BoundaryLayout(2048, 2)
    src = NV.SlotRing(NV.SOURCE, lay, 1, 0)
    first = src.try_acquire(lay.make(1, 0, 0, 0, 1024))
    assert first is not None
    with pytest.raises(NV.BoundaryError):
        src.transition(first, NV.OP_SOURCE_READ_COMPLETE)
    for op in (NV.OP_PRODUCER_RECORDED, NV.OP_TRANSFER_RECORDED, NV.OP_SOURCE_READ_COMPLETE):
        src.transition(first, op)
    assert src.live == 0
    with pytest.raises(NV.BoundaryError):
        src.descriptor(first)
    second = src.try_acquire(lay.make(1, 1, 1, 0, 1024))
    for op in (NV.OP_PRODUCER_RECORDED, NV.OP_TRANSFER_RECORDED, NV.OP_SOURCE_READ_COMPLETE):
        src.transition(second, op)
    reused = src.try_acquire(lay.make(1, 2, 2, 0, 1024))
    assert reused is not None and reused.generation != first.generation
    with pytest.raises(NV.BoundaryError):
        src.transition(first, NV.OP_PRODUCER_RECORDED)
    with pytest.raises(NV.BoundaryError):
        src.try_acquire(lay.make(1, 9, 9, 0, 1))  # out of order
    src.stop()
    src.transition(reused, NV.OP_RELEASE_UNSUBMITTED)
    assert src.live == 0
    with pytest.raises(NV.BoundaryError):
        src.try_acquire(lay.make(1, 3, 3, 0, 1))  # stopped rings never resume


def test_two_rings_share_physical_leases_without_generation_mixups():
    lay7 = NV.BoundaryLayout(2048, 7)
    leases = NV.PhysicalLeases(2)
    fwd = NV.SlotRing(NV.SOURCE, lay7, 1, 1)
    ret = NV.SlotRing(NV.SOURCE, lay7, 1, 5)
    for seq in range(24):
        f = fwd.try_acquire(lay7.make(1, seq, seq, 1, 513))
        r = ret.try_acquire(lay7.make(1, seq, seq, 5, 17))
        fp, rp = leases.acquire(f), leases.acquire(r)
        assert fp != rp and f.slot_id == r.slot_id and leases.live == 2 and not leases.available
        with pytest.raises(NV.BoundaryError):
            leases.release(fp, r)
        stale = NV.QvTicket(f.ring_id, f.sequence, f.generation + 1, f.slot_id)
        with pytest.raises(NV.BoundaryError):
            leases.release(fp, stale)
        for ring, t in ((fwd, f), (ret, r)):
            for op in (NV.OP_PRODUCER_RECORDED, NV.OP_TRANSFER_RECORDED, NV.OP_SOURCE_READ_COMPLETE):
                ring.transition(t, op)
        leases.release(fp, f)
        leases.release(rp, r)
        assert leases.live == 0
        with pytest.raises(NV.BoundaryError):
            leases.release(fp, f)
    assert leases.peak_live == 2


def test_destination_lifecycle_and_discard():
    lay = NV.BoundaryLayout(512, 3, 2, 256)
    dst = NV.SlotRing(NV.DESTINATION, lay, 4, 0)
    t = dst.try_acquire(lay.make(4, 0, 0, 0, 100))
    with pytest.raises(NV.BoundaryError):
        dst.transition(t, NV.OP_PRODUCER_RECORDED)  # source-only transition
    dst.transition(t, NV.OP_TRANSFER_RECORDED)
    assert dst.state(t) == "transferring"
    dst.transition(t, NV.OP_CONSUMER_RECORDED)
    dst.transition(t, NV.OP_CONSUMER_COMPLETE)
    t2 = dst.try_acquire(lay.make(4, 1, 1, 0, 100))
    dst.transition(t2, NV.OP_TRANSFER_RECORDED)
    dst.transition(t2, NV.OP_DISCARD_RECEIVED)
    assert dst.live == 0 and dst.peak_live == 1 and dst.next_sequence == 2


# Every (side, event, state) combination against the slot protocol: the
# legal moves of a message's slot on each side of an edge
# (src/qwen_infra/vpp/native/slot_pool.h:9-75); everything else is refused
# and leaves the slot where it was.
_LEGAL = {
    ("source", NV.OP_PRODUCER_RECORDED, "reserved"): "produced",
    ("source", NV.OP_TRANSFER_RECORDED, "produced"): "transferring",
    ("source", NV.OP_SOURCE_READ_COMPLETE, "transferring"): "free",
    ("destination", NV.OP_TRANSFER_RECORDED, "reserved"): "transferring",
    ("destination", NV.OP_CONSUMER_RECORDED, "transferring"): "consuming",
    ("destination", NV.OP_CONSUMER_COMPLETE, "consuming"): "free",
    ("destination", NV.OP_DISCARD_RECEIVED, "transferring"): "free",
}
_PATH = {"source": [NV.OP_PRODUCER_RECORDED, NV.OP_TRANSFER_RECORDED],
         "destination": [NV.OP_TRANSFER_RECORDED, NV.OP_CONSUMER_RECORDED]}


@pytest.mark.parametrize("side", ["source", "destination"])
def test_every_slot_event_in_every_state(side):
    lay = NV.BoundaryLayout(256, 3, 2, 256)
    role = NV.SOURCE if side == "source" else NV.DESTINATION
    for depth in range(3):  # reserved, then one and two steps along the side's path
        for op in range(7):
            ring = NV.SlotRing(role, lay, 2, 0)
            t = ring.try_acquire(lay.make(2, 0, 0, 0, 8))
            for step in _PATH[side][:depth]:
                ring.transition(t, step)
            before = ring.state(t)
            want = _LEGAL.get((side, op, before))
            if want is None:
                with pytest.raises(NV.BoundaryError):
                    ring.transition(t, op)
                assert ring.state(t) == before and ring.live == 1
            else:
                ring.transition(t, op)
                if want == "free":
                    assert ring.live == 0
                    with pytest.raises(NV.BoundaryError):
                        ring.state(t)
                else:
                    assert ring.state(t) == want
    # abandoning a reserved message is legal on both sides, after stop() only
    ring = NV.SlotRing(role, lay, 2, 0)
    t = ring.try_acquire(lay.make(2, 0, 0, 0, 8))
    with pytest.raises(NV.BoundaryError):
        ring.transition(t, NV.OP_RELEASE_UNSUBMITTED)
    ring.stop()
    ring.transition(t, NV.OP_RELEASE_UNSUBMITTED)
    assert ring.live == 0


def test_lease_arena_capacity_and_lowest_free_slot():
    for bad in (0, 8):
        with pytest.raises(NV.BoundaryError):
            NV.PhysicalLeases(bad)
    lay = NV.BoundaryLayout(256, 7, 2, 256)
    leases = NV.PhysicalLeases(3)
    ring = NV.SlotRing(NV.SOURCE, lay, 2, 0)
    ts = [ring.try_acquire(lay.make(2, s, s, 0, 8)) for s in range(3)]
    got = [leases.acquire(t) for t in ts]
    assert got == [0, 1, 2] and not leases.available
    leases.release(1, ts[1])
    t3 = NV.QvTicket(ts[1].ring_id, 99, 99, 5)
    assert leases.acquire(t3) == 1  # the lowest free physical slot is reused
    with pytest.raises(NV.BoundaryError):
        leases.acquire(ts[0])  # arena full
    leases.release(0, ts[0])
    with pytest.raises(NV.BoundaryError):
        leases.acquire(ts[2])  # logical slot 2 already holds physical slot 2
    assert leases.peak_live == 3


def test_reference_known_answer_binary_when_built():
    exe = REPO / "oracle/_ref/slot_pool_test"
    if not exe.exists():
        pytest.skip("reference checker not built (oracle/build_ref.py)")
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60, check=True)
    assert "passed" in out.stdout


def _receiver(name, n, q):
    page = NV.ControlPage(name, create=True)
    try:
        lay = NV.BoundaryLayout(64, 7, 2, 256)
        got = []
        for seq in range(n):
            page.grant(seq, seq % 3)
            wire = page.wait_published(seq, 20.0)
            got.append(lay.match(wire, 1, 100 + seq, seq, 0).valid_tokens)
        q.put(("ok", got))
        # the sender flags failure; our next wait must end with PeerFailed
        try:
            page.wait_published(n, 20.0)
            q.put(("no-failure", None))
        except NV.PeerFailed:
            q.put(("failed-seen", None))
    finally:
        page.close()


def _sender(name, n, q):
    page = NV.ControlPage(name, create=False, timeout=20.0)
    lay = NV.BoundaryLayout(64, 7, 2, 256)
    slots = []
    for seq in range(n):
        slots.append(page.wait_grant(seq, 20.0))
        page.publish(seq, lay.encode(lay.make(1, 100 + seq, seq, 0, 1 + seq)))
    q.put(("sent", slots))
    page.fail()
    page.close()


def test_control_page_credit_and_publication_across_processes():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    name = f"/qvpp-test-{uuid.uuid4().hex[:10]}"
    n = 20
    rx = ctx.Process(target=_receiver, args=(name, n, q))
    rx.start()
    tx = ctx.Process(target=_sender, args=(name, n, q))
    tx.start()
    tx.join(60)
    rx.join(60)
    msgs = {}
    while not q.empty():
        k, v = q.get()
        msgs[k] = v
    assert tx.exitcode == 0 and rx.exitcode == 0
    assert msgs["sent"] == [s % 3 for s in range(n)]
    assert msgs["ok"] == [1 + s for s in range(n)]
    assert "failed-seen" in msgs


def test_wait_deadline_without_peer():
    page = NV.ControlPage(f"/qvpp-test-{uuid.uuid4().hex[:10]}", create=True)
    try:
        with pytest.raises(NV.TransportTimeout):
            page.wait_published(0, 0.2)
        with pytest.raises(NV.TransportTimeout):
            page.wait_grant(0, 0.2)
        with pytest.raises(NV.BoundaryError):
            page.publish(3, bytes(96))  # publication is strictly in sequence order
    finally:
        page.close()


def _declared(header):
    text = (REPO / "include" / header).read_text()
    return set(re.findall(r"^\s*(?:const\s+)?[\w\*]+\s*\*?\s*(q[iv]_\w+|nvfp4_\w+)\(", text, re.M))


@pytest.mark.parametrize("lib_name,header", [("libqwen_infra_b200.so", "qwen_infra_b200.h"),
                                             ("libqwen_vpp_native.so", "qwen_vpp_native.h")])
def test_libraries_load_and_export_every_declared_symbol(lib_name, header):
    import ctypes

    path = REPO / "qwen3.8-sm120-vpp-bucket-attention_b200" / lib_name
    assert path.exists(), f"{lib_name} not built"
    handle = ctypes.CDLL(str(path))
    declared = _declared(header)
    assert len(declared) > 10
    for name in declared:
        assert hasattr(handle, name), name


def test_kernel_abi_struct_sizes_match_ctypes():
    from qwen_infra_b200 import _native

    _native.lib()  # raises on any size mismatch
