"""Stage-boundary transport of one rank (the reference's ``StageBoundaries``,
``src/qwen_infra/vpp/native/stages.py:70-451``, rebuilt for NVLink).

A slot holds one message = 2 bf16 planes [capacity, H] (hidden at offset 0,
residual at ``plane_bytes``).  Every directed wire edge has a logical ring of
7 slots with generation tickets (``native.SlotRing``) that validates the
message lifecycle.  Physical slots follow the resource layout
(``vpp/native/stages.py:71-102``, ``docs/vpp-resources.md:70-93``):

* ``"rank"`` (default for p2p): rank-shared arenas of 2 source and 3
  destination slots that every edge of the rank leases one at a time;
* ``"edge"`` (default, and the only layout, for nccl): every edge endpoint
  owns its 7 slots, physical slot = ring slot (the reference's comparison
  layout; 28 slots on a middle rank instead of 5).

``backend="p2p"`` (default): the destination arena is exported with CUDA IPC;
the sender's copy stream copies both planes device-to-device straight into the
granted destination slot (copy engines over NVLink), records an interprocess
event and publishes the wire header on the edge's control page.  The receiver
grants destination slots strictly in the order it will consume its inputs (so
the input it needs next always holds a slot) and makes its compute stream wait
on the sender's event.

``backend="nccl"``: the comparison transport (the reference's ``NcclEdge``,
``vpp/native/nccl_edge.cpp:30-107``): one 2-rank NCCL communicator per wire
edge, both planes of a message as one grouped send / receive
(``batch_isend_irecv``), edge-owned slots.  Each edge is used by one stage on
each side, so a rank's two stages may run on two CUDA streams with either
transport.

Every host wait has a deadline (``timeout``, default 60 s); a failure flags the
edge's control page so the peer's waits end too.
"""

import os
import time
import uuid
from datetime import timedelta

import torch
import torch.distributed as dist

from . import layout as L
from . import native as NV

RING_SLOTS = 7
SOURCE_SLOTS = 2
DEST_SLOTS = 3


class _SharedSlots:
    """Rank layout: ``count`` physical slots leased by every edge in turn."""

    def __init__(self, count, stages):
        self.count = count
        self.leases = NV.PhysicalLeases(count)

    def can_take(self, stage, seq):
        return self.leases.available

    def take(self, stage, ticket):
        return self.leases.acquire(ticket)

    def give_back(self, p, ticket):
        self.leases.release(p, ticket)

    def note_stall(self):
        self.leases.note_stall()

    @property
    def peak(self):
        return self.leases.peak_live

    @property
    def stalls(self):
        return self.leases.stalls

    def close(self):
        self.leases.close()


class _EdgeSlots:
    """Edge layout: each edge endpoint owns RING_SLOTS physical slots; the
    physical slot of a message is its ring slot."""

    def __init__(self, count, stages):
        self.base = {s: i * RING_SLOTS for i, s in enumerate(sorted(stages))}
        self.count = RING_SLOTS * len(self.base)
        self.owner = [None] * self.count
        self.live = self.peak = self.stalls = 0

    def can_take(self, stage, seq):
        return self.owner[self.base[stage] + seq % RING_SLOTS] is None

    def take(self, stage, ticket):
        p = self.base[stage] + ticket.slot_id
        if self.owner[p] is not None:
            raise NV.BoundaryError("edge-owned slot still leased")
        self.owner[p] = (ticket.ring_id, ticket.sequence, ticket.generation)
        self.live += 1
        self.peak = max(self.peak, self.live)
        return p

    def give_back(self, p, ticket):
        if self.owner[p] != (ticket.ring_id, ticket.sequence, ticket.generation):
            raise NV.BoundaryError("slot returned by a ticket that does not hold it")
        self.owner[p] = None
        self.live -= 1

    def note_stall(self):
        self.stalls += 1

    def close(self):
        pass


class _Edge:
    def __init__(self, src_stage, ranks):
        self.src_stage = src_stage
        self.dst_stage = src_stage + 1
        self.src_rank = L.stage_rank(src_stage, ranks)
        self.dst_rank = L.stage_rank(src_stage + 1, ranks)
        self.index = NV.edge_index(ranks, src_stage, src_stage + 1)
        self.forward = src_stage < ranks - 1


def boundary_edges(rank, ranks, profile="vpp"):
    """({stage: edge out of it}, {stage: edge into it}) for this rank's stages.
    Folded: stages rank and 2G-1-rank, every boundary but the fold is a wire
    edge.  Conventional: stage rank only, edges s -> s+1 for s < G-1 (the
    forward edges of the folded layout, same indices and rings)."""
    if profile == "vpp":
        stages, n_stages = (rank, 2 * ranks - 1 - rank), 2 * ranks
    elif profile == "cpp":
        stages, n_stages = (rank,), ranks
    else:
        raise ValueError("profile is vpp or cpp")
    out_edges = {s: _Edge(s, ranks) for s in stages if s + 1 < n_stages and L.stage_rank(s + 1, ranks) != rank}
    in_edges = {s: _Edge(s - 1, ranks) for s in stages if s > 0 and L.stage_rank(s - 1, ranks) != rank}
    return out_edges, in_edges


class StageBoundaries:
    def __init__(self, rank, ranks, device, capacity, hidden, *, backend="p2p", epoch=1, timeout=60.0,
                 segment_bytes=0, control_group=None, session=None, profile="vpp", resource_layout=None):
        if ranks < 2:
            raise ValueError("a boundary transport needs at least two ranks")
        if backend not in ("p2p", "nccl"):
            raise ValueError("backend is p2p or nccl")
        resource_layout = resource_layout or ("rank" if backend == "p2p" else "edge")
        if resource_layout not in ("rank", "edge"):
            raise ValueError("resource layout is rank or edge")
        if resource_layout == "rank" and backend != "p2p":
            raise ValueError("rank-shared slots need the peer-to-peer transport")
        self.resource_layout = resource_layout
        if profile not in L.PROFILES:
            raise ValueError("profile is vpp or cpp")
        self.rank, self.ranks, self.backend = rank, ranks, backend
        self.device = torch.device(device)
        self.dev_index = self.device.index
        self.capacity, self.hidden = capacity, hidden
        self.epoch, self.timeout, self.segment = epoch, timeout, segment_bytes
        self.layout = NV.BoundaryLayout(capacity, RING_SLOTS, ranks, hidden)
        self.plane_elems = capacity * hidden
        self.plane_bytes = self.plane_elems * 2
        self.slot_bytes = 2 * self.plane_bytes
        self.closed = self.failed = False
        self.group = control_group or dist.new_group(backend="gloo")
        self.out_edges, self.in_edges = boundary_edges(rank, ranks, profile)
        # logical rings per edge (source side for outgoing, destination side for incoming)
        self.src_rings = {s: NV.SlotRing(NV.SOURCE, self.layout, epoch, e.src_stage) for s, e in self.out_edges.items()}
        self.dst_rings = {s: NV.SlotRing(NV.DESTINATION, self.layout, epoch, e.src_stage)
                          for s, e in self.in_edges.items()}
        slots = _SharedSlots if resource_layout == "rank" else _EdgeSlots
        self.src_leases = slots(SOURCE_SLOTS, self.out_edges)
        self.dst_leases = slots(DEST_SLOTS, self.in_edges)
        n_src, n_dst = self.src_leases.count, max(1, self.dst_leases.count)
        self.out_seq = {s: 0 for s in self.out_edges}
        self.grant_seq = {s: 0 for s in self.in_edges}
        self.recv_seq = {s: 0 for s in self.in_edges}
        self.copy_stream = torch.cuda.Stream(device=self.device)
        # source slots: storage, ready events, copy-done events, owner
        self.n_src, self.n_dst = n_src, n_dst
        self.src_arena = torch.empty((n_src, 2, capacity, hidden), dtype=torch.bfloat16, device=self.device)
        self.src_ready = [[torch.cuda.Event() for _ in range(2)] for _ in range(n_src)]
        self.src_done = [torch.cuda.Event() for _ in range(n_src)]
        self.src_busy = [None] * n_src  # (ticket, stage) until the copy out completes
        self.res_marked = [False] * n_src
        self.src_current = {}  # (batch, stage) -> (physical, ticket)
        # destination slots
        self.dst_done = [torch.cuda.Event() for _ in range(n_dst)]
        self.dst_busy = [None] * n_dst  # ticket held until consumer done completes
        self.dst_pending_free = set()
        self.grants = {}  # (stage, seq) -> (physical, ticket)
        self.schedule = []  # [(batch, stage)] receives in consumption order
        self.sched_pos = 0
        self.received = {}  # (batch, stage) -> (physical, ticket, seq)
        self.stats = dict(credit_waits=0, credit_wait_s=0.0, slot_waits=0, messages_out=0, messages_in=0,
                          bytes_out=0)
        if backend == "p2p":
            self._setup_p2p(session)
        else:
            self._setup_nccl()

    # ------------------------------------------------------------------ setup
    def _setup_p2p(self, session):
        if session is None:
            token = [uuid.uuid4().hex[:12] if self.rank == 0 else None]
            dist.broadcast_object_list(token, src=0, group=self.group)
            session = token[0]
        self.session = session
        ptr, handle = NV.arena_alloc(self.dev_index, self.n_dst * self.slot_bytes)
        self.dst_ptr = ptr
        self.dst_arena = torch.as_tensor(NV.DeviceBuffer(ptr, self.n_dst * self.slot_bytes), device=self.device) \
            .view(torch.bfloat16).view(self.n_dst, 2, self.capacity, self.hidden)
        self.ctrl_in = {s: NV.ControlPage(self._ctrl_name(e), create=True) for s, e in self.in_edges.items()}
        self.ipc_out = {}
        out_handles = {}
        for s, e in self.out_edges.items():
            evs = [NV.ipc_event_create(self.dev_index) for _ in range(8)]
            self.ipc_out[s] = [ev for ev, _ in evs]
            out_handles[e.index] = [h for _, h in evs]
        blob = dict(rank=self.rank, arena=handle, events=out_handles)
        blobs = [None] * self.ranks
        dist.all_gather_object(blobs, blob, group=self.group)
        self.peer_arena = {}
        self.ctrl_out = {}
        for s, e in self.out_edges.items():
            if e.dst_rank not in self.peer_arena:
                self.peer_arena[e.dst_rank] = NV.arena_open(self.dev_index, blobs[e.dst_rank]["arena"])
            self.ctrl_out[s] = NV.ControlPage(self._ctrl_name(e), create=False, timeout=self.timeout)
        self.ipc_in = {}
        for s, e in self.in_edges.items():
            self.ipc_in[s] = [NV.ipc_event_open(self.dev_index, h) for h in blobs[e.src_rank]["events"][e.index]]
        dist.barrier(group=self.group)

    def _ctrl_name(self, e):
        return f"/qvpp-{self.session}-e{e.index}"

    def _setup_nccl(self):
        self.session = None
        # every rank creates every edge's group, in edge order (group creation
        # is collective); a rank uses the groups of its own edges only
        self.edge_groups = {}
        for src in range(2 * self.ranks - 1):
            if L.stage_rank(src, self.ranks) == L.stage_rank(src + 1, self.ranks):
                continue  # the local fold
            e = _Edge(src, self.ranks)
            self.edge_groups[src] = dist.new_group(ranks=sorted((e.src_rank, e.dst_rank)), backend="nccl",
                                                   timeout=timedelta(seconds=self.timeout))
        self.dst_arena = torch.empty((self.n_dst, 2, self.capacity, self.hidden), dtype=torch.bfloat16,
                                     device=self.device)
        self.nccl_sends = {}  # physical source slot -> works

    # --------------------------------------------------------------- schedule
    def set_order(self, order):
        """This rank's op list [(batch, stage)] for the coming bank; receives
        are granted destination slots in exactly this order."""
        self.schedule = [(b, s) for b, s in order if s in self.in_edges]
        self.sched_pos = 0
        self.progress()

    def admit(self, batch):
        self.progress()

    def progress(self):
        """Retire completed copies and consumers, then grant free destination
        slots to the next receives of the schedule (never out of order)."""
        self._reap()
        if self.backend != "p2p":
            return
        while self.sched_pos < len(self.schedule):
            batch, stage = self.schedule[self.sched_pos]
            if not self.dst_leases.can_take(stage, self.grant_seq[stage]):
                break
            self._grant(batch, stage)
            self.sched_pos += 1

    def _reap(self):
        for p in list(self.dst_pending_free):
            if self.dst_done[p].query():
                stage, ticket = self.dst_busy[p]
                self.dst_rings[stage].transition(ticket, NV.OP_CONSUMER_COMPLETE)
                self.dst_leases.give_back(p, ticket)
                self.dst_busy[p] = None
                self.dst_pending_free.discard(p)
        for p in range(self.n_src):
            busy = self.src_busy[p]
            if busy is not None and self._source_done(p):
                stage, ticket = busy
                self.src_rings[stage].transition(ticket, NV.OP_SOURCE_READ_COMPLETE)
                self.src_leases.give_back(p, ticket)
                self.src_busy[p] = None

    def _source_done(self, p):
        if self.backend == "nccl":
            works = self.nccl_sends.get(p, ())
            return all(w.is_completed() for w in works)
        return self.src_done[p].query()

    def _grant(self, batch, stage):
        seq = self.grant_seq[stage]
        d = self.layout.make(self.epoch, batch, seq, stage - 1, self.capacity)
        ticket = self.dst_rings[stage].try_acquire(d)
        if ticket is None:
            raise NV.BoundaryError("destination ring slot still busy")
        p = self.dst_leases.take(stage, ticket)
        self.dst_busy[p] = (stage, ticket)
        self.grants[(stage, seq)] = (p, ticket)
        self.ctrl_in[stage].grant(seq, p)
        self.grant_seq[stage] += 1

    def _wait_progressing(self, what, attempt, slice_s=2e-4):
        """Wait for ``attempt`` (a short bounded native wait that raises
        TransportTimeout when its slice runs out) while still granting credits
        and retiring slots: a rank blocked here must not stop serving its
        peers, or two ranks waiting on each other's credits would deadlock."""
        deadline = time.monotonic() + self.timeout
        while True:
            try:
                return attempt(slice_s)
            except NV.TransportTimeout:
                pass
            except NV.PeerFailed:
                self._fail()
                raise
            self.progress()
            if time.monotonic() > deadline:
                self._fail()
                raise NV.TransportTimeout(f"deadline passed waiting for {what}")

    def _deadline_loop(self, what, ready):
        deadline = time.monotonic() + self.timeout
        spins = 0
        while not ready():
            self._reap()
            if time.monotonic() > deadline:
                self._fail()
                raise NV.TransportTimeout(f"deadline passed waiting for {what}")
            spins += 1
            if spins > 100:
                time.sleep(0.0001)

    # ------------------------------------------------------------------- send
    def prepare_send(self, batch, stage, rows):
        """Reserve a source slot for the output of ``stage`` on ``batch``;
        returns its (hidden, residual) views [rows, H] for the producer."""
        if rows > self.capacity:
            raise ValueError("boundary exceeds capacity")
        self._check_open()
        seq = self.out_seq[stage]
        d = self.layout.make(self.epoch, batch, seq, stage, rows)
        ring = self.src_rings[stage]
        # Wait for the physical slot first: with edge-owned slots it is the
        # ring slot itself, which the message seq - 7 may still hold.
        if not self.src_leases.can_take(stage, seq):
            self.src_leases.note_stall()
            self.stats["slot_waits"] += 1
            self._deadline_loop("a free source slot", lambda: self.src_leases.can_take(stage, seq))
        ticket = ring.try_acquire(d)
        if ticket is None:
            raise NV.BoundaryError("source ring slot still busy")
        p = self.src_leases.take(stage, ticket)
        self.src_busy[p] = None
        self.src_current[(batch, stage)] = (p, ticket, d)
        return self.src_arena[p, 0, :rows], self.src_arena[p, 1, :rows]

    def mark_residual_ready(self, batch, stage):
        """Record that the residual plane is written (it is final before the
        last MLP), so its copy can overlap the rest of the stage."""
        p, _, _ = self.src_current[(batch, stage)]
        self.src_ready[p][1].record(torch.cuda.current_stream(self.device))
        self.res_marked[p] = True

    def send(self, batch, stage, rows):
        p, ticket, d = self.src_current.pop((batch, stage))
        ring = self.src_rings[stage]
        compute = torch.cuda.current_stream(self.device)
        self.src_ready[p][0].record(compute)
        ring.transition(ticket, NV.OP_PRODUCER_RECORDED)
        seq = self.out_seq[stage]
        e = self.out_edges[stage]
        if self.backend == "p2p":
            t0 = time.monotonic()
            ctrl = self.ctrl_out[stage]
            q = self._wait_progressing(f"credit for sequence {seq} on {ctrl.name}",
                                       lambda t: ctrl.wait_grant(seq, t))
            waited = time.monotonic() - t0
            if waited > 1e-4:
                self.stats["credit_waits"] += 1
                self.stats["credit_wait_s"] += waited
            base = self.peer_arena[e.dst_rank] + q * self.slot_bytes
            src_h = self.src_arena[p, 0].data_ptr()
            src_r = self.src_arena[p, 1].data_ptr()
            res_ready = self.src_ready[p][1] if self.res_marked[p] else self.src_ready[p][0]
            self.res_marked[p] = False
            NV.cuda_check(NV.lib().qv_copy_message(
                self.dev_index, self.copy_stream.cuda_stream, res_ready.cuda_event, self.src_ready[p][0].cuda_event,
                src_h, src_r, base, base + self.plane_bytes, rows * self.hidden * 2, self.segment,
                self.ipc_out[stage][seq % 8], self.src_done[p].cuda_event), "peer copy")
            self.ctrl_out[stage].publish(seq, self.layout.encode(d))
        else:
            grp = self.edge_groups[e.src_stage]
            self.nccl_sends[p] = dist.batch_isend_irecv(
                [dist.P2POp(dist.isend, self.src_arena[p, 0, :rows], e.dst_rank, group=grp),
                 dist.P2POp(dist.isend, self.src_arena[p, 1, :rows], e.dst_rank, group=grp)])
        self.res_marked[p] = False
        ring.transition(ticket, NV.OP_TRANSFER_RECORDED)
        self.src_busy[p] = (stage, ticket)
        self.out_seq[stage] += 1
        self.stats["messages_out"] += 1
        self.stats["bytes_out"] += 2 * rows * self.hidden * 2
        self.progress()

    # ---------------------------------------------------------------- receive
    def receive(self, batch, stage, rows):
        """Input planes of ``stage`` for ``batch``: the compute stream waits for
        their arrival on the GPU; returns (hidden, residual) views [rows, H]."""
        self._check_open()
        seq = self.recv_seq[stage]
        compute = torch.cuda.current_stream(self.device)
        if self.backend == "p2p":
            self.progress()
            key = (stage, seq)
            if key not in self.grants:
                self._deadline_loop(f"a destination slot for batch {batch}",
                                    lambda: (self.progress(), key in self.grants)[1])
            p, ticket = self.grants.pop(key)
            ctrl = self.ctrl_in[stage]
            wire = self._wait_progressing(f"publication of sequence {seq} on {ctrl.name}",
                                          lambda t: ctrl.wait_published(seq, t))
            try:
                d = self.layout.match(wire, self.epoch, batch, seq, stage - 1)
            except Exception:
                self._fail()
                raise
            if d.valid_tokens != rows:
                self._fail()
                raise NV.BoundaryError(f"boundary carries {d.valid_tokens} rows, expected {rows}")
            NV.cuda_check(NV.lib().qv_stream_wait_event(self.dev_index, compute.cuda_stream,
                                                        self.ipc_in[stage][seq % 8]), "wait for peer copy")
        else:
            if not self.dst_leases.can_take(stage, seq):
                self._deadline_loop("a free destination slot", lambda: self.dst_leases.can_take(stage, seq))
            d = self.layout.make(self.epoch, batch, seq, stage - 1, rows)
            ticket = self.dst_rings[stage].try_acquire(d)
            p = self.dst_leases.take(stage, ticket)
            self.dst_busy[p] = (stage, ticket)
            e = self.in_edges[stage]
            grp = self.edge_groups[e.src_stage]
            for w in dist.batch_isend_irecv(
                    [dist.P2POp(dist.irecv, self.dst_arena[p, 0, :rows], e.src_rank, group=grp),
                     dist.P2POp(dist.irecv, self.dst_arena[p, 1, :rows], e.src_rank, group=grp)]):
                w.wait()  # the current (consuming) stream waits; the host does not block
        ring = self.dst_rings[stage]
        ring.transition(ticket, NV.OP_TRANSFER_RECORDED)
        ring.transition(ticket, NV.OP_CONSUMER_RECORDED)
        self.received[(batch, stage)] = (p, ticket, seq)
        self.recv_seq[stage] += 1
        self.stats["messages_in"] += 1
        return self.dst_arena[p, 0, :rows], self.dst_arena[p, 1, :rows]

    def retire(self, batch, stage):
        """The consumer of (batch, stage)'s input is enqueued: the destination
        slot is free once the compute stream passes this point."""
        p, ticket, _ = self.received.pop((batch, stage))
        self.dst_done[p].record(torch.cuda.current_stream(self.device))
        self.dst_pending_free.add(p)
        self.progress()

    # ------------------------------------------------------------------ close
    def _check_open(self):
        if self.closed or self.failed:
            raise RuntimeError("transport closed or failed; start a new role epoch")

    def _fail(self):
        self.failed = True
        if self.backend == "p2p":
            for c in list(getattr(self, "ctrl_in", {}).values()) + list(getattr(self, "ctrl_out", {}).values()):
                c.fail()

    def receipt(self):
        return dict(self.stats, backend=self.backend, resource_layout=self.resource_layout,
                    source_peak=self.src_leases.peak, dest_peak=self.dst_leases.peak,
                    source_stalls=self.src_leases.stalls,
                    arena_bytes=(self.src_leases.count + self.dst_leases.count) * self.slot_bytes)

    def close(self):
        if self.closed:
            return self.receipt()
        torch.cuda.synchronize(self.device)
        self._reap()
        receipt = self.receipt()
        if not self.failed:
            dist.barrier(group=self.group)
        self.closed = True
        if self.backend == "p2p":
            for c in list(self.ctrl_out.values()) + list(self.ctrl_in.values()):
                c.close()
            for ptr in self.peer_arena.values():
                NV.lib().qv_arena_close(self.dev_index, ptr)
            for evs in self.ipc_in.values():
                for ev in evs:
                    NV.lib().qv_event_destroy(self.dev_index, ev)
            if not self.failed:
                dist.barrier(group=self.group)
            for evs in self.ipc_out.values():
                for ev in evs:
                    NV.lib().qv_event_destroy(self.dev_index, ev)
            self.dst_arena = None
            NV.lib().qv_arena_free(self.dev_index, self.dst_ptr)
        for r in list(self.src_rings.values()) + list(self.dst_rings.values()):
            r.close()
        self.src_leases.close()
        self.dst_leases.close()
        return receipt
