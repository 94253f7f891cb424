"""Folded virtual-pipeline placement and per-rank stage order, for G ranks.

Generalises the reference's four-rank topology (``src/qwen_infra/vpp/layout.py:14-139``)
to 2G virtual stages on G ranks.  With ``ranks=4`` and 64 layers every
function returns what the reference returns (checked against fixtures recorded
from the reference itself).

Folded placement: rank r runs virtual stage r on the forward traversal and
stage 2G-1-r on the return traversal, so rank G-1 hands stage G-1 to stage G
locally (the fold) and every other stage boundary crosses to a neighbour.
"""

from collections import deque
from dataclasses import dataclass
import json


def _check_rank(rank, ranks):
    if type(ranks) is not int or ranks < 1:
        raise ValueError("Expected a positive number of ranks")
    if type(rank) is not int or not 0 <= rank < ranks:
        raise ValueError("Expected one of the logical P ranks")


def stage_count(ranks):
    return 2 * ranks


def layer_ranges(rank, ranks=4, layers=64):
    """(forward span, return span) of layer indices owned by ``rank``."""
    _check_rank(rank, ranks)
    per = layers // (2 * ranks)
    if per * 2 * ranks != layers:
        raise ValueError("Layers must split evenly into 2G virtual stages")
    back = 2 * ranks - 1 - rank
    return (rank * per, (rank + 1) * per), (back * per, (back + 1) * per)


def stage_rank(stage, ranks=4):
    if type(stage) is not int or not 0 <= stage < 2 * ranks:
        raise ValueError("invalid virtual stage")
    return stage if stage < ranks else 2 * ranks - 1 - stage


def stage_layers(stage, ranks=4, layers=64):
    per = layers // (2 * ranks)
    return stage * per, (stage + 1) * per


def communication(rank, traversal, ranks=4):
    """(source rank, destination rank) of the boundary into / out of this
    rank's stage on the given traversal; None where there is no wire."""
    _check_rank(rank, ranks)
    if traversal not in (0, 1):
        raise ValueError("Expected forward or return traversal")
    last = ranks - 1
    if traversal == 0:
        return (rank - 1 if rank else None, rank + 1 if rank < last else None)
    return (rank + 1 if rank < last else None, rank - 1 if rank else None)


def wire_edges(ranks=4):
    """Source stages whose output crosses to another rank: every stage but
    the fold (G-1 -> G) and the last one.  For G=4: (0, 1, 2, 4, 5, 6)."""
    return tuple(s for s in range(2 * ranks - 1) if s != ranks - 1)


@dataclass
class VppStep:
    scheduler_output: object
    batch_id: int
    traversal: int = 0


@dataclass
class VppContinuation:
    batch_id: int


class RankLocalOrder:
    """Order in which one rank runs its two virtual stages.

    Holds a forward FIFO (admitted, not yet run on the forward stage) and a
    return FIFO (forward stage done, return stage pending).  At most 2G-1
    batches are live.  After admission the rank prefers forward work until
    its warm-up credit (2G-1-2r) is used, then alternates forward / return;
    a drain request runs return work regardless.
    """

    def __init__(self, rank, ranks=4):
        _check_rank(rank, ranks)
        self.rank, self.ranks = rank, ranks
        self.capacity = 2 * ranks - 1
        self.return_stage = 2 * ranks - 1 - rank
        self._reset_credit()
        self.pending, self.returns = deque(), deque()
        self.live, self.returned = set(), set()
        self.last_batch = -1
        self.peak_live = 0

    def _reset_credit(self):
        self.warmup = 2 * self.ranks - 1 - 2 * self.rank
        self.prefer_first = True

    def admit(self, batch):
        if type(batch) is not int or batch <= self.last_batch:
            raise ValueError("Batch IDs must strictly increase")
        if len(self.live) >= self.capacity:
            raise RuntimeError("Admission bound of 2G-1 live batches exceeded")
        self.last_batch = batch
        self.pending.append(batch)
        self.live.add(batch)
        self.peak_live = max(self.peak_live, len(self.live))

    def next(self, *, draining=False):
        """Pick the next (batch, stage) for this rank, or None."""
        forward_first = self.warmup > 0 or self.prefer_first
        if forward_first and self.pending:
            batch = self.pending.popleft()
            self.returns.append(batch)
            if self.warmup > 0:
                self.warmup -= 1
            self.prefer_first = self.warmup > 0
            return batch, self.rank
        if self.returns and (draining or not forward_first):
            batch = self.returns.popleft()
            self.returned.add(batch)
            if self.warmup > 0:
                # A drain took a return before the warm-up window filled:
                # give that credit back for a later admission.
                self.warmup += 1
            self.prefer_first = True
            return batch, self.return_stage
        return None

    def release(self, batch):
        if batch not in self.returned:
            raise ValueError("Cannot release an unreturned or already released batch")
        self.returned.discard(batch)
        self.live.discard(batch)
        if not self.live:
            self._reset_credit()


def rank_local_stage_orders(batch_ids, ranks=4):
    """CPU replay of the admit / return / release messages every rank sees
    for one finite bank; returns each rank's [(batch, stage)] list."""
    bank = tuple(batch_ids)
    if not bank or len(bank) > 65536:
        raise ValueError("Expected one bounded nonempty bank")
    orders = [[] for _ in range(ranks)]
    planners = [RankLocalOrder(r, ranks) for r in range(ranks)]

    def step(r, draining=False):
        op = planners[r].next(draining=draining)
        if op is not None:
            orders[r].append(op)
        return op

    def admit_all(batch):
        for r, plan in enumerate(planners):
            plan.admit(batch)
            step(r)
            if r == ranks - 1:
                step(r)  # the fold: stage G-1 then stage G on the same rank

    window = min(2 * ranks - 1, len(bank))
    for batch in bank[:window]:
        admit_all(batch)
    for index, batch in enumerate(bank):
        for r, plan in enumerate(planners):
            step(r, draining=True)
            while batch not in plan.returned:
                if step(r, draining=True) is None:
                    raise RuntimeError("Missing local dependency while draining")
        for plan in planners:
            plan.release(batch)
        if index + window < len(bank):
            admit_all(bank[index + window])
    return orders


# ---------------------------------------------------------------------------
# Conventional pipeline (the reference's ``--profile cpp``: vLLM pipeline
# parallel with G stages, ``src/qwen_infra/config.py:74-80``), kept as the
# comparison arm for the fold: G stages of L/G layers, stage r on rank r,
# every chunk crossing ranks 0 -> 1 -> ... -> G-1, the last rank producing the
# output.  Its boundaries are the forward wire edges of the folded layout
# (stage s -> s+1 for s < G-1), so the same transport carries them.
# ---------------------------------------------------------------------------

PROFILES = ("vpp", "cpp")


def cpp_layer_range(rank, ranks=4, layers=64):
    """Layer span of ``rank``'s single stage in the conventional pipeline."""
    _check_rank(rank, ranks)
    per = layers // ranks
    if per * ranks != layers:
        raise ValueError("Layers must split evenly into G stages")
    return rank * per, (rank + 1) * per


def cpp_stage_orders(batch_ids, ranks=4):
    """Each rank's [(batch, stage)] list in the conventional pipeline: every
    batch through the rank's one stage, in admission order (per-stage FIFO,
    which keeps each layer's KV history in chunk order)."""
    bank = tuple(batch_ids)
    if not bank or len(bank) > 65536:
        raise ValueError("Expected one bounded nonempty bank")
    if type(ranks) is not int or ranks < 1:
        raise ValueError("Expected a positive number of ranks")
    return [[(b, r) for b in bank] for r in range(ranks)]


def retained_boundary_bytes(tokens, live_batches=6, hidden=5120):
    """Bytes of dual-bf16 boundary planes kept for ``live_batches`` messages."""
    if tokens <= 0 or not 1 <= live_batches <= 6:
        raise ValueError("Positive tokens and bounded in-flight queue required")
    return tokens * hidden * 2 * 2 * live_batches


def profile_annotation(rank, traversal, batch_id, kind, requests, ranks=4, layers=64):
    """Trace scope name of one stage's compute / send / recv span.
    ``requests``: [(request id, query tokens, history tokens)]."""
    spans = layer_ranges(rank, ranks, layers)
    if traversal not in (0, 1) or kind not in ("compute", "send", "recv"):
        raise ValueError("Expected one virtual stage and its compute/transfer scope")
    reqs = [dict(id=str(r), q=q, h=h) for r, q, h in requests]
    if any(r["q"] <= 0 or r["h"] < 0 for r in reqs):
        raise ValueError("Invalid trace query/history metadata")
    return "qwen_infra_vpp:" + json.dumps(
        dict(rank=rank, stage=rank if traversal == 0 else 2 * ranks - 1 - rank, batch=batch_id, kind=kind,
             layers=spans[traversal], requests=reqs),
        separators=(",", ":"))
