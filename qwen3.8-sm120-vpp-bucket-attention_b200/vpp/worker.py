"""Step-wise worker surface of one rank of the folded pipeline: the
reference's ``FoldedWorker`` RPCs (``src/qwen_infra/vpp/worker.py:117-273``)
on this build's ``FoldedRank``, for an engine that schedules one chunk at a
time instead of handing a rank a whole bank.

``execute_model(VppStep(scheduler_output, batch_id, traversal))``:

* traversal 0 admits the batch to the rank's ``RankLocalOrder`` and runs the
  rank's next op (the fold rank G-1 runs two: stage G-1, then stage G on the
  same device), then answers ``VppContinuation(batch_id)``;
* traversal 1 drains: runs return-side ops until the batch has come back,
  then releases it; it answers ``None`` (the engine samples next).

``vpp_return_and_sample(step)`` is traversal 1 followed by the greedy token
of the request the batch completes (output rank only).  ``drive_bank`` is the
engine side of the rank-local route (the reference's
``executor.py:15-73``): admit up to 2G-1 batches, then for each batch in
order drain / sample it and admit the next.  Driven that way, every rank's
ops come out in exactly the order ``layout.rank_local_stage_orders`` replays
for the bank, which is the order the transport grants destination slots in
(``begin_bank`` hands it over); the worker checks every op against it and
refuses to run one out of that order.

There is no vLLM here: ``scheduler_output`` is kept per batch and handed
back on ``schedules`` for an adapter that needs it; the chunk a batch stands
for comes from the rank's bank plan (``FoldedRank.chunks``).
"""

from . import layout as L


class FoldedWorker:
    def __init__(self, runner):
        if getattr(runner, "profile", "vpp") != "vpp":
            raise ValueError("the step-wise worker runs the folded (vpp) order; cpp ranks run run_bank")
        self.runner = runner
        self.rank, self.ranks = runner.rank, runner.ranks
        self.order = L.RankLocalOrder(self.rank, self.ranks)
        self.schedules = {}
        self.executed = []
        self.embeds = self.host_embeds = None
        self.in_bank = False

    # -------------------------------------------------------------- bank
    def begin_bank(self, embeds=None, host_embeds=None):
        """Start a bank: the inputs of its stage-0 ops and, with a
        transport, the grant order (the whole bank's op list)."""
        if self.order.live:
            raise RuntimeError("the previous bank still has live batches")
        self.embeds, self.host_embeds = embeds, host_embeds
        self.executed = []
        self.order = L.RankLocalOrder(self.rank, self.ranks)
        if self.runner.transport is not None:
            self.runner.transport.set_order(self.runner.order)
        self.in_bank = True

    def _advance(self, draining=False):
        op = self.order.next(draining=draining)
        if op is None:
            return None
        i = len(self.executed)
        expected = self.runner.order[i] if i < len(self.runner.order) else None
        if op != expected:
            raise RuntimeError(f"op {op} out of the bank order (expected {expected}): the transport grants "
                               "destination slots in that order")
        self.runner.run_op(*op, self.embeds, self.host_embeds)
        self.executed.append(op)
        return op

    # -------------------------------------------------------------- RPCs
    def execute_model(self, step):
        if not isinstance(step, L.VppStep):
            raise TypeError("FoldedWorker requires an explicit VPP step")
        if not self.in_bank:
            raise RuntimeError("begin_bank first")
        batch = step.batch_id
        if step.traversal == 0:
            self.order.admit(batch)
            self.schedules[batch] = step.scheduler_output
            self._advance()
            if self.rank == self.ranks - 1:
                self._advance()  # the fold: stage G-1, then stage G on this device
            return L.VppContinuation(batch)
        if step.traversal != 1:
            raise ValueError("traversal is 0 (first) or 1 (return)")
        if batch not in self.order.live:
            raise ValueError(f"batch {batch} is not live on rank {self.rank}")
        self._advance(draining=True)
        while batch not in self.order.returned:
            if self._advance(draining=True) is None:
                raise RuntimeError("Missing VPP stage while draining a named batch")
        self.order.release(batch)
        self.schedules.pop(batch, None)
        if not self.order.live and len(self.executed) == len(self.runner.order):
            self.in_bank = False
        return None

    def vpp_return_and_sample(self, step):
        """Traversal 1 and, on the output rank, the greedy token of the
        request this batch completes (``-1`` when it completes none)."""
        if not isinstance(step, L.VppStep) or step.traversal != 1:
            raise ValueError("combined return requires a traversal-1 step")
        self.execute_model(step)
        runner = self.runner
        if runner.rank != runner.output_rank:
            return None
        ch = runner.chunks[step.batch_id]
        if ch.start + ch.rows != runner.request_tokens[ch.request]:
            return -1
        return int(runner.sample([ch.request])[ch.request].item())

    def qwen_infra_vpp_close_transport(self):
        transport = self.runner.transport
        if transport is None:
            return dict(backend="local fold", closed=False)
        if self.order.live:
            raise RuntimeError("Finish all VPP batches before closing transport")
        receipt = transport.close()
        return dict(backend=transport.backend, closed=True, resources=receipt)

    def qwen_infra_vpp_resources(self):
        runner = self.runner
        out = dict(rank=self.rank, live_batches=sorted(self.order.live), peak_live=self.order.peak_live,
                   ops_run=len(self.executed), ops_in_bank=len(runner.order))
        device = getattr(runner, "device", None)
        if device is not None and getattr(device, "type", "cpu") == "cuda":
            import torch

            out["cuda"] = dict(allocated=torch.cuda.memory_allocated(device),
                               reserved=torch.cuda.memory_reserved(device),
                               peak_allocated=torch.cuda.max_memory_allocated(device))
        return out


def drive_bank(worker, batch_ids, schedules=None, sample=True):
    """The engine's rank-local route for one bank, on one worker (every rank
    receives the same step sequence): admit the first 2G-1 batches, then for
    each batch in order return it (and sample on the output rank) and admit
    the next.  Returns the tokens sampled, by batch (output rank)."""
    bank = list(batch_ids)
    window = min(2 * worker.ranks - 1, len(bank))
    schedules = schedules or {}
    tokens = {}
    for batch in bank[:window]:
        worker.execute_model(L.VppStep(schedules.get(batch), batch, 0))
    for index, batch in enumerate(bank):
        step = L.VppStep(schedules.get(batch), batch, 1)
        if sample:
            tok = worker.vpp_return_and_sample(step)
            if tok is not None and tok >= 0:
                tokens[batch] = tok
        else:
            worker.execute_model(step)
        if index + window < len(bank):
            nxt = bank[index + window]
            worker.execute_model(L.VppStep(schedules.get(nxt), nxt, 0))
    return tokens
