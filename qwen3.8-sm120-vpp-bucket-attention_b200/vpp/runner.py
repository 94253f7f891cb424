"""Bank driver of one rank of the folded pipeline (one process per GPU).

A bank is R requests of prompt tokens, cut into chunks of at most C tokens
(request-major, as a first-come-first-served chunked-prefill scheduler would
issue them); every chunk is one batch that flows through the 2G virtual stages.
Each rank runs its precomputed stage order (``layout.rank_local_stage_orders``,
the same order the reference's executor messages produce,
``src/qwen_infra/vpp/executor.py:15-73`` / ``worker.py:117-183``):

    receive (or local fold) -> run the stage's layers -> send -> retire

Per-stage FIFO order makes the KV history of chunk j+1 ready when it reaches
a layer: chunk j passed the same stage, on the same stream, before it.

``profile="cpp"`` runs the conventional pipeline instead (the reference's
``--profile cpp``): one stage of L/G layers per rank, chunks in order through
ranks 0..G-1, output on rank G-1 -- the comparison arm for the fold's bubble.
"""

from dataclasses import dataclass

import torch

from . import layout as L
from .model import StageModel


@dataclass(frozen=True)
class Chunk:
    batch: int
    request: int
    start: int
    rows: int


def plan_bank(request_tokens, chunk):
    chunks = []
    for r, tokens in enumerate(request_tokens):
        for start in range(0, tokens, chunk):
            chunks.append(Chunk(len(chunks), r, start, min(chunk, tokens - start)))
    return chunks


class FoldedRank:
    """Rank ``rank`` of ``ranks``.  Folded (``profile="vpp"``): owns stages
    rank and 2G-1-rank, output on rank 0.  Conventional (``"cpp"``): owns
    stage rank of G, output on rank G-1."""

    def __init__(self, shape, rank, ranks, device, request_tokens, chunk, *, transport=None, base_seed=1234,
                 on_device_init=None, keep_all_outputs=False, profile="vpp", kv_shadow=None, overlap=None,
                 attention="auto"):
        if profile not in L.PROFILES:
            raise ValueError("profile is vpp or cpp")
        self.shape, self.rank, self.ranks, self.profile = shape, rank, ranks, profile
        self.device = torch.device(device)
        self.request_tokens = list(request_tokens)
        self.chunk = chunk
        self.chunks = plan_bank(self.request_tokens, chunk)
        batches = [c.batch for c in self.chunks]
        if profile == "vpp":
            self.spans = L.layer_ranges(rank, ranks, shape.layers)
            self.stage_count, self.output_rank = 2 * ranks, 0
            self.order = L.rank_local_stage_orders(batches, ranks)[rank]
        else:
            self.spans = (L.cpp_layer_range(rank, ranks, shape.layers),)
            self.stage_count, self.output_rank = ranks, ranks - 1
            self.order = L.cpp_stage_orders(batches, ranks)[rank]
        layers = [layer for span in self.spans for layer in range(*span)]
        # A folded rank owns two virtual stages whose chunks are independent
        # of each other at any moment (the first traversal's stage on chunk
        # j + k beside the second traversal's on chunk j), so they run on two
        # CUDA streams and each one's kernels fill the SMs the other leaves
        # idle (partial last waves, small producers).  Default: on for the fold,
        # on one GPU and over either transport: boundary waits are stream waits
        # on the consuming stage's stream (the peer copy's event, or the
        # grouped NCCL receive of the edge's own communicator).
        can = profile == "vpp" and self.device.type == "cuda"
        self.overlap = can if overlap is None else (bool(overlap) and can)
        self.model = StageModel(shape, layers, self.device, max_rows=chunk, request_tokens=self.request_tokens,
                                base_seed=base_seed, on_device_init=on_device_init,
                                final_norm=(rank == self.output_rank), kv_shadow=kv_shadow, attention=attention,
                                streams=2 if self.overlap else 1)
        self.transport = transport
        self.keep_all_outputs = keep_all_outputs
        h = shape.hidden
        self.fold = (torch.empty((chunk, h), dtype=torch.bfloat16, device=self.device),
                     torch.empty((chunk, h), dtype=torch.bfloat16, device=self.device))
        # Overlapped fold: three (hidden, residual) pairs, chunk j in pair j % 3;
        # stage G-1 of chunk j waits for stage G of chunk j - 3 (the pair's
        # last reader).
        self.folds = [self.fold] + [(torch.empty_like(self.fold[0]), torch.empty_like(self.fold[1]))
                                    for _ in range(2 if self.overlap else 0)]
        self.streams = [torch.cuda.Stream(self.device) for _ in range(2)] if self.overlap else None
        self.last_hidden = torch.empty((len(self.request_tokens), h), dtype=torch.bfloat16, device=self.device)
        self.last_tokens = torch.full((len(self.request_tokens),), -1, dtype=torch.int32, device=self.device)
        self.outputs = {}
        self.contexts = None
        self.stage_events = []

    def _contexts(self):
        if self.contexts is None:
            self.contexts = [self.model.chunk_context(c.request, c.start, c.rows) for c in self.chunks]
        return self.contexts

    def run_op(self, batch, stage, embeds=None, host_embeds=None, *, record_events=False):
        """One op of this rank's order, on the current stream: receive (or the
        local fold, or the chunk's embeddings on stage 0) -> the stage's
        layers -> send -> retire; on the last stage the final norm of a
        request's last row.  ``run_bank`` runs its serial path as these ops in
        ``self.order``; ``vpp.worker.FoldedWorker`` runs them one step at a
        time (the transport's grant order must then be ``self.order``)."""
        G = self.ranks
        last_stage = self.stage_count - 1
        folded = self.profile == "vpp"
        ch = self.chunks[batch]
        ctx = self._contexts()[batch]
        stream = torch.cuda.current_stream(self.device)
        if stage == 0:
            if host_embeds is not None:
                hidden = host_embeds[ch.request][ch.start:ch.start + ch.rows].to(self.device, non_blocking=True)
            else:
                hidden = embeds[ch.request][ch.start:ch.start + ch.rows]
            residual = None
        elif folded and stage == G:  # local fold: stage G-1 ran on this rank just before
            hidden, residual = self.fold[0][:ch.rows], self.fold[1][:ch.rows]
        else:
            hidden, residual = self.transport.receive(batch, stage, ch.rows)
        if record_events:  # after the input is ready: stage time excludes waiting
            ev0 = torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
        span = (L.stage_layers(stage, G, self.shape.layers) if folded
                else L.cpp_layer_range(stage, G, self.shape.layers))
        on_residual = None
        if folded and stage == G - 1:
            out_planes = (self.fold[0][:ch.rows], self.fold[1][:ch.rows])
        elif stage == last_stage:
            out_planes = None
        else:
            out_planes = self.transport.prepare_send(batch, stage, ch.rows)
            on_residual = (lambda b=batch, s=stage: self.transport.mark_residual_ready(b, s))
        h, r = self.model.run_layers(span, hidden, residual, ctx, out_planes, on_residual)
        if stage != last_stage and not (folded and stage == G - 1):
            self.transport.send(batch, stage, ch.rows)
        if stage != 0 and not (folded and stage == G):
            self.transport.retire(batch, stage)
        if stage == last_stage:
            if self.keep_all_outputs:
                self.outputs[batch] = self.model.final_norm(h, r)
            if ch.start + ch.rows == self.request_tokens[ch.request]:
                self.model.final_norm(h[-1:], r[-1:], out=self.last_hidden[ch.request:ch.request + 1])
        if record_events:
            ev1 = torch.cuda.Event(enable_timing=True)
            ev1.record(stream)
            self.stage_events.append((batch, stage, ev0, ev1))

    def sample(self, requests=None):
        """P+1 on the output rank: the greedy token of each request in
        ``requests`` (all by default) from its final-normed last row, into
        ``last_tokens``."""
        if self.rank != self.output_rank:
            raise RuntimeError("only the output rank samples")
        if requests is None:
            self.model.sample(self.last_hidden, tokens=self.last_tokens)
        else:
            for q in requests:
                self.model.sample(self.last_hidden[q:q + 1], tokens=self.last_tokens[q:q + 1])
        return self.last_tokens

    def run_bank(self, embeds, *, host_embeds=None, record_events=False):
        """Run this rank's ops for one bank.  ``embeds``: device bf16 [tokens, H]
        per request (list), or None with ``host_embeds`` (pinned host tensors,
        copied chunk by chunk inside the run).  On the output rank, returns the
        final-normed last hidden row of each request and leaves each request's
        greedy output token in ``last_tokens``.  ``record_events`` (per-stage
        device times) runs the stages in series on the current stream."""
        if self.overlap and not record_events:
            return self._run_bank_overlapped(embeds, host_embeds)
        self.stage_events = []
        if self.transport is not None:
            self.transport.set_order(self.order)
        for batch, stage in self.order:
            self.run_op(batch, stage, embeds, host_embeds, record_events=record_events)
        if self.rank == self.output_rank:
            # P+1: the one output token of every request (greedy), part of the bank.
            self.model.sample(self.last_hidden, tokens=self.last_tokens)
        return self.last_hidden

    def _run_bank_overlapped(self, embeds, host_embeds):
        """The folded order with this rank's first-traversal stage (r) on one
        stream and its second-traversal stage (2G-1-r) on another.  Order
        constraints: a stage's chunks run in order on its stream (the KV
        history of chunk j + 1 is written by chunk j); a boundary input is an
        event wait on the consuming stream (``transport.receive``, or for the
        local fold on rank G-1 the event of stage G-1 on the same chunk);
        the fold rotates over three pairs, stage G-1 of chunk j waiting for
        stage G of chunk j - 3.  Transport slot events are recorded on the
        stream of the stage that fills or drains the slot.  The attention
        runs without its key-range split here (the other stream fills the
        last wave's idle SMs).  The caller's stream waits for both at the
        end."""
        G = self.ranks
        last_stage = 2 * G - 1
        local = {self.rank: 0, last_stage - self.rank: 1}
        ctxs = self._contexts()
        main = torch.cuda.current_stream(self.device)
        start = torch.cuda.Event()
        start.record(main)
        for st in self.streams:
            st.wait_event(start)
        if self.transport is not None:
            self.transport.set_order(self.order)
        done = {}
        for batch, stage in self.order:
            ch, ctx = self.chunks[batch], ctxs[batch]
            li = local[stage]
            st, ws = self.streams[li], self.model.ws_sets[li]
            fh, fr = self.folds[batch % 3]
            with torch.cuda.stream(st):
                if stage == 0:
                    if host_embeds is not None:
                        hidden = host_embeds[ch.request][ch.start:ch.start + ch.rows].to(self.device,
                                                                                           non_blocking=True)
                    else:
                        hidden = embeds[ch.request][ch.start:ch.start + ch.rows]
                    residual = None
                elif stage == G:  # local fold: stage G-1 of this chunk ran on this rank
                    st.wait_event(done[(batch, G - 1)])
                    hidden, residual = fh[:ch.rows], fr[:ch.rows]
                else:
                    hidden, residual = self.transport.receive(batch, stage, ch.rows)
                on_residual = None
                if stage == G - 1:
                    if batch >= 3:  # a KeyError here would mean an order that breaks the fold rotation
                        st.wait_event(done[(batch - 3, G)])
                    out_planes = (fh[:ch.rows], fr[:ch.rows])
                elif stage == last_stage:
                    out_planes = None
                else:
                    out_planes = self.transport.prepare_send(batch, stage, ch.rows)
                    on_residual = (lambda b=batch, s=stage: self.transport.mark_residual_ready(b, s))
                h, r = self.model.run_layers(L.stage_layers(stage, G, self.shape.layers), hidden, residual, ctx,
                                             out_planes, on_residual, ws, split=False)
                if stage != last_stage and stage != G - 1:
                    self.transport.send(batch, stage, ch.rows)
                if stage != 0 and stage != G:
                    self.transport.retire(batch, stage)
                if stage == last_stage:
                    if self.keep_all_outputs:
                        self.outputs[batch] = self.model.final_norm(h, r)
                    if ch.start + ch.rows == self.request_tokens[ch.request]:
                        self.model.final_norm(h[-1:], r[-1:], out=self.last_hidden[ch.request:ch.request + 1])
                ev = torch.cuda.Event()
                ev.record(st)
                done[(batch, stage)] = ev
        if self.rank == self.output_rank:
            with torch.cuda.stream(self.streams[local[last_stage]]):
                # P+1: the one output token of every request (greedy), part of the bank.
                self.model.sample(self.last_hidden, tokens=self.last_tokens)
        for st in self.streams:
            main.wait_stream(st)
        return self.last_hidden

    def compute_ms(self):
        """Summed device time of this rank's stages in the last recorded bank."""
        return sum(e0.elapsed_time(e1) for _, _, e0, e1 in self.stage_events)
