"""Stage-boundary transport exerciser (the reference's transport stress
benchmark, ``benchmarks/vpp_resources.py:84-204``, on this build's
``StageBoundaries``).

Every rank walks its folded rank-local order (``layout.rank_local_stage_orders``)
for ``messages`` batches with no model: a stage's "output" is its input planes
refilled with a payload identity -- hidden = the batch id, residual = the
source stage -- and every receive checks on the GPU that the planes carry
exactly that, so a message that lands in the wrong slot, arrives stale or is
torn shows up as mismatching elements.  Valid rows cycle through
{0, 1, 17, C/2, C} (a 0-row boundary included), which exercises ragged
copies, slot wrap-around (7-slot rings, 2 source / 3 destination physical
slots) and the final drain.

``timed=True`` instead sends full-capacity messages and measures, with CUDA
events on the sending rank's copy stream, the bytes moved per second
through the whole protocol (credit waits included).  ``copy_rate`` times the
boundary copy alone (``--copy-rate [--both]``).

    python -m qwen_infra_b200.vpp.stress --gpus 2 [--backend p2p|nccl] [--timed | --copy-rate [--both]]

One process per GPU (spawned here), NCCL process group, gloo control plane.
"""

import argparse
import json
import os
import socket
import tempfile
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from . import layout as L

ROWS_CYCLE = ("0", "1", "17", "C/2", "C")


def rows_for(batch, capacity, timed):
    if timed:
        return capacity
    pick = ROWS_CYCLE[batch % len(ROWS_CYCLE)]
    return {"0": 0, "1": 1, "17": 17, "C/2": capacity // 2, "C": capacity}[pick]


def run_rank(rank, world, device, *, capacity, hidden, messages, backend="p2p", resource_layout=None,
             timed=False, timeout=60.0):
    """One rank's walk; returns its receipt with ``mismatches`` (elements that
    differed from the payload identity), ``received`` and, when timed, the
    copy rate of its outgoing messages."""
    from .stages import StageBoundaries

    if timed and backend != "p2p":
        raise ValueError("timed copies are measured on the peer-to-peer transport's copy stream")
    G = world
    last = 2 * G - 1
    transport = StageBoundaries(rank, world, device, capacity, hidden, backend=backend, timeout=timeout,
                                resource_layout=resource_layout)
    order = L.rank_local_stage_orders(list(range(messages)), G)[rank]
    transport.set_order(order)
    bad = torch.zeros((), dtype=torch.int64, device=device)
    fold = torch.empty((2, capacity, hidden), dtype=torch.bfloat16, device=device)
    received = 0
    sent_bytes = 0
    ev = None
    for batch, stage in order:
        rows = rows_for(batch, capacity, timed)
        if stage == 0:
            pass  # the first stage has no input boundary
        elif stage == G:  # local fold on rank G-1
            h, r = fold[0, :rows], fold[1, :rows]
            bad += (h != batch).sum() + (r != G - 1).sum()
        else:
            h, r = transport.receive(batch, stage, rows)
            if not timed:
                bad += (h != batch).sum() + (r != stage - 1).sum()
            transport.retire(batch, stage)
            received += 1
        if stage == last:
            continue
        if stage == G - 1:
            fold[0, :rows].fill_(batch)
            fold[1, :rows].fill_(stage)
            continue
        hp, rp = transport.prepare_send(batch, stage, rows)
        rp.fill_(stage)
        transport.mark_residual_ready(batch, stage)
        hp.fill_(batch)
        if timed and ev is None and batch >= 2:  # after two warm-up messages per edge
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(transport.copy_stream)
            sent_bytes = 0
        transport.send(batch, stage, rows)
        if ev is not None:
            sent_bytes += 2 * rows * hidden * 2
    end = None
    if timed and ev is not None:
        end = torch.cuda.Event(enable_timing=True)
        end.record(transport.copy_stream)
    torch.cuda.synchronize(device)
    receipt = transport.close()
    receipt.update(rank=rank, mismatches=int(bad.item()), received=received, messages=messages,
                   capacity=capacity, hidden=hidden)
    if end is not None:
        ms = ev.elapsed_time(end)
        receipt.update(copy_ms=ms, copy_bytes=sent_bytes, copy_gbs=sent_bytes / (ms / 1e3) / 1e9 if ms > 0 else None)
    return receipt


def copy_rate(rank, world, device, *, capacity=2048, hidden=5120, reps=50, both=False, segment=0):
    """NVLink rate of the transport's boundary copy itself (qv_copy_message:
    both planes of a C x H bf16 message, peer to peer into an IPC-mapped
    destination), without the credit protocol: rank 0 (and with ``both`` also
    rank 1, to rank 0 at the same time) copies ``reps`` messages back to back
    on one stream, timed with CUDA events on that stream."""
    from . import native as NV

    plane = capacity * hidden * 2
    dst_ptr, handle = NV.arena_alloc(device.index, 2 * plane)
    handles = [None] * world
    dist.all_gather_object(handles, handle)
    src = torch.empty(2 * plane, dtype=torch.uint8, device=device)
    src.fill_(rank + 1)
    torch.cuda.synchronize(device)
    result = dict(rank=rank, capacity=capacity, hidden=hidden, message_bytes=2 * plane, reps=reps, both=both,
                  segment=segment)
    sending = rank == 0 or (both and rank == 1)
    peer = 1 - rank
    peer_ptr = NV.arena_open(device.index, handles[peer]) if sending else None
    dist.barrier()
    if sending:
        stream = torch.cuda.Stream(device=device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

        def issue():
            NV.cuda_check(NV.lib().qv_copy_message(device.index, stream.cuda_stream, None, None, src.data_ptr(),
                                                   src.data_ptr() + plane, peer_ptr, peer_ptr + plane, plane,
                                                   segment, None, None), "peer copy")

        for _ in range(3):
            issue()
        e0.record(stream)
        for _ in range(reps):
            issue()
        e1.record(stream)
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1)
        result.update(ms=ms, gbs=reps * 2 * plane / (ms / 1e3) / 1e9, us_per_message=ms * 1e3 / reps)
    dist.barrier()
    if sending:
        NV.lib().qv_arena_close(device.index, peer_ptr)
    dist.barrier()
    NV.lib().qv_arena_free(device.index, dst_ptr)
    return result


def _worker(rank, world, port, kwargs, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=kwargs.get("timeout", 60.0) + 30))
    try:
        kwargs = dict(kwargs)
        mode = kwargs.pop("mode", "walk")
        receipt = (copy_rate if mode == "copy" else run_rank)(rank, world, dev, **kwargs)
        Path(out_dir, f"rank{rank}.json").write_text(json.dumps(receipt))
    finally:
        dist.destroy_process_group()


def launch(world, **kwargs):
    """Spawn ``world`` ranks (GPU i for rank i); returns their receipts."""
    if world < 2 or world > torch.cuda.device_count():
        raise ValueError(f"needs 2 .. {torch.cuda.device_count()} GPUs, asked {world}")
    import __graft_entry__

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as out_dir:
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=__graft_entry__.spawn_call, args=("qwen_infra_b200.vpp.stress", "_worker",
                                                                      r, world, port, kwargs, out_dir))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=kwargs.get("timeout", 60.0) * 4 + 120)
        codes = [p.exitcode for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        if any(c != 0 for c in codes):
            raise RuntimeError(f"stress ranks exited with {codes}")
        return [json.loads(Path(out_dir, f"rank{r}.json").read_text()) for r in range(world)]


def main(argv=None):
    ap = argparse.ArgumentParser(prog="qwen_infra_b200.vpp.stress")
    ap.add_argument("--gpus", type=int, default=2)
    ap.add_argument("--capacity", type=int, default=2048)
    ap.add_argument("--hidden", type=int, default=5120)
    ap.add_argument("--messages", type=int, default=20)
    ap.add_argument("--backend", choices=("p2p", "nccl"), default="p2p")
    ap.add_argument("--resource-layout", choices=("rank", "edge"), default=None)
    ap.add_argument("--timed", action="store_true")
    ap.add_argument("--copy-rate", action="store_true",
                    help="time back-to-back boundary copies (no credit protocol) instead of the walk")
    ap.add_argument("--both", action="store_true", help="--copy-rate: both directions at once")
    ap.add_argument("--segment", type=int, default=0, help="--copy-rate: bytes per cudaMemcpyAsync (0: whole plane)")
    a = ap.parse_args(argv)
    if a.copy_rate:
        receipts = launch(a.gpus, mode="copy", capacity=a.capacity, hidden=a.hidden, both=a.both, segment=a.segment)
    else:
        receipts = launch(a.gpus, capacity=a.capacity, hidden=a.hidden, messages=a.messages, backend=a.backend,
                          resource_layout=a.resource_layout, timed=a.timed)
    for r in receipts:
        print(json.dumps(r))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
