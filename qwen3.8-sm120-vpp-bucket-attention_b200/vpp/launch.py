"""Launch one bank on G GPUs: one worker process per GPU (spawned here, or
started by torchrun), NCCL process group for the device plumbing, gloo for
the boundary control plane, 2G virtual stages folded onto the G ranks (or,
with ``profile="cpp"``, the conventional G-stage pipeline).
"""

import os
import socket
from dataclasses import asdict, dataclass, field
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


@dataclass
class BankJob:
    model: str = "qwen27b"
    layers: int = 0  # 0: the model's own depth
    requests: int = 4
    prompt_tokens: int = 8192
    chunk: int = 2048
    transport: str = "p2p"  # or "nccl"
    profile: str = "vpp"  # or "cpp" (conventional pipeline, the comparison arm)
    resource_layout: str = ""  # "rank" or "edge"; empty: the transport's default
    seed: int = 4321
    keep_all_outputs: bool = False
    banks: int = 1
    timeout_s: float = 120.0
    request_tokens: list = field(default_factory=list)

    def tokens(self):
        return list(self.request_tokens) or [self.prompt_tokens] * self.requests


def shape_of(job):
    from dataclasses import replace

    from .model import SHAPES

    s = SHAPES[job.model]
    if job.layers and job.layers != s.layers:
        s = replace(s, layers=job.layers)
    return s


def seeded_embeddings(job, hidden, device):
    """Seeded bf16 N(0, 1) prompt embeddings (generated on the CPU so every
    world size sees the same values)."""
    g = torch.Generator().manual_seed(job.seed)
    return [torch.randn(t, hidden, generator=g).to(torch.bfloat16).to(device) for t in job.tokens()]


def run_rank(job, rank, world, local_rank):
    """Body of one rank; returns the output rank's outputs (CPU tensors; rank 0
    folded, rank G-1 conventional) or None, the transport receipt, and the
    output rank's sampled token per request (or None)."""
    from .runner import FoldedRank
    from .stages import StageBoundaries

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    shape = shape_of(job)
    transport = None
    if world > 1:
        transport = StageBoundaries(rank, world, dev, job.chunk, shape.hidden, backend=job.transport,
                                    timeout=job.timeout_s, profile=job.profile,
                                    resource_layout=job.resource_layout or None)
    runner = FoldedRank(shape, rank, world, dev, job.tokens(), job.chunk, transport=transport,
                        keep_all_outputs=job.keep_all_outputs,
                        on_device_init=shape.hidden > 2048, profile=job.profile)
    embeds = seeded_embeddings(job, shape.hidden, dev) if rank == 0 else None
    out = tokens = None
    for _ in range(job.banks):
        last = runner.run_bank(embeds)
    torch.cuda.synchronize(dev)
    runner.model.check_status()
    if rank == runner.output_rank:
        if job.keep_all_outputs:
            out = {b: t.float().cpu() for b, t in runner.outputs.items()}
        else:
            out = last.float().cpu()
        tokens = runner.last_tokens.cpu().tolist()
    receipt = transport.close() if transport is not None else None
    return out, receipt, tokens


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, job_dict, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    job = BankJob(**job_dict)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=job.timeout_s))
    try:
        out, receipt, tokens = run_rank(job, rank, world, rank)
        if rank == (world - 1 if job.profile == "cpp" else 0):  # the output rank writes the result
            torch.save(dict(outputs=out, receipt=receipt, tokens=tokens), result_path)
    finally:
        dist.destroy_process_group()


def launch(job, world, result_path):
    """Spawn ``world`` workers (GPU i for rank i) and run the bank(s); the
    output rank writes its outputs to ``result_path``; returns what it wrote."""
    if world > torch.cuda.device_count():
        raise ValueError(f"{world} ranks but {torch.cuda.device_count()} visible GPUs")
    import __graft_entry__

    mp.spawn(__graft_entry__.spawn_entry, args=(world, _free_port(), asdict(job), str(result_path)), nprocs=world,
             join=True)
    return torch.load(result_path)
