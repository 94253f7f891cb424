"""``qwen-infra prefill`` command surface of the B200 build (the reference's
``src/qwen_infra/cli.py:181-214`` / ``config.py:52-104``).

    qwen-infra prefill --model qwen27b --profile vpp --transport segment-dma \\
        --chunk-size 2048 --requests 4 --prompt-tokens 32768 [--gpus G] [--dry-run]

Models are synthetic (seeded NVFP4 weights of a named shape: ``qwen27b`` or
``tiny``), prompts are seeded embeddings of ``--prompt-tokens`` tokens.
``--transport segment-dma`` selects the peer-to-peer copy-engine transport
(the reference's segmented DMA edge, rebuilt for NVLink); ``nccl`` the NCCL
send/recv comparison.  ``--profile cpp`` runs the conventional G-stage
pipeline on the same kernels and transport (the comparison arm for the fold).
Output: the reference's record per request (``request_id``, ``text``,
``token_ids`` = the greedy output token, ``finished``), printed as a JSON list;
``text`` is empty (the synthetic model has no tokenizer), and each record adds
the norm and a digest of the final-normed hidden state it was sampled from.
"""

import argparse
import hashlib
import json
import sys
import tempfile
from dataclasses import dataclass
from pathlib import Path

PREFILL_PROFILES = ("cpp", "vpp")


@dataclass(frozen=True)
class PrefillConfig:
    model: str
    profile: str = "vpp"
    chunk_size: int = 2048
    max_model_len: int = 32768
    max_num_seqs: int = 8
    gpu_memory_utilization: float = 0.85
    transport: str = "segment-dma"
    resource_layout: str = "rank"

    def engine_options(self):
        """Validated run options (same rules as the reference's PrefillConfig)."""
        if not self.model or self.profile not in PREFILL_PROFILES:
            raise ValueError("A model and cpp/vpp profile are required")
        if not 1 <= self.chunk_size <= 16384 or self.max_model_len <= 1:
            raise ValueError("Use a positive chunk budget up to 16384 and a positive context capacity")
        if not 1 <= self.max_num_seqs or not 0 < self.gpu_memory_utilization < 1:
            raise ValueError("Invalid sequence or GPU memory budget")
        if self.transport not in ("segment-dma", "nccl"):
            raise ValueError("Expected segment-dma or nccl transport")
        if self.resource_layout not in ("rank", "edge"):
            raise ValueError("Expected rank or edge VPP resource layout")
        options = dict(model=self.model, dtype="bfloat16", kv_cache_dtype="nvfp4", max_num_batched_tokens=self.chunk_size,
                       max_model_len=self.max_model_len, max_num_seqs=self.max_num_seqs,
                       gpu_memory_utilization=self.gpu_memory_utilization, profile=self.profile)
        if self.profile == "vpp":
            fast = self.transport == "segment-dma"
            options["additional_config"] = dict(
                qwen_infra_vpp_rank_local=True,
                qwen_infra_vpp_transport="p2p_copy_engine" if fast else "nccl",
                qwen_infra_vpp_resource_layout=self.resource_layout if fast else "edge",
                qwen_infra_vpp_slots=dict(source=2, destination=3, ring=7),
            )
        return options


def _records(outputs, requests, tokens):
    import torch

    recs = []
    for r in range(requests):
        v = outputs[r]
        raw = v.detach().to("cpu").contiguous().view(-1).view(torch.uint8).numpy().tobytes()  # any dtype
        recs.append(dict(request_id=str(r), text="", token_ids=[int(tokens[r])], finished=True,
                         final_hidden_norm=float(v.float().norm()),
                         final_hidden_sha256=hashlib.sha256(raw).hexdigest()[:16]))
    return recs


def _prefill(args):
    config = PrefillConfig(args.model, args.profile, args.chunk_size, args.max_model_len, max(8, args.requests),
                           args.gpu_memory_utilization, args.transport, args.resource_layout)
    options = config.engine_options()
    if args.requests < 1 or args.prompt_tokens < 1:
        raise ValueError("Requests and prompt token counts must be positive")
    if args.prompt_tokens + 1 > args.max_model_len:
        raise ValueError("Prompt plus one output token must fit --max-model-len")
    if args.dry_run:
        print(json.dumps(dict(engine=options, requests=args.requests, prompt_tokens=args.prompt_tokens,
                              gpus=args.gpus), indent=2))
        return 0
    from .vpp.launch import BankJob, launch

    import torch

    gpus = args.gpus or min(4, torch.cuda.device_count())
    job = BankJob(model=args.model, requests=args.requests, prompt_tokens=args.prompt_tokens,
                  chunk=args.chunk_size, transport="p2p" if args.transport == "segment-dma" else "nccl",
                  profile=args.profile,
                  resource_layout=options.get("additional_config", {}).get("qwen_infra_vpp_resource_layout", ""))
    with tempfile.TemporaryDirectory() as tmp:
        result = launch(job, gpus, Path(tmp) / "bank.pt")
    print(json.dumps(_records(result["outputs"], args.requests, result["tokens"]), indent=2))
    return 0


def main(argv=None):
    parser = argparse.ArgumentParser(prog="qwen-infra")
    sub = parser.add_subparsers(dest="command", required=True)
    prefill = sub.add_parser("prefill", help="Run a bounded prefill bank (folded VPP or conventional pipeline)")
    prefill.add_argument("--model", required=True, choices=("qwen27b", "tiny"))
    prefill.add_argument("--profile", choices=PREFILL_PROFILES, default="vpp")
    prefill.add_argument("--transport", choices=("segment-dma", "nccl"), default="segment-dma")
    prefill.add_argument("--resource-layout", choices=("rank", "edge"), default="rank")
    prefill.add_argument("--chunk-size", type=int, default=2048)
    prefill.add_argument("--max-model-len", type=int, default=32768)
    prefill.add_argument("--gpu-memory-utilization", type=float, default=0.85)
    prefill.add_argument("--requests", type=int, default=1)
    prefill.add_argument("--prompt-tokens", type=int, default=2048)
    prefill.add_argument("--gpus", type=int, default=0)
    prefill.add_argument("--dry-run", action="store_true")
    args = parser.parse_args(argv)
    return _prefill(args)


if __name__ == "__main__":
    sys.exit(main())
