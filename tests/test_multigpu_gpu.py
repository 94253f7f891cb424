"""The folded pipeline on 2 GPUs reproduces the single-GPU result bit for bit
(same kernels, same per-layer order; only the stage boundaries move between
GPUs), through the peer-to-peer copy-engine transport and through NCCL; so
does the conventional pipeline (the comparison arm).  Needs two GPUs; skipped
otherwise."""

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _need(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


@pytest.mark.parametrize("transport", ["p2p", "nccl"])
def test_two_rank_fold_matches_single_gpu_bit_exact(tmp_path, transport):
    _need(2)
    from qwen_infra_b200.vpp.launch import BankJob, launch

    job = BankJob(model="tiny", request_tokens=[1024, 700, 512], chunk=256, transport=transport,
                  keep_all_outputs=True, banks=2)
    one = launch(job, 1, tmp_path / "one.pt")["outputs"]
    two = launch(job, 2, tmp_path / "two.pt")
    assert sorted(one) == sorted(two["outputs"])
    for b in one:
        assert torch.equal(one[b], two["outputs"][b]), b
    receipt = two["receipt"]
    budget = (2, 3) if receipt["resource_layout"] == "rank" else (7, 7)  # nccl: edge-owned slots
    assert receipt["source_peak"] <= budget[0] and receipt["dest_peak"] <= budget[1]


@pytest.mark.parametrize("transport", ["p2p", "nccl"])
def test_two_rank_conventional_pipeline_matches_single_gpu_bit_exact(tmp_path, transport):
    _need(2)
    from qwen_infra_b200.vpp.launch import BankJob, launch

    job = BankJob(model="tiny", request_tokens=[1024, 700, 512], chunk=256, transport=transport,
                  keep_all_outputs=True, banks=2)
    one = launch(job, 1, tmp_path / "one.pt")["outputs"]
    job.profile = "cpp"
    two = launch(job, 2, tmp_path / "two.pt")
    assert sorted(one) == sorted(two["outputs"])
    for b in one:
        assert torch.equal(one[b], two["outputs"][b]), b
    receipt = two["receipt"]
    budget = (2, 3) if receipt["resource_layout"] == "rank" else (7, 7)  # nccl: edge-owned slots
    assert receipt["source_peak"] <= budget[0] and receipt["dest_peak"] <= budget[1]
