"""The step-wise worker on a real rank (1 GPU, tiny model, the local fold):
driven through the engine route, its per-request final hidden rows and
greedy tokens equal the serial bank's, bit for bit (same ops, same order,
same stream)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_step_driven_rank_equals_the_serial_bank():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwen_infra_b200.vpp import model as M
    from qwen_infra_b200.vpp.runner import FoldedRank
    from qwen_infra_b200.vpp.worker import FoldedWorker, drive_bank

    dev = torch.device("cuda:0")
    tokens = [700, 512, 300, 900]
    g = torch.Generator().manual_seed(11)
    embeds = [torch.randn(t, M.TINY.hidden, generator=g).to(torch.bfloat16).to(dev) for t in tokens]
    serial = FoldedRank(M.TINY, 0, 1, dev, tokens, 128, overlap=False)
    want = serial.run_bank(embeds).clone()
    want_tokens = serial.last_tokens.clone()
    torch.cuda.synchronize()

    stepped = FoldedRank(M.TINY, 0, 1, dev, tokens, 128, overlap=False)
    worker = FoldedWorker(stepped)
    for _ in range(2):  # two banks in a row through the same worker
        worker.begin_bank(embeds)
        sampled = drive_bank(worker, [c.batch for c in stepped.chunks])
        torch.cuda.synchronize()
        stepped.model.check_status()
        assert worker.executed == stepped.order
        assert torch.equal(stepped.last_hidden.view(torch.int16), want.view(torch.int16))
        assert torch.equal(stepped.last_tokens, want_tokens)
        assert sorted(sampled.values()) == sorted(want_tokens.cpu().tolist())
    assert worker.qwen_infra_vpp_resources()["ops_run"] == len(stepped.order)
