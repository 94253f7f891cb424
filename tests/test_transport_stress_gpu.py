"""Stage-boundary transport under stress on 2 GPUs (the reference's transport
test, benchmarks/vpp_resources.py:84-204): 20 messages per wire edge along the
folded rank-local order, payload identity checked on every receive (hidden =
batch id, residual = source stage), valid rows cycling through
{0, 1, 17, C/2, C}, then every slot and ring drained.  Rank-shared slots peak
at <= 2 source and <= 3 destination; edge-owned slots at <= 7 per edge."""

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _need(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


@pytest.mark.parametrize("backend,layout", [("p2p", "rank"), ("p2p", "edge"), ("nccl", "edge")])
def test_payload_identity_and_slot_budget(backend, layout):
    _need(2)
    from qwen_infra_b200.vpp import stress

    receipts = stress.launch(2, capacity=512, hidden=1024, messages=20, backend=backend, resource_layout=layout)
    for r in receipts:
        assert r["mismatches"] == 0, r
        assert r["resource_layout"] == layout
        if layout == "rank":
            assert r["source_peak"] <= 2 and r["dest_peak"] <= 3, r
        else:
            assert r["source_peak"] <= 7 and r["dest_peak"] <= 7, r
    # G = 2: each rank receives one message per batch over its wire edge
    assert [r["received"] for r in receipts] == [20, 20]
