"""Step-wise worker (``vpp/worker.py``), on CPU with fake ranks: driven the
way the reference's rank-local engine route drives its workers
(``executor.py:15-73``), every rank runs exactly the op order
``layout.rank_local_stage_orders`` replays for the bank -- the order the
transport grants destination slots in -- and the worker refuses anything
else."""

import pytest
import torch

from qwen_infra_b200.vpp import layout as L
from qwen_infra_b200.vpp import runner as R
from qwen_infra_b200.vpp.worker import FoldedWorker, drive_bank


class FakeRank:
    def __init__(self, rank, ranks, request_tokens, chunk):
        self.rank, self.ranks, self.profile = rank, ranks, "vpp"
        self.request_tokens = list(request_tokens)
        self.chunks = R.plan_bank(self.request_tokens, chunk)
        self.order = L.rank_local_stage_orders([c.batch for c in self.chunks], ranks)[rank]
        self.output_rank, self.transport, self.device = 0, None, torch.device("cpu")
        self.ran = []
        self.tokens = torch.full((len(self.request_tokens),), -1, dtype=torch.int32)

    def run_op(self, batch, stage, embeds=None, host_embeds=None):
        self.ran.append((batch, stage))

    def sample(self, requests=None):
        for q in requests:
            self.tokens[q] = 1000 + q
        return self.tokens


@pytest.mark.parametrize("G", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("tokens", [[2048], [8192, 8192, 8192, 8192], [100, 5000, 2048, 70000]])
def test_engine_route_reproduces_the_bank_order_on_every_rank(G, tokens):
    sampled = None
    for rank in range(G):
        fake = FakeRank(rank, G, tokens, 2048)
        w = FoldedWorker(fake)
        w.begin_bank()
        got = drive_bank(w, [c.batch for c in fake.chunks])
        assert fake.ran == fake.order
        assert not w.order.live and not w.in_bank and w.order.peak_live <= 2 * G - 1
        if rank == 0:
            sampled = got
    # one token per request, sampled on the output rank after the request's last chunk
    last = {}
    for c in R.plan_bank(tokens, 2048):
        last[c.request] = c.batch
    assert sampled == {b: 1000 + q for q, b in last.items()}


def test_out_of_order_steps_are_refused():
    fake = FakeRank(1, 4, [8192, 8192], 2048)
    w = FoldedWorker(fake)
    w.begin_bank()
    with pytest.raises(ValueError):  # returning a batch that was never admitted
        w.execute_model(L.VppStep(None, 0, 1))
    w.execute_model(L.VppStep(None, 0, 0))
    with pytest.raises(ValueError):  # batch ids must increase
        w.execute_model(L.VppStep(None, 0, 0))
    with pytest.raises(TypeError):
        w.execute_model("not a step")
    with pytest.raises(ValueError):
        w.vpp_return_and_sample(L.VppStep(None, 0, 0))


def test_an_order_the_transport_did_not_grant_is_refused():
    fake = FakeRank(0, 2, [8192, 8192], 2048)
    fake.order = list(reversed(fake.order))  # a transport granting some other order
    w = FoldedWorker(fake)
    w.begin_bank()
    with pytest.raises(RuntimeError, match="out of the bank order"):
        drive_bank(w, [c.batch for c in fake.chunks])


def test_conventional_ranks_are_not_step_driven_and_transport_close_needs_an_empty_rank():
    fake = FakeRank(0, 2, [4096], 2048)
    fake.profile = "cpp"
    with pytest.raises(ValueError):
        FoldedWorker(fake)
    fake.profile = "vpp"
    w = FoldedWorker(fake)
    w.begin_bank()
    w.execute_model(L.VppStep(None, 0, 0))
    closed = []
    fake.transport = type("T", (), {"backend": "p2p", "close": lambda self: closed.append(1) or {"ok": 1}})()
    with pytest.raises(RuntimeError):
        w.qwen_infra_vpp_close_transport()
    res = w.qwen_infra_vpp_resources()
    assert res["live_batches"] == [0] and res["ops_run"] == 1
