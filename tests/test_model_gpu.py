"""End-to-end parity of the virtual-stage compute on the tiny configuration:
final hidden states of the GPU path against the fp32 dequantised forward
(max |diff| / max |ref| < 2e-2, the tolerance of the benchmark contract)."""

import numpy as np
import pytest
import torch

from oracle import model as OM

pytestmark = pytest.mark.gpu


def test_tiny_model_two_stages_match_oracle():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwen_infra_b200.vpp import model as M

    shape = M.TINY
    tokens, chunk = 1024, 512
    dev = torch.device("cuda:0")
    embeds = (torch.randn(tokens, shape.hidden, generator=torch.Generator().manual_seed(99))).to(torch.bfloat16)
    stage = M.StageModel(shape, range(shape.layers), dev, max_rows=chunk, request_tokens=[tokens], final_norm=True)
    outs = []
    half = shape.layers // 2
    for start in range(0, tokens, chunk):
        ctx = stage.chunk_context(0, start, min(chunk, tokens - start))
        hidden = embeds[start:start + ctx.rows].to(dev)
        h1, r1 = stage.run_layers((0, half), hidden, None, ctx)
        h1, r1 = h1.clone(), r1.clone()
        h2, r2 = stage.run_layers((half, shape.layers), h1, r1, ctx)
        outs.append(stage.final_norm(h2, r2).float().cpu())
    torch.cuda.synchronize()
    stage.check_status()
    got = torch.cat(outs).numpy()
    oracle = OM.OracleModel(OM.TINY, range(OM.TINY.layers), tokens)
    want = oracle.forward_chunks(embeds.float().numpy(), chunk)
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err < 2e-2, err
