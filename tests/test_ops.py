"""The torch.library operators: registered under qwen_b200, fake
implementations give the real ops' output shapes and dtypes without a GPU
(what torch.compile traces with), and on a B200 each op returns what the
plain kernel wrapper returns."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from qwen_infra_b200 import ops

OPS = torch.ops.qwen_b200


def test_every_operator_is_registered():
    for name in ops.OPS:
        assert hasattr(OPS, name), name


def test_fake_shapes_match_the_contracts():
    with FakeTensorMode():
        dev = "cuda"
        bf = dict(dtype=torch.bfloat16, device=dev)
        x = torch.empty(300, 5120, **bf)
        q, sc, upd = OPS.gemma_nvfp4_pack(x, torch.empty_like(x), torch.empty(5120, **bf),
                                          torch.empty(1, device=dev))
        assert q.shape == (300, 2560) and q.dtype == torch.uint8
        assert sc.shape == (384, 80) and sc.dtype == torch.int32 and upd.shape == x.shape
        q, sf, upd = OPS.norm_pack(torch.empty(17, 1024, **bf), None, torch.empty(1024, **bf),
                                   torch.empty(1, device=dev))
        assert q.shape == (17, 512) and sf.shape == (128 * 64,)
        qkv = torch.empty(5, (2 * 64 + 2 * 8) * 128, **bf)
        caches = [torch.empty(4, 16, 8, 64, dtype=torch.uint8, device=dev) for _ in range(2)]
        scales = [torch.empty(4, 16, 8, 8, dtype=torch.uint8, device=dev) for _ in range(2)]
        qo = OPS.qk_rope_kv_append(qkv, torch.empty(5, dtype=torch.int32, device=dev), torch.empty(128, **bf),
                                   torch.empty(128, **bf), torch.empty(64, 128, device=dev),
                                   torch.empty(5, dtype=torch.int32, device=dev), *caches, *scales,
                                   torch.empty(1, device=dev), torch.empty(1, device=dev), 64, 8, 128)
        assert qo.shape == (5, 64 * 128) and qo.dtype == torch.bfloat16
        fp8, s = OPS.gate_fp8(torch.empty(5, 8192, **bf), qkv[:, 128:], 128, 256)
        assert fp8.dtype == torch.float8_e4m3fn and fp8.shape == (5, 8192) and s.shape == (5,)
        a, b = torch.empty(256, 2560, dtype=torch.uint8, device=dev), torch.empty(512, 2560, dtype=torch.uint8,
                                                                                   device=dev)
        out = OPS.nvfp4_gemm(a, torch.empty(1, dtype=torch.uint8, device=dev), b,
                             torch.empty(1, dtype=torch.uint8, device=dev), torch.empty(1, device=dev), 5120)
        assert out.shape == (256, 512) and out.dtype == torch.bfloat16
        act, asf = OPS.nvfp4_gemm_swiglu(a, a, b, b, torch.empty(1, device=dev), torch.empty(1, device=dev), 5120)
        assert act.shape == (256, 128)
        att = OPS.paged_prefill_attention(torch.empty(7, 64 * 128, **bf), *caches, *scales,
                                          torch.empty(4, dtype=torch.int32, device=dev),
                                          torch.empty(1, device=dev), torch.empty(1, device=dev), 30, 64)
        assert att.shape == (7, 64 * 128)
        tok = OPS.lm_head_argmax(torch.empty(4, 5120, **bf), torch.empty(1000, 5120, **bf))
        assert tok.shape == (4,) and tok.dtype == torch.int32


@pytest.mark.gpu
def test_operators_equal_the_kernel_wrappers():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwen_infra_b200 import kernels as K

    dev = torch.device("cuda:0")
    g = torch.Generator(device="cpu").manual_seed(3)
    x = torch.randn(200, 5120, generator=g).to(torch.bfloat16).to(dev)
    r = torch.randn(200, 5120, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(5120, generator=g) * 0.05).to(torch.bfloat16).to(dev)
    gs = torch.tensor([84.0], device=dev)
    q, sc, upd = OPS.gemma_nvfp4_pack(x, r, w, gs)
    q2, sf2, upd2 = K.norm_pack(x, r, w, gs)
    torch.cuda.synchronize()
    assert torch.equal(q, q2) and torch.equal(upd, upd2)
    from oracle import formats as F

    assert (F.unswizzle_scales(sc.view(torch.uint8).view(-1).cpu().numpy(), 200, 5120)
            == F.unswizzle_scales(sf2.cpu().numpy(), 200, 5120)).all()
    out = torch.randn(64, 1024, generator=g).to(torch.bfloat16).to(dev)
    gate = torch.randn(64, 1024, generator=g).to(torch.bfloat16).to(dev)
    fp8, s = OPS.gate_fp8(out, gate)
    fp8b, sb = K.gate_fp8(out, gate)
    assert torch.equal(fp8.view(torch.uint8), fp8b) and torch.equal(s, sb)
    st = torch.tensor([0.02], device=dev)
    assert torch.equal(OPS.gate_fp8_static(out, gate, st).view(torch.uint8), K.gate_fp8_static(out, gate, st))
