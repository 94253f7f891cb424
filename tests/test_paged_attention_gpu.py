"""Prefill attention straight over the paged NVFP4 cache
(qi_paged_prefill_attention): the kernel's producer warps load E2M1 codes and
E4M3 scales through the block table and convert them in shared memory.

Checked against (a) the two-step f16 path (qi_kv_dequant + qi_prefill_attention,
the same tcgen05 math on the same exact f16 values) and (b) a plain fp32 torch
softmax attention over the dequantised cache (TF32 off) within 2e-2 of the
largest output -- the attention tolerance of the other parity tests -- up to
2048 rows over 30,720 keys of history, with the key-range split on and off."""

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0") if torch.cuda.is_available() else None


@pytest.fixture(scope="module")
def K():
    if DEV is None:
        pytest.skip("no CUDA device")
    from qwen_infra_b200 import kernels

    return kernels


def _cache(K, tokens, kvh, d, page_size, seed):
    """Random NVFP4 cache over a shuffled block table (+3 unused pages)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    n_pages = (tokens + page_size - 1) // page_size
    pages = n_pages + 3
    kv = K.PagedKV(pages, page_size, kvh, d, DEV)
    for t in (kv.k, kv.v):
        t.copy_(torch.randint(0, 256, t.shape, generator=g, dtype=torch.int32).to(torch.uint8))
    for t in (kv.ks, kv.vs):
        t.copy_(torch.randint(0x18, 0x58, t.shape, generator=g, dtype=torch.int32).to(torch.uint8))
    table = torch.randperm(pages, generator=g)[:n_pages].to(torch.int32).to(DEV)
    return kv, table


def _fp32_reference(q, k, v, history, qheads, heads, kg, vg):
    """softmax(q k^T / sqrt(D)) v in fp32 on the GPU for the listed heads;
    k, v: f16 [Hkv, T, D] exact cache values (multipliers applied here)."""
    rows, d = q.shape[0], k.shape[2]
    group = qheads // k.shape[0]
    qpos = torch.arange(rows, device=DEV)[:, None] + history
    kpos = torch.arange(k.shape[1], device=DEV)[None, :]
    out = {}
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for h in heads:
            qh = q[:, h * d:(h + 1) * d].float()
            kh = k[h // group].float() * kg
            vh = v[h // group].float() * vg
            s = (qh @ kh.T) / math.sqrt(d)
            s = s.masked_fill(kpos > qpos, float("-inf"))
            out[h] = torch.softmax(s, dim=-1) @ vh
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return out


def _run(K, rows, history, qh, kvh, d, page_size, split, seed, heads=None):
    tokens = history + rows
    kv, table = _cache(K, tokens, kvh, d, page_size, seed)
    g = torch.Generator(device="cpu").manual_seed(seed + 1)
    q = torch.randn(rows, qh * d, generator=g).to(torch.bfloat16).to(DEV)
    kg, vg = torch.tensor([1 / 64], device=DEV), torch.tensor([1 / 32], device=DEV)
    ws = None if split else torch.empty(0, dtype=torch.uint8, device=DEV)
    out = K.paged_prefill_attention(q, kv, table, history=history, qheads=qh, k_global=kg, v_global=vg,
                                    workspace=ws)
    again = K.paged_prefill_attention(q, kv, table, history=history, qheads=qh, k_global=kg, v_global=vg,
                                      workspace=ws)
    kd, vt = K.kv_dequant(kv, table, tokens)
    two_step = K.prefill_attention(q, kd, vt, history=history, qheads=qh, kvheads=kvh, head_dim=d,
                                   k_global=kg, v_global=vg, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(out, again)
    scale = two_step.float().abs().max().item()
    assert (out.float() - two_step.float()).abs().max().item() <= 1e-3 * scale
    heads = heads or list(range(qh))
    v = vt[:, :, :tokens].transpose(1, 2)
    ref = _fp32_reference(q, kd, v, history, qh, heads, 1 / 64, 1 / 32)
    rmax = max(r.abs().max().item() for r in ref.values())
    err = max((out[:, h * d:(h + 1) * d].float() - ref[h]).abs().max().item() for h in heads) / rmax
    assert err < 2e-2, err
    return out


@pytest.mark.parametrize("split", [True, False])
@pytest.mark.parametrize("rows,history,qh,kvh,d,page", [(128, 0, 16, 4, 64, 16), (200, 300, 16, 4, 64, 32),
                                                        (512, 0, 64, 8, 128, 16), (77, 1500, 64, 8, 128, 16),
                                                        (1, 4000, 64, 8, 128, 32), (2048, 1024, 64, 8, 128, 16),
                                                        (300, 333, 8, 1, 128, 16)])
def test_paged_attention_matches_two_step_and_fp32(K, rows, history, qh, kvh, d, page, split):
    _run(K, rows, history, qh, kvh, d, page, split, seed=rows + history)


@pytest.mark.parametrize("split", [True, False])
@pytest.mark.parametrize("history", [8192, 30720])
def test_paged_attention_long_history(K, history, split):
    """2048 rows (one chunk of the 27B bank) over 8192 / 30720 keys of history:
    every unit of the bank's longest launches, with and without the split of
    the last partial wave; the fp32 reference on a sample of 6 heads."""
    _run(K, 2048, history, 64, 8, 128, 16, split, seed=history + int(split), heads=[0, 7, 8, 31, 56, 63])


def test_paged_attention_rejects_bad_requests(K):
    from qwen_infra_b200 import _native as N
    import ctypes as ct

    kv, table = _cache(K, 64, 8, 128, 16, 5)
    q = torch.zeros(64, 64 * 128, dtype=torch.bfloat16, device=DEV)
    out = torch.empty_like(q)
    kg = torch.tensor([1.0], device=DEV)
    base = dict(q=q.data_ptr(), out=out.data_ptr(), kv=kv.view(), block_table=table.data_ptr(),
                k_global=kg.data_ptr(), v_global=kg.data_ptr(), rows=64, history=0, qheads=64,
                q_row=q.stride(0), out_row=out.stride(0), softmax_scale=0.1)
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call(**over):
        p = N.QiPagedAttention()
        for k_, v_ in dict(base, **over).items():
            setattr(p, k_, v_)
        return N.lib().qi_paged_prefill_attention(ct.byref(p), stream)

    assert call() == 0
    bad_view = kv.view()
    bad_view.page_size = 24  # not a power of two
    assert call(kv=bad_view) == 1
    assert call(qheads=60) == 1  # not a multiple of the KV heads
    assert call(q_row=100) == 1  # row stride below Hq * D
    assert call(block_table=None) == 1
    torch.cuda.synchronize()
