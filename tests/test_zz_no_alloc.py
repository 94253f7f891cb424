"""The allocation-free paged attention entry point (for callers that cannot
allocate device memory: allocator callbacks, plugin hosts that only provide
inputs and outputs) must return what the regular
two-call path returns.  Called through the C ABI twice in a row with different
shapes, since every call reuses the same static scratch array.  Collected last
on purpose (file name), so a failure here comes after every other test ran."""

import ctypes as ct
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _entry():
    from qwen_infra_b200 import _native as N

    fn = N.lib().qi_paged_prefill_attention_noalloc
    fn.argtypes = [ct.POINTER(N.QiKvView), ct.c_void_p, ct.c_void_p, ct.c_int64, ct.c_void_p, ct.c_int64, ct.c_int,
                   ct.c_int, ct.c_int, ct.c_void_p, ct.c_void_p, ct.c_float, ct.c_void_p, ct.c_void_p]
    fn.restype = ct.c_int
    return fn


def _case(K, dev, rows, history, qh, kvh, d, seed):
    rng = np.random.default_rng(seed)
    tokens = history + rows
    pages = (tokens + 15) // 16 + 3
    kv = K.PagedKV(pages, 16, kvh, d, dev)
    for t in (kv.k, kv.v):
        t.copy_(torch.from_numpy(rng.integers(0, 256, t.shape, dtype=np.uint8)))
    for t in (kv.ks, kv.vs):
        t.copy_(torch.from_numpy(rng.integers(0x18, 0x58, t.shape, dtype=np.uint8)))
    table = torch.from_numpy(rng.permutation(pages)[: (tokens + 15) // 16].astype(np.int32)).to(dev)
    q = torch.from_numpy(rng.standard_normal((rows, qh * d)).astype(np.float32)).to(torch.bfloat16).to(dev)
    kg = torch.tensor([1 / 64], device=dev)
    vg = torch.tensor([1 / 32], device=dev)
    return kv, table, q, kg, vg


@pytest.mark.parametrize("first,second", [((300, 700, 16, 4, 64), (128, 0, 64, 8, 128)),
                                          ((77, 1500, 64, 8, 128), (512, 3000, 16, 4, 64))])
def test_noalloc_attention_matches_two_call_path_twice(first, second):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwen_infra_b200 import kernels as K

    dev = torch.device("cuda:0")
    fn = _entry()
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    for i, (rows, history, qh, kvh, d) in enumerate((first, second)):
        kv, table, q, kg, vg = _case(K, dev, rows, history, qh, kvh, d, seed=11 + i)
        kd, vt = K.kv_dequant(kv, table, history + rows)
        want = K.prefill_attention(q, kd, vt, history=history, qheads=qh, kvheads=kvh, head_dim=d, k_global=kg,
                                   v_global=vg)
        got = torch.full_like(want, float("nan"))
        view = kv.view()
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(dev)[0]
        rc = fn(ct.byref(view), ct.c_void_p(table.data_ptr()), ct.c_void_p(q.data_ptr()), q.stride(0),
                ct.c_void_p(got.data_ptr()), got.stride(0), rows, history, qh, ct.c_void_p(kg.data_ptr()),
                ct.c_void_p(vg.data_ptr()), 1.0 / math.sqrt(d), None, stream)
        assert rc == 0
        torch.cuda.synchronize()
        if i == 1:
            # the kernels' code is resident after the first call, so a call
            # that allocates nothing leaves the device's free memory as it was
            assert torch.cuda.mem_get_info(dev)[0] == free_before
        err = (got.float() - want.float()).abs().max().item() / want.float().abs().max().item()
        assert err < 2e-2, err  # the tolerance of the attention parity tests
        assert torch.equal(got, want)  # same kernels on the same values: identical in fact


def test_noalloc_rejects_requests_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwen_infra_b200 import kernels as K

    dev = torch.device("cuda:0")
    fn = _entry()
    kv, table, q, kg, vg = _case(K, dev, 64, 0, 64, 8, 128, seed=3)
    out = torch.empty((64, 64 * 128), dtype=torch.bfloat16, device=dev)
    view = kv.view()
    # 8 KV heads of 128: 4 KiB per token; 9000 tokens exceed the 32 MiB array.
    rc = fn(ct.byref(view), ct.c_void_p(table.data_ptr()), ct.c_void_p(q.data_ptr()), q.stride(0),
            ct.c_void_p(out.data_ptr()), out.stride(0), 64, 9000 - 64, 64, ct.c_void_p(kg.data_ptr()),
            ct.c_void_p(vg.data_ptr()), 1.0 / math.sqrt(128), None, ct.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 1  # cudaErrorInvalidValue, nothing launched
