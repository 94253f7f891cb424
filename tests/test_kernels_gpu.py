"""Parity of every sm_100a kernel with the CPU oracle (bit-exact for quantised
bytes; stated tolerances for accumulations).  Runs through the C ABI."""

import math

import numpy as np
import pytest
import torch

from oracle import formats as F
from oracle import producers as P
from oracle import model as OM

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0") if torch.cuda.is_available() else None


@pytest.fixture(scope="module")
def K():
    if DEV is None:
        pytest.skip("no CUDA device")
    from qwen_infra_b200 import kernels

    return kernels


def _bf16(shape, seed, std=1.0, mean=0.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std + mean).to(torch.bfloat16)


def test_conversion_builtins_match_format_definitions(K):
    """E2M1 / E4M3 rounding, nibble order and expf / sigmoid of the device
    helpers against the CPU restatement, including ties and saturation."""
    from qwen_infra_b200 import _native as N
    import ctypes as ct

    grid = np.concatenate([
        np.array([0.0, -0.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 7.0, 100.0, -0.25, -0.3, -5.0, -1e9,
                  1e-9, -1e-9, 448.0, 464.0, 480.0, 1e6, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -10, 0.0136],
                 dtype=np.float32),
        np.random.default_rng(1).standard_normal(1 << 16).astype(np.float32) * 4,
        np.random.default_rng(2).standard_normal(1 << 12).astype(np.float32) * 200,
        np.linspace(-90, 90, 4096, dtype=np.float32),
    ])
    grid = grid[: len(grid) // 8 * 8]
    n = len(grid)
    x = torch.from_numpy(grid).to(DEV)
    e2 = torch.zeros(n, dtype=torch.uint8, device=DEV)
    e4 = torch.zeros(n, dtype=torch.uint8, device=DEV)
    ex = torch.zeros(2 * n, dtype=torch.float32, device=DEV)
    s = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert N.lib().qi_convert_probe(ct.c_void_p(x.data_ptr()), ct.c_void_p(e2.data_ptr()),
                                    ct.c_void_p(e4.data_ptr()), ct.c_void_p(ex.data_ptr()), n, s) == 0
    torch.cuda.synchronize()
    codes = F.e2m1_encode(grid)
    packed = F.pack_nibbles(codes)
    assert np.array_equal(e2.cpu().numpy()[: n // 2], packed)
    assert np.array_equal(e2.cpu().numpy()[n // 2:], packed)
    assert np.array_equal(e4.cpu().numpy(), F.e4m3_encode(grid))
    exv = ex.cpu().numpy().reshape(n, 2)
    # the product library's expf is CUDA's (same values as the oracle's helper
    # built with the reference's flags), and its sigmoid the reference's
    assert np.array_equal(exv[:, 0], P.MATH.exp(grid))
    assert np.array_equal(exv[:, 1], P.sigmoid_f(grid))
    # CUDA's expf: within 2 ulp of exp (the documented maximum ulp error)
    ref = np.exp(np.clip(grid, -80, 80).astype(np.float64))
    mask = np.abs(grid) < 80
    ulp = np.spacing(ref[mask].astype(np.float32)).astype(np.float64)
    assert np.all(np.abs(exv[mask, 0] - ref[mask]) <= 2 * ulp)


@pytest.mark.parametrize("rows,h,with_res", [(1, 1024, True), (17, 1024, False), (129, 1024, True),
                                             (2048, 5120, True), (300, 5120, False)])
def test_norm_pack_bit_exact(K, rows, h, with_res):
    x = _bf16((rows, h), 11)
    r = _bf16((rows, h), 12) if with_res else None
    w = _bf16((h,), 13, 0.05)
    gs = torch.tensor([84.0])
    q, sf, upd = K.norm_pack(x.to(DEV), None if r is None else r.to(DEV), w.to(DEV), gs.to(DEV))
    qo, sfo, updo = P.norm_pack(x.float().numpy(), None if r is None else r.float().numpy(), w.float().numpy(), 84.0)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), qo)
    got_sf = F.unswizzle_scales(sf.cpu().numpy(), rows, h)
    assert np.array_equal(got_sf, F.unswizzle_scales(sfo, rows, h))
    assert np.array_equal(upd.float().cpu().numpy(), updo)


def test_reference_norm_pack_abi_bit_exact(K):
    """The reference entry point nvfp4_norm_pack_launch (H = 5120)."""
    import ctypes as ct
    from qwen_infra_b200 import _native as N

    rows, h = 200, 5120
    x, r, w = _bf16((rows, h), 21), _bf16((rows, h), 22), _bf16((h,), 23, 0.05)
    xd, rd, wd = x.to(DEV), r.to(DEV), w.to(DEV)
    g = torch.tensor([60.0], device=DEV)
    q = torch.empty((rows, 2560), dtype=torch.uint8, device=DEV)
    sc = torch.zeros((((rows + 127) // 128) * 128, 80), dtype=torch.int32, device=DEV)
    upd = torch.empty_like(xd)
    ptr = lambda t: ct.c_void_p(t.data_ptr())
    st = N.lib().nvfp4_norm_pack_launch(ptr(xd), ptr(rd), ptr(wd), ptr(g), ptr(q), ptr(sc), ptr(upd), rows,
                                        ct.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    assert N.lib().nvfp4_norm_pack_launch(ptr(xd), ptr(rd), ptr(wd), ptr(g), ptr(q), ptr(sc), ptr(upd), 0,
                                          None) == 1
    torch.cuda.synchronize()
    qo, sfo, updo = P.norm_pack(x.float().numpy(), r.float().numpy(), w.float().numpy(), 60.0)
    assert np.array_equal(q.cpu().numpy(), qo)
    flat = sc.cpu().numpy().view(np.uint8).reshape(-1)
    assert np.array_equal(F.unswizzle_scales(flat, rows, h), F.unswizzle_scales(sfo, rows, h))
    for row, group in [(0, 0), (37, 319), (199, 123)]:
        assert flat[F.scale_offset(row, group, h)] == F.unswizzle_scales(sfo, rows, h)[row, group]


def _front_case(K, rows, qh, kvh, d, history, seed, page_size=16, slot_dtype=torch.int32):
    rng = np.random.default_rng(seed)
    width = (2 * qh + 2 * kvh) * d
    qkv = _bf16((rows, width), seed, 1.5)
    qw, kw = _bf16((d,), seed + 1, 0.05), _bf16((d,), seed + 2, 0.05)
    maxpos = history + rows
    cs = OM.rope_table(maxpos + 5, d, 1e6)
    pages = (maxpos + page_size - 1) // page_size + 3
    table = rng.permutation(pages)[: (maxpos + page_size - 1) // page_size].astype(np.int32)
    pos = np.arange(history, history + rows)
    slots = table[pos // page_size] * page_size + pos % page_size
    slots[rng.random(rows) < 0.1] = -1  # padding tokens are skipped
    kvc = K.PagedKV(pages, page_size, kvh, d, DEV)
    kvo = OM.KVCache(OM.Shape(1, qh * d, qh, kvh, d, 4 * d, page_size=page_size), pages)
    kg, vg = np.float32(16 / 2688), np.float32(8 / 2688)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    q, gate = K.qk_rope_kv_append(qkv.to(DEV), torch.from_numpy(pos.astype(np.int32)).to(DEV), qw.to(DEV),
                                  kw.to(DEV), torch.from_numpy(cs).to(DEV),
                                  torch.from_numpy(slots).to(slot_dtype).to(DEV), kvc,
                                  torch.tensor([kg], device=DEV), torch.tensor([vg], device=DEV), qheads=qh,
                                  kvheads=kvh, head_dim=d, status=status)
    qo, go = P.qk_rope_append(qkv.float().numpy(), pos, qw.float().numpy(), kw.float().numpy(), cs, slots, kg, vg,
                              kvo.k, kvo.v, kvo.ks, kvo.vs, qheads=qh, kvheads=kvh, head_dim=d,
                              page_size=page_size)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert np.array_equal(q.float().cpu().numpy(), qo)
    assert np.array_equal(gate.float().cpu().numpy(), go)
    for got, want in ((kvc.k, kvo.k), (kvc.v, kvo.v), (kvc.ks, kvo.ks), (kvc.vs, kvo.vs)):
        assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("rows,qh,kvh,d,history", [(64, 16, 4, 64, 0), (33, 16, 4, 64, 100),
                                                    (256, 64, 8, 128, 0), (77, 64, 8, 128, 2000),
                                                    (40, 6, 1, 256, 5)])
def test_qk_rope_kv_append_bit_exact(K, rows, qh, kvh, d, history):
    _front_case(K, rows, qh, kvh, d, history, seed=rows + d)


def test_qk_rope_kv_append_int64_slots_and_bad_scale_status(K):
    _front_case(K, 48, 16, 4, 64, 16, seed=5, slot_dtype=torch.int64)
    rows, qh, kvh, d = 8, 16, 4, 64
    qkv = _bf16((rows, (2 * qh + 2 * kvh) * d), 3).to(DEV)
    kvc = K.PagedKV(4, 16, kvh, d, DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    pos = torch.arange(rows, dtype=torch.int32, device=DEV)
    cs = torch.from_numpy(OM.rope_table(64, d, 1e6)).to(DEV)
    w = _bf16((d,), 4, 0.05).to(DEV)
    K.qk_rope_kv_append(qkv, pos, w, w, cs, pos.clone(), kvc, torch.tensor([float("nan")], device=DEV),
                        torch.tensor([1.0], device=DEV), qheads=qh, kvheads=kvh, head_dim=d, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 1
    assert int(kvc.k.count_nonzero().item()) == 0  # nothing appended with an invalid scale


def test_gate_fp8_bit_exact(K):
    rows, cols = 300, 8192
    out, gate = _bf16((rows, cols), 31), _bf16((rows, cols), 32, 2.0)
    out[5] = 0  # all-zero row: scale clamps to FLT_MIN, codes are zero
    fp8, scale = K.gate_fp8(out.to(DEV), gate.to(DEV))
    co, so = P.gate_fp8(out.float().numpy(), gate.float().numpy())
    torch.cuda.synchronize()
    assert np.array_equal(scale.cpu().numpy(), so)
    assert np.array_equal(fp8.cpu().numpy(), co)


def test_gate_fp8_reads_gate_in_place_from_qkv_rows(K):
    """The model path's gate operand: per head h the gate half of the QKV
    projection row ([q(D) | gate(D)] blocks, then K and V heads), read with a
    head stride of 2D; same bytes as the compact gate."""
    rows, heads, d, kvh = 260, 16, 128, 2
    qkv = _bf16((rows, (2 * heads + 2 * kvh) * d), 33, 2.0)
    out = _bf16((rows, heads * d), 34)
    gate = qkv[:, : 2 * heads * d].reshape(rows, heads, 2, d)[:, :, 1].reshape(rows, heads * d)
    qd = qkv.to(DEV)
    fp8, scale = K.gate_fp8(out.to(DEV), qd[:, d:], head_dim=d, head_stride=2 * d)
    co, so = P.gate_fp8(out.float().numpy(), gate.float().numpy())
    torch.cuda.synchronize()
    assert np.array_equal(scale.cpu().numpy(), so)
    assert np.array_equal(fp8.cpu().numpy(), co)


def test_gate_fp8_bit_exact_across_magnitudes(K):
    """Rows whose values span the bf16 range (tiny, huge, a single outlier,
    subnormal-sized), with a saturated gate so the FP8 quotients run over
    the divisor range."""
    rows, cols = 64, 8192
    g = torch.Generator().manual_seed(35)
    out = torch.randn(rows, cols, generator=g)
    mags = torch.logspace(-36, 36, rows, base=2.0)
    out = (out * mags[:, None]).to(torch.bfloat16)
    out[7, 100] = 3.0e38  # one outlier sets the row's scale
    out[9, :] = 1e-39  # subnormal-sized row
    gate = torch.full((rows, cols), 20.0, dtype=torch.bfloat16)
    gate[::2] = _bf16((rows // 2, cols), 36, 4.0)
    fp8, scale = K.gate_fp8(out.to(DEV), gate.to(DEV))
    co, so = P.gate_fp8(out.float().numpy(), gate.float().numpy())
    torch.cuda.synchronize()
    assert np.array_equal(scale.cpu().numpy(), so)
    assert np.array_equal(fp8.cpu().numpy(), co)


def test_weight_quantizers_bit_exact(K):
    w = torch.randn(512, 1024, generator=torch.Generator().manual_seed(41)) * 0.02
    qo, sfo, go = P.quantize_weight_nvfp4(w.numpy())
    q, sf = K.nvfp4_quantize(w.to(DEV), torch.tensor([go], device=DEV))
    c8o, s8o = P.quantize_weight_fp8_rows(w.numpy())
    c8, s8 = K.fp8_quantize_rows(w.to(DEV))
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(sf.cpu().numpy(), sfo)
    assert np.array_equal(c8.cpu().numpy(), c8o) and np.array_equal(s8.cpu().numpy(), s8o)


def _nvfp4_operand(rows, k, seed, std):
    w = (torch.randn(rows, k, generator=torch.Generator().manual_seed(seed)) * std).numpy()
    q, sf, g = P.quantize_weight_nvfp4(w)
    return q, sf, g, F.nvfp4_dequant(q, sf, rows, k, g)


@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (1, 256, 512), (200, 512, 1024), (2048, 1024, 5120),
                                   (513, 768, 3072)])
def test_nvfp4_gemm_matches_dequantised_product(K, m, n, k):
    aq, asf, ag, a = _nvfp4_operand(m, k, 51 + m, 1.0)
    bq, bsf, bg, b = _nvfp4_operand(n, k, 52 + n, 0.02)
    alpha = float(np.float32(1.0) / (np.float32(ag) * np.float32(bg)))
    t = lambda x: torch.from_numpy(x).to(DEV)
    # The MMA accumulates e2m1*e4m3 products; A.B^T of the dequantised values
    # is the same sum up to fp32 accumulation order -> tight tolerance.
    out32 = K.gemm_nvfp4(t(aq), t(asf), t(bq), t(bsf), m=m, n=n, k=k, alpha_value=alpha, out_dtype=torch.float32)
    out16 = K.gemm_nvfp4(t(aq), t(asf), t(bq), t(bsf), m=m, n=n, k=k, alpha=torch.tensor([alpha], device=DEV))
    ref = (torch.from_numpy(a).double() @ torch.from_numpy(b).double().T).numpy()
    torch.cuda.synchronize()
    scale = np.abs(ref).max()
    assert np.abs(out32.cpu().numpy() - ref).max() / scale < 2e-5
    assert np.abs(out16.float().cpu().numpy() - ref).max() / scale < 8e-3


@pytest.mark.parametrize("m,n,k", [(128, 256, 128), (77, 512, 1024), (2048, 5120, 8192)])
def test_e4m3_gemm_rowcol(K, m, n, k):
    g = torch.Generator().manual_seed(61)
    a = torch.randn(m, k, generator=g).numpy()
    b = (torch.randn(n, k, generator=g) * 0.02).numpy()
    ac, asc = P.quantize_weight_fp8_rows(a)
    bc, bsc = P.quantize_weight_fp8_rows(b)
    t = lambda x: torch.from_numpy(x).to(DEV)
    out = K.gemm_e4m3(t(ac), t(bc), m=m, n=n, k=k, row_scale=t(asc), col_scale=t(bsc))
    ref = (F.e4m3_decode(ac).astype(np.float64) * asc[:, None]) @ (F.e4m3_decode(bc).astype(np.float64) * bsc[:, None]).T
    torch.cuda.synchronize()
    assert np.abs(out.float().cpu().numpy() - ref).max() / np.abs(ref).max() < 8e-3


@pytest.mark.parametrize("m,inter,k", [(128, 128, 256), (300, 512, 1024)])
def test_swiglu_epilogue_bit_exact(K, m, inter, k):
    """The fused SiLU-and-mul -> NVFP4 epilogue reproduces the oracle exactly
    from the same fp32 accumulators (read back with the f32 epilogue)."""
    aq, asf, ag, _ = _nvfp4_operand(m, k, 71, 1.0)
    bq, bsf, bg, _ = _nvfp4_operand(2 * inter, k, 72, 0.05)
    alpha = float(np.float32(1.0) / (np.float32(ag) * np.float32(bg)))
    t = lambda x: torch.from_numpy(x).to(DEV)
    acc = K.gemm_nvfp4(t(aq), t(asf), t(bq), t(bsf), m=m, n=2 * inter, k=k, alpha_value=1.0,
                       out_dtype=torch.float32)
    act_q, act_sf = K.gemm_swiglu_nvfp4(t(aq), t(asf), t(bq), t(bsf), torch.tensor([42.0], device=DEV), m=m,
                                        n=2 * inter, k=k, alpha_value=alpha)
    torch.cuda.synchronize()
    accn = acc.cpu().numpy().reshape(m, inter // 128, 2, 128)
    g_acc = accn[:, :, 0, :].reshape(m, inter)
    u_acc = accn[:, :, 1, :].reshape(m, inter)
    qo, sfo, _ = P.swiglu_nvfp4(g_acc, u_acc, alpha, 42.0)
    assert np.array_equal(act_q.cpu().numpy(), qo)
    assert np.array_equal(F.unswizzle_scales(act_sf.cpu().numpy(), m, inter), F.unswizzle_scales(sfo, m, inter))


@pytest.mark.parametrize("rows,inter", [(1, 128), (300, 512), (2048, 1024)])
def test_swiglu_nvfp4_kernel_bit_exact(K, rows, inter):
    """qi_swiglu_nvfp4 on the bf16 gate_up GEMM output (128-column gate/up
    blocks) reproduces the oracle's SiLU-and-mul + NVFP4 exactly."""
    g = torch.Generator().manual_seed(91 + rows)
    gu = (torch.randn(rows, 2 * inter, generator=g) * 3).to(torch.bfloat16)
    gs = 37.5
    act_q, act_sf = K.swiglu_nvfp4(gu.to(DEV), torch.tensor([gs], device=DEV))
    torch.cuda.synchronize()
    blocks = gu.float().numpy().reshape(rows, inter // 128, 2, 128)
    gate = blocks[:, :, 0, :].reshape(rows, inter)
    up = blocks[:, :, 1, :].reshape(rows, inter)
    qo, sfo, _ = P.swiglu_nvfp4(gate, up, 1.0, gs)
    assert np.array_equal(act_q.cpu().numpy(), qo)
    assert np.array_equal(F.unswizzle_scales(act_sf.cpu().numpy(), rows, inter), F.unswizzle_scales(sfo, rows, inter))


@pytest.mark.parametrize("rows,dim,vocab", [(1, 1024, 4100), (4, 520, 3000), (8, 5120, 1024)])
def test_lm_head_argmax_bit_exact(K, rows, dim, vocab):
    """Logits and greedy tokens of qi_lm_head_argmax equal the oracle's bit for
    bit; a tie at the maximum goes to the lower index; two calls in a row agree
    (the workspace resets itself)."""
    g = torch.Generator().manual_seed(7 + rows)
    h = torch.randn(rows, dim, generator=g).to(torch.bfloat16)
    w = (torch.randn(vocab, dim, generator=g) * 0.05).to(torch.bfloat16)
    _, t0 = P.lm_head_argmax(h.float().numpy(), w.float().numpy())
    w[vocab - 1] = w[int(t0[0])]  # plant a tie with row 0's winner at the last index
    ref_logits, ref_tokens = P.lm_head_argmax(h.float().numpy(), w.float().numpy())
    assert ref_tokens[0] == t0[0]
    logits = torch.empty(rows, vocab, dtype=torch.float32, device=DEV)
    tok = K.lm_head_argmax(h.to(DEV), w.to(DEV), logits=logits)
    again = K.lm_head_argmax(h.to(DEV), w.to(DEV))
    torch.cuda.synchronize()
    assert np.array_equal(logits.cpu().numpy(), ref_logits)
    assert tok.cpu().tolist() == ref_tokens.tolist() == again.cpu().tolist()


def _kv_fixture(K, tokens, kvh, d, seed, page_size=16):
    rng = np.random.default_rng(seed)
    pages = (tokens + page_size - 1) // page_size + 5
    kvc = K.PagedKV(pages, page_size, kvh, d, DEV)
    for t in (kvc.k, kvc.v):
        t.copy_(torch.from_numpy(rng.integers(0, 256, t.shape, dtype=np.uint8)))
    for t in (kvc.ks, kvc.vs):  # positive finite E4M3 scales 2^-4 .. 2^4
        t.copy_(torch.from_numpy(rng.integers(0x18, 0x58, t.shape, dtype=np.uint8)))
    table = rng.permutation(pages)[: (tokens + page_size - 1) // page_size].astype(np.int32)
    return kvc, table


@pytest.mark.parametrize("tokens,d", [(1, 64), (200, 64), (1000, 128), (4096, 128)])
def test_kv_dequant_exact(K, tokens, d):
    kvh = 4 if d == 64 else 8
    kvc, table = _kv_fixture(K, tokens, kvh, d, tokens)
    kd, vt = K.kv_dequant(kvc, torch.from_numpy(table).to(DEV), tokens)
    torch.cuda.synchronize()
    shape = OM.Shape(1, 8 * d, 8, kvh, d, 4 * d)
    cache = OM.KVCache(shape, kvc.pages)
    cache.k, cache.v, cache.ks, cache.vs = (t.cpu().numpy() for t in (kvc.k, kvc.v, kvc.ks, kvc.vs))
    k_ref, v_ref = cache.gather(table, tokens, shape, 1.0, 1.0)  # [T, Hkv, D]
    assert np.array_equal(kd.float().cpu().numpy(), k_ref.transpose(1, 0, 2))
    assert np.array_equal(vt.float().cpu().numpy()[:, :, :tokens], v_ref.transpose(1, 2, 0))


def test_kv_dequant_range_by_chunks_equals_whole_history(K):
    """Chunks of 700 tokens dequantised one after another into buffers sized
    for the whole request equal the whole-history dequantisation; tokens past
    the current length stay zero."""
    tokens, kvh, d, cap = 2500, 8, 128, 2600
    kvc, table = _kv_fixture(K, tokens, kvh, d, tokens)
    tt = torch.from_numpy(table).to(DEV)
    full_k, full_vt = K.kv_dequant(kvc, tt, tokens)
    kd = torch.zeros(kvh, cap, d, dtype=torch.float16, device=DEV)
    vt = torch.zeros(kvh, d, (cap + 63) // 64 * 64, dtype=torch.float16, device=DEV)
    for end in (700, 1400, 2100, 2500):
        hist = end - 700 if end != 2500 else 2100
        K.kv_dequant(kvc, tt, end, first=hist // 64 * 64, k_out=kd, vt_out=vt)
        torch.cuda.synchronize()
        assert torch.equal(kd[:, :end], full_k[:, :end])
        assert torch.equal(vt[:, :, :end], full_vt[:, :, :end])
        assert not kd[:, end:].any() and not vt[:, :, end:].any()


@pytest.mark.parametrize("split", [True, False])
@pytest.mark.parametrize("rows,history,qh,kvh,d", [(128, 0, 16, 4, 64), (200, 300, 16, 4, 64),
                                                   (512, 0, 64, 8, 128), (77, 1500, 64, 8, 128),
                                                   (1, 4000, 64, 8, 128), (2048, 1024, 64, 8, 128)])
def test_prefill_attention_matches_fp32(K, rows, history, qh, kvh, d, split):
    """split=True: the default workspace, so units of the last partly idle
    wave (or all units, when there are fewer than SMs) run as two key-range
    halves combined in the kernel; split=False: no workspace, no split."""
    tokens = history + rows
    g = torch.Generator().manual_seed(81 + rows)
    q = (torch.randn(rows, qh * d, generator=g)).to(torch.bfloat16)
    # K/V held as exact f16 values; the global multipliers are folded in.
    k = (torch.randn(kvh, tokens, d, generator=g) * 64).to(torch.float16)
    v = (torch.randn(kvh, tokens, d, generator=g) * 64).to(torch.float16)
    vt_row = (tokens + 63) // 64 * 64
    vt = torch.zeros(kvh, d, vt_row, dtype=torch.float16)
    vt[:, :, :tokens] = v.transpose(1, 2)
    kg, vg = 1.0 / 64, 1.0 / 64
    ws = None if split else torch.empty(0, dtype=torch.uint8, device=DEV)
    args = dict(history=history, qheads=qh, kvheads=kvh, head_dim=d, k_global=torch.tensor([kg], device=DEV),
                v_global=torch.tensor([vg], device=DEV), workspace=ws)
    out = K.prefill_attention(q.to(DEV), k.to(DEV), vt.to(DEV), **args)
    again = K.prefill_attention(q.to(DEV), k.to(DEV), vt.to(DEV), **args)
    assert torch.equal(out, again)  # the split's arrival counters reset themselves
    ref = OM.attention(q.float().numpy(), (k.float() * kg).transpose(0, 1).contiguous().numpy(),
                       (v.float() * vg).transpose(0, 1).contiguous().numpy(), history,
                       OM.Shape(1, qh * d, qh, kvh, d, 4 * d))
    torch.cuda.synchronize()
    err = np.abs(out.float().cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err < 2e-2, err
