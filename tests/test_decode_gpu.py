"""Bucket decode attention (``qi_decode_assign`` / ``qi_decode_attention``)
against the CPU oracle: the device plan equals the oracle planner (exact), the
output matches the oracle's blockwise evaluation within the bf16 output
rounding, the FP8 tail is bit-exact given the bf16 attention output, and
results are deterministic.  Runs through the C ABI."""

import math

import numpy as np
import pytest
import torch

from oracle import decode as OD
from oracle import formats as F
from oracle import model as OM

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0") if torch.cuda.is_available() else None


@pytest.fixture(scope="module")
def D():
    if DEV is None:
        pytest.skip("no CUDA device")
    from qwen_infra_b200 import decode

    return decode


def _cache(kvheads, pages, page_size, seed):
    from qwen_infra_b200.kernels import PagedKV

    g = np.random.default_rng(seed)
    kv = PagedKV(pages, page_size, kvheads, 128, DEV)
    shape = tuple(kv.k.shape)
    sshape = tuple(kv.ks.shape)
    for t in (kv.k, kv.v):
        t.copy_(torch.from_numpy(g.integers(0, 256, shape, dtype=np.uint8)))
    for t in (kv.ks, kv.vs):
        t.copy_(torch.from_numpy(F.e4m3_encode(g.uniform(0.02, 1.5, sshape).astype(np.float32))))
    return kv


def _oracle_kv(kv, table, lengths, page_size):
    """Per request: the exact e2m1 x e4m3 products [L, Hkv, 128] (globals 1)."""
    cache = OM.KVCache.__new__(OM.KVCache)
    cache.k, cache.v = kv.k.cpu().numpy(), kv.v.cpu().numpy()
    cache.ks, cache.vs = kv.ks.cpu().numpy(), kv.vs.cpu().numpy()

    class _Pages:
        pass

    shape = _Pages()
    shape.page_size = page_size
    pairs = [cache.gather(table[r], n, shape, 1.0, 1.0) for r, n in enumerate(lengths)]
    return [k for k, _ in pairs], [v for _, v in pairs]


def _setup(lengths, qheads, kvheads, seed, extra_width=2, page_size=16):
    width = max(1, max(math.ceil(n / page_size) for n in lengths)) + extra_width
    pages = len(lengths) * width + 3
    kv = _cache(kvheads, pages, page_size, seed)
    g = np.random.default_rng(seed + 1)
    table = g.permutation(pages)[: len(lengths) * width].reshape(len(lengths), width).astype(np.int32)
    q = (torch.randn(len(lengths), qheads, 128, generator=torch.Generator().manual_seed(seed + 2))).to(torch.bfloat16)
    return kv, table, q


def _run(D, lengths, qheads, kvheads, *, ctas, mode, seed=5, gate=None, out_scale=None, ws=None, setup=None):
    kv, table, q = setup or _setup(lengths, qheads, kvheads, seed)
    kg = torch.tensor([0.75], device=DEV)
    vg = torch.tensor([0.5], device=DEV)
    ws = ws or D.Workspace(len(lengths), qheads=qheads, kvheads=kvheads, ctas=ctas, device=DEV)
    ws.release_bindings()
    lt = torch.tensor(lengths, dtype=torch.int32, device=DEV)
    tt = torch.from_numpy(table).to(DEV)
    qd = q.to(DEV)
    ws.bind(qd, kv, tt, lt, k_global=kg, v_global=vg, cyclic=mode == "cyclic", aligned=mode == "aligned",
            persistent=mode == "persistent",
            gate=None if gate is None else gate.to(DEV),
            output_scale=None if out_scale is None else torch.tensor([out_scale], device=DEV))
    out = ws.run().clone()
    torch.cuda.synchronize()
    return out, ws, (kv, table, q)


def _check_plan(ws, lengths, ctas, mode, width):
    got = ws.inspect_plan()
    want = OD.task_plan(list(lengths), ctas=ctas, cyclic=mode == "cyclic", aligned=mode == "aligned",
                        table_width=width, page_size=16)
    assert got["tasks"] == want["tasks"]
    assert got["requests"] == want["requests"]
    assert got["header"] == want["header"]
    if mode != "cyclic":
        assert got["buckets"] == want["buckets"]
    return want


def _check_out(out, lengths, qheads, kvheads, setup, plan):
    kv, table, q = setup
    ks, vs = _oracle_kv(kv, table, lengths, 16)
    qf = q.float().numpy()
    ref = OD.decode_attention(qf, ks, vs, lengths, plan, softmax_scale=1 / math.sqrt(128), k_global=0.75,
                              v_global=0.5)
    got = out.float().cpu().numpy()
    scale = max(1e-6, float(np.abs(ref).max()))
    err = np.abs(got - ref)
    # bf16 output rounding (2^-9 relative) plus accumulation-order and ex2
    # approximation differences.
    assert (err <= 4e-3 * np.abs(ref) + 2e-3 * scale).all(), float(err.max())
    exact = OD.decode_attention_exact(qf, ks, vs, lengths, softmax_scale=1 / math.sqrt(128), k_global=0.75,
                                      v_global=0.5)
    assert np.abs(got - exact).max() <= 1.5e-2 * max(1e-6, float(np.abs(exact).max()))
    for r, n in enumerate(lengths):
        if n == 0:
            assert not got[r].any()


LENGTHS = [0, 1, 127, 128, 129, 256, 257, 3000]


@pytest.mark.parametrize("mode", ["intervals", "persistent", "cyclic", "aligned"])
@pytest.mark.parametrize("ctas", [8, 13, 40])
def test_decode_matches_oracle_all_modes(D, mode, ctas):
    qheads, kvheads = 16, 2
    setup = _setup(LENGTHS, qheads, kvheads, seed=11)
    out, ws, setup = _run(D, LENGTHS, qheads, kvheads, ctas=ctas, mode=mode, setup=setup)
    plan = _check_plan(ws, LENGTHS, ctas, "intervals" if mode == "persistent" else mode, setup[1].shape[1])
    _check_out(out, LENGTHS, qheads, kvheads, setup, plan)
    assert not ws.semaphores.any()
    assert int(ws.status.item()) == 0


@pytest.mark.parametrize("qheads,kvheads", [(8, 2), (32, 2), (24, 3), (64, 8)])
def test_decode_group_sizes(D, qheads, kvheads):
    lengths = [300, 1, 2500, 640]
    out, ws, setup = _run(D, lengths, qheads, kvheads, ctas=10, mode="cyclic", seed=21)
    plan = _check_plan(ws, lengths, 10, "cyclic", setup[1].shape[1])
    _check_out(out, lengths, qheads, kvheads, setup, plan)


def test_decode_27b_shape_long_context(D):
    """64 query heads over 8 KV heads, 4 requests x 8192 keys, default slots."""
    lengths = [8192, 8191, 4097, 8192]
    qheads, kvheads = 64, 8
    setup = _setup(lengths, qheads, kvheads, seed=31, extra_width=0)
    ws = D.Workspace(len(lengths), qheads=qheads, kvheads=kvheads, device=DEV)
    for mode in ("cyclic", "intervals"):
        out, ws, setup = _run(D, lengths, qheads, kvheads, ctas=ws.ctas, mode=mode, setup=setup, ws=ws)
        plan = _check_plan(ws, lengths, ws.ctas, mode, setup[1].shape[1])
        _check_out(out, lengths, qheads, kvheads, setup, plan)


def test_decode_deterministic_and_reusable(D):
    qheads, kvheads = 16, 2
    setup = _setup(LENGTHS, qheads, kvheads, seed=41)
    ws = D.Workspace(len(LENGTHS), qheads=qheads, kvheads=kvheads, ctas=13, device=DEV)
    outs = [_run(D, LENGTHS, qheads, kvheads, ctas=13, mode="intervals", setup=setup, ws=ws)[0] for _ in range(3)]
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    assert not ws.semaphores.any()


def test_decode_fp8_tail_bit_exact(D):
    """Gated FP8 output == e4m3(bf16(bf16(out) * bf16(sigmoid(gate))) / scale)
    of the bf16 output of the same plan."""
    qheads, kvheads = 16, 2
    setup = _setup(LENGTHS, qheads, kvheads, seed=51)
    gate = torch.randn(len(LENGTHS), qheads, 128, generator=torch.Generator().manual_seed(52)).to(torch.bfloat16) * 3
    plain, ws, _ = _run(D, LENGTHS, qheads, kvheads, ctas=13, mode="aligned", setup=setup)
    codes, _, _ = _run(D, LENGTHS, qheads, kvheads, ctas=13, mode="aligned", setup=setup, gate=gate,
                       out_scale=0.01)
    want = OD.fp8_tail(plain.float().cpu().numpy(), gate.float().numpy(), 0.01)
    got = codes.cpu().numpy()
    for r, n in enumerate(LENGTHS):
        if n == 0:
            assert not got[r].any()
        else:
            assert np.array_equal(got[r], want[r])


def test_decode_length_past_table_is_clamped_and_flagged(D):
    qheads, kvheads = 16, 2
    lengths = [100, 200]
    kv, table, q = _setup(lengths, qheads, kvheads, seed=61, extra_width=0)  # width 13 pages = 208 keys
    cap = table.shape[1] * 16
    out, ws, _ = _run(D, [100, cap + 500], qheads, kvheads, ctas=4, mode="intervals", setup=(kv, table, q))
    assert int(ws.status.item()) & 8
    ref, ws2, _ = _run(D, [100, cap], qheads, kvheads, ctas=4, mode="intervals", setup=(kv, table, q))
    assert torch.equal(out, ref)
    assert int(ws2.status.item()) == 0
