"""Producer bytes pinned to the reference's own kernels.

The reference's ``nvfp4_norm_pack.cu`` and ``nvfp4_attention_front.cu`` are
compiled from its sources for sm_100a with its own flags (``oracle/build_ref.py``
-> ``oracle/_ref/``) and run here on the same inputs as this repository's
kernels; every output byte must agree.  The gate epilogue, which in the
reference lives inside its sm_120 decode kernel, is compared with a
restatement of its lines (``oracle/gpu_checks.cu``, built with the same
flags) over every bf16 gate value.  The CPU oracle is held to the same bytes.
"""

import ctypes as ct
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import cuda_math
from oracle import formats as F
from oracle import model as OM
from oracle import producers as P

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"
DEV = torch.device("cuda:0") if torch.cuda.is_available() else None


def _ref_lib(name):
    path = REF / name
    if DEV is None:
        pytest.skip("no CUDA device")
    if not path.exists():
        pytest.skip(f"{path.name} not built (oracle/build_ref.py needs the reference checkout)")
    return ct.CDLL(str(path))


def _ptr(t):
    return ct.c_void_p(t.data_ptr())


def _stream():
    return ct.c_void_p(torch.cuda.current_stream().cuda_stream)


def _bf16(shape, seed, std=1.0, mean=0.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std + mean).to(torch.bfloat16)


def run_norm_pack(lib, x, r, w, g, rows):
    """Call nvfp4_norm_pack_launch (reference ABI) of ``lib`` on device inputs."""
    dev = x.device
    q = torch.zeros((rows, 2560), dtype=torch.uint8, device=dev)
    sc = torch.zeros((((rows + 127) // 128) * 128 * 320,), dtype=torch.uint8, device=dev)
    upd = torch.zeros_like(x)
    fn = lib.nvfp4_norm_pack_launch
    fn.argtypes = [ct.c_void_p] * 7 + [ct.c_int, ct.c_void_p]
    fn.restype = ct.c_int
    assert fn(_ptr(x), _ptr(r), _ptr(w), _ptr(g), _ptr(q), _ptr(sc), _ptr(upd), rows, _stream()) == 0
    torch.cuda.synchronize()
    return q, sc, upd


@pytest.mark.parametrize("rows,std", [(1, 1.0), (127, 1.0), (2048, 1.0), (300, 30.0), (64, 1e-3)])
def test_norm_pack_bytes_equal_the_reference_kernel(rows, std):
    """Config 2's norm-pack (H 5120, up to 2048 rows): the reference kernel,
    this repository's reference-ABI entry point, qi_norm_pack and the CPU
    oracle give the same codes, scales and updated residual."""
    ref = _ref_lib("libref_norm_pack.so")
    from qwen_infra_b200 import _native as N
    from qwen_infra_b200 import kernels as K

    h = 5120
    x, r = _bf16((rows, h), 100 + rows, std), _bf16((rows, h), 200 + rows, std)
    w = _bf16((h,), 300, 0.05)
    xd, rd, wd = x.to(DEV), r.to(DEV), w.to(DEV)
    g = torch.tensor([2688.0 / (4.0 * std)], device=DEV)
    want = run_norm_pack(ref, xd, rd, wd, g, rows)
    ours = run_norm_pack(N.lib(), xd, rd, wd, g, rows)
    for a, b in zip(want, ours):
        assert torch.equal(a, b)
    q, sf, upd = K.norm_pack(xd, rd, wd, g)
    torch.cuda.synchronize()
    assert torch.equal(q, want[0])
    # the scale rows past `rows` in the last 128-row block are padding
    assert np.array_equal(F.unswizzle_scales(sf.cpu().numpy(), rows, h),
                          F.unswizzle_scales(want[1].cpu().numpy(), rows, h))
    assert torch.equal(upd, want[2])
    qo, sfo, updo = P.norm_pack(x.float().numpy(), r.float().numpy(), w.float().numpy(), float(g.item()))
    assert np.array_equal(qo, want[0].cpu().numpy())
    assert np.array_equal(sfo, want[1].cpu().numpy())
    assert np.array_equal(updo, want[2].float().cpu().numpy())


def _front_inputs(rows, qh, kvh, page_size, seed, cos_float, pos_long, slot_long):
    rng = np.random.default_rng(seed)
    d = 256
    qkv = _bf16((rows, (2 * qh + 2 * kvh) * d), seed, 1.5)
    qw, kw = _bf16((d,), seed + 1, 0.05), _bf16((d,), seed + 2, 0.05)
    history = int(rng.integers(0, 3000))
    maxpos = history + rows
    cs = OM.rope_table(maxpos + 3, d, 1e6)
    pages = (maxpos + page_size - 1) // page_size + 2
    table = rng.permutation(pages)[: (maxpos + page_size - 1) // page_size]
    pos = np.arange(history, history + rows)
    slots = (table[pos // page_size] * page_size + pos % page_size).astype(np.int64)
    slots[rng.random(rows) < 0.1] = -1                       # padding token: skipped
    slots[rng.random(rows) < 0.05] = pages * page_size + 7   # past the cache: skipped
    cos_t = torch.from_numpy(cs).to(DEV)
    if not cos_float:
        cos_t = cos_t.to(torch.bfloat16)
    return dict(qkv=qkv.to(DEV), qw=qw.to(DEV), kw=kw.to(DEV), cos=cos_t,
                pos=torch.from_numpy(pos).to(torch.int64 if pos_long else torch.int32).to(DEV),
                slots=torch.from_numpy(slots).to(torch.int64 if slot_long else torch.int32).to(DEV),
                pages=pages, page_size=page_size, rows=rows, qh=qh, kvh=kvh, np_slots=slots, np_pos=pos,
                np_cos=cos_t.float().cpu().numpy(), kg=torch.tensor([16 / 2688], device=DEV),
                vg=torch.tensor([8 / 2688], device=DEV), slot_rows=rows - 3)


def run_front(lib, a):
    """Call nvfp4_attention_front (reference ABI: RefFront by value) of ``lib``."""
    from qwen_infra_b200 import _native as N

    dev = a["qkv"].device
    rows, qh, kvh, ps = a["rows"], a["qh"], a["kvh"], a["page_size"]
    k = torch.zeros((a["pages"], ps, kvh, 128), dtype=torch.uint8, device=dev)
    v = torch.zeros_like(k)
    ks = torch.zeros((a["pages"], ps, kvh, 16), dtype=torch.uint8, device=dev)
    vs = torch.zeros_like(ks)
    q = torch.zeros((rows, qh * 256), dtype=torch.bfloat16, device=dev)
    gate = torch.zeros_like(q)
    f = N.RefFront(_ptr(a["qkv"]), _ptr(a["qw"]), _ptr(a["kw"]), _ptr(a["cos"]), _ptr(a["pos"]), _ptr(a["slots"]),
                   _ptr(a["kg"]), _ptr(a["vg"]), _ptr(k), _ptr(v), _ptr(ks), _ptr(vs), _ptr(q), _ptr(gate),
                   rows, qh, kvh, 256, a["slot_rows"], a["pages"], ps,
                   int(a["cos"].dtype == torch.float32), int(a["pos"].dtype == torch.int64),
                   int(a["slots"].dtype == torch.int64), 0, 0,
                   a["qkv"].stride(0), a["cos"].stride(0), 0, 1,
                   k.stride(0), k.stride(1), k.stride(2), ks.stride(0), ks.stride(1), ks.stride(2), 1e-6)
    fn = lib.nvfp4_attention_front
    fn.argtypes = [N.RefFront, ct.c_void_p]
    fn.restype = ct.c_int
    assert fn(f, _stream()) == 0
    torch.cuda.synchronize()
    return dict(q=q, gate=gate, k=k, v=v, ks=ks, vs=vs)


@pytest.mark.parametrize("rows,qh,kvh,cos_float,pos_long,slot_long",
                         [(150, 4, 1, True, True, True), (64, 6, 2, False, False, False),
                          (257, 8, 2, True, False, True)])
def test_attention_front_bytes_equal_the_reference_kernel(rows, qh, kvh, cos_float, pos_long, slot_long):
    """D 256, page 32 (the reference's ABI): q, gate, K/V codes and scales of
    the reference kernel, of this repository's nvfp4_attention_front and of
    the CPU oracle are the same bytes; padding slots, slots past the cache and
    rows past slot_rows append nothing."""
    ref = _ref_lib("libref_attention_front.so")
    from qwen_infra_b200 import _native as N

    sizes = (ct.c_int * 5)()
    ref.nvfp4_attention_front_resources.argtypes = [ct.POINTER(ct.c_int)]
    assert ref.nvfp4_attention_front_resources(sizes) == 0 and sizes[0] == ct.sizeof(N.RefFront)
    a = _front_inputs(rows, qh, kvh, 32, rows + qh, cos_float, pos_long, slot_long)
    want = run_front(ref, a)
    ours = run_front(N.lib(), a)
    for name in want:
        assert torch.equal(want[name], ours[name]), name
    kvo = OM.KVCache(OM.Shape(1, qh * 256, qh, kvh, 256, 1024, page_size=32), a["pages"])
    slots = a["np_slots"].copy()
    slots[a["slot_rows"]:] = -1
    qo, go = P.qk_rope_append(a["qkv"].float().cpu().numpy(), a["np_pos"], a["qw"].float().cpu().numpy(),
                              a["kw"].float().cpu().numpy(), a["np_cos"], slots, np.float32(16 / 2688),
                              np.float32(8 / 2688), kvo.k, kvo.v, kvo.ks, kvo.vs, qheads=qh, kvheads=kvh,
                              head_dim=256, page_size=32)
    assert np.array_equal(qo, want["q"].float().cpu().numpy())
    assert np.array_equal(go, want["gate"].float().cpu().numpy())
    for got, name in ((kvo.k, "k"), (kvo.v, "v"), (kvo.ks, "ks"), (kvo.vs, "vs")):
        assert np.array_equal(got, want[name].cpu().numpy()), name


def test_gate_fp8_static_equals_the_reference_epilogue_on_every_gate_value():
    """qi_gate_fp8_static against the reference's store_final_fp8 arithmetic
    (nvfp4_bucket_xqa.cu:56-62, restated in oracle/gpu_checks.cu and built
    with the reference's flags) over all 65536 bf16 gate bit patterns, each
    with several attention-output values; and the CPU oracle on the same."""
    _ref_lib("libqo_gpu_checks.so")
    from qwen_infra_b200 import _native as N

    gates = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    gate = gates.repeat(4).reshape(-1, 256)
    rows, cols = gate.shape
    vals = _bf16((rows, cols), 7, 3.0)
    gd, vd = gate.to(DEV), vals.to(DEV)
    scale = torch.tensor([0.0123], device=DEV)
    want = cuda_math.gate_fp8_static_reference(vd, gd, scale)
    got = torch.zeros((rows, cols), dtype=torch.uint8, device=DEV)
    rc = N.lib().qi_gate_fp8_static(_ptr(vd), _ptr(gd), cols, cols, 0, cols, _ptr(got), cols, _ptr(scale), rows,
                                    cols, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    co, _ = P.gate_fp8(vals.float().numpy(), gate.float().numpy(), static_scale=np.float32(0.0123))
    assert np.array_equal(co, want.cpu().numpy())


def test_cuda_math_helper_matches_the_product_library():
    """The oracle's expf helper and the product library's compiled expf
    agree; rsqrtf stays within its documented 2-ulp bound."""
    from qwen_infra_b200 import _native as N

    _ref_lib("libqo_gpu_checks.so")
    grid = np.concatenate([np.linspace(-90, 90, 8192, dtype=np.float32),
                           np.random.default_rng(4).standard_normal(8192).astype(np.float32)])
    n = len(grid)
    x = torch.from_numpy(grid).to(DEV)
    e2 = torch.zeros(n, dtype=torch.uint8, device=DEV)
    e4 = torch.zeros(n, dtype=torch.uint8, device=DEV)
    ex = torch.zeros(2 * n, dtype=torch.float32, device=DEV)
    assert N.lib().qi_convert_probe(_ptr(x), _ptr(e2), _ptr(e4), _ptr(ex), n, _stream()) == 0
    torch.cuda.synchronize()
    assert np.array_equal(ex.cpu().numpy().reshape(n, 2)[:, 0], cuda_math.CudaMath().exp(grid))
    pos = np.abs(grid) + np.float32(1e-3)
    r = cuda_math.CudaMath().rsqrt(pos)
    assert np.all(np.abs(r.astype(np.float64) * np.sqrt(pos.astype(np.float64)) - 1) < 2 ** -21)
