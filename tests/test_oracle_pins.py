"""The CPU oracle pinned against the reference's own outputs and the format
definitions (no GPU).  Fixtures under tests/golden/ were recorded from the
reference project by tests/golden/make_golden.py."""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import formats as F
from oracle import producers as P

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_scale_offset_matches_reference_scale_offset():
    """oracle.formats.scale_offset at K = 5120 equals the reference's
    kernels/nvfp4_norm_pack.py:12-15 on recorded coordinates."""
    for row, group, off in json.loads((GOLDEN / "scale_offset.json").read_text()):
        assert int(F.scale_offset(row, group, 5120)) == off


def test_scale_layout_is_a_bijection():
    for rows, k in ((1, 64), (129, 1024), (300, 5120), (256, 17408)):
        groups = k // 16
        r = np.repeat(np.arange(rows), groups)
        g = np.tile(np.arange(groups), rows)
        offs = F.scale_offset(r, g, k)
        assert len(np.unique(offs)) == offs.size
        assert offs.max() < F.scale_buffer_bytes(rows, k)


def test_e4m3_encoder_matches_torch_float8():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200000).astype(np.float32) * s for s in (1e-3, 0.1, 3, 60, 300)])
    x = np.concatenate([x, F.E4M3_VALUES.astype(np.float32), -F.E4M3_VALUES.astype(np.float32)])
    x = np.clip(x, -448, 448)
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(F.e4m3_encode(x), want)
    # saturation (satfinite) above 448 instead of NaN
    assert np.all(F.e4m3_encode(np.array([500, 1e9, -1e9], np.float32)) == np.array([0x7E, 0x7E, 0xFE]))


def test_e4m3_roundtrip_of_every_code():
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], dtype=np.uint8)
    assert np.array_equal(F.e4m3_encode(F.e4m3_decode(codes)), codes)


def test_e2m1_threshold_encoder_equals_grid_rounding():
    grid = np.concatenate([np.linspace(-8, 8, 200001, dtype=np.float32),
                           np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.0, 0.0], np.float32)])
    assert np.array_equal(F.e2m1_encode(grid), F.e2m1_encode_grid(grid))
    # ties to even mantissa, saturation at 6
    assert list(F.e2m1_encode(np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 9.0], np.float32))) == \
        [0, 2, 2, 4, 4, 6, 6, 7]


def test_nibble_order_low_first():
    packed = F.pack_nibbles(np.array([[1, 2, 3, 4]], np.uint8))
    assert list(packed[0]) == [0x21, 0x43]
    assert np.array_equal(F.unpack_nibbles(packed), [[1, 2, 3, 4]])


def test_bf16_round_matches_torch():
    x = np.random.default_rng(1).standard_normal(100000).astype(np.float32) * 100
    assert np.array_equal(F.bf16_round(x), torch.from_numpy(x).to(torch.bfloat16).float().numpy())


def test_nvfp4_quant_dequant_error_bound():
    w = np.random.default_rng(2).standard_normal((64, 256)).astype(np.float32)
    q, sf, g = P.quantize_weight_nvfp4(w)
    back = F.nvfp4_dequant(q, sf, 64, 256, g)
    blk = np.abs(w).reshape(64, 16, 16).max(-1)
    # half a step of the coarsest e2m1 interval (6-4 = 2 units of amax/6) plus scale rounding
    assert np.all(np.abs(back - w).reshape(64, 16, 16).max(-1) <= blk * (1 / 6 + 1 / 16) + 1e-6)


def test_host_math_and_sigmoid_range():
    x = np.linspace(-80, 80, 100001, dtype=np.float32)
    assert np.array_equal(P.HostMath().exp(x), np.exp(x.astype(np.float64)).astype(np.float32))
    s = P.sigmoid_f(np.array([-1000, -10, 0, 10, 1000], np.float32))
    assert s[0] == 0 and s[2] == 0.5 and s[4] == 1
    rec = P.RecordedMath(rsqrt={int(np.float32(4.0).view(np.uint32)): int(np.float32(0.25).view(np.uint32))})
    assert rec.rsqrt(np.array([4.0, 16.0], np.float32)).tolist() == [0.25, 0.25]
    with P.use_math(rec):
        assert P.MATH is rec
    assert isinstance(P.MATH, P.HostMath) and P.MATH is not rec


def test_gate_fp8_per_token_scale_properties():
    rng = np.random.default_rng(3)
    out = F.bf16_round(rng.standard_normal((8, 256)).astype(np.float32))
    gate = F.bf16_round(rng.standard_normal((8, 256)).astype(np.float32))
    codes, scale = P.gate_fp8(out, gate)
    deq = F.e4m3_decode(codes) * scale[:, None]
    v = F.bf16_round(out * F.bf16_round(P.sigmoid_f(gate)))
    assert np.all(np.abs(F.e4m3_decode(codes)).max(axis=1) <= 448)
    assert np.all(np.abs(deq - v) <= np.abs(v) * 2 ** -4 + scale[:, None] * 2 ** -9 + 1e-12)


def test_lm_head_argmax_oracle_ties_and_nan():
    from oracle import producers as P

    h = np.ones((2, 8), dtype=np.float32)
    w = np.zeros((5, 8), dtype=np.float32)
    w[1] = w[3] = 1.0  # equal best logits at 1 and 3 -> 1
    w[4] = np.nan
    logits, tok = P.lm_head_argmax(h, w)
    assert tok.tolist() == [1, 1]
    assert logits[0, 1] == 8.0 and np.isnan(logits[0, 4])
    w2 = np.full((3, 8), -1.0, dtype=np.float32)
    w2[2] = -0.5  # all negative: the largest (least negative) wins
    assert P.lm_head_argmax(h, w2)[1].tolist() == [2, 2]


def _producer_golden():
    import importlib.util

    path = Path(__file__).resolve().parent / "golden" / "producers_ref.json"
    if not path.exists():
        pytest.skip("producers_ref.json not recorded yet (tests/golden/make_producer_golden.py on a B200)")
    spec = importlib.util.spec_from_file_location("make_producer_golden", path.parent / "make_producer_golden.py")
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    return gen, json.loads(path.read_text())


def test_oracle_reproduces_reference_producer_bytes():
    """The reference's norm-pack, attention front (D 256, page 32) and FP8 gate
    epilogue, run on a B200 from its own sources, recorded as output hashes:
    the CPU oracle rebuilds every output byte from the seeded inputs, given
    CUDA's rsqrtf / expf values where they differ from the correctly rounded
    ones (recorded beside the hashes)."""
    gen, golden = _producer_golden()
    checked = 0
    for kind, cases in golden["cases"].items():
        for case in cases:
            math = P.RecordedMath(rsqrt={int(k): v for k, v in case["rsqrt_differs"].items()},
                                  exp={int(k): v for k, v in case["exp_differs"].items()})
            with P.use_math(math):
                outs = gen.oracle_outputs(kind, case["spec"])
            for name, digest in case["sha256"].items():
                assert gen.sha(np.asarray(outs[name])) == digest, (kind, case["spec"], name)
                checked += 1
    assert checked >= 10
