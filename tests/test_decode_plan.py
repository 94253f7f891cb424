"""Decode task planning and route rule (CPU): the oracle planner and the
package's route rule against outputs recorded from the reference's own
planner (``tests/golden/decode_plans.json``, made by
``tests/golden/make_golden.py``), partition invariants at this build's
16-token pages, and the blockwise decode oracle against exact softmax."""

import json
import math
import random
from pathlib import Path

import numpy as np
import pytest

from oracle import decode as OD

GOLDEN = json.loads((Path(__file__).parent / "golden" / "decode_plans.json").read_text())


def test_oracle_planner_reproduces_reference_plans():
    assert len(GOLDEN["plans"]) >= 60
    for case in GOLDEN["plans"]:
        got = OD.task_plan(case["lengths"], ctas=case["ctas"], cyclic=case["mode"] == "cyclic",
                           aligned=case["mode"] == "aligned", table_width=case["table_width"], page_size=32)
        assert got == case["plan"], (case["lengths"], case["ctas"], case["mode"])


def test_route_rule_reproduces_reference_routes():
    from qwen_infra_b200.decode import route

    for case in GOLDEN["routes"]:
        args = dict(table_width=case["table_width"], sm_count=case["sm_count"], page_size=32)
        assert route(case["lengths"], **args) == case["route"], case
        assert OD.route(case["lengths"], **args) == case["route"], case


@pytest.mark.parametrize("batch", [1, 2, 8, 16, 32])
@pytest.mark.parametrize("mode", ["intervals", "cyclic", "aligned"])
def test_partition_covers_each_tile_once_at_page16(batch, mode):
    rng = random.Random(987 + batch)
    for _ in range(8):
        lengths = [rng.choice([0, 1, 15, 16, 255, 256, 2049, 32768, 131072]) for _ in range(batch)]
        ctas = rng.choice([batch, 37, 148, 340])
        ctas = max(ctas, batch)
        plan = OD.task_plan(lengths, ctas=ctas, cyclic=mode == "cyclic", aligned=mode == "aligned",
                            table_width=8200, page_size=16)
        assert len(plan["tasks"]) <= ctas + batch - 1
        for r, n in enumerate(lengths):
            tasks = [t for t in plan["tasks"] if t[0] == r]
            tiles = sorted(tile for t in tasks for tile in OD.plan_tiles(t))
            assert tiles == list(range(math.ceil(n / 256)))
            first, count = plan["requests"][r]
            assert plan["tasks"][first:first + count] == tasks
        if mode != "cyclic":
            assigned = sorted(s for lo, hi in plan["buckets"] for s in range(lo, hi))
            assert assigned == list(range(len(plan["tasks"])))


def test_planner_rejects_what_the_reference_rejects():
    with pytest.raises(ValueError):
        OD.task_plan([], ctas=4)
    with pytest.raises(ValueError):
        OD.task_plan([1] * 33, ctas=64)
    with pytest.raises(ValueError):
        OD.task_plan([1, 2], ctas=1)
    with pytest.raises(ValueError):
        OD.task_plan([1], ctas=341)
    with pytest.raises(ValueError):
        OD.task_plan([100], ctas=4, table_width=3, page_size=32)
    with pytest.raises(ValueError):
        OD.task_plan([100], ctas=4, cyclic=True, aligned=True)


def test_blockwise_oracle_against_exact_softmax():
    rng = np.random.default_rng(3)
    lengths = [0, 1, 300, 700]
    hq, hkv, d = 8, 2, 128
    q = rng.standard_normal((len(lengths), hq, d)).astype(np.float32)
    k = [rng.standard_normal((n, hkv, d)).astype(np.float32) for n in lengths]
    v = [rng.standard_normal((n, hkv, d)).astype(np.float32) for n in lengths]
    for mode in ("intervals", "cyclic", "aligned"):
        plan = OD.task_plan(lengths, ctas=5, cyclic=mode == "cyclic", aligned=mode == "aligned",
                            table_width=64, page_size=16)
        got = OD.decode_attention(q, k, v, lengths, plan, softmax_scale=1 / math.sqrt(d), k_global=0.5,
                                  v_global=2.0)
        want = OD.decode_attention_exact(q, k, v, lengths, softmax_scale=1 / math.sqrt(d), k_global=0.5,
                                         v_global=2.0)
        assert np.abs(got - want).max() <= 2e-3 * np.abs(want).max()
        assert not got[0].any()


@pytest.mark.parametrize("scale", [1e-3, 1.0, 300.0])
def test_query_terms_reconstruct_the_group(scale):
    """The S product's NVFP4 query terms: power-of-two globals, exact term
    values, and a residual that shrinks about 11x per term."""
    from oracle import formats as F
    q = F.bf16_round(np.random.default_rng(3).standard_normal((12, 128)).astype(np.float32) * np.float32(scale))
    q[5] = 0.0  # a zero head contributes nothing
    terms = OD.q_terms(q)
    assert len(terms) == OD.Q_TERMS
    approx = np.zeros_like(q, dtype=np.float64)
    errs = []
    for unscaled, ig in terms:
        assert ig > 0 and math.frexp(ig)[0] == 0.5  # 1/g is a power of two
        assert not unscaled[5].any()
        approx += unscaled.astype(np.float64) * ig
        errs.append(np.abs(approx - q).max() / np.abs(q).max())
    assert all(b < a / 5 for a, b in zip(errs, errs[1:])), errs
    assert errs[-1] < 2e-4
    zero = OD.q_terms(np.zeros((4, 128), np.float32))
    assert all(ig == 0.0 and not t.any() for t, ig in zero)


@pytest.mark.parametrize("page_size", [0, 3, 24, 48])
def test_plan_rejects_pages_that_are_not_a_power_of_two(page_size):
    from qwen_infra_b200.decode import TaskPlan

    with pytest.raises(ValueError):
        TaskPlan(4, ctas=8, page_size=page_size, device="cpu")
