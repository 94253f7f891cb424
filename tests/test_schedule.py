"""Folded schedule: equal to the reference at G = 4 (fixtures recorded from
src/qwen_infra/vpp/layout.py) and sound for G = 1, 2, 4, 8 (the reference's
tests/test_planning.py:37-60 properties, generalised)."""

import json
from pathlib import Path

import pytest

from qwen_infra_b200.vpp import layout as L

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "layout_g4.json").read_text())


def test_layer_ranges_and_communication_match_reference():
    for r in range(4):
        assert [list(x) for x in L.layer_ranges(r)] == GOLDEN["layer_ranges"][str(r)]
        for t in (0, 1):
            assert list(L.communication(r, t)) == GOLDEN["communication"][f"{r},{t}"]


@pytest.mark.parametrize("size", [1, 2, 4, 7, 8, 9, 20, 64])
def test_rank_orders_match_reference(size):
    orders = L.rank_local_stage_orders(range(10, 10 + size))
    assert [[list(op) for op in o] for o in orders] == GOLDEN["orders"][str(size)]


def test_rank_local_trace_with_early_drain_matches_reference():
    order = L.RankLocalOrder(1)
    trace = []
    for b in range(5):
        order.admit(b)
        trace.append(order.next())
    while 0 not in order.returned:
        trace.append(order.next(draining=True))
    order.release(0)
    trace.append(order.next())
    trace.append(order.next(draining=True))
    assert [list(t) if t else None for t in trace] == GOLDEN["trace_rank1"]


def test_retained_boundary_bytes_match_reference():
    for t, v in GOLDEN["retained_boundary_bytes"].items():
        assert L.retained_boundary_bytes(int(t)) == v


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
def test_folded_ranges_cover_each_layer_once(ranks):
    layers = 64
    owned = [i for r in range(ranks) for lo, hi in L.layer_ranges(r, ranks, layers) for i in range(lo, hi)]
    assert sorted(owned) == list(range(layers))


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
@pytest.mark.parametrize("size", [1, 3, 15, 16, 40])
def test_orders_preserve_stage_fifo_and_dependencies(ranks, size):
    bank = list(range(size))
    orders = L.rank_local_stage_orders(bank, ranks)
    for r, order in enumerate(orders):
        for stage in (r, 2 * ranks - 1 - r):
            assert [b for b, s in order if s == stage] == bank
        assert len(order) == 2 * size
    # A global replay that runs each rank's next op only once its input exists
    # must finish: the per-rank orders admit no cyclic wait.
    done = set()
    pos = [0] * ranks
    progressed = True
    while progressed:
        progressed = False
        for r in range(ranks):
            while pos[r] < len(orders[r]):
                b, s = orders[r][pos[r]]
                if s > 0 and (b, s - 1) not in done:
                    break
                done.add((b, s))
                pos[r] += 1
                progressed = True
    assert all(pos[r] == len(orders[r]) for r in range(ranks))


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
@pytest.mark.parametrize("size", [1, 3, 4, 15, 16, 40, 64])
def test_orders_fit_the_overlapped_fold_rotation(ranks, size):
    """The overlapped runner rotates the local fold over three buffer pairs:
    on rank G-1, stage G-1 of chunk j overwrites the pair stage G of chunk
    j - 3 read, so that read must already be issued (it then waits on its
    event).  Every rank order must also issue stage G of a chunk after
    stage G-1 of it (the event it waits on)."""
    orders = L.rank_local_stage_orders(list(range(size)), ranks)
    pos = {op: i for i, op in enumerate(orders[ranks - 1])}
    for b in range(size):
        assert pos[(b, ranks)] > pos[(b, ranks - 1)]
        if b >= 3:
            assert pos[(b - 3, ranks)] < pos[(b, ranks - 1)]


@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_admission_bound_and_double_release(ranks):
    order = L.RankLocalOrder(0, ranks)
    for b in range(2 * ranks - 1):
        order.admit(b)
    with pytest.raises(RuntimeError):
        order.admit(2 * ranks - 1)
    while 0 not in order.returned:
        assert order.next(draining=True) is not None
    order.release(0)
    with pytest.raises(ValueError):
        order.release(0)
    with pytest.raises(ValueError):
        order.admit(0)  # ids strictly increase


def test_wire_edges_generalise_reference_source_stages():
    assert L.wire_edges(4) == (0, 1, 2, 4, 5, 6)
    assert L.wire_edges(1) == ()
    assert L.wire_edges(2) == (0, 2)
    assert len(L.wire_edges(8)) == 14


def test_profile_annotation():
    text = L.profile_annotation(1, 1, 7, "compute", [(0, 2048, 4096)])
    assert text.startswith("qwen_infra_vpp:")
    body = json.loads(text.split(":", 1)[1])
    assert body["stage"] == 6 and body["layers"] == [48, 56]
    with pytest.raises(ValueError):
        L.profile_annotation(1, 2, 7, "compute", [])


# --- conventional pipeline (the comparison arm) ------------------------------

@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
def test_cpp_ranges_cover_each_layer_once_in_order(ranks):
    spans = [L.cpp_layer_range(r, ranks, 64) for r in range(ranks)]
    assert [i for lo, hi in spans for i in range(lo, hi)] == list(range(64))
    with pytest.raises(ValueError):
        L.cpp_layer_range(0, 3, 64)  # 64 layers do not split into 3 stages


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
def test_cpp_orders_are_per_stage_fifo(ranks):
    bank = list(range(11))
    orders = L.cpp_stage_orders(bank, ranks)
    assert len(orders) == ranks
    for r, order in enumerate(orders):
        assert order == [(b, r) for b in bank]
    with pytest.raises(ValueError):
        L.cpp_stage_orders([], ranks)


@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_cpp_boundaries_are_the_forward_wire_edges(ranks):
    from qwen_infra_b200.vpp.stages import boundary_edges

    for r in range(ranks):
        out_e, in_e = boundary_edges(r, ranks, "cpp")
        assert sorted(out_e) == ([r] if r < ranks - 1 else [])
        assert sorted(in_e) == ([r] if r > 0 else [])
        for s, e in out_e.items():
            assert (e.src_rank, e.dst_rank, e.forward) == (r, r + 1, True)
            # same edge index as the folded layout's forward edge out of stage s
            assert e.index == boundary_edges(r, ranks, "vpp")[0][s].index
    # folded edges are unchanged: every source stage but the fold and the last
    srcs = sorted(s for r in range(ranks) for s in boundary_edges(r, ranks, "vpp")[0])
    assert tuple(srcs) == L.wire_edges(ranks)
