"""The boundary protocol's deadlock freedom, on CPU, for the schedules this
build produces at G = 2, 4 and 8 (folded and conventional).

A random-interleaving model of the rules the transport enforces
(`vpp/stages.py`): per rank 2 shared source slots and 3 shared destination
slots (the rank layout), a 7-slot ring per edge, destination slots granted
eagerly in the rank's consumption order (a rank keeps granting while it
waits), a sender takes its physical source slot before computing the stage
output and sends once its credit is granted, and a copy frees the source slot
when it completes.  Every rank walks the op list of
`layout.rank_local_stage_orders` / `layout.cpp_stage_orders`; the model
fails if all ranks block with no copy in flight."""

import random

import pytest

from qwen_infra_b200.vpp import layout as L


def run(G, B, seed, profile="vpp", src_slots=2, dst_slots=3, ring=7, grant_by_edge=False):
    rnd = random.Random(seed)
    if profile == "vpp":
        orders = L.rank_local_stage_orders(list(range(B)), G)
        last = 2 * G - 1
        srank = lambda s: L.stage_rank(s, G)
    else:
        orders = L.cpp_stage_orders(list(range(B)), G)
        last = G - 1
        srank = lambda s: s
    def out_edge(s):
        return s < last and srank(s) != srank(s + 1)
    def in_edge(s):
        return s > 0 and srank(s - 1) != srank(s)
    pos = [0] * G
    state = [None] * G   # per rank: None (idle), or dict of the op in flight
    src_free = [src_slots] * G
    dst_free = [dst_slots] * G
    # grants: receiver side, per rank: list of receive ops in consumption order
    recv_sched = [[(b, s) for b, s in orders[r] if in_edge(s)] for r in range(G)]
    if grant_by_edge:  # the rule broken on purpose: grants by edge, not by consumption
        recv_sched = [sorted(q, key=lambda x: (x[1], x[0])) for q in recv_sched]
    grant_pos = [0] * G
    granted = set()          # (b, s) messages granted a dst slot
    ring_busy = {}           # (edge dst stage, seq%ring) -> busy
    seq_of = {}              # (b, s) -> per-edge sequence number
    cnt = {}
    for r in range(G):
        for b, s in recv_sched[r]:
            seq_of[(b, s)] = cnt.get(s, 0); cnt[s] = cnt.get(s, 0) + 1
    arrived = set()          # (b, s): data of stage s input landed
    copies = []              # [remaining, (b, s_dst), src_rank]
    done = 0
    total = sum(len(o) for o in orders)
    steps = 0
    while done < total:
        steps += 1
        if steps > 2_000_000:
            return "too many steps"
        progressed = False
        # receivers grant eagerly, in consumption order
        for r in range(G):
            while grant_pos[r] < len(recv_sched[r]) and dst_free[r] > 0:
                b, s = recv_sched[r][grant_pos[r]]
                key = (s, seq_of[(b, s)] % ring)
                if ring_busy.get(key):
                    break
                ring_busy[key] = True
                dst_free[r] -= 1
                granted.add((b, s))
                grant_pos[r] += 1
                progressed = True
        # async copies
        for c in list(copies):
            c[0] -= 1
            if c[0] <= 0:
                copies.remove(c)
                arrived.add(c[1])
                src_free[c[2]] += 1
                progressed = True
        order = list(range(G)); rnd.shuffle(order)
        for r in order:
            if pos[r] >= len(orders[r]):
                continue
            b, s = orders[r][pos[r]]
            st = state[r]
            if st is None:
                st = state[r] = dict(phase="recv")
            if st["phase"] == "recv":
                if in_edge(s) and (b, s) not in arrived:
                    continue
                st["phase"] = "src"
                progressed = True
            if st["phase"] == "src":
                if out_edge(s):
                    if src_free[r] == 0:
                        continue
                    src_free[r] -= 1
                st["phase"] = "compute"; st["t"] = rnd.randint(1, 5)
                progressed = True
            if st["phase"] == "compute":
                st["t"] -= 1
                if st["t"] > 0:
                    progressed = True
                    continue
                if in_edge(s):   # retire: the input's destination slot and ring slot come back
                    dst_free[r] += 1
                    ring_busy[(s, seq_of[(b, s)] % ring)] = False
                st["phase"] = "send"
                progressed = True
            if st["phase"] == "send":
                if out_edge(s):
                    if (b, s + 1) not in granted:
                        continue   # waiting for the credit (grants keep flowing above)
                    copies.append([rnd.randint(1, 8), (b, s + 1), r])
                pos[r] += 1; state[r] = None; done += 1
                progressed = True
        if not progressed and not copies:
            return f"DEADLOCK at done {done}/{total}: pos {pos} states {[ (orders[r][pos[r]] if pos[r] < len(orders[r]) else None, state[r] and state[r]['phase']) for r in range(G)]} src_free {src_free} dst_free {dst_free}"
    return "ok"



@pytest.mark.parametrize("profile", ["vpp", "cpp"])
@pytest.mark.parametrize("G", [2, 4, 8])
def test_orders_and_slot_budget_never_deadlock(profile, G):
    for B in (1, 2, 5, 16, 64):
        for seed in range(6):
            assert run(G, B, seed, profile) == "ok", (profile, G, B, seed)


def test_the_model_catches_grants_out_of_consumption_order():
    """Not vacuous: granting destination slots edge by edge instead of in the
    rank's consumption order deadlocks the same bank."""
    assert all(run(4, 16, seed, "vpp", grant_by_edge=True).startswith("DEADLOCK") for seed in range(4))
