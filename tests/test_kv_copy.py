"""KV page copy engine (``qv_kvcopy_*``).  CPU: validation of copy runs and
page gates (the reference's submit checks, ``native/kv_copy.cpp:299-335``).
GPU: strided offload / reload round trips, page gates between a store and a
load, producer-stream ordering, cancellation, bounded job slots, segments."""

import time

import pytest
import torch

from qwen_infra_b200.vpp import kv_copy as KC


def _runs(rows):
    return torch.tensor(rows, dtype=torch.int64).reshape(-1, 7)


def test_plan_collapses_contiguous_runs_and_groups_gates():
    # one strided TP-head run (16 x 64 B at stride 256 -> compact on host) and
    # two adjacent contiguous runs that merge into one piece
    runs = _runs([[0, 256, 0, 64, 16, 256, 64],
                  [0, 8192, 1024, 4096, 1, 0, 0],
                  [0, 12288, 5120, 4096, 1, 0, 0],
                  [1, 0, 9216, 64, 4, 64, 64]])  # contiguous on both sides: one piece
    units, pieces, nbytes = KC.plan_summary([65536, 4096], 1 << 20, runs)
    assert units == 1 and pieces == 3 and nbytes == 1024 + 8192 + 256
    gates = torch.tensor([[0, 1], [1, 1], [1, 1], [0, 1]], dtype=torch.int64)
    units, pieces, nbytes = KC.plan_summary([65536, 4096], 1 << 20, runs, gates, flag_count=4)
    assert units == 2 and pieces == 3 and nbytes == 1024 + 8192 + 256


@pytest.mark.parametrize("row,why", [
    ([2, 0, 0, 64, 1, 0, 0], "tensor index"),
    ([0, 65500, 0, 64, 1, 0, 0], "device overrun"),
    ([0, 0, (1 << 20) - 10, 64, 1, 0, 0], "host overrun"),
    ([0, 0, 0, 0, 1, 0, 0], "empty run"),
    ([0, 0, 0, 64, 0, 0, 0], "no fragments"),
    ([0, 0, 0, 64, 4, 32, 64], "device stride below the piece"),
    ([0, 0, 0, 64, 2000, 256, 64], "fragments past the buffer"),
    ([0, -1, 0, 64, 1, 0, 0], "negative offset"),
])
def test_plan_rejects_runs_that_escape_their_storage(row, why):
    with pytest.raises(ValueError):
        KC.plan_summary([65536, 4096], 1 << 20, _runs([row]))


def test_plan_rejects_bad_gates():
    runs = _runs([[0, 0, 0, 64, 1, 0, 0], [0, 64, 64, 64, 1, 0, 0]])
    for gates in ([[0, 0], [0, 0]], [[5, 1], [5, 1]], [[0, 1], [0, 2]], [[-1, 1], [0, 1]]):
        with pytest.raises(ValueError):
            KC.plan_summary([65536], 1 << 20, runs, torch.tensor(gates, dtype=torch.int64), flag_count=4)
    with pytest.raises(ValueError):
        KC.plan_summary([65536], 1 << 20, torch.zeros(3, 6, dtype=torch.int64))


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
DEV = torch.device("cuda:0") if torch.cuda.is_available() else None


def _gather(buf, run):
    t, off, hoff, nbytes, frags, ds, hs = run
    return [(hoff + i * hs, buf[off + i * ds: off + i * ds + nbytes]) for i in range(frags)]


def _setup(max_jobs=8):
    if DEV is None:
        pytest.skip("no CUDA device")
    g = torch.Generator().manual_seed(7)
    kcache = torch.randint(0, 256, (64 * 16 * 4 * 64,), generator=g, dtype=torch.uint8).to(DEV)
    scales = torch.randint(0, 256, (64 * 16 * 4 * 8,), generator=g, dtype=torch.uint8).to(DEV)
    big = torch.randint(0, 256, (9 << 20,), generator=g, dtype=torch.uint8).to(DEV)
    host = torch.zeros(12 << 20, dtype=torch.int8).pin_memory()
    eng = KC.KvCopy(DEV, [kcache, scales, big], host, segment_bytes=4 << 20, max_jobs=max_jobs)
    return eng, kcache, scales, big, host


def _offload_runs():
    rows = []
    hoff = 0
    for page in (3, 10, 11, 40):  # head 1 of 4: 16 tokens x 64 B at stride 256 -> compact
        rows.append([0, page * 4096 + 64, hoff, 64, 16, 256, 64])
        hoff += 1024
        rows.append([1, page * 512 + 8, hoff, 8, 16, 32, 8])
        hoff += 128
    rows.append([0, 20 * 4096, hoff, 4096, 1, 0, 0])  # a whole page
    hoff += 4096
    rows.append([2, 1000, hoff, 6 << 20, 1, 0, 0])  # spans two 4 MiB segments
    return rows


@pytest.mark.gpu
def test_offload_then_reload_round_trip():
    eng, kcache, scales, big, host = _setup()
    rows = _offload_runs()
    assert eng.submit(1, 1, _runs(rows), store=True)
    eng.wait([1])
    res = eng.poll()
    total = sum(r[3] * r[4] for r in rows)
    assert len(res) == 1 and res[0].job_id == 1 and res[0].bytes == total and res[0].segments >= 2
    assert not res[0].cancelled and res[0].device_ms > 0
    hb = host.view(torch.uint8)
    srcs = [kcache.cpu(), scales.cpu(), big.cpu()]
    for r in rows:
        for h, data in _gather(srcs[r[0]], r):
            assert torch.equal(hb[h:h + r[3]], data)
    # reload into cleared buffers
    for t in (kcache, scales, big):
        t.zero_()
    assert eng.submit(2, 1, _runs(rows), store=False)
    eng.wait([2])
    assert eng.poll()[0].bytes == total
    back = [kcache.cpu(), scales.cpu(), big.cpu()]
    for r in rows:
        t, off, _, nbytes, frags, ds, _ = r
        for i in range(frags):
            assert torch.equal(back[t][off + i * ds: off + i * ds + nbytes], srcs[t][off + i * ds: off + i * ds + nbytes])
    eng.drain()
    eng.close()
    with pytest.raises(RuntimeError):
        eng.submit(3, 1, _runs(rows), store=True)


@pytest.mark.gpu
def test_producer_stream_orders_the_copy():
    eng, kcache, _, _, host = _setup()
    side = torch.cuda.Stream(DEV)
    with torch.cuda.stream(side):
        torch.cuda._sleep(20_000_000)  # keep the producer busy while the job is admitted
        kcache[:4096].fill_(0x5A)
    assert eng.submit(1, 1, _runs([[0, 0, 0, 4096, 1, 0, 0]]), store=True, producer=side)
    eng.wait([1])
    eng.poll()
    assert (host[:4096].view(torch.uint8) == 0x5A).all()
    eng.drain()
    eng.close()


@pytest.mark.gpu
def test_page_gates_order_load_after_store_and_cancel_stops_waiting_jobs():
    eng, kcache, _, _, host = _setup()
    flags = torch.zeros(8, dtype=torch.int64)
    eng.set_ready(flags)
    run = _runs([[0, 4096, 0, 4096, 1, 0, 0]])
    assert eng.submit(1, 1, run, store=True, gates=torch.tensor([[2, 7]], dtype=torch.int64))
    eng.wait([1])
    eng.poll()
    assert int(flags[2]) == 7  # the store published its page
    ref = kcache[4096:8192].clone()
    kcache[4096:8192].zero_()
    # a load gated on epoch 8 waits until someone publishes it
    assert eng.submit(2, 1, run, store=False, gates=torch.tensor([[2, 8]], dtype=torch.int64))
    time.sleep(0.2)
    snap = eng.snapshot()
    assert len(snap) == 1 and snap[0].bytes == 0
    flags[2] = 8
    eng.wait([2])
    assert eng.poll()[0].bytes == 4096
    assert torch.equal(kcache[4096:8192], ref)
    # a load whose gate never opens is cancelled without copying
    assert eng.submit(3, 4, run, store=False, gates=torch.tensor([[5, 1]], dtype=torch.int64))
    assert eng.cancel(3, 4)
    assert not eng.cancel(3, 5)
    eng.wait([3])
    res = eng.poll()
    assert res[0].cancelled and res[0].bytes == 0
    with pytest.raises(ValueError):  # ids increase
        eng.submit(3, 1, run, store=True)
    eng.drain()
    eng.close()


@pytest.mark.gpu
def test_job_slots_are_bounded():
    eng, _, _, _, _ = _setup(max_jobs=2)
    flags = torch.zeros(4, dtype=torch.int64)
    eng.set_ready(flags)
    run = _runs([[0, 0, 0, 64, 1, 0, 0]])
    gate = torch.tensor([[1, 3]], dtype=torch.int64)
    assert eng.submit(1, 1, run, store=False, gates=gate)
    assert eng.submit(2, 1, run, store=False, gates=gate)
    assert not eng.submit(3, 1, run, store=False, gates=gate)
    with pytest.raises(RuntimeError):
        eng.close()  # jobs still live
    assert eng.cancel(1, 1) and eng.cancel(2, 1)
    eng.drain()
    assert len(eng.poll()) == 2
    assert eng.submit(4, 1, run, store=True)
    eng.wait([4])
    eng.poll()
    eng.close()
