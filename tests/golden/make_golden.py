"""Regenerate the golden fixtures recorded from the reference project itself.

Needs the reference checkout (read-only) at $QVPP_REFERENCE (default: a
checkout named ``reference`` beside this repository) and, for the wire
headers, the reference C++ sources compiled by ``oracle/build_ref.py``.
The committed JSON fixtures are what the tests read; this script is only
how they were made.

    python tests/golden/make_golden.py
"""

import importlib.util
import json
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
REF = Path(os.environ.get("QVPP_REFERENCE", str(REPO.parent / "reference")))


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def layout_fixture():
    lay = _load("ref_layout", REF / "src/qwen_infra/vpp/layout.py")
    out = dict(layer_ranges={r: lay.layer_ranges(r) for r in range(4)},
               communication={f"{r},{t}": lay.communication(r, t) for r in range(4) for t in (0, 1)},
               orders={})
    for size in (1, 2, 4, 7, 8, 9, 20, 64):
        bank = list(range(10, 10 + size))
        out["orders"][str(size)] = lay.rank_local_stage_orders(bank)
    # A rank-local trace with an early drain, to pin the warm-up credit rule.
    trace = []
    order = lay.RankLocalOrder(1)
    for b in range(5):
        order.admit(b)
        trace.append(order.next())
    while 0 not in order.returned:
        trace.append(order.next(draining=True))
    order.release(0)
    trace.append(order.next())
    trace.append(order.next(draining=True))
    out["trace_rank1"] = trace
    out["retained_boundary_bytes"] = {str(t): lay.retained_boundary_bytes(t) for t in (1, 2048, 8192)}
    return out


def scale_offset_fixture():
    pack = _load("ref_norm_pack", REF / "src/qwen_infra/kernels/nvfp4_norm_pack.py")
    pts = [(r, g) for r in (0, 1, 31, 32, 33, 127, 128, 129, 255, 1000, 8191) for g in (0, 1, 3, 4, 5, 79, 80, 318, 319)]
    return [[r, g, pack.scale_offset(r, g)] for r, g in pts]


def wire_fixture():
    exe = REPO / "oracle/_ref/wire_dump"
    if not exe.exists():
        subprocess.run([sys.executable, str(REPO / "oracle/build_ref.py")], check=True)
    return json.loads(subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout)


def decode_plan_fixture():
    """Task plans and routes of the reference's decode planner
    (``kernels/nvfp4_bucket_xqa.py:19-69``, ``kernels/nvfp4_kv_bucket_worker.py:9-31``)."""
    sys.path.insert(0, str(REF / "src"))
    try:
        xqa = _load("ref_xqa", REF / "src/qwen_infra/kernels/nvfp4_bucket_xqa.py")
        worker_src = (REF / "src/qwen_infra/kernels/nvfp4_kv_bucket_worker.py").read_text()
    finally:
        sys.path.pop(0)
    import random
    rng = random.Random(20261202)
    cases = []
    choices = [0, 1, 31, 255, 256, 257, 2049, 8192, 32768, 131072]
    for batch in (1, 2, 4, 8, 16, 32):
        for ctas in (batch, 37, 148, 340):
            if ctas < batch:
                continue
            for _ in range(1):
                lengths = [rng.choice(choices) for _ in range(batch)]
                if not any(lengths):
                    lengths[0] = 4097
                width = max(1, (max(lengths) + 31) // 32) + rng.choice([0, 3])
                for mode in ("intervals", "cyclic", "aligned"):
                    plan = xqa.task_plan(lengths, ctas=ctas, cyclic=mode == "cyclic", aligned=mode == "aligned",
                                         table_width=width)
                    cases.append(dict(lengths=lengths, ctas=ctas, mode=mode, table_width=width, plan=plan))
    # The route rule is a plain function of the lengths; record it through the
    # reference source (its module imports vLLM-side helpers at load time, so
    # only the function's own text is executed, against the reference limits).
    ns = {}
    limits = _load("ref_limits", REF / "src/qwen_infra/limits.py")
    ns["MAX_TABLE_WIDTH"] = limits.MAX_TABLE_WIDTH
    start = worker_src.index("def xqa_route")
    end = worker_src.index("\nclass ", start + 1)
    exec(compile(worker_src[start:end], "xqa_route", "exec"), ns)
    routes = []
    for lengths, width, sms in (([131072] + [256] * 15, 4096, 170), ([256] * 16, 4096, 170),
                                ([32768] * 16, 4096, 170), ([131073] + [256] * 15, 4096, 170),
                                ([32768] * 16, 1, 170), ([32768] * 4 + [0] * 4, 1024, 148),
                                ([8192] * 8, 256, 148), ([1, 256, 512, 131072] * 2, 4096, 148),
                                ([32768] * 4, 1024, 148), ([0] * 8, 16, 148), ([4096, 8192], 256, 148)):
        if max(lengths) > width * 32:
            continue
        routes.append(dict(lengths=lengths, table_width=width, sm_count=sms,
                           route=ns["xqa_route"](lengths, table_width=width, sm_count=sms)))
    return dict(plans=cases, routes=routes)


if __name__ == "__main__":
    (HERE / "layout_g4.json").write_text(json.dumps(layout_fixture(), indent=1) + "\n")
    (HERE / "scale_offset.json").write_text(json.dumps(scale_offset_fixture()) + "\n")
    (HERE / "wire_headers.json").write_text(json.dumps(wire_fixture(), indent=1) + "\n")
    (HERE / "decode_plans.json").write_text(json.dumps(decode_plan_fixture()) + "\n")
    print("golden fixtures written")
