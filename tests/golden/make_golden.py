"""Regenerate the golden fixtures recorded from the reference project itself.

Needs the reference checkout (read-only) at $QVPP_REFERENCE (default
/root/reference) and, for the wire headers, the reference C++ sources
compiled by ``oracle/build_ref.py``.  The committed JSON fixtures are what the
tests read; this script is only how they were made.

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
REF = Path(os.environ.get("QVPP_REFERENCE", "/root/reference"))


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


if __name__ == "__main__":
    (HERE / "layout_g4.json").write_text(json.dumps(layout_fixture(), indent=1) + "\n")
    (HERE / "scale_offset.json").write_text(json.dumps(scale_offset_fixture()) + "\n")
    (HERE / "wire_headers.json").write_text(json.dumps(wire_fixture(), indent=1) + "\n")
    print("golden fixtures written")
