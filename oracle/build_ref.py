"""Build the reference-side checkers into oracle/_ref/ (TEST INFRASTRUCTURE ONLY).

Compiles, from the reference's own sources where they lie (read-only, never
copied), with g++ directly (not the reference's build system):
* ``slot_pool_test``: the reference's C++ known-answer test
  (tests/slot_pool.cpp) of its wire codec and slot-generation lifecycle;
* ``wire_dump``: oracle/wire_dump.cpp linked against the reference codec
  (src/qwen_infra/vpp/native/interface.cpp), printing golden headers.

Skipped silently when the reference checkout is absent (the GPU box): the
committed fixtures under tests/golden/ are used there.
"""

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("QVPP_REFERENCE", "/root/reference"))
OUT = HERE / "_ref"


def build():
    native = REF / "src/qwen_infra/vpp/native"
    if not (native / "interface.cpp").exists():
        return None
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        return None
    OUT.mkdir(exist_ok=True)
    common = [cxx, "-std=c++17", "-O1", "-I", str(native)]
    subprocess.run(common + [str(REF / "tests/slot_pool.cpp"), str(native / "slot_pool.cpp"),
                             str(native / "interface.cpp"), "-o", str(OUT / "slot_pool_test")],
                   check=True, timeout=300)
    subprocess.run(common + [str(HERE / "wire_dump.cpp"), str(native / "interface.cpp"), "-o", str(OUT / "wire_dump")],
                   check=True, timeout=300)
    return OUT


if __name__ == "__main__":
    print(build())
    sys.exit(0)
