"""Build the checkers into oracle/_ref/ (TEST INFRASTRUCTURE ONLY).

From the reference's own sources where they lie (read-only, never copied),
compiled directly (not through the reference's build system):
* ``slot_pool_test``: the reference's C++ known-answer test
  (tests/slot_pool.cpp) of its wire codec and slot-generation lifecycle (g++);
* ``wire_dump``: oracle/wire_dump.cpp linked against the reference codec
  (src/qwen_infra/vpp/native/interface.cpp), printing golden headers (g++);
* ``libref_norm_pack.so`` and ``libref_attention_front.so``: the reference's
  producer kernels src/qwen_infra/kernels/nvfp4_norm_pack.cu and
  nvfp4_attention_front.cu, unmodified, with the flags of their own build
  recipe (kernels/nvfp4_norm_pack.py:26-36: -std=c++17 -O3 --fmad=false
  --shared -Xcompiler=-fPIC -lineinfo) but ``-arch=sm_100a`` for the B200
  instead of sm_120f.  The GPU tests run them on the same inputs as this
  repository's kernels and compare the bytes.

From this repository (needs no reference checkout):
* ``libqo_gpu_checks.so``: oracle/gpu_checks.cu, CUDA's rsqrtf / expf on
  arrays and the reference's FP8 gate epilogue restated, with the same flags.

The reference checkout is found at $QVPP_REFERENCE, else at ``reference``
beside this repository.  Without it (the GPU box) the reference builds are
skipped: the files already in oracle/_ref/ travel with the tree, and the
committed fixtures under tests/golden/ are used.
"""

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
REF = Path(os.environ.get("QVPP_REFERENCE", str(REPO.parent / "reference")))
OUT = HERE / "_ref"
# kernels/nvfp4_norm_pack.py:26-36 (the attention front uses the same list)
REF_CUDA_FLAGS = ["-std=c++17", "-O3", "--fmad=false", "-arch=sm_100a", "--shared", "-Xcompiler=-fPIC", "-lineinfo"]


def _nvcc():
    home = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    nvcc = home / "bin" / "nvcc"
    return str(nvcc) if nvcc.exists() else shutil.which("nvcc")


def _stale(target, sources):
    return not target.exists() or any(s.stat().st_mtime > target.stat().st_mtime for s in sources)


def build_cuda():
    nvcc = _nvcc()
    if nvcc is None:
        return None
    OUT.mkdir(exist_ok=True)
    jobs = [(HERE / "gpu_checks.cu", OUT / "libqo_gpu_checks.so")]
    kernels = REF / "src/qwen_infra/kernels"
    if (kernels / "nvfp4_norm_pack.cu").exists():
        jobs += [(kernels / "nvfp4_norm_pack.cu", OUT / "libref_norm_pack.so"),
                 (kernels / "nvfp4_attention_front.cu", OUT / "libref_attention_front.so")]
    for src, lib in jobs:
        if not _stale(lib, [src, Path(__file__)]):
            continue
        part = lib.with_suffix(".part.so")
        subprocess.run([nvcc, *REF_CUDA_FLAGS, str(src), "-o", str(part)], check=True, timeout=600,
                       stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        os.replace(part, lib)
    return OUT


def build_host():
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


def build():
    host = build_host()
    cuda = build_cuda()
    return host or cuda


if __name__ == "__main__":
    print(build())
    sys.exit(0)
