"""In-tree build of the native libraries (nvcc for sm_100a, g++ for host C++).

``libqwen_infra_b200.so``  : CUDA kernels + C ABI (include/qwen_infra_b200.h)
``libqwen_vpp_native.so``  : stage-boundary transport (wire codec, slot pools,
                            peer-to-peer copy-engine edges, NCCL comparison edge)

Outputs are written next to this file so that they travel with the source tree.
"""

import os
import shutil
import subprocess
import tempfile
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
KERNEL_LIB = PKG / "libqwen_infra_b200.so"
TRANSPORT_LIB = PKG / "libqwen_vpp_native.so"

KERNEL_SOURCES = ["producers.cu", "gemm.cu", "attention.cu", "attention_noalloc.cu", "lm_head.cu", "decode.cu"]
TRANSPORT_SOURCES = ["wire.cpp", "slot_pool.cpp", "edges.cpp", "transport_abi.cpp", "kv_copy.cpp"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo", "--shared", "-Xcompiler", "-fPIC",
    "-Xptxas", "-v", "-cudart", "static",
]


def cuda_home():
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    if not (Path(home) / "bin" / "nvcc").exists():
        found = shutil.which("nvcc")
        if not found:
            raise RuntimeError("nvcc not found: set CUDA_HOME")
        home = str(Path(found).resolve().parent.parent)
    return Path(home)


def _stale(target, sources):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(argv, log):
    with open(log, "w") as out:
        proc = subprocess.run(argv, stdout=out, stderr=subprocess.STDOUT, timeout=900)
    if proc.returncode:
        raise RuntimeError(f"build failed ({' '.join(map(str, argv[:3]))} ...): see {log}\n" + Path(log).read_text()[-4000:])


# Extra flags per source.  The producers compile without FMA contraction, as
# the reference builds its producer kernels (--fmad=false): their own fp32
# steps are explicit IEEE operations either way, and the CUDA math functions
# they call (rsqrtf, expf) are then compiled under the reference's setting.
FILE_FLAGS = {"producers.cu": ["--fmad=false"]}


def build_kernels(force=False):
    sources = [CSRC / s for s in KERNEL_SOURCES]
    deps = sources + [CSRC / "common.cuh", INCLUDE / "qwen_infra_b200.h", Path(__file__)]
    if not force and not _stale(KERNEL_LIB, deps):
        return KERNEL_LIB
    nvcc = cuda_home() / "bin" / "nvcc"
    compile_flags = [f for f in NVCC_FLAGS if f not in ("--shared", "-cudart", "static")]
    log = PKG / "build_kernels.log"
    with tempfile.TemporaryDirectory(prefix="qi_build_") as tmpdir:
        objs = [Path(tmpdir) / (s.stem + ".o") for s in sources]

        def compile_one(i):
            src = sources[i]
            argv = [str(nvcc), *compile_flags, *FILE_FLAGS.get(src.name, []), "-I", str(INCLUDE), "-c", str(src),
                    "-o", str(objs[i])]
            return subprocess.run(argv, capture_output=True, text=True, timeout=900)

        with ThreadPoolExecutor(max_workers=len(sources)) as pool:
            results = list(pool.map(compile_one, range(len(sources))))
        with open(log, "w") as out:
            for src, r in zip(sources, results):
                out.write(f"== {src.name} (rc {r.returncode})\n{r.stdout}{r.stderr}")
        if any(r.returncode for r in results):
            raise RuntimeError(f"kernel build failed: see {log}\n" + log.read_text()[-4000:])
        tmp = KERNEL_LIB.with_suffix(".part.so")
        _run([str(nvcc), "-gencode", "arch=compute_100a,code=sm_100a", "--shared", "-cudart", "static",
              *map(str, objs), "-o", str(tmp)], PKG / "build_link.log")
    os.replace(tmp, KERNEL_LIB)
    return KERNEL_LIB


def build_transport(force=False):
    sources = [CSRC / s for s in TRANSPORT_SOURCES]
    headers = list(CSRC.glob("*.h"))
    if not all(s.exists() for s in sources):
        return None
    if not force and not _stale(TRANSPORT_LIB, sources + headers):
        return TRANSPORT_LIB
    home = cuda_home()
    tmp = TRANSPORT_LIB.with_suffix(".part.so")
    argv = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-Wall", "-I", str(home / "include"), "-I", str(CSRC),
            *map(str, sources), "-o", str(tmp), "-L", str(home / "lib64"), "-lcudart_static", "-ldl", "-lrt",
            "-lpthread"]
    _run(argv, PKG / "build_transport.log")
    os.replace(tmp, TRANSPORT_LIB)
    return TRANSPORT_LIB


def build(force=False):
    return build_kernels(force), build_transport(force)


if __name__ == "__main__":
    print(build(force=True))
