"""CUDA's rsqrtf / expf as black boxes for the oracle (TEST INFRASTRUCTURE ONLY).

The reference's producers call two CUDA math functions whose results are not
correctly rounded: ``rsqrtf`` (nvfp4_norm_pack.cu:39, nvfp4_attention_front.cu:81)
and ``expf`` (nvfp4_bucket_xqa.cu:57).  The CPU restatement in
:mod:`oracle.producers` takes them from a provider: :class:`CudaMath` here
evaluates them on the GPU through oracle/_ref/libqo_gpu_checks.so (built from
oracle/gpu_checks.cu with the reference's flags), so GPU tests hold the
kernels to exact bytes; on the CPU the correctly rounded
:class:`oracle.producers.HostMath` stands in, or a
:class:`oracle.producers.RecordedMath` with the CUDA values recorded in a
golden fixture.
"""

import ctypes as ct
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "_ref" / "libqo_gpu_checks.so"
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            raise FileNotFoundError(f"{LIB} not built (python oracle/build_ref.py)")
        _lib = ct.CDLL(str(LIB))
        for name in ("qo_rsqrtf", "qo_expf"):
            fn = getattr(_lib, name)
            fn.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_int, ct.c_void_p]
            fn.restype = ct.c_int
        _lib.qo_gate_fp8_static.argtypes = [ct.c_void_p] * 4 + [ct.c_int, ct.c_void_p]
        _lib.qo_gate_fp8_static.restype = ct.c_int
    return _lib


def _apply(name, x):
    import torch

    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    flat = x.reshape(-1)
    if flat.size == 0:
        return x.copy()
    dev = torch.device("cuda", torch.cuda.current_device())
    src = torch.from_numpy(flat.copy()).to(dev)
    dst = torch.empty_like(src)
    stream = torch.cuda.current_stream(dev)
    rc = getattr(lib(), name)(ct.c_void_p(src.data_ptr()), ct.c_void_p(dst.data_ptr()), flat.size,
                              ct.c_void_p(stream.cuda_stream))
    if rc:
        raise RuntimeError(f"{name} launch status {rc}")
    return dst.cpu().numpy().reshape(x.shape)


class CudaMath:
    """rsqrtf / expf evaluated by CUDA on the current GPU."""

    name = "cuda"

    def rsqrt(self, x):
        return _apply("qo_rsqrtf", x)

    def exp(self, x):
        return _apply("qo_expf", x)


def gate_fp8_static_reference(values, gates, scale):
    """The reference's FP8 epilogue (nvfp4_bucket_xqa.cu:56-62) element-wise on
    the GPU: values, gates bf16 torch CUDA tensors of one shape, scale an fp32
    device scalar.  Returns the E4M3 codes as a uint8 tensor."""
    import torch

    values = values.contiguous()
    gates = gates.contiguous()
    out = torch.empty(values.shape, dtype=torch.uint8, device=values.device)
    rc = lib().qo_gate_fp8_static(ct.c_void_p(values.data_ptr()), ct.c_void_p(gates.data_ptr()),
                                  ct.c_void_p(scale.data_ptr()), ct.c_void_p(out.data_ptr()), values.numel(),
                                  ct.c_void_p(torch.cuda.current_stream(values.device).cuda_stream))
    if rc:
        raise RuntimeError(f"qo_gate_fp8_static launch status {rc}")
    return out
