"""KV page copy engine (offload / reload of paged KV to a pinned host pool).

Python face of ``qv_kvcopy_*`` (``csrc/kv_copy.cpp``), mirroring the
reference's ``KvCopy`` binding (``src/qwen_infra/vpp/native/kv_copy.h:18-45``):
``submit(id, generation, runs, store, producer, gates)`` admits a job of copy
runs ``int64 [N, 7]`` = [tensor index, device byte offset, host byte offset,
bytes, fragments, device stride, host stride] (False when every job slot is
busy), ``set_ready(flags)`` attaches the shared int64 page-gate words,
``cancel``, ``poll`` (harvest finished jobs), ``snapshot``, ``wait``,
``drain`` and ``close``.  Invalid arguments raise ``ValueError``; deadlines
raise ``TimeoutError``; an engine failure is terminal (``RuntimeError``).
"""

import ctypes as ct
from collections import namedtuple

import torch

from . import native as NV

KvCopyResult = namedtuple("KvCopyResult", "job_id generation bytes segments cancelled device_ms "
                                          "first_issue_ns last_done_ns")


def _kv_err():
    return NV.lib().qv_kvcopy_last_error().decode(errors="replace")


def _rows(t, cols, what):
    if not isinstance(t, torch.Tensor) or t.device.type != "cpu" or t.dtype != torch.int64 \
            or t.dim() != 2 or t.shape[1] != cols or not t.is_contiguous():
        raise ValueError(f"expected a contiguous CPU int64 [N, {cols}] {what}")
    return ct.cast(t.data_ptr(), ct.POINTER(ct.c_int64))


def plan_summary(buffer_bytes, host_bytes, runs, gates=None, flag_count=0, max_runs=1 << 20):
    """Host-only validation of a job: (units, pieces, bytes) after collapsing
    contiguous runs; raises ValueError with the engine's reason."""
    sizes = (ct.c_uint64 * len(buffer_bytes))(*buffer_bytes)
    units, pieces, nbytes = ct.c_int64(), ct.c_int64(), ct.c_uint64()
    rc = NV.lib().qv_kvcopy_plan(sizes, len(buffer_bytes), host_bytes, _rows(runs, 7, "copy runs"), runs.shape[0],
                                 None if gates is None else _rows(gates, 2, "page gates"), flag_count, max_runs,
                                 ct.byref(units), ct.byref(pieces), ct.byref(nbytes))
    if rc:
        raise ValueError(_kv_err())
    return units.value, pieces.value, nbytes.value


class KvCopy:
    def __init__(self, device, gpu, host, segment_bytes=8 << 20, max_jobs=8, max_runs=1 << 20, pitched=True):
        device = torch.device(device)
        if not gpu or any(not t.is_cuda or t.device != device or not t.is_contiguous() for t in gpu):
            raise ValueError("expected contiguous device buffers on the engine's device")
        if host.device.type != "cpu" or not host.is_pinned() or not host.is_contiguous():
            raise ValueError("the host pool must be a contiguous pinned CPU tensor")
        self.device, self.gpu, self.host = device, list(gpu), host
        ptrs = (ct.c_void_p * len(gpu))(*[t.data_ptr() for t in gpu])
        sizes = (ct.c_uint64 * len(gpu))(*[t.numel() * t.element_size() for t in gpu])
        self._h = NV.lib().qv_kvcopy_create(device.index or 0, ptrs, sizes, len(gpu), host.data_ptr(),
                                            host.numel() * host.element_size(), segment_bytes, max_jobs, max_runs,
                                            int(bool(pitched)))
        if not self._h:
            raise ValueError(_kv_err())
        self.max_jobs = max_jobs
        self.flags = None

    def _check(self, rc):
        if rc == -2:
            raise TimeoutError("KV copy wait deadline expired")
        if rc == -1:
            raise ValueError(_kv_err())
        if rc < 0:
            raise RuntimeError(_kv_err())
        return rc

    def submit(self, job_id, generation, runs, store, producer=None, gates=None):
        producer = producer or torch.cuda.current_stream(self.device)
        rc = NV.lib().qv_kvcopy_submit(self._h, job_id, generation, _rows(runs, 7, "copy runs"), runs.shape[0],
                                       int(bool(store)), ct.c_void_p(producer.cuda_stream),
                                       None if gates is None else _rows(gates, 2, "page gates"))
        return bool(self._check(rc))

    def set_ready(self, flags):
        if flags.device.type != "cpu" or flags.dtype != torch.int64 or flags.dim() != 1 or not flags.is_contiguous():
            raise ValueError("ready flags: contiguous CPU int64 vector")
        self._check(NV.lib().qv_kvcopy_set_ready(self._h, ct.cast(flags.data_ptr(), ct.POINTER(ct.c_int64)),
                                                 flags.numel()))
        self.flags = flags

    def cancel(self, job_id, generation):
        return bool(self._check(NV.lib().qv_kvcopy_cancel(self._h, job_id, generation)))

    def _results(self, fn):
        buf = (NV.QvKvCopyResult * self.max_jobs)()
        n = self._check(fn(self._h, buf, self.max_jobs))
        return [KvCopyResult(r.job_id, r.generation, r.bytes, r.segments, bool(r.cancelled), r.device_ms,
                             r.first_issue_ns, r.last_done_ns) for r in buf[:n]]

    def poll(self):
        return self._results(NV.lib().qv_kvcopy_poll)

    def snapshot(self):
        return self._results(NV.lib().qv_kvcopy_snapshot)

    def wait(self, ids, timeout_ms=30000):
        arr = (ct.c_uint64 * len(ids))(*ids)
        self._check(NV.lib().qv_kvcopy_wait(self._h, arr, len(ids), timeout_ms))

    def drain(self, timeout_ms=30000):
        self._check(NV.lib().qv_kvcopy_drain(self._h, timeout_ms))

    def close(self):
        self._check(NV.lib().qv_kvcopy_close(self._h))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            NV.lib().qv_kvcopy_destroy(h)
            self._h = None
