"""Bucket decode attention over the paged NVFP4 KV cache (one query token per
request) -- the host side of ``qi_decode_assign`` / ``qi_decode_attention``.

Mirrors the reference's native-XQA task backend
(``src/qwen_infra/kernels/nvfp4_bucket_xqa.py:248-540``): a ``TaskPlan`` owns
the device plan buffers (tasks, requests, buckets, header) and is refreshed on
the GPU from the device lengths by ``assign()``; a ``Workspace`` owns the
per-layer partials, semaphores and output, ``bind()`` validates the views and
fixes the launch parameters, ``run()`` = ``assign()`` + ``compute()``.  The
route rule choosing the task mode follows
``kernels/nvfp4_kv_bucket_worker.py:9-51``.  Differences: this build's cache
(16-token pages, any power of two accepted; [pages, page, Hkv, D/2] codes in
32-byte aligned rows, head_dim 128, any Hkv with up to 16 query heads per KV
head) instead of the reference's 32-token pages with one KV head of 256; the
dequantisation multipliers are the cache's fp32 globals; q K^T is formed from
q written as four NVFP4 terms (relative error ~7e-5 of the group's largest
query value); there is no CPU path.
"""

import ctypes as ct
import math

import torch

from . import _native as N
from .kernels import PagedKV, _run

TILE = 256  # tokens per plan unit
MAX_BATCH = 32
MAX_CTAS = 340
MODES = {"intervals": 0, "cyclic": 1, "aligned": 2}


def _ceil(a, b):
    return (a + b - 1) // b


def route(lengths, *, table_width, sm_count, forced="auto", page_size=16, diagnostic=False):
    """Task mode for a batch: "persistent" (interval buckets, one CTA per
    bucket) when cyclic splitting would leave one task with at least twice the
    interval budget of tiles, "aligned" when every cyclic task holds at most
    one tile and some would be empty, else "native" (cyclic).  Batches other
    than 1, 8, 16, 24 or 32 rows, and all-empty batches, take "native"."""
    if forced not in ("auto", "native", "persistent", "aligned"):
        raise ValueError("expected auto/native/persistent/aligned route")
    supported = (isinstance(lengths, (tuple, list)) and len(lengths) in (1, 8, 16, 24, 32)
                 and type(sm_count) is int and len(lengths) <= sm_count <= MAX_CTAS
                 and type(table_width) is int and table_width >= 1
                 and all(type(n) is int and 0 <= n <= table_width * page_size for n in lengths) and any(lengths))
    if not supported:
        return dict(route="native", supported=False, reason="unsupported") if diagnostic else "native"
    tiles = [_ceil(n, TILE) for n in lengths]
    splits = min(max(1, sm_count // len(lengths)), _ceil(table_width * page_size, TILE))
    bucket = max(2, _ceil(sum(tiles), sm_count))
    critical = max(_ceil(n, splits) for n in tiles)
    empty = len(lengths) * splits - sum(min(n, splits) for n in tiles)
    auto = "persistent" if critical >= 2 * bucket else "aligned" if critical == 1 and empty > 0 else "native"
    chosen = auto if forced == "auto" else forced
    if not diagnostic:
        return chosen
    return dict(route=chosen, auto_route=auto, supported=True, forced=forced, native_splits=splits,
                native_empty_subsequences=empty, native_critical_tiles=critical, interval_tiles_per_bucket=bucket,
                reason="geometry")


def resources(group=8):
    """Kernel resources for groups of ``group`` query heads per KV head:
    registers, shared bytes, local bytes, resident CTAs per SM."""
    vals = (ct.c_int * 10)()
    N.check(N.lib().qi_decode_resources(vals), "qi_decode_resources")
    if (vals[0], vals[5], vals[6], vals[7]) != (ct.sizeof(N.QiDecode), 16, 8, 8):
        raise RuntimeError("decode C / Python ABI mismatch")
    small = group <= 8
    return dict(registers=vals[1] if small else vals[8], shared_bytes=vals[2], local_bytes=vals[3],
                resident_ctas=vals[4] if small else vals[9], threads=128)


def default_ctas(batch, kvheads, device=None, group=8):
    """Task slots that fill the GPU once: SMs x resident CTAs per SM / Hkv."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    return max(batch, min(MAX_CTAS, sms * resources(group)["resident_ctas"] // kvheads))


def _check_batch(batch, ctas):
    if type(batch) is not int or not 1 <= batch <= MAX_BATCH or type(ctas) is not int or not batch <= ctas <= MAX_CTAS:
        raise ValueError("expected 1..32 requests and batch <= ctas <= 340 task slots")


class TaskPlan:
    """Device plan buffers of one batch shape; ``prepare`` binds them to one
    device lengths buffer and mode, ``assign`` recomputes the plan on the GPU
    (graph-capturable: it reads the lengths on the device)."""

    def __init__(self, batch, *, ctas, page_size=16, device="cuda"):
        _check_batch(batch, ctas)
        if type(page_size) is not int or page_size < 1 or page_size & (page_size - 1):
            raise ValueError("the decode kernel takes pages of a power-of-two token count")
        self.batch, self.ctas, self.page_size = batch, ctas, page_size
        self.capacity = ctas + batch - 1
        self.tasks = torch.empty((self.capacity, 4), dtype=torch.int32, device=device)
        self.requests = torch.empty((batch, 2), dtype=torch.int32, device=device)
        self.buckets = torch.empty((ctas, 2), dtype=torch.int32, device=device)
        self.header = torch.empty(4, dtype=torch.int32, device=device)
        self.binding = None

    @property
    def logical_bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.tasks, self.requests, self.buckets, self.header))

    def prepare(self, lengths, *, table_width, cyclic=False, aligned=False):
        if (type(cyclic) is not bool or type(aligned) is not bool or (cyclic and aligned)
                or type(table_width) is not int or table_width < 1
                or table_width * self.page_size > 2**31 - TILE
                or lengths.device != self.tasks.device or lengths.dtype != torch.int32
                or tuple(lengths.shape) != (self.batch,) or not lengths.is_contiguous()):
            raise ValueError("expected one int32 device-length buffer of the batch and a page-table width")
        key = (lengths.data_ptr(), table_width, cyclic, aligned)
        if self.binding is not None:
            if key != self.binding:
                raise RuntimeError("a bound task plan cannot be rebound; release_binding() first")
            return self
        self.lengths, self.binding = lengths, key
        self.table_width, self.mode = table_width, 1 if cyclic else 2 if aligned else 0
        return self

    def fill(self, p):
        """Write the plan fields of a QiDecode struct."""
        for name in ("tasks", "requests", "buckets", "header"):
            setattr(p, name, getattr(self, name).data_ptr())
        p.lengths = self.lengths.data_ptr()
        p.batch, p.ctas, p.table_width, p.mode = self.batch, self.ctas, self.table_width, self.mode

    def assign(self, kv_view=None):
        if self.binding is None:
            raise RuntimeError("the task plan is not bound")
        p = N.QiDecode()
        self.fill(p)
        if kv_view is not None:
            p.kv = kv_view
        else:
            p.kv.head_dim, p.kv.kvheads, p.kv.page_size = 128, 1, self.page_size
        p.qheads = p.kv.kvheads
        dev = self.tasks.device
        N.check(_run("decode_assign", 0, "B", dev,
                     lambda: N.lib().qi_decode_assign(ct.byref(p), ct.c_void_p(torch.cuda.current_stream(dev).cuda_stream))),
                "qi_decode_assign")

    def release_binding(self):
        for name in ("lengths",):
            if hasattr(self, name):
                delattr(self, name)
        self.binding = None

    def inspect(self):
        count = int(self.header[1].item())
        return dict(tasks=self.tasks[:count].cpu().tolist(), requests=self.requests.cpu().tolist(),
                    buckets=self.buckets.cpu().tolist(), header=self.header.cpu().tolist())


class Workspace:
    """Partials, semaphores and output of one attention layer for a batch shape.

    Sequential layers may share one ``TaskPlan`` (``plan=``) with their own
    workspaces.  Calls through one workspace must be ordered on one stream."""

    def __init__(self, batch, *, qheads, kvheads, ctas=None, page_size=16, device="cuda", plan=None):
        device = torch.device(device)
        if type(qheads) is not int or type(kvheads) is not int or kvheads < 1 or qheads % kvheads \
                or qheads // kvheads > 16:
            raise ValueError("expected qheads = G * kvheads with G <= 16")
        if ctas is None:
            ctas = default_ctas(batch, kvheads, device, group=qheads // kvheads)
        _check_batch(batch, ctas)
        self.batch, self.ctas, self.qheads, self.kvheads = batch, ctas, qheads, kvheads
        self.plan = plan if plan is not None else TaskPlan(batch, ctas=ctas, page_size=page_size, device=device)
        if self.plan.batch != batch or self.plan.ctas != ctas or self.plan.tasks.device != device:
            raise ValueError("a shared plan must match the batch, the task slots and the device")
        self.capacity = ctas + batch - 1
        size = N.lib().qi_decode_scratch_bytes(self.capacity, kvheads)
        if not size:
            raise ValueError("unsupported scratch capacity")
        self.scratch = torch.empty(size, dtype=torch.uint8, device=device)
        self.semaphores = torch.zeros(batch * kvheads, dtype=torch.int32, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.output = torch.empty((batch, qheads, 128), dtype=torch.bfloat16, device=device)

    @property
    def exclusive_bytes(self):
        return sum(t.numel() * t.element_size() for t in (self.semaphores, self.scratch, self.output))

    def bind(self, q, kv, table, lengths, *, k_global, v_global, softmax_scale=None, cyclic=False, aligned=False,
             persistent=False, output=None, gate=None, output_scale=None):
        """q: bf16 [batch, qheads, 128]; kv: ``PagedKV`` (head_dim 128); table:
        int32 [batch, width] page ids; lengths: int32 [batch] keys per request
        (device); k_global / v_global: fp32 device scalars of the cache.  With
        ``gate`` (bf16 like q) and ``output_scale`` (fp32 device scalar) the
        output is e4m3 codes (uint8) of bf16(bf16(out) * bf16(sigmoid(gate))) /
        output_scale."""
        dev = self.output.device
        tail = gate is not None
        out = output if output is not None else (self.output if not tail else
                                                 torch.empty(q.shape, dtype=torch.uint8, device=dev))
        if (not isinstance(kv, PagedKV) or kv.head_dim != 128 or kv.kvheads != self.kvheads
                or kv.page_size != self.plan.page_size or kv.k.device != dev
                or q.device != dev or q.dtype != torch.bfloat16 or tuple(q.shape) != (self.batch, self.qheads, 128)
                or not q.is_contiguous()
                or table.device != dev or table.dtype != torch.int32 or table.ndim != 2
                or table.shape[0] != self.batch or not table.is_contiguous()
                or out.device != dev or tuple(out.shape) != tuple(q.shape) or not out.is_contiguous()
                or out.dtype != (torch.uint8 if tail else torch.bfloat16)
                or (persistent and (cyclic or aligned))):
            raise ValueError("expected bf16 q [batch, qheads, 128], a matching PagedKV, int32 page table")
        if tail and (gate.device != dev or gate.dtype != torch.bfloat16 or gate.shape != q.shape
                     or not gate.is_contiguous() or output_scale is None or output_scale.device != dev
                     or output_scale.dtype != torch.float32 or output_scale.numel() != 1):
            raise ValueError("the FP8 tail takes a bf16 gate like q and an fp32 device output scale")
        if not tail and output_scale is not None:
            raise ValueError("an output scale needs a gate")
        self.plan.prepare(lengths, table_width=table.shape[1], cyclic=cyclic, aligned=aligned)
        self.bound = (q, kv, table, lengths, out, gate, output_scale, k_global, v_global)
        p = N.QiDecode()
        self.plan.fill(p)
        p.q = q.data_ptr()
        p.kv = kv.view()
        p.block_table = table.data_ptr()
        p.semaphores, p.scratch, p.out = self.semaphores.data_ptr(), self.scratch.data_ptr(), out.data_ptr()
        p.gate = gate.data_ptr() if tail else None
        p.out_scale = output_scale.data_ptr() if tail else None
        p.k_global, p.v_global = k_global.data_ptr(), v_global.data_ptr()
        p.status = self.status.data_ptr()
        p.persistent = int(bool(persistent))
        p.qheads = self.qheads
        p.softmax_scale = 1.0 / math.sqrt(128) if softmax_scale is None else float(softmax_scale)
        self.params = p
        return self

    def _stream(self):
        return ct.c_void_p(torch.cuda.current_stream(self.output.device).cuda_stream)

    def assign(self):
        p = self.params
        N.check(_run("decode_assign", 0, "B", self.output.device,
                     lambda: N.lib().qi_decode_assign(ct.byref(p), self._stream())), "qi_decode_assign")

    def compute(self):
        p = self.params
        N.check(_run("decode_attention", 0, "B", self.output.device,
                     lambda: N.lib().qi_decode_attention(ct.byref(p), self._stream())), "qi_decode_attention")

    def run(self, *, assign=True):
        if assign:
            self.assign()
        self.compute()
        return self.bound[4]

    def inspect_plan(self):
        return self.plan.inspect()

    def release_bindings(self):
        for name in ("bound", "params"):
            if hasattr(self, name):
                delattr(self, name)
        self.plan.release_binding()


def decode_attention(q, kv, table, lengths, *, k_global, v_global, route_name="auto", ctas=None, gate=None,
                     output_scale=None, workspace=None, host_lengths=None):
    """One-call form: picks the task mode with ``route`` (from ``host_lengths``,
    a list of ints, when given; "native" cyclic otherwise) and runs it."""
    batch, qheads = q.shape[0], q.shape[1]
    ws = workspace or Workspace(batch, qheads=qheads, kvheads=kv.kvheads, ctas=ctas, page_size=kv.page_size,
                                device=q.device)
    name = route_name
    if name == "auto":
        name = route(list(host_lengths), table_width=table.shape[1], sm_count=ws.ctas,
                     page_size=kv.page_size) if host_lengths is not None else "native"
    ws.bind(q, kv, table, lengths, k_global=k_global, v_global=v_global, cyclic=name == "native",
            aligned=name == "aligned", persistent=name == "persistent", gate=gate, output_scale=output_scale)
    out = ws.run()
    return out, ws
