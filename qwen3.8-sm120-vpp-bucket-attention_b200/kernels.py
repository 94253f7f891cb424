"""Torch-facing operators over the C ABI (one function per kernel entry point).

Mirrors the reference's operator wrappers (``kernels/nvfp4_norm_pack.py:115-159``,
``kernels/nvfp4_attention_front.py:145-237``): arguments are validated on the
host (``ValueError``), outputs are allocated by the caller side in torch, the
launch goes to the current torch stream, and a non-zero launch status raises
``RuntimeError``.  There is no CPU path: every call enters the CUDA library.
"""

import ctypes as ct
import math

import torch

from . import _native as N


class LaunchProfile:
    """Optional launch accounting: counts every kernel entry point called and,
    when ``timing`` is set, brackets each launch with CUDA events on the
    launching stream together with its algorithmic work (FLOPs or bytes)."""

    def __init__(self, timing=False):
        self.timing = timing
        self.launches = 0
        self.records = []  # (name, work, unit, start_event, end_event)

    def launch(self, name, work, unit, stream_dev, fn):
        self.launches += 1
        if not self.timing:
            return fn()
        stream = torch.cuda.current_stream(stream_dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        rc = fn()
        e1.record(stream)
        self.records.append((name, work, unit, e0, e1))
        return rc

    def summary(self):
        """{name: dict(launches, ms, work, unit)} over the recorded launches."""
        out = {}
        for name, work, unit, e0, e1 in self.records:
            d = out.setdefault(name, dict(launches=0, ms=0.0, work=0.0, unit=unit))
            d["launches"] += 1
            d["ms"] += e0.elapsed_time(e1)
            d["work"] += work
        return out


PROFILE = None


def _run(name, work, unit, dev, fn):
    if PROFILE is None:
        return fn()
    return PROFILE.launch(name, work, unit, dev, fn)


def _ptr(t):
    return None if t is None else ct.c_void_p(t.data_ptr())


def _stream(dev):
    return ct.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("the prefill kernels take CUDA tensors only")


def scale_groups_padded(k):
    return ((k // 16) + 3) // 4 * 4


def scale_buffer_bytes(rows, k):
    return (rows + 127) // 128 * 128 * scale_groups_padded(k)


def norm_pack(x, residual, gamma, global_scale, *, eps=1e-6, weight_offset=1.0, q=None, scales=None,
              updated=None, want_updated=True):
    """Residual add + RMSNorm -> NVFP4 (e2m1 codes + swizzled e4m3 scales) and
    the bf16 updated residual.  ``residual=None`` is the first layer."""
    _cuda(x, residual, gamma, global_scale)
    rows, h = x.shape
    if x.dtype != torch.bfloat16 or gamma.dtype != torch.bfloat16 or tuple(gamma.shape) != (h,):
        raise ValueError("norm_pack expects bf16 [rows, H] input and bf16 [H] gamma")
    if residual is not None and (residual.shape != x.shape or residual.dtype != x.dtype):
        raise ValueError("residual must match x")
    if global_scale.dtype != torch.float32 or global_scale.numel() != 1:
        raise ValueError("global scale must be one fp32 device scalar")
    if q is None:
        q = torch.empty((rows, h // 2), dtype=torch.uint8, device=x.device)
    if scales is None:
        scales = torch.empty(scale_buffer_bytes(rows, h), dtype=torch.uint8, device=x.device)
    if updated is None and want_updated:
        updated = torch.empty_like(x)
    N.check(_run("norm_pack", rows * (h * 2 * (2 if residual is not None else 1) + (2 * h if updated is not None else 0) + h // 2 + h // 16), "B", x.device, lambda: N.lib().qi_norm_pack(_ptr(x), _ptr(residual), _ptr(gamma), _ptr(global_scale), _ptr(q), _ptr(scales),
                                 _ptr(updated), rows, h, eps, weight_offset, _stream(x.device))), "qi_norm_pack")
    return q, scales, updated


def rms_norm(x, residual, gamma, *, eps=1e-6, weight_offset=1.0, out=None, updated=None):
    _cuda(x, residual, gamma)
    rows, h = x.shape
    if out is None:
        out = torch.empty_like(x)
    N.check(_run("rms_norm", rows * h * 2 * (3 if residual is not None else 2), "B", x.device, lambda: N.lib().qi_rms_norm(_ptr(x), _ptr(residual), _ptr(gamma), _ptr(out), _ptr(updated), rows, h, eps,
                                weight_offset, _stream(x.device))), "qi_rms_norm")
    return out


class PagedKV:
    """NVFP4 paged KV of one layer: codes [pages, page_size, Hkv, D/2] u8 and
    E4M3 scales [pages, page_size, Hkv, D/16] u8, for K and for V."""

    def __init__(self, pages, page_size, kvheads, head_dim, device):
        self.page_size, self.kvheads, self.head_dim = page_size, kvheads, head_dim
        shape = (pages, page_size, kvheads, head_dim // 2)
        sshape = (pages, page_size, kvheads, head_dim // 16)
        self.k = torch.zeros(shape, dtype=torch.uint8, device=device)
        self.v = torch.zeros(shape, dtype=torch.uint8, device=device)
        self.ks = torch.zeros(sshape, dtype=torch.uint8, device=device)
        self.vs = torch.zeros(sshape, dtype=torch.uint8, device=device)

    @classmethod
    def wrap(cls, k, v, ks, vs):
        """A view over existing cache tensors (codes [pages, page, Hkv, D/2],
        scales [pages, page, Hkv, D/16], uint8)."""
        self = object.__new__(cls)
        if k.dtype != torch.uint8 or k.ndim != 4 or v.shape != k.shape or ks.shape != vs.shape \
                or ks.shape[:3] != k.shape[:3] or ks.shape[3] * 8 != k.shape[3]:
            raise ValueError("expected NVFP4 caches [pages, page, Hkv, D/2] and scales [pages, page, Hkv, D/16]")
        self.k, self.v, self.ks, self.vs = k, v, ks.view(torch.uint8), vs.view(torch.uint8)
        self.page_size, self.kvheads, self.head_dim = k.shape[1], k.shape[2], k.shape[3] * 2
        return self

    @property
    def pages(self):
        return self.k.shape[0]

    def view(self):
        v = N.QiKvView()
        v.k_cache, v.v_cache = self.k.data_ptr(), self.v.data_ptr()
        v.k_scales, v.v_scales = self.ks.data_ptr(), self.vs.data_ptr()
        v.kvheads, v.head_dim, v.page_size = self.kvheads, self.head_dim, self.page_size
        v.data_page, v.data_row, v.data_head = self.k.stride(0), self.k.stride(1), self.k.stride(2)
        v.sf_page, v.sf_row, v.sf_head = self.ks.stride(0), self.ks.stride(1), self.ks.stride(2)
        return v


def qk_rope_kv_append(qkv, positions, q_weight, k_weight, cos_sin, slots, kv, k_global, v_global, *, qheads,
                      kvheads, head_dim, eps=1e-6, weight_offset=1.0, q=None, gate=None, want_gate=True,
                      status=None):
    """QK-norm + RoPE (rotary == head_dim) + gate split + NVFP4 paged KV append."""
    _cuda(qkv, positions, q_weight, k_weight, cos_sin, slots, k_global, v_global)
    rows = qkv.shape[0]
    d = head_dim
    if qkv.dtype != torch.bfloat16 or qkv.stride(-1) != 1 or qkv.shape[1] != (2 * qheads + 2 * kvheads) * d:
        raise ValueError("qkv must be bf16 [rows, (2Hq + 2Hkv) D]")
    if cos_sin.dtype not in (torch.float32, torch.bfloat16) or cos_sin.shape[1] != d:
        raise ValueError("cos_sin must be [maxpos, D] fp32 or bf16")
    if positions.dtype not in (torch.int32, torch.int64) or slots.dtype not in (torch.int32, torch.int64):
        raise ValueError("positions and slots are int32 or int64")
    if q is None:
        q = torch.empty((rows, qheads * d), dtype=torch.bfloat16, device=qkv.device)
    if gate is None and want_gate:
        gate = torch.empty((rows, qheads * d), dtype=torch.bfloat16, device=qkv.device)
    p = N.QiFront()
    p.qkv, p.q_weight, p.k_weight, p.cos_sin = qkv.data_ptr(), q_weight.data_ptr(), k_weight.data_ptr(), cos_sin.data_ptr()
    p.positions, p.slots = positions.data_ptr(), slots.data_ptr()
    p.k_global, p.v_global = k_global.data_ptr(), v_global.data_ptr()
    p.k_cache, p.v_cache, p.k_scales, p.v_scales = kv.k.data_ptr(), kv.v.data_ptr(), kv.ks.data_ptr(), kv.vs.data_ptr()
    p.q = q.data_ptr()
    p.gate = gate.data_ptr() if gate is not None else None
    p.status = status.data_ptr() if status is not None else None
    p.rows, p.qheads, p.kvheads, p.head_dim = rows, qheads, kvheads, d
    p.slot_rows, p.pages, p.page_size = slots.numel(), kv.pages, kv.page_size
    p.cos_float = int(cos_sin.dtype == torch.float32)
    p.pos_long, p.slot_long = int(positions.dtype == torch.int64), int(slots.dtype == torch.int64)
    p.input_row, p.cos_row = qkv.stride(0), cos_sin.stride(0)
    p.q_row = q.stride(0)
    p.gate_row = gate.stride(0) if gate is not None else 0
    p.data_page, p.data_row, p.data_head = kv.k.stride(0), kv.k.stride(1), kv.k.stride(2)
    p.sf_page, p.sf_row, p.sf_head = kv.ks.stride(0), kv.ks.stride(1), kv.ks.stride(2)
    p.eps, p.weight_offset = eps, weight_offset
    # bytes per row: read q, k, v (and the gate when split) + cos/sin; write q
    # (and the gate), K/V codes and scales
    split = 2 * qheads * d * 2 if gate is not None else 0
    work = rows * ((qheads + 2 * kvheads) * d * 2 + d * 4 + qheads * d * 2 + kvheads * (d + d // 8) + split)
    N.check(_run("qk_rope_kv_append", work, "B", qkv.device,
                 lambda: N.lib().qi_qk_rope_kv_append(ct.byref(p), _stream(qkv.device))), "qi_qk_rope_kv_append")
    return q, gate


def gate_fp8(out, gate, *, fp8=None, scale=None, head_dim=None, head_stride=None):
    """bf16(out * bf16(sigmoid(gate))) -> E4M3 with a per-row fp32 scale.
    ``gate`` is a compact [rows, cols] tensor, or (with ``head_dim`` and
    ``head_stride``) a view whose head h starts h * head_stride elements into
    each row, e.g. ``qkv[:, D:]`` with head_stride 2D (the gate halves of the
    QKV projection, read in place)."""
    _cuda(out, gate)
    rows, cols = out.shape
    hd = cols if head_dim is None else head_dim
    hs = 0 if head_stride is None else head_stride
    if gate.stride(-1) != 1 or gate.shape[0] != rows or (head_dim is None and gate.shape[1] != cols) \
            or (head_dim is not None and (cols // hd - 1) * hs + hd > gate.shape[1]):
        raise ValueError("gate must cover [rows, cols] (compact or per head)")
    if fp8 is None:
        fp8 = torch.empty((rows, cols), dtype=torch.uint8, device=out.device)
    if scale is None:
        scale = torch.empty(rows, dtype=torch.float32, device=out.device)
    N.check(_run("gate_fp8", rows * (cols * 5 + 4), "B", out.device,
                 lambda: N.lib().qi_gate_fp8_heads(_ptr(out), _ptr(gate), out.stride(0), gate.stride(0), hs, hd,
                                                   _ptr(fp8), fp8.stride(0), _ptr(scale), rows, cols,
                                                   _stream(out.device))), "qi_gate_fp8_heads")
    return fp8, scale


def gate_fp8_static(out, gate, scale, *, fp8=None, head_dim=None, head_stride=None):
    """The reference's form of the FP8 epilogue: e4m3(bf16(out * bf16(sigmoid(gate))) / scale)
    with one static fp32 device scalar ``scale``; gate addressing as :func:`gate_fp8`."""
    _cuda(out, gate, scale)
    rows, cols = out.shape
    hd = cols if head_dim is None else head_dim
    hs = 0 if head_stride is None else head_stride
    if scale.dtype != torch.float32 or scale.numel() != 1:
        raise ValueError("scale must be one fp32 device scalar")
    if fp8 is None:
        fp8 = torch.empty((rows, cols), dtype=torch.uint8, device=out.device)
    N.check(_run("gate_fp8", rows * cols * 5, "B", out.device,
                 lambda: N.lib().qi_gate_fp8_static(_ptr(out), _ptr(gate), out.stride(0), gate.stride(0), hs, hd,
                                                    _ptr(fp8), fp8.stride(0), _ptr(scale), rows, cols,
                                                    _stream(out.device))), "qi_gate_fp8_static")
    return fp8


def _gemm_struct(kind, epilogue, m, n, k, a, b, sfa=None, sfb=None, alpha=None, alpha_value=1.0):
    g = N.QiGemm()
    g.kind, g.epilogue, g.m, g.n, g.k = kind, epilogue, m, n, k
    g.a, g.b = a.data_ptr(), b.data_ptr()
    g.sfa = sfa.data_ptr() if sfa is not None else None
    g.sfb = sfb.data_ptr() if sfb is not None else None
    g.alpha = alpha.data_ptr() if alpha is not None else None
    g.alpha_value = alpha_value
    return g


def gemm_nvfp4(a, sfa, b, sfb, *, m, n, k, alpha=None, alpha_value=1.0, out=None, out_dtype=torch.bfloat16):
    """A [m, k/2] NVFP4 . B [n, k/2]^T with block scales -> bf16 (or fp32) [m, n]."""
    _cuda(a, sfa, b, sfb, alpha)
    epi = N.EPI_BF16 if out_dtype == torch.bfloat16 else N.EPI_F32
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=a.device)
    g = _gemm_struct(N.GEMM_NVFP4, epi, m, n, k, a, b, sfa, sfb, alpha, alpha_value)
    g.out, g.ldo = out.data_ptr(), out.stride(0)
    N.check(_run("gemm_nvfp4" if g.kind == N.GEMM_NVFP4 else "gemm_e4m3", 2.0 * m * n * k, "FLOP", a.device, lambda: N.lib().qi_gemm(ct.byref(g), _stream(a.device))), "qi_gemm")
    return out


def gemm_swiglu_nvfp4(a, sfa, b, sfb, act_global, *, m, n, k, alpha=None, alpha_value=1.0, act_q=None,
                      act_sf=None):
    """gate_up GEMM with the SiLU-and-mul + NVFP4 epilogue: output [m, n/4]
    codes (n/2 channels) and the swizzled scales of K = n/2."""
    _cuda(a, sfa, b, sfb, alpha, act_global)
    inter = n // 2
    if act_q is None:
        act_q = torch.empty((m, inter // 2), dtype=torch.uint8, device=a.device)
    if act_sf is None:
        act_sf = torch.empty(scale_buffer_bytes(m, inter), dtype=torch.uint8, device=a.device)
    g = _gemm_struct(N.GEMM_NVFP4, N.EPI_SWIGLU_NVFP4, m, n, k, a, b, sfa, sfb, alpha, alpha_value)
    g.act_q, g.act_sf, g.act_global, g.act_ld = act_q.data_ptr(), act_sf.data_ptr(), act_global.data_ptr(), act_q.stride(0)
    N.check(_run("gemm_nvfp4" if g.kind == N.GEMM_NVFP4 else "gemm_e4m3", 2.0 * m * n * k, "FLOP", a.device, lambda: N.lib().qi_gemm(ct.byref(g), _stream(a.device))), "qi_gemm")
    return act_q, act_sf


def swiglu_nvfp4(gate_up, act_global, *, act_q=None, act_sf=None):
    """bf16 gate_up [rows, 2I] (128-column gate/up blocks) -> NVFP4 act codes
    [rows, I/2] and swizzled scales: act = bf16(silu(gate) * up)."""
    _cuda(gate_up, act_global)
    rows, n = gate_up.shape
    inter = n // 2
    if act_q is None:
        act_q = torch.empty((rows, inter // 2), dtype=torch.uint8, device=gate_up.device)
    if act_sf is None:
        act_sf = torch.empty(scale_buffer_bytes(rows, inter), dtype=torch.uint8, device=gate_up.device)
    N.check(_run("swiglu_nvfp4", rows * (2 * n + inter // 2 + inter // 16), "B", gate_up.device,
                 lambda: N.lib().qi_swiglu_nvfp4(_ptr(gate_up), gate_up.stride(0), rows, inter, _ptr(act_global),
                                                 _ptr(act_q), act_q.stride(0), _ptr(act_sf),
                                                 _stream(gate_up.device))), "qi_swiglu_nvfp4")
    return act_q, act_sf


_LM_WORKSPACE = {}


def lm_head_argmax(hidden, weight, *, tokens=None, logits=None):
    """Greedy output token per row: argmax_v <hidden[r], weight[v]> (bf16
    inputs, fp32 logits, lowest index on ties).  ``logits``: optional fp32
    [rows, vocab] to receive the logits.  Returns int32 tokens [rows]."""
    _cuda(hidden, weight)
    rows, dim = hidden.shape
    vocab = weight.shape[0]
    dev = hidden.device
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _LM_WORKSPACE.get(key)
    if ws is None:
        ws = torch.zeros(N.lib().qi_lm_head_workspace_bytes(), dtype=torch.uint8, device=dev)
        _LM_WORKSPACE[key] = ws
    if tokens is None:
        tokens = torch.empty(rows, dtype=torch.int32, device=dev)
    N.check(_run("lm_head", vocab * dim * 2 + rows * dim * 2, "B", dev,
                 lambda: N.lib().qi_lm_head_argmax(_ptr(hidden), hidden.stride(0), rows, dim, _ptr(weight), vocab,
                                                   _ptr(logits), _ptr(ws), _ptr(tokens), _stream(dev))),
            "qi_lm_head_argmax")
    return tokens


def gemm_e4m3(a, b, *, m, n, k, row_scale=None, col_scale=None, alpha_value=1.0, out=None,
              out_dtype=torch.bfloat16):
    """A [m, k] E4M3 . B [n, k]^T -> bf16 scaled by row_scale[m] * col_scale[n]
    (or fp32 times alpha_value when out_dtype is float32)."""
    _cuda(a, b, row_scale, col_scale)
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=a.device)
    if out_dtype == torch.float32:
        epi = N.EPI_F32
    else:
        epi = N.EPI_BF16_ROWCOL if row_scale is not None else N.EPI_BF16
    g = _gemm_struct(N.GEMM_E4M3, epi, m, n, k, a, b, alpha_value=alpha_value)
    g.row_scale = row_scale.data_ptr() if row_scale is not None else None
    g.col_scale = col_scale.data_ptr() if col_scale is not None else None
    g.out, g.ldo = out.data_ptr(), out.stride(0)
    N.check(_run("gemm_nvfp4" if g.kind == N.GEMM_NVFP4 else "gemm_e4m3", 2.0 * m * n * k, "FLOP", a.device, lambda: N.lib().qi_gemm(ct.byref(g), _stream(a.device))), "qi_gemm")
    return out


def kv_dequant(kv, block_table, tokens, *, first=0, k_out=None, vt_out=None):
    """Paged NVFP4 KV of one request -> f16 K [Hkv, capacity, D] and V^T
    [Hkv, D, vt_row] (exact e2m1 x e4m3) for tokens [first, tokens); ``first``
    a multiple of 64 (0: the whole history).  Without outputs, buffers of
    exactly ``tokens`` (vt_row rounded up to 64) are allocated."""
    _cuda(block_table)
    d = kv.head_dim
    if k_out is None:
        k_out = torch.empty((kv.kvheads, tokens, d), dtype=torch.float16, device=kv.k.device)
    if vt_out is None:
        vt_out = torch.empty((kv.kvheads, d, (tokens + 63) // 64 * 64), dtype=torch.float16, device=kv.k.device)
    if k_out.shape[0] != kv.kvheads or k_out.shape[2] != d or not k_out.is_contiguous() \
            or vt_out.shape[:2] != (kv.kvheads, d) or not vt_out.is_contiguous():
        raise ValueError("k_out [Hkv, capacity, D] and vt_out [Hkv, D, vt_row], contiguous")
    view = kv.view()
    n = tokens - first
    N.check(_run("kv_dequant", n * kv.kvheads * (d + d // 8 + 4 * d), "B", kv.k.device,
                 lambda: N.lib().qi_kv_dequant_range(ct.byref(view), _ptr(block_table), first, tokens, _ptr(k_out),
                                                     k_out.shape[1], _ptr(vt_out), vt_out.shape[2],
                                                     _stream(kv.k.device))), "qi_kv_dequant_range")
    return k_out, vt_out


_ATTN_WORKSPACE = {}


def attention_workspace(device, head_dim):
    """Zero-filled key-range split workspace for :func:`prefill_attention` on
    ``device`` (one per device and head_dim, cached; calls on one stream may
    share it)."""
    device = torch.device(device)
    key = (device.index if device.index is not None else torch.cuda.current_device(), head_dim)
    ws = _ATTN_WORKSPACE.get(key)
    if ws is None:
        nbytes = ct.c_int64(0)
        with torch.cuda.device(key[0]):
            N.check(N.lib().qi_prefill_attention_workspace_bytes(head_dim, ct.byref(nbytes)),
                    "qi_prefill_attention_workspace_bytes")
        ws = torch.zeros(nbytes.value, dtype=torch.uint8, device=torch.device("cuda", key[0]))
        _ATTN_WORKSPACE[key] = ws
    return ws


def attention_workspace_new(device, head_dim):
    """A fresh zero-filled key-range split workspace (not the cached one): for
    attention calls on a stream that may run concurrently with another."""
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    nbytes = ct.c_int64(0)
    with torch.cuda.device(idx):
        N.check(N.lib().qi_prefill_attention_workspace_bytes(head_dim, ct.byref(nbytes)),
                "qi_prefill_attention_workspace_bytes")
    return torch.zeros(nbytes.value, dtype=torch.uint8, device=torch.device("cuda", idx))


def prefill_attention(q, k, vt, *, history, qheads, kvheads, head_dim, k_global, v_global, out=None,
                      softmax_scale=None, status=None, kv_tokens=None, workspace=None):
    """Causal GQA attention of ``rows`` queries at positions history.. over
    keys 0 .. history+rows-1 held as f16 K / V^T (from :func:`kv_dequant`).
    ``workspace``: the key-range split workspace (default: the device's cached
    one from :func:`attention_workspace`)."""
    _cuda(q, k, vt, k_global, v_global)
    if workspace is None:
        workspace = attention_workspace(q.device, head_dim)
    rows = q.shape[0]
    if out is None:
        out = torch.empty((rows, qheads * head_dim), dtype=torch.bfloat16, device=q.device)
    p = N.QiAttention()
    p.q, p.k, p.vt, p.out = q.data_ptr(), k.data_ptr(), vt.data_ptr(), out.data_ptr()
    p.k_global, p.v_global = k_global.data_ptr(), v_global.data_ptr()
    p.status = status.data_ptr() if status is not None else None
    p.rows, p.history = rows, history
    p.kv_tokens = kv_tokens if kv_tokens is not None else k.shape[1]
    p.qheads, p.kvheads, p.head_dim = qheads, kvheads, head_dim
    p.q_row, p.out_row, p.vt_row = q.stride(0), out.stride(0), vt.shape[2]
    p.softmax_scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(head_dim)
    p.workspace, p.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    N.check(_run("attention", 4 * qheads * head_dim * (rows * history + rows * (rows + 1) // 2), "FLOP", q.device, lambda: N.lib().qi_prefill_attention(ct.byref(p), _stream(q.device))), "qi_prefill_attention")
    return out


def paged_prefill_attention(q, kv, block_table, *, history, qheads, k_global, v_global, out=None,
                            softmax_scale=None, status=None, workspace=None):
    """Causal GQA attention of ``rows`` queries at positions history.. over the
    request's keys 0 .. history+rows-1, read straight from the paged NVFP4
    cache ``kv`` (a :class:`PagedKV`) through ``block_table``.  ``workspace``:
    the key-range split workspace (default: the device's cached one)."""
    _cuda(q, block_table, k_global, v_global)
    d = kv.head_dim
    if workspace is None:
        workspace = attention_workspace(q.device, d)
    rows = q.shape[0]
    if block_table.dtype != torch.int32 or block_table.numel() * kv.page_size < history + rows:
        raise ValueError("block_table: int32 with a page for every key")
    if out is None:
        out = torch.empty((rows, qheads * d), dtype=torch.bfloat16, device=q.device)
    p = N.QiPagedAttention()
    p.q, p.out, p.kv, p.block_table = q.data_ptr(), out.data_ptr(), kv.view(), block_table.data_ptr()
    p.k_global, p.v_global = k_global.data_ptr(), v_global.data_ptr()
    p.status = status.data_ptr() if status is not None else None
    p.rows, p.history, p.qheads = rows, history, qheads
    p.q_row, p.out_row = q.stride(0), out.stride(0)
    p.softmax_scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(d)
    p.workspace, p.workspace_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    N.check(_run("attention", 4 * qheads * d * (rows * history + rows * (rows + 1) // 2), "FLOP", q.device,
                 lambda: N.lib().qi_paged_prefill_attention(ct.byref(p), _stream(q.device))),
            "qi_paged_prefill_attention")
    return out


def nvfp4_quantize(w, global_scale, *, q=None, scales=None):
    """fp32 [rows, K] -> NVFP4 codes [rows, K/2] + swizzled scales."""
    _cuda(w, global_scale)
    rows, k = w.shape
    if w.dtype != torch.float32 or not w.is_contiguous():
        raise ValueError("weights must be contiguous fp32")
    if q is None:
        q = torch.empty((rows, k // 2), dtype=torch.uint8, device=w.device)
    if scales is None:
        scales = torch.zeros(scale_buffer_bytes(rows, k), dtype=torch.uint8, device=w.device)
    N.check(_run("nvfp4_quantize", rows * k * 4, "B", w.device, lambda: N.lib().qi_nvfp4_quantize(_ptr(w), rows, k, _ptr(global_scale), _ptr(q), _ptr(scales),
                                      _stream(w.device))), "qi_nvfp4_quantize")
    return q, scales


def fp8_quantize_rows(w, *, q=None, scales=None):
    _cuda(w)
    rows, k = w.shape
    if q is None:
        q = torch.empty((rows, k), dtype=torch.uint8, device=w.device)
    if scales is None:
        scales = torch.empty(rows, dtype=torch.float32, device=w.device)
    N.check(_run("fp8_quantize_rows", rows * k * 5, "B", w.device, lambda: N.lib().qi_fp8_quantize_rows(_ptr(w), rows, k, _ptr(q), _ptr(scales), _stream(w.device))), "qi_fp8_quantize_rows")
    return q, scales
