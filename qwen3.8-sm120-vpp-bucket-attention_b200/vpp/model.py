"""Virtual-stage compute of the Qwen-style NVFP4 decoder on sm_100a kernels.

Layer order (the gated-attention decoder the reference runs through vLLM,
``vllm:model_executor/models/qwen3_next.py:285-320``, wrapped by
``src/qwen_infra/vpp/model.py:83-115`` and ``vpp/producer.py:189-210``):

  norm_pack -> QKV GEMM (NVFP4) -> QK-norm/RoPE/NVFP4 KV append
  -> KV dequant + causal GQA attention -> sigmoid gate -> FP8
  -> O GEMM (E4M3) -> norm_pack -> gate_up GEMM + SwiGLU + NVFP4 -> down GEMM

A stage boundary is the pair (hidden, residual) of bf16 [rows, H] planes
(``vpp/model.py:28-47``); the first stage starts from embeddings with no
residual, the last one applies the final norm.
"""

from dataclasses import dataclass
import math

import numpy as np
import torch

from .. import kernels as K


@dataclass(frozen=True)
class ModelShape:
    layers: int
    hidden: int
    qheads: int
    kvheads: int
    head_dim: int
    intermediate: int
    eps: float = 1e-6
    rope_theta: float = 1e6
    page_size: int = 16
    vocab: int = 152064  # LM head rows (the Qwen embedding size)

    @property
    def qkv_out(self):
        return (2 * self.qheads + 2 * self.kvheads) * self.head_dim

    def linear_flops_per_token(self):
        h, d = self.hidden, self.head_dim
        return 2 * (h * self.qkv_out + self.qheads * d * h + h * 2 * self.intermediate + self.intermediate * h)

    def attention_flops(self, history, rows):
        """Causal QK^T + PV FLOPs of one layer for ``rows`` queries after ``history``."""
        pairs = rows * history + rows * (rows + 1) // 2
        return 4 * self.qheads * self.head_dim * pairs


TINY = ModelShape(layers=4, hidden=1024, qheads=16, kvheads=4, head_dim=64, intermediate=3072, vocab=4096)
QWEN27B = ModelShape(layers=64, hidden=5120, qheads=64, kvheads=8, head_dim=128, intermediate=17408)
SHAPES = {"tiny": TINY, "qwen27b": QWEN27B}

# Static activation global scales 448*6/amax (calibration-free constants for
# seeded synthetic weights) and K/V dequantisation multipliers.
ACT_GLOBAL_NORM = float(np.float32(2688.0 / 32.0))
ACT_GLOBAL_DOWN = float(np.float32(2688.0 / 64.0))
KV_GLOBAL_K = float(np.float32(16.0 / 2688.0))
KV_GLOBAL_V = float(np.float32(8.0 / 2688.0))
FINAL_NORM_SEED_OFFSET = 999_983
LM_HEAD_SEED_OFFSET = 999_979


def _seeded_normal(shape, seed, std, device, on_device):
    if on_device:
        g = torch.Generator(device=device).manual_seed(int(seed))
        return torch.randn(*shape, generator=g, dtype=torch.float32, device=device) * std
    g = torch.Generator().manual_seed(int(seed))
    return (torch.randn(*shape, generator=g, dtype=torch.float32) * std).to(device)


def _layer_seed(base, layer, idx):
    return base + layer * 16 + idx


def _interleave_gate_up(w_gate, w_up, block=128):
    i, k = w_gate.shape
    return torch.stack([w_gate.view(i // block, block, k), w_up.view(i // block, block, k)], dim=1).reshape(2 * i, k)


class NVFP4Weight:
    """NVFP4 weight [n, k]: codes [n, k/2], swizzled E4M3 scales, fp32 global."""

    def __init__(self, w_fp32):
        self.n, self.k = w_fp32.shape
        amax = float(w_fp32.abs().max().item())
        self.global_scale = float(np.float32(2688.0) / np.float32(amax))
        self.g = torch.tensor([self.global_scale], dtype=torch.float32, device=w_fp32.device)
        self.q, self.sf = K.nvfp4_quantize(w_fp32.contiguous(), self.g)


class LayerWeights:
    def __init__(self, shape, layer, device, base_seed=1234, on_device=False):
        s = shape
        h, d = s.hidden, s.head_dim

        def normal(shp, idx, std):
            return _seeded_normal(shp, _layer_seed(base_seed, layer, idx), std, device, on_device)

        self.qkv = NVFP4Weight(normal((s.qkv_out, h), 0, 0.02))
        wo = normal((h, s.qheads * d), 1, 0.02)
        self.o_q, self.o_scale = K.fp8_quantize_rows(wo.contiguous())
        del wo
        wg = normal((s.intermediate, h), 2, 0.02)
        wu = normal((s.intermediate, h), 3, 0.02)
        self.gate_up = NVFP4Weight(_interleave_gate_up(wg, wu).contiguous())
        del wg, wu
        self.down = NVFP4Weight(normal((h, s.intermediate), 4, 0.02))
        self.ln_in = normal((h,), 5, 0.05).to(torch.bfloat16)
        self.ln_post = normal((h,), 6, 0.05).to(torch.bfloat16)
        self.q_norm = normal((d,), 7, 0.05).to(torch.bfloat16)
        self.k_norm = normal((d,), 8, 0.05).to(torch.bfloat16)

        def alpha(act_g, w):
            return torch.tensor([float(np.float32(1.0) / (np.float32(act_g) * np.float32(w.global_scale)))],
                                dtype=torch.float32, device=device)

        self.alpha_qkv = alpha(ACT_GLOBAL_NORM, self.qkv)
        self.alpha_gu = alpha(ACT_GLOBAL_NORM, self.gate_up)
        self.alpha_down = alpha(ACT_GLOBAL_DOWN, self.down)

    def nbytes(self):
        ts = [self.qkv.q, self.qkv.sf, self.o_q, self.o_scale, self.gate_up.q, self.gate_up.sf, self.down.q,
              self.down.sf]
        return sum(t.numel() * t.element_size() for t in ts)


def rope_table(max_pos, head_dim, theta, device):
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    t = torch.arange(max_pos, dtype=torch.float64)
    fr = torch.outer(t, inv)
    return torch.cat([fr.cos(), fr.sin()], dim=1).to(torch.float32).to(device)


@dataclass
class ChunkContext:
    """One chunk of one request: rows at positions history .. history+rows-1."""

    request: int
    history: int
    rows: int
    positions: torch.Tensor  # int32 [rows]
    slots: torch.Tensor  # int32 [rows]
    block_table: torch.Tensor  # int32 [pages of the request]


class Workspace:
    """Per-rank scratch sized for the largest chunk and context."""

    def __init__(self, shape, max_rows, max_tokens, device):
        s = shape
        h, d = s.hidden, s.head_dim
        e = dict(device=device)
        self.q_in = torch.empty((max_rows, h // 2), dtype=torch.uint8, **e)
        self.sf_in = torch.empty(K.scale_buffer_bytes(max_rows, h), dtype=torch.uint8, **e)
        self.res1 = torch.empty((max_rows, h), dtype=torch.bfloat16, **e)
        self.qkv = torch.empty((max_rows, s.qkv_out), dtype=torch.bfloat16, **e)
        self.q = torch.empty((max_rows, s.qheads * d), dtype=torch.bfloat16, **e)
        self.att = torch.empty((max_rows, s.qheads * d), dtype=torch.bfloat16, **e)
        self.a8 = torch.empty((max_rows, s.qheads * d), dtype=torch.uint8, **e)
        self.s8 = torch.empty(max_rows, dtype=torch.float32, **e)
        self.o = torch.empty((max_rows, h), dtype=torch.bfloat16, **e)
        self.q_m = torch.empty((max_rows, h // 2), dtype=torch.uint8, **e)
        self.sf_m = torch.empty(K.scale_buffer_bytes(max_rows, h), dtype=torch.uint8, **e)
        self.act_q = torch.empty((max_rows, s.intermediate // 2), dtype=torch.uint8, **e)
        self.act_sf = torch.empty(K.scale_buffer_bytes(max_rows, s.intermediate), dtype=torch.uint8, **e)
        vt_row = (max_tokens + 63) // 64 * 64
        self.kd = torch.empty(s.kvheads * max_tokens * d, dtype=torch.float16, **e)
        self.vt = torch.empty(s.kvheads * d * vt_row, dtype=torch.float16, **e)
        self.status = torch.zeros(1, dtype=torch.int32, **e)
        self.ping = [torch.empty((max_rows, h), dtype=torch.bfloat16, **e) for _ in range(4)]
        # The attention's key-range split workspace: one per workspace, so
        # stages that run concurrently on two streams do not share it.
        self.attn_ws = K.attention_workspace_new(device, d)

    def kv_views(self, shape, tokens):
        vt_row = (tokens + 63) // 64 * 64
        kd = self.kd[: shape.kvheads * tokens * shape.head_dim].view(shape.kvheads, tokens, shape.head_dim)
        vt = self.vt[: shape.kvheads * shape.head_dim * vt_row].view(shape.kvheads, shape.head_dim, vt_row)
        return kd, vt


class StageModel:
    """The layers one rank owns (its two virtual stages), their paged NVFP4 KV
    for every request of a bank, and the stage forward."""

    def __init__(self, shape, layers, device, *, max_rows, request_tokens, base_seed=1234, on_device_init=None,
                 final_norm=False, kv_shadow=None, streams=1, attention="auto"):
        if attention not in ("auto", "paged", "f16"):
            raise ValueError("attention is auto, paged or f16")
        self.shape = shape
        self.device = torch.device(device)
        self.layers = list(layers)
        if on_device_init is None:
            on_device_init = shape.hidden > 2048
        self.weights = {l: LayerWeights(shape, l, self.device, base_seed, on_device_init) for l in self.layers}
        s = shape
        self.max_tokens = max(request_tokens)
        pages = [(t + s.page_size - 1) // s.page_size for t in request_tokens]
        offsets = np.cumsum([0] + pages)
        self.block_tables = [torch.arange(offsets[i], offsets[i + 1], dtype=torch.int32, device=self.device)
                             for i in range(len(pages))]
        self.kv = {l: K.PagedKV(int(offsets[-1]), s.page_size, s.kvheads, s.head_dim, self.device)
                   for l in self.layers}
        self.rope = rope_table(self.max_tokens, s.head_dim, s.rope_theta, self.device)
        # One workspace per concurrently running stage (streams=2: the two
        # virtual stages of a rank overlap on two CUDA streams).
        # Attention: "paged" reads the NVFP4 cache itself (no copy of the
        # cache); "f16" dequantises each chunk's new keys into an f16 K / V^T
        # copy kept per (request, layer) across the request's chunks and runs
        # the TMA-fed kernel on it (faster today: 1.74 vs 2.05 ms for 2048
        # rows over 32K keys, but 4 KB per token per layer of extra memory).
        # "auto": f16 when every request's copy fits in a third of the free
        # memory, else paged (long contexts on few GPUs).
        self.request_tokens = list(request_tokens)
        need = sum(2 * s.kvheads * ((t + 63) // 64 * 64) * s.head_dim * 2 for t in request_tokens) * len(self.layers)
        fits = self.device.type == "cuda" and need < torch.cuda.mem_get_info(self.device)[0] // 3
        if attention == "auto":
            attention = "f16" if fits else "paged"
        self.attention = attention
        self.ws_sets = [Workspace(s, max_rows, self.max_tokens if attention == "f16" else 0, self.device)
                        for _ in range(streams)]
        self.ws = self.ws_sets[0]
        f = lambda v: torch.tensor([v], dtype=torch.float32, device=self.device)
        self.g_norm, self.g_down = f(ACT_GLOBAL_NORM), f(ACT_GLOBAL_DOWN)
        self.kg, self.vg = f(KV_GLOBAL_K), f(KV_GLOBAL_V)
        self.final_gamma = self.lm_head = None
        if final_norm:  # the output rank: final norm, LM head (bf16, unquantised) and sampling
            self.final_gamma = _seeded_normal((s.hidden,), base_seed + FINAL_NORM_SEED_OFFSET, 0.05, self.device,
                                              on_device_init).to(torch.bfloat16)
            self.lm_head = _seeded_normal((s.vocab, s.hidden), base_seed + LM_HEAD_SEED_OFFSET, 0.02, self.device,
                                          on_device_init).to(torch.bfloat16)
        self.softmax_scale = 1.0 / math.sqrt(s.head_dim)
        # attention="f16": the f16 K / V^T copy of each (request, layer) is
        # kept across the request's chunks, so every chunk dequantises only
        # its own new tokens (instead of the whole history again), when it
        # fits (see above).  Zero-filled: keys past the current length read 0.
        if attention == "paged":
            kv_shadow = False
        elif kv_shadow is None:
            kv_shadow = fits
        self.kv_shadow = bool(kv_shadow)
        self.shadow = {}

    def _shadow(self, ctx, layer):
        key = (ctx.request, layer)
        if ctx.history == 0 or key not in self.shadow:
            s, t = self.shape, self.request_tokens[ctx.request]
            self.shadow[key] = (torch.zeros((s.kvheads, t, s.head_dim), dtype=torch.float16, device=self.device),
                                torch.zeros((s.kvheads, s.head_dim, (t + 63) // 64 * 64), dtype=torch.float16,
                                            device=self.device))
        return self.shadow[key]

    def chunk_context(self, request, history, rows):
        s = self.shape
        pos = torch.arange(history, history + rows, dtype=torch.int32, device=self.device)
        bt = self.block_tables[request]
        slots = bt[(pos // s.page_size).long()] * s.page_size + pos % s.page_size
        return ChunkContext(request, history, rows, pos, slots.to(torch.int32), bt)

    def layer_forward(self, layer, hidden, residual, ctx, hidden_out, residual_out, on_residual=None, ws=None,
                      split=True):
        s, w = self.shape, self.weights[layer]
        ws = ws or self.ws
        rows = ctx.rows
        h, d = s.hidden, s.head_dim
        q_in, sf_in, res1 = K.norm_pack(hidden, residual, w.ln_in, self.g_norm, eps=s.eps, q=ws.q_in[:rows],
                                        scales=ws.sf_in, updated=ws.res1[:rows])
        qkv = K.gemm_nvfp4(q_in, sf_in, w.qkv.q, w.qkv.sf, m=rows, n=s.qkv_out, k=h, alpha=w.alpha_qkv,
                           out=ws.qkv[:rows])
        kv = self.kv[layer]
        # The gate halves stay in the QKV output and the gate epilogue reads
        # them there (no split copy).
        q, _ = K.qk_rope_kv_append(qkv, ctx.positions, w.q_norm, w.k_norm, self.rope, ctx.slots, kv, self.kg,
                                   self.vg, qheads=s.qheads, kvheads=s.kvheads, head_dim=d, eps=s.eps,
                                   q=ws.q[:rows], want_gate=False, status=ws.status)
        tokens = ctx.history + rows
        attn_ws = ws.attn_ws if split else ws.attn_ws[:0]
        if self.attention == "paged":
            att = K.paged_prefill_attention(q, kv, ctx.block_table, history=ctx.history, qheads=s.qheads,
                                            k_global=self.kg, v_global=self.vg, out=ws.att[:rows],
                                            softmax_scale=self.softmax_scale, status=ws.status, workspace=attn_ws)
        else:
            if self.kv_shadow:
                kd, vt = self._shadow(ctx, layer)
                K.kv_dequant(kv, ctx.block_table, tokens, first=ctx.history // 64 * 64, k_out=kd, vt_out=vt)
            else:
                kd, vt = ws.kv_views(s, tokens)
                K.kv_dequant(kv, ctx.block_table, tokens, k_out=kd, vt_out=vt)
            att = K.prefill_attention(q, kd, vt, history=ctx.history, qheads=s.qheads, kvheads=s.kvheads,
                                      head_dim=d, k_global=self.kg, v_global=self.vg, out=ws.att[:rows],
                                      softmax_scale=self.softmax_scale, status=ws.status, workspace=attn_ws)
            if self.kv_shadow and tokens >= self.request_tokens[ctx.request]:
                del self.shadow[(ctx.request, layer)]  # last chunk: stream order keeps the buffers until read
        a8, s8 = K.gate_fp8(att, qkv[:, d:], fp8=ws.a8[:rows], scale=ws.s8[:rows], head_dim=d, head_stride=2 * d)
        o = K.gemm_e4m3(a8, w.o_q, m=rows, n=h, k=s.qheads * d, row_scale=s8, col_scale=w.o_scale,
                        out=ws.o[:rows])
        q_m, sf_m, _ = K.norm_pack(o, res1, w.ln_post, self.g_norm, eps=s.eps, q=ws.q_m[:rows], scales=ws.sf_m,
                                   updated=residual_out)
        if on_residual is not None:
            on_residual()  # the residual plane is final here; its transfer may start
        act_q, act_sf = K.gemm_swiglu_nvfp4(q_m, sf_m, w.gate_up.q, w.gate_up.sf, self.g_down, m=rows,
                                            n=2 * s.intermediate, k=h, alpha=w.alpha_gu, act_q=ws.act_q[:rows],
                                            act_sf=ws.act_sf)
        K.gemm_nvfp4(act_q, act_sf, w.down.q, w.down.sf, m=rows, n=h, k=s.intermediate, alpha=w.alpha_down,
                     out=hidden_out)
        return hidden_out, residual_out

    def run_layers(self, span, hidden, residual, ctx, out_planes=None, on_residual=None, ws=None, split=True):
        """Run layers [lo, hi) on one chunk.  ``out_planes`` = (hidden, residual)
        buffers that receive the final layer's output (e.g. a transport slot).
        ``ws``: the workspace set (default the first); stages that run
        concurrently need different ones.  ``split=False``: no key-range split
        of the attention's last partial wave (when another stream fills those
        SMs, the split's extra CTAs and merge cost more than they save)."""
        lo, hi = span
        rows = ctx.rows
        ws = ws or self.ws
        ping = [t[:rows] for t in ws.ping]
        for i, layer in enumerate(range(lo, hi)):
            last = layer == hi - 1
            if last and out_planes is not None:
                ho, ro = out_planes
            else:
                ho, ro = ping[2 * (i % 2)], ping[2 * (i % 2) + 1]
            hidden, residual = self.layer_forward(layer, hidden, residual, ctx, ho, ro,
                                                  on_residual if last else None, ws, split)
        return hidden, residual

    def final_norm(self, hidden, residual, out=None):
        s = self.shape
        return K.rms_norm(hidden, residual, self.final_gamma, eps=s.eps, out=out)

    def sample(self, last_hidden, tokens=None):
        """Greedy output token of each request from its final-normed last hidden
        row (temperature 0, as the reference samples its one output token)."""
        rows = last_hidden.shape[0]
        if tokens is None:
            tokens = torch.empty(rows, dtype=torch.int32, device=self.device)
        for r0 in range(0, rows, 8):  # the kernel takes up to 8 rows per weight pass
            K.lm_head_argmax(last_hidden[r0:r0 + 8], self.lm_head, tokens=tokens[r0:r0 + 8])
        return tokens

    def check_status(self):
        for ws in self.ws_sets:
            st = int(ws.status.item())
            if st:
                raise RuntimeError(f"kernel status word {st:#x}")
