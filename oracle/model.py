"""CPU oracle — fp32 dequantised forward of the Qwen-style NVFP4 decoder
(TEST INFRASTRUCTURE ONLY; also the timed CPU baseline of ``bench.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
may import this module.

Layer order follows the gated-attention decoder the reference runs through
vLLM (``vllm:model_executor/models/qwen3_next.py:285-320``; reference call
sites ``src/qwen_infra/vpp/model.py:83-115`` and ``vpp/producer.py:189-210``):

    norm_pack(hidden, residual) -> QKV GEMM -> QK-norm/RoPE/KV-append
    -> chunked causal GQA attention over the NVFP4 pages -> sigmoid gate -> FP8
    -> O GEMM -> norm_pack -> gate_up GEMM -> SwiGLU -> NVFP4 -> down GEMM

Every quantisation point of the GPU path is reproduced (activations as well
as weights), and all arithmetic in between is fp32 on dequantised values;
that is the "fp32 dequantised forward" the final hidden states are compared
with.  The O projection is FP8 x FP8 (per-token activation scale, per-channel
weight scale), as in the reference checkpoint's mixed NVFP4/FP8 layout
(``docs/architecture.md:123``, ``kernels/nvfp4_attention_fusion.py:46``).
"""

from dataclasses import dataclass

import numpy as np
import torch

from . import formats as F
from . import producers as P

f32 = np.float32


@dataclass(frozen=True)
class Shape:
    layers: int
    hidden: int
    qheads: int
    kvheads: int
    head_dim: int
    intermediate: int
    eps: float = 1e-6
    rope_theta: float = 1e6
    page_size: int = 16

    @property
    def qkv_out(self):
        return (2 * self.qheads + 2 * self.kvheads) * self.head_dim


TINY = Shape(layers=4, hidden=1024, qheads=16, kvheads=4, head_dim=64, intermediate=3072)
QWEN27B = Shape(layers=64, hidden=5120, qheads=64, kvheads=8, head_dim=128, intermediate=17408)

# Static activation global scales (448*6/assumed amax) — the same constants the
# product model uses (``vpp/model.py`` in the package).
ACT_GLOBAL_NORM = f32(2688.0 / 32.0)
ACT_GLOBAL_DOWN = f32(2688.0 / 64.0)
KV_GLOBAL_K = f32(16.0 / 2688.0)
KV_GLOBAL_V = f32(8.0 / 2688.0)


def seeded_normal(shape, seed, std):
    g = torch.Generator().manual_seed(int(seed))
    return (torch.randn(*shape, generator=g, dtype=torch.float32) * std).numpy()


def layer_seed(base, layer, idx):
    return base + layer * 16 + idx


def rope_table(max_pos, head_dim, theta):
    """cos/sin table [max_pos, D] f32: cos in columns [0, D/2), sin in [D/2, D)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    t = torch.arange(max_pos, dtype=torch.float64)
    fr = torch.outer(t, inv)
    return torch.cat([fr.cos(), fr.sin()], dim=1).to(torch.float32).numpy()


def interleave_gate_up(w_gate, w_up, block=128):
    """Row order of the fused gate_up weight: per 128 output channels, the 128
    gate rows then the 128 up rows (so one 256-column GEMM tile holds both
    halves of its SwiGLU)."""
    i, k = w_gate.shape
    return np.stack([w_gate.reshape(i // block, block, k), w_up.reshape(i // block, block, k)],
                    axis=1).reshape(2 * i, k)


def build_layer(shape, layer, base_seed=1234):
    """Synthetic layer weights (seeded N(0,0.02) fp32 -> NVFP4 / FP8), and
    norm weights ~ 1 + N(0, 0.05) rounded to bf16 (stored as raw gamma for
    the Gemma ``(1+w)`` form, i.e. gamma = w_eff - 1)."""
    s = shape
    h, d = s.hidden, s.head_dim
    w = {}
    wqkv = seeded_normal((s.qkv_out, h), layer_seed(base_seed, layer, 0), 0.02)
    wo = seeded_normal((h, s.qheads * d), layer_seed(base_seed, layer, 1), 0.02)
    wg = seeded_normal((s.intermediate, h), layer_seed(base_seed, layer, 2), 0.02)
    wu = seeded_normal((s.intermediate, h), layer_seed(base_seed, layer, 3), 0.02)
    wd = seeded_normal((h, s.intermediate), layer_seed(base_seed, layer, 4), 0.02)
    w["qkv"] = P.quantize_weight_nvfp4(wqkv)
    w["o"] = P.quantize_weight_fp8_rows(wo)
    w["gate_up"] = P.quantize_weight_nvfp4(interleave_gate_up(wg, wu))
    w["down"] = P.quantize_weight_nvfp4(wd)
    for j, name in enumerate(("ln_in", "ln_post")):
        w[name] = F.bf16_round(seeded_normal((h,), layer_seed(base_seed, layer, 5 + j), 0.05))
    w["q_norm"] = F.bf16_round(seeded_normal((d,), layer_seed(base_seed, layer, 7), 0.05))
    w["k_norm"] = F.bf16_round(seeded_normal((d,), layer_seed(base_seed, layer, 8), 0.05))
    return w


def final_norm_weight(shape, base_seed=1234):
    return F.bf16_round(seeded_normal((shape.hidden,), base_seed + 999_983, 0.05))


def dequant_weight(entry, n, k):
    packed, sf, g = entry
    return F.nvfp4_dequant(packed, sf, n, k, g)


class KVCache:
    """Paged NVFP4 KV of one layer: [pages, page, Hkv, D/2] codes + [.., D/16] scales."""

    def __init__(self, shape, pages):
        s = shape
        self.k = np.zeros((pages, s.page_size, s.kvheads, s.head_dim // 2), np.uint8)
        self.v = np.zeros_like(self.k)
        self.ks = np.zeros((pages, s.page_size, s.kvheads, s.head_dim // 16), np.uint8)
        self.vs = np.zeros_like(self.ks)

    def gather(self, block_table, tokens, shape, k_global, v_global):
        """Dequantised K, V [tokens, Hkv, D] of one request."""
        ps = shape.page_size
        pos = np.arange(tokens)
        pages = np.asarray(block_table)[pos // ps]
        ent = pos % ps

        def deq(codes, scales, g):
            vals = F.e2m1_decode(F.unpack_nibbles(codes[pages, ent]))  # [T, Hkv, D]
            sc = F.e4m3_decode(scales[pages, ent])  # [T, Hkv, D/16]
            t, hk, dd = vals.shape
            out = vals.reshape(t, hk, dd // 16, 16) * sc[..., None]
            return (out.reshape(t, hk, dd) * f32(g)).astype(f32)

        return deq(self.k, self.ks, k_global), deq(self.v, self.vs, v_global)


def attention(q, k, v, history, shape, tile=128):
    """Causal GQA softmax(Q K^T / sqrt(D)) V for one chunk of queries at
    positions history .. history+rows-1 over keys 0 .. history+rows-1, with
    the reference's attention precision (bf16 Q/K/V operands, bf16 P for the
    PV product, fp32 softmax statistics and accumulators) evaluated the way a
    tiled prefill kernel evaluates it: keys in tiles of ``tile``, running row
    max m, P = bf16(exp(s - m)), running sum l of the unrounded exponentials,
    O rescaled by exp(m_old - m_new), output O / l."""
    s = shape
    rows = q.shape[0]
    group = s.qheads // s.kvheads
    tokens = k.shape[0]
    qt = torch.from_numpy(np.ascontiguousarray(q)).view(rows, s.qheads, s.head_dim).transpose(0, 1)
    kt = torch.from_numpy(np.ascontiguousarray(k)).transpose(0, 1)  # [Hkv, T, D]
    vt = torch.from_numpy(np.ascontiguousarray(v)).transpose(0, 1)
    qpos = torch.arange(rows)[:, None] + history
    scale = 1.0 / float(np.sqrt(s.head_dim))
    out = torch.empty(s.qheads, rows, s.head_dim)
    for h in range(s.qheads):
        m = torch.full((rows, 1), float("-inf"))
        l = torch.zeros(rows, 1)
        o = torch.zeros(rows, s.head_dim)
        for t0 in range(0, tokens, tile):
            kk = kt[h // group, t0:t0 + tile]
            sc = torch.matmul(qt[h], kk.T) * scale
            kpos = torch.arange(t0, t0 + kk.shape[0])[None, :]
            sc = sc.masked_fill(kpos > qpos, float("-inf"))
            m_new = torch.maximum(m, sc.max(dim=1, keepdim=True).values)
            corr = torch.where(m == float("-inf"), torch.zeros_like(m), torch.exp(m - m_new))
            e = torch.where(sc == float("-inf"), torch.zeros_like(sc), torch.exp(sc - m_new))
            l = l * corr + e.sum(dim=1, keepdim=True)
            o = o * corr + torch.matmul(e.to(torch.bfloat16).float(), vt[h // group, t0:t0 + tile])
            m = m_new
        out[h] = o / l
    return out.transpose(0, 1).reshape(rows, s.qheads * s.head_dim).numpy()


def attention_exact(q, k, v, history, shape):
    """The same attention with fp32 P (no bf16 rounding), one pass per head."""
    s = shape
    rows = q.shape[0]
    group = s.qheads // s.kvheads
    qt = torch.from_numpy(np.ascontiguousarray(q)).view(rows, s.qheads, s.head_dim).transpose(0, 1)
    kt = torch.from_numpy(np.ascontiguousarray(k)).transpose(0, 1)
    vt = torch.from_numpy(np.ascontiguousarray(v)).transpose(0, 1)
    mask = torch.arange(k.shape[0])[None, :] > (torch.arange(rows)[:, None] + history)
    out = torch.empty(s.qheads, rows, s.head_dim)
    for h in range(s.qheads):
        sc = torch.matmul(qt[h], kt[h // group].T) / float(np.sqrt(s.head_dim))
        out[h] = torch.matmul(torch.softmax(sc.masked_fill(mask, float("-inf")), dim=-1), vt[h // group])
    return out.transpose(0, 1).reshape(rows, s.qheads * s.head_dim).numpy()


def _mm(a, w):
    return torch.matmul(torch.from_numpy(np.ascontiguousarray(a)),
                        torch.from_numpy(np.ascontiguousarray(w)).T).numpy()


class OracleModel:
    """Full-precision dequantised forward over chunks, with its own NVFP4 KV."""

    def __init__(self, shape, layers, max_tokens, base_seed=1234):
        self.shape = shape
        self.layers = list(layers)
        self.w = {l: build_layer(shape, l, base_seed) for l in self.layers}
        s = shape
        self.deq = {}
        for l in self.layers:
            w = self.w[l]
            wo_codes, wo_scale = w["o"]
            self.deq[l] = dict(
                qkv=dequant_weight(w["qkv"], s.qkv_out, s.hidden),
                o=(F.e4m3_decode(wo_codes) * wo_scale[:, None]).astype(f32),
                gate_up=dequant_weight(w["gate_up"], 2 * s.intermediate, s.hidden),
                down=dequant_weight(w["down"], s.hidden, s.intermediate),
            )
        self.pages = (max_tokens + s.page_size - 1) // s.page_size
        self.kv = {l: KVCache(s, self.pages) for l in self.layers}
        self.block_table = np.arange(self.pages, dtype=np.int32)
        self.rope = rope_table(max_tokens, s.head_dim, s.rope_theta)
        self.final_gamma = final_norm_weight(shape, base_seed)

    def layer(self, l, hidden, residual, history):
        s = self.shape
        w, dq = self.w[l], self.deq[l]
        rows = hidden.shape[0]
        q_in, sf_in, res1 = P.norm_pack(hidden, residual, w["ln_in"], ACT_GLOBAL_NORM, s.eps)
        a = F.nvfp4_dequant(q_in, sf_in, rows, s.hidden, ACT_GLOBAL_NORM)
        qkv = F.bf16_round(_mm(a, dq["qkv"]))
        positions = np.arange(history, history + rows)
        slots = self.block_table[positions // s.page_size] * s.page_size + positions % s.page_size
        kv = self.kv[l]
        q, gate = P.qk_rope_append(qkv, positions, w["q_norm"], w["k_norm"], self.rope, slots,
                                   KV_GLOBAL_K, KV_GLOBAL_V, kv.k, kv.v, kv.ks, kv.vs,
                                   qheads=s.qheads, kvheads=s.kvheads, head_dim=s.head_dim,
                                   page_size=s.page_size, eps=s.eps)
        kd, vd = kv.gather(self.block_table, history + rows, s, KV_GLOBAL_K, KV_GLOBAL_V)
        # fp32 softmax and fp32 P: the "fp32 dequantised forward" the layer
        # outputs are compared with.  (The bf16-P restatement of the reference's
        # attention precision, ``attention``, differs from it by ~2e-3 relative
        # at the 27B shape, which the FP8 / NVFP4 requantisations downstream
        # amplify ~30x by the layer output; the kernels compute P in f16.)
        att = F.bf16_round(attention_exact(q, kd, vd, history, s))
        a8, s8 = P.gate_fp8(att, gate)
        a8v = (F.e4m3_decode(a8) * s8[:, None]).astype(f32)
        o = F.bf16_round(_mm(a8v, dq["o"]))
        q_m, sf_m, res2 = P.norm_pack(o, res1, w["ln_post"], ACT_GLOBAL_NORM, s.eps)
        am = F.nvfp4_dequant(q_m, sf_m, rows, s.hidden, ACT_GLOBAL_NORM)
        gu = _mm(am, dq["gate_up"]).reshape(rows, s.intermediate // 128, 2, 128)
        g_acc = gu[:, :, 0, :].reshape(rows, s.intermediate)
        u_acc = gu[:, :, 1, :].reshape(rows, s.intermediate)
        q_act, sf_act, _ = P.swiglu_nvfp4(g_acc, u_acc, 1.0, ACT_GLOBAL_DOWN)
        act = F.nvfp4_dequant(q_act, sf_act, rows, s.intermediate, ACT_GLOBAL_DOWN)
        hidden_out = F.bf16_round(_mm(act, dq["down"]))
        return hidden_out, res2

    def forward_chunks(self, embeds, chunk):
        """Run all owned layers over the request in chunks; returns the final
        normed hidden states [tokens, H] (bf16-valued f32)."""
        s = self.shape
        outs = []
        for start in range(0, embeds.shape[0], chunk):
            hidden = embeds[start:start + chunk]
            residual = None
            for l in self.layers:
                hidden, residual = self.layer(l, hidden, residual, start)
            outs.append(P.rms_norm_out(hidden, residual, self.final_gamma, s.eps))
        return np.concatenate(outs, axis=0)
