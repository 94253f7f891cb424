"""The kernels as ``torch.library`` custom operators (namespace ``qwen_b200``).

The reference registers its producer the same way
(``kernels/nvfp4_norm_pack.py:115-167``: ``qwen_sm120::gemma_nvfp4_pack`` with
a ``register_fake`` shape function; the attention adapters at
``kernels/nvfp4_attention_fusion.py:12-35``), so the ops can sit inside a
``torch.compile``'d model: Dynamo and Inductor see opaque CUDA ops with known
output shapes, and the fake implementations below give those shapes without
running anything.  The real implementations enqueue on the current stream
through :mod:`qwen_infra_b200.kernels` (the C ABI); there is no CPU path.

Operators:

* ``gemma_nvfp4_pack(x, residual, raw_gamma, global_inverse) -> (q, scale, updated)``:
  the reference's own contract (H 5120, bf16, scales as int32 [R128, 80]);
* ``norm_pack`` / ``rms_norm``: any hidden size, optional residual;
* ``qk_rope_kv_append``: QK-norm + RoPE + NVFP4 paged append (mutates the
  four cache tensors; returns q);
* ``gate_fp8`` (per-token scale) and ``gate_fp8_static`` (the reference's
  static scale);
* ``nvfp4_gemm`` / ``nvfp4_gemm_swiglu`` / ``e4m3_gemm``;
* ``paged_prefill_attention``: causal GQA over the paged NVFP4 cache;
* ``lm_head_argmax``.
"""

import torch

from . import kernels as K

NS = "qwen_b200"


def _scale_bytes(rows, k):
    return K.scale_buffer_bytes(rows, k)


# ---- norm -> NVFP4 ---------------------------------------------------------

@torch.library.custom_op(f"{NS}::gemma_nvfp4_pack", mutates_args=(), device_types="cuda")
def gemma_nvfp4_pack(x: torch.Tensor, residual: torch.Tensor, raw_gamma: torch.Tensor,
                     global_inverse: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    rows = x.shape[0]
    if (not 1 <= rows <= 8192 or tuple(x.shape) != (rows, 5120) or residual.shape != x.shape
            or x.dtype != torch.bfloat16 or residual.dtype != x.dtype or raw_gamma.dtype != torch.bfloat16
            or tuple(raw_gamma.shape) != (5120,) or global_inverse.dtype != torch.float32
            or global_inverse.numel() != 1
            or any(not t.is_contiguous() or t.data_ptr() % 16 for t in (x, residual, raw_gamma))):
        raise ValueError("expected bf16 [rows <= 8192, 5120] x / residual, bf16 [5120] gamma, fp32 scalar")
    scale = torch.empty((((rows + 127) // 128) * 128, 80), dtype=torch.int32, device=x.device)
    q, _, updated = K.norm_pack(x, residual, raw_gamma, global_inverse, scales=scale.view(torch.uint8).view(-1))
    return q, scale, updated


@gemma_nvfp4_pack.register_fake
def _(x, residual, raw_gamma, global_inverse):
    rows = x.shape[0]
    return (x.new_empty((rows, 2560), dtype=torch.uint8),
            x.new_empty((((rows + 127) // 128) * 128, 80), dtype=torch.int32), torch.empty_like(residual))


@torch.library.custom_op(f"{NS}::norm_pack", mutates_args=(), device_types="cuda")
def norm_pack(x: torch.Tensor, residual: torch.Tensor | None, gamma: torch.Tensor, global_scale: torch.Tensor,
              eps: float = 1e-6, weight_offset: float = 1.0) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return K.norm_pack(x, residual, gamma, global_scale, eps=eps, weight_offset=weight_offset)


@norm_pack.register_fake
def _(x, residual, gamma, global_scale, eps=1e-6, weight_offset=1.0):
    rows, h = x.shape
    return (x.new_empty((rows, h // 2), dtype=torch.uint8), x.new_empty(_scale_bytes(rows, h), dtype=torch.uint8),
            torch.empty_like(x))


@torch.library.custom_op(f"{NS}::rms_norm", mutates_args=(), device_types="cuda")
def rms_norm(x: torch.Tensor, residual: torch.Tensor | None, gamma: torch.Tensor, eps: float = 1e-6,
             weight_offset: float = 1.0) -> torch.Tensor:
    return K.rms_norm(x, residual, gamma, eps=eps, weight_offset=weight_offset)


@rms_norm.register_fake
def _(x, residual, gamma, eps=1e-6, weight_offset=1.0):
    return torch.empty_like(x)


# ---- QK-norm + RoPE + NVFP4 paged KV append ----------------------------------

class _CacheView:
    """The PagedKV fields the append reads, from four cache tensors."""

    def __init__(self, k, v, ks, vs):
        self.k, self.v, self.ks, self.vs = k, v, ks, vs
        self.pages, self.page_size = k.shape[0], k.shape[1]


@torch.library.custom_op(f"{NS}::qk_rope_kv_append", mutates_args=("k_cache", "v_cache", "k_scales", "v_scales"),
                         device_types="cuda")
def qk_rope_kv_append(qkv: torch.Tensor, positions: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                      cos_sin: torch.Tensor, slots: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      k_scales: torch.Tensor, v_scales: torch.Tensor, k_global: torch.Tensor, v_global: torch.Tensor,
                      qheads: int, kvheads: int, head_dim: int, eps: float = 1e-6) -> torch.Tensor:
    q, _ = K.qk_rope_kv_append(qkv, positions, q_weight, k_weight, cos_sin, slots,
                               _CacheView(k_cache, v_cache, k_scales, v_scales), k_global, v_global, qheads=qheads,
                               kvheads=kvheads, head_dim=head_dim, eps=eps, want_gate=False)
    return q


@qk_rope_kv_append.register_fake
def _(qkv, positions, q_weight, k_weight, cos_sin, slots, k_cache, v_cache, k_scales, v_scales, k_global, v_global,
      qheads, kvheads, head_dim, eps=1e-6):
    return qkv.new_empty((qkv.shape[0], qheads * head_dim))


# ---- attention output x sigmoid(gate) -> FP8 ---------------------------------

@torch.library.custom_op(f"{NS}::gate_fp8", mutates_args=(), device_types="cuda")
def gate_fp8(out: torch.Tensor, gate: torch.Tensor, head_dim: int = 0,
             head_stride: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    fp8, scale = K.gate_fp8(out, gate, head_dim=head_dim or None, head_stride=head_stride or None)
    return fp8.view(torch.float8_e4m3fn), scale


@gate_fp8.register_fake
def _(out, gate, head_dim=0, head_stride=0):
    return out.new_empty(out.shape, dtype=torch.float8_e4m3fn), out.new_empty(out.shape[0], dtype=torch.float32)


@torch.library.custom_op(f"{NS}::gate_fp8_static", mutates_args=(), device_types="cuda")
def gate_fp8_static(out: torch.Tensor, gate: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return K.gate_fp8_static(out, gate, scale).view(torch.float8_e4m3fn)


@gate_fp8_static.register_fake
def _(out, gate, scale):
    return out.new_empty(out.shape, dtype=torch.float8_e4m3fn)


# ---- GEMMs -------------------------------------------------------------------

@torch.library.custom_op(f"{NS}::nvfp4_gemm", mutates_args=(), device_types="cuda")
def nvfp4_gemm(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor, alpha: torch.Tensor,
               k: int) -> torch.Tensor:
    return K.gemm_nvfp4(a, sfa, b, sfb, m=a.shape[0], n=b.shape[0], k=k, alpha=alpha)


@nvfp4_gemm.register_fake
def _(a, sfa, b, sfb, alpha, k):
    return a.new_empty((a.shape[0], b.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op(f"{NS}::nvfp4_gemm_swiglu", mutates_args=(), device_types="cuda")
def nvfp4_gemm_swiglu(a: torch.Tensor, sfa: torch.Tensor, b: torch.Tensor, sfb: torch.Tensor, alpha: torch.Tensor,
                      act_global: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    return K.gemm_swiglu_nvfp4(a, sfa, b, sfb, act_global, m=a.shape[0], n=b.shape[0], k=k, alpha=alpha)


@nvfp4_gemm_swiglu.register_fake
def _(a, sfa, b, sfb, alpha, act_global, k):
    m, inter = a.shape[0], b.shape[0] // 2
    return a.new_empty((m, inter // 2), dtype=torch.uint8), a.new_empty(_scale_bytes(m, inter), dtype=torch.uint8)


@torch.library.custom_op(f"{NS}::e4m3_gemm", mutates_args=(), device_types="cuda")
def e4m3_gemm(a: torch.Tensor, b: torch.Tensor, row_scale: torch.Tensor, col_scale: torch.Tensor) -> torch.Tensor:
    return K.gemm_e4m3(a.view(torch.uint8), b.view(torch.uint8), m=a.shape[0], n=b.shape[0], k=a.shape[1],
                       row_scale=row_scale, col_scale=col_scale)


@e4m3_gemm.register_fake
def _(a, b, row_scale, col_scale):
    return a.new_empty((a.shape[0], b.shape[0]), dtype=torch.bfloat16)


# ---- attention and the output token -------------------------------------------

@torch.library.custom_op(f"{NS}::paged_prefill_attention", mutates_args=(), device_types="cuda")
def paged_prefill_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, k_scales: torch.Tensor,
                            v_scales: torch.Tensor, block_table: torch.Tensor, k_global: torch.Tensor,
                            v_global: torch.Tensor, history: int, qheads: int) -> torch.Tensor:
    kv = K.PagedKV.wrap(k_cache, v_cache, k_scales, v_scales)
    return K.paged_prefill_attention(q, kv, block_table, history=history, qheads=qheads, k_global=k_global,
                                     v_global=v_global)


@paged_prefill_attention.register_fake
def _(q, k_cache, v_cache, k_scales, v_scales, block_table, k_global, v_global, history, qheads):
    return torch.empty_like(q)


@torch.library.custom_op(f"{NS}::lm_head_argmax", mutates_args=(), device_types="cuda")
def lm_head_argmax(hidden: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    return K.lm_head_argmax(hidden, weight)


@lm_head_argmax.register_fake
def _(hidden, weight):
    return hidden.new_empty(hidden.shape[0], dtype=torch.int32)


OPS = ("gemma_nvfp4_pack", "norm_pack", "rms_norm", "qk_rope_kv_append", "gate_fp8", "gate_fp8_static",
       "nvfp4_gemm", "nvfp4_gemm_swiglu", "e4m3_gemm", "paged_prefill_attention", "lm_head_argmax")
