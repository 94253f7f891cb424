"""CPU oracle — fused producers of one decoder layer (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
may import this module.  Every function is a numpy restatement of the
reference's semantics, with the fp32 operation order that the sm_100a kernels
use written out explicitly, so that quantised bytes compare bit-exactly:

* every product / sum / quotient is one IEEE fp32 operation, rounded to
  nearest-even, never contracted into an FMA (the kernels use ``__fmul_rn`` /
  ``__fadd_rn`` / ``__fdiv_rn`` / ``__fsqrt_rn``; numpy float32 arithmetic is
  IEEE and never contracts);
* reductions follow the kernels' fixed trees (sequential per-thread partials,
  then xor-butterflies over 32 lanes);
* the exponential is :func:`fexp`, a published method (Cody-Waite split
  ``2^x = 2^n * 2^f`` with a degree-6 Taylor polynomial for ``2^f`` on
  [-1/2, 1/2], Horner form) that both sides evaluate with the same fp32 steps.

Reference semantics followed (file:line inside the reference project):
* norm -> NVFP4: ``src/qwen_infra/kernels/nvfp4_norm_pack.cu:17-64``
* QK-norm / RoPE / gate split / NVFP4 paged KV append:
  ``src/qwen_infra/kernels/nvfp4_attention_front.cu:45-112``
* attention-output x sigmoid(gate) -> FP8: ``src/qwen_infra/kernels/nvfp4_bucket_xqa.cu:48-66``
  (per-token scale instead of the static scalar, as the benchmark configuration asks)
* SwiGLU -> NVFP4 (``vpp/producer.py:197-206``: ``act_fn`` then ``scaled_fp4_quant``).
"""

import numpy as np

from . import formats as F

f32 = np.float32
LOG2E_F = f32(1.4426950408889634)
# Taylor coefficients (ln 2)^k / k!, rounded to fp32, highest degree first.
_LN2 = 0.6931471805599453
EXP2_POLY = [f32(_LN2 ** k / float(np.prod(range(1, k + 1)) if k else 1.0)) for k in range(6, -1, -1)]


def fexp(x):
    """exp(x) in fp32 by 2^(x*log2 e) = 2^n * 2^f (n = rint, |f| <= 1/2)."""
    x = np.asarray(x, dtype=f32)
    t = (x * LOG2E_F).astype(f32)
    big = t >= f32(128.0)
    tiny = t <= f32(-150.0)
    tc = np.clip(t, f32(-149.0), f32(127.0)).astype(f32)
    n = np.rint(tc).astype(f32)
    fr = (tc - n).astype(f32)
    p = np.full_like(fr, EXP2_POLY[0])
    for c in EXP2_POLY[1:]:
        p = (p * fr).astype(f32)
        p = (p + c).astype(f32)
    ni = n.astype(np.int32)
    h1 = ni // 2  # floor division, matches the kernel's arithmetic shift
    h2 = ni - h1
    s1 = ((h1 + 127).astype(np.uint32) << 23).view(f32)
    s2 = ((h2 + 127).astype(np.uint32) << 23).view(f32)
    r = ((p * s1).astype(f32) * s2).astype(f32)
    r = np.where(big, f32(np.inf), r)
    r = np.where(tiny, f32(0.0), r)
    return r.astype(f32)


def sigmoid_f(g):
    g = np.asarray(g, dtype=f32)
    return (f32(1.0) / (f32(1.0) + fexp(-g)).astype(f32)).astype(f32)


def silu_f(g):
    g = np.asarray(g, dtype=f32)
    return (g / (f32(1.0) + fexp(-g)).astype(f32)).astype(f32)


def butterfly_sum(parts):
    """[..., 32] fp32 -> [...]: xor-butterfly over 32 lanes (d = 16,8,4,2,1).
    Addition is commutative, so every lane ends with this same value."""
    x = np.asarray(parts, dtype=f32)
    width = x.shape[-1]
    assert width == 32
    while width > 1:
        width //= 2
        x = (x[..., :width] + x[..., width:2 * width]).astype(f32)
    return x[..., 0]


def _seq_sum_sq(vals):
    """Sequential sum of squares along the last axis, one rounding per op."""
    vals = np.asarray(vals, dtype=f32)
    acc = (vals[..., 0] * vals[..., 0]).astype(f32)
    for i in range(1, vals.shape[-1]):
        acc = (acc + (vals[..., i] * vals[..., i]).astype(f32)).astype(f32)
    return acc


def _block_sum(thread_partials):
    """[rows, T] per-thread partials -> [rows] using warp butterflies and a
    second butterfly over the (zero padded) per-warp results."""
    rows, t = thread_partials.shape
    warps = (t + 31) // 32
    pad = np.zeros((rows, warps * 32), dtype=f32)
    pad[:, :t] = thread_partials
    warp_sums = butterfly_sum(pad.reshape(rows, warps, 32))
    pad2 = np.zeros((rows, 32), dtype=f32)
    pad2[:, :warps] = warp_sums
    return butterfly_sum(pad2)


def nvfp4_quant_rows(y, global_scale):
    """Quantise fp32 rows (already on the values the producer holds) per 16
    elements: scale = e4m3(min(amax*g*(1/6), 448)); code = e2m1(y*g/scale)
    (``nvfp4_norm_pack.cu:50-63``).  Returns (packed [rows,K/2], codes [rows,K/16])."""
    y = np.asarray(y, dtype=f32)
    rows, k = y.shape
    g = f32(global_scale)
    blk = y.reshape(rows, k // 16, 16)
    amax = np.abs(blk).max(axis=-1).astype(f32)
    pre = np.minimum(((amax * g).astype(f32) * f32(1.0 / 6.0)).astype(f32), f32(448.0))
    sf = F.e4m3_encode(pre)
    scale = F.e4m3_decode(sf)
    inv = np.where(scale > 0, (g / np.where(scale > 0, scale, f32(1))).astype(f32), f32(0)).astype(f32)
    codes = F.e2m1_encode((blk * inv[:, :, None]).astype(f32)).reshape(rows, k)
    return F.pack_nibbles(codes), sf


def norm_pack(x, residual, gamma, global_scale, eps=1e-6, weight_offset=1.0):
    """Residual add + RMSNorm + NVFP4 pack (``nvfp4_norm_pack.cu:17-64``).

    x, residual: float32 arrays holding bf16 values [rows, H] (residual may be
    None: the first layer of the first stage); gamma: bf16 values [H].
    weight_offset 1.0 is the Gemma ``(1+w)`` form the reference uses, 0.0 the
    plain ``w`` form.  Returns (q [rows,H/2] u8, scales swizzled u8,
    updated [rows,H] bf16-valued f32)."""
    x = np.asarray(x, dtype=f32)
    rows, h = x.shape
    hv = x if residual is None else (x + np.asarray(residual, dtype=f32)).astype(f32)
    updated = F.bf16_round(hv)
    per_thread = _seq_sum_sq(hv.reshape(rows, h // 16, 16))
    total = _block_sum(per_thread)
    mean = (total / f32(h)).astype(f32)
    inv = (f32(1.0) / np.sqrt((mean + f32(eps)).astype(f32)).astype(f32)).astype(f32)
    weff = (np.asarray(gamma, dtype=f32) + f32(weight_offset)).astype(f32)
    y = F.bf16_round(((hv * inv[:, None]).astype(f32) * weff[None, :]).astype(f32))
    packed, sf = nvfp4_quant_rows(y, global_scale)
    return packed, F.swizzle_scales(sf, h), updated


def rms_norm_out(x, residual, gamma, eps=1e-6, weight_offset=1.0):
    """Final norm of the last virtual stage: the same arithmetic as
    :func:`norm_pack` up to the bf16 normalised value, which is the output."""
    x = np.asarray(x, dtype=f32)
    rows, h = x.shape
    hv = x if residual is None else (x + np.asarray(residual, dtype=f32)).astype(f32)
    per_thread = _seq_sum_sq(hv.reshape(rows, h // 16, 16))
    total = _block_sum(per_thread)
    mean = (total / f32(h)).astype(f32)
    inv = (f32(1.0) / np.sqrt((mean + f32(eps)).astype(f32)).astype(f32)).astype(f32)
    weff = (np.asarray(gamma, dtype=f32) + f32(weight_offset)).astype(f32)
    return F.bf16_round(((hv * inv[:, None]).astype(f32) * weff[None, :]).astype(f32))


def _lane_layout(d):
    """Element ownership of one warp over a head of ``d`` values: lane l owns
    E/2 consecutive elements of each rotary half, E = d/32."""
    e2 = d // 64
    first = np.arange(32)[:, None] * e2 + np.arange(e2)[None, :]
    return first, first + d // 2


def _head_inv_rms(v, d, eps):
    """v: [n, d] fp32 -> [n] inverse RMS with the warp's reduction order:
    lane partial = x0^2 + y0^2 + x1^2 + y1^2 ... (x first half, y second half),
    then the 32-lane butterfly."""
    first, second = _lane_layout(d)
    xs = v[:, first]
    ys = v[:, second]
    inter = np.empty(xs.shape[:-1] + (xs.shape[-1] * 2,), dtype=f32)
    inter[..., 0::2] = xs
    inter[..., 1::2] = ys
    lane = _seq_sum_sq(inter)
    total = butterfly_sum(lane)
    mean = (total / f32(d)).astype(f32)
    return (f32(1.0) / np.sqrt((mean + f32(eps)).astype(f32)).astype(f32)).astype(f32)


def _kv_quant(v, global_scale):
    """K/V NVFP4 per 16 elements (``nvfp4_attention_front.cu:45-66``):
    scale = e4m3(amax/(6*g)); inverse = 1/(scale*g); code = e2m1(v*inverse)."""
    n, d = v.shape
    g = f32(global_scale)
    blk = v.reshape(n, d // 16, 16)
    amax = np.abs(blk).max(axis=-1).astype(f32)
    sf = F.e4m3_encode((amax / (f32(6.0) * g)).astype(f32))
    scale = F.e4m3_decode(sf)
    denom = (scale * g).astype(f32)
    inv = np.where(scale > 0, (f32(1.0) / np.where(scale > 0, denom, f32(1))).astype(f32), f32(0))
    codes = F.e2m1_encode((blk * inv[:, :, None].astype(f32)).astype(f32)).reshape(n, d)
    return F.pack_nibbles(codes), sf


def qk_rope_append(qkv, positions, q_weight, k_weight, cos_sin, slots, k_global, v_global,
                   k_cache, v_cache, k_scales, v_scales, *, qheads, kvheads, head_dim,
                   page_size, eps=1e-6, weight_offset=1.0):
    """QK-norm + NeoX RoPE + gate split + NVFP4 paged KV append
    (``nvfp4_attention_front.cu:68-112``), rotary dimension == head_dim.

    qkv: [rows, (2*Hq + 2*Hkv)*D] bf16-valued f32, each Q head laid out as
    [q(D) | gate(D)], then the K heads, then the V heads.  cos_sin: [maxpos, D]
    f32, cos in the first D/2 columns, sin in the rest.  Caches are updated in
    place: k_cache/v_cache [pages, page_size, Hkv, D/2] u8, k_scales/v_scales
    [pages, page_size, Hkv, D/16] u8.  Returns (q [rows, Hq*D], gate [rows, Hq*D])."""
    qkv = np.asarray(qkv, dtype=f32)
    rows = qkv.shape[0]
    d = head_dim
    half = d // 2
    qoff = 2 * d * qheads
    qw = (np.asarray(q_weight, dtype=f32) + f32(weight_offset)).astype(f32)
    kw = (np.asarray(k_weight, dtype=f32) + f32(weight_offset)).astype(f32)
    pos = np.asarray(positions, dtype=np.int64)
    cs = np.asarray(cos_sin, dtype=f32)
    c = cs[pos, :half]
    s = cs[pos, half:]

    def norm_rope(v, w):  # v [rows, nh, d]
        n = v.shape[1]
        flat = v.reshape(rows * n, d)
        inv = _head_inv_rms(flat, d, eps).reshape(rows, n, 1)
        y = F.bf16_round(((v * inv).astype(f32) * w[None, None, :]).astype(f32))
        a, b = y[..., :half], y[..., half:]
        cc, ss = c[:, None, :], s[:, None, :]
        xo = F.bf16_round(((a * cc).astype(f32) - (b * ss).astype(f32)).astype(f32))
        yo = F.bf16_round(((b * cc).astype(f32) + (a * ss).astype(f32)).astype(f32))
        return np.concatenate([xo, yo], axis=-1)

    qg = qkv[:, :qoff].reshape(rows, qheads, 2 * d)
    q = norm_rope(qg[:, :, :d], qw).reshape(rows, qheads * d)
    gate = qg[:, :, d:].reshape(rows, qheads * d).copy()
    k = norm_rope(qkv[:, qoff:qoff + kvheads * d].reshape(rows, kvheads, d), kw)
    v = qkv[:, qoff + kvheads * d:qoff + 2 * kvheads * d].reshape(rows, kvheads, d)
    kq, ks = _kv_quant(k.reshape(rows * kvheads, d), k_global)
    vq, vs = _kv_quant(v.reshape(rows * kvheads, d), v_global)
    kq = kq.reshape(rows, kvheads, d // 2)
    vq = vq.reshape(rows, kvheads, d // 2)
    ks = ks.reshape(rows, kvheads, d // 16)
    vs = vs.reshape(rows, kvheads, d // 16)
    pages = k_cache.shape[0]
    for r in range(min(rows, len(slots))):
        slot = int(slots[r])
        if slot < 0 or slot >= pages * page_size:
            continue
        pg, en = divmod(slot, page_size)
        k_cache[pg, en] = kq[r]
        v_cache[pg, en] = vq[r]
        k_scales[pg, en] = ks[r]
        v_scales[pg, en] = vs[r]
    return q, gate


def gate_fp8(out, gate):
    """FP8 epilogue (``nvfp4_bucket_xqa.cu:56-62``) with a per-token scale:
    g = bf16(sigmoid(gate)); v = bf16(out*g); scale = max(amax_row/448, FLT_MIN);
    code = e4m3_satfinite(v/scale).  Returns (codes [rows,N] u8, scale [rows] f32)."""
    out = np.asarray(out, dtype=f32)
    sg = F.bf16_round(sigmoid_f(gate))
    v = F.bf16_round((out * sg).astype(f32))
    amax = np.abs(v).max(axis=-1).astype(f32)
    scale = np.maximum((amax / f32(448.0)).astype(f32), f32(np.finfo(np.float32).tiny)).astype(f32)
    codes = F.e4m3_encode((v / scale[:, None]).astype(f32))
    return codes, scale


def swiglu_nvfp4(gate_acc, up_acc, alpha, global_scale):
    """gate_up GEMM epilogue: gate = bf16(acc*alpha), up = bf16(acc*alpha),
    act = bf16(gate/(1+exp(-gate)) * up) (the SiLU-and-mul order), then the
    NVFP4 quantisation of :func:`nvfp4_quant_rows`."""
    g = F.bf16_round((np.asarray(gate_acc, dtype=f32) * f32(alpha)).astype(f32))
    u = F.bf16_round((np.asarray(up_acc, dtype=f32) * f32(alpha)).astype(f32))
    act = F.bf16_round((silu_f(g) * u).astype(f32))
    packed, sf = nvfp4_quant_rows(act, global_scale)
    return packed, F.swizzle_scales(sf, act.shape[1]), act


def weight_global_scale(w):
    """NVFP4 per-tensor global scale g = 448*6/amax (fp32 division)."""
    amax = f32(np.abs(np.asarray(w, dtype=f32)).max())
    return f32(f32(2688.0) / amax)


def quantize_weight_nvfp4(w):
    """fp32 [N, K] -> (packed [N,K/2], swizzled scales, global scale)."""
    w = np.asarray(w, dtype=f32)
    g = weight_global_scale(w)
    packed, sf = nvfp4_quant_rows(w, g)
    return packed, F.swizzle_scales(sf, w.shape[1]), g


def quantize_weight_fp8_rows(w):
    """fp32 [N, K] -> (e4m3 codes [N,K], per-row scale [N] = amax/448)."""
    w = np.asarray(w, dtype=f32)
    amax = np.abs(w).max(axis=1).astype(f32)
    scale = np.maximum((amax / f32(448.0)).astype(f32), f32(np.finfo(np.float32).tiny)).astype(f32)
    return F.e4m3_encode((w / scale[:, None]).astype(f32)), scale


def lm_head_argmax(hidden, weight):
    """Greedy sampling of the output token (the reference samples with
    temperature 0: src/qwen_infra/cli.py:145): logits[r, v] = <hidden[r], W[v]>
    with the kernel's fp32 order -- lane l of a warp sums the 8-element chunks
    l, l+32, ... of the row in order (one rounded multiply and one rounded add
    per element), then the 32 lane sums are combined by the xor butterfly --
    and token[r] = argmax_v, lowest index on ties, NaN never chosen.
    hidden [R, H], weight [V, H]: float32 arrays holding bf16 values.
    Returns (logits [R, V] float32, tokens [R] int)."""
    h = np.asarray(hidden, dtype=f32)
    w = np.asarray(weight, dtype=f32)
    rows, dim = h.shape
    vocab = w.shape[0]
    chunks = dim // 8
    acc = np.zeros((rows, vocab, 32), dtype=f32)
    for step in range((chunks + 31) // 32):
        lanes = np.arange(32)
        c = lanes + 32 * step
        live = c < chunks
        c = np.minimum(c, chunks - 1)
        for e in range(8):
            col = c * 8 + e  # [32]
            prod = (w[None, :, col] * h[:, None, col]).astype(f32)  # [R, V, 32]
            acc = np.where(live[None, None, :], (acc + prod).astype(f32), acc)
    logits = butterfly_sum(acc)
    bits = logits.view(np.uint32)
    ordv = np.where(bits & np.uint32(0x80000000), ~bits, bits | np.uint32(0x80000000)).astype(np.uint64)
    idx = np.arange(vocab, dtype=np.uint64)
    keys = (ordv << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - idx)[None, :]
    keys = np.where(np.isnan(logits), np.uint64(0), keys)
    best = keys.max(axis=1)
    tokens = np.where(best == 0, -1, (np.uint64(0xFFFFFFFF) - (best & np.uint64(0xFFFFFFFF))).astype(np.int64))
    return logits, tokens.astype(np.int64)
