"""CPU oracle — fused producers of one decoder layer (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
may import this module.  Every function is a numpy restatement of the
reference's semantics with the reference kernels' fp32 operation order
written out, so that quantised bytes compare bit-exactly:

* every product / sum / quotient is one IEEE fp32 operation, rounded to
  nearest-even, never contracted into an FMA (the reference builds its
  producers with ``--fmad=false``; numpy float32 arithmetic never contracts);
* reductions follow the reference kernels' trees (per-thread partials in the
  reference's element order, then ``shfl_down`` trees over 32 lanes, which
  leave in lane 0 the same value as an xor-butterfly);
* the two CUDA math functions the reference calls, ``rsqrtf`` and ``expf``,
  come from a provider (:data:`MATH`): :class:`HostMath` (correctly rounded,
  the default on the CPU), :class:`oracle.cuda_math.CudaMath` (CUDA's own
  values, computed on the GPU in the GPU tests) or :class:`RecordedMath`
  (CUDA's values recorded in a golden fixture).

Pinned against the reference itself: the GPU tests run the reference's
``nvfp4_norm_pack.cu`` and ``nvfp4_attention_front.cu`` (compiled for sm_100a
by ``oracle/build_ref.py``) and compare their bytes with this restatement
and with the repository's kernels; ``tests/golden/producers_ref.json`` records
their outputs for the CPU tests.

Reference semantics followed (file:line inside the reference project):
* norm -> NVFP4: ``src/qwen_infra/kernels/nvfp4_norm_pack.cu:17-64``
* QK-norm / RoPE / gate split / NVFP4 paged KV append:
  ``src/qwen_infra/kernels/nvfp4_attention_front.cu:45-112``
* attention-output x sigmoid(gate) -> FP8: ``src/qwen_infra/kernels/nvfp4_bucket_xqa.cu:48-66``
  (static scale as the reference, or a per-token scale as the benchmark
  configuration asks)
* SwiGLU -> NVFP4 (``vpp/producer.py:197-206``: ``act_fn`` then ``scaled_fp4_quant``).
"""

import numpy as np

from . import formats as F

f32 = np.float32


class HostMath:
    """Correctly rounded stand-ins for CUDA's rsqrtf / expf (fp64, rounded)."""

    name = "host"

    def rsqrt(self, x):
        x = np.asarray(x, dtype=f32)
        with np.errstate(divide="ignore", invalid="ignore"):
            return (1.0 / np.sqrt(x.astype(np.float64))).astype(f32)

    def exp(self, x):
        x = np.asarray(x, dtype=f32)
        with np.errstate(over="ignore", under="ignore"):
            return np.exp(x.astype(np.float64)).astype(f32)


class RecordedMath(HostMath):
    """HostMath, except at the inputs where CUDA's value was recorded to
    differ: ``rsqrt`` / ``exp`` map fp32 input bits -> fp32 output bits."""

    name = "recorded"

    def __init__(self, rsqrt=None, exp=None):
        self.tables = {"rsqrt": dict(rsqrt or {}), "exp": dict(exp or {})}

    def _patch(self, which, x, y):
        table = self.tables[which]
        if not table:
            return y
        xb = np.asarray(x, dtype=f32).view(np.uint32).reshape(-1)
        yb = y.view(np.uint32).reshape(-1).copy()
        for i, bits in enumerate(xb.tolist()):
            hit = table.get(bits)
            if hit is not None:
                yb[i] = hit
        return yb.view(f32).reshape(y.shape)

    def rsqrt(self, x):
        return self._patch("rsqrt", x, HostMath.rsqrt(self, x))

    def exp(self, x):
        return self._patch("exp", x, HostMath.exp(self, x))


MATH = HostMath()


class use_math:
    """Context manager: evaluate rsqrtf / expf with ``provider`` inside."""

    def __init__(self, provider):
        self.provider = provider

    def __enter__(self):
        global MATH
        self.saved, MATH = MATH, self.provider
        return self.provider

    def __exit__(self, *exc):
        global MATH
        MATH = self.saved
        return False


def sigmoid_f(g):
    """1/(1+expf(-g)) with one rounding per operation (nvfp4_bucket_xqa.cu:57)."""
    g = np.asarray(g, dtype=f32)
    return (f32(1.0) / (f32(1.0) + MATH.exp(-g)).astype(f32)).astype(f32)


def silu_f(g):
    """g/(1+expf(-g)), the SiLU of the SiLU-and-mul."""
    g = np.asarray(g, dtype=f32)
    return (g / (f32(1.0) + MATH.exp(-g)).astype(f32)).astype(f32)


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


# Element order of one reference thread's 16 values (nvfp4_norm_pack.cu:23-27):
# each step adds one element of the low and one of the high 8.
_NORM_ORDER = [j for i in range(8) for j in (i, i + 8)]


def _row_inv_rms(hv, eps):
    """[rows, H] fp32 -> [rows]: rsqrtf(sum(h^2)/H + eps) with the reference's
    tree: thread t sums its 16 elements in _NORM_ORDER, warps reduce by
    shfl_down, the warp sums by a second zero-padded shfl_down
    (nvfp4_norm_pack.cu:23-40)."""
    rows, h = hv.shape
    per_thread = _seq_sum_sq(hv.reshape(rows, h // 16, 16)[:, :, _NORM_ORDER])
    total = _block_sum(per_thread)
    mean = (total / f32(h)).astype(f32)
    return MATH.rsqrt((mean + f32(eps)).astype(f32))


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
    inv = _row_inv_rms(hv, eps)
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
    inv = _row_inv_rms(hv, eps)
    weff = (np.asarray(gamma, dtype=f32) + f32(weight_offset)).astype(f32)
    return F.bf16_round(((hv * inv[:, None]).astype(f32) * weff[None, :]).astype(f32))


def _head_inv_rms(v, d, eps):
    """v: [n, d] fp32 -> [n] inverse RMS with the reference's tree
    (nvfp4_attention_front.cu:72-82): pair t = (element t, element t + d/2)
    is one thread with partial x^2 + y^2 (two rounded products, one rounded
    sum); 32 consecutive pairs reduce by shfl_down, the warp partials by a
    second zero-padded shfl_down; then rsqrtf(sum/d + eps)."""
    half = d // 2
    x, y = v[:, :half], v[:, half:]
    pairs = ((x * x).astype(f32) + (y * y).astype(f32)).astype(f32)
    total = _block_sum(pairs)
    mean = (total / f32(d)).astype(f32)
    return MATH.rsqrt((mean + f32(eps)).astype(f32))


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


def gate_fp8(out, gate, static_scale=None):
    """FP8 epilogue (``nvfp4_bucket_xqa.cu:56-62``): g = bf16(sigmoid(gate));
    v = bf16(out*g); code = e4m3_satfinite(v/scale) with the reference's
    static per-tensor ``static_scale``, or (None) a per-token scale
    max(amax_row/448, FLT_MIN).  Returns (codes [rows,N] u8, scale [rows] f32)."""
    out = np.asarray(out, dtype=f32)
    sg = F.bf16_round(sigmoid_f(gate))
    v = F.bf16_round((out * sg).astype(f32))
    if static_scale is None:
        amax = np.abs(v).max(axis=-1).astype(f32)
        scale = np.maximum((amax / f32(448.0)).astype(f32), f32(np.finfo(np.float32).tiny)).astype(f32)
    else:
        scale = np.full(v.shape[0], static_scale, dtype=f32)
    codes = F.e4m3_encode((v / scale[:, None]).astype(f32))
    return codes, scale


def swiglu_nvfp4(gate_acc, up_acc, alpha, global_scale):
    """gate_up GEMM epilogue: gate = bf16(acc*alpha), up = bf16(acc*alpha),
    act = bf16(gate/(1+expf(-gate)) * up) (the SiLU-and-mul order), then the
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
