"""CPU oracle of the decode-side bucket attention (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
may import this module.

Two parts:

* ``task_plan`` / ``route``: the KV-tile partition of the bucket decode
  attention, restated from the reference's CPU planner
  (``src/qwen_infra/kernels/nvfp4_bucket_xqa.py:19-69``) and its route rule
  (``src/qwen_infra/kernels/nvfp4_kv_bucket_worker.py:9-31``).  The page size
  is a parameter: the reference hard-codes 32-token pages (its table width
  counts 32-token pages), this build's cache uses 16-token pages.  With
  ``page_size=32`` both reproduce the recorded reference outputs in
  ``tests/golden/decode_plans.json`` exactly.
* ``decode_attention``: one query token per request against its paged NVFP4
  K/V (the same cache the prefill path appends to), softmax(q K^T s) V with the
  arithmetic of the CUDA kernel: K and V are the exact e2m1 x e4m3 products,
  the query group is written as a sum of ``Q_TERMS`` NVFP4 terms (``q_terms``:
  the kernel's S product runs block-scaled on the cached K codes), keys run in
  blocks of 128 with a deferred running max
  (moved only when a score exceeds it by more than 2^8), P is rounded to f16
  for the PV product, the running sum takes the unrounded exponentials, and
  task partials combine by exp2(m_i - m) weights.  The
  optional FP8 tail follows ``kernels/nvfp4_bucket_xqa.cu:48-66``:
  g = bf16(sigmoid(gate)), v = bf16(bf16(out) * g), code = e4m3(v / scale).
"""

import numpy as np
import torch

from . import formats as F
from . import producers as P

f32 = np.float32
TILE = 256  # tokens per plan unit (``nvfp4_bucket_xqa.py:13``)
BLOCK = 128  # keys per MMA block inside a tile


def _ceil(a, b):
    return (a + b - 1) // b


def task_plan(lengths, *, ctas=170, cyclic=False, aligned=False, table_width=None, page_size=32):
    """Tasks [request, begin_tile, end_tile, stride], per-request [first, count],
    per-CTA bucket [begin, end) of task slots, header [budget|splits, tasks,
    active, max count].  Mode 0 (default): requests' tiles laid end to end and
    cut into buckets of ``budget`` tiles; cyclic (mode 1): ``splits`` tasks per
    request taking every splits-th tile; aligned (mode 2): the smallest budget
    whose per-request ceil(tiles/budget) tasks fit in ``ctas``."""
    if (not 1 <= len(lengths) <= 32 or not len(lengths) <= ctas <= 340
            or any(type(n) is not int or n < 0 for n in lengths) or (cyclic and aligned)):
        raise ValueError("expected 1..32 lengths, batch <= ctas <= 340, one mode")
    width = max(1, _ceil(max(lengths), page_size)) if table_width is None else table_width
    if width < 1 or max(lengths) > width * page_size:
        raise ValueError("the page table must cover every length")
    counts = [_ceil(n, TILE) for n in lengths]
    budget = max(2, _ceil(sum(counts), ctas))
    if aligned:
        budget = 1
        while sum(_ceil(n, budget) for n in counts) > ctas:
            budget += 1
    splits = min(max(1, ctas // len(lengths)), _ceil(width * page_size, TILE))
    tasks, requests, buckets, prefix = [], [], [[0, 0] for _ in range(ctas)], 0
    for r, n in enumerate(counts):
        first = len(tasks)
        if cyclic:
            tasks += [[r, s, n, splits] for s in range(splits)]
        elif aligned:
            parts = _ceil(n, budget)
            tasks += [[r, s * n // parts, (s + 1) * n // parts, 1] for s in range(parts)]
        elif n:
            for b in range(prefix // budget, (prefix + n - 1) // budget + 1):
                if buckets[b][0] == buckets[b][1]:
                    buckets[b][0] = len(tasks)
                tasks.append([r, max(prefix, b * budget) - prefix, min(prefix + n, (b + 1) * budget) - prefix, 1])
                buckets[b][1] = len(tasks)
        requests.append([first, len(tasks) - first])
        prefix += n
    if aligned:
        for slot in range(len(tasks)):
            buckets[slot] = [slot, slot + 1]
    active = len(tasks) if cyclic or aligned else _ceil(prefix, budget)
    return dict(tasks=tasks, requests=requests, buckets=buckets,
                header=[splits if cyclic else budget, len(tasks), active, max(c for _, c in requests)])


def route(lengths, *, table_width, sm_count, forced="auto", page_size=32):
    """Geometry rule choosing the task mode: "persistent" (interval buckets)
    when cyclic splitting would leave one task with at least twice the
    interval budget, "aligned" when every cyclic task holds at most one tile
    and some would be empty, else "native" (cyclic).  Batches the reference
    does not pad to (other than 1, 8, 16, 24, 32 rows) and all-empty batches
    take "native"."""
    if forced not in ("auto", "native", "persistent", "aligned"):
        raise ValueError("expected auto/native/persistent/aligned")
    supported = (len(lengths) in (1, 8, 16, 24, 32) and len(lengths) <= sm_count <= 340 and table_width >= 1
                 and all(0 <= n <= table_width * page_size for n in lengths) and any(lengths))
    if not supported:
        return "native"
    tiles = [_ceil(n, TILE) for n in lengths]
    splits = min(max(1, sm_count // len(lengths)), _ceil(table_width * page_size, TILE))
    bucket = max(2, _ceil(sum(tiles), sm_count))
    critical = max(_ceil(n, splits) for n in tiles)
    empty = len(lengths) * splits - sum(min(n, splits) for n in tiles)
    auto = "persistent" if critical >= 2 * bucket else "aligned" if critical == 1 and empty > 0 else "native"
    return auto if forced == "auto" else forced


def plan_tiles(task):
    """KV tiles (256-token units) a task covers, in processing order."""
    _, lo, hi, stride = task
    return list(range(lo, hi, stride))


def _f16(x):
    return x.to(torch.float16).to(torch.float32)


Q_TERMS = 4  # NVFP4 terms of the query group in the kernel's S product


def _e2m1_codes_values(codes):
    return F.e2m1_decode(codes).astype(f32)


def q_terms(qh, terms=Q_TERMS):
    """The query group [G, D] (bf16 values) as a sum of NVFP4 terms, as the
    kernel builds its S operand: term t quantises the residual r_t per 16
    elements with the power-of-two global g_t = 2^floor(log2(2688 / amax_t))
    (amax over the group; 2688/amax clamped to [2^-100, 2^100]), scale =
    e4m3(min(amax16 * g_t * (1/6), 448)), code = e2m1(r * (g_t / scale)), and
    r_{t+1} = r_t - code * scale / g_t (each step one fp32 operation).
    Returns [(code * scale [G, D] float32, 1 / g_t)] per term (a zero group
    gives zero terms)."""
    r = np.asarray(qh, dtype=f32).copy()
    g_rows, d = r.shape
    out = []
    for _ in range(terms):
        amax = f32(np.abs(r).max()) if r.size else f32(0)
        if not amax > 0:
            out.append((np.zeros_like(r), 0.0))
            continue
        y = min(max(f32(f32(2688.0) / amax), f32(2.0 ** -100)), f32(2.0 ** 100))
        g = f32(2.0 ** int(np.floor(np.log2(np.float64(y)))))
        ig = f32(1.0) / g
        blk = r.reshape(g_rows, d // 16, 16)
        am16 = np.abs(blk).max(axis=-1).astype(f32)
        pre = np.minimum(((am16 * g).astype(f32) * f32(1.0 / 6.0)).astype(f32), f32(448.0))
        scale = F.e4m3_decode(F.e4m3_encode(pre)).astype(f32)
        inv = np.where(scale > 0, (g / np.where(scale > 0, scale, f32(1))).astype(f32), f32(0)).astype(f32)
        cv = _e2m1_codes_values(F.e2m1_encode((blk * inv[:, :, None]).astype(f32)))
        unscaled = (cv * scale[:, :, None]).astype(f32)
        r = (blk - (unscaled * ig).astype(f32)).astype(f32).reshape(g_rows, d)
        out.append((unscaled.reshape(g_rows, d), float(ig)))
    return out


MAX_LAG = 8.0  # log2 headroom of the deferred running maximum


def _task_partial(terms, kh, vh, tiles, length, scale2):
    """(O [G, D] unnormalised, m [G] log2 domain, l [G]) of one task for one KV
    head.  The running maxima move (all heads at once, to the block maximum)
    only on the task's first block or when some score of a block exceeds its
    head's maximum by more than ``MAX_LAG``; otherwise P = exp2(s - m) <= 2^8."""
    g = terms[0][0].shape[0]
    tq = [torch.from_numpy(t.astype(np.float64)) for t, _ in terms]
    cg = [float(f32(f32(ig) * f32(scale2))) for _, ig in terms]
    m = torch.full((g,), float("-inf"))
    l = torch.zeros(g)
    o = torch.zeros(g, vh.shape[1])
    for t in tiles:
        for b0 in range(t * TILE, min(t * TILE + TILE, length), BLOCK):
            b1 = min(b0 + BLOCK, length)
            kb = kh[b0:b1].double()
            s = sum((t @ kb.T) * c for t, c in zip(tq, cg)).float()  # [G, keys], log2 units
            if bool(torch.isinf(m).any()) or bool((s > m[:, None] + MAX_LAG).any()):
                m_new = torch.maximum(m, s.max(dim=1).values)
                alpha = torch.where(m == float("-inf"), torch.zeros_like(m), torch.exp2(m - m_new))
                l = l * alpha
                o = o * alpha[:, None]
                m = m_new
            p = torch.exp2(s - m[:, None])
            l = l + p.sum(dim=1)
            o = o + _f16(p) @ vh[b0:b1]
    return o, m, l


def decode_attention(q, k, v, lengths, plan, *, softmax_scale, k_global, v_global):
    """q [B, Hq, D] (bf16 values as float32); k, v [B] lists of [L_b, Hkv, D]
    dequantised unscaled products (``model.KVCache.gather`` with globals 1).
    Returns out [B, Hq, D] float32 (zeros for empty requests)."""
    bsz, hq, d = q.shape
    out = torch.zeros(bsz, hq, d)
    scale2 = float(f32(f32(softmax_scale) * f32(k_global)) * f32(1.4426950408889634))
    for r in range(bsz):
        n = lengths[r]
        if n == 0:
            continue
        first, count = plan["requests"][r]
        kr = torch.from_numpy(np.ascontiguousarray(k[r], dtype=f32))
        vr = torch.from_numpy(np.ascontiguousarray(v[r], dtype=f32))
        hkv = kr.shape[1]
        grp = hq // hkv
        qr = np.ascontiguousarray(q[r], dtype=f32)
        for h in range(hkv):
            terms = q_terms(qr[h * grp:(h + 1) * grp])
            parts = [_task_partial(terms, kr[:, h], vr[:, h], plan_tiles(plan["tasks"][s]), n, scale2)
                     for s in range(first, first + count)]
            mx = torch.stack([p[1] for p in parts]).max(dim=0).values
            o = torch.zeros(grp, d)
            l = torch.zeros(grp)
            for po, pm, pl in parts:
                w = torch.where(pm == float("-inf"), torch.zeros_like(pm), torch.exp2(pm - mx))
                o += po * w[:, None]
                l += pl * w
            out[r, h * grp:(h + 1) * grp] = o * float(v_global) / l[:, None]
    return out.numpy()


def decode_attention_exact(q, k, v, lengths, *, softmax_scale, k_global, v_global):
    """fp64 softmax attention of the same inputs (no f16 rounding of q or P)."""
    bsz, hq, d = q.shape
    out = np.zeros((bsz, hq, d), np.float64)
    for r in range(bsz):
        n = lengths[r]
        if n == 0:
            continue
        kr = np.asarray(k[r], np.float64) * float(k_global)
        vr = np.asarray(v[r], np.float64) * float(v_global)
        grp = hq // kr.shape[1]
        for h in range(hq):
            s = kr[:, h // grp] @ np.asarray(q[r, h], np.float64) * float(softmax_scale)
            p = np.exp(s - s.max())
            out[r, h] = (p / p.sum()) @ vr[:, h // grp]
    return out


def fp8_tail(out, gate, scale):
    """Gated FP8 output with a static scale (``nvfp4_bucket_xqa.cu:48-66``)."""
    ob = F.bf16_round(np.asarray(out, f32))
    sg = F.bf16_round(P.sigmoid_f(np.asarray(gate, f32)))
    v = F.bf16_round((ob * sg).astype(f32))
    return F.e4m3_encode((v / f32(scale)).astype(f32))
