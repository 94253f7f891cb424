"""CPU oracle — number formats of the folded-VPP prefill path (TEST INFRASTRUCTURE ONLY).

This module is a checker.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it; the
product path never does.

Formats are restated from their published definitions (OCP Microscaling v1.0
for E2M1, OCP OFP8 for E4M3), not from any vendor conversion routine:

* E2M1 magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}; round-to-nearest-even on the
  code's mantissa bit; saturate to 6 ("satfinite"); sign bit = bit 3.  Two
  codes per byte, element ``2j`` in the LOW nibble — the order the reference
  producer packs with (``kernels/nvfp4_norm_pack.cu:58-63``: pair ``(y[2j],
  y[2j+1])`` into byte ``j``).
* E4M3 (fn variant): bias 7, subnormals, max 448, NaN = 0x7F/0xFF; conversion
  is round-to-nearest-even with saturation to ±448 — the ``__nv_fp8_e4m3(float)``
  constructor semantics the reference relies on (``nvfp4_norm_pack.cu:53``,
  ``nvfp4_attention_front.cu:50``, ``nvfp4_bucket_xqa.cu:59``).
* The 128x4 swizzled block-scale layout generalises ``scale_offset``
  (``kernels/nvfp4_norm_pack.py:12-15``) from H=5120 to any K with K % 64 == 0.

Parity status: E4M3 is pinned against ``torch.float8_e4m3fn`` conversion and the
swizzle against the reference's ``scale_offset`` (``tests/test_oracle_pins.py``);
E2M1 rounding is checked on the GPU against the hardware ``cvt`` instruction.
"""

import numpy as np

E2M1_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float64)


def _e4m3_positive_values():
    vals = []
    for code in range(127):  # 0x00 .. 0x7E ; 0x7F is NaN
        e = code >> 3
        m = code & 7
        if e == 0:
            vals.append(m / 8.0 * 2.0 ** -6)
        else:
            vals.append((1.0 + m / 8.0) * 2.0 ** (e - 7))
    return np.array(vals, dtype=np.float64)


E4M3_VALUES = _e4m3_positive_values()  # index == code for codes 0..126
E4M3_MAX = 448.0


def _round_to_grid(a, grid):
    """Round non-negative float64 ``a`` onto sorted ``grid`` (index == code),
    nearest with ties to the even code, saturating at the top.  Returns codes."""
    a = np.minimum(a, grid[-1])
    lo = np.searchsorted(grid, a, side="right") - 1
    lo = np.clip(lo, 0, len(grid) - 1)
    hi = np.minimum(lo + 1, len(grid) - 1)
    d_lo = a - grid[lo]
    d_hi = grid[hi] - a
    take_hi = (d_hi < d_lo) | ((d_hi == d_lo) & ((lo & 1) == 1))
    return np.where(take_hi, hi, lo).astype(np.int64)


def e2m1_encode_grid(x):
    """float32 array -> uint8 codes 0..15 by nearest-even search on the grid."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    code = _round_to_grid(a, E2M1_VALUES)
    sign = np.signbit(x).astype(np.int64) << 3
    return (code | sign).astype(np.uint8)


def e2m1_encode(x):
    """float32 array -> uint8 codes 0..15 (one code per element).

    Same result as :func:`e2m1_encode_grid`, written as the count of decision
    thresholds passed: the midpoints 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5 of
    neighbouring codes, where a tie goes to the even code (strict '>' when the
    lower neighbour is even, '>=' when the upper one is)."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x)
    code = ((a > 0.25).astype(np.uint8) + (a >= 0.75) + (a > 1.25) + (a >= 1.75) + (a > 2.5) + (a >= 3.5)
            + (a > 5.0)).astype(np.uint8)
    return (code | (np.signbit(x).astype(np.uint8) << 3)).astype(np.uint8)


def e2m1_decode(codes):
    codes = np.asarray(codes, dtype=np.uint8)
    mag = E2M1_VALUES[codes & 7]
    return np.where(codes & 8, -mag, mag).astype(np.float32)


def e4m3_encode(x):
    """float32 array -> uint8 E4M3 codes (RN-even, satfinite, NaN -> 0x7F)."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    nan = np.isnan(x)
    a = np.where(nan, 0.0, a)
    code = _round_to_grid(a, E4M3_VALUES)
    sign = np.signbit(x).astype(np.int64) << 7
    out = (code | sign).astype(np.uint8)
    return np.where(nan, np.uint8(0x7F), out).astype(np.uint8)


def e4m3_decode(codes):
    codes = np.asarray(codes, dtype=np.uint8)
    mag_code = codes & 0x7F
    mag = np.where(mag_code == 0x7F, np.nan, E4M3_VALUES[np.minimum(mag_code, 126)])
    return np.where(codes & 0x80, -mag, mag).astype(np.float32)


def pack_nibbles(codes):
    """[..., 2n] uint8 codes -> [..., n] bytes, element 2j in the low nibble."""
    codes = np.asarray(codes, dtype=np.uint8)
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(packed):
    packed = np.asarray(packed, dtype=np.uint8)
    out = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = packed & 0xF
    out[..., 1::2] = packed >> 4
    return out


def bf16_round(x):
    """float32 -> float32 holding the nearest bfloat16 (RN-even); NaN kept."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def bf16_bits(x):
    """float32 already on the bf16 grid -> uint16 payload."""
    x = np.ascontiguousarray(bf16_round(x))
    return (x.view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits):
    bits = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return bits.view(np.float32)


def scale_groups_padded(k):
    """Number of 16-element groups per row, padded to the 4-group atom."""
    if k % 16:
        raise ValueError("K must be a multiple of 16")
    g = k // 16
    return (g + 3) // 4 * 4


def scale_offset(row, group, k):
    """Byte offset of the E4M3 scale of (row, 16-element group) in the 128x4
    swizzled layout; generalises ``kernels/nvfp4_norm_pack.py:12-15`` (where
    K = 5120 gives the 40960-byte row-block stride)."""
    gp = scale_groups_padded(k)
    row = np.asarray(row, dtype=np.int64)
    group = np.asarray(group, dtype=np.int64)
    return ((row // 128) * (128 * gp) + (group // 4) * 512 + (row % 32) * 16
            + ((row % 128) // 32) * 4 + group % 4)


def scale_buffer_bytes(rows, k):
    return (rows + 127) // 128 * 128 * scale_groups_padded(k)


def swizzle_scales(codes_rows_groups, k):
    """[rows, K/16] uint8 -> flat swizzled buffer (padding bytes zero)."""
    rows, groups = codes_rows_groups.shape
    out = np.zeros(scale_buffer_bytes(rows, k), dtype=np.uint8)
    r = np.repeat(np.arange(rows), groups)
    g = np.tile(np.arange(groups), rows)
    out[scale_offset(r, g, k)] = codes_rows_groups.reshape(-1)
    return out


def unswizzle_scales(buf, rows, k):
    groups = k // 16
    r = np.repeat(np.arange(rows), groups)
    g = np.tile(np.arange(groups), rows)
    return np.asarray(buf, dtype=np.uint8)[scale_offset(r, g, k)].reshape(rows, groups)


def nvfp4_dequant(packed, scales_swizzled, rows, k, global_scale):
    """NVFP4 bytes [rows, K/2] + swizzled E4M3 scales -> float32 [rows, K]
    with value = e2m1 * scale / global (the convention of
    ``nvfp4_norm_pack.cu:52-54``: scale = amax*global/6, code = y*global/scale)."""
    vals = e2m1_decode(unpack_nibbles(np.asarray(packed).reshape(rows, k // 2)))
    sc = e4m3_decode(unswizzle_scales(scales_swizzled, rows, k)).astype(np.float32)
    vals = vals.reshape(rows, k // 16, 16) * sc[:, :, None]
    return (vals.reshape(rows, k) / np.float32(global_scale)).astype(np.float32)
