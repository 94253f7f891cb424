"""ctypes binding of ``libqwen_infra_b200.so`` (declarations: include/qwen_infra_b200.h).

Loading never falls back to anything: a missing or unloadable library raises.
"""

import ctypes as ct
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqwen_infra_b200.so"

STATUS_BAD_KV_SCALE = 1
STATUS_WAIT_TIMEOUT = 2
STATUS_BAD_SLOT = 4

GEMM_NVFP4, GEMM_E4M3 = 0, 1
EPI_BF16, EPI_F32, EPI_SWIGLU_NVFP4, EPI_BF16_ROWCOL = 0, 1, 2, 3

_vp = ct.c_void_p
_i32, _i64, _f32 = ct.c_int, ct.c_int64, ct.c_float


class RefFront(ct.Structure):
    """Field-for-field the reference's ``Front`` (nvfp4_attention_front.py:13-67)."""

    _fields_ = (
        [(n, _vp) for n in ("qkv", "qw", "kw", "cos_sin", "positions", "slots", "k_scale", "v_scale",
                            "k", "v", "ks", "vs", "q", "gate")]
        + [(n, _i32) for n in ("rows", "qheads", "kvheads", "rotary", "slot_rows", "pages", "page_size",
                               "cos_float", "pos_long", "slot_long", "mrope_h", "mrope_w")]
        + [(n, _i64) for n in ("input_row", "cos_row", "pos_m", "pos_t", "data_page", "data_row", "data_head",
                               "sf_page", "sf_row", "sf_head")]
        + [("epsilon", _f32)]
    )


class QiFront(ct.Structure):
    _fields_ = (
        [(n, _vp) for n in ("qkv", "q_weight", "k_weight", "cos_sin", "positions", "slots", "k_global",
                            "v_global", "k_cache", "v_cache", "k_scales", "v_scales", "q", "gate", "status")]
        + [(n, _i32) for n in ("rows", "qheads", "kvheads", "head_dim", "slot_rows", "pages", "page_size",
                               "cos_float", "pos_long", "slot_long")]
        + [(n, _i64) for n in ("input_row", "cos_row", "q_row", "gate_row", "data_page", "data_row",
                               "data_head", "sf_page", "sf_row", "sf_head")]
        + [("eps", _f32), ("weight_offset", _f32)]
    )


class QiGemm(ct.Structure):
    _fields_ = [
        ("kind", _i32), ("epilogue", _i32), ("m", _i32), ("n", _i32), ("k", _i32),
        ("a", _vp), ("b", _vp), ("sfa", _vp), ("sfb", _vp), ("alpha", _vp), ("alpha_value", _f32),
        ("row_scale", _vp), ("col_scale", _vp), ("out", _vp), ("ldo", _i64),
        ("act_q", _vp), ("act_sf", _vp), ("act_global", _vp), ("act_ld", _i64), ("status", _vp),
    ]


class QiKvView(ct.Structure):
    _fields_ = (
        [(n, _vp) for n in ("k_cache", "v_cache", "k_scales", "v_scales")]
        + [(n, _i32) for n in ("kvheads", "head_dim", "page_size")]
        + [(n, _i64) for n in ("data_page", "data_row", "data_head", "sf_page", "sf_row", "sf_head")]
    )


class QiAttention(ct.Structure):
    _fields_ = (
        [(n, _vp) for n in ("q", "k", "vt", "out", "k_global", "v_global", "status")]
        + [(n, _i32) for n in ("rows", "history", "kv_tokens", "qheads", "kvheads", "head_dim")]
        + [(n, _i64) for n in ("q_row", "out_row", "vt_row")]
        + [("softmax_scale", _f32), ("workspace", _vp), ("workspace_bytes", _i64)]
    )


class QiPagedAttention(ct.Structure):
    _fields_ = (
        [("q", _vp), ("out", _vp), ("kv", QiKvView), ("block_table", _vp), ("k_global", _vp), ("v_global", _vp),
         ("status", _vp)]
        + [(n, _i32) for n in ("rows", "history", "qheads")]
        + [(n, _i64) for n in ("q_row", "out_row")]
        + [("softmax_scale", _f32), ("workspace", _vp), ("workspace_bytes", _i64)]
    )


class QiDecode(ct.Structure):
    _fields_ = (
        [("q", _vp), ("kv", QiKvView)]
        + [(n, _vp) for n in ("block_table", "lengths", "tasks", "requests", "buckets", "header", "semaphores",
                              "scratch", "out", "gate", "out_scale", "k_global", "v_global", "status")]
        + [(n, _i32) for n in ("batch", "ctas", "table_width", "mode", "persistent", "qheads")]
        + [("softmax_scale", _f32)]
    )


EXPORTS = {
    "nvfp4_norm_pack_launch": ([_vp] * 7 + [_i32, _vp], _i32),
    "nvfp4_norm_pack_metadata": ([ct.POINTER(_i32)], _i32),
    "qi_norm_pack": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _f32, _f32, _vp], _i32),
    "qi_rms_norm": ([_vp, _vp, _vp, _vp, _vp, _i32, _i32, _f32, _f32, _vp], _i32),
    "nvfp4_attention_front": ([RefFront, _vp], _i32),
    "nvfp4_attention_front_resources": ([ct.POINTER(_i32)], _i32),
    "qi_qk_rope_kv_append": ([ct.POINTER(QiFront), _vp], _i32),
    "qi_qk_rope_kv_append_resources": ([ct.POINTER(_i32)], _i32),
    "qi_gate_fp8": ([_vp, _vp, _i64, _i64, _vp, _i64, _vp, _i32, _i32, _vp], _i32),
    "qi_gate_fp8_heads": ([_vp, _vp, _i64, _i64, _i64, _i32, _vp, _i64, _vp, _i32, _i32, _vp], _i32),
    "qi_gate_fp8_static": ([_vp, _vp, _i64, _i64, _i64, _i32, _vp, _i64, _vp, _i32, _i32, _vp], _i32),
    "qi_gemm": ([ct.POINTER(QiGemm), _vp], _i32),
    "qi_gemm_resources": ([ct.POINTER(_i32)], _i32),
    "qi_kv_dequant": ([ct.POINTER(QiKvView), _vp, _i32, _vp, _vp, _i64, _vp], _i32),
    "qi_kv_dequant_range": ([ct.POINTER(QiKvView), _vp, _i32, _i32, _vp, _i64, _vp, _i64, _vp], _i32),
    "qi_swiglu_nvfp4": ([_vp, _i64, _i32, _i32, _vp, _vp, _i64, _vp, _vp], _i32),
    "qi_lm_head_argmax": ([_vp, _i64, _i32, _i32, _vp, _i32, _vp, _vp, _vp, _vp], _i32),
    "qi_lm_head_workspace_bytes": ([], _i32),
    "qi_prefill_attention": ([ct.POINTER(QiAttention), _vp], _i32),
    "qi_paged_prefill_attention": ([ct.POINTER(QiPagedAttention), _vp], _i32),
    "qi_prefill_attention_workspace_bytes": ([_i32, ct.POINTER(_i64)], _i32),
    "qi_nvfp4_quantize": ([_vp, _i64, _i32, _vp, _vp, _vp, _vp], _i32),
    "qi_fp8_quantize_rows": ([_vp, _i32, _i32, _vp, _vp, _vp], _i32),
    "qi_abi_struct_sizes": ([ct.POINTER(_i32)], _i32),
    "qi_convert_probe": ([_vp, _vp, _vp, _vp, _i32, _vp], _i32),
    "qi_decode_assign": ([ct.POINTER(QiDecode), _vp], _i32),
    "qi_decode_attention": ([ct.POINTER(QiDecode), _vp], _i32),
    "qi_decode_resources": ([ct.POINTER(_i32)], _i32),
    "qi_decode_scratch_bytes": ([_i32, _i32], ct.c_uint64),
}

_lib = None


def lib():
    """Load the kernel library once; raise if it is missing (no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH.name} is not built; run __graft_entry__.build()")
        handle = ct.CDLL(str(LIB_PATH))
        for name, (args, res) in EXPORTS.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = res
        sizes = (ct.c_int * 7)()
        if handle.qi_abi_struct_sizes(sizes):
            raise RuntimeError("qi_abi_struct_sizes failed")
        expected = [ct.sizeof(c) for c in (RefFront, QiFront, QiGemm, QiKvView, QiAttention, QiDecode,
                                           QiPagedAttention)]
        if list(sizes) != expected:
            raise RuntimeError(f"C ABI struct sizes {list(sizes)} != ctypes {expected}")
        _lib = handle
    return _lib


def check(status, what):
    if status:
        raise RuntimeError(f"{what} CUDA launch status {status}")
