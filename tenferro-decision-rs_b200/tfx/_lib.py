"""ctypes declarations of libtfx's C ABI (include/tfx.h).

The library is the in-tree tenferro-decision-rs_b200/lib/libtfx.so built by
build.py. There is no fallback: if it is missing or does not load, importing
this module raises.
"""

from __future__ import annotations

import ctypes
import os
import re

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "lib", "libtfx.so")
HEADER = os.path.join(ROOT, "include", "tfx.h")

TFX_OK = 0
TFX_ERR_INVALID_ARGUMENT = -1
TFX_ERR_UNSUPPORTED = -2
TFX_ERR_CUDA = -3

TFX_ACT_IDENTITY = 0
TFX_ACT_GELU_ERF = 1
TFX_ACT_RELU = 2

TFX_SOFTMAX_EXCLUDE = 0
TFX_SOFTMAX_FILL = 1


class TfxError(RuntimeError):
    """A libtfx call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


class SoftmaxDesc(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64), ("heads", ctypes.c_int64), ("q_len", ctypes.c_int64),
        ("k_len", ctypes.c_int64), ("scale", ctypes.c_float), ("semantics", ctypes.c_int32),
        ("causal", ctypes.c_int32), ("window_skips_invalid_query", ctypes.c_int32),
        ("window", ctypes.c_int64), ("valid_len", ctypes.c_int64),
        ("valid_lens", ctypes.c_void_p), ("add_mask", ctypes.c_void_p),
        ("add_stride_b", ctypes.c_int64), ("add_stride_q", ctypes.c_int64),
        ("add_stride_k", ctypes.c_int64), ("keep", ctypes.c_void_p),
        ("keep_stride_b", ctypes.c_int64), ("keep_stride_q", ctypes.c_int64),
        ("keep_stride_k", ctypes.c_int64),
    ]


class RopeDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in (
        "n_vec", "seq", "batch", "head_dim", "rotary_dim", "stride_vec", "stride_pos",
        "stride_batch", "stride_feat")]


class AttentionDesc(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64), ("heads", ctypes.c_int64), ("length", ctypes.c_int64),
        ("head_dim", ctypes.c_int64), ("scale", ctypes.c_float), ("empty_rows", ctypes.c_int32),
        ("causal", ctypes.c_int32), ("window", ctypes.c_int64), ("valid_len", ctypes.c_int64),
        ("keep", ctypes.c_void_p), ("bias", ctypes.c_void_p), ("active", ctypes.c_void_p),
        ("gate", ctypes.c_void_p), ("gate_offset", ctypes.c_int64), ("out_tok", ctypes.c_int64),
        ("out_feat", ctypes.c_int64), ("out_batch", ctypes.c_int64),
    ]


_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float

SIGNATURES = {
    "tfx_last_error_string": (ctypes.c_char_p, []),
    "tfx_version": (_int, []),
    "tfx_wait_timeouts": (_int, [_p]),
    "tfx_erf_f32": (_int, [_p, _p, _i64, _p]),
    "tfx_gelu_erf_f32": (_int, [_p, _p, _i64, _p]),
    "tfx_erf_f64": (_int, [_p, _p, _i64, _p]),
    "tfx_gelu_erf_f64": (_int, [_p, _p, _i64, _p]),
    "tfx_geglu_ff_f32": (_int, [_p, _p, _i64, _i64, _p]),
    "tfx_gated_silu_f32": (_int, [_p, _p, _p, _i64, _p]),
    "tfx_gated_silu_stacked_f32": (_int, [_p, _p, _i64, _i64, _p]),
    "tfx_bias_act_ff_f32": (_int, [_p, _p, _p, _i64, _i64, _int, _p]),
    "tfx_add_f32": (_int, [_p, _p, _p, _i64, _p]),
    "tfx_gemm_geglu_ff_f32": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _p]),
    "tfx_gemm_bias_act_ff_f32": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "tfx_layernorm_ff_f32": (_int, [_p, _p, _p, _p, _i64, _i64, ctypes.c_float, _p]),
    "tfx_layernorm_ff_f64": (_int, [_p, _p, _p, _p, _i64, _i64, ctypes.c_double, _p]),
    "tfx_rmsnorm_last_f32": (_int, [_p, _p, _p, _i64, _i64, _int, ctypes.c_float, _p]),
    "tfx_rmsnorm_last_f64": (_int, [_p, _p, _p, _i64, _i64, _int, ctypes.c_double, _p]),
    "tfx_rmsnorm_last_f32_noalloc": (_int, [_p, _p, _p, _i64, _i64, _int, ctypes.c_float, _p]),
    "tfx_softmax_desc_init": (None, [ctypes.POINTER(SoftmaxDesc), _i64, _i64, _i64, _i64]),
    "tfx_masked_softmax_f32": (_int, [_p, _p, ctypes.POINTER(SoftmaxDesc), _p]),
    "tfx_rope_pairhalf_f32": (_int, [_p, _p, _p, _p, ctypes.POINTER(RopeDesc), _p]),
    "tfx_rope_tables_f32": (_int, [ctypes.c_double, _i64, _i64, _p, _p]),
    "tfx_rope_tables_powf_f32": (_int, [_f32, _i64, _i64, _p, _p]),
    "tfx_add_layernorm_ff_f32": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _f32, _p]),
    "tfx_embedding_f32": (_int, [_p, _p, _p, _i64, _i64, _i64, ctypes.c_int32, _p]),
    "tfx_embedding_gather_f32": (_int, [_p, _p, _p, _i64, _i64, _i64, ctypes.c_int32, _p]),
    "tfx_laya_qkv_prep_f32": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p]),
    "tfx_jeff_qkv_prep_f32": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                                     _i64, _f32, _p]),
    "tfx_attention_desc_init": (_int, [ctypes.POINTER(AttentionDesc), _i64, _i64, _i64, _i64]),
    "tfx_attention_f32": (_int, [_p, _p, _p, _p, ctypes.POINTER(AttentionDesc), _p]),
    "tfx_laya_attention_block_f32": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p]),
    "tfx_jeff_attention_f32": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                                      _i64, _f32, _p]),
    "tfx_session_create": (_int, [_int, ctypes.POINTER(ctypes.c_void_p)]),
    "tfx_session_destroy": (_int, [_p]),
    "tfx_session_set_chunk_bytes": (_int, [_p, _i64]),
    "tfx_session_layernorm_ff_f32": (_int, [_p, _p, _p, _p, _p, _i64, _i64, ctypes.c_float]),
    "tfx_session_layernorm_ff_f64": (_int, [_p, _p, _p, _p, _p, _i64, _i64, ctypes.c_double]),
    "tfx_session_rmsnorm_last_f32": (_int, [_p, _p, _p, _p, _i64, _i64, _int, ctypes.c_float]),
    "tfx_session_erf_f32": (_int, [_p, _p, _p, _i64]),
    "tfx_session_gelu_erf_f32": (_int, [_p, _p, _p, _i64]),
    "tfx_session_geglu_ff_f32": (_int, [_p, _p, _p, _i64, _i64]),
    "tfx_session_gated_silu_f32": (_int, [_p, _p, _p, _p, _i64]),
    "tfx_session_bias_act_ff_f32": (_int, [_p, _p, _p, _p, _i64, _i64, _int]),
    "tfx_session_add_f32": (_int, [_p, _p, _p, _p, _i64]),
    "tfx_session_gemm_geglu_ff_f32": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _i64]),
    "tfx_session_gemm_bias_act_ff_f32": (_int, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _int]),
    "tfx_session_add_layernorm_ff_f32": (_int, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64,
                                                ctypes.c_float]),
    "tfx_session_masked_softmax_f32": (_int, [_p, _p, _p, ctypes.POINTER(SoftmaxDesc)]),
    "tfx_session_rope_pairhalf_f32": (_int, [_p, _p, _p, ctypes.c_double,
                                             ctypes.POINTER(RopeDesc)]),
}


def header_symbols(path: str = HEADER) -> list[str]:
    """Every function the public header declares (TFX_API ... tfx_name()."""
    with open(path, encoding="utf-8") as fh:
        text = fh.read()
    return sorted(set(re.findall(r"TFX_API\s+[\w\s\*]+?\b(tfx_\w+)\s*\(", text)))


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libtfx.so not found at {LIB_PATH}; build it with "
            "`python tenferro-decision-rs_b200/build.py` (or __graft_entry__.build())")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error() -> str:
    return (lib.tfx_last_error_string() or b"").decode("utf-8", "replace")


def check(code: int) -> None:
    if code != TFX_OK:
        raise TfxError(code, last_error())
