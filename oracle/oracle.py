"""ctypes binding of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

The oracle (``oracle.cpp``) restates the reference's host arithmetic for the
non-GEMM extension-op path (crates/cpu-kernels/src/lib.rs, crates/tenferro-ext,
crates/tenferro-infer). Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline legs import this module, as the checker or as the
timed CPU baseline; the product path never does.

All arrays are numpy, C-contiguous, float32 / float64 as named.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i64 = ctypes.c_int64
_int = ctypes.c_int


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (gcc, no GPU needed)."""
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH)
        < max(os.path.getmtime(os.path.join(_HERE, f)) for f in ("oracle.cpp", "oracle.h"))
    ):
        subprocess.run(["make", "-s", "-B", "liboracle.so"], cwd=_HERE, check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L: ctypes.CDLL) -> None:
    sig = {
        "orc_set_threads": (None, [_int]),
        "orc_threads": (_int, []),
        "orc_erf_f32": (ctypes.c_float, [ctypes.c_float]),
        "orc_expm1_mlx_f32": (ctypes.c_float, [ctypes.c_float]),
        "orc_gelu_erf_f32": (ctypes.c_float, [ctypes.c_float]),
        "orc_erf_f32_n": (None, [_f32p, _f32p, _i64]),
        "orc_gelu_erf_f32_n": (None, [_f32p, _f32p, _i64]),
        "orc_layer_norm_feature_first_f32": (
            None, [_f32p, _i64, _i64, _f32p, _f32p, ctypes.c_float, _f32p]),
        "orc_geglu_f32": (None, [_f32p, _i64, _i64, _f32p]),
        "orc_rms_norm_last_f32": (None, [_f32p, _i64, _i64, _f32p, _int, ctypes.c_float, _f32p]),
        "orc_gated_silu_f32": (None, [_f32p, _f32p, _f32p, _i64]),
        "orc_bias_add_f32": (None, [_f32p, _f32p, _f32p, _i64, _i64]),
        "orc_bias_act_f32": (None, [_f32p, _f32p, _f32p, _i64, _i64, _int]),
        "orc_gemm_bias_f32": (None, [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64]),
        "orc_add_f32": (None, [_f32p, _f32p, _f32p, _i64]),
        "orc_masked_softmax_f32": (None, [
            _f32p, _f32p, _i64, _i64, _i64, _i64, ctypes.c_float, _int, _int, _i64, _int,
            _i64, _i32p, _f32p, _i64, _i64, _i64, _u8p, _i64, _i64, _i64]),
        "orc_rope_tables_f32": (None, [ctypes.c_double, _i64, _i64, _f32p, _f32p]),
        "orc_rope_tables_f64": (None, [ctypes.c_double, _i64, _i64, _f64p, _f64p]),
        "orc_rope_pairhalf_f32": (None, [
            _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64]),
        "orc_rope_pairhalf_f64": (None, [
            _f64p, _f64p, _f64p, _f64p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64]),
        "orc_rope_tables_powf_f32": (None, [ctypes.c_float, _i64, _i64, _f32p, _f32p]),
        "orc_laya_qkv_prep_f32": (None, [
            _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _f32p, _f32p, _f32p]),
        "orc_laya_attention_block_f32": (None, [
            _f32p, _u8p, _i64, _i64, _i64, _i64, _f32p, _f32p, _f32p]),
        "orc_jeff_qkv_prep_f32": (None, [
            _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64,
            ctypes.c_float, _f32p, _f32p, _f32p]),
        "orc_jeff_full_attention_f32": (None, [
            _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64,
            ctypes.c_float, ctypes.c_float, _f32p]),
        "orc_embedding_f32": (None, [_f32p, ctypes.POINTER(ctypes.c_int64), _f32p, _i64, _i64,
                                     _i64, _i64, _i64, _i64]),
        "orc_erf_f64": (ctypes.c_double, [ctypes.c_double]),
        "orc_erf_f64_n": (None, [_f64p, _f64p, _i64]),
        "orc_gelu_erf_f64_n": (None, [_f64p, _f64p, _i64]),
        "orc_layer_norm_feature_first_f64": (
            None, [_f64p, _i64, _i64, _f64p, _f64p, ctypes.c_double, _f64p]),
        "orc_rms_norm_last_f64": (
            None, [_f64p, _i64, _i64, _f64p, _int, ctypes.c_double, _f64p]),
        "orc_softmax_rows_f64": (None, [_f64p, _f64p, _i64, _i64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p32(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous, (a.dtype, a.flags)
    return a.ctypes.data_as(_f32p)


def _p64(a):
    if a is None:
        return None
    assert a.dtype == np.float64 and a.flags.c_contiguous, (a.dtype, a.flags)
    return a.ctypes.data_as(_f64p)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def threads() -> int:
    return int(lib().orc_threads())


# ---- f32 cpu-kernels restatements ------------------------------------------

def erf_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().orc_erf_f32_n(_p32(x), _p32(y), x.size)
    return y


def gelu_erf_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().orc_gelu_erf_f32_n(_p32(x), _p32(y), x.size)
    return y


def expm1_mlx_f32(a: float) -> float:
    return float(lib().orc_expm1_mlx_f32(ctypes.c_float(a)))


def layer_norm_feature_first_f32(x, d, cols, weight, bias, eps, out=None):
    y = np.empty(d * cols, dtype=np.float32) if out is None else out
    assert y.size == d * cols
    lib().orc_layer_norm_feature_first_f32(_p32(x), d, cols, _p32(weight), _p32(bias),
                                           ctypes.c_float(eps), _p32(y))
    return y


def geglu_f32(u, inter, cols, out=None):
    y = np.empty(inter * cols, dtype=np.float32) if out is None else out
    assert y.size == inter * cols
    lib().orc_geglu_f32(_p32(u), inter, cols, _p32(y))
    return y


def rms_norm_last_f32(x, rows, width, weight, centered, eps):
    y = np.empty(rows * width, dtype=np.float32)
    lib().orc_rms_norm_last_f32(_p32(x), rows, width, _p32(weight), int(bool(centered)),
                                ctypes.c_float(eps), _p32(y))
    return y


def gated_silu_f32(gate, up):
    y = np.empty(gate.size, dtype=np.float32)
    lib().orc_gated_silu_f32(_p32(gate), _p32(up), _p32(y), gate.size)
    return y


def bias_add_f32(x, bias, features, tokens):
    y = np.empty(features * tokens, dtype=np.float32)
    lib().orc_bias_add_f32(_p32(x), _p32(bias), _p32(y), features, tokens)
    return y


def bias_act_f32(x, bias, features, tokens, act):
    y = np.empty(features * tokens, dtype=np.float32)
    lib().orc_bias_act_f32(_p32(x), _p32(bias), _p32(y), features, tokens, int(act))
    return y


def gemm_bias_f32(x, weight, bias, in_dim, out_dim, length):
    y = np.empty(out_dim * length, dtype=np.float32)
    lib().orc_gemm_bias_f32(_p32(x), _p32(weight), _p32(bias), _p32(y), in_dim, out_dim, length)
    return y


def add_f32(a, b, out=None):
    y = np.empty(a.size, dtype=np.float32) if out is None else out
    assert y.size == a.size == b.size
    lib().orc_add_f32(_p32(a), _p32(b), _p32(y), a.size)
    return y


def masked_softmax_f32(scores, batch, heads, q_len, k_len, *, scale=1.0, semantics=0,
                       causal=False, window=-1, window_skips_invalid_query=False,
                       valid_len=-1, valid_lens=None, add_mask=None, add_strides=(0, 0, 0),
                       keep=None, keep_strides=(0, 0, 0), out=None):
    p = np.empty(batch * heads * q_len * k_len, dtype=np.float32) if out is None else out
    assert p.size == batch * heads * q_len * k_len
    vl = None
    if valid_lens is not None:
        valid_lens = np.ascontiguousarray(valid_lens, dtype=np.int32)
        vl = valid_lens.ctypes.data_as(_i32p)
    kp = None
    if keep is not None:
        keep = np.ascontiguousarray(keep, dtype=np.uint8)
        kp = keep.ctypes.data_as(_u8p)
    lib().orc_masked_softmax_f32(
        _p32(scores), _p32(p), batch, heads, q_len, k_len, ctypes.c_float(scale),
        int(semantics), int(bool(causal)), int(window), int(bool(window_skips_invalid_query)),
        int(valid_len), vl, _p32(add_mask), *[int(s) for s in add_strides], kp,
        *[int(s) for s in keep_strides])
    return p


def rope_tables_f32(base, seq, rotary_dim):
    half = rotary_dim // 2
    c = np.empty(seq * half, dtype=np.float32)
    s = np.empty(seq * half, dtype=np.float32)
    lib().orc_rope_tables_f32(ctypes.c_double(base), seq, rotary_dim, _p32(c), _p32(s))
    return c, s


def rope_tables_f64(base, seq, rotary_dim):
    half = rotary_dim // 2
    c = np.empty(seq * half, dtype=np.float64)
    s = np.empty(seq * half, dtype=np.float64)
    lib().orc_rope_tables_f64(ctypes.c_double(base), seq, rotary_dim, _p64(c), _p64(s))
    return c, s


def rope_pairhalf_f32(x, cos_t, sin_t, n_vec, seq, batch, head_dim, rotary_dim, strides,
                      out_size=None, out=None):
    """Rotated copy of x. With `out`, only the described vectors are written
    into it (the rest of `out` is left as it was)."""
    if out is not None:
        assert out.size == x.size
        y = out
    else:
        y = np.array(x, copy=True) if out_size is None else np.zeros(out_size, np.float32)
    lib().orc_rope_pairhalf_f32(_p32(x), _p32(y), _p32(cos_t), _p32(sin_t), n_vec, seq, batch,
                                head_dim, rotary_dim, *[int(s) for s in strides])
    return y


def rope_pairhalf_f64(x, cos_t, sin_t, n_vec, seq, batch, head_dim, rotary_dim, strides):
    y = np.array(x, copy=True)
    lib().orc_rope_pairhalf_f64(_p64(x), _p64(y), _p64(cos_t), _p64(sin_t), n_vec, seq, batch,
                                head_dim, rotary_dim, *[int(s) for s in strides])
    return y


# ---- attention blocks (cpu-kernels lib.rs:618-760, :819-1150) -----------------

def rope_tables_powf_f32(base, seq, rotary_dim):
    half = rotary_dim // 2
    c = np.empty(max(1, seq * half), dtype=np.float32)
    s = np.empty(max(1, seq * half), dtype=np.float32)
    lib().orc_rope_tables_powf_f32(ctypes.c_float(base), seq, rotary_dim, _p32(c), _p32(s))
    return c[:seq * half], s[:seq * half]


def laya_qkv_prep_f32(qkv, hidden, heads, length, batch, cos_t=None, sin_t=None):
    n = hidden * length * batch
    qh, kh, vh = (np.empty(n, np.float32) for _ in range(3))
    lib().orc_laya_qkv_prep_f32(_p32(qkv), _p32(cos_t), _p32(sin_t), hidden, heads, length, batch,
                                _p32(qh), _p32(kh), _p32(vh))
    return qh, kh, vh


def laya_attention_block_f32(qkv, keep, hidden, heads, length, batch, cos_t=None, sin_t=None):
    assert keep.dtype == np.uint8 and keep.size == length * length * batch
    out = np.empty(hidden * length * batch, np.float32)
    lib().orc_laya_attention_block_f32(_p32(qkv), keep.ctypes.data_as(_u8p), hidden, heads,
                                       length, batch, _p32(cos_t), _p32(sin_t), _p32(out))
    return out


def jeff_qkv_prep_f32(q, k, v, q_norm, k_norm, cos_t, sin_t, length, heads, head_dim,
                      rotary_dim, eps):
    n = length * heads * head_dim
    qh, kh, vh = (np.empty(n, np.float32) for _ in range(3))
    dummy = np.zeros(1, np.float32)
    lib().orc_jeff_qkv_prep_f32(
        _p32(q), _p32(k), _p32(v), _p32(q_norm), _p32(k_norm),
        _p32(cos_t if cos_t is not None and cos_t.size else dummy),
        _p32(sin_t if sin_t is not None and sin_t.size else dummy),
        length, heads, head_dim, rotary_dim, ctypes.c_float(eps), _p32(qh), _p32(kh), _p32(vh))
    return qh, kh, vh


def jeff_full_attention_f32(q, k, v, gate, q_norm, k_norm, mask, length, heads, head_dim,
                            rotary_dim, theta, eps):
    out = np.empty(length * heads * head_dim, np.float32)
    lib().orc_jeff_full_attention_f32(
        _p32(q), _p32(k), _p32(v), _p32(gate), _p32(q_norm), _p32(k_norm), _p32(mask), length,
        heads, head_dim, rotary_dim, ctypes.c_float(theta), ctypes.c_float(eps), _p32(out))
    return out


def embedding_f32(table, ids, hidden, vocab, layout):
    """layout 0 (rows): table (hidden, vocab) row-major -> out (length, hidden)
    time-first; layout 1 (columns): table column-major -> out (hidden, length)."""
    length = ids.size
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    out = np.empty(hidden * length, np.float32)
    strides = (1, length, vocab, 1) if layout == 0 else (hidden, 1, 1, hidden)
    lib().orc_embedding_f32(_p32(table), ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                            _p32(out), hidden, length, *strides)
    return out


# ---- f64 composites ----------------------------------------------------------

def erf_f64(x):
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.empty_like(x)
    lib().orc_erf_f64_n(_p64(x), _p64(y), x.size)
    return y


def gelu_erf_f64(x):
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.empty_like(x)
    lib().orc_gelu_erf_f64_n(_p64(x), _p64(y), x.size)
    return y


def layer_norm_feature_first_f64(x, d, cols, weight, bias, eps):
    y = np.empty(d * cols, dtype=np.float64)
    lib().orc_layer_norm_feature_first_f64(_p64(x), d, cols, _p64(weight), _p64(bias),
                                           ctypes.c_double(eps), _p64(y))
    return y


def rms_norm_last_f64(x, rows, width, weight, centered, eps):
    y = np.empty(rows * width, dtype=np.float64)
    lib().orc_rms_norm_last_f64(_p64(x), rows, width, _p64(weight), int(bool(centered)),
                                ctypes.c_double(eps), _p64(y))
    return y


def softmax_rows_f64(x, rows, cols):
    y = np.empty(rows * cols, dtype=np.float64)
    lib().orc_softmax_rows_f64(_p64(x), _p64(y), rows, cols)
    return y


# ---- GEMM with an epilogue (crates/tenferro-ext/src/gemm_geglu.rs:209-238,
# gemm_bias.rs:76-142): the sequential projection, then the epilogue op ------

def gemm_geglu_f32(x, weight, bias, in_dim, intermediate, length):
    """p = bias (or 0) + x.W over (in_dim, length) x (in_dim, 2I), then
    geglu_into over (2I, length) -> (I, length)."""
    out = 2 * intermediate
    b = np.zeros(out, np.float32) if bias is None else bias
    p = gemm_bias_f32(x, weight, b, in_dim, out, length)
    return geglu_f32(p, intermediate, length)


def gemm_bias_act_f32(x, weight, bias, in_dim, out_dim, length, act):
    b = np.zeros(out_dim, np.float32) if bias is None else bias
    p = gemm_bias_f32(x, weight, b, in_dim, out_dim, length)
    return bias_act_f32(p, None, out_dim, length, act)
