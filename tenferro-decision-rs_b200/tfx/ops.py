"""Torch-tensor front end of the libtfx C ABI, named after the reference's
extension-op API (crates/tenferro-ext, crates/tenferro-infer).

Layout convention: the reference's column-major tensors are viewed as torch
row-major tensors with the axes reversed. A feature-first activation (d, cols)
is a torch tensor of shape (cols, d); a feature-last (rows, width) activation is
a torch tensor of shape (width, rows). Every function takes contiguous CUDA
tensors, enqueues on torch's current stream, returns a new tensor (or writes
`out`), and raises TfxError on any failure -- there is no CPU fallback.
"""

from __future__ import annotations

import ctypes

import torch

from ._lib import (RopeDesc, SoftmaxDesc, TFX_ACT_GELU_ERF, TFX_ACT_IDENTITY, TFX_ACT_RELU,
                   TFX_SOFTMAX_EXCLUDE, TFX_SOFTMAX_FILL, check, lib)

__all__ = [
    "erf", "gelu_erf", "geglu", "gated_silu", "gated_silu_stacked", "bias_act", "add",
    "layer_norm_feature_first", "rms_norm_last", "masked_softmax", "rope_tables",
    "rope_pairhalf", "gemm_geglu", "gemm_bias_act", "TFX_ACT_IDENTITY", "TFX_ACT_GELU_ERF", "TFX_ACT_RELU",
    "TFX_SOFTMAX_EXCLUDE", "TFX_SOFTMAX_FILL",
]


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(t=None):
    dev = t.device if t is not None else None
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _cuda(t, dtype, name):
    if t is None:
        return None
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA {dtype} tensor "
                         f"(got {t.device}, {t.dtype}, contiguous={t.is_contiguous()})")
    return t


def erf(x, out=None):
    _cuda(x, x.dtype, "x")
    y = torch.empty_like(x) if out is None else out
    fn = lib.tfx_erf_f32 if x.dtype == torch.float32 else lib.tfx_erf_f64
    check(fn(_ptr(x), _ptr(y), x.numel(), _stream(x)))
    return y


def gelu_erf(x, out=None):
    _cuda(x, x.dtype, "x")
    y = torch.empty_like(x) if out is None else out
    fn = lib.tfx_gelu_erf_f32 if x.dtype == torch.float32 else lib.tfx_gelu_erf_f64
    check(fn(_ptr(x), _ptr(y), x.numel(), _stream(x)))
    return y


def geglu(u, intermediate, out=None):
    """GegluOp: u is feature-first (2*I, cols) = torch (cols, 2*I)."""
    _cuda(u, torch.float32, "u")
    cols = u.numel() // (2 * intermediate)
    y = torch.empty((cols, intermediate), dtype=u.dtype, device=u.device) if out is None else out
    check(lib.tfx_geglu_ff_f32(_ptr(u), _ptr(y), intermediate, cols, _stream(u)))
    return y


def gated_silu(gate, up, out=None):
    _cuda(gate, torch.float32, "gate")
    _cuda(up, torch.float32, "up")
    y = torch.empty_like(gate) if out is None else out
    check(lib.tfx_gated_silu_f32(_ptr(gate), _ptr(up), _ptr(y), gate.numel(), _stream(gate)))
    return y


def gated_silu_stacked(gu, rows, inter, out=None):
    _cuda(gu, torch.float32, "gu")
    y = torch.empty((inter, rows), dtype=gu.dtype, device=gu.device) if out is None else out
    check(lib.tfx_gated_silu_stacked_f32(_ptr(gu), _ptr(y), rows, inter, _stream(gu)))
    return y


def bias_act(x, bias, act=TFX_ACT_IDENTITY, features=None, out=None):
    """x is feature-first (features, tokens) = torch (tokens, features)."""
    _cuda(x, torch.float32, "x")
    _cuda(bias, torch.float32, "bias")
    features = bias.numel() if features is None else features
    tokens = x.numel() // features
    y = torch.empty_like(x) if out is None else out
    check(lib.tfx_bias_act_ff_f32(_ptr(x), _ptr(bias), _ptr(y), features, tokens, act,
                                  _stream(x)))
    return y


def add(a, b, out=None):
    _cuda(a, torch.float32, "a")
    _cuda(b, torch.float32, "b")
    y = torch.empty_like(a) if out is None else out
    check(lib.tfx_add_f32(_ptr(a), _ptr(b), _ptr(y), a.numel(), _stream(a)))
    return y


def layer_norm_feature_first(x, weight, bias=None, eps=1e-5, out=None):
    """LayerNormFeatureFirstOp: x is (d, cols) = torch (cols, d), d = weight.numel()."""
    _cuda(x, x.dtype, "x")
    d = weight.numel()
    cols = x.numel() // d
    y = torch.empty_like(x) if out is None else out
    if x.dtype == torch.float32:
        check(lib.tfx_layernorm_ff_f32(_ptr(x), _ptr(weight), _ptr(bias), _ptr(y), d, cols,
                                       ctypes.c_float(eps), _stream(x)))
    else:
        check(lib.tfx_layernorm_ff_f64(_ptr(x), _ptr(weight), _ptr(bias), _ptr(y), d, cols,
                                       ctypes.c_double(eps), _stream(x)))
    return y


def rms_norm_last(x, weight, centered, eps, out=None):
    """RmsNormLastOp: x is column-major (rows, width) = torch (width, rows).

    As EagerSessionRmsNormExt::rms_norm_last, eps is given as an f64 and used
    as its f32 truncation for f32 inputs (crates/tenferro-ext/src/rms_norm.rs:186)."""
    _cuda(x, x.dtype, "x")
    width = weight.numel()
    rows = x.numel() // width
    y = torch.empty_like(x) if out is None else out
    if x.dtype == torch.float32:
        check(lib.tfx_rmsnorm_last_f32(_ptr(x), _ptr(weight), _ptr(y), rows, width,
                                       int(bool(centered)), ctypes.c_float(eps), _stream(x)))
    else:
        check(lib.tfx_rmsnorm_last_f64(_ptr(x), _ptr(weight), _ptr(y), rows, width,
                                       int(bool(centered)), ctypes.c_double(eps), _stream(x)))
    return y


def masked_softmax(scores, batch, heads, q_len, k_len, *, scale=1.0,
                   semantics=TFX_SOFTMAX_EXCLUDE, causal=False, window=-1,
                   window_skips_invalid_query=False, valid_len=-1, valid_lens=None,
                   add_mask=None, add_strides=(0, 0, 0), keep=None, keep_strides=(0, 0, 0),
                   out=None):
    _cuda(scores, torch.float32, "scores")
    d = SoftmaxDesc()
    lib.tfx_softmax_desc_init(ctypes.byref(d), batch, heads, q_len, k_len)
    d.scale = scale
    d.semantics = semantics
    d.causal = int(bool(causal))
    d.window = window
    d.window_skips_invalid_query = int(bool(window_skips_invalid_query))
    d.valid_len = valid_len
    if valid_lens is not None:
        _cuda(valid_lens, torch.int32, "valid_lens")
        d.valid_lens = valid_lens.data_ptr()
    if add_mask is not None:
        _cuda(add_mask, torch.float32, "add_mask")
        d.add_mask = add_mask.data_ptr()
        d.add_stride_b, d.add_stride_q, d.add_stride_k = add_strides
    if keep is not None:
        _cuda(keep, torch.uint8, "keep")
        d.keep = keep.data_ptr()
        d.keep_stride_b, d.keep_stride_q, d.keep_stride_k = keep_strides
    y = torch.empty_like(scores) if out is None else out
    check(lib.tfx_masked_softmax_f32(_ptr(scores), _ptr(y), ctypes.byref(d), _stream(scores)))
    return y


def rope_tables(base, seq, rotary_dim, device="cuda"):
    """The reference's f64-angle, f32-rounded cos/sin tables (seq, rotary_dim/2)."""
    half = rotary_dim // 2
    c = torch.empty((seq, half), dtype=torch.float32)
    s = torch.empty((seq, half), dtype=torch.float32)
    check(lib.tfx_rope_tables_f32(ctypes.c_double(base), seq, rotary_dim, _ptr(c), _ptr(s)))
    if device == "cpu":
        return c, s
    return c.to(device), s.to(device)


def rope_pairhalf(x, cos_t, sin_t, n_vec, seq, batch, head_dim, rotary_dim, strides,
                  out=None):
    """strides = (stride_vec, stride_pos, stride_batch, stride_feat) in elements."""
    _cuda(x, torch.float32, "x")
    d = RopeDesc(n_vec, seq, batch, head_dim, rotary_dim, *strides)
    y = torch.empty_like(x) if out is None else out
    check(lib.tfx_rope_pairhalf_f32(_ptr(x), _ptr(y), _ptr(cos_t), _ptr(sin_t), ctypes.byref(d),
                                    _stream(x)))
    return y


def rope_tables_powf(base, seq, rotary_dim, device="cuda"):
    """cpu-kernels' f32 tables (powf, cosf, sinf), (seq, rotary_dim/2)."""
    half = rotary_dim // 2
    c = torch.empty((seq, half), dtype=torch.float32)
    s = torch.empty((seq, half), dtype=torch.float32)
    check(lib.tfx_rope_tables_powf_f32(ctypes.c_float(base), seq, rotary_dim, _ptr(c), _ptr(s)))
    if device == "cpu":
        return c, s
    return c.to(device), s.to(device)


def laya_attention_block(qkv, keep, hidden, heads, length, batch, cos_t=None, sin_t=None,
                         out=None):
    """LayaAttentionBlockOp: qkv (3*hidden, length, batch) feature-first, keep
    (length, length, batch) uint8 (query fastest) -> (hidden, length, batch)."""
    _cuda(qkv, torch.float32, "qkv")
    _cuda(keep, torch.uint8, "keep")
    y = torch.empty(hidden * length * batch, device=qkv.device) if out is None else out
    check(lib.tfx_laya_attention_block_f32(_ptr(qkv), _ptr(keep), _ptr(cos_t), _ptr(sin_t),
                                           _ptr(y), hidden, heads, length, batch, _stream(qkv)))
    return y


def jeff_attention(q, k, v, gate, q_norm, k_norm, mask, cos_t, sin_t, length, heads, head_dim,
                   rotary_dim, eps, out=None):
    """jeff_full_attention_into: q, k, v, gate (length, heads*head_dim) time-first."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (gate, "gate")):
        _cuda(t, torch.float32, n)
    y = torch.empty_like(q) if out is None else out
    check(lib.tfx_jeff_attention_f32(_ptr(q), _ptr(k), _ptr(v), _ptr(gate), _ptr(q_norm),
                                     _ptr(k_norm), _ptr(mask), _ptr(cos_t), _ptr(sin_t), _ptr(y),
                                     length, heads, head_dim, rotary_dim, ctypes.c_float(eps),
                                     _stream(q)))
    return y


def add_layer_norm_feature_first(a, b, weight, bias=None, eps=1e-5, sum_out=None, out=None):
    """s = a + b and LayerNorm(s) in one pass (feature-first (d, cols)); returns
    (s or None, y). Bit-identical to add() then layer_norm_feature_first()."""
    _cuda(a, torch.float32, "a")
    _cuda(b, torch.float32, "b")
    d = weight.numel()
    y = torch.empty_like(a) if out is None else out
    check(lib.tfx_add_layernorm_ff_f32(_ptr(a), _ptr(b), _ptr(weight), _ptr(bias), _ptr(sum_out),
                                       _ptr(y), d, a.numel() // d, ctypes.c_float(eps),
                                       _stream(a)))
    return sum_out, y


def embedding_gather(table, ids, hidden, vocab, length, layout, out=None):
    """Gather with device int64 ids; layout 0 rows (time-first out), 1 columns
    (feature-first out)."""
    _cuda(table, torch.float32, "table")
    y = torch.empty(hidden * length, device=table.device) if out is None else out
    check(lib.tfx_embedding_gather_f32(_ptr(table), _ptr(ids), _ptr(y), hidden, vocab, length,
                                       layout, _stream(table)))
    return y


def gemm_geglu(x, weight, bias, intermediate, out=None):
    """GemmGegluOp: x feature-first (in_dim, length) = torch (length, in_dim),
    weight (in_dim, 2*intermediate) column-major = torch (2*intermediate,
    in_dim), bias (2*intermediate) or None -> (intermediate, length) = torch
    (length, intermediate)."""
    _cuda(x, torch.float32, "x")
    _cuda(weight, torch.float32, "weight")
    _cuda(bias, torch.float32, "bias")
    in_dim = weight.numel() // (2 * intermediate) if intermediate else 0
    length = x.numel() // in_dim if in_dim else 0
    y = torch.empty((length, intermediate), dtype=x.dtype, device=x.device) if out is None \
        else out
    check(lib.tfx_gemm_geglu_ff_f32(_ptr(x), _ptr(weight), _ptr(bias), _ptr(y), in_dim,
                                    intermediate, length, _stream(x)))
    return y


def gemm_bias_act(x, weight, bias, out_dim, act=TFX_ACT_IDENTITY, out=None):
    """GemmBiasOp with an activation: x (in_dim, length), weight (in_dim,
    out_dim) column-major = torch (out_dim, in_dim) -> (out_dim, length)."""
    _cuda(x, torch.float32, "x")
    _cuda(weight, torch.float32, "weight")
    _cuda(bias, torch.float32, "bias")
    in_dim = weight.numel() // out_dim if out_dim else 0
    length = x.numel() // in_dim if in_dim else 0
    y = torch.empty((length, out_dim), dtype=x.dtype, device=x.device) if out is None else out
    check(lib.tfx_gemm_bias_act_ff_f32(_ptr(x), _ptr(weight), _ptr(bias), _ptr(y), in_dim,
                                       out_dim, length, act, _stream(x)))
    return y
