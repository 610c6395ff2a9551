"""Host-buffer front end: the extension ops on host arrays through a libtfx
session (tfx_session_* in include/tfx.h) -- the executor a CPU eager session of
the reference would hand its TensorRead slices to.

Arrays may be numpy arrays or CPU torch tensors (pinned ones give the fastest,
fully asynchronous copies). Every call blocks until the outputs are written.
"""

from __future__ import annotations

import ctypes

import numpy as np

from ._lib import RopeDesc, SoftmaxDesc, TFX_ACT_IDENTITY, TFX_SOFTMAX_EXCLUDE, check, lib


def _hptr(a):
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        if not a.flags.c_contiguous:
            raise ValueError("host arrays must be C-contiguous")
        return ctypes.c_void_p(a.ctypes.data)
    if getattr(a, "is_cuda", False):
        raise ValueError("session calls take host arrays, not CUDA tensors")
    if not a.is_contiguous():
        raise ValueError("host tensors must be contiguous")
    return ctypes.c_void_p(a.data_ptr())


def _numel(a):
    return a.size if isinstance(a, np.ndarray) else a.numel()


def _empty_like(a, n=None, dtype=None):
    if isinstance(a, np.ndarray):
        return np.empty(a.size if n is None else n, dtype=a.dtype if dtype is None else dtype)
    import torch
    return torch.empty(a.numel() if n is None else n, dtype=a.dtype if dtype is None else dtype,
                       pin_memory=a.is_pinned())


class Session:
    """One GPU's streams and staging memory for host-buffer ext-op calls."""

    def __init__(self, device: int = 0, chunk_bytes: int | None = None):
        h = ctypes.c_void_p()
        check(lib.tfx_session_create(device, ctypes.byref(h)))
        self._h = h
        self.device = device
        if chunk_bytes is not None:
            check(lib.tfx_session_set_chunk_bytes(self._h, chunk_bytes))

    def close(self):
        if self._h:
            check(lib.tfx_session_destroy(self._h))
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- ops (argument meaning as the device entry points) ------------------------

    def layer_norm_feature_first(self, x, weight, bias=None, eps=1e-5, out=None):
        d = _numel(weight)
        cols = _numel(x) // d
        y = _empty_like(x) if out is None else out
        if (x.dtype == np.float64) or str(x.dtype) == "torch.float64":
            check(lib.tfx_session_layernorm_ff_f64(self._h, _hptr(x), _hptr(weight), _hptr(bias),
                                                   _hptr(y), d, cols, ctypes.c_double(eps)))
        else:
            check(lib.tfx_session_layernorm_ff_f32(self._h, _hptr(x), _hptr(weight), _hptr(bias),
                                                   _hptr(y), d, cols, ctypes.c_float(eps)))
        return y

    def rms_norm_last(self, x, weight, centered, eps, out=None):
        width = _numel(weight)
        rows = _numel(x) // width
        y = _empty_like(x) if out is None else out
        check(lib.tfx_session_rmsnorm_last_f32(self._h, _hptr(x), _hptr(weight), _hptr(y), rows,
                                               width, int(bool(centered)), ctypes.c_float(eps)))
        return y

    def erf(self, x, out=None):
        y = _empty_like(x) if out is None else out
        check(lib.tfx_session_erf_f32(self._h, _hptr(x), _hptr(y), _numel(x)))
        return y

    def gelu_erf(self, x, out=None):
        y = _empty_like(x) if out is None else out
        check(lib.tfx_session_gelu_erf_f32(self._h, _hptr(x), _hptr(y), _numel(x)))
        return y

    def geglu(self, u, intermediate, out=None):
        cols = _numel(u) // (2 * intermediate)
        y = _empty_like(u, intermediate * cols) if out is None else out
        check(lib.tfx_session_geglu_ff_f32(self._h, _hptr(u), _hptr(y), intermediate, cols))
        return y

    def gated_silu(self, gate, up, out=None):
        y = _empty_like(gate) if out is None else out
        check(lib.tfx_session_gated_silu_f32(self._h, _hptr(gate), _hptr(up), _hptr(y),
                                             _numel(gate)))
        return y

    def bias_act(self, x, bias, act=TFX_ACT_IDENTITY, features=None, out=None):
        features = _numel(bias) if features is None else features
        y = _empty_like(x) if out is None else out
        check(lib.tfx_session_bias_act_ff_f32(self._h, _hptr(x), _hptr(bias), _hptr(y), features,
                                              _numel(x) // features, act))
        return y

    def gemm_geglu(self, x, weight, bias, intermediate, out=None):
        """GemmGegluOp on host buffers: x (in_dim, length), weight (in_dim,
        2*intermediate) column-major, bias (2*intermediate) or None."""
        in_dim = _numel(weight) // (2 * intermediate) if intermediate else 0
        length = _numel(x) // in_dim if in_dim else 0
        y = _empty_like(x, intermediate * length) if out is None else out
        check(lib.tfx_session_gemm_geglu_ff_f32(self._h, _hptr(x), _hptr(weight), _hptr(bias),
                                                _hptr(y), in_dim, intermediate, length))
        return y

    def gemm_bias_act(self, x, weight, bias, out_dim, act=TFX_ACT_IDENTITY, out=None):
        """GemmBiasOp (+ activation) on host buffers: weight (in_dim, out_dim)."""
        in_dim = _numel(weight) // out_dim if out_dim else 0
        length = _numel(x) // in_dim if in_dim else 0
        y = _empty_like(x, out_dim * length) if out is None else out
        check(lib.tfx_session_gemm_bias_act_ff_f32(self._h, _hptr(x), _hptr(weight), _hptr(bias),
                                                   _hptr(y), in_dim, out_dim, length, act))
        return y

    def add(self, a, b, out=None):
        y = _empty_like(a) if out is None else out
        check(lib.tfx_session_add_f32(self._h, _hptr(a), _hptr(b), _hptr(y), _numel(a)))
        return y

    def add_layer_norm_feature_first(self, a, b, weight, bias=None, eps=1e-5, sum_out=None,
                                     out=None):
        """s = a + b and LayerNorm(s) on host buffers; returns (s or None, y)."""
        d = _numel(weight)
        y = _empty_like(a) if out is None else out
        check(lib.tfx_session_add_layernorm_ff_f32(self._h, _hptr(a), _hptr(b), _hptr(weight),
                                                   _hptr(bias), _hptr(sum_out), _hptr(y), d,
                                                   _numel(a) // d, ctypes.c_float(eps)))
        return sum_out, y

    def masked_softmax(self, scores, batch, heads, q_len, k_len, *, scale=1.0,
                       semantics=TFX_SOFTMAX_EXCLUDE, causal=False, window=-1,
                       window_skips_invalid_query=False, valid_len=-1, valid_lens=None,
                       add_mask=None, add_strides=(0, 0, 0), keep=None, keep_strides=(0, 0, 0),
                       out=None):
        d = SoftmaxDesc()
        lib.tfx_softmax_desc_init(ctypes.byref(d), batch, heads, q_len, k_len)
        d.scale, d.semantics, d.causal = scale, semantics, int(bool(causal))
        d.window, d.valid_len = window, valid_len
        d.window_skips_invalid_query = int(bool(window_skips_invalid_query))
        keep_alive = []
        if valid_lens is not None:
            vl = np.ascontiguousarray(valid_lens, dtype=np.int32)
            keep_alive.append(vl)
            d.valid_lens = vl.ctypes.data
        if add_mask is not None:
            d.add_mask = _hptr(add_mask).value
            d.add_stride_b, d.add_stride_q, d.add_stride_k = add_strides
        if keep is not None:
            k = np.ascontiguousarray(keep, dtype=np.uint8)
            keep_alive.append(k)
            d.keep = k.ctypes.data
            d.keep_stride_b, d.keep_stride_q, d.keep_stride_k = keep_strides
        y = _empty_like(scores) if out is None else out
        check(lib.tfx_session_masked_softmax_f32(self._h, _hptr(scores), _hptr(y),
                                                 ctypes.byref(d)))
        return y

    def rope_pairhalf(self, x, base, n_vec, seq, batch, head_dim, rotary_dim, strides, out=None):
        d = RopeDesc(n_vec, seq, batch, head_dim, rotary_dim, *strides)
        y = _empty_like(x) if out is None else out
        check(lib.tfx_session_rope_pairhalf_f32(self._h, _hptr(x), _hptr(y),
                                                ctypes.c_double(base), ctypes.byref(d)))
        return y
