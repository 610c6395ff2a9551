"""GPU parity: masked row softmax and RoPE.

Softmax compares within the f32 tolerance (CUDA expf vs glibc expf and the
tree-ordered sum); RoPE is bitwise (same f64-built tables, IEEE products)."""

import math

import numpy as np
import pytest
import torch

from gpu_util import P, S, call, dev, empty, host
from helpers import (golden_case, golden_tensor, assert_bitwise, assert_close, decode_value,
                     splitmix_normal, ulp_distance_f32, F32_RTOL, F32_ATOL_REL)
import tfx
from tfx import _lib
import ctypes

pytestmark = pytest.mark.gpu


def gpu_softmax(s, B, H, Lq, Lk, offset=0, in_place=False, **kw):
    sd = dev(s, offset)
    pd = sd if in_place else empty(s.size, offset_elems=offset)
    d = _lib.SoftmaxDesc()
    _lib.lib.tfx_softmax_desc_init(ctypes.byref(d), B, H, Lq, Lk)
    keepalive = []
    for k, v in kw.items():
        if k in ("valid_lens", "add_mask", "keep"):
            t = dev(v)
            keepalive.append(t)
            setattr(d, k, t.data_ptr())
        elif k == "add_strides":
            d.add_stride_b, d.add_stride_q, d.add_stride_k = v
        elif k == "keep_strides":
            d.keep_stride_b, d.keep_stride_q, d.keep_stride_k = v
        else:
            setattr(d, k, v)
    call("tfx_masked_softmax_f32", P(sd), P(pd), ctypes.byref(d), S())
    return host(pd)


def orc_kwargs(kw):
    out = dict(kw)
    if "window_skips_invalid_query" in out:
        out["window_skips_invalid_query"] = bool(out["window_skips_invalid_query"])
    return out


def test_softmax_config4_full_size(orc):
    """scores [8, 12, 512, 512] ~ N(0, 2); -inf outside a 128-token
    sliding window (|q-k| <= 64) and on the last 37 padded keys."""
    B, H, L = 8, 12, 512
    s = splitmix_normal(B * H * L * L, 0x7E4F0032, std=2.0)
    kw = dict(window=64, valid_len=L - 37)
    got = gpu_softmax(s, B, H, L, L, **kw)
    want = orc.masked_softmax_f32(s, B, H, L, L, **kw)
    st = assert_close(got, want, F32_RTOL, F32_ATOL_REL, "softmax config 4")
    rows = got.reshape(-1, L).astype(np.float64)
    assert np.max(np.abs(rows.sum(1) - 1.0)) < 1e-5
    q = np.arange(L)[:, None]
    k = np.arange(L)[None, :]
    masked = (np.abs(q - k) > 64) | (k >= L - 37)
    assert np.all(got.reshape(B * H, L, L)[:, masked] == 0.0)
    assert st["max_ulp"] <= 64


@pytest.mark.parametrize("semantics", [0, 1])
def test_softmax_additive_and_keep_masks_in_reference_layout(orc, semantics):
    """Masks as the reference stores them: keep / bias tensors (L_q, L_k, B)
    column-major, query fastest (laya-infer/src/model.rs:466-490)."""
    B, H, L = 2, 3, 64
    s = splitmix_normal(B * H * L * L, 0x7E4F0600, std=2.0)
    q = np.arange(L)[:, None, None]
    k = np.arange(L)[None, :, None]
    b = np.arange(B)[None, None, :]
    keep = ((np.abs(q - k) <= 8) & (k < L - 5 - b)).astype(np.uint8)  # [q][k][b]
    keep_cm = np.ascontiguousarray(keep.transpose(2, 1, 0)).ravel()  # q + L*(k + L*b)
    strides = (L * L, 1, L)
    add = np.where(keep_cm == 1, 0.0, -np.inf).astype(np.float32)
    got_keep = gpu_softmax(s, B, H, L, L, semantics=semantics, keep=keep_cm, keep_strides=strides)
    want = orc.masked_softmax_f32(s, B, H, L, L, semantics=semantics, keep=keep_cm,
                                  keep_strides=strides)
    assert_close(got_keep, want, F32_RTOL, F32_ATOL_REL, "softmax keep mask")
    got_add = gpu_softmax(s, B, H, L, L, semantics=0, add_mask=add, add_strides=strides)
    want_add = orc.masked_softmax_f32(s, B, H, L, L, semantics=0, add_mask=add, add_strides=strides)
    assert_close(got_add, want_add, F32_RTOL, F32_ATOL_REL, "softmax additive mask")
    # -inf added == masked (attention_with_bias vs bool mask, primitives.rs:447)
    assert np.max(np.abs(got_add - got_keep)) <= 1e-6


def test_softmax_laya_mask_with_valid_lens(orc):
    """Sliding layer mask of laya-infer/src/model.rs:474-483: padded queries see
    every valid key; per-sequence valid lengths."""
    B, H, L = 3, 2, 128
    s = splitmix_normal(B * H * L * L, 0x7E4F0610, std=2.0)
    vl = np.array([128, 100, 37], dtype=np.int32)
    kw = dict(window=16, valid_lens=vl, window_skips_invalid_query=1, scale=0.125)
    got = gpu_softmax(s, B, H, L, L, **kw)
    want = orc.masked_softmax_f32(s, B, H, L, L, **orc_kwargs(kw))
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, "softmax laya mask")


def test_softmax_empty_rows_and_masked_nonfinite(orc):
    """crates/cpu-kernels/src/lib.rs:1213-1250 on the softmax rows: masked NaN /
    inf never leak; all-masked rows are NaN (EXCLUDE) or uniform (FILL)."""
    c = golden_case("masked_attention_empty_rows_and_masked_nonfinite")
    L, key = c["length"], c["masked_key"]
    base = splitmix_normal(L * L, 0x7E4F0620)
    keep = np.ones((L, L), dtype=np.uint8)
    keep[:, key] = 0
    for q in c["empty_queries"]:
        keep[q, :] = 0
    keep = keep.ravel()
    ref = None
    for excluded in c["excluded_values"]:
        s = base.copy().reshape(L, L)
        s[:, key] = decode_value(excluded)
        s = s.ravel()
        got = gpu_softmax(s, 1, 1, L, L, keep=keep, keep_strides=(0, L, 1))
        want = orc.masked_softmax_f32(s, 1, 1, L, L, keep=keep, keep_strides=(0, L, 1))
        assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"excluded={excluded}")
        g = got.reshape(L, L)
        for q in c["empty_queries"]:
            assert np.all(np.isnan(g[q]))
        if ref is None:
            ref = got
        else:
            assert_bitwise(got, ref, "masked value leaked")
        fill = gpu_softmax(s, 1, 1, L, L, semantics=1, keep=keep, keep_strides=(0, L, 1))
        f = fill.reshape(L, L)
        for q in c["empty_queries"]:
            assert np.allclose(f[q], 1.0 / L)


@pytest.mark.parametrize("Lk,offset,semantics", [
    (1, 0, 0), (3, 0, 0), (20, 0, 0), (32, 0, 1), (65, 0, 1), (128, 1, 0), (320, 0, 0),
    (512, 0, 1), (640, 0, 1), (768, 0, 0), (1000, 0, 0), (1024, 0, 0),
    (2049, 0, 0), (4096, 0, 1), (8192, 0, 0), (9000, 0, 0), (9000, 0, 1)])
def test_softmax_row_lengths(orc, Lk, offset, semantics):
    B, H, Lq = 1, 2, 5
    s = splitmix_normal(B * H * Lq * Lk, 0x7E4F0630 + Lk, std=3.0)
    kw = dict(causal=1, semantics=semantics)
    got = gpu_softmax(s, B, H, Lq, Lk, offset=offset, **kw)
    want = orc.masked_softmax_f32(s, B, H, Lq, Lk, **kw)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"softmax Lk={Lk}")


@pytest.mark.parametrize("Lk", [16, 64, 256, 384, 512, 704, 1024])
@pytest.mark.parametrize("semantics", [0, 1])
def test_softmax_row_lengths_valid_len(orc, Lk, semantics):
    """Every lane-group width of the short-row kernel, rows not a multiple of
    the rows per CTA, a padded key tail (valid_len) instead of causality."""
    B, H, Lq = 3, 1, 7
    s = splitmix_normal(B * H * Lq * Lk, 0x7E4F0680 + Lk, std=3.0)
    kw = dict(valid_len=Lk - 3, semantics=semantics, scale=0.5)
    got = gpu_softmax(s, B, H, Lq, Lk, **kw)
    want = orc.masked_softmax_f32(s, B, H, Lq, Lk, **kw)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"softmax Lk={Lk}")


@pytest.mark.parametrize("window,Lq,Lk,semantics,extra", [
    (0, 40, 164, 0, {}), (1, 33, 256, 1, {"valid_len": 250}), (7, 64, 512, 0, {"causal": 1}),
    (33, 100, 2052, 1, {"scale": 0.125}), (64, 512, 512, 0, {"valid_len": 475}),
    (64, 512, 512, 1, {"valid_len": 475}), (77, 300, 4096, 0, {"valid_len": 200}),
    (78, 160, 640, 0, {}), (50, 9, 9000, 1, {"causal": 1, "valid_len": 7})])
def test_softmax_sliding_window_band(orc, window, Lq, Lk, semantics, extra):
    """Sliding windows short enough for the banded row kernel (|q-k| <= window,
    at most 40 kept float4 chunks, rows longer than that), rows at both sequence
    edges, padded keys, causal, queries past the keys; window 78 just past the
    band limit."""
    B, H = 2, 3
    s = splitmix_normal(B * H * Lq * Lk, 0x7E4F06A0 + window + Lk, std=3.0)
    kw = dict(window=window, semantics=semantics, **extra)
    got = gpu_softmax(s, B, H, Lq, Lk, **kw)
    want = orc.masked_softmax_f32(s, B, H, Lq, Lk, **kw)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"softmax band w={window} Lk={Lk}")
    if semantics == 0:  # keys outside the window: exactly 0 in every non-empty row
        q = np.arange(Lq)[:, None]
        k = np.arange(Lk)[None, :]
        rows_ok = np.isfinite(want.reshape(B * H, Lq, Lk)).all(axis=2)
        sel = rows_ok[:, :, None] & (np.abs(q - k) > window)[None]
        assert np.all(got.reshape(B * H, Lq, Lk)[sel] == 0.0)


def test_softmax_sliding_window_band_in_place(orc):
    B, H, L = 2, 4, 384
    s = splitmix_normal(B * H * L * L, 0x7E4F06B0, std=2.0)
    got = gpu_softmax(s, B, H, L, L, in_place=True, window=16, scale=0.125, valid_len=L - 9)
    want = orc.masked_softmax_f32(s, B, H, L, L, window=16, scale=0.125, valid_len=L - 9)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, "softmax band in place")


@pytest.mark.parametrize("semantics", [0, 1])
def test_softmax_wide_dynamic_range(orc, semantics):
    """Scores ~ N(0, 20): probabilities down to ~1e-40 (subnormal quotients,
    the row-wide IEEE division fallback) against glibc expf in the oracle."""
    B, H, L = 2, 4, 512
    s = splitmix_normal(B * H * L * L, 0x7E4F0670 + semantics, std=20.0)
    got = gpu_softmax(s, B, H, L, L, semantics=semantics, causal=1)
    want = orc.masked_softmax_f32(s, B, H, L, L, semantics=semantics, causal=1)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, "softmax wide range")
    big = want > 1e-30
    assert int(ulp_distance_f32(got[big], want[big]).max()) <= 64


def test_softmax_in_place_and_scale(orc):
    B, H, L = 2, 4, 256
    s = splitmix_normal(B * H * L * L, 0x7E4F0640, std=2.0)
    got = gpu_softmax(s, B, H, L, L, in_place=True, scale=0.125, causal=1)
    want = orc.masked_softmax_f32(s, B, H, L, L, scale=0.125, causal=1)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, "softmax in place")


def test_softmax_f64_primitive_rows(orc):
    """primitives.rs:125-162 data, f32 GPU vs the f64 composite, rows sum to 1."""
    c = golden_case("softmax_f64_primitive")
    rows, cols = c["rows"], c["cols"]
    x = np.ascontiguousarray(golden_tensor(c, "x").reshape(cols, rows).T)
    got = gpu_softmax(x.astype(np.float32).ravel(), 1, 1, rows, cols).reshape(rows, cols)
    want = orc.softmax_rows_f64(x.ravel(), rows, cols).reshape(rows, cols)
    assert np.max(np.abs(got - want)) < 1e-6
    assert np.max(np.abs(got.astype(np.float64).sum(1) - 1.0)) < 1e-6


# ---- RoPE ----------------------------------------------------------------------------

def gpu_rope(x, cos_t, sin_t, n_vec, seq, batch, head_dim, rot, strides, in_place=False,
             out_size=None):
    xd = dev(x)
    cd, sd = dev(cos_t), dev(sin_t)
    if in_place:
        yd = xd
    else:
        yd = torch.zeros(x.size if out_size is None else out_size, dtype=torch.float32,
                         device="cuda")
    desc = _lib.RopeDesc(n_vec, seq, batch, head_dim, rot, *strides)
    call("tfx_rope_pairhalf_f32", P(xd), P(yd), P(cd), P(sd), ctypes.byref(desc), S())
    return host(yd)


def host_tables(base, seq, rot):
    half = rot // 2
    c = np.empty(seq * half, np.float32)
    s = np.empty(seq * half, np.float32)
    rc = _lib.lib.tfx_rope_tables_f32(ctypes.c_double(base), seq, rot,
                                       c.ctypes.data_as(ctypes.c_void_p),
                                       s.ctypes.data_as(ctypes.c_void_p))
    assert rc == 0
    return c, s


@pytest.mark.parametrize("theta", [160000.0, 10000.0])
def test_rope_chain_layout_bitwise(orc, theta):
    """configs[4] layout: q and k blocks of a feature-first qkv (3*768, 512, B),
    head_dim 64, 12 heads each -> 24 rotated vectors per token."""
    hidden, heads, hd, L, B = 768, 12, 64, 512, 8
    x = splitmix_normal(3 * hidden * L * B, 0x7E4F0040)
    c, s = host_tables(theta, L, hd)
    oc, os_ = orc.rope_tables_f32(theta, L, hd)
    assert_bitwise(c, oc, "cos table")
    assert_bitwise(s, os_, "sin table")
    strides = (hd, 3 * hidden, 3 * hidden * L, 1)
    got = gpu_rope(x, c, s, 2 * heads, L, B, hd, hd, strides, in_place=True)
    want = orc.rope_pairhalf_f32(x, c, s, 2 * heads, L, B, hd, hd, strides)
    assert_bitwise(got, want, "rope chain")
    v = slice(2 * hidden, 3 * hidden)
    assert_bitwise(got.reshape(B * L, 3 * hidden)[:, v], x.reshape(B * L, 3 * hidden)[:, v],
                   "v untouched")


def test_rope_tenferro_infer_layout_and_partial(orc):
    """(heads, seq, head) column-major (tenferro-infer rope_qwen_partial layout):
    contiguous leading axis, channel stride heads*seq; partial rotary copies the tail."""
    heads, seq, head, rot = 6, 40, 16, 8
    x = splitmix_normal(heads * seq * head, 0x7E4F0650)
    c, s = host_tables(10000.0, seq, rot)
    strides = (1, heads, 0, heads * seq)
    got = gpu_rope(x, c, s, heads, seq, 1, head, rot, strides)
    want = orc.rope_pairhalf_f32(x, c, s, heads, seq, 1, head, rot, strides)
    assert_bitwise(got, want, "rope partial")


def test_rope_primitive_cases(orc):
    """primitives.rs:299-372: f32 GPU vs the f64 naive loops (1e-6 in f32)."""
    c = golden_case("rope_modernbert_f64_primitive")
    seq, head, base = c["seq"], c["head"], c["base"]
    x = golden_tensor(c, "x")
    ct, st = host_tables(base, seq, head)
    got = gpu_rope(x.astype(np.float32), ct, st, 1, seq, 1, head, head, (0, 1, 0, seq))
    c64, s64 = orc.rope_tables_f64(base, seq, head)
    want = orc.rope_pairhalf_f64(x, c64, s64, 1, seq, 1, head, head, (0, 1, 0, seq))
    assert np.max(np.abs(got - want)) < 1e-6
    for k in range(head):
        assert got[k * seq] == np.float32(x[k * seq])  # position 0 unchanged
    c = golden_case("rope_qwen_partial_f64_primitive")
    heads, seq, head, rot = c["heads"], c["seq"], c["head"], c["rotary"]
    data = np.array([i * 0.1 - 0.3 for i in range(heads * seq * head)])
    ct, st = host_tables(c["base"], seq, rot)
    got = gpu_rope(data.astype(np.float32), ct, st, heads, seq, 1, head, rot,
                   (1, heads, 0, heads * seq))
    c64, s64 = orc.rope_tables_f64(c["base"], seq, rot)
    want = orc.rope_pairhalf_f64(data, c64, s64, heads, seq, 1, head, rot,
                                 (1, heads, 0, heads * seq))
    assert np.max(np.abs(got - want)) < 1e-6


def test_rope_norm_preserving_property(orc):
    """A rotation keeps x_i^2 + x_{i+half}^2 (to rounding) at every position."""
    hidden, hd, L, B = 768, 64, 512, 2
    x = splitmix_normal(3 * hidden * L * B, 0x7E4F0660)
    c, s = host_tables(160000.0, L, hd)
    got = gpu_rope(x, c, s, 24, L, B, hd, hd, (hd, 3 * hidden, 3 * hidden * L, 1))
    a = x.reshape(B * L, 3 * hidden)[:, :2 * hidden].reshape(-1, 2, 32).astype(np.float64)
    r = got.reshape(B * L, 3 * hidden)[:, :2 * hidden].reshape(-1, 2, 32).astype(np.float64)
    assert np.allclose((a ** 2).sum(1), (r ** 2).sum(1), rtol=1e-5, atol=1e-6)


def test_rope_errors():
    x = empty(64)
    desc = _lib.RopeDesc(1, 4, 1, 16, 18, 16, 16, 64, 1)
    with pytest.raises(tfx.TfxError) as e:
        call("tfx_rope_pairhalf_f32", P(x), P(x), P(x), P(x), ctypes.byref(desc), S())
    assert "exceeds head dimension" in str(e.value)
