"""GPU parity: attention prep (bitwise) and masked scaled dot-product attention.

The prep kernels reproduce the cpu-kernels arithmetic exactly (rounded products,
sequential per-token sums) and are compared bit for bit. The attention kernels
use a different summation order (tiled dot products, online softmax, one
division at the end) and are compared within the f32 tolerance."""

import ctypes

import numpy as np
import pytest

from gpu_util import P, S, call, dev, empty, host
from helpers import (assert_bitwise, assert_close, decode_value, golden_case, splitmix_normal,
                     splitmix_uniform, F32_RTOL, F32_ATOL_REL)
from tfx import _lib

pytestmark = pytest.mark.gpu


def keep_window(L, B, window, valid):
    """keep[q + L*(k + L*b)] for |q - k| <= window and k < valid[b]."""
    q = np.arange(L)[None, None, :]
    k = np.arange(L)[None, :, None]
    v = np.asarray(valid)[:, None, None]
    m = (np.abs(q - k) <= window) & (k < v)
    return np.ascontiguousarray(m.astype(np.uint8)).ravel()


def gpu_laya_block(qkv, keep, hidden, heads, L, B, tables=None):
    # Every device tensor stays referenced until the kernels have run: a
    # temporary passed as P(dev(x)) would be freed (and its memory reused)
    # before the call.
    out = empty(hidden * L * B)
    qd, kd = dev(qkv), dev(keep)
    c = s = None
    if tables is not None:
        c, s = dev(tables[0]), dev(tables[1])
    call("tfx_laya_attention_block_f32", P(qd), P(kd), P(c), P(s), P(out), hidden, heads, L, B,
         S())
    return host(out)


@pytest.mark.parametrize("hd,heads,L,B,window,rope", [
    (64, 4, 128, 2, 16, 10000.0), (64, 3, 200, 2, -1, 160000.0), (128, 2, 96, 2, 32, 10000.0),
    (256, 1, 80, 2, -1, 10000.0), (48, 2, 70, 1, 8, 10000.0), (4, 2, 33, 2, -1, 0.0)])
def test_laya_attention_block(orc, hd, heads, L, B, window, rope):
    d = hd * heads
    qkv = splitmix_normal(3 * d * L * B, 0x7E4F0A00 + hd + L)
    valid = [L - 5 * b for b in range(B)]
    keep = keep_window(L, B, window if window >= 0 else L, valid)
    tables = orc.rope_tables_powf_f32(rope, L, hd) if rope else None
    got = gpu_laya_block(qkv, keep, d, heads, L, B, tables)
    want = orc.laya_attention_block_f32(qkv, keep, d, heads, L, B,
                                         *(tables if tables is not None else (None, None)))
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"laya attention hd={hd} L={L}")


def test_laya_attention_block_nonfinite_qk_routed(orc):
    """Heads whose q or k hold NaN / inf leave the tensor-core kernel for the
    f32 one (flags set by the prep kernel); results follow the reference:
    non-finite scores contribute nothing, rows without a finite score are NaN."""
    hd, heads, L, B = 64, 2, 96, 2
    d = hd * heads
    qkv = splitmix_normal(3 * d * L * B, 0x7E4F0A90)
    x = qkv.reshape(B, L, 3, heads, hd)
    x[1, 5, 0, 0, 3] = np.nan          # q of batch 1, head 0, token 5
    x[0, 7, 1, 1, 10] = np.inf         # k of batch 0, head 1, token 7
    keep = keep_window(L, B, 20, [L, L - 9])
    got = gpu_laya_block(qkv, keep, d, heads, L, B)
    want = orc.laya_attention_block_f32(qkv, keep, d, heads, L, B)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, "non-finite q / k")


@pytest.mark.parametrize("hd", [4, 64])
def test_laya_attention_block_known_answer(orc, hd):
    """crates/cpu-kernels/src/lib.rs:1212-1250 through the GPU (hd 4: the row
    kernel; hd 64: the tiled kernel with its non-finite V guard): masked NaN /
    inf never leak, rows without keys are NaN, the rest average v exactly."""
    case = golden_case("laya_attention_block_masked_nonfinite_and_empty_rows")
    L, key = case["length"], case["masked_key"]
    keep = np.ones(L * L, np.uint8)
    keep[np.arange(L) + L * key] = 0
    keep[L * np.arange(L)] = 0
    keep[L - 1 + L * np.arange(L)] = 0
    for excluded in case["excluded_values"]:
        qkv = np.zeros(3 * hd * L, np.float32)
        for k in range(L):
            qkv[3 * hd * k + 2 * hd:3 * hd * k + 3 * hd] = np.arange(1, hd + 1)
        qkv[3 * hd * key + 2 * hd:3 * hd * key + 3 * hd] = decode_value(excluded)
        out = gpu_laya_block(qkv, keep, hd, 1, L, 1).reshape(L, hd)
        for q in range(L):
            if q in case["empty_queries"]:
                assert np.all(np.isnan(out[q])), q
            else:
                assert np.max(np.abs(out[q] - np.arange(1, hd + 1))) <= 1e-6 * hd, q
        if hd == case["hidden"]:
            want = orc.laya_attention_block_f32(qkv, keep, hd, 1, L, 1)
            assert_close(out.ravel(), want, F32_RTOL, F32_ATOL_REL, "known answer vs oracle")


@pytest.mark.parametrize("hd,heads,L,rope", [(64, 4, 96, 10000.0), (128, 2, 50, 0.0), (6, 3, 17, 10000.0)])
def test_laya_qkv_prep_bitwise(orc, hd, heads, L, rope):
    B = 3
    d = hd * heads
    qkv = splitmix_normal(3 * d * L * B, 0x7E4F0A10 + hd)
    n = d * L * B
    qh, kh, vh = empty(n), empty(n), empty(n)
    if rope:
        c, s = orc.rope_tables_powf_f32(rope, L, hd)
        cd, sd = dev(c), dev(s)
        cp, sp = P(cd), P(sd)
    else:
        c = s = None
        cp = sp = None
    xd = dev(qkv)
    call("tfx_laya_qkv_prep_f32", P(xd), cp, sp, P(qh), P(kh), P(vh), d, heads, L, B, S())
    want = orc.laya_qkv_prep_f32(qkv, d, heads, L, B, c, s)
    for got, w, name in zip((qh, kh, vh), want, "qkv"):
        assert_bitwise(host(got), w, f"laya prep {name}")


@pytest.mark.parametrize("hd,rot,heads,L", [(64, 16, 4, 70), (256, 64, 2, 40), (20, 6, 3, 33),
                                            (128, 0, 2, 32)])
def test_jeff_qkv_prep_bitwise(orc, hd, rot, heads, L):
    w = heads * hd
    q, k, v = (splitmix_normal(L * w, 0x7E4F0A20 + i + hd) for i in range(3))
    qn = splitmix_normal(hd, 0x7E4F0A28, std=0.1)
    kn = splitmix_normal(hd, 0x7E4F0A29, std=0.1)
    c, s = orc.rope_tables_powf_f32(1e6, L, rot) if rot else (np.zeros(1, np.float32),) * 2
    n = L * w
    qh, kh, vh = empty(n), empty(n), empty(n)
    ins = [dev(t) for t in (q, k, v, qn, kn, c, s)]
    call("tfx_jeff_qkv_prep_f32", *[P(t) for t in ins], P(qh), P(kh), P(vh), L, heads, hd, rot,
         ctypes.c_float(1e-6), S())
    want = orc.jeff_qkv_prep_f32(q, k, v, qn, kn, c if rot else None, s if rot else None, L, heads,
                                 hd, rot, 1e-6)
    for got, wv, name in zip((qh, kh, vh), want, "qkv"):
        assert_bitwise(host(got), wv, f"jeff prep {name}")


@pytest.mark.parametrize("hd,rot,heads,L", [(64, 16, 4, 130), (256, 64, 2, 72), (20, 6, 2, 31)])
def test_jeff_attention(orc, hd, rot, heads, L):
    w = heads * hd
    theta, eps = 1e7, 1e-6
    q, k, v, g = (splitmix_normal(L * w, 0x7E4F0A30 + i + hd) for i in range(4))
    qn = splitmix_normal(hd, 0x7E4F0A38, std=0.1)
    kn = splitmix_normal(hd, 0x7E4F0A39, std=0.1)
    mask = (splitmix_uniform(L, 0x7E4F0A3A, 0.0, 1.0) > 0.2).astype(np.float32)
    mask[0] = 0.0  # query 0 sees no key: its row is 0
    c, s = orc.rope_tables_powf_f32(theta, L, rot)
    out = empty(L * w)
    ins = [dev(t) for t in (q, k, v, g, qn, kn, mask, c, s)]
    call("tfx_jeff_attention_f32", *[P(t) for t in ins], P(out), L, heads, hd, rot,
         ctypes.c_float(eps), S())
    got = host(out)
    want = orc.jeff_full_attention_f32(q, k, v, g, qn, kn, mask, L, heads, hd, rot, theta, eps)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"jeff attention hd={hd}")
    assert np.all(got.reshape(w, L)[:, 0] == 0.0)


# Lengths that are whole 128-token tiles take the tensor-core route (3xTF32
# GEMMs around the masked softmax); the others the f32 kernel.
@pytest.mark.parametrize("hd,rot,heads,L,big_v", [
    (256, 64, 4, 512, False), (64, 16, 3, 384, False), (128, 32, 2, 256, True),
    (64, 16, 1, 2176, False),   # rows past 2048 keys; an odd number of 128-token tiles
    (64, 16, 1, 4224, False)])  # a long single head: 33 tiles, many slots per tile
def test_jeff_attention_tensor_cores(orc, hd, rot, heads, L, big_v):
    w = heads * hd
    theta, eps = 1e7, 1e-6
    q, k, v, g = (splitmix_normal(L * w, 0x7E4F0A40 + i + hd) for i in range(4))
    qn = splitmix_normal(hd, 0x7E4F0A48, std=0.1)
    kn = splitmix_normal(hd, 0x7E4F0A49, std=0.1)
    mask = (splitmix_uniform(L, 0x7E4F0A4A, 0.0, 1.0) > 0.3).astype(np.float32)
    mask[:3] = 0.0  # queries 0..2 see no key: their rows are 0
    if big_v:
        # a value of 2^41 in head 1's V: that head goes to the f32 kernel
        v.reshape(w, L)[hd + 7, L // 2] = 2.0 ** 41  # (length, hidden) time-first
    c, s = orc.rope_tables_powf_f32(theta, L, rot)
    out = empty(L * w)
    ins = [dev(t) for t in (q, k, v, g, qn, kn, mask, c, s)]
    call("tfx_jeff_attention_f32", *[P(t) for t in ins], P(out), L, heads, hd, rot,
         ctypes.c_float(eps), S())
    got = host(out)
    want = orc.jeff_full_attention_f32(q, k, v, g, qn, kn, mask, L, heads, hd, rot, theta, eps)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"jeff attention (tensor cores) hd={hd}")
    assert np.all(got.reshape(w, L)[:, :3] == 0.0)


def test_jeff_attention_tensor_cores_nonfinite(orc):
    """Non-finite inputs on the tensor-core route: the heads holding them go to
    the f32 kernel (the reference's rules: non-finite scores contribute
    nothing, a NaN in V of a key whose probability is 0 does not leak), the
    others stay on the GEMMs; everything matches the oracle, NaN for NaN."""
    hd, rot, heads, L = 64, 16, 4, 256
    w = heads * hd
    q, k, v, g = (splitmix_normal(L * w, 0x7E4F0A60 + i) for i in range(4))
    qn, kn = splitmix_normal(hd, 0x7E4F0A68, std=0.1), splitmix_normal(hd, 0x7E4F0A69, std=0.1)
    mask = (splitmix_uniform(L, 0x7E4F0A6A, 0.0, 1.0) > 0.25).astype(np.float32)
    mask[0] = 1.0
    mask[3] = 0.0
    # (length, hidden) time-first: element (t, f) at t + L f
    q.reshape(w, L)[0 * hd + 5, 40] = np.inf        # head 0: one query token
    k.reshape(w, L)[1 * hd + 9, 70] = np.nan        # head 1: one key token
    v.reshape(w, L)[2 * hd + 2, 3] = np.nan         # head 2: a masked key's V
    c, s = orc.rope_tables_powf_f32(1e7, L, rot)
    out = empty(L * w)
    ins = [dev(t) for t in (q, k, v, g, qn, kn, mask, c, s)]
    call("tfx_jeff_attention_f32", *[P(t) for t in ins], P(out), L, heads, hd, rot,
         ctypes.c_float(1e-6), S())
    got = host(out)
    want = orc.jeff_full_attention_f32(q, k, v, g, qn, kn, mask, L, heads, hd, rot, 1e7, 1e-6)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, "jeff attention (tensor cores), non-finite")
    assert np.isfinite(got.reshape(w, L)[2 * hd:3 * hd]).all()  # the masked NaN did not leak


@pytest.mark.parametrize("rot,misalign", [(0, False), (32, True)])
def test_jeff_attention_tc_edges(orc, rot, misalign):
    """Rotary width 0 (no tables) on the tensor-core route, and an output /
    gate that is not 16-byte aligned (the f32 route takes the call)."""
    hd, heads, L = 128, 2, 256
    w = heads * hd
    q, k, v, g = (splitmix_normal(L * w, 0x7E4F0A70 + i + rot) for i in range(4))
    qn, kn = splitmix_normal(hd, 0x7E4F0A78, std=0.1), splitmix_normal(hd, 0x7E4F0A79, std=0.1)
    mask = (splitmix_uniform(L, 0x7E4F0A7A, 0.0, 1.0) > 0.2).astype(np.float32)
    mask[0] = 1.0
    want = orc.jeff_full_attention_f32(q, k, v, g, qn, kn, mask, L, heads, hd, rot, 1e7, 1e-6)
    if rot:
        c, s = orc.rope_tables_powf_f32(1e7, L, rot)
        cd, sd = dev(c), dev(s)
    else:
        cd = sd = None
    off = 1 if misalign else 0  # one float off the 16-byte grid
    gd = dev(g, off)
    out = empty(L * w, offset_elems=off)
    ins = [dev(t) for t in (q, k, v)]
    qnd, knd, md = dev(qn), dev(kn), dev(mask)
    call("tfx_jeff_attention_f32", *[P(t) for t in ins], P(gd), P(qnd), P(knd), P(md),
         P(cd), P(sd), P(out), L, heads, hd, rot, ctypes.c_float(1e-6), S())
    got = host(out)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"jeff attention rot={rot} misalign={misalign}")


def test_jeff_attention_no_active_key(orc):
    hd, rot, heads, L = 64, 16, 2, 128
    w = heads * hd
    q, k, v, g = (splitmix_normal(L * w, 0x7E4F0A50 + i) for i in range(4))
    qn, kn = splitmix_normal(hd, 0x7E4F0A58, std=0.1), splitmix_normal(hd, 0x7E4F0A59, std=0.1)
    mask = np.zeros(L, np.float32)
    c, s = orc.rope_tables_powf_f32(1e7, L, rot)
    out = empty(L * w)
    ins = [dev(t) for t in (q, k, v, g, qn, kn, mask, c, s)]
    call("tfx_jeff_attention_f32", *[P(t) for t in ins], P(out), L, heads, hd, rot,
         ctypes.c_float(1e-6), S())
    assert np.all(host(out) == 0.0)


def attention_f64(qh, kh, vh, B, H, L, hd, scale, bias=None, causal=False, active=None):
    """Double-precision restatement of the additive-bias path (fused.cu:239-306)."""
    q = qh.reshape(B, H, L, hd).astype(np.float64)
    k = kh.reshape(B, H, L, hd).astype(np.float64)
    v = vh.reshape(B, H, L, hd).astype(np.float64)
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * scale
    keep = np.ones((B, 1, L, L), bool)
    if bias is not None:
        s = s + bias.reshape(B, L, L).transpose(0, 2, 1)[:, None]  # [b][k][q] -> [b][q][k]
    if causal:
        keep &= np.tril(np.ones((L, L), bool))[None, None]
    if active is not None:
        keep &= (active.reshape(B, 1, 1, L) != 0)
    s = np.where(keep, s, -np.inf)
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    p = p / p.sum(-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v)


@pytest.mark.parametrize("hd", [64, 128, 40])
def test_attention_core_bias_active_causal(hd):
    """The CUDA twin's form: additive (L, L, B) bias, active key mask, causal,
    output (d, L, B) -- against a float64 restatement."""
    B, H, L = 2, 3, 100
    n = B * H * L * hd
    qh, kh, vh = (splitmix_normal(n, 0x7E4F0A40 + i) for i in range(3))
    bias = splitmix_normal(L * L * B, 0x7E4F0A44, std=0.5)
    active = (splitmix_uniform(B * L, 0x7E4F0A45, 0.0, 1.0) > 0.1).astype(np.float32)
    active[0] = 1.0
    active[L] = 1.0
    d = _lib.AttentionDesc()
    _lib.lib.tfx_attention_desc_init(ctypes.byref(d), B, H, L, hd)
    bd, ad = dev(bias), dev(active)
    d.bias, d.active, d.causal = bd.data_ptr(), ad.data_ptr(), 1
    out = empty(n)
    ins = [dev(t) for t in (qh, kh, vh)]
    call("tfx_attention_f32", *[P(t) for t in ins], P(out), ctypes.byref(d), S())
    got = host(out).reshape(B, L, H, hd)  # (d, L, B) with d = H*hd fastest
    want = attention_f64(qh, kh, vh, B, H, L, hd, 1.0 / np.sqrt(np.float32(hd)), bias, True, active)
    want = want.transpose(0, 2, 1, 3).astype(np.float32)  # (B, L, H, hd)
    assert_close(got.ravel(), want.ravel(), 2e-5, F32_ATOL_REL, f"attention core hd={hd}")


@pytest.mark.parametrize("L,causal,B", [(512, 0, 2), (333, 1, 1), (4160, 0, 1)])
def test_attention_core_growing_scores(L, causal, B):
    """Scores that grow along the keys (an additive bias rising by 40 over
    the sequence, added exactly after the product) move each row's running
    max again and again: the tensor-core kernels' rescale path. 4160 keys
    pass the 64 blocks that the per-block keep bits cover and accumulate 65
    blocks of P V; an active mask with holes makes every block a masked one.
    (A steeper rise would push the scores to where one f32 rounding of the
    score alone exceeds the tolerance, in any f32 implementation.)"""
    H, hd = 2, 64
    n = B * H * L * hd
    qh, kh, vh = (splitmix_normal(n, 0x7E4F0B40 + i + L) for i in range(3))
    ramp = (np.arange(L, dtype=np.float32) * np.float32(40.0 / L))[None, :, None]
    bias = (np.broadcast_to(ramp, (B, L, L))
            + splitmix_normal(B * L * L, 0x7E4F0B47 + L, std=0.5).reshape(B, L, L))
    bias = np.ascontiguousarray(bias, np.float32).ravel()  # [b][k][q]
    active = (splitmix_uniform(B * L, 0x7E4F0B44 + L, 0.0, 1.0) > 0.05).astype(np.float32)
    active[0] = 1.0
    d = _lib.AttentionDesc()
    _lib.lib.tfx_attention_desc_init(ctypes.byref(d), B, H, L, hd)
    ad, bd = dev(active), dev(bias)
    d.active, d.bias, d.causal = ad.data_ptr(), bd.data_ptr(), causal
    out = empty(n)
    ins = [dev(t) for t in (qh, kh, vh)]
    call("tfx_attention_f32", *[P(t) for t in ins], P(out), ctypes.byref(d), S())
    got = host(out).reshape(B, L, H, hd)
    want = attention_f64(qh, kh, vh, B, H, L, hd, 1.0 / np.sqrt(np.float32(hd)), bias,
                         bool(causal), active)
    want = want.transpose(0, 2, 1, 3).astype(np.float32)
    assert_close(got.ravel(), want.ravel(), 2e-5, F32_ATOL_REL, f"growing scores L={L}")


@pytest.mark.parametrize("window", [128, -1])
def test_laya_attention_block_bert_shape(orc, window):
    """The ModernBERT layer shape (head_dim 64) at 512 tokens, sliding window
    128 and global with padded keys, against the oracle."""
    hd, heads, L, B = 64, 2, 512, 2
    d = hd * heads
    qkv = splitmix_normal(3 * d * L * B, 0x7E4F0B50 + L + window)
    valid = [L - 37, L - 64]
    keep = keep_window(L, B, window if window >= 0 else L, valid)
    tables = orc.rope_tables_powf_f32(160000.0 if window < 0 else 10000.0, L, hd)
    got = gpu_laya_block(qkv, keep, d, heads, L, B, tables)
    want = orc.laya_attention_block_f32(qkv, keep, d, heads, L, B, *tables)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"laya bert shape window={window}")


def test_attention_rejects_bad_arguments():
    d = _lib.AttentionDesc()
    _lib.lib.tfx_attention_desc_init(ctypes.byref(d), 1, 1, 8, 8)
    d.empty_rows = 7
    rc = _lib.lib.tfx_attention_f32(None, None, None, None, ctypes.byref(d), None)
    assert rc == -1 and b"empty_rows" in _lib.lib.tfx_last_error_string()


def test_attention_no_wait_gave_up():
    """Every bounded wait of the tensor-core kernels completed in the runs above."""
    n = ctypes.c_uint32(99)
    call("tfx_wait_timeouts", ctypes.byref(n))
    assert n.value == 0
