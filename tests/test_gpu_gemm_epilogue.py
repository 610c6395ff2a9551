"""GPU parity: the MLP projection with its epilogue fused on tcgen05
(tfx_gemm_geglu_ff_f32, tfx_gemm_bias_act_ff_f32) against the oracle's
sequential projection followed by its GeGLU / bias-activation
(crates/tenferro-ext/src/gemm_geglu.rs:209-238; cpu-kernels lib.rs:274-288,
:516-538).

The tensor cores compute the projection with the 3xTF32 split, so results are
compared within the f32 bar (the summation order differs from the
reference's); tiles of 128 tokens with a non-finite input, and every tile when
the weight has one, run the reference's sequential arithmetic and are compared
bitwise. The shapes and data of the reference's own test
(crates/tenferro-ext/tests/gemm_geglu.rs:7-93) are included.
"""

import ctypes

import numpy as np
import pytest
import torch

import tfx
from gpu_util import P, S, call, dev, empty, host
from helpers import F32_ATOL_REL, F32_RTOL, assert_bitwise, assert_close, splitmix_normal
from tfx import _lib

pytestmark = pytest.mark.gpu


def gpu_gemm_geglu(x, w, b, in_dim, inter, length, x_offset=0):
    xd, wd = dev(x, x_offset), dev(w)
    bd = None if b is None else dev(b)
    yd = empty(inter * length)
    call("tfx_gemm_geglu_ff_f32", P(xd), P(wd), P(bd), P(yd), in_dim, inter, length, S())
    return host(yd)


def gpu_gemm_bias_act(x, w, b, in_dim, out_dim, length, act):
    xd, wd = dev(x), dev(w)
    bd = None if b is None else dev(b)
    yd = empty(out_dim * length)
    call("tfx_gemm_bias_act_ff_f32", P(xd), P(wd), P(bd), P(yd), in_dim, out_dim, length, act,
         S())
    return host(yd)


@pytest.mark.parametrize("inp,hidden,length,batch",
                         [(7, 5, 1, 1), (7, 5, 3, 2), (33, 17, 65, 2), (129, 129, 129, 1),
                          (7, 5, 0, 2)])
@pytest.mark.parametrize("has_bias", [False, True])
def test_gemm_geglu_reference_test_cases(orc, inp, hidden, length, batch, has_bias):
    """crates/tenferro-ext/tests/gemm_geglu.rs:11-17 shapes and :21-50 data."""
    tokens = length * batch
    x = np.array([((i % 23) - 11) * 0.031 for i in range(inp * tokens)], np.float32)
    w = np.array([((i % 19) - 9) * 0.027 for i in range(inp * 2 * hidden)], np.float32)
    b = np.array([(i % 7) * 0.019 for i in range(2 * hidden)], np.float32) if has_bias else None
    got = gpu_gemm_geglu(x, w, b, inp, hidden, tokens)
    want = orc.gemm_geglu_f32(x, w, b, inp, hidden, tokens)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"gemm_geglu {inp}x{hidden}x{tokens}")
    again = gpu_gemm_geglu(x, w, b, inp, hidden, tokens)
    assert_bitwise(again, got, "gemm_geglu repeated call")


@pytest.mark.parametrize("has_bias", [False, True])
def test_gemm_geglu_modernbert_mlp_shape(orc, has_bias):
    """ModernBERT-base MLP input projection: hidden 768 -> 2 x 1152 over the
    8192 tokens of configs[1] (the GeGLU there is this projection's epilogue)."""
    in_dim, inter, length = 768, 1152, 8192
    x = splitmix_normal(in_dim * length, 0x7E4F0D00)
    w = splitmix_normal(in_dim * 2 * inter, 0x7E4F0D01, std=in_dim ** -0.5)
    b = splitmix_normal(2 * inter, 0x7E4F0D02, std=0.02) if has_bias else None
    got = gpu_gemm_geglu(x, w, b, in_dim, inter, length)
    want = orc.gemm_geglu_f32(x, w, b, in_dim, inter, length)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, "gemm_geglu mlp")


def test_gemm_geglu_unaligned_and_ragged(orc):
    """in_dim not a multiple of 4 or 32, x off the 16-byte grid, I not a
    multiple of 128 or 4, tokens not a multiple of 128."""
    in_dim, inter, length = 130, 100, 333
    x = splitmix_normal(in_dim * length, 0x7E4F0D10)
    w = splitmix_normal(in_dim * 2 * inter, 0x7E4F0D11, std=0.1)
    b = splitmix_normal(2 * inter, 0x7E4F0D12, std=0.02)
    got = gpu_gemm_geglu(x, w, b, in_dim, inter, length, x_offset=1)
    want = orc.gemm_geglu_f32(x, w, b, in_dim, inter, length)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, "gemm_geglu ragged")


def test_gemm_geglu_nonfinite_tiles_take_the_exact_path(orc):
    """inf / NaN in two tokens: their 128-token tiles follow the reference's
    arithmetic bit for bit (inf and NaN where it has them); the other tiles
    stay within the f32 bar."""
    in_dim, inter, length = 96, 64, 640
    x = splitmix_normal(in_dim * length, 0x7E4F0D20)
    w = splitmix_normal(in_dim * 2 * inter, 0x7E4F0D21, std=0.1)
    x[3 + in_dim * 5] = np.inf
    x[7 + in_dim * 300] = np.nan
    x[11 + in_dim * 301] = np.float32(3e30)  # finite but beyond the split's range
    got = gpu_gemm_geglu(x, w, None, in_dim, inter, length)
    want = orc.gemm_geglu_f32(x, w, None, in_dim, inter, length)
    g2, w2 = got.reshape(length, inter), want.reshape(length, inter)
    assert not np.isfinite(w2[5]).all() and np.isnan(w2[300]).all()
    for lo, hi in ((0, 128), (256, 384)):  # the flagged tiles
        assert_bitwise(g2[lo:hi], w2[lo:hi], f"exact tile {lo}")
    rest = np.r_[128:256, 384:640]
    assert_close(g2[rest].ravel(), w2[rest].ravel(), F32_RTOL, F32_ATOL_REL, "unflagged tiles")


def test_gemm_geglu_nonfinite_weight_runs_every_tile_exactly(orc):
    in_dim, inter, length = 40, 24, 300
    x = splitmix_normal(in_dim * length, 0x7E4F0D30)
    w = splitmix_normal(in_dim * 2 * inter, 0x7E4F0D31, std=0.1)
    w[5 + in_dim * 30] = -np.inf  # a gate row
    b = splitmix_normal(2 * inter, 0x7E4F0D32, std=0.02)
    got = gpu_gemm_geglu(x, w, b, in_dim, inter, length)
    assert_bitwise(got, orc.gemm_geglu_f32(x, w, b, in_dim, inter, length), "exact call")


@pytest.mark.parametrize("act", [_lib.TFX_ACT_IDENTITY, _lib.TFX_ACT_GELU_ERF,
                                 _lib.TFX_ACT_RELU])
@pytest.mark.parametrize("has_bias", [False, True])
def test_gemm_bias_act(orc, act, has_bias):
    """The attention output projection shape (768 -> 768) over 1000 tokens (a
    ragged last tile), and 3 x 256 + 17 outputs (a ragged last column tile)."""
    for in_dim, out_dim, length in ((768, 768, 1000), (64, 785, 129)):
        x = splitmix_normal(in_dim * length, 0x7E4F0D40 + out_dim)
        w = splitmix_normal(in_dim * out_dim, 0x7E4F0D41 + out_dim, std=in_dim ** -0.5)
        b = splitmix_normal(out_dim, 0x7E4F0D42, std=0.02) if has_bias else None
        got = gpu_gemm_bias_act(x, w, b, in_dim, out_dim, length, act)
        want = orc.gemm_bias_act_f32(x, w, b, in_dim, out_dim, length, act)
        assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"gemm_bias_act {act} {out_dim}")


def test_gemm_geglu_zero_contraction_is_the_bias_epilogue(orc):
    inter, length = 9, 5
    b = splitmix_normal(2 * inter, 0x7E4F0D50)
    bd = dev(b)
    yd = empty(inter * length)
    # x and weight are empty (in_dim 0): null pointers are accepted
    call("tfx_gemm_geglu_ff_f32", None, None, P(bd), P(yd), 0, inter, length, S())
    want = orc.geglu_f32(np.tile(b, length), inter, length)
    assert_bitwise(host(yd), want, "in_dim 0")


def test_gemm_epilogue_errors():
    x = empty(64)
    with pytest.raises(tfx.TfxError) as e:
        call("tfx_gemm_geglu_ff_f32", P(x), None, None, P(x), 4, 4, 4, S())
    assert "weight: null pointer" in str(e.value)
    with pytest.raises(tfx.TfxError) as e:
        call("tfx_gemm_geglu_ff_f32", P(x), P(x), None, P(x), 4, -1, 4, S())
    assert "non-negative" in str(e.value)
    with pytest.raises(tfx.TfxError) as e:
        call("tfx_gemm_geglu_ff_f32", P(x), P(x), None, P(x), 4, 1 << 40, 4, S())
    assert "overflow" in str(e.value)
    with pytest.raises(tfx.TfxError) as e:
        call("tfx_gemm_bias_act_ff_f32", P(x), P(x), None, P(x), 4, 4, 4, 7, S())
    assert "unknown activation" in str(e.value)
    y = empty(64)
    with pytest.raises(tfx.TfxError) as e:  # y overlapping x
        call("tfx_gemm_bias_act_ff_f32", P(x), P(y), None, P(x), 4, 4, 4, 0, S())
    assert "overlaps x" in str(e.value)
    call("tfx_gemm_geglu_ff_f32", P(x), P(x), None, P(y), 4, 4, 0, S())  # empty: no-op
    torch.cuda.synchronize()
    n = ctypes.c_uint32(0)
    assert _lib.lib.tfx_wait_timeouts(ctypes.byref(n)) == 0 and n.value == 0
